"""Pin the numpy oracle to golden vectors produced by the reference itself.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py,
which imports and runs the reference package (and its two valid Triton decode
kernels under Triton's CPU interpreter).  Integer / fp8 codes and their
reconstructions must match bit-exactly; attention outputs to float32 rounding.
"""

import numpy as np
import pytest

import inputs as gi
from oracle import attention as oatt
from oracle import decode as odec
from oracle import mla as omla
from oracle import quant as oq

PRECS = ["FP16", "FP8", "INT8", "INT4", "INT4_RESIDUAL", "SKIP"]


@pytest.mark.parametrize("prec", PRECS)
def test_fake_quantize_block_granularity_bit_exact(golden, prec):
    g = golden("quant_golden.npz")
    x = gi.normal(11, (2, 3, 20, 64), outlier_frac=0.01)
    r = oq.fake_quantize(x, prec)["recon"]
    np.testing.assert_array_equal(r, g[f"block_{prec}"])


@pytest.mark.parametrize("prec", PRECS)
@pytest.mark.parametrize("mode", ["page", "group32", "channel"])
def test_quantize_pages_matches_reference_reshapes(golden, prec, mode):
    g = golden("quant_golden.npz")
    pages = gi.normal(12, (5, 16, 128), outlier_frac=0.01)
    r = oq.quantize_pages(pages, prec, mode)["recon"]
    np.testing.assert_array_equal(r, g[f"{mode}_{prec}"])


def test_e4m3_matches_torch_cast_sweep(golden):
    g = golden("quant_golden.npz")
    got = oq.e4m3_to_f32(oq.f32_to_e4m3(g["fp8_sweep_in"]))
    ref = g["fp8_sweep_out"]
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan], ref[~nan])


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    vals = oq.e4m3_to_f32(codes)
    finite = ~np.isnan(vals)
    back = oq.f32_to_e4m3(vals[finite])
    # +0 and -0 both round-trip to their own codes
    np.testing.assert_array_equal(back, codes[finite])


def test_int4_pack_roundtrip_and_layout():
    g = np.random.default_rng(5)
    for D in (32, 64, 128):
        c = g.integers(-8, 8, size=(3, 16, D)).astype(np.int8)
        p = oq.pack_int4(c)
        assert p.shape == (3, 16, D // 2) and p.dtype == np.uint8
        np.testing.assert_array_equal(oq.unpack_int4(p), c)
        idx = oq.int4_d_index(D)
        assert sorted(idx.reshape(-1).tolist()) == list(range(D))


def test_dense_attention(golden):
    g = golden("attention_golden.npz")
    q = gi.normal(51, (2, 3, 5, 32)); k = gi.normal(52, (2, 3, 40, 32)); v = gi.normal(53, (2, 3, 40, 32))
    np.testing.assert_allclose(oatt.dense_attention(q, k, v), g["dense"], atol=2e-6, rtol=1e-5)


def _blocks(spec, prec_by_name):
    return [(s, e, prec_by_name[n]) for n, s, e, p, sc in spec if p != "SKIP"]


@pytest.mark.parametrize("mp", [0.0, 0.3, 0.5, 0.8, 0.95])
def test_intent_quant_attention_basic(golden, mp):
    g, meta = golden("attention_golden.npz"), golden("attention_golden.json")
    q = gi.normal(21, (1, 2, 8, 32)); k = gi.normal(22, (1, 2, 64, 32)); v = gi.normal(23, (1, 2, 64, 32))
    precs = meta[f"basic_mp{mp}"]
    out = oatt.intent_quant_attention(q, k, v, _blocks(gi.BASIC_LAYOUT, precs))
    np.testing.assert_allclose(out, g[f"basic_mp{mp}"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("mp", [0.5, 0.8])
def test_intent_quant_attention_e2e_layout(golden, mp):
    g, meta = golden("attention_golden.npz"), golden("attention_golden.json")
    q = gi.normal(31, (2, 4, 1, 64)); k = gi.normal(32, (2, 4, 448, 64), 0.01); v = gi.normal(33, (2, 4, 448, 64), 0.01)
    out = oatt.intent_quant_attention(q, k, v, _blocks(gi.E2E_LAYOUT, meta[f"e2e_mp{mp}"]))
    np.testing.assert_allclose(out, g[f"e2e_mp{mp}"], atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("prec", ["FP8", "INT8", "INT4", "INT4_RESIDUAL"])
def test_intent_quant_attention_forced(golden, prec):
    g = golden("attention_golden.npz")
    q = gi.normal(41, (1, 2, 4, 64)); k = gi.normal(42, (1, 2, 448, 64), 0.01); v = gi.normal(43, (1, 2, 448, 64), 0.01)
    blocks = [(s, e, prec) for n, s, e, p, sc in gi.E2E_LAYOUT if p != "SKIP"]
    np.testing.assert_allclose(oatt.intent_quant_attention(q, k, v, blocks), g[f"forced_{prec}"], atol=2e-6, rtol=1e-5)


def test_c1_reference_granularity(golden):
    g = golden("attention_golden.npz")
    q = gi.normal(1001, (1, 8, 1, 64)); k = gi.normal(1002, (1, 8, 1440, 64)); v = gi.normal(1003, (1, 8, 1440, 64))
    blocks = [(0, 128, "FP16"), (128, 1024, "INT8"), (1280, 1440, "FP16")]
    np.testing.assert_allclose(oatt.intent_quant_attention(q, k, v, blocks), g["c1_refgran"], atol=2e-6, rtol=1e-5)


def test_paged_decode_equals_selected_block_attention():
    """Page-based decode over per-channel-scaled pages == the block oracle."""
    B, H, D, PS = 1, 2, 64, 16
    k = gi.normal(7, (B, H, 448, D), 0.01); v = gi.normal(8, (B, H, 448, D), 0.01); q = gi.normal(9, (B, H, 1, D))
    blocks = [(0, 64, "FP16"), (64, 192, "INT8"), (320, 384, "INT4_RESIDUAL")]
    ref = oatt.intent_quant_attention(q, k, v, blocks)
    # lay the blocks out as single-head pages, one page per 16 tokens per head
    pools = {n: [] for n in ("k_f16", "v_f16", "k_i8", "v_i8", "k_i4", "v_i4", "k_i4r", "v_i4r")}
    sc = {n: [] for n in ("k_scale", "v_scale", "k_res_scale", "v_res_scale")}
    tags, table = [], [[] for _ in range(H)]
    tagnum = {"FP16": 0, "INT8": 1, "INT4_RESIDUAL": 2}
    for h in range(H):
        for s, e, prec in blocks:
            for plane, x in (("k", k), ("v", v)):
                blk = x[:, :, s:e, :]
                full = oq.fake_quantize(blk, prec)
                if prec != "FP16":
                    scale = np.broadcast_to(full["scale"].reshape(1, D), ((e - s) // PS, D))
                    rq = oq.quantize_pages(blk[0, h].reshape(-1, PS, D), prec, "channel", scales=scale,
                                           res_scales=None if prec != "INT4_RESIDUAL" else
                                           np.broadcast_to(full["res_scale"].reshape(1, D), ((e - s) // PS, D)))
                    np.testing.assert_array_equal(rq["recon"], full["recon"][0, h].reshape(-1, PS, D))
    # a direct paged run (per-head pages, per-channel block scales)
    NPg = 0
    for h in range(H):
        for s, e, prec in blocks:
            n = (e - s) // PS
            for plane, x in (("k", k), ("v", v)):
                blk = x[:, :, s:e, :]
                full = oq.fake_quantize(blk, prec)
                pages = blk[0, h].reshape(n, PS, D)
                if prec == "FP16":
                    pools[f"{plane}_f16"].append(pages.astype(np.float16))
                    for other in ("i8", "i4", "i4r"):
                        pools[f"{plane}_{other}"].append(np.zeros((n, PS, D if other == "i8" else D // 2), np.int8 if other == "i8" else np.uint8))
                    sc[f"{plane}_scale"].append(np.ones((n, D), np.float32))
                    sc[f"{plane}_res_scale"].append(np.ones((n, D), np.float32))
                else:
                    scale = np.broadcast_to(full["scale"].reshape(1, D), (n, D))
                    rs = None if prec != "INT4_RESIDUAL" else np.broadcast_to(full["res_scale"].reshape(1, D), (n, D))
                    rq = oq.quantize_pages(pages, prec, "channel", scales=scale, res_scales=rs)
                    pools[f"{plane}_f16"].append(np.zeros((n, PS, D), np.float16))
                    pools[f"{plane}_i8"].append(rq["codes"] if prec == "INT8" else np.zeros((n, PS, D), np.int8))
                    pools[f"{plane}_i4"].append(oq.pack_int4(rq["codes"]) if prec != "INT8" else np.zeros((n, PS, D // 2), np.uint8))
                    pools[f"{plane}_i4r"].append(oq.pack_int4(rq["res_codes"]) if prec == "INT4_RESIDUAL" else np.zeros((n, PS, D // 2), np.uint8))
                    sc[f"{plane}_scale"].append(np.ascontiguousarray(scale))
                    sc[f"{plane}_res_scale"].append(np.ascontiguousarray(rs) if rs is not None else np.ones((n, D), np.float32))
            table[h].extend(range(NPg, NPg + n))
            tags.extend([tagnum[prec]] * n)
            NPg += n
    pools = {kk: np.concatenate(vv) for kk, vv in pools.items()}
    sc = {kk: np.concatenate(vv) for kk, vv in sc.items()}
    out = odec.paged_decode(q[:, :, 0, :], np.array([table]), None, np.array(tags),
                            {0: "F16", 1: "INT8", 2: "INT4R"}, pools, sc, "channel")
    np.testing.assert_allclose(out, ref[:, :, 0, :], atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("case", ["fp16", "int8", "skip", "mixed", "mixed_skip", "zero", "single", "ragged"])
def test_fused_reference_decode(golden, case):
    g = golden("fused_golden.npz")
    kf = gi.normal(61, (8, 16, 64)).astype(np.float16)
    vf = gi.normal(62, (8, 16, 64)).astype(np.float16)
    q = gi.normal(63, (2, 4, 1, 64)).astype(np.float16)
    out = odec.fused_selected_quant_decode_ref(q, kf, vf, g["k_i8"], g["v_i8"], g["k_sc"], g["v_sc"],
                                               g[f"pt_{case}"], g[f"prec_{case}"], g[f"pc_{case}"])
    np.testing.assert_allclose(out.astype(np.float16).astype(np.float32), g[f"out_{case}"].astype(np.float32),
                               atol=1e-3, rtol=0)


def test_fused_int8_page_quantizer(golden):
    """fused_selected_quant_decode.py:521-542: per-page absmax/127, fp16 scales."""
    g = golden("fused_golden.npz")
    kf = gi.normal(61, (8, 16, 64)).astype(np.float16)
    flat = kf.reshape(8, -1)
    absmax = np.maximum(np.abs(flat).max(axis=1, keepdims=True), np.float16(1e-6))
    scales = (absmax / np.float16(127.0)).astype(np.float16)
    codes = np.clip(np.rint(flat / scales), -128, 127).astype(np.int8)
    np.testing.assert_array_equal(codes.reshape(kf.shape), g["k_i8"])
    np.testing.assert_array_equal(scales.reshape(-1), g["k_sc"])


def test_triton6_kernel_semantics(golden):
    """triton_intent_quant_attention.py:272-332 under Triton's interpreter.

    Reference defect, pinned here: when the FIRST slot of a (b, h) is invalid
    (page id -1 or a SKIP tag) the kernel evaluates exp(-inf - -inf) = NaN,
    the NaN survives every later update (NaN * 0) and the final
    ``where(l > 0, acc / l, 0)`` turns the whole head into zeros.  This build
    implements the documented semantics instead (SKIP / -1 contribute nothing),
    so those heads are checked to be zero in the reference and excluded from the
    value comparison.
    """
    g = golden("triton_interp_golden.npz")
    out = odec.intent_quant_decode_triton_ref(g["t6_q"], g["t6_kf"], g["t6_vf"], g["t6_ki"], g["t6_vi"],
                                              g["t6_ks"], g["t6_vs"], g["t6_ids"], g["t6_cnt"], g["t6_prec"])
    ref = g["t6_out"].astype(np.float64)
    ids, cnt, prec = g["t6_ids"], g["t6_cnt"], g["t6_prec"]
    poisoned = np.zeros(cnt.shape, bool)
    for b in range(cnt.shape[0]):
        for h in range(cnt.shape[1]):
            if cnt[b, h] > 0:
                pid = ids[b, h, 0]
                poisoned[b, h] = pid < 0 or prec[pid] == 5
    assert poisoned.any() and (~poisoned).any()
    assert np.all(ref[poisoned] == 0)
    np.testing.assert_allclose(out[~poisoned], ref[~poisoned], atol=2e-3, rtol=0)


def test_adaptive_kernel_semantics(golden):
    g = golden("triton_interp_golden.npz")
    out = odec.adaptive_decode_triton_ref(g["ad_q"], g["ad_ids"], g["ad_fmts"], g["ad_kf"], g["ad_vf"],
                                          g["ad_k8"], g["ad_v8"], g["ad_k8s"], g["ad_v8s"])
    np.testing.assert_allclose(out, g["ad_out"].astype(np.float64), atol=2e-3, rtol=0)


@pytest.mark.parametrize("ps", [8, 16, 32, 64])
def test_mla_cpu_decode(golden, ps):
    g = golden("mla_golden.npz")
    qa = gi.normal(90 + ps, (2, 3, 64)); C = gi.normal(91 + ps, (4 * ps, 64)); W = gi.normal(92 + ps, (64, 128))
    out = omla.mla_decode_cpu(qa, C, W, np.array([2, 0, 3]), page_size=ps)
    np.testing.assert_allclose(out, g[f"cpu_ps{ps}"], atol=1e-4, rtol=1e-5)


def test_mla_sparse_reference(golden):
    g = golden("mla_golden.npz")
    lat = gi.normal(95, (4, 16, 64))
    W_QK = gi.normal(96, (4 * 64, 64)); W_VO = gi.normal(97, (64, 256))
    q = gi.normal(98, (2, 4, 4, 64))
    q_abs = q.transpose(0, 2, 1, 3).reshape(2, 4, 256) @ W_QK
    out = omla.mla_decode_cpu(q_abs, lat.reshape(64, 64), W_VO, np.arange(4), page_size=16)
    # the reference returns float16
    np.testing.assert_allclose(out.astype(np.float16).astype(np.float32), g["sparse_ref"], atol=0.25, rtol=2e-3)


def test_mla_paged_matches_cpu_decode():
    B, H, Dqk, Dv, PS = 2, 5, 96, 64, 16
    q = gi.normal(1, (B, H, Dqk))
    pages = gi.normal(2, (6, PS, Dqk))
    bf = pages.astype(np.float32)
    table = np.array([[0, 3, 5], [1, 2, -1]])
    out = omla.mla_paged_decode(q, table, None, np.zeros(6, np.int64), {"bf16": bf}, None, Dv, 1 / np.sqrt(Dqk))
    for b in range(B):
        ids = [i for i in table[b] if i >= 0]
        K = np.concatenate([bf[i] for i in ids])
        ref = oatt.dense_attention(q[b], K, K[:, :Dv], sm_scale=1 / np.sqrt(Dqk))
        np.testing.assert_allclose(out[b], ref, atol=1e-10)


def test_lse_merge_matches_unsplit():
    g = np.random.default_rng(3)
    s = g.standard_normal((4, 3, 37)) * 3
    vals = g.standard_normal((37, 8))
    m_full = s.max(-1)
    p = np.exp(s - m_full[..., None])
    ref = (p @ vals) / p.sum(-1, keepdims=True)
    cuts = [0, 5, 5, 20, 37]  # includes an empty split
    ms, ls, accs = [], [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        if a == b:
            ms.append(np.full((4, 3), -np.inf)); ls.append(np.zeros((4, 3))); accs.append(np.zeros((4, 3, 8)))
            continue
        mm = s[..., a:b].max(-1)
        pp = np.exp(s[..., a:b] - mm[..., None])
        ms.append(mm); ls.append(pp.sum(-1)); accs.append(pp @ vals[a:b])
    out = odec.lse_merge(np.stack(ms, -1), np.stack(ls, -1), np.stack(accs, -2))
    np.testing.assert_allclose(out, ref, atol=1e-12)
    empty = odec.lse_merge(np.full((2, 3), -np.inf), np.zeros((2, 3)), np.zeros((2, 3, 4)))
    assert np.all(empty == 0)

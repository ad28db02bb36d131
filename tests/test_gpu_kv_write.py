"""GPU parity of KV append (quantise-on-write of open pages) and of page
format transitions (demotion / promotion) with the numpy oracle.

Codes and scales are integer / exactly rounded outputs: bit-exact against
``oracle.quant.quantize_pages`` of the same dense rows.
"""

import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu

FORMATS = ["F16", "FP8", "INT8", "INT4", "INT4R"]
CODE = {"F16": 1, "FP8": 2, "INT8": 3, "INT4": 4, "INT4R": 5}
ORACLE_NAME = {"F16": "FP16", "FP8": "FP8", "INT8": "INT8", "INT4": "INT4", "INT4R": "INT4_RESIDUAL"}
TAG_MAP_FMT = {c: f for f, c in CODE.items()}   # identity tags: tag == format code


def _tag_map():
    from intent_attention.paged import make_tag_map
    return make_tag_map(TAG_MAP_FMT)


def _pool_page(pool, plane, fmt, pid):
    """Stored codes / scales of one pool page, in the oracle's representation."""
    g = lambda name: getattr(pool, f"{plane}_{name}")[pid].cpu().numpy()  # noqa: E731
    if fmt == "F16":
        return {"codes": g("f16")}
    out = {"scale": g("scale")}
    if fmt == "FP8":
        out["codes"] = g("fp8")
    elif fmt == "INT8":
        out["codes"] = g("i8")
    else:
        out["codes"] = oq.unpack_int4(g("i4"))
        if fmt == "INT4R":
            out["res_codes"] = oq.unpack_int4(g("i4r"))
            out["res_scale"] = g("res_scale")
    return out


def _assert_page(pool, plane, fmt, pid, dense, mode):
    ref = oq.quantize_pages(dense[None].astype(np.float32), ORACLE_NAME[fmt], mode)
    got = _pool_page(pool, plane, fmt, pid)
    for key, val in got.items():
        np.testing.assert_array_equal(val, ref[key][0], err_msg=f"{plane} {fmt} page {pid} {key}")


@pytest.mark.parametrize("mode", ["page", "group32", "channel"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_append_one_token_at_a_time(mode, dtype):
    from intent_attention import KVStage, PagePool, append_tokens
    g = np.random.default_rng(len(mode) * 7 + {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype])
    B, Ht, PS, D, n_pages = 3, 2, 16, 128, 3
    units = B * Ht
    pool = PagePool.allocate(units * n_pages, PS, D, FORMATS, mode, "cuda", zero=True)
    # every physical page gets its own format
    fmts = g.integers(1, 6, size=units * n_pages).astype(np.uint8)
    tags = torch.from_numpy(fmts).cuda()
    bases = torch.arange(units, dtype=torch.int32).view(B, Ht).cuda() * n_pages
    stage = KVStage.allocate(units, pool)
    T = n_pages * PS - 5
    dense_k = (g.standard_normal((B, Ht, T, D)) * np.exp(g.standard_normal((1, 1, 1, D)))).astype(np.float32)
    dense_v = g.standard_normal((B, Ht, T, D)).astype(np.float32)
    dense_k[0, 1, 20] *= 30.0                   # an outlier row re-scales its page on arrival
    k_t = torch.from_numpy(dense_k).to("cuda", dtype)
    v_t = torch.from_numpy(dense_v).to("cuda", dtype)
    dense_k, dense_v = k_t.float().cpu().numpy(), v_t.float().cpu().numpy()
    lengths = torch.zeros(B, dtype=torch.int32, device="cuda")
    nxt = torch.empty_like(lengths)
    checkpoints = {0, 1, 15, 16, 17, 20, 31, T - 1}
    for t in range(T):
        append_tokens(pool, k_t[:, :, t:t + 1], v_t[:, :, t:t + 1], lengths, tags, _tag_map(), stage,
                      bases=bases, new_lengths=nxt)
        lengths, nxt = nxt, lengths
        if t not in checkpoints:
            continue
        torch.cuda.synchronize()
        assert lengths.cpu().tolist() == [t + 1] * B
        for u in range(units):
            b, h = divmod(u, Ht)
            for pg in range(t // PS + 1):
                rows = min(PS, t + 1 - pg * PS)
                pid = u * n_pages + pg
                for plane, dense in (("k", dense_k), ("v", dense_v)):
                    page = np.zeros((PS, D), np.float32)
                    page[:rows] = dense[b, h, pg * PS: pg * PS + rows]
                    _assert_page(pool, plane, TAG_MAP_FMT[int(fmts[pid])], pid, page, mode)


@pytest.mark.parametrize("fmt", FORMATS)
def test_append_chunks_equal_whole_page_quantisation(fmt):
    """A prefill chunk, then decode-sized chunks that start mid-page, give the
    pages iak_quantize_pages gives for the same dense rows."""
    from intent_attention import KVStage, PagePool, append_tokens
    g = np.random.default_rng(CODE[fmt])
    B, Ht, PS, D, n_pages = 2, 3, 16, 64, 5
    units = B * Ht
    pool = PagePool.allocate(units * n_pages, PS, D, FORMATS, "group32", "cuda", zero=True)
    tags = torch.full((units * n_pages,), CODE[fmt], dtype=torch.uint8, device="cuda")
    bases = torch.arange(units, dtype=torch.int32).view(B, Ht).cuda() * n_pages
    stage = KVStage.allocate(units, pool)
    T = n_pages * PS
    dk = g.standard_normal((B, Ht, T, D)).astype(np.float32)
    dv = g.standard_normal((B, Ht, T, D)).astype(np.float32)
    pos, cuts = 0, [37, 3, 1, 24, 5]
    for c in cuts:
        positions = torch.full((B,), pos, dtype=torch.int32, device="cuda")
        append_tokens(pool, torch.from_numpy(dk[:, :, pos:pos + c]).cuda(), torch.from_numpy(dv[:, :, pos:pos + c]).cuda(),
                      positions, tags, _tag_map(), stage, bases=bases)
        pos += c
    torch.cuda.synchronize()
    full_pages = pos // PS
    for u in range(units):
        b, h = divmod(u, Ht)
        for pg in range(n_pages):
            rows = max(0, min(PS, pos - pg * PS))
            if rows == 0:
                continue
            for plane, dense in (("k", dk), ("v", dv)):
                page = np.zeros((PS, D), np.float32)
                page[:rows] = dense[b, h, pg * PS: pg * PS + rows]
                _assert_page(pool, plane, fmt, u * n_pages + pg, page, "group32")
    assert full_pages == 4


def test_append_out_of_range_pages_are_counted_not_written():
    from intent_attention import KVStage, PagePool, append_tokens
    PS, D = 16, 128
    pool = PagePool.allocate(4, PS, D, FORMATS, "page", "cuda", zero=True)
    tags = torch.full((4,), CODE["INT8"], dtype=torch.uint8, device="cuda")
    stage = KVStage.allocate(2, pool)
    dropped = torch.zeros(1, dtype=torch.int32, device="cuda")
    k = torch.randn(2, 1, 1, D, device="cuda")
    # sequence 0 lands on page 3 (in range), sequence 1 on page 9 (out of range), then a negative position
    append_tokens(pool, k, k, torch.tensor([3 * PS, 9 * PS], dtype=torch.int32, device="cuda"), tags, _tag_map(),
                  stage, dropped=dropped)
    append_tokens(pool, k, k, torch.tensor([0, -1], dtype=torch.int32, device="cuda"), tags, _tag_map(), stage,
                  dropped=dropped)
    torch.cuda.synchronize()
    assert int(dropped) == 2
    page = np.zeros((PS, D), np.float32)
    page[0] = k[0, 0, 0].cpu().numpy()
    _assert_page(pool, "k", "INT8", 3, page, "page")
    _assert_page(pool, "k", "INT8", 0, page, "page")


@pytest.mark.parametrize("mode", ["page", "group32", "channel"])
def test_convert_pages_matches_oracle(mode):
    """Each page re-quantised from its dequantised contents; tags rewritten."""
    from intent_attention import PagePool, convert_pages
    g = np.random.default_rng(40 + len(mode))
    P, PS, D = 60, 16, 128
    pool = PagePool.allocate(P, PS, D, FORMATS, mode, "cuda", zero=True)
    x = (g.standard_normal((P, PS, D)) * 2).astype(np.float32)
    old = g.integers(0, 5, size=P)
    old_names = [FORMATS[i] for i in old]
    xt = torch.from_numpy(x).cuda()
    pool.quantize_(xt, -xt, old_names)
    tags = torch.tensor([CODE[f] for f in old_names], dtype=torch.uint8, device="cuda")
    ids = g.permutation(P)[:45]
    new = [FORMATS[int(i)] for i in g.integers(0, 5, size=ids.size)]
    before = {plane: _snapshot(pool, plane) for plane in ("k", "v")}
    convert_pages(pool, torch.from_numpy(ids.astype(np.int32)).cuda(), new, tags, _tag_map(),
                  {f: CODE[f] for f in FORMATS})
    torch.cuda.synchronize()
    tags_after = tags.cpu().numpy()
    for pid, nf in zip(ids, new):
        of = old_names[pid]
        assert tags_after[pid] == CODE[nf]
        for plane, sign in (("k", 1.0), ("v", -1.0)):
            src = oq.quantize_pages((sign * x[pid])[None], ORACLE_NAME[of], mode)
            recon = src["recon"][0]
            if of == "F16":
                recon = src["codes"][0].astype(np.float32)
            if nf == of:
                _assert_unchanged(pool, plane, nf, pid, before[plane])
            else:
                _assert_page(pool, plane, nf, pid, recon, mode)
    untouched = np.setdiff1d(np.arange(P), ids)
    assert (tags_after[untouched] == np.array([CODE[old_names[i]] for i in untouched])).all()


def _snapshot(pool, plane):
    """Copies of every pool array of one plane that the pool holds."""
    names = ("f16", "fp8", "i8", "i4", "i4r", "scale", "res_scale")
    return {n: getattr(pool, f"{plane}_{n}").cpu().numpy().copy() for n in names
            if getattr(pool, f"{plane}_{n}") is not None}


def _assert_unchanged(pool, plane, fmt, pid, snap):
    for n, arr in snap.items():
        np.testing.assert_array_equal(getattr(pool, f"{plane}_{n}")[pid].cpu().numpy(), arr[pid])


def test_convert_to_skip_retags_and_missing_pool_rejects():
    from intent_attention import PagePool, convert_pages
    P, PS, D = 6, 16, 64
    pool = PagePool.allocate(P, PS, D, ["F16", "INT8"], "page", "cuda", zero=True)
    x = torch.randn(P, PS, D, device="cuda")
    pool.quantize_(x, x, ["F16"] * P)
    tags = torch.full((P,), CODE["F16"], dtype=torch.int32, device="cuda")
    rejected = torch.zeros(1, dtype=torch.int32, device="cuda")
    snap = _snapshot(pool, "k")
    convert_pages(pool, torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda"), ["SKIP", "INT4", "INT8"], tags,
                  _tag_map(), {"SKIP": 0, "INT4": CODE["INT4"], "INT8": CODE["INT8"]}, rejected=rejected)
    torch.cuda.synchronize()
    assert tags.cpu().tolist()[:3] == [0, CODE["F16"], CODE["INT8"]]
    assert int(rejected) == 1
    _assert_unchanged(pool, "k", "F16", 1, snap)
    _assert_page(pool, "k", "INT8", 2, pool.k_f16[2].float().cpu().numpy(), "page")


def test_demote_then_decode_reads_the_new_format():
    """After demoting pages F16 -> INT8 the decode equals the oracle decode
    over the oracle's re-quantised pages."""
    from intent_attention import PagePool, convert_pages, paged_decode
    g = np.random.default_rng(9)
    B, Hq, PS, D, n = 2, 4, 16, 128, 12
    P = B * n
    pool = PagePool.allocate(P, PS, D, FORMATS, "page", "cuda", zero=True)
    x = g.standard_normal((P, PS, D)).astype(np.float32)
    y = g.standard_normal((P, PS, D)).astype(np.float32)
    pool.quantize_(torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda(), ["F16"] * P)
    tags = torch.full((P,), CODE["F16"], dtype=torch.uint8, device="cuda")
    demote = np.arange(0, P, 3).astype(np.int32)
    convert_pages(pool, torch.from_numpy(demote).cuda(), ["INT8"] * demote.size, tags, _tag_map(),
                  {"INT8": CODE["INT8"]})
    table = torch.arange(P, dtype=torch.int32, device="cuda").view(B, 1, n)
    q = torch.randn(B, Hq, D, device="cuda")
    out = paged_decode(q, pool, table, None, tags, _tag_map())
    torch.cuda.synchronize()
    # oracle pools: F16 pages as half, demoted pages as INT8 of the half values
    xk, xv = x.astype(np.float16).astype(np.float32), y.astype(np.float16).astype(np.float32)
    k8 = oq.quantize_pages(xk[demote], "INT8", "page")
    v8 = oq.quantize_pages(xv[demote], "INT8", "page")
    kd, vd = xk.copy(), xv.copy()
    kd[demote], vd[demote] = k8["recon"], v8["recon"]
    qn = q.cpu().numpy()
    ref = np.zeros((B, Hq, D), np.float32)
    for b in range(B):
        ks = kd[b * n:(b + 1) * n].reshape(-1, D)
        vs = vd[b * n:(b + 1) * n].reshape(-1, D)
        s = qn[b] @ ks.T / np.sqrt(D)
        s = s - s.max(-1, keepdims=True)
        p = np.exp(s)
        ref[b] = (p / p.sum(-1, keepdims=True)) @ vs
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)

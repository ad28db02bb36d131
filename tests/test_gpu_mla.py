"""GPU parity of the MLA decode (``iak_mla_decode``): the CUDA-core kernel and
the tcgen05 / TMEM kernel against the numpy oracle (``oracle/mla.py``), and
the ``mla_decode_triton`` drop-in against outputs of the reference itself.

Tolerance: atol 2e-3 / rtol 1e-2 on fp32-accumulated
outputs.  FP8 latent pages use the reference's FP8 rule (per-page scale =
max(absmax/127, 1e-8), code = e4m3(x / scale))."""

import numpy as np
import pytest
import torch

import inputs as gi
from intent_attention.split_kv import block_floats, block_views, merge_partial_blocks
from intent_attention.triton_mla_decode import make_mla_tag_map, mla_decode_triton, mla_paged_decode
from oracle import mla as omla
from oracle import quant as oq

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
TAGS = make_mla_tag_map({0: "DENSE", 1: "FP8", 2: "SKIP"})


def make_mla_case(seed, B=3, H=128, Dqk=576, Dv=512, PS=64, NP=48, W=12, dense_dtype=torch.bfloat16,
                  q_dtype=torch.bfloat16, probs=(0.3, 0.6, 0.1), counts="ragged", pad_frac=0.1, shared=False):
    g = np.random.default_rng(seed)
    lat = g.standard_normal((NP, PS, Dqk)).astype(np.float32)
    dense = torch.from_numpy(lat).to(dense_dtype)
    scale = np.maximum(np.abs(lat).reshape(NP, -1).max(1) / 127.0, 1e-8).astype(np.float32)
    codes = oq.f32_to_e4m3(lat / scale[:, None, None])
    tags = g.choice([0, 1, 2], size=NP, p=list(probs)).astype(np.uint8)
    rows = 1 if shared else B
    table = np.stack([g.permutation(NP)[:W] for _ in range(rows)]).astype(np.int32)
    table = np.where(g.random(table.shape) < pad_frac, -1, table).astype(np.int32)
    if counts == "ragged":
        cnt = g.integers(0, W + 1, size=B).astype(np.int32)
        cnt[0] = W
    else:
        cnt = None
    q = torch.from_numpy(g.standard_normal((B, H, Dqk)).astype(np.float32)).to(q_dtype)
    dev = "cuda"
    case = dict(q=q.to(dev), table=torch.from_numpy(table if not shared else table[0]).to(dev),
                counts=None if cnt is None else torch.from_numpy(cnt).to(dev), dense=dense.to(dev),
                fp8=torch.from_numpy(codes).to(dev), scale=torch.from_numpy(scale).to(dev),
                tags=torch.from_numpy(tags).to(dev), Dv=Dv)
    np_table = np.broadcast_to(table, (B, W)) if shared else table
    case["oracle"] = lambda sm: omla.mla_paged_decode(q.float().numpy(), np_table, cnt, tags,
                                                      {"bf16": dense.float().numpy(), "fp8": codes}, scale, Dv, sm)
    return case


def run(case, kernel="auto", num_splits=0, out_dtype=torch.float32, sm_scale=None, partial=None):
    return mla_paged_decode(case["q"], case["table"], case["counts"], dense_pages=case["dense"],
                            fp8_pages=case["fp8"], fp8_scale=case["scale"], page_tags=case["tags"], tag_map=TAGS,
                            d_v=case["Dv"], sm_scale=sm_scale, out_dtype=out_dtype, num_splits=num_splits,
                            kernel=kernel, partial=partial)


def _close(got, ref, atol=ATOL, rtol=RTOL):
    np.testing.assert_allclose(got.float().cpu().numpy(), ref, atol=atol, rtol=rtol)


# --------------------------------------------------------------- tcgen05 kernel
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_tensor_kernel_matches_oracle(splits):
    case = make_mla_case(11 + splits)
    sm = 1.0 / np.sqrt(576)
    _close(run(case, "tensor", splits), case["oracle"](sm))


@pytest.mark.parametrize("H", [16, 100])
def test_tensor_kernel_fewer_heads(H):
    case = make_mla_case(21 + H, B=2, H=H, NP=30, W=9)
    _close(run(case, "tensor"), case["oracle"](1.0 / np.sqrt(576)))


def test_tensor_kernel_f16_pages_and_q_and_page_size_128():
    case = make_mla_case(31, B=2, PS=128, NP=40, W=12, dense_dtype=torch.float16, q_dtype=torch.float16)
    _close(run(case, "tensor"), case["oracle"](1.0 / np.sqrt(576)))


def test_tensor_kernel_single_format_pages():
    for probs in ((1.0, 0.0, 0.0), (0.0, 1.0, 0.0)):
        case = make_mla_case(41, B=2, probs=probs, counts=None, pad_frac=0.0)
        _close(run(case, "tensor"), case["oracle"](1.0 / np.sqrt(576)))


def test_tensor_kernel_large_scores_lazy_rescale():
    # a larger softmax scale makes row maxima grow across tiles (O rescaled in TMEM)
    case = make_mla_case(51, B=2, NP=40, W=20, counts=None)
    sm = 0.25
    _close(run(case, "tensor", sm_scale=sm), case["oracle"](sm))


def test_tensor_kernel_empty_rows_and_all_skip():
    case = make_mla_case(61, B=3, NP=20, W=6)
    case["counts"][1] = 0
    case["tags"][:] = 2                       # every page SKIP -> zeros
    out = run(case, "tensor")
    assert torch.count_nonzero(out) == 0


def test_tensor_kernel_bf16_out_matches_generic():
    case = make_mla_case(71, B=2, NP=40, W=16)
    a = run(case, "tensor", out_dtype=torch.bfloat16).float()
    b = run(case, "generic").float()
    np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), atol=1e-2, rtol=1e-2)


def test_tensor_kernel_partial_export_merges_to_full():
    case = make_mla_case(81, B=2, NP=40, W=16, counts="ragged")
    B, H, Dv = 2, 128, 512
    rows = B * H
    blocks = torch.empty((2, block_floats(rows, Dv)), dtype=torch.float32, device="cuda")
    full_table = case["table"]
    cut = 7
    for i, sl in enumerate((slice(0, cut), slice(cut, None))):
        t = full_table[:, sl].contiguous()
        c = None if case["counts"] is None else torch.clamp(case["counts"] - (0 if i == 0 else cut), 0, t.shape[1])
        if i == 0 and case["counts"] is not None:
            c = torch.clamp(case["counts"], 0, cut)
        sub = dict(case, table=t, counts=c.to(torch.int32) if c is not None else None)
        run(sub, "tensor", partial=block_views(blocks[i], rows, Dv))
    out = merge_partial_blocks(blocks, rows, Dv).view(B, H, Dv)
    _close(out, case["oracle"](1.0 / np.sqrt(576)))


def test_tensor_kernel_rejects_other_shapes():
    case = make_mla_case(91, B=1, H=8, Dqk=128, Dv=128, PS=16, NP=10, W=4)
    with pytest.raises(RuntimeError, match="tensor-core MLA"):
        run(case, "tensor")
    case = make_mla_case(92, B=1, H=8, PS=32, NP=10, W=4)      # pages must hold whole 64-token chunks
    with pytest.raises(RuntimeError, match="tensor-core MLA"):
        run(case, "tensor")
    # the automatic choice falls back to the CUDA-core kernel for such shapes
    _close(run(case), case["oracle"](1.0 / np.sqrt(576)))


# --------------------------------------------------------------- CUDA-core kernel
@pytest.mark.parametrize("shape", [(2, 5, 96, 64, 16), (3, 16, 576, 512, 64), (1, 3, 64, 64, 8)])
@pytest.mark.parametrize("splits", [0, 1, 4])
def test_generic_kernel_matches_oracle(shape, splits):
    B, H, Dqk, Dv, PS = shape
    case = make_mla_case(100 + Dqk + splits, B=B, H=H, Dqk=Dqk, Dv=Dv, PS=PS, NP=24, W=10)
    _close(run(case, "generic", splits), case["oracle"](1.0 / np.sqrt(Dqk)))


def test_generic_kernel_fp32_dense_pages_shared_table():
    case = make_mla_case(111, B=3, H=4, Dqk=64, Dv=64, PS=16, NP=12, W=5, dense_dtype=torch.float32,
                         q_dtype=torch.float32, shared=True, counts=None, probs=(1.0, 0.0, 0.0))
    _close(run(case), case["oracle"](1.0 / 8.0), atol=1e-5, rtol=1e-5)


# --------------------------------------------------------------- reference drop-in
@pytest.mark.parametrize("ps", [8, 16, 32, 64])
def test_mla_decode_triton_matches_reference_cpu(golden, ps):
    g = golden("mla_golden.npz")
    qa = gi.normal(90 + ps, (2, 3, 64)); C = gi.normal(91 + ps, (4 * ps, 64)); W = gi.normal(92 + ps, (64, 128))
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).float().cuda()
    out = mla_decode_triton(T(qa), T(C), T(W), torch.tensor([2, 0, 3], dtype=torch.int32, device="cuda"),
                            page_size=ps)
    assert out.dtype == torch.float32 and out.shape == (2, 3, 128)
    np.testing.assert_allclose(out.cpu().numpy(), g[f"cpu_ps{ps}"], atol=2e-3, rtol=1e-2)


def test_mla_decode_triton_empty_table_is_zero_and_cpu_raises():
    q = torch.randn(1, 1, 64, device="cuda"); C = torch.randn(64, 64, device="cuda")
    W = torch.randn(64, 128, device="cuda")
    out = mla_decode_triton(q, C, W, torch.tensor([], dtype=torch.int32, device="cuda"))
    assert out.shape == (1, 1, 128) and torch.count_nonzero(out) == 0
    with pytest.raises(RuntimeError, match="CUDA"):
        mla_decode_triton(q.cpu(), C.cpu(), W.cpu(), torch.tensor([0], dtype=torch.int32))


def test_mla_sparse_reference_pipeline(golden):
    # mla.py:61-92 (q @ W_QK absorption, then decode, then @ W_VO) through the drop-in
    g = golden("mla_golden.npz")
    lat = gi.normal(95, (4, 16, 64))
    W_QK = gi.normal(96, (4 * 64, 64)); W_VO = gi.normal(97, (64, 256))
    q = gi.normal(98, (2, 4, 4, 64))
    q_abs = q.transpose(0, 2, 1, 3).reshape(2, 4, 256) @ W_QK
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x)).float().cuda()
    out = mla_decode_triton(T(q_abs), T(lat.reshape(64, 64)), T(W_VO),
                            torch.arange(4, dtype=torch.int32, device="cuda"), page_size=16)
    # the reference returns float16 (large-magnitude outputs: compare at fp16 resolution)
    np.testing.assert_allclose(out.half().float().cpu().numpy(), g["sparse_ref"], atol=0.25, rtol=2e-3)

"""iak_decode_noalloc: the decode entry point that allocates nothing.

Some callers of this library cannot allocate device memory while they decode:
serving engines that reserve all of HBM up front (most of it for the KV cache)
and forbid allocation on the decode path, and hosts that reach the C ABI
through an FFI with only borrowed device pointers and no allocator.  For them
iak_decode_noalloc keeps its split-KV scratch in a static device array.  These
tests call it through the C ABI and compare it with iak_decode (which takes a
caller-allocated workspace) and with the numpy oracle on the same inputs, on
two calls in a row: a large decode with many splits, then a smaller one with
fewer rows and splits, so that partials left in the shared scratch by the
first call would show in the second.  Both kernels are covered: the
tensor-core path (per-page scales) and the CUDA-core path (per-channel scales,
which uses the scratch when it splits the page lists).
"""

import ctypes

import numpy as np
import pytest
import torch

from gpu_cases import make_case, run_oracle, tag_map_for
from intent_attention import _native as N
from intent_attention.paged import _decode_structs, _stream

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _args(case, q, out, splits):
    return _decode_structs(q, case["pool"], case["table"], case["counts"], case["tags"], tag_map_for(case["formats"]),
                           0, None, out, None, splits)


def _both(case, splits):
    """(iak_decode output, iak_decode_noalloc output) of one case, fp32."""
    L = N.lib()
    q = case["q"]
    stream = _stream(q.device)
    out_ref = torch.full(q.shape, float("nan"), dtype=torch.float32, device="cuda")
    out_na = torch.full(q.shape, float("nan"), dtype=torch.float32, device="cuda")
    P, A = _args(case, q, out_ref, splits)
    nbytes = ctypes.c_size_t(0)
    N.check(L.iak_decode_workspace_size(ctypes.byref(P), ctypes.byref(A), ctypes.byref(nbytes)), "ws size")
    assert 0 < nbytes.value <= N.NOALLOC_SCRATCH_BYTES      # the split-KV scratch is really used
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    N.check(L.iak_decode(ctypes.byref(P), ctypes.byref(A), ws.data_ptr(), nbytes.value, stream), "iak_decode")
    P2, A2 = _args(case, q, out_na, splits)
    N.check(L.iak_decode_noalloc(ctypes.byref(P2), ctypes.byref(A2), stream), "iak_decode_noalloc")
    torch.cuda.synchronize()
    return out_ref.cpu().numpy(), out_na.cpu().numpy()


@pytest.mark.parametrize("mode", ["page", "channel"])
def test_noalloc_decode_matches_allocating_decode_on_two_calls(mode):
    big = make_case(4242, B=4, Hq=16, Ht=4, D=128, W=300, NP=900, counts="full", scale_mode=mode)
    small = make_case(4243, B=1, Hq=8, Ht=2, D=128, W=120, NP=300, counts="ragged", scale_mode=mode)
    for case, splits in ((big, 6), (small, 2)):
        ref, na = _both(case, splits)
        np.testing.assert_allclose(na, ref, atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(na, run_oracle(case), atol=ATOL, rtol=RTOL)


def test_noalloc_rejects_scratch_beyond_its_maximum():
    case = make_case(7, B=1, Hq=8, Ht=1, D=128, W=16, NP=32, counts="full")
    B, Hq, Ht, W = 64, 64, 8, 8192
    q = torch.zeros((B, Hq, 128), dtype=torch.bfloat16, device="cuda")
    out = torch.empty(q.shape, dtype=torch.float32, device="cuda")
    table = torch.full((B, Ht, W), -1, dtype=torch.int32, device="cuda")
    counts = torch.full((B, Ht), W, dtype=torch.int32, device="cuda")
    P, A = _decode_structs(q, case["pool"], table, counts, case["tags"], tag_map_for(case["formats"]), 0, None, out,
                           None, 64)
    st = N.lib().iak_decode_noalloc(ctypes.byref(P), ctypes.byref(A), _stream(q.device))
    assert st == N.IAK_ERR_WORKSPACE
    assert b"static scratch" in N.lib().iak_last_error()

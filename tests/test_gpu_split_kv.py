"""GPU parity of the sequence-sharded split-KV decode.

One GPU emulates N ranks: every rank's page range (``shard_page_lists``) is
decoded into its own partial block through the C ABI, the blocks are stacked
as an all-gather would leave them and merged with ``iak_merge_partial_blocks``;
the result must match the oracle's unsharded decode (atol 2e-3 / rtol 1e-2).
With two or more GPUs the same path also runs as real ranks over NCCL
(``split_kv_nccl_worker.py``, launched with torch.distributed.run).
"""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from gpu_cases import make_case, run_gpu, run_oracle, tag_map_for
from intent_attention.split_kv import (SequenceShardedDecoder, block_floats, decode_partial_block,
                                       merge_partial_blocks, shard_page_lists)

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
HERE = os.path.dirname(os.path.abspath(__file__))


def _sharded(case, world, kernel="auto", out_dtype=torch.float32):
    q = case["q"]
    B, Hq, D = q.shape
    rows = B * Hq
    blocks = torch.empty((world, block_floats(rows, D)), dtype=torch.float32, device=q.device)
    for r in range(world):
        lt, lc = shard_page_lists(case["table"], case["counts"], r, world)
        decode_partial_block(q, case["pool"], lt, lc, case["tags"], tag_map_for(case["formats"]), block=blocks[r],
                             kernel=kernel)
    return merge_partial_blocks(blocks, rows, D, out_dtype=out_dtype).view(B, Hq, D)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("kernel", ["tensor", "generic"])
def test_sharded_blocks_merge_to_unsharded(world, kernel):
    case = make_case(900 + world, B=3, Hq=32, Ht=8, W=120, NP=1500, formats=("F16", "FP8", "INT8", "INT4"))
    got = _sharded(case, world, kernel)
    np.testing.assert_allclose(got.cpu().numpy(), run_oracle(case), atol=ATOL, rtol=RTOL)


def test_sharded_rows_with_empty_shards_are_zero_or_exact():
    # counts 0 / 1 rows: most ranks hold no page of the row, their blocks carry l = 0
    case = make_case(911, B=2, Hq=16, Ht=4, W=9, NP=300, formats=("F16", "INT8"), counts="ragged")
    case["counts"][0, 1] = 0
    case["counts"][1, 2] = 1
    case["np_counts"] = case["counts"].cpu().numpy()
    got = _sharded(case, 8)
    ref = run_oracle(case)
    np.testing.assert_allclose(got.cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
    assert (got[0, 4:8] == 0).all()


def test_sharded_matches_single_device_decode_bf16_out():
    case = make_case(921, B=4, Hq=32, Ht=8, W=200, NP=2500, formats=("F16", "FP8", "INT8", "INT4"), counts="full")
    got = _sharded(case, 4, out_dtype=torch.bfloat16)
    ref = run_gpu(case, out_dtype=torch.float32)
    np.testing.assert_allclose(got.float().cpu().numpy(), ref.cpu().numpy(), atol=1e-2, rtol=1e-2)


def test_single_rank_decoder_is_plain_decode():
    case = make_case(931, B=2, Hq=8, Ht=2, W=64, NP=400)
    dec = SequenceShardedDecoder()
    assert dec.world == 1
    out = dec.decode(case["q"], case["pool"], case["table"], case["counts"], case["tags"],
                     tag_map_for(case["formats"]))
    np.testing.assert_allclose(out.float().cpu().numpy(), run_oracle(case), atol=1e-2, rtol=1e-2)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_two_ranks_match_oracle(tmp_path):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", RESULT_DIR=str(tmp_path))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29631", os.path.join(HERE, "split_kv_nccl_worker.py")]
    subprocess.run(["timeout", "-k", "30", "300"] + cmd, check=True, env=env, cwd=os.path.dirname(HERE))
    for r in range(2):
        assert float(np.load(os.path.join(tmp_path, f"rank{r}.npy"))[0]) == 0.0


# ------------------------------------------------------------------ peer-memory exchange
def test_p2p_single_rank_decoder_is_plain_decode():
    case = make_case(951, B=2, Hq=16, Ht=4, W=80, NP=500)
    dec = SequenceShardedDecoder(transport="p2p")
    for _ in range(3):       # both parities and a reuse
        out = dec.decode(case["q"], case["pool"], case["table"], case["counts"], case["tags"],
                         tag_map_for(case["formats"]), out=torch.empty(case["q"].shape, device="cuda"))
    dec._x.check()
    np.testing.assert_allclose(out.cpu().numpy(), run_oracle(case), atol=ATOL, rtol=RTOL)
    dec.close()


def test_p2p_merge_wait_times_out_with_status_when_a_peer_never_arrives():
    # a two-rank descriptor whose "peer" area is this rank's own: rank 1's flag is never raised,
    # so the bounded wait must give up, report the timeout in the status word and leave the
    # context usable
    import ctypes
    from intent_attention import _native as N
    L = N.lib()
    rows, D = 8, 64
    nbytes = ctypes.c_size_t(0)
    N.check(L.iak_exchange_area_bytes(2, rows, D, ctypes.byref(nbytes)), "area")
    area, handle = ctypes.c_void_p(0), (ctypes.c_uint8 * 64)()
    N.check(L.iak_ipc_alloc(nbytes.value, ctypes.byref(area), handle), "alloc")
    try:
        x = N.PeerExchange()
        x.areas[0] = x.areas[1] = area.value
        x.rank, x.world, x.rows, x.head_dim = 0, 2, rows, D
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        out = torch.zeros((rows, D), device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        N.check(L.iak_exchange_push(ctypes.byref(x), s), "push")
        N.check(L.iak_exchange_merge(ctypes.byref(x), out.data_ptr(), N.DT_F32, D, status.data_ptr(), 200_000, s),
                "merge")
        torch.cuda.synchronize()
        assert int(status.item()) == 1
        # the context is still usable
        assert float((torch.ones(4, device="cuda") * 2).sum().item()) == 8.0
    finally:
        L.iak_ipc_free(area.value)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_exchange_emulated_ranks_two_steps(world):
    """iak_decode_exchange: the decode kernel stores each row's partial into every
    rank's receive slot and raises its flag; iak_exchange_merge then merges.  One GPU
    emulates `world` ranks with one exchange area each.  Every rank's decode is launched
    (and completes, in stream order) before any merge, so no kernel waits on another
    that is still running: the merges find every flag already raised.  Two steps cover
    both parities of the receive arrays."""
    import ctypes
    from intent_attention import _native as N
    from intent_attention.split_kv import decode_exchange
    L = N.lib()
    case = make_case(960 + world, B=2, Hq=16, Ht=4, W=90, NP=900, formats=("F16", "FP8", "INT8", "INT4"))
    B, Hq, D = case["q"].shape
    rows = B * Hq
    nbytes = ctypes.c_size_t(0)
    N.check(L.iak_exchange_area_bytes(world, rows, D, ctypes.byref(nbytes)), "area bytes")
    areas = []
    for _ in range(world):
        a, h = ctypes.c_void_p(0), (ctypes.c_uint8 * 64)()
        N.check(L.iak_ipc_alloc(nbytes.value, ctypes.byref(a), h), "alloc")
        areas.append(a.value)

    class _X:       # the attribute decode_exchange reads
        pass

    try:
        xs = []
        for r in range(world):
            x = N.PeerExchange()
            for j, a in enumerate(areas):
                x.areas[j] = a
            x.rank, x.world, x.rows, x.head_dim = r, world, rows, D
            holder = _X()
            holder.x = x
            xs.append(holder)
        ref = run_oracle(case)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        for step in range(2):
            q = case["q"] if step == 0 else (case["q"].float() * 0.5).to(case["q"].dtype)
            ref_q = ref if step == 0 else run_oracle(dict(case, np_q=q.float().cpu().numpy()))
            for r in range(world):
                t_r, c_r = shard_page_lists(case["table"], case["counts"], r, world)
                decode_exchange(q, case["pool"], t_r, c_r, case["tags"], tag_map_for(case["formats"]), xs[r])
            for r in range(world):
                out = torch.full((rows, D), float("nan"), device="cuda")
                N.check(L.iak_exchange_merge(ctypes.byref(xs[r].x), out.data_ptr(), N.DT_F32, D, status.data_ptr(),
                                             2_000_000, s), "merge")
                torch.cuda.synchronize()
                np.testing.assert_allclose(out.view(B, Hq, D).cpu().numpy(), ref_q, atol=ATOL, rtol=RTOL)
        assert int(status.item()) == 0
    finally:
        torch.cuda.synchronize()
        for a in areas:
            L.iak_ipc_free(a)

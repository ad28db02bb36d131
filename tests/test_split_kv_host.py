"""Host side of the sequence-sharded split-KV decode (no GPU): range cutting,
the partial-block layout, and a world-size-2 gloo exchange + merge checked
against the oracle's unsharded decode."""

import os
import socket

import numpy as np
import pytest
import torch

from intent_attention.split_kv import block_floats, block_views, shard_bounds, shard_page_lists


@pytest.mark.parametrize("n", [0, 1, 7, 64, 1000])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_bounds_partition(n, world):
    spans = [shard_bounds(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1 and sorted(sizes, reverse=True) == sizes


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(10, 0, 0)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_page_lists_concatenate_to_original(world):
    g = np.random.default_rng(world)
    B, Ht, W = 3, 2, 29
    table = torch.from_numpy(g.integers(-1, 500, size=(B, Ht, W)).astype(np.int32))
    counts = torch.from_numpy(g.integers(0, W + 1, size=(B, Ht)).astype(np.int32))
    counts[0, 0], counts[0, 1] = W, 0
    parts = [shard_page_lists(table, counts, r, world) for r in range(world)]
    for lt, lc in parts:
        assert lt.shape == (B, Ht, (W + world - 1) // world) and lt.dtype == torch.int32
    for b in range(B):
        for h in range(Ht):
            got = np.concatenate([lt[b, h, :lc[b, h]].numpy() for lt, lc in parts])
            np.testing.assert_array_equal(got, table[b, h, :counts[b, h]].numpy())
            for lt, lc in parts:
                assert (lt[b, h, lc[b, h]:] == -1).all()
    # counts=None means every slot
    full = [shard_page_lists(table, None, r, world) for r in range(world)]
    np.testing.assert_array_equal(np.concatenate([lt[1, 1, :lc[1, 1]].numpy() for lt, lc in full], 0),
                                  table[1, 1].numpy())


def test_block_views_layout():
    rows, D = 5, 4
    blk = torch.arange(block_floats(rows, D), dtype=torch.float32)
    m, l, acc = block_views(blk, rows, D)
    assert m.tolist() == list(range(rows)) and l.tolist() == list(range(rows, 2 * rows))
    assert acc.shape == (rows, D) and acc[1, 0].item() == 2 * rows + D
    with pytest.raises(ValueError):
        block_views(blk[:-1], rows, D)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_exchange_and_merge_match_unsharded_oracle(tmp_path, world):
    import torch.multiprocessing as mp
    import split_kv_workers as wk
    port = _free_port()
    mp.start_processes(wk.gloo_rank, args=(world, port, 77, str(tmp_path)), nprocs=world, start_method="spawn")
    for r in range(world):
        err = float(np.load(os.path.join(tmp_path, f"rank{r}.npy"))[0])
        # the blocks carry fp32 (m, l, acc): the merge equals the float64 oracle to fp32 rounding
        assert err < 1e-6, f"rank {r}: merged sharded decode differs from the unsharded oracle by {err}"

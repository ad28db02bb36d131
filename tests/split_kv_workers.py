"""Rank bodies for the sequence-sharded decode tests (test infrastructure).

``gloo_rank``: one CPU rank of a world-size-N ``gloo`` group.  Each rank
computes the partial block of its sequence range with the numpy oracle,
exchanges blocks through ``SequenceShardedDecoder.exchange`` and merges them
with the oracle's LSE merge; the result must equal the oracle's unsharded
decode.  It checks the host side of the sharded path (range cutting, block
layout, rank order of the exchange) without a GPU.
"""

from __future__ import annotations

import os

import numpy as np
import torch


def make_numpy_case(seed, B=2, Hq=8, Ht=2, D=64, PS=16, W=37, NP=160):
    from oracle import quant as oq
    g = np.random.default_rng(seed)
    k = g.standard_normal((NP, PS, D)).astype(np.float32)
    v = g.standard_normal((NP, PS, D)).astype(np.float32)
    pools = {"k_f16": k.astype(np.float16), "v_f16": v.astype(np.float16)}
    rk, rv = oq.quantize_pages(k, "INT8", "page"), oq.quantize_pages(v, "INT8", "page")
    pools["k_i8"], pools["v_i8"] = rk["codes"], rv["codes"]
    scales = {"k_scale": rk["scale"], "v_scale": rv["scale"]}
    tags = g.choice([0, 1, 2], size=NP, p=[0.45, 0.45, 0.1]).astype(np.int64)   # F16 / INT8 / SKIP
    table = np.stack([np.stack([g.permutation(NP)[:W] for _ in range(Ht)]) for _ in range(B)]).astype(np.int32)
    table = np.where(g.random(table.shape) < 0.1, -1, table).astype(np.int32)
    counts = g.integers(0, W + 1, size=(B, Ht)).astype(np.int32)
    counts[0, 0] = W
    counts[-1, -1] = 1      # a row whose pages land on rank 0 only
    q = g.standard_normal((B, Hq, D)).astype(np.float32)
    return dict(q=q, table=table, counts=counts, tags=tags, pools=pools, scales=scales)


TAG_MAP = {0: "F16", 1: "INT8", 2: "SKIP"}


def oracle_partial_block(case, table, counts):
    from oracle import decode as odec
    _, (m, l, acc) = odec.paged_decode(case["q"], table, counts, case["tags"], TAG_MAP, case["pools"],
                                       case["scales"], "page", return_partials=True)
    B, Hq, D = case["q"].shape
    rows = B * Hq
    block = np.empty(rows * (D + 2), np.float32)
    block[:rows] = np.where(l.reshape(-1) > 0, m.reshape(-1), -np.inf)
    block[rows:2 * rows] = l.reshape(-1)
    block[2 * rows:] = acc.reshape(-1)
    return block


def gloo_rank(rank, world, port, seed, result_dir):
    import torch.distributed as dist
    from intent_attention.split_kv import SequenceShardedDecoder, block_views, shard_page_lists
    from oracle import decode as odec
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = make_numpy_case(seed)
        B, Hq, D = case["q"].shape
        rows = B * Hq
        lt, lc = shard_page_lists(torch.from_numpy(case["table"]), torch.from_numpy(case["counts"]), rank, world)
        block = torch.from_numpy(oracle_partial_block(case, lt.numpy(), lc.numpy()))
        dec = SequenceShardedDecoder()
        assert dec.world == world
        blocks = dec.exchange(block).view(world, -1)
        ms, ls, accs = zip(*(block_views(blocks[r], rows, D) for r in range(world)))
        merged = odec.lse_merge(torch.stack(ms, -1).double().numpy(), torch.stack(ls, -1).double().numpy(),
                                torch.stack(accs, -2).double().numpy())
        full = odec.paged_decode(case["q"], case["table"], case["counts"], case["tags"], TAG_MAP, case["pools"],
                                 case["scales"], "page").reshape(rows, D)
        err = float(np.abs(merged - full).max())
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([err]))
    finally:
        dist.destroy_process_group()

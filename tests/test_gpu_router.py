"""GPU parity of the device router (iak_route_pages) with the reference's
host routing: BlockRouter.route_layout + selected_page_ids + the page
precision map of routing_to_kernel_metadata, then page-table packing.

Page ids, counts, precisions and tags are integer outputs: bit-exact.
"""

import math

import numpy as np
import random

import pytest
import torch

from intent_attention import (BlockLayout, BlockPolicy, BlockRouter, IntentQuantizer, KVPrecision, RouterConfig,
                              SemanticBlock, routing_to_kernel_metadata)
from intent_attention import _native as N
from intent_attention.device_router import (PRECISION_CODES, LayoutBatch, encode_layouts, route_layouts,
                                            route_pages)

pytestmark = pytest.mark.gpu

POLICIES = list(BlockPolicy)
EDGE_SCORES = [0.0, 0.35, 0.40, 0.75, 1.0, 0.3499999, 0.35000001, 0.7499999]


def _expected(router, layout, total, ps):
    """Reference-semantics page list and per-page precision codes for one sequence."""
    routed = router.route_layout(layout, total)
    ids = router.selected_page_ids(routed, ps)
    meta = routing_to_kernel_metadata(routed, ps)
    precs = [PRECISION_CODES[KVPrecision(meta["block_precision_by_page"][str(p)])] for p in ids]
    return ids, precs


def _random_layout(rng, n_blocks, ps, score_pool=None):
    blocks, t = [], rng.randrange(0, 2 * ps)
    for i in range(n_blocks):
        length = rng.choice([1, 2, ps - 1 if ps > 1 else 1, ps, ps + 1, 3 * ps, rng.randrange(1, 4 * ps + 1)])
        pol = rng.choice(POLICIES)
        if pol == BlockPolicy.ATTEND or rng.random() < 0.6:
            s = rng.choice(score_pool) if score_pool and rng.random() < 0.5 else \
                (rng.choice(EDGE_SCORES) if rng.random() < 0.3 else round(rng.random(), rng.choice([2, 3, 17])))
        else:
            s = None
        blocks.append(SemanticBlock(f"b{i}", t, t + length, pol, score=s))
        t += length + rng.choice([0, 0, 0, 1, ps])
    return BlockLayout(blocks), t


def _check(out, router, layouts, totals, ps, W, Ht, bases):
    pt, pc, ns, pp = (x.cpu() for x in (out.page_table, out.page_counts, out.num_selected, out.page_prec))
    for b, (layout, total) in enumerate(zip(layouts, totals)):
        ids, precs = _expected(router, layout, total, ps)
        n = len(ids)
        k = min(n, W)
        assert int(ns[b]) == n, b
        for h in range(Ht):
            base = int(bases[b, h]) if bases is not None else 0
            assert int(pc[b, h]) == k
            assert pt[b, h, :k].tolist() == [base + p for p in ids[:k]], (b, h)
            assert (pt[b, h, k:] == -1).all()
        assert pp[b, :k].tolist() == precs[:k], b
        assert (pp[b, k:] == N.PREC_SKIP).all()


@pytest.mark.parametrize("seed", range(12))
def test_random_layouts_match_host_router(seed):
    rng = random.Random(seed)
    ps = rng.choice([1, 3, 16, 64])
    mp = rng.choice([0.0, 0.3, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0, rng.random()])
    cfg = RouterConfig(top_k_blocks=rng.choice([0, 1, 3, 8, 50, -2]), score_threshold=rng.choice([0.35, 0.0, 0.6]),
                       memory_pressure=mp, preserve_system_prompt=rng.random() < 0.7,
                       preserve_recent=rng.random() < 0.7)
    router = BlockRouter(cfg)
    B, Ht = rng.choice([1, 5, 17]), rng.choice([1, 2, 3])
    layouts, totals = [], []
    for _ in range(B):
        lay, end = _random_layout(rng, rng.choice([0, 1, 7, 40, 300]), ps, score_pool=[0.5, 0.8, 0.2])
        layouts.append(lay)
        totals.append(end + rng.choice([0, 5]))
    W = rng.choice([4, 64, 4096])
    bases = torch.randint(0, 1000, (B, Ht), dtype=torch.int32)
    out = route_layouts(router, layouts, totals, ps, W, "cuda", table_heads=Ht, bases=bases.cuda())
    torch.cuda.synchronize()
    _check(out, router, layouts, totals, ps, W, Ht, bases)


def test_reference_golden_cases(golden):
    """Every routing case the reference itself produced: page list and precision map."""
    cases = golden("router_golden.json")["cases"]
    for c in cases:
        router = BlockRouter(RouterConfig(**c["config"]))
        layout = BlockLayout([SemanticBlock(n, s, e, BlockPolicy[p], score=sc) for n, s, e, p, sc in c["spec"]])
        ps = c["page_size"]
        W = max(1, len(c["selected_page_ids"]) + 3)
        out = route_layouts(router, [layout], [c["total"]], ps, W, "cuda")
        n = int(out.num_selected[0])
        assert n == len(c["selected_page_ids"]), c["layout"]
        assert out.page_table[0, 0, :n].tolist() == c["selected_page_ids"], c["layout"]
        ref_prec = c["meta"]["block_precision_by_page"]
        got = {str(p): PRECISION_CODES[KVPrecision(ref_prec[str(p)])] for p in c["selected_page_ids"]}
        assert out.page_prec[0, :n].tolist() == [got[str(p)] for p in c["selected_page_ids"]]


def test_quantizer_thresholds_and_flags_forwarded():
    rng = random.Random(5)
    q = IntentQuantizer(memory_pressure=0.55, preserve_recent=False, preserve_global=False,
                        high_score_threshold=0.6, medium_score_threshold=0.2)
    router = BlockRouter(RouterConfig(top_k_blocks=6, memory_pressure=0.55), quantizer=q)
    layouts, totals = [], []
    for _ in range(9):
        lay, end = _random_layout(rng, 60, 8)
        layouts.append(lay)
        totals.append(end)
    out = route_layouts(router, layouts, totals, 8, 512, "cuda")
    torch.cuda.synchronize()
    _check(out, router, layouts, totals, 8, 512, 1, None)


def test_ties_and_signed_zero_keep_layout_order():
    ps = 4
    blocks = [SemanticBlock(f"a{i}", 8 * i, 8 * i + 8, BlockPolicy.ATTEND, score=s)
              for i, s in enumerate([0.5, 0.5, -0.0, 0.0, 0.5, 0.9, 0.0, 0.5])]
    layout = BlockLayout(blocks)
    for k in range(0, 9):
        router = BlockRouter(RouterConfig(top_k_blocks=k, memory_pressure=0.0))
        out = route_layouts(router, [layout], [64], ps, 64, "cuda")
        torch.cuda.synchronize()
        _check(out, router, [layout], [64], ps, 64, 1, None)


def test_shared_boundary_pages_first_block_wins():
    # many short blocks share pages; the precision of a shared page is the first
    # selected block's in routed order, not in layout order
    rng = random.Random(11)
    for trial in range(20):
        ps = rng.choice([8, 16, 32])
        blocks, t = [], 0
        for i in range(rng.randrange(5, 80)):
            ln = rng.randrange(1, ps + 3)
            pol = rng.choice([BlockPolicy.ATTEND, BlockPolicy.ATTEND, BlockPolicy.RECENT, BlockPolicy.SKIP,
                              BlockPolicy.GLOBAL])
            blocks.append(SemanticBlock(f"x{i}", t, t + ln, pol, score=round(rng.random(), 2)))
            t += ln
        layout = BlockLayout(blocks)
        router = BlockRouter(RouterConfig(top_k_blocks=rng.randrange(0, 20), memory_pressure=rng.random()))
        out = route_layouts(router, [layout], [t], ps, 1024, "cuda")
        torch.cuda.synchronize()
        _check(out, router, [layout], [t], ps, 1024, 1, None)


def test_max_blocks_and_truncation():
    rng = random.Random(3)
    blocks, t = [], 0
    for i in range(N.ROUTE_MAX_BLOCKS):
        ln = rng.randrange(1, 40)
        pol = rng.choice(POLICIES)
        blocks.append(SemanticBlock(f"m{i}", t, t + ln, pol,
                                    score=round(rng.random(), 3) if pol == BlockPolicy.ATTEND or rng.random() < 0.5
                                    else None))
        t += ln
    layout = BlockLayout(blocks)
    router = BlockRouter(RouterConfig(top_k_blocks=1500, memory_pressure=0.45))
    for W in (100000, 777):
        out = route_layouts(router, [layout, layout], [t, t], 16, W, "cuda", table_heads=2)
        torch.cuda.synchronize()
        _check(out, router, [layout, layout], [t, t], 16, W, 2, None)


def test_shared_layout_per_sequence_scores_and_tags():
    """One layout row for the whole batch, scores per sequence; page tags scattered."""
    rng = random.Random(21)
    ps, B, Ht, nb = 16, 6, 2, 50
    base_layout, total = _random_layout(rng, nb, ps)
    layouts = []
    for b in range(B):
        blocks = [SemanticBlock(x.name, x.start, x.end, x.policy,
                                score=round(rng.random(), 3) if x.policy == BlockPolicy.ATTEND or rng.random() < 0.5
                                else None) for x in base_layout.blocks]
        layouts.append(BlockLayout(blocks))
    full = encode_layouts(layouts, "cuda")
    shared = LayoutBatch(full.start[:1].contiguous(), full.end[:1].contiguous(), full.policy[:1].contiguous(),
                         full.scores, None)
    cfg = RouterConfig(top_k_blocks=7, memory_pressure=0.45)
    router = BlockRouter(cfg)
    span = total // ps + 2
    bases = (torch.arange(B * Ht, dtype=torch.int32) * span).view(B, Ht)
    tag_of = {KVPrecision.FP16: 1, KVPrecision.FP8: 2, KVPrecision.INT8: 3, KVPrecision.INT4: 4,
              KVPrecision.INT4_RESIDUAL: 5, KVPrecision.SKIP: 0}
    tags = torch.full((B * Ht * span,), 0xEE, dtype=torch.uint8, device="cuda")
    out = route_pages(shared, cfg, ps, 256, table_heads=Ht, bases=bases.cuda(), page_tags=tags, prec_to_tag=tag_of)
    torch.cuda.synchronize()
    _check(out, router, layouts, [total] * B, ps, 256, Ht, bases)
    code_tag = {PRECISION_CODES[p]: t for p, t in tag_of.items()}
    expect = torch.full_like(tags.cpu(), 0xEE)
    for b, lay in enumerate(layouts):
        ids, precs = _expected(router, lay, total, ps)
        for h in range(Ht):
            for p, c in zip(ids, precs):
                expect[int(bases[b, h]) + p] = code_tag[c]
    assert torch.equal(tags.cpu(), expect)


def test_invalid_layouts_flagged_per_sequence():
    """Sequences that fail BlockLayout.validate get num_selected -1 and an
    empty row; their neighbours in the batch are unaffected."""
    ps = 8
    good = BlockLayout([SemanticBlock("s", 0, 20, BlockPolicy.ALWAYS), SemanticBlock("a", 20, 50, BlockPolicy.ATTEND,
                                                                                    score=0.9)])
    bad_sets = [
        [SemanticBlock("a", 0, 20, BlockPolicy.ALWAYS), SemanticBlock("b", 10, 30, BlockPolicy.RECENT)],   # overlap
        [SemanticBlock("a", 20, 30, BlockPolicy.ALWAYS), SemanticBlock("b", 0, 10, BlockPolicy.RECENT)],   # unsorted
        [SemanticBlock("a", 0, 20, BlockPolicy.ATTEND, score=None)],                                       # no score
        [SemanticBlock("a", 5, 5, BlockPolicy.ALWAYS)],                                                    # empty
        [SemanticBlock("a", 0, 70, BlockPolicy.ALWAYS)],                                                   # > total
    ]
    layouts = [good] + [BlockLayout(x) for x in bad_sets] + [good]
    batch = encode_layouts(layouts, "cuda")
    router = BlockRouter(RouterConfig())
    out = route_pages(batch, router.config, ps, 16, seq_lens=torch.full((len(layouts),), 64, dtype=torch.int32).cuda())
    torch.cuda.synchronize()
    ns = out.num_selected.cpu().tolist()
    assert ns[1:-1] == [-1] * len(bad_sets)
    assert (out.page_counts[1:-1].cpu() == 0).all() and (out.page_table[1:-1].cpu() == -1).all()
    ids, _ = _expected(router, good, 64, ps)
    for b in (0, len(layouts) - 1):
        assert ns[b] == len(ids) and out.page_table[b, 0, :len(ids)].tolist() == ids


def test_route_then_decode_matches_host_packed_table():
    """The device-routed table and tags drive the adaptive decode exactly as
    the host-routed, device-packed table does."""
    from intent_attention import PagePool, pack_metadata, paged_decode
    from intent_attention.paged import make_tag_map
    rng = random.Random(8)
    ps, D, B = 16, 128, 4
    layout, total = _random_layout(rng, 30, ps)
    n_pages = (total + ps - 1) // ps + 1
    cfg = RouterConfig(top_k_blocks=5, memory_pressure=0.2)
    router = BlockRouter(cfg)
    bases = (torch.arange(B, dtype=torch.int32) * n_pages).view(B, 1)
    # precision -> decode tag; tags 1..5 equal the pool format codes F16..INT4R
    tag_of = {KVPrecision.FP16: 1, KVPrecision.FP8: 2, KVPrecision.INT8: 3, KVPrecision.INT4: 4,
              KVPrecision.INT4_RESIDUAL: 5, KVPrecision.SKIP: 0}
    tags_dev = torch.zeros(B * n_pages, dtype=torch.uint8, device="cuda")
    out = route_layouts(router, [layout] * B, [total] * B, ps, 256, "cuda", bases=bases.cuda(), page_tags=tags_dev,
                        prec_to_tag=tag_of)
    ids, precs = _expected(router, layout, total, ps)
    ids_t = torch.tensor(ids, dtype=torch.int32, device="cuda")
    pt_h, pc_h = pack_metadata(ids_t, B, 1, 256, bases=bases.cuda())
    assert torch.equal(pt_h, out.page_table) and torch.equal(pc_h, out.page_counts)
    tags_host = torch.zeros(B * n_pages, dtype=torch.uint8)
    code_tag = {PRECISION_CODES[p]: t for p, t in tag_of.items()}
    for b in range(B):
        for p, c in zip(ids, precs):
            tags_host[int(bases[b, 0]) + p] = code_tag[c]
    assert torch.equal(tags_dev.cpu(), tags_host)
    # quantise every page into the format its routed precision names
    fmts = torch.where(tags_host == 0, torch.ones_like(tags_host), tags_host)
    pool = PagePool.allocate(B * n_pages, ps, D, ["F16", "FP8", "INT8", "INT4", "INT4R"], "page", "cuda")
    k = torch.randn(B * n_pages, ps, D, device="cuda")
    pool.quantize_(k, k * 0.5 + 0.1, fmts.cuda())
    q = torch.randn(B, 1, D, device="cuda")
    tag_map = make_tag_map({1: "F16", 2: "FP8", 3: "INT8", 4: "INT4", 5: "INT4R"})
    o_dev = paged_decode(q, pool, out.page_table, out.page_counts, tags_dev, tag_map)
    o_host = paged_decode(q, pool, pt_h, pc_h, tags_host.cuda(), tag_map)
    torch.cuda.synchronize()
    assert torch.isfinite(o_dev).all()
    assert torch.equal(o_dev, o_host)


def test_row_masks_match_selected_block_rows():
    rng = random.Random(31)
    for trial in range(8):
        ps = rng.choice([8, 16, 64])
        layout, total = _random_layout(rng, 60, ps)
        router = BlockRouter(RouterConfig(top_k_blocks=rng.randrange(0, 20), memory_pressure=rng.random()))
        out = route_layouts(router, [layout], [total], ps, 512, "cuda", row_masks=True)
        routed = router.route_layout(layout, total)
        sel = router.selected_blocks(routed)
        ids = router.selected_page_ids(routed, ps)
        expect = []
        for pg in ids:
            m = 0
            for blk in sel:
                for t in range(max(blk.start, pg * ps), min(blk.end, (pg + 1) * ps)):
                    m |= 1 << (t - pg * ps)
            expect.append(m)
        got = out.row_masks[0, :len(ids)].cpu().numpy().view(np.uint64).tolist()
        assert got == expect, trial
        assert (out.row_masks[0, len(ids):] == 0).all()


def test_route_then_prefill_attends_exactly_the_selected_tokens():
    """Router pages + row masks drive the tensor-core prefill; the result is the
    exact-token attention over the router's selected blocks."""
    from intent_attention import PagePool
    from intent_attention.paged import make_tag_map, paged_prefill
    from oracle import prefill as op
    rng = random.Random(41)
    ps, D, B, H = 16, 128, 2, 2
    layout, total = _random_layout(rng, 40, ps)
    total += 7
    n_log = (total + ps - 1) // ps
    g = np.random.default_rng(5)
    k = g.standard_normal((B, H, n_log * ps, D)).astype(np.float32)
    v = g.standard_normal((B, H, n_log * ps, D)).astype(np.float32)
    pool = PagePool.allocate(B * H * n_log, ps, D, ["F16"], "page", "cuda")
    pool.quantize_(torch.from_numpy(k.reshape(-1, ps, D)).cuda(), torch.from_numpy(v.reshape(-1, ps, D)).cuda(),
                   ["F16"] * (B * H * n_log))
    bases = (torch.arange(B * H, dtype=torch.int32) * n_log).view(B, H).cuda()
    router = BlockRouter(RouterConfig(top_k_blocks=6, memory_pressure=0.2))
    out = route_layouts(router, [layout] * B, [total] * B, ps, n_log, "cuda", table_heads=H, bases=bases,
                        row_masks=True)
    M = total
    q = g.standard_normal((B, H, M, D)).astype(np.float32)
    tags = torch.ones(B * H * n_log, dtype=torch.uint8, device="cuda")
    got = paged_prefill(torch.from_numpy(q).cuda(), pool, out.page_table, out.page_counts, tags,
                        make_tag_map({1: "F16"}), causal=True, bases=bases, row_masks=out.row_masks,
                        kernel="tensor")
    routed = router.route_layout(layout, total)
    spec = [(b.name, b.start, b.end, "ALWAYS", None) for b in router.selected_blocks(routed)]
    spec.sort(key=lambda s: s[1])
    kk = torch.from_numpy(k).half().float().numpy()[:, :, :total]
    vv = torch.from_numpy(v).half().float().numpy()[:, :, :total]
    ref = np.nan_to_num(op.semantic_block_attention(q, kk, vv, spec, True), nan=0.0)
    np.testing.assert_allclose(got.cpu().numpy(), ref, atol=2e-3, rtol=1e-2)

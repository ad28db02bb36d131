"""The product's router / precision policy vs outputs of the reference itself."""

import pytest

from intent_attention import (BlockLayout, BlockPolicy, BlockRouter, IntentQuantizer, RouterConfig, SemanticBlock,
                              routing_to_kernel_metadata)


def _layout(spec):
    return BlockLayout([SemanticBlock(n, s, e, BlockPolicy[p], score=sc) for n, s, e, p, sc in spec])


def _cases(golden):
    return golden("router_golden.json")["cases"]


def test_router_cases_match_reference(golden):
    cases = _cases(golden)
    assert len(cases) > 50
    for c in cases:
        router = BlockRouter(RouterConfig(**c["config"]))
        routed = router.route_layout(_layout(c["spec"]), c["total"])
        got = [{"name": r.name, "start": r.start, "end": r.end, "policy": r.policy.value, "score": r.score,
                "decision": r.decision.value, "precision": r.precision.value, "reason": r.reason} for r in routed]
        assert got == c["routed"], (c["layout"], c["config"])
        ps = c["page_size"]
        assert router.selected_page_ids(routed, ps) == c["selected_page_ids"], (c["layout"], c["config"], ps)
        pf = router.prefetch_page_ids(routed, ps)
        assert pf == _intended_prefetch(routed, router.config, ps)
        assert _reference_prefetch_defect(routed, router.config, ps) == c["prefetch_page_ids"]
        meta = routing_to_kernel_metadata(routed, ps)
        ref_meta = dict(c["meta"])
        assert _reference_prefetch_defect(routed, RouterConfig(), ps) == ref_meta.pop("prefetch_page_ids")
        assert meta.pop("prefetch_page_ids") == _intended_prefetch(routed, RouterConfig(), ps)
        assert meta == ref_meta, (c["layout"], c["config"], ps)
        assert router.routing_summary(routed) == c["summary"]


def _candidates(routed, cfg, ps):
    best = {}
    for b in routed:
        if b.decision.value == "SKIP" and b.score is not None and b.score >= cfg.score_threshold:
            for t in range(b.start, b.end):
                best[t // ps] = max(best.get(t // ps, -1.0), b.score)
    for b in routed:
        if b.decision.value in ("SELECT", "PIN_HIGH_PRECISION", "QUANTIZE"):
            for pid in range(max(0, b.start // ps - 1), (b.end + ps - 1) // ps + 1):
                best[pid] = max(best.get(pid, -1.0), 1.0)
    return best


def _intended_prefetch(routed, cfg, ps):
    """Highest-score-first page ids (ties by id), top prefetch_top_k."""
    best = _candidates(routed, cfg, ps)
    return [pid for pid, s in sorted(best.items(), key=lambda kv: (-kv[1], kv[0]))][:cfg.prefetch_top_k]


def _reference_prefetch_defect(routed, cfg, ps):
    """block_router.py:329-337 unpacks (pid, score) items as (score, pid), so the
    reference returns the distinct candidate SCORES in that order.  This build
    returns the page ids; the reference's values are pinned here."""
    best = _candidates(routed, cfg, ps)
    out = []
    for pid, s in sorted(best.items(), key=lambda kv: (-kv[1], kv[0])):
        if s not in out:
            out.append(s)
    return out[:cfg.prefetch_top_k]


def test_quantizer_decision_table_matches_reference(golden):
    table = golden("router_golden.json")["quantizer"]
    assert len(table) == 560
    for mp, pr, pg, pol, sc, prec, reason in table:
        qz = IntentQuantizer(memory_pressure=mp, preserve_recent=pr, preserve_global=pg)
        p = qz.assign_block_precision(SemanticBlock("x", 0, 16, BlockPolicy[pol], score=sc))
        assert (p.precision.value, p.reason) == (prec, reason), (mp, pr, pg, pol, sc)


def test_memory_pressure_range_checked():
    with pytest.raises(ValueError, match="memory_pressure"):
        IntentQuantizer(memory_pressure=1.5)


@pytest.mark.parametrize("spec,msg", [
    ([("", 0, 4, "ALWAYS", None)], "empty name"),
    ([("a", -1, 4, "ALWAYS", None)], "< 0"),
    ([("a", 4, 4, "ALWAYS", None)], "<= start"),
    ([("a", 0, 99, "ALWAYS", None)], "> total_tokens"),
    ([("a", 0, 4, "ATTEND", None)], "score is None"),
    ([("a", 8, 12, "ALWAYS", None), ("b", 0, 4, "ALWAYS", None)], "not sorted"),
    ([("a", 0, 8, "ALWAYS", None), ("b", 4, 12, "ALWAYS", None)], "overlap"),
])
def test_layout_validation_errors(spec, msg):
    with pytest.raises(ValueError, match=msg):
        _layout(spec).validate(32)


def test_page_list_is_linear_in_blocks():
    """A 2M-token layout routes and packs quickly (the reference walks every token)."""
    import time
    blocks = [("sys", 0, 4096, "ALWAYS", None)] + [
        (f"d{i}", 4096 + i * 65536, 4096 + (i + 1) * 65536, "ATTEND", 0.9 - i * 0.01) for i in range(30)]
    T = blocks[-1][2]
    router = BlockRouter(RouterConfig(top_k_blocks=30))
    t0 = time.perf_counter()
    meta = routing_to_kernel_metadata(router.route_layout(_layout(blocks), T), 16)
    assert time.perf_counter() - t0 < 5.0
    assert len(meta["selected_page_ids"]) == T // 16

"""Generate golden vectors by running the REFERENCE implementation itself.

Run from the repository root, in a container that holds the reference source:

    TRITON_INTERPRET=1 PYTHONPATH=<reference>/src python tests/golden/make_golden.py <reference>/src

It imports the reference package ``intent_attention`` (pure Python + torch CPU;
the two Triton decode kernels that are valid Triton run under Triton's CPU
interpreter) on seeded inputs from ``tests/golden/inputs.py`` and writes the
reference's outputs to ``tests/golden/*.npz`` / ``*.json``.  The committed
fixtures are what ``tests/test_oracle_golden.py`` pins the numpy oracle to and
what the product's router / metadata helpers are compared with.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
if len(sys.argv) > 1:
    sys.path.insert(0, sys.argv[1])

import torch  # noqa: E402

import inputs as gi  # noqa: E402
from intent_attention.block_metadata import BlockLayout, BlockPolicy, SemanticBlock  # noqa: E402
from intent_attention.block_router import BlockRouter, RouterConfig, routing_to_kernel_metadata  # noqa: E402
from intent_attention.intent_quant import IntentQuantizer, KVPrecision, QuantPolicy, fake_quantize_tensor  # noqa: E402
from intent_attention.intent_quant_attention import intent_quant_attention_reference  # noqa: E402
from intent_attention.reference import dense_attention  # noqa: E402
import intent_attention.fused_selected_quant_decode  # noqa: E402,F401
# the package re-exports a function under the submodule's name, so take the
# module object from sys.modules
fsq = sys.modules["intent_attention.fused_selected_quant_decode"]
from intent_attention import triton_intent_quant_attention as t6  # noqa: E402
from intent_attention import triton_adaptive_format_attention as ta  # noqa: E402
from intent_attention import triton_mla_decode as tm  # noqa: E402
from intent_attention.mla import MLABlockTable, MLAConfig, mla_sparse_decode_reference  # noqa: E402
from intent_attention.synthetic_traces import generate_agentic_layout  # noqa: E402

T = torch.from_numpy


def layout_of(spec):
    return BlockLayout([SemanticBlock(n, s, e, BlockPolicy[p], score=sc) for n, s, e, p, sc in spec])


def save(name, **arrays):
    np.savez_compressed(os.path.join(HERE, name), **arrays)
    print("wrote", name, sum(a.nbytes for a in arrays.values()), "bytes raw")


# --------------------------------------------------------------------------- #
def gen_quant():
    out = {}
    x = gi.normal(11, (2, 3, 20, 64), outlier_frac=0.01)
    for p in KVPrecision:
        r, meta = fake_quantize_tensor(T(x.copy()), p)
        out[f"block_{p.value}"] = r.float().numpy()
    pages = gi.normal(12, (5, 16, 128), outlier_frac=0.01)
    for p in KVPrecision:
        per_page, per_group, per_chan = [], [], []
        for i in range(pages.shape[0]):
            pg = T(pages[i].copy())
            per_page.append(fake_quantize_tensor(pg.reshape(-1, 1), p)[0].float().reshape(16, 128).numpy())
            g = pg.reshape(16, 4, 32).permute(0, 2, 1).contiguous()
            per_group.append(fake_quantize_tensor(g, p)[0].float().permute(0, 2, 1).reshape(16, 128).numpy())
            per_chan.append(fake_quantize_tensor(pg, p)[0].float().numpy())
        out[f"page_{p.value}"] = np.stack(per_page)
        out[f"group32_{p.value}"] = np.stack(per_group)
        out[f"channel_{p.value}"] = np.stack(per_chan)
    # fp8 cast table over a dense sweep (incl. subnormals, ties, the 448 edge)
    sweep = np.concatenate([np.linspace(-470, 470, 20001, dtype=np.float32),
                            (np.arange(-600, 601, dtype=np.float32) * np.float32(2.0 ** -12)),
                            np.float32([448, 449, 464, 465, 2 ** -9, 2 ** -10, 3 * 2 ** -11, 0.0])])
    out["fp8_sweep_in"] = sweep
    out["fp8_sweep_out"] = T(sweep).to(torch.float8_e4m3fn).float().numpy()
    save("quant_golden.npz", **out)


# --------------------------------------------------------------------------- #
class ForcedQuantizer(IntentQuantizer):
    """Quantizer that returns a fixed precision per block name."""

    def __init__(self, by_name):
        super().__init__()
        self.by_name = by_name

    def assign_block_precision(self, block):
        return QuantPolicy(KVPrecision[self.by_name[block.name]])


def gen_attention():
    out, meta = {}, {}
    # reference test shapes, stock quantizer at several memory pressures
    for mp in (0.0, 0.3, 0.5, 0.8, 0.95):
        q = gi.normal(21, (1, 2, 8, 32)); k = gi.normal(22, (1, 2, 64, 32)); v = gi.normal(23, (1, 2, 64, 32))
        o, dbg = intent_quant_attention_reference(T(q), T(k), T(v), layout_of(gi.BASIC_LAYOUT),
                                                  IntentQuantizer(memory_pressure=mp), return_debug=True)
        out[f"basic_mp{mp}"] = o.numpy()
        meta[f"basic_mp{mp}"] = dbg["precision_by_block"]
    # e2e layout, GQA-style single decode query per head
    for mp in (0.5, 0.8):
        q = gi.normal(31, (2, 4, 1, 64)); k = gi.normal(32, (2, 4, 448, 64), 0.01); v = gi.normal(33, (2, 4, 448, 64), 0.01)
        o, dbg = intent_quant_attention_reference(T(q), T(k), T(v), layout_of(gi.E2E_LAYOUT),
                                                  IntentQuantizer(memory_pressure=mp), return_debug=True)
        out[f"e2e_mp{mp}"] = o.numpy()
        meta[f"e2e_mp{mp}"] = dbg["precision_by_block"]
    # every precision forced onto the e2e layout's selected blocks (an all-FP16
    # selection is not run: the reference then concatenates float16
    # reconstructions and its matmul with the float32 query raises)
    for prec in ("FP8", "INT8", "INT4", "INT4_RESIDUAL"):
        q = gi.normal(41, (1, 2, 4, 64)); k = gi.normal(42, (1, 2, 448, 64), 0.01); v = gi.normal(43, (1, 2, 448, 64), 0.01)
        by = {n: (prec if p != "SKIP" else "SKIP") for n, s, e, p, sc in gi.E2E_LAYOUT}
        o = intent_quant_attention_reference(T(q), T(k), T(v), layout_of(gi.E2E_LAYOUT), ForcedQuantizer(by))
        out[f"forced_{prec}"] = o.numpy()
    # BASELINE config 1 (reference granularity): MHA 8 heads, D64, 1440 tokens
    q = gi.normal(1001, (1, 8, 1, 64)); k = gi.normal(1002, (1, 8, 1440, 64)); v = gi.normal(1003, (1, 8, 1440, 64))
    by = {"system": "FP16", "retrieved": "INT8", "tool_output": "SKIP", "recent": "FP16"}
    out["c1_refgran"] = intent_quant_attention_reference(T(q), T(k), T(v), layout_of(gi.C1_LAYOUT),
                                                         ForcedQuantizer(by)).numpy()
    # plain dense attention
    q = gi.normal(51, (2, 3, 5, 32)); k = gi.normal(52, (2, 3, 40, 32)); v = gi.normal(53, (2, 3, 40, 32))
    out["dense"] = dense_attention(T(q), T(k), T(v)).numpy()
    save("attention_golden.npz", **out)
    with open(os.path.join(HERE, "attention_golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)


# --------------------------------------------------------------------------- #
def _fused_inputs(seed, B=2, H=4, D=64, PS=16, NP=8, W=4):
    kf = gi.normal(seed, (NP, PS, D)).astype(np.float16)
    vf = gi.normal(seed + 1, (NP, PS, D)).astype(np.float16)
    q = gi.normal(seed + 2, (B, H, 1, D)).astype(np.float16)
    return q, kf, vf


def gen_fused():
    out = {}
    cfg = fsq.FusedDecodeConfig(page_size=16, head_dim=64, max_selected_pages=4, block_d=64)
    q, kf, vf = _fused_inputs(61)
    ki, ks = fsq.fake_int8_pages_from_fp16(T(kf))
    vi, vs = fsq.fake_int8_pages_from_fp16(T(vf))
    out.update(k_i8=ki.numpy(), k_sc=ks.numpy(), v_i8=vi.numpy(), v_sc=vs.numpy())
    B, H, NP, W = 2, 4, 8, 4
    pt = np.tile(np.arange(W, dtype=np.int32), (B, H, 1))
    g = gi.rng(62)
    pt_rand = g.integers(0, NP, size=(B, H, W)).astype(np.int32)
    cases = {
        "fp16": (np.zeros(NP, np.int32), np.full((B, H), 4, np.int32), pt),
        "int8": (np.ones(NP, np.int32), np.full((B, H), 4, np.int32), pt),
        "skip": (np.full(NP, 2, np.int32), np.full((B, H), 4, np.int32), pt),
        "mixed": (np.array([0, 0, 0, 0, 1, 1, 1, 1], np.int32), np.full((B, H), 4, np.int32), pt_rand),
        "mixed_skip": (np.array([0, 1, 2, 0, 1, 2, 0, 1], np.int32), np.full((B, H), 4, np.int32), pt_rand),
        "zero": (np.zeros(NP, np.int32), np.zeros((B, H), np.int32), pt),
        "single": (np.array([1, 0, 1, 0, 1, 0, 1, 0], np.int32), np.ones((B, H), np.int32), pt_rand),
        "ragged": (np.array([0, 1, 0, 1, 2, 0, 1, 0], np.int32),
                   np.array([[1, 2, 3, 4], [0, 4, 2, 3]], np.int32), pt_rand),
    }
    for name, (prec, pc, table) in cases.items():
        o = fsq.fused_selected_quant_decode_reference(T(q), T(kf), T(vf), ki, vi, ks, vs, T(table), T(prec), T(pc), cfg)
        out[f"out_{name}"] = o.numpy()
        out[f"prec_{name}"] = prec; out[f"pc_{name}"] = pc; out[f"pt_{name}"] = table
    # metadata_to_kernel_tensors
    metas = {
        "basic": {"selected_page_ids": [0, 3, 5], "block_precision_by_page": {"0": "FP16", "3": "INT8", "5": "SKIP"}},
        "lossy": {"selected_page_ids": [7, 1, 2, 4], "block_precision_by_page":
                  {"7": "FP8", "1": "INT4", "2": "INT4_RESIDUAL", "4": "FP16", "x": "INT8"}},
        "empty": {"selected_page_ids": [], "block_precision_by_page": {}},
        "trunc": {"selected_page_ids": list(range(10)), "block_precision_by_page": {str(i): "INT8" for i in range(10)}},
    }
    for name, m in metas.items():
        for (Bm, Hm, width) in ((1, 1, 64), (2, 3, 4)):
            c = fsq.FusedDecodeConfig(max_selected_pages=width)
            a, b_, c_ = fsq.metadata_to_kernel_tensors(m, num_pages=12, B=Bm, H=Hm, config=c)
            out[f"meta_{name}_{Bm}{Hm}{width}_pt"] = a.numpy()
            out[f"meta_{name}_{Bm}{Hm}{width}_prec"] = b_.numpy()
            out[f"meta_{name}_{Bm}{Hm}{width}_pc"] = c_.numpy()
    with open(os.path.join(HERE, "fused_metas.json"), "w") as f:
        json.dump(metas, f, indent=1)
    # the triton module's int8 page quantiser (fp32 scales, clamp +-127)
    pages = gi.normal(63, (4, 16, 32))
    qi, sc = t6.fake_int8_pages_from_fp16(T(pages))
    out.update(t6_pages=pages, t6_q=qi.numpy(), t6_sc=sc.numpy())
    save("fused_golden.npz", **out)


# --------------------------------------------------------------------------- #
def gen_triton_interp():
    out = {}
    B, H, D, PS, NP, W = 2, 3, 64, 16, 10, 6
    q = gi.normal(71, (B, H, D)).astype(np.float16)
    kf = gi.normal(72, (NP, PS, D)).astype(np.float16); vf = gi.normal(73, (NP, PS, D)).astype(np.float16)
    ki, ks = t6.fake_int8_pages_from_fp16(T(gi.normal(74, (NP, PS, D))))
    vi, vs = t6.fake_int8_pages_from_fp16(T(gi.normal(75, (NP, PS, D))))
    g = gi.rng(76)
    ids = g.integers(0, NP, size=(B, H, W)).astype(np.int32)
    ids[0, 1, 4:] = -1; ids[1, 2, 2] = -1
    cnt = np.array([[6, 4, 5], [3, 6, 0]], np.int32)
    prec = np.array([0, 1, 2, 3, 4, 5, 0, 2, 5, 0], np.int32)
    o = torch.empty(B, H, D, dtype=torch.float16)
    t6._intent_quant_decode_attention_kernel[(B * H,)](
        T(q), T(kf), T(vf), ki, vi, ks, vs, T(ids), T(cnt), T(prec), o,
        B=B, H=H, D=D, PAGE_SIZE=PS, MAX_SELECTED_PAGES=W, BLOCK_D=64)
    out.update(t6_q=q, t6_kf=kf, t6_vf=vf, t6_ki=ki.numpy(), t6_vi=vi.numpy(), t6_ks=ks.numpy(),
               t6_vs=vs.numpy(), t6_ids=ids, t6_cnt=cnt, t6_prec=prec, t6_out=o.numpy())
    # adaptive-format kernel: FP16 / INT8 / SPARSE / SKIP, -1 padding, no counts
    B, H, D, PS, NP, W = 1, 2, 32, 8, 6, 4
    q = gi.normal(81, (B, H, D)).astype(np.float16)
    kf = gi.normal(82, (NP, PS, D)).astype(np.float16); vf = gi.normal(83, (NP, PS, D)).astype(np.float16)
    k8 = gi.rng(84).integers(-127, 128, size=(NP, PS, D)).astype(np.int8)
    v8 = gi.rng(85).integers(-127, 128, size=(NP, PS, D)).astype(np.int8)
    k8s = np.full(NP, 0.02, np.float32); v8s = np.full(NP, 0.03, np.float32)
    fmts = np.array([0, 1, 2, 3, 1, 0], np.int32)
    ids = np.array([[[0, 1, 2, 4], [5, 3, -1, -1]]], np.int32)
    o = torch.empty(B, H, D, dtype=torch.float16)
    e32 = torch.zeros(0, dtype=torch.int32); e16 = torch.zeros(0, dtype=torch.float16)
    ta._adaptive_format_decode_kernel[(B * H,)](
        T(q), T(ids), T(fmts), T(kf), T(vf), T(k8), T(v8), T(k8s), T(v8s), e32, e16, e32, e16, e32, o,
        B=B, H=H, D=D, PAGE_SIZE=PS, MAX_SELECTED_PAGES=W, BLOCK_D=32, SPARSE_MAX_NNZ=4)
    out.update(ad_q=q, ad_kf=kf, ad_vf=vf, ad_k8=k8, ad_v8=v8, ad_k8s=k8s, ad_v8s=v8s, ad_fmts=fmts,
               ad_ids=ids, ad_out=o.numpy())
    # page-table helpers
    p, c = t6.make_page_tables_from_selected_pages(torch.tensor([0, 2, 5], dtype=torch.int32), 2, 3, 8)
    out.update(mk1_ids=p.numpy(), mk1_cnt=c.numpy())
    p, c = t6.make_page_tables_from_selected_pages(torch.arange(12, dtype=torch.int32).reshape(2, 3, 2), 2, 3, 4)
    out.update(mk3_ids=p.numpy(), mk3_cnt=c.numpy())
    out["prec_t"] = t6.make_precision_tensor(10, fp16_pages=torch.tensor([0, 1, 2]), int8_pages=torch.tensor([3, 4])).numpy()
    p, c = ta.make_adaptive_page_tables(torch.tensor([3, 1, 2], dtype=torch.int32), 1, 1)
    out.update(mka_ids=p.numpy(), mka_cnt=c.numpy())
    save("triton_interp_golden.npz", **out)


# --------------------------------------------------------------------------- #
def gen_mla():
    out = {}
    for ps in (8, 16, 32, 64):
        qa = gi.normal(90 + ps, (2, 3, 64)); C = gi.normal(91 + ps, (4 * ps, 64)); W = gi.normal(92 + ps, (64, 128))
        pt = torch.tensor([2, 0, 3], dtype=torch.int32)
        out[f"cpu_ps{ps}"] = tm._mla_decode_cpu(T(qa), T(C), T(W), pt, page_size=ps).numpy()
    d_model, d_c, n_heads, d_head = 256, 64, 4, 64
    cfg = MLAConfig(d_model, d_c, n_heads, d_head)
    table = MLABlockTable(cfg, page_size=16)
    lat = gi.normal(95, (4, 16, 64))
    for bid in range(4):
        table.append(bid, T(lat[bid].copy()))
    W_QK = gi.normal(96, (n_heads * d_head, d_c)); W_VO = gi.normal(97, (d_c, d_model))
    q = gi.normal(98, (2, n_heads, 4, d_head))
    blocks = [SemanticBlock(f"b{i}", i * 16, (i + 1) * 16, BlockPolicy.ATTEND, score=0.9) for i in range(4)]
    ref, _ = mla_sparse_decode_reference(T(q), table, T(W_QK), T(W_VO), BlockLayout(blocks), threshold=0.5)
    out["sparse_ref"] = ref.float().numpy()
    save("mla_golden.npz", **out)


# --------------------------------------------------------------------------- #
def _routed_to_json(routed):
    return [{"name": r.name, "start": r.start, "end": r.end, "policy": r.policy.value, "score": r.score,
             "decision": r.decision.value, "precision": r.precision.value, "reason": r.reason} for r in routed]


def gen_router():
    cases = []
    specs = {
        "e2e": gi.E2E_LAYOUT, "basic": gi.BASIC_LAYOUT, "c1": gi.C1_LAYOUT,
        "many7": gi.many_attend_layout(7), "many8": gi.many_attend_layout(8, n_blocks=40),
    }
    configs = [
        {}, {"score_threshold": 0.3}, {"memory_pressure": 0.8}, {"memory_pressure": 0.95, "top_k_blocks": 3},
        {"memory_pressure": 0.2, "preserve_recent": False}, {"top_k_blocks": 12, "prefetch_top_k": 9},
    ]
    total = {"e2e": 448, "basic": 64, "c1": 1440}
    for lname, spec in specs.items():
        T_tok = total.get(lname, spec[-1][2])
        for ci, cfg in enumerate(configs):
            router = BlockRouter(RouterConfig(**cfg))
            routed = router.route_layout(layout_of(spec), T_tok)
            for ps in (16, 64):
                meta = routing_to_kernel_metadata(routed, page_size=ps)
                cases.append({"layout": lname, "spec": spec, "total": T_tok, "config": cfg, "page_size": ps,
                              "routed": _routed_to_json(routed),
                              "selected_page_ids": router.selected_page_ids(routed, ps),
                              "prefetch_page_ids": router.prefetch_page_ids(routed, ps),
                              "meta": meta, "summary": router.routing_summary(routed)})
    # a synthetic agentic layout from the reference's own generator
    lay = generate_agentic_layout(16384, seed=3)
    spec = [(b.name, b.start, b.end, b.policy.name, b.score) for b in lay.blocks]
    router = BlockRouter(RouterConfig())
    routed = router.route_layout(lay, 16384)
    meta = routing_to_kernel_metadata(routed, page_size=16)
    cases.append({"layout": "agentic", "spec": spec, "total": 16384, "config": {}, "page_size": 16,
                  "routed": _routed_to_json(routed), "selected_page_ids": router.selected_page_ids(routed, 16),
                  "prefetch_page_ids": router.prefetch_page_ids(routed, 16), "meta": meta,
                  "summary": router.routing_summary(routed)})
    # quantizer precision table
    q_table = []
    for mp in (0.0, 0.3, 0.55, 0.65, 0.75, 0.85, 0.95):
        for pr in (True, False):
            for pg in (True, False):
                qz = IntentQuantizer(memory_pressure=mp, preserve_recent=pr, preserve_global=pg)
                for pol in BlockPolicy:
                    for sc in (None, 0.1, 0.5, 0.8):
                        if pol == BlockPolicy.ATTEND and sc is None:
                            pass
                        qp = qz.assign_block_precision(SemanticBlock("x", 0, 16, pol, score=sc))
                        q_table.append([mp, pr, pg, pol.value, sc, qp.precision.value, qp.reason])
    with open(os.path.join(HERE, "router_golden.json"), "w") as f:
        json.dump({"cases": cases, "quantizer": q_table}, f)
    print("wrote router_golden.json", len(cases), "cases")


def gen_prefill():
    """reference.py:82-130 semantic_block_attention (the exact-token CPU path)
    with causal masks on the original token positions (reference.py:16-45)."""
    from intent_attention.reference import semantic_block_attention
    out = {}
    cases = [("e2e_causal", gi.E2E_LAYOUT, (1, 2, 448, 64), 448, True),
             ("e2e_chunk", gi.E2E_LAYOUT, (2, 2, 16, 64), 448, False),
             ("partial_causal", gi.PREFILL_PARTIAL_LAYOUT, (2, 3, 100, 32), 100, True),
             ("gap_causal", gi.PREFILL_GAP_LAYOUT, (1, 2, 96, 32), 96, True),
             ("partial_causal_d128", gi.PREFILL_PARTIAL_LAYOUT, (1, 2, 100, 128), 100, True)]
    for i, (name, spec, qshape, T_kv, causal) in enumerate(cases):
        B, H, M, D = qshape
        q = gi.normal(600 + 3 * i, qshape)
        k = gi.normal(601 + 3 * i, (B, H, T_kv, D))
        v = gi.normal(602 + 3 * i, (B, H, T_kv, D))
        out[name] = semantic_block_attention(T(q), T(k), T(v), layout_of(spec), causal=causal).numpy()
    save("prefill_golden.npz", **out)


if __name__ == "__main__":
    torch.manual_seed(0)
    gen_quant()
    gen_attention()
    gen_fused()
    gen_triton_interp()
    gen_mla()
    gen_router()
    gen_prefill()

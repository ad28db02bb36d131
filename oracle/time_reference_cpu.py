"""Time the REFERENCE's own CPU decode paths on C2-shaped inputs (test / bench
infrastructure; writes ``oracle/reference_cpu_timing.json``).

    python oracle/time_reference_cpu.py <reference>/src

The reference is pure Python + torch and cannot be installed on the GPU box,
so its own CPU paths are timed here, in the build container, and the result
is committed for ``bench.py`` to report beside the numpy port it times on the
box.  Two paths, each on a sample of the C2 workload (Llama-3-8B GQA decode,
32 sequences x 32 query heads / 8 kv heads, head_dim 128, 1024 router-selected
16-token pages per (sequence, kv head)):

* ``fused_selected_quant_decode_reference`` (the drop-in's CPU fallback,
  ``fused_selected_quant_decode.py:267-336``): a Python loop over (b, h) and
  pages.  It has no GQA, so every query head walks its page list; its API has
  FP16 and INT8 pages only, so the sample's FP8 pages are given as INT8 pages
  (same bytes per element).  Timed on a few (sequence, query head) rows and
  scaled to the step's 1024 rows.
* ``intent_quant_attention_reference`` (the oracle,
  ``intent_quant_attention.py:20-119``): fake-quantise every selected block,
  then dense attention, for one (sequence, kv head) with its 4 query heads as
  4 query rows (the GQA view); scaled to the step's 256 units.

``value_gbs`` = the C2 step's algorithmic selected-KV bytes / the scaled step
time, the metric ``bench.py`` reports.
"""

from __future__ import annotations

import json
import math
import os
import platform
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    import torch
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    import intent_attention  # the reference package  # noqa: F401
    fsq = sys.modules["intent_attention.fused_selected_quant_decode"]
    from intent_attention.block_metadata import BlockLayout, BlockPolicy, SemanticBlock
    from intent_attention.block_router import BlockRouter, RouterConfig
    from intent_attention.intent_quant import IntentQuantizer
    from intent_attention.intent_quant_attention import intent_quant_attention_reference

    PS, D, W, T = 16, 128, 1024, 32768
    step_bytes = 1_397_123_072                 # C2 selected-KV bytes per step (bench.step_bytes)
    rows_per_step, units_per_step = 32 * 32, 32 * 8
    g = torch.Generator().manual_seed(1002)
    rec = {"cores": cores, "cpu": platform.processor() or platform.machine(), "torch": torch.__version__,
           "workload": "C2 Llama-3-8B-shape GQA decode (batch 32, 32 q / 8 kv heads, head_dim 128, 1024 "
                       "selected 16-token pages per (sequence, kv head))",
           "measured_on": "the build container's CPU (the reference is pure Python and is not installed on "
                          "the GPU box)"}

    # ---- fused_selected_quant_decode_reference: per (b, h) Python loop over pages
    n_rows = 16
    kf = torch.randn((W, PS, D), generator=g).half()
    vf = torch.randn((W, PS, D), generator=g).half()
    ki = torch.randint(-127, 128, (W, PS, D), generator=g, dtype=torch.int8)
    vi = torch.randint(-127, 128, (W, PS, D), generator=g, dtype=torch.int8)
    ks = torch.rand(W, generator=g) * 0.05
    vs = torch.rand(W, generator=g) * 0.05
    prec = torch.where(torch.rand(W, generator=g) < 0.3, 0, 1).to(torch.int32)   # 30 % FP16, 70 % 8-bit
    table = torch.arange(W, dtype=torch.int32).view(1, 1, W).expand(1, n_rows, W).contiguous()
    counts = torch.full((1, n_rows), W, dtype=torch.int32)
    q = torch.randn((1, n_rows, 1, D), generator=g).half()
    cfg = fsq.FusedDecodeConfig(page_size=PS, head_dim=D, max_selected_pages=W)
    fsq.fused_selected_quant_decode_reference(q[:, :1], kf, vf, ki, vi, ks, vs, table[:, :1], prec, counts[:, :1], cfg)
    t0 = time.perf_counter()
    fsq.fused_selected_quant_decode_reference(q, kf, vf, ki, vi, ks, vs, table, prec, counts, cfg)
    dt = time.perf_counter() - t0
    per_step = dt / n_rows * rows_per_step
    rec["fused_selected_quant_decode_reference"] = {
        "seconds_timed": round(dt, 3), "rows_timed": n_rows, "rows_per_step": rows_per_step,
        "seconds_per_step": round(per_step, 2), "value_gbs": round(step_bytes / per_step / 1e9, 6),
        "sample": f"{n_rows} (sequence, query head) rows of 1024 pages each, scaled to the step's "
                  f"{rows_per_step} rows"}

    # ---- intent_quant_attention_reference: one (sequence, kv head), 4 query rows
    rng = np.random.default_rng(1002)
    blocks = [SemanticBlock("system", 0, 512, BlockPolicy.ALWAYS)]
    n_mid = (T - 512 - 1024) // 64
    for i in range(n_mid):
        blocks.append(SemanticBlock(f"doc{i}", 512 + 64 * i, 512 + 64 * (i + 1), BlockPolicy.ATTEND,
                                    score=float(rng.random())))
    blocks.append(SemanticBlock("recent", T - 1024, T, BlockPolicy.RECENT))
    routed = BlockRouter(RouterConfig(top_k_blocks=(1024 - 96) // 4, memory_pressure=0.0)).route_layout(
        BlockLayout(blocks), T)
    chosen = {r.name for r in routed if r.decision.name != "SKIP"}
    sel_blocks = [b if b.name in chosen else SemanticBlock(b.name, b.start, b.end, BlockPolicy.SKIP, score=b.score)
                  for b in blocks]
    layout = BlockLayout(sel_blocks)
    k = torch.randn((1, 1, T, D), generator=g)
    v = torch.randn((1, 1, T, D), generator=g)
    qa = torch.randn((1, 1, 4, D), generator=g)
    quant = IntentQuantizer(memory_pressure=0.0)
    units = 8
    intent_quant_attention_reference(qa, k, v, layout, quant)
    t0 = time.perf_counter()
    for _ in range(units):
        intent_quant_attention_reference(qa, k, v, layout, quant)
    dt = time.perf_counter() - t0
    per_step = dt / units * units_per_step
    rec["intent_quant_attention_reference"] = {
        "seconds_timed": round(dt, 3), "units_timed": units, "units_per_step": units_per_step,
        "seconds_per_step": round(per_step, 2), "value_gbs": round(step_bytes / per_step / 1e9, 6),
        "sample": f"{units} (sequence, kv head) units (4 query rows each, router-selected blocks of C2's "
                  f"layout), scaled to the step's {units_per_step} units"}
    out = os.path.join(HERE, "reference_cpu_timing.json")
    with open(out, "w") as f:
        json.dump(rec, f, indent=1)
    print(json.dumps(rec, indent=1))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python oracle/time_reference_cpu.py <reference>/src")
    main(sys.argv[1])

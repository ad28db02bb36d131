"""Benchmark: fused selected-quant paged decode on B200 (sm_100a).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c3|c4|c5|c1|route|append|prefill] [--impl b200|reference]

One "step" is one decode step of the workload's whole batch (all sequences,
all heads) over its router-selected pages.  ``value`` is the selected-KV HBM
throughput in GB/s (algorithmic bytes: K+V codes + the scales they need, of
every selected page, divided by the device time of the step) summed over all
ranks; ``ms_per_step`` / ``us_per_step`` give the step time.  Multi-GPU runs
shard the batch (weak scaling: every rank decodes its own full-size batch,
no collective on the data path) and take the max time over ranks; with
``--workload c5`` they instead cut every sequence's selected pages into one
range per rank (strong scaling: the whole C5 step is shared), each rank
decodes its range into partial (m, l, acc) blocks, one NCCL all-gather
exchanges them and every rank LSE-merges the result.

Default workload: Llama-3-8B-shape GQA decode, batch 32,
32 q heads / 8 kv heads, head_dim 128, 32768-token context in 16-token
pages; the router keeps the first 512 and last 1024 tokens plus the top
ATTEND blocks by seeded score (1024 of 2048 pages per sequence and kv head);
selected pages are 30% FP16 / 40% FP8-e4m3 / 30% INT8 with per-page,
per-head scales.  Synthetic seeded data (no dataset is involved).

``--impl reference`` times the reference algorithm's CPU implementation (the
numpy restatement in oracle/, which the tests pin to the reference's own
outputs) on the host cores, on a bounded sample of the same workload, and
reports the same metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "intent-attention-kernel_b200"))

METRIC = "decode-attn µs/step & selected-KV HBM GB/s (vs 8 TB/s) at 1/2/4/8 B200 vs CPU ref"
FALLBACK_HBM_GBS = 6650.0

# name -> [IAK format code, K+V code bytes per page per head-dim element pair]
FMT_CODE = {"F16": 1, "FP8": 2, "INT8": 3, "INT4": 4, "INT4R": 5}


# --------------------------------------------------------------------------- #
#  Workloads
# --------------------------------------------------------------------------- #

def workload(name: str) -> dict:
    if name == "c2":
        return dict(name="C2 Llama-3-8B-shape GQA decode", B=32, Hq=32, Hkv=8, D=128, T=32768, PS=16,
                    head_tokens=512, tail_tokens=1024, attend_block_pages=4, select_pages=1024,
                    mix={"F16": 0.3, "FP8": 0.4, "INT8": 0.3}, scale_mode="page", q_std=1.0, outliers=0.01,
                    seed=1002)
    if name == "c3":
        return dict(name="C3 Llama-3-70B-shape low-bit decode", B=64, Hq=64, Hkv=8, D=128, T=8192, PS=16,
                    head_tokens=8192, tail_tokens=0, attend_block_pages=4, select_pages=512,
                    mix={"F16": 0.2, "INT4": 0.4, "INT4R": 0.4}, scale_mode="group32", q_std=0.5, outliers=0.0,
                    seed=1003)
    if name == "c5":
        return dict(name="C5 long-context decode (single GPU)", B=8, Hq=32, Hkv=8, D=128, T=524288, PS=16,
                    head_tokens=512, tail_tokens=1024, attend_block_pages=4, select_pages=8192,
                    mix={"F16": 0.1, "FP8": 0.3, "INT8": 0.3, "INT4": 0.3}, scale_mode="page", q_std=1.0,
                    outliers=0.0, seed=1005)
    if name == "c1":
        # formats by position: tokens 0-127 (system) FP16, 128-1023 (retrieved) INT8,
        # 1024-1279 (tool output) not selected, 1280-1439 (recent) FP16
        return dict(name="C1 CPU-runnable MHA decode", B=1, Hq=8, Hkv=8, D=64, T=1440, PS=16,
                    head_tokens=128, tail_tokens=160, attend_block_pages=56, select_pages=74,
                    mix={"F16": 0.5, "INT8": 0.5}, scale_mode="page", q_std=1.0, outliers=0.0, seed=1001,
                    format_by_token=[(0, 128, "F16"), (128, 1024, "INT8"), (1280, 1440, "F16")])
    raise SystemExit(f"unknown workload {name}")


def select_pages(w: dict):
    """Router-selected logical pages (shared by every (b, kv head)) + their formats."""
    from intent_attention import BlockLayout, BlockPolicy, BlockRouter, RouterConfig, SemanticBlock
    from intent_attention import routing_to_kernel_metadata
    PS, T = w["PS"], w["T"]
    rng = np.random.default_rng(w["seed"])
    blocks = []
    if w["head_tokens"]:
        blocks.append(SemanticBlock("system", 0, w["head_tokens"], BlockPolicy.ALWAYS))
    mid_start, mid_end = w["head_tokens"], T - w["tail_tokens"]
    bt = w["attend_block_pages"] * PS
    n_mid = (mid_end - mid_start) // bt
    for i in range(n_mid):
        blocks.append(SemanticBlock(f"doc{i}", mid_start + i * bt, mid_start + (i + 1) * bt, BlockPolicy.ATTEND,
                                    score=float(rng.random())))
    if w["tail_tokens"]:
        blocks.append(SemanticBlock("recent", mid_end, T, BlockPolicy.RECENT))
    fixed = (w["head_tokens"] + w["tail_tokens"]) // PS
    top_k = max(0, (w["select_pages"] - fixed) // w["attend_block_pages"])
    router = BlockRouter(RouterConfig(top_k_blocks=top_k, memory_pressure=0.0))
    meta = routing_to_kernel_metadata(router.route_layout(BlockLayout(blocks), T), PS)
    ids = np.asarray(meta["selected_page_ids"], dtype=np.int32)
    n = ids.size
    if "format_by_token" in w:
        fmt = np.zeros(n, np.uint8)
        for t0, t1, name in w["format_by_token"]:
            fmt[(ids * PS >= t0) & (ids * PS < t1)] = FMT_CODE[name]
        if (fmt == 0).any():
            raise SystemExit("a selected page has no format in format_by_token")
        return ids, fmt
    names = list(w["mix"].keys())
    counts = [int(round(w["mix"][k] * n)) for k in names]
    counts[-1] = n - sum(counts[:-1])
    fmt = np.concatenate([np.full(c, FMT_CODE[k], np.uint8) for k, c in zip(names, counts)])
    fmt = fmt[rng.permutation(n)]
    return ids, fmt


def page_bytes(fmt_code: int, PS: int, D: int, ns: int) -> int:
    """Algorithmic bytes of one selected page (K and V planes + their scales)."""
    code = {1: 2 * D, 2: D, 3: D, 4: D // 2, 5: D}[fmt_code] * PS
    scales = {1: 0, 2: 1, 3: 1, 4: 1, 5: 2}[fmt_code] * ns * 4
    return 2 * (code + scales)


def n_scales(mode: str, D: int) -> int:
    return {"page": 1, "group32": D // 32, "channel": D}[mode]


L2_BYTES = 126 * 2 ** 20          # B200 L2


def l2_note(nbytes: int, what: str) -> str:
    """The config's statement on L2 for inputs that are not flushed between timed steps."""
    if nbytes > L2_BYTES:
        return f"inputs larger than L2 ({nbytes / 1e9:.2f} GB of {what} per step)"
    return (f"inputs smaller than L2 ({nbytes / 1e6:.1f} MB of {what} per step), not flushed between steps: "
            "a latency-bound case")


def step_bytes(w: dict, fmt: np.ndarray) -> int:
    ns = n_scales(w["scale_mode"], w["D"])
    per_unit = sum(page_bytes(int(f), w["PS"], w["D"], ns) for f in fmt)
    return per_unit * w["B"] * w["Hkv"]


# --------------------------------------------------------------------------- #
#  CPU (reference algorithm) timing on a bounded sample
# --------------------------------------------------------------------------- #

class CpuDecodeSample:
    """The numpy oracle's decode (the reference algorithm restated, pinned to the
    reference's own outputs by the tests) of (sequence, kv head) units of a
    workload, on the host cores.  Four distinct units of the workload's page
    count and format mix are built once and cycled."""

    def __init__(self, w: dict, ids: np.ndarray, fmt: np.ndarray):
        from oracle import quant as oq
        self.w, self.fmt = w, fmt
        self.cores = len(os.sched_getaffinity(0))
        D, PS, G = w["D"], w["PS"], w["Hq"] // w["Hkv"]
        n = ids.size
        rng = np.random.default_rng(w["seed"] + 7)
        self.units_total = w["B"] * w["Hkv"]
        self.bytes_per_unit = step_bytes(w, fmt) / self.units_total

        def build_unit():
            k = rng.standard_normal((n, PS, D)).astype(np.float32)
            v = rng.standard_normal((n, PS, D)).astype(np.float32)
            pools = {"k_f16": k.astype(np.float16), "v_f16": v.astype(np.float16)}
            sc = {}
            for plane, x in (("k", k), ("v", v)):
                if any(f in (2, 3, 4, 5) for f in fmt):
                    r8 = oq.quantize_pages(x, "INT8", w["scale_mode"])
                    pools[f"{plane}_i8"] = r8["codes"]
                    sc[f"{plane}_scale"] = r8["scale"]
                    pools[f"{plane}_fp8"] = oq.f32_to_e4m3(x / oq.expand_scales(r8["scale"], w["scale_mode"], D))
                    r4 = oq.quantize_pages(x, "INT4_RESIDUAL", w["scale_mode"])
                    pools[f"{plane}_i4"] = oq.pack_int4(r4["codes"])
                    pools[f"{plane}_i4r"] = oq.pack_int4(r4["res_codes"])
                    sc[f"{plane}_res_scale"] = r4["res_scale"]
            q = rng.standard_normal((G, D)).astype(np.float32) * w["q_std"]
            return q, pools, sc

        self.data = [build_unit() for _ in range(min(4, self.units_total))]
        self.tags = fmt.astype(np.int64)
        self.pids = np.arange(n)

    def _one(self, i):
        from oracle import decode as odec
        q, pools, sc = self.data[i % len(self.data)]
        return odec.unit_partial(q, self.pids, self.tags, {1: "F16", 2: "FP8", 3: "INT8", 4: "INT4", 5: "INT4R"},
                                 "SKIP", pools, sc, self.w["scale_mode"], 1.0 / math.sqrt(self.w["D"]))

    def run_for(self, budget_s: float, max_units: int = 0):
        """Decode whole waves of one unit per core until ``budget_s`` has passed
        (at least one wave, at most ``max_units`` units when given).  Returns
        (seconds, units decoded); nothing is extrapolated."""
        import concurrent.futures as cf
        # numpy's BLAS uses every core for the matmuls; a thread pool overlaps the
        # per-unit gather / dequantisation work across cores as well
        limit = max_units or 1 << 30
        done = 0
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(max_workers=self.cores) as ex:
            while done < limit and (done == 0 or time.perf_counter() - t0 < budget_s):
                batch = min(self.cores, limit - done)
                list(ex.map(self._one, range(done, done + batch)))
                done += batch
        return time.perf_counter() - t0, done


def cpu_baseline_record(sample: CpuDecodeSample, budget_s: float) -> dict:
    """The ``cpu_baseline`` object: the numpy port's selected-KV rate on a bounded sample."""
    sec, units = sample.run_for(budget_s)
    return {"value": round(units * sample.bytes_per_unit / sec / 1e9, 4), "unit": "GB/s", "cores": sample.cores,
            "kind": "port", "seconds": round(sec, 3), "units_timed": units, "units_per_step": sample.units_total,
            "sample": f"{units} (sequence, kv head) units of the step's layout (a step has "
                      f"{sample.units_total}) decoded by the numpy oracle on {sample.cores} host threads in "
                      f"{sec:.2f} s; value = their selected-KV bytes / that time"}


REFERENCE_TIMING = os.path.join(ROOT, "oracle", "reference_cpu_timing.json")


def reference_cpu_record(workload_name: str):
    """The reference's own CPU decode paths (fused_selected_quant_decode_reference and
    intent_quant_attention_reference) timed on C2-shaped samples by
    oracle/time_reference_cpu.py in the build container (the reference is pure Python
    and is not installed on the GPU box), or None for other workloads."""
    if workload_name != "c2":
        return None
    try:
        with open(REFERENCE_TIMING) as f:
            t = json.load(f)
    except (OSError, ValueError):
        return None
    fr = t["fused_selected_quant_decode_reference"]
    return {"value": fr["value_gbs"], "unit": "GB/s", "cores": t["cores"], "kind": "reference",
            "seconds_per_step": fr["seconds_per_step"], "sample": fr["sample"],
            "oracle_path_value": t["intent_quant_attention_reference"]["value_gbs"],
            "oracle_path_sample": t["intent_quant_attention_reference"]["sample"],
            "measured_on": t["measured_on"], "source": "oracle/reference_cpu_timing.json"}


def workload_config(w: dict, n_sel_total: int, n_sel_rank: int, world: int, seq_shard: bool, nbytes_rank: int,
                    exchange: str) -> dict:
    """The ``config`` object both arms print for a decode workload."""
    return {"workload": w["name"], "batch_per_gpu": w["B"], "global_batch": w["B"] * (1 if seq_shard else world),
            "q_heads": w["Hq"], "kv_heads": w["Hkv"], "head_dim": w["D"], "ctx": w["T"],
            "page_size": w["PS"], "selected_pages_per_seq_head": n_sel_total,
            "selected_pages_per_seq_head_per_gpu": n_sel_rank,
            "format_mix": ({f"tokens {a}-{b - 1}": f for a, b, f in w["format_by_token"]}
                           if "format_by_token" in w else w["mix"]),
            "scale_mode": w["scale_mode"], "selected_kv_bytes_per_step_per_gpu": nbytes_rank,
            "l2": l2_note(nbytes_rank, "selected KV"),
            "parallelism": (f"sp{world} (each sequence's selected pages cut into {world} ranges; partial "
                            "(m, l, acc) blocks exchanged "
                            + ("by NVLink peer stores with epoch flags (CUDA IPC)" if exchange == "p2p"
                               else "with one NCCL all-gather")
                            + ", LSE-merged on every rank)")
            if seq_shard else f"dp{world} (batch shards, no collective on the data path)"}


# --------------------------------------------------------------------------- #
#  GPU arm
# --------------------------------------------------------------------------- #

class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clocks not sampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) > 8 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows),
                "window": "nvidia-smi every 100 ms over the load window ending with the timed region"}


# DRAM bytes (read + write) of one launch of the workload's hot kernel from an ncu capture
# (--set full) of the same workload at the batch given, and the units (sequences) that
# capture processed.  Traffic grows in proportion to the sequences processed, so it is
# scaled to the benched batch.
NCU_TRAFFIC = {"c2": {"bytes": 356_055_552, "batch": 8,
                      "source": "ncu --set full capture of decode_mma_kernel, C2 at batch 8"},
               "c3": {"bytes": 142_390_528, "batch": 8,
                      "source": "ncu --set full capture of decode_mma_kernel, C3 at batch 8"},
               "c5": {"bytes": 261_946_112, "batch": 1,
                      "source": "ncu --set full capture of decode_mma_kernel, C5 at batch 1"},
               "c4": {"bytes": 58_652_672, "batch": 8,
                      "source": "ncu --set full capture of mla_tc_kernel, C4 at batch 8"},
               "prefill": {"bytes": 140_648_704, "batch": 2,
                           "source": "ncu --set full capture of prefill_tc_kernel<16>, the prefill workload"}}


def ncu_traffic(workload_name, batch, nbytes, shards=1):
    """DRAM bytes of one launch at this batch and a note on where they come from; nbytes = the
    algorithmic bytes of one launch (None: the workload's roofline unit is not bytes); shards =
    the ranks a sequence-sharded launch shares the pages with."""
    rec = NCU_TRAFFIC.get(workload_name)
    if rec is None:
        return None, "null (no ncu capture of this workload)"
    scaled = rec["bytes"] * batch / rec["batch"] / shards
    note = (f"dram__bytes_read.sum + dram__bytes_write.sum of one launch at batch {rec['batch']} "
            f"({rec['source']}), scaled x{batch / rec['batch'] / shards:g} to this launch")
    if nbytes:
        note += f"; {scaled / nbytes:.3f}x the algorithmic bytes"
    return int(scaled), note


def measured_hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def build_gpu_workload(w: dict, ids: np.ndarray, fmt: np.ndarray, device, rank: int):
    import torch
    from intent_attention import PagePool
    B, Hq, Hkv, D, PS, T = w["B"], w["Hq"], w["Hkv"], w["D"], w["PS"], w["T"]
    NLP = T // PS
    units = B * Hkv
    NP = units * NLP
    n = ids.size
    formats = sorted({k for k in w["mix"]})
    pool = PagePool.allocate(NP, PS, D, formats, w["scale_mode"], device)
    g = torch.Generator(device=device).manual_seed(w["seed"] * 131 + rank)
    ids_t = torch.from_numpy(ids).to(device)
    fmt_t = torch.from_numpy(fmt).to(device)
    tags = torch.zeros(NP, dtype=torch.uint8, device=device)
    chunk = max(1, (1 << 27) // (PS * D * n))       # ~512 MB of fp32 per plane per chunk
    for u0 in range(0, units, chunk):
        u1 = min(units, u0 + chunk)
        dst = (torch.arange(u0, u1, device=device, dtype=torch.int32)[:, None] * NLP + ids_t[None, :]).reshape(-1)
        P = dst.numel()
        k = torch.randn((P, PS, D), generator=g, device=device)
        v = torch.randn((P, PS, D), generator=g, device=device)
        if w["outliers"]:
            k = torch.where(torch.rand(k.shape, generator=g, device=device) < w["outliers"], k * 8, k)
            v = torch.where(torch.rand(v.shape, generator=g, device=device) < w["outliers"], v * 8, v)
        f = fmt_t.repeat(u1 - u0)
        pool.quantize_(k, v, f, dst_ids=dst)
        tags[dst.long()] = f
        del k, v
    table = (torch.arange(units, device=device, dtype=torch.int32)[:, None] * NLP + ids_t[None, :]).reshape(B, Hkv, n)
    counts = torch.full((B, Hkv), n, dtype=torch.int32, device=device)
    q = (torch.randn((B, Hq, D), generator=g, device=device) * w["q_std"]).to(torch.bfloat16)
    torch.cuda.synchronize(device)
    return pool, table.contiguous(), counts, tags, q


class _NoClocks:
    rows = ()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False

    def summary(self):
        return None


def pipelined_e2e(device, steps, warmup, h2d_pairs, d2h_pairs, run, world=1):
    """End-to-end steps through the public API with host buffers, as a serving loop runs them:
    every step copies its inputs from pinned host memory, calls the API and copies its result
    back.  Two sets of device buffers let step s+1's input copies (one copy stream) and step
    s-1's result copy (another) run while step s runs on the compute stream; each step's copies
    stay inside the timed region.  h2d_pairs: [(host, (dev0, dev1))]; d2h_pairs: [((dev0, dev1),
    (host0, host1))]; run(b) calls the API on buffer set b.  Returns ms per step (max over ranks)."""
    import torch
    import torch.distributed as dist
    compute = torch.cuda.current_stream(device)
    cin, cout = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev = {name: [torch.cuda.Event() for _ in range(2)] for name in ("in", "run", "out")}
    started = [False, False]

    def one(i):
        b = i & 1
        with torch.cuda.stream(cin):
            if started[b]:
                cin.wait_event(ev["run"][b])          # step i-2 has read these inputs
            for host, devs in h2d_pairs:
                devs[b].copy_(host, non_blocking=True)
            ev["in"][b].record(cin)
        compute.wait_event(ev["in"][b])
        if started[b]:
            compute.wait_event(ev["out"][b])          # step i-2's result has been copied out
        run(b)
        ev["run"][b].record(compute)
        with torch.cuda.stream(cout):
            cout.wait_event(ev["run"][b])
            for devs, hosts in d2h_pairs:
                hosts[b].copy_(devs[b], non_blocking=True)
            ev["out"][b].record(cout)
        started[b] = True

    for i in range(warmup):
        one(i)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    cin.wait_stream(compute)
    for i in range(steps):
        one(warmup + i)
    compute.wait_stream(cout)
    e1.record(compute)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def measure_decode(args, wl_name, world, rank, local, device, clocks_on=True):
    """Build one decode workload on this rank and time it (device step, the decode
    kernel alone, and end to end through the public API); times are max over ranks.
    Returns the numbers the JSON line is made of."""
    import torch
    import torch.distributed as dist
    from intent_attention._native import KernelTimer
    from intent_attention import paged_decode
    from intent_attention.paged import make_tag_map

    w = workload(wl_name)
    if args.batch:
        w["B"] = args.batch
    ids, fmt = select_pages(w)
    n_sel_total = int(ids.size)
    # C5 on several GPUs shards every sequence's selected pages by sequence range
    # (strong scaling, one all-gather of partial blocks per step); the other
    # workloads shard the batch (weak scaling, no collective on the data path)
    seq_shard = wl_name == "c5" and world > 1
    nbytes_total = step_bytes(w, fmt) * (1 if seq_shard else world)
    if seq_shard:
        from intent_attention.split_kv import SequenceShardedDecoder, shard_bounds
        a, b = shard_bounds(ids.size, rank, world)
        ids, fmt = ids[a:b], fmt[a:b]
        w["name"] = "C5 long-context decode, sequence-sharded split-KV"
    if not seq_shard and getattr(args, "shard_of", 0) > 1 and wl_name == "c5":
        # one rank's share of C5 cut over shard_of GPUs, decoded on this GPU alone (no exchange):
        # sizes the per-rank decode of the sequence-sharded case on one GPU
        from intent_attention.split_kv import shard_bounds
        a, b = shard_bounds(ids.size, 0, args.shard_of)
        ids, fmt = ids[a:b], fmt[a:b]
        nbytes_total = step_bytes(w, fmt)
        w["name"] = f"C5 long-context decode, rank 0's share of {args.shard_of} sequence shards (one GPU, no exchange)"
    nbytes = step_bytes(w, fmt)                     # this rank's selected-KV bytes per step
    pool, table, counts, tags, q = build_gpu_workload(w, ids, fmt, device, 0 if seq_shard else rank)
    tag_map = make_tag_map({c: (f if f in w["mix"] else "SKIP") for f, c in FMT_CODE.items()})
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=device)
    decoder = SequenceShardedDecoder(transport=args.exchange) if seq_shard else None

    def decode(q_, table_, counts_, out_=None):
        o = out if out_ is None else out_
        if decoder is not None:
            decoder.decode(q_, pool, table_, counts_, tags, tag_map, 0, out=o, num_splits=args.splits,
                           kernel="tensor")
        else:
            paged_decode(q_, pool, table_, counts_, tags, tag_map, 0, out=o, num_splits=args.splits,
                         kernel="tensor")

    def step():
        decode(q, table, counts)

    # NCCL collectives stay outside graph capture; every other path is captured
    use_graph = not args.no_graph and not (seq_shard and args.exchange == "nccl")

    step()
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with (ClockSampler(local) if clocks_on else _NoClocks()) as clocks:
        # nvidia-smi needs ~0.5 s to start sampling: keep the GPU under the same
        # load until samples arrive, so the clock record covers the load window
        # that ends with the timed region.  Every rank runs the same number of
        # probe rounds (steps may hold a collective).
        t_probe = time.perf_counter()
        while clocks_on:
            for _ in range(20):
                step()
            torch.cuda.synchronize(device)
            done = len(clocks.rows) >= 3 or time.perf_counter() - t_probe >= 3.0
            if world > 1:
                flag = torch.tensor([1 if done else 0], device=device)
                dist.all_reduce(flag, op=dist.ReduceOp.MIN)
                done = bool(flag.item())
            if done:
                break
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        # The step time is taken without the kernel timer: its event records sit between
        # the query preparation and the decode launch and would serialise the two launches
        # that programmatic dependent launch otherwise overlaps.
        if use_graph:
            # the K steps captured once as a CUDA graph (the library never allocates or
            # synchronises while decoding); one warm-up replay, then the timed replay
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(args.steps):
                    step()
            graph.replay()
            torch.cuda.synchronize(device)
            if world > 1:
                dist.barrier()
            ev0.record()
            graph.replay()
            ev1.record()
        else:
            ev0.record()
            for _ in range(args.steps):
                step()
            ev1.record()
        torch.cuda.synchronize(device)
        # the decode kernel's own time: the same steps again with the library's kernel timer
        with KernelTimer(args.steps) as ktimer:
            if use_graph:
                kgraph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(kgraph):
                    for _ in range(args.steps):
                        step()
                kgraph.replay()
                torch.cuda.synchronize(device)
                if world > 1:
                    dist.barrier()
                kgraph.replay()
            else:
                for _ in range(args.steps):
                    step()
            torch.cuda.synchronize(device)
    t_ms = ev0.elapsed_time(ev1) / args.steps
    kernel_ms = ktimer.total_ms / max(1, ktimer.launches)
    if use_graph:
        del graph, kgraph
    if world > 1:
        t = torch.tensor([t_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms = float(t.item())
        dist.barrier()

    # ---- end to end through the public API: host buffers in, host buffer out
    q_host = q.cpu().pin_memory()
    table_host = table.cpu().pin_memory()
    counts_host = counts.cpu().pin_memory()
    out_hosts = tuple(torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2))
    q_devs = (torch.empty_like(q), torch.empty_like(q))
    table_devs = (torch.empty_like(table), torch.empty_like(table))
    counts_devs = (torch.empty_like(counts), torch.empty_like(counts))
    out_devs = (out, torch.empty_like(out))
    h2d = q_host.numel() * q_host.element_size() + table_host.numel() * 4 + counts_host.numel() * 4
    d2h = out.numel() * out.element_size()
    e2e_ms = pipelined_e2e(device, args.steps, args.warmup,
                           [(q_host, q_devs), (table_host, table_devs), (counts_host, counts_devs)],
                           [(out_devs, out_hosts)],
                           lambda b: decode(q_devs[b], table_devs[b], counts_devs[b], out_devs[b]), world)

    # tensor-core path (forced above, so an ineligible shape fails loudly): query-table preparation
    # and the persistent decode kernel, which merges its partials itself
    # + for sequence shards: the block merge after NCCL's all-gather, or (peer stores, issued by the
    # decode kernel itself) one bounded-wait + block-merge kernel
    launches_per_step = 2 + (1 if seq_shard else 0)
    if world > 1:
        t = torch.tensor([kernel_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        kernel_ms = float(t.item())

    if decoder is not None:
        if decoder._x is not None:
            decoder._x.check()
        if world > 1:
            dist.barrier()
        decoder.close()
    return dict(w=w, ids=ids, fmt=fmt, n_sel_total=n_sel_total, seq_shard=seq_shard, nbytes=nbytes,
                nbytes_total=nbytes_total, t_ms=t_ms, kernel_ms=kernel_ms, e2e_ms=e2e_ms, h2d=h2d, d2h=d2h,
                use_graph=use_graph, clocks=clocks.summary(), launches_per_step=launches_per_step)


def run_gpu(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    m = measure_decode(args, args.workload, world, rank, local, device)
    # The sequence-sharded C5 step beside the default C2 line: the same run (and, for the
    # driver's 1-8 GPU scaling run, every N) also times C5 cut by sequence over the ranks
    # (strong scaling; unsharded on one GPU).
    c5 = None
    if args.workload == "c2" and not args.no_c5_strong:
        torch.cuda.empty_cache()
        import copy
        a5 = copy.copy(args)
        a5.workload, a5.batch, a5.exchange = "c5", 0, "p2p"
        c5 = measure_decode(a5, "c5", world, rank, local, device, clocks_on=False)
        torch.cuda.empty_cache()
    w, ids, fmt, n_sel_total, seq_shard = m["w"], m["ids"], m["fmt"], m["n_sel_total"], m["seq_shard"]
    nbytes, nbytes_total, t_ms, kernel_ms, e2e_ms = m["nbytes"], m["nbytes_total"], m["t_ms"], m["kernel_ms"], m["e2e_ms"]
    h2d, d2h, use_graph, launches_per_step = m["h2d"], m["d2h"], m["use_graph"], m["launches_per_step"]
    if rank == 0:
        peak, peak_kind = measured_hbm_peak()
        gbs = nbytes / (t_ms * 1e-3) / 1e9
        kernel_gbs = nbytes / (kernel_ms * 1e-3) / 1e9
        value = nbytes_total / (t_ms * 1e-3) / 1e9
        traffic, traffic_note = ncu_traffic(args.workload, w["B"], nbytes, world if seq_shard else 1)
        rec = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms, 5), "us_per_step": round(t_ms * 1e3, 2),
            "higher_is_better": True, "scaling": "strong" if seq_shard else "weak", "vs_baseline": None, "dtype": "fp16/fp8/int8 pages, fp32 acc",
            "data": "synthetic (seeded N(0,1) K/V with 1% x8 outliers, bf16 Q)",
            "config": workload_config(w, n_sel_total, int(ids.size), world, seq_shard, nbytes, args.exchange),
            "timing": ("one CUDA graph of all timed steps, replayed once after a warm-up replay"
                       if use_graph else "eager launches"),
            "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(kernel_gbs / peak, 4), "traffic": traffic,
                         "kernel": "decode_mma_kernel", "kernel_us": round(kernel_ms * 1e3, 2),
                         "step_frac": round(gbs / peak, 4),
                         "note": f"peak = {peak_kind} HBM copy bandwidth; achieved = algorithmic selected-KV bytes "
                                 "per launch / average CUDA-event duration of the persistent decode kernel over the "
                                 "timed region; step_frac uses the whole step (query preparation + decode, which merges its "
                                 "partials in-kernel); traffic = "
                                 + traffic_note},
            "e2e": {"value": round(nbytes_total / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": ("intent_attention.SequenceShardedDecoder.decode" if seq_shard else
                            "intent_attention.paged_decode") +
                           " with pinned host q / page table / counts in, output out; two buffer sets, the "
                           "next step's input copies and the previous step's output copy on copy streams"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": m["clocks"],
        }
        if world == 1 and not args.no_cpu_baseline:
            rec["cpu_baseline"] = cpu_baseline_record(CpuDecodeSample(w, ids, fmt), args.cpu_budget)
            ref_rec = reference_cpu_record(args.workload)
            if ref_rec is not None:
                rec["cpu_baseline_reference"] = ref_rec
        if c5 is not None:
            c5_peak = measured_hbm_peak()[0]
            rec["c5_strong"] = {
                "workload": "C5 long-context decode (batch 8, 32 q / 8 kv heads, 512k ctx, 8192 selected pages "
                            "per (sequence, kv head))" + (f", cut by sequence over {world} GPUs" if world > 1 else
                                                          ", one GPU"),
                "scaling": "strong" if world > 1 else "single GPU",
                "value": round(c5["nbytes_total"] / (c5["t_ms"] * 1e-3) / 1e9, 2), "unit": "GB/s",
                "us_per_step": round(c5["t_ms"] * 1e3, 2), "kernel_us": round(c5["kernel_ms"] * 1e3, 2),
                "kernel_frac": round(c5["nbytes"] / (c5["kernel_ms"] * 1e-3) / 1e9 / c5_peak, 4),
                "selected_kv_bytes_per_step": c5["nbytes_total"], "selected_kv_bytes_per_gpu": c5["nbytes"],
                "e2e": {"value": round(c5["nbytes_total"] / (c5["e2e_ms"] * 1e-3) / 1e9, 2), "unit": "GB/s",
                        "ms_per_step": round(c5["e2e_ms"], 5)},
                "exchange": ("partial (m, l, acc) rows stored by the decode kernel into every rank's receive "
                             "slot over NVLink, flags raised by its last unit, one bounded-wait + merge kernel"
                             if world > 1 else "none"),
                "gpu_launches_per_step": c5["launches_per_step"],
                "timing": "one CUDA graph of all timed steps, max over ranks"}
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    """The reference arm: the reference algorithm's CPU implementation on the host
    cores (the numpy port that the tests pin to the reference's own outputs), on
    the same workload and config as the GPU arm.  Each step decodes a bounded
    sample of the workload's (sequence, kv head) units, whole waves of one unit
    per host thread for at least ``--ref-step-s`` seconds; ``value`` is the
    sample's selected-KV bytes / its measured time and ``ms_per_step`` the
    sample's measured time (nothing is extrapolated).  Under torchrun rank 0
    alone runs."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "c4":
        return run_reference_mla(args, world)
    w = workload(args.workload)
    if args.batch:
        w["B"] = args.batch
    ids, fmt = select_pages(w)
    n_sel_total = int(ids.size)
    seq_shard = args.workload == "c5" and world > 1
    ids_r, fmt_r = ids, fmt
    if seq_shard:
        from intent_attention.split_kv import shard_bounds
        a, b = shard_bounds(ids.size, 0, world)
        ids_r, fmt_r = ids[a:b], fmt[a:b]
        w["name"] = "C5 long-context decode, sequence-sharded split-KV"
    sample = CpuDecodeSample(w, ids, fmt)
    rates, secs, units = [], [], []
    for i in range(args.warmup + args.steps):
        sec, n = sample.run_for(args.ref_step_s)
        if i >= args.warmup:
            rates.append(n * sample.bytes_per_unit / sec)
            secs.append(sec)
            units.append(n)
    v = statistics.median(rates) / 1e9
    rec = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.median(secs) * 1e3, 3),
           "higher_is_better": True, "scaling": "strong" if seq_shard else "weak", "vs_baseline": None,
           "dtype": "fp32 dequantisation, fp64 attention (numpy)", "data": "synthetic",
           "config": workload_config(w, n_sel_total, int(ids_r.size), world, seq_shard, step_bytes(w, fmt_r),
                                     args.exchange),
           "step": (f"a sample of {int(statistics.median(units))} of the step's {sample.units_total} (sequence, kv "
                    "head) units (median over steps) decoded on the host cores; ms_per_step is the sample's "
                    "measured time"),
           "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": sample.cores, "kind": "port",
                            "sample": f"whole waves of {sample.cores} (sequence, kv head) units per step, at least "
                                      f"{args.ref_step_s} s each, numpy oracle decode of the workload's pages"},
           "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    ref_rec = reference_cpu_record(args.workload)
    if ref_rec is not None:
        rec["cpu_baseline_reference"] = ref_rec
    print(json.dumps(rec), flush=True)


# --------------------------------------------------------------------------- #
#  C4: DeepSeek-V2-shape MLA absorbed decode (tcgen05 / TMEM kernel)
# --------------------------------------------------------------------------- #

C4 = dict(name="C4 DeepSeek-V2-shape MLA absorbed decode", B=64, H=128, Dqk=576, Dv=512, T=16384, PS=64,
          recent_tokens=2048, select_pages=154, seed=1004)


def select_mla_pages(w: dict):
    """Router-selected latent pages (one-page ATTEND blocks with seeded scores
    plus the RECENT tail) and their formats: the last ``recent_tokens`` stay
    BF16 (tag 0), the rest are FP8 (tag 1)."""
    from intent_attention import BlockLayout, BlockPolicy, BlockRouter, RouterConfig, SemanticBlock
    from intent_attention import routing_to_kernel_metadata
    PS, T = w["PS"], w["T"]
    rng = np.random.default_rng(w["seed"])
    tail = T - w["recent_tokens"]
    blocks = [SemanticBlock(f"lat{i}", i * PS, (i + 1) * PS, BlockPolicy.ATTEND, score=float(rng.random()))
              for i in range(tail // PS)]
    blocks.append(SemanticBlock("recent", tail, T, BlockPolicy.RECENT))
    top_k = w["select_pages"] - w["recent_tokens"] // PS
    router = BlockRouter(RouterConfig(top_k_blocks=top_k, memory_pressure=0.0))
    meta = routing_to_kernel_metadata(router.route_layout(BlockLayout(blocks), T), PS)
    ids = np.asarray(meta["selected_page_ids"], dtype=np.int32)
    tags = np.where(ids >= tail // PS, 0, 1).astype(np.uint8)
    return ids, tags


def mla_bytes_flops(w: dict, tags: np.ndarray):
    """Algorithmic bytes (latent codes + FP8 page scales of every selected
    page) and FLOPs (QK over d_qk + PV over d_v per head and token) per step."""
    PS, Dqk = w["PS"], w["Dqk"]
    per_seq = sum(PS * Dqk * 2 if t == 0 else PS * Dqk + 4 for t in tags)
    tokens = tags.size * PS
    flops = 2 * (w["Dqk"] + w["Dv"]) * w["H"] * tokens * w["B"]
    return per_seq * w["B"], flops


def build_mla_workload(w: dict, ids: np.ndarray, tags_sel: np.ndarray, device, rank: int):
    import torch
    B, H, Dqk, PS, T = w["B"], w["H"], w["Dqk"], w["PS"], w["T"]
    NLP = T // PS
    NP = B * NLP
    dense = torch.empty((NP, PS, Dqk), dtype=torch.bfloat16, device=device)
    fp8 = torch.empty((NP, PS, Dqk), dtype=torch.uint8, device=device)
    scale = torch.ones(NP, dtype=torch.float32, device=device)
    tags = torch.full((NP,), 2, dtype=torch.uint8, device=device)   # unselected pages: SKIP
    g = torch.Generator(device=device).manual_seed(w["seed"] * 131 + rank)
    ids_t = torch.from_numpy(ids).to(device).long()
    is_dense = torch.from_numpy(tags_sel).to(device) == 0
    for b in range(B):
        dst = b * NLP + ids_t
        x = torch.randn((ids.size, PS, Dqk), generator=g, device=device)
        dense[dst[is_dense]] = x[is_dense].to(torch.bfloat16)
        xf = x[~is_dense]
        sc = torch.clamp(xf.abs().amax(dim=(1, 2)) / 127.0, min=1e-8)
        fp8[dst[~is_dense]] = (xf / sc[:, None, None]).to(torch.float8_e4m3fn).view(torch.uint8)
        scale[dst[~is_dense]] = sc
        tags[dst] = torch.where(is_dense, 0, 1).to(torch.uint8)
    table = (torch.arange(B, device=device, dtype=torch.int32)[:, None] * NLP + ids_t[None, :].int()).contiguous()
    q = torch.randn((B, H, Dqk), generator=g, device=device).to(torch.bfloat16)
    torch.cuda.synchronize(device)
    return dense, fp8, scale, tags, table, q


class CpuMlaSample:
    """The numpy oracle's per-head MLA decode of whole sequences of the C4
    workload on the host cores (one sequence's latents built once, reused)."""

    def __init__(self, w: dict, ids: np.ndarray, tags_sel: np.ndarray):
        from oracle import quant as oq
        self.w = w
        self.cores = len(os.sched_getaffinity(0))
        PS, Dqk, H = w["PS"], w["Dqk"], w["H"]
        n = ids.size
        rng = np.random.default_rng(w["seed"] + 7)
        lat = rng.standard_normal((n, PS, Dqk)).astype(np.float32)
        self.scale = np.maximum(np.abs(lat).reshape(n, -1).max(1) / 127.0, 1e-8).astype(np.float32)
        self.pools = {"bf16": lat, "fp8": oq.f32_to_e4m3(lat / self.scale[:, None, None])}
        self.q = rng.standard_normal((1, H, Dqk)).astype(np.float32)
        self.table = np.arange(n)[None, :]
        self.tags = tags_sel.astype(np.int64)
        self.bytes_per_seq = mla_bytes_flops(w, tags_sel)[0] / w["B"]

    def _one(self, _):
        from oracle import mla as omla
        return omla.mla_paged_decode(self.q, self.table, None, self.tags, self.pools, self.scale, self.w["Dv"],
                                     1.0 / math.sqrt(self.w["Dqk"]))

    def run_for(self, budget_s: float):
        """Whole waves of one sequence per core until ``budget_s`` has passed (at
        least one wave).  Returns (seconds, sequences decoded)."""
        import concurrent.futures as cf
        done = 0
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(max_workers=self.cores) as ex:
            while done == 0 or time.perf_counter() - t0 < budget_s:
                list(ex.map(self._one, range(self.cores)))
                done += self.cores
        return time.perf_counter() - t0, done


def mla_config(w: dict, ids: np.ndarray, tags_sel: np.ndarray, world: int) -> dict:
    """The ``config`` object both arms print for the C4 workload."""
    nbytes, flops = mla_bytes_flops(w, tags_sel)
    return {"workload": w["name"], "batch_per_gpu": w["B"], "global_batch": w["B"] * world,
            "q_heads": w["H"], "d_qk": w["Dqk"], "d_v": w["Dv"], "ctx": w["T"], "page_size": w["PS"],
            "selected_pages_per_seq": int(ids.size), "bf16_pages_per_seq": int((tags_sel == 0).sum()),
            "fp8_pages_per_seq": int((tags_sel == 1).sum()),
            "selected_kv_bytes_per_step_per_gpu": nbytes, "flops_per_step_per_gpu": flops,
            "l2": l2_note(nbytes, "selected latents"),
            "parallelism": f"dp{world} (batch shards, no collective on the data path)"}


def run_reference_mla(args, world):
    w = dict(C4)
    if args.batch:
        w["B"] = args.batch
    ids, tags_sel = select_mla_pages(w)
    sample = CpuMlaSample(w, ids, tags_sel)
    rates, secs, seqs = [], [], []
    for i in range(args.warmup + args.steps):
        sec, n = sample.run_for(args.ref_step_s)
        if i >= args.warmup:
            rates.append(n * sample.bytes_per_seq / sec)
            secs.append(sec)
            seqs.append(n)
    v = statistics.median(rates) / 1e9
    rec = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(statistics.median(secs) * 1e3, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp64 (numpy)",
           "data": "synthetic", "config": mla_config(w, ids, tags_sel, world),
           "step": (f"a sample of {int(statistics.median(seqs))} of the step's {w['B']} sequences (median over "
                    "steps) decoded on the host cores; ms_per_step is the sample's measured time"),
           "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": sample.cores, "kind": "port",
                            "sample": f"whole waves of {sample.cores} sequences per step, at least "
                                      f"{args.ref_step_s} s each, numpy oracle per-head MLA decode"},
           "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(rec), flush=True)


def measured_tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def run_gpu_mla(args):
    import torch
    import torch.distributed as dist
    from intent_attention._native import KernelTimer
    from intent_attention.triton_mla_decode import make_mla_tag_map, mla_paged_decode

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    w = dict(C4)
    if args.batch:
        w["B"] = args.batch
    ids, tags_sel = select_mla_pages(w)
    nbytes, flops = mla_bytes_flops(w, tags_sel)
    dense, fp8, scale, tags, table, q = build_mla_workload(w, ids, tags_sel, device, rank)
    tag_map = make_mla_tag_map({0: "DENSE", 1: "FP8", 2: "SKIP"})
    out = torch.empty((w["B"], w["H"], w["Dv"]), dtype=torch.bfloat16, device=device)

    def decode(q_, table_, out_=None):
        mla_paged_decode(q_, table_, None, dense_pages=dense, fp8_pages=fp8, fp8_scale=scale, page_tags=tags,
                         tag_map=tag_map, d_v=w["Dv"], out=out if out_ is None else out_, num_splits=args.splits,
                         kernel="tensor")

    decode(q, table)
    torch.cuda.synchronize(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t_probe = time.perf_counter()
        while True:
            for _ in range(10):
                decode(q, table)
            torch.cuda.synchronize(device)
            done = len(clocks.rows) >= 3 or time.perf_counter() - t_probe >= 3.0
            if world > 1:
                flag = torch.tensor([1 if done else 0], device=device)
                dist.all_reduce(flag, op=dist.ReduceOp.MIN)
                done = bool(flag.item())
            if done:
                break
        for _ in range(args.warmup):
            decode(q, table)
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
        with KernelTimer(args.steps) as ktimer:
            ev0.record()
            for _ in range(args.steps):
                decode(q, table)
            ev1.record()
            torch.cuda.synchronize(device)
    t_ms = ev0.elapsed_time(ev1) / args.steps
    kernel_ms = ktimer.total_ms / max(1, ktimer.launches)

    q_host, table_host = q.cpu().pin_memory(), table.cpu().pin_memory()
    out_hosts = tuple(torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2))
    q_devs, table_devs = (torch.empty_like(q), torch.empty_like(q)), (torch.empty_like(table), torch.empty_like(table))
    out_devs = (out, torch.empty_like(out))
    h2d = q_host.numel() * q_host.element_size() + table_host.numel() * 4
    d2h = out.numel() * out.element_size()
    e2e_ms = pipelined_e2e(device, args.steps, args.warmup, [(q_host, q_devs), (table_host, table_devs)],
                           [(out_devs, out_hosts)], lambda b: decode(q_devs[b], table_devs[b], out_devs[b]), world)
    if world > 1:
        t = torch.tensor([t_ms, kernel_ms, e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_ms, kernel_ms, e2e_ms = (float(x) for x in t.tolist())

    if rank == 0:
        hbm_peak, hbm_kind = measured_hbm_peak()
        tc_peak, tc_kind = measured_tensor_peak()
        tflops = flops / (kernel_ms * 1e-3) / 1e12
        kernel_gbs = nbytes / (kernel_ms * 1e-3) / 1e9
        gbs = nbytes / (t_ms * 1e-3) / 1e9
        n_sel = int(ids.size)
        rec = {
            "metric": METRIC, "value": round(gbs * world, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t_ms, 5), "us_per_step": round(t_ms * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16/fp8-e4m3 latent pages, f16 tensor-core operands, fp32 acc",
            "data": "synthetic (seeded N(0,1) latents and bf16 Q)",
            "config": mla_config(w, ids, tags_sel, world),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": tc_peak, "unit": "TFLOP/s",
                         "frac": round(tflops / tc_peak, 4), "traffic": ncu_traffic("c4", w["B"], nbytes)[0],
                         "traffic_note": ncu_traffic("c4", w["B"], nbytes)[1], "kernel": "mla_tc_kernel",
                         "kernel_us": round(kernel_ms * 1e3, 2),
                         "hbm": {"achieved": round(kernel_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                                 "frac": round(kernel_gbs / hbm_peak, 4)},
                         "note": f"peak = {tc_kind} cuBLAS bf16 GEMM (burst); achieved = useful FLOPs per launch "
                                 "(2*(d_qk+d_v) per head and selected token; each work item runs on a pair of "
                                 "CTAs that split the latent channels, so no FLOP is computed twice) / "
                                 "CUDA-event kernel time; hbm = selected "
                                 f"latent bytes / the same time vs the {hbm_kind} copy bandwidth"},
            "e2e": {"value": round(nbytes * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "intent_attention.triton_mla_decode.mla_paged_decode with pinned host q / page table "
                           "in, context out; two buffer sets, the next step's input copies and the previous "
                           "step's output copy on copy streams"},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            mla_sample = CpuMlaSample(w, ids, tags_sel)
            sec, seqs = mla_sample.run_for(args.cpu_budget)
            rec["cpu_baseline"] = {"value": round(seqs * mla_sample.bytes_per_seq / sec / 1e9, 4), "unit": "GB/s",
                                   "cores": mla_sample.cores, "kind": "port", "seconds": round(sec, 3),
                                   "sample": f"{seqs} sequences decoded by the numpy oracle's per-head MLA decode "
                                             f"on {mla_sample.cores} host threads in {sec:.2f} s; value = their "
                                             "selected latent bytes / that time"}
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- #
#  Device router (iak_route_pages) on the C2 layout
# --------------------------------------------------------------------------- #

ROUTE_METRIC = "device router: sequences routed (block routing + page list + precision map + table rows) per s"


def route_workload(batch: int = 0):
    """C2's semantic layout (system prompt, 64-token ATTEND blocks, recent
    tail) for every sequence of the batch, each with its own seeded scores."""
    from intent_attention import BlockLayout, BlockPolicy, RouterConfig, SemanticBlock
    w = workload("c2")
    if batch:
        w["B"] = batch
    PS, T = w["PS"], w["T"]
    rng = np.random.default_rng(w["seed"] + 77)
    bt = w["attend_block_pages"] * PS
    mid_start, mid_end = w["head_tokens"], T - w["tail_tokens"]
    layouts = []
    for _ in range(w["B"]):
        blocks = [SemanticBlock("system", 0, w["head_tokens"], BlockPolicy.ALWAYS)]
        for i in range((mid_end - mid_start) // bt):
            blocks.append(SemanticBlock(f"doc{i}", mid_start + i * bt, mid_start + (i + 1) * bt, BlockPolicy.ATTEND,
                                        score=float(rng.random())))
        blocks.append(SemanticBlock("recent", mid_end, T, BlockPolicy.RECENT))
        layouts.append(BlockLayout(blocks))
    fixed = (w["head_tokens"] + w["tail_tokens"]) // PS
    cfg = RouterConfig(top_k_blocks=(w["select_pages"] - fixed) // w["attend_block_pages"], memory_pressure=0.0)
    return w, layouts, cfg


def cpu_route(w, layouts, cfg, budget_s: float):
    """Host routing per sequence (route_layout + selected_page_ids + the
    precision map of routing_to_kernel_metadata + table rows): seconds per
    sequence over a bounded sample."""
    from intent_attention import BlockRouter, routing_to_kernel_metadata
    router = BlockRouter(cfg)
    PS, T, Hkv, NLP = w["PS"], w["T"], w["Hkv"], w["T"] // w["PS"]
    t0 = time.perf_counter()
    done = 0
    while done < len(layouts) and (time.perf_counter() - t0 < budget_s or done == 0):
        routed = router.route_layout(layouts[done], T)
        meta = routing_to_kernel_metadata(routed, PS)
        ids = np.asarray(meta["selected_page_ids"], dtype=np.int32)
        rows = (np.arange(Hkv, dtype=np.int32)[:, None] + done * Hkv) * NLP + ids[None, :]
        _ = rows, [meta["block_precision_by_page"][str(p)] for p in ids[:4]]
        done += 1
    return (time.perf_counter() - t0) / done, done


def run_route(args):
    import torch
    from intent_attention import KVPrecision, encode_layouts, route_pages
    from intent_attention.device_router import RoutedPages
    w, layouts, cfg = route_workload(args.batch)
    if args.impl == "reference":
        vals, n = [], 0
        for i in range(args.warmup + args.steps):
            sec, n = cpu_route(w, layouts, cfg, args.cpu_budget / max(1, args.steps + args.warmup))
            if i >= args.warmup:
                vals.append(sec)
        v = 1.0 / statistics.median(vals)
        print(json.dumps({"impl": "reference", "metric": ROUTE_METRIC, "value": round(v, 2), "unit": "seq/s",
                          "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": round(w["B"] / v * 1e3, 3), "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "float64 scores", "data": "synthetic",
                          "config": {"workload": "C2 layout routing", "batch": w["B"]},
                          "cpu_baseline": {"value": round(v, 2), "unit": "seq/s", "cores": 1, "kind": "port",
                                           "sample": f"{n} sequences per step through the host BlockRouter"},
                          "e2e": {"value": round(v, 2), "unit": "seq/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B, Hkv, PS, T = w["B"], w["Hkv"], w["PS"], w["T"]
    NLP, W = T // PS, T // PS
    batch = encode_layouts(layouts, device)
    nb = batch.num_blocks
    bases = (torch.arange(B * Hkv, dtype=torch.int32, device=device) * NLP).view(B, Hkv)
    tags = torch.zeros(B * Hkv * NLP, dtype=torch.uint8, device=device)
    prec_to_tag = {KVPrecision.FP16: 1, KVPrecision.FP8: 2, KVPrecision.INT8: 3, KVPrecision.INT4: 4,
                   KVPrecision.INT4_RESIDUAL: 5, KVPrecision.SKIP: 0}
    out = RoutedPages(torch.empty((B, Hkv, W), dtype=torch.int32, device=device),
                      torch.empty((B, Hkv), dtype=torch.int32, device=device),
                      torch.empty(B, dtype=torch.int32, device=device),
                      torch.empty((B, W), dtype=torch.uint8, device=device))

    def step(lb=batch):
        route_pages(lb, cfg, PS, W, table_heads=Hkv, bases=bases, page_tags=tags, prec_to_tag=prec_to_tag, out=out)

    step()
    torch.cuda.synchronize()
    n_sel = out.num_selected.cpu()
    assert (n_sel == w["select_pages"]).all(), n_sel
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        t_probe = time.perf_counter()
        while len(clocks.rows) < 3 and time.perf_counter() - t_probe < 3.0:
            for _ in range(50):
                step()
            torch.cuda.synchronize()
        for _ in range(args.warmup):
            step()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                step()
        graph.replay()
        torch.cuda.synchronize()
        ev0.record()
        graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    t_ms = ev0.elapsed_time(ev1) / args.steps
    del graph
    # end to end: per-sequence scores from pinned host memory, counts and
    # selected totals back to the host
    scores_host = batch.scores.cpu().pin_memory()
    counts_host = torch.empty((B, Hkv), dtype=torch.int32).pin_memory()
    nsel_host = torch.empty(B, dtype=torch.int32).pin_memory()
    scores_dev = torch.empty_like(batch.scores)
    from intent_attention import LayoutBatch
    lb_e2e = LayoutBatch(batch.start, batch.end, batch.policy, scores_dev, batch.counts)

    def e2e_step():
        scores_dev.copy_(scores_host, non_blocking=True)
        step(lb_e2e)
        counts_host.copy_(out.page_counts, non_blocking=True)
        nsel_host.copy_(out.num_selected, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    # algorithmic bytes per launch: layout + scores read, table rows / counts /
    # precisions / tags written
    n = w["select_pages"]
    nbytes = B * (nb * (4 + 4 + 1 + 8) + Hkv * W * 4 + Hkv * 4 + 4 + W + Hkv * n)
    peak, peak_kind = measured_hbm_peak()
    gbs = nbytes / (t_ms * 1e-3) / 1e9
    rec = {"metric": ROUTE_METRIC, "value": round(B / (t_ms * 1e-3), 1), "unit": "seq/s", "n_gpus": 1,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms, 5),
           "us_per_step": round(t_ms * 1e3, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "float64 scores, int32 pages", "data": "synthetic (seeded per-sequence block scores)",
           "config": {"workload": "C2 layout routing (iak_route_pages)", "batch": B, "blocks_per_seq": nb,
                      "kv_heads": Hkv, "page_size": PS, "table_width": W, "pages_listed_per_seq": n,
                      "top_k_blocks": cfg.top_k_blocks,
                      "l2": "inputs smaller than L2 (a per-step router reads its layout from L2 in practice)",
                      "timing": "one CUDA graph of all timed launches, replayed once after a warm-up replay"},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 5), "traffic": None, "kernel": "route_kernel",
                        "kernel_us": round(t_ms * 1e3, 2),
                        "note": f"peak = {peak_kind} HBM copy bandwidth; latency-bound (one CTA per sequence, "
                                "bitonic sort + 4 CTA scans), not bandwidth-bound"},
           "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "seq/s", "ms_per_step": round(e2e_ms, 5),
                   "h2d_bytes_per_step": scores_host.numel() * 8,
                   "d2h_bytes_per_step": counts_host.numel() * 4 + nsel_host.numel() * 4,
                   "api": "intent_attention.route_pages with pinned host scores in, counts out"},
           "gpu_launches": args.steps, "clocks": clocks.summary()}
    if not args.no_cpu_baseline:
        sec, done = cpu_route(w, layouts, cfg, args.cpu_budget)
        rec["cpu_baseline"] = {"value": round(1.0 / sec, 2), "unit": "seq/s", "cores": 1, "kind": "port",
                               "sample": f"{done} sequences through the host BlockRouter (route_layout + "
                                         "routing_to_kernel_metadata + table rows)"}
    print(json.dumps(rec), flush=True)


# --------------------------------------------------------------------------- #
#  Chunked prefill over router-selected pages (iak_prefill, tcgen05 kernel)
# --------------------------------------------------------------------------- #

PREFILL_METRIC = "chunked-prefill attention over router-selected pages: useful TFLOP/s (causal, exact tokens)"
PREFILL = dict(name="Llama-3-8B-shape GQA chunked prefill over router-selected pages", B=2, M=2048)


def prefill_workload(args):
    """C2's model shape and router layout; per sequence the last M tokens of
    the 32k context are the query chunk (positions T - M .. T - 1), attending
    causally to the router-selected pages (1024 of 2048, C2 format mix)."""
    w = workload("c2")
    w["B"] = args.batch or PREFILL["B"]
    w["M"] = PREFILL["M"]
    ids, fmt = select_pages(w)
    PS, T, M, D = w["PS"], w["T"], w["M"], w["D"]
    pos = np.sort((ids.astype(np.int64)[:, None] * PS + np.arange(PS)[None, :]).reshape(-1))
    qpos = T - M + np.arange(M)
    pairs = int(np.searchsorted(pos, qpos, side="right").sum())        # visible (query, key) pairs per q head
    flops = 4 * D * pairs * w["Hq"] * w["B"]
    return w, ids, fmt, qpos, pairs, flops


def cpu_prefill(w, ids, fmt, qpos, budget_s, rows=8):
    """The numpy oracle over a few query rows of one (sequence, kv head) unit,
    extrapolated to the step: seconds per step."""
    import sys as _s
    _s.path.insert(0, ROOT)
    from oracle import prefill as op
    g = np.random.default_rng(3)
    PS, D, n = w["PS"], w["D"], ids.size
    pools = {"k_f16": g.standard_normal((n, PS, D)).astype(np.float32),
             "v_f16": g.standard_normal((n, PS, D)).astype(np.float32)}
    table = np.arange(n, dtype=np.int32).reshape(1, 1, n)
    ppos = (ids.astype(np.int64) * PS).reshape(1, 1, n)
    tags = np.ones(n, np.uint8)
    t0 = time.perf_counter()
    done = 0
    while done == 0 or (time.perf_counter() - t0 < budget_s and done < 64):
        sel = qpos[-rows:] if done % 2 else qpos[:rows]
        q = g.standard_normal((1, 1, rows, D)).astype(np.float32)
        op.paged_prefill(q, table, None, tags, {1: "F16"}, pools, bases=None, q_positions=sel[None],
                         causal=True, page_positions=ppos)
        done += 1
    per_row = (time.perf_counter() - t0) / (done * rows)
    return per_row * w["M"] * w["Hq"] * w["B"], done * rows


def run_prefill(args):
    import torch
    from intent_attention import PagePool
    from intent_attention._native import KernelTimer
    from intent_attention.paged import make_tag_map, paged_prefill
    w, ids, fmt, qpos, pairs, flops = prefill_workload(args)
    if args.impl == "reference":
        vals, rows = [], 0
        for i in range(args.warmup + args.steps):
            sec, rows = cpu_prefill(w, ids, fmt, qpos, args.cpu_budget / max(1, args.steps + args.warmup))
            if i >= args.warmup:
                vals.append(sec)
        sec = statistics.median(vals)
        v = flops / sec / 1e12
        print(json.dumps({"impl": "reference", "metric": PREFILL_METRIC, "value": round(v, 6), "unit": "TFLOP/s",
                          "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1),
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp64 (numpy)",
                          "data": "synthetic", "config": {"workload": PREFILL["name"], "batch": w["B"]},
                          "cpu_baseline": {"value": round(v, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
                                           "sample": f"{rows} query rows of one (sequence, kv head) unit through the "
                                                     "numpy oracle, extrapolated"},
                          "e2e": {"value": round(v, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B, Hq, Hkv, D, PS, T, M = w["B"], w["Hq"], w["Hkv"], w["D"], w["PS"], w["T"], w["M"]
    pool, table, counts, tags, _ = build_gpu_workload(w, ids, fmt, device, 0)
    tag_map = make_tag_map({c: (f if f in w["mix"] else "SKIP") for f, c in FMT_CODE.items()})
    NLP = T // PS
    bases = (torch.arange(B * Hkv, dtype=torch.int32, device=device) * NLP).view(B, Hkv)
    g = torch.Generator(device=device).manual_seed(w["seed"] + 9)
    q = torch.randn((B, Hq, M, D), generator=g, device=device).to(torch.bfloat16)
    qp = torch.from_numpy(np.tile(qpos.astype(np.int32), (B, 1))).to(device)
    out = torch.empty((B, Hq, M, D), dtype=torch.bfloat16, device=device)

    def step(q_=q):
        paged_prefill(q_, pool, table, counts, tags, tag_map, q_positions=qp, causal=True, bases=bases, out=out,
                      kernel="tensor")

    # the selected KV (kv_bytes) and q fit in L2: every timed step starts from a flushed L2 (a write
    # larger than L2 between steps, outside the step's own CUDA events)
    ns = n_scales(w["scale_mode"], D)
    kv_bytes = sum(page_bytes(int(f), PS, D, ns) for f in fmt) * B * Hkv
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=device)

    def timed(fn, n):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for a, b in evs:
            flush.zero_()
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / n

    step()
    torch.cuda.synchronize()
    with ClockSampler(0) as clocks:
        t_probe = time.perf_counter()
        while len(clocks.rows) < 3 and time.perf_counter() - t_probe < 3.0:
            for _ in range(5):
                step()
            torch.cuda.synchronize()
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        with KernelTimer(args.steps) as ktimer:
            t_ms = timed(step, args.steps)
    kernel_ms = ktimer.total_ms / max(1, ktimer.launches)
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    q_dev = torch.empty_like(q)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        step(q_dev)
        out_host.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ms = timed(e2e_step, args.steps)
    peak, peak_kind = measured_tensor_peak()
    tf = flops / (kernel_ms * 1e-3) / 1e12
    rec = {"metric": PREFILL_METRIC, "value": round(flops / (t_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_ms, 4),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16 q, fp16/fp8/int8 pages -> f16 tcgen05 MMA, fp32 accumulate",
           "data": "synthetic (seeded N(0,1) K/V, bf16 Q)",
           "config": {"workload": PREFILL["name"], "batch": B, "query_tokens": M, "q_heads": Hq, "kv_heads": Hkv,
                      "head_dim": D, "ctx": T, "page_size": PS, "selected_pages_per_seq_head": int(ids.size),
                      "format_mix": w["mix"], "visible_pairs_per_q_head": pairs, "useful_flops_per_step": flops,
                      "selected_kv_bytes_per_step": kv_bytes,
                      "l2": f"L2 flushed before every timed step (a {2 * L2_BYTES >> 20} MB write): the selected KV "
                            f"({kv_bytes / 1e6:.0f} MB) and q ({q.numel() * 2 / 1e6:.0f} MB) fit in L2",
                      "timing": "eager launches, CUDA events around each timed step"},
           "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tf / peak, 4), "traffic": ncu_traffic("prefill", B, None)[0],
                        "traffic_note": ncu_traffic("prefill", B, None)[1], "kernel": "prefill_tc_kernel<16>",
                        "kernel_ms": round(kernel_ms, 4),
                        "note": f"peak = {peak_kind} dense bf16 cuBLAS burst; achieved = useful FLOPs (4 x head_dim "
                                "per visible (query, key) pair per q head) / the kernel's CUDA-event time"},
           "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 4),
                   "h2d_bytes_per_step": q_host.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2,
                   "api": "intent_attention.paged_prefill with pinned host q in, output out"},
           "gpu_launches": args.steps, "clocks": clocks.summary()}
    if not args.no_cpu_baseline:
        sec, rows = cpu_prefill(w, ids, fmt, qpos, args.cpu_budget)
        rec["cpu_baseline"] = {"value": round(flops / sec / 1e12, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
                               "sample": f"{rows} query rows of one unit through the numpy oracle, extrapolated"}
    print(json.dumps(rec), flush=True)


# --------------------------------------------------------------------------- #
#  KV append with quantise-on-write (iak_append_tokens) at the C2 shape
# --------------------------------------------------------------------------- #

APPEND_METRIC = "KV append: (sequence, kv-head) rows appended with their open page re-quantised, per s"


def append_page_bytes(fmt_code: int, PS: int, D: int) -> int:
    """Algorithmic bytes of one (unit, plane) append: new bf16 row in, the
    fp32 row into the stage, the staged page read back, the page's codes and
    scale written."""
    codes = {1: 2 * D, 2: D, 3: D}[fmt_code] * PS
    scales = 0 if fmt_code == 1 else 4
    return 2 * D + 4 * D + 4 * PS * D + codes + scales


def cpu_append(w, fmt_units, budget_s):
    """The oracle's page quantiser over sampled units (one page per plane per
    unit): seconds per full step."""
    import sys as _s
    _s.path.insert(0, ROOT)
    from oracle import quant as oq
    g = np.random.default_rng(5)
    PS, D = w["PS"], w["D"]
    names = {1: "FP16", 2: "FP8", 3: "INT8"}
    t0 = time.perf_counter()
    done = 0
    while done < len(fmt_units) and (time.perf_counter() - t0 < budget_s or done == 0):
        page = g.standard_normal((1, PS, D)).astype(np.float32)
        for _ in range(2):
            oq.quantize_pages(page, names[int(fmt_units[done])], w["scale_mode"])
        done += 1
    return (time.perf_counter() - t0) / done * len(fmt_units), done


def run_append(args):
    import torch
    from intent_attention import KVStage, PagePool, append_tokens
    from intent_attention.paged import make_tag_map
    w = workload("c2")
    if args.batch:
        w["B"] = args.batch
    B, Hkv, D, PS = w["B"], w["Hkv"], w["D"], w["PS"]
    units = B * Hkv
    rng = np.random.default_rng(w["seed"] + 5)
    mix = w["mix"]
    fmt_units = rng.choice([FMT_CODE[k] for k in mix], size=units, p=list(mix.values())).astype(np.uint8)
    if args.impl == "reference":
        vals, n = [], 0
        for i in range(args.warmup + args.steps):
            sec, n = cpu_append(w, fmt_units, args.cpu_budget / max(1, args.steps + args.warmup))
            if i >= args.warmup:
                vals.append(sec)
        v = units / statistics.median(vals)
        print(json.dumps({"impl": "reference", "metric": APPEND_METRIC, "value": round(v, 1), "unit": "rows/s",
                          "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": round(units / v * 1e3, 3), "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "fp32 -> fp16/fp8/int8 pages", "data": "synthetic",
                          "config": {"workload": "C2 decode-step KV append", "units": units},
                          "cpu_baseline": {"value": round(v, 1), "unit": "rows/s", "cores": 1, "kind": "port",
                                           "sample": f"{n} units per step through the oracle page quantiser"},
                          "e2e": {"value": round(v, 1), "unit": "rows/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    K = args.steps
    pages_per_unit = (40 + K) // PS + 1
    pool = PagePool.allocate(units * pages_per_unit, PS, D, sorted(mix), w["scale_mode"], device, zero=True)
    tags = torch.from_numpy(np.repeat(fmt_units, pages_per_unit)).to(device)
    bases = (torch.arange(units, dtype=torch.int32, device=device) * pages_per_unit).view(B, Hkv)
    stage = KVStage.allocate(units, pool)
    tag_map = make_tag_map({c: f for f, c in FMT_CODE.items() if f in mix})
    g = torch.Generator(device=device).manual_seed(w["seed"])
    k_rows = torch.randn((K, B, Hkv, 1, D), generator=g, device=device).to(torch.bfloat16)
    v_rows = torch.randn((K, B, Hkv, 1, D), generator=g, device=device).to(torch.bfloat16)
    # step i appends token 40 + i of every sequence: it lands mid-page, so
    # every step re-quantises a partly filled open page
    positions = [torch.full((B,), 40 + i, dtype=torch.int32, device=device) for i in range(K)]

    def step(i):
        append_tokens(pool, k_rows[i], v_rows[i], positions[i], tags, tag_map, stage, bases=bases)

    for i in range(K):
        step(i)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        t_probe = time.perf_counter()
        while len(clocks.rows) < 3 and time.perf_counter() - t_probe < 3.0:
            for i in range(K):
                step(i)
            torch.cuda.synchronize()
        for i in range(min(args.warmup, K)):
            step(i)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(K):
                step(i)
        graph.replay()
        torch.cuda.synchronize()
        ev0.record()
        graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    t_ms = ev0.elapsed_time(ev1) / K
    del graph
    # end to end: the new rows from pinned host memory each step
    k_host = k_rows[0].cpu().pin_memory()
    v_host = v_rows[0].cpu().pin_memory()
    k_dev, v_dev = torch.empty_like(k_rows[0]), torch.empty_like(v_rows[0])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(args.warmup):
        k_dev.copy_(k_host, non_blocking=True)
        v_dev.copy_(v_host, non_blocking=True)
        append_tokens(pool, k_dev, v_dev, positions[i % K], tags, tag_map, stage, bases=bases)
    torch.cuda.synchronize()
    e0.record()
    for i in range(K):
        k_dev.copy_(k_host, non_blocking=True)
        v_dev.copy_(v_host, non_blocking=True)
        append_tokens(pool, k_dev, v_dev, positions[i], tags, tag_map, stage, bases=bases)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K
    nbytes = 2 * sum(append_page_bytes(int(f), PS, D) for f in fmt_units)
    peak, peak_kind = measured_hbm_peak()
    gbs = nbytes / (t_ms * 1e-3) / 1e9
    rec = {"metric": APPEND_METRIC, "value": round(units / (t_ms * 1e-3), 1), "unit": "rows/s", "n_gpus": 1,
           "steps": K, "warmup": args.warmup, "ms_per_step": round(t_ms, 5), "us_per_step": round(t_ms * 1e3, 2),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16 rows -> fp16/fp8/int8 pages (fp32 stage)", "data": "synthetic (seeded N(0,1) rows)",
           "config": {"workload": "C2 decode-step KV append (iak_append_tokens)", "batch": B, "kv_heads": Hkv,
                      "head_dim": D, "page_size": PS, "rows_per_step": units, "format_mix": mix,
                      "scale_mode": w["scale_mode"],
                      "l2": "inputs smaller than L2 (the open pages of a decode step stay L2-resident)",
                      "timing": "one CUDA graph of all timed launches, replayed once after a warm-up replay"},
           "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 5), "traffic": None, "kernel": "append_kernel",
                        "kernel_us": round(t_ms * 1e3, 2),
                        "note": f"peak = {peak_kind} HBM copy bandwidth; {nbytes} algorithmic bytes per launch "
                                "(new rows, stage row write, staged page re-read, page codes + scales); one CTA "
                                "per (unit, plane): latency-bound at this size"},
           "e2e": {"value": round(units / (e2e_ms * 1e-3), 1), "unit": "rows/s", "ms_per_step": round(e2e_ms, 5),
                   "h2d_bytes_per_step": 2 * k_host.numel() * k_host.element_size(), "d2h_bytes_per_step": 0,
                   "api": "intent_attention.append_tokens with pinned host K/V rows in"},
           "gpu_launches": K, "clocks": clocks.summary()}
    if not args.no_cpu_baseline:
        sec, done = cpu_append(w, fmt_units, args.cpu_budget)
        rec["cpu_baseline"] = {"value": round(units / sec, 1), "unit": "rows/s", "cores": 1, "kind": "port",
                               "sample": f"{done} of {units} units through the oracle page quantiser, extrapolated"}
    print(json.dumps(rec), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5", "route", "append", "prefill"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--batch", type=int, default=0, help="override the workload's batch (profiling runs)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="c5 on one GPU: decode rank 0's share of the pages cut over this many GPUs (profiling runs)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="C5 on several GPUs: partial blocks over NVLink peer stores or one NCCL all-gather")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of a captured CUDA graph")
    ap.add_argument("--cpu-budget", type=float, default=12.0,
                    help="seconds of host work for the GPU arm's cpu_baseline sample")
    ap.add_argument("--ref-step-s", type=float, default=0.5,
                    help="--impl reference: at least this many seconds of host work per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c5-strong", action="store_true",
                    help="default workload: skip the sequence-sharded C5 measurement added to the line")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE is {world}: launch one process per GPU "
                         f"(python -m torch.distributed.run --nproc-per-node {args.gpus} ... bench.py --gpus "
                         f"{args.gpus}), or pass --gpus {world}")
    if args.warmup < 3:
        raise SystemExit(f"--warmup {args.warmup}: at least 3 untimed warm-up steps are required")
    if args.workload == "route":
        run_route(args)
    elif args.workload == "append":
        run_append(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "c4":
        run_gpu_mla(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()

"""Benchmark of the Needle 2 CUDA decode engine (one JSON line on rank 0).

Default workload -- BASELINE config 4, ragged continuous-batch decode, full model, per GPU:
256 concurrent sequence slots; prompts of uniform length in [32, 1024] with uniform random token
ids; each sequence generates a uniform number of greedy tokens in [16, 128], then retires and the
next queued sequence is admitted into its slot (seed 4 + rank).  Random-init N(0, 0.02) weights
quantised by the build's CQ quantiser (synthetic data; no checkpoint exists offline).

A *step* is one batched engine step: every busy slot consumes one token through all 27 layers
(a prompt token while it prefills, its last greedy token while it decodes), exactly the
reference's token-serial decoder step (packages/needle.js/src/model/runtime.ts:280-583).
The metric counts *generated* tokens per second -- greedy selections -- like the reference's
GenerationResult.tokensPerSecond (packages/needle.js/src/model/model.ts:142-151), so prefill work
is inside the time but not in the count.  Before timing, a ramp of untimed steps brings the slot
population to the steady-state mix of prefill and decode.

value: device-resident -- the queue of prompts sits in HBM before timing and the device scheduler
       runs the steps without host round trips; CUDA events on the engine stream, max over ranks.
e2e:   the same workload through the host C-ABI step call (needle_cuda_step): host scheduling,
       host item arrays copied in and selected ids / log-probabilities copied out every step.
Multi-GPU: independent sequences per GPU (data parallel, no collectives), weak scaling.

`--impl reference` times the CPU restatement of the reference backend (oracle/, all host cores)
on the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
import __graft_entry__  # noqa: E402  (registers the needle.js_b200/ package as needle_b200)

__graft_entry__.load()

# DRAM bytes (read + write) per timed launch of a kernel class in the benchmarked state, from the
# committed steady-state captures (ncu, one pass), with the sched_chunk they were taken at.  With
# prompt chunks an attention "launch" is the pair of launches of one layer (chunk append, attend).
STEADY_TRAFFIC = {
    "attention": {"bytes": 1054208 + 35696640, "sched_chunk": 8,
                  "source": "profiles/attention_exact_decode_step_steady_state.md"},
    "layer": {"bytes": 5684224, "sched_chunk": 8, "source": "profiles/layer_exact_decode_step_steady_state.md"},
}
SLOTS = 256
PROMPT = (32, 1024)
GEN = (16, 128)
SEED = 4


def workload(rank: int, n_seqs: int):
    from needle_b200 import synth
    plen = synth.integers(SEED + 1000 * rank, n_seqs, PROMPT[1] - PROMPT[0] + 1, stream=1) + PROMPT[0]
    gens = synth.integers(SEED + 1000 * rank, n_seqs, GEN[1] - GEN[0] + 1, stream=2) + GEN[0]
    ids = synth.integers(SEED + 1000 * rank, int(plen.sum()), 8192, stream=3).astype(np.int32)
    offs = np.concatenate([[0], np.cumsum(plen)])
    prompts = [ids[offs[i]:offs[i + 1]] for i in range(n_seqs)]
    return prompts, gens.astype(np.int32)


def sample_clocks(index: int):
    """Starts an nvidia-smi sampler of this GPU's clocks and throttle reasons."""
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    try:
        return subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None


def clocks_summary(proc):
    if proc is None:
        return None
    proc.terminate()
    try:
        out, _ = proc.communicate(timeout=5)
    except subprocess.TimeoutExpired:
        proc.kill()
        out, _ = proc.communicate()
    sm, mx, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in out.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            mx.append(float(f[2]))
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def load_peaks():
    """MEASURED_PEAKS.json (the pool's measured HBM copy bandwidth and bf16 GEMM rates), or None."""
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return None


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference(n_seqs: int = 0):
    """The oracle (C++ restatement of the reference CPU backend) on all host cores, one sequence of
    the workload per thread.  Throughput is the renewal-reward estimate
    threads * sum(generated) / sum(per-sequence compute seconds), free of load imbalance."""
    from oracle import needle_ref
    from needle_b200 import synth
    needle_ref.build()
    threads = cpu_threads()
    n = n_seqs or threads
    model = needle_ref.Model(synth.build_archive(0))
    prompts, gens = workload(0, n)
    t0 = time.perf_counter()
    _, processed, secs = model.decode_many(prompts, gens, threads, seconds=True)
    wall = time.perf_counter() - t0
    gen = int(gens.sum())
    value = threads * gen / float(secs.sum())
    return dict(value=value, processed_per_s=threads * processed / float(secs.sum()), threads=threads, seqs=n,
                seconds=wall, generated=gen, processed=processed)


def aggregate(local_stats, dist=None):
    """Whole-job totals over ranks: (max step-time ms, summed generated, summed processed,
    max e2e ms, summed e2e generated, summed launches).  `local_stats` is this rank's
    [ms, generated, processed, e2e_ms, e2e_generated, launches]; every rank takes the same
    collective (an all_gather over the process group) so ranks never wait on one another."""
    import torch
    stats = torch.tensor([float(v) for v in local_stats], dtype=torch.float64)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        gathered = [torch.zeros_like(stats) for _ in range(dist.get_world_size())]
        dist.all_gather(gathered, stats)
        allst = torch.stack(gathered)
    else:
        allst = stats[None]
    return (float(allst[:, 0].max()), float(allst[:, 1].sum()), float(allst[:, 2].sum()),
            float(allst[:, 3].max()), float(allst[:, 4].sum()), int(allst[:, 5].sum()))


# Binary64 operations the reference performs per unit (its own expressions, not this engine's):
# attention, per visible position, head element and query head: q * code * keyScale (2 multiplies)
# and the add of the score dot, weight * code * valueScale (2) and the add of the value mix -> 6;
# a 2-bit matvec byte (4 weights): 1 multiply + 3 multiply-adds + 1 add = 5 (4-bit: 3 per byte;
# 3-bit: 1 multiply-add per weight).
FP64_OPS_ATTENTION = 6
# FP64 lanes per SM per clock on B200 (spec: 37-40 TFLOP/s FP64 = 148 SMs x 64 FMA lanes x ~2 GHz);
# no FP64 peak is measured on this pool, so the spec-derived figure at the sampled clock is used.
FP64_LANES_PER_SM = 64
SMS = 148


def visible_positions(slots, prompts, chunk, items, steps, window=256):
    """(visible, distinct) KV positions per step over the next `steps` scheduled steps, from the
    slots' (sequence, position, busy): visible summed over the step's items, distinct counted once per
    slot (a chunk's items read one window).  One item per busy slot, or, with prompt chunks, up to
    `chunk` prompt positions of a prefilling slot (never its last, never past the window) while the
    step's `items` last, in slot order (admissions and retirements in between are ignored)."""
    pos = {k: p for k, (sid, p, busy) in enumerate(slots) if busy}
    plen = {k: len(prompts[slots[k][0]]) for k in pos}
    total = distinct = 0
    for _ in range(steps):
        budget = (items if chunk >= 2 else len(pos)) - len(pos)
        for k in sorted(pos):
            p = pos[k]
            n = 1
            if chunk >= 2 and p < plen[k] - 1:
                want = max(1, min(chunk, plen[k] - 1 - p, window - p))
                n = 1 + max(0, min(want - 1, budget))
                budget -= n - 1
            total += sum(min(q + 1, window) for q in range(p, p + n))
            distinct += min(p + n, window + n - 1)
            pos[k] = p + n
    return total / steps, distinct / steps


def roofline_for(prof, n_items, peaks, visible=None, sm_mhz=None, state_chunk=None, unique=None):
    """Roofline of the kernel class with the largest share of step time.  `n_items` is the items of
    one launch, `visible` the number of visible KV positions summed over them (from the slots'
    positions), else full 256-position windows are assumed; `unique` the distinct KV positions among
    them (the items of one chunk share their slot's window), else `visible`.  `state_chunk`: the
    sched_chunk of a config-4 run, whose committed steady-state DRAM capture then applies (None: no
    capture applies)."""
    cls, (ms, launches) = max(prof.items(), key=lambda kv: kv[1][0])
    per_launch_ms = ms / max(launches, 1)
    # algorithmic bytes per launch: the bytes the kernel must touch once per item (KV rows of the
    # visible positions, inputs and outputs) plus, for the GEMVs, every weight byte once
    kv_row = 64 + 64 + 4 + 4
    weights = {"gemv_qkvg": (512 + 256 + 256 + 512) * (128 + 8), "gemv_o": 512 * (192 + 8),
               "gemv_vocab": 8192 * (256 + 8)}
    positions = visible if visible is not None else n_items * 256
    distinct = unique if unique is not None else positions
    fp64_ops = None
    if cls == "layer":
        per_item = 2 * 2048 * 4 + 24 * (1024 + 32) + 5 * 2048 + 80 * 2
        bytes_ = n_items * per_item + 12 * 2048
    elif cls == "attention":
        bytes_ = 4 * distinct * kv_row + n_items * (1536 * 4 + 512 * 4)
        fp64_ops = FP64_OPS_ATTENTION * 8 * 64 * positions  # 8 query heads x 64 elements
    elif cls in weights:
        ins = {"gemv_qkvg": (512, 1536), "gemv_o": (512, 512), "gemv_vocab": (512, 8192)}[cls]
        bytes_ = weights[cls] + n_items * 4 * (ins[0] + ins[1])
    else:
        bytes_ = 0
    achieved = bytes_ / (per_launch_ms * 1e-3) / 1e9
    peak = peaks.get("hbm_gbs") if peaks else None
    src = "measured" if peak else "fallback"
    peak = peak or 6650.0
    # DRAM bytes (read + write) of one launch of the kernel in the benchmarked state (ncu, 1 pass,
    # bench.py --steps 20 --warmup 5 --no-cpu-baseline --e2e-steps 2 --no-fast: the first
    # 256-item launches after the ramp; profiles/attention_exact_decode_step_steady_state.md)
    t = STEADY_TRAFFIC.get(cls)
    if t is not None and (state_chunk is None or max(state_chunk, 1) != max(t["sched_chunk"], 1)):
        t = None
    line = {"kernel": cls, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_source": src,
            "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": t["bytes"] if t else None,
            "launch_ms": round(per_launch_ms, 5), "algorithmic_bytes_per_launch": int(bytes_)}
    if t:
        line["traffic_source"] = t["source"]
    if visible is not None:
        line["visible_positions_per_launch"] = int(visible)
        line["distinct_kv_positions_per_launch"] = int(distinct)
    if cls == "layer":
        # k_layer's bound is the dependent binary64 adds of its sequential sums (512 + 512 + 2048 +
        # 512 terms per item in the reference's order, about 11 cycles each, measured by phase
        # stamps); every item's CTA is resident at once at these counts, so one chain is the floor
        mhz = sm_mhz or 1965.0
        chain_adds, cycles_per_add = 512 + 512 + 2048 + 512, 11
        floor_ms = chain_adds * cycles_per_add / (mhz * 1e3)
        line["latency"] = {"bound": "dependent binary64 adds (sequential sums)", "chain_adds_per_item": chain_adds,
                           "cycles_per_add": cycles_per_add, "floor_ms": round(floor_ms, 5),
                           "frac": round(floor_ms / per_launch_ms, 4),
                           "note": "floor = one item's chain at the sampled clock; the rest is the FWHTs, phi "
                                   "dots and barriers around the chains and the CTAs' contention for the SMs"}
    if fp64_ops is not None:
        mhz = sm_mhz or 1965.0
        fpeak = SMS * FP64_LANES_PER_SM * mhz * 1e6
        line["fp64"] = {"bound": "fp64", "ops_per_launch": int(fp64_ops),
                        "achieved_gops": round(fp64_ops / (per_launch_ms * 1e-3) / 1e9, 1),
                        "peak_gops": round(fpeak / 1e9, 1), "frac": round(fp64_ops / (per_launch_ms * 1e-3) / fpeak, 4),
                        "peak_source": "spec lanes (148 SMs x 64 FP64 lanes) x sampled SM clock, not measured",
                        "ops": "the reference's binary64 multiplies and adds per visible position (6 per element "
                               "and query head)"}
    return line


QMATVEC_SHAPES = [  # (name, rows, inputs, record bits) -- every Needle 2 projection, the stress shape and
    # the four 2-bit projections of a layer stacked (one launch of the exact engine step)
    ("query/gate 512x512 CQ2", 512, 512, 2), ("key/value 256x512 CQ2", 256, 512, 2),
    ("output 512x512 CQ3", 512, 512, 3), ("phi_pre/post layer slice 4x2048 CQ4", 4, 2048, 4),
    ("phi_res layer slice 16x2048 CQ4", 16, 2048, 4), ("phi_pre/post 108x2048 CQ4", 108, 2048, 4),
    ("phi_res 432x2048 CQ4", 432, 2048, 4), ("engram key/value 512x512 ternary", 512, 512, 5),
    ("vocabulary 8192x512 CQ4", 8192, 512, 4), ("stress 8192x8192 CQ4", 8192, 8192, 4),
    ("query|key|value|gate stacked 1536x512 CQ2", 1536, 512, 2)]
ROTATE_BYTES = 256 << 20  # rotated operand sets exceed the 126 MB L2 twice over


def _peak(peaks):
    p = peaks.get("hbm_gbs") if peaks else None
    return (p, "measured") if p else (6650.0, "fallback")


def _time_calls(torch, stream, fn, n_sets, warmup, iters):
    """Device time per call: `iters` calls (rotating operand sets) captured once as a CUDA graph
    after `warmup` eager calls, then the graph replayed between CUDA events, so host call overhead
    stays out of the number.  fn(i, stream_handle) launches call i on the given stream."""
    for i in range(warmup):
        fn(i % n_sets, stream.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.graph(graph, stream=side):
        cap = torch.cuda.current_stream().cuda_stream
        for i in range(iters):
            fn(i % n_sets, cap)
    graph.replay()  # warm the graph
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    del graph
    return e0.elapsed_time(e1) / iters


def fast_matvec_kernels(rows: int, inputs: int, batch: int, sms: int = 148) -> int:
    """Kernel launches of one needle_cuda_cq_matvec_dev_fast call: table GEMV + row totals per 8
    items below 16 items (6 for matrices of 4M weights and more); above, the tensor-core GEMM:
    activation prepare + GEMM (+ split-K sum when the groups are split across CTAs) per 128 items."""
    if batch < 16 and not (batch >= 6 and rows * (-(-inputs // 128) * 128) >= 1 << 22):
        return 2 * -(-batch // 8)
    m_tiles, groups = -(-rows // 128), -(-inputs // 128)
    splits = max(1, min(groups, sms // m_tiles))
    per = -(-groups // splits)
    used = -(-groups // per)
    return (3 if used > 1 else 2) * -(-batch // 128)


def bench_qmatvec(args, peaks):
    """isolated quantised matvec, every projection shape + 8192x8192, batch
    1/8/32/128; indices uniform, fp16 norms |N(0,1)|*0.01, activations N(0,1) (seed 2: generator
    2000 + shape index per shape)."""
    import ctypes as C
    import torch
    from needle_b200 import native, synth
    native.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    cb = synth.lloyd_max_codebook()
    results, launches = [], 0
    batches = [int(b) for b in args.batches.split(",")] if args.batches else [1, 8, 32, 128]
    for si, (name, rows, inputs, bits) in enumerate(QMATVEC_SHAPES):
        if args.cases and args.cases not in name:
            continue
        gen = torch.Generator(device="cuda").manual_seed(2000 + si)  # seed 2, one stream per shape
        pad = -(-inputs // 128) * 128
        row_bytes = pad * (2 if bits == 5 else bits) // 8
        mbytes = rows * row_bytes + rows * (pad // 128) * 2
        n_sets = int(min(4096, max(4, -(-ROTATE_BYTES // mbytes))))
        packed = torch.randint(0, 256, (n_sets, rows * row_bytes + 64), dtype=torch.uint8, device="cuda", generator=gen)
        norms = (torch.randn((n_sets, rows * (pad // 128)), device="cuda", generator=gen).abs() * 0.01).half()
        descs = [native.CqMatrixDesc(packed[i].data_ptr(), norms[i].data_ptr(), rows, inputs, 128, bits)
                 for i in range(n_sets)]
        for batch in batches:
            x = torch.randn((batch, inputs), device="cuda", generator=gen)
            y = torch.empty((batch, rows), device="cuda")
            lib = native.lib()
            modes = []
            if args.numerics in ("both", "exact"):
                modes.append(("exact", lib.needle_cuda_cq_matvec_dev, 3 if (batch <= 8 and pad // 128 >= 16) else 2))
            if bits in (2, 4, 5) and args.numerics in ("both", "fast"):
                modes.append(("fast", lib.needle_cuda_cq_matvec_dev_fast, fast_matvec_kernels(rows, inputs, batch)))
            for mode, fn, kernels in modes:
                def call(i, strm, fn=fn):
                    native.check(fn(C.byref(descs[i]), native.ptr(cb), x.data_ptr(), batch, y.data_ptr(), strm))
                iters = max(20, min(args.steps, 200))
                ms = _time_calls(torch, stream, call, n_sets, max(3, args.warmup), iters)
                launches += kernels * iters
                alg = mbytes + batch * 4 * (inputs + rows)
                results.append({"shape": name, "batch": batch, "numerics": mode, "us": round(ms * 1e3, 3),
                                "gbs": round(alg / (ms * 1e-3) / 1e9, 1), "bytes": alg, "kernels_per_call": kernels})
        del packed, norms
        torch.cuda.empty_cache()
    head = next((r for r in results if r["shape"].startswith("stress") and r["batch"] == 1 and r["numerics"] == "fast"),
                results[0])
    peak, src = _peak(peaks)
    line = {"metric": "qmatvec HBM GB/s", "value": head["gbs"], "unit": "GB/s", "n_gpus": 1,
            "steps": max(20, min(args.steps, 200)), "warmup": max(3, args.warmup), "ms_per_step": head["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fast) / f64 (exact)",
            "data": "synthetic", "config": {"workload": "isolated quantised matvec (BASELINE config 2), headline 8192x8192 CQ4 batch 1, "
                                   "fast numerics; exact-numerics rows alongside",
                       "l2": f"operand sets rotated over > {ROTATE_BYTES >> 20} MB", "cases": results},
            "roofline": {"kernel": "k_cq_gemv_table (+ k_cq_fast_reduce)", "bound": "hbm",
                         "achieved": head["gbs"], "peak": peak, "peak_source": src, "unit": "GB/s",
                         "frac": round(head["gbs"] / peak, 4),
                         # DRAM read + write of one table-kernel launch of the headline case (ncu)
                         "traffic": 33613312 if head["shape"].startswith("stress") and head["batch"] == 1 else None,
                         "traffic_source": "profiles/qmatvec_table_8192x8192_cq4_batch1.md"},
            "gpu_launches": launches}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = {k: v for k, v in cpu_qmatvec().items() if k != "ms"}
    big = next((r for r in results if r["shape"].startswith("stress") and r["batch"] == 128 and r["numerics"] == "fast"),
               None)
    if big is not None:
        # the batched case runs on the tensor cores: algorithmic flops 2 * B * rows * in_pad against the
        # measured dense bf16 GEMM peak (fp16 runs at the same rate); the pipe executes three fp16 products
        # per weight x activation pair
        tflops = 2 * 128 * 8192 * 8192 / (big["us"] * 1e-6) / 1e12
        tpeak = float((peaks or {}).get("bf16_tflops") or 1590.0)
        line["roofline_batched"] = {"kernel": "k_cq_gemm_tc (+ k_cq_prep_f16, k_splitk_sum)", "bound": "tensor",
                                    "case": "stress 8192x8192 CQ4 batch 128", "achieved": round(tflops, 1),
                                    "executed": round(3 * tflops, 1), "peak": tpeak,
                                    "peak_source": "measured" if (peaks or {}).get("bf16_tflops") else "fallback",
                                    "unit": "TFLOP/s", "frac": round(tflops / tpeak, 4),
                                    "source": "profiles/qmatvec_gemm_tc_8192x8192_cq4.md"}
    print(json.dumps(line), flush=True)


def bench_attention(args, peaks):
    """isolated int8-KV decode attention, batch 64, 8 query / 4 KV heads x 64,
    visible counts uniform in [64, L] for L in {512, 2048, 8192}; codes uniform in [-127, 127],
    scales |N(0,1)|*0.02, q N(0,1) (seed 3: generator 3000 + L per length).  Exact and fast numerics."""
    import torch
    from needle_b200 import native
    native.lib()
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    lib = native.lib()
    results, launches = [], 0
    lengths = [int(v) for v in args.cases.split(",")] if args.cases else [512, 2048, 8192]
    for L in lengths:
        gen = torch.Generator(device="cuda").manual_seed(3000 + L)  # seed 3, one stream per L
        batch = 64
        counts = torch.randint(64, L + 1, (batch,), dtype=torch.int32, device="cuda", generator=gen)
        set_bytes = batch * 4 * L * (64 * 2 + 8)
        n_sets = int(max(2, -(-ROTATE_BYTES // set_bytes)))
        kc = torch.randint(-127, 128, (n_sets, batch, 4, L, 64), dtype=torch.int8, device="cuda", generator=gen)
        vc = torch.randint(-127, 128, (n_sets, batch, 4, L, 64), dtype=torch.int8, device="cuda", generator=gen)
        ks = torch.randn((n_sets, batch, 4, L), device="cuda", generator=gen).abs() * 0.02
        vs = torch.randn((n_sets, batch, 4, L), device="cuda", generator=gen).abs() * 0.02
        q = torch.randn((batch, 512), device="cuda", generator=gen)
        out = torch.empty((batch, 512), device="cuda")
        visible = int(counts.sum().item())
        alg = visible * 4 * (64 * 2 + 8) + 2 * batch * 512 * 4 + batch * 4
        modes = [m for m in (("exact", lib.needle_cuda_attention_dev, 1), ("fast", lib.needle_cuda_attention_dev_fast, 2))
                 if args.numerics in ("both", m[0])]
        for mode, fn, kernels in modes:
            def call(i, strm, fn=fn):
                native.check(fn(q.data_ptr(), kc[i].data_ptr(), ks[i].data_ptr(), vc[i].data_ptr(), vs[i].data_ptr(),
                                counts.data_ptr(), batch, L, out.data_ptr(), strm))
            iters = max(10, min(args.steps, 100))
            ms = _time_calls(torch, stream, call, n_sets, max(3, args.warmup), iters)
            launches += kernels * iters
            results.append({"L": L, "numerics": mode, "us": round(ms * 1e3, 2),
                            "gbs": round(alg / (ms * 1e-3) / 1e9, 1), "bytes": alg})
        del kc, vc, ks, vs
        torch.cuda.empty_cache()
    head = next((r for r in results if r["L"] == 8192 and r["numerics"] == "fast"), results[-1])
    peak, src = _peak(peaks)
    line = {"metric": "int8-KV decode attention HBM GB/s", "value": head["gbs"], "unit": "GB/s", "n_gpus": 1,
            "steps": max(10, min(args.steps, 100)), "warmup": max(3, args.warmup), "ms_per_step": head["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (fast) / f64 (exact)",
            "data": "synthetic",
            "config": {"workload": "isolated int8-KV decode attention (BASELINE config 3), headline L=8192 fast",
                       "l2": f"KV sets rotated over > {ROTATE_BYTES >> 20} MB", "cases": results},
            "roofline": {"kernel": "k_attention_fast_mma (+ k_attention_fast_combine)", "bound": "hbm", "achieved": head["gbs"],
                         "peak": peak, "peak_source": src, "unit": "GB/s", "frac": round(head["gbs"] / peak, 4),
                         # DRAM read + write of one k_attention_fast_mma launch at L = 8192 (ncu)
                         "traffic": 152468480 if head["L"] == 8192 and head["numerics"] == "fast" else None,
                         "traffic_source": "profiles/attention_fast_mma_L8192_batch64.md"},
            "gpu_launches": launches}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = {k: v for k, v in cpu_attention().items() if k != "ms"}
    print(json.dumps(line), flush=True)


TOOLCALL_PROMPT = 256
TOOLCALL_MAX_NEW = 256


REFERENCE_CPU_TOKENS_PER_S = 45.3  # pure-TS CPU backend, Apple M4: 13-token prompt, 32 greedy tokens


def bench_single(args):
    """BASELINE config 1 (PR1 ref): one sequence, a --prompt-len prompt of uniform random ids
    (seed 1; 128 by default) fed to prefill, then --new-tokens greedy steps (64; no EOS stop), int8
    KV, sink 0.  `value` is generated tokens over the whole time, prefill included, as
    GenerationResult.tokensPerSecond (model.ts:142-151).  With --prompt-len 13 --new-tokens 32
    (the reference's published setup) `vs_baseline` compares with its 45.3 tok/s on the CPU backend
    (Apple M4).  Every step is a host step through the C-ABI (the selected id stays on the device
    as the next step's pending token), so `e2e` is the same number."""
    import torch
    from needle_b200 import build as nbuild
    from needle_b200 import synth
    from needle_b200.backend import CudaEngine, StepRequest
    nbuild.build()
    torch.cuda.set_device(0)
    archive = synth.build_archive(0)
    P, G = args.prompt_len, args.new_tokens
    prompt = synth.integers(1, P, 8192, stream=0).astype(np.int32)
    eng = CudaEngine(archive, device=0, max_seqs=1, max_len=P + G + 8, max_sink=0)
    stream = torch.cuda.ExternalStream(eng.stream, device=0)

    def generate():
        eng.reset(0, P + G, 0)
        if P > 1:
            eng.prefill(0, prompt[:-1], want_logits=False)
        ids = []
        for k in range(G):
            sel, _ = eng.step([StepRequest(0, int(prompt[-1]) if k == 0 else -1, True)])
            ids.append(sel[0][0])
        return ids

    for _ in range(max(3, args.warmup)):
        generate()
    smi = sample_clocks(int(os.environ.get("CUDA_VISIBLE_DEVICES", "0").split(",")[0]))
    runs = max(1, min(args.steps, 10))
    l0 = eng.kernel_launches()
    times, prefill_ms = [], []
    for _ in range(runs):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        torch.cuda.synchronize()
        e0.record(stream)
        eng.reset(0, P + G, 0)
        if P > 1:
            eng.prefill(0, prompt[:-1], want_logits=False)
        e1.record(stream)
        for k in range(G):
            eng.step([StepRequest(0, int(prompt[-1]) if k == 0 else -1, True)])
        e2.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e2))
        prefill_ms.append(e0.elapsed_time(e1))
    clocks = clocks_summary(smi)
    launches = (eng.kernel_launches() - l0) // runs
    ms = float(np.median(times))
    # per-kernel-class times of 10 decode steps, events around every launch
    eng.reset(0, P + G, 0)
    if P > 1:
        eng.prefill(0, prompt[:-1], want_logits=False)
    eng.profile(True)
    for k in range(min(10, G)):
        eng.step([StepRequest(0, int(prompt[-1]) if k == 0 else -1, True)])
    prof = {k: v for k, v in eng.profile_read().items() if v[1] > 0}
    eng.profile(False)
    eng.close()
    value = G / (ms / 1e3)
    published = (P, G) == (13, 32)
    import ctypes
    from needle_b200 import native
    line = {"metric": "batch-1 greedy decode tokens/s (prefill included)", "value": round(value, 2),
            "unit": "tokens/s", "n_gpus": 1, "steps": runs, "warmup": max(3, args.warmup),
            "ms_per_step": round(ms / (P - 1 + G), 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(value / REFERENCE_CPU_TOKENS_PER_S, 2) if published else None,
            "dtype": "f64", "data": "synthetic",
            "config": {"workload": "single sequence greedy decode (BASELINE config 1)" +
                                   (", the reference's published setup" if published else ""),
                       "prompt_len": P, "new_tokens": G, "seed": 1, "kv_cache": "int8", "sink": 0,
                       "ms_per_generation": round(ms, 3), "prefill_ms": round(float(np.median(prefill_ms)), 3),
                       "decode_ms_per_token": round((ms - float(np.median(prefill_ms))) / G, 4),
                       "runs": runs, "statistic": "median over runs",
                       "numerics": "exact (tokens, logits and int8 KV as the CPU backend's)",
                       "vs_baseline_basis": "the reference's pure-TS CPU backend, 45.3 tok/s on an Apple M4 "
                                            "(13-token prompt, 32 greedy tokens, real weights)" if published else None,
                       "parallelism": "one sequence, one GPU"},
            "e2e": {"value": round(value, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": ctypes.sizeof(native.StepItem),
                    "d2h_bytes_per_step": ctypes.sizeof(native.Selected)},
            "gpu_launches": int(launches),
            "roofline": roofline_for(prof, 1, load_peaks()),
            "kernel_ms_per_step": {k: round(v[0] / min(10, G), 4) for k, v in prof.items()},
            "clocks": clocks}
    if not args.no_cpu_baseline:
        from oracle import needle_ref
        needle_ref.build()
        model = needle_ref.Model(archive)
        t0 = time.perf_counter()
        model.generate_greedy(prompt, G, 0, want_logits=False)
        secs = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(G / secs, 3), "unit": "tokens/s", "cores": 1, "kind": "port",
                                "sample": f"the whole workload ({P}-token prompt, {G} greedy tokens) on one core"}
    print(json.dumps(line), flush=True)


def reference_arm(args):
    """`--impl reference` for the workloads other than the default: the C++ restatement of the
    reference's CPU path (oracle/) on this host's cores, on the CUDA arm's workload, metric and unit,
    each a bounded sample.  One JSON line with "impl": "reference"."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import needle_ref
    from needle_b200 import synth
    needle_ref.build()
    threads = cpu_threads()

    def emit(metric, value, unit, config, sample, cores, ms_per_step):
        line = {"metric": metric, "value": round(value, 3), "unit": unit, "impl": "reference", "n_gpus": args.gpus,
                "steps": 1, "warmup": 0, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f64", "data": "synthetic", "config": config,
                "cpu_baseline": {"value": round(value, 3), "unit": unit, "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": round(value, 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)

    if args.workload == "single":
        P, G = args.prompt_len, args.new_tokens
        model = needle_ref.Model(synth.build_archive(0))
        prompt = synth.integers(1, P, 8192, stream=0).astype(np.int32)
        t0 = time.perf_counter()
        model.generate_greedy(prompt, G, 0, want_logits=False)
        secs = time.perf_counter() - t0
        emit("batch-1 greedy decode tokens/s (prefill included)", G / secs, "tokens/s",
             {"workload": "single sequence greedy decode (BASELINE config 1)", "prompt_len": P, "new_tokens": G},
             f"the whole workload ({P}-token prompt, {G} greedy tokens) on one core", 1, 1e3 * secs / (P - 1 + G))
    elif args.workload == "toolcall":
        from needle_b200 import grammar, toolcall
        pieces, types, _ = synth.tokenizer_pieces(8192, 0)
        vocab = grammar.Vocabulary(pieces, types)
        tools = toolcall.synthetic_tools(5)
        ids = synth.integers(5, threads * TOOLCALL_PROMPT + 1, 8192, stream=7).astype(np.int32)
        prompts = [ids[k * TOOLCALL_PROMPT:(k + 1) * TOOLCALL_PROMPT] for k in range(threads)]
        r = cpu_toolcall(vocab, tools, prompts)
        emit("constrained tool-call tokens/s", r["value"], "tokens/s",
             {"workload": "constrained tool-call decode (BASELINE config 5)", "prompt_len": TOOLCALL_PROMPT,
              "max_new_tokens": TOOLCALL_MAX_NEW}, r["sample"], r["cores"], 1e3 / r["value"] * r["cores"])
    elif args.workload == "qmatvec":
        r = cpu_qmatvec()
        emit("qmatvec HBM GB/s", r["value"], "GB/s", {"workload": "isolated quantised matvec (BASELINE config 2), "
                                                                  "headline 8192x8192 CQ4 batch 1", "numerics": "exact (f64)"},
             r["sample"], r["cores"], r["ms"])
    elif args.workload == "attention":
        r = cpu_attention()
        emit("int8-KV decode attention HBM GB/s", r["value"], "GB/s",
             {"workload": "isolated int8-KV decode attention (BASELINE config 3), headline L=8192", "numerics": "exact (f64)"},
             r["sample"], r["cores"], r["ms"])
    else:
        print(json.dumps({"impl": "reference", "unavailable": f"no reference arm for workload {args.workload}"}))


def cpu_qmatvec():
    """BASELINE config 2's headline case (8192 x 8192 CQ4, batch 1; indices uniform, fp16 norms
    |N(0,1)| * 0.01, x N(0,1), seed 2: generator 2000 + shape index) through the C++ restatement of
    the reference's f64 cqMatvecPrepared, one matvec per host thread at once; GB/s of the same
    algorithmic bytes as the CUDA line."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import needle_ref
    from needle_b200 import synth
    needle_ref.build()
    threads = cpu_threads()
    si = next(i for i, sh in enumerate(QMATVEC_SHAPES) if sh[0].startswith("stress"))
    _, rows, inputs, bits = QMATVEC_SHAPES[si]
    rng = np.random.default_rng(2000 + si)
    pad = -(-inputs // 128) * 128
    row_bytes = pad * bits // 8
    packed = rng.integers(0, 256, rows * row_bytes + 64, dtype=np.uint8)
    norms = (np.abs(rng.standard_normal(rows * (pad // 128))) * 0.01).astype(np.float16)
    cb = synth.lloyd_max_codebook()
    M = needle_ref.CqMatrix(rows, inputs, 128, bits, packed, norms, cb[:4], cb[4:12], cb[12:28])
    xs = [rng.standard_normal(inputs).astype(np.float32) for _ in range(threads)]
    alg = rows * row_bytes + rows * (pad // 128) * 2 + 4 * (inputs + rows)

    def one(x):
        t0 = time.perf_counter()
        M.matvec(x)
        return time.perf_counter() - t0

    with ThreadPoolExecutor(threads) as pool:
        secs = list(pool.map(one, xs))
    mean = float(np.mean(secs))
    return {"value": round(threads * alg / mean / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{threads} concurrent 8192x8192 CQ4 batch-1 matvecs, one per host thread (the reference's "
                      "f64 cqMatvecPrepared)", "ms": 1e3 * mean}


def cpu_attention():
    """BASELINE config 3's headline case (batch 64, visible counts uniform in [64, 8192], codes uniform
    in [-127, 127], scales |N(0,1)| * 0.02, q N(0,1), seed 3: generator 3000 + L) through the C++
    restatement of the reference's attention, one sequence per host thread; GB/s of the same
    algorithmic bytes as the CUDA line."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import needle_ref
    needle_ref.build()
    threads = cpu_threads()
    L, batch = 8192, 64
    rng = np.random.default_rng(3000 + L)
    counts = rng.integers(64, L + 1, batch)
    n = min(batch, max(threads, 8))
    inputs = []
    for k in range(n):
        c = int(counts[k])
        inputs.append((rng.standard_normal(512).astype(np.float32), rng.integers(-127, 128, (4, c, 64), dtype=np.int8),
                       (np.abs(rng.standard_normal((4, c))) * 0.02).astype(np.float32),
                       rng.integers(-127, 128, (4, c, 64), dtype=np.int8),
                       (np.abs(rng.standard_normal((4, c))) * 0.02).astype(np.float32)))

    def one(args_):
        q, kc, ks, vc, vs = args_
        t0 = time.perf_counter()
        needle_ref.attention_int8(q, kc, ks, vc, vs)
        return time.perf_counter() - t0, kc.shape[1] * 4 * (64 * 2 + 8) + 2 * 512 * 4 + 4

    with ThreadPoolExecutor(threads) as pool:
        runs = list(pool.map(one, inputs))
    secs = sum(r[0] for r in runs)
    return {"value": round(threads * sum(r[1] for r in runs) / secs / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port", "sample": f"{n} of the 64 sequences (visible counts uniform in [64, 8192]), one per host "
                                      "thread (the reference's attention over int8 KV)", "ms": 1e3 * secs / n}


def cpu_toolcall(vocab, tools, prompts):
    """BASELINE config 5 on the host cores: the oracle runtime (the C++ restatement of the CPU
    backend) drives the constrained loop of agent.ts:157-210 for one workload sequence per thread
    (its calls release the GIL), selecting like selectToken over the allowed ids.  The allowed ids
    come from this repository's trie scan, which is faster than the reference's clone-and-feed scan,
    so the figure favours the CPU.  Throughput is the renewal-reward estimate
    threads * constrained tokens / per-sequence seconds."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import needle_ref
    from needle_b200 import grammar, synth
    needle_ref.build()
    model = needle_ref.Model(synth.build_archive(0))
    threads = cpu_threads()

    def one(prompt):
        t0 = time.perf_counter()
        rt = needle_ref.Runtime(model)
        rt.reset(prompt.size + TOOLCALL_MAX_NEW + 1, 0)
        logits = None
        for i, t in enumerate(prompt):
            logits = rt.step(int(t), want_logits=(i == prompt.size - 1))
        g = grammar.ToolCallGrammar(tools, 4)
        out = made = 0
        for _ in range(TOOLCALL_MAX_NEW):
            ids = grammar.allowed(g, vocab, out)
            if ids.size == 0:
                break
            tok = int(ids[int(np.argmax(logits[ids]))])
            g.feed(vocab.piece[tok])
            out += len(vocab.piece[tok])
            made += 1
            if g.complete:
                rt.step(tok, want_logits=False)
                break
            logits = rt.step(tok, want_logits=True)
        return made, time.perf_counter() - t0

    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as pool:
        runs = list(pool.map(one, prompts[:threads]))
    wall = time.perf_counter() - t0
    made = sum(r[0] for r in runs)
    secs = sum(r[1] for r in runs)
    return {"value": round(threads * made / secs, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{len(runs)} workload sequences, one per thread ({made} constrained tokens after "
                      f"{len(runs)} x {TOOLCALL_PROMPT} prompt tokens, {wall:.1f} s wall); allowed ids from "
                      "this repository's trie scan (faster than the reference's clone-and-feed scan)"}


# Indices of the per-rank config-5 totals that combine by maximum over ranks (times, steps); the
# rest are summed (tokens, calls, launches, bytes).
TOOLCALL_MAX_FIELDS = (0, 5, 6, 11, 12)


def aggregate_toolcall(local, dist=None):
    """Whole-job config-5 totals from this rank's [ms, constrained, prompt, completed, dead ends,
    steps, grammar s, launches, sequences, h2d, d2h, engine s, wall s, masks put, masked selections,
    allowed ids sent]: every rank takes the same two all-reduces (sum and max over the process
    group)."""
    import torch
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return [float(v) for v in local]
    t = torch.tensor([float(v) for v in local], dtype=torch.float64)
    mx = t.clone()
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    tot = t.tolist()
    for k in TOOLCALL_MAX_FIELDS:
        tot[k] = mx[k].item()
    return tot


def bench_toolcall(args, rank, world, local_rank):
    """constrained tool-call decode, data-parallel.  --sequences sequences (4096)
    split evenly over the GPUs; each a 256-token prompt of random ids (seed 5 + rank), then the
    constrained phase directly after the prompt (random weights never emit <tool_call>), greedy until
    the grammar completes or 256 constrained tokens, over the synthetic schema (3 tools x 2-5
    parameters of string / integer / boolean / enum, seed 5).  --slots engine slots per GPU (512)
    with continuous admission; the allowed ids come from the C++ grammar's byte-trie scan on up to
    16 host threads per GPU."""
    import torch
    from needle_b200 import build as nbuild
    from needle_b200 import grammar, synth, toolcall
    from needle_b200.backend import CudaEngine

    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=900))
    torch.cuda.set_device(local_rank)
    if rank == 0:
        nbuild.build()
    if dist:
        dist.barrier()
    archive = synth.build_archive(0)
    pieces, types, _ = synth.tokenizer_pieces(8192, 0)
    vocab = grammar.Vocabulary(pieces, types)
    tools = toolcall.synthetic_tools(5)
    n_local = args.sequences // world + (1 if rank < args.sequences % world else 0)
    ids = synth.integers(5 + 1000 * rank, n_local * TOOLCALL_PROMPT + 1, 8192, stream=7).astype(np.int32)
    prompts = [ids[k * TOOLCALL_PROMPT:(k + 1) * TOOLCALL_PROMPT] for k in range(n_local)]
    chunk = args.toolcall_chunk
    step_items = args.slots * 3 // 2 if chunk >= 2 else args.slots
    eng = CudaEngine(archive, device=local_rank, max_seqs=args.slots, max_len=TOOLCALL_PROMPT + TOOLCALL_MAX_NEW + 8,
                     max_sink=16, sched_chunk=chunk, sched_items=step_items if chunk >= 2 else 0)
    threads = max(1, min(16, cpu_threads() // max(1, world)))
    dec = toolcall.ConstrainedDecoder(eng, vocab, tools, maximum_new_tokens=TOOLCALL_MAX_NEW, threads=threads,
                                      mask_cache=args.mask_cache, prompt_chunk=chunk, step_items=step_items)
    dec.run(prompts[:min(8, n_local)], max_steps=max(3, args.warmup))  # warm-up steps (untimed)
    stream = torch.cuda.ExternalStream(eng.stream, device=local_rank)
    l0 = eng.kernel_launches()
    smi = sample_clocks(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[0])
                        if "CUDA_VISIBLE_DEVICES" in os.environ and world == 1 else local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    results, st = dec.run(prompts)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    clocks = clocks_summary(smi)
    launches = eng.kernel_launches() - l0

    # per-kernel-class timing for the roofline, after the timed run: 10 steps of the constrained
    # phase (every slot past its prompt), events around every launch
    prof_steps = 10

    def profile_hook(step):
        if step == TOOLCALL_PROMPT + 4:
            eng.profile(True)

    dec.run(prompts[:args.slots], max_steps=TOOLCALL_PROMPT + 4 + prof_steps, hook=profile_hook)
    prof = {k: v for k, v in eng.profile_read().items() if v[1] > 0}
    eng.profile(False)
    import ctypes
    from needle_b200 import native
    mask_bytes = 4 * (vocab.size + 31) // 32 + 4  # one mask and its slot number
    h2d = st.items * ctypes.sizeof(native.StepItem) + 4 * st.allowed_ids + st.masks_put * mask_bytes
    d2h = st.items * ctypes.sizeof(native.Selected)
    local = [ms, st.constrained_tokens, st.prompt_tokens, sum(r.complete for r in results),
             sum(r.dead_end for r in results), st.steps, st.grammar_seconds, launches, len(results), h2d, d2h,
             st.engine_seconds, st.seconds, st.masks_put, st.masked_items, st.allowed_ids]
    tot = aggregate_toolcall(local, dist)
    if rank == 0:
        (ms_max, cons, prompt_toks, done, dead, steps, gsec, launch_all, seqs, h2d_all, d2h_all, esec, wall,
         masks_put, masked_items, allowed_ids) = tot
        secs = ms_max / 1e3
        line = {"metric": "constrained tool-call tokens/s", "value": round(cons / secs, 1), "unit": "tokens/s",
                "n_gpus": world, "steps": int(steps), "warmup": max(3, args.warmup),
                "ms_per_step": round(ms_max / max(steps, 1), 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "config": {"workload": "constrained tool-call decode (BASELINE config 5)", "sequences": int(seqs),
                           "prompt_len": TOOLCALL_PROMPT, "max_new_tokens": TOOLCALL_MAX_NEW, "slots_per_gpu": args.slots,
                           "tools": [{"name": t["name"], "parameters": list(t["parameters"]["properties"])}
                                     for t in tools],
                           "completed_calls": int(done), "dead_ends": int(dead),
                           "processed_tokens_per_s": round((cons + prompt_toks) / secs, 1),
                           "sequences_per_s": round(seqs / secs, 2),
                           "host_grammar_seconds_max_rank": round(gsec, 3), "host_grammar_threads": threads,
                           "engine_call_seconds_max_rank": round(esec, 3),
                           "host_loop_seconds_max_rank": round(max(wall - gsec - esec, 0.0), 3),
                           "allowed": (f"device mask pool, masks cached per grammar state ({args.mask_cache} slots "
                                       f"per GPU)" if args.mask_cache else "id lists per step"),
                           "prompt_chunks": ({"chunk": chunk, "items_per_step": step_items}
                                             if chunk >= 2 else "one position per slot and step"),
                           "masks_put": int(masks_put), "masked_selections": int(masked_items),
                           "allowed_ids_sent": int(allowed_ids),
                           "numerics": "exact (tokens bit-identical to the CPU backend with the same masks)",
                           "parallelism": f"dp{world} (independent sequences per GPU, no collectives)"},
                # the whole run goes through needle_cuda_step with host buffers (items, allowed masks or
                # ids in; selections out), so the measured value is end to end
                "e2e": {"value": round(cons / secs, 1), "unit": "tokens/s",
                        "h2d_bytes_per_step": int(h2d_all / max(steps * world, 1)),
                        "d2h_bytes_per_step": int(d2h_all / max(steps * world, 1))},
                "gpu_launches": int(launch_all),
                "roofline": roofline_for(prof, args.slots, load_peaks()),
                "kernel_ms_per_step": {k: round(v[0] / prof_steps, 4) for k, v in prof.items()},
                "clocks": clocks}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_toolcall(vocab, tools, prompts)
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=["decode", "qmatvec", "attention", "toolcall", "single"], default="decode",
                    help="decode: BASELINE config 4 (default); qmatvec / attention: configs 2 / 3 (1 GPU); "
                         "toolcall: config 5 (constrained tool-call decode, data-parallel); "
                         "single: config 1 (one sequence, batch-1 latency)")
    ap.add_argument("--prompt-len", type=int, default=128, help="single: prompt tokens")
    ap.add_argument("--new-tokens", type=int, default=64, help="single: greedy tokens")
    ap.add_argument("--sequences", type=int, default=4096, help="toolcall: sequences over all GPUs")
    ap.add_argument("--slots", type=int, default=512, help="toolcall: engine slots per GPU")
    ap.add_argument("--sched-chunk", type=int, default=8,
                    help="decode: prompt positions a prefilling slot may take per scheduled step (0: one)")
    ap.add_argument("--sched-items", type=int, default=384, help="decode: items per scheduled step with chunks")
    ap.add_argument("--micro-batches", type=int, default=4,
                    help="decode: micro-batches per step (engine option; 8 measured 1.5 %% more processed tokens in "
                         "the scheduled run but less through host steps and in fast numerics)")
    ap.add_argument("--toolcall-chunk", type=int, default=0,
                    help="toolcall: prompt positions per slot and step (0: one; 512 slots already fill the GPU, "
                         "so chunks of 8 at 768 items per step measured 6 %% slower)")
    ap.add_argument("--mask-cache", type=int, default=4096,
                    help="toolcall: allowed masks cached per grammar state in a device pool of this many "
                         "slots (0: id lists per step)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--ramp", type=int, default=1600, help="untimed steps to reach the steady-state mix")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fast", action="store_true", help="decode: skip the fast-numerics measurement")
    ap.add_argument("--cases", default="", help="qmatvec: shape-name substring; attention: comma list of L")
    ap.add_argument("--batches", default="", help="qmatvec: comma list of batch sizes (default 1,8,32,128)")
    ap.add_argument("--numerics", choices=["both", "exact", "fast"], default="both",
                    help="qmatvec / attention: which numerics to time")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    config = {"workload": "ragged continuous-batch decode, full Needle 2 model (BASELINE config 4)",
              "slots_per_gpu": SLOTS, "prompt_len": list(PROMPT), "gen_tokens": list(GEN), "seed": SEED,
              "numerics": "exact (binary64 in reference order; tokens and int8 KV bit-identical to the CPU backend)",
              "kv_cache": "int8", "l2": "inputs larger than L2: the per-step KV working set is ~1 GB; the 13.7 MB "
                                        "of CQ weights stay L2-resident as in deployment",
              "parallelism": f"dp{args.gpus} (independent sequences per GPU, no collectives)",
              "micro_batches": args.micro_batches,
              "prompt_chunks": ({"sched_chunk": args.sched_chunk, "sched_items": args.sched_items,
                                 "note": "a slot still reading its prompt takes up to sched_chunk positions per "
                                         "step (until its KV window would wrap) beside the other slots' single "
                                         "items, at most sched_items items per step; the same ids and KV"}
                                if args.sched_chunk >= 2 else "one position per slot and step")}
    metric, unit = "decode tokens/s", "tokens/s"

    if args.workload == "single" and args.impl == "cuda":
        if rank == 0:
            bench_single(args)
        return
    if args.workload == "toolcall" and args.impl == "cuda":
        bench_toolcall(args, rank, world, local_rank)
        return

    if args.workload in ("qmatvec", "attention") and args.impl == "cuda":
        if rank != 0:
            return
        peaks = load_peaks()
        from needle_b200 import build as nbuild
        nbuild.build()
        (bench_qmatvec if args.workload == "qmatvec" else bench_attention)(args, peaks)
        return

    if args.impl == "reference" and args.workload != "decode":
        if rank == 0:
            reference_arm(args)
        return
    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_reference()
        sample = (f"{r['seqs']} sequences of the ragged workload (prompt {PROMPT}, gen {GEN}, seed {SEED}), one per "
                  f"host thread, {r['processed']} tokens through the C++ restatement of the reference CPU backend")
        line = {"metric": metric, "value": round(r["value"], 3), "unit": unit, "impl": "reference", "n_gpus": args.gpus,
                "steps": r["processed"], "warmup": 0, "ms_per_step": round(1000 * r["seconds"] / max(r["processed"], 1), 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic", "config": dict(config, slots_per_gpu=r["threads"]),
                "cpu_baseline": {"value": round(r["value"], 3), "unit": unit, "cores": r["threads"], "kind": "port",
                                 "sample": sample},
                "e2e": {"value": round(r["value"], 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    from needle_b200 import build as nbuild
    from needle_b200 import synth
    from needle_b200.backend import CudaEngine, StepRequest

    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=600))
    device = local_rank
    torch.cuda.set_device(device)
    if rank == 0:
        nbuild.build()
    if dist:
        dist.barrier()
    archive = synth.build_archive(0)
    peaks = load_peaks()

    n_seqs = SLOTS * 12
    prompts, gens = workload(rank, n_seqs)
    chunking = dict(sched_chunk=args.sched_chunk, sched_items=args.sched_items if args.sched_chunk >= 2 else 0,
                    micro_batches=args.micro_batches)
    eng = CudaEngine(archive, device=device, max_seqs=SLOTS, max_len=PROMPT[1] + GEN[1], max_sink=0, **chunking)
    stream = torch.cuda.ExternalStream(eng.stream, device=device)

    # ---------------- device-resident run
    eng.sched_load(SLOTS, prompts, gens)
    eng.sched_step(args.ramp + args.warmup)
    p0, g0, _, _ = eng.sched_status()
    l0 = eng.kernel_launches()
    smi = sample_clocks(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(device)).split(",")[0])
                        if "CUDA_VISIBLE_DEVICES" in os.environ and world == 1 else device)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    eng.sched_step(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    clocks = clocks_summary(smi)
    p1, g1, fin, _ = eng.sched_status()
    launches = eng.kernel_launches() - l0
    gen_tokens = g1 - g0
    processed = p1 - p0

    # per-kernel-class timing (events around every launch) for the roofline, after the timed run;
    # the visible KV positions of the profiled steps from the slots' positions (window 256, sink 0)
    slots = [eng.sched_slot(k) for k in range(SLOTS)]
    visible, unique = visible_positions(slots, prompts, args.sched_chunk, args.sched_items, 10)
    pp0 = eng.sched_status()[0]
    eng.profile(True)
    eng.sched_step(10)
    prof = {k: v for k, v in eng.profile_read().items() if v[1] > 0}
    eng.profile(False)
    items_per_launch = (eng.sched_status()[0] - pp0) / 10.0  # profiling runs one micro-batch per step

    # ---------------- end-to-end through the host C-ABI step
    e2e_steps = args.e2e_steps or max(20, min(args.steps, 100))
    e2e = host_driven(eng, stream, prompts, gens, args.ramp, args.warmup, e2e_steps, args.sched_chunk,
                      args.sched_items)

    if world > 1:  # this rank's own figures (stderr: stdout carries rank 0's one line)
        print(json.dumps({"rank": rank, "device": device, "ms": round(ms, 3), "generated": int(gen_tokens),
                          "processed": int(processed), "e2e_ms": round(e2e["ms"], 3)}), file=sys.stderr, flush=True)
    ms_max, gen_all, proc_all, e2e_ms, e2e_gen, launches_all = aggregate(
        [ms, gen_tokens, processed, e2e["ms"], e2e["generated"], launches], dist)
    eng.close()

    # ---------------- the same workload in fast numerics: every projection a tcgen05 GEMM over the
    # step's items (fp16 head/tail operands, fp32 accumulation); device-resident like `value`
    fast = None
    if not args.no_fast:
        feng = CudaEngine(archive, device=device, max_seqs=SLOTS, max_len=PROMPT[1] + GEN[1], max_sink=0,
                          numerics="fast", **chunking)
        fstream = torch.cuda.ExternalStream(feng.stream, device=device)
        feng.sched_load(SLOTS, prompts, gens)
        feng.sched_step(args.ramp + args.warmup)
        fp0, fg0, _, _ = feng.sched_status()
        fl0 = feng.kernel_launches()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(fstream)
        feng.sched_step(args.steps)
        f1.record(fstream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        fms = f0.elapsed_time(f1)
        fp1, fg1, _, _ = feng.sched_status()
        flaunch = feng.kernel_launches() - fl0
        feng.profile(True)
        feng.sched_step(10)
        fprof = {k: v for k, v in feng.profile_read().items() if v[1] > 0}
        feng.profile(False)
        feng.close()
        fms_max, fgen_all, fproc_all, _, _, flaunch_all = aggregate([fms, fg1 - fg0, fp1 - fp0, 0.0, 0, flaunch], dist)
        fast = {"value": round(fgen_all / (fms_max / 1e3), 1), "unit": unit, "ms_per_step": round(fms_max / args.steps, 4),
                "processed_tokens_per_s": round(fproc_all / (fms_max / 1e3), 1), "generated_tokens": int(fgen_all),
                "gpu_launches": flaunch_all,
                "numerics": "fast: projections (Q|K|V|gate, output, engram K|V, vocabulary) as tcgen05 GEMMs with "
                            "fp16 head/tail operands and fp32 accumulation; attention in binary32 over the int8 "
                            "cache; norm sums as block reductions; K/V append, routing and selection binary64 as in "
                            "exact; greedy ids equal to the CPU reference, logits within 1e-3 "
                            "(tests/test_gpu_fast_engine.py)",
                "dtype": "fp16x2 (head/tail) -> fp32 GEMMs; f32 attention; f64 elsewhere",
                "kernel_ms_per_step": {k: round(v[0] / 10, 4) for k, v in fprof.items()},
                "roofline_gemm": gemm_roofline(fprof, SLOTS, peaks)}
    if rank == 0:
        value = gen_all / (ms_max / 1e3)
        line = {"metric": metric, "value": round(value, 1), "unit": unit, "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
                "config": dict(config, ramp_steps=args.ramp, processed_tokens_per_s=round(proc_all / (ms_max / 1e3), 1),
                               generated_tokens=int(gen_all)),
                "e2e": {"value": round(e2e_gen / (e2e_ms / 1e3), 1), "unit": unit,
                        "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"], "steps": e2e_steps},
                "gpu_launches": launches_all,
                "roofline": roofline_for(prof, items_per_launch, peaks, visible=visible,
                                         sm_mhz=(clocks or {}).get("sm_mhz"),
                                         state_chunk=args.sched_chunk, unique=unique),
                "kernel_ms_per_step": {k: round(v[0] / 10, 4) for k, v in prof.items()},
                "kernel_ms_per_step_note": "event-timed per launch with the micro-batches run one after another "
                                           "(their sum exceeds ms_per_step, where they overlap)",
                "clocks": clocks}
        if fast is not None:
            line["fast"] = fast
        if world == 1 and not args.no_cpu_baseline:
            r = cpu_reference()
            line["cpu_baseline"] = {"value": round(r["value"], 3), "unit": unit, "cores": r["threads"], "kind": "port",
                                    "sample": f"{r['seqs']} sequences of the same workload, one per host thread "
                                              f"({r['processed']} tokens, {r['seconds']:.1f} s wall), C++ restatement "
                                              f"of the reference CPU backend"}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def gemm_roofline(prof, n_items, peaks):
    """Tensor roofline of the fast step's GEMMs: algorithmic flops per step (2 x rows x 512 inputs x
    items for Q|K|V|gate and the output projection of every layer, the engram K|V and the vocabulary)
    over their event-timed time per step, against the measured dense bf16 GEMM peak (fp16 runs at the
    same rate; the pipe executes four fp16 products per weight x activation pair)."""
    layers, sites = 27, 2
    flops = 2 * n_items * 512 * (layers * (1536 + 512) + sites * 1024 + 8192)
    ms = sum(prof.get(k, (0.0, 0))[0] for k in ("gemv_qkvg", "gemv_o", "gemv_engram", "gemv_vocab")) / 10
    if ms <= 0:
        return None
    tflops = flops / (ms * 1e-3) / 1e12
    peak = float((peaks or {}).get("bf16_tflops") or 1590.0)
    return {"kernel": "k_cq_gemm_tc (+ k_cq_prep_f16, k_splitk_sum)", "bound": "tensor", "achieved": round(tflops, 2),
            "executed": round(4 * tflops, 2), "peak": peak,
            "peak_source": "measured" if (peaks or {}).get("bf16_tflops") else "fallback", "unit": "TFLOP/s",
            "frac": round(tflops / peak, 5), "gemm_ms_per_step": round(ms, 4), "flops_per_step": flops}


def host_driven(eng, stream, prompts, gens, ramp, warmup, steps, chunk=0, items=0):
    """Continuous batching driven from the host through the C-ABI with host buffers
    (needle_cuda_step_begin / _end: the layers of step t run while the host plans step t + 1, which
    needs no result of step t -- a decode item takes its slot's pending token on the device, and
    the host knows how many tokens each sequence generates).  With `chunk` >= 2 a slot still reading
    its prompt sends up to `chunk` prompt positions as consecutive items (a prompt chunk: never its
    last position, never past the 256-position window), at most `items` items per step, in slot
    order, as the device scheduler does."""
    import torch
    from needle_b200.backend import StepRequest
    n_slots = eng.max_seqs
    queue = 0
    state = [None] * n_slots  # [seq index, position, generated] after every planned step

    def plan():
        """The next step from the planned state: (slot resets to make first, requests, generated)."""
        nonlocal queue
        resets = []
        for s in range(n_slots):
            if state[s] is None and queue < len(prompts):
                resets.append((s, len(prompts[queue]) + int(gens[queue])))
                state[s] = [queue, 0, 0]
                queue += 1
        reqs = []
        budget = items - sum(1 for st in state if st is not None) if chunk >= 2 else 0
        gen = 0
        for s in range(n_slots):
            st = state[s]
            if st is None:
                continue
            q, pos, done = st
            p = prompts[q]
            sel = pos >= len(p) - 1
            n = 1
            if chunk >= 2 and not sel:
                want = max(1, min(chunk, len(p) - 1 - pos, 256 - pos))
                n = 1 + max(0, min(want - 1, budget))
                budget -= n - 1
            if n > 1:
                reqs.extend(StepRequest(s, int(p[pos + j]), False) for j in range(n))
            else:
                reqs.append(StepRequest(s, int(p[pos]) if pos < len(p) else -1, sel))
            st[1] += n
            if sel:
                gen += 1
                st[2] += 1
                if st[2] >= gens[q]:
                    state[s] = None
        return resets, reqs, gen

    def begin(resets, reqs, packed=None):
        for s, max_len in resets:
            eng.reset(s, max_len, 0)
        if reqs:
            eng.step_begin(reqs, packed)

    total = ramp + warmup + steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gen, h2d, d2h = 0, 0, 0
    resets, reqs, g = plan()
    begin(resets, reqs)
    for i in range(total):
        nxt = plan() if i + 1 < total else None
        packed = eng._items(nxt[1])[0] if nxt is not None and nxt[1] else None  # while step i runs
        if reqs:
            eng.step_end(reqs)
        if i >= ramp + warmup:
            gen += g
            n_sel = sum(1 for r in reqs if r.select)
            h2d += 2 * (len(reqs) * 20) + 8
            d2h += n_sel * 12
        if i + 1 == ramp + warmup:
            torch.cuda.synchronize()
            e0.record(stream)
        if nxt is not None:
            resets, reqs, g = nxt
            begin(resets, reqs, packed)
    e1.record(stream)
    torch.cuda.synchronize()
    return {"ms": e0.elapsed_time(e1), "generated": gen, "h2d": int(h2d / steps), "d2h": int(d2h / steps)}

if __name__ == "__main__":
    main()

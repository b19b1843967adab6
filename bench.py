#!/usr/bin/env python
"""Benchmark of the AKV cache-operation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c2|c1|c5|c4|c3m|c4p|c4o|c4m|c3g] [--layers L]

Metric: reposition+drop retained-KV GB/s (algorithmic bytes / time).  At
N = 1 the workload is c2, the GPT-OSS-120B-shaped cache: one 65536-token
request, 36 layers, 8 KV heads, head_dim 64, bf16, about 40 % dropped in
20 spans, Reposition with YaRN RoPE.  One step = one Drop + Reposition:
``DropCompactor`` (keep mask, scan, decode view, transitions, freed slots on
the device; three launches) followed by one ``reposition_kv_layers`` launch
over all 36 layers driven by the device-side transition count.  Moved
tokens are private to the request, so they are rotated in place.

Algorithmic bytes per step (per GPU): reposition, in place: per moved token,
layer and local head 2 * rotary_dim * 2 bytes (read + write the rotary
part); drop: T (keep mask) + 4 T (slot row) + 8 A (decode view) + 4 (T - A)
(freed slots) + 12 per transition.  KV inputs (2.4 GB of K) exceed the
126 MB L2, so no flush is needed between steps.

Multi-GPU: one process per GPU (torchrun); KV heads are split 8 / N per
rank as in SGLang tensor parallelism and every rank computes the same drop
metadata (the scheduler state is replicated per TP rank); no collective on
the data path, a barrier around the timed region and a MAX all-reduce of
the timings afterwards.  The workload is fixed as N grows (strong
scaling); the aggregate counts every rank's bytes.

The same JSON line carries three more sections of the path, each with its own
metric, roofline and CPU reference: ``decode_attention`` (c4: paged GQA
decode with sinks over the compacted cache, batch 128, 36 layers alternating
sliding-window and full attention; tokens/s) and ``event_compiler`` (c3m: the
general multi-stage event compiler over 64 multi-turn agent programs,
1.13M tokens; tokens/s), and ``prefill_attention`` (c4p: the new turn's
prefill over the compacted cache with position holes, tensor-bound;
tokens/s and TFLOP/s).  ``--workload c4`` / ``c3m`` / ``c4p`` run one of
them alone.

``--impl reference``: the reference's CPU implementation of the path on the
host cores (rank 0 only): its own C++ event compiler (oracle/_ref, built
from the reference sources) + the decode view in numpy + the CPU
restatement of its reposition kernel (the reference has no CPU reposition),
each step a bounded sample of the reposition scaled to the full step.
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
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "reposition+drop retained-KV GB/s"
UNIT = "GB/s"

WORKLOADS = {
    # name: (layers, kv heads, head_dim, rope)
    "c1": (1, 8, 64, "rope10000"),
    "c2": (36, 8, 64, "yarn"),
    "c5": (80, 8, 128, "rope500000"),
    "c4": (36, 8, 64, None),  # decode attention only (see bench_attention)
    "c3m": (0, 0, 0, None),   # event compiler only (see bench_compiler)
    "c4p": (36, 8, 64, None),  # prefill attention only (see bench_prefill)
    "c4o": (0, 0, 0, None),   # occurrence binding of a c4p forward only (bench_occurrence)
    "c4m": (0, 0, 0, None),   # decode metadata of the c4 batch only (bench_decode_metadata)
    "c3g": (0, 0, 0, None),   # active-slot gather of the c3 batch only (bench_active_slots)
    "c3": (36, 8, 64, "yarn"),  # batched copy-on-write Drop + Reposition only (bench_c3)
}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="c2")
    p.add_argument("--layers", type=int, default=None,
                   help="override the workload's layer count (a smaller cut for ncu captures)")
    p.add_argument("--shard", type=int, default=1, choices=[1, 2, 4, 8],
                   help="c4 / c3: run one rank's share of an N-way KV-head split on this "
                        "GPU (8/N KV heads; a profiling aid, not a multi-GPU run)")
    p.add_argument("--variant", type=int, default=0,
                   help="c4p: prefill kernel (0 the default for the shape, 1 mma.sync, 2 tcgen05, "
                        "3 tcgen05 warp-specialised, 4 the same with two query tiles per CTA, "
                        "5 / 6: 3 / 4 with P rounded to bf16 for P.V)")
    p.add_argument("--head-dim", type=int, default=64, choices=[64, 128],
                   help="c4p: head_dim of the prefill shape")
    p.add_argument("--page-size", type=int, default=1, choices=[1, 16],
                   help="c3: page size of the KV pool")
    p.add_argument("--slot-layout", default="random", choices=["random", "paged16"],
                   help="c4: where a request's keys sit in the pool")
    p.add_argument("--requests", type=int, default=None,
                   help="c3 / c5: number of requests (a smaller cut for ncu captures)")
    return p.parse_args()


def program_for(name):
    from akv_b200 import workloads

    if name == "c1":
        return workloads.c1_program()
    if name == "c2":
        return workloads.c2_program()
    if name == "c5":
        return workloads.c5_program(requests=1)
    raise ValueError(name)


def cos_sin(name, dim, max_pos):
    from akv_b200.rope import rope_cos_sin_cache, yarn_cos_sin_cache

    rope = WORKLOADS[name][3]
    if rope == "yarn":
        return yarn_cos_sin_cache(max_pos, dim, 150000.0, 32.0, 4096, truncate=False)
    return rope_cos_sin_cache(max_pos, dim, float(rope[4:]))


def plan_stats(prog):
    """Host-side closed form of the single-stage program: kept tokens and
    moved tokens per request (what the kernels will produce)."""
    kept, moved = 0, 0
    for r in range(prog.requests):
        keep = prog.keep_mask(r)
        kept += int(keep.sum())
        dropped = np.flatnonzero(~keep)
        if len(dropped):
            moved += int((keep & (np.arange(len(keep)) > dropped[0])).sum())
    return prog.total_tokens, kept, moved


def algorithmic_bytes(prog, heads_local, layers, dim, rot, elem=2):
    t, a, n = plan_stats(prog)
    reposition = n * layers * heads_local * 2 * rot * elem
    drop = t + 4 * t + 8 * a + 4 * (t - a) + 12 * n
    return reposition, drop


NOMINAL_PEAKS = {"GB/s": 8000.0, "TFLOP/s": 2250.0}  # B200 HBM3e; dense bf16


def with_nominal_fractions(obj):
    """Every ``roofline`` object in ``obj`` also gets its achieved figure as
    a fraction of the B200's nominal peak (8 TB/s HBM3e, 2.25 PFLOP/s dense
    bf16) beside the fraction of the measured one."""
    if isinstance(obj, dict):
        roof = obj.get("roofline")
        if isinstance(roof, dict) and roof.get("unit") in NOMINAL_PEAKS and \
                isinstance(roof.get("achieved"), (int, float)):
            roof["nominal_peak"] = NOMINAL_PEAKS[roof["unit"]]
            roof["frac_of_nominal"] = round(roof["achieved"] / roof["nominal_peak"], 4)
        for v in obj.values():
            with_nominal_fractions(v)
    elif isinstance(obj, list):
        for v in obj:
            with_nominal_fractions(v)
    return obj


def emit(line):
    """Print one result line (JSON) with the nominal-peak fractions added."""
    print(json.dumps(with_nominal_fractions(line)), flush=True)


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic(workload, algorithmic=None):
    """Per-launch DRAM bytes of the reposition kernel from the committed ncu
    summary (profiles/reposition_<workload>.md): its measured bytes per
    launch, or its measured traffic / algorithmic ratio times this launch's
    algorithmic bytes; None if not captured."""
    path = os.path.join(ROOT, "profiles", f"reposition_{workload}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip())
            if line.startswith("traffic_ratio:") and algorithmic is not None:
                return int(round(float(line.split(":")[1].strip()) * algorithmic))
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of this rank's GPU,
    sampled through NVML (read-only queries) every 50 ms on a thread during
    a timed region.  Samples taken while the GPU is busy count as under
    load."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index):
        self.handle = None
        self.samples = []
        self._stop = None
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            uuid = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # no NVML: report the clocks as unknown
            self.error = f"{type(exc).__name__}: {exc}"

    def _run(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                reasons = get_reasons(self.handle)
                util = nv.nvmlDeviceGetUtilizationRates(self.handle).gpu
                self.samples.append((sm, reasons, util))
            except Exception:
                pass
            self._stop.wait(0.05)

    def start(self):
        if self.handle is None:
            return
        import threading

        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self):
        if self.handle is None:
            return {"error": getattr(self, "error", "NVML unavailable")}
        self._stop.set()
        self._thread.join(timeout=2)
        if not self.samples:
            return None
        loaded = [s for s in self.samples if s[2] > 0] or self.samples
        reasons = set()
        for _, bits, _ in loaded:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in loaded), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples),
                "samples_under_load": len(loaded)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        # The path has no exchange: the process group only carries the
        # barriers around timed regions and the MAX of the timings, on the
        # host (gloo), so no NCCL communicator is created at all.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def dist_max(x, world):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def dist_barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def reference_triton():
    """The reference's own Triton kernels, loaded unmodified from the
    reference package installed in baseline/_ref (pip --target of its
    akv/system project): {"reposition": context_reposition module,
    "page_table": context_page_table module}; None when not installed or
    Triton is unusable.  They are the same-box GPU competitor: Triton JITs
    them for sm_100 on first use."""
    base = os.path.join(ROOT, "baseline", "_ref", "akv", "system", "sglang", "kernels", "ops",
                        "attention")
    paths = {"reposition": os.path.join(base, "context_reposition.py"),
             "page_table": os.path.join(base, "context_page_table.py")}
    if not all(os.path.exists(p) for p in paths.values()):
        return None
    import importlib.util

    mods = {}
    try:
        for name, path in paths.items():
            spec = importlib.util.spec_from_file_location(f"akv_reference_{name}", path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mods[name] = mod
    except Exception:
        return None
    return mods


def reference_context_metadata():
    """The reference's ``ContextAttentionMetadata`` class (the native-plan
    builder of its FlashInfer / FA3 context path, context_backend.py:171-222),
    loaded unmodified from the reference package in baseline/_ref under
    stand-in ``sglang`` package names that are removed again; a one-line
    reason instead when the package is not installed or does not load."""
    import importlib.util
    import types

    sg = os.path.join(ROOT, "baseline", "_ref", "akv", "system", "sglang")
    files = [("sglang.srt.context_system.request_storage", "srt/context_system/request_storage.py"),
             ("sglang.srt.context_system.occurrence", "srt/context_system/occurrence.py"),
             ("sglang.srt.layers.attention.context_backend",
              "srt/layers/attention/context_backend.py")]
    if not all(os.path.exists(os.path.join(sg, rel)) for _, rel in files):
        return "the reference package is not installed in baseline/_ref"
    from akv_b200 import context_page_table, context_reposition

    saved = {k: v for k, v in sys.modules.items() if k == "sglang" or k.startswith("sglang.")}
    try:
        for pkg in ("sglang", "sglang.kernels", "sglang.kernels.ops",
                    "sglang.kernels.ops.attention", "sglang.srt", "sglang.srt.context_system",
                    "sglang.srt.layers", "sglang.srt.layers.attention"):
            sys.modules[pkg] = types.ModuleType(pkg)
        sys.modules["sglang.kernels.ops.attention.context_reposition"] = context_reposition
        sys.modules["sglang.kernels.ops.attention.context_page_table"] = context_page_table
        mod = None
        for name, rel in files:
            spec = importlib.util.spec_from_file_location(name, os.path.join(sg, rel))
            mod = importlib.util.module_from_spec(spec)
            sys.modules[name] = mod
            spec.loader.exec_module(mod)
        return mod.ContextAttentionMetadata
    except Exception as exc:
        return f"the reference's context_backend.py did not load: {type(exc).__name__}: {exc}"
    finally:
        for k in [k for k in sys.modules if k == "sglang" or k.startswith("sglang.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def flashinfer_prefill_versus_ours(att, q, k_pool, v_pool, kv_idx, births, qo, kv, qpos, kpos,
                                   window, sinks, out, steps, stream, run_ours):
    """One context-prefill layer through the reference's runtime path and
    through ours, same pools, slots, positions and sinks.  The reference
    (sglang.patch:1303-1331): ``ContextAttentionMetadata.native_plan`` (its
    own code, built once per forward, outside the timing) gives ragged
    segments and the gathered key slots; per layer it gathers K and V at
    those slots, runs FlashInfer's ragged prefill (backend "fa2", causal,
    window_left) with the lse and applies the sink correction.  Returns ms
    of that layer sequence, of the FlashInfer launch alone, of ours, and
    the largest output difference; an "unavailable" note when the reference
    package or FlashInfer is missing here."""
    meta_cls = reference_context_metadata()
    if isinstance(meta_cls, str):
        return {"unavailable": meta_cls}
    try:
        import flashinfer

        dev = q.device
        hq, hkv, d = q.shape[1], k_pool.shape[1], q.shape[2]
        t64 = lambda a: torch.as_tensor(np.asarray(a, np.int64), device=dev)  # noqa: E731
        q_lengths = tuple(int(v) for v in np.diff(qo))
        meta = meta_cls(t64(qo), t64(kv), kv_idx.long(), t64(qpos), t64(kpos), q_lengths,
                        int(qo[-1]), max(q_lengths),
                        (np.asarray(qo, np.int64), np.asarray(kv, np.int64), None,
                         np.asarray(qpos, np.int64), np.asarray(kpos, np.int64)))
        cpu_qo, cpu_kv, _, _, slots, _, _ = meta.native_plan(births.long(), window)
        work = torch.zeros(128 << 20, dtype=torch.uint8, device=dev)
        wrapper = flashinfer.BatchPrefillWithRaggedKVCacheWrapper(work, "NHD", backend="fa2")
        wrapper.plan(cpu_qo, cpu_kv, hq, hkv, d, causal=True, window_left=window,
                     logits_soft_cap=0.0, sm_scale=att.sm_scale, q_data_type=torch.bfloat16,
                     kv_data_type=torch.bfloat16)
        k_g, v_g = k_pool[slots], v_pool[slots]
        fi_out = torch.empty_like(q)
        fi_lse = torch.empty(q.shape[0], hq, dtype=torch.float32, device=dev)

        def kernel_only():
            wrapper.run(q, k_g, v_g, out=fi_out, lse=fi_lse, return_lse=True)

        def theirs():
            o, lse = wrapper.run(q, k_pool[slots], v_pool[slots], out=fi_out, lse=fi_lse,
                                 return_lse=True)
            o.mul_(torch.sigmoid(lse * 0.6931471805599453 - sinks.float()).unsqueeze(-1))

        theirs()
        torch.cuda.synchronize()
    except Exception as exc:  # library missing or its JIT build failing
        return {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}"}
    t_layer = time_launches(theirs, steps, stream)
    t_kernel = time_launches(kernel_only, steps, stream)
    t_ours = time_launches(run_ours, steps, stream)
    theirs()
    run_ours()
    torch.cuda.synchronize()
    diff = float((out.float() - fi_out.float()).abs().max())
    return {"flashinfer": flashinfer.__version__, "segments": len(cpu_qo) - 1,
            "gathered_keys": int(slots.numel()),
            "flashinfer_layer_ms": round(t_layer, 4), "flashinfer_kernel_ms": round(t_kernel, 4),
            "ours_ms": round(t_ours, 4), "speedup": round(t_layer / t_ours, 2),
            "speedup_vs_kernel_alone": round(t_kernel / t_ours, 2),
            "max_abs_diff": round(diff, 5)}


def time_launches(fn, steps, stream, warmup=2):
    """Mean CUDA-event time of ``fn()`` over ``steps`` back-to-back calls
    (after ``warmup`` untimed calls), in ms."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        fn()
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / steps


def triton_versus_ours(ref, k_ptrs, v_ptrs, k0, v0, src, dst, pairs, cache, steps, stream,
                       our_bytes):
    """One reposition list through the reference's Triton launch and through
    ours (same pools, slots and positions): ms of each and the ratio.  The
    reference always moves the K tail and V as well (its contract is a copy
    to fresh slots), so on an in-place list it does more work than ours."""
    from akv_b200.context_reposition import reposition_kv_layers

    def theirs():
        ref["reposition"].reposition_kv_layers(k_ptrs, v_ptrs, k0, v0, src, dst, pairs, cache)

    def ours():
        reposition_kv_layers(k_ptrs, v_ptrs, k0, v0, src, dst, pairs, cache)

    t_ref = time_launches(theirs, steps, stream)
    t_ours = time_launches(ours, steps, stream)
    return {"transitions": int(src.numel()), "triton_ms": round(t_ref, 4),
            "ours_ms": round(t_ours, 4), "speedup": round(t_ref / t_ours, 2),
            "ours_gb_per_s": round(our_bytes / (t_ours / 1e3) / 1e9, 1)}


def flashinfer_versus_ours(attn, q, k_pool, v_pool, indptr, indices, sinks, out, steps, stream):
    """One decode layer through the reference's runtime path and through
    ours, on the same pools, indices and sinks: FlashInfer's
    BatchDecodeWithPagedKVCacheWrapper (page size 1, tensor-core variant, the
    one SGLang takes for GQA groups of 4+ at 16-bit KV) returning the
    log2-sum-exp, then the reference backend's in-place sink correction
    o *= sigmoid(lse * ln 2 - sink) (akv/system/sglang.patch:1535-1551).
    Planning is outside the timed calls on both sides.  Returns ms of each,
    the ratio and the largest output difference; None when FlashInfer cannot
    be imported or built here."""
    try:
        import flashinfer

        bs, hq, d = q.shape
        work = torch.zeros(128 << 20, dtype=torch.uint8, device=q.device)
        wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(work, kv_layout="NHD",
                                                               use_tensor_cores=True)
        wrapper.plan(torch.from_numpy(np.asarray(indptr, np.int32)).to(q.device), indices,
                     torch.ones(bs, dtype=torch.int32, device=q.device), hq, k_pool.shape[1],
                     d, 1, pos_encoding_mode="NONE", q_data_type=torch.bfloat16,
                     kv_data_type=torch.bfloat16, sm_scale=attn.sm_scale)
        kv = (k_pool.unsqueeze(1), v_pool.unsqueeze(1))
        fi_out = torch.empty_like(out)
        fi_lse = torch.empty(bs, hq, dtype=torch.float32, device=q.device)

        def theirs():
            o, lse = wrapper.run(q, kv, out=fi_out, lse=fi_lse, return_lse=True)
            o.mul_(torch.sigmoid(lse * 0.6931471805599453 - sinks.float()).unsqueeze(-1))

        theirs()
        torch.cuda.synchronize()
    except Exception as exc:  # library missing or its JIT build failing
        return {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:160]}"}

    def ours():
        attn.run(q, k_pool, v_pool, indices, sinks=sinks, out=out)

    t_ref = time_launches(theirs, steps, stream)
    t_ours = time_launches(ours, steps, stream)
    theirs()
    ours()
    torch.cuda.synchronize()
    diff = float((out.float() - fi_out.float()).abs().max())
    return {"flashinfer": flashinfer.__version__, "variant": "tensor cores + sink correction",
            "flashinfer_ms": round(t_ref, 4), "ours_ms": round(t_ours, 4),
            "speedup": round(t_ref / t_ours, 2), "max_abs_diff": round(diff, 5)}


def cpu_reference_step(prog, rows, layers, heads, dim, cache_np, sample, rng, threads):
    """One step of the reference's CPU path: its C++ event compiler
    (oracle/_ref) + numpy decode view + the reposition restatement over a
    sample of the moved tokens.  Returns (seconds scaled to the full step,
    sample size)."""
    from oracle import oracle, reference

    t0 = time.perf_counter()
    lays = []
    for r in range(prog.requests):
        t = int(prog.token_counts[r])
        rr = prog.request_ranges(r)
        has = len(rr) > 0
        comp = reference.compile_context_layout if reference.available() else \
            oracle.compile_layout
        lay = comp(np.zeros(t, np.int32), [t] if has else [], [0, len(rr) // 2] if has else [0],
                   rr, [t - 1], [t])
        raw = np.flatnonzero(lay["keep_mask"]).astype(np.int32)
        _ = lay["positions"][raw]
        lays.append(lay)
    t_drop = time.perf_counter() - t0
    lay = lays[0]
    moved = lay["transition_raw_tokens"]
    n = len(moved)
    m = min(sample, n)
    pick = rng.choice(n, size=m, replace=False) if m < n else np.arange(n)
    slots = rows[0][moved[pick]].astype(np.int32)
    pairs = np.stack((lay["transition_old_positions"][pick],
                      lay["transition_new_positions"][pick]), 1).astype(np.int32)
    # K rows of the sampled tokens, all layers, as bf16 bit patterns; the
    # in-place rotation reads and writes exactly these rows.
    k = [np.random.default_rng(l).integers(0, 1 << 16, size=(m, heads, dim), dtype=np.uint16)
         & 0x7F7F for l in range(layers)]
    idx = np.arange(m, dtype=np.int32)
    t1 = time.perf_counter()
    oracle.reposition(k, k, idx, idx, pairs, cache_np, bf16=True, threads=threads)
    t_rep = time.perf_counter() - t1
    del slots
    return t_drop, t_rep * (n / max(1, m)), m, n


def cpu_parts(t_drop, t_rep, m, n, layers, heads, tokens):
    """The two halves of a CPU step, each with its own kind: the event
    compiler is the reference's own code (oracle/_ref) when it was built
    here, the reposition is always this package's restatement (the
    reference has no CPU reposition)."""
    from oracle import reference

    ref = reference.available()
    return {
        "event_compiler": {"kind": "reference" if ref else "port", "ms": round(t_drop * 1e3, 3),
                           "what": f"{'reference C++ (oracle/_ref)' if ref else 'oracle port'} "
                                   f"over all {tokens} tokens + numpy decode view, one thread"},
        "reposition": {"kind": "port", "ms": round(t_rep * 1e3, 3),
                       "what": f"C restatement of the reference kernel on {m} of {n} moved "
                               f"tokens x {layers} layers x {heads} heads, scaled to all {n}"},
    }


def run_reference(args):
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return 0
    from akv_b200 import workloads

    layers, heads, dim, _ = WORKLOADS[args.workload]
    layers = args.layers or layers
    prog = program_for(args.workload)
    rows, _ = workloads.slot_rows(np.random.default_rng(0), prog)
    cache_np = cos_sin(args.workload, dim, 131072).numpy()
    threads = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(0)
    rep_bytes, drop_bytes = algorithmic_bytes(prog, heads, layers, dim, dim)
    sample = 4000
    for _ in range(args.warmup):
        cpu_reference_step(prog, rows, layers, heads, dim, cache_np, sample, rng, threads)
    times, drops, reps = [], [], []
    for _ in range(args.steps):
        t_drop, t_rep, m, n = cpu_reference_step(prog, rows, layers, heads, dim, cache_np,
                                                 sample, rng, threads)
        times.append(t_drop + t_rep)
        drops.append(t_drop)
        reps.append(t_rep)
    sec = sum(times)
    value = (rep_bytes + drop_bytes) * args.steps / sec / 1e9
    desc = (f"{args.workload} per step: event compiler over all {prog.total_tokens} tokens + "
            f"decode view; reposition restatement on {m} of {n} moved tokens x {layers} layers "
            f"x {heads} heads, time scaled to all {n} (parts below)")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * sec / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": args.workload, "layers": layers, "kv_heads": heads, "head_dim": dim,
                   "tokens": prog.total_tokens},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc,
                         "parts": cpu_parts(sum(drops) / args.steps, sum(reps) / args.steps, m,
                                            n, layers, heads, prog.total_tokens)},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)
    return 0


def run_ours(args):
    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor, FreeSlotRing
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers

    layers, heads_total, dim, _ = WORKLOADS[args.workload]
    layers = args.layers or layers
    if heads_total % world:
        raise SystemExit(f"{heads_total} KV heads do not split over {world} GPUs")
    heads = heads_total // world
    prog = program_for(args.workload)
    rows, nslots = workloads.slot_rows(np.random.default_rng(0), prog)
    total, kept, moved = plan_stats(prog)
    freed_per_step = total - kept

    # KV pools of this rank's heads, [slot, head, dim] per layer.
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    k_pools = [torch.randn(nslots, heads, dim, device=dev, generator=g).to(torch.bfloat16)
               for _ in range(layers)]
    v_pools = [torch.empty(nslots, heads, dim, device=dev, dtype=torch.bfloat16)
               for _ in range(layers)]
    k_ptrs, v_ptrs = layer_pointer_table(k_pools), layer_pointer_table(v_pools)
    cache = cos_sin(args.workload, dim, 131072).to(dev)
    table = np.zeros((prog.requests + 1, int(prog.token_counts.max())), np.int32)
    for r in range(prog.requests):
        table[r + 1, : len(rows[r])] = rows[r]
    req_to_token = torch.from_numpy(table).to(dev)
    row_ids = np.arange(1, prog.requests + 1)
    steps_total = args.warmup + 3 * args.steps + 4  # timed, breakdown and e2e passes
    ring = FreeSlotRing(torch.zeros(0, dtype=torch.int32),
                        capacity=freed_per_step * steps_total + 16, device=dev)
    comp = DropCompactor(total, prog.requests, max(1, len(prog.ranges) // 2), dev)
    stream = torch.cuda.current_stream(dev)

    prepared = comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges, row_ids)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]

    def step(i=None):
        if i is not None:
            ev[i][0].record(stream)
        res = comp.launch(prepared, req_to_token, ring)
        if i is not None:
            ev[i][1].record(stream)
        reposition_kv_layers(k_ptrs, v_ptrs, k_pools[0], v_pools[0], res.transition_source,
                             res.transition_destination, res.transition_pairs, cache,
                             count_device=res.transition_count)
        if i is not None:
            ev[i][2].record(stream)
        return res

    for _ in range(args.warmup):
        res = step()
    torch.cuda.synchronize()
    res.check()
    assert int(res.totals[1].item()) == moved

    clocks = ClockSampler(local)
    dist_barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    h0 = time.perf_counter()
    for i in range(args.steps):
        step()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    t_end.record(stream)
    torch.cuda.synchronize()
    dist_barrier(world)
    clock_info = clocks.stop()
    ms = t_start.elapsed_time(t_end)
    ms = dist_max(ms, world)
    # Per-kernel breakdown in a second pass: an event between the drop and
    # the reposition launch stops the reposition blocks from being scheduled
    # while the drop scatter runs, so it is kept out of the timed loop.
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    drop_ms = [a.elapsed_time(b) for a, b, _ in ev]
    rep_ms = [b.elapsed_time(c) for _, b, c in ev]

    # e2e: through the public API with the program in host memory: validate,
    # stage (one pinned H2D copy), launch, and read the decode view back.
    # Like a serving loop, the host issues step i+1 before it waits for the
    # read-back of step i (two pinned result buffers), so host work overlaps
    # the GPU; every step still pays its own H2D and D2H.  The decode view
    # is final once the drop kernels end, so its read-back runs on a second
    # stream beside the reposition launch; the next step's drop waits for it.
    # [raw(kept) | positions(kept) | offsets(n + 1) | next(n) | totals(4) | status]
    n_out = 2 * kept + 2 * prog.requests + 6
    a_host = [torch.empty(n_out, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    viewed = torch.cuda.Event()
    readback = torch.cuda.Stream(dev)
    d2h = 4 * n_out
    h2d = prepared["h2d_bytes"]

    def check(buf):
        if int(buf[-1]) != 0:
            raise RuntimeError("drop_compact status in the e2e loop")

    torch.cuda.synchronize()
    dist_barrier(world)
    torch.cuda.synchronize()
    # Device-clock bracket: the stream is idle when e0 is recorded, so the
    # interval to e1 includes every host-side step in between.
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        if i > 0:
            stream.wait_event(done[(i - 1) % 2])  # the last read-back has left
        res = comp.run(prog.token_counts, prog.range_offsets, prog.ranges, req_to_token,
                       row_ids, ring)
        viewed.record(stream)
        reposition_kv_layers(k_ptrs, v_ptrs, k_pools[0], v_pools[0], res.transition_source,
                             res.transition_destination, res.transition_pairs, cache,
                             count_device=res.transition_count)
        readback.wait_event(viewed)
        res.read_view(a_host[i % 2], stream=readback)  # one library call, five copies
        done[i % 2].record(readback)
        if i > 0:
            done[(i - 1) % 2].synchronize()
            check(a_host[(i - 1) % 2])
    stream.wait_event(done[(args.steps - 1) % 2])
    e1.record(stream)
    done[(args.steps - 1) % 2].synchronize()
    e1.synchronize()
    check(a_host[(args.steps - 1) % 2])
    e2e_s = dist_max(e0.elapsed_time(e1) / 1e3, world)
    dist_barrier(world)

    rep_bytes, drop_bytes = algorithmic_bytes(prog, heads, layers, dim, dim)
    step_bytes = (rep_bytes + drop_bytes) * world
    value = step_bytes * args.steps / (ms / 1e3) / 1e9
    e2e_value = step_bytes * args.steps / e2e_s / 1e9
    rep_mean = statistics.mean(rep_ms)
    peak, peak_kind = measured_peak()
    achieved = rep_bytes / (rep_mean / 1e3) / 1e9
    traffic = ncu_traffic(args.workload) if world == 1 else None

    # The reference's Triton reposition kernel on the same box, on the same
    # transitions (in place: destination = source).
    triton_ref = None
    ref = reference_triton()
    if ref is not None and world == 1:
        n = moved
        triton_ref = triton_versus_ours(
            ref, k_ptrs, v_ptrs, k_pools[0], v_pools[0], res.transition_source[:n],
            res.transition_source[:n], res.transition_pairs[:n], cache, 5, stream, rep_bytes)
        triton_ref["what"] = ("c2 moved tokens in place (destination = source); the Triton "
                              "kernel also rewrites V, which in place is the same bytes")
    # Second metric: paged GQA decode attention over the compacted cache (c4).
    del k_pools, v_pools
    torch.cuda.empty_cache()
    # The other sections have workloads of their own; they run beside the
    # default (c2) line only.
    attention = attention_paged = compiler = prefill = gather = occurrence = metadata = None
    c3 = {}
    c5 = None
    if args.workload == "c2":
        c5 = bench_c5(dev, world, rank, 2, max(3, min(args.steps, 10)))
        c3 = bench_c3(dev, world, rank, 3, max(5, min(args.steps, 20)))
        attention = bench_attention(dev, world, rank, max(3, min(args.warmup, 5)),
                                    max(5, min(args.steps // 20, 20)), compare=world == 1)
        attention_paged = bench_attention(dev, world, rank, max(3, min(args.warmup, 5)),
                                          max(5, min(args.steps // 20, 20)), layout="paged16")
        compiler = bench_compiler(dev, world, rank, 3, 20)
        prefill = bench_prefill(dev, world, rank, 3, 5, compare=world == 1)
        gather = bench_active_slots(dev, world, rank, 3, 20)
        occurrence = bench_occurrence(dev, world, rank, 3, 20)
        metadata = bench_decode_metadata(dev, world, rank, 3, 20)

    cpu = None
    if rank == 0 and world == 1:
        cache_np = cache.cpu().numpy()
        threads = len(os.sched_getaffinity(0))
        t_drop, t_rep, m, n = cpu_reference_step(prog, rows, layers, heads, dim, cache_np, 4000,
                                                 np.random.default_rng(0), threads)
        cpu = {"value": round((rep_bytes + drop_bytes) / (t_drop + t_rep) / 1e9, 3),
               "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"one c2 step: event compiler over all {total} tokens + reposition "
                         f"restatement on {m} of {n} moved tokens, scaled (parts below)",
               "parts": cpu_parts(t_drop, t_rep, m, n, layers, heads, total)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": args.workload, "layers": layers, "kv_heads": heads_total,
                       "kv_heads_per_gpu": heads, "head_dim": dim, "tokens": total,
                       "moved_tokens": moved, "dropped_tokens": total - kept,
                       "reposition": "in place", "rope": WORKLOADS[args.workload][3],
                       "parallelism": f"kv-head tp{world}",
                       "l2": "inputs larger than L2 (K pools 2.4 GB per 36 layers), no flush"},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "kernel": "reposition_kernel",
                         "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": rep_bytes,
                         "ms_per_launch": round(rep_mean, 4)},
            # host time to enqueue one step; below ms_per_step the GPU never waits
            "host_enqueue_ms_per_step": round(host_ms, 4),
            "breakdown_ms": {"drop_compact": round(statistics.mean(drop_ms), 4),
                             "reposition": round(rep_mean, 4)},
            "gpu_launches": 4 * args.steps,
            "cpu_baseline": cpu,
            "triton_reference": triton_ref,
            "event_compiler": compiler,
            "prefill_attention": prefill,
            "active_slots": gather,
            "occurrence_binding": occurrence,
            "decode_metadata": metadata,
            "c5": c5,
            "c3_page_size_1": c3.get(1),
            "c3_page_size_16": c3.get(16),
            "decode_attention": attention,
            "decode_attention_paged16": attention_paged,
            "clocks": clock_info,
        }
        # Last, so that a reader that keeps only the end of the line still
        # sees every section's headline: value, unit, kernel fraction of the
        # HBM (or tensor) peak, e2e and CPU-baseline values.
        summary = {}
        for name, sec in (("c2", line), ("c5", c5), ("c3_ps1", c3.get(1)),
                          ("c3_ps16", c3.get(16)),
                          ("decode_attention", attention),
                          ("decode_attention_paged16", attention_paged),
                          ("prefill_attention", prefill),
                          ("event_compiler", compiler), ("decode_metadata", metadata),
                          ("active_slots", gather), ("occurrence_binding", occurrence)):
            if not sec:
                continue
            item = {"value": sec["value"], "unit": sec["unit"]}
            if sec.get("roofline"):
                item["frac"] = sec["roofline"]["frac"]
            if isinstance(sec.get("e2e"), dict):
                item["e2e"] = sec["e2e"]["value"]
            if isinstance(sec.get("cpu_baseline"), dict):
                item["cpu"] = sec["cpu_baseline"]["value"]
            tri = sec.get("triton_reference")
            if isinstance(tri, dict) and "speedup" in tri:
                item["vs_triton"] = tri["speedup"]
            fi = (sec.get("reference_runtime_decode") or sec.get("reference_runtime_prefill")
                  or {}).get("full_layer")
            if isinstance(fi, dict) and "speedup" in fi:
                item["vs_flashinfer"] = fi["speedup"]
            kinds = sec.get("reposition_by_kind") or {}
            if "copy_on_write" in kinds:
                item["cow_frac"] = kinds["copy_on_write"]["frac"]
                tri = kinds["copy_on_write"].get("triton_reference")
                if tri:
                    item["cow_vs_triton"] = tri["speedup"]
            summary[name] = item
        line["summary"] = summary
        emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def bench_attention(dev, world, rank, warmup, steps, seed=0, layers=36, shard=1,
                    layout="random", compare=False):
    """c4: batch 128, 64 query / 8 KV heads (split 8/N per rank), head_dim 64,
    bf16, lognormal KV lengths (median 8192, sigma 1.0, max 65536), 36 layers
    alternating sliding window 128 and full attention, per-head sinks.  One
    step = one decode token for the whole batch = 36 layer launches (18
    full over all keys, 18 over the 129 visible keys of each request), each
    layer with its own K/V pool.  tokens/s = batch / step time.

    ``layout``: where a request's keys sit in the pool.  "random": every key
    at a random slot (a page_size 1 pool after much churn; the worst case
    for DRAM locality).  "paged16": a page_size 16 pool (the layout the
    paged Drop keeps): a request's keys fill its own 16-slot pages in order,
    the pages at random places in the pool.

    ``compare``: also time the reference's runtime decode (FlashInfer plus
    the sink correction) on one full and one sliding-window layer, outside
    the timed step."""
    from akv_b200 import workloads
    from akv_b200.context_attention import DecodeAttention

    bs, hq_total, hkv_total, d, window = 128, 64, 8, 64, 128
    hkv = hkv_total // (world * shard)
    hq = hq_total // (world * shard)
    lengths = workloads.c4_lengths(seed=seed, batch=bs)
    rng = np.random.default_rng(seed)
    total = int(lengths.sum())
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    full_indptr = np.concatenate(([0], np.cumsum(lengths)))
    swa_len = np.minimum(lengths, window + 1)
    swa_indptr = np.concatenate(([0], np.cumsum(swa_len)))
    def slots_for(lens):
        if layout == "random":
            return rng.permutation(int(lens.sum())).astype(np.int32), int(lens.sum())
        pages_per = -(-lens // 16)
        pages = rng.permutation(int(pages_per.sum())).astype(np.int64)
        firsts = np.concatenate(([0], np.cumsum(pages_per)))
        out = []
        for b, n in enumerate(lens.tolist()):
            i = np.arange(n)
            out.append(pages[firsts[b] + i // 16] * 16 + i % 16)
        return np.concatenate(out).astype(np.int32), int(pages_per.sum()) * 16

    # Keys of a request sit in its layer's pool at the layout's slots.
    full_np, full_slots = slots_for(lengths)
    swa_np, swa_slots = slots_for(swa_len)
    full_idx = torch.from_numpy(full_np).to(dev)
    swa_idx = torch.from_numpy(swa_np).to(dev)
    pools = []
    for layer in range(layers):
        slots = full_slots if layer % 2 else swa_slots
        pools.append((torch.randn(slots, hkv, d, device=dev, generator=g, dtype=torch.bfloat16),
                      torch.randn(slots, hkv, d, device=dev, generator=g, dtype=torch.bfloat16)))
    q = torch.randn(bs, hq, d, device=dev, generator=g, dtype=torch.bfloat16)
    sinks = torch.randn(hq, device=dev, generator=g)
    full = DecodeAttention(hq, hkv, d, bs, dev).plan(full_indptr)
    swa = DecodeAttention(hq, hkv, d, bs, dev).plan(swa_indptr)
    out = torch.empty(bs, hq, d, device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]

    def step(i=None):
        for layer in range(layers):
            if i is not None and layer == 1:
                ev[i][0].record(stream)
            kp, vp = pools[layer]
            if layer % 2:
                full.run(q, kp, vp, full_idx, sinks=sinks, out=out)
            else:
                swa.run(q, kp, vp, swa_idx, sinks=sinks, out=out)
            if i is not None and layer == 1:
                ev[i][1].record(stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    dist_barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        step(i)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = dist_max(t0.elapsed_time(t1) / steps, world)
    full_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    full_bytes = total * hkv * d * 2 * 2
    swa_bytes = int(swa_len.sum()) * hkv * d * 2 * 2
    step_bytes = (layers // 2) * (full_bytes + swa_bytes) * world
    peak, peak_kind = measured_peak()
    achieved = full_bytes / (full_ms / 1e3) / 1e9
    runtime_ref = None
    if compare and layers >= 2:
        # The reference's runtime decode on one full and one sliding-window
        # layer (outside the timed step).
        runtime_ref = {
            "full_layer": flashinfer_versus_ours(full, q, *pools[1], full_indptr, full_idx,
                                                 sinks, out, max(steps, 10), stream),
            "sliding_window_layer": flashinfer_versus_ours(swa, q, *pools[0], swa_indptr,
                                                           swa_idx, sinks, out,
                                                           max(steps, 10), stream)}
    del pools
    torch.cuda.empty_cache()
    return {
        "metric": "paged GQA decode attn tokens/s", "value": round(bs / (ms / 1e3), 1),
        "unit": "tokens/s", "ms_per_step": round(ms, 4), "n_gpus": world,
        "gb_per_s": round(step_bytes / (ms / 1e3) / 1e9, 1),
        "config": {"workload": "c4", "slot_layout": layout, "kv_heads_per_gpu": hkv,
                   "batch": bs, "q_heads": hq_total, "kv_heads": hkv_total,
                   "head_dim": d, "layers": layers, "sliding_window": window,
                   "kv_tokens": total, "lengths": "lognormal median 8192 sigma 1.0",
                   "sinks": True, "work_items_full": full.n_items, "chunk": full.chunk},
        "roofline": {"bound": "hbm", "kernel": "decode_attention_kernel (full layer)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": full_bytes,
                     "ms_per_launch": round(full_ms, 4)},
        "gpu_launches_per_step": layers + (layers // 2 if full.split else 0),
        "reference_runtime_decode": runtime_ref,
    }


def c3_counts(prog, page_size):
    """Closed form of the c3 step on the host (what the kernels produce):
    kept, moved, copy-on-write transitions, copied units (slots at
    page_size 1, pages otherwise) and freed units (slots or pages)."""
    kept = moved = cow = copied = freed = 0
    ps = int(page_size)
    for r in range(prog.requests):
        keep = prog.keep_mask(r)
        t = np.arange(len(keep))
        rr = prog.request_ranges(r)
        first = int(rr[0]) if len(rr) else len(keep)
        mv = keep & (t > first)
        p = int(prog.shared_prefix[r])
        kept += int(keep.sum())
        if ps == 1:
            moved += int(mv.sum())
            cow += int(mv[:p].sum())
            copied += int(mv[:p].sum())
            freed += int((~keep[p:]).sum())
            continue
        n_pages = -(-len(keep) // ps)
        pad = np.zeros(n_pages * ps, bool)
        pad[: len(keep)] = mv
        page_mv = pad.reshape(n_pages, ps).any(1)
        kp = np.ones(n_pages * ps, bool)
        kp[: len(keep)] = keep
        kp[len(keep):] = False
        shared_pages = p // ps
        cow_pages = page_mv[:shared_pages]
        in_cow = np.repeat(np.concatenate((cow_pages, np.zeros(n_pages - shared_pages, bool))),
                           ps)[: len(keep)]
        trans = keep & (mv | in_cow)
        moved += int(trans.sum())
        cow += int((trans & in_cow).sum())
        copied += int(cow_pages.sum())
        freed += int((~kp.reshape(n_pages, ps)[shared_pages:].any(1)).sum())
    return kept, moved, cow, copied, freed


def bench_c3(dev, world, rank, warmup, steps, page_sizes=(1, 16), seed=0, layers=36,
             cpu=True, e2e_steps=8, requests=64, shard=1, bulk_v=None):
    """c3: batched agent serving -- 64 requests (lengths U{2K..32K}, 1.18M
    tokens), one radix-shared prefix of 1K..4K tokens (a whole number of
    16-token pages) whose moved tokens must copy-on-write, per-request drop
    fraction U[0.1, 0.6], GPT-OSS-120B KV shape (36 layers, 8 KV heads split
    8/N per rank, head_dim 64), YaRN RoPE; at page_size 1 and 16.

    One step = restore the rows and the ring head that the previous step's
    copy-on-write changed (one 8 MB device copy of req_to_token and one of
    the 16-byte ring state; the bytes are not counted) + the Drop (three
    launches) + the reposition over all 36 layers (``bulk_copy_v``: the V
    rows of the copies by TMA bulk copies in one launch, K in another).  Algorithmic
    bytes: per (transition, layer, local head) 2 * rotary_dim * 2 B in place
    and 4 * head_dim * 2 B for copy-on-write (K read + write, V read +
    write); Drop: T + 4 T + 8 A + 4 per freed unit + 12 per transition +
    4 per rewritten row entry.  The K pools (49 GB) exceed L2."""
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor, FreeSlotRing
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers
    from akv_b200.rope import yarn_cos_sin_cache

    heads_total, dim = 8, 64
    heads = heads_total // (world * shard)
    if bulk_v is None:
        # The TMA bulk move of the copies' V rows pays from 512-byte rows on
        # (4+ local heads); at one head (128 B) it loses to one-pass staging.
        bulk_v = heads * dim * 2 >= 512
    prog = workloads.c3_program(seed=seed, page_align=16, requests=requests)
    total = prog.total_tokens
    layouts = {}
    pool_slots = 0
    for ps in page_sizes:
        kept, moved, cow, copied, freed = c3_counts(prog, ps)
        rng = np.random.default_rng(seed)
        if ps == 1:
            rows, n_units = workloads.slot_rows(rng, prog)
            slots = n_units + copied
        else:
            rows, n_units = workloads.paged_slot_rows(rng, prog, ps)
            slots = (n_units + copied) * ps
        layouts[ps] = (rows, n_units, (kept, moved, cow, copied, freed))
        pool_slots = max(pool_slots, slots)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    k_pools = [torch.randn(pool_slots, heads, dim, device=dev, generator=g, dtype=torch.bfloat16)
               for _ in range(layers)]
    v_pools = [torch.empty(pool_slots, heads, dim, device=dev, dtype=torch.bfloat16)
               for _ in range(layers)]
    k_ptrs, v_ptrs = layer_pointer_table(k_pools), layer_pointer_table(v_pools)
    cache = yarn_cos_sin_cache(32768, dim, 150000.0, 32.0, 4096, truncate=False).to(dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = measured_peak()
    comp = DropCompactor(total, prog.requests, max(1, len(prog.ranges) // 2), dev)
    ref = reference_triton()
    out = {}
    for ps in page_sizes:
        rows, n_units, (kept, moved, cow, copied, freed) = layouts[ps]
        table = np.zeros((prog.requests + 1, int(prog.token_counts.max())), np.int32)
        for r in range(prog.requests):
            table[r + 1, : len(rows[r])] = rows[r]
        rtt0 = torch.from_numpy(table).to(dev)
        rtt = rtt0.clone()
        row_ids = np.arange(1, prog.requests + 1)
        ring = FreeSlotRing(torch.arange(n_units, n_units + copied, dtype=torch.int32),
                            capacity=copied + freed + 16, device=dev)
        state0 = ring.state.clone()
        prepared = comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges, row_ids,
                                shared_prefix=prog.shared_prefix, page_size=ps)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]

        def step(i=None):
            rtt.copy_(rtt0)
            ring.state.copy_(state0)
            if i is not None:
                ev[i][0].record(stream)
            res = comp.launch(prepared, rtt, ring)
            if i is not None:
                ev[i][1].record(stream)
            reposition_kv_layers(k_ptrs, v_ptrs, k_pools[0], v_pools[0], res.transition_source,
                                 res.transition_destination, res.transition_pairs, cache,
                                 count_device=res.transition_count, page_size=ps,
                                 bulk_copy_v=bulk_v)
            if i is not None:
                ev[i][2].record(stream)
            return res

        for _ in range(warmup):
            res = step()
        torch.cuda.synchronize()
        res.check()
        assert res.totals.cpu().tolist() == [kept, moved, copied, freed], \
            (res.totals.cpu().tolist(), [kept, moved, copied, freed])
        n = moved
        src = res.transition_source[:n]
        n_cow = int((src != res.transition_destination[:n]).sum().item())
        assert n_cow == cow
        rep_bytes = ((n - n_cow) * 2 * dim * 2 + n_cow * 4 * dim * 2) * layers * heads
        row_writes = copied if ps == 1 else copied * ps
        drop_bytes = total + 4 * total + 8 * kept + 4 * freed + 12 * n + 4 * row_writes
        dist_barrier(world)
        torch.cuda.synchronize()
        clocks = ClockSampler(dev.index)
        clocks.start()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        clock_info = clocks.stop()
        ms = dist_max(t0.elapsed_time(t1) / steps, world)
        for i in range(steps):
            step(i)
        torch.cuda.synchronize()
        drop_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
        rep_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
        # The two kinds of transition in separate launches (split once,
        # outside any timed region): copy-on-write moves K and V to fresh
        # slots, in-place rotates the rotary part only.
        split = {}
        cow_mask = src != res.transition_destination[:n]
        for kind, sel, bulk in (("copy_on_write", cow_mask, True), ("in_place", ~cow_mask, True),
                                ("copy_on_write_one_pass", cow_mask, False)):
            s_src = src[sel].contiguous()
            s_dst = res.transition_destination[:n][sel].contiguous()
            s_pairs = res.transition_pairs[:n][sel].contiguous()
            cnt = int(s_src.numel())
            per = (2 if kind == "in_place" else 4) * dim * 2 * layers * heads
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(steps)]
            for a0, a1 in [(None, None)] * 2 + evs:
                if a0 is not None:
                    a0.record(stream)
                reposition_kv_layers(k_ptrs, v_ptrs, k_pools[0], v_pools[0], s_src, s_dst,
                                     s_pairs, cache, bulk_copy_v=bulk)
                if a1 is not None:
                    a1.record(stream)
            torch.cuda.synchronize()
            k_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
            split[kind] = {"transitions": cnt, "ms": round(k_ms, 4),
                           "algorithmic_bytes": cnt * per,
                           "achieved": round(cnt * per / (k_ms / 1e3) / 1e9, 1),
                           "frac": round(cnt * per / (k_ms / 1e3) / 1e9 / peak, 4)}
            if ref is not None and world == 1 and cnt and kind != "copy_on_write_one_pass":
                split[kind]["triton_reference"] = triton_versus_ours(
                    ref, k_ptrs, v_ptrs, k_pools[0], v_pools[0], s_src, s_dst, s_pairs, cache,
                    3, stream, cnt * per)
        # e2e through the public API from host memory: validate + pack + one
        # H2D copy + launches, and the decode view read back every step.  As
        # in a serving loop (and the c2 e2e), the host issues step i + 1
        # before it waits for the read-back of step i (two pinned buffers).
        n_view = 2 * kept + 2 * prog.requests + 6  # the layout of DropResult.read_view
        views = [torch.empty(n_view, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]
        dist_barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(e2e_steps):
            rtt.copy_(rtt0)
            ring.state.copy_(state0)
            r2 = comp.run(prog.token_counts, prog.range_offsets, prog.ranges, rtt, row_ids, ring,
                          shared_prefix=prog.shared_prefix, page_size=ps)
            reposition_kv_layers(k_ptrs, v_ptrs, k_pools[0], v_pools[0], r2.transition_source,
                                 r2.transition_destination, r2.transition_pairs, cache,
                                 count_device=r2.transition_count, page_size=ps,
                                 bulk_copy_v=bulk_v)
            r2.read_view(views[i % 2])
            read[i % 2].record(stream)
            if i > 0:
                read[(i - 1) % 2].synchronize()
                if int(views[(i - 1) % 2][-1]) != 0:
                    raise RuntimeError("drop_compact status in the c3 e2e loop")
        e1.record(stream)
        e1.synchronize()
        if int(views[(e2e_steps - 1) % 2][-1]) != 0:
            raise RuntimeError("drop_compact status in the c3 e2e loop")
        e2e_s = dist_max(e0.elapsed_time(e1) / 1e3, world)
        step_bytes = (rep_bytes + drop_bytes) * world
        achieved = rep_bytes / (rep_ms / 1e3) / 1e9
        sec = {
            "metric": METRIC, "value": round(step_bytes / (ms / 1e3) / 1e9, 2), "unit": UNIT,
            "ms_per_step": round(ms, 4), "n_gpus": world, "scaling": "strong",
            "config": {"workload": f"c3 page_size {ps}", "requests": prog.requests,
                       "tokens": total, "shared_prefix": int(prog.shared_prefix.max()),
                       "layers": layers, "kv_heads": heads_total, "kv_heads_per_gpu": heads,
                       "head_dim": dim, "page_size": ps, "rope": "yarn",
                       "bulk_copy_v": bool(bulk_v),
                       "moved_tokens": n, "cow_transitions": n_cow,
                       "in_place_transitions": n - n_cow,
                       ("copied_pages" if ps > 1 else "copied_slots"): copied,
                       ("freed_pages" if ps > 1 else "freed_slots"): freed,
                       "l2": "K pools 49 GB, larger than L2; no flush",
                       "restore": "rows + ring head restored on the device each step"},
            "e2e": {"value": round(step_bytes * e2e_steps / e2e_s / 1e9, 2), "unit": UNIT,
                    "h2d_bytes_per_step": prepared["h2d_bytes"],
                    "d2h_bytes_per_step": 4 * n_view},
            "breakdown_ms": {"drop_compact": round(drop_ms, 4), "reposition": round(rep_ms, 4)},
            "reposition_by_kind": split,
            "roofline": {"bound": "hbm", "kernel": "reposition_kernel",
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": rep_bytes,
                         "ms_per_launch": round(rep_ms, 4),
                         "traffic": ncu_traffic("c3", rep_bytes) if world == 1 else None,
                         "traffic_source": "profiles/reposition_c3.md (4-request cut, "
                                           "traffic / algorithmic ratio)"},
            "gpu_launches_per_step": 5,
            "clocks": clock_info,
        }
        if cpu and rank == 0 and world == 1:
            sec["cpu_baseline"] = cpu_reference_c3(prog, rows, layers, heads, dim,
                                                   cache.cpu().numpy(), rep_bytes + drop_bytes)
        out[ps] = sec
    del k_pools, v_pools
    torch.cuda.empty_cache()
    return out


def bench_c5(dev, world, rank, warmup, steps, requests=8, layers=80, budget_gb=96.0, seed=0):
    """c5, the scaling configuration at its stated size: Llama-3-70B-shaped
    cache (80 layers, 8 KV heads split 8/N per rank as SGLang TP does,
    head_dim 128, bf16), 8 requests of 131072 tokens, 30 % dropped in 20
    seed-placed spans each, plain RoPE theta 500000; every moved token is
    private and rotates in place.  The full cache (344 GB) does not fit one
    GPU or two: when this rank's share exceeds ``budget_gb``, as many layers
    as fit are resident and each step runs the 80 layers as consecutive
    launches over those resident layers (chunks of the pointer table), the
    same bytes and the same per-launch shape as 80 resident layers.  At 4
    and 8 GPUs all 80 layers are resident (one launch).  Every rank computes
    the same drop metadata (three launches) and no collective runs."""
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor, FreeSlotRing
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers
    from akv_b200.rope import rope_cos_sin_cache

    heads_total, dim = 8, 128
    heads = heads_total // world
    prog = workloads.c5_program(seed=seed, requests=requests)
    rows, nslots = workloads.slot_rows(np.random.default_rng(seed), prog)
    total, kept, moved = plan_stats(prog)
    per_layer = nslots * heads * dim * 2 * 2  # K and V
    resident = max(1, min(layers, int(budget_gb * 1e9 // per_layer)))
    chunks = [min(resident, layers - c) for c in range(0, layers, resident)]
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    k_pools = [torch.randn(nslots, heads, dim, device=dev, generator=g, dtype=torch.bfloat16)
               for _ in range(resident)]
    v_pools = [torch.empty(nslots, heads, dim, device=dev, dtype=torch.bfloat16)
               for _ in range(resident)]
    k_ptrs, v_ptrs = layer_pointer_table(k_pools), layer_pointer_table(v_pools)
    cache = rope_cos_sin_cache(131072, dim, 500000.0).to(dev)
    table = np.zeros((prog.requests + 1, int(prog.token_counts.max())), np.int32)
    for r in range(prog.requests):
        table[r + 1, : len(rows[r])] = rows[r]
    rtt = torch.from_numpy(table).to(dev)
    row_ids = np.arange(1, prog.requests + 1)
    freed = total - kept
    ring = FreeSlotRing(torch.zeros(0, dtype=torch.int32),
                        capacity=freed * (warmup + 2 * steps + 4) + 16, device=dev)
    comp = DropCompactor(total, prog.requests, max(1, len(prog.ranges) // 2), dev)
    prepared = comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges, row_ids)
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(chunks) + 1)]
          for _ in range(steps)]

    def step(i=None):
        res = comp.launch(prepared, rtt, ring)
        if i is not None:
            ev[i][0].record(stream)
        for c, n in enumerate(chunks):
            reposition_kv_layers(k_ptrs[:n], v_ptrs[:n], k_pools[0], v_pools[0],
                                 res.transition_source, res.transition_destination,
                                 res.transition_pairs, cache, count_device=res.transition_count)
            if i is not None:
                ev[i][c + 1].record(stream)
        return res

    for _ in range(warmup):
        res = step()
    torch.cuda.synchronize()
    res.check()
    assert int(res.totals[1].item()) == moved
    dist_barrier(world)
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = dist_max(t0.elapsed_time(t1) / steps, world)
    dist_barrier(world)
    for i in range(steps):
        step(i)
    torch.cuda.synchronize()
    launch_ms = statistics.mean(e[c].elapsed_time(e[c + 1]) for e in ev
                                for c in range(len(chunks)))
    rep_ms = statistics.mean(e[0].elapsed_time(e[-1]) for e in ev)  # all launches of a step
    rep_bytes = moved * layers * heads * 2 * dim * 2
    drop_bytes = total + 4 * total + 8 * kept + 4 * (total - kept) + 12 * moved
    per_launch = moved * chunks[0] * heads * 2 * dim * 2
    peak, peak_kind = measured_peak()
    achieved = rep_bytes / (rep_ms / 1e3) / 1e9
    achieved_max = dist_max(achieved, world)
    achieved_min = -dist_max(-achieved, world)
    del k_pools, v_pools
    torch.cuda.empty_cache()
    return {
        "metric": METRIC, "value": round((rep_bytes + drop_bytes) * world / (ms / 1e3) / 1e9, 2),
        "unit": UNIT, "ms_per_step": round(ms, 4), "n_gpus": world, "scaling": "strong",
        "config": {"workload": "c5", "requests": prog.requests, "tokens": total,
                   "moved_tokens": moved, "layers": layers, "kv_heads": heads_total,
                   "kv_heads_per_gpu": heads, "head_dim": dim, "rope": "rope500000",
                   "resident_layers": resident, "launches_per_step": len(chunks),
                   "reposition": "in place", "parallelism": f"kv-head tp{world}",
                   "l2": f"resident K pools {resident * nslots * heads * dim * 2 / 1e9:.0f} GB "
                         "per GPU, larger than L2; no flush"},
        "roofline": {"bound": "hbm", "kernel": "reposition_kernel",
                     "achieved": round(achieved_min, 1), "achieved_max_rank": round(achieved_max, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved_min / peak, 4),
                     "peak_source": peak_kind, "algorithmic_bytes_per_launch": per_launch,
                     "ms_per_launch": round(launch_ms, 4),
                     "traffic": ncu_traffic("c5", per_launch),
                     "traffic_source": "profiles/reposition_c5.md (one-request, 10-layer cut, "
                                       "traffic / algorithmic ratio)",
                     "reposition_ms_per_step": round(rep_ms, 4), "per": "GPU (slowest rank)"},
        "gpu_launches_per_step": 3 + len(chunks),
        "clocks": clock_info,
    }


def cpu_reference_c3(prog, rows, layers, heads, dim, cache_np, step_bytes, sample=2000):
    """The reference's CPU path for one c3 step, on the host cores: its C++
    event compiler (oracle/_ref) over every request + the numpy decode view,
    and the CPU restatement of its reposition kernel (the reference has no
    CPU reposition; it copies every moved token, so the restatement moves
    K and V of a sample of the transitions, copy-on-write ones included)
    scaled to all transitions.  The reference has no paged Reposition, so
    both page sizes are measured against this page_size 1 path."""
    from oracle import oracle, reference

    threads = len(os.sched_getaffinity(0))
    comp = reference.compile_context_layout if reference.available() else oracle.compile_layout
    t0 = time.perf_counter()
    trans = []
    for r in range(prog.requests):
        t = int(prog.token_counts[r])
        rr = prog.request_ranges(r)
        lay = comp(np.zeros(t, np.int32), [t], [0, len(rr) // 2], rr, [t - 1], [t])
        raw = np.flatnonzero(lay["keep_mask"]).astype(np.int32)
        _ = lay["positions"][raw]
        trans.append(np.stack((lay["transition_old_positions"],
                               lay["transition_new_positions"]), 1))
    t_drop = time.perf_counter() - t0
    pairs = np.concatenate(trans).astype(np.int32)
    n = len(pairs)
    rng = np.random.default_rng(0)
    m = min(sample, n)
    pick = rng.choice(n, size=m, replace=False)
    k = [np.random.default_rng(l).integers(0, 1 << 16, size=(2 * m, heads, dim),
                                           dtype=np.uint16) & 0x7F7F for l in range(layers)]
    v = [np.zeros((2 * m, heads, dim), np.uint16) for _ in range(layers)]
    src = np.arange(m, dtype=np.int32)
    t1 = time.perf_counter()
    oracle.reposition(k, v, src, src + m, pairs[pick], cache_np, bf16=True, threads=threads)
    t_rep = (time.perf_counter() - t1) * n / m
    sec = t_drop + t_rep
    kind = "reference" if reference.available() else "port"
    return {"value": round(step_bytes / sec / 1e9, 3), "unit": UNIT, "cores": threads,
            "kind": kind,
            "sample": f"event compiler ({'reference C++' if kind == 'reference' else 'port'}) "
                      f"over all {prog.requests} requests ({t_drop * 1e3:.1f} ms) + reposition "
                      f"restatement (port) moving K and V of {m} of {n} transitions x {layers} "
                      f"layers x {heads} heads, scaled to all {n} ({t_rep * 1e3:.1f} ms)"}


def measured_tensor_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def bench_prefill(dev, world, rank, warmup, steps, seed=0, layers=36, variant=0, head_dim=64,
                  compare=False):
    """c4p: prefill of a new agent turn over the compacted cache -- 16
    requests, each a compacted prefix (lognormal length, median 8192, with
    position holes from dropped tokens) plus 1,024 new tokens; GPT-OSS-120B
    shape (64 query / 8 KV heads split 8/N per rank, head_dim 64), sinks,
    36 layers alternating sliding window 128 and full attention.  Tensor
    bound: FLOPs = 4 * head_dim per visible (query, key, query head).
    ``compare``: also time the reference's runtime context prefill
    (its native plan + FlashInfer ragged prefill + sink correction) on one
    full and one sliding-window layer, outside the timed step."""
    from akv_b200 import workloads
    from akv_b200.context_prefill import ContextPrefillAttention

    bs, new, hq_total, hkv_total, d, window = 16, 1024, 64, 8, head_dim, 128
    hkv, hq = hkv_total // world, hq_total // world
    rng = np.random.default_rng(seed)
    prefix = workloads.c4_lengths(seed=seed, batch=bs)
    qo = np.concatenate(([0], np.cumsum([new] * bs))).astype(np.int64)
    kv = np.concatenate(([0], np.cumsum(prefix))).astype(np.int64)
    kpos, qpos = [], []
    for p in prefix:
        pp = np.cumsum(rng.integers(1, 3, size=int(p))) - 1  # about a third dropped
        kpos.append(pp)
        qpos.append((pp[-1] if len(pp) else -1) + 1 + np.arange(new))
    kpos = np.concatenate(kpos).astype(np.int32)
    qpos = np.concatenate(qpos).astype(np.int32)
    n_keys = int(kv[-1] + qo[-1])
    perm = torch.from_numpy(rng.permutation(n_keys).astype(np.int32)).to(dev)
    kv_idx, births = perm[: kv[-1]], perm[kv[-1]:]
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    pools = [(torch.randn(n_keys, hkv, d, device=dev, generator=g, dtype=torch.bfloat16),
              torch.randn(n_keys, hkv, d, device=dev, generator=g, dtype=torch.bfloat16))
             for _ in range(2)]
    q = torch.randn(int(qo[-1]), hq, d, device=dev, generator=g, dtype=torch.bfloat16)
    sinks = torch.randn(hq, device=dev, generator=g)
    t_qpos = torch.from_numpy(qpos).to(dev)
    t_kpos = torch.from_numpy(kpos).to(dev)
    full = ContextPrefillAttention(hq, hkv, d, dev).plan(qo, kv, qpos, kpos, window=-1)
    swa = ContextPrefillAttention(hq, hkv, d, dev).plan(qo, kv, qpos, kpos, window=window)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)

    def layer(i):
        kp, vp = pools[i % 2]
        (full if i % 2 else swa).run(q, kp, vp, kv_idx, births, t_qpos, t_kpos, sinks=sinks,
                                     out=out, variant=variant)

    for _ in range(warmup):
        for i in range(layers):
            layer(i)
    torch.cuda.synchronize()
    dist_barrier(world)
    ev_full = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for s in range(steps):
        for i in range(layers):
            if i == 1:
                ev_full[s][0].record(stream)
            layer(i)
            if i == 1:
                ev_full[s][1].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    for att in (full, swa):
        att.check()
    ms = dist_max(t0.elapsed_time(t1) / steps, world)
    full_ms = statistics.median(a.elapsed_time(b) for a, b in ev_full)
    full_flops = 4.0 * d * hq * full.visible
    step_flops = (layers // 2) * 4.0 * d * hq * (full.visible + swa.visible) * world
    peak, peak_kind = measured_tensor_peak()
    achieved = full_flops / (full_ms / 1e3) / 1e12
    bf16_p = None
    if variant == 0 and layers >= 2:
        # The same full layer with P rounded to bf16 for P.V (variant 5, or 6
        # at head_dim 128): FlashInfer's precision, one P.V MMA per key block.
        fv = 6 if d == 128 else 5
        kp, vp = pools[1]
        fast_ms = time_launches(
            lambda: full.run(q, kp, vp, kv_idx, births, t_qpos, t_kpos, sinks=sinks, out=out,
                             variant=fv), max(steps, 3), stream)
        full.check()
        fast = full_flops / (fast_ms / 1e3) / 1e12
        bf16_p = {"variant": fv, "p_in_pv": "bf16 (FlashInfer's precision; default: hi + lo)",
                  "ms_per_launch": round(fast_ms, 4), "achieved": round(fast, 1),
                  "unit": "TFLOP/s", "frac": round(fast / peak, 4)}
    runtime_ref = None
    if compare and layers >= 2:
        # The reference's runtime context prefill on one sliding-window and
        # one full layer (outside the timed step).
        runtime_ref = {}
        for name, i, att, win in (("full_layer", 1, full, -1),
                                  ("sliding_window_layer", 0, swa, window)):
            kp, vp = pools[i % 2]
            runtime_ref[name] = flashinfer_prefill_versus_ours(
                att, q, kp, vp, kv_idx, births, qo, kv, qpos, kpos, win, sinks, out,
                max(steps, 3), stream, lambda i=i: layer(i))
    cpu = None
    if rank == 0 and world == 1:
        # Torch fp32 on the host cores over a bounded sample (the reference
        # has no CPU path for this kernel): one request, 64 of its queries,
        # full attention; scaled to the full layer by visible pairs.
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        kq = q[:64].float().cpu()
        slots = torch.cat((kv_idx[: kv[1]], births[:64])).long()
        kk = pools[1][0][slots].float().cpu().repeat_interleave(8, dim=1)
        vv = pools[1][1][slots].float().cpu().repeat_interleave(8, dim=1)
        n_p = int(kv[1])
        vis = (torch.arange(n_p + 64)[None, :] < n_p) | \
            (torch.arange(n_p + 64)[None, :] - n_p <= torch.arange(64)[:, None])
        t_cpu = time.perf_counter()
        sc = torch.einsum("qhd,khd->hqk", kq, kk) / np.sqrt(d)
        sc = sc.masked_fill(~vis[None], float("-inf"))
        torch.einsum("hqk,khd->qhd", torch.softmax(sc, dim=2), vv)
        sec = time.perf_counter() - t_cpu
        pairs = int(vis.sum())
        cpu = {"value": round(4.0 * d * hq * pairs / sec / 1e12, 4), "unit": "TFLOP/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"torch fp32 CPU, request 0, 64 of its queries x {n_p + 64} keys, "
                         f"full attention, all {hq} heads"}
    del pools
    torch.cuda.empty_cache()
    return {
        "metric": "context prefill attention new tokens/s",
        "value": round(int(qo[-1]) / (ms / 1e3), 1), "unit": "tokens/s",
        "ms_per_step": round(ms, 4), "n_gpus": world,
        "tflops": round(step_flops / (ms / 1e3) / 1e12, 1),
        "config": {"workload": "c4p", "kernel_variant": variant, "requests": bs,
                   "new_tokens_per_request": new,
                   "prefix_keys": int(kv[-1]), "q_heads": hq_total, "kv_heads": hkv_total,
                   "head_dim": d, "layers": layers, "sliding_window": window, "sinks": True,
                   "positions": "prefix with holes (about a third dropped)"},
        "roofline": {"bound": "tensor",
                     "kernel": {1: "prefill_attention_kernel", 2: "prefill_attention_tc_kernel",
                                4: "prefill_attention_tc_ws_kernel, two query tiles",
                                5: "prefill_attention_tc_ws_kernel, bf16 P",
                                6: "prefill_attention_tc_ws_kernel, two query tiles, bf16 P"}
                     .get(variant, "prefill_attention_tc_ws_kernel") + " (full layer)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "algorithmic_flops_per_launch": full_flops,
                     "ms_per_launch": round(full_ms, 4)},
        "gpu_launches_per_step": layers,
        "cpu_baseline": cpu,
        "bf16_p_form": bf16_p,
        "reference_runtime_prefill": runtime_ref,
    }


def bench_active_slots(dev, world, rank, warmup, steps, seed=0, copies=12):
    """PD offload / transfer gather (context_transfer.py:110-128): the active
    slots of 64 requests (c3 lengths, 1.13M prompt tokens, about 70 % kept,
    128 generated tokens each) in one ``ActiveSlotGather`` launch.  ``copies``
    independent batches (rows, raw indices, outputs: about 12 MB each, 140 MB
    together, more than L2) are gathered in turn.  The per-request call the
    reference makes (``active_slots``, one launch each) is timed beside it.
    Bytes per slot: 4 B raw index + 4 B row slot read + 4 B written."""
    from akv_b200 import workloads
    from akv_b200.context_transfer import ActiveSlotGather, active_slots

    prog = workloads.c3_program()
    rng = np.random.default_rng(seed)
    base = []
    total = 0
    for T in prog.token_counts:
        T = int(T)
        raw = np.flatnonzero(rng.random(T) < 0.7).astype(np.int32)
        row = rng.permutation(4 * (T + 128))[: T + 128].astype(np.int32)
        base.append((row, raw, T, T + 128))
        total += len(raw) + 128
    sets = []
    for c in range(copies):
        reqs = [(torch.from_numpy(row).to(dev), torch.from_numpy(raw).to(dev), g, e)
                for row, raw, g, e in base]
        gather = ActiveSlotGather(dev).plan([r[0] for r in reqs], [r[1] for r in reqs],
                                            [0] * len(reqs), [r[2] for r in reqs],
                                            [r[3] for r in reqs])
        sets.append((reqs, gather, torch.empty(gather.total, dtype=torch.int32, device=dev)))
    reqs = sets[0][0]
    outs = [torch.empty(len(r[1]) + 128, dtype=torch.int32, device=dev) for r in reqs]
    stream = torch.cuda.current_stream(dev)
    turn = [0]

    def batched():
        _, gather, packed = sets[turn[0] % copies]
        turn[0] += 1
        gather.run(out=packed)

    def per_request():
        for (row, idx, gen0, end), out in zip(reqs, outs):
            active_slots(row, idx, 0, gen0, end, out=out)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize()
        return dist_max(t0.elapsed_time(t1) / steps, world)

    # One call enqueues in ~10 us of host time, about as long as the kernel
    # runs: the batched launches are timed from a captured graph of `steps`
    # consecutive launches (cycling through the copies), so the device time
    # is what is measured.
    for _ in range(copies):
        batched()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            batched()
    graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    graph.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    ms = dist_max(t0.elapsed_time(t1) / steps, world)
    del graph
    ms_eager = timed(batched)
    ms_per_request = timed(per_request)
    del sets
    peak, peak_kind = measured_peak()
    gbs = 12.0 * total / (ms / 1e3) / 1e9
    return {
        "metric": "active-slot gather slots/s", "value": round(total / (ms / 1e3), 1),
        "unit": "slots/s", "ms_per_step": round(ms, 4), "n_gpus": world, "scaling": "replicas",
        "config": {"workload": "c3 offload", "requests": len(reqs), "slots": total,
                   "launches_per_step": 1,
                   "l2": f"{copies} independent batches gathered in turn (more than L2)"},
        "roofline": {"bound": "hbm", "kernel": "active_slots_batch_kernel",
                     "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": 12 * total},
        "eager_call_ms": round(ms_eager, 4),
        "per_request_launches_ms": round(ms_per_request, 4),
        "gpu_launches_per_step": 1,
    }


def bench_occurrence(dev, world, rank, warmup, steps, seed=0, requests=16, prefix=9000,
                     queries=1024, copies=600):
    """Occurrence binding of one prefill forward (the device part of
    OccurrenceState.advance, srt/context_system/occurrence.py:644-755, and
    the scheduler's concatenation, sglang.patch:3133-3180), c4p shape:
    ``requests`` requests, each with ``prefix`` slots of earlier chunks,
    ``queries`` new query slots and ``copies`` extra slots for repositioned
    copies.  Per request: occurrence slots (all rows, mostly in order),
    copy sources and destinations, retained and retired slots, copy position
    pairs.  The index arrays are synthetic with those sizes (the ownership
    decisions that produce them are scheduler CPU work, the same in both
    arms).  Timed: this build's one copy + one launch (host packing
    included), the kernel alone (graph replay over prepacked programs), and
    the reference's per-request torch sequence (concatenation, one pageable
    copy, gathers, int32 casts, then four batch concatenations).  Bytes per
    output: 4 B index + 8 B slot read + 8 B written (4 B for int32 fields)."""
    from akv_b200 import _native
    from akv_b200.context_occurrence import SlotGather

    rng = np.random.default_rng(seed)
    stream = torch.cuda.current_stream(dev)
    reqs = []
    for _ in range(requests):
        old = torch.from_numpy(rng.permutation(40 * prefix)[:prefix]).to(dev)
        q = torch.from_numpy(rng.permutation(40 * queries)[:queries]).to(dev)
        e = torch.from_numpy(rng.permutation(40 * copies)[:copies]).to(dev)
        total = prefix + queries + copies
        occ = np.arange(total)
        swap = rng.random(total) < 0.1
        occ[swap] = rng.integers(0, total, int(swap.sum()))
        src = rng.integers(0, prefix, copies)
        dst = np.arange(prefix + queries, total)
        keep = np.sort(rng.choice(total, total - copies, replace=False))
        release = np.setdiff1d(np.arange(total), keep)
        pairs = rng.integers(0, 10**5, 2 * copies)
        # int32 row vectors, as the host derivation of advance returns them
        reqs.append(dict(seg=(old, q, e), occ=occ.astype(np.int32), src=src.astype(np.int32),
                         dst=dst.astype(np.int32), keep=keep.astype(np.int32),
                         release=release.astype(np.int32), pairs=pairs.astype(np.int32)))
    n_slots = sum(len(r["occ"]) for r in reqs)
    n_copy = requests * copies
    out_slots = torch.empty(n_slots, dtype=torch.int64, device=dev)
    i32 = torch.empty(4 * n_copy, dtype=torch.int32, device=dev)
    succ = [torch.empty(len(r["keep"]), dtype=torch.int64, device=dev) for r in reqs]
    retired = [torch.empty(len(r["release"]), dtype=torch.int64, device=dev) for r in reqs]

    occ_sizes = [len(r["occ"]) for r in reqs]

    def queue():
        # the tasks OccurrenceBatch queues per request (its internal
        # _add_fields / _add: per-request views of batch buffers it
        # allocated, indices that fit int32 by construction)
        g = SlotGather(dev)
        v_slots = out_slots.split_with_sizes(occ_sizes)
        v_src, v_dst, v_pairs = (i32[:n_copy].split(copies), i32[n_copy:2 * n_copy].split(copies),
                                 i32[2 * n_copy:].split(2 * copies))
        for j, r in enumerate(reqs):
            g._add_fields([(v_slots[j], r["occ"]), (v_src[j], r["src"]), (v_dst[j], r["dst"]),
                           (succ[j], r["keep"]), (retired[j], r["release"])], r["seg"])
            g._add(v_pairs[j], r["pairs"], literal=True)
        return g

    def ours():
        queue().launch()

    def reference_sequence():
        slots, sources, dests, positions = [], [], [], []
        for r in reqs:
            all_slots = torch.cat(r["seg"])
            fields = (r["occ"], r["src"], r["dst"], r["keep"], r["release"], r["pairs"])
            offsets = np.r_[0, np.cumsum([len(f) for f in fields])]
            packed = torch.from_numpy(np.concatenate(fields).astype(np.int64)).to(
                dev, non_blocking=True)
            o, sr, ds, kp, rl, pr = (packed[a:b] for a, b in zip(offsets[:-1], offsets[1:]))
            slots.append(all_slots[o])
            sources.append(all_slots[sr].to(torch.int32))
            dests.append(all_slots[ds].to(torch.int32))
            all_slots[kp], all_slots[rl]  # noqa: B018 - successor slots, retired slots
            positions.append(pr.reshape(-1, 2).to(torch.int32))
        torch.cat(slots), torch.cat(sources), torch.cat(dests), torch.cat(positions)  # noqa: B018

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            fn()
        t1.record(stream)
        torch.cuda.synchronize()
        return dist_max(t0.elapsed_time(t1) / steps, world)

    ms_ours = timed(ours)
    ms_ref = timed(reference_sequence)
    # kernel alone: the packed program resident on the device, graph replay
    words, n_tasks, n_chunks = queue().pack()
    prog = torch.from_numpy(words).to(dev)
    base = prog.data_ptr()

    def kernel():
        st = _native.lib.akv_gather_slots(base, base + 96 * n_tasks, n_chunks,
                                          base + 8 * (12 * n_tasks + n_chunks), None,
                                          _native.stream_of(dev))
        assert st == 0

    kernel()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            kernel()
    graph.replay()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    graph.replay()
    t1.record(stream)
    torch.cuda.synchronize()
    ms_kernel = dist_max(t0.elapsed_time(t1) / steps, world)
    del graph
    n_out64 = n_slots + sum(len(r["keep"]) + len(r["release"]) for r in reqs)
    gathered32 = 2 * n_copy
    alg = 20 * n_out64 + 16 * gathered32 + 8 * 2 * n_copy
    peak, peak_kind = measured_peak()
    gbs = alg / (ms_kernel / 1e3) / 1e9
    return {
        "metric": "occurrence binding ms per forward", "value": round(ms_ours, 4),
        "unit": "ms", "higher_is_better": False, "n_gpus": world, "scaling": "replicas",
        "config": {"workload": "c4p forward", "requests": requests, "prefix_slots": prefix,
                   "query_slots": queries, "copies": copies, "occurrence_slots": n_slots,
                   "index_data": "synthetic, sizes of the c4p forward"},
        "reference_torch_sequence_ms": round(ms_ref, 4),
        "kernel_ms": round(ms_kernel, 4),
        "roofline": {"bound": "hbm", "kernel": "gather_slots_kernel", "achieved": round(gbs, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "peak_source": peak_kind, "algorithmic_bytes_per_launch": alg},
        "gpu_launches_per_step": 1,
        "reference_launches_per_step": requests * 10 + 4,
    }


def bench_decode_metadata(dev, world, rank, warmup, steps, seed=0, generated=4):
    """Per-step decode metadata of the c4 batch (ContextDecodeRegistry.fill /
    fill_window, srt/layers/attention/context_backend.py:754-809): 128
    requests with lognormal prompt lengths (median 8K, max 64K), about 70 %
    of each prompt kept (a sorted random decode view at compact positions),
    ``generated`` generated tokens each; every step builds the full-attention
    metadata and the sliding-window (128) metadata, two launches each
    (``build_decode_metadata``).  Bytes per key: 4 B decode-view raw index
    + 4 B req_to_token slot read + 4 B kv_indices written (generated keys
    have no raw-index read).  Registry rows, decode views and the table
    are synthetic with those shapes."""
    from akv_b200 import workloads
    from akv_b200.context_page_table import build_decode_metadata

    rng = np.random.default_rng(seed)
    lengths = workloads.c4_lengths(seed=seed)
    batch = len(lengths)
    max_ctx = int(lengths.max()) + generated
    table = torch.from_numpy(rng.integers(1, 1 << 24, size=(batch, max_ctx)).astype(
        np.int32)).to(dev)
    registry = torch.zeros((batch, 6), dtype=torch.int64, device=dev)
    keep, seq, prefix_keys = [], [], 0
    for b, t in enumerate(lengths.tolist()):
        raw = np.flatnonzero(rng.random(t) < 0.7).astype(np.int32)
        if len(raw) == 0:
            raw = np.zeros(1, np.int32)
        packed = torch.from_numpy(np.concatenate((raw, np.arange(len(raw), dtype=np.int32))))
        packed = packed.to(dev)
        keep.append(packed)
        registry[b] = torch.tensor([packed.data_ptr(), packed.data_ptr() + 4 * len(raw), t,
                                    len(raw), len(raw), 0], dtype=torch.int64)
        seq.append(len(raw) + generated)
        prefix_keys += len(raw)
    rows = torch.arange(batch, dtype=torch.int64, device=dev)
    seq_lens = torch.tensor(seq, dtype=torch.int64, device=dev)
    n_full = int(sum(seq))
    kv_indptr = torch.empty(batch + 1, dtype=torch.int32, device=dev)
    kv_indices = torch.empty(n_full, dtype=torch.int32, device=dev)
    w_indptr = torch.empty(batch + 1, dtype=torch.int32, device=dev)
    w_indices = torch.empty(batch * 128, dtype=torch.int32, device=dev)
    w_len = torch.empty(batch, dtype=torch.int64, device=dev)
    w_start = torch.empty(batch, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        build_decode_metadata(registry, table, rows, seq_lens, kv_indptr, kv_indices)
        build_decode_metadata(registry, table, rows, seq_lens, w_indptr, w_indices, window=128,
                              lengths_out=w_len, starts_out=w_start)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    assert int(kv_indptr[-1].item()) == n_full

    def timed(run):
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        run()
        t1.record(stream)
        torch.cuda.synchronize()
        return dist_max(t0.elapsed_time(t1) / steps, world)

    # Two Python calls a step enqueue in about as long as the kernels run, so
    # the device time comes from a captured graph of `steps` steps; the eager
    # loop (host enqueue included) is reported beside it.
    ms_eager = timed(lambda: [step() for _ in range(steps)])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            step()
    graph.replay()
    torch.cuda.synchronize()
    ms = timed(graph.replay)
    del graph
    n_window = int(w_len.sum().item())
    alg = 12 * prefix_keys + 8 * (n_full - prefix_keys) + 12 * n_window
    # The reference's Triton page-table kernels on the same registry, as its
    # ContextDecodeRegistry drives them (context_backend.py:754-809): full
    # indices over the cumulative lengths; window lengths, their cumsum and
    # starts, then window indices.  Checked equal to ours, then timed the
    # same way (graph of `steps` steps).
    triton_ref = None
    ref = reference_triton()
    if ref is not None:
        pt = ref["page_table"]
        r_indptr = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
        r_indices = torch.empty_like(kv_indices)
        r_wlen = torch.empty_like(seq_lens)
        r_windptr = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
        r_windices = torch.empty_like(w_indices)

        def ref_step():
            r_indptr[1:] = seq_lens.cumsum(0)
            pt.context_decode_indices[(batch,)](
                registry, table, rows, seq_lens, r_indptr, r_indices, None, None,
                ROW_STRIDE=table.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=False)
            pt.context_window_lengths[(batch,)](registry, rows, seq_lens, r_wlen, 128)
            r_windptr[1:] = r_wlen.cumsum(0)
            starts = seq_lens - r_wlen
            pt.context_decode_indices[(batch,)](
                registry, table, rows, r_wlen, r_windptr, r_windices, starts, None,
                ROW_STRIDE=table.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=True)

        for _ in range(warmup):
            ref_step()
        torch.cuda.synchronize()
        same = (torch.equal(r_indptr, kv_indptr) and torch.equal(r_indices, kv_indices) and
                torch.equal(r_wlen, w_len) and torch.equal(r_windptr, w_indptr) and
                torch.equal(r_windices[:n_window], w_indices[:n_window]))
        ref_eager = timed(lambda: [ref_step() for _ in range(steps)])
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(steps):
                ref_step()
        graph.replay()
        torch.cuda.synchronize()
        ref_ms = timed(graph.replay)
        del graph
        # Kernel by kernel: the reference's Triton launch and this package's
        # drop-in launcher of the same name, same arguments, graph-captured.
        from akv_b200 import context_page_table as ours_pt

        w_starts = (seq_lens - r_wlen).contiguous()
        o_wlen = torch.empty_like(seq_lens)
        o_idx = torch.empty_like(kv_indices)
        per_kernel = {}
        for name, theirs, mine in (
            ("context_window_lengths",
             lambda: pt.context_window_lengths[(batch,)](registry, rows, seq_lens, r_wlen, 128),
             lambda: ours_pt.context_window_lengths[(batch,)](registry, rows, seq_lens, o_wlen,
                                                              128)),
            ("context_decode_indices",
             lambda: pt.context_decode_indices[(batch,)](
                 registry, table, rows, seq_lens, r_indptr, r_indices, None, None,
                 ROW_STRIDE=table.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=False),
             lambda: ours_pt.context_decode_indices[(batch,)](
                 registry, table, rows, seq_lens, r_indptr, o_idx, None, None,
                 ROW_STRIDE=table.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=False)),
        ):
            times = []
            for fn in (theirs, mine):
                fn()
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(steps):
                        fn()
                g.replay()
                torch.cuda.synchronize()
                times.append(timed(g.replay))
                del g
            torch.cuda.synchronize()
            equal = torch.equal(o_wlen, r_wlen) if name == "context_window_lengths" else \
                torch.equal(o_idx, r_indices)
            per_kernel[name] = {"triton_us": round(1e3 * times[0], 2),
                                "ours_us": round(1e3 * times[1], 2),
                                "speedup": round(times[0] / times[1], 2),
                                "outputs_equal": bool(equal)}
        del w_starts
        triton_ref = {"triton_ms_per_step": round(ref_ms, 4),
                      "triton_eager_ms_per_step": round(ref_eager, 4),
                      "ours_ms_per_step": round(ms, 4), "speedup": round(ref_ms / ms, 2),
                      "outputs_equal": bool(same),
                      "what": "context_decode_indices (full) + context_window_lengths + "
                              "context_decode_indices (window 128) with the registry's "
                              "cumsum / starts, graph-captured like ours",
                      "per_kernel": per_kernel}
    peak, peak_kind = measured_peak()
    gbs = alg / (ms / 1e3) / 1e9
    return {
        "metric": "decode metadata keys/s", "value": round((n_full + n_window) / (ms / 1e3), 1),
        "unit": "keys/s", "ms_per_step": round(ms, 4), "n_gpus": world, "scaling": "replicas",
        "config": {"workload": "c4 decode metadata", "requests": batch, "full_keys": n_full,
                   "window_keys": n_window, "launches_per_step": 4},
        "roofline": {"bound": "hbm", "kernel": "decode_indices_kernel + decode_lengths_scan",
                     "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_source": peak_kind,
                     "algorithmic_bytes_per_step": alg},
        "eager_ms_per_step": round(ms_eager, 4),
        "gpu_launches_per_step": 4,
        "triton_reference": triton_ref,
    }


def bench_compiler(dev, world, rank, warmup, steps, seed=0):
    """c3m: the general event compiler over 64 multi-turn agent programs
    (c3 request lengths, 8 turns each: a Drop event then a Reposition at the
    end of every turn; 1.13M tokens at seed 0).  The program is the same on
    every rank (scheduler state is replicated per TP rank), so this is a
    replica measurement.  Device: the four launches on resident inputs.
    e2e: host programs -> packing -> H2D -> launches -> D2H of the
    per-request status and the totals.  CPU: the reference's C++ compiler
    (oracle/_ref), request by request on one thread as its scheduler runs
    it."""
    from akv_b200 import workloads
    from akv_b200.context_plan import LayoutCompiler, Program

    progs = [Program.of(*p) for p in workloads.agent_turn_programs(seed=seed)]
    tokens = sum(len(p.token_ids) for p in progs)
    comp = LayoutCompiler(dev, max_tokens=tokens, max_requests=len(progs),
                          max_events=sum(len(p.drop_insert_offsets) for p in progs),
                          max_ranges=sum(len(p.drop_ranges) // 2 for p in progs),
                          max_repositions=sum(len(p.reposition_raw_boundaries) for p in progs),
                          transition_capacity=4 * tokens)
    stream = torch.cuda.current_stream(dev)
    prepared = comp.prepare(progs)
    for _ in range(warmup):
        comp.launch(prepared)
    torch.cuda.synchronize()
    totals = comp.totals.cpu().tolist()
    if totals[3]:
        raise RuntimeError(f"event compiler benchmark: status bits {totals[3]}")
    dist_barrier(world)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for a, b in ev:
        a.record(stream)
        comp.launch(prepared)
        b.record(stream)
    torch.cuda.synchronize()
    dev_ms = dist_max(statistics.median(a.elapsed_time(b) for a, b in ev), world)
    # End to end through the public API, one step after another.
    status_host = torch.empty_like(comp.status, device="cpu").pin_memory()
    totals_host = torch.empty(4, dtype=torch.int64).pin_memory()
    e2e = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        comp.compile(progs)
        status_host.copy_(comp.status, non_blocking=True)
        totals_host.copy_(comp.totals, non_blocking=True)
        b.record(stream)
        b.synchronize()
        e2e.append(a.elapsed_time(b))
    e2e_ms = dist_max(statistics.median(e2e), world)
    h2d = prepared[1]["h2d_bytes"]
    d2h = status_host.numel() * 8 + 32
    transitions, kept = int(totals[0]), int(totals[1])
    # Algorithmic bytes: ids in; per token 4+1+4+4+4+8 (positions, keep, stage, birth
    # position and stage, token_to_key) + 12+1+8 (record, virtual flag, key_to_token)
    # out; 8 per kept token (decode view); 12 per transition.
    alg = tokens * (8 + 25 + 21) + kept * 8 + transitions * 12
    peak, peak_kind = measured_peak()
    cpu = None
    if rank == 0 and world == 1:
        from oracle import oracle, reference

        comp_fn = reference.compile_context_layout if reference.available() else \
            oracle.compile_layout
        t0 = time.perf_counter()
        for p in progs:
            comp_fn(p.token_ids, p.drop_insert_offsets, p.drop_range_offsets, p.drop_ranges,
                    p.reposition_raw_boundaries, p.reposition_raw_boundaries.astype(np.int64) + 1)
        sec = time.perf_counter() - t0
        cpu = {"value": round(tokens / sec, 1), "unit": "tokens/s", "cores": 1,
               "kind": "reference" if reference.available() else "port",
               "sample": f"all {len(progs)} programs ({tokens} tokens), compile_context_layout "
                         f"count + compile passes, one request at a time"}
    return {
        "metric": "event compiler tokens/s", "value": round(tokens * world / (dev_ms / 1e3), 1),
        "unit": "tokens/s", "ms_per_step": round(dev_ms, 4), "n_gpus": world,
        "scaling": "replicas",
        "config": {"workload": "c3m", "requests": len(progs), "tokens": tokens, "turns": 8,
                   "transitions": transitions, "kept": kept},
        "e2e": {"value": round(tokens * world / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "layout_* (4 launches)",
                     "achieved": round(alg / (dev_ms / 1e3) / 1e9, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(alg / (dev_ms / 1e3) / 1e9 / peak, 4),
                     "peak_source": peak_kind, "algorithmic_bytes_per_launch": alg},
        "gpu_launches_per_step": 4,
        "cpu_baseline": cpu,
    }


def main():
    args = parse_args()
    if args.workload == "c4p" and args.impl == "ours":
        # Prefill attention alone.
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = bench_prefill(dev, world, rank, max(3, min(args.warmup, 5)),
                            max(3, min(args.steps, 20)), layers=args.layers or 36,
                            variant=args.variant, head_dim=args.head_dim,
                            compare=world == 1)
        if rank == 0:
            emit(res)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.workload == "c3m" and args.impl == "ours":
        # The event compiler alone.
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = bench_compiler(dev, world, rank, max(3, args.warmup), max(3, min(args.steps, 50)))
        if rank == 0:
            emit(res)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.workload in ("c4m", "c3g") and args.impl == "ours":
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        fn = bench_decode_metadata if args.workload == "c4m" else bench_active_slots
        res = fn(dev, world, rank, max(3, args.warmup), max(3, min(args.steps, 50)))
        if rank == 0:
            emit(res)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.workload == "c4o" and args.impl == "ours":
        # Occurrence binding of one forward alone.
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = bench_occurrence(dev, world, rank, max(3, args.warmup), max(3, min(args.steps, 50)))
        if rank == 0:
            emit(res)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.workload == "c4" and args.impl == "ours":
        # Decode attention alone (for profiling cuts: --layers 2).
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = bench_attention(dev, world, rank, max(3, args.warmup), max(3, args.steps // 20),
                              layers=args.layers or 36, shard=args.shard,
                              layout=args.slot_layout, compare=world == 1)
        if rank == 0:
            emit(res)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.workload == "c5" and args.impl == "ours":
        # The scaling configuration alone, at its stated size (--requests for
        # a smaller cut).
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = bench_c5(dev, world, rank, max(2, args.warmup), max(3, min(args.steps, 30)),
                       requests=args.requests or 8, layers=args.layers or 80)
        if rank == 0:
            emit(res)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.workload == "c3" and args.impl == "ours":
        # The batched copy-on-write step alone (--page-size 1 or 16; --layers
        # for a smaller cut under a profiler).
        world, rank, local = dist_setup()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = bench_c3(dev, world, rank, max(3, args.warmup), max(3, min(args.steps, 50)),
                       page_sizes=(args.page_size,), layers=args.layers or 36, cpu=False,
                       requests=args.requests or 64, shard=args.shard)
        if rank == 0:
            emit(res[args.page_size])
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

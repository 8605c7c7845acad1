"""Benchmark of the attention hot path (decode, Llama-3.1-8B shapes, 8K context).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = the attention block of one decode token through all 32 layers at
position 8191 of an 8192-entry fp32 KV cache: per layer, the device-side
append of the token's K/V row and the decode attention (q.K^T, softmax, .V)
over all 8192 positions, one fused kernel launch
per layer (l3p_attn_step_dev).  Per step the KV traffic
is 32 x 64 MiB = 2 GiB, far larger than the 126 MB L2, so no step reuses
another's cache lines.

Printed on rank 0 as one JSON line:
  value      fp32-equivalent KV bytes read per second (GB/s), whole job,
             inputs resident in HBM, device time (CUDA events, max over ranks)
  e2e        the same metric through the host-pointer C ABI (l3p_attn_step
             per layer: pinned host q/k/v in, host output back, per step)
  roofline   the decode kernel: algorithmic bytes per launch / average launch
             time over the timed region (every launch in it is this kernel),
             against MEASURED_PEAKS.json's HBM copy bandwidth; the same kernel
             timed in isolation (launches without overlap) beside it
  exchange   (N > 1) the head-sharded block's exchange per layer: the
             tensor-parallel wo sum over NVLink, timed inside the step
  configs    BASELINE configs[0], [2], [3] at this GPU count (us/layer,
             tokens/s, fraction of HBM per GPU); prefill = configs[4] with the
             heads sharded over the ranks
  parity     every multi-GPU data path (KV-head shards, sequence parts merged
             over NVLink and over NCCL, the tensor-parallel wo sum) on seeded
             inputs against the CPU oracle, outside the timed regions; a
             mismatch makes the run exit 1
  cpu_baseline  the reference's own CPU attention (oracle/_ref, compiled from
             llama3pure-c-engine.c with its OpenMP flags) on a bounded sample
Multi-GPU (torchrun): each rank owns n_kv/N KV heads (head sharding, no
collective on the data path); value = all ranks' bytes / max-rank time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from llama3pure_b200.synth import CONFIGS, decode_inputs  # noqa: E402

WORKLOAD = "llama31_8b_decode_8k"
# dram__bytes_read.sum + dram__bytes_write.sum of one decode launch on this
# workload (67.18 MB + 0.59 MB), from the ncu capture summarised in
# profiles/decode_f32_kernel_llama31_8b_8k.md; --traffic overrides it
NCU_TRAFFIC_PER_LAUNCH = 67.77e6
METRIC = "decode-attn KV GB/s (fp32-equivalent), Llama-3.1-8B shapes, ctx 8K, 32 layers, append+decode per layer"


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# --------------------------------------------------------------------------
# clocks


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------
# reference / CPU baseline


class CpuReference:
    """The reference's own decode attention (Q8_0 cache as shipped, OpenMP
    over KV heads as at llama3pure-c-engine.c:3327-3328) on `layers` layers of
    the workload, each timed call = append row pos + attend, per layer.
    fast: True = the harness built -march=x86-64-v3, "v4" = -march=x86-64-v4."""

    def __init__(self, layers: int = 2, fast=True):
        O = oracle_module()
        self.kind = "reference" if O.ref_available(fast=fast) else "port"
        self.impl = "ref" if self.kind == "reference" else "port"
        self.fast = fast if self.kind == "reference" else True
        self.sh = sh = CONFIGS[WORKLOAD]
        self.layers = layers
        self.o = O.Oracle(sh, O.MODE_Q8, self.impl, fast=self.fast, n_layers=layers)
        self.rows = []
        for layer in range(layers):
            k, v, q = decode_inputs(sh, layer)
            self.o.load_kv(layer, 0, k[:, : sh.pos], v[:, : sh.pos])
            self.rows.append((q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos])))
            del k, v
        self.omp_threads = O.threads(self.impl, fast=self.fast)
        self.threads = min(self.omp_threads, sh.n_kv_heads)
        self.bytes_per_layer = 2 * (sh.pos + 1) * sh.n_kv_heads * sh.head_dim * 4
        self.o.decode(0, sh.pos, *self.rows[0])  # warm

    def step(self) -> float:
        t0 = time.perf_counter()
        for layer in range(self.layers):
            self.o.decode(layer, self.sh.pos, *self.rows[layer])
        return time.perf_counter() - t0

    def describe(self, reps: int, seconds: float) -> str:
        return (f"{self.layers} of 32 layers x {reps} steps of {WORKLOAD} decode at pos {self.sh.pos} "
                f"(Q8_0 cache as shipped, append+attend per layer), {seconds:.1f} s of CPU time")

    def close(self):
        self.o.close()


def oracle_module():
    """The CPU oracle / reference harness (test infrastructure): bench.py runs
    it only as the timed CPU baseline and as the parity leg's checker."""
    p = os.path.join(ROOT, "oracle")
    if p not in sys.path:
        sys.path.insert(0, p)
    import oracle as O

    return O


BUILD_FLAGS = {True: "-Ofast -fopenmp -march=x86-64-v3", "v4": "-Ofast -fopenmp -march=x86-64-v4"}


def pick_reference_build():
    """The reference harness build to time on this host: x86-64-v3, or
    x86-64-v4 (AVX-512) when the CPU has it and it is faster on a 4-layer
    sample.  (The reference's own flag is -march=native, Makefile:33; the
    harness is compiled where the reference source is, not on this host.)
    Returns (fast, {build: GB/s on the sample})."""
    O = oracle_module()
    cands = [True] + (["v4"] if O.ref_available("v4") and O.cpu_has_v4() else [])
    if not O.ref_available(True) or len(cands) == 1:
        return True, {}
    gbs = {}
    for c in cands:
        r = CpuReference(layers=4, fast=c)
        t = min(r.step() for _ in range(3))
        gbs[c] = r.bytes_per_layer * r.layers / t / 1e9
        r.close()
    best = max(gbs, key=gbs.get)
    return best, {BUILD_FLAGS[c]: round(v, 2) for c, v in gbs.items()}


def cpu_facts(ref: CpuReference, sample_gbs: dict) -> dict:
    O = oracle_module()
    return {"host_cpus": os.cpu_count(), "cpu_model": O.cpu_model(), "omp_threads": ref.omp_threads,
            "threads_used": ref.threads,
            "threads_note": "the reference parallelises decode attention over KV heads only "
                            "(llama3pure-c-engine.c:3327-3328): at most n_kv_heads = 8 threads work",
            "build": BUILD_FLAGS.get(ref.fast, "-Ofast -fopenmp -march=x86-64-v3") +
                     (" (reference harness, llama3pure-c-engine.c compiled in place)" if ref.kind == "reference"
                      else " (restated port)"),
            "builds_sampled_gbs": sample_gbs}


def cpu_baseline(min_seconds: float = 10.0):
    host_threads_for_reference()
    fast, sampled = pick_reference_build()
    ref = CpuReference(layers=CONFIGS[WORKLOAD].n_layers, fast=fast)
    dts = []
    while sum(dts) < min_seconds or len(dts) < 3:
        dts.append(ref.step())
    gbs = ref.bytes_per_layer * ref.layers * len(dts) / sum(dts) / 1e9
    out = {"value": round(gbs, 3), "unit": "GB/s", "cores": ref.threads, "kind": ref.kind,
           "sample": ref.describe(len(dts), sum(dts)), **cpu_facts(ref, sampled)}
    ref.close()
    return out


def host_threads_for_reference() -> None:
    """torchrun sets OMP_NUM_THREADS=1 in every rank; the reference arm runs
    on rank 0 alone and must use the host's cores (OpenMP reads the variable
    when the reference library first loads, which happens after this)."""
    if os.environ.get("OMP_NUM_THREADS") in (None, "1"):
        os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    host_threads_for_reference()
    fast, sampled = pick_reference_build()
    ref = CpuReference(layers=CONFIGS[WORKLOAD].n_layers, fast=fast)
    for _ in range(args.warmup):
        ref.step()
    dts = [ref.step() for _ in range(args.steps)]
    value = ref.bytes_per_layer * ref.layers * len(dts) / sum(dts) / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.median(dts) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 (Q8_0) + f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "layers_per_step": ref.layers, "pos": ref.sh.pos,
                   "note": "every step is the full 32-layer workload"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": ref.threads, "kind": ref.kind,
                         "sample": ref.describe(len(dts), sum(dts)), **cpu_facts(ref, sampled)},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    ref.close()
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------
# our arm


class DevView:
    """A raw device range seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class Job:
    """The job's ranks: torch, the process group (or None) and timing helpers."""

    def __init__(self, torch, dist, world: int, rank: int, local: int):
        self.torch, self.dist, self.world, self.rank, self.local = torch, dist, world, rank, local

    def max(self, *vals):
        if self.world == 1:
            return list(vals)
        t = self.torch.tensor(list(vals), device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.tolist()

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def graph(self, fn):
        """CUDA graph of fn(stream), captured on a side stream."""
        torch = self.torch
        g = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(cs):
            with torch.cuda.graph(g, stream=cs):
                fn(cs)
        torch.cuda.current_stream().wait_stream(cs)
        return g

    def time_graph(self, g, reps: int, warmup: int = 3) -> float:
        """ms per replay, max over ranks (ranks start together after a barrier)."""
        torch = self.torch
        s = torch.cuda.current_stream()
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        for _ in range(reps):
            g.replay()
        b.record(s)
        torch.cuda.synchronize()
        return self.max(a.elapsed_time(b) / reps)[0]

    def fill_cache(self, ctx, n_layers: int, heads: int, rows: int, hd: int, seed: int, k_scale: float = 1.0,
                   n_rows: int | None = None):
        """N(0,1) rows [0, n_rows) of every owned cache row block, on the device."""
        torch = self.torch
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        for layer in range(n_layers):
            kp, vp = ctx.kv_device_ptr(layer)
            kt = torch.as_tensor(DevView(kp, (heads, rows, hd)), device="cuda")
            vt = torch.as_tensor(DevView(vp, (heads, rows, hd)), device="cuda")
            kt[:, : n_rows or rows].normal_(generator=g)
            if k_scale != 1.0:
                kt.mul_(k_scale)
            vt[:, : n_rows or rows].normal_(generator=g)
        return g


def _peak():
    import json

    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p.get("bf16_tflops", 0.0)), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _decode_record(us_per_layer: float, L: int, bytes_per_layer_job: float, bytes_per_layer_rank: float,
                   world: int, peak: float):
    return {"us_per_layer": round(us_per_layer, 3), "tokens_per_s": round(1e6 / (us_per_layer * L), 1),
            "job_gbs": round(bytes_per_layer_job / us_per_layer / 1e3, 1),
            "frac_of_hbm_per_gpu": round(bytes_per_layer_rank / us_per_layer / 1e3 / peak, 4)}


# --------------------------------------------------------------------------
# Llama-3.2-1B shapes, 16 layers, 1024 positions, head_dim 64


def config1(job: Job, reps: int):
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.shard import plan_shards
    from llama3pure_b200.synth import CONFIGS

    torch = job.torch
    sh = CONFIGS["llama32_1b_decode"]
    L, P, hd = sh.n_layers, sh.pos + 1, sh.head_dim
    me = plan_shards(sh.n_kv_heads, sh.seq_len, job.world, 1)[job.rank]
    hk = me.kv_head_count
    peak, _, pk = _peak()
    res = {"workload": sh.name, "n_layers": L, "kv_positions": P, "head_dim": hd,
           "parallelism": f"kv-head shards x{job.world} ({hk} KV heads per GPU)", "peak_kind": pk}
    with AttnContext.for_shape(sh, device=job.local, kv_head_begin=me.kv_head_begin, kv_head_count=hk) as ctx:
        g = job.fill_cache(ctx, L, hk, sh.seq_len, hd, 3000 + job.rank)
        q = torch.randn((L, sh.n_heads * hd), device="cuda", generator=g)
        kn = torch.randn((L, sh.n_kv_heads * hd), device="cuda", generator=g)
        vn = torch.randn((L, sh.n_kv_heads * hd), device="cuda", generator=g)
        out = torch.zeros_like(q)
        ctx.set_overlap(True)
        n0 = ctx.launch_count()
        gs = job.graph(lambda s: [ctx.step_dev(l, sh.pos, q[l], kn[l], vn[l], out[l], s) for l in range(L)])
        step_launches = ctx.launch_count() - n0
        gd = job.graph(lambda s: [ctx.decode_dev(l, sh.pos, q[l], out[l], s) for l in range(L)])
        n0 = ctx.launch_count()
        gb = job.graph(lambda s: ctx.decode_layers_dev(0, L, sh.pos, q, out, s))
        batched_launches = ctx.launch_count() - n0
        step_ms = job.time_graph(gs, reps)
        dec_ms = job.time_graph(gd, reps)
        bat_ms = job.time_graph(gb, reps)
        ctx.check()
        plan = ctx.decode_plan(sh.pos)
        del gs, gd, gb
    rank_b = 2 * P * hk * hd * 4
    job_b = rank_b * job.world
    res["per_call_step"] = {"api": "l3p_attn_step_dev per layer (append + decode), graph + programmatic "
                                   "dependent launch", "launches_per_layer": step_launches // L,
                            **_decode_record(step_ms * 1e3 / L, L, job_b, rank_b, job.world, peak)}
    res["per_call_decode"] = {"api": "l3p_attn_decode_dev per layer, graph + programmatic dependent launch",
                              **_decode_record(dec_ms * 1e3 / L, L, job_b, rank_b, job.world, peak)}
    res["layer_batched"] = {"api": "l3p_attn_decode_layers_dev: all 16 layers in one launch",
                            "launches_per_step": batched_launches,
                            **_decode_record(bat_ms * 1e3 / L, L, job_b, rank_b, job.world, peak)}
    res["split_k"] = {"ctas_per_kv_head": plan[0], "cluster": plan[1]}
    res["bytes_per_layer"] = job_b
    return res


# --------------------------------------------------------------------------
# 131072 cached positions, 1 GiB of K+V per layer, 32 layers


def config3(job: Job, reps: int, seq_parts_list=(1, 2)):
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.shard import plan_shards
    from llama3pure_b200.synth import CONFIGS

    torch = job.torch
    sh = CONFIGS["llama31_8b_decode_128k"]
    L, P, hd = sh.n_layers, sh.pos + 1, sh.head_dim
    peak, _, pk = _peak()
    job_b = 2 * P * sh.n_kv_heads * hd * 4
    res = {"workload": sh.name, "n_layers": L, "kv_positions": P, "bytes_per_layer": job_b, "peak_kind": pk,
           "decompositions": []}
    for sp in seq_parts_list:
        if job.world % sp or sh.n_kv_heads % (job.world // sp) or (sp > 1 and job.world < 2):
            continue
        me = plan_shards(sh.n_kv_heads, sh.seq_len, job.world, sp)[job.rank]
        g0 = me.head_group * sp
        with AttnContext.for_shape(sh, device=job.local, kv_head_begin=me.kv_head_begin,
                                   kv_head_count=me.kv_head_count, seq_begin=me.seq_begin,
                                   seq_count=me.seq_count) as ctx:
            g = job.fill_cache(ctx, L, me.kv_head_count, me.seq_count, hd, 4000 + job.rank, k_scale=sh.k_scale)
            q = torch.randn((L, sh.n_heads * hd), device="cuda", generator=g)
            out = torch.zeros_like(q)
            if sp > 1:
                h = ctx.seq_group_export(sp, me.seq_part)
                hs = [None] * job.world
                job.dist.all_gather_object(hs, h)
                ctx.seq_group_import(hs[g0:g0 + sp])
            # programmatic dependent launch only with the merge kernel between
            # the decodes: back to back, 1 GiB launches measured ~9 us per
            # layer slower with it (158.5 vs 167.7 us on one B200)
            ctx.set_overlap(sp > 1)
            if sp > 1:
                gr = job.graph(lambda s: [ctx.decode_seq_dev(l, sh.pos, q[l], out[l], s) for l in range(L)])
            else:
                gr = job.graph(lambda s: [ctx.decode_dev(l, sh.pos, q[l], out[l], s) for l in range(L)])
            ms = job.time_graph(gr, reps)
            ctx.check()
            del gr
            rank_b = 2 * me.seq_count * me.kv_head_count * hd * 4
        rec = {"head_groups": job.world // sp, "seq_parts": sp,
               "exchange": "none" if sp == 1 else "partial triples read from the peers over NVLink in the merge "
                                                  "kernel (l3p_attn_decode_seq_dev)",
               **_decode_record(ms * 1e3 / L, L, job_b, rank_b, job.world, peak)}
        res["decompositions"].append(rec)
    best = min(res["decompositions"], key=lambda r: r["us_per_layer"])
    res["best"] = {k: best[k] for k in ("head_groups", "seq_parts", "us_per_layer", "tokens_per_s",
                                        "frac_of_hbm_per_gpu")}
    return res


# --------------------------------------------------------------------------
# Gemma-2B shapes, 18 layers, 8 q heads, 1 KV head, head_dim 256


def config4(job: Job, reps: int):
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.synth import CONFIGS

    torch = job.torch
    sh = CONFIGS["gemma_2b_decode"]
    L, P, hd = sh.n_layers, sh.pos + 1, sh.head_dim
    W = job.world
    b, e = sh.seq_len * job.rank // W, sh.seq_len * (job.rank + 1) // W
    peak, _, pk = _peak()
    res = {"workload": sh.name, "n_layers": L, "kv_positions": P, "head_dim": hd, "peak_kind": pk,
           "parallelism": "one GPU" if W == 1 else f"{W} sequence parts of the single KV head over NVLink "
                                                   "(l3p_attn_decode_seq_dev)"}
    with AttnContext.for_shape(sh, device=job.local, seq_begin=b, seq_count=e - b) as ctx:
        g = job.fill_cache(ctx, L, 1, e - b, hd, 5000 + job.rank)
        q = torch.randn((L, sh.n_heads * hd), device="cuda", generator=g)
        kn = torch.randn((L, hd), device="cuda", generator=g)
        vn = torch.randn((L, hd), device="cuda", generator=g)
        out = torch.zeros_like(q)
        if W > 1:
            h = ctx.seq_group_export(W, job.rank)
            hs = [None] * W
            job.dist.all_gather_object(hs, h)
            ctx.seq_group_import(hs)
        ctx.set_overlap(True)
        if W > 1:
            gd = job.graph(lambda s: [ctx.decode_seq_dev(l, sh.pos, q[l], out[l], s) for l in range(L)])
            gs = None
        else:
            gd = job.graph(lambda s: [ctx.decode_dev(l, sh.pos, q[l], out[l], s) for l in range(L)])
            gs = job.graph(lambda s: [ctx.step_dev(l, sh.pos, q[l], kn[l], vn[l], out[l], s) for l in range(L)])
        dec_ms = job.time_graph(gd, reps)
        step_ms = job.time_graph(gs, reps) if gs is not None else None
        ctx.check()
        del gd, gs
    job_b = 2 * P * hd * 4
    rank_b = 2 * (e - b) * hd * 4
    res["decode"] = {"api": "l3p_attn_decode_dev" if W == 1 else "l3p_attn_decode_seq_dev",
                     **_decode_record(dec_ms * 1e3 / L, L, job_b, rank_b, W, peak)}
    if step_ms is not None:
        res["step"] = {"api": "l3p_attn_step_dev (append + decode)",
                       **_decode_record(step_ms * 1e3 / L, L, job_b, rank_b, W, peak)}
    res["bytes_per_layer"] = job_b
    return res


# --------------------------------------------------------------------------
# causal prefill, 2048 tokens, heads sharded by KV-head group


def measure_tf32_peak(torch):
    """Dense TF32 tensor throughput of this GPU, measured live: an fp32
    torch.matmul (cuBLAS) with TF32 enabled, 8192^3, best of 5 (2*N^3 flops).
    The 3xTF32 prefill roofline is a third of it."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn((n, n), device="cuda")
    b = torch.randn((n, n), device="cuda")
    c = a @ b
    best = 1e9
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        c = a @ b
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b, c
    return 2 * n ** 3 / (best / 1e3) / 1e12


def config5(job: Job, reps: int, raw: bool = True):
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.shard import plan_shards
    from llama3pure_b200.synth import CONFIGS, prefill_flops

    torch = job.torch
    sh = CONFIGS["llama31_8b_prefill_2k"]
    S, hd = sh.pos + 1, sh.head_dim
    L = 4  # layers cycled (16 MiB of K/V each)
    me = plan_shards(sh.n_kv_heads, sh.seq_len, job.world, 1)[job.rank]
    with AttnContext.for_shape(sh, n_layers=L, device=job.local, kv_head_begin=me.kv_head_begin,
                               kv_head_count=me.kv_head_count) as ctx:
        g = torch.Generator(device="cuda")
        g.manual_seed(6000 + job.rank)
        q = torch.randn((L, S, sh.n_heads, hd), device="cuda", generator=g)
        k = torch.randn((L, S, sh.n_kv_heads, hd), device="cuda", generator=g)
        v = torch.randn((L, S, sh.n_kv_heads, hd), device="cuda", generator=g)
        out = torch.zeros_like(q)
        s = torch.cuda.current_stream()

        def timed(fn):
            for i in range(3):
                fn(i % L)
            torch.cuda.synchronize()
            job.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for i in range(reps):
                fn(i % L)
            e1.record(s)
            torch.cuda.synchronize()
            return job.max(e0.elapsed_time(e1) / reps)[0]

        n0 = ctx.launch_count()
        ctx.prefill_dev(0, 0, S, q[0], k[0], v[0], out[0], s)
        launches = ctx.launch_count() - n0
        ms = timed(lambda i: ctx.prefill_dev(i, 0, S, q[i], k[i], v[i], out[i], s))
        raw_ms = None
        if raw:
            ctx.set_rope()
            raw_ms = timed(lambda i: ctx.prefill_raw_dev(i, 0, S, q[i], k[i], v[i], out[i], s))
        ctx.check()
    flops = prefill_flops(sh)
    tflops = flops / (ms / 1e3) / 1e12
    tf32 = measure_tf32_peak(torch)
    _, bf16, _ = _peak()
    res = {"workload": sh.name, "tokens": S, "head_dim": hd, "ms_per_layer": round(ms, 4),
           "tflops": round(tflops, 2), "flops_per_layer": flops, "launches_per_layer": launches,
           "parallelism": f"kv-head shards x{job.world} ({me.kv_head_count} KV heads, "
                          f"{me.kv_head_count * sh.kv_mul} q heads per GPU)",
           "kernel": "prefill_tc_kernel (tcgen05 3xTF32) + prefill_prep_kernel + kv_append_kernel",
           "tf32_dense_tflops_measured": round(tf32, 1),
           "tf32_how": "torch.matmul fp32 with allow_tf32 (cuBLAS), 8192^3, best of 5, this GPU, this run",
           "roofline_3xtf32_tflops_per_gpu": round(tf32 / 3, 1),
           "frac_of_3xtf32_per_gpu": round(tflops / job.world / (tf32 / 3), 4)}
    if bf16 > 0:
        # TF32 dense peak taken as half the driver-measured bf16 burst peak
        res["frac_of_3xtf32_from_half_bf16_per_gpu"] = round(tflops / job.world / (bf16 / 2 / 3), 4)
    if raw_ms is not None:
        res["raw_ms_per_layer"] = round(raw_ms, 4)
        res["raw_api"] = "l3p_attn_prefill_raw_dev (RoPE + cache write, then prep + attention)"
    res["tokens_per_s_32_layers"] = round(S / (ms * 32 / 1e3), 1)
    return res


def prefill_other_head_dims(job: Job, reps: int, tf32: float):
    """Causal prefill of 2048 tokens at the other two head sizes on one GPU:
    Llama-3.2-1B shapes (head_dim 64, the tcgen05 kernel) and Gemma-2B shapes
    (head_dim 256, MQA: the decode kernel in token mode, one grid slice per
    token -- Q hi and O alone would fill the tensor memory at head_dim 256)."""
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.synth import CONFIGS, prefill_flops

    torch = job.torch
    res = {}
    for name, base, path in (("llama32_1b_hd64", CONFIGS["llama32_1b_decode"], "prefill_tc_kernel<1,64> (tcgen05 3xTF32)"),
                             ("gemma_2b_hd256", CONFIGS["gemma_2b_decode"],
                              "decode_f32_kernel<256,8> in token mode (FFMA, fp32)")):
        sh = base.with_(seq_len=2048, pos=2047, n_layers=2)
        S, hd = 2048, sh.head_dim
        with AttnContext.for_shape(sh, device=job.local) as ctx:
            g = torch.Generator(device="cuda")
            g.manual_seed(7000)
            L = 2
            q = torch.randn((L, S, sh.n_heads, hd), device="cuda", generator=g)
            k = torch.randn((L, S, sh.n_kv_heads, hd), device="cuda", generator=g)
            v = torch.randn((L, S, sh.n_kv_heads, hd), device="cuda", generator=g)
            out = torch.zeros_like(q)
            s = torch.cuda.current_stream()
            for i in range(3):
                ctx.prefill_dev(i % L, 0, S, q[i % L], k[i % L], v[i % L], out[i % L], s)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for i in range(reps):
                ctx.prefill_dev(i % L, 0, S, q[i % L], k[i % L], v[i % L], out[i % L], s)
            e1.record(s)
            torch.cuda.synchronize()
            ctx.check()
            ms = e0.elapsed_time(e1) / reps
        flops = prefill_flops(sh)
        tflops = flops / (ms / 1e3) / 1e12
        res[name] = {"shape": f"{sh.n_heads} q heads / {sh.n_kv_heads} KV heads, head_dim {hd}, 2048 tokens",
                     "path": path, "ms_per_layer": round(ms, 4), "tflops": round(tflops, 2), "flops_per_layer": flops,
                     "frac_of_3xtf32": round(tflops / (tf32 / 3), 4)}
    # the FFMA path's own ceiling: fp32 FMA issue of every SM at the clock the GPU reports
    props = torch.cuda.get_device_properties(job.local)
    clock_ghz = getattr(props, "clock_rate", 0) / 1e6 or 1.965
    ffma = props.multi_processor_count * 128 * 2 * clock_ghz / 1e3
    res["gemma_2b_hd256"]["frac_of_ffma_peak"] = round(res["gemma_2b_hd256"]["tflops"] / ffma, 4)
    res["ffma_peak_tflops"] = round(ffma, 1)
    res["ffma_peak_how"] = "SMs x 128 fp32 FMA lanes x 2 flop x the SM clock the device reports"
    return res


# --------------------------------------------------------------------------
# parity leg: seeded inputs (BASELINE generator) through every multi-GPU path


def _cmp(got, want):
    from llama3pure_b200.synth import tolerance_ok

    ok, ma, mr = tolerance_ok(got, want)
    return {"ok": ok, "max_abs": float(f"{ma:.3e}"), "max_rel": float(f"{mr:.3e}")}


def _worst(recs):
    """One record for several compared outputs (all ranks, repeated calls)."""
    return {"ok": all(r["ok"] for r in recs), "max_abs": max(r["max_abs"] for r in recs),
            "max_rel": max(r["max_rel"] for r in recs), "outputs_compared": len(recs)}


def parity_leg(job: Job):
    """Returns {path: {ok, max_abs, max_rel, ...}} on rank 0 (None elsewhere)."""
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.shard import plan_shards
    from llama3pure_b200.synth import CONFIGS, decode_inputs, wo_input, wo_weights

    torch, dist, W, rank = job.torch, job.dist, job.world, job.rank
    O = oracle_module() if rank == 0 else None
    res = {}

    def gather(arr):
        """Every rank's numpy array, on rank 0."""
        if W == 1:
            return [arr]
        out = [None] * W
        dist.all_gather_object(out, arr)
        return out if rank == 0 else None

    # KV-head shards: configs[1] layer 0 (seed 1), append of row 8191 + decode,
    # through the host C ABI (l3p_attn_step) on every rank; rows concatenated
    sh = CONFIGS["llama31_8b_decode_8k"]
    k, v, q = decode_inputs(sh, 0)
    me = plan_shards(sh.n_kv_heads, sh.seq_len, W, 1)[rank]
    with AttnContext.for_shape(sh, n_layers=1, device=job.local, kv_head_begin=me.kv_head_begin,
                               kv_head_count=me.kv_head_count) as ctx:
        ctx.load_kv(0, 0, np.ascontiguousarray(k[:, : sh.pos]), np.ascontiguousarray(v[:, : sh.pos]))
        out = ctx.step(0, sh.pos, q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos]))
        r0, r1 = ctx.owned_rows
    parts = gather((r0, r1, out[r0:r1].copy()))
    if rank == 0:
        full = np.full((sh.n_heads, sh.head_dim), np.nan, np.float32)
        for a, b, rows in parts:
            full[a:b] = rows
        o = O.Oracle(sh, O.MODE_F32, "port", n_layers=1)
        o.load_kv(0, 0, k, v)
        want, _ = o.decode(0, sh.pos, q)
        o.close()
        res["kv_head_shards"] = {"workload": sh.name + " layer 0 (append + decode, l3p_attn_step)",
                                 "ranks": W, **_cmp(full, want.reshape(full.shape))}
    del k, v

    # sequence parts of one KV head: configs[3] layer 0 (seed 3) split over the ranks
    gs = CONFIGS["gemma_2b_decode"]
    k, v, q = decode_inputs(gs, 0)
    want = None
    if rank == 0:
        o = O.Oracle(gs, O.MODE_F32, "port", n_layers=1)
        o.load_kv(0, 0, k, v)
        want, _ = o.decode(0, gs.pos, q)
        o.close()
        want = want.reshape(gs.n_heads, gs.head_dim)
    if W > 1:
        b, e = gs.seq_len * rank // W, gs.seq_len * (rank + 1) // W
        with AttnContext.for_shape(gs, n_layers=1, device=job.local, seq_begin=b, seq_count=e - b) as ctx:
            ctx.load_kv(0, b, np.ascontiguousarray(k[:, b:e]), np.ascontiguousarray(v[:, b:e]))
            dq = torch.from_numpy(q.reshape(-1).copy()).cuda()
            # over NVLink peer memory, three steps (device step counter, slot reuse)
            h = ctx.seq_group_export(W, rank)
            hs = [None] * W
            dist.all_gather_object(hs, h)
            ctx.seq_group_import(hs)
            outs = []
            for _ in range(3):
                dout = torch.zeros_like(dq)
                ctx.decode_seq_dev(0, gs.pos, dq, dout)
                outs.append(dout)
            ctx.check()
            nv = [o_.cpu().numpy().reshape(gs.n_heads, gs.head_dim) for o_ in outs]
            # NCCL all-gather of the partial triples + the LSE merge kernel
            po = torch.zeros(gs.n_heads * gs.head_dim, device="cuda")
            pml = torch.zeros(gs.n_heads * 2, device="cuda")
            ctx.decode_partial_dev(0, gs.pos, dq, po, pml)
            go = torch.zeros((W, po.numel()), device="cuda")
            gml = torch.zeros((W, pml.numel()), device="cuda")
            dist.all_gather_into_tensor(go, po)
            dist.all_gather_into_tensor(gml, pml)
            mout = torch.zeros_like(dq)
            ctx.lse_merge_dev(W, gs.n_heads, 0, gs.n_heads, go, gml, mout)
            ctx.check()
            nc = mout.cpu().numpy().reshape(gs.n_heads, gs.head_dim)
        all_nv, all_nc = gather(nv), gather(nc)
        if rank == 0:
            res["seq_parts_nvlink_merge"] = {
                "workload": gs.name + f" layer 0, {W} sequence parts (l3p_attn_decode_seq_dev, 3 steps)",
                **_worst([_cmp(x, want) for outs_r in all_nv for x in outs_r])}
            res["seq_parts_nccl_lse_merge"] = {
                "workload": gs.name + f" layer 0, {W} sequence parts (decode_partial_dev + NCCL all-gather + "
                                      "lse_merge_dev)",
                **_worst([_cmp(x, want) for x in all_nc])}
    else:
        with AttnContext.for_shape(gs, n_layers=1, device=job.local) as ctx:
            ctx.load_kv(0, 0, k, v)
            got = ctx.decode(0, gs.pos, q)
        res["gemma_mqa_decode"] = {"workload": gs.name + " layer 0 (one GPU)", **_cmp(got, want)}
    del k, v

    # the wo projection: 4096 x 4096 (Llama-3.1-8B), every GGUF weight type; at N > 1
    # the tensor-parallel sum over NVLink on every rank, two steps
    dim = cols = sh.n_heads * sh.head_dim
    x = wo_input(cols, seed=7)
    for name, wt in (("q8_0", 8), ("q2_k", 10), ("q3_k", 11), ("q4_k", 12), ("q5_k", 13), ("q6_k", 14), ("q4_0", 2),
                     ("q4_1", 3), ("q5_0", 6), ("q5_1", 7), ("iq4_nl", 20), ("f32", 0), ("f16", 1), ("bf16", 29)):
        w = wo_weights(wt, dim, cols, seed=6)
        with AttnContext.for_shape(sh, n_layers=1, seq_len=16, device=job.local, kv_head_begin=me.kv_head_begin,
                                   kv_head_count=me.kv_head_count) as ctx:
            ctx.set_wo(0, wt, w)
            dx = torch.from_numpy(x).cuda()
            outs = []
            if W > 1:
                h = ctx.tp_group_export(W, rank, dim)
                hs = [None] * W
                dist.all_gather_object(hs, h)
                ctx.tp_group_import(hs)
                for _ in range(2):
                    y = torch.zeros(dim, device="cuda")
                    ctx.wo_allreduce_dev(0, dx, y)
                    outs.append(y)
            else:
                y = torch.zeros(dim, device="cuda")
                ctx.wo_dev(0, dx, y)
                outs.append(y)
            ctx.check()
            got = [o_.cpu().numpy() for o_ in outs]
        allg = gather(got)
        if rank == 0:
            want = O.matvec(wt, w, dim, cols, x)
            key = f"tp_wo_sum_{name}" if W > 1 else f"wo_{name}"
            res[key] = {"workload": f"wo {dim} x {cols} {name}" +
                                    (" (l3p_attn_wo_allreduce_dev, 2 steps, every rank)" if W > 1 else " (l3p_attn_wo_dev)"),
                        **_worst([_cmp(g_, want) for r_ in allg for g_ in r_])}
    if rank == 0:
        res["tolerance"] = "|gpu - oracle| <= 1e-4 + 1e-4*|oracle| element-wise (fp32 oracle, f32 mode)"
        res["all_ok"] = all(r["ok"] for r in res.values() if isinstance(r, dict))
    return res if rank == 0 else None


# --------------------------------------------------------------------------
# the headline line


def run_ours(args):
    import torch
    import torch.distributed as dist

    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.shard import plan_shards

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    sh = CONFIGS[WORKLOAD]
    L, P = sh.n_layers, sh.pos + 1
    shard = plan_shards(sh.n_kv_heads, sh.seq_len, world, seq_parts=1)[rank]
    ctx = AttnContext.for_shape(sh, device=local, kv_head_begin=shard.kv_head_begin,
                                kv_head_count=shard.kv_head_count)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream)

    # resident cache: positions [0, pos) filled on the device, row pos appended per step
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + rank)
    hk = shard.kv_head_count
    for layer in range(L):
        kp, vp = ctx.kv_device_ptr(layer)
        kt = torch.as_tensor(DevView(kp, (hk, sh.seq_len, sh.head_dim)), device="cuda")
        vt = torch.as_tensor(DevView(vp, (hk, sh.seq_len, sh.head_dim)), device="cuda")
        kt[:, : sh.pos].normal_(generator=g)
        vt[:, : sh.pos].normal_(generator=g)
    q = torch.randn((L, sh.n_heads, sh.head_dim), device="cuda", generator=g)
    knew = torch.randn((L, sh.n_kv_heads, sh.head_dim), device="cuda", generator=g)
    vnew = torch.randn((L, sh.n_kv_heads, sh.head_dim), device="cuda", generator=g)
    out = torch.zeros_like(q)
    torch.cuda.synchronize()

    def step():
        # per layer ONE launch: the new K/V row is appended and attended in the decode kernel
        for layer in range(L):
            ctx.step_dev(layer, sh.pos, q[layer], knew[layer], vnew[layer], out[layer], stream)

    # consecutive step launches belong to different layers, so a launch may
    # start streaming its cache while the previous layer's kernel finishes
    # (programmatic dependent launch; see l3p_attn_set_overlap)
    if not args.no_overlap:
        ctx.set_overlap(True)
    # capture one step as a CUDA graph (the step is L launches)
    n0 = ctx.launch_count()
    step()
    torch.cuda.synchronize()
    launches_per_step = ctx.launch_count() - n0
    graph = None
    if not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        cap_stream = torch.cuda.Stream()
        cap_stream.wait_stream(stream)
        with torch.cuda.stream(cap_stream):
            ctx.set_stream(cap_stream)
            with torch.cuda.graph(graph, stream=cap_stream):
                for layer in range(L):
                    ctx.step_dev(layer, sh.pos, q[layer], knew[layer], vnew[layer], out[layer], cap_stream)
        stream.wait_stream(cap_stream)
        ctx.set_stream(stream)

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step()

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    ctx.check()

    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        run_step()
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    ctx.check()

    # decode kernel alone (roofline): a CUDA graph of 2*L decode launches with
    # no overlap between them, timed with CUDA events on the launching stream
    ctx.set_overlap(False)
    kgraph = torch.cuda.CUDAGraph()
    kstream = torch.cuda.Stream()
    kstream.wait_stream(stream)
    with torch.cuda.stream(kstream):
        ctx.set_stream(kstream)
        with torch.cuda.graph(kgraph, stream=kstream):
            for i in range(2 * L):
                ctx.decode_dev(i % L, sh.pos, q[i % L], out[i % L], kstream)
    stream.wait_stream(kstream)
    ctx.set_stream(stream)
    kgraph.replay()
    torch.cuda.synchronize()
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(3):
        kgraph.replay()
    k1.record(stream)
    torch.cuda.synchronize()
    kern_ms = k0.elapsed_time(k1) / (3 * 2 * L)
    del kgraph

    # the same step from the raw projections (l3p_attn_step_raw_dev: RoPE and
    # the cache write on the device, then the decode), as a graph of L layers
    raw = None
    exchange = None
    if not args.no_raw:
        ctx.set_rope()
        ctx.set_overlap(not args.no_overlap)
        rgraph = torch.cuda.CUDAGraph()
        rstream = torch.cuda.Stream()
        rstream.wait_stream(stream)
        n0 = ctx.launch_count()
        with torch.cuda.stream(rstream):
            ctx.set_stream(rstream)
            with torch.cuda.graph(rgraph, stream=rstream):
                for layer in range(L):
                    ctx.step_raw_dev(layer, sh.pos, q[layer], knew[layer], vnew[layer], out[layer], rstream)
        raw_launches = ctx.launch_count() - n0
        stream.wait_stream(rstream)
        ctx.set_stream(stream)
        for _ in range(max(3, args.warmup)):
            rgraph.replay()
        torch.cuda.synchronize()
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        r0.record(stream)
        for _ in range(args.steps):
            rgraph.replay()
        r1.record(stream)
        torch.cuda.synchronize()
        ctx.check()
        raw_ms = r0.elapsed_time(r1) / args.steps
        del rgraph
        raw = {"api": "l3p_attn_step_raw_dev (QK-norm/RoPE + cache write + decode)",
               "us_per_layer": round(raw_ms * 1e3 / L, 3), "launches_per_layer": raw_launches // L,
               "post_rope_step_us_per_layer": round(ms / args.steps * 1e3 / L, 3)}
        if not args.no_wo:
            # and on to the wo projection (Q8_0 weights, 4096 x 4096 per layer): at N = 1 the
            # local projection; at N > 1 each rank's partial over its heads, then (a) left
            # partial and (b) summed over NVLink on every rank -- (b) - (a) is the exchange
            from llama3pure_b200.synth import wo_weights

            dim = sh.n_heads * sh.head_dim
            w = wo_weights(8, dim, dim, seed=3)
            for layer in range(L):
                ctx.set_wo(layer, 8, w)
            xb2 = torch.zeros((L, dim), device="cuda")
            job = Job(torch, dist, world, rank, local)
            ctx.set_stream(stream)
            bgraph = job.graph(lambda s: [(ctx.step_raw_dev(l, sh.pos, q[l], knew[l], vnew[l], out[l], s),
                                           ctx.wo_dev(l, out[l], xb2[l], s)) for l in range(L)])
            wo_ms = job.time_graph(bgraph, args.steps, max(3, args.warmup))
            ctx.check()
            del bgraph
            raw["with_wo_q8_0_us_per_layer"] = round(wo_ms * 1e3 / L, 3)
            if world > 1:
                h = ctx.tp_group_export(world, rank, dim)
                hs = [None] * world
                dist.all_gather_object(hs, h)
                ctx.tp_group_import(hs)
                agraph = job.graph(lambda s: [(ctx.step_raw_dev(l, sh.pos, q[l], knew[l], vnew[l], out[l], s),
                                               ctx.wo_allreduce_dev(l, out[l], xb2[l], s)) for l in range(L)])
                ar_ms = job.time_graph(agraph, args.steps, max(3, args.warmup))
                ctx.check()
                del agraph
                raw["with_wo_allreduce_q8_0_us_per_layer"] = round(ar_ms * 1e3 / L, 3)
                raw["wo_allreduce"] = ("each rank's partial wo over its heads, summed over NVLink peer memory "
                                       "(l3p_attn_wo_allreduce_dev)")
                exchange = {"us_per_layer": round((ar_ms - wo_ms) * 1e3 / L, 3),
                            "what": "the tensor-parallel wo sum of the head-sharded step: 16 KiB partial per rank, "
                                    "reduce-scattered and all-gathered over NVLink inside the projection; "
                                    "= with_wo_allreduce - with_wo (same graph without the sum)"}
    if clocks:
        clk = clocks.stop()
    else:
        clk = None

    if world > 1:
        t = torch.tensor([ms, kern_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kern_ms = t.tolist()

    bytes_per_layer_rank = 2 * P * hk * sh.head_dim * 4
    total_bytes = bytes_per_layer_rank * world * L * args.steps
    value = total_bytes / (ms / 1e3) / 1e9
    ms_step = ms / args.steps
    peak, peak_kind = measured_peaks()
    # every launch of the timed region is the decode kernel (one per layer)
    launch_ms = ms_step / launches_per_step
    achieved = bytes_per_layer_rank / (launch_ms / 1e3) / 1e9
    split_k = dict(zip(("ctas_per_kv_head", "cluster"), ctx.decode_plan(sh.pos)))

    # end to end through the host-pointer C ABI (every rank runs it; max over ranks)
    e2e = None
    if not args.no_e2e:
        legs = [run_e2e(ctx, sh, world, args, torch, server=False)]
        if not args.no_server:
            legs.append(run_e2e(ctx, sh, world, args, torch, server=True))
        for leg in legs:
            if world > 1:
                t = torch.tensor([leg["ms_per_step"]], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                leg["ms_per_step"] = round(t.item(), 4)
                leg["us_per_layer"] = round(leg["ms_per_step"] * 1e3 / L, 2)
                leg["value"] = round(bytes_per_layer_rank * world * L / (leg["ms_per_step"] / 1e3) / 1e9, 3)
        # the headline e2e is the faster of the two forms of the same call
        e2e = dict(min(legs, key=lambda d: d["ms_per_step"]))
        e2e["legs"] = {d["leg"]: {k: d[k] for k in ("value", "ms_per_step", "us_per_layer", "api")} for d in legs}
    del graph
    ctx.close()

    # every BASELINE configuration at this GPU count, then the parity leg
    job = Job(torch, dist, world, rank, local)
    configs = None
    if not args.no_configs:
        reps = max(args.steps // 2, 5)
        configs = {"llama32_1b_decode": config1(job, reps),
                   "llama31_8b_decode_128k": config3(job, max(reps // 2, 3)),
                   "gemma_2b_decode": config4(job, reps)}
    prefill = None
    if not args.no_prefill:
        prefill = config5(job, max(args.steps // 2, 4), raw=not args.no_raw)
        if world == 1:
            prefill["other_head_dims"] = prefill_other_head_dims(job, max(args.steps // 4, 3),
                                                                 prefill["tf32_dense_tflops_measured"])
    parity = None
    if not args.no_parity:
        parity = parity_leg(job)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline()
    q8 = None
    if rank == 0 and world == 1 and not args.no_q8:
        q8 = run_q8(args, torch)
    wo = None
    if rank == 0 and world == 1 and not args.no_wo:
        wo = run_wo(args, torch)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": ("synthetic: the timed caches and q/k/v are N(0,1) fp32 from torch's device generator "
                     "(Philox, seed 1000 + rank); the parity leg uses the BASELINE generator (numpy PCG64, "
                     "SeedSequence([seed, layer]))"),
            "config": {"workload": WORKLOAD, "n_layers": L, "n_heads": sh.n_heads, "n_kv_heads": sh.n_kv_heads,
                       "head_dim": sh.head_dim, "pos": sh.pos, "kv_positions": P,
                       "parallelism": f"kv-head shards x{world}",
                       "launch": ("cuda graph" if not args.no_graph else "stream") +
                                 ("" if args.no_overlap else " + programmatic dependent launch"),
                       "split_k": split_k,
                       "l2": "inputs larger than L2 (2 GiB KV per step vs 126 MB L2)"},
            "us_per_layer": round(ms_step * 1e3 / L, 3),
            "tokens_per_s": round(1e3 / ms_step, 2),
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "kernel": "decode_f32_kernel<128,4>", "kernel_us": round(launch_ms * 1e3, 3),
                         "kernel_timing": "timed region / its launches (one decode launch per layer, CUDA graph "
                                          "with programmatic dependent launch, CUDA events)",
                         "isolated_kernel_us": round(kern_ms * 1e3, 3),
                         "isolated_frac": round(bytes_per_layer_rank / kern_ms / 1e6 / peak, 4),
                         "isolated_timing": "graph of 64 decode launches without overlap, CUDA events",
                         "algorithmic_bytes_per_launch": bytes_per_layer_rank,
                         "traffic": args.traffic if args.traffic is not None else
                         (NCU_TRAFFIC_PER_LAUNCH if world == 1 else None)},
            "exchange_us_per_layer": exchange["us_per_layer"] if exchange else None,
            "exchange": exchange,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "parity": parity,
            "configs": configs,
            "pre_attention_step": raw,
            "wo_projection": wo,
            "prefill": prefill,
            "q8_decode": q8,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    rc = 0
    if rank == 0 and parity is not None and not parity["all_ok"]:
        print("parity leg FAILED: " + json.dumps({k: r for k, r in parity.items()
                                                  if isinstance(r, dict) and not r["ok"]}), file=sys.stderr)
        rc = 1
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return rc


def run_long(args):
    """Llama-3.1-8B shapes at position 131071 of a
    131072-entry fp32 cache (1 GiB of K+V per layer, K rows x 0.5), 32 layers,
    split over the ranks as head groups x sequence parts (--seq-parts).  Per
    layer each rank runs the partial decode over its positions; ranks sharing
    a head group all-gather their (m, l, o) triples over NCCL and merge them
    with the LSE kernel.  One JSON line on rank 0 (device time, max over
    ranks)."""
    import datetime

    import torch
    import torch.distributed as dist

    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.shard import plan_shards

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    sh = CONFIGS["llama31_8b_decode_128k"]
    L, P, hd = sh.n_layers, sh.pos + 1, sh.head_dim
    seq_parts = args.seq_parts if args.seq_parts > 0 else 1
    shards = plan_shards(sh.n_kv_heads, sh.seq_len, world, seq_parts)
    me = shards[rank]
    ctx = AttnContext.for_shape(sh, device=local, kv_head_begin=me.kv_head_begin, kv_head_count=me.kv_head_count,
                                seq_begin=me.seq_begin, seq_count=me.seq_count)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream)
    g = torch.Generator(device="cuda")
    g.manual_seed(2000 + rank)
    for layer in range(L):
        kp, vp = ctx.kv_device_ptr(layer)
        kt = torch.as_tensor(DevView(kp, (me.kv_head_count, me.seq_count, hd)), device="cuda")
        vt = torch.as_tensor(DevView(vp, (me.kv_head_count, me.seq_count, hd)), device="cuda")
        kt.normal_(generator=g).mul_(sh.k_scale)
        vt.normal_(generator=g)
    q = torch.randn((L, sh.n_heads * hd), device="cuda", generator=g)
    out = torch.zeros_like(q)
    part_o = torch.zeros((L, sh.n_heads * hd), device="cuda")
    part_ml = torch.zeros((L, sh.n_heads * 2), device="cuda")
    gat_o = torch.zeros((L, world, sh.n_heads * hd), device="cuda")
    gat_ml = torch.zeros((L, world, sh.n_heads * 2), device="cuda")
    r0 = me.kv_head_begin * sh.kv_mul
    nr = me.kv_head_count * sh.kv_mul
    g0 = me.head_group * seq_parts  # first rank of this head group

    nvlink = seq_parts > 1 and args.xchg == "nvlink"
    if nvlink:
        # the members of this head group map each other's exchange regions
        h = ctx.seq_group_export(seq_parts, me.seq_part)
        hs = [None] * world
        dist.all_gather_object(hs, h)
        ctx.seq_group_import(hs[g0:g0 + seq_parts])
        ctx.set_overlap(True)

    def step(s):
        for layer in range(L):
            if seq_parts == 1:
                ctx.decode_dev(layer, sh.pos, q[layer], out[layer], s)
                continue
            if nvlink:
                ctx.decode_seq_dev(layer, sh.pos, q[layer], out[layer], s)
                continue
            ctx.decode_partial_dev(layer, sh.pos, q[layer], part_o[layer], part_ml[layer], s)
            dist.all_gather_into_tensor(gat_o[layer], part_o[layer])
            dist.all_gather_into_tensor(gat_ml[layer], part_ml[layer])
            ctx.lse_merge_dev(seq_parts, sh.n_heads, r0, nr, gat_o[layer, g0], gat_ml[layer, g0], out[layer], s)

    for _ in range(args.warmup):
        step(stream)
    torch.cuda.synchronize()
    ctx.check()
    # a CUDA graph when the step holds no collective (every rank takes the same branch)
    graph = None
    if not args.no_graph and (seq_parts == 1 or nvlink):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step(stream)

    def run_step():
        if graph is not None:
            graph.replay()
        else:
            step(stream)

    for _ in range(args.warmup):
        run_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        run_step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    ctx.check()
    total_bytes = 2 * P * sh.n_kv_heads * hd * 4 * L * args.steps
    if rank == 0:
        peak, peak_kind = measured_peaks()
        gbs = total_bytes / (ms / 1e3) / 1e9
        print(json.dumps({
            "metric": "decode-attn KV GB/s (fp32-equivalent), Llama-3.1-8B shapes, ctx 128K, 32 layers",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "us_per_layer": round(ms / args.steps * 1e3 / L, 2),
            "tokens_per_s": round(1e3 / (ms / args.steps), 2), "higher_is_better": True, "scaling": "strong",
            "dtype": "f32", "data": "synthetic (on-device N(0,1), K x 0.5)",
            "config": {"workload": "llama31_8b_decode_128k", "head_groups": world // seq_parts,
                       "seq_parts": seq_parts,
                       "exchange": ("none" if seq_parts == 1 else
                                    "peer reads over NVLink inside the merge kernel (l3p_attn_decode_seq_dev)"
                                    if nvlink else "NCCL all-gather + LSE merge kernel"),
                       "launch": "cuda graph" if graph is not None else "stream"},
            "frac_of_hbm_per_gpu": round(gbs / world / peak, 4), "peak_kind": peak_kind,
        }), flush=True)
    del graph
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_kernel_only(args):
    """Decode kernel alone on `--layers` layers of the workload (a small case
    for ncu captures: layers x 64 MiB of KV, still larger than L2)."""
    import torch

    from llama3pure_b200.attn import AttnContext

    sh = CONFIGS[WORKLOAD]
    L = args.layers
    ctx = AttnContext.for_shape(sh, n_layers=L)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream)
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    for layer in range(L):
        for p in ctx.kv_device_ptr(layer):
            torch.as_tensor(DevView(p, (sh.n_kv_heads, sh.seq_len, sh.head_dim)), device="cuda").normal_(generator=g)
    q = torch.randn((L, sh.n_heads, sh.head_dim), device="cuda", generator=g)
    out = torch.zeros_like(q)
    for _ in range(args.warmup):
        for layer in range(L):
            ctx.decode_dev(layer, sh.pos, q[layer], out[layer], stream)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        for layer in range(L):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ctx.decode_dev(layer, sh.pos, q[layer], out[layer], stream)
            b.record(stream)
            times.append((a, b))
    torch.cuda.synchronize()
    ctx.check()
    us = statistics.median(a.elapsed_time(b) * 1e3 for a, b in times)
    nbytes = 2 * (sh.pos + 1) * sh.n_kv_heads * sh.head_dim * 4
    print(json.dumps({"mode": "kernel-only", "layers": L, "launches": len(times), "median_us": round(us, 3),
                      "gbs": round(nbytes / us / 1e3, 1)}), flush=True)
    ctx.close()
    return 0


def run_decode_trace(args):
    """Per-stage timeline of the decode launches of a step graph (the headline
    form: 32 layers of l3p_attn_step_dev with programmatic dependent launch,
    and the same launches without it), from a build of the library with
    -DL3P_DECODE_TRACE: every CTA stamps %globaltimer at its start, when
    griddepcontrol.wait returns, when q is ready, when its last tile is done,
    when its partial is published and at its exit.  --kv-heads H owns H of
    the 8 KV heads (the per-rank work at N = 8/H GPUs); --q8 uses a Q8_0 cache.
    Prints medians over the layers of one replay, in microseconds."""
    import tempfile as _tf

    import torch

    from llama3pure_b200.attn import AttnContext, load_library
    from llama3pure_b200.build import LIB_PATH
    from llama3pure_b200.build import build as build_lib

    torch.cuda.set_device(0)
    lib_path = os.path.join(os.path.dirname(LIB_PATH), "libllama3pure_attn_trace.so")
    build_lib(out=lib_path, extra=["-DL3P_DECODE_TRACE"])
    lib = load_library(lib_path)
    sh = CONFIGS[WORKLOAD]
    L, hk = sh.n_layers, args.kv_heads
    job = Job(torch, None, 1, 0, 0)
    out_json = {"workload": WORKLOAD, "kv_heads": hk, "kv_format": "q8_0" if args.q8 else "f32", "n_layers": L}
    for overlap in (True, False):
        ctx = AttnContext.for_shape(sh, device=0, kv_head_begin=0, kv_head_count=hk, kv_format=1 if args.q8 else 0,
                                    lib=lib)
        if args.q8:
            for layer in range(L):  # random blocks (any bytes time the same)
                rng = np.random.default_rng(layer)
                nb = sh.head_dim // 32
                b = rng.integers(0, 256, size=(sh.n_kv_heads, sh.seq_len, nb * 34), dtype=np.uint8)
                b.reshape(sh.n_kv_heads, sh.seq_len, nb, 34)[..., 1] = 0x20  # fp16 scales ~0.008
                ctx.load_kv_q8(layer, 0, b, b)
            g = torch.Generator(device="cuda")
            g.manual_seed(3)
        else:
            g = job.fill_cache(ctx, L, hk, sh.seq_len, sh.head_dim, 3)
        q = torch.randn((L, sh.n_heads * sh.head_dim), device="cuda", generator=g)
        kn = torch.randn((L, sh.n_kv_heads * sh.head_dim), device="cuda", generator=g)
        vn = torch.randn_like(kn)
        o = torch.zeros_like(q)
        ctx.set_overlap(overlap)
        gr = job.graph(lambda s: [ctx.step_dev(l, sh.pos, q[l], kn[l], vn[l], o[l], s) for l in range(L)])
        ms = job.time_graph(gr, args.steps)
        gr.replay()  # the traced replay (slots hold the last launch of each layer)
        torch.cuda.synchronize()
        ctx.check()
        fd, path = _tf.mkstemp(suffix=".bin")
        os.close(fd)
        os.environ["L3P_TRACE_FILE"] = path
        plan = ctx.decode_plan(sh.pos)
        del gr
        ctx.close()
        os.environ.pop("L3P_TRACE_FILE", None)
        raw = np.fromfile(path, dtype=np.int64)
        os.unlink(path)
        n, ctas = int(raw[0]), int(raw[1])
        recs = []
        off = 2
        for _ in range(n):
            meta = raw[off:off + 6]
            st = raw[off + 6:off + 6 + ctas * 8].reshape(ctas, 8)[: int(meta[1] * meta[2] * meta[3])].astype(np.float64)
            recs.append((meta, st))
            off += 6 + ctas * 8
        # the launches of the last replay: the L with the highest launch sequence numbers
        recs = sorted(recs, key=lambda r: r[0][0])[-L:]
        rows = []
        for i in range(1, len(recs)):
            prev_end = recs[i - 1][1][:, 5].max()
            st = recs[i][1]
            rows.append({
                "first_cta_start_after_prev_end": st[:, 0].min() - prev_end,
                "wait_release_after_prev_end": st[:, 1].min() - prev_end,
                "ctas_started_before_prev_end": float((st[:, 0] < prev_end).mean()),
                "q_ready_after_release": np.median(st[:, 2] - st[:, 1]),
                "last_tile_after_release": st[:, 3].max() - st[:, 1].min(),
                "median_tile_done_after_release": np.median(st[:, 3] - st[:, 1]),
                "ticket_after_last_tile": st[:, 4].max() - st[:, 3].max(),
                "merge_tail_after_last_tile": st[:, 5].max() - st[:, 3].max(),
                "period": st[:, 5].max() - prev_end,
            })
        out_json["overlap" if overlap else "no_overlap"] = {
            "us_per_layer_timed": round(ms * 1e3 / L, 3), "split_k": plan,
            **{k: round(float(np.median([r[k] for r in rows])) / (1.0 if k.startswith("ctas") else 1e3), 3)
               for k in rows[0]}}
    print(json.dumps({"mode": "decode-trace", **out_json}), flush=True)
    return 0


def run_server_trace(args, lib_path=None):
    """Stage timeline of calls served by the host-call server
    (l3p_attn_set_host_server) on the headline workload, from the
    -DL3P_DECODE_TRACE build: the host stamps CLOCK_REALTIME when it posts a
    call and when it has read every output packet; every CTA stamps
    %globaltimer when it sees the call (fetchers: the mailbox; the others: the
    go word), (fetchers) when it has published go, and at the decode body's
    stages.  Prints medians over the last 32 calls, in microseconds (host and
    GPU stamps on the clock the driver keeps %globaltimer on)."""
    import tempfile as _tf

    import torch

    from llama3pure_b200.attn import AttnContext, load_library
    from llama3pure_b200.build import LIB_PATH
    from llama3pure_b200.build import build as build_lib

    torch.cuda.set_device(0)
    if lib_path is None:
        lib_path = os.path.join(os.path.dirname(LIB_PATH), "libllama3pure_attn_trace.so")
        build_lib(out=lib_path, extra=["-DL3P_DECODE_TRACE"])
    lib = load_library(lib_path)
    sh = CONFIGS[WORKLOAD]
    L, hk = sh.n_layers, args.kv_heads
    job = Job(torch, None, 1, 0, 0)
    ctx = AttnContext.for_shape(sh, device=0, kv_head_begin=0, kv_head_count=hk, lib=lib)
    job.fill_cache(ctx, L, hk, sh.seq_len, sh.head_dim, 3)
    torch.cuda.synchronize()
    qh = torch.randn((L, sh.n_heads, sh.head_dim)).pin_memory().numpy()
    kh = torch.randn((L, sh.n_kv_heads, sh.head_dim)).pin_memory().numpy()
    vh = torch.randn((L, sh.n_kv_heads, sh.head_dim)).pin_memory().numpy()
    oh = torch.zeros((L, sh.n_heads, sh.head_dim)).pin_memory().numpy()
    fn, h = ctx.lib.l3p_attn_step, ctx.h
    calls = [(layer, qh[layer].ctypes.data, kh[layer].ctypes.data, vh[layer].ctypes.data, oh[layer].ctypes.data)
             for layer in range(L)]
    ctx.set_host_server(True)
    t0 = time.perf_counter()
    n_steps = max(3, args.warmup) + args.steps
    for _ in range(n_steps):
        for layer, qp, kp, vp, op in calls:
            rc = fn(h, layer, sh.pos, qp, kp, vp, op)
            if rc:
                ctx._ok(rc, "l3p_attn_step")
    us_per_call = (time.perf_counter() - t0) / (n_steps * L) * 1e6
    fd, path = _tf.mkstemp(suffix=".bin")
    os.close(fd)
    os.environ["L3P_TRACE_FILE"] = path
    ctx.close()
    os.environ.pop("L3P_TRACE_FILE", None)
    raw = np.fromfile(path, dtype=np.int64)
    os.unlink(path)
    n, ctas = int(raw[0]), int(raw[1])
    recs = []
    off = 2
    for _ in range(n):
        meta = raw[off:off + 6]
        st = raw[off + 6:off + 6 + ctas * 8].reshape(ctas, 8)
        recs.append((meta, st[: int(meta[1] * meta[2])].astype(np.float64), st[ctas - 1].astype(np.float64)))
        off += 6 + ctas * 8
    recs = sorted(recs, key=lambda r: r[0][0])[-32:]
    rows = []
    for meta, st, host in recs:
        gx, gy = int(meta[1]), int(meta[2])
        fetch = st.reshape(gy, gx, 8)[:, 0, :]  # split 0 of every unit: the fetchers (n_hg = 1 here)
        others = st.reshape(gy, gx, 8)[:, 1:, :].reshape(-1, 8)
        go = fetch[:, 7].max()
        rows.append({
            "host_pack_and_copy_call": host[2] - host[0],
            # the two host<->GPU crossings, summed so that the clocks' offset cancels
            "copy_to_header_seen_plus_flags_to_host": (fetch[:, 6].min() - host[2]) + (host[3] - st[:, 5].max()),
            "last_fetcher_sees_header_after_first": fetch[:, 6].max() - fetch[:, 6].min(),
            "go_published_after_call_seen": np.median(fetch[:, 7] - fetch[:, 6]),
            "others_see_go_after_published": np.median(others[:, 6]) - go if len(others) else 0.0,
            "q_ready_after_go": np.median(st[:, 2]) - go,
            "last_tile_after_go": st[:, 3].max() - go,
            "merged_after_last_tile": st[:, 5].max() - st[:, 3].max(),
            "host_output_copy": host[1] - host[3],
            "call": host[1] - host[0],
        })
    out = {"mode": "server-trace", "workload": WORKLOAD, "kv_heads": hk, "us_per_call_loop": round(us_per_call, 2),
           "grid": [int(recs[-1][0][1]), int(recs[-1][0][2])],
           **{k: round(float(np.median([r[k] for r in rows])) / 1e3, 3) for k in rows[0]}}
    print(json.dumps(out), flush=True)
    return 0


def run_tp_trace(args):
    """Under torchrun (N >= 2): stage timeline of the tensor-parallel wo sum
    (l3p_attn_wo_allreduce_dev, Q8_0 4096 x 4096, each rank the columns of its
    KV-head shard) from the -DL3P_DECODE_TRACE build, alone (32 launches in a
    graph) and inside the head-sharded block (raw step + wo + sum per layer).
    Every CTA stamps %globaltimer at its start, after griddepcontrol.wait,
    after its GEMV rows, after sending them to every member, when every
    member's rows of its block have arrived and are summed, and at its exit.  Medians over the launches of one replay, per rank, in us (each
    GPU's own timer: only differences within one GPU are used)."""
    import datetime
    import tempfile as _tf

    import torch
    import torch.distributed as dist

    from llama3pure_b200.attn import AttnContext, load_library
    from llama3pure_b200.build import LIB_PATH
    from llama3pure_b200.build import build as build_lib
    from llama3pure_b200.shard import plan_shards
    from llama3pure_b200.synth import wo_weights

    world, rank, local = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    lib_path = os.path.join(os.path.dirname(LIB_PATH), "libllama3pure_attn_trace.so")
    if rank == 0:
        build_lib(out=lib_path, extra=["-DL3P_DECODE_TRACE"])
    dist.barrier()
    lib = load_library(lib_path)
    job = Job(torch, dist, world, rank, local)
    sh = CONFIGS[WORKLOAD]
    L, dim = sh.n_layers, sh.n_heads * sh.head_dim
    me = plan_shards(sh.n_kv_heads, sh.seq_len, world, 1)[rank]
    res = {}
    for name in ("wo_allreduce_alone", "block"):
        ctx = AttnContext.for_shape(sh, device=local, kv_head_begin=me.kv_head_begin, kv_head_count=me.kv_head_count,
                                    lib=lib)
        g = job.fill_cache(ctx, L, me.kv_head_count, sh.seq_len, sh.head_dim, 11 + rank)
        q = torch.randn((L, dim), device="cuda", generator=g)
        kn = torch.randn((L, sh.n_kv_heads * sh.head_dim), device="cuda", generator=g)
        vn = torch.randn_like(kn)
        out = torch.zeros_like(q)
        xb2 = torch.zeros((L, dim), device="cuda")
        w = wo_weights(8, dim, dim, seed=3)
        for l in range(L):
            ctx.set_wo(l, 8, w)
        ctx.set_rope()
        h = ctx.tp_group_export(world, rank, dim)
        hs = [None] * world
        dist.all_gather_object(hs, h)
        ctx.tp_group_import(hs)
        ctx.set_overlap(True)
        if name == "block":
            gr = job.graph(lambda s: [(ctx.step_raw_dev(l, sh.pos, q[l], kn[l], vn[l], out[l], s),
                                       ctx.wo_allreduce_dev(l, out[l], xb2[l], s)) for l in range(L)])
        else:
            gr = job.graph(lambda s: [ctx.wo_allreduce_dev(l, out[l], xb2[l], s) for l in range(L)])
        ms = job.time_graph(gr, args.steps)
        gr.replay()
        torch.cuda.synchronize()
        ctx.check()
        fd, path = _tf.mkstemp(suffix=".bin")
        os.close(fd)
        os.environ["L3P_TRACE_FILE"] = path
        del gr
        ctx.close()
        os.environ.pop("L3P_TRACE_FILE", None)
        raw = np.fromfile(path, dtype=np.int64)
        os.unlink(path)
        n, ctas = int(raw[0]), int(raw[1])
        recs, off = [], 2
        for _ in range(n):
            meta = raw[off:off + 6]
            st = raw[off + 6:off + 6 + ctas * 8].reshape(ctas, 8)[: int(meta[1] * meta[2] * meta[3])].astype(np.float64)
            if meta[5] == -1:  # wo launches
                recs.append((meta, st))
            off += 6 + ctas * 8
        recs = sorted(recs, key=lambda r: r[0][0])[-L:]
        rows = []
        for i in range(1, len(recs)):
            st, prev = recs[i][1], recs[i - 1][1]
            rows.append({
                "release_after_prev_exit": st[:, 1].min() - prev[:, 5].max(),
                "gemv_done_after_release": st[:, 2].max() - st[:, 1].min(),
                "sent_after_gemv": np.median(st[:, 3] - st[:, 2]),
                "summed_after_sent": np.median(st[:, 4] - st[:, 3]),
                "exit_after_summed": np.median(st[:, 5] - st[:, 4]),
                "last_exit_after_release": st[:, 5].max() - st[:, 1].min(),
                "period": st[:, 5].max() - prev[:, 5].max(),
            })
        summary = {k: round(float(np.median([r[k] for r in rows])) / 1e3, 3) for k in rows[0]}
        summary["us_per_layer_timed"] = round(ms * 1e3 / L, 3)
        per_rank = [None] * world
        dist.all_gather_object(per_rank, summary)
        res[name] = per_rank
    if rank == 0:
        print(json.dumps({"mode": "tp-trace", "n_gpus": world, **res}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_q8(args, torch, layers: int = 16):
    """Decode over the reference's own cache format (kv_format L3P_KV_Q8_0,
    272 bytes per position and KV head instead of 1024) on the workload's
    geometry: `layers` layers of random Q8_0 blocks (285 MB at 16 layers, more
    than L2), the decode kernel alone timed over a CUDA graph of 2*layers
    launches, and the engine's per-layer step (append + decode)."""
    from llama3pure_b200.attn import AttnContext

    sh = CONFIGS[WORKLOAD]
    L = layers
    ctx = AttnContext.for_shape(sh, n_layers=L, kv_format=1)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream)
    rng = np.random.default_rng(77)
    nb = sh.head_dim // 32
    for layer in range(L):
        blocks = []
        for _ in range(2):
            b = rng.integers(-127, 128, size=(sh.n_kv_heads, sh.seq_len, nb, 34), dtype=np.int16).astype(np.int8)
            d = rng.uniform(0.005, 0.03, size=(sh.n_kv_heads, sh.seq_len, nb)).astype(np.float16)
            b = b.view(np.uint8)
            b[..., :2] = d.view(np.uint8).reshape(sh.n_kv_heads, sh.seq_len, nb, 2)
            blocks.append(np.ascontiguousarray(b.reshape(sh.n_kv_heads, sh.seq_len, nb * 34)))
        ctx.load_kv_q8(layer, 0, blocks[0], blocks[1])
    g = torch.Generator(device="cuda")
    g.manual_seed(78)
    q = torch.randn((L, sh.n_heads, sh.head_dim), device="cuda", generator=g)
    knew = torch.randn((L, sh.n_kv_heads, sh.head_dim), device="cuda", generator=g)
    vnew = torch.randn((L, sh.n_kv_heads, sh.head_dim), device="cuda", generator=g)
    out = torch.zeros_like(q)

    def graph_of(fn):
        gr = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(stream)
        with torch.cuda.stream(cs):
            ctx.set_stream(cs)
            with torch.cuda.graph(gr, stream=cs):
                fn(cs)
        stream.wait_stream(cs)
        ctx.set_stream(stream)
        return gr

    def timed(gr, reps):
        for _ in range(max(3, args.warmup)):
            gr.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            gr.replay()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    kgr = graph_of(lambda cs: [ctx.decode_dev(i % L, sh.pos, q[i % L], out[i % L], cs) for i in range(2 * L)])
    kern_us = timed(kgr, 5) * 1e3 / (2 * L)
    n0 = ctx.launch_count()
    sgr = graph_of(lambda cs: [ctx.step_dev(i, sh.pos, q[i], knew[i], vnew[i], out[i], cs) for i in range(L)])
    launches = ctx.launch_count() - n0
    step_us = timed(sgr, max(args.steps, 5)) * 1e3 / L
    # the same step with programmatic dependent launch (as the headline step)
    ctx.set_overlap(not args.no_overlap)
    ogr = graph_of(lambda cs: [ctx.step_dev(i, sh.pos, q[i], knew[i], vnew[i], out[i], cs) for i in range(L)])
    step_overlap_us = timed(ogr, max(args.steps, 5)) * 1e3 / L
    ctx.check()
    del kgr, sgr, ogr
    raw_us = None
    if not getattr(args, "no_raw", False):
        ctx.set_rope()
        rgr = graph_of(lambda cs: [ctx.step_raw_dev(i, sh.pos, q[i], knew[i], vnew[i], out[i], cs) for i in range(L)])
        raw_us = round(timed(rgr, max(args.steps, 5)) * 1e3 / L, 3)
        ctx.check()
        del rgr
    ctx.close()
    nbytes = 2 * (sh.pos + 1) * sh.n_kv_heads * (sh.head_dim + sh.head_dim // 16)
    peak, peak_kind = measured_peaks()
    return {"workload": WORKLOAD + " with a Q8_0 cache", "layers_cycled": L, "kernel": "decode_q8_kernel<128,4>",
            "bytes_per_layer": nbytes, "kernel_us": round(kern_us, 3),
            "kernel_gbs": round(nbytes / kern_us / 1e3, 1), "frac_of_hbm": round(nbytes / kern_us / 1e3 / peak, 4),
            "peak_kind": peak_kind, "step_us_per_layer": round(step_us, 3),
            "step_launches_per_layer": launches // L, "step_overlap_us_per_layer": round(step_overlap_us, 3),
            "raw_step_us_per_layer": raw_us,
            "tokens_per_s_32_layers": round(1e6 / (step_us * 32), 1)}


def run_wo(args, torch, layers: int = 16):
    """The wo projection (attention output -> dim) on the workload's geometry
    (4096 x 4096) for each weight type: `layers` layers of random GGUF rows
    cycled (more than L2 in total), the kernel alone timed over a CUDA graph of
    2*layers launches without overlap."""
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.synth import wo_weights

    sh = CONFIGS[WORKLOAD]
    dim = cols = sh.n_heads * sh.head_dim
    stream = torch.cuda.Stream()
    peak, peak_kind = measured_peaks()
    res = {"shape": f"{dim} x {cols}", "layers_cycled": layers, "peak_kind": peak_kind}
    for name, wt, nbytes in (("q8_0", 8, cols // 32 * 34), ("q2_k", 10, cols // 256 * 84),
                             ("q3_k", 11, cols // 256 * 110), ("q4_k", 12, cols // 256 * 144),
                             ("q5_k", 13, cols // 256 * 176), ("q6_k", 14, cols // 256 * 210),
                             ("q4_0", 2, cols // 32 * 18), ("q4_1", 3, cols // 32 * 20), ("q5_0", 6, cols // 32 * 22),
                             ("q5_1", 7, cols // 32 * 24), ("iq4_nl", 20, cols // 32 * 18), ("f32", 0, cols * 4),
                             ("f16", 1, cols * 2), ("bf16", 29, cols * 2)):
        ctx = AttnContext.for_shape(sh, n_layers=layers, seq_len=16)
        ctx.set_stream(stream)
        w = wo_weights(wt, dim, cols, seed=5)
        for layer in range(layers):
            ctx.set_wo(layer, wt, w)
        x = torch.randn((layers, cols), device="cuda")
        y = torch.zeros((layers, dim), device="cuda")
        gr = torch.cuda.CUDAGraph()
        cs = torch.cuda.Stream()
        cs.wait_stream(stream)
        with torch.cuda.stream(cs):
            with torch.cuda.graph(gr, stream=cs):
                for i in range(2 * layers):
                    ctx.wo_dev(i % layers, x[i % layers], y[i % layers], cs)
        reps = 5
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(cs):  # replays run on the current stream; time them there
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            a.record(cs)
            for _ in range(reps):
                gr.replay()
            b.record(cs)
        torch.cuda.synchronize()
        ctx.check()
        us = a.elapsed_time(b) * 1e3 / (reps * 2 * layers)
        algo = dim * nbytes + cols * 4 + dim * 4  # GGUF weight bytes + x + y
        res[name] = {"us": round(us, 3), "bytes": algo, "gbs": round(algo / us / 1e3, 1),
                     "frac_of_hbm": round(algo / us / 1e3 / peak, 4)}
        del gr
        ctx.close()
    return res


def run_e2e(ctx, sh, world, args, torch, server=False):
    """l3p_attn_step per layer with pinned host buffers: H2D of q/k/v, append,
    decode, D2H of the output, every step.  server=True: the same calls with
    the host-call server on (l3p_attn_set_host_server): the inputs cross into
    a mailbox the resident grid reads, the output comes back as packets."""
    L = sh.n_layers
    qh = torch.randn((L, sh.n_heads, sh.head_dim)).pin_memory().numpy()
    kh = torch.randn((L, sh.n_kv_heads, sh.head_dim)).pin_memory().numpy()
    vh = torch.randn((L, sh.n_kv_heads, sh.head_dim)).pin_memory().numpy()
    oh = torch.zeros((L, sh.n_heads, sh.head_dim)).pin_memory().numpy()
    ctx.set_stream(None)
    # the C-ABI call itself, with the buffers' addresses taken once (the
    # AttnContext.step wrapper re-validates its numpy arguments on every call,
    # which costs the Python loop ~4 us per layer)
    fn, h, pos = ctx.lib.l3p_attn_step, ctx.h, sh.pos
    calls = [(layer, qh[layer].ctypes.data, kh[layer].ctypes.data, vh[layer].ctypes.data, oh[layer].ctypes.data)
             for layer in range(L)]

    def step():
        for layer, qp, kp, vp, op in calls:
            rc = fn(h, layer, pos, qp, kp, vp, op)
            if rc:
                ctx._ok(rc, "l3p_attn_step")

    if server:
        ctx.set_host_server(True)
    for _ in range(max(3, args.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    if server:
        ctx.set_host_server(False)  # ends the resident grid: the GPU is free again
    r0, r1 = ctx.owned_rows
    h2d = L * ((r1 - r0) * sh.head_dim + 2 * sh.n_kv_heads * sh.head_dim) * 4
    d2h = L * (r1 - r0) * sh.head_dim * 4
    hk = ctx.kv_head_count
    bytes_step = 2 * (sh.pos + 1) * hk * sh.head_dim * 4 * L * world
    return {"value": round(bytes_step / dt / 1e9, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(dt * 1e3, 4),
            "us_per_layer": round(dt * 1e6 / L, 2), "leg": "host_server" if server else "launch_per_call",
            "api": ("l3p_attn_step (host pointers, pinned) with the host-call server (l3p_attn_set_host_server)"
                    if server else "l3p_attn_step (host pointers, pinned), one launch + stream synchronisation per call"),
            "timing": "wall clock around the host loop (time.perf_counter), max over ranks"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-overlap", action="store_true", help="no programmatic dependent launch between layers")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-server", action="store_true", help="e2e: skip the host-call server leg")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-q8", action="store_true", help="skip the Q8_0-cache decode measurement")
    ap.add_argument("--no-raw", action="store_true", help="skip the raw-projection (RoPE on device) measurements")
    ap.add_argument("--no-wo", action="store_true", help="skip the wo projection measurement")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[0], [2], [3] sub-records")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity leg")
    ap.add_argument("--wo-only", action="store_true", help="wo projection measurement alone (ncu case)")
    ap.add_argument("--long", action="store_true", help="BASELINE configs[2] (128K context) over --gpus ranks")
    ap.add_argument("--seq-parts", type=int, default=1, help="--long: sequence parts per head group")
    ap.add_argument("--xchg", default="nvlink", choices=["nvlink", "nccl"],
                    help="--long: exchange of the sequence parts' partials")
    ap.add_argument("--q8-only", action="store_true", help="Q8_0-cache decode measurement alone")
    ap.add_argument("--kernel-only", action="store_true", help="decode kernel alone on --layers layers (ncu case)")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--trace-decode", action="store_true",
                    help="per-stage timeline of the step graph's decode launches (a -DL3P_DECODE_TRACE build)")
    ap.add_argument("--kv-heads", type=int, default=8, help="--trace-decode: KV heads owned (8/N at N GPUs)")
    ap.add_argument("--q8", action="store_true", help="--trace-decode: Q8_0 cache")
    ap.add_argument("--trace-server", action="store_true",
                    help="stage timeline of calls served by the host-call server (a -DL3P_DECODE_TRACE build)")
    ap.add_argument("--trace-tp", action="store_true",
                    help="(torchrun, N >= 2) stage timeline of the tensor-parallel wo sum (a -DL3P_DECODE_TRACE build)")
    ap.add_argument("--prefill-only", action="store_true", help="prefill measurement alone (ncu case)")
    ap.add_argument("--traffic", type=float, default=None,
                    help="ncu dram bytes per decode launch, if captured (reported as roofline.traffic)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.kernel_only:
        return run_kernel_only(args)
    if args.trace_decode:
        return run_decode_trace(args)
    if args.trace_server:
        return run_server_trace(args)
    if args.trace_tp:
        return run_tp_trace(args)
    if args.long:
        return run_long(args)
    if args.q8_only:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps({"mode": "q8-only", **run_q8(args, torch)}), flush=True)
        return 0
    if args.wo_only:
        import torch

        torch.cuda.set_device(0)
        print(json.dumps({"mode": "wo-only", **run_wo(args, torch)}), flush=True)
        return 0
    if args.prefill_only:
        import torch

        torch.cuda.set_device(0)
        line = config5(Job(torch, None, 1, 0, 0), max(args.steps // 2, 4), raw=not args.no_raw)
        print(json.dumps({"mode": "prefill-only", **line}), flush=True)
        return 0
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

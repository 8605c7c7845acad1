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
    the workload, each timed call = append row pos + attend, per layer."""

    def __init__(self, layers: int = 2):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O

        self.kind = "reference" if O.ref_available(fast=True) else "port"
        self.impl = "ref" if self.kind == "reference" else "port"
        self.sh = sh = CONFIGS[WORKLOAD]
        self.layers = layers
        self.o = O.Oracle(sh, O.MODE_Q8, self.impl, fast=True, n_layers=layers)
        self.rows = []
        for layer in range(layers):
            k, v, q = decode_inputs(sh, layer)
            self.o.load_kv(layer, 0, k[:, : sh.pos], v[:, : sh.pos])
            self.rows.append((q, np.ascontiguousarray(k[:, sh.pos]), np.ascontiguousarray(v[:, sh.pos])))
            del k, v
        self.threads = min(O.threads(self.impl, fast=True), sh.n_kv_heads)
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


def cpu_baseline(min_seconds: float = 10.0):
    host_threads_for_reference()
    ref = CpuReference(layers=CONFIGS[WORKLOAD].n_layers)
    dts = []
    while sum(dts) < min_seconds or len(dts) < 3:
        dts.append(ref.step())
    gbs = ref.bytes_per_layer * ref.layers * len(dts) / sum(dts) / 1e9
    out = {"value": round(gbs, 3), "unit": "GB/s", "cores": ref.threads, "kind": ref.kind,
           "sample": ref.describe(len(dts), sum(dts))}
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
    ref = CpuReference(layers=CONFIGS[WORKLOAD].n_layers)
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
                         "sample": ref.describe(len(dts), sum(dts))},
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
        if not args.no_wo and world == 1:
            # and on to the wo projection (Q8_0 weights, 4096 x 4096 per layer)
            from llama3pure_b200.synth import wo_weights

            w = wo_weights(8, sh.n_heads * sh.head_dim, sh.n_heads * sh.head_dim, seed=3)
            for layer in range(L):
                ctx.set_wo(layer, 8, w)
            xb2 = torch.zeros((L, sh.n_heads * sh.head_dim), device="cuda")
            bgraph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(rstream):
                ctx.set_stream(rstream)
                with torch.cuda.graph(bgraph, stream=rstream):
                    for layer in range(L):
                        ctx.step_raw_dev(layer, sh.pos, q[layer], knew[layer], vnew[layer], out[layer], rstream)
                        ctx.wo_dev(layer, out[layer], xb2[layer], rstream)
            stream.wait_stream(rstream)
            ctx.set_stream(stream)
            for _ in range(max(3, args.warmup)):
                bgraph.replay()
            torch.cuda.synchronize()
            r0.record(stream)
            for _ in range(args.steps):
                bgraph.replay()
            r1.record(stream)
            torch.cuda.synchronize()
            ctx.check()
            raw["with_wo_q8_0_us_per_layer"] = round(r0.elapsed_time(r1) / args.steps * 1e3 / L, 3)
            del bgraph
        if not args.no_wo and world > 1:
            # the tensor-parallel block: every rank's partial wo summed over NVLink (Q8_0, 4096 x 4096)
            from llama3pure_b200.synth import wo_weights

            dim = sh.n_heads * sh.head_dim
            w = wo_weights(8, dim, dim, seed=3)
            for layer in range(L):
                ctx.set_wo(layer, 8, w)
            h = ctx.tp_group_export(world, rank, dim)
            hs = [None] * world
            dist.all_gather_object(hs, h)
            ctx.tp_group_import(hs)
            xb2 = torch.zeros((L, dim), device="cuda")
            bgraph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(rstream):
                ctx.set_stream(rstream)
                with torch.cuda.graph(bgraph, stream=rstream):
                    for layer in range(L):
                        ctx.step_raw_dev(layer, sh.pos, q[layer], knew[layer], vnew[layer], out[layer], rstream)
                        ctx.wo_allreduce_dev(layer, out[layer], xb2[layer], rstream)
            stream.wait_stream(rstream)
            ctx.set_stream(stream)
            for _ in range(max(3, args.warmup)):
                bgraph.replay()
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            r0.record(stream)
            for _ in range(args.steps):
                bgraph.replay()
            r1.record(stream)
            torch.cuda.synchronize()
            ctx.check()
            t = torch.tensor([r0.elapsed_time(r1)], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            raw["with_wo_allreduce_q8_0_us_per_layer"] = round(t.item() / args.steps * 1e3 / L, 3)
            raw["wo_allreduce"] = "partial wo per rank, summed over NVLink peer stores (l3p_attn_wo_allreduce_dev)"
            del bgraph
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

    # end to end through the host-pointer C ABI (rank 0 at N GPUs: every rank runs it)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(ctx, sh, world, args, torch)
        if world > 1:
            t = torch.tensor([e2e["ms_per_step"]], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e["ms_per_step"] = t.item()
            e2e["value"] = round(bytes_per_layer_rank * world * L / (e2e["ms_per_step"] / 1e3) / 1e9, 3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline()
    q8 = None
    if rank == 0 and world == 1 and not args.no_q8:
        q8 = run_q8(args, torch)
    wo = None
    if rank == 0 and world == 1 and not args.no_wo:
        wo = run_wo(args, torch)
    prefill = None
    if rank == 0 and not args.no_prefill:
        prefill = run_prefill(args, torch)
        tf32 = measure_tf32_peak(torch)
        prefill["tf32_dense_tflops_measured"] = round(tf32, 1)
        prefill["roofline_3xtf32_tflops"] = round(tf32 / 3, 1)
        prefill["frac_of_3xtf32"] = round(prefill["tflops"] / (tf32 / 3), 4)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) fp32 q/K/V, generated on device)",
            "config": {"workload": WORKLOAD, "n_layers": L, "n_heads": sh.n_heads, "n_kv_heads": sh.n_kv_heads,
                       "head_dim": sh.head_dim, "pos": sh.pos, "kv_positions": P,
                       "parallelism": f"kv-head shards x{world}",
                       "launch": ("cuda graph" if graph else "stream") + ("" if args.no_overlap else " + programmatic dependent launch"),
                       "split_k": dict(zip(("ctas_per_kv_head", "cluster"), ctx.decode_plan(sh.pos))),
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
            "e2e": e2e,
            "cpu_baseline": cpu,
            "pre_attention_step": raw,
            "wo_projection": wo,
            "prefill": prefill,
            "q8_decode": q8,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    del graph
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


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


def measure_tf32_peak(torch):
    """Dense TF32 tensor throughput of this GPU, measured live: an fp32
    torch.matmul with TF32 enabled, 8192^3, best of 5 (2*N^3 flops).  The
    3xTF32 prefill roofline is a third of it."""
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


def run_prefill(args, torch):
    """Causal prefill of BASELINE configs[4] (Llama-3.1-8B shapes, 2048
    tokens, one layer per launch) through l3p_attn_prefill_dev."""
    from llama3pure_b200.attn import AttnContext
    from llama3pure_b200.synth import prefill_flops

    sh = CONFIGS["llama31_8b_prefill_2k"]
    S = sh.pos + 1
    L = 4  # layers cycled (16 MiB of K/V each)
    ctx = AttnContext.for_shape(sh, n_layers=L)
    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    q = torch.randn((L, S, sh.n_heads, sh.head_dim), device="cuda", generator=g)
    k = torch.randn((L, S, sh.n_kv_heads, sh.head_dim), device="cuda", generator=g)
    v = torch.randn((L, S, sh.n_kv_heads, sh.head_dim), device="cuda", generator=g)
    out = torch.zeros_like(q)
    for i in range(args.warmup):
        ctx.prefill_dev(i % L, 0, S, q[i % L], k[i % L], v[i % L], out[i % L], stream)
    torch.cuda.synchronize()
    reps = max(args.steps // 2, 4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(reps):
        ctx.prefill_dev(i % L, 0, S, q[i % L], k[i % L], v[i % L], out[i % L], stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ctx.check()
    ms = e0.elapsed_time(e1) / reps
    tflops = prefill_flops(sh) / (ms / 1e3) / 1e12
    res = {"workload": "llama31_8b_prefill_2k", "ms_per_layer": round(ms, 4), "tflops": round(tflops, 2),
           "flops_per_layer": prefill_flops(sh), "kernel": "prefill_tc_kernel (tcgen05 3xTF32) + prefill_prep_kernel"}
    if not getattr(args, "no_raw", False):
        # from the raw projections: RoPE + cache write in the pre-attention kernel
        ctx.set_rope()
        for i in range(args.warmup):
            ctx.prefill_raw_dev(i % L, 0, S, q[i % L], k[i % L], v[i % L], out[i % L], stream)
        torch.cuda.synchronize()
        e0.record(stream)
        for i in range(reps):
            ctx.prefill_raw_dev(i % L, 0, S, q[i % L], k[i % L], v[i % L], out[i % L], stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.check()
        res["raw_ms_per_layer"] = round(e0.elapsed_time(e1) / reps, 4)
        res["raw_api"] = "l3p_attn_prefill_raw_dev (RoPE + cache write, then prep + attention)"
    ctx.close()
    return res


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
    for name, wt, nbytes in (("q8_0", 8, cols // 32 * 34), ("q4_k", 12, cols // 256 * 144),
                             ("q6_k", 14, cols // 256 * 210)):
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


def run_e2e(ctx, sh, world, args, torch):
    """l3p_attn_step per layer with pinned host buffers: H2D of q/k/v, append,
    decode, D2H of the output, every step."""
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

    for _ in range(max(3, args.warmup)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    r0, r1 = ctx.owned_rows
    h2d = L * ((r1 - r0) * sh.head_dim + 2 * sh.n_kv_heads * sh.head_dim) * 4
    d2h = L * (r1 - r0) * sh.head_dim * 4
    hk = ctx.kv_head_count
    bytes_step = 2 * (sh.pos + 1) * hk * sh.head_dim * 4 * L * world
    return {"value": round(bytes_step / dt / 1e9, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(dt * 1e3, 4),
            "api": "l3p_attn_step (host pointers, pinned)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-overlap", action="store_true", help="no programmatic dependent launch between layers")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-q8", action="store_true", help="skip the Q8_0-cache decode measurement")
    ap.add_argument("--no-raw", action="store_true", help="skip the raw-projection (RoPE on device) measurements")
    ap.add_argument("--no-wo", action="store_true", help="skip the wo projection measurement")
    ap.add_argument("--wo-only", action="store_true", help="wo projection measurement alone (ncu case)")
    ap.add_argument("--long", action="store_true", help="BASELINE configs[2] (128K context) over --gpus ranks")
    ap.add_argument("--seq-parts", type=int, default=1, help="--long: sequence parts per head group")
    ap.add_argument("--xchg", default="nvlink", choices=["nvlink", "nccl"],
                    help="--long: exchange of the sequence parts' partials")
    ap.add_argument("--q8-only", action="store_true", help="Q8_0-cache decode measurement alone")
    ap.add_argument("--kernel-only", action="store_true", help="decode kernel alone on --layers layers (ncu case)")
    ap.add_argument("--layers", type=int, default=4)
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
        line = run_prefill(args, torch)
        line["tf32_dense_tflops_measured"] = round(measure_tf32_peak(torch), 1)
        print(json.dumps({"mode": "prefill-only", **line}), flush=True)
        return 0
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

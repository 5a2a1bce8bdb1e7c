#!/usr/bin/env python
"""Benchmark of the B200 ternary BitLinear path (decode GEMV sweep, config 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Step: the BitLinear forwards of a BitNet-b1.58-2B decoder for every batch size
of the sweep: for B in {1, 8, 32, 64}, 30 layers x 5 projections (fused QKV
3840x2560, o 2560x2560, gate 6912x2560, up 6912x2560, down 2560x6912), each a
fused RMSNorm + per-token int8 quantize + ternary matmul through the C ABI.
The 150 weight matrices (521 MB packed) exceed L2, so every pass streams them
from HBM. Each B is one CUDA graph of the 150 forwards (captured through the
public API), replayed per step.

value  = algorithmic bytes of the step / device time (GB/s, summed over ranks);
         bytes per forward = M*K/4 + B*K*4 + K*4 + B*M*4 + 4.
e2e    = the same through host buffers: per step one H2D copy of all inputs
         from pinned memory and one D2H copy of all outputs, timed with the
         graph replays (double-buffered on a copy stream, so a step's copies
         overlap its neighbours' kernels).
Multi-GPU (torchrun): independent decode sequences per GPU, full weight
replicas, no collective on the data path (weak scaling); the max over ranks
of the device time is reported.

--impl reference times the reference algorithm's CPU restatement (oracle/,
OpenMP over all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ternary decode GEMV GB/s"
BATCHES = (1, 8, 32, 64)
LAYERS = 30


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--layers", type=int, default=LAYERS)
    p.add_argument("--batches", type=str, default=",".join(map(str, BATCHES)))
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--prefill", type=str, default="512,2048,8192",
                   help="config-2 token counts for the prefill TOPS block ('' to skip)")
    p.add_argument("--no-generate", dest="generate", action="store_false",
                   help="skip the end-to-end model (GGUF -> oxbitnet_generate_ids) run")
    p.add_argument("--no-decoder", dest="decoder", action="store_false",
                   help="skip the config-3 decoder tok/s block")
    p.add_argument("--tp-tokens", type=int, default=16384,
                   help="config-4 tensor-parallel prefill tokens when run on N > 1 GPUs (0 skips)")
    p.add_argument("--case", type=str, default=None,
                   help="SHAPE:B — run a few forwards of one 2B shape (or of 'all' five in "
                        "turn; or 'lmhead' / 'attn' / 'attnpf' / 'attndec' / 'decoder' / 'prefill' / "
                        "'prefilltrace' / 'gateup' / 'quant' / 'mmarate') at B and exit (a "
                        "small, self-contained workload for ncu captures)")
    return p.parse_args()


def synthetic_standalone():
    """The package's pure-numpy generators (0xbitnet_b200/synthetic.py and i2s.py),
    loaded by file path under a private package name so that the CPU legs never run
    the package __init__, which maps libobn.so."""
    import importlib.util
    import types
    name = "_obn_synthetic_pkg"
    if name + ".synthetic" in sys.modules:
        return sys.modules[name + ".synthetic"]
    pkg_dir = os.path.join(ROOT, "0xbitnet_b200")
    pkg = types.ModuleType(name)
    pkg.__path__ = [pkg_dir]
    sys.modules[name] = pkg
    for sub in ("i2s", "synthetic"):
        spec = importlib.util.spec_from_file_location(f"{name}.{sub}",
                                                      os.path.join(pkg_dir, sub + ".py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = mod
        spec.loader.exec_module(mod)
        setattr(pkg, sub, mod)
    return sys.modules[name + ".synthetic"]


def shapes():
    return list(synthetic_standalone().SHAPES_2B.items())


def fwd_bytes(M: int, K: int, B: int) -> int:
    return M * K // 4 + B * K * 4 + K * 4 + B * M * 4 + 4


def gemv_kernel_bytes(M: int, K: int, B: int) -> int:
    # matmul kernel alone: packed weights + int8 activations + per-token scale
    # and code sum + per-row scales + f32 output
    return M * K // 4 + B * K + 8 * B + 4 * M + 4 * B * M


def config(args, world):
    return {
        "workload": "cfg1 decode GEMV sweep: B in {%s} x %d layers x 5 BitNet-2B BitLinear shapes "
                    "(qkv 3840x2560, o 2560x2560, gate 6912x2560, up 6912x2560, down 2560x6912); "
                    "fused RMSNorm + int8 absmax quantize + ternary matmul per forward"
                    % (args.batches, args.layers),
        "batches": [int(b) for b in args.batches.split(",")],
        "layers": args.layers,
        "weights_bytes_per_pass": sum(M * K // 4 for _, (M, K) in shapes()) * args.layers,
        "l2": "inputs larger than L2: each batch pass streams 521 MB of packed weights",
        "parallelism": f"dp{world} (independent decode sequences per GPU, no collective)",
    }


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[4:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i - 1] for r in rows for i in range(1, 5)
                          if r[3][i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows),
                "samples": len(rows), "reasons": reasons}


# ----------------------------------------------------------------------------- CPU baseline
def host_threads() -> int:
    # torchrun exports OMP_NUM_THREADS=1; the CPU baseline is timed on every core
    # this process may run on instead.
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def reference_sample(args):
    """1 layer x 5 shapes x every B of the sweep, seeded; numpy only (no libobn)."""
    synth = synthetic_standalone()
    batches = [int(b) for b in args.batches.split(",")]
    data = []
    for i, (name, (M, K)) in enumerate(shapes()):
        L = synth.layer(900 + i, M, K)
        xs = {B: synth.activations(950 + i * 10 + B, B, K) for B in batches}
        data.append((M, K, L, xs))
    step_bytes = sum(fwd_bytes(M, K, B) for M, K, _, _ in data for B in batches)
    return batches, data, step_bytes


def time_oracle(data, batches, threads, min_seconds, max_reps):
    """Repetitions of the sample through the oracle's BitLinear: the literal
    single-thread restatement (threads == 1) or its OpenMP form (row-parallel,
    identical results). Returns (reps, seconds)."""
    import oracle as orc

    def rep():
        for M, K, L, xs in data:
            for B in batches:
                if threads == 1:
                    orc.bitlinear(xs[B], L.packed, L.row_scales(), M, K, norm_w=L.gamma)
                else:
                    orc.bitlinear_omp(xs[B], L.packed, L.row_scales(), M, K, norm_w=L.gamma,
                                      threads=threads)
    rep()  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        rep()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or reps >= max_reps:
            return reps, el


def cpu_sample(args, min_seconds=10.0, max_reps=50):
    """Times the oracle on 1 layer x 5 shapes x every B: OpenMP over all host
    threads (the reported value) and the literal single-thread build beside it."""
    batches, data, bytes_per_rep = reference_sample(args)
    threads = host_threads()
    reps, el = time_oracle(data, batches, threads, min_seconds, max_reps)
    reps1, el1 = time_oracle(data, batches, 1, min_seconds / 2, max_reps)
    return {"value": bytes_per_rep * reps / el / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"1 layer x 5 shapes x B in {{{args.batches}}} ({reps} reps, "
                      f"{el:.1f} s): the oracle's C restatement of the WGSL kernels, OpenMP",
            "single_thread": {"value": bytes_per_rep * reps1 / el1 / 1e9, "unit": "GB/s",
                              "cores": 1, "kind": "port",
                              "sample": f"same sample, literal single-thread build "
                                        f"({reps1} reps, {el1:.1f} s)"}}


def run_reference(args):
    """The reference algorithm on the host cores: the oracle's C restatement of
    the WGSL kernels (OpenMP over all host threads), one layer x 5 shapes x every
    B per step. Nothing here imports the 0xbitnet_b200 package or maps libobn.so."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle as orc
    batches, data, step_bytes = reference_sample(args)
    threads = host_threads()

    def step():
        for M, K, L, xs in data:
            for B in batches:
                orc.bitlinear_omp(xs[B], L.packed, L.row_scales(), M, K, norm_w=L.gamma,
                                  threads=threads)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = step_bytes * args.steps / el / 1e9
    reps1, el1 = time_oracle(data, batches, 1, 5.0, 10)
    sample = (f"each step: 1 of the {args.layers} layers (5 shapes) x B in {{{args.batches}}}, "
              f"{step_bytes} algorithmic bytes; oracle C restatement, OpenMP")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded)",
        "config": config(args, world),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample,
                         "single_thread": {"value": step_bytes * reps1 / el1 / 1e9,
                                           "unit": "GB/s", "cores": 1, "kind": "port",
                                           "sample": f"same step, literal single-thread build "
                                                     f"({reps1} reps, {el1:.1f} s)"}},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- ours
def load_profile_traffic():
    """DRAM traffic of the dominant kernel from the committed ncu summary
    (profiles/traffic.json: batch, kernel, dram_bytes_per_launch), or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        return json.load(open(path))
    except (OSError, ValueError):
        return None


def measure_int8_peak(dev) -> float:
    """Dense int8 tensor throughput of this GPU: torch._int_mm 8192^3, best of 10."""
    import torch
    a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b)
    best = float("inf")
    for _ in range(10):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return 2.0 * 8192 ** 3 / (best / 1e3) / 1e12


def measure_prefill(args, obn, synth, dev, stream):
    """Config 2: the 5 BitNet-2B shapes at M_tok prefill tokens (one layer's
    weights each), timed as the tcgen05 GEMM alone and as the full BitLinear
    forward (RMSNorm + quantize + GEMM), in TOPS = 2*M_tok*M*K / time."""
    import torch
    toks = [int(t) for t in args.prefill.split(",") if t]
    peak = measure_int8_peak(dev)
    shp = shapes()
    layers = []
    for i, (name, (M, K)) in enumerate(shp):
        packed, s_w, gamma = synth.layer_device(20_000 + i, M, K, dev)
        layers.append(obn.BitLinear(packed, s_w, gamma, K, M))
    out = {"int8_peak_tops": peak, "int8_peak_how": "torch._int_mm 8192^3 best of 10 (cuBLASLt)",
           "gemm_tops": {}, "forward_tops": {}}
    for T in toks:
        ops = sum(2.0 * T * M * K for _, (M, K) in shp)
        xs = [torch.randn(T, K, device=dev) for _, (M, K) in shp]
        ys = [torch.empty(T, M, device=dev) for _, (M, K) in shp]
        with torch.cuda.stream(stream):
            qin = [obn.rmsnorm_quantize(x) for x in xs]
            for i, L in enumerate(layers):
                L.forward(xs[i], out=ys[i])
            stream.synchronize()
            res = {}
            for mode in ("gemm", "forward"):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for i, L in enumerate(layers):
                        if mode == "gemm":
                            q, sc, qs = qin[i]
                            obn._lib.check(obn.lib().obn_ternary_matmul(
                                L.handle, q.data_ptr(), sc.data_ptr(), qs.data_ptr(), T,
                                ys[i].data_ptr(), stream.cuda_stream))
                        else:
                            L.forward(xs[i], out=ys[i])
                for _ in range(2):
                    g.replay()
                stream.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                reps = 5
                e0.record(stream)
                for _ in range(reps):
                    g.replay()
                e1.record(stream)
                stream.synchronize()
                res[mode] = ops / (e0.elapsed_time(e1) / reps / 1e3) / 1e12
                del g
        out["gemm_tops"][str(T)] = res["gemm"]
        out["forward_tops"][str(T)] = res["forward"]
        del xs, ys, qin
    best = max(out["gemm_tops"].values()) if out["gemm_tops"] else 0.0
    out["gemm_frac_of_int8_peak"] = best / peak if peak else None
    for L in layers:
        L.close()
    torch.cuda.synchronize()
    return out


def measure_tp_prefill(args, obn, synth, dev, stream, world, rank):
    """Config 4 on N > 1 GPUs: the 3B-class shapes (hidden 3072, FFN 9216; QKV
    assumed MHA 9216x3072), --tp-tokens prefill tokens, one layer of 5 BitLinears,
    output features split over the ranks and gathered on every rank. Two forms:
    "fused" = obn_bitlinear_forward_tp (each GEMM epilogue stores its columns into
    every rank's output, NVLS multicast when the group has it, else peer stores)
    + one stream barrier; "nccl" = the same row-slice GEMM into a local buffer,
    NCCL all_gather_into_tensor, re-layout to [tokens, out] on every rank. Whole-job
    TOPS = sum 2*T*M*K / device time (max over ranks)."""
    import torch
    import torch.distributed as dist
    tp = importlib.import_module("0xbitnet_b200.tp")
    T = args.tp_tokens
    shp = list(synth.SHAPES_3B.items())
    parts, outs, xs, locs, gath = [], [], [], [], []
    for i, (name, (M, K)) in enumerate(shp):
        L = synth.layer(30_000 + i, M, K)  # seeded: identical on every rank
        parts.append(tp.TPBitLinear(L.blob(), K, M, world, rank, norm_weight=L.gamma,
                                    device=dev.index))
        outs.append(tp.GatherOutput(T, M, device=dev))
        g = torch.Generator(device=dev)
        g.manual_seed(31_000 + i)
        xs.append(torch.randn(T, K, generator=g, device=dev))
        locs.append(torch.empty(T, M // world, device=dev))
        gath.append(torch.empty(world, T, M // world, device=dev))
    ops = sum(2.0 * T * M * K for _, (M, K) in shp)
    has_mc = bool(outs[0].mc_ptr)

    def fused(mc=False):
        for i in range(len(shp)):
            parts[i].forward(xs[i], outs[i], multicast=mc)
        outs[-1].barrier()  # one stream barrier after all five gathered GEMMs

    def local():
        for i in range(len(shp)):
            parts[i].layer.forward(xs[i], out=locs[i])

    def nccl():
        for i, (name, (M, K)) in enumerate(shp):
            parts[i].layer.forward(xs[i], out=locs[i])
            dist.all_gather_into_tensor(gath[i], locs[i])
            outs[i].view(T).view(T, world, M // world).copy_(gath[i].permute(1, 0, 2))

    def timed(fn, reps=3):
        with torch.cuda.stream(stream):
            fn()
            stream.synchronize()
            dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            stream.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # parity: the gathered output equals the NCCL all-gather of the same slices
    with torch.cuda.stream(stream):
        nccl()
        stream.synchronize()
        ref = [o.view(T).clone() for o in outs]
        for o in outs:
            o.view(T).fill_(float("nan"))
        outs[-1].barrier()
        fused(has_mc)
        stream.synchronize()
    same = all(torch.equal(o.view(T), r) for o, r in zip(outs, ref))
    if has_mc:  # and the peer-store form
        with torch.cuda.stream(stream):
            for o in outs:
                o.view(T).fill_(float("nan"))
            outs[-1].barrier()
            fused(False)
            stream.synchronize()
        same = same and all(torch.equal(o.view(T), r) for o, r in zip(outs, ref))
    flag = torch.tensor([1 if same else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    del ref
    peers_ms = timed(lambda: fused(False))
    mc_ms = timed(lambda: fused(True)) if has_mc else None
    fused_ms = min(peers_ms, mc_ms) if mc_ms is not None else peers_ms
    nccl_ms = timed(nccl)
    local_ms = timed(local)
    # NVLink bound: every rank must receive (world-1)/world of each f32 output
    ingress = sum(T * M * 4 * (world - 1) / world for _, (M, K) in shp)
    out = {
        "workload": "config 4: 3B-class shapes (hidden 3072, FFN 9216, QKV assumed MHA "
                    "9216x3072), %d tokens, 1 layer x 5 BitLinears, output features split "
                    "over %d GPUs and gathered on every rank" % (T, world),
        "tokens": T, "world": world,
        "fused_form": "NVLS multicast stores" if fused_ms == mc_ms else "peer stores over NVLink",
        "fused_ms": fused_ms, "fused_tops": ops / (fused_ms / 1e3) / 1e12,
        "fused_peer_stores_ms": peers_ms, "fused_multicast_ms": mc_ms,
        "nccl_allgather_ms": nccl_ms, "nccl_allgather_tops": ops / (nccl_ms / 1e3) / 1e12,
        "local_gemm_ms": local_ms,
        "nvlink_ingress_bytes_per_gpu": ingress,
        "nvlink_bound_ms": ingress / 770e9 * 1e3,
        "parity_bitexact_vs_nccl": bool(flag.item()),
    }
    for p_ in parts:
        p_.close()
    del outs, xs, locs, gath
    torch.cuda.synchronize()
    dist.barrier()
    return out


def measure_ffn_gate_up(args, obn, synth, dev, stream, batches):
    """Next-row measurement: the FFN's gate and up projections of BitNet-2B (6912x2560
    each) for 30 layers, as the reference runs them (two BitLinear forwards on the
    same input, each quantizing it) against the merged gated layer (one quantize, one
    matmul over the interleaved rows, ReLU^2 x up fused: one more pass than nothing,
    two fewer than the reference's activation + multiply). Device time per layer."""
    import torch
    M, K = synth.SHAPES_2B["gate"]
    nl = args.layers
    sep, merged = [], []
    for l in range(nl):
        g = synth.layer(50_000 + 2 * l, M, K)
        u = synth.layer(50_001 + 2 * l, M, K)
        sep.append((obn.BitLinear.from_i2s(g.blob(), K, M, norm_weight=g.gamma, device=dev.index),
                    obn.BitLinear.from_i2s(u.blob(), K, M, norm_weight=g.gamma, device=dev.index)))
        merged.append(obn.BitLinear.from_i2s_gated(g.blob(), u.blob(), K, M, norm_weight=g.gamma,
                                                   device=dev.index))
    out = {"shape": [M, K], "layers": nl, "per_batch": {}}
    # the decode batches, then two prefill chunk sizes (tensor-core GEMM epilogue)
    for B in list(batches) + [512, 2048]:
        x = torch.randn(B, K, device=dev)
        yg, yu, ym = (torch.empty(B, M, device=dev) for _ in range(3))

        def run_sep():
            for a, b in sep:
                a.forward(x, out=yg)
                b.forward(x, out=yu)

        def run_merged():
            for L in merged:
                L.forward(x, out=ym)
        res = {}
        for name, fn in (("separate_gate_up_us", run_sep), ("merged_gated_us", run_merged)):
            with torch.cuda.stream(stream):
                fn()
                stream.synchronize()
                gph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gph, stream=stream):
                    fn()
                for _ in range(3):
                    gph.replay()
                stream.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                reps = 10
                e0.record(stream)
                for _ in range(reps):
                    gph.replay()
                e1.record(stream)
                stream.synchronize()
                res[name] = e0.elapsed_time(e1) * 1e3 / (reps * nl)
                del gph
        res["speedup"] = res["separate_gate_up_us"] / res["merged_gated_us"]
        out["per_batch"][str(B)] = res
    for a, b in sep:
        a.close()
        b.close()
    for L in merged:
        L.close()
    torch.cuda.synchronize()
    return out


def measure_attention(dev, stream, peak, layers):
    """Next-row kernels: one decode step's attention for BitNet-2B (20 heads, 5 KV
    heads, head_dim 128) at context 2048 over `layers` layers, fp16 KV: RoPE + KV
    append of the new token fused into the split-KV attention for small batches
    (obn_attention_decode_rope), a separate RoPE pass before it for large ones, then
    the combine. Bytes per layer and
    sequence = the K and V cache read (2 * 2048 * 5 * 128 * 2) + q, out, new k/v."""
    import torch
    att = importlib.import_module("0xbitnet_b200.attention")
    H, Hkv, Dh, ctx = 20, 5, 128, 2048
    out = {"heads": H, "kv_heads": Hkv, "head_dim": Dh, "context": ctx, "layers": layers,
           "per_batch": {}}
    for B in (1, 64):
        caches = [att.KVCache(B, ctx, Hkv, Dh, device=dev) for _ in range(layers)]
        for c in caches:
            c.k.normal_()
            c.v.normal_()
            c.seq_len = ctx - 1
        qkv = torch.randn(B, (H + 2 * Hkv) * Dh, device=dev)

        fused = B <= importlib.import_module("0xbitnet_b200.decoder").FUSED_ROPE_MAX_BATCH

        def step():  # the decoder's path for this batch size
            for c in caches:
                if fused:
                    att.attention_rope(qkv, c, H, ctx - 1)
                else:
                    q = att.rope_kv_append(qkv, c, H, 1)
                    att.attention(q, c, H, 1, ctx)
        with torch.cuda.stream(stream):
            step()
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step()
            for _ in range(3):
                g.replay()
            stream.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = 10
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            stream.synchronize()
            del g
        us = e0.elapsed_time(e1) * 1e3 / (reps * layers)
        nbytes = B * (2 * ctx * Hkv * Dh * 2 + (H + 2 * Hkv) * Dh * 4 + H * Dh * 8)
        out["per_batch"][str(B)] = {"us_per_layer": us, "bytes_per_layer": nbytes,
                                    "achieved_gbs": nbytes / (us * 1e-6) / 1e9,
                                    "frac": nbytes / (us * 1e-6) / 1e9 / peak}
        del caches
    torch.cuda.synchronize()
    return out


def measure_decoder(dev, stream, world, rank, ctx=2048, total_batch=64):
    """Config 3: one decode step of the random-init BitNet-2B-class decoder (30
    layers, hidden 2560, FFN 6912 ReLU^2-gated, 20/5 heads x 128, RoPE 500000,
    fp16 KV cache at context `ctx`, tied fp16 embedding / LM head, vocab 128256).
    Batch 1 on every rank, and `total_batch` sequences sharded over the ranks
    (total_batch / world each, no collective). tok/s = sequences / step time
    (max over ranks for the sharded batch)."""
    import torch
    import torch.distributed as dist
    D_ = importlib.import_module("0xbitnet_b200.decoder")
    cfg = D_.DecoderConfig()
    out = {"config": "30 layers, hidden 2560, FFN 6912, 20/5 heads x 128, vocab 128256, "
                     "fp16 KV cache, context %d" % ctx, "per_batch": {}}
    for B, sharded in ((1, False), (max(1, total_batch // world), True)):
        m = D_.BitNetDecoder(cfg, B, ctx, device=dev, seed=70_000)
        m.fill_caches(ctx - 1, seed=70_001)
        with torch.cuda.stream(stream):
            m.step(ctx - 1)  # warm-up outside the graph: workspaces
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                m.step(ctx - 1)
            for _ in range(3):
                g.replay()
            stream.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = 10
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            stream.synchronize()
            del g
        ms = e0.elapsed_time(e1) / reps
        if sharded and world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        key = "sharded_%d_over_%d_gpus" % (B * world, world) if sharded else "1"
        seqs = B * world if sharded else B
        out["per_batch"][key] = {"ms_per_step": ms, "tokens_per_s": seqs / (ms / 1e3),
                                 "sequences": seqs}
        m.close()
        del m
        torch.cuda.synchronize()
    return out


def measure_generate(dev):
    """Config 3 end to end through the drop-in model ABI (include/oxbitnet.h): a
    random-init BitNet-2B GGUF (the reference's tensor names, I2_S ternary
    weights, f16 tied embedding, synthetic 128256-token vocabulary) is written to
    a temporary file, loaded with oxbitnet_load, and driven with
    oxbitnet_forward (prefill) and oxbitnet_generate_ids (sampling with the
    reference's default options: T 1.0, top-k 50, penalty 1.1 over 64 tokens).
    Decode tok/s = generated tokens / wall time between the first and the last
    token (host sampling and the per-token callback included)."""
    import shutil
    import tempfile

    import numpy as np
    W = importlib.import_module("0xbitnet_b200.gguf_writer")
    ox = importlib.import_module("0xbitnet_b200.oxbitnet")
    tmp = tempfile.mkdtemp(prefix="obn_gguf_")
    out = {"model": "BitNet-2B shape (30 layers, 2560/6912, 20/5 heads x 128, vocab 128256), "
                    "random weights, through oxbitnet_load / oxbitnet_forward / "
                    "oxbitnet_generate_ids"}
    try:
        path = os.path.join(tmp, "bitnet2b.gguf")
        t0 = time.perf_counter()
        toks, merges, bos, eos = W.synthetic_vocab(128256)
        W.write_bitnet_model(path, W.BitNetShape(), toks, merges, bos, eos, seed=0, fast=True)
        out["file_gb"] = os.path.getsize(path) / 1e9
        t1 = time.perf_counter()
        m = ox.BitNet.load_sync(path)
        out["load_s"] = time.perf_counter() - t1
        out["write_s"] = t1 - t0
        rng = np.random.default_rng(0)
        prompt = [bos] + [int(x) for x in rng.integers(0, 128000, 511)]
        m.forward(prompt, reset=True)
        ts = []
        for _ in range(3):
            t = time.perf_counter()
            m.forward(prompt, reset=True)
            ts.append(time.perf_counter() - t)
        out["prefill_tokens"] = len(prompt)
        out["prefill_ms"] = min(ts) * 1e3
        out["prefill_tok_s"] = len(prompt) / min(ts)
        m.set_seed(1)
        m.generate_ids(prompt[:16], max_tokens=8)  # warm-up (captures the decode graph)
        stamps = []
        n_new = 256

        def timed(ids, max_tokens):
            got = []
            L = ox.lib()

            def cb(i, _p, _n, _ud):
                stamps.append(time.perf_counter())
                got.append(i)
                return 0
            c = ox.TokenIdFn(cb)
            arr = (ox._U32 * len(ids))(*ids)
            o = ox.GenerateOptions(max_tokens, 1.0, 50, 1.1, 64)
            if L.oxbitnet_generate_ids(m._handle(), arr, len(ids), ox.ctypes.byref(o), c,
                                       None) != 0:
                raise RuntimeError(ox.error_message())
            return got
        best = None
        for _ in range(2):
            stamps.clear()
            got = timed(prompt[:16], n_new)
            if len(got) > 1:
                rate = (len(got) - 1) / (stamps[-1] - stamps[0])
                best = rate if best is None else max(best, rate)
        out["decode_tokens"] = n_new
        out["decode_tok_s"] = best
        out["decode_ms_per_token"] = 1e3 / best if best else None
        m.dispose()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return out


def measure_lm_head(obn, dev, stream, peak):
    """Next-row kernel: the f16 LM head of BitNet-2B (128256 x 2560, 656.7 MB) behind
    the final RMSNorm, one token as the reference runs it; the table exceeds L2, so
    every launch streams it from HBM. Bytes per launch = V*D*2 + D*4 (x) + D*4
    (gamma) + V*4 (logits)."""
    import torch
    V, D = 128256, 2560
    g = torch.Generator(device=dev)
    g.manual_seed(40_000)
    embed = (torch.randn(V, D, generator=g, device=dev) * 0.05).to(torch.float16)
    x = torch.randn(1, D, generator=g, device=dev)
    gamma = 1 + 0.1 * torch.randn(D, generator=g, device=dev)
    with torch.cuda.stream(stream):
        for _ in range(3):
            obn.lm_head_f16(embed, x, gamma)
        stream.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = 20
        e0.record(stream)
        for _ in range(reps):
            obn.lm_head_f16(embed, x, gamma)
        e1.record(stream)
        stream.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    nbytes = V * D * 2 + D * 8 + V * 4
    ach = nbytes / (us * 1e-6) / 1e9
    del embed
    return {"kernel": "k_lm_head_f16<1> (final RMSNorm + f16 LM head GEMV, 1 token)",
            "shape": [V, D], "bytes_per_launch": nbytes, "avg_launch_us": us,
            "achieved_gbs": ach, "peak_gbs": peak, "frac": ach / peak,
            "tokens_per_s": 1e6 / us}


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and "WORLD_SIZE" in os.environ:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    obn = importlib.import_module("0xbitnet_b200")
    synth = importlib.import_module("0xbitnet_b200.synthetic")
    batches = [int(b) for b in args.batches.split(",")]
    shp = shapes()

    # Weights: one replica per GPU (independent decode sequences need no exchange).
    layers = []
    for l in range(args.layers):
        row = []
        for i, (name, (M, K)) in enumerate(shp):
            packed, s_w, gamma = synth.layer_device(10_000 + 10 * l + i, M, K, dev)
            row.append(obn.BitLinear(packed, s_w, gamma, K, M))
            del packed
        layers.append(row)
    torch.cuda.synchronize()

    # Activations: flat device buffers so the e2e copies are one H2D + one D2H per step.
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    x_total = sum(B * K for B in batches for _, (M, K) in shp)
    y_total = sum(B * M for B in batches for _, (M, K) in shp)
    x_flat = torch.randn(x_total, generator=gen, device=dev)
    y_flat = torch.empty(y_total, device=dev)
    xs, ys = {}, {}
    xo = yo = 0
    for B in batches:
        for i, (name, (M, K)) in enumerate(shp):
            xs[B, i] = x_flat[xo:xo + B * K].view(B, K)
            ys[B, i] = y_flat[yo:yo + B * M].view(B, M)
            xo += B * K
            yo += B * M

    def views(xf, yf):
        vx, vy = {}, {}
        xo = yo = 0
        for B in batches:
            for i, (name, (M, K)) in enumerate(shp):
                vx[B, i] = xf[xo:xo + B * K].view(B, K)
                vy[B, i] = yf[yo:yo + B * M].view(B, M)
                xo += B * K
                yo += B * M
        return vx, vy

    def capture(vx, vy):
        gs = {}
        for B in batches:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for row in layers:
                    for i, L in enumerate(row):
                        L.forward(vx[B, i], out=vy[B, i])
            gs[B] = g
        return gs

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for B in batches:  # eager warm-up allocates every layer's workspace
            for row in layers:
                for i, L in enumerate(row):
                    L.forward(xs[B, i], out=ys[B, i])
        stream.synchronize()
        graphs = capture(xs, ys)
    torch.cuda.synchronize()
    obn.check_device_errors()

    step_bytes = {B: args.layers * sum(fwd_bytes(M, K, B) for _, (M, K) in shp) for B in batches}
    # B = 1: one fused kernel per forward; B > 1: RMSNorm+quantize, then the matmul.
    launches_per_step = sum(1 if B == 1 else 2 for B in batches) * args.layers * len(shp)

    def step(evs=None, gs=None):
        gs = graphs if gs is None else gs
        for j, B in enumerate(batches):
            if evs is not None:
                evs[j][0].record(stream)
            gs[B].replay()
            if evs is not None:
                evs[j][1].record(stream)

    clocks = ClockSampler(local)
    clocks.start()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
        stream.synchronize()
        barrier()
        per_b_ms = {B: 0.0 for B in batches}
        evs_all = []
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t_start.record(stream)
        for _ in range(args.steps):
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in batches]
            step(evs)
            evs_all.append(evs)
        t_end.record(stream)
        torch.cuda.synchronize()
        barrier()
    clock_info = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    for evs in evs_all:
        for j, B in enumerate(batches):
            per_b_ms[B] += evs[j][0].elapsed_time(evs[j][1])
    total_ms_max = max_over_ranks(total_ms)
    bytes_all = world * args.steps * sum(step_bytes.values())
    value = bytes_all / (total_ms_max / 1e3) / 1e9

    # e2e: every step copies its inputs from pinned host memory to the device and
    # its outputs back, as a serving loop would: two sets of device buffers (one
    # graph set each) and a copy stream, so step k's H2D overlaps step k-1's
    # kernels and its D2H overlaps step k+1's. The timed region runs from before
    # the first H2D to after the last D2H.
    x_host = torch.empty(x_total, dtype=torch.float32, pin_memory=True)
    x_host.copy_(x_flat.cpu())
    y_host = [torch.empty(y_total, dtype=torch.float32, pin_memory=True) for _ in range(2)]
    x_dev = [x_flat, torch.empty_like(x_flat)]
    y_dev = [y_flat, torch.empty_like(y_flat)]
    with torch.cuda.stream(stream):
        graph_sets = [graphs, capture(*views(x_dev[1], y_dev[1]))]
    torch.cuda.synchronize()
    h2d = torch.cuda.Stream(device=dev)  # inputs in, one stream per direction so a
    d2h = torch.cuda.Stream(device=dev)  # step's outputs never queue before the next inputs

    def e2e_steps(count):
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        h2d.wait_stream(stream)
        d2h.wait_stream(stream)

        def load(k):
            j = k & 1
            with torch.cuda.stream(h2d):
                if k >= 2:
                    h2d.wait_event(ev_done[j])  # step k - 2 has read x_dev[j]
                x_dev[j].copy_(x_host, non_blocking=True)
                ev_in[j].record(h2d)

        load(0)
        for k in range(count):
            j = k & 1
            if k + 1 < count:
                load(k + 1)  # overlaps step k's kernels
            stream.wait_event(ev_in[j])
            if k >= 2:
                stream.wait_event(ev_out[j])  # step k - 2's outputs have left y_dev[j]
            step(gs=graph_sets[j])
            ev_done[j].record(stream)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_done[j])
                y_host[j].copy_(y_dev[j], non_blocking=True)  # overlaps step k + 1's kernels
                ev_out[j].record(d2h)
        for j in range(min(2, count)):
            stream.wait_event(ev_out[j])

    with torch.cuda.stream(stream):
        e2e_steps(max(1, args.warmup))
        stream.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_steps(args.steps)
        e1.record(stream)
        stream.synchronize()
        barrier()
    if not torch.equal(y_host[(args.steps - 1) & 1], y_flat.cpu()):
        raise RuntimeError("e2e outputs differ from the device-timed run's")
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = bytes_all / (e2e_ms / 1e3) / 1e9

    # Per-batch kernel timings. B = 1 runs one fused kernel per forward, so its
    # step graph is the kernel alone; for B > 1 the matmul kernel (dp4a GEMV or
    # tcgen05 GEMM) is timed alone over the same 150 weights with pre-quantized
    # activations. The roofline is reported for the kernel with the largest
    # total time in the step.
    kernels = {}
    n1_bytes = args.layers * sum(fwd_bytes(M, K, 1) for _, (M, K) in shp)
    if 1 in batches:
        kernels[1] = {"kernel": "k_bitlinear_n1 (fused RMSNorm+quantize+GEMV, B=1)",
                      "bound": "hbm", "us": per_b_ms[1] * 1e3 / (args.steps * args.layers * len(shp)),
                      "bytes": n1_bytes / (args.layers * len(shp)),
                      "step_share_ms": per_b_ms[1] / args.steps}
    with torch.cuda.stream(stream):
        for B in [b for b in batches if b > 1]:
            qin = {}
            for i, (name, (M, K)) in enumerate(shp):
                qin[i] = obn.rmsnorm_quantize(xs[B, i].contiguous())
            outs = {i: torch.empty((B, M), device=dev) for i, (_, (M, K)) in enumerate(shp)}
            torch.cuda.synchronize()
            gk = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gk, stream=stream):
                for row in layers:
                    for i, L in enumerate(row):
                        q, sc, qs = qin[i]
                        obn._lib.check(obn.lib().obn_ternary_matmul(
                            L.handle, q.data_ptr(), sc.data_ptr(), qs.data_ptr(), B,
                            outs[i].data_ptr(), stream.cuda_stream))
            for _ in range(3):
                gk.replay()
            stream.synchronize()
            k0 = torch.cuda.Event(enable_timing=True)
            k1 = torch.cuda.Event(enable_timing=True)
            reps = max(5, min(args.steps, 50))
            k0.record(stream)
            for _ in range(reps):
                gk.replay()
            k1.record(stream)
            stream.synchronize()
            ms = k0.elapsed_time(k1) / reps
            nl = args.layers * len(shp)
            kb = args.layers * sum(gemv_kernel_bytes(M, K, B) for _, (M, K) in shp)
            # 2..16 tokens: the warp-MMA decode kernel; from 17 tokens every
            # BitNet-2B shape (< 74 row tiles) takes the split-K cluster GEMM.
            name = ("k_mma_gemv (mma.sync m16n8k32 u8 x s8, B=%d)" % B) if B <= 16 else (
                "k_gemm_sk (tcgen05 kind::i8, split-K over clusters, B=%d)" % B)
            kernels[B] = {"kernel": name, "bound": "hbm", "us": ms * 1e3 / nl, "bytes": kb / nl,
                          "step_share_ms": ms}
            del gk
    torch.cuda.synchronize()
    obn.check_device_errors()

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("hbm_gbs")
    peak_note = "measured" if peak else "fallback"
    peak = peak or 6650.0
    rooflines = {}
    for B, k in kernels.items():
        ach = k["bytes"] / (k["us"] * 1e-6) / 1e9
        rooflines[str(B)] = {"kernel": k["kernel"], "avg_launch_us": k["us"],
                             "bytes_per_launch_avg": k["bytes"], "achieved_gbs": ach,
                             "frac": ach / peak}
    dom = max(kernels, key=lambda b: kernels[b]["step_share_ms"]) if kernels else None
    traffic = load_profile_traffic()
    roofline = None
    if dom is not None:
        k = kernels[dom]
        ach = k["bytes"] / (k["us"] * 1e-6) / 1e9
        tr = None
        if traffic and traffic.get("batch") == dom:
            tr = traffic.get("dram_bytes_per_launch")
        roofline = {"kernel": k["kernel"], "bound": k["bound"], "achieved": ach, "peak": peak,
                    "peak_source": peak_note, "unit": "GB/s", "frac": ach / peak,
                    "avg_launch_us": k["us"], "bytes_per_launch_avg": k["bytes"], "traffic": tr}

    prefill = measure_prefill(args, obn, synth, dev, stream) if args.prefill else None
    lm_head = measure_lm_head(obn, dev, stream, peak)
    ffn_gate_up = measure_ffn_gate_up(args, obn, synth, dev, stream, batches)
    attention = measure_attention(dev, stream, peak, min(args.layers, 30))
    decoder = measure_decoder(dev, stream, world, rank) if args.decoder else None
    generate = measure_generate(dev) if (args.generate and world == 1) else None
    tp_prefill = None
    if world > 1 and args.tp_tokens > 0:
        tp_prefill = measure_tp_prefill(args, obn, synth, dev, stream, world, rank)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_sample(args)

    if rank == 0:
        # per-batch figures are rank 0's own device time (ranks run identical work)
        per_b = {str(B): step_bytes[B] * args.steps * world / (per_b_ms[B] / 1e3) / 1e9
                 for B in batches}
        tok_s = {str(B): B * world * args.steps / (per_b_ms[B] / 1e3) for B in batches}
        out = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded): N(0,1) activations, RMSNorm gamma N(1,0.1), i.i.d. "
                    "ternary weights P(-1)=P(+1)=0.3, per-tensor scale U(0.5,2)",
            "config": config(args, world),
            "per_batch_gbs": per_b,
            "bitlinear_stack_tok_s": tok_s,
            "roofline": roofline,
            "rooflines_per_batch": rooflines,
            "prefill": prefill,
            "tp_prefill": tp_prefill,
            "lm_head": lm_head,
            "ffn_gate_up": ffn_gate_up,
            "attention_decode": attention,
            "decode_tok_s": decoder,
            "generate": generate,
            "cpu_baseline": cpu,
            "clocks": clock_info,
            "e2e": {"value": e2e_value, "unit": "GB/s",
                    "h2d_bytes_per_step": x_total * 4, "d2h_bytes_per_step": y_total * 4,
                    "copies": "double-buffered on H2D and D2H streams beside the kernels; "
                              "outputs checked against the device-timed run"},
            "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(out), flush=True)
    for gs in graph_sets:
        gs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_case(spec: str):
    """A few BitLinear forwards of one shape, or of every shape in turn ("all"),
    4 layers each with distinct weights, for profilers: SHAPE:B, e.g. gate:64."""
    import torch
    obn = importlib.import_module("0xbitnet_b200")
    synth = importlib.import_module("0xbitnet_b200.synthetic")
    name, B = spec.split(":")
    B = int(B)
    if name == "lmhead":  # the 128256 x 2560 f16 LM head, B tokens, 3 launches
        g = torch.Generator(device="cuda")
        g.manual_seed(5)
        embed = (torch.randn(128256, 2560, generator=g, device="cuda") * 0.05).half()
        x = torch.randn(B, 2560, generator=g, device="cuda")
        gamma = torch.ones(2560, device="cuda")
        for _ in range(3):
            (obn.lm_head_f16 if B <= 4 else obn.lm_head_f16_batched)(embed, x, gamma)
        torch.cuda.synchronize()
        obn.check_device_errors()
        print(f"case lmhead B={B}: ok")
        return
    if name == "mmarate":  # MACs per cycle per SM of the integer MMA forms (B = MMAs per burst)
        import ctypes
        L = obn.lib()
        out = {}
        for form, label in ((0, "tcgen05 kind::i8 A=TMEM"), (1, "tcgen05 kind::i8 A=smem")):
            for N in (8, 16, 32, 64, 128, 256):
                r = ctypes.c_double()
                obn._lib.check(L.obn_measure_mma_rate(form, N, B, ctypes.byref(r)))
                out[f"{label} N={N}"] = r.value
        for form, label in ((2, "mma.sync m16n8k32 u8.s8"), (3, "dp4a")):
            r = ctypes.c_double()
            obn._lib.check(L.obn_measure_mma_rate(form, 8, 4 * B, ctypes.byref(r)))
            out[label] = r.value
        print(json.dumps({"case": "mmarate", "ops_per_burst": B,
                          "macs_per_cycle_per_sm": {k: round(v, 1) for k, v in out.items()}}))
        return
    if name == "quant":  # fused RMSNorm + int8 quantize alone, B tokens at K = 2560 and 6912
        for K in (2560, 6912):
            x = torch.randn(B, K, device="cuda")
            gamma = torch.ones(K, device="cuda")
            for _ in range(3):
                obn.rmsnorm_quantize(x, gamma)
        torch.cuda.synchronize()
        obn.check_device_errors()
        print(f"case quant B={B}: ok")
        return
    if name == "prefill":  # the config-2 block alone at B tokens
        import types
        dev = torch.device("cuda", 0)
        res = measure_prefill(types.SimpleNamespace(prefill=str(B)), obn, synth, dev,
                              torch.cuda.Stream(dev))
        print(json.dumps({"prefill": res}), flush=True)
        return
    if name in ("attndec", "decoder"):  # the full-run blocks alone: B = layers / context
        dev = torch.device("cuda", 0)
        stream = torch.cuda.Stream(dev)
        try:
            peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
        except (OSError, ValueError, KeyError):
            peak = 6650.0  # the pool's fallback copy bandwidth
        res = (measure_attention(dev, stream, peak, B) if name == "attndec"
               else measure_decoder(dev, stream, 1, 0, ctx=B))
        print(json.dumps({name: res}), flush=True)
        return
    if name == "attn":  # decode attention, 5 KV heads, context 2048, B sequences, 3 steps
        att = importlib.import_module("0xbitnet_b200.attention")
        cache = att.KVCache(B, 2048, 5, 128)
        cache.k.normal_()
        cache.v.normal_()
        q = torch.randn(B, 20 * 128, device="cuda")
        for _ in range(3):
            att.attention(q, cache, 20, 1, 2048)
        torch.cuda.synchronize()
        print(f"case attn B={B}: ok")
        return
    if name == "prefilltrace":  # kernel timeline (CUPTI) of one B-token prompt through the model ABI
        import re
        import shutil
        import tempfile

        import numpy as np
        from torch.profiler import ProfilerActivity, profile
        W = importlib.import_module("0xbitnet_b200.gguf_writer")
        ox = importlib.import_module("0xbitnet_b200.oxbitnet")
        tmp = tempfile.mkdtemp(prefix="obn_gguf_")
        try:
            path = os.path.join(tmp, "bitnet2b.gguf")
            toks, merges, bos, eos = W.synthetic_vocab(128256)
            W.write_bitnet_model(path, W.BitNetShape(), toks, merges, bos, eos, seed=0, fast=True)
            m = ox.BitNet.load_sync(path)
            rng = np.random.default_rng(0)
            prompt = [bos] + [int(x) for x in rng.integers(0, 128000, B - 1)]
            m.forward(prompt, reset=True)
            torch.cuda.synchronize()
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                m.forward(prompt, reset=True)
                torch.cuda.synchronize()
            ev = sorted((e for e in prof.events() if e.device_type.name == "CUDA"),
                        key=lambda e: e.time_range.start)
            kinds = {}
            for i, e in enumerate(ev):
                mt = re.search(r"(k_\w+)", e.name)
                k = mt.group(1) if mt else e.name[:40]
                end_prev = ev[i - 1].time_range.end if i else e.time_range.start
                a = kinds.setdefault(k, [0, 0.0])
                a[0] += 1
                a[1] += e.time_range.end - end_prev  # end-to-end increment, us
            span = (ev[-1].time_range.end - ev[0].time_range.start) if ev else 0
            print(json.dumps({"prefilltrace": {
                "tokens": B, "gpu_span_us": span,
                "kernels": {k: {"launches": n, "end_increment_us": round(t, 1)}
                            for k, (n, t) in sorted(kinds.items(), key=lambda x: -x[1][1])}}}),
                flush=True)
            del m
        finally:
            shutil.rmtree(tmp, ignore_errors=True)
        return
    if name == "attnpf":  # prefill attention: one sequence, B new rows on an empty cache, 3 runs
        att = importlib.import_module("0xbitnet_b200.attention")
        cache = att.KVCache(1, B, 5, 128)
        cache.k.normal_()
        cache.v.normal_()
        q = torch.randn(B, 20 * 128, device="cuda")
        for _ in range(3):
            att.attention(q, cache, 20, B, B)
        torch.cuda.synchronize()
        print(f"case attnpf n={B}: ok")
        return
    if name == "gateup":  # merged 6912 x 2560 gate|up layer, ReLU^2 x up in the matmul epilogue
        M, K = synth.SHAPES_2B["gate"]
        layers = []
        for i in range(4):
            gp, gs, gamma = synth.layer_device(91 + 2 * i, M, K)
            up, us, _ = synth.layer_device(92 + 2 * i, M, K)
            layers.append(obn.BitLinear.create_gated(gp, gs, up, us, gamma, K, M))
        x = torch.randn(B, K, device="cuda")
        for _ in range(3):
            for L in layers:
                L.forward(x)
        torch.cuda.synchronize()
        obn.check_device_errors()
        for L in layers:
            L.close()
        print(f"case gateup {M}x{K} B={B}: ok")
        return
    names = list(synth.SHAPES_2B) if name == "all" else [name]
    for nm in names:
        M, K = synth.SHAPES_2B[nm]
        layers = []
        for i in range(4):
            packed, s_w, gamma = synth.layer_device(77 + i, M, K)
            layers.append(obn.BitLinear(packed, s_w, gamma, K, M))
        x = torch.randn(B, K, device="cuda")
        for _ in range(3):
            for L in layers:
                L.forward(x)
        torch.cuda.synchronize()
        obn.check_device_errors()
        for L in layers:
            L.close()
        print(f"case {nm} {M}x{K} B={B}: ok")


def main():
    args = parse_args()
    if args.case:
        run_case(args.case)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark of the decode-step hot path.

Workload: one decode token through a stack of 26 Gemma-2-2B-shape layers
(hidden 2304, 8 Q / 4 KV heads, head_dim 256, FFN 2304->9216->2304, GeGLU)
at batch 1 with a KV context of 4096, f16 weights N(0, 0.02), KV cache and
input N(0, 1), seeded. A step = one token through all 26 layers (QKV with
fused RMSNorm + KV write, split-KV flash-decode, o_proj + residual, fused
gate/up GeGLU, down_proj + residual), replayed from one CUDA graph. The
weights and caches of the stack (4.5 GB) are far larger than the 126 MB L2,
so every step streams them from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

At N > 1 (torchrun, one process per GPU) every rank runs its own replica
(the config-2 decode path at batch 1 does not shard: replicas only);
`value` is the tokens/s of all ranks together, timed as the max over ranks.
The same line then carries the other BASELINE configs: at N = 1 the single
FlashDecoding op (`fd_config1`), the 16-point FlashDecoding sweep
(`fd_sweep`) and the prefill GEMM and attention (`prefill`); at every N the
tensor-parallel 9B-shape decode at TP = N (`tp9b`: tok/s, per-role
breakdown, all-reduce share, clocks and a peer-vs-NCCL parity check) — the
scaling curve. Rank 0 prints one JSON line.
"""
import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LAYERS = 26
CTX = 4096
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one gemv_tma_kernel
# <f16,f16,f16,NORM,kGated> launch (one layer's gate/up), from an ncu
# capture of that launch (bench.py --layers 4 --profile-steps 1).
GEGLU_NCU_TRAFFIC = 87_360_256
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", FALLBACK_BF16_TFLOPS)), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def metric_name(layers=LAYERS):
    return "Gemma-2-2B-shape decode tok/s (%d-layer stack, batch 1, ctx 4096)" % layers


def config_dict(parallelism, layers=LAYERS):
    return {"workload": "config2: Gemma-2-2B-shape decode layer x%d, batch 1, KV ctx %d, f16" % (layers, CTX),
            "layers": layers, "hidden": 2304, "q_heads": 8, "kv_heads": 4, "head_dim": 256, "ffn": 9216,
            "global_batch": 1, "seq_len": CTX, "activation": "gelu_tanh (GeGLU)",
            "l2": "inputs larger than L2 (weights + KV of the stack stream from HBM every step)",
            "parallelism": parallelism}


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.path = os.path.join("/tmp", "pc_clocks_%d_%d.csv" % (os.getpid(), device_index))

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        med = sm[len(sm) // 2] if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU legs (oracle port) — the reported baseline and the reference arm
# ---------------------------------------------------------------------------

def host_layer(seed=1234):
    """One layer's weights / caches / input on the host in the oracle's layout."""
    import numpy as np
    import oracle
    rng = np.random.default_rng(seed)
    H, Nq, Nkv, Hd, F = 2304, 8, 4, 256, 9216

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float16)

    d = dict(x=rng.standard_normal((H,), dtype=np.float32).astype(np.float16),
             w_attn_norm=(rng.standard_normal(H) * 0.1).astype(np.float32),
             w_mlp_norm=(rng.standard_normal(H) * 0.1).astype(np.float32),
             w_qkv=w((Nq + 2 * Nkv) * Hd, H), w_o=w(H, Nq * Hd), w_gate=w(F, H), w_up=w(F, H), w_down=w(H, F),
             k_cache=rng.standard_normal((Nkv, CTX, Hd), dtype=np.float32).astype(np.float16),
             v_cache=rng.standard_normal((Nkv, CTX, Hd), dtype=np.float32).astype(np.float16))
    return d, oracle


def time_cpu_layer(reps_min=1, budget_s=15.0, threads=None):
    """Seconds per layer of the oracle decode layer on the host cores."""
    d, oracle = host_layer()
    if threads:
        oracle.set_threads(threads)
    cores = oracle.threads()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < reps_min or (time.perf_counter() < t_end and len(times) < 50):
        t0 = time.perf_counter()
        oracle.decode_layer(d["x"], "f16", d["w_attn_norm"], d["w_mlp_norm"], d["w_qkv"], d["w_o"], d["w_gate"],
                            d["w_up"], d["w_down"], d["k_cache"], d["v_cache"], 8, 4, 256, CTX - 1)
        times.append(time.perf_counter() - t0)
    times.sort()
    return times[len(times) // 2], cores, len(times)


def run_reference(args):
    """The reference arm: the CPU restatement of the reference's kernels
    (oracle/) over the whole 26-layer step, every step, on all host cores.
    Each step runs the oracle decode layer 26 times (one layer's weights and
    caches reused: on the host they stream from DRAM either way), so
    ms_per_step is measured, not multiplied."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    d, oracle = host_layer()
    oracle.set_threads(os.cpu_count() or 1)
    cores = oracle.threads()

    def layer():
        oracle.decode_layer(d["x"], "f16", d["w_attn_norm"], d["w_mlp_norm"], d["w_qkv"], d["w_o"], d["w_gate"],
                            d["w_up"], d["w_down"], d["k_cache"], d["v_cache"], 8, 4, 256, CTX - 1)

    def step():
        for _ in range(LAYERS):
            layer()

    steps = max(1, min(args.steps, args.ref_steps))
    warmup = max(1, min(args.warmup, 3))
    for _ in range(warmup):
        layer()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    tok_s = 1.0 / dt
    sample = ("each step: all %d layers (ctx %d) on the host, one layer's weights and caches reused; "
              "%d timed step(s) after %d warm-up layer(s)" % (LAYERS, CTX, steps, warmup))
    line = {"impl": "reference", "metric": metric_name(), "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": dt * 1000.0,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV cache and input)",
            "config": config_dict("cpu, %d threads" % cores),
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference = the C++ restatement of the reference's Metal kernels (oracle/); the Swift/Metal "
                    "original cannot run on Linux. steps capped at --ref-steps (%d) to bound the run" % args.ref_steps}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# FlashDecoding sweep
# ---------------------------------------------------------------------------

def fd_sweep_points(pc, lib, hbm_gbs):
    """Config 3: batch {1,8,32,64} x ctx {1k,4k,16k,32k}, 16 Q / 8 KV heads,
    head_dim 256, bf16 K/V N(0,1), ragged lengths U[ctx/2, ctx] (seeded),
    split count chosen by the library. Each point: K/V bytes actually read
    (sum of lengths x 8 heads x 256 x 2 B x 2) / time of one ragged
    FlashDecoding call (partial + combine), CUDA events over graph replays.
    Points smaller than 2x L2 rotate over several cache copies so every call
    reads from HBM."""
    import torch
    Nq, Nkv, Hd = 16, 8, 256
    points = []
    gen = torch.Generator(device="cuda").manual_seed(7)
    for B in (1, 8, 32, 64):
        for ctx in (1024, 4096, 16384, 32768):
            lens_h = torch.randint(ctx // 2, ctx + 1, (B,), generator=torch.Generator().manual_seed(B * 7 + ctx),
                                   dtype=torch.int32)
            kv_bytes = int(lens_h.sum()) * Nkv * Hd * 2 * 2
            cache_bytes = B * Nkv * ctx * Hd * 2 * 2
            copies = max(1, -(-(256 << 20) // cache_bytes))
            caches = []
            for _ in range(copies):
                k = torch.randn(B, Nkv, ctx, Hd, device="cuda", dtype=torch.bfloat16, generator=gen)
                v = torch.randn(B, Nkv, ctx, Hd, device="cuda", dtype=torch.bfloat16, generator=gen)
                caches.append((k, v))
            q = torch.randn(B, Nq, 1, Hd, device="cuda", dtype=torch.bfloat16, generator=gen)
            out = torch.empty_like(q)
            lens = lens_h.cuda()
            stream = torch.cuda.Stream()
            scratch = pc.FixedScratch(64 << 20)
            with torch.cuda.stream(stream):
                enc = pc.KernelCommandEncoder(lib, stream=stream, scratch=scratch)
                kerns = [pc.Kernels.FlashDecodingRagged(q, k, v, lens, into=out, scale=1.0 / 16) for k, v in caches]
                enc.encode(*kerns)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    enc.encode(*kerns)
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                reps = max(3, min(50, int(2e9 // max(1, kv_bytes * copies))))
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(reps):
                    g.replay()
                b.record(stream)
                torch.cuda.synchronize()
                us = a.elapsed_time(b) * 1000.0 / (reps * copies)
            gbs = kv_bytes / (us * 1e-6) / 1e9
            points.append({"batch": B, "ctx": ctx, "us": round(us, 2), "kv_bytes": kv_bytes, "gbs": round(gbs, 1),
                           "frac_of_measured_hbm": round(gbs / hbm_gbs, 3)})
            del caches, kerns, g, k, v
            torch.cuda.empty_cache()
    return points


def fd_config1(pc, lib, hbm_gbs):
    """Config 1: one FlashDecoding op (B 1, one query token, 8 Q / 4 KV heads,
    head_dim 256, KV context 1024, f16 N(0,1) q/k/v, scale 1/16, causal):
    4 202 496 algorithmic bytes per call (K + V + q + out). One call's data
    (4.2 MB) fits in L2, so the timed graph rotates over 64 distinct K/V
    copies (269 MB > L2) and every call reads from HBM. CUDA events over
    graph replays; the per-call time includes the split combine."""
    import torch
    B, Nq, Nkv, S, Hd, copies = 1, 8, 4, 1024, 256, 64
    gen = torch.Generator(device="cuda").manual_seed(1234)
    kv = [(torch.randn(B, Nkv, S, Hd, device="cuda", generator=gen).half(),
           torch.randn(B, Nkv, S, Hd, device="cuda", generator=gen).half()) for _ in range(copies)]
    q = torch.randn(B, Nq, 1, Hd, device="cuda", generator=gen).half()
    out = torch.empty_like(q)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        enc = pc.KernelCommandEncoder(lib, stream=stream, scratch=pc.FixedScratch(16 << 20))
        kerns = [pc.Kernels.FlashAttention(q, k, v, into=out, scale=1.0 / 16) for k, v in kv]
        enc.encode(*kerns)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            enc.encode(*kerns)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = 20
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1000.0 / (reps * copies)
    nbytes = 2 * B * Nkv * S * Hd * 2 + 2 * B * Nq * Hd * 2
    gbs = nbytes / (us * 1e-6) / 1e9
    names = kerns[0].function_names
    del kv, kerns, g
    torch.cuda.empty_cache()
    return {"kernels": "+".join(names), "us": us, "bytes": nbytes, "gbs": gbs, "frac_of_measured_hbm": gbs / hbm_gbs,
            "timing": "64 distinct K/V copies (269 MB) per graph replay, CUDA events"}


def run_fd_sweep(args):
    import torch
    import popcorn_b200 as pc
    torch.cuda.set_device(0)
    hbm_gbs, _, peak_kind = peaks()
    points = fd_sweep_points(pc, pc.KernelLibrary(0), hbm_gbs)
    line = {"metric": "FlashDecoding sweep HBM GB/s (config 3)", "unit": "GB/s", "peak": hbm_gbs,
            "peak_kind": peak_kind, "dtype": "bf16", "data": "synthetic seeded N(0,1) K/V, ragged U[ctx/2, ctx]",
            "config": {"workload": "config3: B {1,8,32,64} x ctx {1k,4k,16k,32k}, 16Q/8KV, hd 256"},
            "points": points}
    print(json.dumps(line), flush=True)
    return 0


def prefill_kernels(pc, lib, steps, warmup, tf_peak):
    """Config 4: the prefill GEMM (M 8192 x K 2304 x N 9216, bf16, transposeB,
    2*M*N*K = 347.9 GFLOP) and causal FlashAttention (B 4, 8 Q / 4 KV heads,
    S 2048, hd 256, bf16: 4*B*Nq*(S(S+1)/2)*hd = 68.75 GFLOP), each on the
    tcgen05 tensor cores, CUDA events over graph replays after warm-up.
    Operands (GEMM 370 MB in+out) exceed L2."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(4)
    M, K, N = 8192, 2304, 9216
    a = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    B, Nq, Nkv, S, Hd = 4, 8, 4, 2048, 256
    q = torch.randn(B, Nq, S, Hd, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, Nkv, S, Hd, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, Nkv, S, Hd, device="cuda", generator=g).to(torch.bfloat16)
    o = torch.empty_like(q)
    gemm = pc.Kernels.Matmul(a, w, into=c, transpose_b=True)
    fa = pc.Kernels.FlashAttention(q, k, v, into=o, scale=1.0 / 16, mask=pc.AttentionMask.causal)
    stream = torch.cuda.Stream()
    res = {}
    with torch.cuda.stream(stream):
        enc = pc.KernelCommandEncoder(lib, stream=stream)
        for name, kern, flops in (("gemm", gemm, 2.0 * M * N * K),
                                  ("flash_attention", fa, 4.0 * B * Nq * (S * (S + 1) / 2) * Hd)):
            enc.encode(kern)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                enc.encode(kern)
            for _ in range(max(warmup, 3)):
                graph.replay()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = max(steps, 5)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000.0 / reps
            tf = flops / (us * 1e-6) / 1e12
            res[name] = {"kernel": kern.function_names[0], "us": round(us, 2), "gflop": round(flops / 1e9, 2),
                         "tflops": round(tf, 1), "frac_of_measured_bf16": round(tf / tf_peak, 3)}
            del graph
    del a, w, c, q, k, v, o, gemm, fa
    torch.cuda.empty_cache()
    return res


def run_prefill(args):
    import torch
    import popcorn_b200 as pc
    torch.cuda.set_device(0)
    _, tf_peak, peak_kind = peaks()
    res = prefill_kernels(pc, pc.KernelLibrary(0), args.steps, args.warmup, tf_peak)
    line = {"metric": "prefill TFLOP/s (config 4)", "unit": "TFLOP/s", "peak": tf_peak, "peak_kind": peak_kind,
            "dtype": "bf16", "data": "synthetic seeded N(0,1) activations / q,k,v, N(0,0.02) weights",
            "config": {"workload": "config4: GEMM 8192x2304x9216 tb; causal FA B4 8Q/4KV S2048 hd256"},
            "kernels": res, "device_error_word": pc.device_error_check(0)}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Tensor-parallel 9B-shape batched decode
# ---------------------------------------------------------------------------

TP_ROLES = ("qkv_gemm", "qkv_scatter", "attention", "o_proj_gemm", "allreduce_o_add_norm", "gate_up_gemm",
            "gated_act", "down_gemm", "allreduce_down_add_norm")


def _graph_time(stream, encode, reps, warmup=3):
    """ms per replay of a graph holding what encode() enqueues."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        encode()
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(reps):
        g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / reps


def tp9b_leg(args, world, rank, local):
    """Config 5: Gemma-2-9B-shape decoder (42 layers, vocab 256000), batch 32,
    KV context 8192, bf16, tensor-parallel over the torchrun ranks (one
    process per GPU): Q/KV heads, FFN columns and the vocabulary sharded,
    an all-reduce after o_proj and after down_proj. A step = one token for
    all 32 sequences through every layer and the LM head, replayed from one
    CUDA graph. Total work is fixed as N grows (strong scaling); tok/s =
    32 / step time (max over ranks).

    Before timing, one step runs on the NCCL path (torch.distributed
    all-reduce + AddRMSNorm) and one on the peer path (the one-shot
    all-reduce over NVLink peer memory fused with Add + RMSNorm) from the
    same input; `parity` is the largest logit difference between them
    relative to the logits' RMS, and whether the two paths pick the same
    argmax token for every sequence. The timed step uses the peer path.
    `breakdown` replays each role's 42 launches from its own graph (all
    ranks together), so `allreduce_share` = the two all-reduce roles' time
    / the step time."""
    import torch
    import torch.distributed as dist
    import popcorn_b200 as pc
    from popcorn_b200.tp import TPDecodeModel, TPShape
    hbm_gbs, _, peak_kind = peaks()
    shape = TPShape(layers=args.tp_layers)
    model = TPDecodeModel(pc.KernelLibrary(local), shape, rank=rank, world=world, seed=5, device=local)
    stream = torch.cuda.Stream(device=local)

    def all_reduce(t):
        # the reference path of the parity check: NCCL sums the partials in
        # fp32 and the sum is rounded once, as the peer kernel does (a bf16
        # NCCL reduction rounds every partial sum of its ring, which differs
        # from any single-rounding sum from 4 ranks on)
        if world > 1:
            t32 = t.float()
            dist.all_reduce(t32)
            t.copy_(t32)

    def all_gather(blob):
        if world == 1:
            return [blob]
        out = [None] * world
        dist.all_gather_object(out, blob)
        return out

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def parity_of(m):
        """One step on the NCCL path, then one on the peer path, from the same
        input; returns the comparison of the two paths' logits."""
        m.x.normal_(generator=torch.Generator(device=m.x.device).manual_seed(11))
        x_in = m.x.clone()
        e = m.encoder(stream)
        m.step(e, all_reduce)
        sync_all()
        ref = m.logits.float()
        m.x.copy_(x_in)
        m.use_peer_allreduce(all_gather, fuse_gemm=args.allreduce == "peer-fused")
        e = m.encoder(stream)
        m.step(e, all_reduce)
        sync_all()
        got = m.logits.float()
        m.x.copy_(x_in)
        rms = ref.pow(2).mean().sqrt()
        d = (got - ref).abs()
        # the bound of a chain of rounding points (bf16): relative L2 below
        # 5e-3 and every logit within 8 bf16 ulps at the logits' RMS scale
        ulp = torch.exp2(torch.floor(torch.log2(torch.maximum(ref.abs(), rms))) - 7)
        red = torch.stack([d.max() / rms, (d.pow(2).sum().sqrt() / ref.pow(2).sum().sqrt()),
                           (d > 8 * ulp).any().float(), (got.argmax(1) != ref.argmax(1)).any().float(),
                           (d == 0).all().logical_not().float()])
        if world > 1:
            dist.all_reduce(red, op=dist.ReduceOp.MAX)
        return {"max_abs_diff_over_rms": float(red[0]), "rel_l2": float(red[1]),
                "within_chain_tolerance": bool(red[1] < 5e-3 and red[2] == 0), "argmax_equal": bool(red[3] == 0),
                "bit_identical": bool(red[4] == 0)}

    with torch.cuda.stream(stream):
        # ---- parity: a 2-layer model of the same shapes and sharding (a
        # short chain of rounding points), then the full 42-layer model ----
        short = TPDecodeModel(pc.KernelLibrary(local), TPShape(layers=2), rank=rank, world=world, seed=5,
                              device=local)
        parity = {"paths": "NCCL all-reduce (fp32 sum, one rounding) + AddRMSNorm vs peer all-reduce fused with "
                           "Add + RMSNorm",
                  "argmax": "per rank over its vocabulary slice", "two_layer": parity_of(short)}
        del short
        torch.cuda.empty_cache()
        parity["full_depth"] = parity_of(model)
        enc = model.encoder(stream)
        x0 = model.x.clone()

        # ---- the timed step (peer path), graph-captured ----
        model.x.copy_(x0)
        n0 = enc.dispatch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            model.step(enc, all_reduce)
        launches = enc.dispatch_count - n0
        for _ in range(args.warmup):
            graph.replay()
        sync_all()
        clocks = ClockSampler(local)
        clocks.start()
        time.sleep(0.2)
        sync_all()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        clk = clocks.stop()
        sync_all()
        del graph

        # ---- per-role breakdown (peer path; 9 launches per layer) ----
        ks = model.kernels()
        body = ks[1:-1]
        per_layer = len(TP_ROLES)
        breakdown = {}
        if len(body) == per_layer * shape.L:
            for i, role in enumerate(TP_ROLES):
                sel = body[i::per_layer]
                breakdown[role] = _graph_time(stream, lambda sel=sel: enc.encode(*sel), reps=5)
            breakdown["lm_head_gemm"] = _graph_time(stream, lambda: enc.encode(ks[-1]), reps=5)
            sync_all()
    vals = [ms] + [breakdown[k] for k in sorted(breakdown)]
    if world > 1:
        t = torch.tensor(vals, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = [float(x) for x in t]
    ms = vals[0]
    breakdown = {k: round(v, 4) for k, v in zip(sorted(breakdown), vals[1:])}
    err = pc.device_error_check(local)
    per_rank_bytes = model.bytes_per_step()
    ar_ms = breakdown.get("allreduce_o_add_norm", 0.0) + breakdown.get("allreduce_down_add_norm", 0.0)
    top = max((k for k in breakdown), key=lambda k: breakdown[k]) if breakdown else None
    res = {"workload": "config5: Gemma-2-9B-shape decode, %d layers, vocab 256000, batch 32, KV ctx 8192, bf16"
                       % shape.L,
           "parallelism": "tp%d" % world, "allreduce": args.allreduce, "scaling": "strong",
           "tok_s": shape.B * 1000.0 / ms, "ms_per_step": ms,
           "per_rank_bytes_per_step": per_rank_bytes,
           "per_rank_hbm_gbs": per_rank_bytes / (ms * 1e-3) / 1e9,
           "per_rank_frac_of_measured_hbm": per_rank_bytes / (ms * 1e-3) / 1e9 / hbm_gbs, "peak_kind": peak_kind,
           "allreduce_per_step": 2 * shape.L, "allreduce_bytes": shape.B * shape.H * 2,
           "breakdown_ms_per_step": breakdown,
           "breakdown_note": "each role's launches of one step replayed from their own graph, max over ranks",
           "allreduce_share": ar_ms / ms if ms > 0 else None, "largest_role": top,
           "gpu_launches_per_step": launches, "parity": parity, "clocks": clk, "device_error_word": err}
    del model, ks, body
    torch.cuda.empty_cache()
    return res


def run_tp(args):
    """bench.py --workload tp9b: the config-5 leg alone, as its own JSON line."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    res = tp9b_leg(args, world, rank, local)
    line = {"metric": "Gemma-2-9B-shape batched decode tok/s (42 layers, batch 32, ctx 8192, TP)",
            "value": res["tok_s"], "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) weights, N(0,1) KV)",
            "config": {"workload": res["workload"], "global_batch": 32, "seq_len": 8192,
                       "parallelism": res["parallelism"], "l2": "inputs larger than L2"},
            "tp9b": res, "gpu_launches": res["gpu_launches_per_step"] * args.steps, "clocks": res["clocks"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        os._exit(0)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def time_aq_matvec(pc, enc, stream, shape, copies=4, reps=10):
    """Affine 4-bit quantized Matmul (Kernels.Matmul with an
    AffineQuantizedTensor) at batch 1: algorithmic bytes = packed weights +
    scales + biases + x + out, CUDA events over graph replays."""
    import torch
    hbm = peaks()[0]

    def qt(n, k):
        packed = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=torch.int32, device="cuda")
        sc = (torch.rand(n, k // 64, device="cuda") * 0.002).bfloat16()
        bi = (torch.randn(n, k // 64, device="cuda") * 0.01).bfloat16()
        return pc.AffineQuantizedTensor(packed, sc, bi, (n, k))

    def qbytes(n, k):
        return n * k // 2 + 2 * n * (k // 64) * 2 + k * 2 + n * 2

    def timed(kernels, nbytes):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            enc.encode(*kernels)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        us = a.elapsed_time(b) * 1000.0 / reps
        del g
        return us, nbytes / (us * 1e-6) / 1e9

    H, F, Nq, Nkv, Hd = shape.H, shape.F, shape.Nq, shape.Nkv, shape.Hd
    shapes = [((Nq + 2 * Nkv) * Hd, H), (H, Nq * Hd), (F, H), (F, H), (H, F)]
    x_in = {k: torch.randn(1, k, device="cuda").bfloat16() for k in {s_[1] for s_ in shapes}}
    # the 4-bit LM head first (its first launch is the one a profile captures)
    head = qt(256000, H)
    head_us, head_gbs = timed([pc.Kernels.Matmul(x_in[H], head, torch.empty(1, 256000, device="cuda",
                                                                            dtype=torch.bfloat16))],
                              qbytes(256000, H))
    del head
    ks, nbytes = [], 0
    for _ in range(copies):
        for n, k in shapes:
            ks.append(pc.Kernels.Matmul(x_in[k], qt(n, k), torch.empty(1, n, device="cuda", dtype=torch.bfloat16)))
            nbytes += qbytes(n, k)
    layer_us, layer_gbs = timed(ks, nbytes)
    del ks
    return {"kernel": "aq_qmv_tma (mma.sync m16n8k16 bf16, TMA rings), bf16 x / scales / out",
            "layer_us": layer_us / copies, "layer_gbs": layer_gbs, "layer_frac_of_measured_hbm": layer_gbs / hbm,
            "lm_head_us": head_us, "lm_head_gbs": head_gbs, "lm_head_frac_of_measured_hbm": head_gbs / hbm,
            "bytes_per_layer": nbytes // copies}


def time_qk_rope_step(lib, stream, n_layers, pos, warmup, steps, device):
    """The config-2 step with the Gemma-3/4 attention prologue (per-head
    q/k/v RMSNorm + RoPE): the per-op graph (one QKNormRope launch per
    layer) and the fused one-launch step (folded into its attention items)."""
    import torch
    from popcorn_b200.decode import DecodeStack, LayerShape
    out = {}
    for fused in (False, True):
        st = DecodeStack(lib, LayerShape(), n_layers, seed=55, device=device, fused=fused, qk_norm_rope=True)
        st.set_position(pos)
        st.x.normal_()
        enc = st.encoder(stream)
        st.kernels()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            st.encode_step(enc)
        for _ in range(warmup):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        out["fused_ms_per_step" if fused else "ms_per_step"] = a.elapsed_time(b) / steps
        del g, st
    return out


def time_aq_step(pc, lib, stream, n_layers, pos, warmup, steps, device):
    """The decode step over 4-bit affine weights (AqDecodeStack, bf16
    activations, ctx 4096): CUDA events over graph replays."""
    import torch
    from popcorn_b200.decode import AqDecodeStack, LayerShape
    st = AqDecodeStack(lib, LayerShape(dtype="bf16"), n_layers, seed=77, device=device, vocab=256000)
    st.set_position(pos)
    st.x.normal_()
    enc = st.encoder(stream)
    st.kernels()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        st.encode_step(enc)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        g.replay()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    nbytes = st.algorithmic_bytes_per_step(pos + 1)
    del g, st
    return {"stack": "AqDecodeStack, %d layers + 4-bit LM head (vocab 256000) + Argmax, batch 1, ctx 4096, "
                     "bf16 activations" % n_layers,
            "ms_per_step": ms, "tok_s": 1000.0 / ms, "bytes_per_step": nbytes,
            "step_hbm_gbs": nbytes / (ms * 1e-3) / 1e9}


def run_aq(args):
    """The affine 4-bit GEMV alone (config-2 layer shapes and the LM head)."""
    import torch
    import popcorn_b200 as pc
    from popcorn_b200.decode import LayerShape
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream()
    enc = pc.KernelCommandEncoder(pc.KernelLibrary(0), stream=stream, scratch=pc.ScratchPool())
    with torch.cuda.stream(stream):
        res = time_aq_matvec(pc, enc, stream, LayerShape(dtype="bf16"))
    print(json.dumps({"workload": "aq", "aq_matvec": res, "device_error_word": pc.device_error_check(0)}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-steps", type=int, default=20,
                    help="reference arm: at most this many timed steps (each is 26 oracle layers on the host)")
    ap.add_argument("--no-extra", action="store_true",
                    help="config-2 line only (skip the config-1/3/4/5 objects)")
    ap.add_argument("--l2-prefetch", action="store_true",
                    help="each kernel of the step pulls the start of the next kernel's operand into L2")
    ap.add_argument("--profile-steps", type=int, default=5)
    ap.add_argument("--workload", default="config2", choices=["config2", "fd_sweep", "tp9b", "prefill", "aq"])
    ap.add_argument("--tp-layers", type=int, default=42)
    ap.add_argument("--allreduce", default="peer", choices=["peer", "peer-fused", "nccl"],
                    help="tp9b: all-reduce over peer memory with Add + RMSNorm as one kernel after the GEMM "
                         "(peer), the same fused into the o_proj / down GEMM (peer-fused), or NCCL")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="config-2 stack depth (26 for the bench line; fewer for small profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "fd_sweep":
        return run_fd_sweep(args)
    if args.workload == "tp9b":
        return run_tp(args)
    if args.workload == "prefill":
        return run_prefill(args)
    if args.workload == "aq":
        return run_aq(args)

    import torch
    import torch.distributed as dist
    import popcorn_b200 as pc
    from popcorn_b200 import _native as N
    from popcorn_b200.decode import DecodeStack, LayerShape

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    n_layers = args.layers
    shape = LayerShape(max_ctx=CTX, dtype="f16")
    lib = pc.KernelLibrary(local)
    stack = DecodeStack(lib, shape, n_layers, seed=1234 + rank, device=local, l2_prefetch=args.l2_prefetch)
    stream = torch.cuda.Stream(device=local)
    pos = CTX - 1
    hbm_gbs, _, peak_kind = peaks()

    with torch.cuda.stream(stream):
        stack.set_position(pos)
        stack.x.normal_()
        enc = stack.encoder(stream)
        # eager run once (validates launches), then capture one step
        stack.encode_step(enc)
        torch.cuda.synchronize()
        n0 = enc.dispatch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            stack.encode_step(enc)
        launches_per_step = enc.dispatch_count - n0
        torch.cuda.synchronize()

        # ---- device-timed region: inputs resident in HBM ----
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
        barrier()
        clocks = ClockSampler(local)
        clocks.start()
        time.sleep(0.3)
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        barrier()
        t_start.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t_end.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = t_start.elapsed_time(t_end) / args.steps

        # ---- end to end through the C ABI with host buffers ----
        H = shape.H
        # the step's inputs as laid out in stack.io: x (f16), then [pos, pos + 1]
        io_bytes = stack.io_pos_offset + 8
        host_io = torch.zeros(io_bytes, dtype=torch.uint8).pin_memory()
        host_io[:H * 2].view(torch.float16).normal_()
        host_io[stack.io_pos_offset:io_bytes].view(torch.int32).copy_(torch.tensor([pos, pos + 1], dtype=torch.int32))
        host_out = torch.empty(H, dtype=torch.float16).pin_memory()
        L = N.lib()
        sptr = torch.cuda.current_stream().cuda_stream

        def e2e_step():
            L.pc_memcpy_htod_async(stack.io.data_ptr(), host_io.data_ptr(), io_bytes, sptr)
            graph.replay()
            L.pc_memcpy_dtoh_async(host_out.data_ptr(), stack.out.data_ptr(), H * 2, sptr)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e_end.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e_start.elapsed_time(e_end) / args.steps
        clk = clocks.stop()
        barrier()

        # ---- per-kernel rates: each role's 26 launches replayed from their own
        # graph (back to back, as in the step), CUDA events on this stream ----
        ks = stack.kernels()
        role_idx = {"qkv_matvec_f16": 0, "flash_decoding_f16": 1, "o_proj_residual_f16": 2, "geglu_matvec_f16": 3,
                    "down_proj_residual_f16": 4}
        kern_us = {}
        for name, idx in role_idx.items():
            sel = [ks[l * 5 + idx] for l in range(n_layers)]
            g_role = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_role, stream=stream):
                enc.encode(*sel)
            for _ in range(3):
                g_role.replay()
            torch.cuda.synchronize()
            a_ev = torch.cuda.Event(enable_timing=True)
            b_ev = torch.cuda.Event(enable_timing=True)
            reps = max(5, args.profile_steps * 4)
            a_ev.record(stream)
            for _ in range(reps):
                g_role.replay()
            b_ev.record(stream)
            torch.cuda.synchronize()
            kern_us[name] = a_ev.elapsed_time(b_ev) * 1000.0 / reps / n_layers
            del g_role

        # ---- the step's tail at Gemma-2 vocabulary size: final RMSNorm fused into
        # the LM head GEMV (256000 x 2304, 1.18 GB) + Argmax, from its own graph ----
        tail = DecodeStack(lib, shape, 1, seed=99 + rank, device=local, vocab=256000)
        tail.set_position(pos)
        tail.x.normal_()
        tail_ks = tail.kernels()[-2:]
        g_t = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_t, stream=stream):
            enc.encode(*tail_ks)
        for _ in range(3):
            g_t.replay()
        torch.cuda.synchronize()
        t0e = torch.cuda.Event(enable_timing=True)
        t1e = torch.cuda.Event(enable_timing=True)
        t0e.record(stream)
        for _ in range(10):
            g_t.replay()
        t1e.record(stream)
        torch.cuda.synchronize()
        tail_us = t0e.elapsed_time(t1e) * 100.0
        tail_bytes = 256000 * shape.H * 2 + 256000 * 2
        del g_t, tail

        # ---- 4-bit affine weights (MLX format, group 64, bf16 scales / biases):
        # the config-2 layer's five GEMVs at batch 1 over 4 distinct layer copies
        # (175 MB > L2) and the LM head (256000 x 2304), each from a graph ----
        aq = time_aq_matvec(pc, enc, stream, shape)
        aq["decode_step"] = time_aq_step(pc, lib, stream, n_layers, pos, args.warmup, min(args.steps, 50), local)
        qk_rope = time_qk_rope_step(lib, stream, n_layers, pos, args.warmup, min(args.steps, 50), local)

        # ---- the same step as one persistent kernel (DecodeStack(fused=True)) ----
        fused = DecodeStack(lib, shape, n_layers, seed=1234 + rank, device=local, fused=True)
        fused.set_position(pos)
        fused.x.normal_()
        fused.kernels()
        enc_f = fused.encoder(stream)
        g_f = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_f, stream=stream):
            fused.encode_step(enc_f)
        for _ in range(args.warmup):
            g_f.replay()
        torch.cuda.synchronize()
        f_start = torch.cuda.Event(enable_timing=True)
        f_end = torch.cuda.Event(enable_timing=True)
        f_start.record(stream)
        for _ in range(args.steps):
            g_f.replay()
        f_end.record(stream)
        torch.cuda.synchronize()
        fused_ms = f_start.elapsed_time(f_end) / args.steps
        fused_err = pc.device_error_check(local)
        del g_f, fused

    # max over ranks of the timed step
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])

    s = shape
    F, Hd = s.F, s.Hd
    per_launch_bytes = {
        "qkv_matvec_f16": (s.Nq + 2 * s.Nkv) * Hd * s.H * 2 + s.H * 2 + 2 * s.Nkv * Hd * 2 + s.Nq * Hd * 2,
        "flash_decoding_f16": s.kv_bytes(CTX) + 2 * s.Nq * Hd * 2,
        "o_proj_residual_f16": s.H * s.Nq * Hd * 2 + s.Nq * Hd * 2 + 2 * s.H * 2,
        "geglu_matvec_f16": 2 * F * s.H * 2 + s.H * 2 + F * 2,
        "down_proj_residual_f16": s.H * F * 2 + F * 2 + 2 * s.H * 2,
    }
    kernels = {}
    for n, us in kern_us.items():
        b = per_launch_bytes[n]
        kernels[n] = {"us": us, "bytes": b, "gbs": b / (us * 1e-6) / 1e9,
                      "frac_of_measured_hbm": b / (us * 1e-6) / 1e9 / hbm_gbs}
    dom = "geglu_matvec_f16"
    dom_gbs = kernels[dom]["gbs"]
    fd = kernels["flash_decoding_f16"]

    tok_s = world * 1000.0 / ms
    e2e_tok_s = world * 1000.0 / e2e_ms
    bytes_step = stack.algorithmic_bytes_per_step(CTX)
    line = {
        "metric": metric_name(n_layers), "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) KV cache and input)",
        "config": config_dict("replicas" if world > 1 else "single GPU", n_layers),
        "step_hbm_gbs": bytes_step / (ms * 1e-3) / 1e9,
        "step_frac_of_measured_hbm": bytes_step / (ms * 1e-3) / 1e9 / hbm_gbs,
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": dom_gbs, "peak": hbm_gbs, "unit": "GB/s",
                     "frac": dom_gbs / hbm_gbs, "peak_kind": peak_kind,
                     "traffic": GEGLU_NCU_TRAFFIC,
                     "algorithmic_bytes_per_launch": per_launch_bytes[dom],
                     "timing": "26 launches (one per layer, distinct weights) replayed from a graph, CUDA events"},
        "flash_decode": {"kernel": "flash_decoding_f16 (partial + combine)", "achieved_gbs": fd["gbs"],
                         "frac_of_measured_hbm": fd["frac_of_measured_hbm"], "bytes_per_launch": fd["bytes"]},
        "kernels": kernels,
        "lm_head_argmax": {"kernels": "RMSNorm + LM head GEMV (vocab 256000) + Argmax", "us": tail_us,
                           "bytes": tail_bytes, "gbs": tail_bytes / (tail_us * 1e-6) / 1e9,
                           "frac_of_measured_hbm": tail_bytes / (tail_us * 1e-6) / 1e9 / hbm_gbs},
        "aq_matvec": aq,
        "qk_norm_rope_step": qk_rope,
        "fused_step": {"kernel": "decode_step_f16 (one persistent launch per token, all 26 layers)",
                       "ms_per_step": fused_ms, "tok_s": 1000.0 / fused_ms,
                       "step_hbm_gbs": bytes_step / (fused_ms * 1e-3) / 1e9, "device_error_word": fused_err},
        "e2e": {"value": e2e_tok_s, "unit": "tok/s", "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": H * 2,
                "path": "pc_memcpy_htod_async (pinned host) -> graph of C-ABI kernels -> pc_memcpy_dtoh_async"},
        "gpu_launches": launches_per_step * args.steps,
        "launches_per_step": launches_per_step,
        "clocks": clk,
    }
    if not args.no_extra:
        # The other BASELINE configs, measured by the same run: config 1 (one
        # FlashDecoding op), config 3 (the FlashDecoding sweep) and config 4
        # (prefill GEMM + attention) on one GPU; config 5 (tensor-parallel
        # 9B-shape decode) on every rank of this run, so a run at N GPUs
        # reports TP-N. The config-2 stack is freed first (config 5 holds
        # 108.7 GB / N per rank).
        del graph, stack, enc, ks
        import gc
        gc.collect()
        torch.cuda.empty_cache()
        if world == 1:
            line["fd_config1"] = fd_config1(pc, lib, hbm_gbs)
            line["fd_sweep"] = {"kernels": "flash_decoding_partial_bf16 + flash_decoding_reduce_bf16 (ragged)",
                                "points": fd_sweep_points(pc, lib, hbm_gbs)}
            _, tf_peak, tf_kind = peaks()
            line["prefill"] = prefill_kernels(pc, lib, 10, args.warmup, tf_peak)
            line["prefill"]["peak_tflops"] = tf_peak
            line["prefill"]["peak_kind"] = tf_kind
        line["tp9b"] = tp9b_leg(args, world, rank, local)
        line["gpu_launches_tp9b"] = line["tp9b"]["gpu_launches_per_step"] * args.steps

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t_layer, cores, reps = time_cpu_layer()
        line["cpu_baseline"] = {"value": 1.0 / (t_layer * n_layers), "unit": "tok/s", "cores": cores, "kind": "port",
                                "sample": "%d run(s) of one layer (ctx %d) of the oracle on the host, median; "
                                          "tok/s = 1 / (%d x layer time)" % (reps, CTX, n_layers)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        # Leave without tearing the communicator down: a destroy after a
        # graph-captured NCCL collective was seen to block for minutes.
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        os._exit(0)
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Benchmark of the B200 quantized matvec path (one JSON line on rank 0).

Workload: Q4_K weight 11008 x 4096 in GGUF blocks,
f32 activations x[1, 4096] ~ N(0, 1), batch 1, float path
(c = x . dequant(W)^T).  Synthetic seeded blocks with the benchmark's value
distributions (tcb_b200/synth.py); no model files exist on the box.

A step is one pass over a cold ring of R distinct weight copies (together
well above the 126 MB L2), i.e. R matvecs, so every launch streams its
weight from HBM.  The ring sweep is captured once in a CUDA graph and
replayed.  `value` is the algorithmic bytes (weight blocks + x + y) of all
ranks / the max over ranks of the device time.  `e2e` repeats the metric
through the public C ABI with host buffers: every step is one
tcb_qgemm_host call that moves x in from pinned host memory, runs the
product and writes y into pinned host memory (the same step as
cudaMemcpyAsync + tcb_qgemm + cudaMemcpyAsync is reported beside it).  `decode` adds the
metric's second half: 8B-shape Q4_K_M greedy decode tokens/s at batch 1
through the tcb_llama engine.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N   (one process per GPU)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K matvec HBM GB/s (% of peak); 8B-shape Q4_K_M decode tokens/sec @ batch 1"
WORKLOAD = {"workload": "q4_k_matvec", "wtype": "q4_k", "N": 11008, "K": 4096, "batch": 1,
            "x_dtype": "f32", "path": "float"}
Q4_0, Q8_0, Q4_K = 2, 8, 12


def algorithmic_bytes(N: int, K: int, M: int = 1) -> int:
    """Bytes one Q4_K product must move: the weight blocks (144 B per 256
    weights), x (f32) and y (f32)."""
    return N * K // 256 * 144 + M * K * 4 + M * N * 4


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", 1400.0)), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of the
# batch-1 Q4_K kernel on WORKLOAD, taken by ncu on that launch: ncu cannot run
# inside the timed region, so the figure is the capture's, reported beside the
# algorithmic bytes
TRAFFIC_BYTES_PER_LAUNCH = 25_445_888


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            names = {
                "hw_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwSlowdown", 0x8),
                "hw_thermal_slowdown": getattr(pynvml, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
                "sw_thermal_slowdown": getattr(pynvml, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
                "sw_power_cap": getattr(pynvml, "nvmlClocksEventReasonSwPowerCap", 0x4),
            }

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for k, bit in names.items():
                            if r & bit:
                                self.reasons.add(k)
                    except Exception:
                        pass
                    time.sleep(0.01)

            self._t = threading.Thread(target=run, daemon=True)
            self._t.start()
        except Exception:
            self._t = None
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_baseline(seconds: float = 12.0) -> dict:
    """TR's AVX2 float path restated (oracle, all host threads) on a bounded
    sample of the same workload: repeated 11008 x 4096 Q4_K matvecs."""
    from oracle import oracle as O
    from tcb_b200 import synth

    N, K = WORKLOAD["N"], WORKLOAD["K"]
    w = synth.weight(Q4_K, N, K, seed=7)
    x = synth.activations(1, K, seed=8)
    threads = len(os.sched_getaffinity(0))
    O.set_pinning(True)
    try:
        O.qgemm_float(Q4_K, x, w, N, nthreads=threads)  # warm
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            O.qgemm_float(Q4_K, x, w, N, nthreads=threads)
            n += 1
        dt = time.perf_counter() - t0
    finally:
        O.set_pinning(False)
    return {"value": round(algorithmic_bytes(N, K) * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port", "pinning": f"one worker thread per allowed CPU ({threads} of os.cpu_count() = "
                                       f"{os.cpu_count()}), pthread_setaffinity_np",
            "sample": f"{n} matvecs of Q4_K 11008x4096 (float path, oracle AVX2 restatement) in {dt:.1f} s"}


def decode_bench(ctx, rank: int, world: int, peak_gbs: float) -> dict:
    """8B-shape Q4_K_M greedy decode at batch 1: a
    512-token random prompt fed by the prompt pass (tcb_llama_prefill: 511
    rows through the tensor-core products, the last token by the first step),
    then 256 greedy tokens, every step one replay of the captured CUDA graph
    (token, position and prompt stay on the device).  Random-init synthetic
    weights (fp16 block scales sized for order-one activations,
    tcb_b200/llama.py)."""
    import torch

    from tcb_b200 import llama

    cfg = llama.LLAMA3_8B
    model = llama.device_model(cfg, seed=7, varied=True)
    eng = llama.Llama(ctx, model)
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 512)
    stream = torch.cuda.Stream()
    eng.start(prompt, stream)
    eng.capture(stream)
    kernels_per_token = eng.step_kernels()
    eng.start(prompt, stream)
    eng.prefill(stream)  # warm-up of the prompt pass (workspace, kernel attributes)
    eng.start(prompt, stream)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    with torch.cuda.stream(stream):
        e0.record(stream)
        eng.prefill(stream)
        e1.record(stream)
        eng.step(256, stream)
        e2.record(stream)
    e2.synchronize()
    t = torch.tensor([e1.elapsed_time(e2)], dtype=torch.float64, device="cuda")
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    toks = eng.tokens(768, stream)
    bpt = llama.weight_bytes_per_token(cfg)
    kv = 2 * cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * (512 + 128)  # fp16 K/V read per token (mean position)
    per_tok_s = ms / 1e3 / 256
    eng.close()
    del model
    return {
        "model": "llama3-8b-shape q4_k_m (random init, synthetic)", "prompt_tokens": 512, "generated_tokens": 256,
        "tokens_per_s": round(256 * world / (ms / 1e3), 2), "ms_per_token": round(ms / 256, 4),
        "prompt_pass_ms": round(e0.elapsed_time(e1), 2),
        "bytes_per_token": bpt + kv, "weight_bytes_per_token": bpt,
        "roofline": {"bound": "hbm", "achieved": round((bpt + kv) / per_tok_s / 1e9, 2), "peak": peak_gbs,
                     "unit": "GB/s", "frac": round((bpt + kv) / per_tok_s / 1e9 / peak_gbs, 4),
                     "ceiling_tokens_per_s": round(peak_gbs * 1e9 / (bpt + kv), 1)},
        "gpu_launches_per_token": kernels_per_token, "last_tokens": [int(v) for v in toks[-8:]],
        "distinct_generated_tokens": len(set(int(v) for v in toks[512:])),
        "timing": "CUDA events around 256 graph replays on the engine's stream",
    }


def matvec_table_bench(ctx, rank: int, peak_gbs: float) -> dict:
    """BASELINE configs 1 and 2 beside the headline shape: Q8_0 4096x4096 at
    batch 1 (float path and int8-activation path), Q4_0 and Q4_K at
    11008x4096 and 4096x11008 for batch 1, 4 and 8 (f32 x ~ N(0, 1), f32 y).
    Each case sweeps a cold ring of at least 512 MiB of distinct weight copies
    (one code byte per block flipped), captured in a CUDA graph; CUDA events
    around 20 sweeps after 3 warm-up sweeps.  GB/s = algorithmic bytes
    (weight blocks + M*K*4 + M*N*4) per call / time."""
    import torch

    from tcb_b200 import synth

    code_off = {Q8_0: 2, Q4_0: 2, Q4_K: 16}
    code_len = {Q8_0: 32, Q4_0: 16, Q4_K: 128}
    blk = {Q8_0: (32, 34), Q4_0: (32, 18), Q4_K: (256, 144)}
    names = {Q8_0: "q8_0", Q4_0: "q4_0", Q4_K: "q4_k"}
    cases = [(Q8_0, 4096, 4096, (1,), (False, True))]
    for wt in (Q4_0, Q4_K):
        for N, K in ((11008, 4096), (4096, 11008)):
            cases.append((wt, N, K, (1, 4, 8), (False,)))
    rows = []
    stream = torch.cuda.Stream()
    for wt, N, K, Ms, modes in cases:
        E, B = blk[wt]
        wbytes = N * K // E * B
        ring = max(4, -(-512 * 2 ** 20 // wbytes))
        base = torch.from_numpy(synth.weight(wt, N, K, seed=41 + rank)).cuda()
        weights = [base]
        for i in range(1, ring):
            w = base.clone()
            w[code_off[wt] + (i % code_len[wt])::B] ^= 0x11
            weights.append(w)
        for M in Ms:
            x = torch.from_numpy(synth.activations(M, K, seed=43 + rank)).cuda()
            y = torch.empty((M, N), dtype=torch.float32, device="cuda")
            for act8 in modes:
                def sweep():
                    for w in weights:
                        ctx.qgemm(wt, w, x, y, stream=stream, act8=act8)

                with torch.cuda.stream(stream):
                    sweep()
                    stream.synchronize()
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        sweep()
                    for _ in range(3):
                        g.replay()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(20):
                        g.replay()
                    e1.record(stream)
                    e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (20 * ring)
                gbs = (wbytes + M * K * 4 + M * N * 4) / (us * 1e-6) / 1e9
                rows.append([names[wt], N, K, M, "act8" if act8 else "float", round(us, 2), round(gbs, 1),
                             round(gbs / peak_gbs, 4)])
                del g
        del weights, base
    return {"timing": "CUDA graph of one sweep over a cold weight ring (>= 512 MiB), 20 sweeps",
            "peak_gbs": peak_gbs, "columns": ["wtype", "N", "K", "M", "path", "us_per_call", "GB/s", "frac"],
            "cases": rows}


def model_prefill_bench(ctx, peaks: dict, layers: int = 0) -> dict:
    """8B-shape model prefill (second part): a batch of 4
    random 2048-token prompts, one engine (KV cache) per sequence on the same
    weights, fed by one batched prompt pass (tcb_llama_prefill_batch: the
    products over all 4 x 2047 rows at once, rotary, cache append and causal
    flash attention per sequence), then each sequence's first decode step
    (its last prompt token and first greedy token): the time is the batch's
    time to first token.  CUDA events around the pass and the 4 steps, after
    one warm-up batch.  Tensor roofline: the products' 2*rows*N*K flops plus
    the causal attention's 4*hd per (query head, query, key) pair, against
    the measured sustained dense bf16 peak (a pass of over a hundred
    milliseconds)."""
    import dataclasses

    import torch

    from tcb_b200 import llama

    T_, B = 2048, 4
    cfg = dataclasses.replace(llama.LLAMA3_8B, max_ctx=T_ + 1)
    if layers:  # profiling: the same layer shapes, fewer layers
        cfg = dataclasses.replace(cfg, n_layers=layers)
    model = llama.device_model(cfg, seed=7)
    engines = [llama.Llama(ctx, model) for _ in range(B)]
    stream = torch.cuda.Stream()
    rng = np.random.default_rng(17)
    ms = []
    for rep in range(2):  # the first batch warms up (row buffers, workspace)
        prompts = [rng.integers(0, cfg.vocab, T_) for _ in range(B)]
        for eng, p in zip(engines, prompts):
            eng.start(p, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            llama.prefill_batch(engines, stream)
            for eng in engines:
                eng.step(1, stream)
            e1.record(stream)
        e1.synchronize()
        if rep:
            ms.append(e0.elapsed_time(e1))
    toks = engines[0].tokens(T_ + 1, stream)
    for eng in engines:
        eng.close()
    del model
    D, H, KVH, hd, F, L = cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.n_layers
    rows = T_ - 1
    per_row = 2 * ((H + 2 * KVH) * hd * D + D * H * hd + 2 * F * D + D * F)
    attn = 4 * hd * H * (rows * (rows + 1) // 2)
    flops = L * (rows * per_row + attn)
    total = sum(ms)
    peak = peaks.get("bf16_tflops_sustained") or peaks.get("bf16_tflops")
    tf = flops * B / (total / 1e3) / 1e12
    return {"model": "llama3-8b-shape q4_k_m (random init, synthetic)", "prompt_tokens": T_, "batch": B,
            "batch_mode": "one prompt pass over all sequences' rows (an engine and KV cache per sequence)",
            "tokens_per_s": round(T_ * B / (total / 1e3), 1), "ms_per_batch": round(total, 2),
            "time_to_first_token_ms": round(total, 2),
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tf / peak, 4) if peak else None,
                         "flops_per_sequence": flops,
                         "peak_source": ("measured (sustained)" if peaks.get("source") == "measured" else "fallback")},
            "first_token": int(toks[-1])}


def prefill_bench(ctx, rank: int, peaks: dict, cpu: bool) -> dict:
    """Prefill product: Q4_K weights 14336x4096 and
    4096x14336 against bf16 activations of M = 2048 rows, f32 output, through
    the tcgen05 kernel.  Each shape cycles through 4 weight copies (more than
    the 126 MB L2 together); CUDA events around 20 calls after 3 warm-up
    calls.  Tensor roofline: 2*M*N*K flops against the measured dense bf16
    peak (burst figure: the kernel is timed alone)."""
    import torch

    from tcb_b200 import synth

    M = 2048
    out = {"model": "q4_k x bf16 prefill products (synthetic)", "M": M, "x_dtype": "bf16", "c_dtype": "f32",
           "shapes": []}
    peak = peaks.get("bf16_tflops")
    stream = torch.cuda.Stream()
    for N, K in ((14336, 4096), (4096, 14336)):
        ring = [torch.from_numpy(synth.weight(Q4_K, N, K, seed=31 + i + rank)).cuda() for i in range(4)]
        x = torch.from_numpy(synth.activations(M, K, seed=33 + rank)).cuda().to(torch.bfloat16)
        c = torch.empty((M, N), dtype=torch.float32, device="cuda")
        with torch.cuda.stream(stream):
            for i in range(3):
                ctx.qgemm(Q4_K, ring[i % 4], x, c, stream=stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = 20
            e0.record(stream)
            for i in range(n):
                ctx.qgemm(Q4_K, ring[i % 4], x, c, stream=stream)
            e1.record(stream)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / n
        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
        row = {"N": N, "K": K, "us_per_call": round(ms * 1e3, 1), "tflops": round(tf, 1),
               "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                            "frac": round(tf / peak, 4) if peak else None,
                            "peak_source": ("measured (burst)" if peaks.get("source") == "measured" else "fallback")}}
        if cpu and rank == 0:
            # the oracle's float path on the host cores, on a sample of rows
            from oracle import oracle as O

            xs = x[:16].float().cpu().numpy()
            w = ring[0].cpu().numpy()
            t0 = time.perf_counter()
            O.qgemm_float(Q4_K, xs, w, N)
            dt = time.perf_counter() - t0
            row["cpu_baseline"] = {"value": round(2.0 * 16 * N * K / dt / 1e12, 4), "unit": "TFLOP/s",
                                   "cores": os.cpu_count(), "kind": "port",
                                   "sample": f"16 of {M} rows through the oracle's float path"}
        out["shapes"].append(row)
        if N == 14336:
            # the same product with int8-quantised activations (TR's
            # quantGemmQ8, bit-exact): integer block sums on tcgen05 kind::i8
            with torch.cuda.stream(stream):
                for i in range(2):
                    ctx.qgemm_act8(Q4_K, ring[i % 4], x, c, stream=stream)
                e0.record(stream)
                for i in range(n):
                    ctx.qgemm_act8(Q4_K, ring[i % 4], x, c, stream=stream)
                e1.record(stream)
                e1.synchronize()
            ms8 = e0.elapsed_time(e1) / n
            tops = 2.0 * M * N * K / (ms8 / 1e3) / 1e12
            peak8 = 2.0 * peak if peak else None
            out["act8"] = {"N": N, "K": K, "M": M, "us_per_call": round(ms8 * 1e3, 1), "tops": round(tops, 1),
                           "roofline": {"bound": "tensor", "achieved": round(tops, 1), "peak": peak8, "unit": "TOP/s",
                                        "frac": round(tops / peak8, 4) if peak8 else None,
                                        "peak_source": "int8 dense = 2 x the measured dense bf16 burst"},
                           "path": "int8 activations (bit-exact), tcgen05.mma.kind::i8"}
        del ring, x, c
    return out


def decode_tp_bench(ctx, rank: int, world: int, peak_gbs: float, batch16: bool = True) -> dict:
    """70B-shape Q4_K_M greedy decode at batch 1, on one GPU or
    tensor-parallel over the world's GPUs (QKV/gate/up
    column-parallel, o/down row-parallel with a residual all-reduce each,
    vocabulary-parallel head): a 1024-token random prompt fed by the prompt
    pass (1023 rows through the tensor-core products, residual rows summed by
    NCCL), then 128 greedy tokens, every step one replay of the captured
    graph.  The weights are one model at every degree (each global tensor
    from its own counter-based generator, each rank keeping its slice), so
    the tokens are comparable across N."""
    import torch
    import torch.distributed as dist

    from tcb_b200 import llama

    cfg = llama.LLAMA3_70B
    model = llama.device_model(cfg, seed=9, tp=(world, rank), varied=True)
    eng = llama.Llama(ctx, model, tp=(world, rank))
    if world > 1:
        eng.tp_init(llama.share_id(llama.nccl_unique_id, rank))
    prompt = np.random.default_rng(13).integers(0, cfg.vocab, 1024)
    stream = torch.cuda.Stream()
    eng.start(prompt, stream)
    eng.capture(stream)
    eng.start(prompt, stream)
    eng.prefill(stream)  # warm-up of the prompt pass
    eng.start(prompt, stream)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    with torch.cuda.stream(stream):
        e0.record(stream)
        eng.prefill(stream)
        e1.record(stream)
        eng.step(128, stream)
        e2.record(stream)
    e2.synchronize()
    t = torch.tensor([e1.elapsed_time(e2), e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, pms = float(t[0].item()), float(t[1].item())
    toks = eng.tokens(1152, stream)
    eng.close()
    batch = decode_batch_bench(ctx, model, rank, world, peak_gbs, stream) if batch16 else None
    del model
    bpt = llama.weight_bytes_per_token(cfg)
    per_gpu = bpt / world
    out = {
        "model": "llama3-70b-shape q4_k_m (random init, synthetic)", "tensor_parallel": world,
        "prompt_tokens": 1024, "generated_tokens": 128, "tokens_per_s": round(128 / (ms / 1e3), 2),
        "prompt_pass_ms": round(pms, 2),
        "ms_per_token": round(ms / 128, 4), "weight_bytes_per_token": bpt, "weight_bytes_per_gpu_per_token": per_gpu,
        "roofline": {"bound": "hbm", "achieved_per_gpu": round(per_gpu / (ms / 1e3 / 128) / 1e9, 2),
                     "peak": peak_gbs, "unit": "GB/s", "frac": round(per_gpu / (ms / 1e3 / 128) / 1e9 / peak_gbs, 4),
                     "ceiling_tokens_per_s": round(peak_gbs * 1e9 / per_gpu, 1)},
        "allreduce": ("none (one GPU)" if world == 1 else
                      "peer memory (NVLink)" if getattr(eng, "peer_active", False) else "nccl"),
        "collectives_per_token": 0 if world == 1 else 2 * cfg.n_layers + 1,
        "last_tokens": [int(v) for v in toks[-8:]],
        "distinct_generated_tokens": len(set(int(v) for v in toks[1024:])),
        "timing": "CUDA events around 128 graph replays, max over ranks",
    }
    if batch is not None:
        out["batch16"] = batch
    return out


def decode_batch_bench(ctx, model, rank: int, world: int, peak_gbs: float, stream, B: int = 16, cfg=None) -> dict:
    """BASELINE config 5 at batch 16: 16 sequences on the same 70B-shape
    weights, each with its own 1024-token random prompt and K/V cache, fed by
    one batched prompt pass (tcb_llama_prefill_batch), then 128 greedy steps
    of all 16 together (tcb_llama_batch: each product once over the 16 rows,
    attention per sequence), every step one replay of the captured graph.
    tokens/s counts the tokens of all sequences."""
    import torch
    import torch.distributed as dist

    from tcb_b200 import llama

    cfg = cfg or llama.LLAMA3_70B
    engines = [llama.Llama(ctx, model, tp=(world, rank)) for _ in range(B)]
    if world > 1:
        engines[0].tp_init(llama.share_id(llama.nccl_unique_id, rank))
    rng = np.random.default_rng(19)
    prompts = [rng.integers(0, cfg.vocab, 1024) for _ in range(B)]
    for e, p in zip(engines, prompts):
        e.start(p, stream)
    batch = llama.Batch(engines)
    batch.step(1, stream)  # sizes the products' scratch before the capture
    batch.capture(stream)
    for e, p in zip(engines, prompts):
        e.start(p, stream)
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    with torch.cuda.stream(stream):
        e0.record(stream)
        llama.prefill_batch(engines, stream)
        e1.record(stream)
        batch.step(128, stream)
        e2.record(stream)
    e2.synchronize()
    t = torch.tensor([e1.elapsed_time(e2), e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, pms = float(t[0].item()), float(t[1].item())
    toks = [e.tokens(1152, stream) for e in engines]
    # the engine sums the residual rows over peer memory up to 16 sequences
    allreduce = ("none (one GPU)" if world == 1 else
                 "peer memory (NVLink)" if getattr(engines[0], "peer_active", False) and B <= 16 else "nccl")
    batch.close()
    for e in engines:
        e.close()
    bpt = llama.weight_bytes_per_token(cfg)
    per_gpu_step = bpt / world
    return {"batch": B, "prompt_tokens": 1024, "generated_tokens": 128, "allreduce": allreduce,
            "tokens_per_s": round(B * 128 / (ms / 1e3), 2), "ms_per_step": round(ms / 128, 4),
            "prompt_pass_ms": round(pms, 2),
            "roofline": {"bound": "hbm", "achieved_per_gpu": round(per_gpu_step / (ms / 1e3 / 128) / 1e9, 2),
                         "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(per_gpu_step / (ms / 1e3 / 128) / 1e9 / peak_gbs, 4),
                         "note": "weight bytes of one step (once per step, as if every product streamed "
                                 "its weights once for all rows)"},
            "last_tokens": [[int(v) for v in t[-4:]] for t in toks[:4]],
            "distinct_generated_tokens": len(set(int(v) for t in toks for v in t[1024:])),
            "timing": "CUDA events around 128 replays of the batch step graph, max over ranks"}


def dist_init():
    if "RANK" not in os.environ:
        return 0, 1, 0
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local


def run_config(world: int) -> dict:
    """The workload's config object, the same on both arms."""
    wbytes = WORKLOAD["N"] * WORKLOAD["K"] // 256 * 144
    ring = max(4, -(-512 * 2 ** 20 // wbytes))  # >= 512 MiB of distinct weights
    return dict(WORKLOAD, ring=ring, ring_bytes=ring * wbytes, l2="inputs larger than L2 (cold ring)",
                parallelism=f"replicas{world}")


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    cb = cpu_baseline()
    line = {"metric": METRIC, "value": cb["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "impl": "reference", "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": run_config(world), "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


_RESULT = None  # the process's original stdout, kept for the JSON line


def claim_stdout():
    """Point fd 1 at stderr for the rest of the run, so that what libraries
    print on stdout (NCCL's version banner when a debug level is set) cannot
    mix with the result; the JSON line goes to the original stdout."""
    global _RESULT
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def emit(obj: dict):
    out = _RESULT if _RESULT is not None else sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def product_bench(ctx, wname: str, n: str, k: str, m: str, act8: bool = False) -> dict:
    """One product (synthetic weights and activations), 4 warm-up and 10 timed
    calls on the default stream: the profiling case of a kernel."""
    import torch

    import tcb_b200 as T
    from tcb_b200 import synth

    wt = {"q4_k": T.Q4_K, "q6_k": T.Q6_K, "q4_0": T.Q4_0, "q8_0": T.Q8_0}[wname]
    N, K, M = int(n), int(k), int(m)
    w = torch.from_numpy(synth.weight(wt, N, K, seed=1)).cuda()
    x = torch.from_numpy(synth.activations(M, K, seed=2)).cuda()
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    for _ in range(4):
        ctx.qgemm(wt, w, x, c, act8=act8)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        ctx.qgemm(wt, w, x, c, act8=act8)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / 10
    wb = N * K // T.BLOCK[wt][0] * T.BLOCK[wt][1]
    return {"wtype": wname, "N": N, "K": K, "M": M, "act8": act8, "us_per_call": round(us, 2),
            "weight_GBs": round(wb / us / 1e3, 1), "device_error": ctx.device_error()}


def main():
    claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the 8B-shape decode measurement")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill-product measurement")
    ap.add_argument("--no-configs", action="store_true", help="skip the BASELINE config 1/2 matvec table")
    ap.add_argument("--only-model-prefill", action="store_true",
                    help="run only the 8B model prefill and print its object (for profiling)")
    ap.add_argument("--layers", type=int, default=0,
                    help="with --only-model-prefill / --only-batch16: this many layers (small profiling case)")
    ap.add_argument("--only-product", nargs=4, metavar=("WTYPE", "N", "K", "M"),
                    help="run only one product (q4_k, q6_k, q4_0, q8_0; N x K weight, M rows of x) a few "
                         "times and print its time (for profiling)")
    ap.add_argument("--act8", action="store_true", help="with --only-product: the int8-activation product")
    ap.add_argument("--only-decode", action="store_true", help="run only the 8B decode and print its object")
    ap.add_argument("--only-batch16", action="store_true",
                    help="run only the 70B-shape batch-16 decode (with --layers: fewer layers) and print it")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank, world, local = dist_init()
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    import torch

    import tcb_b200 as T
    from tcb_b200 import synth

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.only_model_prefill:
        emit({"model_prefill": model_prefill_bench(T.Context(local), load_peaks(), args.layers)})
        return
    if args.only_product:
        emit({"product": product_bench(T.Context(local), *args.only_product, act8=args.act8)})
        return
    if args.only_decode:
        emit({"decode": decode_bench(T.Context(local), rank, world, load_peaks()["hbm_gbs"])})
        return
    if args.only_batch16:
        import dataclasses

        from tcb_b200 import llama

        cfg = llama.LLAMA3_70B if not args.layers else dataclasses.replace(llama.LLAMA3_70B, n_layers=args.layers)
        ctx = T.Context(local)
        model = llama.device_model(cfg, seed=9, varied=True)
        emit({"batch16": decode_batch_bench(ctx, model, rank, world, load_peaks()["hbm_gbs"],
                                            torch.cuda.Stream(dev), cfg=cfg)})
        return
    N, K = WORKLOAD["N"], WORKLOAD["K"]
    config = run_config(world)
    ring = config["ring"]
    ctx = T.Context(local)
    base = torch.from_numpy(synth.weight(Q4_K, N, K, seed=1 + rank)).to(dev)
    weights = [base]
    for i in range(1, ring):
        # distinct copies: flip the nibbles of one byte per block row so no two are equal
        w = base.clone()
        w[16 + (i % 128)::144] ^= 0x11
        weights.append(w)
    x = torch.from_numpy(synth.activations(1, K, seed=2 + rank)).to(dev)
    ys = [torch.empty((1, N), dtype=torch.float32, device=dev) for _ in range(ring)]
    stream = torch.cuda.Stream(dev)

    def sweep():
        for i in range(ring):
            ctx.qgemm(Q4_K, weights[i], x, ys[i], accumulate=False, stream=stream)

    with torch.cuda.stream(stream):
        sweep()  # first call outside capture (lazy attributes)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            sweep()
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                g.replay()
            stop.record(stream)
        stop.synchronize()
    barrier()
    ms = start.elapsed_time(stop)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    launches = args.steps * ring
    per_launch_bytes = algorithmic_bytes(N, K)
    value = per_launch_bytes * launches * world / (ms_max / 1e3) / 1e9
    kernel_s = ms / 1e3 / launches  # this rank's average duration per launch
    peaks = load_peaks()
    achieved = per_launch_bytes / kernel_s / 1e9

    # e2e with host buffers, eager calls, every step: x moved in from pinned
    # memory, the product, y moved back.  Headline: the host-buffer entry
    # tcb_qgemm_host called as a cgo/purego host calls it (one call a step,
    # the pointers resolved once).  Beside it: the same step as three calls
    # (cudaMemcpyAsync, tcb_qgemm, cudaMemcpyAsync) and the Python mirror
    # (torch tensor copies and Context.qgemm).
    import ctypes

    xh = torch.from_numpy(synth.activations(1, K, seed=2 + rank)).pin_memory()
    yh = torch.empty((1, N), dtype=torch.float32).pin_memory()
    e2e_steps = max(200, args.steps // 4)
    rt = ctypes.CDLL("libcudart.so.12")
    rt.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p]
    rt.cudaMemcpyAsync.restype = ctypes.c_int
    qgemm = T.lib().tcb_qgemm
    qgemm_host = T.lib().tcb_qgemm_host
    sh, hctx = stream.cuda_stream, ctx._h
    xp, xhp, yp, yhp = x.data_ptr(), xh.data_ptr(), ys[0].data_ptr(), yh.data_ptr()
    wps = [w.data_ptr() for w in weights]

    def host_step(i):
        # x read from pinned host memory by the library's staging kernel, y
        # written into pinned host memory by the product
        return qgemm_host(hctx, Q4_K, 1, N, K, wps[i % ring], xhp, T.F32, K, yhp, T.F32, N, 0, sh)

    def capi_step(i):
        rc = rt.cudaMemcpyAsync(xp, xhp, K * 4, 1, sh)  # cudaMemcpyHostToDevice
        rc |= qgemm(hctx, Q4_K, 1, N, K, wps[i % ring], xp, T.F32, K, yp, T.F32, N, 0, sh)
        return rc | rt.cudaMemcpyAsync(yhp, yp, N * 4, 2, sh)  # cudaMemcpyDeviceToHost

    def torch_step(i):
        x.copy_(xh, non_blocking=True)
        ctx.qgemm(Q4_K, weights[i % ring], x, ys[0], accumulate=False, stream=stream)
        yh.copy_(ys[0], non_blocking=True)
        return 0

    def e2e(step_fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rc = 0
        with torch.cuda.stream(stream):
            for i in range(20):
                rc |= step_fn(i)
            barrier()
            e0.record(stream)
            for i in range(e2e_steps):
                rc |= step_fn(i)
            e1.record(stream)
            e1.synchronize()
        if rc:
            raise RuntimeError(f"e2e step failed (status {rc})")
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        return per_launch_bytes * e2e_steps * world / (float(et.item()) / 1e3) / 1e9

    e2e_value = e2e(host_step)
    e2e_copies = e2e(capi_step)
    e2e_torch = e2e(torch_step)
    del g
    decode = decode70 = None
    if not args.no_decode:
        if world == 1:
            decode = decode_bench(ctx, rank, world, peaks["hbm_gbs"])
        torch.cuda.empty_cache()
        decode70 = decode_tp_bench(ctx, rank, world, peaks["hbm_gbs"])
        torch.cuda.empty_cache()

    table = matvec_table_bench(ctx, rank, peaks["hbm_gbs"]) if world == 1 and not args.no_configs else None
    prefill = model_prefill = None
    if world == 1 and not args.no_prefill:
        prefill = prefill_bench(ctx, rank, peaks, not args.no_cpu_baseline)
        model_prefill = model_prefill_bench(ctx, peaks)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "pct_of_peak": round(100 * value / world / peaks["hbm_gbs"], 2),
            "config": config,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                         "traffic": TRAFFIC_BYTES_PER_LAUNCH,
                         "traffic_source": "dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
                                           "kernel under ncu, summarised in profiles/q4k_matvec_11008x4096.md",
                         "algorithmic_bytes_per_launch": per_launch_bytes},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": K * 4,
                    "d2h_bytes_per_step": N * 4, "steps": e2e_steps,
                    "calls": "per step: one tcb_qgemm_host over pinned host x and y (x read over the host link "
                             "by a staging kernel, y written into host memory by the product)",
                    "copy_engine": {"value": round(e2e_copies, 2),
                                    "calls": "per step: cudaMemcpyAsync x from pinned memory, tcb_qgemm, "
                                             "cudaMemcpyAsync y back"},
                    "python_mirror": {"value": round(e2e_torch, 2),
                                      "calls": "torch copy_ of x, Context.qgemm, torch copy_ of y, per step"}},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        # the driver keeps the end of stdout: the long table first, the
        # decoder figures last
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        if table is not None:
            line["matvec_configs"] = table
        if prefill is not None:
            line["prefill"] = prefill
        if model_prefill is not None:
            line["model_prefill"] = model_prefill
        if decode70 is not None:
            line["decode_70b"] = decode70
        if decode is not None:
            line["decode"] = decode
        emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""bench.py -- AR semantic tokens/s of the B200 hot path on BASELINE config 4 (box-wide serving).

One bench step = one serving job per GPU: 64 sequence slots, prefixes U[80,400] split 70/30
phones/prompt codes, 1500 decode iterations with top_k 15 / rep 1.35 sampling and EOS (1024) on;
finished slots are refilled from a seeded request queue every 16 iterations. Weak scaling: every
rank runs its own 64-slot shard with its own request stream (no data-path collective).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gsvcu|reference]

value: job throughput with the requests' BERT features already in HBM (device pointers to the C ABI);
e2e:   the same jobs through the same C ABI with every input in host memory (H2D inside the timed
       region) and every finished sequence's tokens read back to the host.
Timing: CUDA events on the library's stream, barrier + synchronize on both sides, max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for sub in ("gsv.cpp_b200", "oracle"):
    sys.path.insert(0, os.path.join(ROOT, sub))

METRIC = "AR semantic tokens/s (batched decode, box)"
MODEL_CACHE = os.environ.get("GSVCU_MODEL_CACHE", "/tmp/gsvcu_models")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="gsvcu", choices=["gsvcu", "reference"])
    ap.add_argument("--slots", type=int, default=64)
    ap.add_argument("--iters", type=int, default=1500)
    ap.add_argument("--refill-every", type=int, default=16)
    ap.add_argument("--kv", default="f16", choices=["f16", "f32"])
    ap.add_argument("--format", default="q8_0", choices=list(FORMATS),
                    help="model file of the serve workload: q8_0 (the exporter's --q8, the headline), f16 (its --f16 "
                         "preset: F16 matrices, predict and embeddings), f32 (no flags), q6_k (--spec "
                         "attn=q8_0,ffn=q6_k,predict=f16,emb=f16) or q4_1 (--spec attn=q4_1,ffn=q4_1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-chunks", type=int, default=3,
                    help="chunks (of --refill-every iterations) of the job the cpu_baseline sample runs")
    ap.add_argument("--dit-steps", type=int, default=8, help="Euler steps per sample call of the dit workload")
    ap.add_argument("--kv-f32-steps", type=int, default=3,
                    help="jobs of the extra F32-KV (reference-exact) measurement; 0 skips it")
    ap.add_argument("--lookahead", action="store_true",
                    help="serve with gsvcu_set_serve_lookahead (the next chunk runs while the host handles results)")
    ap.add_argument("--workload", default="serve", choices=["serve", "attn", "gemv", "prefill", "single", "bert", "dit"],
                    help="serve: config-4 serving shard (the bench line); attn: config-3 decode-attention sweep; "
                         "gemv: config-3 Q8_0 GEMV sweep; prefill: config-2 prefill attention + GEMMs; "
                         "single: config-0 single-sequence decode latency; bert: the BERT feature producer "
                         "(published 1024 / 16 / 4096 shape, 22 layers used, F16 matrices)")
    ap.add_argument("--attn-batches", default="1,8,32,64,128")
    ap.add_argument("--prefill-gemm", default="auto", choices=["auto", "tc", "mma"],
                    help="prefill Q8_0 GEMMs: tc = tcgen05/TMEM kernel, mma = mma.sync tiles, auto = the library default")
    return ap.parse_args()


def attn_sweep(args):
    """decode attention alone, B in {1,8,32,64,128}, per-sequence lengths U[256,2048],
    one layer of a paged F16 (or F32) pool, q ~ N(0,1). Prints one JSON line per B with the achieved
    algorithmic GB/s (K+V rows of every key + q in + Q8_0 out) against the measured HBM peak."""
    import torch
    import gsvcu
    ctx = gsvcu.Context(0)
    kv = gsvcu.KV_F16 if args.kv == "f16" else gsvcu.KV_F32
    elem = 2 if kv == gsvcu.KV_F16 else 4
    peak, peak_kind = measured_peaks()
    for B in [int(b) for b in args.attn_batches.split(",")]:
        rng = np.random.default_rng(B)
        lens = rng.integers(256, 2049, B)
        pages = [(int(l) + 63) // 64 for l in lens]
        maxp = max(pages) + 1
        npages = sum(pages) + 1
        dt = torch.float16 if kv == gsvcu.KV_F16 else torch.float32
        pool = torch.randn((npages, 1, 2, 16, 64, 32), device="cuda", dtype=torch.float32).to(dt)
        perm = torch.randperm(npages, device="cpu").numpy().astype(np.int32)
        bt = np.zeros((B, maxp), np.int32)
        at = 0
        for b, n in enumerate(pages):
            bt[b, :n] = perm[at:at + n]
            at += n
        q = torch.randn((B, 512), device="cuda")
        kvpos = torch.tensor(lens - 1, dtype=torch.int32, device="cuda")
        active = torch.ones(B, dtype=torch.int32, device="cuda")
        btd = torch.from_numpy(bt).cuda()
        oq = torch.empty((B, 512), dtype=torch.int8, device="cuda")
        od = torch.empty((B, 16), dtype=torch.int16, device="cuda")
        ext = torch.cuda.ExternalStream(ctx.stream_handle())
        call = lambda: ctx.op_decode_attention(q, 512, pool, kv, 1, 0, btd, maxp, kvpos, active, B, oq, od)
        for _ in range(max(args.warmup, 200)):   # also lets the SM clock ramp up before timing
            call()
        ctx.sync()
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")   # > L2 between timed launches
        times = []
        for _ in range(max(args.steps, 5)):
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(ext):
                # the flush runs on the library's stream, so the launch below is queued while it runs
                # and the timed interval holds no host-side launch latency
                flush.zero_()
            e0.record(ext)
            call()
            e1.record(ext)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = float(np.median(times))
        keys = int(lens.sum())
        nbytes = keys * 2 * 512 * elem + B * (512 * 4 + 512 + 32)
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"workload": "cfg3 decode attention", "B": B, "kv": args.kv, "keys": keys,
                          "algorithmic_bytes": nbytes, "ms": ms, "GBps": gbs, "peak": peak, "peak_kind": peak_kind,
                          "frac": gbs / peak, "l2": "256 MiB flush between launches"}))
        del pool, flush
        torch.cuda.empty_cache()
    ctx.close()


def _flush_and_time(ext, flush, call, reps):
    """Median CUDA-event time (ms) of call() on the library stream, L2 flushed before each launch."""
    import torch
    times = []
    for _ in range(reps):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(ext):
            flush.zero_()
        e0.record(ext)
        call()
        e1.record(ext)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    return float(np.median(times))


def _rand_q8(rng, rows, K):
    """Random Q8_0 blocks in GGUF layout [rows][K/32][34]: fp16 scale + 32 int8 (no quantizer needed)."""
    raw = np.zeros((rows, K // 32, 34), np.uint8)
    raw[..., :2] = (rng.uniform(0.0005, 0.002, (rows, K // 32)).astype(np.float16)).view(np.uint8).reshape(rows, K // 32, 2)
    raw[..., 2:] = rng.integers(-127, 128, (rows, K // 32, 32)).astype(np.int8).view(np.uint8)
    return raw


def gemv_sweep(args):
    """BASELINE config 3, GEMV half: Q8_0 GEMM/GEMV shapes 512x1536, 512x512, 512x2048, 2048x512 (the unfused
    decode kernels, one launch each) and the 512x1025 F32 logits projection, at B in {1,8,32,64,128}, with a
    256 MiB L2 flush before each launch. Algorithmic bytes: weights (34/32 B per Q8_0 weight, 4 B per F32
    weight) + activations in + outputs."""
    import torch
    import gsvcu
    ctx = gsvcu.Context(0)
    ext = torch.cuda.ExternalStream(ctx.stream_handle())
    peak, peak_kind = measured_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(3)
    for (N, K) in [(1536, 512), (512, 512), (2048, 512), (512, 2048)]:
        raw = _rand_q8(rng, N, K)
        wq = torch.empty(N * K, dtype=torch.uint8, device="cuda")
        wd = torch.empty(N * K // 32, dtype=torch.int16, device="cuda")
        ctx.op_pack_q8_0(raw, N, K, wq, wd)
        bias = torch.randn(N, device="cuda")
        for B in [int(b) for b in args.attn_batches.split(",")]:
            xraw = _rand_q8(rng, B, K)
            xq = torch.from_numpy(np.ascontiguousarray(xraw[..., 2:]).reshape(B, K).view(np.int8)).cuda()
            xd = torch.from_numpy(np.ascontiguousarray(xraw[..., :2]).reshape(B, K // 32, 2).view(np.int16)
                                  .reshape(B, K // 32)).cuda()
            y = torch.empty((B, N), device="cuda")
            call = lambda: ctx.op_q8_gemm(xq, xd, B, wq, wd, N, K, bias, None, gsvcu.EPI_BIAS, y=y)
            for _ in range(max(args.warmup, 50)):
                call()
            ms = _flush_and_time(ext, flush, call, max(args.steps, 5))
            nbytes = N * K * 34 // 32 + B * (K + K // 16) + B * N * 4 + N * 4
            gbs = nbytes / (ms * 1e-3) / 1e9
            print(json.dumps({"workload": "cfg3 Q8_0 GEMV", "shape": f"{K}x{N}", "B": B, "algorithmic_bytes": nbytes,
                              "ms": ms, "GBps": gbs, "peak": peak, "peak_kind": peak_kind, "frac": gbs / peak,
                              "kernel": "k_gemm_q8 (unfused decode path, one launch)",
                              "l2": "256 MiB flush before each launch"}))
    N, K = 1025, 512
    w = torch.randn((N, K), device="cuda") * 0.02
    for B in [int(b) for b in args.attn_batches.split(",")]:
        x = torch.randn((B, K), device="cuda")
        y = torch.empty((B, N), device="cuda")
        call = lambda: ctx.op_f32_gemm(x, B, w, N, K, None, y)
        for _ in range(max(args.warmup, 50)):
            call()
        ms = _flush_and_time(ext, flush, call, max(args.steps, 5))
        nbytes = N * K * 4 + B * K * 4 + B * N * 4
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"workload": "cfg3 logits GEMV (F32 predict)", "shape": f"{K}x{N}", "B": B,
                          "algorithmic_bytes": nbytes, "ms": ms, "GBps": gbs, "peak": peak, "peak_kind": peak_kind,
                          "frac": gbs / peak, "kernel": "k_logits512", "l2": "256 MiB flush before each launch"}))
    ctx.close()


def prefill_bench(args):
    """B=8 sequences of 512 positions, the first 256 bidirectional text positions, the last
    256 semantic positions causal with full access to the text; 16 heads x 32, Q/K/V ~ N(0,1). Times the
    prefix-masked prefill attention (one layer) and the four Q8_0 GEMMs at M = 8*512 = 4096, and measures
    the int8 tensor peak in this run (torch._int_mm, cuBLASLt, 8192^3) as the GEMMs' denominator."""
    import torch
    import gsvcu
    ctx = gsvcu.Context(0)
    ext = torch.cuda.ExternalStream(ctx.stream_handle())
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    B, S, T = 8, 512, 256
    M = B * S
    qkv = torch.randn((M, 1536), device="cuda")
    out_q = torch.empty((M, 512), dtype=torch.int8, device="cuda")
    out_d = torch.empty((M, 16), dtype=torch.int16, device="cuda")
    starts = np.arange(B, dtype=np.int32) * S
    call = lambda: ctx.op_prefill_attention(qkv, starts, [S] * B, [T] * B, out_q, out_d)
    for _ in range(max(args.warmup, 10)):
        call()
    ms = _flush_and_time(ext, flush, call, max(args.steps, 5))
    pairs = T * T + T * T + T * (T + 1) // 2          # visible (query, key) pairs per sequence
    flops = 4 * 512 * pairs * B
    print(json.dumps({"workload": "cfg2 prefill attention (one layer)", "B": B, "S": S, "text": T,
                      "visible_pairs_per_seq": pairs, "mask_density": pairs / (S * S), "algorithmic_flops": flops,
                      "ms": ms, "TFLOPs": flops / (ms * 1e-3) / 1e12,
                      "bound": "FP64 tensor cores (k_prefill_attn_mma: mma.sync m8n8k4 .f64 for q.k and P.V, softmax in double)"}))
    # int8 tensor-core peak measured here (the GEMMs' denominator)
    a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    int8_tops = 2 * 8192 ** 3 / (best * 1e-3) / 1e12
    del a, b
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            bf16_peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        bf16_peak = 1590.0
    rng = np.random.default_rng(4)
    for (N, K) in [(1536, 512), (512, 512), (2048, 512), (512, 2048)]:
        raw = _rand_q8(rng, N, K)
        wq = torch.empty(N * K, dtype=torch.uint8, device="cuda")
        wd = torch.empty(N * K // 32, dtype=torch.int16, device="cuda")
        ctx.op_pack_q8_0(raw, N, K, wq, wd)
        xraw = _rand_q8(rng, M, K)
        xq = torch.from_numpy(np.ascontiguousarray(xraw[..., 2:]).reshape(M, K).view(np.int8)).cuda()
        xd = torch.from_numpy(np.ascontiguousarray(xraw[..., :2]).reshape(M, K // 32, 2).view(np.int16)
                              .reshape(M, K // 32)).cuda()
        y = torch.empty((M, N), device="cuda")
        bias = torch.randn(N, device="cuda")
        w16 = torch.empty(N * K, dtype=torch.float16, device="cuda")
        ctx.op_pack_q8_0_f16(raw, N, K, w16)
        variants = [("k_gemm_q8_tile (mma.m16n8k32 s8 per Q8_0 block + pinned float chain)",
                     lambda: ctx.op_q8_gemm(xq, xd, M, wq, wd, N, K, bias, None, gsvcu.EPI_BIAS, y=y)),
                    ("k_tc_prep + k_gemm_q8_tc (persistent; tcgen05.mma kind::f16 into TMEM, TMA tiles, per-block float "
                     "chain in the epilogue warps)",
                     lambda: ctx.op_q8_gemm_tc(xq, xd, M, w16, wd, N, K, bias, None, gsvcu.EPI_BIAS, y=y))]
        for name, call in variants:
            for _ in range(max(args.warmup, 10)):
                call()
            ms = _flush_and_time(ext, flush, call, max(args.steps, 5))
            tops = 2 * M * N * K / (ms * 1e-3) / 1e12
            print(json.dumps({"workload": "cfg2 prefill Q8_0 GEMM", "M": M, "shape": f"{K}x{N}", "ms": ms,
                              "TOPs": tops, "peak_int8_TOPs_measured_here": int8_tops, "frac_int8": tops / int8_tops,
                              "peak_bf16_TFLOPs_measured": bf16_peak, "frac_bf16": tops / bf16_peak,
                              "kernel": name}))
    ctx.close()


def single_bench(args):
    """one sequence, 120 phones with BERT features + 40 prompt codes, greedy decode
    (top_k 1), early stop off, up to 500 steps; reports per-token decode latency (the reference's published
    CPU figure is 12.55 ms/token on 4 threads)."""
    import torch
    import gsv_synth as S
    import gsvcu
    model = S.cached_model(MODEL_CACHE, seed=0, n_layer=24)
    ctx = gsvcu.Context(0)
    ctx.load(model)
    ctx.kv_reserve(1, 700, gsvcu.KV_F16 if args.kv == "f16" else gsvcu.KV_F32)
    rng = np.random.default_rng(120)
    req = S.make_request(rng, 120, 40)
    ext = torch.cuda.ExternalStream(ctx.stream_handle())
    for _ in range(max(args.warmup, 3)):
        ctx.generate([req], top_k=1, seed_base=1, max_steps=500)
    res = []
    for _ in range(max(args.steps, 3)):
        ctx.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        toks, lens = ctx.generate([req], top_k=1, seed_base=1, max_steps=500)
        e1.record(ext)
        torch.cuda.synchronize()
        res.append((e0.elapsed_time(e1), int(lens[0])))
    ms, n = min(res)
    print(json.dumps({"workload": "cfg0 single sequence, greedy", "prefix": "120 phones + 40 prompt",
                      "tokens": n, "ms_total": ms, "ms_per_token": ms / max(n, 1),
                      "note": "wall time on the library stream incl. prefill and the 16-step status reads",
                      "reference_cpu_ms_per_token": 12.55}))
    ctx.close()


def dit_bench(args):
    """The DiT / CFM estimator (gsv.cpp's gsv_dit, the stage after the AR path) at a production chunk: T =
    1140 frames (500 reference frames + 640 generated, src/gsv_dit.cpp synthesize's chunk), 22 blocks of
    1024 / 16 x 64 / FFN 2048, F16 matrices (the exporter's --spec lin=f16), seeded synthetic weights,
    guided sampling (cfg 2: both branches, 2T rows, per step). Device time per guided step by CUDA events
    on the DiT stream over `sample` calls of --dit-steps steps (inputs and outputs in host memory, so the
    events also cover one H2D of x0 and one D2H of the mel per call), tensor FLOP/s against the measured
    bf16 peak; beside it the CPU restatement (oracle) timed on one DiT block of one branch."""
    import torch
    import gsv_synth as S
    import gsvcu
    import dit_oracle as DO
    path = S.cached_dit_model(MODEL_CACHE, seed=0, depth=22)
    d = gsvcu.Dit(path)
    T, P, steps, cfg = 1140, 500, args.dit_steps, 2.0
    rng = np.random.default_rng(0)
    x0 = rng.standard_normal((100, T)).astype(np.float32)
    cond = rng.standard_normal((T, 1024)).astype(np.float32)
    neg = rng.standard_normal((T, 1024)).astype(np.float32)
    d.set_condition(cond, neg)
    stream = torch.cuda.ExternalStream(d.stream_handle())
    for _ in range(max(args.warmup, 3)):
        d.sample(x0, P, steps, cfg)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dev_ms, wall_ms = [], []
    for _ in range(max(args.steps, 3)):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ev0.record(stream)
        d.sample(x0, P, steps, cfg)
        ev1.record(stream)
        ev1.synchronize()
        wall_ms.append(1e3 * (time.perf_counter() - t0))
        dev_ms.append(ev0.elapsed_time(ev1))
    ms = float(np.median(dev_ms)) / steps
    R = 2 * T
    flop_gemm = 2 * R * (4 * 1024 * 1024 + 2 * 1024 * 2048) * 22 + 2 * 2 * R * 1024 * 64 * 31 + 2 * R * 1024 * (128 + 128)
    flop_attn = 4 * R * T * 1024 * 22
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        peak = 1590.0   # the pool's earlier measurement, when the file is absent
    tflops = (flop_gemm + flop_attn) / (ms * 1e-3) / 1e12
    cpu = None
    if not args.no_cpu_baseline:   # CPU restatement: one block of one branch (a step runs 44, trunk and head)
        W = DO.load(path)
        W1 = {k: v for k, v in W.items()
              if not k.startswith("dit.transformer_blocks.") or k.startswith("dit.transformer_blocks.0.")}
        W1["depth"] = 1
        t0 = time.perf_counter()
        DO.branch(W1, x0, 0.5, cond, T, n_blocks=1, head=False)
        t1 = time.perf_counter()
        DO.branch(W1, x0, 0.5, cond, T, n_blocks=0, head=False)
        t2 = time.perf_counter()
        blk = (t1 - t0) - (t2 - t1)
        cpu = {"ms_per_guided_step": 1e3 * (44 * max(blk, 1e-3) + 2 * (t2 - t1)), "cores": os.cpu_count() or 1,
               "kind": "port", "sample": "oracle (numpy) DiT block 0 of one branch timed, x 44 blocks + 2 x trunk "
               "per guided step"}
    print(json.dumps({"workload": "DiT / CFM guided sampling (gsv_dit::sample)", "model": "22 blocks, 1024 / 16 x 64 / "
                      "FFN 2048, F16 matrices", "T": T, "prompt_frames": P, "steps_per_call": steps, "cfg": cfg,
                      "ms_per_guided_step": ms, "frames_per_s": (T - P) / (ms * steps * 1e-3),
                      "wall_ms_per_call": float(np.median(wall_ms)),
                      "gflop_per_step": {"gemm": flop_gemm / 1e9, "attention": flop_attn / 1e9},
                      "tflops": tflops, "peak_bf16_tflops": peak, "frac_of_peak": tflops / peak if peak else None,
                      "cpu_baseline": cpu}))
    d.close()


def bert_bench(args):
    """The BERT feature producer (gsv.cpp's gsv_bert, the AR path's `bert` input) at the published
    chinese-roberta-wwm-ext-large shape (hidden 1024, 16 heads, FFN 4096, 24 layers of which 22 run, F16
    matrices as the exporter's --spec writes them, seeded synthetic weights): encode_feat_batch of 16
    sentences of 20-60 tokens, features to host memory; tokens/s over all sentence tokens. Beside it the
    CPU restatement (oracle) on the box's host cores for the first 4 sentences."""
    import torch
    import gsv_synth as S
    import gsvcu
    import oracle as O
    path = os.path.join(MODEL_CACHE, "bert_large_f16_seed21.gguf")
    if not os.path.exists(path):
        os.makedirs(MODEL_CACHE, exist_ok=True)
        S.write_bert_model(path + ".tmp", seed=21, dims=S.BertDims(), mat_type="f16")
        os.replace(path + ".tmp", path)
    g = gsvcu.Bert(path)
    rng = np.random.default_rng(22)
    B, tmax = 16, 64
    lens = rng.integers(20, 61, B).astype(np.int32)
    ids = rng.integers(672, 8000, (B, tmax)).astype(np.int32)
    ids[:, 0] = 101
    for b in range(B):
        ids[b, lens[b] - 1] = 102
    for _ in range(max(args.warmup, 3)):
        g.encode_feat_batch(ids.ravel(), lens, tmax)
    times = []
    for _ in range(max(args.steps, 5)):
        t0 = time.perf_counter()
        g.encode_feat_batch(ids.ravel(), lens, tmax)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * float(np.median(times))
    ntok = int(lens.sum())
    cores = os.cpu_count() or 1
    O.set_threads(cores)
    orc = O.BertOracle(path)
    t0 = time.perf_counter()
    for b in range(4):
        orc.encode_feat(ids[b, :lens[b]])
    cpu_s = time.perf_counter() - t0
    cpu_tok = int(lens[:4].sum())
    print(json.dumps({"workload": "BERT features (gsv_bert::encode_feat_batch)", "model": "1024 / 16 heads / 4096, "
                      "22 layers used, F16 matrices", "sentences": B, "tokens": ntok, "ms": ms,
                      "tokens_per_s": ntok / (ms * 1e-3), "timing": "host wall clock around the call (inputs and "
                      "features in host memory)",
                      "cpu_baseline": {"tokens_per_s": cpu_tok / cpu_s, "cores": cores, "kind": "port",
                                       "sample": f"oracle encode_feat of 4 sentences ({cpu_tok} tokens)"}}))
    g.close()


class RequestStream:
    """Seeded queue of BASELINE config-4 requests for one (rank, job)."""

    def __init__(self, rank, job, device=None):
        import gsv_synth as S
        self.S = S
        self.rng = np.random.default_rng([20261201, rank, job])
        self.device = device
        self.n = 0
        self.rank, self.job = rank, job

    def next(self):
        P = int(self.rng.integers(80, 401))
        T = int(round(0.7 * P))
        r = self.S.make_request(self.rng, T, P - T)
        seed = (self.rank << 40) | (self.job << 20) | self.n
        self.n += 1
        return r, seed


def stage(stream, count, device):
    """Pre-generate `count` requests; with device, their BERT features are moved into HBM."""
    import torch
    out = []
    for _ in range(count):
        r, seed = stream.next()
        if device is not None:
            r = type(r)(phones=r.phones, bert=torch.from_numpy(np.ascontiguousarray(r.bert)).to(device), prompt=r.prompt)
        out.append((r, seed))
    return out


def reduce_over_ranks(ms, tokens, seqs, world, device):
    """Whole-job numbers over the ranks: the slowest rank's time (max) and the tokens and sequences of
    all ranks (sum); the identity on one rank. Every rank takes the same two collectives."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms, float(tokens), float(seqs)], dtype=torch.float64, device=device)
    if world > 1:
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        t[0] = mx[0]
    return float(t[0]), float(t[1]), float(t[2])


def job_chunks(srv, queue, args, counters):
    """One serving job as a generator: admits the first `slots` requests, then runs chunks of
    `refill_every` decode iterations, refilling finished slots from the queue after each chunk, for
    `iters` iterations; yields after each chunk. `srv` is the library context (gsvcu.Context) or the
    CPU arm's OracleServing, which expose the same serve_* calls."""
    srv.serve_reset()
    t0 = srv.serve_tokens_total()
    at = 0

    def admit(k):
        nonlocal at
        if at + k > len(queue):
            raise RuntimeError("request queue exhausted; enlarge the staged queue")
        items = queue[at:at + k]
        at += k
        reqs = [r for r, _ in items]
        srv.serve_admit(reqs, [s for _, s in items], list(range(at - k, at)), max_steps=args.iters)
        for r in reqs:
            T, P = len(r.phones), len(r.prompt)
            counters["h2d"] += 4 * T + 4 * P + (0 if hasattr(r.bert, "data_ptr") else 4 * 1024 * T)
        counters["seqs"] += k

    admit(args.slots)
    lookahead = args.lookahead
    srv.set_serve_lookahead(lookahead)
    it = 0
    if lookahead:   # the first call only starts a chunk; each later call reports the previous one
        it = min(args.refill_every, args.iters)
        srv.serve_step(it, max_done=args.slots, tok_cap=args.slots * args.iters)
    while True:
        n = min(args.refill_every, args.iters - it)
        if not lookahead and n == 0:
            break
        done = srv.serve_step(n, max_done=args.slots, tok_cap=args.slots * args.iters)
        counters["d2h"] += 64 * srv.serve_active() + sum(4 * len(d["tokens"]) for d in done)
        if lookahead and n == 0:
            break
        it += n
        if done and it < args.iters:
            admit(len(done))
        yield it
    counters["tokens"] = srv.serve_tokens_total() - t0
    srv.serve_reset()
    srv.set_serve_lookahead(False)


def run_job(ctx, queue, args, counters):
    """One serving job: returns generated tokens."""
    for _ in job_chunks(ctx, queue, args, counters):
        pass
    return counters["tokens"]


class OracleServing:
    """The serve_* calls of gsvcu.Context on the CPU oracle's serving loop (oracle.OracleServer), so the
    CPU arm runs the job loop of job_chunks unchanged."""

    def __init__(self, orc, slots, max_ctx, kv_f16=False):
        import oracle as O
        self.srv = O.OracleServer(orc, slots, max_ctx, kv_f16=kv_f16)

    def serve_reset(self):
        self.srv.reset()

    def serve_tokens_total(self):
        return self.srv.tokens_total()

    def serve_admit(self, reqs, seeds, tags, max_steps):
        self.srv.admit(reqs, seeds, tags, max_steps=max_steps)

    def serve_step(self, n, max_done, tok_cap):
        return self.srv.step(n, max_done=max_done, tok_cap=tok_cap)

    def serve_active(self):
        return self.srv.active()

    def set_serve_lookahead(self, on):
        pass


def sample_clocks(local_rank):
    try:
        return subprocess.Popen(
            ["nvidia-smi", "-i", str(local_rank),
             "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
             "--format=csv,noheader,nounits", "-lms", "200"],
            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except Exception:
        return None


def clock_summary(proc):
    if proc is None:
        return None
    proc.terminate()
    try:
        out = proc.communicate(timeout=5)[0]
    except Exception:
        return None
    rows = [[c.strip() for c in l.split(",")] for l in out.strip().splitlines() if l.count(",") >= 8]
    if not rows:
        return None
    sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
    mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
    return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_per_key():
    """DRAM bytes per attended key of one decode-attention launch, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "decode_attention_cfg3_b64.md")
    try:
        for line in open(p):
            if line.startswith("dram_bytes_per_key:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


def _oracle_setup(args):
    import gsv_synth as S
    import oracle as O
    fmt_kw = FORMATS[args.format][0]
    model = S.cached_model(MODEL_CACHE, seed=0, n_layer=24, **fmt_kw)
    cores = os.cpu_count() or 1
    O.set_threads(cores)
    orc = O.OracleModel(model)
    return orc, cores


def cpu_baseline(args):
    """The oracle (CPU restatement of the reference's ggml CPU path, F32 KV as the reference caches) on a
    bounded sample of the same workload: the first --cpu-sample-chunks chunks of job 2000 of rank 0 (the
    GPU arm's first timed job), initial 64-sequence admission and the refills included, timed on the host
    clock. Early iterations have the shortest contexts, so this sample is optimistic for the CPU; the
    reference arm (--impl reference) times the whole job."""
    orc, cores = _oracle_setup(args)
    srv = OracleServing(orc, args.slots, 400 + args.iters + 8)
    queue = stage(RequestStream(0, 2000), args.slots * 5, None)
    counters = {"h2d": 0, "d2h": 0, "seqs": 0}
    n_chunks = max(1, args.cpu_sample_chunks)
    t0 = time.perf_counter()
    gen = job_chunks(srv, queue, args, counters)
    it = 0
    for _ in range(n_chunks):
        it = next(gen)
    sec = time.perf_counter() - t0
    tokens = srv.serve_tokens_total()
    srv.serve_reset()
    return {"value": tokens / sec, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"config-4 job 2000 of rank 0 (64 slots) on the oracle, {cores} threads, F32 KV: admission of "
                      f"{counters['seqs']} sequences and iterations 0-{it} ({tokens} tokens) in {sec:.1f} s; "
                      f"contexts of these early iterations are short (<= {400 + it} keys)"}


def reference_arm(args, n_gpus):
    """--impl reference: the reference's CPU path (the oracle port of the ggml CPU backend; ggml itself is
    not buildable offline) runs one whole config-4 job -- rank 0's job 2000, the GPU arm's first timed job:
    64 slots, 1500 iterations, refills every 16, F32 KV as the reference caches -- on all host threads. The
    job's chunks are split into the K timed steps (step k = its share of the chunks, host clock), so the
    timed region is exactly one job and value = its tokens / its time."""
    orc, cores = _oracle_setup(args)
    srv = OracleServing(orc, args.slots, 400 + args.iters + 8)
    counters = {"h2d": 0, "d2h": 0, "seqs": 0}
    # warm-up (untimed): W decode iterations of a 4-slot batch from another stream
    wq = stage(RequestStream(0, 999), 8, None)
    wa = argparse.Namespace(**{**vars(args), "slots": 4, "iters": max(args.warmup, 1), "refill_every": 1})
    for _ in job_chunks(srv, wq, wa, dict(counters)):
        pass
    queue = stage(RequestStream(0, 2000), args.slots * 5, None)
    n_chunks = -(-args.iters // args.refill_every)
    K = max(1, min(args.steps, n_chunks))
    bounds = [round(k * n_chunks / K) for k in range(K + 1)]
    gen = job_chunks(srv, queue, args, counters)
    step_s = []
    done = 0
    t_start = time.perf_counter()
    for k in range(K):
        t0 = time.perf_counter()
        for _ in range(bounds[k + 1] - bounds[k]):
            next(gen)
            done += 1
        step_s.append(time.perf_counter() - t0)
    tokens = srv.serve_tokens_total()
    for _ in gen:   # nothing left: closes the job (counts, reset)
        pass
    total = time.perf_counter() - t_start
    value = tokens / sum(step_s)
    return {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": n_gpus, "steps": K,
        "warmup": args.warmup, "ms_per_step": 1e3 * sum(step_s) / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q8_0 int8 dot / f32 softmax / f32 KV", "data": DATA,
        "config": serve_config(args, n_gpus),
        "kv_cache": "f32 per sequence (the reference's cache type, src/gsv_ar.cpp:107-108)",
        "job": {"tokens": tokens, "sequences": counters["seqs"], "iterations": args.iters, "chunks": done,
                "seconds": total},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"one whole config-4 job (rank 0, job 2000: {counters['seqs']} sequences, "
                                   f"{args.iters} iterations, {tokens} tokens) on the oracle port of the ggml CPU "
                                   f"path, {cores} threads, F32 KV; the K steps are consecutive shares of its "
                                   f"{n_chunks} chunks"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


DATA = "synthetic (seeded GGUF weights N(0,0.02), requests U[80,400])"


def serve_config(args, n_gpus):
    """The config key both arms print for the serve workload."""
    return {"workload": "cfg4: box-wide serving shard per GPU (BASELINE configs[4])",
            "model": f"gsv AR 24 x 512, 16 heads x 32, FFN 2048, vocab 1025, {FORMATS[args.format][2]}",
            "slots_per_gpu": args.slots, "iters_per_job": args.iters, "refill_every": args.refill_every,
            "sampler": "top_k 15, top_p 1.0, temperature 1.0, rep 1.35, EOS 1024",
            "parallelism": f"dp{n_gpus} (replicas, batch-sharded)",
            "l2": "no flush; KV working set per step (>1 GB) exceeds the 126 MB L2"}


# serve-workload model formats: cached_model arguments and the weight bytes one decode step reads
# (24 layers x 3,145,728 matrix weights + 26,624 B of F32 biases / LN per layer + the 1025 x 512 predict)
FORMATS = {
    "q8_0": (dict(mat_type="q8_0"), 82954240, "Q8_0 attn/FFN, F32 predict"),
    "f16": (dict(mat_type="f16", predict_type="f16", emb_type="f16"), 152683520, "F16 attn/FFN/predict/embeddings"),
    "f32": (dict(mat_type="f32"), 304728064, "F32 attn/FFN/predict"),
    # the exporter's own example: --spec attn=q8_0,ffn=q6_k,predict=f16,emb=f16 (file bytes of the matrices)
    "q6_k": (dict(mat_type="q8_0", ffn_type="q6_k", predict_type="f16", emb_type="f16"), 69714944,
             "Q8_0 attn, Q6_K FFN, F16 predict/embeddings"),
    # --spec attn=q4_1,ffn=q4_1 (the k_gemm_qm path), F32 predict
    "q4_1": (dict(mat_type="q4_1"), 49924096, "Q4_1 attn/FFN, F32 predict"),
}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n_gpus = max(args.gpus, world)

    if args.workload != "serve":
        if rank == 0:
            {"attn": attn_sweep, "gemv": gemv_sweep, "prefill": prefill_bench, "single": single_bench,
             "bert": bert_bench, "dit": dit_bench}[args.workload](args)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(reference_arm(args, n_gpus)))
        return

    import torch
    import torch.distributed as dist
    import gsv_synth as S
    import gsvcu

    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    fmt_kw, weight_bytes, fmt_desc = FORMATS[args.format]
    if rank == 0:
        model = S.cached_model(MODEL_CACHE, seed=0, n_layer=24, **fmt_kw)
    if world > 1:
        dist.barrier()
    model = S.cached_model(MODEL_CACHE, seed=0, n_layer=24, **fmt_kw)

    ctx = gsvcu.Context(local_rank)
    ctx.load(model)
    if args.prefill_gemm != "auto":
        ctx.set_prefill_gemm(1 if args.prefill_gemm == "tc" else 0)
    max_ctx = 400 + args.iters + 8
    ctx.kv_reserve(args.slots, max_ctx, gsvcu.KV_F16 if args.kv == "f16" else gsvcu.KV_F32)
    ext = torch.cuda.ExternalStream(ctx.stream_handle())
    queue_len = args.slots * 5
    counters = {"h2d": 0, "d2h": 0, "seqs": 0}

    for w in range(args.warmup):
        run_job(ctx, stage(RequestStream(rank, 1000 + w), queue_len, None), args, counters)

    def timed(device_inputs, job0):
        queues = [stage(RequestStream(rank, job0 + k), queue_len, local_rank if device_inputs else None)
                  for k in range(args.steps)]
        counters.update(h2d=0, d2h=0, seqs=0)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        l0 = ctx.kernel_launches()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(ext)
        tokens = 0
        for q in queues:
            tokens += run_job(ctx, q, args, counters)
        ev1.record(ext)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        if world > 1:
            dist.barrier()
        launches = ctx.kernel_launches() - l0
        return (*reduce_over_ranks(ms, tokens, counters["seqs"], world, "cuda"), launches, dict(counters))

    clk = sample_clocks(local_rank)
    ms_v, tok_v, seqs_v, launches_v, _ = timed(True, 2000)
    clocks = clock_summary(clk)
    ms_e, tok_e, seqs_e, _, cnt_e = timed(False, 2000)

    # roofline of the dominant kernel (decode attention) on a mid-job state of the same workload
    prof_q = stage(RequestStream(rank, 3000), queue_len, None)
    ctx.serve_reset()
    ctx.serve_admit([r for r, _ in prof_q[:args.slots]], [s for _, s in prof_q[:args.slots]],
                    list(range(args.slots)), max_steps=args.iters)
    ctx.serve_step(args.iters // 2)
    # whole decode step (graph replay) at this state: weights + every decoding slot's K/V
    ctx.sync()
    se0, se1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    se0.record(ext)
    ctx.serve_step(16)
    se1.record(ext)
    torch.cuda.synchronize()
    step_ms = se0.elapsed_time(se1) / 16
    prof_steps = 8
    ms_cls, attn_bytes = ctx.step_profile(prof_steps)
    ctx.serve_reset()
    n_launch = prof_steps * ctx.hp.n_layer
    attn_ms = ms_cls["decode_attn"] / n_launch
    bytes_launch = attn_bytes / n_launch
    peak, peak_kind = measured_peaks()
    achieved = bytes_launch / (attn_ms * 1e-3) / 1e9
    tpk = traffic_per_key()
    keys_launch = bytes_launch / (2 * 512 * (2 if args.kv == "f16" else 4))

    # the reference-exact configuration: the same jobs with an F32 KV cache (the reference caches F32,
    # src/gsv_ar.cpp:107-108; with it every token equals the oracle's). Every rank takes these steps.
    kv32 = None
    if args.kv == "f16" and args.kv_f32_steps > 0:
        ctx.kv_reserve(args.slots, max_ctx, gsvcu.KV_F32)
        run_job(ctx, stage(RequestStream(rank, 1000), queue_len, None), args, counters)   # warm-up
        steps_saved = args.steps
        args.steps = args.kv_f32_steps
        ms_32, tok_32, seqs_32, _, _ = timed(True, 2000)
        args.steps = steps_saved
        kv32 = {"value": tok_32 / (ms_32 * 1e-3), "unit": "tokens/s", "steps": args.kv_f32_steps,
                "ms_per_step": ms_32 / args.kv_f32_steps, "kv_cache": "paged f32, 64-token pages",
                "jobs": "the first jobs of the timed set above, device-resident inputs",
                "parity": "tokens identical to the oracle with the reference's F32 cache (the F16 cache rounds "
                          "K/V and diverges from it after a few to ~100 greedy steps)"}

    value = tok_v / (ms_v * 1e-3)
    e2e = tok_e / (ms_e * 1e-3)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": n_gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_v / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": ("q8_0 int8 MMA" if args.format == "q8_0" else
                  "q8_0 int8 MMA + q6_k dp2a" if args.format == "q6_k" else
                  "q4_1 dp4a" if args.format == "q4_1" else f"{args.format} weights / f32 FMA") +
                 f" / f32 softmax / {args.kv} KV",
        "data": DATA,
        "config": serve_config(args, n_gpus),
        "kv_cache": f"paged {args.kv}, 64-token pages",
        "serve_lookahead": args.lookahead,
        "job": {"tokens_per_step": tok_v / args.steps, "sequences_per_step": seqs_v / args.steps},
        "gpu_launches": launches_v,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": cnt_e["h2d"] // args.steps,
                "d2h_bytes_per_step": cnt_e["d2h"] // args.steps},
        "roofline": {"kernel": "k_decode_attn<__half>", "bound": "hbm", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": (tpk * keys_launch) if tpk else None, "algorithmic_bytes_per_launch": bytes_launch,
                     "avg_launch_ms": attn_ms},
        "decode_step_roofline": {"bytes_per_step": weight_bytes + attn_bytes / prof_steps, "ms_per_step": step_ms,
                                 "achieved": (weight_bytes + attn_bytes / prof_steps) / (step_ms * 1e-3) / 1e9,
                                 "peak": peak, "unit": "GB/s",
                                 "frac": (weight_bytes + attn_bytes / prof_steps) / (step_ms * 1e-3) / 1e9 / peak,
                                 "state": f"mid-job (iteration ~iters/2), 16 graph-replayed steps; bytes = weights "
                                          f"({weight_bytes / 1e6:.2f} MB) + K/V and q/out of every decoding slot"},
        "step_profile_ms": {k: round(v / prof_steps, 4) for k, v in ms_cls.items()},
        "clocks": clocks,
    }
    if kv32:
        line["kv_f32"] = kv32
    if n_gpus == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

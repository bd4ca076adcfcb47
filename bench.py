#!/usr/bin/env python
"""Batch-1 decode benchmark of the Qwen3-0.6B engine (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference] [--mode replicas|shard]

Workload: Qwen3-0.6B architecture, bf16 weights from the seed-0 synthetic
checkpoint, a 1024-token seeded prompt, then greedy decode at context 1024-1279
(positions are rewound to 1024 after every 256 tokens, so every step decodes at
1K context).  A step is one decoded token: the whole forward (28 layers, LM
head) plus the device sampler, one kernel launch.  Weights (1.19 GB) stream
from HBM every step, far larger than the 126 MB L2.

--impl mine       the engine.  value = device time of K chained steps from CUDA
                  events (max over ranks; N ranks = N independent replicas);
                  e2e = qwen_decode_step per token through the C ABI with the
                  token in and out of pinned host memory.
--mode shard      the vocabulary-sharded LM head over the N ranks: per-token
                  decode latency (ms/token, max over ranks) of the device loop
                  (trunk + shard rows, NCCL all-gather of the shards' top-k,
                  device merge and sampling), greedy and sampled.
--impl reference  the reference's path on the host cores: the oracle's
                  restatement of forward() in the reference's own bf16 rounding
                  (qwen_model.cuh:772-851; the reference has no CPU forward) and
                  the reference's own sampler.h compiled from its sources, all
                  host threads, same workload.  Rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "oracle"))

METRIC = "batch-1 decode tok/s (Qwen3-0.6B bf16) and % of B200 HBM roofline; prefill tok/s"
PROMPT_LEN = 1024
WINDOW = 256
WEIGHT_BYTES = 1_192_101_888      # weights read per token (28 layers + LM head + final norm + embedding row)
KV_BYTES_PER_POS = 114_688        # 28 layers x (K + V) x 1024 bf16 per cached position
CONFIG = {
    "workload": "Qwen3-0.6B batch-1 greedy decode at 1K context: 1024-token seeded prompt, decode positions 1024-1279 "
                "(rewound every 256 tokens), random-init bf16 weights (seed 0)",
    "model": "Qwen3-0.6B architecture (28 layers, hidden 1024, 16/8 heads, vocab 151936)",
    "batch": 1,
    "prompt_tokens": PROMPT_LEN,
    "decode_positions": [PROMPT_LEN, PROMPT_LEN + WINDOW - 1],
    "l2": "inputs larger than L2: 1.19 GB of weights stream from HBM every step (L2 126 MB)",
}


def load_qb():
    import importlib.util
    spec = importlib.util.spec_from_file_location("qwen_b200", os.path.join(REPO, "qwen600-rocm-inference_b200", "qwen_b200.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def measured_peak():
    try:
        d = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def measured_bf16_peak():
    """Dense bf16 TFLOP/s of a cuBLAS GEMM timed as a burst on this pool's B200s
    (the kernels below are timed alone), else the 1,590 fallback."""
    try:
        return float(json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))["bf16_tflops"])
    except Exception:
        return 1590.0


def profiled_traffic():
    """dram read+write bytes per decode launch from the committed ncu summary."""
    p = os.path.join(REPO, "profiles", "decode_kernel_ncu.md")
    try:
        for line in open(p):
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":")[1].split()[0])
    except OSError:
        pass
    return None


class Clocks:
    """nvidia-smi samples (100 ms) of one GPU while the timed region runs."""
    FIELDS = "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device):
        self.device = device
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.p is None:
            return
        time.sleep(0.15)
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) == 7:
                self.rows.append(f)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i].lower() == "active"})
        pw = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows), "power_w_max": max(pw) if pw else None}


def cpu_oracle_rate(ck, mode, budget_s, max_tokens, threads):
    """Tokens/s of the oracle decoding at context 1024 on the host cores."""
    import oracle_py as O
    O.set_threads(threads)
    o = O.Oracle(ck, mode, PROMPT_LEN + WINDOW + 1)
    o.fill_kv(PROMPT_LEN)
    ref_samp = O.ref_sampler()
    rng = np.random.default_rng(11)
    tok = int(rng.integers(0, 151936))
    o.forward(tok, PROMPT_LEN)          # warm-up
    n, t0 = 0, time.perf_counter()
    while n < max_tokens and (n == 0 or time.perf_counter() - t0 < budget_s):
        lg = o.forward(tok, PROMPT_LEN + 1 + (n % (WINDOW - 1)))
        if ref_samp is not None:        # the reference's own sampler.h, argmax path
            import ctypes
            r = ctypes.c_ulonglong(1)
            tok = ref_samp.ref_sample(lg.ctypes.data, 0.0, 0.95, 20, ctypes.byref(r))
        else:
            tok = O.sample(lg, 0.0, 0.95, 20, 1)[0]
        n += 1
    dt = time.perf_counter() - t0
    o.close()
    return n / dt, n, dt


def ref_cuda_rate(ck, n_prompt=768, n_timed=200):
    """The reference's own CUDA forward (cuBLAS, compiled for sm_100a) on this
    GPU: forward + its host argmax sampler per token, positions below 1024 only
    (its attention is valid there).  Informational."""
    import ctypes
    import oracle_py as O
    L, S = O.ref_model(), O.ref_sampler()
    if L is None or S is None:
        return None
    if L.ref_build(ck.encode()) != 0:
        return None
    lg = np.zeros(151936, dtype=np.float32)
    toks = np.random.default_rng(5).integers(0, 151936, n_prompt).tolist()
    for pos, t in enumerate(toks):
        L.ref_forward(t, pos, lg.ctypes.data)
    r = ctypes.c_ulonglong(1)
    tok = S.ref_sample(lg.ctypes.data, 0.0, 0.95, 20, ctypes.byref(r))
    t0 = time.perf_counter()
    for i in range(n_timed):
        L.ref_forward(tok, n_prompt + i, lg.ctypes.data)
        tok = S.ref_sample(lg.ctypes.data, 0.0, 0.95, 20, ctypes.byref(r))
    dt = time.perf_counter() - t0
    L.ref_free()
    return {"value": n_timed / dt, "unit": "tok/s", "positions": [n_prompt, n_prompt + n_timed - 1],
            "note": "reference qwen_model.cuh + sampler.h built for sm_100a with cuBLAS, on this GPU; context below 1024 "
                    "because its attention is wrong beyond 1024 positions"}


GEMV_SHAPES = [(1024, 4096), (2048, 1024), (1024, 6144), (3072, 1024), (1024, 151936)]   # (K, N)


def gemv_sweep(qb, peak, reps=64):
    """Isolated bf16 GEMV y = bf16(W x) through qwen_gemv_bf16 at the decode
    chain's shapes: x ~ N(0,1), W ~ N(0,0.02) from a seed, fp32 accumulate, bf16
    out.  `reps` calls back to back, each on the next of enough copies of W that
    together exceed twice the 126 MB L2 (every launch reads its W from HBM),
    captured once as a CUDA graph and replayed between two CUDA events on the
    replaying stream: `us` = device time per GEMV, median of 5 replays.  The
    same calls issued one by one from Python (`us_host_issued`) are bound by the
    host's per-call cost (~6 us) below ~13 MB, so the graph is what isolates the
    kernel."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(0)
    out = []
    for k, n in GEMV_SHAPES:
        nbytes_w = n * k * 2
        copies = max(1, -(-(256 << 20) // nbytes_w))
        W = [(torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn(k, generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty(n, dtype=torch.bfloat16, device="cuda")
        ptrs = [w.data_ptr() for w in W]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        call = lambda i, st: qb.gemv_bf16(ptrs[i % copies], x.data_ptr(), y.data_ptr(), n, k, st.cuda_stream)
        with torch.cuda.stream(side):
            for i in range(copies + 3):   # first call sets up the device; the rest warm up
                call(i, side)
            ts_host = []
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(side)
                for i in range(reps):
                    call(i, side)
                e1.record(side)
                e1.synchronize()
                ts_host.append(e0.elapsed_time(e1) * 1e3 / reps)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream()
            for i in range(reps):
                call(i, cs)
        rs = torch.cuda.Stream()
        rs.wait_stream(torch.cuda.current_stream())
        ts = []
        with torch.cuda.stream(rs):
            graph.replay()   # warm-up replay
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(rs)
                graph.replay()
                e1.record(rs)
                e1.synchronize()
                ts.append(e0.elapsed_time(e1) * 1e3 / reps)
        torch.cuda.current_stream().wait_stream(rs)
        qb.gemv_status(rs.cuda_stream)
        us = float(np.median(ts))
        nbytes = n * k * 2 + k * 2 + n * 2
        out.append({"k": k, "n": n, "bytes": nbytes, "us": us, "gbs": nbytes / (us * 1e-6) / 1e9,
                    "frac": nbytes / (us * 1e-6) / 1e9 / peak, "copies_of_w": copies, "us_host_issued": float(np.median(ts_host))})
        del graph, W, x, y
    torch.cuda.empty_cache()
    return out


# (M, N, K): the prefill projections of a 2048-row pass as the engine runs them
# (K = 3 x the input width: activations split into three bf16 parts) — q|k|v,
# gate|up, O, down
GEMM_SHAPES = [(2048, 4096, 3072), (2048, 6144, 3072), (2048, 1024, 6144), (2048, 1024, 9216)]


def gemm_sweep(qb, peak_tflops):
    """Isolated tcgen05 GEMM C = A B^T (bf16 in, fp32 out) through qwen_gemm_bf16
    at the prefill shapes: A ~ N(0,1), B ~ N(0,0.05) from a seed.  Each timed
    launch is bracketed alone by CUDA events with a 256 MB write before it to
    flush L2; the reported time is the median of 10 after 3 warm-up launches.
    TFLOP/s counts the executed 2 M N K."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(1)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    out = []
    for m, n, k in GEMM_SHAPES:
        A = torch.randn(m, k, generator=g, device="cuda").to(torch.bfloat16)
        B = (torch.randn(n, k, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
        C = torch.empty(m, n, dtype=torch.float32, device="cuda")
        call = lambda: qb.gemm_bf16(A.data_ptr(), B.data_ptr(), C.data_ptr(), m, n, k, True, stream.cuda_stream)
        for _ in range(3):
            call()
        ts = []
        for _ in range(10):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call()
            e1.record(stream)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        us = float(np.median(ts))
        tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
        out.append({"m": m, "n": n, "k": k, "us": us, "tflops": tf, "frac": tf / peak_tflops})
        del A, B, C
    del flush
    torch.cuda.empty_cache()
    return out


def long_context(qb, ck, n_prompt=4096, n_gen=512):
    """4096 seeded prompt tokens, then 512 sampled tokens (temperature 0.6,
    top-k 20, top-p 0.95, seeded xorshift64*), KV cache sized 8192: decode
    tok/s from the device time of the 512 chained launches.  The prompt is
    prefilled twice (the second call writes the same cache): prefill_tok_s is
    the second, synchronous call's wall time; the first call, which also sets
    up the handle's prompt-pass buffers and tensor maps, is reported beside it."""
    eng = qb.Engine(ck, 0)
    try:
        prompt = np.random.default_rng(4096).integers(0, 151936, n_prompt).tolist()
        t0 = time.perf_counter()
        eng.prefill(prompt, 0)
        first_s = time.perf_counter() - t0
        t0 = time.perf_counter()
        eng.prefill(prompt, 0)
        pre_s = time.perf_counter() - t0
        sp = qb.Sampling(0.6, 0.95, 20)
        toks, rng, ms = eng.generate_timed(prompt[-1], n_prompt, n_gen, sp, 0x5EED)
    finally:
        eng.close()
    return {"value": n_gen / (ms / 1e3), "unit": "tok/s", "prompt_tokens": n_prompt, "sampled_tokens": n_gen,
            "sampling": {"temperature": 0.6, "top_k": 20, "top_p": 0.95}, "ms_per_token": ms / n_gen,
            "prefill_tok_s": n_prompt / pre_s, "prefill_first_call_tok_s": n_prompt / first_s}


def batched_decode(qb, ck, batches=(8, 32, 128), n_prompt=1024, n_steps=24, warmup=3, sampled=(32,)):
    """qwen_batch_step at 1K context: 128 slots prefilled with seeded 1024-token
    prompts, then for each B greedy steps over slots 0..B-1 (every slot at its
    own next position), and for each B in `sampled` steps sampled at
    temperature 0.6, top-p 0.95, top-k 20 (device top-k, host draw per row).
    Wall time of the synchronous calls (inputs from host memory, next tokens
    back to host memory every step) after `warmup` steps; aggregate tok/s =
    B x steps / time."""
    eng = qb.Engine(ck, 0)
    out = []
    try:
        top = max(tuple(batches) + tuple(sampled))
        eng.batch_init(top)
        pos = []
        for slot in range(top):
            prompt = np.random.default_rng(5000 + slot).integers(0, 151936, n_prompt).tolist()
            eng.batch_prefill(slot, prompt)
            pos.append(n_prompt)
        runs = [(b, "greedy") for b in batches] + [(b, "top_k 20") for b in sampled]
        for b, mode in runs:
            toks = [5] * b
            sp = qb.GREEDY if mode == "greedy" else qb.Sampling(0.6, 0.95, 20)
            rs = None if mode == "greedy" else list(range(1, b + 1))
            for i in range(warmup + n_steps):
                if i == warmup:
                    t0 = time.perf_counter()
                toks, rs = eng.batch_step(toks, pos[:b], sp, rs)
                for r in range(b):
                    pos[r] += 1
            dt = time.perf_counter() - t0
            out.append({"batch": b, "sampling": mode, "tok_s": b * n_steps / dt, "ms_per_step": dt / n_steps * 1e3,
                        "context": [min(pos[:b]) - n_steps, max(pos[:b])]})
    finally:
        eng.close()
    return {"unit": "tok/s (aggregate over the batch)", "prompt_tokens": n_prompt, "points": out,
            "path": "qwen_batch_step: projections and LM head as tcgen05 GEMMs over the batch rows, fp32 attention per row"}


PREFILL_LINEAR_FLOP = 2 * 440_401_920     # per prompt token: 2 x the 28 layers' projection weights (q, k, v, o, gate, up, down)


def prefill_bench(qb, ck, n_prompt=2048, n_gen=32):
    """2048 seeded prompt tokens through qwen_prefill (tensor-core passes over all
    positions, the last one's logits from an LM-head GEMV), then 32 greedy
    tokens; prefill time is the wall time of the synchronous call after one
    warm-up call.  Algorithmic FLOPs: the projections (2 x 440,401,920 per
    token) plus causal attention (28 x 16 x 2 x S^2 x 128 for QK^T and P.V
    over the lower triangle); the passes execute both twice (the fp32
    activations, Q and P enter the bf16 tensor-core products as two bf16
    parts)."""
    eng = qb.Engine(ck, 0)
    try:
        prompt = np.random.default_rng(2048).integers(0, 151936, n_prompt).tolist()
        eng.prefill(prompt, 0)                       # warm-up (buffers, tensor maps)
        t0 = time.perf_counter()
        eng.prefill(prompt, 0)
        dt = time.perf_counter() - t0
        toks, _, ms = eng.generate_timed(prompt[-1], n_prompt, n_gen)
    finally:
        eng.close()
    attn = 28 * 16 * 2 * 2 * (n_prompt * (n_prompt + 1) / 2) * 128
    alg = PREFILL_LINEAR_FLOP * n_prompt + attn
    return {"value": n_prompt / dt, "unit": "tok/s", "prompt_tokens": n_prompt, "ms": dt * 1e3,
            "algorithmic_tflop": alg / 1e12, "achieved_tflops": alg / dt / 1e12,
            "executed_tensor_tflop": 2 * alg / 1e12,
            "path": "28 layers x (4 persistent tcgen05 GEMM launches over all prompt rows, 256 x 256 tiles on SM pairs "
                    "(cta_group::2) + causal attention on tcgen05/TMEM, one pass, online softmax), two bf16 parts per "
                    "fp32 operand; last position's logits by fp32 RMSNorm + LM-head GEMV",
            "decode_after": {"tokens": n_gen, "tok_s": n_gen / (ms / 1e3)}}


def reference_checkpoint(seed=0):
    """The seed-0 synthetic checkpoint for the reference arm, at the path the
    engine uses, written by the oracle when absent (this arm never loads the
    engine library; the two writers produce the same bytes)."""
    import oracle_py as O
    d = os.environ.get("QWEN_B200_CACHE", os.path.join(REPO, ".cache"))
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"qwen3-0.6b-synthetic-seed{seed}.safetensors")
    if not os.path.exists(path):
        tmp = f"{path}.tmp.{os.getpid()}"
        try:
            O.write_synthetic_checkpoint(tmp, seed)
            os.replace(tmp, path)
        finally:
            if os.path.exists(tmp):
                os.remove(tmp)
    return path


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ck = reference_checkpoint(0)
    import oracle_py as O
    threads = os.cpu_count() or 1
    budget = min(240.0, max(20.0, 0.05 * args.steps))
    rate, n, dt = cpu_oracle_rate(ck, O.BF16, budget, args.steps, threads)
    sample = f"{n} decode tokens at context 1024-{1024 + min(n, WINDOW - 1)} ({dt:.1f} s), oracle bf16-faithful forward + reference sampler.h"
    line = {"metric": METRIC, "value": rate, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus, "steps": n,
            "warmup": 1, "ms_per_step": 1000.0 / rate, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": CONFIG,
            "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_mine(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    qb = load_qb()
    ck = qb.default_checkpoint(0)
    eng = qb.Engine(ck, local)
    prompt = np.random.default_rng(1000 + rank).integers(0, 151936, PROMPT_LEN).tolist()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            t = torch.zeros(1, device="cuda")
            dist.all_reduce(t)
            torch.cuda.synchronize()

    t0 = time.perf_counter()
    eng.prefill(prompt, 0)
    prefill_s = time.perf_counter() - t0
    tok = prompt[-1]
    # warm-up
    w = max(args.warmup, 3)
    toks, _, _ = eng.generate_timed(tok, PROMPT_LEN - 1, min(w, WINDOW))
    tok = toks[-1]
    # timed region: K chained steps in windows of 256 positions
    barrier()
    dev_ms, done, ctx_sum = 0.0, 0, 0.0
    with Clocks(local) as clk:
        wall0 = time.perf_counter()
        while done < args.steps:
            n = min(WINDOW, args.steps - done)
            toks, _, ms = eng.generate_timed(tok, PROMPT_LEN, n)
            dev_ms += ms
            ctx_sum += n * (PROMPT_LEN + 1 + (n - 1) / 2.0)
            tok = toks[-1]
            done += n
        barrier()
        wall = time.perf_counter() - wall0
    t = torch.tensor([dev_ms], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    # e2e: one qwen_decode_step per token, token in / token out through pinned host memory.
    # The handle's first decode_step captures and instantiates its step graph: that
    # one-time set-up call stays outside the timed region.
    n_e2e = min(args.steps, 512)
    tok, _ = eng.decode_step(tok, PROMPT_LEN)
    barrier()
    e0 = time.perf_counter()
    for i in range(n_e2e):
        tok, _ = eng.decode_step(tok, PROMPT_LEN + (i % WINDOW))
    barrier()
    e2e_s = time.perf_counter() - e0
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())

    if rank == 0:
        peak, peak_kind = measured_peak()
        ms_step = max_ms / args.steps
        ctx = ctx_sum / args.steps
        bytes_step = WEIGHT_BYTES + KV_BYTES_PER_POS * ctx
        achieved = bytes_step / (ms_step * 1e-3) / 1e9
        line = {"metric": METRIC, "value": world * args.steps / (max_ms / 1000.0), "unit": "tok/s", "n_gpus": world,
                "steps": args.steps, "warmup": w, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": dict(CONFIG, parallelism=f"{world} independent replicas" if world > 1 else "single GPU"),
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                             "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback 6.65 TB/s",
                             "traffic": profiled_traffic(), "algorithmic_bytes_per_step": bytes_step,
                             "kernel": "qb::decode_kernel (one launch per token)"},
                "e2e": {"value": world * n_e2e / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 32, "d2h_bytes_per_step": 32,
                        "steps": n_e2e, "call": "qwen_decode_step"},
                "gpu_launches": args.steps,
                "clocks": clk.summary(),
                "wall_s_timed_region": wall,
                "prefill_1k_first_call": {"value": PROMPT_LEN / prefill_s, "unit": "tok/s", "tokens": PROMPT_LEN,
                                          "note": "first qwen_prefill of the handle (includes one-time buffer and tensor-map setup)"}}
        if world == 1:
            eng.close()
            torch.cuda.empty_cache()
            def extra(name, fn):
                # secondary fields: a failure (e.g. no room for 128 KV slots on a shared GPU)
                # is reported in the field and never costs the headline line
                try:
                    line[name] = fn()
                except Exception as e:
                    line[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:200]}"}
                torch.cuda.empty_cache()

            extra("gemv_sweep", lambda: {"shapes": gemv_sweep(qb, peak), "peak_gbs": peak, "method": "64 launches replayed as one CUDA graph",
                                         "l2": "inputs larger than L2: 64 launches rotate over copies of W totalling >= 256 MB"})
            bf16_peak = measured_bf16_peak()
            extra("gemm_sweep", lambda: {"shapes": gemm_sweep(qb, bf16_peak), "peak_tflops": bf16_peak,
                                         "peak_source": "bf16_tflops (burst, MEASURED_PEAKS.json)",
                                         "l2": "flushed (256 MB write) between timed launches"})
            extra("long_context", lambda: long_context(qb, ck))
            extra("prefill", lambda: prefill_bench(qb, ck))
            extra("batched_decode", lambda: batched_decode(qb, ck))
            import oracle_py as O
            threads = os.cpu_count() or 1
            rate, n, dt = cpu_oracle_rate(ck, O.FP32, 15.0, 400, threads)
            line["cpu_baseline"] = {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
                                    "sample": f"{n} decode tokens at context 1024 ({dt:.1f} s), fp32 oracle, {threads} threads"}
            try:
                line["reference_cuda_b200"] = ref_cuda_rate(ck)
            except Exception as e:   # informational only
                line["reference_cuda_b200"] = {"unavailable": str(e)[:200]}
        print(json.dumps(line), flush=True)
    else:
        eng.close()
    if dist is not None:
        barrier()
        dist.destroy_process_group()


def run_shard(args):
    """--mode shard: the 151936-row LM head split across the N ranks (rows
    [r V / N, (r+1) V / N) on rank r), every rank running the same trunk on the
    same 1024-token prompt, the ranks' top-k exchanged per token by an NCCL
    all-gather on the engine's stream and merged on the device
    (sharding.ShardedHead).  value = per-token device latency, max over ranks,
    greedy and sampled (temperature 0.6, top-p 0.95, top-k 20)."""
    import datetime
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    qb = load_qb()
    import importlib.util
    spec = importlib.util.spec_from_file_location("sharding", os.path.join(REPO, "qwen600-rocm-inference_b200", "sharding.py"))
    sh = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(sh)
    ck = qb.default_checkpoint(0)
    eng = qb.Engine(ck, local)
    eng.set_vocab_shard(*sh.shard_range(rank, world))
    prompt = np.random.default_rng(1000).integers(0, 151936, PROMPT_LEN).tolist()
    eng.prefill(prompt, 0)
    head = sh.ShardedHead(eng)
    out = {}
    for name, sp in (("greedy", qb.GREEDY), ("top_k 20", qb.Sampling(0.6, 0.95, 20))):
        head.generate(prompt[-1], PROMPT_LEN - 1, max(args.warmup, 3), sp, 7)
        toks, _, ms = head.timed(prompt[-1], PROMPT_LEN - 1, args.steps, sp, 7)
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out[name] = float(t.item())
    if rank == 0:
        line = {"metric": "vocab-sharded LM head: batch-1 decode latency per token (Qwen3-0.6B bf16)", "value": out["greedy"],
                "unit": "ms/token", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3), "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": dict(CONFIG, parallelism=f"LM head rows split over {world} ranks, top-k all-gather (NCCL) + device merge"),
                "sampled_top_k20_ms_per_token": out["top_k 20"],
                "gpu_launches": 2 * args.steps}
        print(json.dumps(line), flush=True)
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--mode", default="replicas", choices=["replicas", "shard"])
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "shard":
        run_shard(args)
    else:
        run_mine(args)


if __name__ == "__main__":
    main()

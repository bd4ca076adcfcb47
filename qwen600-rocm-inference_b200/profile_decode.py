"""A small decode case for profilers (ncu) and quick timing.

    python qwen600-rocm-inference_b200/profile_decode.py [--prompt N] [--steps K] [--device D]

Builds an Engine on the seed-0 synthetic checkpoint, prefills N seeded prompt
tokens (rng 1000) with qwen_prefill — for N >= 65 the tensor-core passes over
positions 0..N-2 and one decode-kernel launch for the last token; below that,
N decode-kernel launches — then decodes K greedy positions with
qwen_decode_step (one launch each) and prints the host wall time per step.
ncu counts --launch-skip over the launches that match its kernel filter, so
for N >= 65

    ncu --set full --clock-control none -k regex:decode_kernel -s 2 -c 1 ...

captures the second decode step: position N + 1, context N + 2.  After the
K host-timed steps it re-decodes the same positions as K chained launches and
prints their device time per step.

With --batch B it profiles batched decode instead: B slots, each prefilled
with its own seeded N-token prompt (qwen_batch_prefill), then K greedy
qwen_batch_step calls over the B slots; --top-k k > 1 samples them instead
(temperature 0.6, top-p 0.95, top-k k, one RNG state per slot).
"""
import argparse
import importlib.util
import os
import time

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--top-k", type=int, default=1)
    a = ap.parse_args()
    spec = importlib.util.spec_from_file_location("qwen_b200", os.path.join(HERE, "qwen_b200.py"))
    qb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(qb)
    import numpy as np
    eng = qb.Engine(qb.default_checkpoint(0), a.device)
    if a.batch:
        eng.batch_init(a.batch)
        for slot in range(a.batch):
            eng.batch_prefill(slot, np.random.default_rng(1000 + slot).integers(0, qb.VOCAB_SIZE, a.prompt).tolist())
        toks, pos = [5] * a.batch, [a.prompt] * a.batch
        sp = qb.GREEDY if a.top_k <= 1 else qb.Sampling(0.6, 0.95, a.top_k)
        rs = None if a.top_k <= 1 else list(range(1, a.batch + 1))
        t0 = time.perf_counter()
        for _ in range(a.steps):
            toks, rs = eng.batch_step(toks, pos, sp, rs)
            pos = [p + 1 for p in pos]
        dt = time.perf_counter() - t0
        eng.close()
        print(f"batch {a.batch} top-k {a.top_k} prompt {a.prompt} steps {a.steps}: {dt / max(a.steps, 1) * 1e3:.2f} ms per step (host wall time)")
        return
    prompt = np.random.default_rng(1000).integers(0, qb.VOCAB_SIZE, a.prompt).tolist()
    eng.prefill(prompt, 0)
    tok = prompt[-1]
    t0 = time.perf_counter()
    for pos in range(a.prompt, a.prompt + a.steps):
        tok, _ = eng.decode_step(tok, pos)
    dt = time.perf_counter() - t0
    # the same positions again as chained launches, timed on the device (CUDA events)
    _, _, ms = eng.generate_timed(prompt[-1], a.prompt, a.steps)
    eng.close()
    print(f"prompt {a.prompt} steps {a.steps}: {dt / max(a.steps, 1) * 1e6:.1f} us per step (host wall time), "
          f"{ms * 1e3 / max(a.steps, 1):.1f} us per step (device time of chained launches)")


if __name__ == "__main__":
    main()

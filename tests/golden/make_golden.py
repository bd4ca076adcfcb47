"""Generate the golden fixtures in tests/golden/ from the reference's own code.

    python tests/golden/make_golden.py table     # needs the reference tree (CPU)
    python tests/golden/make_golden.py sampler   # needs oracle/_ref/libref_sampler.so (CPU)
    python tests/golden/make_golden.py forward   # needs oracle/_ref/libref_model.so and a GPU

table    tensor_table.json: the 311 (name, offset, bytes) entries of the
         reference's TENSOR_METADATA (static_loader.h:83-400), read as text.
sampler  sampler_cases.json: tokens and RNG states returned by the reference's
         own sample() (sampler.h:120-175), compiled from the reference tree, for
         seeded logit vectors (the test regenerates them from their seeds).
forward  ref_forward_seed0.npz: the reference's own CUDA forward()
         (qwen_model.cuh:772-851, compiled for sm_100a with cuBLAS) on the
         seed-0 synthetic checkpoint: 16 seeded prompt tokens then 24 greedy
         tokens (its own argmax), with logits summaries per position.  All
         positions stay below 1024, where the reference's attention is valid
         (qwen_model.cuh:560-564, 626).
"""
import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
REF = os.environ.get("REFERENCE_DIR") or os.path.normpath(os.path.join(REPO, os.pardir, "reference"))
VOCAB = 151936

# (logit seed, scale, temperature, topp, top_k, rng seed, bf16-valued logits)
SAMPLER_CASES = [
    (1, 0.64, 0.6, 0.95, 20, 12345, False),
    (2, 0.64, 0.6, 0.95, 20, 777, False),
    (3, 1.50, 0.6, 0.95, 20, 4242, False),
    (4, 0.64, 1.0, 0.90, 40, 99, False),
    (5, 0.64, 0.8, 0.50, 10, 2024, False),
    (6, 2.00, 0.3, 0.95, 20, 31337, False),
    (7, 0.64, 0.6, 0.95, 64, 5, False),
    (8, 0.64, 0.0, 0.95, 20, 11, False),     # temperature 0: argmax
    (9, 0.64, 0.7, 0.95, 1, 13, False),      # top_k 1: argmax
    (10, 0.64, 0.6, 1.00, 20, 17, False),    # top-p off: quickselect order
    (11, 0.64, 0.6, 0.00, 20, 19, False),    # top-p off
    # top_k 0 (whole vocabulary) is left out: the reference's quick_select then
    # reads its pivot one past the end (sampler.h:63, k == n) and never returns.
    (13, 0.64, 0.6, 0.95, 20, 29, True),     # bf16-valued logits (ties)
    (14, 3.00, 0.6, 0.95, 20, 31, True),
]


def sampler_logits(seed, scale, bf16):
    x = (np.random.default_rng(seed).standard_normal(VOCAB) * scale).astype(np.float32)
    if bf16:
        u = x.view(np.uint32).astype(np.uint64)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
        x = u.astype(np.uint32).view(np.float32)
    return x


def make_table():
    src = open(os.path.join(REF, "static_loader.h")).read()
    rows = re.findall(r'\{"([^"]+)",\s*(\d+),\s*(\d+)\}', src)
    tot = re.search(r"TOTAL_WEIGHTS_BYTES\s*=\s*(\d+)", src).group(1)
    out = {"total_bytes": int(tot), "tensors": [[n, int(o), int(b)] for n, o, b in rows]}
    with open(os.path.join(HERE, "tensor_table.json"), "w") as f:
        json.dump(out, f, indent=0)
    print("tensor_table.json:", len(rows), "tensors")


def make_sampler():
    import ctypes
    import oracle_py as O
    L = O.ref_sampler()
    if L is None:
        raise SystemExit("oracle/_ref/libref_sampler.so not built")
    cases = []
    for (ls, sc, T, p, k, rs, bf) in SAMPLER_CASES:
        lg = sampler_logits(ls, sc, bf)
        r = ctypes.c_ulonglong(rs)
        draws = []
        for _ in range(4):   # four consecutive draws on the same logits
            t = L.ref_sample(lg.ctypes.data, T, p, k, ctypes.byref(r))
            draws.append([int(t), int(r.value)])
        cases.append({"logit_seed": ls, "scale": sc, "temperature": T, "topp": p, "top_k": k, "rng": rs, "bf16": bf,
                      "draws": draws})
    with open(os.path.join(HERE, "sampler_cases.json"), "w") as f:
        json.dump({"cases": cases}, f, indent=1)
    print("sampler_cases.json:", len(cases), "cases")


def make_forward():
    import importlib.util
    import oracle_py as O
    spec = importlib.util.spec_from_file_location("qwen_b200", os.path.join(REPO, "qwen600-rocm-inference_b200", "qwen_b200.py"))
    qb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(qb)
    ck = qb.default_checkpoint(0)
    L = O.ref_model()
    if L is None:
        raise SystemExit("oracle/_ref/libref_model.so not built")
    if L.ref_build(ck.encode()) != 0:
        raise SystemExit("ref_build failed")
    prompt = np.random.default_rng(0).integers(0, VOCAB, 16).tolist()
    n_gen = 24
    probe = np.sort(np.random.default_rng(7).choice(VOCAB, 512, replace=False)).astype(np.int32)
    toks, top_i, top_v, probe_v, stats = [], [], [], [], []
    lg = np.zeros(VOCAB, dtype=np.float32)
    nxt = None
    for pos in range(16 + n_gen):
        tok = prompt[pos] if pos < 16 else nxt
        toks.append(tok)
        if L.ref_forward(tok, pos, lg.ctypes.data) != 0:
            raise SystemExit("ref_forward failed")
        nxt = int(np.argmax(lg))   # first maximum, as sample_argmax (sampler.h:82-97)
        order = np.argsort(-lg, kind="stable")[:32]
        top_i.append(order.astype(np.int32))
        top_v.append(lg[order])
        probe_v.append(lg[probe])
        d = lg.astype(np.float64)
        stats.append([d.sum(), (d * d).sum(), d.max()])
    L.ref_free()
    np.savez_compressed(os.path.join(HERE, "ref_forward_seed0.npz"), tokens=np.array(toks, np.int32), prompt_len=16,
                        top_i=np.array(top_i), top_v=np.array(top_v), probe_idx=probe, probe_v=np.array(probe_v),
                        stats=np.array(stats))
    print("ref_forward_seed0.npz:", len(toks), "positions")


if __name__ == "__main__":
    for what in sys.argv[1:] or ["table", "sampler"]:
        {"table": make_table, "sampler": make_sampler, "forward": make_forward}[what]()

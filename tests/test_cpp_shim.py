"""The reference-named C++ API (include/qwen_model_b200.h: Transformer,
build_transformer, forward, Sampler, build_sampler, sample — qwen_model.cuh:51-94,
:772 and sampler.h:11-120; Tokenizer, build_tokenizer, encode, decode —
tokenizer.h:14-104) compiled as plain C++ programs against libqwen_b200.so,
the way a maintainer swaps the reference's headers."""
import json
import sys
import os
import subprocess

import numpy as np
import pytest

from conftest import PKG, REPO

SRC = os.path.join(REPO, "tests", "cpp", "shim_greedy.cpp")
LIB_DIR = os.path.join(PKG, "lib")


def _build(tmp_path):
    exe = str(tmp_path / "shim_greedy")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"), SRC,
           "-o", exe, "-L", LIB_DIR, "-lqwen_b200", "-Wl,-rpath," + LIB_DIR]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_shim_compiles_and_links(qb, tmp_path):
    qb.load_library()          # the library is built
    exe = _build(tmp_path)
    assert os.path.exists(exe)
    # two translation units may include the header (everything is inline)
    a, b = tmp_path / "a.cpp", tmp_path / "b.cpp"
    a.write_text('#include "qwen_model_b200.h"\nint fa() { return qwen_vocab_size(); }\n')
    b.write_text('#include "qwen_model_b200.h"\nint fa();\nint main() { return fa() == 151936 ? 0 : 1; }\n')
    exe2 = str(tmp_path / "two_tu")
    r = subprocess.run(["g++", "-std=c++17", "-I", os.path.join(REPO, "include"), str(a), str(b), "-o", exe2,
                        "-L", LIB_DIR, "-lqwen_b200", "-Wl,-rpath," + LIB_DIR], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert subprocess.run([exe2]).returncode == 0   # qwen_vocab_size needs no GPU


@pytest.mark.gpu
def test_shim_greedy_matches_engine(qb, checkpoint, tmp_path):
    exe = _build(tmp_path)
    prompt = np.random.default_rng(5).integers(0, 151936, 8).tolist()
    r = subprocess.run([exe, checkpoint, str(len(prompt)), "12"] + [str(t) for t in prompt],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    got = [int(t) for t in r.stdout.split()]
    eng = qb.Engine(checkpoint, 0)
    try:
        eng.prefill(prompt[:-1], 0)
        want, _ = eng.generate(prompt[-1], len(prompt) - 1, 12)
    finally:
        eng.close()
    assert got == want


def test_shim_tokenizer_matches_reference_ids(qb, tmp_path):
    """Host-only: the tokenizer calls of tokenizer.h through the C++ names give
    the reference's own ids (tests/golden/tokenizer_cases.json)."""
    qb.load_library()
    sys.path.insert(0, os.path.join(REPO, "tests", "golden"))
    import make_tokenizer_golden as G
    d = tmp_path / "model"
    d.mkdir()
    G.write_model_dir(str(d))
    exe = str(tmp_path / "shim_tokenizer")
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
                        os.path.join(REPO, "tests", "cpp", "shim_tokenizer.cpp"), "-o", exe, "-L", LIB_DIR, "-lqwen_b200",
                        "-Wl,-rpath," + LIB_DIR], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    cases = json.load(open(os.path.join(REPO, "tests", "golden", "tokenizer_cases.json"), encoding="utf-8"))["cases"]
    for case in cases:
        if not case["text"]:
            continue                      # (an empty argv string is fine too, but keeps the output format simple)
        out = subprocess.run([exe, str(d), case["text"]], capture_output=True, timeout=60)
        assert out.returncode == 0, out.stderr
        lines = out.stdout.split(b"\n")
        k = lines.index(next(l for l in lines if l.startswith(b"#")))
        assert [int(x) for x in lines[:k]] == case["ids"]
        assert b"\n".join(lines[k:])[1:].rstrip(b"\n") == case["text"].encode("utf-8").rstrip(b"\n")


def _build_loader(tmp_path):
    exe = str(tmp_path / "shim_loader")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"), "-I", os.path.join(cuda, "include"),
           os.path.join(REPO, "tests", "cpp", "shim_loader.cpp"), "-o", exe, "-L", LIB_DIR, "-lqwen_b200",
           "-L", os.path.join(cuda, "lib64"), "-lcudart", "-Wl,-rpath," + LIB_DIR]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_loader_names_give_reference_table(qb, tmp_path):
    """static_loader.h's names (NUM_TENSORS, TOTAL_WEIGHTS_BYTES,
    TENSOR_METADATA[i].name/.offset/.size_bytes) compile against the library and
    hold the reference's own table (tests/golden/tensor_table.json, read from
    static_loader.h:80-400).  No GPU needed."""
    qb.load_library()
    exe = _build_loader(tmp_path)
    r = subprocess.run([exe, "table"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.split("\n")
    n, total = map(int, lines[0].split())
    gold = json.load(open(os.path.join(REPO, "tests", "golden", "tensor_table.json")))
    assert n == 311 and total == gold["total_bytes"]
    got = [(l.split()[0], int(l.split()[1]), int(l.split()[2])) for l in lines[1:1 + n]]
    want = [tuple(t) for t in gold["tensors"]]
    assert got == want                    # same entries, same index order as the reference's array


@pytest.mark.gpu
def test_loader_names_point_into_the_weight_block(qb, checkpoint, tmp_path):
    """load_qwen_weights and Transformer.weights: every member points at its
    tensor's canonical offset, and the tensors read back through them equal the
    checkpoint's bytes."""
    exe = _build_loader(tmp_path)
    r = subprocess.run([exe, "load", checkpoint], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr + r.stdout
    rows = [l.split() for l in r.stdout.strip().split("\n")]
    hdr = int.from_bytes(open(checkpoint, "rb").read(8), "little")
    meta = json.loads(open(checkpoint, "rb").read(8 + hdr)[8:])

    def fnv(name):
        a, b = meta[name]["data_offsets"]
        with open(checkpoint, "rb") as f:
            f.seek(8 + hdr + a)
            data = np.frombuffer(f.read(b - a), dtype=np.uint8)
        h = 1469598103934665603           # FNV-1a, as shim_loader.cpp hashes
        for x in data.tobytes():
            h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
        return f"{h:016x}"

    names = ["model.layers.5.self_attn.q_proj.weight", "model.layers.27.mlp.down_proj.weight", "model.norm.weight"]
    for row, name in zip(rows, names):
        want = fnv(name)
        assert row == [want, want], name

"""The reference-named C++ API (include/qwen_model_b200.h: Transformer,
build_transformer, forward, Sampler, build_sampler, sample — qwen_model.cuh:51-94,
:772 and sampler.h:11-120) compiled as a plain C++ program against
libqwen_b200.so, the way a maintainer swaps the reference's headers."""
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

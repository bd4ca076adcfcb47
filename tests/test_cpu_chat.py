"""Chat driver host logic: the reference's command-line defaults and clamps
(main.cu:236-270) and the sampler RNG advance used to keep the token stream
equal to the reference's (checked against the reference's own random_u32,
compiled into oracle/_ref/ where the reference tree was available)."""
import ctypes
import importlib.util
import os

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _chat():
    spec = importlib.util.spec_from_file_location("qwen_chat", os.path.join(REPO, "qwen600-rocm-inference_b200", "chat.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


C = _chat()


def test_defaults_and_clamps():
    a = C.parse_args(["model"])
    assert (a.temperature, a.top_p, a.top_k, a.prompt, a.system_prompt, a.thinking) == (0.6, 0.95, 20, None, None, 0)
    assert a.seed > 0                                # seed <= 0 -> the clock
    a = C.parse_args(["m", "-t", "-1", "-p", "1.5", "-k", "5", "-s", "42", "-i", "hi", "-y", "sys", "-r", "1"])
    assert (a.temperature, a.top_p, a.top_k, a.seed, a.prompt, a.system_prompt, a.thinking) == (0.0, 0.95, 5, 42, "hi", "sys", 1)
    assert C.parse_args(["m", "-p", "-0.1"]).top_p == 0.95


def test_rng_advance_matches_reference_generator():
    lib_path = os.path.join(REPO, "oracle", "_ref", "libref_sampler.so")
    if not os.path.exists(lib_path):
        pytest.skip("reference sampler not built (no reference tree when it was built)")
    lib = ctypes.CDLL(lib_path)
    lib.ref_random_u32.restype = ctypes.c_uint
    lib.ref_random_u32.argtypes = [ctypes.POINTER(ctypes.c_ulonglong)]
    for seed in (1, 42, 0x5EED, (1 << 63) + 12345):
        for k in (0, 1, 7, 100):
            r = ctypes.c_ulonglong(seed)
            for _ in range(k):
                lib.ref_random_u32(ctypes.byref(r))
            assert C.rng_advance(seed, k) == r.value

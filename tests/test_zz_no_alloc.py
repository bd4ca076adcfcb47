"""qwen_gemv_bf16_static: the GEMV entry point that allocates nothing.

It exists for callers that may not call cudaMalloc (code running during a
stream capture, or inside a framework whose allocator owns the device memory).
It runs the same kernels on the same inputs as qwen_gemv_bf16, so its output
must equal that entry point's bit for bit, on two calls in a row (its scratch
array keeps the previous call's contents; the error word it holds must read
clear through qwen_gemv_bf16_static_status after both).  The shapes cover both
kernels: the direct-load one (up to 64 MB) and the TMA-ring one (the LM head),
whose error word is the scratch.  Collected last on purpose, and it passes
alone in a fresh process too."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k,n", [(1024, 4096), (3072, 1024), (1024, 151936)])
def test_static_gemv_matches_allocating_gemv(qb, O, k, n):
    import torch
    g = np.random.default_rng(n + k)
    W = O.bf16_bits(g.standard_normal((n, k), dtype=np.float32) * 0.02)
    x = O.bf16_bits(g.standard_normal(k, dtype=np.float32))
    Wd = torch.from_numpy(W.view(np.int16)).cuda()
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    y_ref = torch.zeros(n, dtype=torch.int16, device="cuda")
    qb.gemv_bf16(Wd.data_ptr(), xd.data_ptr(), y_ref.data_ptr(), n, k)
    qb.gemv_status()
    want = y_ref.cpu().numpy().view(np.uint16)
    for call in range(2):
        y = torch.full((n,), -1, dtype=torch.int16, device="cuda")
        qb.gemv_bf16_static(Wd.data_ptr(), xd.data_ptr(), y.data_ptr(), n, k)
        qb.gemv_status(static=True)
        got = y.cpu().numpy().view(np.uint16)
        assert np.array_equal(got, want), (call, int(np.count_nonzero(got != want)))


def test_static_gemv_rejects_oversized_k(qb):
    import torch
    t = torch.zeros(8192, dtype=torch.int16, device="cuda")
    with pytest.raises(qb.QwenError) as e:
        qb.gemv_bf16_static(t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 8192)
    assert e.value.code == -1 and "4096" in str(e.value)

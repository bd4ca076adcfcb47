"""qwen_gemv_bf16_static: the GEMV entry point that allocates nothing.

It exists for callers that may not call cudaMalloc (code running during a
stream capture, or inside a framework whose allocator owns the device memory).
It must give the same result as qwen_gemv_bf16 on the same inputs, on two
calls in a row (its scratch array keeps the previous call's contents, so the
second call checks that the entry point clears what must start at zero).
Collected last on purpose, and it passes alone in a fresh process too."""
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
    torch.cuda.synchronize()
    want = y_ref.cpu().numpy().view(np.uint16)
    for call in range(2):
        y = torch.full((n,), -1, dtype=torch.int16, device="cuda")
        qb.gemv_bf16_static(Wd.data_ptr(), xd.data_ptr(), y.data_ptr(), n, k)
        torch.cuda.synchronize()
        got = y.cpu().numpy().view(np.uint16)
        a, b = O.bf16_to_f32(got), O.bf16_to_f32(want)
        tol = np.maximum(np.abs(b) * 2.0 ** -7, 1e-4)   # the GEMV tests' tolerance
        assert (np.abs(a - b) <= tol).all(), (call, float(np.abs(a - b).max()))


def test_static_gemv_rejects_oversized_k(qb):
    import torch
    t = torch.zeros(8192, dtype=torch.int16, device="cuda")
    with pytest.raises(qb.QwenError) as e:
        qb.gemv_bf16_static(t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 8192)
    assert e.value.code == -1 and "4096" in str(e.value)

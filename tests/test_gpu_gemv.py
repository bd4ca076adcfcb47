"""Isolated bf16 GEMV (qwen_gemv_bf16) against the oracle on the sweep shapes
K->N: 1024->4096 (QKV), 2048->1024 (O), 1024->6144 (gate|up), 3072->1024
(down), 1024->151936 (LM head), plus edge shapes: row counts that leave a
CTA's row group or row pair partly empty, every segment count (k = 256 ..
4096), and matrices on both sides of the 64 MB switch from the direct-load
kernel to the TMA-ring kernel.  After each call the error word reads clear
(qwen_gemv_bf16_status).

Tolerance: both sides accumulate exactly enough that the bf16 outputs agree
bit for bit except where the fp32 sum sits next to a bf16 rounding boundary;
there they may differ by one bf16 step, and near zero by 1e-4 absolute."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(1024, 4096), (2048, 1024), (1024, 6144), (3072, 1024), (1024, 151936), (256, 1), (256, 7), (4096, 300), (1280, 149),
          (2048, 3), (3072, 5), (768, 33), (3072, 10922), (3072, 10923), (4096, 70000)]


@pytest.mark.parametrize("k,n", SHAPES)
def test_gemv_matches_oracle(qb, O, k, n):
    import torch
    g = np.random.default_rng(k * 7 + n)
    W = O.bf16_bits(g.standard_normal((n, k), dtype=np.float32) * 0.02)
    x = O.bf16_bits(g.standard_normal(k, dtype=np.float32))
    want = O.gemv_bf16(W, x)
    Wd = torch.from_numpy(W.view(np.int16)).cuda()
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    yd = torch.full((n,), -1, dtype=torch.int16, device="cuda")
    qb.gemv_bf16(Wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), n, k)
    qb.gemv_status()
    got = yd.cpu().numpy().view(np.uint16)
    a, b = O.bf16_to_f32(got), O.bf16_to_f32(want)
    tol = np.maximum(np.abs(b) * 2.0 ** -7, 1e-4)
    assert (np.abs(a - b) <= tol).all(), float(np.abs(a - b).max())
    assert np.mean(got == want) > 0.999


def test_gemv_rejects_bad_shapes(qb):
    import torch
    t = torch.zeros(4096, dtype=torch.int16, device="cuda")
    for n, k in [(4, 100), (4, 8192), (0, 256)]:
        with pytest.raises(qb.QwenError) as e:
            qb.gemv_bf16(t.data_ptr(), t.data_ptr(), t.data_ptr(), n, k)
        assert e.value.code == -1

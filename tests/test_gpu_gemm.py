"""qwen_gemm_bf16 (persistent tcgen05 tensor-core GEMM) against float64 products of the same
bf16 inputs: C = A B^T with A [M][K], B [N][K] row-major.  fp32 output within
1e-5 of sum |a_k b_k| per element (fp32 accumulation of exact bf16 products);
bf16 output within one bf16 rounding of that."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _case(qb, M, N, K, c_fp32, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.randn(M, K, generator=g, device="cuda")).to(torch.bfloat16)
    B = (torch.randn(N, K, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    C = torch.empty(M, N, dtype=torch.float32 if c_fp32 else torch.bfloat16, device="cuda")
    qb.gemm_bf16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, c_fp32, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = A.double() @ B.double().T
    mag = A.double().abs() @ B.double().abs().T
    return C.double(), ref, mag


# M and N multiples of 256 run in the pair form (256 x 256 tiles on two SMs of a
# cluster): (2048, 4096), (2048, 6144) and (4096, 4096) give a pair two to four
# tiles, alternating its two TMEM accumulators.  The others run single-CTA tiles:
# (1920, 4096) and (1920, 1024) 128 x 256 tiles, several per CTA; the small ones
# one 128 x 128 tile per CTA.
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 384, 512), (384, 512, 1024), (2048, 4096, 1024), (2048, 1024, 3072),
                                   (2048, 6144, 1024), (4096, 4096, 256), (1920, 4096, 1024), (1920, 1024, 3072)])
def test_gemm_fp32_out(qb, M, N, K):
    C, ref, mag = _case(qb, M, N, K, True, M + N + K)
    err = ((C - ref).abs() / (mag + 1e-30)).max().item()
    assert err <= 1e-5, err


def test_gemm_bf16_out(qb):
    C, ref, mag = _case(qb, 256, 512, 1024, False, 7)
    # one bf16 rounding of the fp32 result (relative 2^-8) plus the accumulation error
    assert ((C - ref).abs() <= ref.abs() * 2.0 ** -8 + mag * 1e-5).all()


def test_gemm_rejects_bad_shapes(qb):
    import torch
    A = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    B = torch.zeros(256, 64, dtype=torch.bfloat16, device="cuda")
    C = torch.zeros(128, 256, dtype=torch.float32, device="cuda")
    for (M, N, K) in [(100, 256, 64), (128, 200, 64), (128, 256, 48)]:
        with pytest.raises(qb.QwenError) as e:
            qb.gemm_bf16(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, True)
        assert e.value.code == -1

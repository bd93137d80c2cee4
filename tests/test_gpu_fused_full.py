"""dense_fused_i8 end to end at every shape the benchmark times, whole matrices.

Config 2 (square, N(0,1), scale 1, no ReLU) at 1024, 2048, 4096 and 8192, and
config 4 (M tokens x 14336 x 4096, N(0,1) with 1 % of A's entries x20, ReLU,
scale 0.125) at M = 1, 8, 64 and 512: the GPU's int8 codes, scales, int32
accumulators and fp32 C are each compared with the oracle over the whole
tensor (tests/fused_check.py).  Calls go through the C ABI (ane_b200 wraps
ane_dense_fused_i8_dev, ane_quantize_pair_dev and ane_gemm_s8_dev).
"""
import pytest

from fused_check import check_dense_fused

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1024, 2048, 4096, 8192])
def test_config2_square_whole_matrix(ane, n):
    import torch

    g = torch.Generator(device="cuda").manual_seed(1234 + n)
    A = torch.randn((n, n), device="cuda", generator=g)
    B = torch.randn((n, n), device="cuda", generator=g)
    C = ane.dense_fused_i8(A, B, 1.0, False)
    check_dense_fused(ane, torch, A, B, C, 1.0, False)


@pytest.mark.parametrize("m", [1, 8, 64, 512])
def test_config4_projection_whole_matrix(ane, m):
    import torch

    g = torch.Generator(device="cuda").manual_seed(4 + m)
    A = torch.randn((m, 4096), device="cuda", generator=g)
    A = torch.where(torch.rand(A.shape, device="cuda", generator=g) < 0.01, A * 20, A)
    B = torch.randn((4096, 14336), device="cuda", generator=g)
    C = ane.dense_fused_i8(A, B, 0.125, True)
    check_dense_fused(ane, torch, A, B, C, 0.125, True)

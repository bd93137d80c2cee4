"""GPU test of ane_dense_fused_i8_noalloc_dev, the allocation-free dense_fused_i8.

That entry point is for callers that cannot allocate device memory when they
run the op (a framework that already holds nearly all GPU memory in its own
pool, a ggml-style backend inside graph_compute, latency-critical loops where
cudaMalloc/cudaFree would synchronise).  It keeps its scratch in a fixed 40 MiB
array inside the library instead of a workspace.

Checked through the C ABI, two calls in a row each time (the second reuses the
array the first left behind):
* against the oracle: small shapes with the oracle's full dense_fused_i8, and
  M = N = K = 4096 -- the largest problem the array takes, which runs the
  cooperative prologue -- piece by piece over the whole matrix
  (tests/fused_check.py); bit for bit, with the 1e-5 relative bar asserted too;
* against ane_dense_fused_i8_dev (the workspace entry point): bit for bit;
* the limit: the first shape past the array's size is refused with
  ANE_ERR_INVALID_ARGUMENT before any pointer is touched.
The file name sorts last so a stop-at-first-failure run has finished every
other test before this one; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

import oracle
from fused_check import bits_equal, check_dense_fused, reference_parts

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 40 << 20


def _noalloc(ane, torch, A, B, scale, relu):
    M, K = A.shape
    N = B.shape[1]
    C = torch.full((M, N), float("nan"), device=A.device)
    ane.check(ane.lib.ane_dense_fused_i8_noalloc_dev(M, N, K, scale, int(relu), A.data_ptr(), B.data_ptr(),
                                                     C.data_ptr(), ane._stream_ptr()))
    return C


@pytest.mark.parametrize("M,N,K,scale,relu", [(50, 128, 784, 1.0, True), (512, 1000, 4096, 0.125, False),
                                              (64, 4096, 4096, 0.125, True)])
def test_noalloc_matches_oracle_small(M, N, K, scale, relu):
    import torch

    import ane_b200 as ane

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(M + N + K)
    A = torch.randn((M, K), device=dev, generator=g)
    B = torch.randn((K, N), device=dev, generator=g)
    ref = oracle.dense_fused_i8_omp(A.cpu().numpy(), B.cpu().numpy(), scale, relu)
    ws = ane.dense_fused_i8(A, B, scale, relu)  # workspace entry point
    for _ in range(2):  # two calls in a row share the fixed scratch array
        C = _noalloc(ane, torch, A, B, scale, relu)
        torch.cuda.synchronize()
        c = C.cpu().numpy()
        assert bits_equal(c, ref)
        np.testing.assert_allclose(c, ref, rtol=1e-5, atol=0)
        assert bits_equal(c, ws.cpu().numpy())
    assert ane.lib.ane_device_timeouts() == 0


def test_noalloc_matches_oracle_at_the_largest_size():
    import torch

    import ane_b200 as ane

    M = N = K = 4096
    assert ane.lib.ane_dense_fused_i8_workspace_size(M, N, K) <= SCRATCH_BYTES
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(99)
    A = torch.randn((M, K), device=dev, generator=g)
    B = torch.randn((K, N), device=dev, generator=g)
    parts = reference_parts(torch, A, B, 1.0, False)
    ws = ane.dense_fused_i8(A, B, 1.0, False)
    for _ in range(2):
        C = _noalloc(ane, torch, A, B, 1.0, False)
        torch.cuda.synchronize()
        check_dense_fused(ane, torch, A, B, C, 1.0, False, parts=parts, check_stages=False)
        assert torch.equal(C.view(torch.int32), ws.view(torch.int32))
    assert ane.lib.ane_device_timeouts() == 0


def test_noalloc_refuses_the_first_shape_past_the_array():
    import ane_b200 as ane

    # K = 5104 still fits (2 x 4096 x 5104 int8 codes + scales + partials);
    # K = 5120 (the next multiple of 16) does not
    assert ane.lib.ane_dense_fused_i8_workspace_size(4096, 4096, 5104) <= SCRATCH_BYTES
    assert ane.lib.ane_dense_fused_i8_workspace_size(4096, 4096, 5120) > SCRATCH_BYTES
    rc = ane.lib.ane_dense_fused_i8_noalloc_dev(4096, 4096, 5120, 1.0, 0, 1, 1, 1, None)
    assert rc == 1  # ANE_ERR_INVALID_ARGUMENT, before touching any pointer
    assert b"fixed buffer" in ane.lib.ane_last_error_string()
    rc = ane.lib.ane_dense_fused_i8_noalloc_dev(8192, 8192, 8192, 1.0, 0, 1, 1, 1, None)
    assert rc == 1

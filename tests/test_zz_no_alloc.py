"""GPU test of ane_dense_fused_i8_noalloc_dev, the allocation-free dense_fused_i8.

That entry point is for callers that cannot allocate device memory when they
run the op (a framework that already holds nearly all GPU memory in its own
pool, a ggml-style backend inside graph_compute, latency-critical loops where
cudaMalloc/cudaFree would synchronise).  It keeps its scratch in a fixed 40 MiB
array inside the library instead of a workspace.

Checked through the C ABI: two calls in a row (the second reuses the array the
first left behind) must match ane_dense_fused_i8_dev bit for bit -- the
tolerance the other parity tests use, with the 1e-5 relative bar asserted too --
and a problem too large for the array must be refused with
ANE_ERR_INVALID_ARGUMENT.  The file name sorts last so a stop-at-first-failure
run has finished every other test before this one; it also passes on its own in
a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits_equal(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    nan = np.isnan(a) | np.isnan(b)
    return np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32),
                                                                       b[~nan].view(np.uint32))


def test_noalloc_matches_workspace_entry_twice():
    import torch

    assert torch.cuda.is_available()
    import ane_b200 as ane

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream().cuda_stream
    cases = [(50, 128, 784, 1.0, True), (512, 1000, 4096, 0.125, False)]
    for M, N, K, scale, relu in cases:
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        A = torch.randn((M, K), device=dev, generator=g)
        B = torch.randn((K, N), device=dev, generator=g)
        ref = ane.dense_fused_i8(A, B, scale, relu)  # workspace entry point
        outs = []
        for _ in range(2):  # two calls in a row share the fixed scratch array
            C = torch.full((M, N), float("nan"), device=dev)
            ane.check(ane.lib.ane_dense_fused_i8_noalloc_dev(M, N, K, scale, int(relu), A.data_ptr(), B.data_ptr(),
                                                             C.data_ptr(), stream))
            outs.append(C)
        torch.cuda.synchronize()
        r = ref.cpu().numpy()
        for C in outs:
            c = C.cpu().numpy()
            assert _bits_equal(c, r)
            np.testing.assert_allclose(c, r, rtol=1e-5, atol=0)


def test_noalloc_refuses_problems_beyond_the_fixed_buffer():
    import ane_b200 as ane

    # 8192^3 needs 2 x 64 MiB of int8 scratch > 40 MiB
    rc = ane.lib.ane_dense_fused_i8_noalloc_dev(8192, 8192, 8192, 1.0, 0, 1, 1, 1, None)
    assert rc == 1  # ANE_ERR_INVALID_ARGUMENT, before touching any pointer
    assert b"fixed buffer" in ane.lib.ane_last_error_string()

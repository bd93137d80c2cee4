"""Failure detection on one GPU, without a fault: a bounded device wait runs out.

The N-sharded dense_fused_i8 gathers C with NVLink peer stores from the GEMM
epilogue; every CTA then bumps each rank's arrival counter and a one-thread
kernel on each GPU waits (bounded, about 2 s) until all ranks' CTAs arrived.
Here both "ranks" live on one GPU: rank 1's output buffer and counter are
ordinary local buffers.

* When rank 1's counter is a different word from rank 0's, rank 0's counter
  only ever receives rank 0's own arrivals -- exactly what a peer that died
  between steps looks like.  The wait gives up, counts one device timeout and
  returns; the stream and the context stay usable.
* When both counter pointers name the same word, the arrivals of "both ranks"
  reach it, the wait completes, and C equals the single-GPU result bit for bit.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(torch, ane, dev, M=512, N=512, K=512):
    g = torch.Generator(device=dev).manual_seed(7)
    A = torch.randn((M, K), device=dev, generator=g)
    B = torch.randn((K, N), device=dev, generator=g)
    Aq, Bq, scales = ane.quantize_pair(A, B)
    ref = ane.dense_fused_i8(A, B, 1.0, False)
    return Aq, Bq, scales, ref


def _gather(ane, torch, Aq, Bq, scales, C_ranks, ctr_ranks, epoch):
    import ctypes

    M, K16 = Aq.shape
    N = C_ranks[0].shape[1]
    c_arr = (ctypes.c_void_p * 2)(*[c.data_ptr() for c in C_ranks])
    k_arr = (ctypes.c_void_p * 2)(*[c.data_ptr() for c in ctr_ranks])
    return ane.lib.ane_gemm_s8_gather_dev(M, N, K16, Aq.data_ptr(), Bq.data_ptr(), scales.data_ptr(), 1.0, 0, 2, 0,
                                          c_arr, N, k_arr, epoch.data_ptr(), ane._stream_ptr())


def test_gather_wait_times_out_when_a_rank_never_arrives():
    import torch

    import ane_b200 as ane

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Aq, Bq, scales, ref = _setup(torch, ane, dev)
    assert ane.lib.ane_device_timeouts() == 0
    C0, C1 = torch.zeros_like(ref), torch.zeros_like(ref)
    ctr0 = torch.zeros(1, dtype=torch.int32, device=dev)
    ctr1 = torch.zeros(1, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    ane.check(_gather(ane, torch, Aq, Bq, scales, [C0, C1], [ctr0, ctr1], epoch))
    torch.cuda.synchronize()  # returns after the bounded wait gave up (about 2 s)
    assert ane.lib.ane_device_timeouts() == 1
    assert ane.lib.ane_device_timeouts() == 0  # read and reset
    assert int(epoch.item()) == 1  # the wait kernel still finished its call
    # the local tiles were written before the wait; the context is still usable
    assert torch.equal(C0.view(torch.int32), ref.view(torch.int32))
    again = ane.dense_fused_i8(torch.randn(64, 64, device=dev), torch.randn(64, 64, device=dev))
    torch.cuda.synchronize()
    assert bool(torch.isfinite(again).all())
    assert ane.lib.ane_device_timeouts() == 0


def test_gather_wait_completes_when_every_rank_arrives():
    import torch

    import ane_b200 as ane

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Aq, Bq, scales, ref = _setup(torch, ane, dev)
    C0, C1 = torch.zeros_like(ref), torch.zeros_like(ref)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int32, device=dev)
    for step in range(3):  # counters only grow; each call waits for its own arrivals
        ane.check(_gather(ane, torch, Aq, Bq, scales, [C0, C1], [ctr, ctr], epoch))
        torch.cuda.synchronize()
        assert ane.lib.ane_device_timeouts() == 0
        assert int(epoch.item()) == step + 1
    for C in (C0, C1):
        np.testing.assert_array_equal(C.view(torch.int32).cpu().numpy(), ref.view(torch.int32).cpu().numpy())

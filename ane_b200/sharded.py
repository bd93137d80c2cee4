"""N-sharded dense_fused_i8 across GPUs (one process per GPU, NCCL over NVLink).

Partitioning: every rank holds the full A (M x K) and a column shard of B
(K x N_local); rank r produces columns [r*N_local, (r+1)*N_local) of C.
The only cross-rank dependencies are

1. the per-tensor absmax: each rank reduces its local absmax of A and B into
   two floats and the ranks all-reduce them with MAX, so every shard is
   quantized with exactly the scales one GPU would compute;
2. the output (optional): the M x N_local shards are all-gathered and
   interleaved into the row-major M x (world*N_local) result.

Because the global scales are identical and all per-element arithmetic is
unchanged, the sharded result is bit-identical to the 1-GPU dense_fused_i8.

`ShardPlan` holds the collective orchestration and is independent of where
the compute runs (the CPU tests drive it with gloo ranks and the oracle);
`ShardedDense` binds it to libane_b200's kernels and NCCL.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def global_absmax(local_absmax2: torch.Tensor, group=None) -> torch.Tensor:
    """All-reduce (MAX) the per-rank absmax of A and of B, in place.

    The values are non-negative floats or NaN, whose bit patterns order as
    integers exactly like the reference's propagating max (NaN > inf >
    finite); reducing the int32 view keeps a NaN on any rank, which a float
    MAX collective may drop."""
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(local_absmax2.view(torch.int32), op=dist.ReduceOp.MAX, group=group)
    return local_absmax2


def interleave_shards(gathered: torch.Tensor) -> torch.Tensor:
    """[world, M, N_local] -> [M, world * N_local] (column shards side by side)."""
    world, M, n_local = gathered.shape
    return gathered.permute(1, 0, 2).reshape(M, world * n_local)


class ShardPlan:
    """Collective steps of the sharded op around two compute callables:
    absmax2(A_part, B_part) -> float[2] (local absmax of the two operands) and
    quantize_gemm(A_part, B_part, absmax2) -> C_part.

    shard="cols": every rank has all of A and a column block of B; C blocks are
    interleaved after the gather.  shard="rows": every rank has a row block of
    A and all of B; the gathered row blocks are already the row-major C."""

    def __init__(self, world: int, group=None, shard: str = "cols"):
        assert shard in ("cols", "rows")
        self.world = world
        self.group = group
        self.shard = shard

    def run(self, A, B, absmax2_fn: Callable, quantize_gemm_fn: Callable, gather: bool = True,
            gathered_out: torch.Tensor | None = None):
        absmax2 = global_absmax(absmax2_fn(A, B), self.group)
        C_local = quantize_gemm_fn(A, B, absmax2)
        if not gather:
            return C_local
        if self.world > 1:
            if gathered_out is None:
                gathered_out = torch.empty((self.world,) + tuple(C_local.shape), dtype=C_local.dtype,
                                           device=C_local.device)
            if gathered_out.is_cuda:
                dist.all_gather_into_tensor(gathered_out, C_local, group=self.group)
            else:  # gloo has no all_gather_into_tensor
                dist.all_gather(list(gathered_out.unbind(0)), C_local, group=self.group)
            if self.shard == "rows":
                return gathered_out.view(self.world * C_local.shape[0], C_local.shape[1])
            return interleave_shards(gathered_out)
        return C_local


class PeerBuffers:
    """A device tensor of this rank, opened on every rank through CUDA IPC:
    ptrs[q] is rank q's copy of the same-shaped buffer as seen from this GPU
    (ptrs[rank] is local).  Collective: every rank constructs it together."""

    def __init__(self, nbytes: int, device, group=None):
        import ctypes

        import ane_b200 as ane

        self._ane = ane
        self.tensor = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        base = self.tensor.data_ptr()
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_uint64()
        ane.check(ane.lib.ane_ipc_get_handle(base, handle, ctypes.byref(off)))
        everyone = [None] * world
        dist.all_gather_object(everyone, (bytes(handle), off.value), group=group)
        self._opened = []
        self.ptrs = []
        for q in range(world):
            if q == rank:
                self.ptrs.append(base)
                continue
            h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[q][0])
            b = ctypes.c_void_p()
            ane.check(ane.lib.ane_ipc_open_handle(h, ctypes.byref(b)))
            self._opened.append(b.value)
            self.ptrs.append(b.value + everyone[q][1])

    def close(self):
        for b in self._opened:
            self._ane.lib.ane_ipc_close_handle(b)
        self._opened = []


class ShardedDense:
    """dense_fused_i8 over this rank's part on its GPU.

    shard="cols": operands A (M x K) and a column block of B (K x N_local).
    shard="rows": operands a row block of A (M x K, M = rows per rank) and all
    of B (K x N_local, N_local = N)."""

    def __init__(self, M: int, N_local: int, K: int, world: int, device, group=None, shard: str = "cols",
                 fused_gather: bool = False):
        import ane_b200 as ane

        self.ane = ane
        self.group, self.shard = group, shard
        self.M, self.N_local, self.K, self.world = M, N_local, K, world
        self.plan = ShardPlan(world, group, shard)
        K16 = (K + 15) // 16 * 16
        self.absmax2 = torch.empty(2, dtype=torch.float32, device=device)
        self.partials = torch.empty(int(ane.lib.ane_absmax_partials_count(M * K, K * N_local)),
                                    dtype=torch.float32, device=device)
        self.Aq = torch.empty((M, K16), dtype=torch.int8, device=device)
        # codes of this rank's B block in B's layout (K16 rows of N16 bytes)
        self.Bq = torch.empty((K16, (N_local + 15) // 16 * 16), dtype=torch.int8, device=device)
        self.scales = torch.empty(2, dtype=torch.float32, device=device)
        self.C_local = torch.empty((M, N_local), dtype=torch.float32, device=device)
        self.gathered = torch.empty((world, M, N_local), dtype=torch.float32, device=device)
        # fused gather: the GEMM epilogue stores each tile into every rank's
        # gathered C (one IPC-shared buffer per rank: C, then a counter and the
        # call count); rows -> [world*M, N_local], cols -> [M, world*N_local]
        self.fused = None
        if fused_gather and world > 1:
            import ctypes

            c_bytes = world * M * N_local * 4
            # after C: gather counter (+0), gather call count (+128), the
            # prologue's absmax exchange area (+256, 2 words per rank), its
            # control words (+512)
            self.fused = PeerBuffers(c_bytes + 1024, device, group)
            rank = dist.get_rank(group)
            if shard == "rows":
                off, self.ldc = rank * M * N_local * 4, N_local
                shape = (world * M, N_local)
            else:
                off, self.ldc = rank * N_local * 4, world * N_local
                shape = (M, world * N_local)
            self._c_ranks = (ctypes.c_void_p * world)(*[b + off for b in self.fused.ptrs])
            self._ctr_ranks = (ctypes.c_void_p * world)(*[b + c_bytes for b in self.fused.ptrs])
            self._epoch = self.fused.ptrs[rank] + c_bytes + 128
            self._slot_peer = (ctypes.c_void_p * world)(*[b + c_bytes + 256 + 16 * rank for b in self.fused.ptrs])
            self._slots = self.fused.ptrs[rank] + c_bytes + 256
            self._xctl = self.fused.ptrs[rank] + c_bytes + 512
            K16 = (K + 15) // 16 * 16
            self._coop = (K % 16 == 0 and N_local % 16 == 0 and M * K + K * N_local >= (1 << 22)
                          and K16 == K)
            self._rank = rank
            self.C_gathered = self.fused.tensor[:c_bytes].view(torch.float32).view(*shape)

    def _absmax2(self, A, B_local):
        ane = self.ane
        ane.check(ane.lib.ane_absmax_pair_dev(A.data_ptr(), self.M * self.K, B_local.data_ptr(),
                                              self.K * self.N_local, self.absmax2.data_ptr(),
                                              self.partials.data_ptr(), ane._stream_ptr()))
        return self.absmax2

    def forward(self, A, B_local, scale: float = 1.0, relu: bool = False, gather: bool = True):
        ane = self.ane
        if self.fused is not None and gather:
            # the absmax exchange (tagged peer words, or the NCCL all-reduce) is
            # also the handshake: every rank has entered this call (its earlier
            # readers of C_gathered are done) before any GEMM epilogue stores
            # into peers
            if self._coop and A.data_ptr() % 16 == 0 and B_local.data_ptr() % 16 == 0:
                # one cooperative launch: A and B read once, absmax exchanged
                # with the peers through tagged words (also the handshake)
                ane.check(ane.lib.ane_quantize_pair_xrank_dev(
                    self.M, self.N_local, self.K, A.data_ptr(), B_local.data_ptr(), self.Aq.data_ptr(),
                    self.Bq.data_ptr(), self.scales.data_ptr(), self.partials.data_ptr(), self.world, self._rank,
                    self._slot_peer, self._slots, self._xctl, ane._stream_ptr()))
            else:
                absmax2 = global_absmax(self._absmax2(A, B_local), self.group)
                ane.check(ane.lib.ane_quantize_pair_absmax_dev(self.M, self.N_local, self.K, A.data_ptr(),
                                                               B_local.data_ptr(), self.Aq.data_ptr(),
                                                               self.Bq.data_ptr(), absmax2.data_ptr(),
                                                               self.scales.data_ptr(), ane._stream_ptr()))
            ane.check(ane.lib.ane_gemm_s8_gather_dev(self.M, self.N_local, self.Aq.shape[1], self.Aq.data_ptr(),
                                                     self.Bq.data_ptr(), self.scales.data_ptr(), float(scale),
                                                     int(bool(relu)), self.world, self._rank, self._c_ranks,
                                                     self.ldc, self._ctr_ranks, self._epoch, ane._stream_ptr()))
            return self.C_gathered

        def quantize_gemm(A, B_local, absmax2):
            ane.check(ane.lib.ane_quantize_pair_absmax_dev(self.M, self.N_local, self.K, A.data_ptr(),
                                                           B_local.data_ptr(), self.Aq.data_ptr(),
                                                           self.Bq.data_ptr(), absmax2.data_ptr(),
                                                           self.scales.data_ptr(), ane._stream_ptr()))
            return ane.gemm_s8_kn(self.Aq, self.Bq, self.N_local, self.scales, scale, relu, out=self.C_local)

        return self.plan.run(A, B_local, self._absmax2, quantize_gemm, gather, self.gathered)

    def close(self):
        if self.fused is not None:
            self.fused.close()
            self.fused = None

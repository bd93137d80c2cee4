"""N-sharded dense_fused_i8 across GPUs (one process per GPU, NCCL over NVLink).

Partitioning: every rank holds the full A (M x K) and a column shard of B
(K x N_local); rank r produces columns [r*N_local, (r+1)*N_local) of C.
The only cross-rank dependencies are

1. the per-tensor absmax: each rank reduces its local absmax of A and B into
   two floats (ane_absmax_pair_dev) and the ranks all-reduce them with MAX, so
   every shard is quantized with exactly the scales a single GPU would use;
2. the output: the M x N_local shards are all-gathered and interleaved into the
   row-major M x (world*N_local) result.

Because the global scales are identical and all per-element arithmetic is
unchanged, the sharded result is bit-identical to the 1-GPU dense_fused_i8.
The collectives go through torch.distributed (NCCL); the compute is
libane_b200's kernels.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

import ane_b200 as ane


class ShardedDense:
    def __init__(self, M: int, N_local: int, K: int, world: int, device, group=None):
        self.M, self.N_local, self.K, self.world = M, N_local, K, world
        self.group = group
        K16 = (K + 15) // 16 * 16
        self.absmax2 = torch.empty(2, dtype=torch.float32, device=device)
        self.partials = torch.empty(int(ane.lib.ane_absmax_partials_count(M * K, K * N_local)),
                                    dtype=torch.float32, device=device)
        self.Aq = torch.empty((M, K16), dtype=torch.int8, device=device)
        self.Bt = torch.empty((N_local, K16), dtype=torch.int8, device=device)
        self.scales = torch.empty(2, dtype=torch.float32, device=device)
        self.C_local = torch.empty((M, N_local), dtype=torch.float32, device=device)
        self.gathered = torch.empty((world, M, N_local), dtype=torch.float32, device=device)

    def forward(self, A, B_local, scale: float = 1.0, relu: bool = False, gather: bool = True):
        M, N_local, K = self.M, self.N_local, self.K
        s = ane._stream_ptr()
        ane.check(ane.lib.ane_absmax_pair_dev(A.data_ptr(), M * K, B_local.data_ptr(), K * N_local,
                                              self.absmax2.data_ptr(), self.partials.data_ptr(), s))
        if self.world > 1:
            dist.all_reduce(self.absmax2, op=dist.ReduceOp.MAX, group=self.group)
        ane.check(ane.lib.ane_quantize_pair_absmax_dev(M, N_local, K, A.data_ptr(), B_local.data_ptr(),
                                                       self.Aq.data_ptr(), self.Bt.data_ptr(),
                                                       self.absmax2.data_ptr(), self.scales.data_ptr(), s))
        ane.gemm_s8(self.Aq, self.Bt, self.scales, scale, relu, out=self.C_local)
        if not gather:
            return self.C_local
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.C_local, group=self.group)
        else:
            self.gathered[0].copy_(self.C_local)
        # [world, M, N_local] -> [M, world * N_local]
        return self.gathered.permute(1, 0, 2).reshape(M, self.world * N_local)

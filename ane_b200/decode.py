"""Q8_0 decode stack: a 7B-shaped stack of Q8_0 matvecs, N-sharded by rows.

Per layer four projections run back to back (ggml MUL_MAT at batch 1 with
Q8_0 weights, src/ggml-backend/ggml-ane.cpp:142-177), in one of two
arithmetics: mode "q" quantizes each matvec's activation to Q8_0 first (the
ggml CPU convention for Q8_0 weights); mode "r" keeps the
activation in fp32 and runs the reference's q8_0_gemv, as its ggml backend
does:

    QKV      12288 x 4096
    O         4096 x 4096
    gate+up  22016 x 4096
    down      4096 x 11008

Attention, norms and the SwiGLU product are outside the quantized hot path.
Every layer starts from its own seeded fp32 activation vector (norms would keep
a real stack's scale bounded; a raw chain of N(0, 0.02) projections grows ~4x
per layer and would overflow the fp16 block scales after ~10 layers); inside a
layer each projection consumes the first K entries of the previous one's output
(QKV -> O takes q, gate+up -> down takes the gate half), so the stack exercises
exactly the quantize / matvec / all-gather path with its true dependencies.

Sharding: every rank owns rows [r*M/world, (r+1)*M/world) of every weight
matrix and computes that slice of every output; the slices are all-gathered
into the full vector before the next projection.  Weight rows are generated
from per-64-row-block seeds, so the logical matrices -- and, since each output
row is computed the same way on any rank, the outputs -- do not depend on the
number of ranks.

`DecodeStack` takes its three steps (quantize, matvec, all-gather) as
callables: the GPU path binds them to libane_b200 and NCCL, the CPU tests bind
them to the oracle and gloo ranks.
"""
from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist

LAYER_SHAPES = (("qkv", 12288, 4096), ("o", 4096, 4096), ("gate_up", 22016, 4096), ("down", 4096, 11008))
ROW_BLOCK = 64
BLOCK_BYTES = 34  # Q8_0: fp16 d + 32 int8


def q8_row_bytes(K: int) -> int:
    return K // 32 * BLOCK_BYTES


def stack_weight_bytes(layers: int, shapes=LAYER_SHAPES) -> int:
    return layers * sum(M * q8_row_bytes(K) for _, M, K in shapes)


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    if M % world or (M // world) % ROW_BLOCK:
        raise ValueError(f"{M} rows do not split into {world} shards of whole {ROW_BLOCK}-row blocks")
    m = M // world
    return rank * m, (rank + 1) * m


def block_seed(seed: int, layer: int, proj: int, block: int) -> int:
    return (seed * 1_000_003 + layer * 10_007 + proj * 101 + block) & 0x7FFFFFFF


class DecodeStack:
    """Row-sharded stack of Q8_0 projections.

    quantize(x_fp32[K]) -> xq (K/32 Q8_0 blocks, uint8)
    matvec(W_local, xq, rows, K, out) -> out fp32[rows]
    gather(y_local, y_full) -> y_full fp32[M]  (not called when world == 1: the
        matvec then writes the full output directly)
    make_rows(layer, proj, block, K) -> uint8 [ROW_BLOCK * row_bytes]  (one block of weight rows)
    """

    def __init__(self, layers: int, world: int, rank: int, make_rows: Callable, quantize: Callable,
                 matvec: Callable, gather: Callable, shapes: Sequence = LAYER_SHAPES, alloc=None,
                 make_inputs: Callable | None = None, batch: int = 1, weights: list | None = None):
        self.layers, self.world, self.rank, self.batch = layers, world, rank, batch
        self.shapes = tuple(shapes)
        for (_, M_prev, _), (name, _, K) in zip(self.shapes, self.shapes[1:]):
            if K > M_prev:
                raise ValueError(f"projection {name} reads {K} entries of a {M_prev}-entry vector")
        self.quantize, self.matvec, self.gather = quantize, matvec, gather
        alloc = alloc or (lambda n, dtype: torch.empty(n, dtype=dtype))
        self.weights = weights if weights is not None else []  # reuse another stack's shards
        for layer in range(layers if weights is None else 0):
            ws = []
            for p, (_, M, K) in enumerate(self.shapes):
                r0, r1 = shard_rows(M, world, rank)
                rb = q8_row_bytes(K)
                W = alloc((r1 - r0) * rb, torch.uint8)
                for i, blk in enumerate(range(r0 // ROW_BLOCK, r1 // ROW_BLOCK)):
                    W[i * ROW_BLOCK * rb:(i + 1) * ROW_BLOCK * rb] = make_rows(layer, p, blk, K)
                ws.append(W)
            self.weights.append(ws)
        width = max(max(M, K) for _, M, K in self.shapes)
        k0 = self.shapes[0][2]
        if batch == 1:
            self.h = [alloc(width, torch.float32), alloc(width, torch.float32)]
            self.inputs = make_inputs(layers, k0) if make_inputs else torch.randn(layers, k0)  # per-layer x
            self.y_local = {M: alloc(M // world, torch.float32) for _, M, _ in self.shapes} if world > 1 else {}
        else:
            # token t is row t of every activation: h[i] is [batch, width], inputs [layers, batch, K]
            self.h = [alloc(batch * width, torch.float32).view(batch, width) for _ in range(2)]
            self.inputs = (make_inputs(layers * batch, k0) if make_inputs
                           else torch.randn(layers * batch, k0)).view(layers, batch, k0)
            self.y_local = ({M: alloc(batch * (M // world), torch.float32).view(batch, M // world)
                             for _, M, _ in self.shapes} if world > 1 else {})

    def forward(self, trace: list | None = None) -> torch.Tensor:
        """One step (one token, or `batch` tokens as rows) through every layer;
        returns the last projection's full output."""
        cur = 0
        for layer in range(self.layers):
            for p, (_, M, K) in enumerate(self.shapes):
                xin = self.inputs[layer] if p == 0 else self.h[cur][..., :K]
                xq = self.quantize(xin)
                out = self.h[1 - cur][..., :M]
                if self.world == 1:
                    self.matvec(self.weights[layer][p], xq, M, K, out)
                else:
                    y_loc = self.matvec(self.weights[layer][p], xq, M // self.world, K, self.y_local[M])
                    self.gather(y_loc, out)
                if trace is not None:
                    trace.append((layer, p, xin.clone(), out.clone()))
                cur = 1 - cur
        return self.h[cur][..., :self.shapes[-1][1]]


# ------------------------------------------------------------------ GPU binding
def gpu_stack(layers: int, device, world: int = 1, rank: int = 0, group=None, seed: int = 5,
              shapes: Sequence = LAYER_SHAPES, static_weights: bool = True, batch: int = 1,
              weights: list | None = None, first_layer: int = 0, mode: str = "q") -> DecodeStack:
    """DecodeStack on libane_b200 with an NCCL all-gather.  batch 1: one launch
    per projection (Q8_0 activation quantization fused into the Q8_0 x Q8_0
    matvec); batch > 1: the batched MUL_MAT (weights read once for all tokens).
    first_layer: the stack holds layers first_layer .. first_layer+layers-1 of
    the seeded model (same weights and inputs as those layers of a taller stack),
    so one GPU can recompute the last layer of a sharded run.
    mode "q": the activation is quantized to Q8_0 and multiplied block by block
    in int32 (ggml's CPU convention for Q8_0 weights); mode "r": the
    reference's own arithmetic -- q8_0_gemv on the fp32 activation
    (src/ggml-backend/ggml-ane.cpp:160-166 hands src1 to q8_0_gemv, whose
    handler keeps x in fp32, src/bytecode_interpreter.s:7010-7063), batch 1."""
    if mode not in ("q", "r"):
        raise ValueError("mode is 'q' (Q8_0 activation) or 'r' (fp32 activation, reference arithmetic)")
    if mode == "r" and batch != 1:
        raise ValueError("mode 'r' runs one token per step: the reference's MUL_MAT computes column 0 only")
    import ane_b200 as ane

    workspaces, gather_bufs = {}, {}

    def make_rows(layer, p, blk, K):
        g = torch.Generator(device=device).manual_seed(block_seed(seed, first_layer + layer, p, blk))
        w = torch.randn(ROW_BLOCK * K, device=device, generator=g) * 0.02
        return ane.quantize_q8_0(w)

    # the activation's Q8_0 quantization runs inside the matvec (ggml MUL_MAT at batch 1)
    def quantize(x):
        return x

    def matvec(W, x, rows, K, out):
        if mode == "r":
            return ane.q8_0_gemv(W, x, rows, K, out=out, static_weights=static_weights)
        if batch == 1:
            return ane.mul_mat_q8_0(W, x, rows, K, out=out, static_weights=static_weights)
        if (rows, K) not in workspaces:
            workspaces[(rows, K)] = ane.mul_mat_q8_0_batch_workspace(rows, K, device)
        return ane.mul_mat_q8_0_batch(W, x, rows, K, out=out, workspace=workspaces[(rows, K)],
                                      static_weights=static_weights)

    def gather(y_loc, y_full):
        if batch == 1:
            dist.all_gather_into_tensor(y_full, y_loc, group=group)
            return
        # [batch, m] slices -> [world, batch, m] -> token rows of [batch, world * m]
        m = y_loc.shape[1]
        if m not in gather_bufs:
            gather_bufs[m] = torch.empty(world * batch * m, dtype=torch.float32, device=device)
        buf = gather_bufs[m]
        dist.all_gather_into_tensor(buf, y_loc, group=group)
        y_full.copy_(buf.view(world, batch, m).permute(1, 0, 2).reshape(batch, world * m))

    def make_inputs(n, K):
        g = torch.Generator(device=device).manual_seed(seed + 17)
        skip = first_layer * batch  # rows of the layers below first_layer
        return torch.randn(skip + n, K, device=device, generator=g)[skip:]

    alloc = lambda n, dtype: torch.empty(n, dtype=dtype, device=device)  # noqa: E731
    return DecodeStack(layers, world, rank, make_rows, quantize, matvec, gather, shapes, alloc, make_inputs, batch,
                       weights)


# ------------------------------------------------- one persistent launch per token
class FusedDecodeStack:
    """The weights and inputs of a DecodeStack run as ONE persistent kernel per
    token (ane_q8_stack_*): weight streaming never stops between projections,
    and with world > 1 every CTA stores its output rows straight into every
    rank's activation vector (CUDA-IPC peer pointers over NVLink) -- the
    all-gather is part of the matvec.

    Activations are two ping-pong TAGGED vectors per rank (projection j writes
    vector j % 2; element = 8-byte {fp32 value, u32 tag} word) followed by two
    control words, all zero at creation and never reset.
    """

    def __init__(self, stack: DecodeStack, device, group=None):
        import ctypes

        import ane_b200 as ane

        self._ane = ane
        world, rank = stack.world, stack.rank
        self.nproj = stack.layers * len(stack.shapes)
        width = stack.h[0].numel()
        vec_bytes = width * 8
        ctl_off = 2 * vec_bytes
        self.block = torch.zeros(ctl_off + 64, dtype=torch.uint8, device=device)
        base = self.block.data_ptr()
        self._opened = []
        peer = [0] * world
        peer[rank] = base
        if world > 1:
            handle = (ctypes.c_uint8 * 64)()
            off = ctypes.c_uint64()
            ane.check(ane.lib.ane_ipc_get_handle(base, handle, ctypes.byref(off)))
            everyone = [None] * world
            dist.all_gather_object(everyone, (bytes(handle), off.value), group=group)
            for r in range(world):
                if r == rank:
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[r][0])
                b = ctypes.c_void_p()
                ane.check(ane.lib.ane_ipc_open_handle(h, ctypes.byref(b)))
                self._opened.append(b.value)
                peer[r] = b.value + everyone[r][1]
        projs = (ane.Q8StackProj * self.nproj)()
        j = 0
        for layer in range(stack.layers):
            for p, (_, M, K) in enumerate(stack.shapes):
                rows = M // world
                pr = projs[j]
                pr.W = stack.weights[layer][p].data_ptr()
                pr.rows_local = rows
                pr.K = K
                if p == 0:
                    pr.x, pr.x_tagged = stack.inputs[layer].data_ptr(), 0
                else:
                    pr.x, pr.x_tagged = base + ((j - 1) % 2) * vec_bytes, 1
                for r in range(world):
                    pr.out[r] = peer[r] + (j % 2) * vec_bytes + 8 * rank * rows
                pr.out_all = base + (j % 2) * vec_bytes
                j += 1
        self.plan = ctypes.c_void_p()
        ane.check(ane.lib.ane_q8_stack_plan_create(projs, self.nproj, world, rank, base + ctl_off,
                                                   ctypes.byref(self.plan)))
        words = self.block[:ctl_off].view(torch.float32).view(2, width, 2)
        self.out = words[(self.nproj - 1) % 2, :stack.shapes[-1][1], 0]  # values of the last output

    def forward(self, stream=None) -> torch.Tensor:
        self._ane.check(self._ane.lib.ane_q8_stack_run(self.plan, self._ane._stream_ptr(stream)))
        return self.out

    def close(self):
        if self.plan:
            self._ane.lib.ane_q8_stack_plan_free(self.plan)
            self.plan = None
        for b in self._opened:
            self._ane.lib.ane_ipc_close_handle(b)
        self._opened = []


# ------------------------------------------- per-projection launches, fused gather
class PeerChainDecodeStack:
    """The weights and inputs of a batch-1 DecodeStack run as one MUL_MAT
    launch per projection (mode q: ane_mul_mat_q8_0_gather_dev; mode r:
    ane_q8_0_gemv_gather_dev, the reference's q8_0_gemv arithmetic) whose rows
    go straight into every rank's next input vector over NVLink -- no NCCL
    call -- plus one token-end launch; the whole token captures into a CUDA
    graph.

    Per rank one zeroed buffer holds two TAGGED vectors (8-byte {fp32 value,
    u32 tag} words; projection j writes vector j % 2) and the token count; the
    other ranks' buffers are mapped with CUDA IPC.  Projection j reads the
    previous projection's vector: as its input x (when it chains), and always
    one guard word per (rank, CTA) of that projection, so a fast rank never
    overwrites a vector a slow one still reads.
    """

    def __init__(self, stack: DecodeStack, device, group=None, mode: str = "q"):
        """mode "q": each link is the Q8_0-activation MUL_MAT; mode "r": the
        reference's arithmetic, q8_0_gemv on the fp32 activation (an extra launch
        per projection writes the previous vector's values as fp32 first)."""
        import ctypes

        import ane_b200 as ane

        if stack.batch != 1:
            raise ValueError("the fused-gather chain runs one token per step")
        if mode not in ("q", "r"):
            raise ValueError("mode is 'q' or 'r'")
        self._ane, self.stack, self.mode = ane, stack, mode
        world, rank = stack.world, stack.rank
        width = stack.h[0].numel()
        vec_bytes = (width * 8 + 255) // 256 * 256
        tok_off = 2 * vec_bytes
        self.block = torch.zeros(tok_off + 256, dtype=torch.uint8, device=device)
        base = self.block.data_ptr()
        self._opened = []
        peer = [0] * world
        peer[rank] = base
        if world > 1:
            handle = (ctypes.c_uint8 * 64)()
            off = ctypes.c_uint64()
            ane.check(ane.lib.ane_ipc_get_handle(base, handle, ctypes.byref(off)))
            everyone = [None] * world
            dist.all_gather_object(everyone, (bytes(handle), off.value), group=group)
            for r in range(world):
                if r == rank:
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[r][0])
                b = ctypes.c_void_p()
                ane.check(ane.lib.ane_ipc_open_handle(h, ctypes.byref(b)))
                self._opened.append(b.value)
                peer[r] = b.value + everyone[r][1]
        self._tok = base + tok_off
        projs = [(layer, p, M, K) for layer in range(stack.layers) for p, (_, M, K) in enumerate(stack.shapes)]
        self.nproj = len(projs)
        split = [(M // world, int(ane.lib.ane_mul_mat_q8_0_ctas(M // world, K))) for _, _, M, K in projs]
        # mode r: the fp32 input of a chained projection, written from the tagged vector
        self._xbuf = torch.empty(max(K for _, _, _, K in projs), dtype=torch.float32, device=device)
        self._calls = []
        for j, (layer, p, M, K) in enumerate(projs):
            rows = M // world
            jp = (j - 1) % self.nproj  # the previous projection (of the previous token for j = 0)
            prev = base + (jp % 2) * vec_bytes
            chained = p != 0
            x = 0 if chained else stack.inputs[layer].data_ptr()
            outs = (ctypes.c_void_p * world)(*[q + (j % 2) * vec_bytes + 8 * rank * rows for q in peer])
            self._calls.append((rows, K, x, stack.weights[layer][p].data_ptr(), outs, prev, int(chained),
                                split[jp][0], split[jp][1], j))
        last_M = stack.shapes[-1][1]
        self._last = base + ((self.nproj - 1) % 2) * vec_bytes
        self._last_len = last_M
        words = self.block[:tok_off].view(torch.float32).view(2, vec_bytes // 8, 2)
        self.out = words[(self.nproj - 1) % 2, :last_M, 0]  # values of the last output

    def forward(self, stream=None) -> torch.Tensor:
        ane, world = self._ane, self.stack.world
        s = ane._stream_ptr(stream)
        if self.mode == "r":
            xbuf = self._xbuf.data_ptr()
            for rows, K, x, W, outs, prev, chained, prev_rows, _, j in self._calls:
                ane.check(ane.lib.ane_q8_0_gemv_gather_dev(rows, K, x or None, xbuf, W, world, outs, prev, chained,
                                                           prev_rows, self._tok, self.nproj, j, ane.WEIGHTS_STATIC,
                                                           s))
        else:
            for rows, K, x, W, outs, prev, chained, prev_rows, prev_ctas, j in self._calls:
                ane.check(ane.lib.ane_mul_mat_q8_0_gather_dev(rows, K, x or None, W, world, outs, prev, chained,
                                                              prev_rows, prev_ctas, self._tok, self.nproj, j,
                                                              ane.WEIGHTS_STATIC, s))
        ane.check(ane.lib.ane_q8_chain_token_end_dev(self._last, self._last_len, self.nproj, self._tok, s))
        return self.out

    def close(self):
        for b in self._opened:
            self._ane.lib.ane_ipc_close_handle(b)
        self._opened = []


# ------------------------------------------- batch > 1: the same chain, batched
class PeerBatchDecodeStack:
    """The weights and inputs of a batch-NT (NT <= 16) mode-Q DecodeStack run
    as one batched MUL_MAT per projection (ane_mul_mat_q8_0_batch_gather_dev:
    the activation quantize launch and the GEMM launch) whose outputs go
    straight into every rank's next vector over NVLink -- no NCCL call -- plus
    one step-end launch; the whole step captures into a CUDA graph.

    Per rank one zeroed buffer holds two TAGGED vectors of NT token rows
    (8-byte {fp32 value, u32 tag} words, row stride ldw; projection j writes
    vector j % 2) and the step count; the other ranks' buffers are mapped with
    CUDA IPC.  Each projection also waits for one word per rank of the
    previous projection, so a fast rank never overwrites a vector a slow one
    still reads.
    """

    def __init__(self, stack: DecodeStack, device, group=None):
        import ctypes

        import ane_b200 as ane

        if stack.batch == 1:
            raise ValueError("batch 1 runs as PeerChainDecodeStack or FusedDecodeStack")
        self._ane, self.stack = ane, stack
        world, rank, NT = stack.world, stack.rank, stack.batch
        ldw = (stack.h[0].shape[1] + 1) // 2 * 2
        vec_bytes = (NT * ldw * 8 + 255) // 256 * 256
        tok_off = 2 * vec_bytes
        self.block = torch.zeros(tok_off + 256, dtype=torch.uint8, device=device)
        base = self.block.data_ptr()
        self._opened = []
        peer = [0] * world
        peer[rank] = base
        if world > 1:
            handle = (ctypes.c_uint8 * 64)()
            off = ctypes.c_uint64()
            ane.check(ane.lib.ane_ipc_get_handle(base, handle, ctypes.byref(off)))
            everyone = [None] * world
            dist.all_gather_object(everyone, (bytes(handle), off.value), group=group)
            for r in range(world):
                if r == rank:
                    continue
                h = (ctypes.c_uint8 * 64).from_buffer_copy(everyone[r][0])
                b = ctypes.c_void_p()
                ane.check(ane.lib.ane_ipc_open_handle(h, ctypes.byref(b)))
                self._opened.append(b.value)
                peer[r] = b.value + everyone[r][1]
        self._tok = base + tok_off
        projs = [(layer, p, M, K) for layer in range(stack.layers) for p, (_, M, K) in enumerate(stack.shapes)]
        self.nproj = len(projs)
        self._ws = {}
        self._calls = []
        for j, (layer, p, M, K) in enumerate(projs):
            rows = M // world
            jp = (j - 1) % self.nproj  # the previous projection (of the previous step for j = 0)
            prev = base + (jp % 2) * vec_bytes
            chained = p != 0
            x = stack.inputs[layer]
            if (rows, K) not in self._ws:
                self._ws[(rows, K)] = ane.mul_mat_q8_0_batch_workspace(rows, K, device)
            outs = (ctypes.c_void_p * world)(*[q + (j % 2) * vec_bytes + 8 * rank * rows for q in peer])
            self._calls.append((rows, K, 0 if chained else x.data_ptr(), x.stride(0), stack.weights[layer][p].data_ptr(),
                                self._ws[(rows, K)].data_ptr(), outs, prev, int(chained), projs[jp][2] // world, j))
        self._ldw, self._NT = ldw, NT
        last_M = stack.shapes[-1][1]
        self._last = base + ((self.nproj - 1) % 2) * vec_bytes
        self._last_rows = last_M
        words = self.block[:tok_off].view(torch.float32).view(2, vec_bytes // 8, 2)
        # values of the last output, [NT, last_M]
        self.out = words[(self.nproj - 1) % 2, :NT * ldw, 0].view(NT, ldw)[:, :last_M]

    def forward(self, stream=None) -> torch.Tensor:
        ane, world = self._ane, self.stack.world
        s = ane._stream_ptr(stream)
        for rows, K, x, ldx, W, ws, outs, prev, chained, prev_rows, j in self._calls:
            ane.check(ane.lib.ane_mul_mat_q8_0_batch_gather_dev(rows, K, self._NT, x or None, ldx, W, ws, world, outs,
                                                                self._ldw, prev, chained, prev_rows, self._tok,
                                                                self.nproj, j, ane.WEIGHTS_STATIC, s))
        ane.check(ane.lib.ane_q8_batch_step_end_dev(self._last, self._last_rows, self._ldw, self._NT, self.nproj,
                                                    self._tok, s))
        return self.out

    def close(self):
        for b in self._opened:
            self._ane.lib.ane_ipc_close_handle(b)
        self._opened = []

"""ane_b200 -- B200 (sm_100a) implementation of ane's quantized dense hot path.

The product is ``ane_b200/_lib/libane_b200.so``: hand-written CUDA kernels
behind the C ABI declared in ``include/ane_b200.h``.  This Python module is a
thin ctypes binding over that ABI, used by the tests, the benchmark and the
multi-GPU driver.  It never computes anything itself: if the library is
missing, importing the module raises, and there is no CPU fallback.

Mirrors of the reference's interface (joshmorgan1000/ane):

* ``Op`` -- the opcode enum of include/ane/ane.hpp:47-177, plus
  ``dense_fused_i8 = 0x80`` (README.md:87-97).
* ``dispatch(op, *args)`` -- packs arguments by size with no padding, exactly as
  ``ane::dispatch`` (include/ane/ane.hpp:206-220), then calls ``stream_exec``.
* ``Program`` -- multi-op byte stream like ``ane::program`` (ane.hpp:229-352).
"""
from __future__ import annotations

import ctypes
import enum
import os
import struct

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libane_b200.so")
ROOT = os.path.dirname(_HERE)
INCLUDE_DIR = os.path.join(ROOT, "include")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"ane_b200: native library {LIB_PATH} is missing; build it with "
        "`make -C ane_b200/csrc` (or __graft_entry__.build()). There is no CPU fallback.")

_lib = ctypes.CDLL(LIB_PATH)

_u8, _u32, _i32, _f, _sz, _vp, _u64 = (ctypes.c_uint8, ctypes.c_uint32, ctypes.c_int, ctypes.c_float,
                                       ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint64)

# name -> (restype, argtypes); every symbol declared in include/ane_b200.h
SIGNATURES = {
    "ane_last_error": (_i32, []),
    "ane_last_error_string": (ctypes.c_char_p, []),
    "ane_clear_error": (None, []),
    "ane_version": (ctypes.c_char_p, []),
    "ane_opcode_supported": (_i32, [_u8]),
    "ane_opcode_payload_size": (_i32, [_u8]),
    "stream_exec": (None, [_vp, _sz]),
    "ane_quantize_fp32_i8": (_i32, [_u32, _vp, _vp, _vp]),
    "ane_dequantize_i8_fp32": (_i32, [_u32, _f, _vp, _vp]),
    "ane_pack_b_i8": (_i32, [_u32, _u32, _vp, _vp]),
    "ane_quantize_fp32_i8_channelwise": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_dense_i8": (_i32, [_u32, _u32, _u32, _f, _f, _u8, _vp, _vp, _vp, _vp]),
    "ane_dense_u8s8": (_i32, [_u32, _u32, _u32, _f, _f, _u8, _vp, _vp, _vp, _vp]),
    "ane_get_rows_q8_0": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_q4_0_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_get_rows_q4_0": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_q4_k_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_q2_k_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_q3_k_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_q5_k_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_q6_k_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_elementwise_scaled_add_fp32": (_i32, [_u32, _f, _vp, _vp, _vp]),
    "ane_relu_backward_fp32": (_i32, [_u32, _vp, _vp, _vp]),
    "ane_transpose_fp32": (_i32, [_u32, _u32, _vp, _vp]),
    "ane_softmax_argmax_fp32": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp, _vp]),
    "ane_dense_fp32": (_i32, [_u32, _u32, _u32, _f, _u8, _vp, _vp, _vp, _vp]),
    "ane_count_matches": (_i32, [_u32, _vp, _vp, _vp]),
    "ane_elementwise_scaled_add_fp32_dev": (_i32, [_u32, _f, _vp, _vp, _vp, _vp]),
    "ane_relu_backward_fp32_dev": (_i32, [_u32, _vp, _vp, _vp, _vp]),
    "ane_transpose_fp32_dev": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_count_matches_dev": (_i32, [_u32, _vp, _vp, _vp, _vp]),
    "ane_dense_fp32_dev": (_i32, [_u32, _u32, _u32, _f, _u8, _vp, _vp, _vp, _vp, _vp]),
    "ane_softmax_argmax_fp32_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ane_q4_0_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_q4_0_gemv_ex_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _u32, _vp]),
    "ane_get_rows_q8_0_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_get_rows_q4_0_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_q4_k_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_q2_k_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_q3_k_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_q5_k_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_q6_k_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_kquant_gemv_ex_dev": (_i32, [_u8, _u32, _u32, _vp, _vp, _vp, _u32, _vp]),
    "ane_cblas_igemm": (_i32, [_u8, _u32, _u32, _u32, _u32, _u32, _u32, _f, _f, _vp, _vp, _vp]),
    "ane_cblas_ugemm": (_i32, [_u8, _u32, _u32, _u32, _u32, _u32, _u32, _f, _f, _vp, _vp, _vp]),
    "ane_cblas_usgemm": (_i32, [_u8, _u32, _u32, _u32, _u32, _u32, _u32, _f, _f, _vp, _vp, _vp]),
    "ane_dense_fused_i8": (_i32, [_u32, _u32, _u32, _f, _u8, _vp, _vp, _vp]),
    "ane_q8_0_gemv": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_dense_fused_i8_workspace_size": (_sz, [_u32, _u32, _u32]),
    "ane_dense_fused_i8_dev": (_i32, [_u32, _u32, _u32, _f, _u8, _vp, _vp, _vp, _vp, _sz, _vp]),
    "ane_dense_fused_i8_noalloc_dev": (_i32, [_u32, _u32, _u32, _f, _u8, _vp, _vp, _vp, _vp]),
    "ane_absmax_partials_count": (_sz, [_sz, _sz]),
    "ane_quantize_pair_dev": (_i32, [_u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ane_absmax_pair_dev": (_i32, [_vp, _sz, _vp, _sz, _vp, _vp, _vp]),
    "ane_quantize_pair_absmax_dev": (_i32, [_u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "ane_gemm_s8_dev": (_i32, [_u32, _u32, _u32, _vp, _vp, _vp, _f, _u8, _i32, _vp, _vp]),
    "ane_gemm_s8_kn_dev": (_i32, [_u32, _u32, _u32, _vp, _vp, _u32, _vp, _f, _u8, _i32, _vp, _vp]),
    "ane_quantize_fp32_i8_dev": (_i32, [_u32, _vp, _vp, _vp, _vp]),
    "ane_pack_b_i8_dev": (_i32, [_u32, _u32, _vp, _vp, _vp]),
    "ane_dense_i8_dev": (_i32, [_u32, _u32, _u32, _f, _f, _u8, _vp, _vp, _vp, _vp, _vp]),
    "ane_dense_u8s8_dev": (_i32, [_u32, _u32, _u32, _f, _f, _u8, _vp, _vp, _vp, _vp, _vp]),
    "ane_cblas_int_gemm_dev": (_i32, [_i32, _u8, _u32, _u32, _u32, _u32, _u32, _u32, _f, _f, _vp, _vp, _vp, _vp]),
    "ane_q8_0_gemv_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp]),
    "ane_quantize_q8_0_dev": (_i32, [_u32, _vp, _vp, _vp]),
    "ane_q8_0_gemv_q8_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp, _vp]),
    "ane_q8_0_gemv_ex_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _u32, _vp]),
    "ane_q8_0_gemv_q8_ex_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp, _u32, _vp]),
    "ane_mul_mat_q8_0_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _vp, _u32, _vp]),
    "ane_mul_mat_q8_0_batch_workspace_size": (_sz, [_u32, _u32]),
    "ane_mul_mat_q8_0_ctas": (_u32, [_u32, _u32]),
    "ane_mul_mat_q8_0_gather_dev": (_i32, [_u32, _u32, _vp, _vp, _u32, _vp, _vp, _u32, _u32, _u32, _vp, _u32, _u32,
                                           _u32, _vp]),
    "ane_q8_chain_token_end_dev": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "ane_q8_0_gemv_gather_dev": (_i32, [_u32, _u32, _vp, _vp, _vp, _u32, _vp, _vp, _u32, _u32, _vp, _u32, _u32, _u32,
                                        _vp]),
    "ane_mul_mat_q8_0_batch_dev": (_i32, [_u32, _u32, _u32, _vp, _sz, _vp, _vp, _sz, _vp, _u32, _vp]),
    "ane_mul_mat_q8_0_batch_gather_dev": (_i32, [_u32, _u32, _u32, _vp, _sz, _vp, _vp, _u32, _vp, _sz, _vp, _u32,
                                                 _u32, _vp, _u32, _u32, _u32, _vp]),
    "ane_q8_batch_step_end_dev": (_i32, [_vp, _u32, _sz, _u32, _u32, _vp, _vp]),
    "ane_q8_stack_plan_create": (_i32, [_vp, _u32, _u32, _u32, _vp, _vp]),
    "ane_q8_stack_run": (_i32, [_vp, _vp]),
    "ane_q8_stack_plan_free": (None, [_vp]),
    "ane_quantize_pair_xrank_dev": (_i32, [_u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _vp, _vp,
                                           _vp, _vp]),
    "ane_gemm_s8_gather_dev": (_i32, [_u32, _u32, _u32, _vp, _vp, _vp, _f, _u8, _u32, _u32, _vp, _u32, _vp, _vp,
                                      _vp]),
    "ane_ipc_get_handle": (_i32, [_vp, _vp, _vp]),
    "ane_ipc_open_handle": (_i32, [_vp, _vp]),
    "ane_ipc_close_handle": (_i32, [_vp]),
    "ane_device_timeouts": (_i32, []),
    "ane_kernel_launch_count": (_u64, []),
}
for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(_lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

lib = _lib


class AneError(RuntimeError):
    """A libane_b200 call returned a non-zero ane_status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ane_status {code}: {msg}")
        self.code = code


STATUS = {0: "ANE_OK", 1: "ANE_ERR_INVALID_ARGUMENT", 2: "ANE_ERR_UNSUPPORTED_OPCODE",
          3: "ANE_ERR_TRUNCATED_STREAM", 4: "ANE_ERR_CUDA", 5: "ANE_ERR_NO_DEVICE",
          6: "ANE_ERR_OUT_OF_MEMORY", 7: "ANE_ERR_DEVICE_TIMEOUT"}


def check(rc: int) -> None:
    if rc != 0:
        raise AneError(rc, (_lib.ane_last_error_string() or b"").decode())


def last_error() -> int:
    return _lib.ane_last_error()


def launch_count() -> int:
    """Kernel launches issued by libane_b200 in this process."""
    return int(_lib.ane_kernel_launch_count())


# ----------------------------------------------------------------- opcodes
class Op(enum.IntEnum):
    """Opcode values of the reference (include/ane/ane.hpp:47-177) + dense_fused_i8."""
    reserved_0x00 = 0x00
    elementwise_scaled_add_fp32 = 0x0D
    relu_backward_fp32 = 0x0F
    transpose_fp32 = 0x11
    softmax_argmax_fp32 = 0x12
    dense_fp32 = 0x15
    count_matches = 0x16
    dense_i8 = 0x18
    quantize_fp32_i8 = 0x19
    dequantize_i8_fp32 = 0x1A
    pack_b_i8 = 0x1B
    quantize_fp32_i8_channelwise = 0x1C
    transpose_i8 = 0x1D
    dense_u8s8 = 0x1E
    q8_0_gemv = 0x57
    q4_0_gemv = 0x58
    cblas_igemm = 0x61
    cblas_ugemm = 0x62
    cblas_usgemm = 0x63
    q4_k_gemv = 0x75
    q2_k_gemv = 0x76
    q3_k_gemv = 0x77
    q5_k_gemv = 0x78
    q6_k_gemv = 0x79
    get_rows_q8_0 = 0x7C
    get_rows_q4_0 = 0x7D
    dense_fused_i8 = 0x80


class U8(int):
    """1-byte immediate (uint8_t / bool in ane::dispatch)."""


class U32(int):
    """4-byte unsigned immediate (uint32_t / int)."""


class I32(int):
    """4-byte signed immediate."""


class F32(float):
    """4-byte float immediate."""


class Ptr(int):
    """8-byte pointer operand."""


def _pack(arg) -> bytes:
    if isinstance(arg, bool):
        return struct.pack("<B", int(arg))
    if isinstance(arg, U8):
        return struct.pack("<B", int(arg) & 0xFF)
    if isinstance(arg, U32):
        return struct.pack("<I", int(arg) & 0xFFFFFFFF)
    if isinstance(arg, I32):
        return struct.pack("<i", int(arg))
    if isinstance(arg, F32):
        return struct.pack("<f", float(arg))
    if isinstance(arg, Ptr):
        return struct.pack("<Q", int(arg))
    raise TypeError(f"dispatch argument {arg!r} needs an explicit width (U8/U32/I32/F32/Ptr)")


def encode(op: int, *args) -> bytes:
    """Byte encoding of one opcode, identical to ane::dispatch's stack buffer."""
    return bytes([int(op)]) + b"".join(_pack(a) for a in args)


def stream_exec(data: bytes) -> None:
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    _lib.stream_exec(buf, len(data))
    check(_lib.ane_last_error())


def dispatch(op: int, *args) -> None:
    """ane::dispatch: encode one opcode and run it through stream_exec."""
    stream_exec(encode(op, *args))


class Program:
    """ane::program: accumulate several opcodes and run them in one stream_exec."""

    def __init__(self):
        self._bytes = bytearray()

    def emit(self, op: int, *args) -> "Program":
        self._bytes += encode(op, *args)
        return self

    def exec(self) -> None:
        if self._bytes:
            stream_exec(bytes(self._bytes))

    def clear(self) -> None:
        self._bytes.clear()

    def size(self) -> int:
        return len(self._bytes)


# ------------------------------------------------- torch-tensor conveniences
def _torch():
    import torch  # plumbing only: device memory and streams

    return torch


def _stream_ptr(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def dense_fused_i8(A, B, scale: float = 1.0, relu: bool = False, out=None, workspace=None, stream=None):
    """C = dense_fused_i8(A, B) on CUDA fp32 tensors (A: M x K, B: K x N)."""
    torch = _torch()
    M, K = A.shape
    K2, N = B.shape
    assert K == K2 and A.is_cuda and B.is_cuda
    A = A.contiguous()
    B = B.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    ws_ptr, ws_bytes = (0, 0) if workspace is None else (workspace.data_ptr(), workspace.numel())
    check(_lib.ane_dense_fused_i8_dev(M, N, K, float(scale), int(bool(relu)), A.data_ptr(), B.data_ptr(),
                                      out.data_ptr(), ws_ptr or None, ws_bytes, _stream_ptr(stream)))
    return out


def dense_fused_i8_workspace(M: int, N: int, K: int, device="cuda"):
    torch = _torch()
    return torch.empty(int(_lib.ane_dense_fused_i8_workspace_size(M, N, K)), dtype=torch.uint8, device=device)


def quantize_pair(A, B, stream=None):
    """Stage 1 of dense_fused_i8: returns (Aq [M x K16], Bq [K16 x N16], scales[2]).

    Bq holds the codes of B in B's own layout (row k = codes of B[k, :], pad
    columns zero); its rows K..K16-1 are not written (they meet Aq's zero pad
    columns in the GEMM)."""
    torch = _torch()
    M, K = A.shape
    N = B.shape[1]
    K16 = (K + 15) // 16 * 16
    N16 = (N + 15) // 16 * 16
    Aq = torch.empty((M, K16), dtype=torch.int8, device=A.device)
    Bq = torch.empty((K16, N16), dtype=torch.int8, device=A.device)
    scales = torch.empty(2, dtype=torch.float32, device=A.device)
    partials = torch.empty(int(_lib.ane_absmax_partials_count(M * K, K * N)), dtype=torch.float32, device=A.device)
    check(_lib.ane_quantize_pair_dev(M, N, K, A.contiguous().data_ptr(), B.contiguous().data_ptr(), Aq.data_ptr(),
                                     Bq.data_ptr(), scales.data_ptr(), partials.data_ptr(), _stream_ptr(stream)))
    return Aq, Bq, scales


INT_GEMM_KINDS = {"igemm": 0, "ugemm": 1, "usgemm": 2}


def cblas_int_gemm(kind: str, A, B, C, M: int, N: int, K: int, lda: int, ldb: int, ldc: int, alpha: float = 1.0,
                   beta: float = 0.0, trans_a: bool = False, trans_b: bool = False, stream=None):
    """cblas_igemm / ugemm / usgemm on device tensors (byte strides lda / ldb, ldc
    in floats): C = alpha * cvt(op(A) @ op(B)) [beta: see ane_cblas_igemm]."""
    flags = (1 if trans_a else 0) | (2 if trans_b else 0)
    check(_lib.ane_cblas_int_gemm_dev(INT_GEMM_KINDS[kind], flags, M, N, K, lda, ldb, ldc, float(alpha), float(beta),
                                      A.data_ptr(), B.data_ptr(), C.data_ptr(), _stream_ptr(stream)))
    return C


def gemm_s8(Aq, Bt, scales=None, scale: float = 1.0, relu: bool = False, raw_i32: bool = False, out=None,
            stream=None):
    """Tensor-core int8 GEMM on resident operands: Aq [M x K16], Bt [N x K16] (K-major)."""
    torch = _torch()
    M, K16 = Aq.shape
    N = Bt.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.int32 if raw_i32 else torch.float32, device=Aq.device)
    check(_lib.ane_gemm_s8_dev(M, N, K16, Aq.data_ptr(), Bt.data_ptr(),
                               scales.data_ptr() if scales is not None else None, float(scale), int(bool(relu)),
                               1 if raw_i32 else 0, out.data_ptr(), _stream_ptr(stream)))
    return out


def gemm_s8_kn(Aq, Bq, N: int, scales=None, scale: float = 1.0, relu: bool = False, raw_i32: bool = False,
               out=None, stream=None):
    """Tensor-core int8 GEMM with B stored K x N: Aq [M x K16], Bq [K16 x ldb] (the
    layout quantize_pair returns), N <= ldb output columns."""
    torch = _torch()
    M, K16 = Aq.shape
    assert Bq.shape[0] >= K16 and Bq.shape[1] >= N
    if out is None:
        out = torch.empty((M, N), dtype=torch.int32 if raw_i32 else torch.float32, device=Aq.device)
    check(_lib.ane_gemm_s8_kn_dev(M, N, K16, Aq.data_ptr(), Bq.data_ptr(), Bq.stride(0),
                                  scales.data_ptr() if scales is not None else None, float(scale), int(bool(relu)),
                                  1 if raw_i32 else 0, out.data_ptr(), _stream_ptr(stream)))
    return out


def quantize_q8_0(x, out=None, stream=None):
    """fp32 x[K] -> K/32 Q8_0 blocks (uint8 tensor of K/32*34 bytes)."""
    torch = _torch()
    K = x.numel()
    if out is None:
        out = torch.empty(K // 32 * 34, dtype=torch.uint8, device=x.device)
    check(_lib.ane_quantize_q8_0_dev(K, x.data_ptr(), out.data_ptr(), _stream_ptr(stream)))
    return out


WEIGHTS_STATIC = 1  # ANE_Q8_WEIGHTS_STATIC: W is not written by the kernel just before the call


class Q8StackProj(ctypes.Structure):
    """ane_q8_stack_proj (include/ane_b200.h)."""
    _fields_ = [("W", ctypes.c_void_p), ("rows_local", ctypes.c_uint32), ("K", ctypes.c_uint32),
                ("x", ctypes.c_void_p), ("x_tagged", ctypes.c_uint32), ("out", ctypes.c_void_p * 8),
                ("out_all", ctypes.c_void_p)]


def q8_0_gemv_q8(W, xq, M: int, K: int, out=None, block_dots=None, stream=None, static_weights=False):
    """Q8_0 weights x Q8_0 activation blocks -> fp32 out[M] (optionally the int32 block dots).

    static_weights promises that W was not written by the kernel queued just
    before this call, so the kernel may start streaming W early."""
    torch = _torch()
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=W.device)
    check(_lib.ane_q8_0_gemv_q8_ex_dev(M, K, xq.data_ptr(), W.data_ptr(), out.data_ptr(),
                                       block_dots.data_ptr() if block_dots is not None else None,
                                       WEIGHTS_STATIC if static_weights else 0, _stream_ptr(stream)))
    return out


def mul_mat_q8_0(W, x, M: int, K: int, out=None, block_dots=None, stream=None, static_weights=False):
    """ggml MUL_MAT at batch 1: fp32 x[K] quantized to Q8_0 inside the Q8_0 x Q8_0 matvec."""
    torch = _torch()
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=W.device)
    check(_lib.ane_mul_mat_q8_0_dev(M, K, x.data_ptr(), W.data_ptr(), out.data_ptr(),
                                    block_dots.data_ptr() if block_dots is not None else None,
                                    WEIGHTS_STATIC if static_weights else 0, _stream_ptr(stream)))
    return out


def mul_mat_q8_0_batch_workspace(M: int, K: int, device):
    """Workspace for mul_mat_q8_0_batch: the quantized activation (reusable by calls on one stream)."""
    torch = _torch()
    n = int(_lib.ane_mul_mat_q8_0_batch_workspace_size(M, K))
    return torch.zeros(n, dtype=torch.uint8, device=device)


def mul_mat_q8_0_batch(W, x, M: int, K: int, out=None, workspace=None, stream=None, static_weights=False):
    """ggml MUL_MAT for NT <= 16 fp32 activation rows x [NT, K] (row stride
    x.stride(0)) against Q8_0 weights W: out [NT, M] (row stride out.stride(0))."""
    torch = _torch()
    NT = x.shape[0]
    assert x.dim() == 2 and x.shape[1] == K and x.stride(1) == 1
    if out is None:
        out = torch.empty((NT, M), dtype=torch.float32, device=W.device)
    assert out.dim() == 2 and out.shape == (NT, M) and out.stride(1) == 1
    if workspace is None:
        workspace = mul_mat_q8_0_batch_workspace(M, K, W.device)
    check(_lib.ane_mul_mat_q8_0_batch_dev(M, K, NT, x.data_ptr(), x.stride(0), W.data_ptr(), out.data_ptr(),
                                          out.stride(0), workspace.data_ptr(), WEIGHTS_STATIC if static_weights else 0,
                                          _stream_ptr(stream)))
    return out


def q4_0_gemv(W, x, M: int, K: int, out=None, stream=None, static_weights=False):
    """out[M] = Q4_0 matrix W (M rows of K/32 18-byte blocks, uint8 tensor) times fp32 x[K]."""
    torch = _torch()
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    check(_lib.ane_q4_0_gemv_ex_dev(M, K, x.data_ptr(), W.data_ptr(), out.data_ptr(),
                                    WEIGHTS_STATIC if static_weights else 0, _stream_ptr(stream)))
    return out


# K-quant super-block sizes (bytes per 256 weights), by format name
KQUANT_BLOCK_BYTES = {"q2_k": 84, "q3_k": 110, "q4_k": 144, "q5_k": 176, "q6_k": 210}


KQUANT_OPCODES = {"q4_k": 0x75, "q2_k": 0x76, "q3_k": 0x77, "q5_k": 0x78, "q6_k": 0x79}


def kquant_gemv(fmt: str, W, x, M: int, K: int, out=None, stream=None, static_weights=False):
    """out[M] = K-quant matrix W (M rows of K/256 super-blocks of format `fmt`,
    a key of KQUANT_BLOCK_BYTES; uint8 tensor) times fp32 x[K].
    static_weights: W is not written by the kernel before this call on the
    stream, so the matvec may start reading it early (ANE_Q8_WEIGHTS_STATIC)."""
    torch = _torch()
    if fmt not in KQUANT_BLOCK_BYTES:
        raise ValueError("unknown K-quant format %r" % (fmt,))
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    if static_weights:
        check(_lib.ane_kquant_gemv_ex_dev(KQUANT_OPCODES[fmt], M, K, x.data_ptr(), W.data_ptr(), out.data_ptr(),
                                          WEIGHTS_STATIC, _stream_ptr(stream)))
        return out
    fn = getattr(_lib, "ane_%s_gemv_dev" % fmt)
    check(fn(M, K, x.data_ptr(), W.data_ptr(), out.data_ptr(), _stream_ptr(stream)))
    return out


def get_rows_q4_0(table, indices, dim: int, out=None, stream=None):
    """Rows `indices` (uint32/int32 tensor) of a Q4_0 table, dequantized: out [n, dim]."""
    torch = _torch()
    n = indices.numel()
    if out is None:
        out = torch.empty((n, dim), dtype=torch.float32, device=table.device)
    check(_lib.ane_get_rows_q4_0_dev(n, dim, table.data_ptr(), indices.data_ptr(), out.data_ptr(),
                                     _stream_ptr(stream)))
    return out


def q8_0_gemv(W, x, M: int, K: int, out=None, stream=None, static_weights=False):
    """out[M] = Q8_0 matrix W (M rows of K/32 34-byte blocks, uint8 tensor) times fp32 x[K]."""
    torch = _torch()
    if out is None:
        out = torch.empty(M, dtype=torch.float32, device=x.device)
    check(_lib.ane_q8_0_gemv_ex_dev(M, K, x.data_ptr(), W.data_ptr(), out.data_ptr(),
                                    WEIGHTS_STATIC if static_weights else 0, _stream_ptr(stream)))
    return out

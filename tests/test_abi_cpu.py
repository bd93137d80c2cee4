"""CPU-side checks of the C ABI boundary (no GPU needed, no compute calls).

* libane_b200.so loads and exports every function include/ane_b200.h declares;
* the Python `encode` packs opcodes byte-for-byte like ane::dispatch
  (include/ane/ane.hpp:206-220) -- payload sizes of the hot-path opcodes;
* stream_exec rejects unsupported opcodes and truncated payloads before any
  device work, and a supported opcode without a GPU fails loudly (no fallback).
"""
import os
import re
import struct

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "ane_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\([^;{]*\)\s*;", text)
    return sorted(set(n for n in names if n not in ("if", "while", "for", "return")))


def test_library_exports_every_declared_symbol():
    import ane_b200

    names = header_functions()
    assert "stream_exec" in names and "ane_dense_fused_i8" in names and "ane_q8_0_gemv" in names
    for n in names:
        assert hasattr(ane_b200.lib, n), f"{n} declared in include/ane_b200.h but not exported"
        assert n in ane_b200.SIGNATURES, f"{n} has no ctypes signature"


def test_encoding_sizes_match_reference_dispatch():
    from ane_b200 import F32, U8, U32, Op, Ptr, encode

    # README.md:87-97 dense_fused_i8 call: int M,N,K, float scale, bool relu, 3 pointers
    b = encode(Op.dense_fused_i8, U32(50), U32(128), U32(784), F32(1.0), True, Ptr(1), Ptr(2), Ptr(3))
    assert len(b) == 42
    assert b[0] == 0x80 and struct.unpack_from("<IIIf?QQQ", b, 1) == (50, 128, 784, 1.0, True, 1, 2, 3)
    # tests/test_mnist_i8.cpp:309-314 dense_i8 call
    b = encode(Op.dense_i8, U32(50), U32(16), U32(128), F32(0.5), F32(0.25), False, Ptr(1), Ptr(2), Ptr(3), Ptr(4))
    assert len(b) == 54
    assert len(encode(Op.q8_0_gemv, U32(4096), U32(4096), Ptr(1), Ptr(2), Ptr(3))) == 33
    assert len(encode(Op.quantize_fp32_i8, U32(256), Ptr(1), Ptr(2), Ptr(3))) == 29
    assert len(encode(Op.pack_b_i8, U32(832), U32(128), Ptr(1), Ptr(2))) == 25
    with pytest.raises(TypeError):
        encode(Op.q8_0_gemv, 4096)  # widths must be explicit, like C++ types


def test_payload_size_table_matches_encoding():
    import ane_b200

    L = ane_b200.lib
    for op, n in [(0x18, 53), (0x19, 28), (0x1A, 24), (0x1B, 24), (0x1C, 32), (0x57, 32), (0x80, 41),
                  (0x1E, 53), (0x58, 32), (0x61, 57), (0x62, 57), (0x63, 57), (0x7C, 32),
                  (0x0D, 32), (0x0F, 28), (0x11, 24), (0x12, 48), (0x15, 49), (0x16, 28),
                  (0x75, 32), (0x76, 32), (0x77, 32), (0x78, 32), (0x79, 32), (0x7D, 32)]:
        assert L.ane_opcode_payload_size(op) == n, hex(op)
        assert L.ane_opcode_supported(op) == 1
    for op in (0x01, 0x14, 0x4D, 0x7A, 0x7F, 0xFF):
        assert L.ane_opcode_supported(op) == 0
        assert L.ane_opcode_payload_size(op) == -1


def test_stream_exec_rejects_unsupported_and_truncated():
    import ane_b200
    from ane_b200 import U32, Op, Ptr, encode

    with pytest.raises(ane_b200.AneError) as e:
        ane_b200.stream_exec(bytes([0x14]) + bytes(40))  # luti2_op: not executed here
    assert e.value.code == 2
    full = encode(Op.q8_0_gemv, U32(32), U32(32), Ptr(1), Ptr(2), Ptr(3))
    with pytest.raises(ane_b200.AneError) as e:
        ane_b200.stream_exec(full[:-1])
    assert e.value.code == 3
    for op in (Op.q4_k_gemv, Op.q2_k_gemv, Op.q3_k_gemv, Op.q5_k_gemv, Op.q6_k_gemv, Op.get_rows_q4_0):
        full = encode(op, U32(32), U32(256), Ptr(1), Ptr(2), Ptr(3))
        assert len(full) == 33
        with pytest.raises(ane_b200.AneError) as e:
            ane_b200.stream_exec(full[:-3])
        assert e.value.code == 3, op
    # 0x00 ends the stream (jump-table slot 0 = exit) and an empty stream is a no-op
    ane_b200.stream_exec(bytes([0x00]) + bytes([0x14]))
    ane_b200.stream_exec(b"")


def test_program_concatenates_streams():
    from ane_b200 import U32, Op, Program, Ptr, encode

    p = Program().emit(Op.pack_b_i8, U32(4), U32(16), Ptr(1), Ptr(2)).emit(Op.q8_0_gemv, U32(1), U32(32), Ptr(1),
                                                                             Ptr(2), Ptr(3))
    assert p.size() == 25 + 33
    assert bytes(p._bytes) == encode(Op.pack_b_i8, U32(4), U32(16), Ptr(1), Ptr(2)) + encode(
        Op.q8_0_gemv, U32(1), U32(32), Ptr(1), Ptr(2), Ptr(3))


def test_no_gpu_means_loud_failure():
    """Without a B200 the product path errors out; it never computes on the CPU."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import ane_b200
    import numpy as np

    x = np.ones(16, np.float32)
    q = np.zeros(16, np.int8)
    s = np.zeros(1, np.float32)
    rc = ane_b200.lib.ane_quantize_fp32_i8(16, x.ctypes.data, q.ctypes.data, s.ctypes.data)
    assert rc == 5  # ANE_ERR_NO_DEVICE
    assert not q.any() and s[0] == 0
    # the K-quant matvecs and get_rows_q4_0 likewise: no CPU fallback
    xk = np.ones(256, np.float32)
    W = np.zeros(210, np.uint8)
    out = np.full(1, 7.0, np.float32)
    for fmt in ("q2_k", "q3_k", "q4_k", "q5_k", "q6_k"):
        fn = getattr(ane_b200.lib, "ane_%s_gemv" % fmt)
        assert fn(1, 256, xk.ctypes.data, W.ctypes.data, out.ctypes.data) == 5, fmt
        assert out[0] == 7.0
    # the flags entry: an opcode outside 0x75-0x79 is an argument error before
    # any device work; a valid one fails loudly without a GPU
    ex = ane_b200.lib.ane_kquant_gemv_ex_dev
    assert ex(0x74, 1, 256, xk.ctypes.data, W.ctypes.data, out.ctypes.data, 1, None) == 1
    assert ex(0x7A, 1, 256, xk.ctypes.data, W.ctypes.data, out.ctypes.data, 1, None) == 1
    assert ex(0x79, 1, 256, xk.ctypes.data, W.ctypes.data, out.ctypes.data, 1, None) == 5
    assert out[0] == 7.0
    idx = np.zeros(1, np.uint32)
    rows = np.full(32, 7.0, np.float32)
    assert ane_b200.lib.ane_get_rows_q4_0(1, 32, W.ctypes.data, idx.ctypes.data, rows.ctypes.data) == 5
    assert (rows == 7.0).all()


def test_cpp_header_compiles_on_linux(tmp_path):
    """include/ane/ane.hpp (the drop-in C++ front end) builds with g++ -std=c++20."""
    import subprocess

    src = tmp_path / "t.cpp"
    src.write_text(
        '#include <ane/ane.hpp>\n'
        'int main() { float a[16]={0}, b[16]={0}, c[16]={0};\n'
        '  ane::program p; p.emit(ane::Op::dense_fused_i8, 1, 1, 16, 1.0f, true, a, b, c);\n'
        '  return p.size() == 42 ? 0 : 1; }\n')
    exe = tmp_path / "t"
    r = subprocess.run(["g++", "-std=c++20", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                        "-L", os.path.join(ROOT, "ane_b200", "_lib"), "-lane_b200",
                        "-Wl,-rpath," + os.path.join(ROOT, "ane_b200", "_lib")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert subprocess.run([str(exe)]).returncode == 0

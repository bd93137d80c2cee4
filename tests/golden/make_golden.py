"""Generate the known-answer fixtures in this folder from the reference's own tests.

The reference (joshmorgan1000/ane) is AArch64 SME2 assembly and cannot run on
x86, so its outputs cannot be recorded here.  What its test files do pin is
(a) deterministic input patterns and (b) expected values computed by plain CPU
loops in those tests.  This script restates those patterns and those CPU
loops in numpy (double precision where the reference test uses it) and writes
them to ``reference_kats.npz``:

* ``igemm_*``  tests/test_remaining_ops.cpp:131-184 -- int8 GEMM M=16 N=32 K=64,
  A[i] = (i % 11) - 5, B[i] = (i % 13) - 6, exact integer sums, alpha 1.0 / 0.5.
* ``q8rows32_*`` / ``q8rows64_*``  tests/test_remaining_ops.cpp:230-325 -- Q8_0
  tables (fp16 d = 0.1*(v+1) resp. 0.05*(v+b+1), qs = (q+7v)%21-10 resp.
  (q+3v+5b)%19-9), rows {1, 3}, expected float(q)*float(d), tolerance 1e-4.
* ``qrt_*``  tests/test_dsl_coverage.cpp:334-368 -- quantize round trip on
  x[i] = (i-128)*0.1f, 256 values, bound max|x - deq(q(x))| < 1.5*scale.
* ``mnist_*``  tests/test_mnist_i8.cpp:43-50,165-169 -- padding constants and
  the packed-B byte count for W1 (832 x 128) and W2 (128 x 16).

Run:  python tests/golden/make_golden.py   (writes reference_kats.npz)
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def c_mod(a: int, b: int) -> int:
    """C's % on ints (truncating toward zero)."""
    r = abs(a) % b
    return -r if a < 0 else r


def igemm():
    M, N, K = 16, 32, 64
    A = np.array([c_mod(i, 11) - 5 for i in range(M * K)], np.int8).reshape(M, K)
    B = np.array([c_mod(i, 13) - 6 for i in range(K * N)], np.int8).reshape(K, N)
    ref = A.astype(np.int64) @ B.astype(np.int64)
    return {
        "igemm_A": A, "igemm_B": B, "igemm_ref_i32": ref.astype(np.int32),
        "igemm_ref_alpha1": (ref.astype(np.float32) * np.float32(1.0)),
        "igemm_ref_alpha05": (ref.astype(np.float32) * np.float32(0.5)),
        "igemm_tol": np.float32(1e-3),
    }


def q8_table(vocab: int, dim: int, scale_fn, q_fn):
    nb = dim // 32
    table = np.zeros((vocab, nb * 34), np.uint8)
    for v in range(vocab):
        for b in range(nb):
            d = np.float32(scale_fn(v, b))
            bits = np.array([d], np.float32).astype(np.float16).view(np.uint16)[0]  # (__fp16)f, RN
            blk = table[v, b * 34:(b + 1) * 34]
            blk[0] = bits & 0xFF
            blk[1] = bits >> 8
            for q in range(32):
                blk[2 + q] = np.uint8(np.int8(q_fn(q, v, b)).view(np.uint8))
    return table


def q8_expected(table, indices, dim):
    nb = dim // 32
    out = np.zeros((len(indices), dim), np.float64)
    for r, idx in enumerate(indices):
        row = table[idx]
        for b in range(nb):
            blk = row[b * 34:(b + 1) * 34]
            d = float(np.array([int(blk[0]) | (int(blk[1]) << 8)], np.uint16).view(np.float16)[0])
            qs = blk[2:34].view(np.int8).astype(np.float64)
            out[r, b * 32:(b + 1) * 32] = qs * d
    return out.astype(np.float32)


def q8rows():
    idx = np.array([1, 3], np.uint32)
    t32 = q8_table(4, 32, lambda v, b: 0.1 * (v + 1), lambda q, v, b: c_mod(q + v * 7, 21) - 10)
    t64 = q8_table(4, 64, lambda v, b: 0.05 * (v + b + 1), lambda q, v, b: c_mod(q + v * 3 + b * 5, 19) - 9)
    return {
        "q8rows_idx": idx,
        "q8rows32_table": t32, "q8rows32_ref": q8_expected(t32, idx, 32),
        "q8rows64_table": t64, "q8rows64_ref": q8_expected(t64, idx, 64),
        "q8rows_tol": np.float32(1e-4),
    }


def quant_roundtrip():
    x = (np.arange(256, dtype=np.int32) - 128).astype(np.float32) * np.float32(0.1)
    absmax = np.max(np.abs(x))
    scale = absmax / np.float32(127.0)
    inv = np.float32(127.0) / absmax
    q = np.rint(np.clip(x * inv, np.float32(-127.0), np.float32(127.0))).astype(np.int8)
    return {"qrt_x": x, "qrt_scale": np.float32(scale), "qrt_q": q, "qrt_bound_factor": np.float32(1.5)}


def mnist_consts():
    INPUT_DIM, HIDDEN_DIM, OUTPUT_DIM = 784, 128, 10
    INP_K = (INPUT_DIM + 63) // 64 * 64
    HID_K = (HIDDEN_DIM + 63) // 64 * 64
    OUT_PAD = (OUTPUT_DIM + 15) // 16 * 16

    def packed(K, N):
        return ((K + 3) // 4 * 4 // 4) * ((N + 15) // 16 * 16 // 16) * 64

    return {"mnist_dims": np.array([INPUT_DIM, HIDDEN_DIM, OUTPUT_DIM, INP_K, HID_K, OUT_PAD], np.int32),
            "mnist_packed_bytes": np.array([packed(INP_K, HIDDEN_DIM), packed(HID_K, OUT_PAD)], np.int64)}


def main():
    d = {}
    for f in (igemm, q8rows, quant_roundtrip, mnist_consts):
        d.update(f())
    np.savez(os.path.join(HERE, "reference_kats.npz"), **d)
    print("wrote", os.path.join(HERE, "reference_kats.npz"), len(d), "arrays")


if __name__ == "__main__":
    main()

"""The two facts the K-quant decoders of kquant_gemv.cu rest on, checked on
the CPU.

1. Code extraction.  Thread t of a row holds lanes 2t and 2t+1.  The decoders
   leave a code at a bit position p (value q·2^p) where that saves a shift, and
   pair it with the scale times 2^-p; q3_k's second half shifts its packed word
   by the first half's x bits first (amounts >= 32 give 0).  For every t and
   random words, the extracted values equal the handlers' codes times 2^p.
2. Exact products.  A sub-block scale is an fp16 d times a code of at most 6
   bits (8 for q6_k), and element codes have at most 6 bits, so d·sc and
   q·(d·sc) are exact in fp32.  That makes the handlers' RN(RN(q·dsc) + dmm)
   equal to one fma(q, dsc, dmm), and RN((q - off)·dsc) equal to
   RN(q·2^p·(dsc·2^-p)), for every finite fp16 scale.
"""
import numpy as np


def test_code_extraction_matches_the_handlers_codes():
    rng = np.random.default_rng(0)
    n = 50000
    b16 = rng.integers(0, 1 << 16, n, dtype=np.uint64)
    w = rng.integers(0, 1 << 32, n, dtype=np.uint64)
    h = rng.integers(0, 1 << 32, n, dtype=np.uint64)
    s0 = rng.integers(0, 40, n, dtype=np.uint64)  # q3_k stale shift amounts, some >= 32
    mask32 = 0xFFFFFFFF

    def shr_clamp(x, s):
        return np.where(s >= 32, 0, (x >> np.minimum(s, 31)) & mask32)

    for t in range(8):
        l0, l1 = 2 * t, 2 * t + 1
        # q4_k: the two bytes of lanes 2t, 2t+1; low nibbles at bits 0, 8, high at 4, 12
        assert np.array_equal(b16 & 0xF, b16 & 0x000F)
        assert np.array_equal(((b16 >> 8) & 0xF) << 8, b16 & 0x0F00)
        assert np.array_equal(((b16 >> 4) & 0xF) << 4, b16 & 0x00F0)
        assert np.array_equal(((b16 >> 12) & 0xF) << 12, b16 & 0xF000)
        # q2_k: lane 2t at bits 4t..4t+1 (x 1), lane 2t+1 at 4t+2..4t+3 (x 4)
        ws = w >> (4 * t)
        assert np.array_equal((w >> (4 * t)) & 3, ws & 3)
        assert np.array_equal(((w >> (4 * t + 2)) & 3) * 4, ws & 0xC)
        # q5_k: the four 5-bit codes as bytes, high bits moved by one multiply
        ref = [(b16 & 0xF) | (((h >> l0) & 1) << 4), ((b16 >> 8) & 0xF) | (((h >> l1) & 1) << 4),
               ((b16 >> 4) & 0xF) | (((h >> (16 + l0)) & 1) << 4),
               ((b16 >> 12) & 0xF) | (((h >> (16 + l1)) & 1) << 4)]
        hb = (h >> (2 * t)) & 0x00030003
        v = (((b16 | (b16 << 12)) & 0x0F0F0F0F) | ((hb * 0x810) & 0x10101010)) & mask32
        for k in range(4):
            assert np.array_equal((v >> (8 * k)) & 0xFF, ref[k])
        # q3_k: first half (x 1, x 4) and second half after the stale shift
        h0 = h & 0xFFFF
        q00 = ((w >> (2 * l0)) & 3) | (((h0 >> l0) & 1) << 2)
        q01 = ((w >> (2 * l1)) & 3) | (((h0 >> l1) & 1) << 2)
        assert np.array_equal(q00, (ws & 3) | (((h0 >> l0) & 1) << 2))
        assert np.array_equal(q01 * 4, (ws & 0xC) | (((h0 >> l1) & 1) << 4))
        t1 = shr_clamp(w, s0)
        q11 = ((t1 >> (2 * l1)) & 3) | (((h0 >> l1) & 1) << 2)
        assert np.array_equal(q11 * 4, ((t1 >> (4 * t)) & 0xC) | (((h0 >> l1) & 1) << 4))
        # q6_k: lane 2t low nibble | 2 high bits (x 1), lane 2t+1 high nibble | 2 bits (x 16)
        b8 = b16 & 0xFF
        hs = h >> (4 * t)
        q0 = (b8 & 0xF) | (((h >> (4 * t)) & 3) << 4)
        q1 = (b8 >> 4) | (((h >> (4 * t + 2)) & 3) << 4)
        assert np.array_equal(q0, (b8 & 0x0F) | ((hs << 4) & 0x30))
        assert np.array_equal(q1 * 16, (b8 & 0xF0) | ((hs << 6) & 0x300))


def test_scale_and_code_products_are_exact_in_fp32():
    # every finite fp16 value as d
    d = np.arange(1 << 16, dtype=np.uint16).view(np.float16).astype(np.float64)
    d = d[np.isfinite(d)]
    for sc_bits, q_bits, signed in ((6, 5, False), (4, 2, False), (6, 3, True), (8, 6, True)):
        scs = np.arange(-(1 << (sc_bits - 1)), 1 << (sc_bits - 1)) if signed else np.arange(1 << sc_bits)
        for sc in scs:
            dsc64 = d * float(sc)
            dsc32 = (d.astype(np.float32) * np.float32(sc)).astype(np.float64)
            assert np.array_equal(dsc64, dsc32), (sc_bits, sc)  # d·sc exact
            qmax = 1 << q_bits
            for q in (1, 3, qmax - 1, -(qmax // 2)) if signed else (1, 3, qmax - 1):
                p64 = dsc64 * q
                p32 = (dsc32.astype(np.float32) * np.float32(q)).astype(np.float64)
                assert np.array_equal(p64, p32), (sc_bits, sc, q)  # q·dsc exact
                for p in (2, 4, 8, 12):  # a code at bit p paired with dsc·2^-p
                    scaled = (dsc32.astype(np.float32) * np.float32(2.0 ** -p)).astype(np.float64)
                    assert np.array_equal(scaled * (2.0 ** p), dsc64)

"""Test helpers for the K-quant matvecs and get_rows_q4_0: random super-blocks
with controlled fp16 scales, and an independent numpy dequantizer of each
layout as the reference handlers read it (src/bytecode_interpreter.s:
11024-11620), used to cross-check the C oracle's decoding."""
import numpy as np

BLOCK_BYTES = {"q2_k": 84, "q3_k": 110, "q4_k": 144, "q5_k": 176, "q6_k": 210}
# byte offsets of the fp16 fields (d, dmin) per format
_D_OFF = {"q4_k": (0, 2), "q5_k": (0, 2), "q2_k": (80, 82), "q3_k": (108, None), "q6_k": (208, None)}


def random_blocks(fmt, M, K, rng, scale=0.01):
    """M rows of K/256 random super-blocks; d (and dmin) set to small positive fp16."""
    nsb = K // 256
    bb = BLOCK_BYTES[fmt]
    W = rng.integers(0, 256, size=(M, nsb, bb), dtype=np.uint8)
    d_off, m_off = _D_OFF[fmt]
    for off in (d_off, m_off):
        if off is None:
            continue
        h = (rng.random((M, nsb)) * scale + scale / 8).astype(np.float16).view(np.uint8).reshape(M, nsb, 2)
        W[:, :, off:off + 2] = h
    return W.reshape(-1)


def set_scale(W, fmt, M, K, row, sb, value, which=0):
    """Overwrite d (which=0) or dmin (which=1) of one super-block with an fp16 value."""
    nsb = K // 256
    off = _D_OFF[fmt][which]
    blk = W.reshape(M, nsb, BLOCK_BYTES[fmt])
    blk[row, sb, off:off + 2] = np.frombuffer(np.float16(value).tobytes(), np.uint8)


def _f16(b, off):
    return float(b[off:off + 2].copy().view(np.float16)[0])


def _scale_min(s, j):
    if j < 4:
        return s[j] & 0x3F, s[j + 4] & 0x3F
    return (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4), (s[j + 4] >> 4) | ((s[j] >> 6) << 4)


def dequant_row(fmt, row_bytes, x):
    """float64 values of one row's K weights (the handlers' element order), and
    for q3_k the dependence of the second-half codes on x (the stale shift)."""
    nsb = len(row_bytes) // BLOCK_BYTES[fmt]
    out = np.zeros(nsb * 256)
    xb_all = np.asarray(x, np.float32)
    for b in range(nsb):
        blk = row_bytes[b * BLOCK_BYTES[fmt]:(b + 1) * BLOCK_BYTES[fmt]].astype(np.int64)
        raw = row_bytes[b * BLOCK_BYTES[fmt]:(b + 1) * BLOCK_BYTES[fmt]]
        v = out[b * 256:(b + 1) * 256]
        xb = xb_all[b * 256:(b + 1) * 256]
        if fmt in ("q4_k", "q5_k"):
            d, dmin = _f16(raw, 0), _f16(raw, 2)
            qs = blk[16:144] if fmt == "q4_k" else blk[48:176]
            for j in range(8):
                sc, mn = _scale_min(blk[4:16], j)
                h = int.from_bytes(bytes(raw[16 + 4 * j:20 + 4 * j]), "little") if fmt == "q5_k" else 0
                for i in range(16):
                    lo, hi = qs[16 * j + i] & 15, qs[16 * j + i] >> 4
                    if fmt == "q5_k":
                        lo |= ((h >> i) & 1) << 4
                        hi |= ((h >> (16 + i)) & 1) << 4
                    v[32 * j + i] = d * sc * lo - dmin * mn
                    v[32 * j + 16 + i] = d * sc * hi - dmin * mn
        elif fmt == "q2_k":
            d, dmin = _f16(raw, 80), _f16(raw, 82)
            for j in range(16):
                w = int.from_bytes(bytes(raw[16 + 4 * j:20 + 4 * j]), "little")
                for i in range(16):
                    v[16 * j + i] = d * (blk[j] & 15) * ((w >> (2 * i)) & 3) - dmin * (blk[j] >> 4)
        elif fmt == "q3_k":
            d = _f16(raw, 108)
            sc = blk[96:108]
            for j in range(8):
                s6 = (sc[j] & 0x3F) if j < 4 else ((sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4))
                w0 = int.from_bytes(bytes(raw[32 + 8 * j:36 + 8 * j]), "little")
                w1 = int.from_bytes(bytes(raw[36 + 8 * j:40 + 8 * j]), "little")
                h0 = int.from_bytes(bytes(raw[4 * j:4 * j + 2]), "little")
                h1 = int.from_bytes(bytes(raw[4 * j + 2:4 * j + 4]), "little")
                for i in range(16):
                    q = ((w0 >> (2 * i)) & 3) | (((h0 >> i) & 1) << 2)
                    v[32 * j + i] = d * (s6 - 32) * (q - 4)
                    xs = int(xb[32 * j + i:32 * j + i + 1].view(np.uint32)[0])
                    t = 0 if xs >= 32 else (w1 >> xs)
                    q = ((t >> (2 * i)) & 3) | (((h1 >> i) & 1) << 2)
                    v[32 * j + 16 + i] = d * (s6 - 32) * (q - 4)
        elif fmt == "q6_k":
            d = _f16(raw, 208)
            sc = raw[192:208].view(np.int8).astype(np.int64)
            for j in range(16):
                h = int.from_bytes(bytes(raw[128 + 4 * j:132 + 4 * j]), "little")
                for n in range(16):
                    byte = blk[8 * j + n // 2]
                    nib = (byte >> 4) if n & 1 else (byte & 15)
                    q = nib | (((h >> (2 * n)) & 3) << 4)
                    v[16 * j + n] = d * sc[j] * (q - 32)
    return out


def get_rows_q4_0_kat_tables():
    """The reference's get_rows_q4_0 test tables (tests/test_remaining_ops.cpp:
    328-430): vocab 4; dim 32 (scale 0.2 (v+1), nibbles (i+v) % 16 and
    (i+v+3) % 16) and dim 64 (scale 0.15 (v+b+1), nibbles (i+v+2b) % 16 and
    (i+v+2b+5) % 16); rows [0, 2]; expected (nibble - 8) * float(fp16(scale))."""
    cases = []
    for dim, sc, lo_off, hi_off in ((32, lambda v, b: 0.2 * (v + 1), lambda v, b: v, lambda v, b: v + 3),
                                    (64, lambda v, b: 0.15 * (v + b + 1), lambda v, b: v + 2 * b,
                                     lambda v, b: v + 2 * b + 5)):
        nb = dim // 32
        table = np.zeros((4, nb, 18), np.uint8)
        for v in range(4):
            for b in range(nb):
                table[v, b, 0:2] = np.frombuffer(np.float16(np.float32(sc(v, b))).tobytes(), np.uint8)
                for i in range(16):
                    table[v, b, 2 + i] = (((i + hi_off(v, b)) % 16) << 4) | ((i + lo_off(v, b)) % 16)
        idx = np.array([0, 2], np.uint32)
        ref = np.zeros((2, dim), np.float32)
        for r, v in enumerate(idx):
            for b in range(nb):
                s = np.float32(table[v, b, 0:2].copy().view(np.float16)[0])
                for i in range(16):
                    q = int(table[v, b, 2 + i])
                    ref[r, 32 * b + i] = np.float32((q & 15) - 8) * s
                    ref[r, 32 * b + 16 + i] = np.float32((q >> 4) - 8) * s
        cases.append((table.reshape(-1), idx, dim, ref))
    return cases

"""The activation quantizer of the Q8_0 MUL_MAT kernel splits each 32-element
block over 4 lanes: lane i folds the absmax of elements 8i..8i+7 with ggml's
sequential compare (acc = acc > a ? acc : a, a = |x|) from 0 and records
whether it saw a NaN; the 4 results combine in order as
acc = nan_i ? r_i : (acc > r_i ? acc : r_i).  The compare restarts at a NaN
(both NaN > a and a > NaN are false), so this equals the sequential fold over
all 32 elements for every input.  This test restates the combine in numpy and
checks the block scale it implies against the oracle's sequential quantizer
(ane_ref_quantize_q8_0), on blocks with NaN, inf and zeros at every quarter
position.  The kernel itself is checked against the one-thread-per-block
quantize_q8_0 kernel, bit for bit, by the GPU parity tests."""
import numpy as np

import oracle


def _fold(acc, a):
    return acc if acc > a else a


def _segmented_amax(block):
    acc = np.float32(0.0)
    for i in range(4):
        r, nan = np.float32(0.0), False
        for a in np.abs(block[8 * i:8 * i + 8]):
            nan |= bool(a != a)
            r = _fold(r, a)
        acc = r if nan else _fold(acc, r)
    return acc


def test_segmented_absmax_gives_the_oracle_block_scales():
    rng = np.random.default_rng(11)
    nb = 512
    x = rng.standard_normal(nb * 32).astype(np.float32)
    specials = [np.nan, np.inf, -np.inf, 0.0, np.float32(6.0), np.float32(-9.5)]
    for b in range(nb):
        for _ in range(b % 5):  # 0-4 special values per block, anywhere in it
            x[b * 32 + rng.integers(0, 32)] = specials[rng.integers(0, len(specials))]
    x[32 * 7 + 7] = np.nan    # NaN as the last element of a quarter
    x[32 * 8 + 31] = np.nan   # NaN as the block's last element: the scale is NaN
    x[32 * 9 + 8] = np.nan    # NaN as the first element of a quarter, larger values before it
    x[32 * 9 + 0] = 50.0
    ref = oracle.quantize_q8_0(x, 1, nb * 32).reshape(nb, 34)
    ref_d = ref[:, :2].copy().view(np.float16).ravel().astype(np.float32)
    checked = 0
    for b in range(nb):
        amax = _segmented_amax(x[b * 32:(b + 1) * 32])
        d = np.float16(np.float32(amax) / np.float32(127.0)).astype(np.float32)
        if np.isnan(d):
            assert np.isnan(ref_d[b]), b
        else:
            assert d.view(np.uint32) == ref_d[b].view(np.uint32), (b, d, ref_d[b])
        checked += 1
    assert checked == nb
    # the restart really is exercised: block 9's scale ignores the 50.0 before its NaN
    assert ref_d[9] < np.float32(50.0) / 127
    assert np.isnan(ref_d[8])

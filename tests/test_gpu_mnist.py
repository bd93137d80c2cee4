"""The reference's MNIST-i8 training step (tests/test_mnist_i8.cpp:304-346) on
the GPU opcode by opcode through ane::dispatch byte streams, bit-exact against
the oracle chain; and each of its fp32 opcodes alone (0x0D, 0x0F, 0x11, 0x12,
0x15, 0x16), including the edge cases the handlers define (NaN, ties, labels
outside the first 16 columns, K not a multiple of 16)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
F32 = np.float32
INP_K, HID, HID_K, OUT_PAD, B = 832, 128, 128, 16, 50


def _bits_equal(a, b):
    a, b = np.asarray(a, F32), np.asarray(b, F32)
    nan = np.isnan(a)
    return np.array_equal(nan, np.isnan(b)) and np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


def test_fp32_ops_exact(ane):
    rng = np.random.default_rng(21)
    n = 4096 + 7
    a = rng.standard_normal(n).astype(F32)
    b = rng.standard_normal(n).astype(F32)
    a[5] = np.nan
    b[6] = np.inf
    out = np.empty(n, F32)
    ane.dispatch(ane.Op.elementwise_scaled_add_fp32, ane.U32(n), ane.F32(-0.013), ane.Ptr(a.ctypes.data),
                 ane.Ptr(b.ctypes.data), ane.Ptr(out.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert _bits_equal(out, oracle.elementwise_scaled_add_fp32(np.float32(-0.013), a, b))
    act = rng.standard_normal(n).astype(F32)
    act[:4] = [0.0, -0.0, np.nan, 1e-45]
    out2 = np.empty(n, F32)
    ane.dispatch(ane.Op.relu_backward_fp32, ane.U32(n), ane.Ptr(act.ctypes.data), ane.Ptr(b.ctypes.data),
                 ane.Ptr(out2.ctypes.data))
    assert _bits_equal(out2, oracle.relu_backward_fp32(act, b))
    src = rng.standard_normal((333, 77)).astype(F32)
    dst = np.empty((77, 333), F32)
    ane.dispatch(ane.Op.transpose_fp32, ane.U32(333), ane.U32(77), ane.Ptr(src.ctypes.data), ane.Ptr(dst.ctypes.data))
    assert np.array_equal(dst, src.T)
    pred = rng.integers(0, 12, 1000).astype(np.int32)
    lab = rng.integers(0, 12, 1000).astype(np.uint8)
    cnt = np.zeros(1, np.int32)
    ane.dispatch(ane.Op.count_matches, ane.U32(1000), ane.Ptr(pred.ctypes.data), ane.Ptr(lab.ctypes.data),
                 ane.Ptr(cnt.ctypes.data))
    assert cnt[0] == oracle.count_matches(pred, lab)


@pytest.mark.parametrize("M,N,K,flags", [(128, 16, 50, 0), (50, 128, 16, 1), (832, 128, 50, 0), (33, 40, 64, 1)])
def test_dense_fp32_exact(ane, M, N, K, flags):
    rng = np.random.default_rng(M + N + K)
    M16 = (M + 15) // 16 * 16
    A = rng.standard_normal((M16, K)).astype(F32)
    Bm = rng.standard_normal((K, N)).astype(F32)
    bias = rng.standard_normal(N).astype(F32)
    ref = oracle.dense_fp32(M, N, K, 0.75, flags, A, Bm, bias)
    C = np.empty((M16, N), F32)
    ane.dispatch(ane.Op.dense_fp32, ane.U32(M), ane.U32(N), ane.U32(K), ane.F32(0.75), ane.U8(flags),
                 ane.Ptr(A.ctypes.data), ane.Ptr(Bm.ctypes.data), ane.Ptr(bias.ctypes.data), ane.Ptr(C.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert _bits_equal(C, ref)


@pytest.mark.parametrize("cols", [16, 48])
def test_softmax_argmax_exact(ane, cols):
    rng = np.random.default_rng(cols)
    batch = 37
    logits = (rng.standard_normal((batch, cols)) * 5).astype(F32)
    logits[3, 2] = logits[3, 9] = 40.0      # tie for the max: first index wins
    logits[4, :] = -1000.0                   # all equal
    logits[5, 7] = np.nan
    logits[6, 0] = np.inf
    labels = rng.integers(0, cols, batch).astype(np.uint8)
    labels[7] = 200                          # no column gets the -1
    g0 = np.full((batch, cols), 5.0, F32)    # only the first 16 columns are written
    probs_r, g_r, am_r = oracle.softmax_argmax_fp32(logits, labels, g0)
    probs = np.empty_like(logits)
    g = g0.copy()
    am = np.empty(batch, np.int32)
    ane.dispatch(ane.Op.softmax_argmax_fp32, ane.U32(batch), ane.U32(cols), ane.Ptr(logits.ctypes.data),
                 ane.Ptr(probs.ctypes.data), ane.Ptr(labels.ctypes.data), ane.Ptr(g.ctypes.data),
                 ane.Ptr(am.ctypes.data))
    assert ane.lib.ane_last_error() == 0
    assert _bits_equal(probs, probs_r) and _bits_equal(g, g_r) and np.array_equal(am, am_r)


def test_mnist_i8_training_step(ane):
    """Two SGD steps of the reference's training loop, every opcode dispatched
    as a byte stream on host buffers, against the same chain on the oracle."""
    rng = np.random.default_rng(1)
    W1 = (rng.standard_normal((INP_K, HID)) * np.sqrt(2.0 / 784)).astype(F32)
    W1[784:] = 0
    W2 = (rng.standard_normal((HID, OUT_PAD)) * np.sqrt(2.0 / HID)).astype(F32)
    xu8 = np.zeros((64, INP_K), np.uint8)
    xu8[:B, :784] = rng.integers(0, 256, (B, 784), dtype=np.uint8)
    xfp = (xu8.astype(F32) / F32(255.0))
    labels = rng.integers(0, 10, B).astype(np.uint8)
    logit_bias = np.array([0.0] * 10 + [-1000.0] * 6 + [0.0] * 16, F32)
    zero_bias = np.zeros(INP_K, F32)
    u8_scale, lr = F32(1.0 / 255.0), F32(0.05)

    def step(backend, W1, W2):
        # weights quantized and packed per step (the reference repacks them periodically)
        W1q, sW1 = oracle.quantize_fp32_i8(W1)
        W2q, sW2 = oracle.quantize_fp32_i8(W2)
        W1p = oracle.pack_b_i8(W1q.reshape(INP_K, HID), INP_K, HID)
        W2p = oracle.pack_b_i8(W2q.reshape(HID, OUT_PAD), HID_K, OUT_PAD)
        return backend(W1, W2, W1p, W2p, np.float32(sW1), np.float32(sW2))

    def gpu(W1, W2, W1p, W2p, sW1, sW2):
        W1, W2 = W1.copy(), W2.copy()
        hidden = np.zeros((64, HID), F32)
        ane.dispatch(ane.Op.dense_u8s8, ane.U32(B), ane.U32(HID), ane.U32(INP_K), ane.F32(u8_scale), ane.F32(sW1),
                     True, ane.Ptr(xu8.ctypes.data), ane.Ptr(W1p.ctypes.data), ane.Ptr(zero_bias.ctypes.data),
                     ane.Ptr(hidden.ctypes.data))
        hid_i8 = np.zeros((64, HID_K), np.int8)
        sh = np.zeros(1, F32)
        ane.dispatch(ane.Op.quantize_fp32_i8, ane.U32(B * HID_K), ane.Ptr(hidden.ctypes.data),
                     ane.Ptr(hid_i8.ctypes.data), ane.Ptr(sh.ctypes.data))
        logits = np.zeros((64, OUT_PAD), F32)
        ane.dispatch(ane.Op.dense_i8, ane.U32(B), ane.U32(OUT_PAD), ane.U32(HID_K), ane.F32(sh[0]), ane.F32(sW2),
                     False, ane.Ptr(hid_i8.ctypes.data), ane.Ptr(W2p.ctypes.data), ane.Ptr(logit_bias.ctypes.data),
                     ane.Ptr(logits.ctypes.data))
        probs = np.zeros((B, OUT_PAD), F32)
        g_out = np.zeros((64, OUT_PAD), F32)
        pred = np.zeros(B, np.int32)
        ane.dispatch(ane.Op.softmax_argmax_fp32, ane.U32(B), ane.U32(OUT_PAD), ane.Ptr(logits.ctypes.data),
                     ane.Ptr(probs.ctypes.data), ane.Ptr(labels.ctypes.data), ane.Ptr(g_out.ctypes.data),
                     ane.Ptr(pred.ctypes.data))
        correct = np.zeros(1, np.int32)
        ane.dispatch(ane.Op.count_matches, ane.U32(B), ane.Ptr(pred.ctypes.data), ane.Ptr(labels.ctypes.data),
                     ane.Ptr(correct.ctypes.data))
        h_T = np.zeros((HID, B), F32)
        ane.dispatch(ane.Op.transpose_fp32, ane.U32(B), ane.U32(HID), ane.Ptr(hidden.ctypes.data),
                     ane.Ptr(h_T.ctypes.data))
        gW2 = np.zeros((HID, OUT_PAD), F32)
        ane.dispatch(ane.Op.dense_fp32, ane.U32(HID), ane.U32(OUT_PAD), ane.U32(B), ane.F32(1.0), False,
                     ane.Ptr(h_T.ctypes.data), ane.Ptr(g_out.ctypes.data), ane.Ptr(zero_bias.ctypes.data),
                     ane.Ptr(gW2.ctypes.data))
        W2_T = np.zeros((OUT_PAD, HID), F32)
        ane.dispatch(ane.Op.transpose_fp32, ane.U32(HID), ane.U32(OUT_PAD), ane.Ptr(W2.ctypes.data),
                     ane.Ptr(W2_T.ctypes.data))
        g_hid = np.zeros((64, HID), F32)
        ane.dispatch(ane.Op.dense_fp32, ane.U32(B), ane.U32(HID), ane.U32(OUT_PAD), ane.F32(1.0), False,
                     ane.Ptr(g_out.ctypes.data), ane.Ptr(W2_T.ctypes.data), ane.Ptr(zero_bias.ctypes.data),
                     ane.Ptr(g_hid.ctypes.data))
        g_hid_r = np.zeros((64, HID), F32)
        ane.dispatch(ane.Op.relu_backward_fp32, ane.U32(B * HID_K), ane.Ptr(hidden.ctypes.data),
                     ane.Ptr(g_hid.ctypes.data), ane.Ptr(g_hid_r.ctypes.data))
        x_T = np.zeros((INP_K, B), F32)
        ane.dispatch(ane.Op.transpose_fp32, ane.U32(B), ane.U32(INP_K), ane.Ptr(xfp.ctypes.data),
                     ane.Ptr(x_T.ctypes.data))
        gW1 = np.zeros((INP_K, HID), F32)
        ane.dispatch(ane.Op.dense_fp32, ane.U32(INP_K), ane.U32(HID), ane.U32(B), ane.F32(1.0), False,
                     ane.Ptr(x_T.ctypes.data), ane.Ptr(g_hid_r.ctypes.data), ane.Ptr(zero_bias.ctypes.data),
                     ane.Ptr(gW1.ctypes.data))
        stp = F32(-lr / B)
        ane.dispatch(ane.Op.elementwise_scaled_add_fp32, ane.U32(INP_K * HID), ane.F32(stp), ane.Ptr(W1.ctypes.data),
                     ane.Ptr(gW1.ctypes.data), ane.Ptr(W1.ctypes.data))
        ane.dispatch(ane.Op.elementwise_scaled_add_fp32, ane.U32(HID * OUT_PAD), ane.F32(stp),
                     ane.Ptr(W2.ctypes.data), ane.Ptr(gW2.ctypes.data), ane.Ptr(W2.ctypes.data))
        assert ane.lib.ane_last_error() == 0
        return W1, W2, probs, pred, int(correct[0])

    def ref(W1, W2, W1p, W2p, sW1, sW2):
        hidden = oracle.dense_u8s8(B, HID, INP_K, u8_scale, sW1, 1, xu8, W1p, zero_bias)
        hq, sh = oracle.quantize_fp32_i8(hidden[:B].ravel())
        hid_i8 = np.zeros((64, HID_K), np.int8)
        hid_i8[:B] = hq.reshape(B, HID_K)
        logits = oracle.dense_i8(B, OUT_PAD, HID_K, np.float32(sh), sW2, 0, hid_i8, W2p, logit_bias)
        probs, g16, pred = oracle.softmax_argmax_fp32(logits[:B], labels)
        g_out = np.zeros((64, OUT_PAD), F32)
        g_out[:B] = g16
        correct = oracle.count_matches(pred, labels)
        h_T = oracle.transpose_fp32(hidden[:B])
        gW2 = oracle.dense_fp32(HID, OUT_PAD, B, 1.0, 0, h_T, g_out[:B], zero_bias)
        W2_T = oracle.transpose_fp32(W2)
        g_hid = oracle.dense_fp32(B, HID, OUT_PAD, 1.0, 0, g_out, W2_T, zero_bias)
        g_hid_r = np.zeros((64, HID), F32)
        g_hid_r[:B] = oracle.relu_backward_fp32(hidden[:B], g_hid[:B]).reshape(B, HID)
        x_T = oracle.transpose_fp32(xfp[:B])
        gW1 = oracle.dense_fp32(INP_K, HID, B, 1.0, 0, x_T, g_hid_r[:B], zero_bias)
        stp = F32(-lr / B)
        W1n = oracle.elementwise_scaled_add_fp32(stp, W1, gW1[:INP_K]).reshape(INP_K, HID)
        W2n = oracle.elementwise_scaled_add_fp32(stp, W2, gW2[:HID]).reshape(HID, OUT_PAD)
        return W1n, W2n, probs, pred, correct

    Wg = (W1, W2)
    Wr = (W1, W2)
    for _ in range(2):
        g = step(gpu, *Wg)
        r = step(ref, *Wr)
        assert _bits_equal(g[2], r[2]) and np.array_equal(g[3], r[3]) and g[4] == r[4]
        assert _bits_equal(g[0], r[0]) and _bits_equal(g[1], r[1])
        Wg, Wr = g[:2], r[:2]

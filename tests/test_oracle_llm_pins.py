"""Pins of the oracle's LLM helper restatements (shape_ops.rs rope_f32,
softmax_last_axis_f32, silu_gate_mul_up_f32, dequantize_q6_k,
dequant_matmul_f16_f32) against known answers and independent numpy
transcriptions of the reference loops. The reference ships no golden vectors
for these NIFs."""
import numpy as np
import pytest

import ref

RNG = np.random.default_rng(5)


def test_softmax_known_answers(built):
    out = ref.softmax_last_axis_f32(np.array([[0.0, np.log(2.0)]], np.float32), 1, 2)
    np.testing.assert_allclose(out, [[1 / 3, 2 / 3]], rtol=1e-6)
    # the reference scans the max from src[0] with `v > max`: a NaN there
    # poisons the row, a later NaN is skipped by the scan but not by exp
    out = ref.softmax_last_axis_f32(np.array([[np.nan, 1.0], [1.0, np.nan]], np.float32), 2, 2)
    assert np.isnan(out).all()
    out = ref.softmax_last_axis_f32(np.array([[5.0, 5.0, 5.0, 5.0]], np.float32), 1, 4)
    assert np.array_equal(out, np.full((1, 4), 0.25, np.float32))


def test_silu_gate_mul_up_known_answers(built):
    g = np.array([0.0, 30.0, -30.0, 1.0], np.float32)
    u = np.array([5.0, 2.0, 2.0, 1.0], np.float32)
    out = ref.silu_gate_mul_up_f32(g, u)
    assert out[0] == 0.0 and out[1] == np.float32(60.0)
    assert abs(out[2]) < 1e-11
    np.testing.assert_allclose(out[3], 1.0 / (1.0 + np.exp(-1.0)), rtol=1e-6)


def test_rope_known_answers(built):
    x = np.array([[1.0, 0.0], [0.0, 1.0]], np.float32)
    out = ref.rope_f32(x, np.array([0, 1], np.int64), np.array([1.0], np.float32), 2, 2, 1)
    np.testing.assert_allclose(out[0], [1.0, 0.0])
    np.testing.assert_allclose(out[1], [-np.sin(1.0), np.cos(1.0)], rtol=1e-6)
    # heads_per_token: rows 0..2 share token 0's position
    x = RNG.uniform(-1, 1, (6, 4)).astype(np.float32)
    f = np.array([1.0, 0.01], np.float32)
    out = ref.rope_f32(x, np.array([3, 0], np.int64), f, 6, 4, 3)
    assert np.array_equal(out[3:], x[3:])
    assert not np.array_equal(out[:3], x[:3])


def q6k_reference_loop(raw):
    """shape_ops.rs:2848-2899 transcribed: scales[8n + {0,2,4,6}] for every l."""
    nb = raw.shape[0]
    out = np.empty((nb, 256), np.float32)
    d = raw[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(nb)
    sc = raw[:, 192:208].view(np.int8).astype(np.int32)
    for n in range(2):
        ql, qh = raw[:, 64 * n: 64 * n + 64].astype(np.int32), raw[:, 128 + 32 * n: 160 + 32 * n].astype(np.int32)
        q1 = ((ql[:, :32] & 0xF) | ((qh & 3) << 4)) - 32
        q2 = ((ql[:, 32:] & 0xF) | (((qh >> 2) & 3) << 4)) - 32
        q3 = ((ql[:, :32] >> 4) | (((qh >> 4) & 3) << 4)) - 32
        q4 = ((ql[:, 32:] >> 4) | (((qh >> 6) & 3) << 4)) - 32
        for g, q in enumerate((q1, q2, q3, q4)):
            out[:, 128 * n + 32 * g: 128 * n + 32 * g + 32] = d[:, None] * (sc[:, 8 * n + 2 * g, None] * q).astype(np.float32)
    return out


def q6k_blocks(nb, equal_pairs=False):
    raw = RNG.integers(0, 256, (nb, 210), dtype=np.uint8)
    if equal_pairs:
        raw[:, 193:208:2] = raw[:, 192:208:2]
    raw[:, 208:210] = RNG.uniform(1e-4, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return raw


def test_dequantize_q6_k_follows_reference_loop(built):
    raw = q6k_blocks(37)
    assert np.array_equal(ref.dequantize_q6_k(raw, 37).reshape(37, 256), q6k_reference_loop(raw))


def test_dequantize_q6_k_subscale_order_vs_ggml(built):
    """The reference uses sub-scale 2g for the whole 32-value group; ggml uses
    2g + l/16. They agree exactly when the paired sub-scales are equal."""
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    same = q6k_blocks(8, equal_pairs=True)
    ggml = dequantize(same.reshape(-1), gguf.GGMLQuantizationType.Q6_K).reshape(8, 256)
    assert np.array_equal(ref.dequantize_q6_k(same, 8).reshape(8, 256), ggml.astype(np.float32))
    diff = q6k_blocks(8)
    ggml = dequantize(diff.reshape(-1), gguf.GGMLQuantizationType.Q6_K).reshape(8, 256).astype(np.float32)
    ours = ref.dequantize_q6_k(diff, 8).reshape(8, 256)
    first_half = np.concatenate([np.arange(32 * g, 32 * g + 16) for g in range(8)])
    assert np.array_equal(ours[:, first_half], ggml[:, first_half])
    assert not np.array_equal(ours, ggml)


def test_dequant_matmul_f16_serial_order(built):
    b, m, n, k = 1, 3, 5, 37
    a = RNG.uniform(-1, 1, (b * m, k)).astype(np.float32)
    w = RNG.uniform(-1, 1, (n, k)).astype(np.float16)
    acc = np.zeros((b * m, n), np.float32)
    wf = w.astype(np.float32)
    for kk in range(k):  # total += a[kk] * f32(w[kk]), f32 rounding at each step
        acc = (acc + (a[:, kk, None] * wf[None, :, kk]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(ref.dequant_matmul_f16_f32(a, w.view(np.uint16), b, m, n, k), acc)

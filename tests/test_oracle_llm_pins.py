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
    """shape_ops.rs:2848-2899 transcribed: scales[8n + {0,2,4,6}] for every l,
    and `let scales = &block[192..208]` is a `&[u8]`, so `scales[i] as i32`
    zero-extends: the sub-scales are unsigned 0..255."""
    nb = raw.shape[0]
    out = np.empty((nb, 256), np.float32)
    d = raw[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(nb)
    sc = raw[:, 192:208].astype(np.int32)
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


def q6k_known_block(d_bits):
    """One hand-built Q6_K block: ql[0] = 0x21, ql[32] = 0x43, qh[0] = 0xE4,
    every other ql/qh byte 0; sub-scale bytes scales[0] = 0x80,
    scales[2] = 0xC0, scales[4] = 0xFF, scales[6] = 0x01, scales[8] = 0x7F,
    the rest 0; f16 d from `d_bits`."""
    blk = np.zeros(210, np.uint8)
    blk[0], blk[32], blk[128] = 0x21, 0x43, 0xE4
    blk[192], blk[194], blk[196], blk[198], blk[200] = 0x80, 0xC0, 0xFF, 0x01, 0x7F
    blk[208], blk[209] = d_bits & 0xFF, d_bits >> 8
    return blk


def q6k_known_answer(d):
    """Expected output of q6k_known_block, written out from the Rust loop
    (shape_ops.rs:2870-2895) by hand. For n = 0, l = 0:
      q1 = (0x21 & 0xF | ((0xE4 >> 0) & 3) << 4) - 32 = (1 | 0) - 32 = -31
      q2 = (0x43 & 0xF | ((0xE4 >> 2) & 3) << 4) - 32 = (3 | 16) - 32 = -13
      q3 = (0x21 >> 4  | ((0xE4 >> 4) & 3) << 4) - 32 = (2 | 32) - 32 = 2
      q4 = (0x43 >> 4  | ((0xE4 >> 6) & 3) << 4) - 32 = (4 | 48) - 32 = 20
    and the sub-scales `scales[i] as i32` of u8 bytes: s1 = 0x80 = 128,
    s2 = 0xC0 = 192, s3 = 0xFF = 255, s4 = 0x01 = 1 (int8 would read -128,
    -64, -1, 1). out = d * (s * q) as f32:
      out[0] = 128 * -31 = -3968, out[32] = 192 * -13 = -2496,
      out[64] = 255 * 2 = 510,     out[96] = 1 * 20 = 20.
    Every other l of n = 0 has ql = qh = 0, q = -32: 128 * -32 = -4096,
    192 * -32 = -6144, 255 * -32 = -8160, 1 * -32 = -32. For n = 1 all q are
    -32 with s = scales[8] = 127 (values 128..159: -4064) and
    scales[10 / 12 / 14] = 0 (values 160..255: 0)."""
    out = np.zeros(256, np.float64)
    out[0:32], out[32:64], out[64:96], out[96:128] = -4096, -6144, -8160, -32
    out[0], out[32], out[64], out[96] = -3968, -2496, 510, 20
    out[128:160] = -4064
    return (out * d).astype(np.float32)


@pytest.mark.parametrize("d_bits,d", [(0x3C00, 1.0), (0x3000, 0.125), (0xB800, -0.5)])
def test_dequantize_q6_k_known_answer_unsigned_subscales(built, d_bits, d):
    got = ref.dequantize_q6_k(q6k_known_block(d_bits)[None, :], 1).reshape(256)
    assert np.array_equal(got, q6k_known_answer(d))


def test_dequantize_q6_k_subscale_order_vs_ggml(built):
    """The reference uses sub-scale 2g for the whole 32-value group; ggml uses
    2g + l/16. It also reads the sub-scale bytes unsigned where ggml reads
    int8. The two agree exactly when the paired sub-scales are equal and
    every sub-scale byte is below 0x80."""
    gguf = pytest.importorskip("gguf")
    from gguf.quants import dequantize
    same = q6k_blocks(8, equal_pairs=True)
    same[:, 192:208] &= 0x7F
    ggml = dequantize(same.reshape(-1), gguf.GGMLQuantizationType.Q6_K).reshape(8, 256)
    assert np.array_equal(ref.dequantize_q6_k(same, 8).reshape(8, 256), ggml.astype(np.float32))
    # a sub-scale byte >= 0x80 is s under the reference, s - 256 under ggml
    neg = same.copy()
    neg[:, 192:194] |= 0x80
    ggml = dequantize(neg.reshape(-1), gguf.GGMLQuantizationType.Q6_K).reshape(8, 256).astype(np.float32)
    ours = ref.dequantize_q6_k(neg, 8).reshape(8, 256)
    assert np.array_equal(ours[:, 32:], ggml[:, 32:])
    s = neg[:, 192].astype(np.float64)
    np.testing.assert_allclose(ours[:, :32].astype(np.float64) * (s - 256)[:, None] / s[:, None],
                               ggml[:, :32], rtol=1e-6)
    diff = q6k_blocks(8)
    diff[:, 192:208] &= 0x7F
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

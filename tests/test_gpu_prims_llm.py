"""LLM helper NIFs on the GPU (rope, softmax, silu(gate) * up, Q6_K
dequantisation, f16-weight matmul) vs the oracle's restatement of
shape_ops.rs.

Bit-exact: dequantize_q6_k (one f32 product per value) and
dequant_matmul_f16_f32 (the reference's serial k-order chain, products and
sums rounded separately). Tolerances: rope 2e-6 (CUDA cosf / sinf against
glibc's, each within 2 ulp), silu(gate) * up 1e-6 relative (expf), softmax
2e-6 relative to the exact (f64) softmax, and against the oracle the larger
of 1e-5 and inner * 2^-24 (the error bound of the reference's serial f32
sum).
"""
import numpy as np
import pytest

import ref
from arm_ai_b200 import prims
from arm_ai_b200.native import NifError

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(77)


def inv_freq(head_dim, base=10000.0):
    return (1.0 / base ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)).astype(np.float32)


@pytest.mark.parametrize("tokens,heads,hd", [(1, 32, 64), (7, 8, 128), (512, 4, 64), (3, 1, 2)])
def test_rope_matches_oracle(built, tokens, heads, hd):
    x = RNG.uniform(-1, 1, (tokens * heads, hd)).astype(np.float32)
    pos = RNG.integers(0, 8192, tokens).astype(np.int64)
    f = inv_freq(hd)
    got = prims.rope_f32_op(x, pos, f, tokens * heads, hd, heads).reshape(tokens * heads, hd)
    exp = ref.rope_f32(x, pos, f, tokens * heads, hd, heads)
    np.testing.assert_allclose(got, exp, rtol=0, atol=2e-6)


def test_rope_position_zero_is_identity(built):
    x = RNG.uniform(-1, 1, (4, 64)).astype(np.float32)
    got = prims.rope_f32_op(x, np.zeros(4, np.int64), inv_freq(64), 4, 64, 1)
    assert np.array_equal(got, x.reshape(-1))


@pytest.mark.parametrize("outer,inner", [(1, 1), (3, 7), (64, 4096), (2, 32000), (1000, 33)])
def test_softmax_matches_oracle(built, outer, inner):
    x = RNG.normal(0, 4, (outer, inner)).astype(np.float32)
    got = prims.softmax_last_axis_f32_op(x, outer, inner).reshape(outer, inner)
    exp = ref.softmax_last_axis_f32(x, outer, inner)
    # the reference normalises by a serial f32 sum, whose relative error is
    # bounded by inner * 2^-24; the parallel sum is far closer to exact.
    # "exact": f64 from the f32-rounded x - max that both compute
    diff = (x - x.max(axis=1, keepdims=True)).astype(np.float32).astype(np.float64)
    exact = np.exp(diff)
    exact /= exact.sum(axis=1, keepdims=True)
    np.testing.assert_allclose(got, exact, rtol=2e-6, atol=1e-30)
    np.testing.assert_allclose(got, exp, rtol=max(1e-5, inner * 2.0 ** -24), atol=1e-30)


def test_softmax_nan_and_inf_rows(built):
    x = np.array([[np.nan, 1, 2], [1, np.nan, 2], [-np.inf, 0, 1], [-np.inf, -np.inf, -np.inf]], np.float32)
    got = prims.softmax_last_axis_f32_op(x, 4, 3).reshape(4, 3)
    exp = ref.softmax_last_axis_f32(x, 4, 3)
    assert np.array_equal(np.isnan(got), np.isnan(exp))
    ok = ~np.isnan(exp)
    np.testing.assert_allclose(got[ok], exp[ok], rtol=1e-6)


@pytest.mark.parametrize("n", [1, 1000, 5632 * 16, 14336])
def test_silu_gate_mul_up_matches_oracle(built, n):
    g = RNG.normal(0, 3, n).astype(np.float32)
    u = RNG.normal(0, 1, n).astype(np.float32)
    got = prims.silu_gate_mul_up_f32_op(g, u)
    np.testing.assert_allclose(got, ref.silu_gate_mul_up_f32(g, u), rtol=1e-6, atol=1e-37)


def q6k_blocks(nb):
    raw = RNG.integers(0, 256, (nb, 210), dtype=np.uint8)
    d = RNG.uniform(1e-4, 1e-2, nb).astype(np.float16)
    raw[:, 208:210] = d.view(np.uint8).reshape(nb, 2)
    return raw


@pytest.mark.parametrize("nb", [1, 3, 4096])
def test_dequantize_q6_k_bit_exact(built, nb):
    raw = q6k_blocks(nb)
    # at least half of the sub-scale bytes at or above 0x80, where an int8
    # reading of the reference's u8 scales would differ
    raw[:, 192:208:2] |= 0x80
    assert (raw[:, 192:208] >= 0x80).mean() >= 0.5
    got = prims.dequantize_q6_k_op(raw.tobytes(), nb * 256)
    assert np.array_equal(got, ref.dequantize_q6_k(raw, nb))


def test_dequantize_q6_k_known_answer(built):
    """Hand-derived values (tests/test_oracle_llm_pins.py: q6k_known_answer)
    for sub-scale bytes 0x80, 0xC0 and 0xFF, read unsigned as the reference's
    `scales[i] as i32` over a `&[u8]` does."""
    from test_oracle_llm_pins import q6k_known_answer, q6k_known_block
    raw = np.stack([q6k_known_block(0x3C00), q6k_known_block(0x3000), q6k_known_block(0xB800)])
    got = prims.dequantize_q6_k_op(raw.tobytes(), 3 * 256).reshape(3, 256)
    for i, d in enumerate((1.0, 0.125, -0.5)):
        assert np.array_equal(got[i], q6k_known_answer(d))


@pytest.mark.parametrize("b,m,n,k", [(1, 1, 4096, 4096), (1, 3, 100, 33), (2, 16, 512, 1024), (1, 64, 2048, 256)])
def test_dequant_matmul_f16_bit_exact(built, b, m, n, k):
    a = RNG.uniform(-1, 1, (b * m, k)).astype(np.float32)
    w = RNG.uniform(-1, 1, (n, k)).astype(np.float16)
    got = prims.dequant_matmul_f16_f32_op(a, w, b, m, n, k).reshape(b * m, n)
    assert np.array_equal(got, ref.dequant_matmul_f16_f32(a, w.view(np.uint16), b, m, n, k))


def test_llm_helper_errors_and_empty(built):
    with pytest.raises(NifError, match=r"rope: head_dim 3 must be even"):
        prims.rope_f32_op(np.zeros(3, np.float32), [0], np.zeros(1, np.float32), 1, 3, 1)
    with pytest.raises(NifError, match=r"rope: inv_freq len 1 != head_dim/2 = 2"):
        prims.rope_f32_op(np.zeros(4, np.float32), [0], np.zeros(1, np.float32), 1, 4, 1)
    with pytest.raises(NifError, match=r"rope: n_rows 2 != n_tokens \* heads_per_token = 1"):
        prims.rope_f32_op(np.zeros(8, np.float32), [0], np.zeros(2, np.float32), 2, 4, 1)
    with pytest.raises(NifError, match=r"dequant_matmul_f16: weights len 3 != N\*K = 4"):
        prims.dequant_matmul_f16_f32_op(np.zeros(2, np.float32), np.zeros(3, np.uint16), 1, 1, 2, 2)
    with pytest.raises(NifError, match=r"softmax: inner must be positive"):
        prims.softmax_last_axis_f32_op(np.zeros(0, np.float32), 0, 0)
    with pytest.raises(NifError, match=r"silu_gate_mul_up: up len 2 != gate len 3"):
        prims.silu_gate_mul_up_f32_op(np.zeros(3, np.float32), np.zeros(2, np.float32))
    with pytest.raises(NifError, match=r"dequantize_q6_k: n_elements 255 != 256 \* blocks = 256"):
        prims.dequantize_q6_k_op(bytes(210), 255)
    assert prims.softmax_last_axis_f32_op(np.zeros(0, np.float32), 0, 5).size == 0
    assert prims.dequantize_q6_k_op(bytes(209), 0).size == 0
    assert prims.dequant_matmul_f16_f32_op(np.zeros(0, np.float32), np.zeros(0, np.uint16), 0, 1, 0, 0).size == 0

"""Primitive NIFs on the GPU vs the oracle's restatement of shape_ops.rs.

Bit-exact: every integer output (s32 accumulators, int8 / int4 quantisation)
and the f32 outputs whose reference order the kernels reproduce (int8 scale
products, int4 f32 / q4xq8 sequential group folds, the weight-only int8 dot).
Tolerances: rmsnorm 2e-6 relative (parallel sum of squares); flash attention
2e-5 absolute for f32 inputs, 2e-3 for f16 inputs against the f32 oracle on
the f16-rounded values.
"""
import numpy as np
import pytest

import ref
from arm_ai_b200 import prims
from arm_ai_b200.native import NifError

pytestmark = pytest.mark.gpu
RNG = np.random.default_rng(2026)


def i8(shape):
    return RNG.integers(-127, 128, size=shape, dtype=np.int8)


# M >= 64 runs the tcgen05 kind::i8 kernel (TMA boxes of 128 x 128 bytes,
# zero-filled past the edges): ragged M / N / K cover its tile edges.
@pytest.mark.parametrize("m,n,k", [(1, 2048, 2048), (16, 4096, 4096), (512, 2048, 2048), (3, 100, 48),
                                   (512, 4096, 4096), (64, 256, 272), (200, 300, 144), (130, 129, 4112)])
def test_int8_gemm_bit_exact(built, m, n, k):
    a, w = i8((m, k)), i8((n, k))
    ws = RNG.uniform(1e-3, 1e-1, n).astype(np.float32)
    acs = RNG.uniform(1e-3, 1e-1, m).astype(np.float32)
    assert np.array_equal(prims.int8_matmul_s32(a, w, m, n, k).reshape(m, n), ref.int8_matmul_s32(a, w, m, n, k))
    got = prims.int8_matmul_f32_op(a, w, ws, 0.0125, m, n, k).reshape(m, n)
    exp = ref.int8_matmul_f32(a, w, np.float32(0.0125), ws, m, n, k)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
    got = prims.int8_matmul_f32_per_token_op(a, w, acs, ws, m, n, k).reshape(m, n)
    exp = ref.int8_matmul_f32_per_token(a, w, acs, ws, m, n, k)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_quantize_int8_per_token_bit_exact(built):
    a = RNG.uniform(-1, 1, (17, 4096)).astype(np.float32)
    a[3] = 0
    a[5, 7] = 1e-30
    q, s = prims.quantize_int8_per_token_op(a, 17, 4096)
    rq, rs = ref.quantize_int8_per_token(a, 17, 4096)
    assert np.array_equal(q.reshape(17, 4096), rq) and np.array_equal(s.view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 1), (14336, 4096, 1), (64, 256, 5)])
def test_int4_f32_bit_exact(built, n, k, m):
    w = RNG.uniform(-1, 1, (n, k)).astype(np.float32)
    packed, scales = ref.quantize_int4_q4_0(w, n, k)
    gp, gs = prims.quantize_int4_q4_0_op(w, n, k)
    assert np.array_equal(gp.reshape(n, k // 2), packed) and np.array_equal(gs.reshape(n, -1).view(np.uint32),
                                                                            scales.view(np.uint32))
    a = RNG.uniform(-1, 1, (m, k)).astype(np.float32)
    got = prims.int4_matmul_f32_op(a, packed, scales, m, n, k).reshape(m, n)
    exp = ref.int4_matmul_f32(a, packed, scales, m, n, k)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
    if m == 1:
        g2 = prims.int4_matmul_gemv_neon_op(a, packed, scales, n, k)
        assert np.array_equal(g2.view(np.uint32), exp[0].view(np.uint32))
        g3 = prims.int4_matmul_gemv_q4_x_q8_neon_op(a, packed, scales, n, k)
        e3 = ref.int4_matmul_q4_x_q8(a, packed, scales, n, k)
        assert np.array_equal(g3.view(np.uint32), e3.view(np.uint32))


def test_rmsnorm_matches(built):
    x = RNG.uniform(-1, 1, (512, 4096)).astype(np.float32)
    g = RNG.uniform(0.5, 1.5, 4096).astype(np.float32)
    got = prims.rmsnorm_f32_op(x, g, 512, 4096, 1e-5).reshape(512, 4096)
    exp = ref.rmsnorm_f32(x, g, 512, 4096, np.float32(1e-5))
    assert np.max(np.abs(got - exp) / np.maximum(np.abs(exp), 1e-30)) < 2e-6


@pytest.mark.parametrize("causal", [True, False])
def test_flash_attention_f32(built, causal):
    b, h, s, d = 1, 4, 200, 64
    q, k, v = (RNG.uniform(-1, 1, (b, h, s, d)).astype(np.float32) for _ in range(3))
    scale = 1.0 / np.sqrt(d)
    got = prims.flash_attention_f32_op(q, k, v, scale, b, h, s, s, d, causal).reshape(b, h, s, d)
    exp = ref.flash_attention_f32(q, k, v, np.float32(scale), b, h, s, s, d, causal)
    assert np.max(np.abs(got - exp)) < 2e-5


def test_dequant_matmul_int8_bit_exact(built):
    b, m, n, k = 2, 3, 257, 1024
    act = RNG.uniform(-1, 1, (b * m, k)).astype(np.float32)
    w = i8((n, k))
    sc = RNG.uniform(1e-3, 1e-1, n).astype(np.float32)
    got = prims.dequant_matmul_int8_f32_op(act, w, sc, b, m, n, k).reshape(b * m, n)
    exp = ref.dequant_matmul_int8_f32(act, w, sc, b, m, n, k)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_length_errors_use_reference_wording(built):
    with pytest.raises(NifError, match=r"int8_matmul: a len 3 != M\*K = 4"):
        prims.int8_matmul_f32_op(np.zeros(3, np.int8), np.zeros(4, np.int8), np.zeros(1, np.float32), 1.0, 1, 1, 4)
    with pytest.raises(NifError, match="int4_matmul: K=40 must be multiple of 32"):
        prims.int4_matmul_f32_op(np.zeros(40, np.float32), np.zeros(20, np.uint8), np.zeros(1, np.float32), 1, 1, 40)
    with pytest.raises(NifError, match="rmsnorm: gamma len 3 != inner 4"):
        prims.rmsnorm_f32_op(np.zeros(8, np.float32), np.zeros(3, np.float32), 2, 4, 1e-5)
    with pytest.raises(NifError, match=r"flash_attn: q len 1 != B\*H\*Sq\*D = 2"):
        prims.flash_attention_f32_op(np.zeros(1, np.float32), np.zeros(2, np.float32), np.zeros(2, np.float32),
                                     1.0, 1, 1, 1, 1, 2, True)

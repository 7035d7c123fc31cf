"""Bit-exact checks of the CUDA k-quant building blocks against the oracle.

Integer work (Q8_K bytes and bsums, per-super-block integer dot products) must
be identical; QMatMul's f32 output differs from candle's only in the order of
the f32 combine of exact integers, so it is held to 2e-6 of the magnitude
sum (sum_i |w_i x_i|).
"""
import ctypes

import numpy as np
import pytest

import ref
from arm_ai_b200 import kquant
from arm_ai_b200._lib import load_synth

pytestmark = pytest.mark.gpu


def _rows(qtype, rows, k, seed, std=0.02):
    lib = load_synth()
    bb = 144 if qtype == kquant.Q4_K else 210
    out = np.empty((rows, (k // 256) * bb), dtype=np.uint8)
    assert lib.synth_tensor(ctypes.c_uint64(seed), rows, k, ctypes.c_float(std), qtype,
                            out.ctypes.data_as(ctypes.c_void_p)) == 0
    return out


def _activations(m, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[0, :256] = 0.0                                   # all-zero block
    if m > 1:
        x[1, :256] = np.float32(0.75)                  # every value ties on |x|
        x[1, 44] = np.float32(-0.75)
    if m > 2:
        # max |x| = 2 -> iscale = 64; 64 * (i + 0.5)/64 = i + 0.5 exactly, so
        # every value sits on a rounding tie (half away from zero).
        x[2, 0] = np.float32(-2.0)
        x[2, 1:256] = (np.arange(255, dtype=np.float32) - 127 + np.float32(0.5)) / np.float32(64.0)
    return x


@pytest.mark.parametrize("k", [256, 2048, 5632])
def test_q8k_quantize_bit_exact(built, k):
    x = _activations(5, k, k)
    ours = kquant.quantize_q8k(x)
    theirs = ref.quantize_q8k(x)
    assert np.array_equal(ours["qs"], theirs["qs"])
    assert np.array_equal(ours["bsums"], theirs["bsums"])
    assert np.array_equal(ours["d"].view(np.uint32), theirs["d"].view(np.uint32))


def _q6k_subscales(w):
    """The int8 sub-scales of every Q6_K super-block of rows `w`."""
    return w.reshape(-1, 210)[:, 192:208].view(np.int8)


def _random_q6k_rows(rows, k, seed):
    """Q6_K rows of random bytes (every ql / qh / sub-scale byte, so sub-scales
    span -128..127) with finite f16 d of either sign."""
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, (rows * (k // 256), 210), dtype=np.uint8)
    d = (rng.uniform(1e-5, 1e-3, raw.shape[0]) * rng.choice([-1, 1], raw.shape[0])).astype(np.float16)
    raw[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return raw.reshape(rows, -1)


def test_synthetic_q6k_has_negative_subscales(built):
    sc = _q6k_subscales(_rows(kquant.Q6_K, 64, 2048, seed=1))
    assert 0.3 < (sc < 0).mean() < 0.7


@pytest.mark.parametrize("qtype", [kquant.Q4_K, kquant.Q6_K, "q6k_random"])
@pytest.mark.parametrize("k", [2048, 5632])
def test_block_dots_bit_exact(built, qtype, k):
    if qtype == "q6k_random":
        qtype, w = kquant.Q6_K, _random_q6k_rows(37, k, seed=k)
    else:
        w = _rows(qtype, 37, k, seed=k + qtype)
    if qtype == kquant.Q6_K:
        assert (_q6k_subscales(w) < 0).mean() > 0.3
    q8 = ref.quantize_q8k(_activations(3, k, 7))
    isum, msum = kquant.block_dots(qtype, w, k, q8)
    risum, rmsum = ref.block_ints(qtype, w, q8, k)
    assert np.array_equal(isum, risum)
    if qtype == kquant.Q4_K:
        assert np.array_equal(msum, rmsum)


@pytest.mark.parametrize("qtype", [kquant.Q4_K, kquant.Q6_K])
@pytest.mark.parametrize("k,n,m", [(2048, 2560, 1), (5632, 2048, 1), (2048, 300, 11)])
def test_qmatmul_matches_oracle(built, qtype, k, n, m):
    w = _rows(qtype, n, k, seed=n + k)
    x = _activations(m, k, 3)
    ours = kquant.qmatmul(qtype, w, k, x)
    theirs = ref.qmatmul(qtype, w, k, x)
    deq = ref.dequant_rows(qtype, w, k).astype(np.float64)
    q8 = ref.quantize_q8k(x)
    xq = (q8["qs"].astype(np.float64) * q8["d"][..., None]).reshape(m, k)
    mag = np.abs(xq) @ np.abs(deq).T
    assert np.all(np.abs(ours - theirs) <= 2e-6 * mag + 1e-12)


def _f16_operands(qtype, w, k, x):
    """The prefill GEMM's operands in f64: Q8_K q * d rounded to f16, and the
    dequantised weights rounded to f16."""
    q8 = ref.quantize_q8k(x)
    a = (q8["qs"].astype(np.float32) * q8["d"][..., None].astype(np.float32)).astype(np.float16)
    a = a.reshape(x.shape[0], k).astype(np.float64)
    wd = ref.dequant_rows(qtype, w, k).astype(np.float16).astype(np.float64)
    return a, wd


@pytest.mark.parametrize("qtype", [kquant.Q4_K, kquant.Q6_K, "q6k_random"])
@pytest.mark.parametrize("k,n,m", [(256, 128, 128), (2048, 384, 200), (5632, 256, 77), (2048, 1000, 5)])
def test_qgemm_tensor_cores(built, qtype, k, n, m):
    """tcgen05 prefill GEMM: exactly the f16 operands' product up to the f32
    summation order (2e-6 of the magnitude sum), ragged m and n included.
    Q6_K rows carry negative sub-scales (synthetic: about half; random bytes:
    the full int8 range)."""
    if qtype == "q6k_random":
        qtype, w = kquant.Q6_K, _random_q6k_rows(n, k, seed=7 * n + k)
    else:
        w = _rows(qtype, n, k, seed=7 * n + k)
    if qtype == kquant.Q6_K:
        assert (_q6k_subscales(w) < 0).mean() > 0.3
    x = _activations(m, k, 5)
    ours = kquant.qgemm(qtype, w, k, x)
    a, wd = _f16_operands(qtype, w, k, x)
    exact = a @ wd.T
    mag = np.abs(a) @ np.abs(wd).T
    assert np.all(np.abs(ours - exact) <= 2e-6 * mag + 1e-12)
    # and against candle's integer path (QMatMul) at f16 precision
    theirs = ref.qmatmul(qtype, w, k, x)
    assert np.all(np.abs(ours - theirs) <= 2e-3 * mag + 1e-9)


def test_qgemm_with_rms_norm(built):
    k, n, m = 2048, 256, 130
    w = _rows(kquant.Q4_K, n, k, seed=99)
    rng = np.random.default_rng(8)
    x = rng.standard_normal((m, k)).astype(np.float32)
    g = (1.0 + 0.05 * rng.standard_normal(k)).astype(np.float32)
    ours = kquant.qgemm(kquant.Q4_K, w, k, x, gamma=g, eps=1e-5)
    xn = (x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=1, keepdims=True) + 1e-5) * g).astype(np.float32)
    a, wd = _f16_operands(kquant.Q4_K, w, k, xn)
    mag = np.abs(a) @ np.abs(wd).T
    # one activation may round the other way (norm summation order): 2e-3
    assert np.all(np.abs(ours - a @ wd.T) <= 2e-3 * mag + 1e-9)

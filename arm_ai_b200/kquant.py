"""k-quant building blocks of the CUDA path, through the C ABI.

These call the same device code the decode kernels run and exist so that the
integer parts (Q8_K bytes, bsums, per-super-block integer dot products) can be
checked bit for bit against the CPU oracle.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import check, load_cuda, ptr

Q4_K, Q6_K = 12, 14
Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])


def quantize_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    rows = x.reshape(-1, k)
    out = np.zeros((rows.shape[0], k // 256), dtype=Q8K_DTYPE)
    check(load_cuda().armai_quantize_q8k(ptr(rows), rows.shape[0], k, ptr(out)))
    return out


def block_dots(wtype: int, w_rows: np.ndarray, k: int, q8: np.ndarray):
    w_rows = np.ascontiguousarray(w_rows, dtype=np.uint8)
    q8 = np.ascontiguousarray(q8, dtype=Q8K_DTYPE)
    n, m, nb = w_rows.shape[0], q8.shape[0], k // 256
    isum = np.zeros((m, n, nb), dtype=np.int32)
    msum = np.zeros((m, n, nb), dtype=np.int32)
    check(load_cuda().armai_kquant_block_dots(ptr(w_rows), wtype, n, k, ptr(q8), m, ptr(isum), ptr(msum)))
    return isum, (msum if wtype == Q4_K else None)


def qmatmul(wtype: int, w_rows: np.ndarray, k: int, x: np.ndarray) -> np.ndarray:
    w_rows = np.ascontiguousarray(w_rows, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    out = np.empty((x.shape[0], w_rows.shape[0]), dtype=np.float32)
    check(load_cuda().armai_qmatmul(ptr(w_rows), wtype, w_rows.shape[0], k, ptr(x), x.shape[0], ptr(out)))
    return out


def qgemm(wtype: int, w_rows: np.ndarray, k: int, x: np.ndarray, gamma=None, eps: float = 1e-5) -> np.ndarray:
    """Prefill tensor-core GEMM (armai_qgemm): x [m, k] f32 (rms-normalised
    with gamma when given) quantised per token to Q8_K and expanded to f16,
    times the f16-dequantised weight rows: [m, n] f32."""
    w_rows = np.ascontiguousarray(w_rows, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, k)
    g = None if gamma is None else np.ascontiguousarray(gamma, dtype=np.float32)
    out = np.empty((x.shape[0], w_rows.shape[0]), dtype=np.float32)
    check(load_cuda().armai_qgemm(ptr(w_rows), wtype, w_rows.shape[0], k, ptr(x), x.shape[0], ptr(g),
                                  ctypes.c_float(eps), ptr(out)))
    return out

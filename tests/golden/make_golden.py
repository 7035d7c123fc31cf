"""Regenerate the committed golden fixtures of tests/golden/.

q4k_golden.npz / q6k_golden.npz: seeded random GGML Q4_K / Q6_K rows (every
scale/min/nibble byte random, f16 super-scales drawn from a normal range)
and their f32 dequantisation by gguf-py 0.19.0 (gguf.quants), the GGML
format's own Python implementation. They pin the block layouts used by the
oracle and by the CUDA embedding/dequant code.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    import gguf
    rng = np.random.default_rng(20261201)
    k, rows = 512, 24
    # Q4_K: f16 d, f16 dmin, 12 B scales, 128 B nibbles
    raw = rng.integers(0, 256, size=(rows, (k // 256) * 144), dtype=np.uint8)
    blocks = raw.reshape(rows, k // 256, 144)
    d = (rng.standard_normal((rows, k // 256)) * 1e-3).astype(np.float16)
    dm = np.abs(rng.standard_normal((rows, k // 256)) * 1e-3).astype(np.float16)
    blocks[:, :, 0:2] = d.view(np.uint8).reshape(rows, k // 256, 2)
    blocks[:, :, 2:4] = dm.view(np.uint8).reshape(rows, k // 256, 2)
    deq = gguf.dequantize(raw, gguf.GGMLQuantizationType.Q4_K).astype(np.float32).reshape(rows, k)
    np.savez_compressed(os.path.join(HERE, "q4k_golden.npz"), raw=raw, deq=deq, k=np.int64(k))
    # Q6_K: 128 B ql, 64 B qh, 16 i8 scales, f16 d
    raw6 = rng.integers(0, 256, size=(rows, (k // 256) * 210), dtype=np.uint8)
    b6 = raw6.reshape(rows, k // 256, 210)
    d6 = (rng.standard_normal((rows, k // 256)) * 1e-3).astype(np.float16)
    b6[:, :, 208:210] = d6.view(np.uint8).reshape(rows, k // 256, 2)
    deq6 = gguf.dequantize(raw6, gguf.GGMLQuantizationType.Q6_K).astype(np.float32).reshape(rows, k)
    np.savez_compressed(os.path.join(HERE, "q6k_golden.npz"), raw=raw6, deq=deq6, k=np.int64(k))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()

"""Test models whose matrices use the other GGML weight types candle's
loader accepts (Q4_0, Q5_0, Q8_0, Q5_K) beside Q4_K / Q6_K. Test
infrastructure: the legacy types are quantised by gguf-py; Q5_K by
quantize_q5k below (a plain per-sub-block affine encoding — any valid Q5_K
block serves a synthetic model)."""
from __future__ import annotations

import os

import numpy as np

from arm_ai_b200 import synth

GGML = {"Q4_0": 2, "Q5_0": 6, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}


def quantize_q5k(x: np.ndarray) -> np.ndarray:
    """Rows of x (length % 256 == 0) as Q5_K blocks: value = d*sc*q - dmin*m,
    q in [0, 31], 6-bit sc and m per 32-value sub-block, f16 d and dmin."""
    x = np.asarray(x, dtype=np.float32)
    rows, k = x.shape
    sb = x.reshape(rows, k // 256, 8, 32)
    lo = np.minimum(sb.min(axis=-1), 0.0)
    hi = sb.max(axis=-1)
    scale = np.maximum(hi - lo, 1e-12) / 31.0
    mins = -lo
    d = (scale.max(axis=-1) / 63.0).astype(np.float16)
    dmin = (mins.max(axis=-1) / 63.0).astype(np.float16)
    df, dminf = d.astype(np.float32)[..., None], dmin.astype(np.float32)[..., None]
    sc = np.clip(np.rint(scale / np.where(df > 0, df, 1)), 0, 63).astype(np.int32)
    mm = np.clip(np.rint(mins / np.where(dminf > 0, dminf, 1)), 0, 63).astype(np.int32)
    step = (df * sc)[..., None]
    off = (dminf * mm)[..., None]
    q = np.clip(np.rint((sb + off) / np.where(step > 0, step, 1)), 0, 31).astype(np.int32)
    nb = k // 256
    out = np.zeros((rows, nb, 176), dtype=np.uint8)
    out[..., 0:2] = d.reshape(rows, nb, 1).view(np.uint8).reshape(rows, nb, 2)
    out[..., 2:4] = dmin.reshape(rows, nb, 1).view(np.uint8).reshape(rows, nb, 2)
    s12 = np.zeros((rows, nb, 12), dtype=np.int32)
    for j in range(4):
        s12[..., j] = sc[..., j] | ((sc[..., j + 4] >> 4) << 6)
        s12[..., j + 4] = mm[..., j] | ((mm[..., j + 4] >> 4) << 6)
        s12[..., j + 8] = (sc[..., j + 4] & 0xF) | ((mm[..., j + 4] & 0xF) << 4)
    out[..., 4:16] = s12.astype(np.uint8)
    qv = q.reshape(rows, nb, 256)
    qh = np.zeros((rows, nb, 32), dtype=np.int32)
    qs = np.zeros((rows, nb, 128), dtype=np.int32)
    for g in range(4):
        a, b = qv[..., 64 * g: 64 * g + 32], qv[..., 64 * g + 32: 64 * g + 64]
        qs[..., 32 * g: 32 * g + 32] = (a & 0xF) | ((b & 0xF) << 4)
        qh |= ((a >> 4) << (2 * g)) | ((b >> 4) << (2 * g + 1))
    out[..., 16:48] = qh.astype(np.uint8)
    out[..., 48:176] = qs.astype(np.uint8)
    return out.reshape(rows, nb * 176)


def _quantize(x: np.ndarray, tname: str) -> np.ndarray:
    import gguf
    from gguf.quants import quantize
    if tname == "Q5_K":
        return quantize_q5k(x)
    return quantize(x, gguf.GGMLQuantizationType[tname])


def write_mixed_model(path: str, arch_name: str, seed: int, types: dict[str, str]) -> str:
    """A random-init GGUF of arch_name whose tensors named in `types`
    (e.g. "attn_q", "ffn_up", "output", "token_embd"; per layer or all
    layers) use the given GGML type; the others follow synth.quant_type."""
    import gguf
    if os.path.exists(path):
        return path
    a = synth.ARCHS[arch_name]
    rng = np.random.default_rng(seed)
    w = gguf.GGUFWriter(path + ".tmp", "llama")
    w.add_name(f"armai-mixed-{arch_name}-s{seed}")
    w.add_block_count(a.n_layer)
    w.add_context_length(a.context_length)
    w.add_embedding_length(a.n_embd)
    w.add_feed_forward_length(a.n_ff)
    w.add_head_count(a.n_head)
    w.add_head_count_kv(a.n_head_kv)
    w.add_rope_dimension_count(a.head_dim)
    w.add_layer_norm_rms_eps(a.eps)
    w.add_rope_freq_base(a.rope_theta)

    def mat(name, layer, rows, k):
        full = name if layer is None else f"blk.{layer}.{name}"
        tname = types.get(name)
        if tname is None:
            tname = "Q6_K" if synth.quant_type(name, layer) == synth.Q6_K else "Q4_K"
        x = rng.normal(0.0, 0.02, (rows, k)).astype(np.float32)
        w.add_tensor(full + ".weight", _quantize(x, tname), raw_dtype=gguf.GGMLQuantizationType[tname])

    def norm(name, n):
        w.add_tensor(name, (1.0 + rng.normal(0.0, 0.05, n)).astype(np.float32))

    hd = a.head_dim
    mat("token_embd", None, a.n_vocab, a.n_embd)
    for l in range(a.n_layer):
        norm(f"blk.{l}.attn_norm.weight", a.n_embd)
        mat("attn_q", l, a.n_head * hd, a.n_embd)
        mat("attn_k", l, a.n_head_kv * hd, a.n_embd)
        mat("attn_v", l, a.n_head_kv * hd, a.n_embd)
        mat("attn_output", l, a.n_embd, a.n_head * hd)
        norm(f"blk.{l}.ffn_norm.weight", a.n_embd)
        mat("ffn_gate", l, a.n_ff, a.n_embd)
        mat("ffn_up", l, a.n_ff, a.n_embd)
        mat("ffn_down", l, a.n_embd, a.n_ff)
    norm("output_norm.weight", a.n_embd)
    mat("output", None, a.n_vocab, a.n_embd)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    os.replace(path + ".tmp", path)
    return path

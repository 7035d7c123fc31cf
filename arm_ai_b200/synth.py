"""Seeded synthetic Llama-architecture GGUF models (random init, Q4_K_M-style).

The reference's headline numbers use real model files that are not available
here, so benchmarks and parity tests run on random-init models with the
architectures the benchmarks use. Every tensor is drawn N(0, 0.02) from a
seed derived from (model seed, tensor name) and quantised by
``csrc/synth.c``: Q4_K for every 2-D tensor, Q6_K for ``output`` and for
``attn_v`` / ``ffn_down`` on even layers (a stated simplification of
llama.cpp's Q4_K_M mix). Q6_K sub-scales are signed as llama.cpp makes them
(about half negative). Norm gains are f32, 1 + N(0, 0.05).

The file is written with gguf-py's ``GGUFWriter``; the loader in
``libarmai_cuda.so`` parses it with its own reader, so the container format is
cross-checked by construction.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
from dataclasses import dataclass, asdict

import numpy as np

from ._lib import load_synth

Q4_K = 12
Q6_K = 14
F32 = 0


@dataclass(frozen=True)
class LlamaArch:
    n_layer: int
    n_embd: int
    n_ff: int
    n_head: int
    n_head_kv: int
    n_vocab: int
    rope_theta: float = 10000.0
    eps: float = 1e-5
    context_length: int = 4096

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


ARCHS = {
    # the headline b=1 decode and the batched decode workloads
    "tinyllama-1.1b": LlamaArch(22, 2048, 5632, 32, 4, 32000, 10000.0, 1e-5, 2048),
    # configs[2]
    "mistral-7b": LlamaArch(32, 4096, 14336, 32, 8, 32000, 10000.0, 1e-5, 32768),
    # configs[3]
    "llama-3-8b": LlamaArch(32, 4096, 14336, 32, 8, 128256, 500000.0, 1e-5, 8192),
    # small shapes for CPU-checkable parity tests
    "tiny": LlamaArch(2, 256, 512, 4, 2, 1000, 10000.0, 1e-5, 4096),
    "small": LlamaArch(4, 512, 1536, 8, 2, 4096, 10000.0, 1e-5, 4096),
    # head_dim 128 (the Mistral / Llama-3 attention shape) at CPU-checkable size
    "tiny128": LlamaArch(2, 512, 1024, 4, 2, 1000, 500000.0, 1e-5, 8192),
    # tensor parallelism over 4 ranks: 16 / 4 query heads, 4 / 4 KV heads,
    # 256 attn_output columns and 512 FFN rows per rank
    "tp4": LlamaArch(2, 1024, 2048, 16, 4, 4096, 10000.0, 1e-5, 4096),
    # FFN 12288: 16 activation rows of ffn_down's K exceed shared memory, so
    # batched decode runs its 8-row kernels (as for 7B/8B models on one GPU)
    "wide": LlamaArch(1, 256, 12288, 4, 2, 1000, 10000.0, 1e-5, 4096),
}


def tensor_seed(model_seed: int, name: str) -> int:
    h = hashlib.sha256(f"{model_seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little")


def quant_type(name: str, layer: int | None) -> int:
    if name == "output":
        return Q6_K
    if name in ("attn_v", "ffn_down") and layer is not None and layer % 2 == 0:
        return Q6_K
    return Q4_K


def _gen_quant(lib, seed: int, rows: int, k: int, qtype: int, std: float = 0.02) -> np.ndarray:
    bb = 144 if qtype == Q4_K else 210
    out = np.empty((rows, (k // 256) * bb), dtype=np.uint8)
    rc = lib.synth_tensor(ctypes.c_uint64(seed), rows, k, ctypes.c_float(std), qtype,
                          out.ctypes.data_as(ctypes.c_void_p))
    if rc != 0:
        raise ValueError(f"synth_tensor failed ({rc}) for rows={rows} k={k}")
    return out


def _gen_norm(lib, seed: int, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib.synth_fill_normal(out.ctypes.data_as(ctypes.c_void_p), n, ctypes.c_uint64(seed),
                          ctypes.c_float(1.0), ctypes.c_float(0.05))
    return out


def write_model(path: str, arch: LlamaArch, seed: int = 0, tie_output: bool = False) -> str:
    """Write a seeded random-init GGUF model for ``arch`` to ``path``."""
    import gguf  # gguf-py, present in the image

    lib = load_synth()
    a = arch
    tmp = path + ".tmp"
    w = gguf.GGUFWriter(tmp, "llama")
    w.add_name(f"armai-synthetic-seed{seed}")
    w.add_block_count(a.n_layer)
    w.add_context_length(a.context_length)
    w.add_embedding_length(a.n_embd)
    w.add_feed_forward_length(a.n_ff)
    w.add_head_count(a.n_head)
    w.add_head_count_kv(a.n_head_kv)
    w.add_rope_dimension_count(a.head_dim)
    w.add_layer_norm_rms_eps(a.eps)
    w.add_rope_freq_base(a.rope_theta)

    def qt(name, layer, rows, k):
        t = quant_type(name, layer)
        full = name if layer is None else f"blk.{layer}.{name}"
        data = _gen_quant(lib, tensor_seed(seed, full), rows, k, t)
        w.add_tensor(full + ".weight", data, raw_dtype=gguf.GGMLQuantizationType(t))

    qt("token_embd", None, a.n_vocab, a.n_embd)
    hd = a.head_dim
    for l in range(a.n_layer):
        w.add_tensor(f"blk.{l}.attn_norm.weight", _gen_norm(lib, tensor_seed(seed, f"blk.{l}.attn_norm"), a.n_embd))
        qt("attn_q", l, a.n_head * hd, a.n_embd)
        qt("attn_k", l, a.n_head_kv * hd, a.n_embd)
        qt("attn_v", l, a.n_head_kv * hd, a.n_embd)
        qt("attn_output", l, a.n_embd, a.n_head * hd)
        w.add_tensor(f"blk.{l}.ffn_norm.weight", _gen_norm(lib, tensor_seed(seed, f"blk.{l}.ffn_norm"), a.n_embd))
        qt("ffn_gate", l, a.n_ff, a.n_embd)
        qt("ffn_up", l, a.n_ff, a.n_embd)
        qt("ffn_down", l, a.n_embd, a.n_ff)
    w.add_tensor("output_norm.weight", _gen_norm(lib, tensor_seed(seed, "output_norm"), a.n_embd))
    if not tie_output:
        qt("output", None, a.n_vocab, a.n_embd)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    os.replace(tmp, path)
    return path


def model_path(arch_name: str, seed: int = 0, cache_dir: str | None = None, tie_output: bool = False) -> str:
    """Path of the cached synthetic model, generating it on first use."""
    cache_dir = cache_dir or os.environ.get("ARMAI_MODEL_CACHE", "/tmp/armai_models")
    os.makedirs(cache_dir, exist_ok=True)
    arch = ARCHS[arch_name]
    # the last field versions the quantiser (2: signed Q6_K sub-scales)
    key = hashlib.sha256(repr((asdict(arch), seed, tie_output, 2)).encode()).hexdigest()[:12]
    p = os.path.join(cache_dir, f"{arch_name}-s{seed}{'-tied' if tie_output else ''}-{key}.gguf")
    if not os.path.exists(p):
        tmp = f"{p}.{os.getpid()}.tmp"  # complete files only, even if interrupted or raced
        write_model(tmp, arch, seed, tie_output)
        os.replace(tmp, p)
    return p


def prompt_tokens(n: int, vocab: int, seed: int) -> list[int]:
    """Seeded prompt: token ids uniform in [3, vocab)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return [int(t) for t in rng.integers(3, vocab, size=n)]

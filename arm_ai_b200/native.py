"""NIF-level mirror of ArmAI.Native for the decode path (lib/arm_ai/native.ex).

Same names, arities, argument order, return shapes and error wording as the
reference's Rust NIFs (native/arm_ai_nif/src/lib.rs), implemented by calling
the C ABI of libarmai_cuda.so. Binaries are numpy arrays (or bytes).
Errors raise ``NifError`` whose message carries the reference's prefix
("candle load: ", "candle generate: "), as ``rustler::Error::Term`` does.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_size_t, c_uint32, c_uint64, c_void_p

import numpy as np

from . import _lib
from ._lib import ArmaiError, LlamaInfo, LlamaOpts, TOKEN_CB, check, load_cuda, ptr


class NifError(RuntimeError):
    """The NIF raised (Elixir sees ErlangError with `original` = message)."""


class LlamaResource:
    """ResourceArc<LlamaResource>: owns an armai_llama handle, freed on GC."""

    def __init__(self, handle: int, lib):
        self._h = c_void_p(handle)
        self._lib = lib

    @property
    def handle(self) -> c_void_p:
        if not self._h:
            raise NifError("model handle already released")
        return self._h

    def info(self) -> LlamaInfo:
        inf = LlamaInfo()
        check(self._lib.armai_llama_get_info(self.handle, ctypes.byref(inf)))
        return inf

    def close(self) -> None:
        if self._h:
            self._lib.armai_llama_free(self._h)
            self._h = c_void_p(None)

    def __del__(self):  # BEAM GC -> Drop
        try:
            self.close()
        except Exception:
            pass


def default_opts(**kw) -> LlamaOpts:
    lib = load_cuda()
    o = LlamaOpts()
    lib.armai_llama_default_opts(ctypes.byref(o))
    for k, v in kw.items():
        if not hasattr(o, k):
            raise TypeError(f"unknown model option {k!r}")
        setattr(o, k, v)
    return o


def llama_candle_load_op(path: str, **opts) -> LlamaResource:
    """lib.rs:1659-1665. Raises NifError("candle load: ...")."""
    lib = load_cuda()
    o = default_opts(**opts)
    h = c_void_p()
    rc = lib.armai_llama_load(str(path).encode(), ctypes.byref(o), ctypes.byref(h))
    if rc != 0:
        raise NifError("candle load: " + _lib.last_error())
    return LlamaResource(h.value, lib)


def _u32(seq) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(seq), dtype=np.uint32))


def _generate(model: LlamaResource, prompt, max_new: int, stop_tokens, on_token=None):
    lib = load_cuda()
    p = _u32(prompt)
    st = _u32(stop_tokens)
    out = np.zeros(max(int(max_new), 1), dtype=np.uint32)
    n_out = c_size_t(0)
    pre = c_uint64(0)
    dec = c_uint64(0)
    errors = []

    def _cb(_user, tok):
        try:
            on_token(int(tok))
        except Exception as e:  # surface callback failures after the call
            errors.append(e)

    cb = TOKEN_CB(_cb) if on_token is not None else TOKEN_CB()
    rc = lib.armai_llama_generate(model.handle, ptr(p), p.size, int(max_new), ptr(st), st.size, cb,
                                  None, ptr(out), ctypes.byref(n_out), ctypes.byref(pre),
                                  ctypes.byref(dec))
    if rc != 0:
        raise NifError("candle generate: " + _lib.last_error())
    if errors:
        raise errors[0]
    return [int(t) for t in out[: n_out.value]], int(pre.value), int(dec.value)


def llama_candle_generate_op(model: LlamaResource, prompt, max_new: int, stop_tokens):
    """lib.rs:1667-1678 -> {tokens, prefill_us, decode_us}."""
    return _generate(model, prompt, max_new, stop_tokens)


def llama_candle_stream_op(model: LlamaResource, prompt, max_new: int, stop_tokens, pid):
    """lib.rs:1682-1699: like generate, also sending ("llama_token", id) to
    `pid` (any object with a ``send`` method, or a callable) per token."""
    send = pid.send if hasattr(pid, "send") else pid
    return _generate(model, prompt, max_new, stop_tokens, on_token=lambda t: send(("llama_token", t)))


def llama_generate_batch(model: LlamaResource, prompts, max_new: int, stop_tokens=()):
    """Batched greedy decode of independent sequences (several independent sequences; no
    reference counterpart, the reference holds one cache per handle):
    ([tokens per sequence], prefill_us, decode_us). Each sequence behaves as
    one llama_candle_generate_op call; the model must be loaded with
    max_batch >= len(prompts)."""
    lib = load_cuda()
    n = len(prompts)
    lens = np.array([len(p) for p in prompts], dtype=np.uint64)
    flat = _u32([t for p in prompts for t in p]) if lens.sum() else np.zeros(1, np.uint32)
    stop = _u32(list(stop_tokens))
    out = np.zeros(max(n * max_new, 1), dtype=np.uint32)
    n_out = np.zeros(max(n, 1), dtype=np.uint64)
    pre, dec = c_uint64(0), c_uint64(0)
    try:
        check(lib.armai_llama_generate_batch(model.handle, ptr(flat), ptr(lens), n, int(max_new), ptr(stop),
                                             stop.size, ptr(out), ptr(n_out), ctypes.byref(pre),
                                             ctypes.byref(dec)))
    except ArmaiError as e:
        raise NifError("candle generate: " + str(e)) from None
    toks = [out[i * max_new: i * max_new + int(n_out[i])].tolist() for i in range(n)]
    return toks, int(pre.value), int(dec.value)


def llama_forward(model: LlamaResource, tokens, index_pos: int, want_logits: bool = True):
    """ModelWeights::forward(tokens, index_pos): (logits f32[n_vocab] | None, argmax)."""
    lib = load_cuda()
    t = _u32(tokens)
    logits = np.empty(model.info().n_vocab, dtype=np.float32) if want_logits else None
    tok = c_uint32(0)
    check(lib.armai_llama_forward(model.handle, ptr(t), t.size, int(index_pos), ptr(logits),
                                  ctypes.byref(tok)))
    return logits, int(tok.value)


def llama_bench_decode(model: LlamaResource, n_steps: int) -> float:
    """Device time (ms) of n_steps back-to-back decode steps (CUDA events)."""
    ms = c_float(0)
    check(load_cuda().armai_llama_bench_decode(model.handle, int(n_steps), ctypes.byref(ms)))
    return float(ms.value)


KERNEL_KINDS = {"gateup": 0, "qkv": 1, "attn_output": 2, "ffn_down": 3, "head": 4, "attention": 5}


def llama_bench_kernel(model: LlamaResource, kind: str, rounds: int = 3):
    """(avg device ms per launch, weight bytes per launch) of one decode kernel kind."""
    ms = c_float(0)
    nbytes = ctypes.c_int64(0)
    check(load_cuda().armai_llama_bench_kernel(model.handle, KERNEL_KINDS[kind], int(rounds),
                                               ctypes.byref(ms), ctypes.byref(nbytes)))
    return float(ms.value), int(nbytes.value)


def llama_trace_decode(model: LlamaResource):
    """One decode step of the persistent kernel with per-phase, per-CTA
    globaltimer stamps: uint64 array [n_phases, n_ctas, 12] (ns)."""
    cap = 1 << 20
    buf = np.zeros(cap, dtype=np.uint64)
    nph, nct = ctypes.c_int32(0), ctypes.c_int32(0)
    check(load_cuda().armai_llama_trace_decode(model.handle, buf.ctypes.data, cap, ctypes.byref(nph),
                                               ctypes.byref(nct)))
    return buf[: nph.value * nct.value * 12].reshape(nph.value, nct.value, 12)


__all__ = ["llama_bench_kernel", "llama_trace_decode", "llama_generate_batch", "NifError", "LlamaResource", "llama_candle_load_op", "llama_candle_generate_op",
           "llama_candle_stream_op", "llama_forward", "llama_bench_decode", "default_opts",
           "ArmaiError"]

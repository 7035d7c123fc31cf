"""Mirror of ArmAI.LlamaCandle (lib/arm_ai/llama_candle.ex) over the CUDA path.

    status, model = LlamaCandle.load("/data/models/tinyllama.gguf",
                                     tokenizer="/data/models/tinyllama-tokenizer.json")
    reply, stats = LlamaCandle.generate(model, prompt="...", max_new=64, stop_tokens=[2])

``load`` returns ``("ok", model)`` or ``("error", reason)`` and never raises
(llama_candle.ex:31-57). ``generate`` raises ``ArgumentError`` for bad
arguments before touching the model (llama_candle.ex:199-215) and returns
``(generated, stats)`` with the reference's stats keys
(llama_candle.ex:94-102). ``stream`` yields text pieces as tokens arrive
(llama_candle.ex:137-197).
"""
from __future__ import annotations

import os
import queue
import threading
from dataclasses import dataclass
from typing import Any, Iterator

from . import native


class ArgumentError(ValueError):
    """Elixir ArgumentError."""


@dataclass
class LlamaCandle:
    handle: Any = None
    tokenizer: Any = None

    # ---------------------------------------------------------------- load
    @staticmethod
    def load(path: str, tokenizer: str | None = None, **model_opts) -> tuple[str, Any]:
        tok = _load_tokenizer(tokenizer)
        if tok[0] == "error":
            return tok
        res = _load_model(path, **model_opts)
        if res[0] == "error":
            return res
        return ("ok", LlamaCandle(handle=res[1], tokenizer=tok[1]))

    # ------------------------------------------------------------ generate
    @staticmethod
    def generate(model: "LlamaCandle", prompt: str | None = None, prompt_tokens=None,
                 max_new: int = 16, stop_tokens=(), performance_governor: bool = True):
        tokens_in, return_string = _encode_prompt(model.tokenizer, prompt, prompt_tokens)
        stop = list(stop_tokens)
        # performance_governor scopes the CPU governor in the reference
        # (llama_candle.ex:115-119); the option is accepted, and a no-op here.
        del performance_governor
        toks, prefill_us, decode_us = native.llama_candle_generate_op(model.handle, tokens_in,
                                                                      max_new, stop)
        if toks and toks[-1] in stop:
            toks = toks[:-1]
        n_new = len(toks)
        stats = {
            "n_prompt": len(tokens_in),
            "n_new": n_new,
            "prefill_ms": prefill_us / 1000.0,
            "decode_total_ms": decode_us / 1000.0,
            "decode_ms_per_tok": decode_us / 1000.0 / (n_new - 1) if n_new > 1 else None,
            "prefill_tokens_per_sec": len(tokens_in) * 1.0e6 / max(prefill_us, 1),
            "cpu_temp_c": None,
        }
        if return_string:
            return model.tokenizer.decode(toks), stats
        return toks, stats

    # -------------------------------------------------------------- stream
    @staticmethod
    def stream(model: "LlamaCandle", prompt: str | None = None, max_new: int = 16, stop_tokens=(),
               performance_governor: bool = True, **_ignored) -> Iterator[str]:
        if prompt is None or model.tokenizer is None:
            raise ArgumentError("stream/2 needs a string :prompt and load/2 with a `tokenizer:` path")
        tokens_in, _ = _encode_prompt(model.tokenizer, prompt, None)
        stop = list(stop_tokens)
        del performance_governor
        return _stream_iter(model, tokens_in, max_new, stop)


def _stream_iter(model, tokens_in, max_new, stop):
    q: queue.Queue = queue.Queue()
    done = object()

    class _Pid:
        def send(self, msg):
            q.put(msg)

    def run():
        try:
            native.llama_candle_stream_op(model.handle, tokens_in, max_new, stop, _Pid())
            q.put(done)
        except BaseException as e:  # the Task's :DOWN
            q.put(e)

    th = threading.Thread(target=run, daemon=True)
    th.start()
    ids: list[int] = []
    text = ""
    while True:
        msg = q.get()
        if msg is done:
            break
        if isinstance(msg, BaseException):
            raise msg
        _, tid = msg
        if tid in stop:
            continue
        ids.append(tid)
        new_text = model.tokenizer.decode(ids)
        yield new_text[len(text):] if new_text.startswith(text) else ""
        text = new_text
    th.join()


def _load_tokenizer(path):
    if path is None:
        return ("ok", None)
    try:
        from tokenizers import Tokenizer
        return ("ok", _Tok(Tokenizer.from_file(str(path))))
    except Exception as e:  # missing file / bad json
        return ("error", ("tokenizer", str(e)))


def _load_model(path, **opts):
    if not isinstance(path, (str, os.PathLike)) or not os.path.isfile(path):
        return ("error", ("enoent", path))
    try:
        return ("ok", native.llama_candle_load_op(str(path), **opts))
    except native.NifError as e:
        return ("error", str(e))
    except Exception as e:
        return ("error", e)


class _Tok:
    def __init__(self, tok):
        self._t = tok

    def encode(self, text: str) -> list[int]:
        return list(self._t.encode(text).ids)

    def decode(self, ids) -> str:
        return self._t.decode(list(ids))


def _encode_prompt(tokenizer, prompt, prompt_tokens):
    if prompt is not None:
        if tokenizer is None:
            raise ArgumentError("a string :prompt requires load/2 with a `tokenizer:` path")
        return tokenizer.encode(prompt), True
    if prompt_tokens is not None:
        return [int(t) for t in prompt_tokens], False
    raise ArgumentError("pass :prompt (string) or :prompt_tokens (list)")


__all__ = ["LlamaCandle", "ArgumentError"]

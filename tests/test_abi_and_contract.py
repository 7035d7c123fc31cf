"""C-ABI surface and host-side contract tests (no GPU).

* libarmai_cuda.so loads and exports every entry point include/armai.h declares.
* The ArmAI.LlamaCandle contract of the reference's own ExUnit tests
  (test/llama_candle_test.exs:15-58, test/models_api_test.exs:13-24): load
  error paths return ("error", _), generate raises ArgumentError before
  touching the NIF.
* GGUF parse errors surface as errors before any CUDA call.
* generate's stats/stop-token trimming (llama_candle.ex:86-102) with a fake NIF.
"""
import os
import re
import struct

import pytest

from arm_ai_b200 import native
from arm_ai_b200.llama_candle import ArgumentError, LlamaCandle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "armai.h")).read()
    return sorted(set(re.findall(r"ARMAI_API\s+[\w\s\*]+?\b(armai_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol(built):
    import ctypes
    from arm_ai_b200._lib import CUDA_LIB
    lib = ctypes.CDLL(CUDA_LIB)
    syms = declared_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_integration_rust_block_matches_header():
    """INTEGRATION.md's FFI block declares exactly the header's functions and
    the option / info structs' fields in the header's order."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    assert sorted(set(re.findall(r"pub fn (armai_\w+)\(", doc))) == declared_symbols()
    hdr = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "armai.h")).read(), flags=re.S)
    for name in ("armai_llama_opts", "armai_llama_info"):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), hdr, re.S).group(1)
        c_fields = []
        for decl in filter(str.strip, body.split(";")):
            first, *more = decl.replace("*", " ").split(",")
            c_fields += [n.strip().split("[")[0] for n in [first.split()[-1], *more]]
        rs = re.search(r"pub struct %s \{(.*?)\}" % name, doc, re.S).group(1)
        assert re.findall(r"pub (\w+):", rs) == c_fields, name


def test_missing_gguf_returns_error(built):
    assert LlamaCandle.load("/tmp/__nope.gguf")[0] == "error"


def test_missing_tokenizer_returns_error(built):
    assert LlamaCandle.load("/tmp/__nope.gguf", tokenizer="/tmp/__nope_tokenizer.json")[0] == "error"


def test_empty_path_returns_error(built):
    assert LlamaCandle.load("")[0] == "error"


def test_generate_raises_without_prompt():
    fake = LlamaCandle(handle=None, tokenizer=None)
    with pytest.raises(ArgumentError, match=re.compile("prompt", re.I)):
        LlamaCandle.generate(fake, max_new=4)


def test_generate_raises_for_string_prompt_without_tokenizer():
    fake = LlamaCandle(handle=None, tokenizer=None)
    with pytest.raises(ArgumentError, match="tokenizer"):
        LlamaCandle.generate(fake, prompt="hello", max_new=4)


def test_stream_requires_tokenizer():
    fake = LlamaCandle(handle=None, tokenizer=None)
    with pytest.raises(ArgumentError):
        LlamaCandle.stream(fake, prompt="hi")


def test_struct_fields_stable():
    m = LlamaCandle(handle="placeholder", tokenizer=None)
    assert m.handle == "placeholder" and m.tokenizer is None


def _write(path, data):
    with open(path, "wb") as f:
        f.write(data)


def test_gguf_errors_before_cuda(built, tmp_path):
    bad = tmp_path / "bad.gguf"
    _write(bad, b"NOPE" + b"\0" * 64)
    with pytest.raises(native.NifError, match="candle load: .*magic"):
        native.llama_candle_load_op(str(bad))
    trunc = tmp_path / "trunc.gguf"
    _write(trunc, b"GGUF" + struct.pack("<IQQ", 3, 5, 100))
    with pytest.raises(native.NifError, match="candle load: .*truncated"):
        native.llama_candle_load_op(str(trunc))
    # valid header, no llama metadata
    empty = tmp_path / "empty.gguf"
    _write(empty, b"GGUF" + struct.pack("<IQQ", 3, 0, 0))
    with pytest.raises(native.NifError, match="cannot find llama.attention.head_count"):
        native.llama_candle_load_op(str(empty))


def test_gguf_missing_tensor_and_bad_type(built, tmp_path):
    import gguf
    import numpy as np
    p = str(tmp_path / "m.gguf")
    w = gguf.GGUFWriter(p, "llama")
    w.add_block_count(1)
    w.add_embedding_length(256)
    w.add_head_count(4)
    w.add_head_count_kv(2)
    w.add_rope_dimension_count(64)
    w.add_layer_norm_rms_eps(1e-5)
    w.add_tensor("token_embd.weight", np.zeros((10, 256), dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(native.NifError, match="token_embd.weight has type F32"):
        native.llama_candle_load_op(p)


def test_generate_stats_and_stop_trim(monkeypatch):
    calls = {}

    def fake_generate(handle, prompt, max_new, stop):
        calls["args"] = (handle, list(prompt), max_new, list(stop))
        return [5, 6, 7, 2], 2000, 9000

    monkeypatch.setattr(native, "llama_candle_generate_op", fake_generate)
    m = LlamaCandle(handle="h", tokenizer=None)
    toks, stats = LlamaCandle.generate(m, prompt_tokens=[1, 2, 3], max_new=8, stop_tokens=[2])
    assert calls["args"] == ("h", [1, 2, 3], 8, [2])
    assert toks == [5, 6, 7]
    assert stats["n_new"] == 3 and stats["n_prompt"] == 3
    assert stats["prefill_ms"] == 2.0 and stats["decode_total_ms"] == 9.0
    assert stats["decode_ms_per_tok"] == 4.5
    assert stats["prefill_tokens_per_sec"] == 3 * 1e6 / 2000
    toks, stats = LlamaCandle.generate(m, prompt_tokens=[1], max_new=8, stop_tokens=[9])
    assert toks == [5, 6, 7, 2] and stats["decode_ms_per_tok"] == 9.0 / 3
    monkeypatch.setattr(native, "llama_candle_generate_op", lambda *a: ([2], 0, 0))
    toks, stats = LlamaCandle.generate(m, prompt_tokens=[1], stop_tokens=[2])
    assert toks == [] and stats["decode_ms_per_tok"] is None and stats["prefill_tokens_per_sec"] == 1e6


def test_bench_reads_profiled_traffic():
    """bench.py's roofline `traffic` comes from the committed ncu summary of the
    decode kernel; the summary must keep the line it parses."""
    import sys
    sys.path.insert(0, ROOT)
    import bench
    t = bench.profiled_traffic("k_decode_mega")
    assert t is not None and 600e6 < t < 700e6  # ~one TinyLlama token's weights

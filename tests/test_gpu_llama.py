"""Parity of the CUDA decode path with the CPU oracle, through the C ABI.

Bar: final logits within 1e-2 relative max-abs
(max |ours - oracle| / max |oracle|), greedy token ids identical for the
first 32 tokens. The integer parts are bit-exact (test_gpu_kquant.py); the
remaining differences are f32 summation orders, which now and then flip one
activation's Q8_K rounding. tests/parity.py explains the resulting criteria:
every result within the model's flip bound, a quarter of the tiny-model
inputs within 1e-5, greedy ids consistent with the oracle's argmax.
"""
import numpy as np
import pytest

import ref
from arm_ai_b200 import native, synth
from arm_ai_b200.llama_candle import LlamaCandle
from parity import TIGHT, check_errors, flip_bound, greedy_consistent, rel_maxabs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(tiny_model):
    return tiny_model, native.llama_candle_load_op(tiny_model), ref.OracleLlama(tiny_model)


PREFILL_LENGTHS = [1, 2, 7, 8, 19, 20, 40, 63, 64, 65, 70, 100, 128, 129, 200, 300]
SMALL_LENGTHS = (16, 24, 64, 100, 128)  # the small-model tests use short contexts


def test_prefill_logits_match_oracle(tiny):
    """Prompt lengths across the prefill tiling (8-token tiles, 64-token
    attention launches): final logits and argmax."""
    path, gpu, orc = tiny
    errs = []
    for n in PREFILL_LENGTHS:
        prompt = synth.prompt_tokens(n, orc.n_vocab, 100 + n)
        lg, tok = native.llama_forward(gpu, prompt, 0)
        errs.append(rel_maxabs(lg, orc.forward(prompt, 0)))
        assert tok == int(np.argmax(lg)) and tok == ref.argmax(lg), n
    check_errors(errs, flip_bound(path), min_tight_frac=0.25)


def test_teacher_forced_decode_matches_oracle(tiny):
    path, gpu, orc = tiny
    prompt = synth.prompt_tokens(9, orc.n_vocab, 5)
    native.llama_forward(gpu, prompt, 0)
    orc.forward(prompt, 0)
    rng = np.random.default_rng(3)
    errs = []
    for i in range(40):
        t = int(rng.integers(3, orc.n_vocab))
        lg, _ = native.llama_forward(gpu, [t], len(prompt) + i)
        errs.append(rel_maxabs(lg, orc.forward([t], len(prompt) + i)))
    check_errors(errs, flip_bound(path), min_tight_frac=0.25)


@pytest.mark.parametrize("decode_kernel", [0, 1])
@pytest.mark.parametrize("n_prompt,steps,check", [
    # the persistent kernel splits the context across CTAs every 128
    # positions (head_dim 64): boundaries at 512 and 640 here; the per-kernel
    # chain's attention takes one CTA per 64 positions (9 .. 11 CTAs here)
    (450, 200, {0, 60, 61, 62, 63, 188, 189, 190, 199}),
    # persistent kernel: 16 splits of one tile each end at 2048, beyond them
    # splits take two tiles; per-kernel chain: 16 CTAs of two to three
    # 64-position tiles, and its prompt runs every context length below
    (2040, 16, set(range(16))),
])
def test_long_context_decode_matches_oracle(tiny, n_prompt, steps, check, decode_kernel):
    # the integer (dp4a) prefill, so that only the decode attention is on trial
    path, _, orc = tiny
    gpu = native.llama_candle_load_op(path, prefill_gemm=1, decode_kernel=decode_kernel)
    prompt = synth.prompt_tokens(n_prompt, orc.n_vocab, 77)
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    orc.forward(prompt, 0)
    rng = np.random.default_rng(4)
    errs = []
    for i in range(steps):
        t = int(rng.integers(3, orc.n_vocab))
        lg, _ = native.llama_forward(gpu, [t], n_prompt + i, want_logits=i in check)
        lo = orc.forward([t], n_prompt + i)
        if i in check:
            errs.append(rel_maxabs(lg, lo))
    check_errors(errs, flip_bound(path))
    gpu.close()


@pytest.mark.parametrize("seed", [11, 12, 13])
def test_greedy_tokens_identical(tiny, seed):
    path, gpu, orc = tiny
    prompt = synth.prompt_tokens(16, orc.n_vocab, seed)
    ours, pre, dec = native.llama_candle_generate_op(gpu, prompt, 40, [])
    assert len(ours) == 40
    assert greedy_consistent(path, prompt, ours[:32], tol=2 * flip_bound(path)) is None
    assert pre > 0 and dec > 0


def test_stop_tokens_and_edge_cases(tiny):
    path, gpu, orc = tiny
    prompt = synth.prompt_tokens(12, orc.n_vocab, 21)
    full, _, _ = orc.generate(prompt, 20)
    stop = [full[5]]
    first = full.index(stop[0])
    ours, _, _ = native.llama_candle_generate_op(gpu, prompt, 20, stop)
    theirs, _, _ = orc.generate(prompt, 20, stop)
    assert ours == theirs == full[: first + 1]      # the stop token is included
    assert native.llama_candle_generate_op(gpu, prompt, 0, []) == ([], 0, 0)
    assert native.llama_candle_generate_op(gpu, [], 5, []) == ([], 0, 0)
    one, _, _ = native.llama_candle_generate_op(gpu, prompt, 1, [])
    assert one == full[:1]
    # stop on the very first token
    ours, _, _ = native.llama_candle_generate_op(gpu, prompt, 20, [full[0]])
    assert ours == full[:1]


def test_llama_candle_api_stats(tiny):
    path, gpu, orc = tiny
    status, model = LlamaCandle.load(path)
    assert status == "ok"
    prompt = synth.prompt_tokens(10, orc.n_vocab, 31)
    full, _, _ = orc.generate(prompt, 12)
    toks, stats = LlamaCandle.generate(model, prompt_tokens=prompt, max_new=12, stop_tokens=[full[4]])
    assert toks == full[:4]                 # trailing stop token trimmed
    assert stats["n_new"] == 4 and stats["n_prompt"] == 10
    assert stats["decode_ms_per_tok"] == pytest.approx(stats["decode_total_ms"] / 3)
    assert stats["prefill_tokens_per_sec"] > 0


def test_stream_op_sends_each_token(tiny):
    path, gpu, orc = tiny
    prompt = synth.prompt_tokens(6, orc.n_vocab, 41)
    got = []
    toks, _, _ = native.llama_candle_stream_op(gpu, prompt, 10, [], got.append)
    assert [t for (_, t) in got] == toks and all(tag == "llama_token" for tag, _ in got)


def test_errors(tiny):
    path, gpu, orc = tiny
    with pytest.raises(Exception):
        native.llama_forward(gpu, [orc.n_vocab + 5], 0)
    with pytest.raises(native.NifError, match="candle generate: .*max_seq_len"):
        native.llama_candle_generate_op(gpu, [5] * 4000, 200, [])
    # the model still works after host-side errors
    lg, _ = native.llama_forward(gpu, [5, 6], 0)
    assert np.isfinite(lg).all()


def test_tied_output_model(tied_model):
    gpu = native.llama_candle_load_op(tied_model)
    orc = ref.OracleLlama(tied_model)
    prompt = synth.prompt_tokens(5, orc.n_vocab, 3)
    lg, _ = native.llama_forward(gpu, prompt, 0)
    bound = flip_bound(tied_model)
    assert rel_maxabs(lg, orc.forward(prompt, 0)) < bound
    ours = native.llama_candle_generate_op(gpu, prompt, 24, [])[0]
    assert greedy_consistent(tied_model, prompt, ours, tol=2 * bound) is None


@pytest.mark.parametrize("opts", [{}, {"decode_kernel": 1}, {"decode_kernel": 1, "use_graph": 0},
                                  {"decode_kernel": 1, "use_pdl": 0}])
def test_small_model_decode_kernels(small_model, opts):
    """Both decode paths (persistent kernel; per-kernel chain with/without
    graph and PDL) on the 4-layer model: prompt logits within the sized bound,
    33 greedy tokens consistent with the oracle."""
    prompt = synth.prompt_tokens(13, 4096, 8)
    gpu = native.llama_candle_load_op(small_model, **opts)
    lg, _ = native.llama_forward(gpu, prompt, 0)
    bound = flip_bound(small_model, lengths=SMALL_LENGTHS)
    assert rel_maxabs(lg, ref.OracleLlama(small_model).forward(prompt, 0)) < bound
    ours = native.llama_candle_generate_op(gpu, prompt, 33, [])[0]
    assert len(ours) == 33
    assert greedy_consistent(small_model, prompt, ours[:32], tol=2 * bound) is None
    gpu.close()


def test_f16_kv_cache(small_model):
    """f16 KV cache (config 3) against the oracle with the same binary16
    rounding of cache entries: teacher-forced logits within the flip bound,
    greedy tokens consistent with the oracle."""
    orc = ref.OracleLlama(small_model, kv_f16=True)
    gpu = native.llama_candle_load_op(small_model, kv_f16=1)
    bound = flip_bound(small_model, kv_f16=True, lengths=SMALL_LENGTHS)
    prompt = synth.prompt_tokens(20, orc.n_vocab, 9)
    lg, _ = native.llama_forward(gpu, prompt, 0)
    errs = [rel_maxabs(lg, orc.forward(prompt, 0))]
    for i in range(8):
        lg, _ = native.llama_forward(gpu, [100 + i], 20 + i)
        errs.append(rel_maxabs(lg, orc.forward([100 + i], 20 + i)))
    check_errors(errs, bound)
    ours = native.llama_candle_generate_op(gpu, prompt, 33, [])[0]
    assert greedy_consistent(small_model, prompt, ours[:32], tol=2 * bound, kv_f16=True) is None


@pytest.mark.parametrize("n", [8, 64, 130, 300, 2040])
def test_prefill_tensor_core_gemm(tiny_model, n):
    """Prompt through the tcgen05 GEMM path (prefill_gemm = 2: f16 operands,
    f32 accumulation): final logits and the KV cache it leaves behind (decode
    steps after it). The f16 rounding of both operands is an approximation of
    candle's int8 dots on top of the flip noise, so the bound is 1.5 x the
    flip bound."""
    gpu = native.llama_candle_load_op(tiny_model, prefill_gemm=2)
    orc = ref.OracleLlama(tiny_model)
    prompt = synth.prompt_tokens(n, orc.n_vocab, 4000 + n)
    lg, tok = native.llama_forward(gpu, prompt, 0)
    bound = 1.5 * flip_bound(tiny_model)
    errs = [rel_maxabs(lg, orc.forward(prompt, 0))]
    assert tok == int(np.argmax(lg))
    for i in range(4):
        lg, _ = native.llama_forward(gpu, [50 + i], n + i)
        errs.append(rel_maxabs(lg, orc.forward([50 + i], n + i)))
    check_errors(errs, bound)
    gpu.close()


def test_prefill_gemm_small_model(small_model):
    gpu = native.llama_candle_load_op(small_model, prefill_gemm=2)
    orc = ref.OracleLlama(small_model)
    prompt = synth.prompt_tokens(200, orc.n_vocab, 77)
    lg, _ = native.llama_forward(gpu, prompt, 0)
    assert rel_maxabs(lg, orc.forward(prompt, 0)) < 1.5 * flip_bound(small_model, lengths=SMALL_LENGTHS)
    gpu.close()

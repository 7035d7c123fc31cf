"""Batched greedy decode (independent sequences per GPU): armai_llama_generate_batch.

Each sequence must behave as one armai_llama_generate call. Two batched
steps exist:
  * batch_gemm=1, the integer matvec step: the same per-row arithmetic as the
    per-kernel decode chain (one weight pass serves 16 sequences), so against
    that chain it is compared token for token;
  * batch_gemm=2 (the default for Q4_K / Q6_K models on one GPU), the
    tensor-core GEMM step: f16 operands, so it is held to the oracle with the
    same greedy criterion as the single-sequence path (tests/parity.py).
"""
import pytest

from arm_ai_b200 import native, synth
from parity import flip_bound, greedy_consistent

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def models(tiny_model):
    batch = native.llama_candle_load_op(tiny_model, decode_kernel=1, max_batch=20, batch_gemm=1)
    return tiny_model, batch


@pytest.fixture(scope="module")
def gemm_models(tiny_model):
    batch = native.llama_candle_load_op(tiny_model, max_batch=20, batch_gemm=2)
    return tiny_model, batch


def _prompts(n, vocab, seed):
    return [synth.prompt_tokens(1 + (7 * i + 3) % 37, vocab, seed + i) for i in range(n)]


@pytest.mark.parametrize("n_seq", [1, 5, 16, 20])
def test_batch_matches_single_sequence_chain(models, n_seq):
    path, gpu = models
    vocab = gpu.info().n_vocab
    prompts = _prompts(n_seq, vocab, 500)
    toks, pre, dec = native.llama_generate_batch(gpu, prompts, 24)
    assert len(toks) == n_seq and pre > 0 and dec > 0
    for p, t in zip(prompts, toks):
        single, _, _ = native.llama_candle_generate_op(gpu, p, 24, [])
        assert t == single


def test_batch_greedy_consistent_with_oracle(models):
    path, gpu = models
    vocab = gpu.info().n_vocab
    prompts = _prompts(6, vocab, 900)
    toks, _, _ = native.llama_generate_batch(gpu, prompts, 20)
    tol = 2 * flip_bound(path)
    for p, t in zip(prompts, toks):
        assert greedy_consistent(path, p, t, tol=tol) is None


@pytest.mark.parametrize("n_seq", [1, 5, 16, 20])
def test_batch_gemm_greedy_consistent_with_oracle(gemm_models, n_seq):
    path, gpu = gemm_models
    vocab = gpu.info().n_vocab
    prompts = _prompts(n_seq, vocab, 2100 + n_seq)
    toks, pre, dec = native.llama_generate_batch(gpu, prompts, 20)
    assert len(toks) == n_seq and pre > 0 and dec > 0
    assert all(len(t) == 20 for t in toks)
    tol = 2 * flip_bound(path)
    for p, t in list(zip(prompts, toks))[:4]:
        assert greedy_consistent(path, p, t, tol=tol) is None


def test_batch_gemm_is_deterministic_and_order_free(gemm_models):
    """Split-K partial sums are added in split order, so a batch repeats
    exactly, and a sequence's tokens do not depend on its neighbours."""
    path, gpu = gemm_models
    vocab = gpu.info().n_vocab
    prompts = _prompts(9, vocab, 2600)
    a, _, _ = native.llama_generate_batch(gpu, prompts, 16)
    b, _, _ = native.llama_generate_batch(gpu, prompts, 16)
    assert a == b
    c, _, _ = native.llama_generate_batch(gpu, prompts[::-1], 16)
    assert c[::-1] == a


@pytest.mark.parametrize("which", ["models", "gemm_models"])
def test_batch_stops_and_edges(request, which):
    path, gpu = request.getfixturevalue(which)
    vocab = gpu.info().n_vocab
    prompts = _prompts(4, vocab, 1300)
    full, _, _ = native.llama_generate_batch(gpu, prompts, 16)
    stop = [full[1][3]]
    toks, _, _ = native.llama_generate_batch(gpu, prompts, 16, stop)
    for f, t in zip(full, toks):
        cut = f.index(stop[0]) + 1 if stop[0] in f else len(f)
        assert t == f[:cut]      # the stop token is included, per sequence
    # an empty prompt yields no tokens and does not disturb the others
    toks, _, _ = native.llama_generate_batch(gpu, [prompts[0], [], prompts[2]], 16)
    assert toks[1] == [] and toks[0] == full[0] and toks[2] == full[2]
    assert native.llama_generate_batch(gpu, prompts, 0) == ([[], [], [], []], 0, 0)
    with pytest.raises(native.NifError, match="max_batch"):
        native.llama_generate_batch(gpu, _prompts(21, vocab, 1), 4)
    with pytest.raises(native.NifError, match="max_seq_len"):
        native.llama_generate_batch(gpu, [[5] * 4000], 200)
    # the handle still serves single-sequence calls (token for token the
    # batched integer step; the GEMM step is checked against the oracle above)
    single, _, _ = native.llama_candle_generate_op(gpu, prompts[0], 16, [])
    if which == "models":
        assert single == full[0]


def test_batch_wide_model_8_row_kernels(built):
    """ffn_down K = 12288: the batched step falls back to 8 sequences per
    weight pass; still token for token the single-sequence chain."""
    path = synth.model_path("wide", seed=6)
    gpu = native.llama_candle_load_op(path, decode_kernel=1, max_batch=12, batch_gemm=1)
    vocab = gpu.info().n_vocab
    prompts = _prompts(11, vocab, 1700)
    toks, _, _ = native.llama_generate_batch(gpu, prompts, 12)
    for p, t in zip(prompts, toks):
        single, _, _ = native.llama_candle_generate_op(gpu, p, 12, [])
        assert t == single
    tol = 2 * flip_bound(path, lengths=(16, 24, 64))
    for p, t in list(zip(prompts, toks))[:3]:
        assert greedy_consistent(path, p, t, tol=tol) is None
    gpu.close()

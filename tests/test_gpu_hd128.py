"""head_dim 128 (the Mistral-7B / Llama-3-8B attention shape) on a
CPU-checkable model: the persistent decode kernel's HD = 128 instantiation
and the long-context configuration's structure — f16 KV cache, a ~4096-token prompt and
decode steps across position 4096 (split attention of 16 context slices of
several 32-position tiles) — against the oracle, under the same flip-bound
criteria as tests/test_gpu_llama.py."""
import numpy as np
import pytest

import ref
from arm_ai_b200 import native, synth
from parity import check_errors, flip_bound, greedy_consistent, rel_maxabs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prefill_gemm", [1, 0])
def test_hd128_prefill_and_decode_match_oracle(hd128_model, prefill_gemm):
    """prefill_gemm=1: every prompt through the integer matvec kernels, held
    to the flip bound. prefill_gemm=0 (the default): prompts of 64 tokens or
    more run the tensor-core GEMMs and attention (f16 operands), held to
    1.5 x the flip bound as in tests/test_gpu_llama.py, and so are the decode
    steps that read the KV cache those prompts wrote."""
    path = hd128_model
    gpu = native.llama_candle_load_op(path, prefill_gemm=prefill_gemm)
    assert gpu.info().head_dim == 128
    orc = ref.OracleLlama(path)
    bound = flip_bound(path, lengths=(16, 24, 64, 100, 128))
    if prefill_gemm == 0:
        bound *= 1.5
    errs = []
    for n in (1, 20, 70, 129):
        prompt = synth.prompt_tokens(n, orc.n_vocab, 300 + n)
        lg, tok = native.llama_forward(gpu, prompt, 0)
        errs.append(rel_maxabs(lg, orc.forward(prompt, 0)))
        assert tok == ref.argmax(lg)
    rng = np.random.default_rng(8)
    for i in range(40):  # decode steps after the 129-token prompt
        t = int(rng.integers(3, orc.n_vocab))
        lg, _ = native.llama_forward(gpu, [t], 129 + i)
        errs.append(rel_maxabs(lg, orc.forward([t], 129 + i)))
    check_errors(errs, bound)
    prompt = synth.prompt_tokens(16, orc.n_vocab, 31)
    ours = native.llama_candle_generate_op(gpu, prompt, 32, [])[0]
    assert greedy_consistent(path, prompt, ours, tol=2 * bound) is None
    gpu.close()


def test_hd128_long_context_f16_kv(hd128_model):
    path = hd128_model
    n_prompt, steps = 4090, 16  # decode positions 4090 .. 4105 cross 4096
    gpu = native.llama_candle_load_op(path, kv_f16=1, max_seq_len=8192, prefill_gemm=1)
    orc = ref.OracleLlama(path, max_seq=8192, kv_f16=True)
    prompt = synth.prompt_tokens(n_prompt, orc.n_vocab, 55)
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    orc.forward(prompt, 0)
    rng = np.random.default_rng(9)
    errs = []
    for i in range(steps):
        t = int(rng.integers(3, orc.n_vocab))
        lg, _ = native.llama_forward(gpu, [t], n_prompt + i)
        errs.append(rel_maxabs(lg, orc.forward([t], n_prompt + i)))
    check_errors(errs, flip_bound(path, kv_f16=True, lengths=(16, 128, 1024, 4096)))
    gpu.close()

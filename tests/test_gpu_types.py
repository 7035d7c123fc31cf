"""Weight types beyond Q4_K / Q6_K (Q5_K with Q8_K activations; Q4_0, Q5_0,
Q8_0 with candle's Q8_0 activations) through the GPU path, against the
oracle, on tiny models that use one type throughout or mix them (prompts of
these models run the integer per-kernel chain; decode the persistent kernel).
The oracle side of these types is pinned in tests/test_oracle_types_pins.py."""
import os

import numpy as np
import pytest

import ref
from arm_ai_b200 import native, synth
from mixed_models import write_mixed_model
from parity import check_errors, flip_bound, greedy_consistent, rel_maxabs

pytestmark = pytest.mark.gpu

ALL = ("token_embd", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down", "output")
CASES = {
    "q5k": {n: "Q5_K" for n in ALL},
    "q8_0": {n: "Q8_0" for n in ALL},
    "q4_0": {n: "Q4_0" for n in ALL},
    "q5_0": {n: "Q5_0" for n in ALL},
    "mixed": {"token_embd": "Q5_K", "attn_q": "Q5_K", "attn_k": "Q8_0", "attn_v": "Q4_0",
              "attn_output": "Q5_0", "ffn_gate": "Q5_K", "ffn_up": "Q8_0", "ffn_down": "Q4_0", "output": "Q8_0"},
}


@pytest.mark.parametrize("case", list(CASES))
def test_weight_types_match_oracle(built, case):
    d = os.environ.get("ARMAI_MODEL_CACHE", "/tmp/armai_models")
    os.makedirs(d, exist_ok=True)
    path = write_mixed_model(os.path.join(d, f"tiny-{case}-s21-v1.gguf"), "tiny", 21, CASES[case])
    gpu = native.llama_candle_load_op(path)
    orc = ref.OracleLlama(path)
    bound = flip_bound(path, lengths=(16, 24, 64, 100, 128))
    errs = []
    for n in (1, 12, 70):
        prompt = synth.prompt_tokens(n, orc.n_vocab, 500 + n)
        lg, tok = native.llama_forward(gpu, prompt, 0)
        errs.append(rel_maxabs(lg, orc.forward(prompt, 0)))
        assert tok == ref.argmax(lg)
    rng = np.random.default_rng(5)
    for i in range(16):
        t = int(rng.integers(3, orc.n_vocab))
        lg, _ = native.llama_forward(gpu, [t], 70 + i)
        errs.append(rel_maxabs(lg, orc.forward([t], 70 + i)))
    check_errors(errs, bound)
    prompt = synth.prompt_tokens(10, orc.n_vocab, 77)
    ours = native.llama_candle_generate_op(gpu, prompt, 20, [])[0]
    assert greedy_consistent(path, prompt, ours, tol=2 * bound) is None
    gpu.close()

"""Failure detection and concurrency on one GPU, in the forms this pool
allows (no GPU fault, trap or unbounded wait is provoked):

* a device-side bounded wait that runs out: armai_llama_test_stall makes one
  phase of the persistent decode kernel publish nothing and shortens the
  waits; the decode call must come back with ARMAI_E_DEVICE well within
  seconds, the model must then refuse further work ("reload the model"),
  and a model loaded afterwards on the same GPU must work (the context
  survived);
* several host threads calling generate on one handle: the per-model mutex
  (reference native/arm_ai_nif/src/llama_candle.rs:24-32,80) serialises them,
  so every thread gets the tokens of a lone call.
"""
import threading
import time

import numpy as np
import pytest

import ref
from arm_ai_b200 import native, synth
from arm_ai_b200._lib import ArmaiError, load_cuda
from arm_ai_b200.native import NifError
from parity import flip_bound, rel_maxabs

pytestmark = pytest.mark.gpu


def test_stalled_phase_times_out_and_model_asks_for_reload(tiny_model):
    gpu = native.llama_candle_load_op(tiny_model)
    prompt = synth.prompt_tokens(8, 1000, 3)
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    # phase 2 = layer 0's attn_output: its row sums are never published, so
    # layer 0's gate/up waits (at most 2^14 polls) for them in vain
    assert load_cuda().armai_llama_test_stall(gpu.handle, 2, 1 << 14) == 0
    t0 = time.time()
    with pytest.raises(ArmaiError, match="reload the model"):
        native.llama_forward(gpu, [5], len(prompt))
    assert time.time() - t0 < 30
    with pytest.raises((NifError, ArmaiError), match="reload"):
        native.llama_candle_generate_op(gpu, prompt, 4, [])
    gpu.close()
    fresh = native.llama_candle_load_op(tiny_model)
    lg, tok = native.llama_forward(fresh, prompt, 0)
    assert rel_maxabs(lg, ref.OracleLlama(tiny_model).forward(prompt, 0)) < flip_bound(tiny_model)
    assert len(native.llama_candle_generate_op(fresh, prompt, 8, [])[0]) == 8
    fresh.close()


@pytest.mark.parametrize("decode_kernel", [0, 1])
def test_concurrent_generate_calls_are_serialised(tiny_model, decode_kernel):
    gpu = native.llama_candle_load_op(tiny_model, decode_kernel=decode_kernel)
    prompt = synth.prompt_tokens(20, 1000, 11)
    lone = native.llama_candle_generate_op(gpu, prompt, 32, [])[0]
    results, errors = [None] * 4, []

    def work(i):
        try:
            results[i] = native.llama_candle_generate_op(gpu, prompt, 32, [])[0]
        except Exception as e:  # surfaced below
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    assert all(r == lone for r in results), (lone, results)
    gpu.close()

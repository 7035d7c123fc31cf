"""Parity on the benchmarked configuration, measured and reported: the
TinyLlama-1.1B-architecture Q4_K_M model (22 layers, random-init weights),
b = 1, 32-token seeded prompts, 32 greedy tokens, through the persistent
decode kernel that the benchmark times.

For each of 8 prompts (seed 1000 is the benchmark's own prompt):
  * prefill logits: relative max-abs error against the oracle;
  * teacher-forced decode along the oracle's greedy trajectory (both sides
    fed the oracle's tokens): the relative max-abs logit error of every
    step, and at every step whether the GPU's argmax is the oracle's;
  * free-running greedy decode on the GPU (armai_llama_generate): how many of
    the 32 ids equal the oracle's greedy ids before the first difference.
At a step where the argmax differs, the oracle's top-2 margin (relative to
max |logit|) is reported, and the oracle is re-run under its one-ulp
rms_norm perturbations to see whether one of them also picks the GPU's token
(a single Q8_K rounding flip moves these logits by up to the model's flip
bound, see tests/parity.py).

Asserted: every logit error within max(1e-2, flip bound); the argmax equal to
the oracle's at every teacher-forced step whose oracle top-2 margin exceeds
2 x the flip bound (a difference there cannot be a rounding flip). The
measured figures are printed in the run's "parity report" section.
"""
import numpy as np
import pytest

import ref
from arm_ai_b200 import native, synth
from parity import LOGIT_TOL, flip_bound, rel_maxabs

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

N_PROMPTS, N_PROMPT, N_IDS = 8, 32, 32


def top2_margin(lo):
    s = np.sort(lo)
    return float((s[-1] - s[-2]) / max(np.max(np.abs(lo)), 1e-30))


def oracle_picks_under_perturbation(path, prompt, prefix, token):
    """Variants (1..4) of the oracle's one-ulp rms_norm perturbation under
    which its logits after prompt + prefix have `token` as the argmax."""
    hits = []
    for v in (1, 2, 3, 4):
        with ref.norm_perturbed(v):
            orc = ref.OracleLlama(path)
            lo = orc.forward(prompt, 0)
            for i, t in enumerate(prefix):
                lo = orc.forward([t], len(prompt) + i)
            orc.close()
        if ref.argmax(lo) == token:
            hits.append(v)
    return hits


@pytest.fixture(scope="module")
def tinyllama(built):
    return synth.model_path("tinyllama-1.1b", seed=0)


def test_config1_logits_and_greedy_ids(tinyllama, parity_report):
    fb = flip_bound(tinyllama, lengths=(32,))
    bound = max(LOGIT_TOL, fb)
    gpu = native.llama_candle_load_op(tinyllama)
    rows, failures = [], []
    for s in range(N_PROMPTS):
        prompt = synth.prompt_tokens(N_PROMPT, 32000, 1000 + s)
        orc = ref.OracleLlama(tinyllama)
        lo = orc.forward(prompt, 0)
        lg, _ = native.llama_forward(gpu, prompt, 0)
        pre_err = rel_maxabs(lg, lo)
        tf_errs, ids_o, same, notes = [], [], 0, []
        for i in range(N_IDS):
            o, g = ref.argmax(lo), ref.argmax(lg)
            ids_o.append(o)
            if g == o:
                same += 1
            else:
                m = top2_margin(lo)
                if len(notes) < 2:  # the perturbed re-runs cost seconds each
                    hits = oracle_picks_under_perturbation(tinyllama, prompt, ids_o[:-1], g)
                    notes.append(f"step {i}: gpu {g} oracle {o}, oracle top-2 margin {m:.2e}, "
                                 f"perturbed oracle picks gpu's token under variants {hits}")
                else:
                    notes.append(f"step {i}: gpu {g} oracle {o}, oracle top-2 margin {m:.2e}")
                if m > 2 * fb:
                    failures.append((s, i, m))
            if i + 1 < N_IDS:
                lo = orc.forward([o], N_PROMPT + i)
                lg, _ = native.llama_forward(gpu, [o], N_PROMPT + i)
                tf_errs.append(rel_maxabs(lg, lo))
        orc.close()
        ours = native.llama_candle_generate_op(gpu, prompt, N_IDS, [])[0]
        prefix = next((i for i, (a, b) in enumerate(zip(ours, ids_o)) if a != b), len(ours))
        rows.append((s, pre_err, max(tf_errs), float(np.median(tf_errs)), same, prefix, notes))
        assert pre_err < bound and max(tf_errs) < bound, (s, pre_err, max(tf_errs), bound)
    gpu.close()
    parity_report.append(f"config 1 (tinyllama-1.1b Q4_K_M, b=1, {N_PROMPT}-token prompts, {N_IDS} ids): "
                         f"flip bound {fb:.2e}, logit bar max(1e-2, flip bound) = {bound:.2e}")
    for s, pe, tm, tmed, same, prefix, notes in rows:
        parity_report.append(f"  prompt seed {1000 + s}: prefill logits rel max-abs {pe:.2e}; teacher-forced "
                             f"max {tm:.2e} median {tmed:.2e}; argmax equal at {same}/{N_IDS} steps; "
                             f"free-running greedy identical for the first {prefix}/{N_IDS} ids")
        for n in notes:
            parity_report.append("    " + n)
    tot_same = sum(r[4] for r in rows)
    parity_report.append(f"  total: argmax equal at {tot_same}/{N_PROMPTS * N_IDS} teacher-forced steps; "
                         f"{sum(r[5] == N_IDS for r in rows)}/{N_PROMPTS} prompts identical for all {N_IDS} ids")
    assert not failures, failures

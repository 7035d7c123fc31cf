"""Pins of the oracle's other GGML weight types (Q4_0, Q5_0, Q8_0, Q5_K)
and of candle's Q8_0 activation quantisation, which the legacy types' matmuls
use (k_quants.rs, candle-core 0.8.4): against gguf-py's independent
quantiser / dequantisers, against f64 dots of the dequantised operands, and,
for a model mixing the types, against transformers' Llama."""
import os

import numpy as np
import pytest

import ref
from arm_ai_b200 import synth
from mixed_models import GGML, quantize_q5k, write_mixed_model
from parity import TIGHT, rel_maxabs

gguf = pytest.importorskip("gguf")
from gguf.quants import dequantize, quantize  # noqa: E402

T = gguf.GGMLQuantizationType
RNG = np.random.default_rng(11)


def test_q8_0_quantise_bit_exact(built):
    x = RNG.normal(0, 0.05, (16, 512)).astype(np.float32)
    x[3, :32] = 0.0                      # all-zero block: d = 0, q = 0
    x[5, 40] = 7.5                       # one large value per block
    ours = ref.quantize_q8_0(x).view(np.uint8).reshape(16, -1)
    assert np.array_equal(ours, quantize(x, T.Q8_0).reshape(16, -1))


@pytest.mark.parametrize("tname", ["Q4_0", "Q5_0", "Q8_0", "Q5_K"])
def test_dequant_bit_exact(built, tname):
    x = RNG.normal(0, 0.02, (12, 512)).astype(np.float32)
    raw = quantize_q5k(x) if tname == "Q5_K" else quantize(x, T[tname]).reshape(12, -1)
    want = dequantize(raw.reshape(-1), T[tname]).reshape(12, 512).astype(np.float32)
    assert np.array_equal(ref.dequant_rows(GGML[tname], raw, 512), want)


def test_q5k_dequant_of_arbitrary_bytes(built):
    raw = RNG.integers(0, 256, (6, 2 * 176), dtype=np.uint8)
    for off, v in ((0, 0.01), (2, 0.005), (176, 0.02), (178, 0.003)):
        raw[:, off:off + 2] = np.frombuffer(np.float16(v).tobytes(), np.uint8)
    want = dequantize(raw.reshape(-1), T.Q5_K).reshape(6, 512).astype(np.float32)
    assert np.array_equal(ref.dequant_rows(GGML["Q5_K"], raw, 512), want)


@pytest.mark.parametrize("tname", ["Q4_0", "Q5_0", "Q8_0", "Q5_K"])
def test_qmatmul_equals_dot_of_dequantised_operands(built, tname):
    k, n, m = 1024, 24, 3
    w = RNG.normal(0, 0.02, (n, k)).astype(np.float32)
    raw = quantize_q5k(w) if tname == "Q5_K" else quantize(w, T[tname]).reshape(n, -1)
    x = RNG.normal(0, 1.0, (m, k)).astype(np.float32)
    got = ref.qmatmul(GGML[tname], raw, k, x)
    wd = ref.dequant_rows(GGML[tname], raw, k).astype(np.float64)
    if tname == "Q5_K":  # the lhs as Q8_K: q * d
        q8 = ref.quantize_q8k(x)
        xd = (q8["qs"].astype(np.float64) * q8["d"][..., None]).reshape(m, k)
    else:                # the lhs as Q8_0: q * f16(d)
        q8 = ref.quantize_q8_0(x)
        d = q8["d"].view(np.float16).astype(np.float64)
        xd = (q8["qs"].astype(np.float64) * d[..., None]).reshape(m, k)
    want = xd @ wd.T
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5 * np.abs(want).max())


def test_q5k_without_high_bits_is_q4k(built):
    """With qh = 0 a Q5_K block is a Q4_K block (same d, dmin, scales, qs)."""
    k = 512
    q5 = quantize_q5k(RNG.normal(0, 0.02, (8, k)).astype(np.float32)).reshape(8, 2, 176)
    q5[..., 16:48] = 0
    q4 = np.concatenate([q5[..., 0:16], q5[..., 48:176]], axis=-1).reshape(8, 2 * 144)
    x = RNG.normal(0, 1.0, (2, k)).astype(np.float32)
    assert np.array_equal(ref.qmatmul(GGML["Q5_K"], q5.reshape(8, -1), k, x), ref.qmatmul(GGML["Q4_K"], q4, k, x))


# ---- a whole model mixing the types, against transformers' Llama ----
MIXED = {"token_embd": "Q5_K", "attn_q": "Q5_K", "attn_k": "Q8_0", "attn_v": "Q4_0",
         "attn_output": "Q5_0", "ffn_gate": "Q5_K", "ffn_up": "Q8_0", "ffn_down": "Q4_0", "output": "Q8_0"}
HF_NAME = {"q_proj": "attn_q", "k_proj": "attn_k", "v_proj": "attn_v", "o_proj": "attn_output",
           "gate_proj": "ffn_gate", "up_proj": "ffn_up", "down_proj": "ffn_down", "lm_head": "output"}


@pytest.fixture(scope="module")
def mixed_model(built, tmp_path_factory):
    d = os.environ.get("ARMAI_MODEL_CACHE", "/tmp/armai_models")
    os.makedirs(d, exist_ok=True)
    return write_mixed_model(os.path.join(d, "tiny-mixed-s12-v1.gguf"), "tiny", 12, MIXED)


def test_mixed_model_matches_transformers(built, mixed_model):
    torch = pytest.importorskip("torch")
    pytest.importorskip("transformers")
    from test_oracle_hf_pin import candle_rmsnorm, hf_model, q8k_roundtrip
    from transformers.models.llama import modeling_llama

    def q8_0_roundtrip(x):
        v = x.reshape(-1, 32).to(torch.float32)
        d = v.abs().max(dim=1, keepdim=True).values / 127.0
        iv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
        t = v * iv
        q = torch.sign(t) * torch.floor(t.abs() + 0.5)
        return (q * d.half().float()).reshape(x.shape)

    orc = ref.OracleLlama(mixed_model)
    old = modeling_llama.LlamaRMSNorm.forward
    modeling_llama.LlamaRMSNorm.forward = candle_rmsnorm
    try:
        model = hf_model(mixed_model, orc.n_vocab)  # Q8_K pre-hooks on every Linear
        for name, mod in model.named_modules():     # ... replaced by Q8_0 for the legacy types
            if isinstance(mod, torch.nn.Linear) and MIXED[HF_NAME[name.split(".")[-1]]] in ("Q4_0", "Q5_0", "Q8_0"):
                mod._forward_pre_hooks.clear()
                mod.register_forward_pre_hook(lambda _m, args: (q8_0_roundtrip(args[0]),))
        errs = []
        for n in (1, 5, 16, 40):
            prompt = synth.prompt_tokens(n, orc.n_vocab, 300 + n)
            with torch.no_grad():
                lg = model(torch.tensor([prompt])).logits[0, -1].numpy()
            errs.append(rel_maxabs(lg, ref.OracleLlama(mixed_model).forward(prompt, 0)))
    finally:
        modeling_llama.LlamaRMSNorm.forward = old
    assert max(errs) < 5e-2, errs
    assert np.mean(np.array(errs) < TIGHT) >= 0.5, errs

"""Cross-check of the oracle's forward pass against an independent Llama
implementation: transformers' LlamaForCausalLM, built from our synthetic
GGUF files through transformers' own GGUF reader (tensors dequantised by the
gguf package, q/k un-permuted to its rotate-half RoPE).

candle (the reference's engine) quantises every matmul input to Q8_K; the
HF model gets the same rounding from forward pre-hooks on its Linear layers,
and candle's rms_norm formula (serial f32 sum of squares, x / sqrt(sum/K +
eps) * w). What remains differs only in f32 summation order, which now and
then flips one activation's Q8_K rounding (tests/parity.py). So: every
prompt within the model's flip bound, at least 40 % of them within 1e-5, and
the same argmax wherever they agree that closely. This pins the oracle's
model structure (RoPE convention and theta, GQA, norms, SiLU * up, residuals,
output head) and our GGUF writer; the reference's own Rust engine cannot be
built here.
"""
import numpy as np
import pytest

import ref
from arm_ai_b200 import synth
from parity import TIGHT, flip_bound, rel_maxabs

torch = pytest.importorskip("torch")
pytest.importorskip("transformers")
pytest.importorskip("gguf")


def q8k_roundtrip(x):
    """BlockQ8K::from_float then dequantise, per 256 values: the value of
    largest magnitude (first on ties) m, iscale = -128 / m,
    q = min(round-half-away(iscale * x), 127), value q / iscale."""
    shp = x.shape
    v = x.reshape(-1, 256).to(torch.float32)
    m = torch.gather(v, 1, v.abs().argmax(dim=1, keepdim=True))
    iscale = -128.0 / m
    t = iscale * v
    q = torch.clamp(torch.sign(t) * torch.floor(t.abs() + 0.5), max=127.0)
    out = torch.where(m == 0, torch.zeros_like(v), q * (1.0 / iscale))
    return out.reshape(shp)


def candle_rmsnorm(self, x):
    xn = x.detach().numpy().astype(np.float32)
    s = np.cumsum(xn * xn, axis=-1, dtype=np.float32)[..., -1:]  # serial f32 sum
    m = np.sqrt(s / np.float32(xn.shape[-1]) + np.float32(self.variance_epsilon)).astype(np.float32)
    return torch.from_numpy(((xn / m).astype(np.float32) * self.weight.detach().numpy()).astype(np.float32))


def hf_model(path, vocab):
    from transformers import LlamaConfig, LlamaForCausalLM
    from transformers.modeling_gguf_pytorch_utils import load_gguf_checkpoint
    cfg = load_gguf_checkpoint(path, return_tensors=False)["config"]
    kw = {k: v for k, v in cfg.items() if k not in ("tokenizer", "model_type", "_model_name_or_path", "architectures")}
    kw["vocab_size"] = vocab  # the synthetic files carry no tokenizer
    model = LlamaForCausalLM(LlamaConfig(**kw)).float().eval()
    ts = load_gguf_checkpoint(path, return_tensors=True, model_to_load=model)["tensors"]
    model.load_state_dict({k: torch.as_tensor(np.asarray(v)).float() for k, v in ts.items()}, strict=True)
    for mod in model.modules():
        if isinstance(mod, torch.nn.Linear):
            mod.register_forward_pre_hook(lambda _m, args: (q8k_roundtrip(args[0]),))
    return model


@pytest.fixture
def candle_norm(monkeypatch):
    from transformers.models.llama import modeling_llama
    monkeypatch.setattr(modeling_llama.LlamaRMSNorm, "forward", candle_rmsnorm)


def test_oracle_matches_transformers_llama(built, candle_norm, tiny_model, small_model, hd128_model):
    errs, tight_argmax_ok = [], True
    for path in (tiny_model, small_model, hd128_model):
        vocab = ref.OracleLlama(path).n_vocab
        model = hf_model(path, vocab)
        bound = flip_bound(path, lengths=(16, 24, 64, 100, 128))
        for n in (1, 5, 16, 40, 100):
            prompt = synth.prompt_tokens(n, vocab, 70 + n)
            with torch.no_grad():
                lg = model(torch.tensor([prompt])).logits[0, -1].numpy()
            lo = ref.OracleLlama(path).forward(prompt, 0)
            e = rel_maxabs(lg, lo)
            assert e < bound, (path, n, e, bound)
            errs.append(e)
            if e < TIGHT:
                tight_argmax_ok &= int(np.argmax(lg)) == int(np.argmax(lo))
    assert np.mean(np.array(errs) < TIGHT) >= 0.4, errs
    assert tight_argmax_ok

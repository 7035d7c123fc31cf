"""Tensor-core attention (tcgen05: Q K^T and P V on the tensor cores, online
softmax in f32) through armai_dev_flash_attention_f16, against a PyTorch fp32
reference on the same f16 inputs: softmax(scale * q k^T, causal mask aligned at
0 as the reference's flash_attention_f32_op, shape_ops.rs:464-558) @ v.

Tolerance: P is rounded to f16 before P V (2^-11 relative per weight), so the
output's error is bounded by a few 2^-11 of the output scale; the bound used is
4e-3 x max|reference| (about 8 half-ulps)."""
import ctypes

import pytest

torch = pytest.importorskip("torch")

from arm_ai_b200._lib import load_cuda

pytestmark = pytest.mark.gpu


def _ref(q, k, v, scale, causal):
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), k.float()) * scale
    if causal:
        sq, sk = s.shape[-2], s.shape[-1]
        mask = torch.arange(sk, device=s.device)[None, :] > torch.arange(sq, device=s.device)[:, None]
        s = s.masked_fill(mask, float("-inf"))
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, dim=-1), v.float())


def _run(q, k, v, scale, causal):
    b, h, sq, d = q.shape
    sk = k.shape[2]
    out = torch.full((b, h, sq, d), float("nan"), device="cuda", dtype=torch.float32)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = load_cuda().armai_dev_flash_attention_f16(P(q), P(k), P(v), P(out), ctypes.c_float(scale), b, h, sq, sk,
                                                   d, int(causal), None)
    assert rc == 0
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("b,h,sq,sk,d,causal", [
    (1, 4, 200, 200, 64, True),      # ragged last tile, causal diagonal
    (1, 4, 200, 200, 64, False),
    (2, 3, 300, 300, 128, True),     # batch, head dim 128
    (1, 2, 128, 128, 64, True),      # exactly one tile
    (1, 2, 100, 333, 64, False),     # more keys than queries
    (1, 2, 1, 1, 128, True),         # a single query
    (1, 32, 2048, 2048, 128, True),  # the config-5 shape
])
def test_tc_attention_matches_fp32(built, b, h, sq, sk, d, causal):
    g = torch.Generator(device="cuda").manual_seed(1000 * sq + sk + d)
    q, k, v = (torch.rand((b, h, n, d), generator=g, device="cuda") * 2 - 1 for n in (sq, sk, sk))
    q, k, v = q.half(), k.half(), v.half()
    scale = d ** -0.5
    got = _run(q, k, v, scale, causal)
    exp = _ref(q, k, v, scale, causal)
    assert torch.isfinite(got).all()
    err = (got - exp).abs().max().item()
    assert err <= 4e-3 * exp.abs().max().item(), err


def test_tc_attention_large_scores(built):
    """Scores of magnitude ~30: the running max moves across key tiles, so the
    output is rescaled in tensor memory several times."""
    g = torch.Generator(device="cuda").manual_seed(7)
    b, h, s, d = 1, 2, 640, 64
    q = (torch.rand((b, h, s, d), generator=g, device="cuda") * 2 - 1).half()
    k = (torch.rand((b, h, s, d), generator=g, device="cuda") * 2 - 1).half()
    # later keys get larger scores: the max grows tile by tile
    k = (k.float() * torch.linspace(0.2, 3.0, s, device="cuda")[None, None, :, None]).half()
    v = (torch.rand((b, h, s, d), generator=g, device="cuda") * 2 - 1).half()
    got = _run(q, k, v, 1.0, True)
    exp = _ref(q, k, v, 1.0, True)
    assert (got - exp).abs().max().item() <= 4e-3 * exp.abs().max().item()

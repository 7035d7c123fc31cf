"""The loader's weight-type check, on the CPU: a GGUF whose attn_q has a type
outside the ones the reference's loader documents (Q4_0, Q5_0, Q8_0, Q4_K,
Q5_K, Q6_K; lib/arm_ai/native.ex:551-556) is rejected before any device
work, with the tensor and its type in the message."""
import numpy as np
import pytest

from arm_ai_b200 import native, synth
from arm_ai_b200.native import NifError

gguf = pytest.importorskip("gguf")


def _write_model(path, q_type_name):
    from gguf.quants import quantize
    a = synth.ARCHS["tiny"]
    lib = synth.load_synth()
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_name("armai-loader-type-test")
    w.add_block_count(a.n_layer)
    w.add_context_length(a.context_length)
    w.add_embedding_length(a.n_embd)
    w.add_feed_forward_length(a.n_ff)
    w.add_head_count(a.n_head)
    w.add_head_count_kv(a.n_head_kv)
    w.add_rope_dimension_count(a.head_dim)
    w.add_layer_norm_rms_eps(a.eps)
    w.add_rope_freq_base(a.rope_theta)
    rng = np.random.default_rng(0)

    def mat(name, rows, k, qtype=synth.Q4_K):
        if name == "blk.0.attn_q":
            x = rng.normal(0, 0.02, (rows, k)).astype(np.float32)
            t = gguf.GGMLQuantizationType[q_type_name]
            w.add_tensor(name + ".weight", quantize(x, t), raw_dtype=t)
        else:
            w.add_tensor(name + ".weight", synth._gen_quant(lib, 7, rows, k, qtype),
                         raw_dtype=gguf.GGMLQuantizationType(qtype))

    mat("token_embd", a.n_vocab, a.n_embd)
    for l in range(a.n_layer):
        w.add_tensor(f"blk.{l}.attn_norm.weight", np.ones(a.n_embd, np.float32))
        mat(f"blk.{l}.attn_q", a.n_head * a.head_dim, a.n_embd)
        mat(f"blk.{l}.attn_k", a.n_head_kv * a.head_dim, a.n_embd)
        mat(f"blk.{l}.attn_v", a.n_head_kv * a.head_dim, a.n_embd)
        mat(f"blk.{l}.attn_output", a.n_embd, a.n_head * a.head_dim)
        w.add_tensor(f"blk.{l}.ffn_norm.weight", np.ones(a.n_embd, np.float32))
        mat(f"blk.{l}.ffn_gate", a.n_ff, a.n_embd)
        mat(f"blk.{l}.ffn_up", a.n_ff, a.n_embd)
        mat(f"blk.{l}.ffn_down", a.n_embd, a.n_ff)
    w.add_tensor("output_norm.weight", np.ones(a.n_embd, np.float32))
    mat("output", a.n_vocab, a.n_embd, synth.Q6_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.mark.parametrize("qtype", ["Q4_1", "Q5_1"])
def test_unsupported_weight_type_rejected(built, tmp_path, qtype):
    p = tmp_path / f"attn_q_{qtype}.gguf"
    _write_model(p, qtype)
    with pytest.raises(NifError, match=rf"tensor blk\.0\.attn_q\.weight has type {qtype}; this build supports "
                                       r"Q4_0, Q5_0, Q8_0, Q4_K, Q5_K and Q6_K matrices"):
        native.llama_candle_load_op(str(p))

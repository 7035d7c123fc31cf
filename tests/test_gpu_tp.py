"""Tensor parallelism on two and four GPUs (the Llama-3-8B sharding on small
test models: 2 ranks on 8 query / 2 KV heads, FFN 1536; 4 ranks on 16 query
/ 4 KV heads, FFN 2048; vocab 4096 split over the ranks).

Each rank holds half the heads, gate/up rows and vocab rows and a K-half of
attn_output / ffn_down; the halves are summed through peer memory (the
persistent decode kernel) or by NCCL (per-kernel chain, prefill, batched
decode). Against the oracle: prompt logits (gathered from both ranks) within
the model's flip bound and greedy tokens consistent with the oracle,
identical on every rank, for single-sequence and batched decode. Skipped
with fewer GPUs than ranks.
"""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


BATCH_PROMPTS = [(13, 21), (20, 22), (7, 23)]  # (length, seed)


def _rank(rank, world, port, path, prompt, q):
    import datetime

    import numpy as np
    import torch.distributed as dist

    from arm_ai_b200 import native, synth, tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")  # plain NVLink transfers, no multicast objects
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        out = []
        for kernel in (0, 1):  # persistent kernel (peer memory), per-kernel chain (NCCL)
            uid = tp.share_unique_id(rank)
            gpu = tp.load_tp(path, rank, world, rank, uid, decode_kernel=kernel)
            lg, tok = native.llama_forward(gpu, prompt, 0)
            lg1, _ = native.llama_forward(gpu, [77], len(prompt))  # one decode step's logits
            toks = native.llama_candle_generate_op(gpu, prompt, 24, [])[0]
            long_prompt = list(prompt) * 8  # 104 tokens: the GEMM prefill path
            lg2, _ = native.llama_forward(gpu, long_prompt, 0)
            gpu.close()
            out.append((np.asarray(lg), tok, toks, np.asarray(lg1), np.asarray(lg2)))
        # batched decode (config 4's batch case): sharded weights, every
        # sequence on every rank, row-split sums and head winners through NCCL
        uid = tp.share_unique_id(rank)
        gpu = tp.load_tp(path, rank, world, rank, uid, max_batch=4)
        prompts = [synth.prompt_tokens(n, 4096, sd) for n, sd in BATCH_PROMPTS]
        btoks = [[int(t) for t in seq] for seq in native.llama_generate_batch(gpu, prompts, 20)[0]]
        gpu.close()
        q.put((rank, out, btoks))
    except Exception as e:  # report instead of hanging the other rank
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_matches_oracle(request, world):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    import ref
    from arm_ai_b200 import synth
    from parity import flip_bound, greedy_consistent, rel_maxabs

    small_model = request.getfixturevalue("small_model" if world == 2 else "tp4_model")
    prompt = synth.prompt_tokens(13, 4096, 21)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, small_model, prompt, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert not isinstance(r[1], str), r[1]
    bt = [r[2] for r in res]
    assert all(b == bt[0] for b in bt)  # every rank decodes the same batch
    btol = 2 * flip_bound(small_model, lengths=(16, 24, 64))
    for (n, sd), toks in zip(BATCH_PROMPTS, bt[0]):
        assert len(toks) == 20
        assert greedy_consistent(small_model, synth.prompt_tokens(n, 4096, sd), toks, tol=btol) is None
    bound = flip_bound(small_model, lengths=(16, 24, 64, 100, 128))
    orc = ref.OracleLlama(small_model)
    lo = orc.forward(prompt, 0)
    lo1 = orc.forward([77], len(prompt))
    lo2 = ref.OracleLlama(small_model).forward(list(prompt) * 8, 0)
    for kernel in (0, 1):
        for r in res:
            out = r[1]
            lg, tok, toks, lg1, lg2 = out[kernel]
            assert rel_maxabs(lg, lo) < bound, kernel
            assert rel_maxabs(lg1, lo1) < bound, kernel
            assert greedy_consistent(small_model, prompt, toks, tol=2 * bound) is None, kernel
            assert rel_maxabs(lg2, lo2) < 1.5 * bound, kernel  # GEMM prefill: f16 operands
        for r in res[1:]:  # every rank decodes the same tokens
            assert r[1][kernel][2] == res[0][1][kernel][2]
            assert r[1][kernel][1] == res[0][1][kernel][1]

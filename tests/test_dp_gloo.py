"""Host-side data-parallel logic of batched decode (arm_ai_b200/dp.py) on two
gloo ranks on the CPU. The per-rank generate is a stand-in with the same
contract as native.llama_generate_batch (no GPU here)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from arm_ai_b200.dp import generate_batch_dp, shard


def test_shard_covers_each_sequence_once():
    for n in (0, 1, 5, 16, 17):
        for w in (1, 2, 3, 4, 8):
            got = [i for r in range(w) for i in shard(n, w, r)]
            assert got == list(range(n))
            sizes = [len(shard(n, w, r)) for r in range(w)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def _fake_generate(prompts, max_new, stop):
    # deterministic per sequence: continue the prompt's last id
    out = [[(p[-1] + k + 1) % 1000 for k in range(max_new)] if p else [] for p in prompts]
    return out, 10 * len(prompts), 20 * len(prompts)


def _worker(rank, world, port, prompts, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        toks, pre, dec = generate_batch_dp(_fake_generate, prompts, 5)
        q.put((rank, toks, pre, dec))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_generate_batch_dp_two_gloo_ranks():
    prompts = [[3 + i] * (1 + i % 4) for i in range(7)] + [[]]
    want, _, _ = _fake_generate(prompts, 5, ())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, toks, pre, dec in results:
        assert toks == want
        assert pre == 40 and dec == 80  # max over ranks: 4 sequences each

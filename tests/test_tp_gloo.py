"""Host side of tensor parallelism on the CPU (no GPU here): rank 0's NCCL
unique id reaches every rank through torch.distributed (two gloo ranks), and
the loader rejects shardings the kernels cannot run before it touches a GPU
(arm_ai_b200/tp.py, armai_llama_load's tensor-parallel checks)."""
import ctypes
import os
import socket

import pytest
import torch.multiprocessing as mp

from arm_ai_b200 import native, tp
from arm_ai_b200.native import NifError


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, tp.share_unique_id(rank)))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_unique_id_shared_by_two_gloo_ranks(built):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert isinstance(got[0], bytes) and len(got[0]) == 128
    assert got[0] == got[1]


def test_load_tp_rejects_bad_unique_id(built, small_model):
    with pytest.raises(ValueError, match="128 bytes"):
        tp.load_tp(small_model, 0, 2, 0, b"short")


def _load(path, **opts):
    uid = ctypes.create_string_buffer(tp.nccl_unique_id(), 128)
    return native.llama_candle_load_op(path, tp_unique_id=ctypes.cast(uid, ctypes.c_void_p).value, **opts)


def test_loader_rejects_unrunnable_shardings(built, tiny_model, small_model):
    with pytest.raises(NifError, match=r"tp_rank must be in \[0, tp_size\)"):
        _load(small_model, tp_size=2, tp_rank=2)
    with pytest.raises(NifError, match=r"prefill_gemm 1 is not available with tp_size > 1"):
        _load(small_model, tp_size=2, tp_rank=0, prefill_gemm=1)
    # small: 8 query / 2 KV heads -> 3 ranks do not divide them
    with pytest.raises(NifError, match=r"3 ranks must divide the query heads \(8\) and KV heads \(2\)"):
        _load(small_model, tp_size=3, tp_rank=0)
    # tiny: 4 x 64-wide heads -> 2 ranks leave half a 256-value block of attn_output each
    with pytest.raises(NifError, match=r"whole 256-value blocks of attn_output per rank"):
        _load(tiny_model, tp_size=2, tp_rank=1)


def _worker_absent(rank, world, port, q):
    """Rank 1 never takes part in the id exchange (it leaves right after
    joining the group); rank 0's exchange must end with an error within the
    group's short timeout instead of waiting for ever."""
    import datetime
    import time

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((rank, "left"))
        return
    t0 = time.time()
    try:
        tp.share_unique_id(rank)
        q.put((rank, "completed"))
    except Exception as e:
        q.put((rank, ("error", type(e).__name__, time.time() - t0)))


def test_unique_id_exchange_ends_when_a_rank_never_joins(built):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_absent, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert isinstance(got[0], tuple) and got[0][0] == "error", got[0]
    assert got[0][2] < 60, got[0]

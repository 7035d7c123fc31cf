"""Tensor-parallel model loading (7B/8B-class models such as Llama-3-8B) across the GPUs of one
node: one process per GPU, every rank loads the same GGUF with its
tp_rank, all ranks share rank 0's NCCL unique id (armai_nccl_unique_id)
through the already-initialised torch.distributed group. The reference runs
on one CPU and has no counterpart.
"""
from __future__ import annotations

import ctypes

from ._lib import check, load_cuda


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(load_cuda().armai_nccl_unique_id(ctypes.cast(buf, ctypes.c_void_p)))
    return buf.raw


def share_unique_id(rank: int, group=None) -> bytes:
    """Rank 0's NCCL unique id on every rank (torch.distributed broadcast)."""
    import torch.distributed as dist
    obj = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def load_tp(path: str, device: int, tp_size: int, tp_rank: int, unique_id: bytes, **opts):
    """llama_candle_load_op for one tensor-parallel rank; all ranks must call it
    together (NCCL communicator creation is collective)."""
    from .native import llama_candle_load_op
    if len(unique_id) != 128:
        raise ValueError("NCCL unique id must be 128 bytes")
    buf = ctypes.create_string_buffer(unique_id, 128)
    return llama_candle_load_op(path, device=device, tp_size=tp_size, tp_rank=tp_rank,
                                tp_unique_id=ctypes.cast(buf, ctypes.c_void_p).value, **opts)

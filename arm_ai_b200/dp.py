"""Data-parallel batched decode across the GPUs of one node (many independent sequences, e.g. 16 x 512-token prompts).

Independent sequences shard with no data-path collective: rank r of W takes
a contiguous block of the sequences, decodes it with one batched call on its
own GPU (armai_llama_generate_batch), and the token lists are gathered on the
host afterwards. The reference has no counterpart (one KV cache per handle,
native/arm_ai_nif/src/llama_candle.rs:27-29); each sequence's result is the
single-sequence result.
"""
from __future__ import annotations


def shard(n_seq: int, world: int, rank: int) -> range:
    """Contiguous block of sequence indices for `rank`; the first n_seq % world
    ranks take one extra sequence."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n_seq, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def generate_batch_dp(generate, prompts, max_new: int, stop_tokens=(), group=None):
    """Run `generate(local_prompts, max_new, stop_tokens) -> (tokens, prefill_us,
    decode_us)` on this rank's shard and gather every rank's tokens in
    sequence order. Returns (tokens for all sequences, max prefill_us, max
    decode_us) on every rank. Without an initialised process group this is
    the single-process call."""
    import torch.distributed as dist
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return generate(list(prompts), max_new, stop_tokens)
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    idx = shard(len(prompts), world, rank)
    local = [prompts[i] for i in idx]
    toks, pre, dec = generate(local, max_new, stop_tokens) if local else ([], 0, 0)
    parts = [None] * world
    dist.all_gather_object(parts, (idx.start, toks, pre, dec), group=group)
    out = [None] * len(prompts)
    for start, ts, _, _ in parts:
        for j, t in enumerate(ts):
            out[start + j] = t
    return out, max(p[2] for p in parts), max(p[3] for p in parts)

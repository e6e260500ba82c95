"""Multi-GPU plumbing for the attention path (one process per GPU).

Two ways the work spreads over the GPUs of one box:

* a batched decode step shards whole sequences (attention of a sequence reads
  only its own blocks, legal_sources in kernels/attention_cpu.cpp:113-123 is
  per sequence), so no collective is needed: `shard_sequences` balances
  K/V bytes with a longest-processing-time greedy assignment;
* one very long sequence splits its block list into contiguous ranges
  (`split_range`), each GPU decodes its range into (m, l, o) partials
  (inferlab_cuda_paged_decode_partials), the partials are all-gathered over
  the process group (NCCL on GPUs, gloo in the CPU tests) and merged in rank
  order (inferlab_cuda_lse_combine), which makes the result independent of
  arrival order.
"""
from __future__ import annotations

import numpy as np


def shard_sequences(contexts, world: int) -> np.ndarray:
    """Owner rank of every sequence: longest context first onto the least
    loaded rank (ties to the lowest rank). Deterministic."""
    contexts = np.asarray(contexts, dtype=np.int64)
    order = np.argsort(-contexts, kind="stable")
    loads = np.zeros(world, np.int64)
    owner = np.zeros(len(contexts), np.int64)
    for i in order:
        r = int(np.argmin(loads))
        owner[i] = r
        loads[r] += contexts[i]
    return owner


def split_range(num_blocks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block range [lo, hi) of `rank` when `num_blocks` blocks are
    split as evenly as possible over `world` ranks (earlier ranks take the
    remainder)."""
    base, extra = divmod(num_blocks, world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def local_tokens(total_tokens: int, block_tokens: int, world: int, rank: int) -> tuple[int, int]:
    """Token range [lo, hi) of `rank` for a sequence of total_tokens tokens
    whose blocks are split by split_range (the last block may be partial)."""
    nblk = (total_tokens + block_tokens - 1) // block_tokens
    lo_b, hi_b = split_range(nblk, world, rank)
    return lo_b * block_tokens, min(hi_b * block_tokens, total_tokens)


def all_gather_partials(m, l, o, group=None):
    """Stack every rank's (m, l, o) partials in rank order: returns tensors of
    shape [world, ...]. Works for the NCCL (GPU tensors) and gloo (CPU
    tensors) backends."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = []
    for t in (m, l, o):
        t = t.contiguous()
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t, group=group)
        out.append(torch.stack(parts))
    return tuple(out)


def decode_split_sequence(pool, queries, block_table, local_len: int, group=None, workspace=None):
    """Decode one query per row against a sequence whose blocks are spread
    over the ranks: this rank's blocks are `block_table` (device int32
    [rows, blocks]) covering `local_len` tokens. Returns the merged output
    [rows, q_heads, head_dim] on every rank.

    The partials are written straight into one packed [m | l | o] block, the
    blocks of all ranks are exchanged with a single all-gather (NCCL), and
    one kernel merges them in rank order."""
    import torch
    import torch.distributed as dist

    from .paged import lse_combine_packed

    rows, q_heads, hd = queries.shape
    nrows = rows * q_heads
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    send = torch.empty(nrows * (hd + 2), dtype=torch.float32, device=queries.device)
    if local_len > 0:
        lens = torch.full((rows,), local_len, dtype=torch.int32, device=queries.device)
        pool.decode_partials(queries, block_table, lens, local_len, workspace=workspace,
                             packed=send)
    else:
        send[:nrows].fill_(float("-inf"))
        send[nrows:].zero_()
    if world > 1:
        recv = torch.empty(world * send.numel(), dtype=torch.float32, device=queries.device)
        dist.all_gather_into_tensor(recv, send, group=group)
    else:
        recv = send
    return lse_combine_packed(recv, world, nrows, hd).view(rows, q_heads, hd)

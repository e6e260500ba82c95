"""Seeded synthetic batches with the shapes of the benchmark configurations.

Inputs are synthetic (no dataset is involved): Q/K/V ~ N(0, sigma^2) from a
seeded generator, contexts drawn from the stated distributions, block tables
dealt from a seeded permutation of the pool. The KV arenas are filled on the
device in one pass (every slot of every block holds a sample), which is the
state a pool is in after the corresponding appends.

    decode_fp32   64 sequences, context ~ U[64, 2048], 8 heads x 64 (MHA),
                  fp32, 16-token blocks, tables from a permutation of 8192 blocks
    prefill_f16   8 x 1024-token causal prefill, 16 heads x 128, f16,
                  inputs ~ N(0, 0.5^2), paged K/V with 16-token blocks
    mixed_bf16    32 decode sequences with context Zipf(1.1) clipped to
                  [32, 8192] + 4 chunked-prefill segments of 512 tokens whose
                  prior context is drawn from the same clipped Zipf, GQA
                  32 q / 8 kv heads x 128, bf16, pool of 65536 blocks
    longctx_bf16  256 sequences, context ~ U[4096, 32768], GQA 32/8 x 128,
                  bf16 (sharded by sequence across GPUs), plus one
                  131072-token sequence split across GPUs
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from .paged import KV_BF16, KV_F16, KV_FP32, TORCH_DTYPES, CudaKvPool

BLOCK_TOKENS = 16


@dataclass
class PagedBatch:
    """A pool plus decode sequences and/or prefill segments over it."""

    pool: CudaKvPool
    q_heads: int
    # decode part
    queries: torch.Tensor | None = None          # [B][Hq][D] fp32
    block_tables: torch.Tensor | None = None     # [B][max_blocks] int32
    context_lens: torch.Tensor | None = None     # [B] int32
    contexts: np.ndarray | None = None
    tables_host: np.ndarray | None = None
    max_context_len: int = 0
    # prefill part
    prefill_queries: torch.Tensor | None = None  # [total][Hq][D] (pool dtype)
    prefill_tables: torch.Tensor | None = None
    prefill_tables_host: np.ndarray | None = None
    starts: np.ndarray | None = None
    counts: np.ndarray | None = None
    starts_dev: torch.Tensor | None = None
    counts_dev: torch.Tensor | None = None
    offsets_dev: torch.Tensor | None = None
    extra: dict = field(default_factory=dict)

    @property
    def kv_heads(self) -> int:
        return self.pool.kv_heads

    @property
    def head_dim(self) -> int:
        return self.pool.head_dim

    def decode_bytes(self) -> int:
        """Algorithmic HBM bytes of one decode step: every context K and V row
        once per (sequence, kv-head), the fp32 queries and outputs, the table
        entries and context lengths."""
        ctx = self.contexts.astype(np.int64)
        kv = int(ctx.sum()) * self.kv_heads * self.head_dim * 2 * self.pool.element_bytes
        b = len(ctx)
        qo = 2 * b * self.q_heads * self.head_dim * 4
        tables = int(((ctx + BLOCK_TOKENS - 1) // BLOCK_TOKENS).sum()) * 4 + b * 4
        return kv + qo + tables

    def prefill_flops(self) -> int:
        """4 * head_dim * score_elements, score_elements counted as the
        reference does (kernels/attention_cpu.cpp:149-168): for a chunk with
        prior context P and C queries, heads * (C * P + C * (C + 1) / 2)."""
        total = 0
        for p, c in zip(self.starts.tolist(), self.counts.tolist()):
            total += self.q_heads * (c * p + c * (c + 1) // 2)
        return 4 * self.head_dim * total


def _generator(seed: int, device: int) -> torch.Generator:
    gen = torch.Generator(device=f"cuda:{device}")
    gen.manual_seed(seed)
    return gen


def _fill_arenas(pool: CudaKvPool, gen: torch.Generator, sigma: float) -> None:
    dtype = TORCH_DTYPES[pool.dtype]
    for arena in (pool.key_arena, pool.value_arena):
        flat = arena.view(-1)
        step = 1 << 28
        for start in range(0, flat.numel(), step):
            chunk = flat[start:start + step]
            sample = torch.randn(chunk.numel(), generator=gen, device=chunk.device,
                                 dtype=torch.float32)
            if sigma != 1.0:
                sample.mul_(sigma)
            chunk.copy_(sample.to(dtype))


def _deal_tables(rng: np.random.Generator, num_blocks: int, blocks_needed, max_blocks: int):
    perm = rng.permutation(num_blocks).astype(np.int32)
    if int(np.sum(blocks_needed)) > num_blocks:
        raise ValueError("pool too small for the batch")
    tables = np.zeros((len(blocks_needed), max_blocks), np.int32)
    used = 0
    for i, n in enumerate(blocks_needed):
        tables[i, :n] = perm[used:used + n]
        used += n
    return tables


def decode_batch(device: int, seed: int, num_seqs: int, contexts: np.ndarray, q_heads: int,
                 kv_heads: int, head_dim: int, dtype: int, num_blocks: int | None = None,
                 sigma: float = 1.0, max_context_len: int | None = None) -> PagedBatch:
    rng = np.random.Generator(np.random.PCG64(seed))
    contexts = np.asarray(contexts, dtype=np.int64)
    need = (contexts + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    max_ctx = int(max_context_len or contexts.max())
    max_blocks = (max_ctx + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    if num_blocks is None:
        num_blocks = int(need.sum())
    tables = _deal_tables(rng, num_blocks, need, max_blocks)
    pool = CudaKvPool(device, dtype, num_blocks, BLOCK_TOKENS, kv_heads, head_dim)
    gen = _generator(seed + 1, device)
    _fill_arenas(pool, gen, sigma)
    dev = f"cuda:{device}"
    queries = torch.randn((num_seqs, q_heads, head_dim), generator=gen, device=dev,
                          dtype=torch.float32)
    if sigma != 1.0:
        queries.mul_(sigma)
    return PagedBatch(
        pool=pool, q_heads=q_heads, queries=queries,
        block_tables=torch.from_numpy(tables).to(dev),
        context_lens=torch.from_numpy(contexts.astype(np.int32)).to(dev),
        contexts=contexts, tables_host=tables, max_context_len=max_ctx)


def decode_fp32(device: int = 0, seed: int = 2026, num_seqs: int = 64) -> PagedBatch:
    """Paged decode, fp32: 64 x U[64, 2048], 8 heads x 64, pool of 8192 blocks."""
    rng = np.random.Generator(np.random.PCG64(seed))
    contexts = rng.integers(64, 2048, size=num_seqs, endpoint=True)
    return decode_batch(device, seed, num_seqs, contexts, 8, 8, 64, KV_FP32, num_blocks=8192,
                        max_context_len=2048)


def zipf_contexts(rng: np.random.Generator, n: int, low: int = 32, high: int = 8192) -> np.ndarray:
    return np.clip(rng.zipf(1.1, size=n), low, high).astype(np.int64)


def longctx_contexts(seed: int, num_seqs: int = 256) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(4096, 32768, size=num_seqs, endpoint=True).astype(np.int64)


def longctx_bf16(device: int = 0, seed: int = 2027, contexts: np.ndarray | None = None) -> PagedBatch:
    """Long-context paged decode, bf16, GQA 32/8 x 128 (one shard of sequences)."""
    if contexts is None:
        contexts = longctx_contexts(seed)
    return decode_batch(device, seed, len(contexts), contexts, 32, 8, 128, KV_BF16,
                        max_context_len=32768)


def prefill_batch(device: int, seed: int, starts, counts, q_heads: int, kv_heads: int,
                  head_dim: int, dtype: int, sigma: float, num_blocks: int | None = None,
                  extra_blocks: int = 0) -> PagedBatch:
    """Prefill segments: segment s has counts[s] queries at positions
    [starts[s], starts[s] + counts[s]); its K/V for [0, starts[s] + counts[s])
    are in the pool under table row s."""
    rng = np.random.Generator(np.random.PCG64(seed))
    starts = np.asarray(starts, dtype=np.int64)
    counts = np.asarray(counts, dtype=np.int64)
    totals = starts + counts
    need = (totals + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    max_blocks = int(need.max())
    if num_blocks is None:
        num_blocks = int(need.sum()) + extra_blocks
    tables = _deal_tables(rng, num_blocks, need, max_blocks)
    pool = CudaKvPool(device, dtype, num_blocks, BLOCK_TOKENS, kv_heads, head_dim)
    gen = _generator(seed + 1, device)
    _fill_arenas(pool, gen, sigma)
    dev = f"cuda:{device}"
    total_q = int(counts.sum())
    q = torch.randn((total_q, q_heads, head_dim), generator=gen, device=dev, dtype=torch.float32)
    if sigma != 1.0:
        q.mul_(sigma)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    return PagedBatch(
        pool=pool, q_heads=q_heads,
        prefill_queries=q.to(TORCH_DTYPES[dtype]) if dtype != KV_FP32 else q,
        prefill_tables=torch.from_numpy(tables).to(dev), prefill_tables_host=tables,
        starts=starts, counts=counts,
        starts_dev=torch.from_numpy(starts.astype(np.int32)).to(dev),
        counts_dev=torch.from_numpy(counts.astype(np.int32)).to(dev),
        offsets_dev=torch.from_numpy(offsets).to(dev))


def prefill_f16(device: int = 0, seed: int = 2028, num_seqs: int = 8,
                tokens: int = 1024) -> PagedBatch:
    """Causal prefill, f16: 8 x 1024 tokens, 16 heads x 128, N(0, 0.5^2)."""
    return prefill_batch(device, seed, [0] * num_seqs, [tokens] * num_seqs, 16, 16, 128, KV_F16,
                         0.5)


def mixed_bf16(device: int = 0, seed: int = 2029, num_decode: int = 32, num_chunks: int = 4,
               chunk_tokens: int = 512, num_blocks: int = 65536) -> PagedBatch:
    """Continuous-batching step: num_decode decode sequences with context
    Zipf(1.1) clipped to [32, 8192], plus num_chunks chunked-prefill segments
    of chunk_tokens queries whose prior context is drawn from the same clipped
    Zipf (so a chunk covers positions [prior, prior + chunk_tokens)). GQA
    32 q / 8 kv heads x 128, bf16, one pool of num_blocks blocks with tables
    dealt from a seeded permutation."""
    rng = np.random.Generator(np.random.PCG64(seed))
    contexts = zipf_contexts(rng, num_decode)
    priors = zipf_contexts(rng, num_chunks)
    counts = np.full(num_chunks, chunk_tokens, np.int64)
    totals = np.concatenate([contexts, priors + counts])
    need = (totals + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    max_blocks = int(need.max())
    tables = _deal_tables(rng, num_blocks, need, max_blocks)
    pool = CudaKvPool(device, KV_BF16, num_blocks, BLOCK_TOKENS, 8, 128)
    gen = _generator(seed + 1, device)
    _fill_arenas(pool, gen, 1.0)
    dev = f"cuda:{device}"
    queries = torch.randn((num_decode, 32, 128), generator=gen, device=dev, dtype=torch.float32)
    pq = torch.randn((int(counts.sum()), 32, 128), generator=gen, device=dev,
                     dtype=torch.float32).to(torch.bfloat16)
    offsets = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    dt = tables[:num_decode]
    pt = tables[num_decode:]
    return PagedBatch(
        pool=pool, q_heads=32, queries=queries, block_tables=torch.from_numpy(dt).to(dev),
        context_lens=torch.from_numpy(contexts.astype(np.int32)).to(dev), contexts=contexts,
        tables_host=dt, max_context_len=int(contexts.max()),
        prefill_queries=pq, prefill_tables=torch.from_numpy(pt).to(dev), prefill_tables_host=pt,
        starts=priors, counts=counts,
        starts_dev=torch.from_numpy(priors.astype(np.int32)).to(dev),
        counts_dev=torch.from_numpy(counts.astype(np.int32)).to(dev),
        offsets_dev=torch.from_numpy(offsets).to(dev))


@dataclass
class ProjectionBatch:
    pool: CudaKvPool
    hidden: torch.Tensor        # [tokens][model_dim], pool type
    weights: torch.Tensor       # [(q_heads + 2 kv_heads) head_dim][model_dim], pool type
    q_heads: int
    row_sequences: torch.Tensor
    positions: torch.Tensor
    block_tables: torch.Tensor
    tables_host: np.ndarray

    def flops(self) -> int:
        return 2 * self.hidden.shape[0] * self.weights.shape[0] * self.hidden.shape[1]


def qkv_append_bf16(device: int = 0, seed: int = 2030, num_chunks: int = 4,
                    chunk_tokens: int = 512, model_dim: int = 4096,
                    num_blocks: int = 16384) -> ProjectionBatch:
    """The projection beside a continuous-batching step's prefill chunks:
    num_chunks x chunk_tokens tokens (positions [prior, prior + chunk_tokens)
    with prior from the clipped Zipf of the mixed step), hidden states
    N(0, 1) of model_dim 4096, stacked W_q / W_k / W_v for GQA 32 q / 8 kv
    heads x 128 (N = 6144) scaled by 1/sqrt(model_dim), bf16; the K/V rows go
    to a pool of num_blocks blocks through seeded tables."""
    rng = np.random.Generator(np.random.PCG64(seed))
    priors = zipf_contexts(rng, num_chunks)
    need = (priors + chunk_tokens + BLOCK_TOKENS - 1) // BLOCK_TOKENS
    max_blocks = int(need.max())
    tables = _deal_tables(rng, num_blocks, need, max_blocks)
    pool = CudaKvPool(device, KV_BF16, num_blocks, BLOCK_TOKENS, 8, 128)
    gen = _generator(seed + 1, device)
    dev = f"cuda:{device}"
    tokens = num_chunks * chunk_tokens
    hidden = torch.randn((tokens, model_dim), generator=gen, device=dev).to(torch.bfloat16)
    weights = (torch.randn(((32 + 16) * 128, model_dim), generator=gen, device=dev) /
               model_dim ** 0.5).to(torch.bfloat16)
    seq = np.repeat(np.arange(num_chunks, dtype=np.int32), chunk_tokens)
    pos = np.concatenate([np.arange(p, p + chunk_tokens, dtype=np.int32) for p in priors])
    return ProjectionBatch(pool=pool, hidden=hidden, weights=weights, q_heads=32,
                           row_sequences=torch.from_numpy(seq).to(dev),
                           positions=torch.from_numpy(pos).to(dev),
                           block_tables=torch.from_numpy(tables).to(dev), tables_host=tables)


def long_sequence_shard(device: int, rank: int, world: int, total_tokens: int = 131072,
                        seed: int = 2030) -> PagedBatch:
    """One total_tokens-token sequence (GQA 32/8 x 128, bf16) whose blocks are
    split into `world` contiguous ranges; this rank's pool holds its range and
    the batch's single decode row covers it. The query is the same on every
    rank (seeded); K/V differ per range (seed + rank)."""
    from .distributed import local_tokens

    lo, hi = local_tokens(total_tokens, BLOCK_TOKENS, world, rank)
    local = hi - lo
    batch = decode_batch(device, seed + 1000 * (rank + 1), 1, np.array([local]), 32, 8, 128,
                         KV_BF16, max_context_len=local)
    gen = _generator(seed, device)
    batch.queries = torch.randn((1, 32, 128), generator=gen, device=f"cuda:{device}",
                                dtype=torch.float32)
    batch.extra.update({"token_range": (lo, hi), "total_tokens": total_tokens})
    return batch


def host_arenas(pool: CudaKvPool):
    """Host copies of the arenas as numpy (fp32, or uint16 storage bits)."""
    def grab(t):
        if pool.dtype == KV_FP32:
            return t.cpu().numpy()
        return t.view(torch.int16).cpu().numpy().view(np.uint16)

    return grab(pool.key_arena), grab(pool.value_arena)


def round_queries(queries: torch.Tensor, dtype: int) -> np.ndarray:
    """Queries as the kernels see them: rounded to the pool type, widened."""
    if dtype == KV_FP32:
        return queries.cpu().numpy()
    return queries.to(TORCH_DTYPES[dtype]).to(torch.float32).cpu().numpy()


__all__ = [
    "PagedBatch", "decode_batch", "decode_fp32", "longctx_bf16", "longctx_contexts",
    "prefill_batch", "prefill_f16", "zipf_contexts", "host_arenas", "round_queries",
    "mixed_bf16", "long_sequence_shard", "KV_FP32", "KV_F16", "KV_BF16",
]

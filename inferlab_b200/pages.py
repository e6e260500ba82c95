"""Block ownership for the device KV pool: a thin wrapper over the C ABI
(inferlab_cuda_pages_*, include/inferlab_attention.h).

The manager keeps the reference PagedKvPool's ownership model
(worker/cpp/inferlab_runtime.cpp:649-1032) on the host - free list,
reference counts, published prefixes with longest-prefix lookup and
least-recently-used eviction, copy on write of a shared tail block - while the
rows themselves live in a CudaKvPool on the device. A sequence is a block
table (list of block ids) plus its cached token count, as in the reference's
Session.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from .attention import AttentionError


def _check(status: int, error) -> None:
    if status != 0:
        raise AttentionError(error.value.decode())


def _i32(values) -> np.ndarray:
    return np.ascontiguousarray(values, dtype=np.int32)


class PageManager:
    """Host metadata of `page_count` blocks of `block_tokens` rows each;
    `row_bytes` = one token row of K and V over all kv-heads."""

    def __init__(self, page_count: int, block_tokens: int, row_bytes: int,
                 prefix_capacity: int = 0):
        self._lib = _lib.lib()
        handle = ctypes.c_void_p()
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_create(page_count, block_tokens, row_bytes,
                                                     prefix_capacity, ctypes.byref(handle),
                                                     error, len(error)), error)
        self._handle = handle
        self.block_tokens = block_tokens

    @classmethod
    def for_pool(cls, pool, prefix_capacity: int = 0) -> "PageManager":
        """A manager of every block of a CudaKvPool."""
        row = pool.kv_heads * pool.head_dim * 2 * pool.element_bytes
        return cls(pool.num_blocks, pool.block_tokens, row, prefix_capacity)

    def close(self) -> None:
        if self._handle:
            self._lib.inferlab_cuda_pages_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def prepare_append(self, table: list[int], cached_tokens: int):
        """Reserve the slot of token `cached_tokens`; returns the new table and
        the (from, to) block copy to run on the device first, or None
        (PagedKvPool::append's allocation policy, :710-767)."""
        cap = len(table) + 1
        buf = np.zeros(cap, np.int32)
        buf[:len(table)] = table
        length = ctypes.c_uint32(len(table))
        src = ctypes.c_int32(-1)
        dst = ctypes.c_int32(-1)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_prepare_append(
            self._handle, buf.ctypes.data_as(_lib.c_i32p), cap, ctypes.byref(length),
            cached_tokens, ctypes.byref(src), ctypes.byref(dst), error, len(error)), error)
        copy = None if src.value < 0 else (src.value, dst.value)
        return [int(x) for x in buf[:length.value]], copy

    def release(self, table: list[int]) -> None:
        buf = _i32(table)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_release(
            self._handle, buf.ctypes.data_as(_lib.c_i32p), len(buf), error, len(error)), error)

    def publish_prefix(self, tokens, table: list[int], cached_tokens: int) -> None:
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        buf = _i32(table)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_publish_prefix(
            self._handle, toks.ctypes.data_as(_lib.c_u32p), len(toks),
            buf.ctypes.data_as(_lib.c_i32p), len(buf), cached_tokens, error, len(error)), error)

    def acquire_prefix(self, tokens):
        """(blocks, prefix_tokens) of the longest published prefix, or ([], 0)."""
        toks = np.ascontiguousarray(tokens, dtype=np.uint32)
        cap = max(1, (len(toks) + self.block_tokens - 1) // self.block_tokens)
        buf = np.zeros(cap, np.int32)
        length = ctypes.c_uint32(0)
        ntok = ctypes.c_uint64(0)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_acquire_prefix(
            self._handle, toks.ctypes.data_as(_lib.c_u32p), len(toks),
            buf.ctypes.data_as(_lib.c_i32p), cap, ctypes.byref(length), ctypes.byref(ntok),
            error, len(error)), error)
        return [int(x) for x in buf[:length.value]], int(ntok.value)

    def shared_pages(self, table: list[int]) -> int:
        buf = _i32(table)
        out = ctypes.c_uint64(0)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_shared(
            self._handle, buf.ctypes.data_as(_lib.c_i32p), len(buf), ctypes.byref(out),
            error, len(error)), error)
        return int(out.value)

    def stats(self) -> dict:
        raw = _lib.InferlabPagedCacheStats()
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pages_stats(self._handle, ctypes.byref(raw), error,
                                                    len(error)), error)
        return {name: int(getattr(raw, name)) for name, _ in raw._fields_}


def copy_blocks(pool, copies, stream=None) -> None:
    """Run copy-on-write block copies [(from, to), ...] on the device pool."""
    if not copies:
        return
    import torch

    src = _i32([c[0] for c in copies])
    dst = _i32([c[1] for c in copies])
    if stream is None:
        stream = torch.cuda.current_stream(pool.device)
    error = _lib.error_buffer()
    _check(_lib.lib().inferlab_cuda_pages_copy(
        pool._handle, src.ctypes.data_as(_lib.c_i32p), dst.ctypes.data_as(_lib.c_i32p),
        len(copies), ctypes.c_void_p(stream.cuda_stream), error, len(error)), error)

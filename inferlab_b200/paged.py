"""Host-side API of the device-resident paged KV pool.

A CudaKvPool owns the HBM arenas that replace PagedKvPool's page storage
(worker/cpp/inferlab_runtime.cpp:649-1026). Block ids, block tables and
context lengths stay the caller's business, as in the reference where
the pool's host policy hands out page ids and the attention only follows the
table (docs/rfcs/0014-paged-kv-cache-prefix-ownership.md, "Logical block
tables"). Device arrays are torch tensors here only as HBM plumbing; every
kernel is a call into libinferlab_attention_cuda.so.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .attention import AttentionError

KV_FP32, KV_F16, KV_BF16 = 0, 1, 2
TORCH_DTYPES = {KV_FP32: torch.float32, KV_F16: torch.float16, KV_BF16: torch.bfloat16}
_TYPESTR = {KV_FP32: "<f4", KV_F16: "<f2", KV_BF16: "<u2"}


def _check(status: int, error) -> None:
    if status != 0:
        raise AttentionError(error.value.decode())


def _vp(tensor):
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def _stream_handle(device: int, stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream(device)
    return ctypes.c_void_p(stream.cuda_stream)


class _DeviceView:
    """Exposes a raw device range through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3,
            "strides": None,
        }


def _require(tensor: torch.Tensor, name: str, dtype, device: int) -> torch.Tensor:
    if not isinstance(tensor, torch.Tensor):
        raise AttentionError(f"{name} must be a torch tensor on cuda:{device}")
    if tensor.device.type != "cuda" or tensor.device.index != device:
        raise AttentionError(f"{name} must live on cuda:{device}")
    if dtype is not None and tensor.dtype != dtype:
        raise AttentionError(f"{name} must have dtype {dtype}")
    if not tensor.is_contiguous():
        raise AttentionError(f"{name} must be contiguous")
    return tensor


class CudaKvPool:
    """HBM block pool: arenas [num_blocks][kv_heads][block_tokens][head_dim]."""

    def __init__(self, device: int, dtype: int, num_blocks: int, block_tokens: int,
                 kv_heads: int, head_dim: int):
        self._lib = _lib.lib()
        handle = ctypes.c_void_p()
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pool_create(device, dtype, num_blocks, block_tokens,
                                                   kv_heads, head_dim, ctypes.byref(handle),
                                                   error, len(error)), error)
        self._handle = handle
        info = _lib.InferlabCudaPoolInfo()
        _check(self._lib.inferlab_cuda_pool_info(handle, ctypes.byref(info), error, len(error)),
               error)
        self.device = info.device
        self.dtype = info.dtype
        self.num_blocks = info.num_blocks
        self.block_tokens = info.block_tokens
        self.kv_heads = info.kv_heads
        self.head_dim = info.head_dim
        self.element_bytes = info.element_bytes
        self.arena_bytes = info.arena_bytes
        self._key_ptr = info.key_arena
        self._value_ptr = info.value_arena
        self._workspaces: dict = {}

    # -- lifetime -----------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_handle", None) is not None and self._handle.value:
            self._lib.inferlab_cuda_pool_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- views ----------------------------------------------------------------
    def _arena(self, ptr: int) -> torch.Tensor:
        shape = (self.num_blocks, self.kv_heads, self.block_tokens, self.head_dim)
        view = torch.as_tensor(_DeviceView(ptr, shape, _TYPESTR[self.dtype]),
                               device=f"cuda:{self.device}")
        return view.view(TORCH_DTYPES[self.dtype]) if self.dtype == KV_BF16 else view

    @property
    def key_arena(self) -> torch.Tensor:
        """A torch view of the key arena (no copy; valid while the pool lives)."""
        return self._arena(self._key_ptr)

    @property
    def value_arena(self) -> torch.Tensor:
        return self._arena(self._value_ptr)

    # -- kernels ----------------------------------------------------------------
    def synchronize(self, stream=None, timeout_ms: int = 0) -> None:
        """Bounded wait on the stream, then raise any error a kernel recorded."""
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pool_synchronize(
            self._handle, _stream_handle(self.device, stream), timeout_ms, error, len(error)),
            error)

    def append(self, key_rows: torch.Tensor, value_rows: torch.Tensor,
               row_sequences: torch.Tensor, positions: torch.Tensor, block_tables: torch.Tensor,
               stream=None) -> None:
        """Write token rows [n][kv_heads][head_dim] at (sequence, position) via the tables."""
        dev = self.device
        row_dtype = KV_FP32 if key_rows.dtype == torch.float32 else self.dtype
        if key_rows.dtype not in (torch.float32, TORCH_DTYPES[self.dtype]):
            raise AttentionError("paged KV row dtype must be FP32 or the pool dtype")
        _require(key_rows, "key_rows", key_rows.dtype, dev)
        _require(value_rows, "value_rows", key_rows.dtype, dev)
        _require(row_sequences, "row_sequences", torch.int32, dev)
        _require(positions, "positions", torch.int32, dev)
        _require(block_tables, "block_tables", torch.int32, dev)
        rows = key_rows.shape[0]
        if key_rows.numel() != rows * self.kv_heads * self.head_dim or \
                value_rows.shape != key_rows.shape or row_sequences.numel() != rows or \
                positions.numel() != rows:
            raise AttentionError("paged KV append shapes do not match the pool")
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_kv_append(
            self._handle, _vp(key_rows), _vp(value_rows), row_dtype, _vp(row_sequences),
            _vp(positions), rows, _vp(block_tables), block_tables.shape[-1],
            _stream_handle(dev, stream), error, len(error)), error)

    def project_append(self, hidden: torch.Tensor, weights: torch.Tensor, q_heads: int,
                       row_sequences: torch.Tensor, positions: torch.Tensor,
                       block_tables: torch.Tensor, q_out: torch.Tensor | None = None,
                       stream=None) -> torch.Tensor:
        """Q/K/V projection of hidden [tokens][model_dim] by the stacked
        weights [(q_heads + 2 kv_heads) head_dim][model_dim] (pool type, F16 or
        BF16 pools): returns Q [tokens][q_heads][head_dim] and writes every
        token's K/V rows into the pool at (row_sequences[t], positions[t])
        (inferlab_cuda_qkv_project_append)."""
        dev = self.device
        dtype = TORCH_DTYPES.get(self.dtype)
        _require(hidden, "hidden", dtype, dev)
        _require(weights, "weights", dtype, dev)
        _require(row_sequences, "row_sequences", torch.int32, dev)
        _require(positions, "positions", torch.int32, dev)
        _require(block_tables, "block_tables", torch.int32, dev)
        tokens, model_dim = hidden.shape
        if weights.shape != ((q_heads + 2 * self.kv_heads) * self.head_dim, model_dim) or \
                row_sequences.numel() != tokens or positions.numel() != tokens or \
                block_tables.dim() != 2:
            raise AttentionError("projection shapes do not match the pool")
        if q_out is None:
            q_out = torch.empty((tokens, q_heads, self.head_dim), dtype=dtype, device=f"cuda:{dev}")
        _require(q_out, "q_out", dtype, dev)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_qkv_project_append(
            self._handle, _vp(hidden), _vp(weights), tokens, model_dim, q_heads,
            _vp(row_sequences), _vp(positions), _vp(block_tables), block_tables.shape[0],
            block_tables.shape[1], _vp(q_out), _stream_handle(dev, stream), error, len(error)),
            error)
        return q_out

    def output_project(self, attention: torch.Tensor, weights: torch.Tensor,
                       residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
                       stream=None) -> torch.Tensor:
        """out = residual + attention @ weights.T on the tensor cores
        (inferlab_cuda_output_project): attention [tokens][in_dim] fp32 or
        the pool type, weights [out_dim][in_dim] in the pool type, residual /
        out [tokens][out_dim] fp32."""
        dev = self.device
        dtype = TORCH_DTYPES.get(self.dtype)
        if attention.dtype not in (torch.float32, dtype):
            raise AttentionError("projection input dtype must be FP32 or the pool dtype")
        _require(attention, "attention", attention.dtype, dev)
        _require(weights, "weights", dtype, dev)
        tokens, in_dim = attention.shape
        out_dim = weights.shape[0]
        if weights.shape[1] != in_dim:
            raise AttentionError("projection shapes do not match")
        if residual is not None:
            _require(residual, "residual", torch.float32, dev)
            if residual.shape != (tokens, out_dim):
                raise AttentionError("projection shapes do not match")
        if out is None:
            out = torch.empty((tokens, out_dim), dtype=torch.float32, device=f"cuda:{dev}")
        _require(out, "out", torch.float32, dev)
        a_dtype = KV_FP32 if attention.dtype == torch.float32 else self.dtype
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_output_project(
            self._handle, _vp(attention), a_dtype, _vp(weights),
            None if residual is None else _vp(residual), tokens, in_dim, out_dim, _vp(out),
            _stream_handle(dev, stream), error, len(error)), error)
        return out

    def gather(self, block_table: torch.Tensor, tokens: int, stream=None):
        """Contiguous copies [tokens][kv_heads][head_dim] of one sequence's K and V."""
        dev = self.device
        _require(block_table, "block_table", torch.int32, dev)
        if block_table.numel() != (tokens + self.block_tokens - 1) // self.block_tokens:
            raise AttentionError("paged KV block table length is inconsistent")
        shape = (tokens, self.kv_heads, self.head_dim)
        keys = torch.empty(shape, dtype=TORCH_DTYPES[self.dtype], device=f"cuda:{dev}")
        values = torch.empty_like(keys)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_kv_gather(
            self._handle, _vp(block_table), tokens, _vp(keys), _vp(values),
            _stream_handle(dev, stream), error, len(error)), error)
        return keys, values

    def workspace_size(self, num_seqs: int, q_heads: int, max_context_len: int) -> int:
        return int(self._lib.inferlab_cuda_paged_decode_workspace_size(
            self._handle, num_seqs, q_heads, max_context_len))

    def make_workspace(self, num_seqs: int, q_heads: int, max_context_len: int,
                       stream=None) -> torch.Tensor:
        """A zero-initialised decode workspace for this batch shape."""
        size = max(16, self.workspace_size(num_seqs, q_heads, max_context_len))
        ws = torch.empty(size, dtype=torch.uint8, device=f"cuda:{self.device}")
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_paged_decode_workspace_init(
            _vp(ws), size, _stream_handle(self.device, stream), error, len(error)), error)
        return ws

    def set_decode_split(self, blocks_per_split: int) -> None:
        """Fixes later decodes' split length at blocks_per_split 16-token
        blocks (0: the planner chooses, the default). A tuning and test knob
        (inferlab_cuda_pool_set_decode_split)."""
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_pool_set_decode_split(
            self._handle, int(blocks_per_split), error, len(error)), error)

    def _cached_workspace(self, num_seqs, q_heads, max_context_len, stream):
        """The pool's own decode workspace, kept per stream: decodes on one
        stream run in order and may share it, decodes on two streams would race
        on its split counters and partials. A workspace outgrown on a stream is
        replaced only after that stream has finished with it (record_stream)."""
        need = self.workspace_size(num_seqs, q_heads, max_context_len)
        key = _stream_handle(self.device, stream).value
        ws = self._workspaces.get(key)
        if ws is None or ws.numel() < need:
            if ws is not None:
                ws.record_stream(stream if stream is not None
                                 else torch.cuda.current_stream(self.device))
            ws = self.make_workspace(num_seqs, q_heads, max_context_len, stream)
            self._workspaces[key] = ws
        return ws

    def decode(self, queries: torch.Tensor, block_tables: torch.Tensor,
               context_lens: torch.Tensor, max_context_len: int | None = None,
               out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
        """One decode step: queries [num_seqs][q_heads][head_dim] fp32 -> fp32 output."""
        dev = self.device
        _require(queries, "queries", torch.float32, dev)
        _require(block_tables, "block_tables", torch.int32, dev)
        _require(context_lens, "context_lens", torch.int32, dev)
        num_seqs, q_heads, hd = queries.shape
        if hd != self.head_dim or context_lens.numel() != num_seqs or \
                block_tables.shape[0] != num_seqs:
            raise AttentionError("paged decode shapes do not match the pool")
        if max_context_len is None:
            max_context_len = int(context_lens.max().item())
        if out is None:
            out = torch.empty_like(queries)
        _require(out, "out", torch.float32, dev)
        if workspace is None:
            workspace = self._cached_workspace(num_seqs, q_heads, max_context_len, stream)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_paged_decode(
            self._handle, _vp(queries), _vp(block_tables), block_tables.shape[1],
            _vp(context_lens), num_seqs, q_heads, max_context_len, _vp(out), _vp(workspace),
            workspace.numel(), _stream_handle(dev, stream), error, len(error)), error)
        return out

    def decode_step_host(self, queries, block_tables, context_lens, new_keys=None,
                         new_values=None, out=None, stream=None, timeout_ms: int = 0,
                         block_copies=None):
        """One synchronous decode step from host (numpy) arrays: append the new
        token rows at context_lens - 1 (if given), decode every sequence, return
        the output as a host array. One C call (inferlab_cuda_decode_step_host).
        block_copies: per sequence the (from, to) copy-on-write pair that
        PageManager.prepare_append returned, or (-1, -1); the copies run in the
        same call before the rows are written (inferlab_cuda_decode_step_host_cow)."""
        import numpy as np

        q = np.ascontiguousarray(queries, dtype=np.float32)
        tables = np.ascontiguousarray(block_tables, dtype=np.int32)
        lens = np.ascontiguousarray(context_lens, dtype=np.int32)
        num_seqs, q_heads, _ = q.shape
        if out is None:
            out = np.empty_like(q)
        elif not (isinstance(out, np.ndarray) and out.dtype == np.float32 and
                  out.flags.c_contiguous and out.shape == q.shape):
            raise AttentionError("decode step output must be a contiguous float32 array shaped "
                                 "like the queries")
        keys = None if new_keys is None else np.ascontiguousarray(new_keys, dtype=np.float32)
        values = None if new_values is None else np.ascontiguousarray(new_values, dtype=np.float32)
        error = _lib.error_buffer()
        # Plain addresses: the per-step path avoids ctypes pointer objects.
        kp = None if keys is None else keys.ctypes.data
        vp = None if values is None else values.ctypes.data
        if block_copies is None:
            _check(self._lib.inferlab_cuda_decode_step_host(
                self._handle, q.ctypes.data, kp, vp, tables.ctypes.data, tables.shape[1],
                lens.ctypes.data, num_seqs, q_heads, out.ctypes.data,
                _stream_handle(self.device, stream), timeout_ms, error, len(error)), error)
            return out
        copies = np.ascontiguousarray(block_copies, dtype=np.int32)
        if copies.shape != (num_seqs, 2):
            raise AttentionError("decode step block copies must be [num_seqs][2]")
        _check(self._lib.inferlab_cuda_decode_step_host_cow(
            self._handle, q.ctypes.data, kp, vp, copies.ctypes.data, tables.ctypes.data,
            tables.shape[1], lens.ctypes.data, num_seqs, q_heads, out.ctypes.data,
            _stream_handle(self.device, stream), timeout_ms, error, len(error)), error)
        return out

    def decode_partials(self, queries: torch.Tensor, block_tables: torch.Tensor,
                        context_lens: torch.Tensor, max_context_len: int | None = None,
                        workspace: torch.Tensor | None = None, stream=None,
                        packed: torch.Tensor | None = None):
        """Split-KV partials (m, l, o) over this pool's part of each context.
        With `packed` (fp32, rows * (head_dim + 2) elements, rows = num_seqs *
        q_heads) they are written into it as [m | l | o], the layout
        lse_combine_packed merges after an all-gather."""
        dev = self.device
        _require(queries, "queries", torch.float32, dev)
        _require(block_tables, "block_tables", torch.int32, dev)
        _require(context_lens, "context_lens", torch.int32, dev)
        num_seqs, q_heads, hd = queries.shape
        if max_context_len is None:
            max_context_len = int(context_lens.max().item())
        if packed is not None:
            rows = num_seqs * q_heads
            _require(packed, "packed", torch.float32, dev)
            if packed.numel() != rows * (hd + 2):
                raise AttentionError("packed partials buffer has the wrong size")
            flat = packed.view(-1)
            m = flat[:rows].view(num_seqs, q_heads)
            l = flat[rows:2 * rows].view(num_seqs, q_heads)
            o = flat[2 * rows:].view(num_seqs, q_heads, hd)
        else:
            m = torch.empty((num_seqs, q_heads), dtype=torch.float32, device=f"cuda:{dev}")
            l = torch.empty_like(m)
            o = torch.empty_like(queries)
        if workspace is None:
            workspace = self._cached_workspace(num_seqs, q_heads, max_context_len, stream)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_paged_decode_partials(
            self._handle, _vp(queries), _vp(block_tables), block_tables.shape[1],
            _vp(context_lens), num_seqs, q_heads, max_context_len, _vp(m), _vp(l), _vp(o),
            _vp(workspace), workspace.numel(), _stream_handle(dev, stream), error, len(error)),
            error)
        return m, l, o

    def prefill(self, queries: torch.Tensor, block_tables: torch.Tensor,
                query_starts: torch.Tensor, query_counts: torch.Tensor,
                query_offsets: torch.Tensor, max_query_count: int,
                out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Causal (chunked) prefill of segments whose K/V are already in the pool."""
        dev = self.device
        if queries.dtype == torch.float32:
            qtype = KV_FP32
        elif queries.dtype == TORCH_DTYPES[self.dtype]:
            qtype = self.dtype
        else:
            raise AttentionError("paged prefill query dtype must be FP32 or the pool dtype")
        _require(queries, "queries", None, dev)
        for name, t in (("block_tables", block_tables), ("query_starts", query_starts),
                        ("query_counts", query_counts), ("query_offsets", query_offsets)):
            _require(t, name, torch.int32, dev)
        total, q_heads, hd = queries.shape
        if hd != self.head_dim:
            raise AttentionError("paged prefill head_dim does not match the pool")
        if out is None:
            out = torch.empty((total, q_heads, hd), dtype=torch.float32, device=f"cuda:{dev}")
        _require(out, "out", torch.float32, dev)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_paged_prefill(
            self._handle, _vp(queries), qtype, _vp(block_tables), block_tables.shape[1],
            _vp(query_starts), _vp(query_counts), _vp(query_offsets), query_starts.numel(),
            q_heads, max_query_count, total, _vp(out), _stream_handle(dev, stream), error,
            len(error)), error)
        return out


def lse_combine(part_m: torch.Tensor, part_l: torch.Tensor, part_o: torch.Tensor,
                out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Merge partials [parts][rows], [parts][rows][head_dim] in part order."""
    dev = part_o.device.index
    parts = part_o.shape[0]
    rows = math.prod(part_o.shape[1:-1])
    hd = part_o.shape[-1]
    for name, t in (("part_m", part_m), ("part_l", part_l), ("part_o", part_o)):
        _require(t, name, torch.float32, dev)
    if out is None:
        out = torch.empty(part_o.shape[1:], dtype=torch.float32, device=part_o.device)
    error = _lib.error_buffer()
    _check(_lib.lib().inferlab_cuda_lse_combine(
        _vp(part_m), _vp(part_l), _vp(part_o), parts, rows, hd, _vp(out),
        _stream_handle(dev, stream), error, len(error)), error)
    return out


def lse_combine_packed(packed: torch.Tensor, parts: int, rows: int, head_dim: int,
                       out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Merge `parts` packed [m | l | o] partial blocks (part order) into
    [rows][head_dim]."""
    dev = packed.device.index
    _require(packed, "packed", torch.float32, dev)
    if packed.numel() != parts * rows * (head_dim + 2):
        raise AttentionError("packed partials buffer has the wrong size")
    if out is None:
        out = torch.empty((rows, head_dim), dtype=torch.float32, device=packed.device)
    error = _lib.error_buffer()
    _check(_lib.lib().inferlab_cuda_lse_combine_packed(
        _vp(packed), parts, rows, head_dim, _vp(out), _stream_handle(dev, stream), error,
        len(error)), error)
    return out

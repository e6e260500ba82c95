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
  arrival order; on GPUs `PeerExchange` does the exchange and the merge in one
  kernel over NVLink peer memory instead.
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


class PeerExchange:
    """The all-gather of packed [m | l | o] partials and their rank-order merge
    in one kernel over NVLink peer memory (inferlab_cuda_peer_exchange_*): each
    rank's receive buffer is opened by its peers through CUDA IPC handles swapped
    over the process group once; per call the kernel stores this rank's block
    into every peer's buffer as 8-byte words tagged with the call's step number,
    waits (bounded) until every rank's words carry that step and merges. The
    fused form (`decode`) does the same from inside the decode kernel. One
    process per GPU, every rank on its own GPU (ranks sharing a GPU would wait
    on each other from separate launches), every rank makes the same sequence
    of calls, and a rank's calls run in order on the GPU (one stream, or
    streams ordered by events). Setting up is collective and agreed: if any
    rank cannot allocate or open a buffer, every rank raises RuntimeError (and
    holds nothing), so callers can fall back together."""

    def __init__(self, rows: int, head_dim: int, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib
        from .paged import _check

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.head_dim = int(rows), int(head_dim)
        self.device = torch.cuda.current_device()
        self._lib = _lib.lib()
        if self.world > 8:
            raise ValueError("the peer exchange covers up to 8 ranks")
        uuids = [None] * self.world
        dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid),
                               group=group)
        if len(set(uuids)) != self.world:
            raise ValueError("the peer exchange needs one GPU per rank")
        def agree(ok: bool) -> bool:
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=f"cuda:{self.device}")
            dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
            return bool(flag.item())

        nbytes = self._lib.inferlab_cuda_peer_buffer_bytes(self.world, self.rows, self.head_dim)
        handle = ctypes.create_string_buffer(64)
        self._buffer = ctypes.c_void_p()
        self._handle = None
        error = _lib.error_buffer()
        status = self._lib.inferlab_cuda_peer_buffer_alloc(self.device, nbytes, ctypes.byref(self._buffer),
                                                           handle, error, len(error))
        if not agree(status == 0):
            if status == 0:
                self._lib.inferlab_cuda_peer_buffer_free(self.device, self._buffer, error, len(error))
            raise RuntimeError("peer exchange buffers could not be allocated on every rank: "
                               + error.value.decode())
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        joined = ctypes.create_string_buffer(b"".join(handles), 64 * self.world)
        made = ctypes.c_void_p()
        status = self._lib.inferlab_cuda_peer_exchange_create(
            self.device, self.world, self.rank, self.rows, self.head_dim, self._buffer, joined,
            ctypes.byref(made), error, len(error))
        if not agree(status == 0):
            if status == 0:
                self._lib.inferlab_cuda_peer_exchange_destroy(made)
            dist.barrier(group=group)  # no rank still holds a peer's buffer open
            self._lib.inferlab_cuda_peer_buffer_free(self.device, self._buffer, error, len(error))
            raise RuntimeError("peer exchange buffers could not be opened on every rank: "
                               + error.value.decode())
        self._handle = made
        dist.barrier(group=group)  # every rank's buffer is open before the first push

    def combine(self, packed, out=None, stream=None):
        """Merged [rows, head_dim] output of every rank's packed block (this
        rank's is `packed`); asynchronous on the current stream."""
        import torch

        from . import _lib
        from .paged import _check, _stream_handle, _vp

        if out is None:
            out = torch.empty((self.rows, self.head_dim), dtype=torch.float32, device=packed.device)
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_peer_exchange_combine(
            self._handle, _vp(packed), _vp(out), _stream_handle(self.device, stream), error,
            len(error)), error)
        return out

    def decode(self, pool, queries, block_table, context_lens, max_context_len: int, workspace=None,
               out=None, stream=None):
        """This rank's block range decoded and exchanged in one kernel
        (inferlab_cuda_paged_decode_exchange): the merged [rows, q_heads,
        head_dim] output of all ranks' ranges, asynchronous."""
        import torch

        from . import _lib
        from .paged import _check, _stream_handle, _vp

        num_seqs, q_heads, hd = queries.shape
        if out is None:
            out = torch.empty((num_seqs, q_heads, hd), dtype=torch.float32, device=queries.device)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_paged_decode_exchange(
            pool._handle, _vp(queries), _vp(block_table), block_table.shape[1], _vp(context_lens),
            num_seqs, q_heads, int(max_context_len), _vp(workspace), ws_bytes, self._handle,
            _vp(out), _stream_handle(self.device, stream), error, len(error)), error)
        return out

    def synchronize(self, stream=None, timeout_ms: int = 0) -> None:
        """Waits for the stream and raises if a peer's block never arrived."""
        from . import _lib
        from .paged import _check, _stream_handle

        error = _lib.error_buffer()
        _check(self._lib.inferlab_cuda_peer_exchange_synchronize(
            self._handle, _stream_handle(self.device, stream), int(timeout_ms), error, len(error)),
            error)

    def close(self) -> None:
        """Releases the peers' buffers and this rank's (after every rank's last
        exchange: a barrier first)."""
        import torch
        import torch.distributed as dist

        from . import _lib

        if self._handle is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._lib.inferlab_cuda_peer_exchange_destroy(self._handle)
        self._handle = None
        dist.barrier(group=self.group)  # no peer still holds this rank's buffer open
        error = _lib.error_buffer()
        self._lib.inferlab_cuda_peer_buffer_free(self.device, self._buffer, error, len(error))


# Per (device, rows, local length): the constant lengths tensor of the split decode.
_LENGTHS: dict = {}


def decode_split_sequence(pool, queries, block_table, local_len: int, group=None, workspace=None,
                          exchange: PeerExchange | None = None):
    """Decode one query per row against a sequence whose blocks are spread
    over the ranks: this rank's blocks are `block_table` (device int32
    [rows, blocks]) covering `local_len` tokens. Returns the merged output
    [rows, q_heads, head_dim] on every rank.

    With `exchange`, one kernel decodes this rank's range and exchanges and
    merges the partials of all ranks over NVLink (a rank without blocks
    exchanges an empty block). Otherwise the partials are written straight
    into one packed [m | l | o] block, the blocks of all ranks are exchanged
    with a single all-gather (NCCL), and one kernel merges them."""
    import torch
    import torch.distributed as dist

    from .paged import lse_combine_packed

    rows, q_heads, hd = queries.shape
    nrows = rows * q_heads
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if exchange is not None and local_len > 0:
        key = (queries.device.index, rows, local_len)
        lens = _LENGTHS.get(key)
        if lens is None:
            lens = _LENGTHS[key] = torch.full((rows,), local_len, dtype=torch.int32,
                                              device=queries.device)
        if workspace is None:
            workspace = pool.make_workspace(rows, q_heads, local_len)
        return exchange.decode(pool, queries, block_table, lens, local_len, workspace=workspace)
    send = torch.empty(nrows * (hd + 2), dtype=torch.float32, device=queries.device)
    if local_len > 0:
        key = (queries.device.index, rows, local_len)
        lens = _LENGTHS.get(key)
        if lens is None:  # made once: a fill kernel per call would sit in every step
            lens = _LENGTHS[key] = torch.full((rows,), local_len, dtype=torch.int32,
                                              device=queries.device)
        pool.decode_partials(queries, block_table, lens, local_len, workspace=workspace,
                             packed=send)
    else:
        send[:nrows].fill_(float("-inf"))
        send[nrows:].zero_()
    if exchange is not None:
        return exchange.combine(send).view(rows, q_heads, hd)
    if world > 1:
        recv = torch.empty(world * send.numel(), dtype=torch.float32, device=queries.device)
        dist.all_gather_into_tensor(recv, send, group=group)
    else:
        recv = send
    return lse_combine_packed(recv, world, nrows, hd).view(rows, q_heads, hd)

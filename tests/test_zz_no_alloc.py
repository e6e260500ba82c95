"""The allocation-free decode entry point, checked against the workspace one.

inferlab_cuda_paged_decode_noalloc serves callers that cannot allocate device
memory (for example a process whose GPU memory is reserved up front by another
framework's allocator): its split-KV scratch is an array built into the
library instead of a caller workspace. Called through the C ABI, twice in a
row (the array keeps the previous call's contents), it must give the same
output as inferlab_cuda_paged_decode within the fp32 tolerance
|a - b| <= 1e-6 + 1e-5 * |b|. This file is collected last so that a run that
stops at its first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def close(got, ref):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    err = np.abs(got - ref)
    bad = err > 1e-6 + 1e-5 * np.abs(ref)
    assert not bad.any(), f"{bad.sum()}/{bad.size} outside tolerance, max abs err {err.max():.3e}"


def call_noalloc(pool, queries, tables, lens, max_ctx, out):
    import torch

    from inferlab_b200 import _lib

    err = ctypes.create_string_buffer(512)
    status = _lib.lib().inferlab_cuda_paged_decode_noalloc(
        pool._handle, ctypes.c_void_p(queries.data_ptr()), ctypes.c_void_p(tables.data_ptr()),
        tables.shape[1], ctypes.c_void_p(lens.data_ptr()), queries.shape[0], queries.shape[1],
        max_ctx, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream(pool.device).cuda_stream), err, 512)
    return status, err.value.decode()


@pytest.mark.parametrize("kind", ["fp32_mha", "bf16_gqa"])
def test_noalloc_decode_matches_workspace_decode(kind):
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    from inferlab_b200 import workloads as wl

    if kind == "fp32_mha":
        batch = wl.decode_fp32(device=0, seed=303)  # 64 seqs, contexts split across CTAs
    else:
        contexts = np.array([1, 17, 2048, 5000, 8192, 300])
        batch = wl.decode_batch(0, 304, len(contexts), contexts, 32, 8, 128, wl.KV_BF16,
                                max_context_len=8192)
    pool = batch.pool
    ref = pool.decode(batch.queries, batch.block_tables, batch.context_lens,
                      batch.max_context_len)
    pool.synchronize()
    ref = ref.cpu().numpy()
    for _ in range(2):
        out = torch.full_like(batch.queries, float("nan"))
        status, message = call_noalloc(pool, batch.queries, batch.block_tables,
                                       batch.context_lens, batch.max_context_len, out)
        assert status == 0, message
        pool.synchronize()
        close(out.cpu().numpy(), ref)
    pool.close()


SCRATCH_BYTES = 16 << 20  # the array built into the library


def test_noalloc_decode_rejects_split_batches_beyond_its_scratch():
    """64 sequences x 64 q-heads over 8 kv-heads x 128 at a 32768-token bound:
    the contexts split 8 ways and the partials need more than 16 MiB."""
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    from inferlab_b200 import workloads as wl

    batch = wl.decode_batch(0, 305, 1, np.array([16]), 8, 8, 128, wl.KV_BF16,
                            max_context_len=16)
    assert batch.pool.workspace_size(64, 64, 32768) > SCRATCH_BYTES
    queries = torch.zeros((64, 64, 128), dtype=torch.float32, device="cuda:0")
    tables = torch.zeros((64, 2048), dtype=torch.int32, device="cuda:0")
    lens = torch.full((64,), 32768, dtype=torch.int32, device="cuda:0")
    out = torch.empty_like(queries)
    status, message = call_noalloc(batch.pool, queries, tables, lens, 32768, out)
    assert status == -1
    assert "bytes of scratch" in message and "16777216" in message
    batch.pool.close()


def test_noalloc_decode_single_split_batch_needs_no_scratch():
    """1024 sequences x 32 q-heads x 128 with contexts <= 512: every context
    fits one split, so no scratch is read even though a caller workspace for
    the shape would be larger than the built-in array."""
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    from inferlab_b200 import workloads as wl

    rng = np.random.Generator(np.random.PCG64(306))
    contexts = rng.integers(1, 512, size=1024, endpoint=True)
    batch = wl.decode_batch(0, 306, len(contexts), contexts, 32, 8, 128, wl.KV_BF16,
                            max_context_len=512)
    pool = batch.pool
    assert pool.workspace_size(1024, 32, 512) > SCRATCH_BYTES
    ref = pool.decode(batch.queries, batch.block_tables, batch.context_lens, 512)
    pool.synchronize()
    ref = ref.cpu().numpy()
    out = torch.full_like(batch.queries, float("nan"))
    status, message = call_noalloc(pool, batch.queries, batch.block_tables, batch.context_lens,
                                   512, out)
    assert status == 0, message
    pool.synchronize()
    close(out.cpu().numpy(), ref)
    pool.close()


def test_noalloc_decode_split_batch_just_under_the_limit_twice():
    """120 sequences x 32 q-heads x 128 at a 32768-token bound split 8 ways:
    the partials take about 95% of the array. Two calls in a row."""
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    from inferlab_b200 import workloads as wl

    rng = np.random.Generator(np.random.PCG64(307))
    contexts = rng.integers(1, 32768, size=120, endpoint=True)
    contexts[:6] = [32768, 32767, 4097, 4096, 17, 1]
    batch = wl.decode_batch(0, 307, len(contexts), contexts, 32, 8, 128, wl.KV_BF16,
                            max_context_len=32768)
    pool = batch.pool
    need = pool.workspace_size(120, 32, 32768)
    assert 0.9 * SCRATCH_BYTES < need <= SCRATCH_BYTES
    ref = pool.decode(batch.queries, batch.block_tables, batch.context_lens, 32768)
    pool.synchronize()
    ref = ref.cpu().numpy()
    for _ in range(2):
        out = torch.full_like(batch.queries, float("nan"))
        status, message = call_noalloc(pool, batch.queries, batch.block_tables,
                                       batch.context_lens, 32768, out)
        assert status == 0, message
        pool.synchronize()
        close(out.cpu().numpy(), ref)
    pool.close()

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


def test_noalloc_decode_rejects_batches_beyond_its_scratch():
    import torch

    assert torch.cuda.is_available(), "this test needs a CUDA device"
    from inferlab_b200 import workloads as wl

    contexts = np.full(64, 32768)
    batch = wl.decode_batch(0, 305, 1, contexts[:1], 32, 8, 128, wl.KV_BF16,
                            max_context_len=32768)
    queries = torch.zeros((4096, 32, 128), dtype=torch.float32, device="cuda:0")
    tables = torch.zeros((4096, 2048), dtype=torch.int32, device="cuda:0")
    lens = torch.full((4096,), 32768, dtype=torch.int32, device="cuda:0")
    out = torch.empty_like(queries)
    status, message = call_noalloc(batch.pool, queries, tables, lens, 32768, out)
    assert status == -1
    assert "bytes of scratch" in message and "16777216" in message
    batch.pool.close()

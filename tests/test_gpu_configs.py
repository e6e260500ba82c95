"""GPU parity at the benchmark configurations that combine several launches.

- The continuous-batching mixed step at its full configuration: 32 decode
  sequences with contexts Zipf(1.1) clipped to [32, 8192] and 4 chunked
  prefill segments of 512 tokens with prior context from the same clipped
  Zipf; GQA 32 q / 8 kv heads x 128, bf16 KV, 16-token blocks, a 65,536-block
  pool (seed 2029, the bench's). Both launches of the step run; every decode
  row is compared with the reference's decode call shape per (sequence,
  q-head), attention_forward(q, K, V, 1, T, 1, d, T - 1)
  (worker/cpp/inferlab_runtime.cpp:1458-1470), and every chunk row with its
  causal rule (query i of a chunk at prior P sees keys [0, P + i],
  kernels/attention_cpu.cpp:113-123), both through the oracle.
  Decode (fp32 arithmetic on the stored bf16 values): |gpu - ref| <= 1e-6 +
  1e-5 |ref|. Chunks (tensor cores, fp16 probabilities): |gpu - ref| <=
  2e-3 |ref| + 1e-3 max|ref row|.
- One 131,072-token sequence (GQA 32/8 x 128, bf16) split into 8 contiguous
  block ranges exactly as the 8-GPU split assigns them
  (inferlab_b200.distributed.local_tokens): each range is decoded into
  packed [m | l | o] partials, the 8 blocks are merged in range order by
  inferlab_cuda_lse_combine_packed (what each rank runs after the NCCL
  all-gather), and the result is compared with the oracle's whole-sequence
  attention within the fp32 tolerance.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL_16, ROW_ATOL_16 = 2e-3, 1e-3


@pytest.fixture(scope="module")
def wl():
    import torch

    assert torch.cuda.is_available(), "these tests need a CUDA device"
    from inferlab_b200 import workloads

    return workloads


def compact_arenas(pool, rows):
    """Host copies of only the blocks that `rows` name: rows is a list of
    (table row, blocks used). Returns (k, v, remap) with remap[old id] = new
    index, so a table maps with remap[table]."""
    import torch

    ids = np.unique(np.concatenate([np.asarray(t[:n]) for t, n in rows]).astype(np.int64))
    index = torch.from_numpy(ids).to(f"cuda:{pool.device}")

    def grab(arena):
        part = arena.index_select(0, index)
        if part.dtype == torch.float32:
            return part.cpu().numpy()
        return part.view(torch.int16).cpu().numpy().view(np.uint16)

    remap = np.full(pool.num_blocks, -1, np.int64)
    remap[ids] = np.arange(len(ids))
    return grab(pool.key_arena), grab(pool.value_arena), remap


def errors(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    row = np.max(np.abs(ref), axis=-1, keepdims=True)
    big = np.abs(ref) > 1e-2
    return {"max_abs": float(err.max()),
            "max_rel_ref_gt_1e-2": float((err[big] / np.abs(ref[big])).max()) if big.any() else 0.0,
            "max_err_over_rowmax": float(np.max(err / np.maximum(row, 1e-30)))}


def test_mixed_step_full_configuration(wl, oracle_mod):
    import torch

    batch = wl.mixed_bf16(device=0, seed=2029)
    pool = batch.pool
    # the realised lengths of this seed, recorded
    assert int(batch.contexts.sum()) == 102644 and batch.contexts.max() == 8192
    assert batch.starts.tolist() == [33, 8192, 8192, 8192]
    out_d = pool.decode(batch.queries, batch.block_tables, batch.context_lens,
                        batch.max_context_len)
    out_p = torch.empty((batch.prefill_queries.shape[0], 32, 128), dtype=torch.float32,
                        device="cuda:0")
    pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev, batch.counts_dev,
                 batch.offsets_dev, int(batch.counts.max()), out=out_p)
    pool.synchronize()

    need_d = (batch.contexts + 15) // 16
    need_p = (batch.starts + batch.counts + 15) // 16
    rows = [(batch.tables_host[i], int(n)) for i, n in enumerate(need_d)]
    rows += [(batch.prefill_tables_host[i], int(n)) for i, n in enumerate(need_p)]
    k_host, v_host, remap = compact_arenas(pool, rows)
    tables_d = np.where(np.arange(batch.tables_host.shape[1])[None, :] < need_d[:, None],
                        remap[batch.tables_host], 0).astype(np.int32)
    tables_p = np.where(np.arange(batch.prefill_tables_host.shape[1])[None, :] < need_p[:, None],
                        remap[batch.prefill_tables_host], 0).astype(np.int32)

    ref_d = oracle_mod.paged_attention(k_host, v_host, wl.KV_BF16, tables_d, batch.contexts - 1,
                                       np.ones(len(batch.contexts)),
                                       wl.round_queries(batch.queries, wl.KV_BF16), 32)
    got_d = out_d.cpu().numpy().astype(np.float64)
    err_d = np.abs(got_d - ref_d)
    bad = err_d > 1e-6 + 1e-5 * np.abs(ref_d)
    assert not bad.any(), f"decode: {bad.sum()}/{bad.size} outside, max abs {err_d.max():.3e}"

    ref_p = oracle_mod.paged_attention(k_host, v_host, wl.KV_BF16, tables_p, batch.starts,
                                       batch.counts, batch.prefill_queries.float().cpu().numpy(),
                                       32)
    got_p = out_p.cpu().numpy().astype(np.float64)
    row = np.max(np.abs(ref_p), axis=-1, keepdims=True)
    err_p = np.abs(got_p - ref_p)
    print("mixed step chunk parity:", errors(got_p, ref_p))
    bad = err_p > RTOL_16 * np.abs(ref_p) + ROW_ATOL_16 * row
    assert not bad.any(), f"chunks: {bad.sum()}/{bad.size} outside, {errors(got_p, ref_p)}"
    pool.close()


def test_long_sequence_split_eight_ways(wl, oracle_mod):
    import torch

    from inferlab_b200 import distributed
    from inferlab_b200.paged import lse_combine_packed

    total, world = 131072, 8
    batch = wl.decode_batch(0, 2030, 1, np.array([total]), 32, 8, 128, wl.KV_BF16,
                            max_context_len=total)
    pool = batch.pool
    rows = 32
    packed = torch.empty((world, rows * (128 + 2)), dtype=torch.float32, device="cuda:0")
    ranges = []
    for rank in range(world):
        lo, hi = distributed.local_tokens(total, 16, world, rank)
        ranges.append((lo, hi))
        table = batch.block_tables[:, lo // 16:(hi + 15) // 16].contiguous()
        lens = torch.full((1,), hi - lo, dtype=torch.int32, device="cuda:0")
        pool.decode_partials(batch.queries, table, lens, hi - lo, packed=packed[rank])
    assert ranges[0] == (0, 16384) and ranges[-1] == (114688, 131072)
    merged = lse_combine_packed(packed.view(-1), world, rows, 128)
    whole = pool.decode(batch.queries, batch.block_tables, batch.context_lens, total)
    pool.synchronize()

    k_host, v_host = wl.host_arenas(pool)
    ref = oracle_mod.paged_attention(k_host, v_host, wl.KV_BF16, batch.tables_host,
                                     np.array([total - 1]), np.ones(1),
                                     wl.round_queries(batch.queries, wl.KV_BF16), 32)
    got = merged.view(1, 32, 128).cpu().numpy().astype(np.float64)
    err = np.abs(got - ref)
    bad = err > 1e-6 + 1e-5 * np.abs(ref)
    assert not bad.any(), f"split: {bad.sum()}/{bad.size} outside, max abs {err.max():.3e}"
    # the single-launch decode of the whole sequence agrees as well
    err = np.abs(whole.cpu().numpy().astype(np.float64) - ref)
    assert np.all(err <= 1e-6 + 1e-5 * np.abs(ref)), float(err.max())
    pool.close()

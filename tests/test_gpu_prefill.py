"""GPU parity of the tcgen05 tensor-core prefill against the oracle.

The oracle is the fp32 CPU attention fed the same 16-bit inputs widened to
fp32 (the reference kernel in Fp32 mode on f16/bf16-rounded data). The kernel
multiplies fp16 probabilities, so the tolerance is the f16/bf16 one:
|gpu - oracle| <= 2e-3 * |oracle| + 1e-3 * max|oracle row|, where a row is one
(query, head) output vector. The row term is the fp16 probability rounding:
each p_j carries up to 2^-11 relative error, so with the normaliser summed
from the same rounded p_j the output moves by at most 2^-11 * max_j |v_j - o|,
a bound on the scale of the values, which shows on rows with few keys whose
outputs cancel. A masking or tiling bug moves outputs by O(|v|), ~500x more.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 2e-3
ROW_ATOL = 1e-3


def check_f16(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    row_scale = np.max(np.abs(ref), axis=-1, keepdims=True)
    err = np.abs(got - ref)
    bad = err > RTOL * np.abs(ref) + ROW_ATOL * row_scale
    rel = err / np.maximum(np.abs(ref), 1e-30)
    row_ratio = float(np.max(err / np.maximum(row_scale, 1e-30)))
    print(f"f16 parity: max abs {err.max():.3e}, max err/rowmax {row_ratio:.3e}, "
          f"max rel (|ref|>1e-2) {rel[np.abs(ref) > 1e-2].max():.3e}")
    assert not bad.any(), (f"{bad.sum()}/{bad.size} outside tolerance; max abs {err.max():.3e}, "
                           f"max err/rowmax {row_ratio:.3e}, "
                           f"max rel (|ref|>1e-2) {rel[np.abs(ref) > 1e-2].max():.3e}")
    return float(err.max())


@pytest.fixture(scope="module")
def wl():
    import torch

    assert torch.cuda.is_available(), "these tests need a CUDA device"
    from inferlab_b200 import workloads

    return workloads


def oracle_prefill(oracle_mod, wl, batch):
    k_arena, v_arena = wl.host_arenas(batch.pool)
    q = batch.prefill_queries.float().cpu().numpy()
    return oracle_mod.paged_attention(k_arena, v_arena, batch.pool.dtype,
                                      batch.prefill_tables_host, batch.starts, batch.counts, q,
                                      batch.q_heads)


def test_tc_prefill_single_tile(wl, oracle_mod):
    """One 128-query tile of one head: the smallest tensor-core case."""
    batch = wl.prefill_batch(0, 51, [0], [128], 1, 1, 128, 1, 0.5)
    out = batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                             batch.counts_dev, batch.offsets_dev, 128)
    batch.pool.synchronize()
    check_f16(out.cpu().numpy(), oracle_prefill(oracle_mod, wl, batch))
    batch.pool.close()


@pytest.mark.parametrize("dtype", [1, 2])
def test_tc_prefill_ragged_chunks(wl, oracle_mod, dtype):
    """Full prompts and chunks with prior context, lengths off the 16/128 grid."""
    q_heads, kv_heads = (16, 16) if dtype == 1 else (32, 8)
    batch = wl.prefill_batch(0, 60 + dtype, [0, 0, 300, 37, 1000], [256, 100, 512, 129, 1],
                             q_heads, kv_heads, 128, dtype, 0.5)
    out = batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                             batch.counts_dev, batch.offsets_dev, 512)
    batch.pool.synchronize()
    check_f16(out.cpu().numpy(), oracle_prefill(oracle_mod, wl, batch))
    batch.pool.close()


def test_tc_prefill_fp32_queries_are_rounded(wl, oracle_mod):
    """fp32 queries are rounded to the pool type first; same result as passing f16."""
    import torch

    batch = wl.prefill_batch(0, 71, [0, 64], [200, 64], 8, 8, 128, 1, 0.5)
    q32 = batch.prefill_queries.float().contiguous()
    a = batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                           batch.counts_dev, batch.offsets_dev, 200)
    b = batch.pool.prefill(q32, batch.prefill_tables, batch.starts_dev, batch.counts_dev,
                           batch.offsets_dev, 200)
    batch.pool.synchronize()
    assert torch.equal(a, b)
    check_f16(a.cpu().numpy(), oracle_prefill(oracle_mod, wl, batch))
    batch.pool.close()


def test_tc_prefill_full_workload(wl, oracle_mod):
    """8 x 1024-token causal prefill, 16 heads x 128, f16, N(0, 0.5^2)."""
    batch = wl.prefill_f16(device=0, seed=2028)
    out = batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                             batch.counts_dev, batch.offsets_dev, 1024)
    batch.pool.synchronize()
    check_f16(out.cpu().numpy(), oracle_prefill(oracle_mod, wl, batch))
    batch.pool.close()


def test_tc_prefill_last_row_equals_decode(wl):
    """Size-independent cross-check at a long context: the last query of a
    chunk equals the decode kernel's output for the same position."""
    import torch

    batch = wl.prefill_batch(0, 81, [8000], [192], 32, 8, 128, 2, 1.0)
    out = batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                             batch.counts_dev, batch.offsets_dev, 192)
    q_last = batch.prefill_queries[-1:].float().contiguous()
    lens = torch.tensor([8192], dtype=torch.int32, device="cuda:0")
    dec = batch.pool.decode(q_last, batch.prefill_tables, lens, 8192)
    batch.pool.synchronize()
    check_f16(out[-1:].cpu().numpy(), dec.cpu().numpy())
    batch.pool.close()


def test_tc_prefill_reports_bad_segment(wl):
    import torch

    from inferlab_b200 import AttentionError

    batch = wl.prefill_batch(0, 91, [0], [64], 8, 8, 128, 1, 0.5)
    bad_starts = torch.tensor([batch.prefill_tables.shape[1] * 16], dtype=torch.int32,
                              device="cuda:0")
    batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, bad_starts, batch.counts_dev,
                       batch.offsets_dev, 64)
    with pytest.raises(AttentionError, match="^paged prefill segment is invalid$"):
        batch.pool.synchronize()
    batch.pool.close()

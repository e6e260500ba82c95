"""GPU parity of the paged KV pool kernels against the oracle.

- append / gather: bit-exact against the oracle's restatement of
  PagedKvPool::append / materialize (worker/cpp/inferlab_runtime.cpp:713-803);
- paged decode (fp32 and 16-bit pools, MHA and GQA, split and unsplit):
  |gpu - oracle| <= 1e-6 + 1e-5 * |oracle| (both compute in fp32 on the same
  stored values; the decode call shape of worker/cpp/inferlab_runtime.cpp:1458-1470);
- split partials merged by inferlab_cuda_lse_combine equal the whole-context result;
- device-detected errors surface through inferlab_cuda_pool_synchronize.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-6, 1e-5


def close(got, ref, atol=ATOL, rtol=RTOL):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), f"{bad.sum()}/{bad.size} outside tolerance, max abs err {err.max():.3e}"


@pytest.fixture(scope="module")
def torch_mod():
    import torch

    assert torch.cuda.is_available(), "these tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def wl(torch_mod):
    from inferlab_b200 import workloads

    return workloads


def oracle_decode(oracle_mod, wl, batch):
    k_host, v_host = wl.host_arenas(batch.pool)
    q = wl.round_queries(batch.queries, batch.pool.dtype)
    return oracle_mod.paged_attention(k_host, v_host, batch.pool.dtype, batch.tables_host,
                                      batch.contexts - 1, np.ones(len(batch.contexts)), q,
                                      batch.q_heads)


def test_decode_fp32_full_workload(torch_mod, wl, oracle_mod):
    """64 sequences x U[64, 2048], 8 heads x 64, fp32, 8192-block pool."""
    batch = wl.decode_fp32(device=0, seed=11)
    out = batch.pool.decode(batch.queries, batch.block_tables, batch.context_lens,
                            batch.max_context_len)
    batch.pool.synchronize()
    close(out.cpu().numpy(), oracle_decode(oracle_mod, wl, batch))
    # the split-free path (one split per sequence) agrees too
    batch.pool.set_decode_split(256)
    try:
        out2 = batch.pool.decode(batch.queries, batch.block_tables, batch.context_lens,
                                 batch.max_context_len, workspace=batch.pool.make_workspace(
                                     64, 8, 2048))
    finally:
        batch.pool.set_decode_split(0)
    batch.pool.synchronize()
    close(out2.cpu().numpy(), out.cpu().numpy())
    batch.pool.close()


@pytest.mark.parametrize("dtype", [1, 2])
@pytest.mark.parametrize("q_heads,kv_heads,head_dim", [(32, 8, 128), (8, 8, 128), (16, 2, 64),
                                                       (4, 2, 64), (8, 1, 128)])
def test_decode_16bit_gqa(torch_mod, wl, oracle_mod, dtype, q_heads, kv_heads, head_dim):
    rng = np.random.Generator(np.random.PCG64(q_heads * 100 + kv_heads + dtype))
    contexts = np.concatenate([[1, 15, 16, 17, 4096], rng.integers(1, 3000, size=11)])
    batch = wl.decode_batch(0, 7 + dtype, len(contexts), contexts, q_heads, kv_heads, head_dim,
                            dtype, max_context_len=4096)
    out = batch.pool.decode(batch.queries, batch.block_tables, batch.context_lens,
                            batch.max_context_len)
    batch.pool.synchronize()
    close(out.cpu().numpy(), oracle_decode(oracle_mod, wl, batch))
    batch.pool.close()


def test_decode_long_context_sample(torch_mod, wl, oracle_mod):
    """Sequences from the long-context workload (bf16, GQA 32/8 x 128,
    context U[4096, 32768]); a 24-sequence sample keeps the oracle quick."""
    contexts = wl.longctx_contexts(2027)[:24]
    contexts[0] = 32768
    batch = wl.decode_batch(0, 5, len(contexts), contexts, 32, 8, 128, wl.KV_BF16,
                            max_context_len=32768)
    out = batch.pool.decode(batch.queries, batch.block_tables, batch.context_lens, 32768)
    batch.pool.synchronize()
    close(out.cpu().numpy(), oracle_decode(oracle_mod, wl, batch))
    batch.pool.close()


def test_partials_and_combine_equal_whole_context(torch_mod, wl, oracle_mod):
    """One 2048-token sequence split into 4 contiguous block ranges (as the
    cross-GPU split does), each decoded into partials, then merged in order."""
    torch = torch_mod
    from inferlab_b200 import lse_combine

    contexts = np.array([2048, 1000])
    batch = wl.decode_batch(0, 21, 2, contexts, 32, 8, 128, wl.KV_BF16, max_context_len=2048)
    whole = batch.pool.decode(batch.queries, batch.block_tables, batch.context_lens, 2048)
    parts_m, parts_l, parts_o = [], [], []
    for part in range(4):
        lo, hi = part * 32, (part + 1) * 32  # 32 blocks = 512 tokens per part
        tables = torch.zeros((2, 32), dtype=torch.int32, device="cuda:0")
        tables[0] = batch.block_tables[0, lo:hi]
        lens = torch.tensor([512, 1], dtype=torch.int32, device="cuda:0")
        tables[1, :1] = batch.block_tables[1, 0]
        m, l, o = batch.pool.decode_partials(batch.queries, tables, lens, 512)
        if part > 0:  # the second sequence only has one token, in part 0
            m[1] = -float("inf")
            l[1] = 0
            o[1] = 0
        parts_m.append(m)
        parts_l.append(l)
        parts_o.append(o)
    merged = lse_combine(torch.stack(parts_m), torch.stack(parts_l), torch.stack(parts_o))
    # the packed layout (one [m | l | o] block per part, as an all-gather
    # delivers it) merges to the same bits
    from inferlab_b200.paged import lse_combine_packed

    packed = torch.cat([torch.cat([pm.reshape(-1), pl.reshape(-1), po.reshape(-1)])
                        for pm, pl, po in zip(parts_m, parts_l, parts_o)])
    rows = parts_m[0].numel()
    merged_packed = lse_combine_packed(packed, len(parts_m), rows, parts_o[0].shape[-1])
    assert torch.equal(merged_packed.view_as(merged), merged)
    batch.pool.synchronize()
    close(merged[0].cpu().numpy(), whole[0].cpu().numpy(), atol=2e-6, rtol=2e-5)
    # the oracle's merge of the same partials agrees with the device merge
    ref = oracle_mod.lse_merge(torch.stack(parts_m).cpu().numpy().reshape(4, -1),
                               torch.stack(parts_l).cpu().numpy().reshape(4, -1),
                               torch.stack(parts_o).cpu().numpy().reshape(4, -1, 128))
    close(merged.cpu().numpy().reshape(-1, 128)[:32], ref[:32], atol=2e-6, rtol=2e-5)
    batch.pool.close()


def test_decode_step_host_matches_device_calls(torch_mod, wl, oracle_mod):
    """inferlab_cuda_decode_step_host (host buffers, append + decode in one
    call) equals kv_append followed by paged decode, and the oracle."""
    torch = torch_mod
    contexts = np.array([1, 16, 17, 700, 2048, 33])
    batch = wl.decode_batch(0, 17, len(contexts), contexts, 32, 8, 128, wl.KV_BF16,
                            max_context_len=2048)
    rng = np.random.Generator(np.random.PCG64(18))
    q = rng.standard_normal((len(contexts), 32, 128), dtype=np.float32)
    k_new = rng.standard_normal((len(contexts), 8, 128), dtype=np.float32)
    v_new = rng.standard_normal((len(contexts), 8, 128), dtype=np.float32)
    for repeat in range(2):  # the second call reuses the pool's staging
        got = batch.pool.decode_step_host(q, batch.tables_host, contexts, k_new, v_new)
    dev = "cuda:0"
    ref = batch.pool.decode(torch.from_numpy(q).to(dev), batch.block_tables, batch.context_lens,
                            2048)
    batch.pool.synchronize()
    close(got, ref.cpu().numpy())
    k_host, v_host = wl.host_arenas(batch.pool)
    ref_o = oracle_mod.paged_attention(k_host, v_host, wl.KV_BF16, batch.tables_host,
                                       contexts - 1, np.ones(len(contexts)),
                                       wl.round_queries(torch.from_numpy(q), wl.KV_BF16), 32)
    close(got, ref_o)
    # the appended rows are in the pool at position ctx - 1
    kg, _ = batch.pool.gather(batch.block_tables[4, :128].contiguous(), 2048)
    assert torch.equal(kg[2047].cpu(), torch.from_numpy(k_new[4]).to(torch.bfloat16))
    # invalid block ids and context lengths fail the call with the reference's messages
    from inferlab_b200 import AttentionError

    bad = batch.tables_host.copy()
    bad[2, 1] = -3
    with pytest.raises(AttentionError, match="^paged KV block table contains an invalid page$"):
        batch.pool.decode_step_host(q, bad, contexts)
    with pytest.raises(AttentionError, match="^paged KV context length is invalid$"):
        batch.pool.decode_step_host(q, batch.tables_host, contexts * 0)
    batch.pool.close()


@pytest.mark.parametrize("kv_dtype,q_heads,kv_heads,head_dim", [(0, 16, 4, 64), (2, 32, 8, 128)])
def test_decode_step_host_pinned_buffers_match_staged(torch_mod, wl, kv_dtype, q_heads, kv_heads,
                                                      head_dim):
    """Page-locked caller buffers take the mapped path (a prologue kernel reads
    them over the bus, the decode writes the caller's output directly); the
    result equals the staged path on pageable copies of the same arrays, bit
    for bit, and so does the appended row."""
    torch = torch_mod
    contexts = np.array([5, 300, 1024, 77])
    rng = np.random.Generator(np.random.PCG64(28))
    q = rng.standard_normal((len(contexts), q_heads, head_dim), dtype=np.float32)
    k_new = rng.standard_normal((len(contexts), kv_heads, head_dim), dtype=np.float32)
    v_new = rng.standard_normal((len(contexts), kv_heads, head_dim), dtype=np.float32)

    def pinned(a):
        t = torch.empty(a.shape, dtype=getattr(torch, str(a.dtype)), pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()

    results, rows = [], []
    for use_pinned in (False, True):
        batch = wl.decode_batch(0, 27, len(contexts), contexts, q_heads, kv_heads, head_dim,
                                kv_dtype, max_context_len=1024)
        tables = np.ascontiguousarray(batch.tables_host, dtype=np.int32)
        lens = contexts.astype(np.int32)
        args = (q, tables, lens, k_new, v_new)
        if use_pinned:
            args = tuple(pinned(a) for a in args)
            out = pinned(np.zeros_like(q))
        else:
            out = np.zeros_like(q)
        got = batch.pool.decode_step_host(args[0], args[1], args[2], args[3], args[4], out=out)
        assert got is out
        results.append(np.array(got))
        kg, vg = batch.pool.gather(batch.block_tables[2, :64].contiguous(), 1024)
        rows.append((kg[1023].cpu(), vg[1023].cpu()))
        if use_pinned:
            # a non-finite new row is rejected and leaves the pool untouched
            bad_k = pinned(k_new)
            bad_k[1, 0, 3] = np.inf
            from inferlab_b200 import AttentionError

            with pytest.raises(AttentionError, match="^attention input must be finite$"):
                batch.pool.decode_step_host(args[0], args[1], args[2], bad_k, args[4], out=out)
            kg2, _ = batch.pool.gather(batch.block_tables[1, :19].contiguous(), 300)
            assert torch.equal(kg2[299].cpu(), kg2[299].cpu().nan_to_num())
        batch.pool.close()
    assert np.array_equal(results[0], results[1])
    assert torch.equal(rows[0][0], rows[1][0]) and torch.equal(rows[0][1], rows[1][1])


def test_append_then_gather_bit_exact(torch_mod, wl, oracle_mod):
    torch = torch_mod
    from inferlab_b200 import CudaKvPool

    for dtype in (0, 1, 2):
        pool = CudaKvPool(0, dtype, 64, 16, 4, 64)
        rng = np.random.Generator(np.random.PCG64(dtype))
        contexts = [37, 16, 1]
        tables = np.full((3, 4), -1, np.int32)
        perm = rng.permutation(64).astype(np.int32)
        used = 0
        for s, c in enumerate(contexts):
            n = (c + 15) // 16
            tables[s, :n] = perm[used:used + n]
            used += n
        rows = [(s, p) for s, c in enumerate(contexts) for p in range(c)]
        rng.shuffle(rows)
        seqs = np.array([r[0] for r in rows], np.int32)
        pos = np.array([r[1] for r in rows], np.int32)
        k_rows = rng.standard_normal((len(rows), 4, 64), dtype=np.float32) * 3
        v_rows = rng.standard_normal((len(rows), 4, 64), dtype=np.float32)
        dev = "cuda:0"
        pool.append(torch.from_numpy(k_rows).to(dev), torch.from_numpy(v_rows).to(dev),
                    torch.from_numpy(seqs).to(dev), torch.from_numpy(pos).to(dev),
                    torch.from_numpy(tables).to(dev))
        pool.synchronize()
        k_arena, v_arena = wl.host_arenas(pool)
        for s, c in enumerate(contexts):
            n = (c + 15) // 16
            kg, vg = pool.gather(torch.from_numpy(tables[s, :n].copy()).to(dev), c)
            pool.synchronize()
            k_ref = oracle_mod.materialize(k_arena, dtype, tables[s, :n], c)
            v_ref = oracle_mod.materialize(v_arena, dtype, tables[s, :n], c)
            kg = kg.float().cpu().numpy()
            vg = vg.float().cpu().numpy()
            assert np.array_equal(kg, k_ref) and np.array_equal(vg, v_ref)
            # the stored values are the rows rounded like round_attention_value
            mine = [i for i, r in enumerate(rows) if r[0] == s]
            order = np.argsort(pos[mine])
            expect_k = oracle_mod.round_values_ieee(k_rows[mine][order], dtype)
            assert np.array_equal(kg, expect_k)
        pool.close()


def test_generic_geometry_decode_and_prefill(torch_mod, wl, oracle_mod):
    """Block size 4 and head_dim 8 (the reference worker's default page size)
    take the generic CUDA-core kernel; same tolerance."""
    torch = torch_mod
    from inferlab_b200 import CudaKvPool

    rng = np.random.Generator(np.random.PCG64(31))
    pool = CudaKvPool(0, 0, 40, 4, 2, 8)
    k_rows = rng.standard_normal((160, 2, 8), dtype=np.float32)
    v_rows = rng.standard_normal((160, 2, 8), dtype=np.float32)
    table = rng.permutation(40).astype(np.int32).reshape(1, 40)
    dev = "cuda:0"
    pool.append(torch.from_numpy(k_rows).to(dev), torch.from_numpy(v_rows).to(dev),
                torch.zeros(160, dtype=torch.int32, device=dev),
                torch.arange(160, dtype=torch.int32, device=dev), torch.from_numpy(table).to(dev))
    q = rng.standard_normal((1, 4, 8), dtype=np.float32)
    out = pool.decode(torch.from_numpy(q).to(dev), torch.from_numpy(table).to(dev),
                      torch.tensor([150], dtype=torch.int32, device=dev), 160)
    k_arena, v_arena = wl.host_arenas(pool)
    ref = oracle_mod.paged_attention(k_arena, v_arena, 0, table, [149], [1], q, 4)
    pool.synchronize()
    close(out.cpu().numpy(), ref)
    # chunked prefill: 10 queries at positions 140..149
    qp = rng.standard_normal((10, 4, 8), dtype=np.float32)
    outp = pool.prefill(torch.from_numpy(qp).to(dev), torch.from_numpy(table).to(dev),
                        torch.tensor([140], dtype=torch.int32, device=dev),
                        torch.tensor([10], dtype=torch.int32, device=dev),
                        torch.tensor([0], dtype=torch.int32, device=dev), 10)
    refp = oracle_mod.paged_attention(k_arena, v_arena, 0, table, [140], [10], qp, 4)
    pool.synchronize()
    close(outp.cpu().numpy(), refp)
    pool.close()


def test_prefill_fp32_matches_oracle(torch_mod, wl, oracle_mod):
    """fp32 pools run the CUDA-core prefill: two segments (a full prompt and a
    chunk with prior context), GQA 8/2 x 64."""
    batch = wl.prefill_batch(0, 41, [0, 300], [200, 77], 8, 2, 64, wl.KV_FP32, 1.0)
    out = batch.pool.prefill(batch.prefill_queries, batch.prefill_tables, batch.starts_dev,
                             batch.counts_dev, batch.offsets_dev, 200)
    k_arena, v_arena = wl.host_arenas(batch.pool)
    ref = oracle_mod.paged_attention(k_arena, v_arena, 0, batch.prefill_tables_host, batch.starts,
                                     batch.counts, batch.prefill_queries.cpu().numpy(), 8)
    batch.pool.synchronize()
    close(out.cpu().numpy(), ref)
    batch.pool.close()


def test_invalid_block_id_is_reported(torch_mod, wl):
    torch = torch_mod
    from inferlab_b200 import AttentionError

    batch = wl.decode_batch(0, 3, 2, np.array([40, 40]), 8, 8, 64, wl.KV_FP32,
                            max_context_len=64)
    tables = batch.block_tables.clone()
    tables[1, 1] = batch.pool.num_blocks + 5
    batch.pool.decode(batch.queries, tables, batch.context_lens, 64)
    with pytest.raises(AttentionError, match="^paged KV block table contains an invalid page$"):
        batch.pool.synchronize()
    # the error word is cleared and the pool keeps working
    batch.pool.decode(batch.queries, batch.block_tables, batch.context_lens, 64)
    batch.pool.synchronize()
    bad_lens = torch.tensor([40, 65], dtype=torch.int32, device="cuda:0")
    batch.pool.decode(batch.queries, batch.block_tables, bad_lens, 64)
    with pytest.raises(AttentionError, match="^paged KV context length is invalid$"):
        batch.pool.synchronize()
    batch.pool.close()


def test_non_finite_rows_are_rejected_on_append(torch_mod):
    torch = torch_mod
    from inferlab_b200 import AttentionError, CudaKvPool

    pool = CudaKvPool(0, 2, 4, 16, 1, 64)
    dev = "cuda:0"
    rows = torch.ones((2, 1, 64), device=dev)
    rows[1, 0, 3] = float("inf")
    table = torch.tensor([[0]], dtype=torch.int32, device=dev)
    pool.append(rows, torch.ones_like(rows), torch.zeros(2, dtype=torch.int32, device=dev),
                torch.tensor([0, 1], dtype=torch.int32, device=dev), table)
    with pytest.raises(AttentionError, match="^attention input must be finite$"):
        pool.synchronize()
    assert torch.all(pool.key_arena[0, 0, 1] == 0)  # the bad row was not written
    assert torch.all(pool.key_arena[0, 0, 0] == 1)
    pool.close()

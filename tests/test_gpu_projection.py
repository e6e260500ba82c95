"""inferlab_cuda_qkv_project_append against the projection oracle
(oracle/projection.py: the reference's fp32 linear, pinned bit for bit, and
PagedKvPool::append's placement). The GPU multiplies the pool-type (f16 /
bf16) operands with fp32 accumulation and rounds to the pool type, so every
element must satisfy |gpu - ref| <= 2^-7 |ref| + 2^-8 rms(ref) (a little over
one rounding step of bf16) against the fp32 oracle fed the same rounded
operands; tokens' K/V rows must sit exactly where the block tables say."""
import numpy as np
import pytest

from oracle import projection

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod():
    import torch

    assert torch.cuda.is_available(), "these tests need a CUDA device"
    return torch


def _case(torch, dtype, tokens, model_dim, q_heads, kv_heads, head_dim, seed):
    from inferlab_b200 import CudaKvPool
    from inferlab_b200 import workloads as wl

    tdt = wl.TORCH_DTYPES[dtype]
    dev = "cuda:0"
    pool = CudaKvPool(0, dtype, 256, 16, kv_heads, head_dim)
    rng = np.random.Generator(np.random.PCG64(seed))
    gen = torch.Generator(device=dev).manual_seed(seed)
    hidden = torch.randn((tokens, model_dim), generator=gen, device=dev).to(tdt)
    n = (q_heads + 2 * kv_heads) * head_dim
    weights = (torch.randn((n, model_dim), generator=gen, device=dev) / model_dim ** 0.5).to(tdt)
    # three sequences, each a run of consecutive positions (a prefill chunk)
    starts = [0, 40, 7]
    counts = [tokens // 3, tokens // 3, tokens - 2 * (tokens // 3)]
    seq = np.concatenate([np.full(c, s, np.int32) for s, c in enumerate(counts)])
    pos = np.concatenate([np.arange(st, st + c, dtype=np.int32) for st, c in zip(starts, counts)])
    max_blocks = int((pos.max() + 16) // 16)
    tables = rng.permutation(256)[:3 * max_blocks].astype(np.int32).reshape(3, max_blocks)
    q = pool.project_append(hidden, weights, q_heads,
                            torch.from_numpy(seq).to(dev), torch.from_numpy(pos).to(dev),
                            torch.from_numpy(tables).to(dev))
    pool.synchronize()
    x32 = hidden.float().cpu().numpy()
    w32 = weights.float().cpu().numpy()
    rq, rk, rv, blocks, slots = projection.project_append(
        x32, w32, q_heads, kv_heads, head_dim, seq, pos, tables, 16)

    def close(got, ref):
        tol = 2.0 ** -7 * np.abs(ref) + 2.0 ** -8 * float(np.sqrt(np.mean(ref ** 2)))
        assert np.all(np.abs(got - ref) <= tol), float(np.max(np.abs(got - ref) - tol))

    close(q.float().cpu().numpy(), rq)
    karena = pool.key_arena.float().cpu().numpy()    # [blocks][kv_heads][16][d]
    varena = pool.value_arena.float().cpu().numpy()
    close(karena[blocks, :, slots, :], rk)
    close(varena[blocks, :, slots, :], rv)
    # nothing else of the pool was written
    mask = np.zeros(karena.shape[0] * 16, bool)
    mask[blocks * 16 + slots] = True
    rest = karena.transpose(0, 2, 1, 3).reshape(-1, kv_heads * head_dim)[~mask]
    assert not np.any(rest)
    pool.close()


@pytest.mark.parametrize("dtype", [1, 2])
def test_projection_gqa_ragged_tokens(torch_mod, dtype):
    # 300 tokens (last 128-token tile ragged), 8 q / 2 kv heads x 128: N = 1536
    _case(torch_mod, dtype, 300, 256, 8, 2, 128, 5)


def test_projection_small_heads_partial_feature_tile(torch_mod):
    # the single-sequence configuration's shape: 4 heads x 32 (N = 384, a
    # partial 256-feature tile), model_dim 200 (a partial 64-wide K stage)
    _case(torch_mod, 2, 129, 200, 4, 4, 32, 6)


def test_projection_rejects_bad_block(torch_mod):
    import torch

    from inferlab_b200 import AttentionError, CudaKvPool

    dev = "cuda:0"
    pool = CudaKvPool(0, 2, 8, 16, 1, 32)
    hidden = torch.ones((4, 64), dtype=torch.bfloat16, device=dev)
    weights = torch.ones((3 * 32, 64), dtype=torch.bfloat16, device=dev)
    tables = torch.tensor([[99]], dtype=torch.int32, device=dev)
    pool.project_append(hidden, weights, 1, torch.zeros(4, dtype=torch.int32, device=dev),
                        torch.arange(4, dtype=torch.int32, device=dev), tables)
    with pytest.raises(AttentionError, match="^paged KV block table contains an invalid page$"):
        pool.synchronize()
    with pytest.raises(AttentionError, match="^projection needs an F16 or BF16 pool$"):
        CudaKvPool(0, 0, 8, 16, 1, 32).project_append(
            hidden.float(), weights.float(), 1, torch.zeros(4, dtype=torch.int32, device=dev),
            torch.arange(4, dtype=torch.int32, device=dev), tables)
    pool.close()


@pytest.mark.parametrize("dtype,fp32_input", [(2, True), (1, False)])
def test_output_projection_with_residual(torch_mod, dtype, fp32_input):
    """out = residual + attention x W_o^T (inferlab_cuda_output_project) against
    the oracle's fp32 linear fed the same pool-type operands. Products of two
    16-bit values are exact in fp32, so only the summation order differs:
    |gpu - ref| <= 1e-4 |ref| + 1e-4 rms(ref)."""
    torch = torch_mod
    from inferlab_b200 import CudaKvPool
    from inferlab_b200 import workloads as wl

    dev = "cuda:0"
    tdt = wl.TORCH_DTYPES[dtype]
    pool = CudaKvPool(0, dtype, 4, 16, 1, 32)
    gen = torch.Generator(device=dev).manual_seed(11 + dtype)
    tokens, in_dim, out_dim = 200, 512, 352  # ragged token tile, partial feature tile
    attn = torch.randn((tokens, in_dim), generator=gen, device=dev)
    if not fp32_input:
        attn = attn.to(tdt)
    weights = (torch.randn((out_dim, in_dim), generator=gen, device=dev) / in_dim ** 0.5).to(tdt)
    residual = torch.randn((tokens, out_dim), generator=gen, device=dev)
    out = pool.output_project(attn, weights, residual)
    pool.synchronize()
    a32 = attn.to(tdt).float().cpu().numpy()
    ref = projection.output_project(a32, weights.float().cpu().numpy(), residual.cpu().numpy())
    got = out.cpu().numpy()
    tol = 1e-4 * np.abs(ref) + 1e-4 * float(np.sqrt(np.mean(ref ** 2)))
    assert np.all(np.abs(got - ref) <= tol), float(np.max(np.abs(got - ref) - tol))
    # without a residual
    out2 = pool.output_project(attn, weights)
    pool.synchronize()
    ref2 = projection.output_project(a32, weights.float().cpu().numpy())
    tol2 = 1e-4 * np.abs(ref2) + 1e-4 * float(np.sqrt(np.mean(ref2 ** 2)))
    assert np.all(np.abs(out2.cpu().numpy() - ref2) <= tol2)
    pool.close()


def test_attention_layer_chain(torch_mod, oracle_mod):
    """One prefill chunk through the three device stages a layer needs:
    inferlab_cuda_qkv_project_append -> inferlab_cuda_paged_prefill ->
    inferlab_cuda_output_project, each stage checked against its oracle fed
    the previous stage's device results (projection tolerances as above; the
    attention stage with the f16/bf16 prefill tolerance 2e-3 |ref| + 1e-3 row
    max). Two 100-token sequences from position 0, model_dim 256, 4 q / 2 kv
    heads x 128, bf16."""
    torch = torch_mod
    from inferlab_b200 import CudaKvPool
    from inferlab_b200 import workloads as wl

    from tests.test_gpu_prefill import check_f16

    dev = "cuda:0"
    pool = CudaKvPool(0, 2, 64, 16, 2, 128)
    gen = torch.Generator(device=dev).manual_seed(21)
    tokens, model_dim = 200, 256
    hidden = torch.randn((tokens, model_dim), generator=gen, device=dev)
    h16 = hidden.to(torch.bfloat16)
    w_qkv = (torch.randn(((4 + 4) * 128, model_dim), generator=gen, device=dev) /
             model_dim ** 0.5).to(torch.bfloat16)
    w_o = (torch.randn((model_dim, 4 * 128), generator=gen, device=dev) / 512 ** 0.5).to(torch.bfloat16)
    tables = np.arange(16, dtype=np.int32).reshape(2, 8)
    seq = np.repeat(np.arange(2, dtype=np.int32), 100)
    pos = np.tile(np.arange(100, dtype=np.int32), 2)
    d_tables = torch.from_numpy(tables).to(dev)

    q = pool.project_append(h16, w_qkv, 4, torch.from_numpy(seq).to(dev),
                            torch.from_numpy(pos).to(dev), d_tables)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=dev)  # noqa: E731
    attn = pool.prefill(q, d_tables, i32([0, 0]), i32([100, 100]), i32([0, 100]), 100)
    out = pool.output_project(attn.view(tokens, -1), w_o, residual=hidden)
    pool.synchronize()

    # stage 1: projection
    rq, _, _, _, _ = projection.project_append(h16.float().cpu().numpy(), w_qkv.float().cpu().numpy(),
                                               4, 2, 128, seq, pos, tables, 16)
    tol = 2.0 ** -7 * np.abs(rq) + 2.0 ** -8 * float(np.sqrt(np.mean(rq ** 2)))
    assert np.all(np.abs(q.float().cpu().numpy() - rq) <= tol)
    # stage 2: attention over the pool the projection filled
    k_host, v_host = wl.host_arenas(pool)
    ref_attn = oracle_mod.paged_attention(k_host, v_host, 2, tables, np.array([0, 0]),
                                          np.array([100, 100]), q.float().cpu().numpy(), 4)
    check_f16(attn.cpu().numpy(), ref_attn)
    # stage 3: output projection + residual of the device attention output
    a16 = attn.view(tokens, -1).to(torch.bfloat16).float().cpu().numpy()
    ref_out = projection.output_project(a16, w_o.float().cpu().numpy(), hidden.cpu().numpy())
    tol3 = 1e-4 * np.abs(ref_out) + 1e-4 * float(np.sqrt(np.mean(ref_out ** 2)))
    assert np.all(np.abs(out.cpu().numpy() - ref_out) <= tol3)
    pool.close()

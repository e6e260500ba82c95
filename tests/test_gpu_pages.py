"""Copy on write through the device pool: a sequence that starts from a shared
prefix gets its tail block copied on the device (inferlab_cuda_pages_copy)
before the next row is written; the copied rows are bit-exact, the shared
block is untouched, and both sequences decode to the oracle's answer within
the fp32 tolerance |gpu - ref| <= 1e-6 + 1e-5 |ref|."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_copy_on_write_on_the_device(oracle_mod):
    import torch

    from inferlab_b200 import CudaKvPool, PageManager
    from inferlab_b200 import workloads as wl
    from inferlab_b200.pages import copy_blocks

    dev = "cuda:0"
    pool = CudaKvPool(0, wl.KV_FP32, 16, 16, 2, 64)
    m = PageManager.for_pool(pool, prefix_capacity=4)
    rng = np.random.Generator(np.random.PCG64(41))

    def append(table, n, copy=None):
        """Reserve slot n, run any block copy, write one random row there."""
        if copy is not None:
            copy_blocks(pool, [copy])
        k = torch.from_numpy(rng.standard_normal((1, 2, 64), dtype=np.float32)).to(dev)
        v = torch.from_numpy(rng.standard_normal((1, 2, 64), dtype=np.float32)).to(dev)
        tab = torch.zeros((1, 8), dtype=torch.int32, device=dev)
        tab[0, :len(table)] = torch.tensor(table, dtype=torch.int32)
        pool.append(k, v, torch.zeros(1, dtype=torch.int32, device=dev),
                    torch.tensor([n], dtype=torch.int32, device=dev), tab)

    # sequence A: 21 tokens (one full block + 5 rows), published as a prefix
    a, n = [], 0
    for _ in range(21):
        a, copy = m.prepare_append(a, n)
        assert copy is None
        append(a, n)
        n += 1
    tokens = list(range(21))
    m.publish_prefix(tokens, a, 21)

    # sequence B starts from the prefix and appends: its shared tail is copied
    b, reused = m.acquire_prefix(tokens + [99])
    assert reused == 21 and b == a
    b, copy = m.prepare_append(b, 21)
    assert copy is not None and copy[0] == a[1] and b[0] == a[0] and b[1] == copy[1]
    append(b, 21, copy)
    pool.synchronize()

    ka, va = pool.gather(torch.tensor(a, dtype=torch.int32, device=dev), 21)
    kb, vb = pool.gather(torch.tensor(b, dtype=torch.int32, device=dev), 22)
    assert torch.equal(kb[:21], ka) and torch.equal(vb[:21], va)  # copied rows bit-exact
    s = m.stats()
    # a[0] is held by A, B and the prefix, a[1] by A and the prefix
    assert s["copy_on_write_copies"] == 1 and s["shared_pages"] == 2
    assert s["maximum_refcount"] == 3

    # both decode to the oracle's answer
    q = torch.from_numpy(rng.standard_normal((2, 2, 64), dtype=np.float32)).to(dev)
    tables = torch.zeros((2, 8), dtype=torch.int32, device=dev)
    tables[0, :2] = torch.tensor(a, dtype=torch.int32)
    tables[1, :2] = torch.tensor(b, dtype=torch.int32)
    lens = torch.tensor([21, 22], dtype=torch.int32, device=dev)
    got = pool.decode(q, tables, lens, 22).cpu().numpy()
    pool.synchronize()
    k_host, v_host = wl.host_arenas(pool)
    ref = oracle_mod.paged_attention(k_host, v_host, wl.KV_FP32, tables.cpu().numpy(),
                                     np.array([20, 21]), np.ones(2), q.cpu().numpy(), 2)
    assert np.all(np.abs(got - ref) <= 1e-6 + 1e-5 * np.abs(ref))
    m.release(a)
    m.release(b)
    m.close()
    pool.close()


@pytest.mark.parametrize("page_locked", [False, True])
def test_copy_on_write_fused_into_the_decode_step(oracle_mod, page_locked):
    """The copy-on-write pair prepare_append returns goes into the same host
    decode step call (inferlab_cuda_decode_step_host_cow): the shared tail
    block is copied, the new row lands in the copy, the shared block keeps its
    rows, and the step's output matches the oracle (fp32 tolerance)."""
    import torch

    from inferlab_b200 import CudaKvPool, PageManager
    from inferlab_b200 import workloads as wl

    dev = "cuda:0"
    pool = CudaKvPool(0, wl.KV_FP32, 16, 16, 2, 64)
    m = PageManager.for_pool(pool, prefix_capacity=4)
    rng = np.random.Generator(np.random.PCG64(43))

    def host(a):
        if not page_locked:
            return a
        t = torch.empty(a.shape, dtype=getattr(torch, str(a.dtype)), pin_memory=True)
        t.numpy()[...] = a
        return t.numpy()

    # sequence A: 21 tokens through device appends, published as a prefix
    a, n = [], 0
    for _ in range(21):
        a, copy = m.prepare_append(a, n)
        k = torch.from_numpy(rng.standard_normal((1, 2, 64), dtype=np.float32)).to(dev)
        v = torch.from_numpy(rng.standard_normal((1, 2, 64), dtype=np.float32)).to(dev)
        tab = torch.zeros((1, 8), dtype=torch.int32, device=dev)
        tab[0, :len(a)] = torch.tensor(a, dtype=torch.int32)
        pool.append(k, v, torch.zeros(1, dtype=torch.int32, device=dev),
                    torch.tensor([n], dtype=torch.int32, device=dev), tab)
        n += 1
    tokens = list(range(21))
    m.publish_prefix(tokens, a, 21)

    # sequence B takes the prefix; its first own token needs a copy of a[1]
    b, reused = m.acquire_prefix(tokens + [7])
    assert reused == 21
    b, copy = m.prepare_append(b, 21)
    assert copy is not None and copy[0] == a[1]
    tables = np.zeros((1, 8), np.int32)
    tables[0, :len(b)] = b
    q = rng.standard_normal((1, 2, 64), dtype=np.float32)
    k_new = rng.standard_normal((1, 2, 64), dtype=np.float32)
    v_new = rng.standard_normal((1, 2, 64), dtype=np.float32)
    copies = np.array([list(copy)], np.int32)
    out = host(np.zeros_like(q))
    got = pool.decode_step_host(host(q), host(tables), host(np.array([22], np.int32)), host(k_new),
                                host(v_new), out=out, block_copies=host(copies))
    pool.synchronize()

    ka, va = pool.gather(torch.tensor(a, dtype=torch.int32, device=dev), 21)
    kb, vb = pool.gather(torch.tensor(b, dtype=torch.int32, device=dev), 22)
    assert torch.equal(kb[:21], ka) and torch.equal(vb[:21], va)  # copied rows bit-exact
    assert torch.equal(kb[21].cpu(), torch.from_numpy(k_new[0]))
    assert torch.equal(vb[21].cpu(), torch.from_numpy(v_new[0]))
    # the shared block still ends after A's 21 rows: its slot 5 was not written
    ka2, _ = pool.gather(torch.tensor(a, dtype=torch.int32, device=dev), 22)
    assert torch.count_nonzero(ka2[21]).item() == 0

    k_host, v_host = wl.host_arenas(pool)
    ref = oracle_mod.paged_attention(k_host, v_host, wl.KV_FP32, tables, np.array([21]),
                                     np.ones(1), q, 2)
    assert np.all(np.abs(np.array(got) - ref) <= 1e-6 + 1e-5 * np.abs(ref))
    m.release(a)
    m.release(b)
    m.close()
    pool.close()

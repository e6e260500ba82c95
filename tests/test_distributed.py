"""CPU tests (gloo, world size 2) of the multi-GPU host logic.

Sequence sharding has no collective; the split-KV path for one long sequence
does: each rank computes (m, l, o) partials over its contiguous block range,
the partials are all-gathered in rank order, and the log-sum-exp merge of the
gathered parts must equal attention over the whole context. The partial math
here is the oracle's (float64 numpy); the CUDA kernels that produce and merge
partials on GPUs are checked in tests/test_gpu_paged.py.
"""
import math
import os
import socket

import numpy as np
import pytest


def test_shard_sequences_balances_and_is_deterministic():
    from inferlab_b200.distributed import shard_sequences

    rng = np.random.Generator(np.random.PCG64(0))
    contexts = rng.integers(4096, 32768, size=256, endpoint=True)
    for world in (1, 2, 4, 8):
        owner = shard_sequences(contexts, world)
        loads = np.bincount(owner, weights=contexts, minlength=world)
        assert owner.min() >= 0 and owner.max() < world
        assert loads.max() - loads.min() <= contexts.max()
        assert np.array_equal(owner, shard_sequences(contexts, world))


def test_split_range_covers_every_block_once():
    from inferlab_b200.distributed import local_tokens, split_range

    for total in (1, 7, 8, 1000, 8192):
        for world in (1, 2, 3, 8):
            covered = []
            for rank in range(world):
                lo, hi = split_range(total, world, rank)
                covered.extend(range(lo, hi))
            assert covered == list(range(total))
    assert sum(hi - lo for lo, hi in (local_tokens(131072, 16, 8, r) for r in range(8))) == 131072
    assert local_tokens(100, 16, 2, 1) == (64, 100)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partials(q, k, v, scale):
    s = (k.astype(np.float64) @ q.astype(np.float64)) * scale  # [tokens]
    if s.size == 0:
        return -np.inf, 0.0, np.zeros(q.shape[-1])
    m = s.max()
    p = np.exp(s - m)
    return m, p.sum(), p @ v.astype(np.float64)


def _worker(rank, world, port, tokens, result_path):
    import torch
    import torch.distributed as dist

    from inferlab_b200.distributed import all_gather_partials, local_tokens

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.Generator(np.random.PCG64(9))
        heads, dim = 4, 16
        q = rng.standard_normal((heads, dim))
        k = rng.standard_normal((tokens, heads, dim))
        v = rng.standard_normal((tokens, heads, dim))
        lo, hi = local_tokens(tokens, 16, world, rank)
        scale = 1 / math.sqrt(dim)
        m = torch.zeros(heads, dtype=torch.float64)
        l = torch.zeros(heads, dtype=torch.float64)
        o = torch.zeros((heads, dim), dtype=torch.float64)
        for h in range(heads):
            mh, lh, oh = _partials(q[h], k[lo:hi, h], v[lo:hi, h], scale)
            m[h], l[h], o[h] = mh, lh, torch.from_numpy(np.asarray(oh))
        gm, gl, go = all_gather_partials(m, l, o)
        assert gm.shape == (world, heads)
        if rank == 0:
            merged = np.zeros((heads, dim))
            for h in range(heads):
                # rank-order log-sum-exp merge (what inferlab_cuda_lse_combine does)
                big = gm[:, h].max().item()
                weight = torch.exp(gm[:, h] - big)
                den = (weight * gl[:, h]).sum()
                merged[h] = ((weight[:, None] * go[:, h]).sum(0) / den).numpy()
            whole = np.zeros((heads, dim))
            for h in range(heads):
                mh, lh, oh = _partials(q[h], k[:, h], v[:, h], scale)
                whole[h] = oh / lh
            np.save(result_path, np.stack([merged, whole]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens", [1000, 37])
def test_split_kv_merge_over_gloo(tmp_path, tokens):
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    path = str(tmp_path / "merged.npy")
    mp.start_processes(_worker, args=(world, port, tokens, path), nprocs=world,
                       start_method="spawn", join=True)
    merged, whole = np.load(path)
    assert np.max(np.abs(merged - whole)) <= 1e-12 + 1e-10 * np.max(np.abs(whole))

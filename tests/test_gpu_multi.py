"""Multi-GPU parity (needs 2, 4 or 8 GPUs; each case is skipped otherwise).

One 131,072-token sequence (GQA 32/8 x 128, bf16) split across the GPUs by
contiguous block ranges: each rank decodes its range into (m, l, o)
partials, the partials are all-gathered over NCCL and merged in rank order;
the result must equal the whole-context decode on one GPU within the fp32
tolerance |a - b| <= 1e-6 + 1e-5 |b|. The decode with the exchange fused
into it over NVLink peer memory (distributed.PeerExchange, five steps in a
row so both buffer parities are reused, with a call rejected on one rank
between them that must leave the ranks' step counts in step), and then the packed partials
through the standalone exchange kernel, must equal the NCCL result bit for
bit. Ranks are spawned processes with a short process-group timeout.
"""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path):
    import torch
    import torch.distributed as dist

    from inferlab_b200 import distributed, paged, workloads as wl

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        total = 131072
        # every rank builds the same full sequence (same seed) so rank 0 can
        # also decode it whole; each rank then keeps only its own block range
        full = wl.decode_batch(rank, 77, 1, np.array([total]), 32, 8, 128, wl.KV_BF16,
                               max_context_len=total)
        lo, hi = distributed.local_tokens(total, 16, world, rank)
        blocks = full.block_tables[:, lo // 16:(hi + 15) // 16].contiguous()
        merged = distributed.decode_split_sequence(full.pool, full.queries, blocks, hi - lo)
        exchange = distributed.PeerExchange(32, 128)
        lens = torch.full((1,), hi - lo, dtype=torch.int32, device=f"cuda:{rank}")

        def fused():
            return distributed.decode_split_sequence(full.pool, full.queries, blocks, hi - lo,
                                                     exchange=exchange).clone()

        # the decode and the exchange in one kernel, five steps in a row; after
        # the second, rank 0 alone makes a call that is rejected (no split
        # workspace): it must take no exchange step, or the ranks' later
        # exchanges no longer pair up and their waits time out
        peer = [fused() for _ in range(2)]
        if rank == 0:
            try:
                exchange.decode(full.pool, full.queries, blocks, lens, hi - lo)
            except paged.AttentionError as e:
                assert "workspace is too small" in str(e), e
            else:
                raise AssertionError("a decode exchange without workspace was accepted")
        peer += [fused() for _ in range(3)]
        # then the packed partials through the standalone exchange kernel
        send = torch.empty(32 * 130, dtype=torch.float32, device=f"cuda:{rank}")
        for _ in range(2):
            full.pool.decode_partials(full.queries, blocks, lens, hi - lo, packed=send)
            peer.append(exchange.combine(send).view(1, 32, 128).clone())
        exchange.synchronize(timeout_ms=20000)
        exchange.close()
        whole = full.pool.decode(full.queries, full.block_tables, full.context_lens, total)
        full.pool.synchronize()
        if rank == 0:
            np.save(path, np.stack([merged.cpu().numpy(), whole.cpu().numpy()] +
                                   [x.cpu().numpy() for x in peer]))
        full.pool.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_split_sequence_over_nccl_matches_single_gpu(tmp_path, world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    path = str(tmp_path / "out.npy")
    mp.start_processes(_rank_main, args=(world, _port(), path), nprocs=world,
                       start_method="spawn", join=True)
    merged, whole, *peer = np.load(path)
    err = np.abs(merged.astype(np.float64) - whole)
    assert np.all(err <= 1e-6 + 1e-5 * np.abs(whole)), float(err.max())
    for x in peer:
        assert np.array_equal(x, merged)


def _missing_peer_main(rank, world, port, path):
    import torch
    import torch.distributed as dist

    from inferlab_b200 import AttentionError, distributed

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        exchange = distributed.PeerExchange(4, 64)
        block = torch.zeros(4 * 66, dtype=torch.float32, device=f"cuda:{rank}")
        block[4:8] = 1.0  # l = 1 for every row, m = 0, o = 0
        outcome = "no error"
        if rank == 0:
            # rank 1 leaves this step out (between steps, nothing of its own in
            # flight): rank 0's bounded wait runs out and reports it
            exchange.combine(block)
            try:
                exchange.synchronize(timeout_ms=30000)
            except AttentionError as caught:
                outcome = str(caught)
            with open(path, "w") as f:
                f.write(outcome)
        dist.barrier()
        exchange.close()
    finally:
        dist.destroy_process_group()


def test_peer_exchange_reports_a_missing_peer(tmp_path):
    """Failure detection without a GPU fault: one rank skips an exchange, the
    other's bounded wait (about 2 s) gives up and its synchronize raises
    "device wait timed out"; the CUDA context stays usable and both ranks
    close cleanly. NVLS stays off (NCCL_NVLS_ENABLE=0); the exchange itself
    uses plain peer stores."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    path = str(tmp_path / "outcome.txt")
    mp.start_processes(_missing_peer_main, args=(2, _port(), path), nprocs=2,
                       start_method="spawn", join=True)
    with open(path) as f:
        assert f.read() == "device wait timed out"

"""Block ownership (inferlab_cuda_pages_*) against the reference's behaviour.

CPU only: the manager is host metadata. Pinned two ways:
  * the reference's own known-answer tests for the paged cache
    (worker/src/lib.rs:2261-2358), replayed at the page level - the token
    counts, page sizes and expected statistics are theirs;
  * a differential test against oracle/page_pool.py, the CPU restatement of
    PagedKvPool (worker/cpp/inferlab_runtime.cpp:649-1032), over seeded random
    sequences of appends, releases, prefix publications and lookups: tables,
    copy-on-write decisions, statistics and error messages must agree.
"""
import numpy as np
import pytest

from inferlab_b200 import AttentionError, PageManager
from oracle.page_pool import PagePool, PagePoolError


def test_shared_partial_prefix_is_copied_before_append():
    """worker/src/lib.rs:2261-2318: page_tokens 4, 8 pages, prefix capacity 4;
    a 3-token prompt (rows of 128 bytes: the tiny model's 16 floats x K,V x 4 B)."""
    m = PageManager(8, 4, 128, 4)
    cold, n = [], 0
    for _ in range(3):
        cold, copy = m.prepare_append(cold, n)
        assert copy is None
        n += 1
    m.publish_prefix([11, 12, 13], cold, 3)
    m.release(cold)

    warm, reused = m.acquire_prefix([11, 12, 13])
    assert reused == 3
    s = m.stats()
    assert (s["allocated_pages"], s["shared_pages"], s["maximum_refcount"],
            s["bytes_saved_by_sharing"]) == (1, 1, 2, 384)
    assert s["prefix_hits"] == 1 and s["prefix_tokens_reused"] == 3

    warm, copy = m.prepare_append(warm, 3)  # the shared tail is copied first
    assert copy == (0, 1) and warm == [1]
    s = m.stats()
    assert s["copy_on_write_copies"] == 1 and s["allocated_pages"] == 2
    m.release(warm)
    assert m.stats()["allocated_pages"] == 1


def test_paged_capacity_is_bounded_and_pages_return_after_drop():
    """worker/src/lib.rs:2320-2358: page_tokens 4, 16 pages, no prefixes; eight
    sessions of 8 tokens fill the pool, the ninth fails, dropping frees all."""
    m = PageManager(16, 4, 128, 0)
    tables = []
    for _ in range(8):
        t = []
        for n in range(8):
            t, _ = m.prepare_append(t, n)
        tables.append(t)
    s = m.stats()
    assert (s["allocated_pages"], s["free_pages"], s["used_token_slots"]) == (16, 0, 64)
    with pytest.raises(AttentionError, match="capacity exhausted"):
        m.prepare_append([], 0)
    for t in tables:
        m.release(t)
    s = m.stats()
    assert (s["allocated_pages"], s["free_pages"], s["allocation_failures"]) == (0, 16, 1)


def test_dimensions_must_be_positive():
    with pytest.raises(AttentionError, match="^paged KV cache dimensions must be positive$"):
        PageManager(0, 16, 128)
    with pytest.raises(PagePoolError, match="^paged KV cache dimensions must be positive$"):
        PagePool(0, 16, 128, 0)


def _run_differential(seed: int, pages: int, page_tokens: int, prefix_capacity: int, ops: int):
    rng = np.random.Generator(np.random.PCG64(seed))
    ours = PageManager(pages, page_tokens, 96, prefix_capacity)
    ref = PagePool(pages, page_tokens, 96, prefix_capacity)
    seqs = []  # [tokens, our table, reference table]
    vocab = 4  # small, so prefixes collide and get reused
    for step in range(ops):
        op = rng.integers(0, 10)
        if op < 5 and seqs:  # append one token to a sequence
            s = seqs[rng.integers(0, len(seqs))]
            n = len(s[0])
            got = err_ours = err_ref = None
            try:
                table, copy = ours.prepare_append(s[1], n)
            except AttentionError as e:
                err_ours = str(e)
            try:
                rcopy = ref.append(s[2], n)
            except PagePoolError as e:
                err_ref = str(e)
            assert err_ours == err_ref, (step, err_ours, err_ref)
            if err_ours is None:
                assert copy == rcopy and table == s[2], (step, copy, rcopy, table, s[2])
                s[1] = table
                s[0].append(int(rng.integers(0, vocab)))
        elif op < 7:  # a new sequence, starting from the longest published prefix
            tokens = [int(x) for x in rng.integers(0, vocab, size=int(rng.integers(1, 12)))]
            blocks, reused = ours.acquire_prefix(tokens)
            rblocks, rreused = ref.acquire_longest_prefix(tokens)
            assert (blocks, reused) == (rblocks, rreused), step
            seqs.append([tokens[:reused], blocks, rblocks])
        elif op < 8 and seqs:  # publish a sequence's tokens as a prefix
            s = seqs[rng.integers(0, len(seqs))]
            if s[0]:
                cut = int(rng.integers(1, len(s[0]) + 1))
                ours.publish_prefix(s[0][:cut], s[1], len(s[0]))
                ref.publish_prefix(s[0][:cut], s[2], len(s[0]))
        elif seqs:  # a sequence ends
            s = seqs.pop(int(rng.integers(0, len(seqs))))
            ours.release(s[1])
            ref.release_table(s[2])
        for s in seqs:
            assert ours.shared_pages(s[1]) == ref.shared_pages(s[2])
        assert ours.stats() == ref.stats(), step
    return ours.stats()


@pytest.mark.parametrize("seed,pages,page_tokens,prefix_capacity", [
    (1, 12, 4, 3), (2, 6, 2, 2), (3, 40, 16, 0), (4, 9, 3, 8),
    (5, 3, 1, 1),    # one-token pages, a single prefix slot, constant exhaustion
    (6, 20, 7, 5)])  # page size that divides nothing in the token stream
def test_matches_restated_pool_on_random_operations(seed, pages, page_tokens, prefix_capacity):
    final = _run_differential(seed, pages, page_tokens, prefix_capacity, 400)
    # the seeds reach the interesting paths
    if prefix_capacity:
        assert final["prefix_hits"] > 0
    if seed in (1, 2):
        assert final["copy_on_write_copies"] > 0 and final["evictions"] > 0

"""The projection oracle (oracle/projection.py) against the reference's own
fp32 linear (worker/cpp/inferlab_runtime.cpp:1266-1285), bit for bit. CPU only."""
import numpy as np
import pytest

from oracle import projection


@pytest.mark.parametrize("rows,inputs,outputs", [(1, 16, 48), (7, 64, 96), (33, 128, 384)])
def test_linear_matches_the_reference_bit_for_bit(rows, inputs, outputs):
    rng = np.random.Generator(np.random.PCG64(rows * 1000 + inputs))
    x = rng.standard_normal((rows, inputs), dtype=np.float32)
    w = rng.standard_normal((outputs, inputs), dtype=np.float32) * np.float32(0.1)
    ref = projection.ref_linear(x, w)
    if ref is None:
        pytest.skip("oracle/_ref/libref_linear.so is not built (no reference tree)")
    got = projection.linear(x, w)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_placement_follows_the_block_table():
    tables = np.array([[5, 9, 2], [7, 1, 3]], np.int32)
    hidden = np.ones((3, 8), np.float32)
    weights = np.ones(((1 + 2) * 32, 8), np.float32)
    q, k, v, blocks, slots = projection.project_append(
        hidden, weights, 1, 1, 32, [0, 1, 1], [3, 17, 40], tables, 16)
    assert q.shape == (3, 1, 32) and k.shape == (3, 1, 32) and v.shape == (3, 1, 32)
    assert blocks.tolist() == [5, 1, 3] and slots.tolist() == [3, 1, 8]
    assert np.all(q == 8.0)

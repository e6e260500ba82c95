"""GPU parity of the drop-in entry inferlab_attention_forward against the oracle.

Every call goes through the C ABI (run_attention -> libinferlab_attention_cuda.so).
Tolerance (fp32 arithmetic on both sides): |gpu - oracle| <= 1e-6 + 1e-5 * |oracle|.
Stats are integer and must match exactly.
"""
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATOL, RTOL = 1e-6, 1e-5


def close(got, ref):
    got = np.asarray(got, np.float64).reshape(-1)
    ref = np.asarray(ref, np.float64).reshape(-1)
    bad = np.abs(got - ref) > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), (f"{bad.sum()} of {bad.size} outside tolerance; max abs err "
                           f"{np.max(np.abs(got - ref)):.3e}")


@pytest.fixture(scope="module")
def il():
    import torch

    assert torch.cuda.is_available(), "these tests need a CUDA device"
    import inferlab_b200

    return inferlab_b200


def run(il, q, k, v, tq, tkv, h, d, start, algorithm=0, precision=0, tile=16, causal=True):
    cfg = il.AttentionConfig(il.AttentionAlgorithm(algorithm), il.AttentionPrecision(precision),
                             tile, causal)
    return il.run_attention(q, k, v, tq, tkv, h, d, start, cfg)


def test_probe_fixture_all_variants(il, oracle_mod):
    with open(os.path.join(GOLDEN, "attention_probe_v012.json")) as handle:
        probe = json.load(handle)
    t, h, d = probe["tokens"], probe["heads"], probe["head_dimension"]
    algos = {"materialized": 0, "online-tiled": 1}
    precs = {"fp32": 0, "fp16": 1, "bf16": 2}
    for variant in probe["variants"]:
        a, p = algos[variant["algorithm"]], precs[variant["precision"]]
        got = run(il, probe["queries"], probe["keys"], probe["values"], t, t, h, d, 0, a, p,
                  probe["tile_tokens"])
        ref, ref_stats = oracle_mod.attention_forward(probe["queries"], probe["keys"],
                                                      probe["values"], t, t, h, d, 0, a, p,
                                                      probe["tile_tokens"])
        close(got.output, ref)
        # and within the reference checker's 2e-6 of the retained goldens
        assert np.max(np.abs(got.output - np.array(variant["output"], np.float32))) <= 2e-6
        assert got.stats.as_dict() == variant["stats"] == ref_stats


def test_single_sequence_workload_reference_fixture(il):
    """1 x 128 tokens, 4 heads x 32, fp32: prefill then decode of token 129,
    against outputs of the reference's own build (tests/golden/ref_cfg1.npz)."""
    data = np.load(os.path.join(GOLDEN, "ref_cfg1.npz"))
    q, k, v = data["q"], data["k"], data["v"]
    for algorithm in (0, 1):
        for precision in (0, 1, 2):
            tag = f"a{algorithm}p{precision}"
            pre = run(il, q[:128], k[:128], v[:128], 128, 128, 4, 32, 0, algorithm, precision)
            dec = run(il, q[128:], k, v, 1, 129, 4, 32, 128, algorithm, precision)
            close(pre.output, data[f"prefill_{tag}"])
            close(dec.output, data[f"decode_{tag}"])
            assert list(pre.stats.as_dict().values()) == data[f"prefill_stats_{tag}"].tolist()
            assert list(dec.stats.as_dict().values()) == data[f"decode_stats_{tag}"].tolist()


@pytest.mark.parametrize("seed", range(8))
def test_random_shapes_match_oracle(il, oracle_mod, seed):
    rng = np.random.Generator(np.random.PCG64(100 + seed))
    for _ in range(3):
        heads = int(rng.integers(1, 6))
        dim = int(rng.choice([1, 2, 7, 8, 32, 64, 96, 128, 257]))
        kv = int(rng.integers(1, 700))
        causal = bool(rng.integers(0, 2))
        start = int(rng.integers(0, kv)) if causal else int(rng.integers(0, 50))
        tq = int(rng.integers(1, min(kv - start, 64) + 1)) if causal else int(rng.integers(1, 40))
        tile = int(rng.choice([1, 5, 16, 4096]))
        q = rng.standard_normal(tq * heads * dim, dtype=np.float32) * 2
        k = rng.standard_normal(kv * heads * dim, dtype=np.float32) * 2
        v = rng.standard_normal(kv * heads * dim, dtype=np.float32)
        for algorithm in (0, 1):
            for precision in (0, 1, 2):
                got = run(il, q, k, v, tq, kv, heads, dim, start, algorithm, precision, tile, causal)
                ref, stats = oracle_mod.attention_forward(q, k, v, tq, kv, heads, dim, start,
                                                          algorithm, precision, tile, causal)
                close(got.output, ref)
                assert got.stats.as_dict() == stats


def test_known_answers(il):
    """worker/src/lib.rs:2850-2869: future K/V never leak; exact [0.25, -0.5]."""
    q = [1000.0, -1000.0]
    k = [1000.0, -1000.0, 4.0, 5.0, -8.0, 9.0]
    a = run(il, q, k, [0.25, -0.5, 10.0, 20.0, 30.0, 40.0], 1, 3, 1, 2, 0, 1, 1, 2)
    b = run(il, q, k, [0.25, -0.5, -100.0, 200.0, 300.0, -400.0], 1, 3, 1, 2, 0, 1, 1, 2)
    assert a.output.tolist() == [0.25, -0.5]
    assert b.output.tolist() == [0.25, -0.5]


def test_large_scores_stay_finite(il, oracle_mod):
    """worker/src/bin/inferlab-attention-probe.rs:262-316 (scores ~1e5)."""
    tokens, heads, dim = 9, 2, 8
    idx = np.arange(tokens * heads * dim)
    q = np.where(idx % 3 == 0, 220.0, -180.0).astype(np.float32)
    k = np.where(idx % 5 < 2, 190.0, -210.0).astype(np.float32)
    v = np.sin(idx * 0.29).astype(np.float32)
    for precision in (0, 1, 2):
        for algorithm in (0, 1):
            got = run(il, q, k, v, tokens, tokens, heads, dim, 0, algorithm, precision, 3)
            ref, _ = oracle_mod.attention_forward(q, k, v, tokens, tokens, heads, dim, 0,
                                                  algorithm, precision, 3)
            assert np.all(np.isfinite(got.output))
            close(got.output, ref)


def test_non_finite_input_is_rejected(il):
    q = np.ones(8, np.float32)
    k = np.ones(16, np.float32)
    v = np.ones(16, np.float32)
    v[-1] = np.nan  # outside the causal range of query 0, still rejected as in the reference
    with pytest.raises(il.AttentionError, match="^attention input must be finite$"):
        run(il, q, k, v, 1, 2, 2, 4, 0)
    k[3] = np.inf
    with pytest.raises(il.AttentionError, match="^attention input must be finite$"):
        run(il, q, k, np.ones(16, np.float32), 1, 2, 2, 4, 0)
    # and the device context stays usable afterwards
    good = run(il, q, np.ones(16, np.float32), np.ones(16, np.float32), 1, 2, 2, 4, 0)
    assert np.allclose(good.output, 1.0)


def test_head_dim_limit(il):
    with pytest.raises(il.AttentionError, match="exceeds the CUDA kernel limit"):
        run(il, np.ones(4097, np.float32), np.ones(4097, np.float32), np.ones(4097, np.float32),
            1, 1, 1, 4097, 0)


def test_cpp_api_matches_c_api(il, oracle_mod):
    """The C++ entry inferlab::attention_forward is the same implementation."""
    import ctypes
    import subprocess
    import tempfile

    from inferlab_b200 import _lib

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    source = r'''
#include "attention_cuda.h"
#include <cstdio>
#include <stdexcept>
#include <vector>
int main() {
    std::vector<float> q(3 * 2 * 8), k(5 * 2 * 8), v(5 * 2 * 8), out(3 * 2 * 8);
    for (size_t i = 0; i < k.size(); ++i) { k[i] = 0.01f * i; v[i] = 0.5f - 0.02f * i; }
    for (size_t i = 0; i < q.size(); ++i) q[i] = 0.03f * i - 0.2f;
    inferlab::AttentionConfig cfg;
    cfg.algorithm = inferlab::AttentionAlgorithm::OnlineTiled;
    inferlab::AttentionStats stats;
    inferlab::attention_forward(q.data(), k.data(), v.data(), 3, 5, 2, 8, 2, cfg, out.data(), &stats);
    for (float x : out) std::printf("%.9g\n", x);
    std::printf("%llu\n", (unsigned long long)stats.score_elements);
    try {
        inferlab::attention_forward(q.data(), k.data(), v.data(), 3, 5, 2, 8, 3, cfg, out.data(), &stats);
    } catch (const std::runtime_error& e) { std::printf("%s\n", e.what()); }
    return 0;
}
'''
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "main.cpp")
        exe = os.path.join(tmp, "main")
        with open(src, "w") as handle:
            handle.write(source)
        subprocess.run(["g++", "-std=c++17", "-I", os.path.join(root, "include"), src, "-o", exe,
                        _lib.LIBPATH, f"-Wl,-rpath,{os.path.dirname(_lib.LIBPATH)}"],
                       check=True)
        lines = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    got = np.array([float(x) for x in lines[:48]], np.float32)
    q = (0.03 * np.arange(48, dtype=np.float32) - np.float32(0.2)).astype(np.float32)
    k = (0.01 * np.arange(80, dtype=np.float32)).astype(np.float32)
    v = (np.float32(0.5) - 0.02 * np.arange(80, dtype=np.float32)).astype(np.float32)
    ref, stats = oracle_mod.attention_forward(q, k, v, 3, 5, 2, 8, 2, 1, 0, 16)
    close(got, ref)
    assert int(lines[48]) == stats["score_elements"]
    assert " ".join(lines[49:]) == "causal query positions exceed the KV sequence"


@pytest.mark.parametrize("precision", [1, 2])
@pytest.mark.parametrize("algorithm", [0, 1])
@pytest.mark.parametrize("tq,tkv,h,start", [(512, 512, 8, 0), (300, 700, 4, 400),
                                            (1024, 1030, 2, 6)])
def test_tensor_route_fp16_bf16_modes(il, oracle_mod, precision, algorithm, tq, tkv, h, start):
    """Fp16 / Bf16 storage mode, head_dim 128, causal, at least 1024 query rows:
    the drop-in entry runs the tensor-core prefill. Against the reference's
    own mode (the oracle rounds inputs as round_attention_value does, then
    computes in fp32) the tolerance is the f16/bf16 one, |gpu - ref| <=
    2e-3 |ref| + 1e-3 max|ref row| (fp16 probabilities); stats are exact."""
    rng = np.random.Generator(np.random.PCG64(tq + 10 * h + precision))
    q = rng.standard_normal(tq * h * 128, dtype=np.float32)
    k = rng.standard_normal(tkv * h * 128, dtype=np.float32)
    v = rng.standard_normal(tkv * h * 128, dtype=np.float32)
    got = run(il, q, k, v, tq, tkv, h, 128, start, algorithm, precision)
    ref, ref_stats = oracle_mod.attention_forward(q, k, v, tq, tkv, h, 128, start, algorithm,
                                                  precision, 16)
    got_rows = np.asarray(got.output, np.float64).reshape(-1, 128)
    ref_rows = np.asarray(ref, np.float64).reshape(-1, 128)
    err = np.abs(got_rows - ref_rows)
    bound = 2e-3 * np.abs(ref_rows) + 1e-3 * np.max(np.abs(ref_rows), axis=1, keepdims=True)
    assert np.all(err <= bound), f"max abs err {err.max():.3e}"
    assert got.stats.as_dict() == ref_stats


def test_tensor_route_falls_back_for_values_beyond_fp16(il, oracle_mod):
    """A Bf16-mode V value beyond fp16's range (the tensor path widens V to
    fp16) sends the call back to the fp32 kernel: the result then meets the
    fp32 tolerance against the oracle."""
    rng = np.random.Generator(np.random.PCG64(77))
    tq, h = 512, 4
    q = rng.standard_normal(tq * h * 128, dtype=np.float32)
    k = rng.standard_normal(tq * h * 128, dtype=np.float32)
    v = rng.standard_normal(tq * h * 128, dtype=np.float32)
    v[12345] = 1.0e5
    got = run(il, q, k, v, tq, tq, h, 128, 0, 1, 2)
    ref, ref_stats = oracle_mod.attention_forward(q, k, v, tq, tq, h, 128, 0, 1, 2, 16)
    close(got.output, ref)
    assert got.stats.as_dict() == ref_stats

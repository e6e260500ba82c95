#!/usr/bin/env python3
"""Regenerate the golden fixtures in this directory.

Run where the reference tree is mounted (it is read, never written):

    python tests/golden/make_golden.py --reference-root <reference checkout>

Writes:
  attention_probe_v012.json  - the reference's retained attention probe
      fixture (docs/results/v0.12/raw/attention-probe.json: T=11, H=3, d=8
      inputs, six algorithm x precision outputs with their stats, scaling
      stats and checksums) and its PyTorch oracle outputs
      (docs/results/v0.12/raw/attention-torch.json). Copied field by field.
  ref_cfg1.npz  - outputs of the reference's own kernel (oracle/_ref/libref.so,
      compiled from kernels/attention_cpu.cpp by oracle/Makefile) on the
      single-sequence workload: 1 x 128 tokens, 4 heads x head_dim 32, fp32,
      Q/K/V ~ N(0,1) from PCG64(seed 20261201) over 129 tokens; causal prefill
      of the first 128 queries (start 0), then decode of query 128 against all
      129 keys (start 128), for both algorithms and all three precisions.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402


def probe_fixture(reference_root: str) -> dict:
    raw = os.path.join(reference_root, "docs", "results", "v0.12", "raw")
    with open(os.path.join(raw, "attention-probe.json")) as handle:
        probe = json.load(handle)
    with open(os.path.join(raw, "attention-torch.json")) as handle:
        torch_ref = json.load(handle)
    fixture = probe["fixture"]
    return {
        "source": "docs/results/v0.12/raw/attention-probe.json + attention-torch.json",
        "tokens": fixture["tokens"],
        "heads": fixture["heads"],
        "head_dimension": fixture["head_dimension"],
        "tile_tokens": fixture["tile_tokens"],
        "queries": fixture["queries"],
        "keys": fixture["keys"],
        "values": fixture["values"],
        "variants": [
            {
                "algorithm": variant["algorithm"],
                "precision": variant["precision"],
                "output": variant["output"],
                "stats": variant["stats"],
            }
            for variant in fixture["variants"]
        ],
        "torch": [
            {"precision": entry["precision"], "output": entry["output"]}
            for entry in torch_ref["references"]
        ],
        "causal_isolation": probe["causal_isolation"],
        "large_score_stability": probe["large_score_stability"],
        "sequence_scaling": [
            {
                "tokens": entry["tokens"],
                "heads": entry["heads"],
                "head_dimension": entry["head_dimension"],
                "tile_tokens": probe["benchmark_tile_tokens"],
                "profiles": [
                    {"algorithm": prof["algorithm"], "checksum": prof["checksum"],
                     "stats": prof["stats"]}
                    for prof in entry["profiles"]
                ],
            }
            for entry in probe["sequence_scaling"]
        ],
    }


def cfg1_reference() -> dict:
    if oracle.ref_lib() is None:
        raise SystemExit("oracle/_ref/libref.so is missing: run `make -C oracle` first")
    rng = np.random.Generator(np.random.PCG64(20261201))
    tokens, heads, dim = 129, 4, 32
    q = rng.standard_normal((tokens, heads, dim), dtype=np.float32)
    k = rng.standard_normal((tokens, heads, dim), dtype=np.float32)
    v = rng.standard_normal((tokens, heads, dim), dtype=np.float32)
    arrays = {"q": q, "k": k, "v": v}
    for algorithm in (oracle.MATERIALIZED, oracle.ONLINE_TILED):
        for precision in (oracle.FP32, oracle.FP16, oracle.BF16):
            tag = f"a{algorithm}p{precision}"
            prefill, stats_p = oracle.attention_forward(
                q[:128], k[:128], v[:128], 128, 128, heads, dim, 0, algorithm, precision, 16,
                True, impl="reference")
            decode, stats_d = oracle.attention_forward(
                q[128:], k, v, 1, 129, heads, dim, 128, algorithm, precision, 16, True,
                impl="reference")
            arrays[f"prefill_{tag}"] = prefill.reshape(128, heads, dim)
            arrays[f"decode_{tag}"] = decode.reshape(1, heads, dim)
            arrays[f"prefill_stats_{tag}"] = np.array(
                [stats_p[name] for name in oracle.STAT_FIELDS], dtype=np.uint64)
            arrays[f"decode_stats_{tag}"] = np.array(
                [stats_d[name] for name in oracle.STAT_FIELDS], dtype=np.uint64)
    return arrays


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-root", required=True,
                        help="root of the reference checkout (read only)")
    args = parser.parse_args()
    oracle.build(args.reference_root)
    with open(os.path.join(HERE, "attention_probe_v012.json"), "w") as handle:
        json.dump(probe_fixture(args.reference_root), handle)
        handle.write("\n")
    np.savez_compressed(os.path.join(HERE, "ref_cfg1.npz"), **cfg1_reference())


if __name__ == "__main__":
    main()

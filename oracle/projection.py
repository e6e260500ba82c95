"""CPU restatement of the Q/K/V projection beside attention.

TEST INFRASTRUCTURE ONLY: tests and bench.py's cpu_baseline use it as the
checker for inferlab_cuda_qkv_project_append. Restates:
  * `linear` (worker/cpp/inferlab_runtime.cpp:1266-1285): for every row and
    output feature, value = 0 (no bias), then value += input[row][in] *
    weight(out, in) for in = 0, 1, ... in fp32 (separate multiply and add);
    the loop over `in` is kept, vectorised over rows and outputs, so the
    rounding sequence is the reference's;
  * the forward pass's three projections (:1318-1325) as one stacked weight
    [W_q; W_k; W_v];
  * PagedKvPool::append's placement (:713-767): token t's row goes to block
    table[seq][pos // block_tokens], slot pos % block_tokens;
  * the output projection and residual add (:1340-1350): hidden +
    linear(attention_context, attention_output_weight).
Pinned: tests/test_projection_oracle.py checks `linear` bit for bit against
the reference's own function (oracle/_ref/libref_linear.so, built from
worker/cpp/inferlab_runtime.cpp in place).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """x [rows][in] fp32, w [out][in] fp32 -> [rows][out] fp32, the reference's order."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    acc = np.zeros((x.shape[0], w.shape[0]), dtype=np.float32)
    for i in range(x.shape[1]):
        acc += np.multiply.outer(x[:, i], w[:, i]).astype(np.float32)
    return acc


def ref_linear(x: np.ndarray, w: np.ndarray) -> np.ndarray | None:
    """The reference's own linear() through oracle/_ref/libref_linear.so, or None."""
    path = os.path.join(_HERE, "_ref", "libref_linear.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    f = lib.oracle_ref_linear
    f.restype = ctypes.c_int
    fp = ctypes.POINTER(ctypes.c_float)
    f.argtypes = [fp, ctypes.c_size_t, ctypes.c_size_t, fp, ctypes.c_size_t, fp]
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty((x.shape[0], w.shape[0]), dtype=np.float32)
    if f(x.ctypes.data_as(fp), x.shape[0], x.shape[1], w.ctypes.data_as(fp), w.shape[0],
         out.ctypes.data_as(fp)) != 0:
        raise RuntimeError("reference linear failed")
    return out


def project_append(hidden: np.ndarray, weights: np.ndarray, q_heads: int, kv_heads: int,
                   head_dim: int, row_sequences, positions, tables, block_tokens: int):
    """Q [T][q_heads][d] and the K/V rows with their (block, slot) placements:
    returns (q, k_rows [T][kv_heads][d], v_rows, blocks [T], slots [T])."""
    y = linear(hidden, weights)
    t = hidden.shape[0]
    qd, kd = q_heads * head_dim, kv_heads * head_dim
    q = y[:, :qd].reshape(t, q_heads, head_dim)
    k = y[:, qd:qd + kd].reshape(t, kv_heads, head_dim)
    v = y[:, qd + kd:].reshape(t, kv_heads, head_dim)
    pos = np.asarray(positions)
    seq = np.asarray(row_sequences)
    blocks = np.asarray(tables)[seq, pos // block_tokens]
    return q, k, v, blocks, pos % block_tokens


def output_project(attention: np.ndarray, weights: np.ndarray, residual=None) -> np.ndarray:
    """residual + linear(attention, weights), fp32, the reference's order
    (the residual is added after the full sum, as hidden += attention_output)."""
    y = linear(attention, weights)
    return y if residual is None else (np.asarray(residual, np.float32) + y).astype(np.float32)

"""ctypes bindings for the CPU oracle (liboracle.so) and the reference build
(_ref/libref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker. The product package
(inferlab_b200) never imports this module.

liboracle.so is the C restatement in attention_oracle.c; libref.so is the
reference's kernels/attention_cpu.cpp + worker/cpp/inferlab_runtime.cpp
compiled by oracle/Makefile. Both are built on demand with `make -C oracle`
(gcc/g++ only, no GPU).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref.so")

FP32, FP16, BF16 = 0, 1, 2
MATERIALIZED, ONLINE_TILED = 0, 1

_lock = threading.Lock()
_oracle = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_sz = ctypes.c_size_t


class InferlabAttentionConfig(ctypes.Structure):
    """worker/cpp/inferlab_runtime.h:67-72."""

    _fields_ = [
        ("algorithm", ctypes.c_uint32),
        ("precision", ctypes.c_uint32),
        ("tile_tokens", ctypes.c_uint32),
        ("causal", ctypes.c_uint32),
    ]


class InferlabAttentionStats(ctypes.Structure):
    """worker/cpp/inferlab_runtime.h:74-83."""

    _fields_ = [
        ("score_elements", ctypes.c_uint64),
        ("masked_score_elements", ctypes.c_uint64),
        ("score_buffer_bytes", ctypes.c_uint64),
        ("working_set_bytes", ctypes.c_uint64),
        ("modeled_external_read_bytes", ctypes.c_uint64),
        ("modeled_external_write_bytes", ctypes.c_uint64),
        ("modeled_external_total_bytes", ctypes.c_uint64),
        ("key_tiles", ctypes.c_uint64),
    ]


STAT_FIELDS = [name for name, _ in InferlabAttentionStats._fields_]


def build(reference_root: str | None = None) -> None:
    """Compile liboracle.so, and the reference's own kernel into _ref/ when
    reference_root (or the INFERLAB_REFERENCE_ROOT environment variable) names
    a reference checkout."""
    root = reference_root or os.environ.get("INFERLAB_REFERENCE_ROOT", "")
    cmd = ["make", "-s", "-C", HERE]
    if root:
        cmd.append(f"REFERENCE_ROOT={root}")
    subprocess.run(cmd, check=True)


def _ptr(array: np.ndarray, ctype):
    return array.ctypes.data_as(ctypes.POINTER(ctype))


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    with _lock:
        if _oracle is None:
            if not os.path.exists(ORACLE_SO):
                build()
            lib = ctypes.CDLL(ORACLE_SO)
            lib.oracle_attention_forward.restype = ctypes.c_int
            lib.oracle_attention_forward.argtypes = [
                _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _u32p, _f32p, _sz, _u64p,
                ctypes.c_char_p, _sz,
            ]
            lib.oracle_half_bits_to_float.restype = ctypes.c_float
            lib.oracle_half_bits_to_float.argtypes = [ctypes.c_uint16]
            lib.oracle_half_bits_to_float_ieee.restype = ctypes.c_float
            lib.oracle_half_bits_to_float_ieee.argtypes = [ctypes.c_uint16]
            lib.oracle_round_value.restype = ctypes.c_float
            lib.oracle_round_value.argtypes = [ctypes.c_float, ctypes.c_uint32]
            lib.oracle_float_to_half_bits.restype = ctypes.c_uint16
            lib.oracle_float_to_half_bits.argtypes = [ctypes.c_float]
            lib.oracle_float_to_bf16_bits.restype = ctypes.c_uint16
            lib.oracle_float_to_bf16_bits.argtypes = [ctypes.c_float]
            lib.oracle_materialize.restype = ctypes.c_int
            lib.oracle_materialize.argtypes = [
                ctypes.c_void_p, ctypes.c_uint32, _sz, _sz, _sz, _sz, _i32p, _sz, _sz, _f32p,
            ]
            lib.oracle_paged_attention.restype = ctypes.c_int
            lib.oracle_paged_attention.argtypes = [
                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, _sz, _sz, _sz, _sz, _sz,
                _i32p, _sz, _sz, _i64p, _i64p, _i64p, _f32p, ctypes.c_uint32, _sz, _f32p,
                ctypes.c_int,
            ]
            lib.oracle_lse_merge.restype = None
            lib.oracle_lse_merge.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p, _f32p]
            _oracle = lib
    return _oracle


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own kernel built from its sources, or None if absent."""
    global _ref
    with _lock:
        if _ref is None:
            if not os.path.exists(REF_SO):
                return None
            lib = ctypes.CDLL(REF_SO)
            lib.inferlab_attention_forward.restype = ctypes.c_int
            lib.inferlab_attention_forward.argtypes = [
                _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz,
                ctypes.POINTER(InferlabAttentionConfig), _f32p, _sz,
                ctypes.POINTER(InferlabAttentionStats), ctypes.c_char_p, _sz,
            ]
            # C++ inferlab::round_attention_value(float, AttentionPrecision)
            fn = getattr(lib, "_ZN8inferlab21round_attention_valueEfNS_18AttentionPrecisionE")
            fn.restype = ctypes.c_float
            fn.argtypes = [ctypes.c_float, ctypes.c_uint32]
            lib.round_attention_value = fn
            _ref = lib
    return _ref


class OracleError(RuntimeError):
    pass


def attention_forward(q, k, v, q_tokens, kv_tokens, heads, head_dim, start=0,
                      algorithm=MATERIALIZED, precision=FP32, tile_tokens=16, causal=True,
                      impl="oracle"):
    """Run the CPU attention on flat fp32 arrays; returns (output, stats dict).

    impl="oracle" uses the C restatement, impl="reference" the reference build.
    Raises OracleError with the library's message on failure.
    """
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1)
    k = np.ascontiguousarray(k, dtype=np.float32).reshape(-1)
    v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1)
    out = np.zeros(q_tokens * heads * head_dim, dtype=np.float32)
    err = ctypes.create_string_buffer(512)
    if impl == "oracle":
        lib = oracle_lib()
        config = np.array([algorithm, precision, tile_tokens, 1 if causal else 0], np.uint32)
        stats = np.zeros(8, np.uint64)
        status = lib.oracle_attention_forward(
            _ptr(q, ctypes.c_float), _ptr(k, ctypes.c_float), _ptr(v, ctypes.c_float),
            q_tokens, kv_tokens, heads, head_dim, start, _ptr(config, ctypes.c_uint32),
            _ptr(out, ctypes.c_float), out.size, _ptr(stats, ctypes.c_uint64), err, 512)
        stats_dict = dict(zip(STAT_FIELDS, (int(x) for x in stats)))
    else:
        lib = ref_lib()
        if lib is None:
            raise OracleError("reference library is not built")
        config = InferlabAttentionConfig(algorithm, precision, tile_tokens, 1 if causal else 0)
        stats = InferlabAttentionStats()
        status = lib.inferlab_attention_forward(
            _ptr(q, ctypes.c_float), _ptr(k, ctypes.c_float), _ptr(v, ctypes.c_float),
            q_tokens, kv_tokens, heads, head_dim, start, ctypes.byref(config),
            _ptr(out, ctypes.c_float), out.size, ctypes.byref(stats), err, 512)
        stats_dict = {name: int(getattr(stats, name)) for name in STAT_FIELDS}
    if status != 0:
        raise OracleError(err.value.decode())
    return out, stats_dict


def round_values(values: np.ndarray, precision: int) -> np.ndarray:
    """The reference's storage rounding of every element
    (round_attention_value, kernels/attention_cpu.cpp:405-417), including its
    widening of fp16 subnormals to half their value (:86-88)."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    if precision == FP32:
        return values.copy()
    if precision == FP16:
        widened = half_bits_to_float(float_to_half_bits(values))
        return np.where(np.abs(widened) < np.float32(2.0**-14), widened * np.float32(0.5),
                        widened).astype(np.float32)
    return bf16_bits_to_float(float_to_bf16_bits(values))


def round_values_ieee(values: np.ndarray, precision: int) -> np.ndarray:
    """IEEE round-to-nearest-even storage rounding (what the device pool stores)."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    if precision == FP32:
        return values.copy()
    if precision == FP16:
        return half_bits_to_float(float_to_half_bits(values))
    return bf16_bits_to_float(float_to_bf16_bits(values))


def float_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Vectorised restatement of kernels/attention_cpu.cpp:412-416."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_float(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def float_to_half_bits(values: np.ndarray) -> np.ndarray:
    """Element-wise oracle_float_to_half_bits (kernels/attention_cpu.cpp:15-67).

    Vectorised restatement of the same bit algorithm, checked against the C
    function in tests/test_oracle.py.
    """
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    biased = (bits >> 23) & 0xFF
    fraction = bits & 0x7FFFFF
    exponent = biased - 127 + 15
    out = np.zeros(bits.shape, dtype=np.int64)
    # normal
    result = (np.clip(exponent, 0, 31) << 10) | (fraction >> 13)
    dropped = fraction & 0x1FFF
    up = (dropped > 0x1000) | ((dropped == 0x1000) & ((result & 1) == 1))
    result = result + up
    result = np.where((result >> 10) >= 31, 0x7C00, result)
    normal = (exponent > 0) & (exponent < 31)
    out = np.where(normal, result, out)
    # subnormal
    sub = (exponent <= 0) & (exponent >= -10)
    shift = np.where(sub, 14 - exponent, 1)
    significand = fraction | 0x800000
    res_s = significand >> shift
    dropped_s = significand & ((1 << shift) - 1)
    half = 1 << (shift - 1)
    up_s = (dropped_s > half) | ((dropped_s == half) & ((res_s & 1) == 1))
    out = np.where(sub, res_s + up_s, out)
    # overflow / inf / nan
    out = np.where((exponent >= 31) & (biased != 0xFF), 0x7C00, out)
    out = np.where(biased == 0xFF, 0x7C00 | np.where(fraction != 0, 0x200, 0), out)
    return (out | sign).astype(np.uint16)


def half_bits_to_float(bits: np.ndarray) -> np.ndarray:
    """binary16 -> binary32, exact (numpy's float16 widening is exact)."""
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def materialize(arena_bits: np.ndarray, dtype: int, table: np.ndarray, tokens: int) -> np.ndarray:
    """Gather one sequence from an arena [num_blocks][kv_heads][block_tokens][head_dim]
    into [tokens][kv_heads][head_dim] fp32 (worker/cpp/inferlab_runtime.cpp:769-803)."""
    lib = oracle_lib()
    arena_bits = np.ascontiguousarray(arena_bits)
    nb, kvh, bt, hd = arena_bits.shape
    table = np.ascontiguousarray(table, dtype=np.int32)
    out = np.zeros((tokens, kvh, hd), dtype=np.float32)
    status = lib.oracle_materialize(arena_bits.ctypes.data, dtype, nb, kvh, bt, hd,
                                    _ptr(table, ctypes.c_int32), table.size, tokens,
                                    _ptr(out, ctypes.c_float))
    if status != 0:
        raise OracleError("paged KV block table is inconsistent" if status == -1
                          else "paged KV block table contains an invalid page")
    return out


def paged_attention(k_arena, v_arena, dtype, tables, starts, q_counts, q, q_heads,
                    algorithm=ONLINE_TILED, tile_tokens=16, threads=None):
    """Reference attention for a paged batch (see oracle_paged_attention).

    k_arena/v_arena: [num_blocks][kv_heads][block_tokens][head_dim] arrays of
    fp32 or 16-bit storage bits; tables [segments][max_blocks] int32; starts and
    q_counts per segment; q [total_q][q_heads][head_dim] fp32 (already rounded
    to the storage precision). Returns [total_q][q_heads][head_dim] fp32.
    """
    lib = oracle_lib()
    k_arena = np.ascontiguousarray(k_arena)
    v_arena = np.ascontiguousarray(v_arena)
    nb, kvh, bt, hd = k_arena.shape
    tables = np.ascontiguousarray(tables, dtype=np.int32)
    starts = np.ascontiguousarray(starts, dtype=np.int64)
    q_counts = np.ascontiguousarray(q_counts, dtype=np.int64)
    q_offsets = np.concatenate([[0], np.cumsum(q_counts)[:-1]]).astype(np.int64)
    q = np.ascontiguousarray(q, dtype=np.float32)
    out = np.zeros_like(q)
    if threads is None:
        threads = len(os.sched_getaffinity(0))
    status = lib.oracle_paged_attention(
        k_arena.ctypes.data, v_arena.ctypes.data, dtype, nb, kvh, bt, hd, q_heads,
        _ptr(tables, ctypes.c_int32), tables.shape[1], tables.shape[0],
        _ptr(starts, ctypes.c_int64), _ptr(q_counts, ctypes.c_int64),
        _ptr(q_offsets, ctypes.c_int64), _ptr(q, ctypes.c_float), algorithm, tile_tokens,
        _ptr(out, ctypes.c_float), threads)
    if status != 0:
        raise OracleError("oracle paged attention failed")
    return out


def lse_merge(m, l, o):
    """Merge split-KV partials m,l [parts][rows], o [parts][rows][head_dim]."""
    lib = oracle_lib()
    m = np.ascontiguousarray(m, dtype=np.float32)
    l = np.ascontiguousarray(l, dtype=np.float32)
    o = np.ascontiguousarray(o, dtype=np.float32)
    parts, rows, hd = o.shape
    out = np.zeros((rows, hd), dtype=np.float32)
    lib.oracle_lse_merge(parts, rows, hd, _ptr(m, ctypes.c_float), _ptr(l, ctypes.c_float),
                         _ptr(o, ctypes.c_float), _ptr(out, ctypes.c_float))
    return out


def reference_paged_decode_timed(k_arena, v_arena, dtype, tables, contexts, q, q_heads,
                                 threads, tile_tokens=16):
    """The reference's CPU paged decode step over a batch, on `threads` host threads.

    Per sequence: gather the pages (PagedKvPool::materialize,
    worker/cpp/inferlab_runtime.cpp:769-803) and call the reference's
    inferlab_attention_forward (OnlineTiled) once per q-head on its kv-head
    slice. One task per sequence when there are at least as many sequences as
    threads, else one task per (sequence, q-head) call.
    ctypes releases the GIL during the call, so the pool runs in parallel.
    Returns the output [num_seqs][q_heads][head_dim].
    """
    lib = ref_lib()
    if lib is None:
        raise OracleError("reference library is not built")
    nb, kvh, bt, hd = k_arena.shape
    group = q_heads // kvh
    out = np.zeros((len(contexts), q_heads, hd), dtype=np.float32)
    config = InferlabAttentionConfig(ONLINE_TILED, FP32, tile_tokens, 1)

    def widen(blocks):
        if dtype == FP32:
            return blocks.astype(np.float32, copy=False)
        if dtype == FP16:
            return blocks.view(np.float16).astype(np.float32)
        return (blocks.astype(np.uint32) << 16).view(np.float32)

    def gather(s):
        ctx = int(contexts[s])
        nblk = (ctx + bt - 1) // bt
        ids = tables[s, :nblk]
        kk = widen(k_arena[ids])  # [nblk][kvh][bt][hd]
        vv = widen(v_arena[ids])
        kk = np.ascontiguousarray(kk.transpose(1, 0, 2, 3).reshape(kvh, nblk * bt, hd)[:, :ctx])
        vv = np.ascontiguousarray(vv.transpose(1, 0, 2, 3).reshape(kvh, nblk * bt, hd)[:, :ctx])
        return kk, vv

    def head(task, kv=None):
        s, h = divmod(task, q_heads)
        ctx = int(contexts[s])
        kk, vv = pages[s] if kv is None else kv
        kh = kk[h // group]
        vh = vv[h // group]
        qh = np.ascontiguousarray(q[s, h])
        oh = np.zeros(hd, dtype=np.float32)
        err = ctypes.create_string_buffer(512)
        stats = InferlabAttentionStats()
        status = lib.inferlab_attention_forward(
            _ptr(qh, ctypes.c_float), _ptr(kh, ctypes.c_float), _ptr(vh, ctypes.c_float),
            1, ctx, 1, hd, ctx - 1, ctypes.byref(config), _ptr(oh, ctypes.c_float), hd,
            ctypes.byref(stats), err, 512)
        if status != 0:
            raise OracleError(err.value.decode())
        out[s, h] = oh

    def sequence(s):
        kv = gather(s)
        for h in range(q_heads):
            head(s * q_heads + h, kv)

    with ThreadPoolExecutor(max_workers=max(1, threads)) as pool:
        if len(contexts) >= threads:
            # enough sequences to occupy every thread: one task per sequence
            list(pool.map(sequence, range(len(contexts))))
        else:
            # few long sequences: pages first, then every (sequence, q-head)
            # call as its own task, so that every thread has work
            pages = list(pool.map(gather, range(len(contexts))))
            list(pool.map(head, range(len(contexts) * q_heads)))
    return out

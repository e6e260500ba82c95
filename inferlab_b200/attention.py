"""Host-side mirror of the reference's attention facade over the CUDA library.

run_attention() follows worker/src/lib.rs:743-819 (the safe wrapper the
worker and its probe binaries call): the same validation order and messages,
then the C entry inferlab_attention_forward, then the stats copied out. The
difference is underneath: the C entry here is libinferlab_attention_cuda.so,
which runs the attention on the GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from enum import IntEnum

import numpy as np

from . import _lib


class AttentionAlgorithm(IntEnum):
    """kernels/attention_cpu.h:8-11."""

    MATERIALIZED = 0
    ONLINE_TILED = 1


class AttentionPrecision(IntEnum):
    """kernels/attention_cpu.h:13-17 (storage rounding of the inputs)."""

    FP32 = 0
    FP16 = 1
    BF16 = 2


@dataclass(frozen=True)
class AttentionConfig:
    """worker/src/lib.rs:480-515 (defaults from :488-497)."""

    algorithm: AttentionAlgorithm = AttentionAlgorithm.MATERIALIZED
    precision: AttentionPrecision = AttentionPrecision.FP32
    tile_tokens: int = 16
    causal: bool = True

    def validate(self) -> None:
        if self.tile_tokens == 0 or self.tile_tokens > 4096:
            raise AttentionError("attention tile_tokens must be between 1 and 4096")

    def raw(self) -> _lib.InferlabAttentionConfig:
        return _lib.InferlabAttentionConfig(int(self.algorithm), int(self.precision),
                                            int(self.tile_tokens), 1 if self.causal else 0)


@dataclass(frozen=True)
class AttentionStats:
    """worker/src/lib.rs:517-527."""

    score_elements: int
    masked_score_elements: int
    score_buffer_bytes: int
    working_set_bytes: int
    modeled_external_read_bytes: int
    modeled_external_write_bytes: int
    modeled_external_total_bytes: int
    key_tiles: int

    def as_dict(self) -> dict:
        return dict(self.__dict__)


@dataclass
class AttentionRun:
    """worker/src/lib.rs:529-533."""

    output: np.ndarray
    stats: AttentionStats


class AttentionError(RuntimeError):
    """An error string returned by the library (or by the facade's own checks)."""


def _as_f32(name: str, values) -> np.ndarray:
    array = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    return array


def run_attention(queries, keys, values, query_tokens: int, key_value_tokens: int, heads: int,
                  head_dimension: int, query_start_position: int,
                  config: AttentionConfig = AttentionConfig()) -> AttentionRun:
    """Scaled dot-product attention on [tokens][heads][head_dim] fp32 inputs.

    Validation mirrors worker/src/lib.rs:755-779; the computation runs on the
    current CUDA device through inferlab_attention_forward.
    """
    config.validate()
    if query_tokens == 0 or key_value_tokens == 0 or heads == 0 or head_dimension == 0:
        raise AttentionError("attention dimensions must be positive")
    token_width = heads * head_dimension
    query_values = query_tokens * token_width
    key_value_values = key_value_tokens * token_width
    if max(query_values, key_value_values) >= 2**63:
        raise AttentionError("attention KV shape overflows")
    q = _as_f32("queries", queries)
    k = _as_f32("keys", keys)
    v = _as_f32("values", values)
    if q.size != query_values or k.size != key_value_values or v.size != key_value_values:
        raise AttentionError("attention input lengths do not match their declared shapes")
    if config.causal and (query_start_position >= key_value_tokens
                          or query_tokens > key_value_tokens - query_start_position):
        raise AttentionError("causal query positions exceed the KV sequence")
    output = np.zeros(query_values, dtype=np.float32)
    raw_stats = _lib.InferlabAttentionStats()
    raw_config = config.raw()
    error = _lib.error_buffer()
    f32 = ctypes.POINTER(ctypes.c_float)
    status = _lib.lib().inferlab_attention_forward(
        q.ctypes.data_as(f32), k.ctypes.data_as(f32), v.ctypes.data_as(f32), query_tokens,
        key_value_tokens, heads, head_dimension, query_start_position, ctypes.byref(raw_config),
        output.ctypes.data_as(f32), output.size, ctypes.byref(raw_stats), error, len(error))
    if status != 0:
        raise AttentionError(error.value.decode())
    stats = AttentionStats(*(int(getattr(raw_stats, name)) for name, _ in raw_stats._fields_))
    return AttentionRun(output=output, stats=stats)

"""Loads libinferlab_attention_cuda.so and declares its C ABI (include/inferlab_attention.h).

The library is the product: there is no other implementation behind this
package. If it has not been built, importing fails with an error that says
how to build it (python -m inferlab_b200.build).
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIBPATH = os.path.join(HERE, "lib", "libinferlab_attention_cuda.so")

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

c_f32p = ctypes.POINTER(ctypes.c_float)
c_i32p = ctypes.POINTER(ctypes.c_int32)
c_sz = ctypes.c_size_t
c_vp = ctypes.c_void_p
c_err = ctypes.c_char_p


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


class InferlabCudaPoolInfo(ctypes.Structure):
    _fields_ = [
        ("device", ctypes.c_int32),
        ("dtype", ctypes.c_uint32),
        ("block_tokens", ctypes.c_uint32),
        ("kv_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32),
        ("element_bytes", ctypes.c_uint32),
        ("num_blocks", ctypes.c_uint64),
        ("block_bytes", ctypes.c_uint64),
        ("arena_bytes", ctypes.c_uint64),
        ("key_arena", ctypes.c_void_p),
        ("value_arena", ctypes.c_void_p),
    ]


class InferlabPagedCacheStats(ctypes.Structure):
    """worker/cpp/inferlab_runtime.h:7-31."""

    _fields_ = [(name, ctypes.c_uint64) for name in (
        "page_tokens", "page_count", "prefix_capacity", "page_bytes", "capacity_bytes",
        "allocated_pages", "free_pages", "used_token_slots", "allocated_token_slots",
        "internal_fragmentation_bytes", "live_references", "shared_pages", "maximum_refcount",
        "logical_referenced_bytes", "physical_used_bytes", "bytes_saved_by_sharing",
        "prefix_entries", "prefix_hits", "prefix_misses", "prefix_tokens_reused",
        "copy_on_write_copies", "evictions", "allocation_failures")]


c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_u64p = ctypes.POINTER(ctypes.c_uint64)

# name -> (restype, argtypes)
SIGNATURES = {
    "inferlab_attention_forward": (ctypes.c_int, [
        c_f32p, c_f32p, c_f32p, c_sz, c_sz, c_sz, c_sz, c_sz,
        ctypes.POINTER(InferlabAttentionConfig), c_f32p, c_sz,
        ctypes.POINTER(InferlabAttentionStats), c_err, c_sz]),
    "inferlab_cuda_pool_create": (ctypes.c_int, [
        ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.c_uint32, ctypes.POINTER(c_vp), c_err, c_sz]),
    "inferlab_cuda_pool_destroy": (None, [c_vp]),
    "inferlab_cuda_peer_buffer_bytes": (ctypes.c_uint64, [ctypes.c_uint32, ctypes.c_uint64,
                                                          ctypes.c_uint32]),
    "inferlab_cuda_peer_buffer_alloc": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_uint64, ctypes.POINTER(c_vp), c_vp, c_err, c_sz]),
    "inferlab_cuda_peer_buffer_free": (ctypes.c_int, [ctypes.c_int, c_vp, c_err, c_sz]),
    "inferlab_cuda_peer_exchange_create": (ctypes.c_int, [
        ctypes.c_int, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, c_vp,
        c_vp, ctypes.POINTER(c_vp), c_err, c_sz]),
    "inferlab_cuda_peer_exchange_combine": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_peer_exchange_synchronize": (ctypes.c_int, [
        c_vp, c_vp, ctypes.c_uint32, c_err, c_sz]),
    "inferlab_cuda_peer_exchange_destroy": (None, [c_vp]),
    "inferlab_cuda_paged_decode_exchange": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_sz, c_vp, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_pool_info": (ctypes.c_int, [
        c_vp, ctypes.POINTER(InferlabCudaPoolInfo), c_err, c_sz]),
    "inferlab_cuda_pool_synchronize": (ctypes.c_int, [c_vp, c_vp, ctypes.c_uint32, c_err, c_sz]),
    "inferlab_cuda_kv_append": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint64, c_vp, ctypes.c_uint32,
        c_vp, c_err, c_sz]),
    "inferlab_cuda_kv_gather": (ctypes.c_int, [
        c_vp, c_vp, ctypes.c_uint64, c_vp, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_paged_decode_workspace_size": (c_sz, [
        c_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]),
    "inferlab_cuda_paged_decode_workspace_init": (ctypes.c_int, [c_vp, c_sz, c_vp, c_err, c_sz]),
    "inferlab_cuda_pool_set_decode_split": (ctypes.c_int, [c_vp, ctypes.c_uint32, c_err, c_sz]),
    "inferlab_cuda_paged_decode": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_vp, c_sz, c_vp, c_err, c_sz]),
    "inferlab_cuda_paged_decode_noalloc": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_vp, c_err, c_sz]),
    # host-array pointers passed as plain addresses (the per-step call path)
    "inferlab_cuda_decode_step_host": (ctypes.c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, c_err, c_sz]),
    "inferlab_cuda_qkv_project_append": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_vp,
        ctypes.c_uint32, ctypes.c_uint32, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_output_project": (ctypes.c_int, [
        c_vp, c_vp, ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_decode_step_host_cow": (ctypes.c_int, [
        c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_vp, ctypes.c_uint32, c_err, c_sz]),
    "inferlab_cuda_paged_decode_partials": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, ctypes.c_uint32,
        ctypes.c_uint32, c_vp, c_vp, c_vp, c_vp, c_sz, c_vp, c_err, c_sz]),
    "inferlab_cuda_lse_combine": (ctypes.c_int, [
        c_vp, c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, c_vp, c_vp, c_err,
        c_sz]),
    "inferlab_cuda_lse_combine_packed": (ctypes.c_int, [
        c_vp, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_paged_prefill": (ctypes.c_int, [
        c_vp, c_vp, ctypes.c_uint32, c_vp, ctypes.c_uint32, c_vp, c_vp, c_vp, ctypes.c_uint32,
        ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64, c_vp, c_vp, c_err, c_sz]),
    "inferlab_cuda_pages_create": (ctypes.c_int, [
        ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(c_vp),
        c_err, c_sz]),
    "inferlab_cuda_pages_destroy": (None, [c_vp]),
    "inferlab_cuda_pages_prepare_append": (ctypes.c_int, [
        c_vp, c_i32p, ctypes.c_uint32, c_u32p, ctypes.c_uint64, c_i32p, c_i32p, c_err, c_sz]),
    "inferlab_cuda_pages_release": (ctypes.c_int, [c_vp, c_i32p, ctypes.c_uint32, c_err, c_sz]),
    "inferlab_cuda_pages_publish_prefix": (ctypes.c_int, [
        c_vp, c_u32p, ctypes.c_uint64, c_i32p, ctypes.c_uint32, ctypes.c_uint64, c_err, c_sz]),
    "inferlab_cuda_pages_acquire_prefix": (ctypes.c_int, [
        c_vp, c_u32p, ctypes.c_uint64, c_i32p, ctypes.c_uint32, c_u32p, c_u64p, c_err, c_sz]),
    "inferlab_cuda_pages_shared": (ctypes.c_int, [
        c_vp, c_i32p, ctypes.c_uint32, c_u64p, c_err, c_sz]),
    "inferlab_cuda_pages_stats": (ctypes.c_int, [
        c_vp, ctypes.POINTER(InferlabPagedCacheStats), c_err, c_sz]),
    "inferlab_cuda_pages_copy": (ctypes.c_int, [
        c_vp, c_i32p, c_i32p, ctypes.c_uint32, c_vp, c_err, c_sz]),
    "inferlab_cuda_version": (ctypes.c_char_p, []),
}


class LibraryNotBuilt(ImportError):
    pass


def lib() -> ctypes.CDLL:
    """The loaded CUDA library (raises LibraryNotBuilt when it is missing)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIBPATH):
                raise LibraryNotBuilt(
                    f"{LIBPATH} is missing: build the CUDA library with "
                    "`python -m inferlab_b200.build` (nvcc, sm_100a)")
            handle = ctypes.CDLL(LIBPATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def error_buffer(size: int = 512):
    """Same 512-byte error buffer the Rust facade passes (worker/src/lib.rs:40)."""
    return ctypes.create_string_buffer(size)

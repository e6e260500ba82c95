"""CPU checks of the CUDA library: it loads, exports every entry point the
headers declare, and its host-side validation (which runs before any CUDA
call) returns the reference's status codes and messages.

Validation order and messages: worker/cpp/inferlab_runtime.cpp:2577-2593,
the config mapping at :446-490, kernels/attention_cpu.cpp:432-447, and the
Rust facade's own checks at worker/src/lib.rs:755-779.
"""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_c_functions():
    with open(os.path.join(ROOT, "include", "inferlab_attention.h")) as handle:
        text = handle.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(inferlab_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from inferlab_b200 import _lib

    lib = _lib.lib()
    declared = declared_c_functions()
    assert "inferlab_attention_forward" in declared
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.SIGNATURES)
    # C++ API of include/attention_cuda.h (kernels/attention_cpu.h:37-51)
    out = subprocess.run(["nm", "-DC", "--defined-only", _lib.LIBPATH], capture_output=True,
                         text=True, check=True).stdout
    assert "inferlab::attention_forward(" in out
    assert "inferlab::round_attention_value(" in out


def test_library_is_sm100a_and_names_no_multicast():
    from inferlab_b200 import _lib

    assert _lib.lib().inferlab_cuda_version() == b"inferlab-b200 0.1 sm_100a"
    csrc = os.path.join(ROOT, "inferlab_b200", "csrc")
    # the qualifier is assembled here so this test file itself does not carry it
    qualifier = ".".join(["", "multicast"]) + "::" + "cluster"
    for name in os.listdir(csrc):
        if name.endswith((".cu", ".cuh")):
            with open(os.path.join(csrc, name)) as handle:
                assert qualifier not in handle.read(), name


def _call(q, k, v, tq, tkv, heads, dim, start, config, out, out_cap, stats=True):
    from inferlab_b200 import _lib

    f32 = ctypes.POINTER(ctypes.c_float)
    raw_stats = _lib.InferlabAttentionStats()
    err = ctypes.create_string_buffer(512)
    err.value = b"stale"

    def ptr(a):
        return None if a is None else a.ctypes.data_as(f32)

    status = _lib.lib().inferlab_attention_forward(
        ptr(q), ptr(k), ptr(v), tq, tkv, heads, dim, start,
        ctypes.byref(config) if config is not None else None, ptr(out), out_cap,
        ctypes.byref(raw_stats) if stats else None, err, 512)
    return status, err.value.decode()


def _cfg(algorithm=0, precision=0, tile=16, causal=1):
    from inferlab_b200 import _lib

    return _lib.InferlabAttentionConfig(algorithm, precision, tile, causal)


ABI_CASES = [
    (dict(config=None), "attention config or stats pointer is null"),
    (dict(stats=False), "attention config or stats pointer is null"),
    (dict(out_cap=3), "attention output buffer is too small"),
    (dict(out=None), "attention output buffer is too small"),
    (dict(tile=0), "attention tile_tokens must be between 1 and 4096"),
    (dict(tile=5000, algorithm=7), "attention tile_tokens must be between 1 and 4096"),
    (dict(algorithm=2), "attention algorithm must be 0 (materialized) or 1 (online tiled)"),
    (dict(precision=9), "attention precision must be 0 (FP32), 1 (FP16), or 2 (BF16)"),
    (dict(q=None), "attention input or output pointer is null"),
    (dict(heads=0, out_cap=0), "attention dimensions must be positive"),
    (dict(start=4), "causal query positions exceed the KV sequence"),
    (dict(tq=5, out_cap=5 * 8), "causal query positions exceed the KV sequence"),
]


@pytest.mark.parametrize("override,message", ABI_CASES)
def test_c_abi_validation_matches_reference(override, message, oracle_mod):
    tq, tkv, heads, dim, start = 2, 4, 2, 4, 0
    tq = override.get("tq", tq)
    heads = override.get("heads", heads)
    start = override.get("start", start)
    q = np.ones(max(1, tq * heads * dim), np.float32)
    k = np.ones(tkv * 2 * dim, np.float32)
    v = np.ones_like(k)
    out = np.zeros(max(1, tq * heads * dim), np.float32)
    config = None if "config" in override and override["config"] is None else _cfg(
        override.get("algorithm", 0), override.get("precision", 0), override.get("tile", 16))
    status, text = _call(None if "q" in override else q, k, v, tq, tkv, heads, dim, start, config,
                         None if "out" in override else out,
                         override.get("out_cap", out.size), override.get("stats", True))
    assert status == -1
    assert text == message
    # The reference build agrees, case for case.
    ref = oracle_mod.ref_lib()
    if ref is not None and "config" not in override and "stats" not in override:
        err = ctypes.create_string_buffer(512)
        f32 = ctypes.POINTER(ctypes.c_float)
        rs = oracle_mod.InferlabAttentionStats()
        rc = oracle_mod.InferlabAttentionConfig(override.get("algorithm", 0),
                                                override.get("precision", 0),
                                                override.get("tile", 16), 1)
        st = ref.inferlab_attention_forward(
            None if "q" in override else q.ctypes.data_as(f32), k.ctypes.data_as(f32),
            v.ctypes.data_as(f32), tq, tkv, heads, dim, start, ctypes.byref(rc),
            None if "out" in override else out.ctypes.data_as(f32),
            override.get("out_cap", out.size), ctypes.byref(rs), err, 512)
        assert st == -1 and err.value.decode() == message


def test_error_text_truncates_to_capacity():
    from inferlab_b200 import _lib

    err = ctypes.create_string_buffer(8)
    status = _lib.lib().inferlab_attention_forward(None, None, None, 1, 1, 1, 1, 0, None, None, 0,
                                                   None, err, 8)
    assert status == -1
    assert err.value == b"attenti"  # capacity 8 = 7 characters + NUL


def test_facade_validation_messages():
    """worker/src/lib.rs:755-779 checks, before the C call."""
    import inferlab_b200 as il

    with pytest.raises(il.AttentionError, match="tile_tokens must be between 1 and 4096"):
        il.run_attention([0.0], [0.0], [0.0], 1, 1, 1, 1, 0, il.AttentionConfig(tile_tokens=0))
    with pytest.raises(il.AttentionError, match="dimensions must be positive"):
        il.run_attention([], [], [], 0, 1, 1, 1, 0)
    with pytest.raises(il.AttentionError, match="do not match their declared shapes"):
        il.run_attention([0.0] * 3, [0.0] * 4, [0.0] * 4, 1, 1, 1, 4, 0)
    with pytest.raises(il.AttentionError, match="causal query positions exceed"):
        il.run_attention([0.0] * 8, [0.0] * 4, [0.0] * 4, 2, 1, 1, 4, 0)


def test_pool_api_rejects_bad_arguments_without_gpu():
    from inferlab_b200 import _lib

    lib = _lib.lib()
    err = ctypes.create_string_buffer(256)
    handle = ctypes.c_void_p()
    assert lib.inferlab_cuda_pool_create(0, 5, 16, 16, 8, 64, ctypes.byref(handle), err, 256) == -1
    assert err.value == b"paged KV dtype must be 0 (FP32), 1 (FP16), or 2 (BF16)"
    assert lib.inferlab_cuda_pool_create(0, 0, 0, 16, 8, 64, ctypes.byref(handle), err, 256) == -1
    assert err.value == b"paged KV cache dimensions must be positive"
    assert lib.inferlab_cuda_pool_create(0, 0, 1 << 31, 16, 8, 64, ctypes.byref(handle), err,
                                         256) == -1
    assert err.value == b"paged KV num_blocks must fit a 32-bit block id"
    assert lib.inferlab_cuda_pool_info(None, None, err, 256) == -1
    assert err.value == b"paged KV pool pointer is null"
    assert lib.inferlab_cuda_paged_decode(None, None, None, 1, None, 1, 1, 1, None, None, 0, None,
                                          err, 256) == -1
    assert err.value == b"paged KV pool pointer is null"
    assert lib.inferlab_cuda_lse_combine(None, None, None, 1, 1, 1, None, None, err, 256) == -1
    assert err.value == b"lse combine pointer is null"
    assert lib.inferlab_cuda_paged_decode_workspace_size(None, 1, 1, 1) == 0
    assert lib.inferlab_cuda_qkv_project_append(None, None, None, 1, 64, 1, None, None, None, 1, 1,
                                                None, None, err, 256) == -1
    assert err.value == b"paged KV pool pointer is null"
    assert lib.inferlab_cuda_decode_step_host_cow(None, None, None, None, None, None, 1, None, 1,
                                                  1, None, None, 0, err, 256) == -1
    assert err.value == b"paged KV pool pointer is null"
    lib.inferlab_cuda_pool_destroy(None)


def test_header_compiles_as_c_and_links(tmp_path):
    """include/inferlab_attention.h is plain C: a C11 program that includes it,
    links the library and calls entries whose host-side checks fail before any
    CUDA work gets the reference's status and messages (no GPU needed)."""
    from inferlab_b200 import _lib

    src = tmp_path / "main.c"
    src.write_text(r'''
#include "inferlab_attention.h"
#include <stdio.h>
#include <string.h>
int main(void) {
    char err[512];
    float q[4] = {0}, out[4] = {0};
    InferlabAttentionStats stats;
    int rc = inferlab_attention_forward(q, q, q, 1, 1, 1, 4, 0, NULL, out, 4, &stats, err,
                                        sizeof err);
    if (rc != -1 || strcmp(err, "attention config or stats pointer is null") != 0) {
        printf("forward: %d %s\n", rc, err);
        return 1;
    }
    InferlabCudaKvPool* pool = NULL;
    rc = inferlab_cuda_pool_create(0, 5, 16, 16, 8, 64, &pool, err, sizeof err);
    if (rc != -1 || pool != NULL) return 2;
    rc = inferlab_cuda_qkv_project_append(NULL, NULL, NULL, 1, 64, 1, NULL, NULL, NULL, 1, 1,
                                          NULL, NULL, err, sizeof err);
    if (rc != -1 || strcmp(err, "paged KV pool pointer is null") != 0) return 3;
    puts("ok");
    return 0;
}
''')
    exe = tmp_path / "main"
    libdir = os.path.dirname(_lib.LIBPATH)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I",
                    os.path.join(ROOT, "include"), str(src), "-o", str(exe), "-L", libdir,
                    "-linferlab_attention_cuda", f"-Wl,-rpath,{libdir}"], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "ok", (run.returncode, run.stdout)

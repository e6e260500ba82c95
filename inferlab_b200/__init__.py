"""inferlab_b200 - B200 (sm_100a) attention hot path for InferLab.

Drop-in for the reference's kernels/attention_cpu + paged KV cache:
  * run_attention: the worker's attention facade (worker/src/lib.rs:743-819)
    over the C entry inferlab_attention_forward, executed on the GPU;
  * CudaKvPool: the HBM block pool with append / gather / paged decode /
    paged prefill kernels that follow the reference's block tables;
  * PageManager: the block ownership model (reference counts, prefixes,
    copy on write, eviction, InferlabPagedCacheStats) kept on the host.
All compute is in libinferlab_attention_cuda.so (built by
`python -m inferlab_b200.build`); importing this package does not need a GPU,
calling it does.
"""
from .attention import (AttentionAlgorithm, AttentionConfig, AttentionError,  # noqa: F401
                        AttentionPrecision, AttentionRun, AttentionStats, run_attention)

__all__ = [
    "AttentionAlgorithm", "AttentionConfig", "AttentionError", "AttentionPrecision",
    "AttentionRun", "AttentionStats", "run_attention", "CudaKvPool", "lse_combine",
    "PageManager",
]


def __getattr__(name):
    # The pool API needs torch; load it lazily so the facade imports without it.
    if name in ("CudaKvPool", "lse_combine"):
        from . import paged

        return getattr(paged, name)
    if name == "PageManager":
        from . import pages

        return pages.PageManager
    raise AttributeError(name)

"""Build and load the in-tree sm_100a extension (`_bdh_cuda`).

The extension is compiled with nvcc for `sm_100a` only (tcgen05 / TMA / TMEM are
architecture-specific features) into ``burn_dragon_b200/csrc/build`` so the shared
object lives inside the repository tree. ``load()`` never silently falls back: the
caller gets the compiled module or an exception.
"""

from __future__ import annotations

import os
import threading

_LOCK = threading.Lock()
_MOD = None

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(CSRC, "build")

SOURCES = ["bindings.cpp", "gemm_host.cu", "gemm_inst_a.cu", "gemm_inst_b.cu", "gemm_inst_c.cu", "gemm_inst_d.cu", "gemm_inst_e.cu", "rowwise.cu", "noalloc_decoder.cu", "decode.cu", "scaffold.cu", "comm.cu", "gdpo.cu", "ssd_chunk.cu"]

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
]
if os.environ.get("BDH_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")


# Kernels launched by one call of each binding (for the bench's launch count).
_LAUNCHES_PER_CALL = {"grad_clip_coef": 2}


class _Counted:
    """Proxy over the extension module that counts kernel launches."""

    def __init__(self, mod):
        self._mod = mod
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        per = _LAUNCHES_PER_CALL.get(name, 1)

        def call(*args, **kwargs):
            self.launches += per
            return fn(*args, **kwargs)

        return call


def add_launches(n: int) -> None:
    """Account for kernels launched by replaying a captured CUDA graph."""
    if _MOD is not None:
        _MOD.launches += n


def launch_count() -> int:
    """Kernels of this package launched so far in this process."""
    return _MOD.launches if _MOD is not None else 0


def load(verbose: bool = False):
    """Compile (if stale) and import the extension. Thread-safe, cached."""
    global _MOD
    if _MOD is not None:
        return _MOD
    with _LOCK:
        if _MOD is not None:
            return _MOD
        # Pin the arch list so torch adds no -gencode flags of its own.
        os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
        from torch.utils.cpp_extension import load as _load

        os.makedirs(BUILD_DIR, exist_ok=True)
        raw = _load(
            name="_bdh_cuda",
            sources=[os.path.join(CSRC, s) for s in SOURCES],
            extra_cflags=["-O3", "-std=c++17"],
            extra_cuda_cflags=NVCC_FLAGS,
            extra_include_paths=[CSRC],
            build_directory=BUILD_DIR,
            verbose=verbose,
        )
        _MOD = _Counted(raw)
        return _MOD

"""Python front of the tcgen05 GEMM engine (``csrc/gemm_sm100.cuh``).

Each BDH contraction is expressed as one engine call: an operand is described by a
4-D geometry ``(inner, outer, outer_stride, z1, z2)`` of bf16 memory and a majorness
(K-major = the reduction index is contiguous; MN-major = the output row/column index
is contiguous), so every operand is read in place — no transposed copies in HBM.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from .. import _ext

EPI_BF16, EPI_F32, EPI_RELU_ROPE, EPI_SCORES, EPI_GATE, EPI_DEC_BWD, EPI_DQ, EPI_F32_SCATTER = range(8)


@dataclass(frozen=True)
class Operand:
    t: torch.Tensor
    mn: bool
    inner: int
    outer: int
    stride: int
    z1: tuple[int, int] | None = None  # (count, stride) or None when unused
    z2: tuple[int, int] | None = None

    def geom(self) -> list[int]:
        z1c, z1s = self.z1 if self.z1 else (1, 0)
        z2c, z2s = self.z2 if self.z2 else (1, 0)
        return [self.inner, self.outer, self.stride, z1c, z1s, z2c, z2s,
                int(self.z1 is not None), int(self.z2 is not None)]


_ERR: dict[int, torch.Tensor] = {}

# CTA-pair (cta_group::2) kernels for the MMA-bound contractions: on unless BDH_GEMM_PAIR=0.
PAIR = os.environ.get("BDH_GEMM_PAIR", "1") != "0"


# Bounds checks of data-dependent indices (token ids, CE targets) in the row kernels:
# DRAGON_DEBUG_BOUNDS=1 registers the device's error word with them, so an id outside the
# vocabulary is recorded (codes 201-203) and skipped instead of read out of bounds.
DEBUG_BOUNDS = os.environ.get("DRAGON_DEBUG_BOUNDS", "0") == "1"
BOUNDS_CODES = {201: "embedding gather: token id outside the table",
                202: "cross-entropy: target outside the vocabulary",
                203: "embedding gradient: token id outside the table"}


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 the kernels set when a bounded wait times out or (with
    DRAGON_DEBUG_BOUNDS=1) a bounds check fails (0 = healthy)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _ERR:
        _ERR[idx] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        if DEBUG_BOUNDS:
            set_debug_bounds(torch.device("cuda", idx), True)
    return _ERR[idx]


def set_debug_bounds(device: torch.device, on: bool) -> None:
    """Turn the row kernels' bounds checks on `device` on (reporting into its error word)
    or off."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    word = error_word(device) if on else None
    _ext.load().set_debug_bounds(idx, word)


def check_errors(device: torch.device) -> None:
    """Raise if any launch on `device` recorded a timeout or a failed bounds check
    (synchronizes)."""
    e = error_word(device)
    code = int(e.item())
    if code:
        e.zero_()
        if code in BOUNDS_CODES:
            raise IndexError(f"bounds check failed (code {code}): {BOUNDS_CODES[code]}")
        raise RuntimeError(f"tcgen05 GEMM engine reported a bounded-wait timeout (code {code})")


# Tile N of the TMA-epilogue modes (x-projection, gate, decoder backward, dQ): 128 runs
# the 1-CTA 128 x 128 kernel, 256 a CTA pair with 256 x 256 tiles and 16 epilogue warps
# (where M >= 256). Measured at BDH-GPU batch 32 (CUDA events): the pair's mainloop is
# about twice as fast, which pays for dQ (K = T = 512: 841 vs 895 us) but not for the
# K = 256 modes, whose epilogues bound both (x-projection 596 vs 587, gate 539 vs 476,
# decoder backward 1190 vs 880 us). ``BDH_TMA_BN`` = 128 / 256 forces one tile for all.
TMA_BN = os.environ.get("BDH_TMA_BN")
_TMA_BN_DEFAULT = {"dq": 256}


def tma_bn(M: int, N: int, mode: str = "") -> int:
    """Tile N for a TMA-epilogue GEMM of M x N outputs (per batch matrix)."""
    want = int(TMA_BN) if TMA_BN else _TMA_BN_DEFAULT.get(mode, 128)
    if want == 256 and PAIR and M >= 256 and N % 256 == 0:
        return 256
    return 128


def pick_bn(n: int) -> int:
    for bn in (256, 128, 64):
        if n % bn == 0:
            return bn
    return 64


def fit_splits(kb: int, want: int) -> int:
    """Largest split count <= want that the engine's even K partition reproduces."""
    want = max(1, min(want, kb))
    per = -(-kb // want)
    return -(-kb // per)


def gemm(epi: int, a: Operand, b: Operand, M: int, N: int, K: int, out0: torch.Tensor, *,
         Z1: int = 1, Z2: int = 1, bn: int | None = None, splits: int = 1, causal_skip: bool = False,
         out1=None, aux0=None, aux1=None, ld: int, sz1: int = 0, sz2: int = 0, split_stride: int = 0,
         alpha: float = 1.0, thr: float = 0.0, freq=None, log2_decay=None, T: int = 1, pos0: int = 0,
         Nh: int = 1, accumulate: bool = False, row_decay: bool = False, pair: bool | None = None,
         scatter: list[int] | None = None, acc_src: torch.Tensor | None = None, src_decay_T: int = 0,
         rope_tab: torch.Tensor | None = None) -> None:
    """``scatter`` (EPI_F32_SCATTER): [world, rows per owner, rank, slot stride, slot
    pointer of every rank] — rows go straight to their owner's slot over NVLink.

    EPI_F32 extras: ``out1`` a bf16 copy of the stored values; ``acc_src`` with
    ``accumulate``: out0 = alpha * acc + acc_src (* 2^(src_decay_T * log2_decay[z1]) when
    ``src_decay_T`` > 0) instead of adding out0's old contents.

    ``rope_tab`` (x-projection / dQ with ``freq``): the half2 (cos, sin) table of
    ``rope_table`` for this call's positions pos0 .. pos0 + T - 1. The x-projection
    stages its tiles through the epilogue's TMA ring; dQ reads it with plain loads."""
    mod = _ext.load()
    bn = bn or pick_bn(N)
    mod.gemm(epi, bn, a.t, a.mn, a.geom(), b.t, b.mn, b.geom(), M, N, K, Z1, Z2, splits, causal_skip,
             out0, out1, aux0, aux1, ld, sz1, sz2, split_stride, alpha, thr, freq, log2_decay, T, pos0, Nh,
             accumulate, row_decay, int(PAIR if pair is None else pair), error_word(out0.device), scatter,
             acc_src, src_decay_T, rope_tab)


def rope_table(freq: torch.Tensor, pos0: int, T: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """(cos, sin) half2 pairs of the RoPE phases for positions pos0 .. pos0 + T - 1 and the
    latent pairs of ``freq`` ([T, Nh / 2] int32), the table the epilogues read."""
    if out is None:
        out = torch.empty(T, freq.numel() // 2, dtype=torch.int32, device=freq.device)
    _ext.load().rope_table(freq, pos0, T, out)
    return out


def matmul(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.float32, a_t: bool = False,
           b_t: bool = False) -> torch.Tensor:
    """C = op(a) @ op(b) for 2-D bf16 tensors on the engine (op = transpose if *_t).

    a is [M,K] (or [K,M] with a_t), b is [K,N] (or [N,K] with b_t). Used by tests and
    small contractions; the BDH stack calls ``gemm`` directly.
    """
    assert a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
    a = a.contiguous()
    b = b.contiguous()
    if a_t:
        K, M = a.shape
        A = Operand(a, True, M, K, M)
    else:
        M, K = a.shape
        A = Operand(a, False, K, M, K)
    if b_t:
        N, K2 = b.shape
        B = Operand(b, False, K2, N, K2)
    else:
        K2, N = b.shape
        B = Operand(b, True, N, K2, N)
    assert K2 == K
    out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    gemm(EPI_F32 if out_dtype == torch.float32 else EPI_BF16, A, B, M, N, K, out, ld=N)
    return out

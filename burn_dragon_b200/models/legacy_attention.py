"""Block patterns and the legacy row-normalised causal attention with a KV cache.

* ``BlockPattern1d``: latent-axis block mask (all blocks active = dense). In the BDH
  layer an inactive latent block zeroes those x and y neurons (the reference
  multiplies both projections by the mask; kernel/block_sparse.rs:13-60).
* ``BlockPattern2d``: (query block, key block) pairs for block-sparse time attention;
  dense = every causal block pair (block_sparse.rs:62-110).
* ``row_normalized_attention``: ``S = tril(QK^T, -1) (+ ALiBi slope*(j-i))``, rows
  divided by ``sum|S| + 1e-6``, then ``S V`` (model/attention.rs:304-335,482-486), with
  the time pattern restricting which key blocks a query block sees (the reference's
  block-tiled form, kernel/linear_attention.rs:11-107). The ALiBi bias is applied
  strictly below the diagonal in both forms here (the reference's tiled form also
  adds it above the diagonal of diagonal blocks).
* ``AttentionCache`` / ``forward_cached``: incremental decoding that keeps the rotated
  keys and values of earlier tokens (attention.rs:363-480).

This path is superseded by the linear-attention recurrence for training and decode;
it is kept for models and checkpoints that use it.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import reference as R

ROW_NORM_EPS = 1e-6


@dataclass
class BlockPattern1d:
    block_size: int = 64
    active_blocks: set[int] | None = None

    def is_sparse(self) -> bool:
        return self.active_blocks is not None

    def is_block_active(self, b: int) -> bool:
        return self.active_blocks is None or b in self.active_blocks

    def mask(self, elements: int, device=None, dtype=torch.float32) -> torch.Tensor:
        bs = max(self.block_size, 1)
        idx = torch.arange(elements) // bs
        keep = torch.tensor([self.is_block_active(int(b)) for b in idx], dtype=dtype)
        return keep.to(device)


@dataclass
class BlockPattern2d:
    block_size: int = 64
    active_pairs: set[tuple[int, int]] | None = None

    def is_sparse(self) -> bool:
        return self.active_pairs is not None

    def is_active(self, row: int, col: int) -> bool:
        return col <= row if self.active_pairs is None else (row, col) in self.active_pairs

    def element_mask(self, time: int, device=None) -> torch.Tensor:
        """[T, T] 0/1 mask of the key positions each query may see (block level)."""
        bs = max(self.block_size, 1)
        nb = -(-time // bs)
        blk = torch.tensor([[self.is_active(r, c) for c in range(nb)] for r in range(nb)], dtype=torch.float32)
        return blk.repeat_interleave(bs, 0).repeat_interleave(bs, 1)[:time, :time].to(device)


def _rotate(x, cfg_rot: str, freqs, start: int):
    if cfg_rot == "alibi" or freqs is None:
        return x
    T = x.shape[2]
    ph = R.rope_phases(torch.arange(start, start + T, device=x.device), freqs)[None, None]
    return R.pope_apply(x, ph) if cfg_rot == "pope" else R.rope_apply(x, ph)


def _alibi(slopes, rows: torch.Tensor, cols: torch.Tensor):
    """slope_h * (col - row) as [1, H, R, C]."""
    return slopes.view(1, -1, 1, 1) * (cols.view(1, 1, 1, -1) - rows.view(1, 1, -1, 1)).to(slopes.dtype)


def row_normalized_attention(q, v, rotary: str = "rope", freqs=None, alibi_slopes=None,
                             time_pattern: BlockPattern2d | None = None):
    """q [B,H,T,N], v [B,1|H,T,D] -> [B,H,T,D]."""
    B, H, T, _ = q.shape
    qr = _rotate(q, rotary, freqs, 0)
    s = torch.tril(qr @ qr.transpose(-1, -2), -1)
    pos = torch.arange(T, device=q.device)
    if alibi_slopes is not None:
        s = s + torch.tril(_alibi(alibi_slopes, pos, pos).expand(B, H, T, T), -1)
    if time_pattern is not None:
        s = s * time_pattern.element_mask(T, q.device)
    s = s / (s.abs().sum(-1, keepdim=True) + ROW_NORM_EPS)
    return s @ v.expand(B, H, T, v.shape[-1])


@dataclass
class AttentionCache:
    q_rot: torch.Tensor | None = None  # [B,H,P,N]
    value: torch.Tensor | None = None  # [B,H,P,D]

    def __len__(self) -> int:
        return 0 if self.q_rot is None else self.q_rot.shape[2]

    def append(self, k_rot, v) -> None:
        self.q_rot = k_rot if self.q_rot is None else torch.cat([self.q_rot, k_rot], 2)
        self.value = v if self.value is None else torch.cat([self.value, v], 2)


def forward_cached(q, v, cache: AttentionCache, rotary: str = "rope", freqs=None, alibi_slopes=None):
    """Attention of new tokens over the cached prefix plus themselves (strictly causal)."""
    B, H, Tn, _ = q.shape
    P = len(cache)
    qr = _rotate(q, rotary, freqs, P)
    vr = v.expand(B, H, Tn, v.shape[-1])
    rows = torch.arange(P, P + Tn, device=q.device)
    self_s = torch.tril(qr @ qr.transpose(-1, -2), -1)
    if alibi_slopes is not None:
        self_s = self_s + torch.tril(_alibi(alibi_slopes, rows, rows).expand(B, H, Tn, Tn), -1)
    if P:
        prev = qr @ cache.q_rot.transpose(-1, -2)
        if alibi_slopes is not None:
            prev = prev + _alibi(alibi_slopes, rows, torch.arange(P, device=q.device))
        s = torch.cat([prev, self_s], -1)
        vals = torch.cat([cache.value, vr], 2)
    else:
        s, vals = self_s, vr
    s = s / (s.abs().sum(-1, keepdim=True) + ROW_NORM_EPS)
    cache.append(qr, vr)
    return s @ vals

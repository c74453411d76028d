"""Recurrent model state (burn_dragon_core/src/model/state.rs).

Each layer carries the linear-attention state rho [B, H, Nh, D]; ``position`` is the
absolute position of the next token (the RoPE phase origin). ``detach_in_place`` is the
TBPTT boundary; ``repeat_batch`` broadcasts a prompt state to a batch.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class ModelState:
    rhos: list[torch.Tensor] | None = None
    position: int = 0

    @staticmethod
    def empty() -> "ModelState":
        return ModelState(None, 0)

    def detach_in_place(self) -> None:
        if self.rhos is not None:
            self.rhos = [r.detach() for r in self.rhos]

    def reset(self) -> None:
        self.rhos = None
        self.position = 0

    def repeat_batch(self, n: int) -> "ModelState":
        rhos = None if self.rhos is None else [r.repeat(n, 1, 1, 1) for r in self.rhos]
        return ModelState(rhos, self.position)

    def select(self, mask: torch.Tensor) -> None:
        """Zero the state of the streams where ``mask`` is True (document boundaries)."""
        if self.rhos is None:
            return
        keep = (~mask).to(self.rhos[0].dtype).view(-1, 1, 1, 1)
        self.rhos = [r * keep for r in self.rhos]

    def to_dict(self) -> dict:
        return {"position": self.position,
                "rhos": None if self.rhos is None else [r.detach().cpu() for r in self.rhos]}

    @staticmethod
    def from_dict(d: dict, device=None) -> "ModelState":
        rhos = d.get("rhos")
        if rhos is not None:
            rhos = [r.to(device) for r in rhos]
        return ModelState(rhos, int(d.get("position", 0)))

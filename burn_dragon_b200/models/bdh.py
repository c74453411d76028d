"""BDH (Dragon Hatchling) language model with shared layer weights.

Parameters live in one flat fp32 master buffer (``ParamStore``) so the optimizer, the
gradient all-reduce and the bf16 GEMM shadow each touch one contiguous allocation; the
``nn.Parameter`` objects are views into it. Names and shapes follow the reference's
record paths (burn_dragon_core/src/model/dragon.rs:203-272, 711-754): ``embed.weight``
[V, D], ``encoder`` [H, D, Nh], ``encoder_v`` [H, D, Nh], ``decoder`` [N, D], ``lm_head``
[D, V], ``norm.gamma`` / ``norm.beta`` [D].

Two execution paths share these parameters:
* ``forward`` — the PyTorch statement of the math (``models.reference``), with autograd.
  This is the CPU path and the oracle.
* ``fused_step`` — forward + cross-entropy + backward on the sm_100a kernels
  (``models.bdh_fused``). On a CUDA device it is the training path; it raises if the
  extension cannot be loaded (no silent fallback).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..config import DragonConfig
from . import reference as R

PARAM_ORDER = ("encoder", "encoder_v", "decoder", "embed", "lm_head", "norm_gamma", "norm_beta")
RECORD_NAMES = {
    "encoder": "encoder",
    "encoder_v": "encoder_v",
    "decoder": "decoder",
    "embed": "embed.weight",
    "lm_head": "lm_head",
    "norm_gamma": "norm.gamma",
    "norm_beta": "norm.beta",
}


def param_shapes(cfg: DragonConfig) -> dict[str, tuple[int, ...]]:
    D, H, Nh, V = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.vocab_size
    shapes = {
        "encoder": (H, D, Nh),
        "encoder_v": (H, D, Nh),
        "decoder": (H * Nh, D),
        "embed": (V, D),
        "lm_head": (D, V),
        "norm_gamma": (D,),
        "norm_beta": (D,),
    }
    if cfg.tie_input_output_embeddings:
        del shapes["lm_head"]
    return shapes


class ParamStore:
    """Flat fp32 master buffer + flat grad buffer + flat bf16 shadow, with named views."""

    ALIGN = 64  # elements: keeps every view 256-byte aligned in fp32 and 128-byte in bf16

    def __init__(self, shapes: dict[str, tuple[int, ...]], device, with_shadow: bool):
        self.shapes = dict(shapes)
        self.offsets: dict[str, int] = {}
        off = 0
        for name, shp in shapes.items():
            self.offsets[name] = off
            n = math.prod(shp)
            off += -(-n // self.ALIGN) * self.ALIGN
        self.numel = off
        self.data = torch.zeros(off, dtype=torch.float32, device=device)
        self.grad = torch.zeros(off, dtype=torch.float32, device=device)
        self.shadow = torch.zeros(off, dtype=torch.bfloat16, device=device) if with_shadow else None

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        o = self.offsets[name]
        shp = self.shapes[name]
        return buf[o:o + math.prod(shp)].view(shp)

    def views(self, buf: torch.Tensor) -> dict[str, torch.Tensor]:
        return {n: self.view(buf, n) for n in self.shapes}

    def refresh_shadow(self) -> None:
        if self.shadow is not None:
            self.shadow.copy_(self.data)


class BDH(nn.Module):
    def __init__(self, cfg: DragonConfig, device=None, seed: int | None = None):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        device = torch.device(device) if device is not None else torch.device("cpu")
        self.store = ParamStore(param_shapes(cfg), device, with_shadow=device.type == "cuda")
        gen = torch.Generator(device="cpu")
        gen.manual_seed(1337 if seed is None else seed)
        self._init_weights(gen)
        for name in self.store.shapes:
            p = nn.Parameter(self.store.view(self.store.data, name))
            p.grad = self.store.view(self.store.grad, name)
            self.register_parameter(name, p)
        self.store.refresh_shadow()
        self._fused = None

    # SimpleNormal(0.02) for every projection and the embedding, LayerNorm gamma=1,
    # beta=0 (burn_dragon_core/src/model/init.rs:10,448-520,593-650).
    def _init_weights(self, gen: torch.Generator) -> None:
        std = self.cfg.init_std
        for name, shp in self.store.shapes.items():
            view = self.store.view(self.store.data, name)
            if name == "norm_gamma":
                view.fill_(1.0)
            elif name == "norm_beta":
                view.zero_()
            else:
                view.copy_(torch.randn(shp, generator=gen, dtype=torch.float32) * std)

    # ---------------------------------------------------------------- helpers
    def param_dict(self) -> dict[str, torch.Tensor]:
        d = {n: getattr(self, n) for n in self.store.shapes}
        if "lm_head" not in d:
            d["lm_head"] = None
        return d

    def shadow_dict(self) -> dict[str, torch.Tensor]:
        assert self.store.shadow is not None
        return self.store.views(self.store.shadow)

    def grad_dict(self) -> dict[str, torch.Tensor]:
        return self.store.views(self.store.grad)

    def num_params(self) -> int:
        return sum(math.prod(s) for s in self.store.shapes.values())

    # ---------------------------------------------------------------- reference path
    def forward(self, tokens: torch.Tensor, state=None, need_state: bool = False):
        """Logits [B, T, V] through the PyTorch path. ``state`` is a ``ModelState``."""
        rho0s = state.rhos if state is not None and state.rhos is not None else None
        pos0 = state.position if state is not None else 0
        logits, rhos = R.bdh_forward(tokens, self.param_dict(), self.cfg, rho0s=rho0s, pos0=pos0,
                                     need_state=need_state or state is not None, training=self.training)
        if state is not None:
            state.rhos = rhos
            state.position += tokens.shape[1]
        return logits

    def loss(self, tokens: torch.Tensor, targets: torch.Tensor, mask=None, state=None) -> torch.Tensor:
        return R.cross_entropy(self.forward(tokens, state=state), targets, mask)

    # ---------------------------------------------------------------- fused path
    def fused_step(self, tokens: torch.Tensor, targets: torch.Tensor, mask=None, state=None) -> torch.Tensor:
        """Forward + CE + backward on the sm_100a kernels. Writes ``.grad`` of every
        parameter (the flat grad buffer) and returns the loss as a device scalar.

        With a ``ModelState`` the chunk continues that state (stateful TBPTT: the state
        enters detached and leaves detached, burn_dragon_language/src/train/steps.rs:
        2698-2731) and the state is advanced in place."""
        from .bdh_fused import FusedBDH, FusedWorkspace

        B, T = tokens.shape
        if self._fused is None or self._fused.ws.B != B or self._fused.ws.T != T:
            self._fused = None
            torch.cuda.empty_cache()
            self._fused = FusedBDH(self.cfg, FusedWorkspace(self.cfg, B, T, tokens.device))
        f = self._fused
        p32 = self.store.views(self.store.data)
        p16 = self.shadow_dict()
        pos0 = state.position if state is not None else 0
        rho0s = state.rhos if state is not None else None
        outs = f.forward(p16, p32, tokens, pos0=pos0, rho0s=rho0s, want_state=state is not None)
        loss = f.loss(targets, mask)
        f.backward(p16, p32, self.grad_dict(), tokens, pos0=pos0)
        if state is not None:
            state.rhos = outs
            state.position += T
        return loss

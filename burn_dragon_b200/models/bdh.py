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

import copy
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
    "norm_alpha": "norm.alpha",
    "norm_shift": "norm.shift",
}


SCAFFOLD_RECORD = "random_scaffold_adapters.fast"


def param_shapes(cfg: DragonConfig) -> dict[str, tuple[int, ...]]:
    D, H, Nh, V = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.vocab_size
    if cfg.random_scaffold.enabled:
        from .scaffold import adapter_shapes

        shapes = {}
        for k, shp in adapter_shapes(cfg).items():
            if k.endswith(".gain") and not cfg.random_scaffold.trainable_gain:
                continue
            shapes[k.replace(".", "_")] = shp
    else:
        shapes = {"encoder": (H, D, Nh), "encoder_v": (H, D, Nh), "decoder": (H * Nh, D)}
    shapes.update({"embed": (V, D), "lm_head": (D, V), "norm_gamma": (D,), "norm_beta": (D,),
                   "norm_alpha": (1,), "norm_shift": (1,)})
    if cfg.tie_input_output_embeddings:
        del shapes["lm_head"]
    if cfg.mhc_streams > 1:
        S, L = cfg.mhc_streams, cfg.n_layer
        shapes.update({"mhc_res": (L, S, S), "mhc_pre": (L, 1, S), "mhc_post": (L, 1, S)})
        if cfg.mhc_policy == "dynamic_positive":
            from .mhc import dynamic_shapes

            shapes.update(dynamic_shapes(L, S, D))
    return shapes


def record_name(name: str) -> str:
    """Reference record path of a parameter (scaffold adapters under
    ``random_scaffold_adapters.fast.<proj>.<a|b|gain>``)."""
    if name in RECORD_NAMES:
        return RECORD_NAMES[name]
    for proj in ("encoder_v", "encoder", "decoder"):
        if name.startswith(proj + "_"):
            return f"{SCAFFOLD_RECORD}.{proj}.{name[len(proj) + 1:]}"
    return name


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

    def rebind(self, data: torch.Tensor, grad: torch.Tensor, shadow: torch.Tensor | None) -> None:
        """Move the flat buffers into caller-owned memory (e.g. symmetric IPC memory);
        the new buffers may be longer than ``numel`` (the tail stays zero)."""
        with torch.no_grad():
            data[:self.numel].copy_(self.data)
            grad[:self.numel].copy_(self.grad)
            if shadow is not None:
                shadow[:self.numel].copy_(self.data)
        self.data, self.grad = data, grad
        self.shadow = shadow if shadow is not None else self.shadow


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
        self.tp = None  # parallel.tp.TensorParallel when this model holds a head shard
        self.scaffold = cfg.random_scaffold.enabled
        if self.scaffold:
            self._init_scaffold(device)

    # SimpleNormal(0.02) for every projection and the embedding, LayerNorm gamma=1,
    # beta=0 (burn_dragon_core/src/model/init.rs:10,448-520,593-650); scaffold adapters:
    # A from the scaffold generator, B = 0, gain = 1 (scaffold.rs:31-55).
    def _init_weights(self, gen: torch.Generator) -> None:
        from .init import init_param
        from .scaffold import PATHS, adapter_a_init

        cfg = self.cfg
        rs = cfg.random_scaffold
        for name, shp in self.store.shapes.items():
            view = self.store.view(self.store.data, name)
            if name.startswith("mhc_"):
                from .mhc import init_logits

                view.copy_(init_logits(cfg.n_layer, cfg.mhc_streams, dim=cfg.n_embd,
                                       dynamic=cfg.mhc_policy == "dynamic_positive")[name])
            elif name == "norm_gamma" or name.endswith("_gain"):
                view.fill_(1.0)
            elif name == "norm_alpha":
                view.fill_(cfg.norm_alpha())
            elif name == "norm_shift":
                view.fill_(cfg.norm_shift_init)
            elif name == "norm_beta" or name.endswith("_b"):
                view.zero_()
            elif name.endswith("_a") and rs.enabled:
                proj = name[:-2]
                fan_in = shp[-2]
                view.copy_(adapter_a_init(rs.seed, PATHS[proj], shp, fan_in))
            else:
                view.copy_(init_param(cfg, name, shp, gen))

    def _init_scaffold(self, device) -> None:
        """Frozen bases: kept on the host (CPU path) or regenerated by the device kernel."""
        from .scaffold import PATHS, base_shape, dist_code, scaffold_tensor_cpu, signed64, tensor_key

        rs = self.cfg.random_scaffold
        self.scaffold_keys = {n: signed64(tensor_key(rs.seed, PATHS[n])) for n in PATHS}
        self.scaffold_dist = dist_code(rs.distribution)
        self._bases: dict[str, torch.Tensor] = {}
        if device.type != "cuda":
            for n in PATHS:
                self._bases[n] = scaffold_tensor_cpu(rs.seed, PATHS[n], base_shape(self.cfg, n), self.cfg.init_std,
                                                     rs.distribution)
        self._eff16 = None
        self._geff = None
        self._scaffold_work = None
        # W_seed is generated from the seed on the device once and kept (fp32, 4 bytes per
        # frozen element); BDH_SCAFFOLD_CACHE_BASE=0 regenerates it in the fold and
        # gain-gradient kernels every step instead (no copy held, about 1.7 ms more per
        # BDH-GPU step: the generator's 24 64-bit mixes per element)
        import os as _os

        self.scaffold_cache_base = device.type == "cuda" and _os.environ.get("BDH_SCAFFOLD_CACHE_BASE", "1") == "1"

    def scaffold_base(self, name: str) -> torch.Tensor:
        """W_seed of a projection (fp32), regenerated on the device when needed."""
        if name not in self._bases:
            from .. import _ext
            from .scaffold import base_shape

            shp = base_shape(self.cfg, name)
            out = torch.empty(shp, device=self.store.data.device)
            rows = shp[0] * shp[1] if len(shp) == 3 else shp[0]
            _ext.load().scaffold_effective(self.scaffold_keys[name], self.cfg.init_std, self.scaffold_dist, rows,
                                           shp[-2] if len(shp) == 3 else rows, shp[-1], 0, None, None, None, 0.0,
                                           None, None, out, None)
            self._bases[name] = out
        return self._bases[name]

    def _scaffold_parts(self, name: str):
        a = getattr(self, f"{name}_a")
        b = getattr(self, f"{name}_b")
        g = getattr(self, f"{name}_gain") if self.cfg.random_scaffold.trainable_gain else \
            torch.ones(1, device=a.device, dtype=a.dtype)
        return a, b, g

    def __deepcopy__(self, memo):
        """A copy whose parameters are views of its own copied flat store (a plain deep
        copy would give them separate storage, and an optimizer stepping the copy's store
        would then miss them)."""
        new = self.__class__.__new__(self.__class__)
        memo[id(self)] = new
        for k, v in self.__dict__.items():
            new.__dict__[k] = copy.deepcopy(v, memo)
        st = new.store
        with torch.no_grad():
            for name in st.shapes:  # the copied parameters hold the current values
                st.view(st.data, name).copy_(getattr(self, name).detach())
        new.attach_buffers(st.data, st.grad, st.shadow)
        return new

    def attach_buffers(self, data: torch.Tensor, grad: torch.Tensor, shadow: torch.Tensor | None) -> None:
        """Re-home parameters, grads and the bf16 shadow (see ``ParamStore.rebind``)."""
        self.store.rebind(data, grad, shadow)
        for name in self.store.shapes:
            p = nn.Parameter(self.store.view(self.store.data, name))
            p.grad = self.store.view(self.store.grad, name)
            setattr(self, name, p)
        self._fused = None

    # ---------------------------------------------------------------- helpers
    def param_dict(self) -> dict[str, torch.Tensor]:
        """The BDH weights the math consumes (effective projections for scaffold runs)."""
        d = {n: getattr(self, n) for n in ("embed", "lm_head", "norm_gamma", "norm_beta", "norm_alpha", "norm_shift",
                                           "mhc_res", "mhc_pre", "mhc_post")
             if n in self.store.shapes}
        d.update({n: getattr(self, n) for n in self.store.shapes if n.startswith("mhc_")})
        if self.scaffold:
            from .scaffold import effective_weight

            for n in ("encoder", "encoder_v", "decoder"):
                a, b, g = self._scaffold_parts(n)
                d[n] = effective_weight(self.cfg, n, a, b, g, self.scaffold_base(n).to(a.dtype))
        else:
            for n in ("encoder", "encoder_v", "decoder"):
                d[n] = getattr(self, n)
        if "lm_head" not in d:
            d["lm_head"] = None
        return d

    def fold_scaffold_for_inference(self) -> "BDH":
        """Dense model with W = gain*W_seed + s*A@B folded in (dragon.rs:1126-1180)."""
        import copy

        cfg = copy.deepcopy(self.cfg)
        cfg.random_scaffold.enabled = False
        dense = BDH(cfg, device=self.store.data.device)
        with torch.no_grad():
            src = self.param_dict()
            for n in dense.store.shapes:
                getattr(dense, n).copy_(src[n].detach())
        dense.store.refresh_shadow()
        return dense

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

    # ---------------------------------------------------------------- scaffold (fused path)
    def _scaffold_prepare(self, p16: dict, g32: dict) -> None:
        """Fold gain*W_seed + s*A@B into bf16 GEMM operands (W_seed regenerated in the
        kernel, never stored) and point the projection grads at fp32 scratch buffers."""
        from .. import _ext
        from .scaffold import base_shape

        mod = _ext.load()
        dev = self.store.data.device
        if self._eff16 is None:
            self._eff16 = {n: torch.empty(base_shape(self.cfg, n), dtype=torch.bfloat16, device=dev)
                           for n in ("encoder", "encoder_v", "decoder")}
            self._geff = {n: torch.empty(base_shape(self.cfg, n), device=dev) for n in ("encoder", "encoder_v", "decoder")}
        s = self.cfg.random_scaffold.adapter_scale()
        r = self.cfg.random_scaffold.rank
        for n in ("encoder", "encoder_v", "decoder"):
            shp = base_shape(self.cfg, n)
            a, b, g = self._scaffold_parts(n)
            rows = shp[0] * shp[1] if len(shp) == 3 else shp[0]
            I = shp[1] if len(shp) == 3 else shp[0]
            base = self.scaffold_base(n) if self.scaffold_cache_base else None
            mod.scaffold_effective(self.scaffold_keys[n], self.cfg.init_std, self.scaffold_dist, rows, I, shp[-1], r,
                                   a.detach().reshape(rows, r), b.detach(), g.detach(), s, self._eff16[n], None, None,
                                   base)
            p16[n] = self._eff16[n]
            g32[n] = self._geff[n]

    def _scaffold_backward(self, g32: dict) -> None:
        """Adapter grads from d(W_eff), one pass over dW per projection on the device
        (``scaffold_adapter_grad``): dA = s dW B^T, dB = s A^T dW, dgain = sum(dW * W_seed)
        with W_seed regenerated from the seed (or read from the cached base)."""
        from .. import _ext
        from .scaffold import base_shape

        mod = _ext.load()
        s = self.cfg.random_scaffold.adapter_scale()
        r = self.cfg.random_scaffold.rank
        for n in ("encoder", "encoder_v", "decoder"):
            dW = self._geff[n]
            a, b, _ = self._scaffold_parts(n)
            shp = base_shape(self.cfg, n)
            Hm, I, O = (shp[0], shp[1], shp[2]) if len(shp) == 3 else (1, shp[0], shp[1])
            ga = self.store.view(self.store.grad, f"{n}_a")
            gb = self.store.view(self.store.grad, f"{n}_b")
            need = mod.scaffold_adapter_work(Hm, I, O, r)
            if self._scaffold_work is None or self._scaffold_work.numel() < need:
                self._scaffold_work = torch.empty(need, device=dW.device)
            gg = self.store.view(self.store.grad, f"{n}_gain") if self.cfg.random_scaffold.trainable_gain else None
            mod.scaffold_adapter_grad(self.scaffold_keys[n], self.cfg.init_std, self.scaffold_dist, Hm, I, O, r, dW,
                                      a.detach(), b.detach(), self.scaffold_base(n) if self.scaffold_cache_base else None,
                                      s, ga, gb, gg, self._scaffold_work)

    # ---------------------------------------------------------------- fused path
    def fused_step(self, tokens: torch.Tensor, targets: torch.Tensor, mask=None, state=None,
                   accumulate: bool = False, loss_scale: float = 1.0, grad_ready=None,
                   grad16: dict | None = None) -> torch.Tensor:
        """Forward + CE + backward on the sm_100a kernels. Writes ``.grad`` of every
        parameter (the flat grad buffer) and returns the loss as a device scalar.

        With a ``ModelState`` the chunk continues that state (stateful TBPTT: the state
        enters detached and leaves detached, burn_dragon_language/src/train/steps.rs:
        2698-2731) and the state is advanced in place. ``grad_ready(name)`` is called on the
        current stream as soon as a shared projection's gradient is final (data-parallel
        overlap)."""
        from .bdh_fused import FusedBDH, FusedWorkspace

        B, T = tokens.shape
        if self._fused is None or self._fused.ws.B != B or self._fused.ws.T != T:
            self._fused = None
            torch.cuda.empty_cache()
            self._fused = FusedBDH(self.cfg, FusedWorkspace(self.cfg, B, T, tokens.device), tp=self.tp)
        f = self._fused
        p32 = self.store.views(self.store.data)
        p16 = self.shadow_dict()
        g32 = self.grad_dict()
        if self.scaffold:
            self._scaffold_prepare(p16, g32)
        pos0 = state.position if state is not None else 0
        rho0s = state.rhos if state is not None else None
        outs = f.forward(p16, p32, tokens, pos0=pos0, rho0s=rho0s, want_state=state is not None)
        loss = f.loss(targets, mask, scale=loss_scale)
        f.backward(p16, p32, g32, tokens, pos0=pos0, accumulate=accumulate, grad_ready=grad_ready, grad16=grad16)
        if self.scaffold:
            self._scaffold_backward(g32)
        if state is not None:
            state.rhos = outs
            state.position += T
        return loss

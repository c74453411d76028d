"""Stateful Dragon runtime: the BDH layer loop with the optional residual connectors,
auxiliary memories, hierarchical cycles, rollout fast steps and latent-reasoning heads.

These variants change the layer loop itself (extra passes over a layer, per-chunk
recurrences, history attention), so they run on the PyTorch layer path built from the
same shared weights as the fused training step (``models.bdh.BDH``); the fused tcgen05
step stays the path for the plain BDH layer. Everything here is differentiable.

Reference behaviour:

* layer loop, connectors and the branch split / merge:
  burn_dragon_core/src/model/dragon/language_pipeline.rs:67-414,
  dragon/connector.rs:5-212 (attention-residual connectors merge as
  ``norm(current + branch_out)``; vanilla keeps ``branch_out``);
* attention residual over the history of layer deltas: model/attention_residual/
  reference.rs (softmax over history with an RMS-normalised key, recency bias
  ``-bias*(age)``, tanh mix gate), block.rs (block summaries + recent raw deltas),
  history.rs (anchor, then deltas ``next - previous``);
* auxiliary memories: dragon/auxiliary_memory.rs:4-376 (y-neuron state
  stabilisation / injection / update, clocked slow memory, surprise-gated summary
  memory with optional write-trigger events);
* y-neuron recurrence single pass: dragon.rs:3338-3768;
* hierarchical Dragon (fast / slow cycles, shared or split rho and weights):
  dragon.rs:1893-2168;
* rollout fast steps (host loop: F passes at the token's position; fused: the token
  repeated F times in one pass at a fixed position): dragon.rs:2721-2995;
* latent reasoning (refiner with optional gate, adaptive halting, energy head,
  step-conditioned decoder, JEPA predictor, next-latent transition, sequence score
  head): dragon.rs:3770-4100, construction dragon.rs:929-1000.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F
from torch import nn

from ..config import DragonConfig
from . import reference as R
from .bdh import BDH


@dataclass
class LayerState:
    rho: torch.Tensor | None = None
    slow_rho: torch.Tensor | None = None
    y_state: torch.Tensor | None = None  # [B, H, Nh]
    clocked_hidden: torch.Tensor | None = None  # [B, 1, D]
    summary_hidden: torch.Tensor | None = None  # [B, 1, D]
    hier_slow: torch.Tensor | None = None  # [B, 1, D]
    mamba: dict | None = None  # Mamba-3 ssm / angle / k / v
    slow_mamba: dict | None = None

    def detach(self) -> None:
        for k, v in vars(self).items():
            if isinstance(v, torch.Tensor):
                setattr(self, k, v.detach())
            elif isinstance(v, dict):
                setattr(self, k, {n: t.detach() for n, t in v.items()})


@dataclass
class RuntimeState:
    layers: list[LayerState] = field(default_factory=list)
    position: int = 0

    @staticmethod
    def new(n_layer: int) -> "RuntimeState":
        return RuntimeState([LayerState() for _ in range(n_layer)], 0)

    def detach(self) -> None:
        for ls in self.layers:
            ls.detach()

    def to_tensors(self) -> dict[str, torch.Tensor]:
        """Flat ``<layer>.<field>[.<key>]`` tensors for a runtime-state checkpoint."""
        out = {}
        for i, ls in enumerate(self.layers):
            for k, v in vars(ls).items():
                if isinstance(v, torch.Tensor):
                    out[f"{i}.{k}"] = v.detach()
                elif isinstance(v, dict):
                    out.update({f"{i}.{k}.{n}": t.detach() for n, t in v.items()})
        return out

    @staticmethod
    def from_tensors(n_layer: int, tensors: dict[str, torch.Tensor], position: int = 0) -> "RuntimeState":
        st = RuntimeState.new(n_layer)
        for name, t in tensors.items():
            parts = name.split(".")
            ls = st.layers[int(parts[0])]
            if len(parts) == 2:
                setattr(ls, parts[1], t)
            else:
                d = getattr(ls, parts[1]) or {}
                d[parts[2]] = t
                setattr(ls, parts[1], d)
        st.position = position
        return st


def _applies(last_layers: int | None, layer: int, n_layer: int) -> bool:
    if last_layers is None:
        return True
    if last_layers == 0:
        return False
    return layer >= max(n_layer, 1) - last_layers


def _first_layer(last_layers: int | None, n_layer: int) -> int:
    return 0 if last_layers is None else max(max(n_layer, 1) - last_layers, 0)


class AttentionResidual(nn.Module):
    """Branch input = current + tanh(g)·(attend(history) − current)."""

    def __init__(self, dim: int, num_heads: int, history_window, recency_bias: float, dropout: float):
        super().__init__()
        self.h = max(1, min(num_heads, dim))
        self.hd = dim // self.h
        self.window = history_window
        self.recency_bias = recency_bias
        self.dropout = dropout
        eye = torch.eye(dim)
        self.mix_gate = nn.Parameter(torch.zeros(1))
        self.query = nn.Parameter(torch.zeros(self.h, self.hd))
        self.key_proj = nn.Parameter(eye.clone())
        self.value_proj = nn.Parameter(eye.clone())
        self.out_proj = nn.Parameter(eye.clone())

    def attend(self, current: torch.Tensor, candidates: list[torch.Tensor]) -> torch.Tensor:
        if not candidates:
            candidates = [current]
        w = len(candidates) if self.window is None else max(self.window, 1)
        hist = torch.stack(candidates[-w:], dim=1)  # [B, L, T, D]
        B, L, T, D = hist.shape
        if L == 1:
            mixed = hist[:, 0]
        else:
            k = (hist @ self.key_proj).view(B, L, T, self.h, self.hd)
            k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6)
            v = (hist @ self.value_proj).view(B, L, T, self.h, self.hd)
            bias = -self.recency_bias * torch.arange(L - 1, -1, -1, device=hist.device, dtype=hist.dtype)
            s = (k * self.query).sum(-1) / math.sqrt(max(self.hd, 1)) + bias.view(1, L, 1, 1)
            p = torch.softmax(s, dim=1)  # over history
            mixed = (p.unsqueeze(-1) * v).sum(1).reshape(B, T, D) @ self.out_proj
            if self.dropout > 0 and self.training:
                mixed = F.dropout(mixed, self.dropout, True)
        g = torch.tanh(self.mix_gate)
        return current + (mixed - current) * g


class BlockAttentionResidual(nn.Module):
    """Attention residual over per-block summaries of older deltas plus recent raw ones."""

    def __init__(self, dim: int, c):
        super().__init__()
        self.attn = AttentionResidual(dim, c.num_heads, None, c.recency_bias, c.dropout)
        self.per_block = max(1, c.layers_per_block)
        self.block_window = c.block_history_window
        self.local_window = max(1, c.intra_block_history_window or self.per_block)
        self.mode = c.summary_mode
        self.summary_proj = nn.Parameter(torch.eye(dim))

    def candidates(self, current: torch.Tensor, history: list[torch.Tensor]) -> list[torch.Tensor]:
        cands = list(history) or [current]
        total = len(cands)
        raw_start = total - min(self.local_window, total)
        out = []
        if raw_start > 0:
            blocks = -(-raw_start // self.per_block)
            keep = max(1, min(self.block_window or blocks, blocks))
            for b in range(blocks - keep, blocks):
                seg = cands[b * self.per_block:min((b + 1) * self.per_block, raw_start)]
                s = torch.stack(seg, 1).mean(1)
                out.append(s @ self.summary_proj if self.mode == "learned_projection" else s)
        return out + cands[raw_start:]

    def attend(self, current, history):
        return self.attn.attend(current, self.candidates(current, history))


class Linear(nn.Module):
    """x @ W + b with W [in, out] (the reference's Linear layout)."""

    def __init__(self, fan_in: int, fan_out: int, gen: torch.Generator, zero: bool = False, bias_value=None):
        super().__init__()
        bound = 1.0 / math.sqrt(max(fan_in, 1))
        w = torch.zeros(fan_in, fan_out) if zero else (torch.rand(fan_in, fan_out, generator=gen) * 2 - 1) * bound
        self.weight = nn.Parameter(w)
        b = torch.zeros(fan_out) if zero else (torch.rand(fan_out, generator=gen) * 2 - 1) * bound
        if bias_value is not None:
            b = torch.full((fan_out,), float(bias_value))
        self.bias = nn.Parameter(b)

    def forward(self, x):
        return x @ self.weight + self.bias


@dataclass
class LatentReasoningOutput:
    raw_hidden: torch.Tensor
    final_hidden: torch.Tensor
    step_hiddens: list
    energies: list
    stop_logits: list
    stop_probs: list
    steps_used: int


class DragonRuntime(nn.Module):
    """BDH core (``self.core``) plus the optional modules the config enables."""

    def __init__(self, cfg: DragonConfig, device=None, seed: int | None = None, rollout_mode: str = "fused"):
        super().__init__()
        cfg.validate()
        self.cfg = cfg
        self.core = BDH(cfg, device=device, seed=seed)
        dev = self.core.store.data.device
        gen = torch.Generator().manual_seed((1337 if seed is None else seed) + 97)
        D, L = cfg.n_embd, cfg.n_layer
        self.connector = cfg.resolved_residual_connector()
        self.rollout_mode = rollout_mode
        if self.connector == "attention_residual":
            c = cfg.attention_residual
            self.attn_res = AttentionResidual(D, c.num_heads, c.history_window, c.recency_bias, c.dropout)
            self.conn_first = _first_layer(c.last_layers, L)
        elif self.connector == "block_attention_residual":
            self.attn_res = BlockAttentionResidual(D, cfg.block_attention_residual)
            self.conn_first = _first_layer(cfg.block_attention_residual.last_layers, L)
        hd = cfg.hierarchical_dragon
        if hd.enabled and hd.weight_sharing == "split":
            from .init import init_param

            H, Nh, N = cfg.n_head, cfg.latent_per_head, cfg.latent_total
            mk = lambda role, shp: nn.Parameter(init_param(cfg, role, shp, gen))  # noqa: E731
            self.slow_encoder = mk("encoder", (H, D, Nh))
            self.slow_encoder_v = mk("encoder_v", (H, D, Nh))
            self.slow_decoder = mk("decoder", (N, D))
        lr = cfg.latent_reasoning
        if lr.enabled:
            hid = D * max(1, lr.refiner_hidden_multiplier)
            self.refiner_in = Linear(D, hid, gen)
            self.refiner_out = Linear(hid, D, gen, zero=True)
            if lr.residual_refinement_gate:
                g0 = lr.residual_refinement_gate_init
                self.refiner_gate = nn.Parameter(torch.full((D,), math.log(g0 / (1 - g0))))
            if lr.energy_head:
                self.energy_head = Linear(D, 1, gen)
            if lr.adaptive_halting:
                self.stop_head = Linear(D, 1, gen, bias_value=lr.stop_bias_init)
            self.jepa_predictor = Linear(D, D, gen)
            if lr.step_conditioned_decoder:
                self.step_decoder_embedding = nn.Parameter(torch.zeros(lr.max_steps + 1, D))
        nl = cfg.next_latent_transition
        if nl.enabled:
            hid = D * max(1, nl.hidden_multiplier)
            self.transition_in = Linear(2 * D, hid, gen)
            self.transition_mid = Linear(hid, hid, gen)
            self.transition_out = Linear(hid, D, gen, zero=nl.zero_init_output)
        if cfg.sequence_score_head.enabled:
            p = cfg.sequence_score_head.projection_dim
            sg = lambda s: torch.Generator().manual_seed(s)
            self.score_query = Linear(D, p, sg(0x7175_6572_795F_6B31 & 0x7FFF_FFFF_FFFF_FFFF))
            self.score_candidate = Linear(D, p, sg(0x6361_6E64_5F6B_6579))
            self.score_out = Linear(p, 1, sg(0x7363_6F72_655F_7631))
        for name, mod in list(self._modules.items()):
            if name != "core":
                mod.to(dev)
        for name, p in list(self._parameters.items()):
            self._parameters[name] = nn.Parameter(p.data.to(dev))
        if cfg.sequence_memory_system == "gated_deltanet2":
            from .sequence import GDN2Params

            self.gdn2 = GDN2Params(cfg.n_head, D, cfg.latent_per_head, cfg.gated_deltanet2, gen).to(dev)
        elif cfg.sequence_memory_system == "mamba3_state_space_duality":
            from .sequence import Mamba3Params

            self.mamba = Mamba3Params(D, cfg.mamba, gen).to(dev)
        Nh = cfg.latent_per_head
        self._freqs = None
        if cfg.rotary_embedding in ("rope", "pope"):
            f = R.rope_freqs if cfg.rotary_embedding == "rope" else R.pope_freqs
            self._freqs = f(Nh, cfg.rope_theta, device=dev)
        self._latent_mask = None
        if cfg.latent_active_blocks is not None:
            from .legacy_attention import BlockPattern1d

            pat = BlockPattern1d(cfg.latent_block_size, set(cfg.latent_active_blocks))
            self._latent_mask = pat.mask(cfg.latent_per_head, device=dev)
        self._decay = R.decay_vector(cfg.decay_slopes(), device=dev) if cfg.uses_decay() else None

    # ------------------------------------------------------------------ pieces
    def _weights(self, slow: bool = False):
        p = self.core.param_dict()
        if slow and hasattr(self, "slow_encoder"):
            return self.slow_encoder, self.slow_encoder_v, self.slow_decoder, p
        return p["encoder"], p["encoder_v"], p["decoder"], p

    def _norm(self, p):
        c = self.cfg
        return R.make_norm(c.norm_kind, p["norm_gamma"], p["norm_beta"], c.norm_eps, p.get("norm_alpha"),
                           p.get("norm_shift"))

    def _rotate(self, x, pos: int, fixed: bool):
        T = x.shape[2]
        if self._freqs is None:
            return x
        positions = torch.full((T,), pos, device=x.device) if fixed else torch.arange(pos, pos + T, device=x.device)
        ph = R.rope_phases(positions, self._freqs)[None, None]
        return R.pope_apply(x, ph) if self.cfg.rotary_embedding == "pope" else R.rope_apply(x, ph)

    def _attend(self, x, v, ls: LayerState, pos: int, fixed: bool, slot: str = "fast"):
        """The sequence memory read / write (sequence_dispatch.rs:83-403): linear
        attention on rho, Gated DeltaNet-2 on its delta-rule state, or Mamba-3 on the
        dense stream. Slot ``slow`` uses the split (hierarchical slow) state."""
        fam = self.cfg.sequence_memory_system
        attr = "slow_rho" if slot == "slow" else "rho"
        rho0 = getattr(ls, attr)
        if rho0 is not None and rho0.shape[0] != x.shape[0]:
            rho0 = None
        if fam == "mamba3_state_space_duality":
            mattr = "slow_mamba" if slot == "slow" else "mamba"
            ctx, st = self.mamba(v, getattr(ls, mattr))
            setattr(ls, mattr, st)
            return ctx[:, None]
        if fam == "gated_deltanet2":
            from .sequence import gdn2_chunk_wy, gdn2_recurrent, l2_normalize

            c = self.cfg.gated_deltanet2
            key, erase, write, log_decay = self.gdn2.project(v)
            q, k = self._rotate(x, pos, fixed), self._rotate(key, pos, fixed)
            if c.qk_l2_norm:
                q, k = l2_normalize(q, c.state_epsilon), l2_normalize(k, c.state_epsilon)
            if self.cfg.sequence_executor == "gated_delta_chunk_wy":
                out, S = gdn2_chunk_wy(q, k, v[:, None], erase, write, log_decay, rho0, c.chunk_size)
            else:
                out, S = gdn2_recurrent(q, k, v[:, None], erase, write, log_decay, rho0)
            setattr(ls, attr, S)
            return out * self.gdn2.output_scale
        q = self._rotate(x, pos, fixed)
        a, rho = R.linear_attention_chunked(q, v[:, None], rho0=rho0, decay=self._decay, need_state=True,
                                            chunk=getattr(self.cfg, "dense_score_row_chunk", 0) or 0)
        setattr(ls, attr, rho)
        return a

    def _lowrank_step(self, v, ls, pos, fixed, *, slow_weights=False, slot="fast", x_inject=None, want_y=False):
        enc, enc_v, dec, p = self._weights(slow_weights)
        nf = self._norm(p)
        thr, thr_y = self.cfg.thresholds()
        lm = self._latent_mask
        x = torch.relu(torch.einsum("btd,hdn->bhtn", v, enc) - thr)
        if lm is not None:
            x = x * lm
        if x_inject is not None:
            x = x + x_inject
        a = nf(self._attend(x, v, ls, pos, fixed, slot))
        y = torch.relu(torch.einsum("bhtd,hdn->bhtn", a, enc_v) - thr_y)
        if lm is not None:
            y = y * lm
        yn = x * y
        if self.cfg.dropout > 0 and self.training:
            yn = F.dropout(yn, self.cfg.dropout, True)
        B, H, T, Nh = yn.shape
        m = nf(yn.permute(0, 2, 1, 3).reshape(B, T, H * Nh) @ dec)
        out = nf(v + m)
        return (out, yn) if want_y else out

    # ------------------------------------------------------------------ memories
    def _summary_branch(self, inp, ls: LayerState, start_pos: int, event_mask):
        c = self.cfg.summary_memory
        B, T, D = inp.shape
        ck = max(1, c.chunk_tokens)
        carry = ls.summary_hidden if ls.summary_hidden is not None and ls.summary_hidden.shape[0] == B else None
        if T == 1 and ck > 1 and start_pos % ck and carry is not None:
            return inp + carry * c.residual_scale
        trigger = bool(c.write_trigger_token_ids)
        outs = []
        for s in range(0, T, ck):
            e = min(s + ck, T)
            chunk = inp[:, s:e]
            summary = chunk.mean(1, keepdim=True)
            outs.append(chunk if carry is None else chunk + carry * c.residual_scale)
            gate = None
            if trigger:
                if event_mask is None:
                    gate = torch.zeros(B, 1, 1, device=inp.device, dtype=inp.dtype)
                else:
                    hits = event_mask[:, s:e].to(inp.dtype).sum(1).view(B, 1, 1)
                    gate = hits / (hits + 1e-6)
            if carry is None:
                nxt = summary * c.state_update_scale
                carry = nxt * gate if gate is not None else nxt
            else:
                upd = self._summary_update(carry, summary)
                carry = carry * (1 - gate) + upd * gate if gate is not None else upd
        ls.summary_hidden = carry
        return torch.cat(outs, 1)

    def _summary_update(self, prev, summary):
        c = self.cfg.summary_memory
        ungated = prev * c.state_decay + summary * c.state_update_scale
        if c.surprise_gate_threshold <= 0:
            return ungated
        z = torch.relu(((summary - prev).abs().mean(-1, keepdim=True) - c.surprise_gate_threshold)
                       * c.surprise_gate_sharpness)
        g = z / (z + 1)
        return prev * (1 - g) + ungated * g

    def _clocked_branch(self, inp, ls: LayerState, start_pos: int, fixed: bool):
        c = self.cfg.clocked_slow_memory
        B, T, D = inp.shape
        ck = max(1, min(c.chunk_tokens, T))
        if T == 1 and c.chunk_tokens > 1 and start_pos % c.chunk_tokens and ls.clocked_hidden is not None \
                and ls.clocked_hidden.shape[0] == B:
            return inp + ls.clocked_hidden * c.residual_scale
        outs, last = [], None
        for i, s in enumerate(range(0, T, ck)):
            e = min(s + ck, T)
            chunk = inp[:, s:e]
            slow_pos = start_pos // ck if fixed else start_pos // ck + i
            h = self._lowrank_step(chunk.mean(1, keepdim=True), ls, slow_pos, fixed)
            last = h
            outs.append(chunk + h * c.residual_scale)
        ls.clocked_hidden = last
        return torch.cat(outs, 1)

    def _stabilize(self, s):
        cap = self.cfg.y_neuron_recurrence.state_rms_cap
        if cap is None:
            return s
        # clamp before the square root (same value as clamping the rms at 1e-6) so an
        # all-zero row has a finite gradient
        rms = s.pow(2).mean(-1, keepdim=True).clamp_min(1e-12).sqrt()
        return s / (rms / cap).clamp_min(1.0)

    def _y_recurrent_layer(self, v, ls: LayerState, start_pos: int, fixed: bool):
        c = self.cfg.y_neuron_recurrence
        enc, enc_v, dec, p = self._weights()
        nf = self._norm(p)
        thr, thr_y = self.cfg.thresholds()
        B, T, D = v.shape
        H, Nh = self.cfg.n_head, self.cfg.latent_per_head
        st = ls.y_state
        st = self._stabilize(st) if st is not None and st.shape == (B, H, Nh) else v.new_zeros(B, H, Nh)
        x_base = torch.relu(torch.einsum("btd,hdn->bhtn", v, enc) - thr)
        if self._latent_mask is not None:
            x_base = x_base * self._latent_mask
        ck = max(1, min(c.chunk_tokens, T))
        outs = []
        for s in range(0, T, ck):
            e = min(s + ck, T)
            x = x_base[:, :, s:e]
            if c.carry_in_scale != 0.0:
                x = x + st.unsqueeze(2) * c.carry_in_scale
            tok = v[:, s:e]
            a = nf(self._attend(x, tok, ls, start_pos if fixed else start_pos + s, fixed))
            y = torch.relu(torch.einsum("bhtd,hdn->bhtn", a, enc_v) - thr_y)
            if self._latent_mask is not None:
                y = y * self._latent_mask
            yn = x * y
            if self.cfg.dropout > 0 and self.training:
                yn = F.dropout(yn, self.cfg.dropout, True)
            m = nf(yn.permute(0, 2, 1, 3).reshape(B, e - s, H * Nh) @ dec)
            outs.append(nf(tok + m))
            st = self._stabilize(st * c.state_decay + yn[:, :, -1] * c.state_update_scale)
        ls.y_state = st
        return torch.cat(outs, 1)

    def _hierarchical_layer(self, v, ls: LayerState, start_pos: int, fixed: bool):
        c = self.cfg.hierarchical_dragon
        nf = self._norm(self.core.param_dict())
        B, T, D = v.shape
        fast = v
        slow = ls.hier_slow if ls.hier_slow is not None and ls.hier_slow.shape == (B, 1, D) else None
        s2f, f2s = max(c.slow_to_fast_scale, 0.0), max(c.fast_to_slow_scale, 0.0)
        slot = "slow" if c.rho_sharing == "split" else "fast"
        split_w = c.weight_sharing == "split"
        for _ in range(max(1, c.slow_cycles)):
            if s2f > 0 and slow is not None:
                fast = nf(fast + slow * s2f)
            for _ in range(max(1, c.fast_cycles)):
                fast = self._lowrank_step(fast, ls, start_pos, fixed)
            sin = fast.mean(1, keepdim=True)
            if f2s > 0 and slow is not None:
                sin = nf(sin + slow * f2s)
            slow = self._lowrank_step(sin, ls, start_pos, fixed, slow_weights=split_w, slot=slot)
            if s2f > 0:
                fast = nf(fast + slow * s2f)
        ls.hier_slow = slow
        return fast

    # ------------------------------------------------------------------ passes
    def hidden_single_pass(self, embedded, state: RuntimeState, start_pos: int, fixed: bool = False,
                           event_mask=None):
        """One pass of the layer loop over [B, T, D] embeddings (position not advanced)."""
        cfg = self.cfg
        p = self.core.param_dict()
        nf = self._norm(p)
        cur = nf(embedded)
        conn = self.connector
        history = [cur] if conn in ("attention_residual", "block_attention_residual") else None
        streams = cfg.mhc_streams if conn == "mhc" else 1
        dyn = streams > 1 and cfg.mhc_policy == "dynamic_positive"
        if streams > 1:
            from . import mhc as MHC

            Rs = MHC.bootstrap(cur, streams, p["mhc_boot"] if dyn else None)
        yrec = cfg.y_neuron_recurrence.enabled
        for li in range(cfg.n_layer):
            ls = state.layers[li]
            before = cur
            use_conn = history is not None and li >= self.conn_first
            if dyn:
                branch, Rs, w_out = MHC.dynamic_split(Rs, p, li, cfg.mhc_tau, cfg.mhc_iters)
            elif streams > 1:
                branch, Rs = MHC.layer_split(Rs, p["mhc_res"][li], p["mhc_pre"][li], cfg.mhc_tau, cfg.mhc_iters)
            elif use_conn:
                branch = self.attn_res.attend(cur, history)
            else:
                branch = cur
            if yrec:
                ls.clocked_hidden = ls.summary_hidden = None
                if _applies(cfg.y_neuron_recurrence.last_layers, li, cfg.n_layer):
                    out = self._y_recurrent_layer(branch, ls, start_pos, fixed)
                else:
                    ls.y_state = None
                    out = self._lowrank_step(branch, ls, start_pos, fixed)
            else:
                if cfg.summary_memory.enabled and _applies(cfg.summary_memory.last_layers, li, cfg.n_layer):
                    branch = self._summary_branch(branch, ls, start_pos, event_mask)
                else:
                    ls.summary_hidden = None
                hd = cfg.hierarchical_dragon
                if cfg.clocked_slow_memory.enabled and _applies(cfg.clocked_slow_memory.last_layers, li, cfg.n_layer):
                    out = self._clocked_branch(branch, ls, start_pos, fixed)
                elif hd.enabled and li >= _first_layer(hd.last_layers, cfg.n_layer):
                    ls.clocked_hidden = ls.y_state = None
                    out = self._hierarchical_layer(branch, ls, start_pos, fixed)
                else:
                    ls.clocked_hidden = None
                    ls.hier_slow = ls.slow_rho = None
                    out = self._lowrank_step(branch, ls, start_pos, fixed)
            if streams > 1:
                Rs = MHC.dynamic_merge(Rs, out, w_out) if dyn else MHC.layer_merge(Rs, out, p["mhc_post"][li])
                cur = out
            elif use_conn:
                cur = nf(cur + out)
            else:
                cur = out
            if history is not None:
                history.append(cur - before)
        if streams > 1:
            cur = Rs.mean(dim=1)
        return cur

    def forward_hidden(self, tokens, state: RuntimeState | None = None, event_mask=None):
        """Final hidden [B, T, D] after the layer loop, rollout and latent reasoning."""
        h, _ = self._forward(tokens, state, event_mask, logits=False)
        return h

    def forward(self, tokens, state: RuntimeState | None = None, event_mask=None):
        """Logits [B, T, V]; ``state`` (``RuntimeState``) is read and advanced."""
        _, lg = self._forward(tokens, state, event_mask, logits=True)
        return lg

    def loss(self, tokens, targets, mask=None, state=None, event_mask=None):
        return R.cross_entropy(self.forward(tokens, state, event_mask), targets, mask)

    def _forward(self, tokens, state, event_mask, logits: bool):
        if state is None:
            state = RuntimeState.new(self.cfg.n_layer)
        p = self.core.param_dict()
        emb = p["embed"][tokens]
        Fs = self.cfg.rollout_fast_steps_per_slow_step
        if Fs <= 1:
            h = self.hidden_single_pass(emb, state, state.position, False, event_mask)
            state.position += tokens.shape[1]
            h = self.reason_hidden_final(h)
            return h, (self.logits_from_hidden(h) if logits else None)
        hs = []
        for t in range(tokens.shape[1]):
            tok = emb[:, t:t + 1]
            em = None if event_mask is None else event_mask[:, t:t + 1]
            if self.rollout_mode == "host_loop":
                for _ in range(Fs):
                    h = self.hidden_single_pass(tok, state, state.position, False, em)
            else:  # the token repeated F times in one pass at a fixed position
                h = self.hidden_single_pass(tok.expand(-1, Fs, -1), state, state.position, True, em)[:, -1:]
            hs.append(self.reason_hidden_final(h))
            state.position += 1
        h = torch.cat(hs, 1)
        return h, (self.logits_from_hidden(h) if logits else None)

    # ------------------------------------------------------------------ heads
    def latent_reasoning_enabled(self) -> bool:
        lr = self.cfg.latent_reasoning
        return lr.enabled and lr.max_steps > 0 and hasattr(self, "refiner_in") and \
            (not lr.adaptive_halting or hasattr(self, "stop_head"))

    def _refine(self, cur):
        upd = self.refiner_out(F.gelu(self.refiner_in(cur)))
        if hasattr(self, "refiner_gate"):
            upd = upd * torch.sigmoid(self.refiner_gate)
        nxt = cur + upd
        return self._norm(self.core.param_dict())(nxt) if self.cfg.latent_reasoning.normalize_steps else nxt

    def reason_hidden(self, hidden) -> LatentReasoningOutput:
        if not self.latent_reasoning_enabled():
            return LatentReasoningOutput(hidden, hidden, [], [], [], [], 0)
        lr = self.cfg.latent_reasoning
        cur = hidden
        final = torch.zeros_like(hidden)
        remaining = hidden.new_ones(*hidden.shape[:-1], 1)
        steps, energies, logits_l, probs_l = [], [], [], []
        for s in range(lr.max_steps):
            cur = self._refine(cur)
            if hasattr(self, "energy_head"):
                energies.append(self.energy_head(cur))
            if hasattr(self, "stop_head"):
                lg = self.stop_head(cur)
                pr = torch.zeros_like(lg) if s + 1 < lr.min_steps else torch.sigmoid(lg)
                halt = (pr >= lr.halt_threshold).to(cur.dtype) * remaining
                final = final + cur * halt
                remaining = remaining * (1 - halt)
                logits_l.append(lg)
                probs_l.append(pr)
            steps.append(cur)
        final = final + cur * remaining if lr.adaptive_halting else cur
        return LatentReasoningOutput(hidden, final, steps, energies, logits_l, probs_l, lr.max_steps)

    def reason_hidden_final(self, hidden):
        return self.reason_hidden(hidden).final_hidden

    def logits_from_hidden(self, hidden, step: int | None = None):
        lr = self.cfg.latent_reasoning
        if step is None:
            step = lr.max_steps if self.latent_reasoning_enabled() else 0
        if hasattr(self, "step_decoder_embedding") and lr.step_conditioned_decoder_scale > 1.1920929e-07:
            emb = self.step_decoder_embedding
            hidden = hidden + emb[min(step, emb.shape[0] - 1)] * lr.step_conditioned_decoder_scale
        p = self.core.param_dict()
        head = p["embed"].t() if p.get("lm_head") is None else p["lm_head"]
        return hidden @ head

    def latent_jepa_prediction(self, hidden):
        return self.jepa_predictor(hidden) if hasattr(self, "jepa_predictor") else hidden

    def latent_energy(self, hidden):
        return self.energy_head(hidden) if hasattr(self, "energy_head") else None

    def next_latent_prediction(self, hidden, action_embedding):
        if not hasattr(self, "transition_in") or action_embedding.shape != hidden.shape:
            return None
        x = torch.cat([hidden, action_embedding], -1)
        if self.cfg.next_latent_transition.normalize_input:
            mu = x.mean(-1, keepdim=True)
            c = x - mu
            x = c / (c.pow(2).mean(-1, keepdim=True) + 1e-5).sqrt()
        return hidden + self.transition_out(F.gelu(self.transition_mid(F.gelu(self.transition_in(x)))))

    def sequence_scores(self, hidden):
        return self.score_out(self.score_candidate(hidden)) if hasattr(self, "score_out") else None

    def sequence_scores_pair(self, prompt_hidden, terminal_hidden):
        if not hasattr(self, "score_out") or prompt_hidden.shape != terminal_hidden.shape:
            return None
        return self.score_out(self.score_query(prompt_hidden) * self.score_candidate(terminal_hidden))

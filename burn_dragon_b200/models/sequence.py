"""Alternate sequence-memory systems for the Dragon layer: Gated DeltaNet-2 and Mamba-3.

Both replace the linear-attention read/write of rho inside the BDH layer; the rest of
the layer (x / y projections, gating, decoder, norms) is unchanged.

Gated DeltaNet-2 (burn_dragon_core/src/model/sequence/gdn2.rs). Per head, with state
``S [L, D]``, decay ``a_t = exp(log_decay_t)`` (per latent channel), erase gate ``e_t``,
write gate ``w_t``, key ``k_t`` and value ``v_t``::

    A_t S_{t-1} = diag(a_t) S_{t-1}
    u_t         = w_t * v_t - (e_t * k_t)^T (A_t S_{t-1})
    S_t         = A_t S_{t-1} + k_t u_t^T
    o_t         = q_t^T S_t / sqrt(L)

(golden one-step vector: gdn2.rs ``reference_matches_one_step_paper_update``). Two
executors: ``reference`` (the token recurrence) and ``gated_delta_chunk_wy``, the
chunked WY form that turns each chunk into GEMMs plus one unit-lower-triangular solve:
with cumulative decay ``c = exp(cumsum log a)``, ``W = K / c``, ``M = E*K*c``,
``Z = (I + tril(M W^T, -1))^{-1} (w*V - M S_0)``, the chunk output is
``(Q*c) S_0 + tril((Q*c) W^T) Z`` and the carried state ``diag(c_C) (S_0 + W^T Z)``
(the same algebra as gdn2.rs ``wy_chunk_reference``). Projections (key / erase /
decay / write, gate modes channel / scalar / disabled, ``allow_neg_eigval``):
gdn2.rs:180-430.

Mamba-3 state-space duality, SISO (burn_dragon_kernel/src/sequence/mamba3/forward.rs:
1738-2346, parameters burn_dragon_core/src/model/sequence/mamba.rs:300-420): one input
projection gives z, x, B, C, dt, A, trapezoid gate and shared rotary angles; B and C
are RMS-normalised per group, expanded to heads and biased; data-dependent rotary
angles accumulate ``tanh(angle) * dt * pi``; per chunk the output is the carried-state
read ``q S~^T * exp(dA prefix)`` + the strictly causal intra-chunk scores
``(q k^T) * exp(min(dA_i - dA_j, 0))`` applied to x + the diagonal term
``(D + gamma * q.k) * x``, gated by ``silu(z)`` and projected out; the state carries the
SSM matrix, the angle, and the last key / value for the trapezoid term.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

# ----------------------------------------------------------------------- GDN-2


def l2_normalize(x: torch.Tensor, eps: float) -> torch.Tensor:
    return x / (x.pow(2).sum(-1, keepdim=True) + eps).sqrt()


def gdn2_recurrent(q, k, v, erase, write, log_decay, state=None):
    """q, k, erase, log_decay [B,H,T,L]; v, write [B,H,T,D] (v may have H=1).
    Returns (out [B,H,T,D], state [B,H,L,D])."""
    B, H, T, L = q.shape
    v = v.expand(B, H, T, v.shape[-1])
    D = v.shape[-1]
    S = q.new_zeros(B, H, L, D) if state is None else state
    outs = []
    a = log_decay.exp()
    for t in range(T):
        S = S * a[:, :, t, :, None]
        ek = erase[:, :, t] * k[:, :, t]
        u = write[:, :, t] * v[:, :, t] - torch.einsum("bhl,bhld->bhd", ek, S)
        S = S + k[:, :, t, :, None] * u[:, :, None, :]
        outs.append(torch.einsum("bhl,bhld->bhd", q[:, :, t], S))
    return torch.stack(outs, 2) / math.sqrt(L), S


def gdn2_chunk_wy(q, k, v, erase, write, log_decay, state=None, chunk: int = 64):
    """Chunked WY executor of the same recurrence (GEMMs + a triangular solve per chunk)."""
    B, H, T, L = q.shape
    v = v.expand(B, H, T, v.shape[-1])
    D = v.shape[-1]
    S = q.new_zeros(B, H, L, D) if state is None else state
    outs = []
    for s in range(0, T, chunk):
        e = min(s + chunk, T)
        C = e - s
        c = log_decay[:, :, s:e].cumsum(2).exp()  # [B,H,C,L]
        kk = k[:, :, s:e]
        W = kk / c
        M = erase[:, :, s:e] * kk * c
        A = torch.tril(M @ W.transpose(-1, -2), -1)
        rhs = write[:, :, s:e] * v[:, :, s:e] - M @ S
        eye = torch.eye(C, device=q.device, dtype=q.dtype)
        Z = torch.linalg.solve_triangular(eye + A, rhs, upper=False, unitriangular=True)
        Qc = q[:, :, s:e] * c
        outs.append(Qc @ S + torch.tril(Qc @ W.transpose(-1, -2)) @ Z)
        S = c[:, :, -1, :, None] * (S + W.transpose(-1, -2) @ Z)
    return torch.cat(outs, 2) / math.sqrt(L), S


def _gate(logits: torch.Tensor, mode: str, neg_eig: bool) -> torch.Tensor:
    if mode == "disabled":
        return torch.ones_like(logits)
    g = torch.sigmoid(logits) if mode == "channel" else torch.sigmoid(logits.mean(-1, keepdim=True)).expand_as(logits)
    return g * 2.0 if neg_eig else g


class GDN2Params(nn.Module):
    """Key / erase / decay / write projections shared by every layer (gdn2.rs:180-240)."""

    def __init__(self, n_head: int, dim: int, latent: int, cfg, gen: torch.Generator):
        super().__init__()
        self.cfg = cfg
        std = min(math.sqrt(1.0 / max(dim, 1)), 0.02)
        rn = lambda *s: torch.randn(*s, generator=gen) * std
        self.key_proj = nn.Parameter(rn(n_head, dim, latent))
        self.erase_proj = nn.Parameter(rn(n_head, dim, latent))
        self.erase_bias = nn.Parameter(torch.zeros(n_head, latent))
        self.decay_proj = nn.Parameter(rn(n_head, dim, latent))
        self.decay_log = nn.Parameter(torch.zeros(n_head, latent))
        self.decay_bias = nn.Parameter(torch.full((n_head, latent), -4.6))
        self.write_proj = nn.Parameter(rn(n_head, dim, dim))
        self.write_bias = nn.Parameter(torch.zeros(n_head, dim))
        self.register_buffer("output_scale", torch.full((1,), float(cfg.output_scale)))

    def project(self, dense: torch.Tensor):
        """dense [B,T,D] -> key, erase, write, log_decay (each [B,H,T,*])."""
        c = self.cfg
        key = torch.einsum("btd,hdl->bhtl", dense, self.key_proj)
        erase = torch.einsum("btd,hdl->bhtl", dense, self.erase_proj) + self.erase_bias[None, :, None]
        dec = torch.einsum("btd,hdl->bhtl", dense, self.decay_proj) + self.decay_bias[None, :, None]
        write = torch.einsum("btd,hde->bhte", dense, self.write_proj) + self.write_bias[None, :, None]
        erase = _gate(erase, c.erase_gate, c.allow_neg_eigval)
        write = _gate(write, c.write_gate, False)
        if c.decay_gate == "disabled":
            log_decay = torch.zeros_like(dec)
        else:
            if c.decay_gate == "scalar":
                dec = dec.mean(-1, keepdim=True).expand_as(dec)
            log_decay = -F.softplus(dec) * self.decay_log.exp()[None, :, None]
        return key, erase, write, log_decay


# ----------------------------------------------------------------------- Mamba-3


class Mamba3Params(nn.Module):
    """Mamba-3 SISO parameters (mamba.rs:300-380)."""

    def __init__(self, d_model: int, cfg, gen: torch.Generator):
        super().__init__()
        self.d_model = d_model
        self.d_inner = d_model * cfg.expand
        self.headdim = cfg.headdim
        self.nheads = self.d_inner // cfg.headdim
        self.ngroups = cfg.ngroups
        self.d_state = cfg.d_state
        split = int(cfg.d_state * cfg.rope_fraction)
        split -= split % 2
        self.n_angles = max(split // 2, 1)
        self.eps, self.a_floor, self.chunk = cfg.norm_eps, cfg.a_floor, cfg.chunk_size
        in_dim = 2 * self.d_inner + 2 * self.ngroups * self.d_state + 3 * self.nheads + self.n_angles
        self.in_proj = nn.Parameter(torch.randn(d_model, in_dim, generator=gen) / math.sqrt(d_model))
        lo, hi = math.log(cfg.dt_min), math.log(cfg.dt_max)
        dt = (torch.rand(self.nheads, generator=gen) * (hi - lo) + lo).exp().clamp_min(cfg.dt_init_floor)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))  # softplus^-1(dt)
        self.b_bias = nn.Parameter(torch.ones(self.nheads, self.d_state))
        self.c_bias = nn.Parameter(torch.ones(self.nheads, self.d_state))
        self.b_norm_weight = nn.Parameter(torch.ones(self.d_state))
        self.c_norm_weight = nn.Parameter(torch.ones(self.d_state))
        self.d_skip = nn.Parameter(torch.ones(self.nheads))
        self.out_proj = nn.Parameter(torch.randn(self.d_inner, d_model, generator=gen) / math.sqrt(self.d_inner))

    def _bc(self, raw, weight, bias):
        B, T = raw.shape[:2]
        g = raw.view(B, T, self.ngroups, self.d_state)
        g = g * torch.rsqrt(g.pow(2).mean(-1, keepdim=True) + self.eps) * weight
        return g.repeat_interleave(self.nheads // self.ngroups, dim=2) + bias

    @staticmethod
    def _rotate(x, ang, n):
        """Pairwise rotation of the first 2n channels of x [B,T,H,S] by ang [B,T,H,n]."""
        r = x[..., :2 * n].unflatten(-1, (n, 2))
        c, s = ang.cos(), ang.sin()
        rot = torch.stack((r[..., 0] * c - r[..., 1] * s, r[..., 0] * s + r[..., 1] * c), -1).flatten(-2)
        return torch.cat((rot, x[..., 2 * n:]), -1)

    def forward(self, hidden: torch.Tensor, state: dict | None):
        """hidden [B,T,D] -> (context [B,T,D], state dict ssm/angle/k/v). On CUDA the chunk
        scan runs in the ``ssd_chunk`` kernels (``forward_fused``); elsewhere in the chunk
        loop below."""
        if hidden.is_cuda and fused_ssd_ok(self):
            return self.forward_fused(hidden, state)
        B, T, Dm = hidden.shape
        H, P, S, n = self.nheads, self.headdim, self.d_state, self.n_angles
        di, gs = self.d_inner, self.ngroups * S
        pr = hidden @ self.in_proj
        z = pr[..., :di].view(B, T, H, P)
        x = pr[..., di:2 * di].view(B, T, H, P)
        k_pre = self._bc(pr[..., 2 * di:2 * di + gs], self.b_norm_weight, self.b_bias)
        q_pre = self._bc(pr[..., 2 * di + gs:2 * di + 2 * gs], self.c_norm_weight, self.c_bias)
        o = 2 * di + 2 * gs
        dt = F.softplus(self.dt_bias + pr[..., o:o + H])  # [B,T,H]
        a = (-F.softplus(pr[..., o + H:o + 2 * H])).clamp_max(-self.a_floor)
        trap = torch.sigmoid(pr[..., o + 2 * H:o + 3 * H])
        ang_proj = pr[..., o + 3 * H:].unsqueeze(2).expand(B, T, H, n)
        gamma = dt * trap
        beta = dt * (1 - trap)  # trapezoid weight of the previous token
        st = state or {}
        ssm = st.get("ssm", hidden.new_zeros(B, H, P, S))
        ang_s = st.get("angle", hidden.new_zeros(B, H, n))
        k_s = st.get("k", hidden.new_zeros(B, H, S))
        v_s = st.get("v", hidden.new_zeros(B, H, P))
        outs = []
        for s0 in range(0, T, self.chunk):
            s1 = min(s0 + self.chunk, T)
            sl = slice(s0, s1)
            tilde = ssm + v_s[..., None] * k_s[:, :, None, :] * (dt[:, s0] * (1 - trap[:, s0]))[..., None, None]
            ang = (torch.tanh(ang_proj[:, sl]) * dt[:, sl, :, None] * math.pi).cumsum(1) + ang_s[:, None]
            q_rot = self._rotate(q_pre[:, sl], ang, n)
            k_rot = self._rotate(k_pre[:, sl], ang, n)
            qk_dot = (q_pre[:, sl] * k_pre[:, sl]).sum(-1) * gamma[:, sl]  # [B,C,H]
            q = q_rot.transpose(1, 2)  # [B,H,C,S]
            # a token's key carries its own gamma plus the next token's beta; the next
            # token's beta for the chunk's last token enters through the carried
            # trapezoid term of the following chunk instead, so the result does not
            # depend on the chunk size
            shifted = torch.cat((beta[:, s0 + 1:s1], beta.new_zeros(B, 1, H)), 1)
            kc = (k_rot * (gamma[:, sl] + shifted)[..., None]).transpose(1, 2)
            v = x[:, sl].transpose(1, 2)  # [B,H,C,P]
            da = (a[:, sl] * dt[:, sl]).transpose(1, 2).cumsum(2)  # [B,H,C]
            prev = (q @ tilde.transpose(-1, -2)) * da.exp()[..., None]
            dec = (da[..., :, None] - da[..., None, :]).clamp_max(0).exp()
            cur = torch.tril((q @ kc.transpose(-1, -2)) * dec, -1) @ v
            y = prev + cur + (self.d_skip[None, :, None, None] + qk_dot.transpose(1, 2)[..., None]) * v
            y = F.silu(z[:, sl].transpose(1, 2)) * y
            outs.append(y.transpose(1, 2).reshape(B, s1 - s0, di) @ self.out_proj)
            last = da[..., -1]
            wv = v * (last[..., None] - da).exp()[..., None]
            ssm = tilde * last.exp()[..., None, None] + wv.transpose(-1, -2) @ kc
            ang_s = ang[:, -1]
            k_s = k_rot[:, -1]
            v_s = x[:, s1 - 1]
        return torch.cat(outs, 1), {"ssm": ssm, "angle": ang_s, "k": k_s, "v": v_s}


# ----------------------------------------------------------------------- Mamba-3 on the device


def fused_ssd_ok(m: "Mamba3Params") -> bool:
    """The ``ssd_chunk`` kernels' limits: chunk <= 64, state <= 64, head dim <= 256."""
    return m.chunk <= 64 and m.d_state <= 64 and m.headdim <= 256


class SSDChunkScan(torch.autograd.Function):
    """The chunk scan of the state-space duality on the device (``csrc/ssd_chunk.cu``).

    Inputs (fp32, [BH, ...]): q, k [BH, T, S]; v [BH, T, P]; da [BH, T] (chunk-local
    cumulative log decay); s0 [BH, P, S]; vs [BH, n, P], ks [BH, n, S], cf [BH, n] (the
    trapezoid term of each chunk). Outputs: y [BH, T, P] (carried-state read + causal
    intra-chunk term) and the final state [BH, P, S]."""

    @staticmethod
    def forward(ctx, q, k, v, da, s0, vs, ks, cf, chunk: int):
        from .. import _ext

        BH, T, S = q.shape
        P = v.shape[-1]
        n = -(-T // chunk)
        y = torch.empty(BH, T, P, device=q.device)
        sf = torch.empty(BH, P, S, device=q.device)
        sc = torch.empty(BH, n, P, S, device=q.device)
        _ext.load().ssd_chunk_fwd(q, k, v, da, s0, vs, ks, cf, chunk, y, sf, sc)
        ctx.save_for_backward(q, k, v, da, vs, ks, cf, sc)
        ctx.chunk = chunk
        return y, sf

    @staticmethod
    def backward(ctx, dy, dsf):
        from .. import _ext

        q, k, v, da, vs, ks, cf, sc = ctx.saved_tensors
        dy = torch.zeros_like(v) if dy is None else dy.contiguous()
        BH, T, S = q.shape
        P = v.shape[-1]
        dsf = torch.zeros(BH, P, S, device=q.device) if dsf is None else dsf.contiguous()
        g = [torch.empty_like(t) for t in (q, k, v, da)]
        ds0 = torch.empty(BH, P, S, device=q.device)
        dvs, dks, dcf = torch.empty_like(vs), torch.empty_like(ks), torch.empty_like(cf)
        _ext.load().ssd_chunk_bwd(q, k, v, da, vs, ks, cf, sc, dy, dsf, ctx.chunk, *g, ds0, dvs, dks, dcf)
        return (*g, ds0, dvs, dks, dcf, None)


def ssd_scan_reference(q, k, v, da, s0, vs, ks, cf, chunk: int):
    """PyTorch restatement of ``SSDChunkScan`` (same inputs and outputs; the oracle)."""
    BH, T, S = q.shape
    st = s0
    ys = []
    for c, t0 in enumerate(range(0, T, chunk)):
        t1 = min(t0 + chunk, T)
        qc, kcc, vc, dc = q[:, t0:t1], k[:, t0:t1], v[:, t0:t1], da[:, t0:t1]
        tl = st + cf[:, c, None, None] * vs[:, c, :, None] * ks[:, c, None, :]
        dec = (dc[:, :, None] - dc[:, None, :]).clamp_max(0).exp()
        ys.append((qc @ tl.transpose(-1, -2)) * dc.exp()[..., None]
                  + torch.tril((qc @ kcc.transpose(-1, -2)) * dec, -1) @ vc)
        last = dc[:, -1]
        st = tl * last.exp()[:, None, None] + (vc * (last[:, None] - dc).exp()[..., None]).transpose(-1, -2) @ kcc
    return torch.cat(ys, 1), st


def _forward_fused(self, hidden: torch.Tensor, state: dict | None, scan=None):
    """Mamba-3 SISO with the projections, norms and rotations vectorised over the whole
    sequence and the chunk scan in ``SSDChunkScan`` (the same function as the chunk loop of
    ``forward``: the rotary angle accumulates over the sequence, a token's key carries
    its own gamma plus the next token's beta inside its chunk, and each chunk's first
    token's beta enters through the trapezoid term on the previous token's key / value)."""
    B, T, Dm = hidden.shape
    H, P, S, n = self.nheads, self.headdim, self.d_state, self.n_angles
    di, gs, C = self.d_inner, self.ngroups * S, self.chunk
    pr = hidden @ self.in_proj
    z = pr[..., :di].view(B, T, H, P)
    x = pr[..., di:2 * di].view(B, T, H, P)
    k_pre = self._bc(pr[..., 2 * di:2 * di + gs], self.b_norm_weight, self.b_bias)
    q_pre = self._bc(pr[..., 2 * di + gs:2 * di + 2 * gs], self.c_norm_weight, self.c_bias)
    o = 2 * di + 2 * gs
    dt = F.softplus(self.dt_bias + pr[..., o:o + H])
    a = (-F.softplus(pr[..., o + H:o + 2 * H])).clamp_max(-self.a_floor)
    trap = torch.sigmoid(pr[..., o + 2 * H:o + 3 * H])
    ang_proj = pr[..., o + 3 * H:].unsqueeze(2).expand(B, T, H, n)
    gamma = dt * trap
    beta = dt * (1 - trap)
    st = state or {}
    ssm = st.get("ssm", hidden.new_zeros(B, H, P, S))
    ang_s = st.get("angle", hidden.new_zeros(B, H, n))
    k_s = st.get("k", hidden.new_zeros(B, H, S))
    v_s = st.get("v", hidden.new_zeros(B, H, P))
    ang = (torch.tanh(ang_proj) * dt[..., None] * math.pi).cumsum(1) + ang_s[:, None]
    q_rot = self._rotate(q_pre, ang, n)
    k_rot = self._rotate(k_pre, ang, n)
    qk_dot = (q_pre * k_pre).sum(-1) * gamma                         # [B,T,H]
    t_idx = torch.arange(T, device=hidden.device)
    chunk_end = ((t_idx + 1) % C == 0) | (t_idx == T - 1)
    nxt = torch.cat((beta[:, 1:], beta.new_zeros(B, 1, H)), 1) * (~chunk_end)[None, :, None]
    kc = k_rot * (gamma + nxt)[..., None]
    nch = -(-T // C)
    pad = nch * C - T
    adt = F.pad(a * dt, (0, 0, 0, pad)).view(B, nch, C, H).cumsum(2).view(B, nch * C, H)[:, :T]
    starts = torch.arange(nch, device=hidden.device) * C
    cf = beta[:, starts]                                               # [B, n, H]
    prev_idx = (starts - 1).clamp_min(0)
    vs = x[:, prev_idx].clone()                                        # [B, n, H, P]
    ks = k_rot[:, prev_idx].clone()
    vs[:, 0] = v_s
    ks[:, 0] = k_s
    cdt = hidden.dtype if scan is not None else torch.float32  # the kernels run in fp32
    scan = scan or SSDChunkScan.apply
    bh = lambda t: t.transpose(1, 2).reshape(B * H, *t.shape[1:2], *t.shape[3:]).contiguous().to(cdt)  # noqa: E731
    y, sf = scan(bh(q_rot), bh(kc), bh(x), adt.transpose(1, 2).reshape(B * H, T).contiguous().to(cdt),
                 ssm.reshape(B * H, P, S).contiguous().to(cdt), bh(vs), bh(ks),
                 cf.transpose(1, 2).reshape(B * H, nch).contiguous().to(cdt), C)
    y = y.to(hidden.dtype)
    sf = sf.to(hidden.dtype)
    y = y.view(B, H, T, P)
    v = x.transpose(1, 2)
    y = y + (self.d_skip[None, :, None, None] + qk_dot.transpose(1, 2)[..., None]) * v
    y = F.silu(z.transpose(1, 2)) * y
    out = y.transpose(1, 2).reshape(B, T, di) @ self.out_proj
    return out, {"ssm": sf.view(B, H, P, S), "angle": ang[:, -1], "k": k_rot[:, -1], "v": x[:, -1]}


Mamba3Params.forward_fused = _forward_fused

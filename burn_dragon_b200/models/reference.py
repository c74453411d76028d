"""Pure-PyTorch statement of the BDH math: the oracle every kernel is tested against,
and the CPU execution path.

Everything here follows the reference's own reference math:

* linear attention, strictly causal, read-before-update recurrence
  ``a_t = rho^T q_t ; rho <- (rho + q_t (x) v_t) * gamma``
  (burn_dragon_core/src/model/sequence/linear.rs:18-60) and its dense-score form
  ``S = tril_{-1}(Q Q^T) * gamma^(i-j)``, ``C = gamma^i Q rho0 + S V``,
  ``rho_T = gamma^T rho0 + (Q * gamma^(T-i))^T V`` (linear.rs:105-430);
* RoPE with frequencies ``theta^(-2 floor(i/2)/Nh) / 2pi``, wrapped phase
  ``frac(pos*freq)*2pi`` and adjacent (even, odd) pairs (attention.rs:488-575);
* the low-rank residual step (residual_stream.rs:323-572): x = relu(v W_x - thr),
  a = LN(LinAttn(rope(x), v)), y = relu(a W_y - thr), yn = x*y, m = LN(yn_flat E),
  v' = LN(v + m), with the single shared LayerNorm (norm.rs:302-327).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rope_freqs(latent: int, theta: float, device=None, dtype=torch.float32) -> torch.Tensor:
    """Per-column frequency in cycles per position (attention.rs:553-575)."""
    idx = torch.arange(latent, dtype=torch.float64)
    exponent = (torch.floor(idx / 2.0) * 2.0) / latent
    f = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64), exponent) / (2.0 * math.pi)
    return f.to(dtype=torch.float32).to(device=device, dtype=dtype)


def pope_freqs(latent: int, theta: float, device=None, dtype=torch.float32) -> torch.Tensor:
    """PoPE frequencies theta^(-i/Nh) / 2pi (attention.rs:561-564)."""
    idx = torch.arange(latent, dtype=torch.float64)
    f = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64), idx / latent) / (2.0 * math.pi)
    return f.to(dtype=torch.float32).to(device=device, dtype=dtype)


def pope_apply(x: torch.Tensor, phases: torch.Tensor) -> torch.Tensor:
    """softplus(x) as magnitude of a complex embedding: [|x| cos, |x| sin] (2 Nh wide;
    attention.rs:503-510)."""
    mag = F.softplus(x)
    return torch.cat([mag * torch.cos(phases).to(x.dtype), mag * torch.sin(phases).to(x.dtype)], dim=-1)


def make_norm(kind: str, gamma, beta, eps: float, alpha=None, shift=None):
    """DragonNorm (norm.rs:302-327): LayerNorm / RMSNorm / DynamicTanh / Derf, then x*gamma+beta."""
    def f(x):
        if kind == "layer_norm":
            return F.layer_norm(x, (x.shape[-1],), gamma, beta, eps)
        if kind == "rms_norm":
            y = x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps)
        elif kind == "dynamic_tanh":
            y = torch.tanh(x * alpha)
        elif kind == "derf":
            y = torch.erf(x * alpha + shift)
        else:
            raise ValueError(kind)
        return y * gamma + beta
    return f


def rope_phases(positions: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """phase[t, j] = frac(pos_t * f_j) * 2pi, computed in fp32 like the reference."""
    raw = positions.to(torch.float32)[:, None] * freqs.to(torch.float32)[None, :]
    return (raw - torch.floor(raw)) * (2.0 * math.pi)


def rope_apply(x: torch.Tensor, phases: torch.Tensor) -> torch.Tensor:
    """x * cos + rot(x) * sin with rot(x)[2i] = -x[2i+1], rot(x)[2i+1] = x[2i]."""
    cos = torch.cos(phases).to(x.dtype)
    sin = torch.sin(phases).to(x.dtype)
    pairs = x.reshape(*x.shape[:-1], x.shape[-1] // 2, 2)
    rot = torch.stack((-pairs[..., 1], pairs[..., 0]), dim=-1).reshape(x.shape)
    return x * cos + rot * sin


def decay_vector(slopes: list[float], device=None, dtype=torch.float32) -> torch.Tensor:
    """gamma_h = exp(-slope_h)."""
    return torch.exp(-torch.tensor(slopes, dtype=torch.float64)).to(device=device, dtype=dtype)


def linear_attention_recurrent(q, v, rho0=None, decay=None):
    """Time-step recurrence. q [B,H,T,N], v [B,1|H,T,D], rho0 [B,H,N,D], decay [H]."""
    B, H, T, N = q.shape
    D = v.shape[-1]
    v = v.expand(B, H, T, D)
    rho = rho0.clone() if rho0 is not None else q.new_zeros(B, H, N, D)
    outs = []
    g = decay.view(1, H, 1, 1) if decay is not None else None
    for t in range(T):
        qt = q[:, :, t, :]
        outs.append(torch.einsum("bhn,bhnd->bhd", qt, rho))
        rho = rho + qt[..., :, None] * v[:, :, t, None, :]
        if g is not None:
            rho = rho * g
    return torch.stack(outs, dim=2), rho


def _decay_powers(T: int, decay: torch.Tensor | None, device, dtype):
    """Gamma matrix gamma^(i-j) for j<i (0 elsewhere), and the gamma^i / gamma^(T-i) vectors."""
    i = torch.arange(T, device=device)
    diff = (i[:, None] - i[None, :]).to(dtype)
    mask = (i[None, :] < i[:, None]).to(dtype)
    if decay is None:
        return mask[None], None, None
    lg = torch.log(decay.to(dtype))[:, None, None]  # [H,1,1]
    gam = torch.exp(lg * diff.clamp_min(0)[None]) * mask[None]
    pow_i = torch.exp(torch.log(decay.to(dtype))[:, None] * i.to(dtype)[None, :])  # [H,T]
    pow_ti = torch.exp(torch.log(decay.to(dtype))[:, None] * (T - i).to(dtype)[None, :])
    return gam, pow_i, pow_ti


def linear_attention_dense(q, v, rho0=None, decay=None, need_state: bool = True):
    """Dense-score form (the reference's CUDA training executor)."""
    B, H, T, N = q.shape
    D = v.shape[-1]
    v = v.expand(B, H, T, D)
    gam, pow_i, pow_ti = _decay_powers(T, decay, q.device, q.dtype)
    s = torch.matmul(q, q.transpose(-1, -2)) * gam[None]
    c = torch.matmul(s, v)
    if rho0 is not None:
        init = torch.matmul(q, rho0)
        if pow_i is not None:
            init = init * pow_i[None, :, :, None]
        c = c + init
    rho = None
    if need_state:
        qw = q * pow_ti[None, :, :, None] if pow_ti is not None else q
        rho = torch.matmul(qw.transpose(-1, -2), v)
        if rho0 is not None:
            base = rho0 * (decay.view(1, H, 1, 1) ** T if decay is not None else 1.0)
            rho = rho + base
    return c, rho


def linear_attention_chunked(q, v, rho0=None, decay=None, need_state: bool = True, chunk: int = 512):
    """The dense-score form over row chunks of ``chunk`` positions with the state carried
    between them: chunk c computes its causal scores against itself only and reads the
    state that enters it (rho_c = gamma^c0 rho0 + sum_{j < c0} gamma^(c0-j) q_j^T v_j), so the
    scores take O(T chunk) memory instead of O(T^2) and the result (and its autograd
    gradient, which flows through the carried states) equals ``linear_attention_dense``.
    The reference's dense executor chunks its rows the same way (``dense_score_row_chunk``,
    burn_dragon_core/src/model/sequence/config.rs)."""
    T = q.shape[2]
    if chunk <= 0 or T <= chunk:
        return linear_attention_dense(q, v, rho0=rho0, decay=decay, need_state=need_state)
    outs, rho = [], rho0
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        vc = v[:, :, c0:c1]
        a, rho = linear_attention_dense(q[:, :, c0:c1], vc, rho0=rho, decay=decay,
                                        need_state=need_state or c1 < T)
        outs.append(a)
    return torch.cat(outs, dim=2), (rho if need_state else None)


def linear_attention_dense_vjp(q, v, dc, rho0=None, decay=None, drho=None):
    """Analytic backward of ``linear_attention_dense``: the data flow the fused backward
    runs on tensor cores (dense_causal_attention/backward_runtime.rs:36-148 in the
    reference). With S = (Q Q^T) . Gamma and P = dC V^T:

        dV    = sum_h S^T dC                      (+ (Q . g^(T-i))^T-side of drho)
        dS    = P . Gamma                         (strictly causal, decayed)
        dQ    = (dS + dS^T) Q                     (Q is both query and key)
                + (dC . g^i) rho0^T + (V drho^T) . g^(T-i)
        drho0 = Q^T (dC . g^i) + drho g^T

    ``v`` [B,1|H,T,D] (a broadcast value gets its head-sum); returns (dq, dv, drho0)."""
    B, H, T, N = q.shape
    D = v.shape[-1]
    ve = v.expand(B, H, T, D)
    gam, pow_i, pow_ti = _decay_powers(T, decay, q.device, q.dtype)
    s = torch.matmul(q, q.transpose(-1, -2)) * gam[None]
    dv = torch.matmul(s.transpose(-1, -2), dc)
    ds = torch.matmul(dc, ve.transpose(-1, -2)) * gam[None]
    dq = torch.matmul(ds + ds.transpose(-1, -2), q)
    drho0 = None
    if rho0 is not None:
        dci = dc * pow_i[None, :, :, None] if pow_i is not None else dc
        dq = dq + torch.matmul(dci, rho0.transpose(-1, -2))
        drho0 = torch.matmul(q.transpose(-1, -2), dci)
    if drho is not None:
        wt = pow_ti[None, :, :, None] if pow_ti is not None else 1.0
        dq = dq + torch.matmul(ve, drho.transpose(-1, -2)) * wt
        dv = dv + torch.matmul(q * wt, drho)
        if rho0 is not None:
            drho0 = drho0 + drho * (decay.view(1, H, 1, 1) ** T if decay is not None else 1.0)
    if v.shape[1] == 1 and H > 1:
        dv = dv.sum(1, keepdim=True)
    return dq, dv, drho0


def layer_norm(x, gamma, beta, eps):
    return F.layer_norm(x, (x.shape[-1],), gamma, beta, eps)


def bdh_layer(v, enc, enc_v, dec, gamma, beta, *, eps, thr, freqs, positions, decay, rho0=None,
              need_state=False, dropout=0.0, training=False, norm=None, pope=False, attention=None, thr_y=None,
              row_chunk: int = 0):
    """One shared-weight BDH layer. v [B,T,D]; enc/enc_v [H,D,Nh]; dec [N,D].
    ``norm`` overrides the LayerNorm (other DragonNorm kinds); ``pope`` switches the
    query embedding to PoPE (``freqs`` then holds the PoPE frequencies). ``thr`` is the
    x ReLU threshold, ``thr_y`` the y one (default: the same).

    ``row_chunk`` > 0: the attention runs over row chunks of that many positions with
    the state carried between them (``linear_attention_chunked``).

    Returns (v', rho_T or None, aux dict of the intermediate activations).
    """
    B, T, D = v.shape
    H, _, Nh = enc.shape
    nf = norm if norm is not None else (lambda z: layer_norm(z, gamma, beta, eps))
    x = torch.relu(torch.einsum("btd,hdn->bhtn", v, enc) - thr)  # [B,H,T,Nh]
    if freqs is None:
        q = x
    elif pope:
        q = pope_apply(x, rope_phases(positions, freqs)[None, None])
    else:
        q = rope_apply(x, rope_phases(positions, freqs)[None, None])
    if attention is not None:  # e.g. context parallelism: the sequence is split over ranks
        a, rho = attention(q, v[:, None])
    else:
        a, rho = linear_attention_chunked(q, v[:, None], rho0=rho0, decay=decay, need_state=need_state,
                                          chunk=row_chunk)
    a = nf(a)  # [B,H,T,D]
    y = torch.relu(torch.einsum("bhtd,hdn->bhtn", a, enc_v) - (thr if thr_y is None else thr_y))
    yn = x * y
    if dropout > 0.0 and training:
        yn = F.dropout(yn, dropout, training=True)
    m = yn.permute(0, 2, 1, 3).reshape(B, T, H * Nh) @ dec
    m = nf(m)
    v_next = nf(v + m)
    return v_next, rho, {"x": x, "q": q, "a": a, "y": y, "yn": yn}


def layer_weights(params: dict, cfg, layer: int, freqs):
    """The shared projections a layer uses: all of them, or under a latent fan-out
    schedule the first ``nh`` neurons of every head (encoder / encoder_v columns, the
    head's first ``nh`` decoder rows) with the RoPE / PoPE table cut to ``nh``."""
    enc, enc_v, dec = params["encoder"], params["encoder_v"], params["decoder"]
    nh = cfg.latent_per_head_for_layer(layer) if getattr(cfg, "latent_fanout_schedule", None) else enc.shape[-1]
    cap = enc.shape[-1]
    if nh == cap:
        return enc, enc_v, dec, freqs
    H = enc.shape[0]
    dec = dec.reshape(H, cap, -1)[:, :nh].reshape(H * nh, -1)
    return enc[..., :nh], enc_v[..., :nh], dec, None if freqs is None else freqs[:nh]


def bdh_forward(tokens, params: dict, cfg, rho0s=None, pos0: int = 0, need_state=False, training=False):
    """Full BDH forward (logits). params: embed [V,D], encoder, encoder_v, decoder,
    lm_head [D,V] (or None for tied), norm_gamma, norm_beta."""
    B, T = tokens.shape
    gamma, beta = params["norm_gamma"], params["norm_beta"]
    norm = make_norm(getattr(cfg, "norm_kind", "layer_norm"), gamma, beta, cfg.norm_eps, params.get("norm_alpha"),
                     params.get("norm_shift"))
    v = norm(params["embed"][tokens])
    Nh = cfg.latent_per_head
    freqs = None
    if cfg.rotary_embedding == "rope":
        freqs = rope_freqs(Nh, cfg.rope_theta, device=v.device, dtype=v.dtype)
    elif cfg.rotary_embedding == "pope":
        freqs = pope_freqs(Nh, cfg.rope_theta, device=v.device, dtype=v.dtype)
    decay = decay_vector(cfg.decay_slopes(), device=v.device, dtype=v.dtype) if cfg.uses_decay() else None
    positions = torch.arange(pos0, pos0 + T, device=v.device)
    rhos = []
    streams = getattr(cfg, "mhc_streams", 1)
    dyn = streams > 1 and getattr(cfg, "mhc_policy", "static_sinkhorn") == "dynamic_positive"
    if streams > 1:
        from . import mhc as MHC

        R = MHC.bootstrap(v, streams, params["mhc_boot"] if dyn else None)
    for layer in range(cfg.n_layer):
        r0 = rho0s[layer] if rho0s is not None else None
        if dyn:
            v, R, w_out = MHC.dynamic_split(R, params, layer, cfg.mhc_tau, cfg.mhc_iters)
        elif streams > 1:
            v, R = MHC.layer_split(R, params["mhc_res"][layer], params["mhc_pre"][layer], cfg.mhc_tau, cfg.mhc_iters)
        enc, enc_v, dec, fq = layer_weights(params, cfg, layer, freqs)
        v, rho, _ = bdh_layer(v, enc, enc_v, dec, gamma, beta,
                              eps=cfg.norm_eps, thr=cfg.thresholds()[0], thr_y=cfg.thresholds()[1], freqs=fq,
                              positions=positions,
                              decay=decay, rho0=r0, need_state=need_state, dropout=cfg.dropout,
                              training=training, norm=norm, pope=cfg.rotary_embedding == "pope",
                              row_chunk=getattr(cfg, "dense_score_row_chunk", 0) or 0)
        if dyn:
            R = MHC.dynamic_merge(R, v, w_out)
        elif streams > 1:
            R = MHC.layer_merge(R, v, params["mhc_post"][layer])
        rhos.append(rho)
    if streams > 1:
        v = R.mean(dim=1)
    head = params["embed"].t() if params.get("lm_head") is None else params["lm_head"]
    logits = v @ head
    return logits, rhos


def cross_entropy(logits, targets, mask=None):
    """Token-mean CE (language_head.rs:549-572), optional loss mask."""
    V = logits.shape[-1]
    lp = F.log_softmax(logits.reshape(-1, V).float(), dim=-1)
    nll = -lp.gather(1, targets.reshape(-1, 1)).squeeze(1)
    if mask is None:
        return nll.mean()
    w = mask.reshape(-1).to(nll.dtype)
    return (nll * w).sum() / w.sum().clamp_min(1.0)

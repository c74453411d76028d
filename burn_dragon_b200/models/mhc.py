"""Manifold-constrained hyper-connections (mHC): static-Sinkhorn and dynamic-positive
coefficient policies (burn_dragon_core/src/model/mhc/reference.rs:18-675,
mhc/config.rs:9-24).

The residual stream becomes S parallel streams R [B, S, T, D]. Per layer:
  H_res  = Sinkhorn(h_res / tau) (doubly stochastic S x S; iters of row / column
           log-softmax), initialised near the identity (diagonal 0, off-diagonal -8);
  H_pre  = softmax(h_pre, over streams) [V, S]: the branch input is the stream mixture
           sum_s H_pre[v, s] R_s (one view, V = 1);
  H_post = softmax(h_post, over streams) [V, S]: the branch output is distributed back,
  R <- H_res-mixed R + sum_v H_post[v, s] * branch_out_v.
The initial streams repeat the embedded input; the LM head reads the mean of the
streams. Only the PyTorch path implements mHC.

dynamic_positive (reference.rs:291-408): the coefficients become per-token functions of
the residual streams. Controller features f = flatten_s(R[b, :, t, :]) / rms(f) [S*D];
  branch input weights   sigmoid(h_pre[0]  + (f A_w + A_b) * sigmoid(g_A))   [S]
  branch output weights  sigmoid(h_post[0] + (f B_w + B_b) * sigmoid(g_B))   [S]
  residual weights       Sinkhorn(C_b + (f C_w) * sigmoid(g_C))               [S, S]
(positive sigmoids, not softmaxes; the controller weights start at zero and the gates
at sigmoid(-4.59512) ~ 0.01, C_b at the static h_res logits). The initial streams get a
small fixed bootstrap bias 1e-3 * (s - (S-1)/2) / S * ((d mod 7) / 6 - 1/2) so that
they differ (reference.rs:141-160).
"""

from __future__ import annotations

import torch


def sinkhorn(logits: torch.Tensor, tau: float = 1.0, iters: int = 10) -> torch.Tensor:
    z = logits / max(tau, 1e-6)
    for _ in range(iters):
        z = torch.log_softmax(z, dim=-1)
        z = torch.log_softmax(z, dim=-2)
    return z.exp()


def mix(streams: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """streams [B, S_in, T, D], w [S_in, S_out] -> [B, S_out, T, D]."""
    return torch.einsum("bitd,io->botd", streams, w)


SELECTED_STREAM_LOGIT = 2.0     # reference.rs:13
DYNAMIC_GATE_INIT_LOGIT = -4.59512  # reference.rs:12


def init_logits(n_layer: int, streams: int, views: int = 1, dim: int = 0,
                dynamic: bool = False) -> dict[str, torch.Tensor]:
    res = torch.full((n_layer, streams, streams), -8.0)
    pre = torch.full((n_layer, views, streams), -8.0)
    post = torch.full((n_layer, views, streams), -8.0)
    for l in range(n_layer):
        res[l].fill_diagonal_(0.0)
        pre[l, :, l % streams] = SELECTED_STREAM_LOGIT
        post[l, :, l % streams] = SELECTED_STREAM_LOGIT
    out = {"mhc_res": res, "mhc_pre": pre, "mhc_post": post}
    if dynamic:
        S, L = streams, n_layer
        out.update(dynamic_init(L, S, dim, res))
    return out


def dynamic_shapes(n_layer: int, streams: int, dim: int) -> dict[str, tuple[int, ...]]:
    S, L, F = streams, n_layer, streams * dim
    return {"mhc_alpha_w": (L, F, S), "mhc_alpha_b": (L, S), "mhc_alpha_gate": (L, 1),
            "mhc_beta_w": (L, F, S), "mhc_beta_b": (L, S), "mhc_beta_gate": (L, 1),
            "mhc_carry_w": (L, F, S * S), "mhc_carry_b": (L, S * S), "mhc_carry_gate": (L, 1),
            "mhc_boot": (S, dim)}


def dynamic_init(n_layer: int, streams: int, dim: int, res_logits: torch.Tensor) -> dict[str, torch.Tensor]:
    S, L = streams, n_layer
    out = {k: torch.zeros(shp) for k, shp in dynamic_shapes(L, S, dim).items()}
    for k in ("mhc_alpha_gate", "mhc_beta_gate", "mhc_carry_gate"):
        out[k].fill_(DYNAMIC_GATE_INIT_LOGIT)
    out["mhc_carry_b"].copy_(res_logits.reshape(L, S * S))
    center = (S - 1) * 0.5
    s_term = (torch.arange(S, dtype=torch.float32) - center) / S
    d_phase = (torch.arange(dim) % 7).float() / 6.0 - 0.5
    out["mhc_boot"].copy_(1e-3 * s_term[:, None] * d_phase[None, :])
    return out


def bootstrap(v: torch.Tensor, streams: int, boot: torch.Tensor | None) -> torch.Tensor:
    """[B, T, D] -> initial streams [B, S, T, D] (plus the bootstrap bias, dynamic policy)."""
    R = v[:, None].expand(v.shape[0], streams, v.shape[1], v.shape[2])
    return R + boot[None, :, None, :] if boot is not None else R


def controller_features(R: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """[B, S, T, D] -> per-token features [B, T, S*D] divided by their RMS."""
    B, S, T, D = R.shape
    f = R.permute(0, 2, 1, 3).reshape(B, T, S * D)
    return f / f.pow(2).mean(-1, keepdim=True).sqrt().clamp_min(eps)


def dynamic_split(R: torch.Tensor, p: dict, layer: int, tau: float, iters: int):
    """Dynamic-positive width connection: (branch input [B, T, D], mixed streams, output
    weights [B, T, S])."""
    B, S, T, D = R.shape
    f = controller_features(R)
    g = lambda k: torch.sigmoid(p[k][layer])  # noqa: E731
    w_in = torch.sigmoid(p["mhc_pre"][layer][0] + (f @ p["mhc_alpha_w"][layer] + p["mhc_alpha_b"][layer])
                         * g("mhc_alpha_gate"))                       # [B, T, S]
    w_out = torch.sigmoid(p["mhc_post"][layer][0] + (f @ p["mhc_beta_w"][layer] + p["mhc_beta_b"][layer])
                          * g("mhc_beta_gate"))                       # [B, T, S]
    carry = (p["mhc_carry_b"][layer] + (f @ p["mhc_carry_w"][layer]) * g("mhc_carry_gate")).reshape(B, T, S, S)
    w_res = sinkhorn(carry, tau, iters)                               # [B, T, S_in, S_out]
    branch_in = torch.einsum("bstd,bts->btd", R, w_in)
    mixed = torch.einsum("bitd,btio->botd", R, w_res)
    return branch_in, mixed, w_out


def dynamic_merge(R_mixed: torch.Tensor, branch_out: torch.Tensor, w_out: torch.Tensor) -> torch.Tensor:
    return R_mixed + torch.einsum("btd,bts->bstd", branch_out, w_out)


def layer_split(R: torch.Tensor, res_logits, pre_logits, tau: float, iters: int):
    """Returns (branch input [B, T, D], mixed residual streams)."""
    h_res = sinkhorn(res_logits, tau, iters)
    h_pre = torch.softmax(pre_logits, dim=-1)  # [V, S]
    branch_in = mix(R, h_pre.t())[:, 0]
    return branch_in, mix(R, h_res)


def layer_merge(R_mixed: torch.Tensor, branch_out: torch.Tensor, post_logits) -> torch.Tensor:
    h_post = torch.softmax(post_logits, dim=-1)  # [V, S]
    return R_mixed + mix(branch_out[:, None], h_post)

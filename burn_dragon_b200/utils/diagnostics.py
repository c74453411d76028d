"""Model and state diagnostics (interpretability probes).

Reference: burn_dragon_core/src/model/dragon/interpretability.rs (tensor distribution,
per-head geometry of the shared projections, weight comparisons, recurrent-state
summaries and deltas) and dragon/diagnostics.rs (collection entry points).

Everything is reduced on the tensor's device and returned as plain floats / dicts
(JSON-serialisable); nothing here is on a training hot path.
"""

from __future__ import annotations

import torch


def tensor_distribution(t: torch.Tensor) -> dict:
    """finite, mean, std, rms, mean|x|, max|x|, positive / nonzero / tiny (<0.1 rms)
    fractions, excess kurtosis."""
    x = t.detach().double().reshape(-1)
    if x.numel() == 0:
        return {"finite": True, "mean": 0.0, "std": 0.0, "rms": 0.0, "mean_abs": 0.0, "abs_max": 0.0,
                "positive_fraction": 0.0, "nonzero_fraction": 0.0, "tiny_fraction_0p1_rms": 0.0,
                "kurtosis_excess": None}
    mean = x.mean()
    c = x - mean
    var = c.pow(2).mean()
    rms = x.pow(2).mean().sqrt()
    kurt = float(c.pow(4).mean() / var.pow(2) - 3.0) if float(var) > 0 else None
    return {
        "finite": bool(torch.isfinite(x).all()),
        "mean": float(mean), "std": float(var.sqrt()), "rms": float(rms),
        "mean_abs": float(x.abs().mean()), "abs_max": float(x.abs().max()),
        "positive_fraction": float((x > 0).double().mean()),
        "nonzero_fraction": float((x != 0).double().mean()),
        "tiny_fraction_0p1_rms": float((x.abs() < 0.1 * rms).double().mean()),
        "kurtosis_excess": kurt,
    }


def head_geometry(w: torch.Tensor) -> dict:
    """Per-head geometry of a [H, rows, cols] tensor: head norms (mean, CV, max energy
    share), pairwise / nearest-neighbour cosine between flattened heads, stable rank
    ||W||_F^2 / sigma_max^2 and top-singular energy share."""
    w = w.detach().double()
    H = w.shape[0]
    flat = w.reshape(H, -1)
    norms = flat.norm(dim=1)
    energy = norms.pow(2)
    out = {"head_count": H, "rows": w.shape[1], "cols": w.shape[2],
           "mean_head_norm": float(norms.mean()),
           "head_norm_cv": float(norms.std(unbiased=False) / norms.mean().clamp_min(1e-30)),
           "max_head_energy_share": float(energy.max() / energy.sum().clamp_min(1e-30))}
    if H > 1:
        u = flat / norms.clamp_min(1e-30)[:, None]
        cos = u @ u.t()
        off = cos[~torch.eye(H, dtype=torch.bool)]
        out["pairwise_cosine_mean"] = float(off.mean())
        out["pairwise_cosine_max"] = float(off.max())
        out["nearest_neighbor_cosine_mean"] = float((cos - 2 * torch.eye(H, dtype=cos.dtype)).max(1).values.mean())
    else:
        out["pairwise_cosine_mean"] = out["pairwise_cosine_max"] = out["nearest_neighbor_cosine_mean"] = None
    sv = torch.linalg.svdvals(w)
    top = sv[:, 0].pow(2)
    fro = sv.pow(2).sum(1).clamp_min(1e-30)
    sr = fro / top.clamp_min(1e-30)
    out["stable_rank_mean"] = float(sr.mean())
    out["stable_rank_min"] = float(sr.min())
    out["top_singular_energy_mean"] = float((top / fro).mean())
    out["tensor"] = tensor_distribution(w)
    return out


def compare_tensors(a: torch.Tensor, b: torch.Tensor) -> dict:
    """cosine, relative L2 ||a - b|| / ||b||, mean |a - b|."""
    a, b = a.detach().double().reshape(-1), b.detach().double().reshape(-1)
    if a.shape != b.shape or a.numel() == 0:
        return {"cosine": None, "relative_l2": None, "mean_abs_delta": None}
    na, nb = a.norm(), b.norm()
    return {"cosine": float(a @ b / (na * nb)) if float(na * nb) > 0 else None,
            "relative_l2": float((a - b).norm() / nb) if float(nb) > 0 else None,
            "mean_abs_delta": float((a - b).abs().mean())}


def lowrank_geometry(model) -> dict:
    """Geometry of the shared projections of a ``BDH`` model (encoder / encoder_v as
    [H, D, Nh], the decoder as [H, Nh, D])."""
    p = model.param_dict()
    H = model.cfg.n_head
    dec = p["decoder"].reshape(H, -1, p["decoder"].shape[-1])
    return {"latent_per_head": model.cfg.latent_per_head, "encoder": head_geometry(p["encoder"]),
            "encoder_v": head_geometry(p["encoder_v"]), "decoder": head_geometry(dec)}


def compare_lowrank(model_a, model_b) -> dict:
    pa, pb = model_a.param_dict(), model_b.param_dict()
    H = model_a.cfg.n_head
    out = {}
    for n in ("encoder", "encoder_v", "decoder"):
        out[n] = compare_tensors(pa[n], pb[n])
        ha, hb = pa[n].reshape(H, -1), pb[n].reshape(H, -1)
        per = [compare_tensors(ha[h], hb[h]) for h in range(H)]
        cs = [c["cosine"] for c in per if c["cosine"] is not None]
        rl = [c["relative_l2"] for c in per if c["relative_l2"] is not None]
        out[n + "_heads"] = {"paired_head_cosine_mean": sum(cs) / len(cs) if cs else None,
                             "paired_head_relative_l2_mean": sum(rl) / len(rl) if rl else None}
    return out


def state_summary(t: torch.Tensor | None) -> dict:
    if t is None:
        return {"present": False, "finite": True, "rms": None, "mean_abs": None, "abs_max": None,
                "positive_fraction": None, "nonzero_fraction": None}
    d = tensor_distribution(t)
    return {"present": True, "finite": d["finite"], "rms": d["rms"], "mean_abs": d["mean_abs"],
            "abs_max": d["abs_max"], "positive_fraction": d["positive_fraction"],
            "nonzero_fraction": d["nonzero_fraction"]}


def state_delta(before: torch.Tensor | None, after: torch.Tensor | None) -> dict:
    out = {"present_before": before is not None, "present_after": after is not None, "cosine": None,
           "delta_rms": None, "relative_update": None, "after_rms": None}
    if after is not None:
        out["after_rms"] = float(after.detach().double().pow(2).mean().sqrt())
    if before is None or after is None or before.shape != after.shape:
        return out
    a, b = before.detach().double().reshape(-1), after.detach().double().reshape(-1)
    d = b - a
    out["cosine"] = float(a @ b / (a.norm() * b.norm())) if float(a.norm() * b.norm()) > 0 else None
    out["delta_rms"] = float(d.pow(2).mean().sqrt())
    out["relative_update"] = float(d.norm() / a.norm()) if float(a.norm()) > 0 else None
    return out


_STATE_FIELDS = ("rho", "slow_rho", "y_state", "clocked_hidden", "summary_hidden", "hier_slow")


def _layer_tensors(state, i: int) -> dict:
    if hasattr(state, "layers"):  # RuntimeState
        ls = state.layers[i]
        d = {f: getattr(ls, f) for f in _STATE_FIELDS}
        for k, v in (ls.mamba or {}).items():
            d[f"mamba_{k}"] = v
        return d
    return {"rho": None if state.rhos is None else state.rhos[i]}  # ModelState


def summarize_state(state, n_layer: int) -> list[dict]:
    return [{"layer_index": i, **{k: state_summary(v) for k, v in _layer_tensors(state, i).items()}}
            for i in range(n_layer)]


def compare_states(before, after, n_layer: int) -> list[dict]:
    out = []
    for i in range(n_layer):
        b, a = _layer_tensors(before, i), _layer_tensors(after, i)
        out.append({"layer_index": i, **{k: state_delta(b.get(k), a.get(k)) for k in sorted(set(a) | set(b))}})
    return out


def neuron_activity(model, tokens: torch.Tensor) -> list[dict]:
    """Per layer: distributions of x, y and x*y and the fraction of silent neurons
    (never positive over the batch) from a no-grad PyTorch-path forward."""
    from ..models import reference as R

    cfg = model.cfg
    p = model.param_dict()
    out = []
    with torch.no_grad():
        norm = R.make_norm(cfg.norm_kind, p["norm_gamma"], p["norm_beta"], cfg.norm_eps, p.get("norm_alpha"),
                           p.get("norm_shift"))
        v = norm(p["embed"][tokens])
        freqs = R.rope_freqs(cfg.latent_per_head, cfg.rope_theta, device=v.device) \
            if cfg.rotary_embedding == "rope" else None
        decay = R.decay_vector(cfg.decay_slopes(), device=v.device) if cfg.uses_decay() else None
        pos = torch.arange(tokens.shape[1], device=v.device)
        for i in range(cfg.n_layer):
            v, _, aux = R.bdh_layer(v, p["encoder"], p["encoder_v"], p["decoder"], p["norm_gamma"], p["norm_beta"],
                                    eps=cfg.norm_eps, thr=cfg.thresholds()[0], thr_y=cfg.thresholds()[1], freqs=freqs, positions=pos, decay=decay,
                                    norm=norm)
            yn = aux["yn"]
            silent = (yn.reshape(-1, yn.shape[1], yn.shape[-1]) > 0).any(0).logical_not().double().mean()
            out.append({"layer_index": i, "x": tensor_distribution(aux["x"]), "y": tensor_distribution(aux["y"]),
                        "yn": tensor_distribution(yn), "silent_neuron_fraction": float(silent),
                        "sparsity_x": 1.0 - tensor_distribution(aux["x"])["nonzero_fraction"]})
    return out

"""Local predictive-coding (PC) training for the Dragon layer stack.

The factor graph (burn_dragon_language/src/train/local_predictive_coding.rs:70-115):
activity nodes ``a_0 .. a_L`` ([B, T, D] each; ``a_0`` = the normalised embedding,
clamped), one factor per layer predicting ``a_{l+1}`` from ``a_l`` with the shared BDH
layer, and a terminal next-token factor on ``a_L``. Energy::

    E = s * ( p/2 * sum_l ||f_l(a_l) - a_{l+1}||^2 + CE_sum(head(a_L)) )

with precision ``p`` and factor scale ``s`` (1, or 1/(L+1) for ``mean`` reduction).

Step (local_predictive_coding.rs:680-1030):

1. feed-forward pass initialises every activity (predictions = activities);
2. activity inference for ``steps`` iterations: ``synchronous_equilibrium`` updates
   all free activities from one trace; ``reverse_gauss_seidel`` sweeps from the last
   activity to the first, each update using the already-updated child. The update is
   SGD on ``dE/da`` with a per-row gradient-norm clip (``max_grad_norm``) and optional
   ``latent_decay`` (the burn_pc inference rule);
3. parameter derivatives are layer-local: each factor's VJP with its inputs held fixed,
   prediction errors divided by the supervised-token count, plus the head's CE
   gradient at ``a_L`` and the embedding gradient through ``a_0``.

``fixed_prediction`` keeps the feed-forward activities and chains the factor VJPs from
the head back to the embedding, which is ordinary backpropagation.

Here every "local VJP" is an autograd call on one factor whose inputs are detached
tensors, so no gradient crosses a factor boundary.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..config import LocalPredictiveCodingConfig, PCInferenceConfig  # noqa: F401 (re-exported)
from ..models import reference as R


@dataclass
class PCStepReport:
    solver: str
    inference_steps: int
    factors: int
    local_vjp_calls: int
    global_backward_calls: int
    energy_before: float | None = None
    energy_after: float | None = None


class _Stack:
    """The model pieces the factors need, bound once per step."""

    def __init__(self, model, tokens):
        cfg = model.cfg
        self.cfg = cfg
        self.p = model.param_dict()
        p = self.p
        self.norm = R.make_norm(cfg.norm_kind, p["norm_gamma"], p["norm_beta"], cfg.norm_eps, p.get("norm_alpha"),
                                p.get("norm_shift"))
        T = tokens.shape[1]
        self.freqs = None
        if cfg.rotary_embedding in ("rope", "pope"):
            f = R.rope_freqs if cfg.rotary_embedding == "rope" else R.pope_freqs
            self.freqs = f(cfg.latent_per_head, cfg.rope_theta, device=tokens.device)
        self.decay = R.decay_vector(cfg.decay_slopes(), device=tokens.device) if cfg.uses_decay() else None
        self.pos = torch.arange(T, device=tokens.device)
        self.head = p["embed"].t() if p.get("lm_head") is None else p["lm_head"]

    def layer(self, a, rho0=None, need_state=False):
        c = self.cfg
        out, rho, _ = R.bdh_layer(a, self.p["encoder"], self.p["encoder_v"], self.p["decoder"], self.p["norm_gamma"],
                                  self.p["norm_beta"], eps=c.norm_eps, thr=c.thresholds()[0], thr_y=c.thresholds()[1], freqs=self.freqs,
                                  positions=self.pos, decay=self.decay, rho0=rho0, need_state=need_state,
                                  norm=self.norm, pope=c.rotary_embedding == "pope")
        return out, rho

    def ce_sum(self, a, targets, mask):
        lp = F.log_softmax((a @ self.head).float(), -1)
        nll = -lp.gather(-1, targets.unsqueeze(-1)).squeeze(-1)
        w = torch.ones_like(nll) if mask is None else mask.to(nll.dtype)
        return (nll * w).sum(), w.sum()


def _detach_params(p: dict) -> dict:
    return {k: (v.detach() if isinstance(v, torch.Tensor) else v) for k, v in p.items()}


def _sgd(a, g, inf: PCInferenceConfig):
    if inf.latent_decay:
        g = g + inf.latent_decay * a
    if inf.max_grad_norm is not None:
        if inf.gradient_norm_scope == "per_row":
            n = g.norm(dim=-1, keepdim=True)
        else:
            n = g.norm()
        g = g * (inf.max_grad_norm / (n + inf.eps)).clamp(max=1.0)
    return a - inf.step_size * g


def local_pc_step(model, tokens, targets, cfg: LocalPredictiveCodingConfig, mask=None, rho0s=None):
    """One PC step on a ``BDH`` model: writes every parameter's ``.grad`` (the flat
    gradient buffer) and returns (feed-forward loss, report)."""
    if cfg.learning_schedule != "equilibrium":
        raise ValueError("local predictive coding supports only learning_schedule = \"equilibrium\"")
    L = model.cfg.n_layer
    scale = 1.0 if cfg.factor_reduction == "sum" else 1.0 / (L + 1)
    prec = cfg.prediction_precision
    params = [p for p in model.parameters()]
    st = _Stack(model, tokens)
    rho0s = rho0s or [None] * L

    # 1. feed-forward initialisation (no parameter graph)
    with torch.no_grad():
        a0 = st.norm(st.p["embed"][tokens])
        acts = [a0]
        for layer in range(L):
            acts.append(st.layer(acts[-1], rho0s[layer])[0])
        ce, ntok = st.ce_sum(acts[-1], targets, mask)
        ff_loss = ce / ntok.clamp_min(1)
    calls = 0
    report = PCStepReport(cfg.solver, cfg.inference.steps, L + 1, 0, 0)

    if cfg.solver == "fixed_prediction":
        # chained factor VJPs == backpropagation from the head to the embedding
        st_g = _Stack(model, tokens)
        a = st_g.norm(st_g.p["embed"][tokens])
        for layer in range(L):
            a = st_g.layer(a, rho0s[layer])[0]
        ce, ntok = st_g.ce_sum(a, targets, mask)
        loss = ce / ntok.clamp_min(1) * scale
        grads = torch.autograd.grad(loss, params, allow_unused=True)
        _write(model, grads)
        report.local_vjp_calls = L + 2
        report.inference_steps = 1
        return ff_loss.detach(), report

    # frozen-parameter view for activity inference
    frozen = _Stack(model, tokens)
    frozen.p = _detach_params(frozen.p)
    frozen.head = frozen.head.detach()
    frozen.norm = R.make_norm(model.cfg.norm_kind, frozen.p["norm_gamma"], frozen.p["norm_beta"], model.cfg.norm_eps,
                              frozen.p.get("norm_alpha"), frozen.p.get("norm_shift"))

    def energy(activities):
        e = 0.0
        for layer in range(L):
            pred = frozen.layer(activities[layer], rho0s[layer])[0]
            e = e + 0.5 * prec * (pred - activities[layer + 1]).pow(2).sum()
        return scale * (e + frozen.ce_sum(activities[-1], targets, mask)[0])

    if cfg.sync_diagnostics:
        with torch.no_grad():
            report.energy_before = float(energy(acts))
    acts = [a.detach() for a in acts]
    for _ in range(cfg.inference.steps):
        if cfg.solver == "synchronous_equilibrium":
            free = [a.requires_grad_(True) for a in acts[1:]]
            e = energy([acts[0]] + free)
            g = torch.autograd.grad(e, free)
            calls += L + 1
            acts = [acts[0]] + [_sgd(a.detach(), gi, cfg.inference).detach() for a, gi in zip(free, g)]
        elif cfg.solver == "reverse_gauss_seidel":
            with torch.no_grad():
                preds = [frozen.layer(acts[layer], rho0s[layer])[0] for layer in range(L)]
            for i in range(L, 0, -1):
                ai = acts[i].detach().requires_grad_(True)
                own = prec * scale * (ai - preds[i - 1])
                if i == L:
                    child_e = scale * frozen.ce_sum(ai, targets, mask)[0]
                else:
                    child_e = 0.5 * prec * scale * (frozen.layer(ai, rho0s[i])[0] - acts[i + 1]).pow(2).sum()
                child = torch.autograd.grad(child_e, ai)[0]
                calls += 1
                acts[i] = _sgd(ai.detach(), own.detach() + child, cfg.inference).detach()
        else:
            raise ValueError(f"unknown predictive-coding solver {cfg.solver!r}")
    if cfg.sync_diagnostics:
        with torch.no_grad():
            report.energy_after = float(energy(acts))

    # 3. layer-local parameter derivatives at the inferred activities
    st_g = _Stack(model, tokens)
    a0 = st_g.norm(st_g.p["embed"][tokens])
    n = None
    ce, ntok = st_g.ce_sum(acts[-1], targets, mask)
    n = ntok.clamp_min(1)
    total = scale * ce / n
    for layer in range(L):
        inp = a0 if layer == 0 else acts[layer]
        pred = st_g.layer(inp, rho0s[layer])[0]
        total = total + scale * 0.5 * prec * (pred - acts[layer + 1]).pow(2).sum() / n
    grads = torch.autograd.grad(total, params, allow_unused=True)
    _write(model, grads)
    report.local_vjp_calls = calls + L + 1
    return ff_loss.detach(), report


def _write(model, grads):
    """Store the derivatives in the model's flat gradient buffer."""
    for (name, _), g in zip(model.named_parameters(), grads):
        view = model.store.view(model.store.grad, name)
        if g is None:
            view.zero_()
        else:
            view.copy_(g)


# ------------------------------------------------------------------ gradient fidelity
def _stats(pc: torch.Tensor, ref: torch.Tensor, family: str, present: bool | None) -> dict:
    """Agreement of a PC derivative with the exact gradient (cosine, norm ratio, relative
    L2 error, least-squares scale, sign agreement) as in the reference's diagnostics
    (burn_dragon_language/src/train/local_predictive_coding/diagnostics.rs:16-120)."""
    p, r = pc.double().reshape(-1), ref.double().reshape(-1)
    return _finish({"elements": p.numel(), "dot": float(p @ r), "pc2": float(p @ p), "ref2": float(r @ r),
                    "err2": float((p - r).pow(2).sum()), "nonneg": float((p * r >= 0).double().sum())},
                   family, present)


def _finish(raw: dict, family: str, present: bool | None) -> dict:
    def ratio(a, b):
        return a / b if abs(b) > 1e-30 and math.isfinite(a / b) else None

    pn, rn = math.sqrt(max(raw["pc2"], 0.0)), math.sqrt(max(raw["ref2"], 0.0))
    return {"parameter_family": family, "elements": raw["elements"], "reference_gradient_present": present,
            "dot_product": raw["dot"], "pc_norm": pn, "reference_norm": rn, "cosine": ratio(raw["dot"], pn * rn),
            "pc_to_reference_norm_ratio": ratio(pn, rn),
            "relative_l2_error": ratio(math.sqrt(max(raw["err2"], 0.0)), rn),
            "least_squares_scale": ratio(raw["dot"], raw["pc2"]),
            "nonnegative_product_fraction": raw["nonneg"] / raw["elements"] if raw["elements"] else 0.0,
            "_raw": raw}


def pc_gradient_fidelity(model, tokens, targets, cfg: LocalPredictiveCodingConfig, mask=None, rho0s=None) -> dict:
    """One local-PC derivative step against exact backpropagation of the same masked
    next-token loss (an offline diagnostic: it runs one global backward)."""
    loss_pc, report = local_pc_step(model, tokens, targets, cfg, mask=mask, rho0s=rho0s)
    pc = {n: model.store.view(model.store.grad, n).clone() for n, _ in model.named_parameters()}
    names = [n for n, _ in model.named_parameters()]
    params = [p for _, p in model.named_parameters()]
    from ..models.state import ModelState

    st = None if rho0s is None else ModelState([r.detach() for r in rho0s], 0)
    ref_loss = R.cross_entropy(model(tokens, state=st), targets, mask)
    ref = torch.autograd.grad(ref_loss, params, allow_unused=True)
    fams, tot = [], None
    for n, p, g in zip(names, params, ref):
        f = _stats(pc[n], torch.zeros_like(p) if g is None else g, n, g is not None)
        fams.append(f)
        raw = f["_raw"]
        tot = dict(raw) if tot is None else {k: tot[k] + raw[k] for k in tot}
    glob = _finish(tot, "global", None)
    for f in fams + [glob]:
        f.pop("_raw")
    lp, lr = float(loss_pc), float(ref_loss.detach())
    return {"pc_loss": lp, "reference_loss": lr, "loss_absolute_error": abs(lp - lr), "reference_backward_calls": 1,
            "pc_step": {"solver": report.solver, "inference_steps": report.inference_steps,
                        "factors": report.factors, "local_vjp_calls": report.local_vjp_calls,
                        "global_backward_calls": report.global_backward_calls},
            "global": glob, "parameter_families": fams}

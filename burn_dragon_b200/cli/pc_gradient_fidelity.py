"""Local predictive-coding gradient fidelity sweep: for each solver setting (inference
steps x step size) one PC derivative step is compared with exact backpropagation of the
same masked next-token loss on one synthetic batch; one JSON document with every arm
(the reference's pc_gradient_fidelity example,
burn_dragon_language/examples/pc_gradient_fidelity.rs).

  python -m burn_dragon_b200.cli.pc_gradient_fidelity [--backend cpu|cuda]
         [--solver synchronous_equilibrium|reverse_gauss_seidel|fixed_prediction] [--seed N]
         [--n-layer N --n-embd N --n-head N --latent-total N --vocab-size N]
         [--batch-size N --block-size N] [--inference-steps 1,2,4,8] [--step-sizes 0.01,0.05,0.1]
         [--max-grad-norm N|none] [--mask-period N]

The loss mask drops every ``mask-period``-th token (0: no mask).
"""

from __future__ import annotations

import argparse
import copy
import json

import torch

from ..config import DragonConfig, LocalPredictiveCodingConfig, PCInferenceConfig
from ..models.bdh import BDH
from ..train.predictive_coding import pc_gradient_fidelity


def _ints(s):
    return [int(x) for x in s.split(",") if x]


def _floats(s):
    return [float(x) for x in s.split(",") if x]


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser()
    ap.add_argument("--backend", choices=("cpu", "cuda"), default="cpu")
    ap.add_argument("--solver", default="synchronous_equilibrium",
                    choices=("synchronous_equilibrium", "reverse_gauss_seidel", "fixed_prediction"))
    ap.add_argument("--seed", type=int, default=20260804)
    ap.add_argument("--n-layer", type=int, default=4)
    ap.add_argument("--n-embd", type=int, default=96)
    ap.add_argument("--n-head", type=int, default=4)
    ap.add_argument("--latent-total", type=int, default=3072)
    ap.add_argument("--vocab-size", type=int, default=272)
    ap.add_argument("--batch-size", type=int, default=32)
    ap.add_argument("--block-size", type=int, default=128)
    ap.add_argument("--inference-steps", type=_ints, default=[1, 2, 4, 8])
    ap.add_argument("--step-sizes", type=_floats, default=[0.01, 0.05, 0.1])
    ap.add_argument("--max-grad-norm", default="1.0")
    ap.add_argument("--mask-period", type=int, default=5)
    a = ap.parse_args(argv)
    dev = torch.device(a.backend if a.backend == "cpu" else "cuda")
    if a.latent_total % a.n_embd:
        raise SystemExit("--latent-total must be a multiple of --n-embd")
    cfg = DragonConfig(n_layer=a.n_layer, n_embd=a.n_embd, n_head=a.n_head,
                       mlp_internal_dim_multiplier=a.latent_total // a.n_embd, vocab_size=a.vocab_size, dropout=0.0)
    cfg.validate()
    g = torch.Generator().manual_seed(a.seed)
    stream = torch.randint(0, a.vocab_size, (a.batch_size, a.block_size + 1), generator=g)
    x, y = stream[:, :-1].to(dev), stream[:, 1:].to(dev)
    mask = None
    if a.mask_period > 0:
        idx = torch.arange(a.batch_size * a.block_size).reshape(a.batch_size, a.block_size)
        mask = (idx % a.mask_period != 0).to(torch.int64).to(dev)
    base = BDH(cfg, device=dev, seed=a.seed)
    mgn = None if a.max_grad_norm.lower() == "none" else float(a.max_grad_norm)
    arms = []
    steps = [1] if a.solver == "fixed_prediction" else a.inference_steps
    sizes = [0.0] if a.solver == "fixed_prediction" else a.step_sizes
    for k in steps:
        for lr in sizes:
            model = copy.deepcopy(base)
            pcc = LocalPredictiveCodingConfig(solver=a.solver,
                                              inference=PCInferenceConfig(steps=k, step_size=lr, max_grad_norm=mgn))
            arms.append({"solver": a.solver, "inference_steps": k, "step_size": lr, "max_grad_norm": mgn,
                         "report": pc_gradient_fidelity(model, x, y, pcc, mask=mask)})
    out = {"backend": a.backend, "seed": a.seed, "n_layer": a.n_layer, "n_embd": a.n_embd, "n_head": a.n_head,
           "latent_total": a.latent_total, "vocab_size": a.vocab_size, "batch_size": a.batch_size,
           "block_size": a.block_size, "mask_period": a.mask_period, "arms": arms}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    main()

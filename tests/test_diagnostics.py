"""Diagnostics: tensor distributions, head geometry, comparisons, state summaries (CPU)."""

import json

import torch

from burn_dragon_b200.config import DragonConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.models.dragon_runtime import DragonRuntime, RuntimeState
from burn_dragon_b200.models.state import ModelState
from burn_dragon_b200.utils import diagnostics as DG


def cfg():
    return DragonConfig(n_layer=2, n_embd=16, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope", initialization="simple_normal", vocab_size=32)


def test_distribution_and_geometry():
    d = DG.tensor_distribution(torch.tensor([1.0, -1.0, 0.0, 2.0]))
    assert d["finite"] and abs(d["mean"] - 0.5) < 1e-12 and d["positive_fraction"] == 0.5
    assert d["nonzero_fraction"] == 0.75 and d["abs_max"] == 2.0
    # two identical heads: cosine 1, rank-1 heads: stable rank 1
    h = torch.outer(torch.arange(1.0, 4.0), torch.ones(5))
    g = DG.head_geometry(torch.stack([h, h]))
    assert abs(g["pairwise_cosine_mean"] - 1.0) < 1e-9 and abs(g["stable_rank_min"] - 1.0) < 1e-9
    assert abs(g["max_head_energy_share"] - 0.5) < 1e-12 and abs(g["head_norm_cv"]) < 1e-12


def test_model_and_state_diagnostics_are_json():
    m = BDH(cfg(), seed=0)
    geo = DG.lowrank_geometry(m)
    cmp_ = DG.compare_lowrank(m, BDH(cfg(), seed=0))
    assert abs(cmp_["encoder"]["cosine"] - 1.0) < 1e-9 and cmp_["decoder"]["relative_l2"] == 0.0
    t = torch.randint(0, 32, (2, 6))
    acts = DG.neuron_activity(m, t)
    assert len(acts) == 2 and 0.0 <= acts[0]["silent_neuron_fraction"] <= 1.0
    st = ModelState.empty()
    m.forward(t, state=st)
    before = ModelState([r.clone() for r in st.rhos], st.position)
    m.forward(t, state=st)
    delta = DG.compare_states(before, st, 2)
    assert delta[0]["rho"]["relative_update"] > 0
    rt = DragonRuntime(cfg(), seed=0)
    rs = RuntimeState.new(2)
    rt.forward(t, rs)
    summ = DG.summarize_state(rs, 2)
    assert summ[0]["rho"]["present"] and not summ[0]["y_state"]["present"]
    json.dumps({"geo": geo, "acts": acts, "delta": delta, "summ": summ})

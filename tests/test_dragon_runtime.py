"""Layer-loop variants on the PyTorch path: connectors, auxiliary memories, hierarchical
cycles, rollout fast steps, latent-reasoning heads (CPU)."""

import copy

import pytest
import torch

from burn_dragon_b200.config import DragonConfig, training_config_from_dict
from burn_dragon_b200.models.dragon_runtime import DragonRuntime, RuntimeState


def tiny(**kw) -> DragonConfig:
    c = DragonConfig(n_layer=3, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                     rotary_embedding="rope", initialization="simple_normal", vocab_size=64)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def toks(B=2, T=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 64, (B, T), generator=g)


def test_plain_runtime_matches_bdh_reference_path():
    cfg = tiny()
    rt = DragonRuntime(cfg, seed=3)
    t = toks()
    ref = rt.core.forward(t)
    got = rt.forward(t)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rot", ["rope", "alibi"])
def test_state_carry_token_by_token_equals_full_pass(rot):
    cfg = tiny(rotary_embedding=rot)
    rt = DragonRuntime(cfg, seed=1)
    t = toks(T=6)
    full = rt.forward(t)
    st = RuntimeState.new(cfg.n_layer)
    parts = [rt.forward(t[:, i:i + 1], st) for i in range(6)]
    torch.testing.assert_close(torch.cat(parts, 1), full, rtol=1e-4, atol=1e-5)
    assert st.position == 6


def test_y_neuron_recurrence_chunked_state_and_stabilization():
    cfg = tiny()
    cfg.y_neuron_recurrence.enabled = True
    cfg.y_neuron_recurrence.state_rms_cap = 0.5
    rt = DragonRuntime(cfg, seed=2)
    t = toks(T=6)
    st = RuntimeState.new(cfg.n_layer)
    full = rt.forward(t, st)
    for ls in st.layers:
        rms = ls.y_state.pow(2).mean(-1).sqrt()
        assert float(rms.max()) <= 0.5 + 1e-5
    st2 = RuntimeState.new(cfg.n_layer)
    parts = [rt.forward(t[:, i:i + 2], st2) for i in range(0, 6, 2)]
    torch.testing.assert_close(torch.cat(parts, 1), full, rtol=1e-4, atol=1e-5)
    # the carry changes the output relative to the plain model
    assert not torch.allclose(full, rt.core.forward(t), atol=1e-4)
    # carry_in_scale 0 keeps the state but does not inject it
    cfg0 = copy.deepcopy(cfg)
    cfg0.y_neuron_recurrence.carry_in_scale = 0.0
    rt0 = DragonRuntime(cfg0, seed=2)
    torch.testing.assert_close(rt0.forward(t), rt0.core.forward(t), rtol=1e-4, atol=1e-5)


def test_y_neuron_last_layers_limits_recurrence():
    cfg = tiny()
    cfg.y_neuron_recurrence.enabled = True
    cfg.y_neuron_recurrence.last_layers = 1
    rt = DragonRuntime(cfg, seed=2)
    st = RuntimeState.new(cfg.n_layer)
    rt.forward(toks(), st)
    assert st.layers[0].y_state is None and st.layers[1].y_state is None
    assert st.layers[2].y_state is not None


def test_summary_memory_chunks_and_write_trigger():
    cfg = tiny()
    sm = cfg.summary_memory
    sm.enabled, sm.chunk_tokens, sm.surprise_gate_threshold = True, 4, 0.01
    rt = DragonRuntime(cfg, seed=4)
    t = toks(T=8)
    full = rt.forward(t)
    st = RuntimeState.new(cfg.n_layer)
    parts = [rt.forward(t[:, :4], st), rt.forward(t[:, 4:], st)]
    torch.testing.assert_close(torch.cat(parts, 1), full, rtol=1e-4, atol=1e-5)
    # first chunk sees no carry: identical to the plain model on its tokens
    torch.testing.assert_close(full[:, :4], rt.core.forward(t[:, :4]), rtol=1e-4, atol=1e-5)
    # with a write trigger and no events the carry stays zero
    sm.write_trigger_token_ids = [5]
    st = RuntimeState.new(cfg.n_layer)
    rt.forward(t, st)
    assert all(float(ls.summary_hidden.abs().max()) == 0.0 for ls in st.layers)
    ev = torch.zeros_like(t)
    ev[:, 1] = 1
    st = RuntimeState.new(cfg.n_layer)
    rt.forward(t, st, event_mask=ev)
    assert float(st.layers[0].summary_hidden.abs().max()) > 0


def test_clocked_slow_memory_cached_token_path():
    cfg = tiny()
    cs = cfg.clocked_slow_memory
    cs.enabled, cs.chunk_tokens, cs.last_layers = True, 4, 2
    rt = DragonRuntime(cfg, seed=5)
    t = toks(T=8)
    st = RuntimeState.new(cfg.n_layer)
    full = rt.forward(t, st)
    assert full.shape == (2, 8, 64)
    assert st.layers[0].clocked_hidden is None and st.layers[2].clocked_hidden.shape == (2, 1, 32)
    # a single token at a non-boundary position reuses the cached slow hidden (no rho update)
    rho_before = st.layers[2].rho.clone()
    st.position = 9
    rt.forward(t[:, :1], st)
    torch.testing.assert_close(st.layers[2].rho, rho_before)


@pytest.mark.parametrize("split", [False, True])
def test_hierarchical_dragon_cycles_and_split(split):
    cfg = tiny()
    hd = cfg.hierarchical_dragon
    hd.enabled, hd.fast_cycles, hd.slow_cycles = True, 2, 2
    if split:
        hd.rho_sharing = hd.weight_sharing = "split"
    rt = DragonRuntime(cfg, seed=6)
    st = RuntimeState.new(cfg.n_layer)
    t = toks(T=4)
    loss = rt.loss(t, toks(T=4, seed=9), state=st)
    loss.backward()
    assert torch.isfinite(loss)
    assert st.layers[0].hier_slow.shape == (2, 1, 32)
    assert (st.layers[0].slow_rho is not None) == split
    if split:
        assert rt.slow_encoder.grad is not None and float(rt.slow_encoder.grad.abs().sum()) > 0


def test_attention_residual_zero_gate_is_identity_and_history_is_deltas():
    cfg = tiny(residual_connector="attention_residual")
    rt = DragonRuntime(cfg, seed=7)
    cur = torch.randn(2, 5, 32)
    hist = [torch.randn(2, 5, 32) for _ in range(3)]
    torch.testing.assert_close(rt.attn_res.attend(cur, hist), cur)
    with torch.no_grad():
        rt.attn_res.mix_gate.fill_(10.0)  # tanh -> 1: pure history mix
    out = rt.attn_res.attend(cur, hist[:1])
    torch.testing.assert_close(out, hist[0], rtol=1e-5, atol=1e-5)
    logits = rt.forward(toks())
    assert torch.isfinite(logits).all()


def test_block_attention_residual_candidate_layout():
    cfg = tiny(residual_connector="block_attention_residual")
    cfg.block_attention_residual.layers_per_block = 2
    cfg.block_attention_residual.summary_mode = "mean_pool"
    rt = DragonRuntime(cfg, seed=8)
    hist = [torch.full((1, 1, 32), float(i)) for i in range(5)]
    c = rt.attn_res.candidates(hist[0], hist)
    # 5 entries, local window 2 -> raw [3, 4]; older 3 -> blocks [0,1] and [2]
    vals = [float(x.mean()) for x in c]
    assert vals == [0.5, 2.0, 3.0, 4.0]
    assert torch.isfinite(rt.forward(toks())).all()


def test_rollout_fast_steps_modes():
    t = toks(T=3)
    base = DragonRuntime(tiny(), seed=10)
    st = RuntimeState.new(3)
    one = DragonRuntime(tiny(rollout_fast_steps_per_slow_step=1), seed=10).forward(t, st)
    torch.testing.assert_close(one, base.forward(t))
    for mode in ("host_loop", "fused"):
        rt = DragonRuntime(tiny(rollout_fast_steps_per_slow_step=4), seed=10, rollout_mode=mode)
        st = RuntimeState.new(3)
        out = rt.forward(t, st)
        assert out.shape == (2, 3, 64) and st.position == 3
        assert torch.isfinite(out).all()
    # fused rollout of one token == the token repeated F times at a fixed position
    rt = DragonRuntime(tiny(rollout_fast_steps_per_slow_step=2), seed=10)
    st = RuntimeState.new(3)
    out = rt.forward(t[:, :1], st)
    st2 = RuntimeState.new(3)
    emb = rt.core.param_dict()["embed"][t[:, :1]].expand(-1, 2, -1)
    h = rt.hidden_single_pass(emb, st2, 0, fixed=True)[:, -1:]
    torch.testing.assert_close(out, rt.logits_from_hidden(h))


def test_latent_reasoning_zero_init_gate_and_halting():
    cfg = tiny()
    lr = cfg.latent_reasoning
    lr.enabled, lr.max_steps, lr.min_steps = True, 3, 1
    rt = DragonRuntime(cfg, seed=11)
    h = torch.randn(2, 4, 32)
    torch.testing.assert_close(rt.reason_hidden_final(h), h)  # zero-initialised refiner output
    with torch.no_grad():
        rt.refiner_out.weight.normal_(0, 0.1)
    cfg_g = copy.deepcopy(cfg)
    cfg_g.latent_reasoning.residual_refinement_gate = True
    cfg_g.latent_reasoning.max_steps = cfg_g.latent_reasoning.min_steps = 1
    rg = DragonRuntime(cfg_g, seed=11)
    rg.refiner_in.load_state_dict(rt.refiner_in.state_dict())
    rg.refiner_out.load_state_dict(rt.refiner_out.state_dict())
    gated = rg.reason_hidden_final(h) - h
    with torch.no_grad():
        rg.refiner_gate.fill_(40.0)
    open_ = rg.reason_hidden_final(h) - h
    torch.testing.assert_close(gated, open_ * 0.25, rtol=1e-4, atol=1e-6)
    # adaptive halting: a large stop bias halts every position at min_steps
    cfg_h = copy.deepcopy(cfg)
    cfg_h.latent_reasoning.adaptive_halting = True
    cfg_h.latent_reasoning.min_steps = 2
    cfg_h.latent_reasoning.stop_bias_init = 50.0
    rh = DragonRuntime(cfg_h, seed=11)
    rh.refiner_in.load_state_dict(rt.refiner_in.state_dict())
    rh.refiner_out.load_state_dict(rt.refiner_out.state_dict())
    out = rh.reason_hidden(h)
    assert len(out.step_hiddens) == 3 and len(out.stop_probs) == 3
    assert float(out.stop_probs[0].abs().max()) == 0.0
    torch.testing.assert_close(out.final_hidden, out.step_hiddens[1])


def test_step_conditioned_decoder_and_aux_heads():
    cfg = tiny()
    cfg.latent_reasoning.enabled = True
    cfg.latent_reasoning.step_conditioned_decoder = True
    cfg.latent_reasoning.max_steps = 2
    cfg.next_latent_transition.enabled = True
    cfg.sequence_score_head.enabled = True
    rt = DragonRuntime(cfg, seed=12)
    h = torch.randn(1, 3, 32)
    with torch.no_grad():
        rt.step_decoder_embedding[2].fill_(1.0)
    head = rt.core.param_dict()["lm_head"]
    torch.testing.assert_close(rt.logits_from_hidden(h), (h + 1.0) @ head)
    torch.testing.assert_close(rt.logits_from_hidden(h, step=0), h @ head)
    # zero-initialised transition output: prediction == hidden
    torch.testing.assert_close(rt.next_latent_prediction(h, torch.randn(1, 3, 32)), h)
    assert rt.sequence_scores(h).shape == (1, 3, 1)
    assert rt.sequence_scores_pair(h, h).shape == (1, 3, 1)


def test_toml_sections_for_runtime_features():
    cfg = training_config_from_dict({
        "model": {"n_layer": 2, "n_embd": 32, "n_head": 2, "mlp_internal_dim_multiplier": 4,
                  "residual_connector": "block_attention_residual",
                  "block_attention_residual": {"layers_per_block": 3, "summary_mode": "mean_pool"},
                  "y_neuron_recurrence": {"enabled": True, "chunk_tokens": 2},
                  "hierarchical_dragon": {"enabled": True, "rho_sharing": "split"},
                  "latent_reasoning": {"enabled": True, "max_steps": 2, "min_steps": 1}},
    })
    m = cfg.model
    assert m.block_attention_residual.layers_per_block == 3
    assert m.y_neuron_recurrence.chunk_tokens == 2 and m.y_neuron_recurrence.state_decay == 0.5
    assert m.hierarchical_dragon.rho_sharing == "split"
    assert m.uses_extended_runtime()
    with pytest.raises(ValueError):
        training_config_from_dict({"model": {"latent_reasoning": {"enabled": True, "max_steps": 1,
                                                                  "min_steps": 2}}})


@pytest.mark.gpu
def test_runtime_variants_on_cuda_match_cpu():
    cfg = tiny()
    cfg.y_neuron_recurrence.enabled = True
    cfg.summary_memory.enabled = True
    cfg.summary_memory.chunk_tokens = 4
    cpu = DragonRuntime(cfg, seed=13)
    gpu = DragonRuntime(copy.deepcopy(cfg), device="cuda", seed=13)
    t = toks(T=8)
    ref = cpu.forward(t)
    got = gpu.forward(t.cuda())
    torch.testing.assert_close(got.cpu(), ref, rtol=2e-3, atol=2e-3)
    gpu.loss(t.cuda(), t.cuda()).backward()
    assert torch.isfinite(gpu.core.encoder.grad).all()


def test_y_neuron_recurrence_gradients_finite_with_silent_rows():
    cfg = tiny(relu_threshold=0.05)
    cfg.y_neuron_recurrence.enabled = True
    rt = DragonRuntime(cfg, seed=14)
    rt.loss(toks(T=6), toks(T=6, seed=3)).backward()
    for p in rt.parameters():
        assert p.grad is None or torch.isfinite(p.grad).all()

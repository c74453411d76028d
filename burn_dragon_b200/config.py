"""Configuration: model hyper-parameters and the training TOML schema.

The key names follow the reference's serde schema so a reference TOML file loads here:
``DragonConfig`` (burn_dragon_core/src/model/config.rs:979-1063), ``FusedKernelConfig``
(config.rs:51-85; it carries ``rope_theta``, ``relu_threshold``, ``rotary_embedding``),
``DragonRandomScaffoldConfig`` (config.rs:884-962) and the language ``TrainingConfig``
sections ``[dataset] [model] [training] [optimizer] [parallel] [generation]``
(burn_dragon_language/src/config/train/schema.rs:1209-2224). ``extends = "base.toml"``
inheritance and ordered ``--config`` overlays merge tables recursively, later files
winning (burn_dragon_language/src/config/merge.rs:8-164). Keys this framework does not
implement are kept in ``extras`` and reported once as a warning.
"""

from __future__ import annotations

import copy
import dataclasses
import math
import os
import tomllib
import warnings
from dataclasses import dataclass, field
from typing import Any

ROTARY_KINDS = ("rope", "alibi", "pope")


@dataclass
class RandomScaffoldConfig:
    """Frozen seeded projection + trainable low-rank adapter (config.rs:884-906)."""

    enabled: bool = False
    seed: int = 1337
    distribution: str = "gaussian_clt12"  # or "rademacher"
    rank: int = 8
    alpha: float = 16.0
    scaling: str = "standard"  # or "rank_stabilized"
    trainable_gain: bool = True

    def adapter_scale(self) -> float:
        if self.scaling == "rank_stabilized":
            return self.alpha / math.sqrt(self.rank)
        return self.alpha / self.rank


@dataclass
class YNeuronRecurrenceConfig:
    """Token-wise carry of the y-neuron activity into the next token's x-neurons
    (config.rs:196-224, defaults config.rs:594-612)."""

    enabled: bool = False
    carry_in_scale: float = 0.125
    last_layers: int | None = None
    chunk_tokens: int = 1
    state_decay: float = 0.5
    state_update_scale: float = 1.0
    state_rms_cap: float | None = 1.0


@dataclass
class ClockedSlowMemoryConfig:
    """A second low-rank step on chunk means, broadcast back to the chunk (config.rs:226-260)."""

    enabled: bool = False
    last_layers: int | None = None
    chunk_tokens: int = 4
    residual_scale: float = 1.0


@dataclass
class SummaryMemoryConfig:
    """Surprise-gated running summary of chunk means added to later chunks (config.rs:318-380)."""

    enabled: bool = False
    last_layers: int | None = None
    chunk_tokens: int = 32
    residual_scale: float = 0.25
    state_decay: float = 0.75
    state_update_scale: float = 0.5
    surprise_gate_threshold: float = 0.0
    surprise_gate_sharpness: float = 8.0
    write_trigger_text: str | None = None
    write_trigger_token_ids: list[int] | None = None


@dataclass
class HierarchicalDragonConfig:
    """Fast/slow cycles per layer with shared or split rho / weights (config.rs:452-520)."""

    enabled: bool = False
    last_layers: int | None = None
    fast_cycles: int = 3
    slow_cycles: int = 2
    rho_sharing: str = "shared"  # or "split"
    weight_sharing: str = "shared"  # or "split"
    slow_to_fast_scale: float = 0.25
    fast_to_slow_scale: float = 0.25


@dataclass
class AttentionResidualConfig:
    """Softmax attention over the history of layer deltas as the branch input
    (attention_residual/config.rs:70-116)."""

    enabled: bool = False
    last_layers: int | None = None
    num_heads: int = 4
    history_window: int | None = None
    dropout: float = 0.0
    recency_bias: float = 2.0


@dataclass
class BlockAttentionResidualConfig:
    """Attention residual over block summaries plus the recent raw deltas
    (attention_residual/config.rs:240-305)."""

    enabled: bool = False
    last_layers: int | None = None
    num_heads: int = 4
    layers_per_block: int = 2
    block_history_window: int | None = None
    intra_block_history_window: int | None = None
    summary_mode: str = "learned_projection"  # or "mean_pool"
    dropout: float = 0.0
    recency_bias: float = 2.0
    cache_block_summaries: bool = True
    two_phase_compute: bool = True


@dataclass
class LatentReasoningConfig:
    """Iterated latent refiner with optional adaptive halting (config.rs:744-843)."""

    enabled: bool = False
    max_steps: int = 1
    min_steps: int = 1
    adaptive_halting: bool = False
    halt_threshold: float = 0.55
    refiner_hidden_multiplier: int = 1
    normalize_steps: bool = False
    residual_refinement_gate: bool = False
    residual_refinement_gate_init: float = 0.25
    energy_head: bool = False
    step_conditioned_decoder: bool = False
    step_conditioned_decoder_scale: float = 1.0
    stop_bias_init: float = -2.0
    energy_margin: float = 1.0

    def validate(self) -> None:
        if not self.enabled:
            return
        if self.max_steps < 1 or self.min_steps < 1 or self.min_steps > self.max_steps:
            raise ValueError("latent_reasoning needs 1 <= min_steps <= max_steps")
        if self.adaptive_halting and not 0.0 <= self.halt_threshold <= 1.0:
            raise ValueError("latent_reasoning.halt_threshold must be in [0, 1]")
        if self.refiner_hidden_multiplier < 1:
            raise ValueError("latent_reasoning.refiner_hidden_multiplier must be > 0")
        if not 0.0 < self.residual_refinement_gate_init < 1.0:
            raise ValueError("latent_reasoning.residual_refinement_gate_init must be in (0, 1)")
        if self.step_conditioned_decoder_scale < 0 or self.energy_margin < 0:
            raise ValueError("latent_reasoning scales must be >= 0")


@dataclass
class NextLatentTransitionConfig:
    """Action-conditioned next-latent predictor (config.rs:845-883)."""

    enabled: bool = False
    hidden_multiplier: int = 2
    normalize_input: bool = True
    zero_init_output: bool = True


@dataclass
class SequenceScoreHeadConfig:
    """Low-rank prompt/candidate compatibility score head (config.rs:963-978)."""

    enabled: bool = False
    projection_dim: int = 64


@dataclass
class GatedDeltaNet2Config:
    """Gated DeltaNet-2 memory (burn_dragon_core/src/model/sequence/gdn2.rs:28-80)."""

    chunk_size: int = 64
    implementation: str = "bdh_adapter_legacy"
    qk_l2_norm: bool = True
    allow_neg_eigval: bool = False
    erase_gate: str = "channel"  # channel | scalar | disabled
    write_gate: str = "channel"
    decay_gate: str = "channel"
    state_precision: str = "f32"
    state_epsilon: float = 1.0e-6
    output_scale: float = 1.0


@dataclass
class MambaSequenceConfig:
    """Mamba-3 SISO memory (burn_dragon_core/src/model/sequence/mamba.rs:60-130)."""

    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    dt_rank: int | None = None
    dt_min: float = 1.0e-3
    dt_max: float = 1.0e-1
    dt_scale: float = 1.0
    conv_bias: bool = True
    use_fast_path: bool = True
    headdim: int = 128
    ngroups: int = 1
    a_init_min: float = 1.0
    a_init_max: float = 16.0
    norm_eps: float = 1.0e-5
    rope_fraction: float = 0.5
    dt_init_floor: float = 1.0e-4
    a_floor: float = 1.0e-4
    chunk_size: int = 64
    is_outproj_norm: bool = False
    is_mimo: bool = False
    mimo_rank: int = 1

    def validate(self, d_model: int) -> None:
        d_inner = d_model * self.expand
        if self.headdim <= 0 or d_inner % self.headdim:
            raise ValueError(f"mamba: d_inner {d_inner} must be divisible by headdim {self.headdim}")
        if (d_inner // self.headdim) % self.ngroups:
            raise ValueError("mamba: nheads must be divisible by ngroups")
        if abs(self.rope_fraction - 0.5) > 1e-6 and abs(self.rope_fraction - 1.0) > 1e-6:
            raise ValueError("mamba: rope_fraction must be 0.5 or 1.0")
        split = int(self.d_state * self.rope_fraction)
        if split - split % 2 < 2:
            raise ValueError("mamba: d_state * rope_fraction needs at least one rotary pair")
        if self.is_mimo:
            raise ValueError("mamba: MIMO is not implemented (set is_mimo = false)")
        if self.chunk_size <= 0 or self.dt_min <= 0 or self.dt_max < self.dt_min:
            raise ValueError("mamba: invalid chunk_size / dt range")


@dataclass
class DragonConfig:
    """BDH model hyper-parameters (defaults as in config.rs:1030-1063)."""

    n_layer: int = 6
    n_embd: int = 256
    dropout: float = 0.1
    n_head: int = 4
    mlp_internal_dim_multiplier: int = 4
    vocab_size: int = 256
    n_expert: int = 1
    # {type = "late_layer", base_latent_total, last_layers} | {type = "geometric",
    # min_latent_total}: layer l uses the first latent_total_for_layer(l) / n_head neurons
    # of every head of the shared weights (burn_dragon_core/src/model/config.rs:584-592,
    # 1125-1260; dragon.rs:1855-1880)
    latent_fanout_schedule: dict | None = None
    tie_input_output_embeddings: bool = False
    rollout_fast_steps_per_slow_step: int = 1
    # FusedKernelConfig fields that change the math
    rotary_embedding: str = "alibi"
    rope_theta: float = 65536.0
    relu_threshold: float = 0.0
    alibi_slopes: list[float] | None = None
    # DragonNorm
    norm_eps: float = 1e-5
    # initialization family (init.rs:18-25; the reference defaults to near_critical) and
    # the SimpleNormal std (init.rs:810)
    initialization: str = "simple_normal"
    init_std: float = 0.02
    reservoir_density: float = 0.1
    # DragonInitializationConfig sub-tables (init.rs:24-190). Without an
    # [model.initialization] table the reference uses its promoted default: simple_normal
    # with depth-scaled residual projections and heavy-tailed log-normal neuron gains.
    residual_scaling: str = "depth_scaled"  # family_default | disabled | depth_scaled
    residual_scaling_gain: float = 1.0
    neuron_gains: str = "heavy_tailed_log_normal"  # iid | heavy_tailed_log_normal
    neuron_gain_log_sigma: float = 0.75
    neuron_gain_max: float = 4.0
    topology_prior: str = "iid"  # iid | modular_bridges
    topology_community_count: int = 4
    topology_bridge_fraction: float = 0.05
    topology_intra_community_gain: float = 1.5
    topology_inter_community_gain: float = 0.5
    topology_bridge_gain: float = 1.0
    firing_targets: str = "disabled"  # disabled | gaussian_estimate | explicit_thresholds
    x_firing_target: float = 0.15
    y_firing_target: float = 0.05
    x_firing_threshold: float = 0.0
    y_firing_threshold: float = 0.0
    # DragonNormConfig (norm.rs:11-125): layer_norm | rms_norm | dynamic_tanh | derf
    norm_kind: str = "layer_norm"
    norm_alpha_init: float | None = None
    norm_shift_init: float = 0.0
    # ManifoldHyperConnectionsConfig (mhc/config.rs): 1 stream = vanilla residual
    mhc_streams: int = 1
    mhc_tau: float = 1.0
    mhc_iters: int = 10
    # coefficient policy (mhc/config.rs:9-24): "static_sinkhorn" (learned constants) or
    # "dynamic_positive" (a per-token stream controller)
    mhc_policy: str = "static_sinkhorn"
    # latent block pattern (kernel/block_sparse.rs): None = dense; otherwise the active
    # latent blocks (of latent_block_size neurons within each head)
    latent_block_size: int = 64
    latent_active_blocks: list[int] | None = None
    # dense-score row chunk (sequence/config.rs)
    dense_score_row_chunk: int = 512
    random_scaffold: RandomScaffoldConfig = field(default_factory=RandomScaffoldConfig)
    # sequence memory system (sequence/config.rs:12-120): linear_attention |
    # mamba3_state_space_duality | gated_deltanet2; executor reference |
    # dense_score_short_context | gated_delta_chunk_wy
    sequence_memory_system: str = "linear_attention"
    sequence_executor: str = "reference"
    mamba: MambaSequenceConfig = field(default_factory=MambaSequenceConfig)
    gated_deltanet2: GatedDeltaNet2Config = field(default_factory=GatedDeltaNet2Config)
    # residual connector: vanilla | mhc | attention_residual | block_attention_residual
    residual_connector: str = "vanilla"
    attention_residual: AttentionResidualConfig = field(default_factory=AttentionResidualConfig)
    block_attention_residual: BlockAttentionResidualConfig = field(default_factory=BlockAttentionResidualConfig)
    y_neuron_recurrence: YNeuronRecurrenceConfig = field(default_factory=YNeuronRecurrenceConfig)
    clocked_slow_memory: ClockedSlowMemoryConfig = field(default_factory=ClockedSlowMemoryConfig)
    summary_memory: SummaryMemoryConfig = field(default_factory=SummaryMemoryConfig)
    hierarchical_dragon: HierarchicalDragonConfig = field(default_factory=HierarchicalDragonConfig)
    latent_reasoning: LatentReasoningConfig = field(default_factory=LatentReasoningConfig)
    next_latent_transition: NextLatentTransitionConfig = field(default_factory=NextLatentTransitionConfig)
    sequence_score_head: SequenceScoreHeadConfig = field(default_factory=SequenceScoreHeadConfig)

    @property
    def latent_total(self) -> int:
        return self.mlp_internal_dim_multiplier * self.n_embd

    @property
    def latent_per_head(self) -> int:
        total = self.latent_total
        if total % self.n_head:
            raise ValueError("latent size must be divisible by the number of heads")
        return total // self.n_head

    def _latent_quantum(self) -> int:
        return math.lcm(max(self.n_embd, 1), max(self.n_head, 1) * max(self.n_expert, 1))

    def latent_total_for_layer(self, layer: int) -> int:
        full = self.latent_total
        f = self.latent_fanout_schedule
        if not f:
            return full
        if f.get("type") == "late_layer":
            first_full = max(max(self.n_layer, 1) - max(int(f["last_layers"]), 1), 0)
            return full if layer >= first_full else int(f["base_latent_total"])
        lo = int(f["min_latent_total"])
        if self.n_layer <= 1 or layer + 1 >= self.n_layer:
            return full
        if layer == 0:
            return lo
        raw = round(lo * (full / lo) ** (layer / (self.n_layer - 1)))
        q = self._latent_quantum()
        c = min(max(raw, lo), full)
        lower = max((c // q) * q, lo)
        upper = min(lower + q, full)
        if upper < lo:
            return lo
        return lower if c - lower <= upper - c else upper

    def latent_per_head_for_layer(self, layer: int) -> int:
        return self.latent_total_for_layer(layer) // self.n_head

    def uniform_latent_fanout(self) -> bool:
        return all(self.latent_total_for_layer(i) == self.latent_total for i in range(self.n_layer))

    def _validate_fanout(self) -> None:
        f = self.latent_fanout_schedule
        if not f:
            return
        kind = f.get("type")
        keys = {"late_layer": ("base_latent_total",), "geometric": ("min_latent_total",)}.get(kind)
        if keys is None:
            raise ValueError(f"model.latent_fanout_schedule type {kind!r}")
        for k in keys:
            t = int(f.get(k, 0))
            if t <= 0 or t > self.latent_total or t % self._latent_quantum():
                raise ValueError(f"model.latent_fanout_schedule.{k} must be in (0, latent_total] and divisible by "
                                 f"lcm(n_embd, n_head*n_expert) (got {t})")
        if kind == "late_layer" and int(f.get("last_layers", 0)) <= 0:
            raise ValueError("model.latent_fanout_schedule.last_layers must be > 0")

    def residual_depth(self) -> int:
        return max(self.n_layer, 1) * max(self.rollout_fast_steps_per_slow_step, 1)

    def thresholds(self) -> tuple[float, float]:
        """(x, y) ReLU thresholds: the shared ``relu_threshold`` unless firing targets set
        them (init.rs:544-580): ``gaussian_estimate`` places each threshold at the
        (1 - target) quantile of the estimated pre-activation N(0, sqrt(D) * std)."""
        if self.firing_targets == "disabled":
            return self.relu_threshold, self.relu_threshold
        if self.firing_targets == "explicit_thresholds":
            return self.x_firing_threshold, self.y_firing_threshold
        from statistics import NormalDist

        from .models.init import projection_std

        out = []
        for role, target in (("encoder", self.x_firing_target), ("encoder_v", self.y_firing_target)):
            sigma = math.sqrt(max(self.n_embd, 1)) * projection_std(self, role, self.n_embd, self.latent_per_head)
            p = min(max(1.0 - target, 1e-12), 1.0 - 1e-12)
            out.append(sigma * NormalDist().inv_cdf(p))
        return out[0], out[1]

    def norm_alpha(self) -> float:
        if self.norm_alpha_init is not None:
            return self.norm_alpha_init
        return {"dynamic_tanh": 0.5, "derf": 0.88622695}.get(self.norm_kind, 1.0)

    def validate(self) -> None:
        if self.norm_kind not in ("layer_norm", "rms_norm", "dynamic_tanh", "derf"):
            raise ValueError(f"unknown normalization kind {self.norm_kind!r}")
        if self.initialization not in ("simple_normal", "near_critical", "he_glorot", "headwise_semi_orthogonal",
                                       "reservoir"):
            raise ValueError(f"unknown initialization kind {self.initialization!r}")
        if self.residual_scaling not in ("family_default", "disabled", "depth_scaled") or \
                not self.residual_scaling_gain > 0:
            raise ValueError("initialization.residual_scaling: kind family_default | disabled | depth_scaled, gain > 0")
        if self.neuron_gains not in ("iid", "heavy_tailed_log_normal") or self.neuron_gain_log_sigma < 0 or \
                not self.neuron_gain_max > 0:
            raise ValueError("initialization.neuron_gains: kind iid | heavy_tailed_log_normal, log_sigma >= 0, "
                             "max_gain > 0")
        if self.topology_prior not in ("iid", "modular_bridges") or self.topology_community_count < 1 or \
                not 0 <= self.topology_bridge_fraction <= 1:
            raise ValueError("initialization.topology_prior: kind iid | modular_bridges, community_count > 0, "
                             "bridge_fraction in [0, 1]")
        if self.firing_targets not in ("disabled", "gaussian_estimate", "explicit_thresholds"):
            raise ValueError("initialization.firing_targets.kind: disabled | gaussian_estimate | explicit_thresholds")
        if self.firing_targets == "gaussian_estimate" and not (0 < self.x_firing_target < 1
                                                               and 0 < self.y_firing_target < 1):
            raise ValueError("initialization.firing_targets: targets must be probabilities in (0, 1)")
        if self.rotary_embedding not in ROTARY_KINDS:
            raise ValueError(f"rotary_embedding must be one of {ROTARY_KINDS}")
        if self.rollout_fast_steps_per_slow_step not in (1, 2, 4, 8, 16):
            raise ValueError("rollout_fast_steps_per_slow_step must be one of [1, 2, 4, 8, 16]")
        if self.rotary_embedding == "rope" and self.latent_per_head % 2:
            raise ValueError("RoPE needs an even latent per head")
        _ = self.latent_per_head
        self._validate_fanout()
        if self.latent_fanout_schedule and self.uses_extended_runtime():
            raise ValueError("model.latent_fanout_schedule is implemented on the BDH layer path, not with the "
                             "layer-loop variants")
        if self.residual_connector not in ("vanilla", "mhc", "attention_residual", "block_attention_residual"):
            raise ValueError(f"unknown residual_connector {self.residual_connector!r}")
        if self.mhc_policy not in ("static_sinkhorn", "dynamic_positive"):
            raise ValueError(f"unknown mHC coefficient policy {self.mhc_policy!r}")
        self.latent_reasoning.validate()
        ok = {("linear_attention", "reference"), ("linear_attention", "dense_score_short_context"),
              ("mamba3_state_space_duality", "reference"), ("gated_deltanet2", "reference"),
              ("gated_deltanet2", "gated_delta_chunk_wy")}
        if (self.sequence_memory_system, self.sequence_executor) not in ok:
            raise ValueError(f"sequence kernel family {self.sequence_memory_system!r} with executor "
                             f"{self.sequence_executor!r} is not supported")
        if self.sequence_memory_system == "mamba3_state_space_duality":
            self.mamba.validate(self.n_embd)
        for name in ("rho_sharing", "weight_sharing"):
            if getattr(self.hierarchical_dragon, name) not in ("shared", "split"):
                raise ValueError(f"hierarchical_dragon.{name} must be 'shared' or 'split'")

    def resolved_residual_connector(self) -> str:
        """``vanilla`` defers to the enabled sub-config (config.rs:1067-1086)."""
        if self.residual_connector != "vanilla":
            return self.residual_connector
        if self.block_attention_residual.enabled:
            return "block_attention_residual"
        if self.attention_residual.enabled:
            return "attention_residual"
        if self.mhc_streams > 1:
            return "mhc"
        return "vanilla"

    def uses_extended_runtime(self) -> bool:
        """True when a feature outside the fused BDH step is on (these run on the PyTorch
        layer path of ``models.dragon_runtime``)."""
        return (self.sequence_memory_system != "linear_attention" or self.latent_active_blocks is not None
                or self.resolved_residual_connector() in ("attention_residual", "block_attention_residual")
                or self.y_neuron_recurrence.enabled or self.clocked_slow_memory.enabled
                or self.summary_memory.enabled or self.hierarchical_dragon.enabled
                or self.latent_reasoning.enabled or self.rollout_fast_steps_per_slow_step > 1)

    def decay_slopes(self) -> list[float]:
        """ALiBi slopes 1/2^(h/H) (burn_dragon_core/src/kernel/linear_attention.rs:149-160)."""
        if self.alibi_slopes is not None:
            return list(self.alibi_slopes)
        return [1.0 / (2.0 ** (h / self.n_head)) for h in range(self.n_head)]

    def uses_decay(self) -> bool:
        return self.rotary_embedding == "alibi"

    def param_count(self) -> int:
        d, n, v = self.n_embd, self.latent_total, self.vocab_size
        head = 0 if self.tie_input_output_embeddings else d * v
        return 3 * d * n + v * d + head + 2 * d

    @staticmethod
    def bdh_gpu() -> "DragonConfig":
        """BDH-GPU: d=256, n=32768, h=4, L=6, RoPE, byte vocab (the flagship config)."""
        return DragonConfig(n_layer=6, n_embd=256, n_head=4, mlp_internal_dim_multiplier=128,
                            dropout=0.0, rotary_embedding="rope", initialization="simple_normal")

    @staticmethod
    def tiny() -> "DragonConfig":
        """Tiny CPU config: d=64, n=2048, h=4, L=2."""
        return DragonConfig(n_layer=2, n_embd=64, n_head=4, mlp_internal_dim_multiplier=32,
                            dropout=0.0, rotary_embedding="rope", initialization="simple_normal")


@dataclass
class OptimizerConfig:
    name: str = "adamw"
    learning_rate: float = 1e-3
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    grad_clip_norm: float | None = None
    # element-wise gradient clamp, used when grad_clip_norm is unset
    # (burn_dragon_train/src/train/pipeline/optimizer.rs:225-240)
    grad_clip_value: float | None = None
    # validated and recorded; the reference applies no schedule from it either
    weight_decay_final: float | None = None
    lr_schedule: dict[str, Any] = field(default_factory=lambda: {"type": "constant"})
    # name = "eggroll": {sigma, population = {population_size (members, antithetic pairs
    # x 2), population_chunk_size (pairs per batched forward), rank}}
    # (burn_dragon_train/src/config/optimizer.rs:239-310)
    eggroll: dict[str, Any] = field(default_factory=dict)
    # {enabled, min_population_size 8, max_population_size 4096, population_per_batch 128,
    # population_chunk_size, prefer_power_of_two true}: population size from the batch size
    # (burn_dragon_train/src/config/optimizer.rs:108-135, 276-310, 382-406)
    eggroll_auto_population: dict[str, Any] = field(default_factory=dict)
    # {backend = auto | reference | cuda | factorized, perturbation_scope =
    # dragon_core_projection}: the population always runs as one batched (vmapped) forward
    # over the shared projections here, so every backend value takes that path
    eggroll_population_execution: dict[str, Any] = field(default_factory=dict)
    # the retired predictive-coding update transforms (only meaningful with the retired
    # optimizer.name = "predictive_coding", which is rejected)
    predictive_coding: dict[str, Any] = field(default_factory=dict)
    # the reference's only schedule mode
    schedule_mode: str = "dragon_reference"

    def apply_auto_eggroll_population(self, batch_size: int) -> dict | None:
        a = dict(self.eggroll_auto_population)
        if self.name != "eggroll" or not a.get("enabled"):
            return None

        def even(v):
            return max(v - v % 2, 2)

        pop = dict(dict(self.eggroll).get("population", {}))
        conf_size = int(pop.get("population_size", 16))
        conf_chunk = pop.get("population_chunk_size")
        lo = even(int(a.get("min_population_size", 8)))
        hi = even(max(int(a.get("max_population_size", 4096)), lo))
        req = max(conf_size, int(a.get("min_population_size", 8)),
                  max(batch_size, 1) * int(a.get("population_per_batch", 128)))
        req = min(max(even(req), lo), hi)
        size = req
        if a.get("prefer_power_of_two", True):
            nxt = 1 << (req - 1).bit_length()
            if lo <= nxt <= hi:
                size = nxt
            elif (1 << (req.bit_length() - 1)) >= lo:
                size = 1 << (req.bit_length() - 1)
        chunk = a.get("population_chunk_size", conf_chunk)
        chunk = size if chunk is None else int(chunk)
        chunk = min(even(max(min(chunk, size), 2)), size)
        pop.update(population_size=size, population_chunk_size=chunk)
        self.eggroll = {**dict(self.eggroll), "population": pop}
        return {"configured_population_size": conf_size, "resolved_population_size": size,
                "resolved_population_chunk_size": chunk, "batch_size": batch_size}

    def eggroll_settings(self) -> dict:
        e = dict(self.eggroll)
        pop = dict(e.get("population", {}))
        upd = dict(e.get("update", {}))
        out = {"sigma": float(e.get("sigma", 0.01)), "members": int(pop.get("population_size", 16)),
               "chunk": pop.get("population_chunk_size"), "rank": int(pop.get("rank", 4)),
               "fitness_normalization": str(e.get("fitness_normalization", "none")),
               "coefficient_clip": e.get("coefficient_clip"),
               "max_delta_rms": upd.get("max_delta_rms", e.get("max_delta_rms"))}
        if out["fitness_normalization"] not in ("none", "center", "rank"):
            raise ValueError(f"optimizer.eggroll.fitness_normalization {out['fitness_normalization']!r}")
        if not out["sigma"] > 0:
            raise ValueError("optimizer.eggroll.sigma must be > 0")
        if out["members"] < 2 or out["members"] % 2:
            raise ValueError("optimizer.eggroll.population.population_size must be an even number >= 2 "
                             "(antithetic pairs)")
        if out["rank"] <= 0:
            raise ValueError("optimizer.eggroll.population.rank must be > 0")
        if self.grad_clip_norm is not None:
            raise ValueError("optimizer.name = eggroll does not use gradients: grad clipping is not supported")
        return out


@dataclass
class ParallelConfig:
    mode: str = "single"  # single | ddp | fsdp | tensor_parallel_neuron | hybrid_2d | pipeline
    world_size: int | None = None
    # data: shard-the-loader keys of the reference, plus transport = "p2p" | "nvls" (the
    # NVLink data-parallel step's exchange: peer loads / stores or NVLink multicast)
    data: dict[str, Any] = field(default_factory=dict)
    tensor: dict[str, Any] = field(default_factory=dict)
    pipeline: dict[str, Any] = field(default_factory=dict)
    fsdp: dict[str, Any] = field(default_factory=dict)
    checkpoint: dict[str, Any] = field(default_factory=dict)


@dataclass
class ContinualBackpropConfig:
    """Utility-based replacement of shared low-rank features (burn_dragon_train/src/
    config/continual_backprop.rs:1-120; defaults as there)."""

    enabled: bool = False
    target: str = "shared_lowrank_latents"
    utility_decay: float = 0.99
    replacement_rate: float = 1.0e-5
    maturity_steps: int = 1024
    sample_interval_steps: int = 8
    replace_interval_steps: int = 256
    utility_epsilon: float = 1.0e-6
    lr_coupling: str = "global_ratio"  # none | global_ratio | target_group_ratio
    lr_coupling_power: float = 1.0
    warmup_steps: int = 1024
    cooldown_steps: int = 256
    max_replacements_per_interval: int = 1
    regression_pause_steps: int = 1024


@dataclass
class PCInferenceConfig:
    """Activity-inference rule of local predictive coding (burn_pc PcInferenceConfig;
    defaults burn_dragon_language/src/config/train/schema.rs:621-639)."""

    steps: int = 4
    step_size: float = 0.05
    latent_decay: float = 0.0
    max_grad_norm: float | None = 1.0
    gradient_norm_scope: str = "per_row"  # per_row | global
    eps: float = 1.0e-8


@dataclass
class LocalPredictiveCodingConfig:
    solver: str = "synchronous_equilibrium"  # | reverse_gauss_seidel | fixed_prediction
    inference: PCInferenceConfig = field(default_factory=PCInferenceConfig)
    prediction_precision: float = 1.0
    factor_reduction: str = "sum"  # sum | mean
    sync_diagnostics: bool = False
    # parameters learn once the activities have settled; the reference accepts only this
    # schedule for Dragon (validate.rs:3610-3618)
    learning_schedule: str = "equilibrium"


@dataclass
class AutoBatchSizeConfig:
    """Startup batch-size selection (burn_dragon_language/src/config/train/schema.rs:
    209-255; defaults :179-205)."""

    enabled: bool = False
    max_batch_size: int | None = None
    max_probe_batch_size: int | None = None
    min_batch_size: int = 1
    target_device_memory_mb: int = 0
    probe_steps: int = 1
    binary_search: bool = True
    recompute_on_neuron_scale: bool = True
    scale_memory_exponent: float = 1.0
    max_system_memory_fraction: float = 0.9
    probe_safety_margin: float = 1.15


@dataclass
class NeuronScalingStabilizationConfig:
    freeze_base_steps: int = 256
    unfreeze_ramp_steps: int = 256
    new_slice_lr_scale: float = 1.0
    base_lr_scale_after_ramp: float = 1.0


@dataclass
class NeuronScalingConfig:
    """Latent-width doubling on a validation plateau (schema.rs:151-300; defaults there)."""

    enabled: bool = False
    max_latent_total: int = 8192
    growth: str = "double"
    min_steps_between_scales: int = 2000
    max_scale_events: int = 4
    capacity_patience_epochs: int = 2
    require_live_source_selection: bool = True
    stabilization: NeuronScalingStabilizationConfig = field(default_factory=NeuronScalingStabilizationConfig)


@dataclass
class ValidationConfig:
    """Teacher-forced validation (schema.rs:1088-1160): ``fixed_holdout`` evaluates the
    same windows every time (drawn with ``seed``, independent of the training seed);
    ``live_source_selection`` draws fresh windows; ``external_evaluator`` leaves
    validation to a separate process reading the checkpoints."""

    execution: str = "local"  # local | external_evaluator
    sampling: str = "fixed_holdout"  # fixed_holdout | live_source_selection
    seed: int = 0xD12A60A5

    def validate(self) -> None:
        if self.execution not in ("local", "external_evaluator"):
            raise ValueError(f"training.validation.execution {self.execution!r}")
        if self.sampling not in ("fixed_holdout", "live_source_selection"):
            raise ValueError(f"training.validation.sampling {self.sampling!r}")


@dataclass
class DynamicsAnchorConfig:
    """Self-distillation anchor to an EMA teacher of the student (schema.rs, DynamicsAnchorConfig)."""

    enabled: bool = False
    weight: float = 0.0
    teacher_update_rate: float = 0.01
    kl: str = "jensen_shannon"  # forward | reverse | jensen_shannon
    mask: str = "all_tokens"  # all_tokens | context_tokens | target_tokens
    warmup_steps: int = 0
    ramp_steps: int = 0
    every_steps: int = 1

    def validate(self) -> None:
        if not self.enabled:
            return
        if self.kl not in ("forward", "reverse", "jensen_shannon"):
            raise ValueError(f"training.dynamics_anchor.kl {self.kl!r}")
        if self.mask not in ("all_tokens", "context_tokens", "target_tokens"):
            raise ValueError(f"training.dynamics_anchor.mask {self.mask!r}")
        if not self.weight >= 0.0 or self.every_steps == 0:
            raise ValueError("training.dynamics_anchor.weight must be >= 0 and every_steps > 0")


@dataclass
class GreedyRolloutUnlikelihoodConfig:
    """Unlikelihood on short greedy rollouts (schema.rs, GreedyRolloutUnlikelihoodConfig)."""

    enabled: bool = False
    # only while the dynamics monitor reports a recovery; that monitor belongs to the
    # absent event crate, so a recovery-only rollout never runs here
    recovery_only: bool = False
    weight: float = 0.0
    margin_weight: float = 0.0
    margin: float = 0.0
    recovery_weight: float = 0.0
    sequence_recovery_weight: float = 0.0
    entropy_floor_weight: float = 0.0
    target_entropy_bits: float = 0.0
    cycle_weight: float = 0.0
    cycle_margin_weight: float = 0.0
    cycle_min_lag: int = 2
    cycle_max_lag: int = 64
    warmup_steps: int = 0
    ramp_steps: int = 0
    every_steps: int = 128
    prompt_tokens: int = 32
    rollout_tokens: int = 8
    history_tokens: int = 8
    batch_prompts: int = 1
    epsilon: float = 1e-4

    def validate(self) -> None:
        if not self.enabled:
            return
        if self.every_steps == 0:
            raise ValueError("training.greedy_rollout_unlikelihood.every_steps must be > 0")
        if not 0.0 < self.epsilon < 1.0:
            raise ValueError("training.greedy_rollout_unlikelihood.epsilon must be in (0, 1)")
        for k in ("weight", "margin_weight", "recovery_weight", "sequence_recovery_weight", "entropy_floor_weight",
                  "target_entropy_bits", "cycle_weight", "cycle_margin_weight"):
            if not getattr(self, k) >= 0.0:
                raise ValueError(f"training.greedy_rollout_unlikelihood.{k} must be finite and >= 0")


@dataclass
class LogitEntropyFloorConfig:
    """Entropy / marginal-entropy floors and target coverage on the predicted
    distribution (schema.rs:340-371)."""

    enabled: bool = False
    weight: float = 0.0
    target_entropy_bits: float = 0.0
    marginal_weight: float = 0.0
    target_marginal_entropy_bits: float = 0.0
    target_coverage_weight: float = 0.0
    target_coverage_epsilon: float = 1e-8
    warmup_steps: int = 0
    ramp_steps: int = 0
    every_steps: int = 1

    def validate(self) -> None:
        if not self.enabled:
            return
        for k in ("weight", "marginal_weight", "target_coverage_weight", "target_entropy_bits",
                  "target_marginal_entropy_bits"):
            v = getattr(self, k)
            if not (v >= 0.0 and v != float("inf")):
                raise ValueError(f"training.logit_entropy_floor.{k} must be finite and >= 0")
        if not 0.0 < self.target_coverage_epsilon < 1.0:
            raise ValueError("training.logit_entropy_floor.target_coverage_epsilon must be finite and in (0, 1)")
        if self.every_steps == 0:
            raise ValueError("training.logit_entropy_floor.every_steps must be > 0")


@dataclass
class RepeatUnlikelihoodConfig:
    """Unlikelihood of repeating recent input tokens (schema.rs:372-407)."""

    enabled: bool = False
    weight: float = 0.0
    cycle_weight: float = 0.0
    cycle_margin_weight: float = 0.0
    cycle_margin: float = 0.0
    cycle_min_lag: int = 2
    cycle_max_lag: int = 64
    cycle_lags_per_step: int = 8
    warmup_steps: int = 0
    ramp_steps: int = 0
    every_steps: int = 1
    history_lags: list[int] = field(default_factory=list)
    epsilon: float = 1e-4

    def validate(self) -> None:
        if not self.enabled:
            return
        for k in ("weight", "cycle_weight", "cycle_margin_weight"):
            if not getattr(self, k) >= 0.0:
                raise ValueError(f"training.repeat_unlikelihood.{k} must be finite and >= 0")
        if not 0.0 < self.epsilon < 1.0:
            raise ValueError("training.repeat_unlikelihood.epsilon must be in (0, 1)")
        if self.every_steps == 0:
            raise ValueError("training.repeat_unlikelihood.every_steps must be > 0")


@dataclass
class CausalInputCorruptionConfig:
    """Replace input tokens (never targets) at a ramped probability (schema.rs:321-339)."""

    enabled: bool = False
    probability: float = 0.0
    warmup_steps: int = 0
    ramp_steps: int = 0
    replacement_token_id: int | None = None

    def probability_at(self, step: int) -> float:
        """0 before warm-up, then linear over ``ramp_steps`` to ``probability``
        (burn_dragon_language/src/train/steps.rs:3368-3388)."""
        p = min(max(self.probability, 0.0), 1.0)
        if not self.enabled or p <= 1.1920929e-07 or step < self.warmup_steps:
            return 0.0
        if self.ramp_steps == 0:
            return p
        return p * min(max((step - self.warmup_steps + 1) / self.ramp_steps, 0.0), 1.0)


@dataclass
class TrainingSection:
    block_size: int = 512
    batch_size: int = 32
    max_iters: int = 1000
    tbptt_chunk_size: int | None = None
    tbptt_persist_across_steps: bool = False
    # auto: streaming when rho persists across steps, random windows otherwise (schema.rs,
    # SequenceBatchingMode)
    sequence_batching: str = "auto"  # auto | random | streaming
    gradient_accumulation_steps: int = 1
    seed: int = 1337
    log_frequency: int = 10
    checkpoint_interval_iters: int | None = None
    validation_interval_iters: int | None = None
    continual_backprop: ContinualBackpropConfig = field(default_factory=ContinualBackpropConfig)
    auto_batch_size: AutoBatchSizeConfig = field(default_factory=AutoBatchSizeConfig)
    neuron_scaling: NeuronScalingConfig = field(default_factory=NeuronScalingConfig)
    input_corruption: CausalInputCorruptionConfig = field(default_factory=CausalInputCorruptionConfig)
    init_transfer: dict[str, Any] = field(default_factory=dict)
    # [{target, scale, schedule = {final_scale, start_fraction, end_fraction}}] (train.module_lr)
    module_lr_scales: list[dict[str, Any]] = field(default_factory=list)
    # run control (schema.rs TrainingHyperparameters; run_dirs.rs:13-19, 236-290):
    # epochs: when set, max_iters = epochs x the dataset's steps per epoch
    epochs: int | None = None
    # None: resume the named run if it has a checkpoint. fresh | resume_exact_run (needs
    # resume_run_dir) | resume_latest_checkpoint_if_present (the run root's latest run) |
    # init_from_checkpoint (needs init_checkpoint_path)
    launch_mode: str | None = None
    resume_run_dir: str | None = None
    resume_checkpoint_epoch: int | None = None  # which checkpoint to resume (default newest)
    init_checkpoint_epoch: int | None = None  # which checkpoint of init_checkpoint_path
    # streaming documents are at least this long (rounded up to block_size multiples)
    min_logical_block_size: int | None = None
    # the reference's ablation switch to keep an unused terminal state; the fused step
    # writes the state only when it is consumed, so this changes nothing here
    retain_ephemeral_terminal_sequence_state: bool = False
    # {enabled, paired_batches, max_rho_slots}: stream-warm validation with a warm / cold
    # carry probe (train.state_probe)
    sequence_state_probe: dict[str, Any] = field(default_factory=dict)
    # recurrent-state predictive coding (train.state_pc.RecurrentStatePCConfig keys)
    predictive_coding: dict[str, Any] = field(default_factory=dict)
    # training-side latent reasoning (train.latent_reasoning.LatentReasoningTraining keys)
    latent_reasoning: dict[str, Any] = field(default_factory=dict)
    # legacy: enabling it is rejected in favour of training.objective (validate.rs:2854-2860)
    gdpo: dict[str, Any] | None = None
    # a [model.sequence_kernel] table that replaces the model's for training (applied by
    # the loader; burn_dragon_language/src/train/backend.rs:755-770)
    sequence_kernel_override: dict[str, Any] | None = None
    # context strategy of generation done during training ({type = "infinite"} |
    # {type = "sliding", window}), checked like generation.context_strategy
    context_strategy: dict[str, Any] = field(default_factory=lambda: {"type": "infinite"})
    validation: ValidationConfig = field(default_factory=ValidationConfig)
    logit_entropy_floor: LogitEntropyFloorConfig = field(default_factory=LogitEntropyFloorConfig)
    dynamics_anchor: DynamicsAnchorConfig = field(default_factory=DynamicsAnchorConfig)
    greedy_rollout_unlikelihood: GreedyRolloutUnlikelihoodConfig = field(
        default_factory=GreedyRolloutUnlikelihoodConfig)
    repeat_unlikelihood: RepeatUnlikelihoodConfig = field(default_factory=RepeatUnlikelihoodConfig)  # train.init_transfer.InitTransferConfig keys
    # batches from the native prefetching loader (csrc/host/loader.cpp) instead of the
    # Python generators
    native_loader: bool = True
    loader_workers: int = 2
    target_effective_batch_size: int | None = None
    # initialise the weights from this run directory's newest checkpoint (a fresh run only)
    init_checkpoint_path: str | None = None
    # auto | backpropagation | predictive_coding | eggroll (schema.rs:569-577)
    algorithm: str = "auto"
    local_predictive_coding: LocalPredictiveCodingConfig = field(default_factory=LocalPredictiveCodingConfig)
    # training objective table (objective.rs TrainingObjectiveConfig): {type = "next_token"
    # | "sdft" | "sdpo" | "sdft_sdpo", sdft = {...}, sdpo = {...}, sdft_weight, sdpo_weight}
    objective: dict[str, Any] = field(default_factory=lambda: {"type": "next_token"})


@dataclass
class DatasetConfig:
    # synthetic_bytes | file (a byte file) | jsonl | parquet | text (a corpus tokenised
    # once into cache_dir, then read like a file) | nemotron_climb_mix (the reference's
    # Hugging Face preset, schema.rs:37-52) | huggingface (a dataset repository of the local
    # hub cache described by the ``huggingface`` table: repo_id, revision, format,
    # train_files, auto_discover_train_files, validation_files, text_fields,
    # sequence_field, field_separator, template, max_records; schema.rs:64-96)
    type: str = "synthetic_bytes"
    revision: str | None = None      # nemotron_climb_mix
    max_records: int | None = None   # nemotron_climb_mix
    huggingface: dict[str, Any] | None = None
    cache_dir: str = "data"
    train_split_ratio: float = 0.9
    path: str | None = None
    text_field: str = "text"
    tokenizer: str | None = None  # a tokenizer.json (BPE) for jsonl / parquet / text corpora
    # a separate held-out source: {type = file | jsonl | parquet | text, path, text_field,
    # cache_dir, train_split_ratio (default 0: the whole source is validation data)}
    # (schema.rs:13-35, ValidationDatasetConfig)
    validation: dict[str, Any] | None = None


@dataclass
class GenerationConfig:
    prompt: str = ""
    max_tokens: int = 256
    max_chars: int | None = None
    temperature: float = 1.0
    top_k: int | None = None
    device_buffer_tokens: int = 64
    output_format: str = "auto"  # auto | decoded_text | token_ids (burn_dragon_language/src/config/core.rs:18-60)
    # {type = "infinite"} or {type = "sliding", window = W}; window 0 means block_size
    # (core.rs:60-68, generation.rs:1317-1332)
    context_strategy: dict[str, Any] = field(default_factory=lambda: {"type": "infinite"})
    # {source = "dataset"} (the run's tokenizer.json) or {source = "config", path = a
    # tokenizer.json | type = "byte"} (core.rs:40-52)
    prompt_tokenizer: dict[str, Any] = field(default_factory=lambda: {"source": "dataset"})
    decode_tokenizer: dict[str, Any] = field(default_factory=lambda: {"source": "dataset"})

    def sliding_window(self, block_size: int) -> int | None:
        kind = self.context_strategy.get("type", "infinite")
        if kind == "infinite":
            return None
        if kind != "sliding":
            raise ValueError(f"generation.context_strategy type {kind!r}")
        w = int(self.context_strategy.get("window", 0))
        return w if w > 0 else max(block_size, 1)


@dataclass
class RunLayoutConfig:
    """Where runs live (burn_dragon_train/src/config/run_layout.rs:6-35; path rules in
    burn_dragon_train/src/train/pipeline/run_dirs.rs:46-141)."""

    base_dir: str | None = None
    category: str | None = None
    mirror_config_path: bool = True
    bundle: str | None = None
    stage: str | None = None
    variant: str | None = None


@dataclass
class TrainingConfig:
    dataset: DatasetConfig = field(default_factory=DatasetConfig)
    model: DragonConfig = field(default_factory=DragonConfig)
    training: TrainingSection = field(default_factory=TrainingSection)
    optimizer: OptimizerConfig = field(default_factory=OptimizerConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    generation: GenerationConfig = field(default_factory=GenerationConfig)
    run_layout: RunLayoutConfig = field(default_factory=RunLayoutConfig)
    config_paths: list[str] = field(default_factory=list)
    extras: dict[str, Any] = field(default_factory=dict)

    def validate(self) -> None:
        self.model.validate()
        self.training.validation.validate()
        t = self.training
        if t.gdpo and t.gdpo.get("enabled"):
            raise ValueError("training.gdpo.enabled is a legacy objective flag; use training.objective.type = "
                             "\"sdpo\" for self-distilled policy optimization")
        if t.launch_mode not in (None, "fresh", "resume_exact_run", "resume_latest_checkpoint_if_present",
                                 "init_from_checkpoint"):
            raise ValueError(f"training.launch_mode {t.launch_mode!r}")
        if t.launch_mode in ("fresh", "init_from_checkpoint", "resume_latest_checkpoint_if_present") \
                and t.resume_run_dir:
            raise ValueError(f"training.launch_mode = \"{t.launch_mode}\" cannot be combined with "
                             "training.resume_run_dir")
        if t.launch_mode == "resume_exact_run" and not t.resume_run_dir:
            raise ValueError("training.launch_mode = \"resume_exact_run\" requires training.resume_run_dir")
        if t.launch_mode == "init_from_checkpoint" and not t.init_checkpoint_path:
            raise ValueError("training.launch_mode = \"init_from_checkpoint\" requires training.init_checkpoint_path")
        if t.min_logical_block_size is not None and t.min_logical_block_size <= 0:
            raise ValueError("training.min_logical_block_size must be > 0 when set")
        if t.epochs is not None and t.epochs <= 0:
            raise ValueError("training.epochs must be > 0 when set")
        o = self.optimizer
        if o.name == "predictive_coding":
            # burn_dragon_train/src/train/pipeline/optimizer.rs:250-256
            raise ValueError("optimizer.name=predictive_coding is retired; predictive coding is a training "
                             "algorithm: use training.algorithm=predictive_coding with an ordinary update")
        ex = dict(o.eggroll_population_execution)
        if ex.get("backend", "auto") not in ("auto", "reference", "cuda", "factorized") or \
                ex.get("perturbation_scope", "dragon_core_projection") != "dragon_core_projection":
            raise ValueError(f"optimizer.eggroll_population_execution {ex}")
        if o.schedule_mode != "dragon_reference":
            raise ValueError(f"optimizer.schedule_mode {o.schedule_mode!r}")
        if o.name not in ("adamw", "eggroll"):
            raise ValueError(f"optimizer.name {o.name!r} (adamw | eggroll)")
        if o.weight_decay_final is not None and o.weight_decay_final < 0:
            raise ValueError("optimizer.weight_decay_final must be >= 0")
        if o.grad_clip_value is not None and not o.grad_clip_value > 0:
            raise ValueError("optimizer.grad_clip_value must be > 0")
        if self.generation.output_format not in ("auto", "decoded_text", "token_ids"):
            raise ValueError(f"generation.output_format {self.generation.output_format!r}")
        self.generation.sliding_window(self.training.block_size)
        GenerationConfig(context_strategy=dict(self.training.context_strategy)).sliding_window(
            self.training.block_size)
        p = self.parallel.mode
        if p not in ("single", "ddp", "fsdp", "tensor_parallel_neuron", "hybrid_2d", "pipeline"):
            raise ValueError(f"unknown parallel.mode {p!r}")
        if self.parallel.data.get("transport", "p2p") not in ("p2p", "nvls"):
            raise ValueError("parallel.data.transport must be 'p2p' or 'nvls'")
        if p in ("tensor_parallel_neuron", "hybrid_2d"):
            tpc = self.parallel.tensor
            if tpc.get("axis", "neuron") != "neuron":
                raise ValueError("parallel.tensor.axis: only the neuron axis exists")
            part = tpc.get("partition", "contiguous")
            if part not in ("contiguous", "head_aligned"):
                raise ValueError(f"parallel.tensor.partition {part!r}")
            size = tpc.get("size")
            if size is not None:
                size = int(size)
                if part == "head_aligned" and size > self.model.n_head:
                    raise ValueError(f"parallel.tensor.partition=head_aligned requires parallel.tensor.size <= "
                                     f"model.n_head (got tensor_size={size} n_head={self.model.n_head})")
                # the decoder rows are head-major, so contiguous neuron ranges are whole heads
                # exactly when the size divides the head count; a split inside a head would
                # cut a head's attention across ranks, which this implementation keeps local
                if self.model.n_head % size:
                    raise ValueError(f"parallel.tensor.size {size} must divide model.n_head {self.model.n_head} "
                                     "(shards are whole heads)")
        if p == "pipeline" and self.training.tbptt_chunk_size:
            raise ValueError("pipeline parallelism does not support TBPTT chunking")
        if self.training.sequence_batching not in ("auto", "random", "streaming"):
            raise ValueError(f"training.sequence_batching {self.training.sequence_batching!r}")
        if self.training.tbptt_persist_across_steps and self.training.sequence_batching == "random":
            raise ValueError("training.sequence_batching=random is incompatible with "
                             "training.tbptt_persist_across_steps=true")
        if self.training.tbptt_chunk_size is not None:
            if self.training.tbptt_chunk_size <= 0 or self.training.block_size % self.training.tbptt_chunk_size:
                raise ValueError("tbptt_chunk_size must divide block_size")


# ------------------------------------------------------------------ TOML loading


def merge_tables(base: dict, overlay: dict) -> dict:
    """Recursive table merge; overlay scalars and arrays replace base values."""
    out = copy.deepcopy(base)
    for k, v in overlay.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = merge_tables(out[k], v)
        else:
            out[k] = copy.deepcopy(v)
    return out


def load_toml_with_extends(path: str, _seen: tuple[str, ...] = ()) -> dict:
    path = os.path.abspath(path)
    if path in _seen:
        raise ValueError(f"circular extends: {' -> '.join(_seen + (path,))}")
    with open(path, "rb") as f:
        data = tomllib.load(f)
    parent = data.pop("extends", None)
    if parent is None:
        return data
    parents = parent if isinstance(parent, list) else [parent]
    merged: dict = {}
    for p in parents:
        p_path = p if os.path.isabs(p) else os.path.join(os.path.dirname(path), p)
        merged = merge_tables(merged, load_toml_with_extends(p_path, _seen + (path,)))
    return merge_tables(merged, data)


def _fill(cls, table: dict, extras: dict, prefix: str):
    names = {f.name: f for f in dataclasses.fields(cls)}
    kwargs = {}
    for k, v in table.items():
        if k in names:
            f = names[k]
            if dataclasses.is_dataclass(f.default_factory() if callable(f.default_factory) else None) \
                    and isinstance(v, dict):
                sub_cls = type(f.default_factory())
                kwargs[k] = _fill(sub_cls, v, extras, f"{prefix}{k}.")
            else:
                kwargs[k] = v
        else:
            extras[f"{prefix}{k}"] = v
    return cls(**kwargs)


def _model_table(table: dict) -> dict:
    """Flatten the reference's nested [model.fused_kernels] keys into DragonConfig fields."""
    t = dict(table)
    fk = t.pop("fused_kernels", None)
    if isinstance(fk, dict):
        for k in ("rope_theta", "relu_threshold", "alibi_slopes", "rotary_embedding"):
            if k in fk:
                t[k] = fk[k]
        lat = (fk.get("block_sparse") or {}).get("latent") if isinstance(fk.get("block_sparse"), dict) else None
        if isinstance(lat, dict):
            t["latent_block_size"] = int(lat.get("block_size", 64))
            if lat.get("active_blocks") is not None:
                t["latent_active_blocks"] = sorted(int(b) for b in lat["active_blocks"])
    if "rotary_embedding" in t and isinstance(t["rotary_embedding"], str):
        t["rotary_embedding"] = t["rotary_embedding"].lower()
    norm = t.pop("normalization", None)
    if isinstance(norm, dict):
        kind = norm.get("kind", "layer_norm").lower()
        t["norm_kind"] = {"rmsnorm": "rms_norm", "dyt": "dynamic_tanh"}.get(kind, kind)
        if "eps" in norm:
            t["norm_eps"] = norm["eps"]
        if norm.get("alpha_init") is not None:
            t["norm_alpha_init"] = norm["alpha_init"]
        if norm.get("shift_init") is not None:
            t["norm_shift_init"] = norm["shift_init"]
    head = t.pop("language_head", None)
    if isinstance(head, dict) and head.get("type", "standard_token_classification") != "standard_token_classification":
        # the factorized NCA patch head serves the NCA universality data, which is not built here
        raise ValueError(f"model.language_head type {head.get('type')!r} is not implemented "
                         "(standard_token_classification is)")
    mhc = t.pop("mhc", None)
    if isinstance(mhc, dict) and mhc.get("enabled"):
        t["mhc_streams"] = int(mhc.get("num_streams", 4))
        t["mhc_tau"] = float(mhc.get("mhc_tau", 1.0))
        t["mhc_iters"] = int(mhc.get("mhc_iters", 10))
        t["mhc_policy"] = str(mhc.get("coefficient_policy", "static_sinkhorn"))
    sk = t.pop("sequence_kernel", None)
    if isinstance(sk, str):
        sk = {"memory_system": sk}
    if isinstance(sk, dict):
        fam = str(sk.get("memory_system", sk.get("family", "linear_attention"))).lower()
        fam = {"gdn2": "gated_deltanet2"}.get(fam, fam)
        t["sequence_memory_system"] = fam
        ex = str(sk.get("executor") or "reference").lower()
        t["sequence_executor"] = {"gdn2_chunk_wy": "gated_delta_chunk_wy"}.get(ex, ex)
        if "dense_score_row_chunk" in sk:
            t["dense_score_row_chunk"] = sk["dense_score_row_chunk"]
    ini = t.get("initialization")
    if isinstance(ini, dict):
        # a present table takes each sub-table's own defaults (init.rs:24-160)
        t["initialization"] = ini.get("kind", "near_critical")
        if "simple_normal_std" in ini:
            t["init_std"] = ini["simple_normal_std"]
        rs = ini.get("residual_scaling", {})
        t["residual_scaling"] = rs.get("kind", "family_default")
        t["residual_scaling_gain"] = rs.get("gain", 1.0)
        ng = ini.get("neuron_gains", {})
        t["neuron_gains"] = ng.get("kind", "iid")
        t["neuron_gain_log_sigma"] = ng.get("log_sigma", 0.75)
        t["neuron_gain_max"] = ng.get("max_gain", 4.0)
        tp = ini.get("topology_prior", {})
        t["topology_prior"] = tp.get("kind", "iid")
        for k in ("community_count", "bridge_fraction", "intra_community_gain", "inter_community_gain",
                  "bridge_gain"):
            if k in tp:
                t["topology_" + k] = tp[k]
        ft = ini.get("firing_targets", {})
        t["firing_targets"] = ft.get("kind", "disabled")
        for a, b in (("x_target", "x_firing_target"), ("y_target", "y_firing_target"),
                     ("x_threshold", "x_firing_threshold"), ("y_threshold", "y_firing_threshold")):
            if a in ft:
                t[b] = ft[a]
        if isinstance(ini.get("reservoir"), dict) and "density" in ini["reservoir"]:
            t["reservoir_density"] = ini["reservoir"]["density"]
    if "latent_total" in t:
        lt = t.pop("latent_total")
        d = t.get("n_embd", DragonConfig.n_embd)
        if lt % d:
            raise ValueError("latent_total must be a multiple of n_embd")
        t["mlp_internal_dim_multiplier"] = lt // d
    return t


def training_config_from_dict(data: dict) -> TrainingConfig:
    extras: dict = {}
    cfg = TrainingConfig()
    for section, cls in (("dataset", DatasetConfig), ("training", TrainingSection),
                         ("optimizer", OptimizerConfig), ("parallel", ParallelConfig),
                         ("generation", GenerationConfig), ("run_layout", RunLayoutConfig)):
        if section in data:
            setattr(cfg, section, _fill(cls, data[section], extras, f"{section}."))
    sko = (data.get("training") or {}).get("sequence_kernel_override")
    if sko is not None:
        data = dict(data)
        data["model"] = {**dict(data.get("model") or {}), "sequence_kernel": sko}
    if "model" in data:
        cfg.model = _fill(DragonConfig, _model_table(data["model"]), extras, "model.")
    for k, v in data.items():
        if k == "config_paths":  # written back by a run directory's training_config.json
            cfg.config_paths = list(v)
        elif k == "extras":
            extras.update(v or {})
        elif k not in ("dataset", "training", "optimizer", "parallel", "generation", "model", "run_layout"):
            extras[k] = v
    cfg.extras = extras
    if extras:
        warnings.warn(f"ignoring config keys not implemented here: {sorted(extras)}", stacklevel=2)
    cfg.validate()
    return cfg


def load_training_config(paths: list[str] | str, overrides: dict | None = None) -> TrainingConfig:
    """Load one or more TOML files (each may `extends` others), merged in order."""
    if isinstance(paths, str):
        paths = [paths]
    merged: dict = {}
    for p in paths:
        merged = merge_tables(merged, load_toml_with_extends(p))
    if overrides:
        merged = merge_tables(merged, overrides)
    cfg = training_config_from_dict(merged)
    cfg.config_paths = [str(p) for p in paths]
    return cfg

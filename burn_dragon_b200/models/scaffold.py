"""Random-scaffold projections with low-rank adapters.

The three shared projections become ``W = gain * W_seed + s * A @ B`` where ``W_seed`` is
a frozen tensor regenerated from (seed, path) and only A, B (and the scalar gain, when
``trainable_gain``) train (burn_dragon_core/src/model/scaffold.rs:21-124; frozen ids
dragon.rs:1190-1222). ``s = alpha / r`` ("standard") or ``alpha / sqrt(r)``
("rank_stabilized"). Shapes: headwise ``A [H, D, r]``, ``B [H, r, Nh]`` for ``encoder`` /
``encoder_v`` (paths ``shared.encoder`` / ``shared.encoder_v``), matrix ``A [N, r]``,
``B [r, D]`` for ``decoder`` (``shared.decoder``). B starts at zero, so a fresh adapter
is function-preserving; A starts uniform in +-1/sqrt(fan_in) from the same generator
(path ``<path>.adapter_a``).

Generator contract ``dragon-scaffold-v1`` (see csrc/scaffold.cu for the device side):
key = mix64(seed ^ fnv1a64(path)); u_k(i) = (mix64(key ^ mix64(12 i + k + 1)) >> 40) / 2^24;
gaussian_clt12: std * (sum_{k<12} u_k - 6); rademacher: +-std from the top bit of
mix64(key ^ mix64(12 i + 1)). ``random_scaffold_manifest.json`` records this contract
and resume refuses a different one (burn_dragon_language/src/checkpoint.rs:37-85).
"""

from __future__ import annotations

import json
import math

import numpy as np
import torch

GENERATOR_VERSION = "dragon-scaffold-v1"
PATHS = {"encoder": "shared.encoder", "encoder_v": "shared.encoder_v", "decoder": "shared.decoder"}
_M64 = (1 << 64) - 1


def fnv1a64(text: str) -> int:
    h = 0xCBF29CE484222325
    for b in text.encode():
        h ^= b
        h = (h * 0x100000001B3) & _M64
    return h


def _mix64_np(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.uint64, copy=True)
    with np.errstate(over="ignore"):
        z ^= z >> np.uint64(30)
        z *= np.uint64(0xBF58476D1CE4E5B9)
        z ^= z >> np.uint64(27)
        z *= np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return z


def _mix64_int(z: int) -> int:
    return int(_mix64_np(np.array([z], dtype=np.uint64))[0])


def tensor_key(seed: int, path: str) -> int:
    return _mix64_int((seed & _M64) ^ fnv1a64(path))


def signed64(x: int) -> int:
    return x - (1 << 64) if x >= (1 << 63) else x


def uniforms(key: int, idx: np.ndarray, k: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        c = idx.astype(np.uint64) * np.uint64(12) + np.uint64(k + 1)
    h = _mix64_np(np.uint64(key) ^ _mix64_np(c))
    return (h >> np.uint64(40)).astype(np.float64) / float(1 << 24)


def scaffold_tensor_cpu(seed: int, path: str, shape, std: float, distribution: str = "gaussian_clt12"):
    """The oracle: W_seed on the host (float32)."""
    key = tensor_key(seed, path)
    n = math.prod(shape)
    idx = np.arange(n, dtype=np.uint64)
    if distribution == "rademacher":
        with np.errstate(over="ignore"):
            c = idx * np.uint64(12) + np.uint64(1)
        h = _mix64_np(np.uint64(key) ^ _mix64_np(c))
        w = np.where((h >> np.uint64(63)) == 1, std, -std)
    elif distribution == "gaussian_clt12":
        s = np.zeros(n, dtype=np.float64)
        for k in range(12):
            s += uniforms(key, idx, k)
        w = std * (s - 6.0)
    else:
        raise ValueError(f"unknown scaffold distribution {distribution!r}")
    return torch.from_numpy(w.astype(np.float32)).reshape(shape)


def adapter_a_init(seed: int, path: str, shape, fan_in: int) -> torch.Tensor:
    key = tensor_key(seed, path + ".adapter_a")
    u = uniforms(key, np.arange(math.prod(shape), dtype=np.uint64), 0)
    bound = 1.0 / math.sqrt(fan_in)
    return torch.from_numpy(((2.0 * u - 1.0) * bound).astype(np.float32)).reshape(shape)


def adapter_shapes(cfg) -> dict[str, tuple[int, ...]]:
    D, H, Nh, r = cfg.n_embd, cfg.n_head, cfg.latent_per_head, cfg.random_scaffold.rank
    N = H * Nh
    out = {}
    for name in ("encoder", "encoder_v"):
        out[f"{name}.a"] = (H, D, r)
        out[f"{name}.b"] = (H, r, Nh)
        out[f"{name}.gain"] = (1,)
    out["decoder.a"] = (N, r)
    out["decoder.b"] = (r, D)
    out["decoder.gain"] = (1,)
    return out


def base_shape(cfg, name: str) -> tuple[int, ...]:
    D, H, Nh = cfg.n_embd, cfg.n_head, cfg.latent_per_head
    return (H * Nh, D) if name == "decoder" else (H, D, Nh)


def dist_code(distribution: str) -> int:
    return {"gaussian_clt12": 0, "rademacher": 1}[distribution]


def effective_weight(cfg, name: str, a: torch.Tensor, b: torch.Tensor, gain: torch.Tensor,
                     base: torch.Tensor) -> torch.Tensor:
    """PyTorch path (autograd through a, b, gain; base frozen)."""
    s = cfg.random_scaffold.adapter_scale()
    return base.detach() * gain.reshape([1] * base.dim()) + s * torch.matmul(a, b)


def manifest(cfg) -> dict:
    rs = cfg.random_scaffold
    full = sum(math.prod(base_shape(cfg, n)) for n in PATHS)
    shapes = adapter_shapes(cfg)
    trainable = sum(math.prod(s) for k, s in shapes.items() if not k.endswith("gain"))
    if rs.trainable_gain:
        trainable += 3
    return {
        "manifest": {
            "generator": GENERATOR_VERSION,
            "seed": rs.seed,
            "distribution": rs.distribution,
            "rank": rs.rank,
            "alpha": rs.alpha,
            "scaling": rs.scaling,
            "trainable_gain": rs.trainable_gain,
            "tensors": {PATHS[n]: {"shape": list(base_shape(cfg, n)), "std": cfg.init_std} for n in PATHS},
        },
        "full_projection_elements": full,
        "trainable_adapter_elements": trainable,
        "frozen_scaffold_elements": full,
        "fp32_size": 4 * full,
    }


def check_manifest(saved: dict, cfg) -> None:
    """Resume guard: the saved scaffold contract must equal this config's."""
    want = manifest(cfg)["manifest"]
    got = saved.get("manifest", saved)
    for k in ("generator", "seed", "distribution", "rank", "alpha", "scaling", "trainable_gain", "tensors"):
        if got.get(k) != want.get(k):
            raise ValueError(f"random scaffold manifest mismatch on {k!r}: saved {got.get(k)!r} != {want.get(k)!r}")


def write_manifest(path: str, cfg) -> None:
    with open(path, "w") as f:
        json.dump(manifest(cfg), f, indent=2, sort_keys=True)

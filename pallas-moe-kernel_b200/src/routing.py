"""Group-size generators and seeded synthetic inputs for the expert MLP.

* ``make_group_sizes`` -- ``src/benchmark.py:42-91`` of the reference
  (linspace(0.85, 1.15) weights by default, largest-remainder rounding).
* ``routing_weights`` / ``make_group_sizes_pattern`` --
  ``src/ragged_moe_speedup_experiment.py:455-493`` (balanced / mild /
  skewed Zipf(1.25) / one_dominant 70%, at least one token per expert).
* Seeded generators for the five benchmark configurations (uniform
  multinomial routing, Zipf(1.2) skew with empty experts, top-k routers),
  with X ~ N(0, 1), W_up ~ N(0, 1/D), W_down ~ N(0, 1/F).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np


# --------------------------------------------------------------------- reference generators
def make_group_sizes(M: int, E: int, group_fractions: Optional[Sequence[float]] = None) -> np.ndarray:
    """Largest-remainder split of M rows over E experts
    (``src/benchmark.py:42-91``)."""
    if M < E:
        raise ValueError(f"need M >= E to give each of the {E} experts a row (M={M})")
    if group_fractions is None:
        weights = np.linspace(0.85, 1.15, E, dtype=np.float64)
    else:
        weights = np.asarray(group_fractions, dtype=np.float64)
        if weights.shape != (E,):
            raise ValueError(f"group_fractions: expected {E} values, got shape {weights.shape}")
        if np.any(weights <= 0):
            raise ValueError("group_fractions: all values must be > 0")
    weights = weights / weights.sum()
    exact = M * weights
    sizes = np.floor(exact).astype(np.int32)
    remainder = M - int(sizes.sum())
    order = np.argsort(-(exact - sizes))
    sizes[order[:remainder]] += 1
    assert int(sizes.sum()) == M
    return sizes


def routing_weights(E: int, pattern: str) -> np.ndarray:
    """Normalised expert weights per routing pattern
    (``src/ragged_moe_speedup_experiment.py:455-472``)."""
    if pattern == "balanced":
        w = np.ones(E, dtype=np.float64)
    elif pattern == "mild":
        w = np.linspace(0.85, 1.15, E, dtype=np.float64)
    elif pattern == "skewed":
        ranks = np.arange(1, E + 1, dtype=np.float64)
        w = 1.0 / np.power(ranks, 1.25)
    elif pattern == "one_dominant":
        if E == 1:
            w = np.ones(1, dtype=np.float64)
        else:
            w = np.full(E, 0.30 / (E - 1), dtype=np.float64)
            w[0] = 0.70
    else:
        raise ValueError(f"routing pattern {pattern!r} is not one of balanced, mild, skewed, one_dominant")
    return w / w.sum()


def make_group_sizes_pattern(M: int, E: int, pattern: str) -> np.ndarray:
    """At least one token per expert, the rest by largest remainders
    (``src/ragged_moe_speedup_experiment.py:475-493``)."""
    if M < E:
        raise ValueError(f"need M >= E (M={M}, E={E})")
    w = routing_weights(E, pattern)
    remaining = M - E
    exact = remaining * w
    extra = np.floor(exact).astype(np.int64)
    rem = remaining - int(extra.sum())
    if rem > 0:
        order = np.argsort(-(exact - extra))
        extra[order[:rem]] += 1
    sizes = (extra + 1).astype(np.int32)
    if int(sizes.sum()) != M:
        raise AssertionError(f"group sizes sum to {int(sizes.sum())}, expected {M}")
    return sizes


# --------------------------------------------------------------------- synthetic routing
def multinomial_group_sizes(M: int, E: int, rng: np.random.Generator) -> np.ndarray:
    """Uniform multinomial routing of M rows over E experts."""
    return rng.multinomial(M, np.full(E, 1.0 / E)).astype(np.int32)


def zipf_group_sizes(M: int, E: int, rng: np.random.Generator, s: float = 1.2, min_empty: int = 3,
                     dominant: float = 0.5) -> np.ndarray:
    """Zipf(s) routing over a random expert order, with at least ``min_empty``
    experts receiving no rows and the top expert holding >= ``dominant`` of M."""
    perm = rng.permutation(E)
    ranks = np.arange(1, E + 1, dtype=np.float64)
    w = 1.0 / ranks ** s
    w[E - min_empty:] = 0.0            # the lowest-ranked experts stay empty
    w /= w.sum()
    counts = rng.multinomial(M, w).astype(np.int64)
    need = int(np.ceil(dominant * M)) - int(counts[0])
    if need > 0:                        # move rows from the tail into the top expert
        for r in range(E - 1, 0, -1):
            take = min(need, int(counts[r]))
            counts[r] -= take
            counts[0] += take
            need -= take
            if need == 0:
                break
    out = np.zeros(E, dtype=np.int32)
    out[perm] = counts
    return out


def topk_group_sizes(tokens: int, E: int, k: int, rng: np.random.Generator,
                     softmax: bool = False) -> np.ndarray:
    """Router with N(0, 1) logits (optionally softmaxed), top-k experts per
    token; returns the per-expert row counts of the k*tokens routed rows."""
    logits = rng.standard_normal((tokens, E), dtype=np.float32)
    if softmax:
        logits = np.exp(logits - logits.max(axis=1, keepdims=True))
        logits /= logits.sum(axis=1, keepdims=True)
    top = np.argpartition(-logits, k - 1, axis=1)[:, :k]
    return np.bincount(top.reshape(-1), minlength=E).astype(np.int32)


# --------------------------------------------------------------------- configurations
@dataclass(frozen=True)
class MoeConfig:
    name: str
    M: int
    D: int
    F: int
    E: int
    dtype: str          # "f32", "bf16" or "fp8"
    routing: str        # "multinomial", "zipf", "top2", "top8_softmax"
    tokens: int = 0     # router input tokens (top-k configs)

    @property
    def flops(self) -> int:
        return 4 * self.M * self.D * self.F


CONFIGS = {
    "c1": MoeConfig("c1_fp32_M4096_D128_F1024_E8", 4096, 128, 1024, 8, "f32", "multinomial"),
    "c2": MoeConfig("c2_fp32_M65536_D128_F512_E8", 65536, 128, 512, 8, "f32", "multinomial"),
    "c3": MoeConfig("c3_fp32_M4096_D256_F2048_E16_zipf", 4096, 256, 2048, 16, "f32", "zipf"),
    "c4": MoeConfig("c4_bf16_M32768_D4096_F14336_E8_top2", 32768, 4096, 14336, 8, "bf16", "top2", 16384),
    "c5": MoeConfig("c5_fp8_M65536_D7168_F2048_E256_top8", 65536, 7168, 2048, 256, "fp8", "top8_softmax", 8192),
}


def config_group_sizes(cfg: MoeConfig, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if cfg.routing == "multinomial":
        return multinomial_group_sizes(cfg.M, cfg.E, rng)
    if cfg.routing == "zipf":
        return zipf_group_sizes(cfg.M, cfg.E, rng)
    if cfg.routing == "top2":
        return topk_group_sizes(cfg.tokens, cfg.E, 2, rng)
    if cfg.routing == "top8_softmax":
        return topk_group_sizes(cfg.tokens, cfg.E, 8, rng, softmax=True)
    raise ValueError(cfg.routing)


def with_shape(cfg: MoeConfig, **kw) -> MoeConfig:
    d = dict(cfg.__dict__)
    d.update(kw)
    return MoeConfig(**d)


def make_inputs_numpy(M: int, D: int, F: int, E: int, seed: int = 0):
    """X ~ N(0,1) (M, D), W_up ~ N(0, 1/D) (E, D, F), W_down ~ N(0, 1/F)
    (E, F, D), float32."""
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((M, D), dtype=np.float32)
    w_up = rng.standard_normal((E, D, F), dtype=np.float32) * np.float32(1.0 / np.sqrt(D))
    w_down = rng.standard_normal((E, F, D), dtype=np.float32) * np.float32(1.0 / np.sqrt(F))
    return x, w_up, w_down


def quantize_e4m3_blockwise(w, block: int = 128):
    """FP8 e4m3 weights with per-(block x block) f32 scales: for each block of
    the last two dims, scale = amax / 448 (the e4m3 maximum) and
    q = round_to_e4m3(w / scale).  ``w`` is a torch tensor (..., R, C); a
    partial block at the end of R or C has a scale of its own.  Returns
    (q float8_e4m3fn (..., R, C), scale f32 (..., ceil(R/block),
    ceil(C/block))); dequantisation is q * scale per block."""
    import torch
    *lead, R, C = w.shape
    rb, cb = -(-R // block), -(-C // block)
    wp = torch.zeros((*lead, rb * block, cb * block), dtype=torch.float32, device=w.device)
    wp[..., :R, :C] = w.float()
    wb = wp.reshape(*lead, rb, block, cb, block)
    amax = wb.abs().amax(dim=(-3, -1))                         # (..., rb, cb)
    scale = torch.clamp(amax, min=1e-30) / 448.0
    q = (wb / scale[..., :, None, :, None]).reshape(*lead, rb * block, cb * block)[..., :R, :C]
    return q.contiguous().to(torch.float8_e4m3fn), scale.contiguous()


def dequantize_e4m3_blockwise(q, scale, block: int = 128):
    """q * scale per (block x block) tile (partial tiles at the ends), as float32."""
    *lead, R, C = q.shape
    s = scale.repeat_interleave(block, dim=-2).repeat_interleave(block, dim=-1)[..., :R, :C]
    return q.float() * s

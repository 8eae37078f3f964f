"""Seeded synthetic weights and inputs for BASELINE's configs.

There is no checkpoint or dataset here, so every run uses random-init weights of the named shape
and N(0, 1) input embeddings, drawn by numpy's PCG64 generator (`np.random.default_rng(seed)`,
`standard_normal` in float32), which gives the same numbers on every machine:

- weights: per layer, in this order, q_proj, k_proj, v_proj, o_proj, gate_proj, up_proj,
  down_proj, each N(0, 0.02) from one generator seeded `seed`; RMSNorm gains 1 (input,
  post-attention and the final norm), or 1 + 0.1 N(0, 1) from a generator seeded `seed + 1000`
  when `jitter_gains` (tests use that, so that a gain left out shows);
- bf16 weights are the f32 draws rounded to nearest even (`bf16_round`).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

WEIGHT_ORDER = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


@dataclass(frozen=True)
class Config:
    name: str
    hidden: int
    inner: int
    heads: int
    kv_heads: int
    head_dim: int
    layers: int
    dtype: str
    eps: float = 1e-5
    rope_theta: float = 10000.0

    @property
    def residual_scale(self) -> float:
        """1.4 / sqrt(layers), as f32 ("residual scale 1.4/sqrt(layers)")."""
        return float(np.float32(1.4 / math.sqrt(self.layers)))


# BASELINE.json configs[0] and configs[1..4]'s backbone.
TINY = Config("tiny", hidden=256, inner=1024, heads=4, kv_heads=1, head_dim=64, layers=4, dtype="f32")
S05B = Config("0p5b", hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=24, dtype="bf16")
CONFIGS = {"tiny": TINY, "0p5b": S05B}


def shape_of(cfg: Config, capacity: int, layers: int | None = None):
    """The package's Shape for `cfg` with a cache of `capacity` positions."""
    from . import Shape

    return Shape(hidden=cfg.hidden, inner=cfg.inner, heads=cfg.heads, kv_heads=cfg.kv_heads,
                 head_dim=cfg.head_dim, layers=cfg.layers if layers is None else layers,
                 capacity=capacity, eps=cfg.eps, rope_theta=cfg.rope_theta,
                 residual_scale=cfg.residual_scale)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The bf16 bits of f32 values, rounded to nearest even (finite values: the low 16 bits are
    rounded into the high 16, ties to the even result)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 values rounded to bf16 and widened back: the values a bf16 copy holds."""
    return bf16_to_f32(bf16_bits(x))


def weight_shapes(cfg: Config, layers: int | None = None) -> dict[str, tuple[int, ...]]:
    L = cfg.layers if layers is None else layers
    h, i, d = cfg.hidden, cfg.inner, cfg.head_dim
    out: dict[str, tuple[int, ...]] = {}
    for l in range(L):
        out[f"layers.{l}.self_attn.q_proj.weight"] = (cfg.heads * d, h)
        out[f"layers.{l}.self_attn.k_proj.weight"] = (cfg.kv_heads * d, h)
        out[f"layers.{l}.self_attn.v_proj.weight"] = (cfg.kv_heads * d, h)
        out[f"layers.{l}.self_attn.o_proj.weight"] = (h, cfg.heads * d)
        out[f"layers.{l}.mlp.gate_proj.weight"] = (i, h)
        out[f"layers.{l}.mlp.up_proj.weight"] = (i, h)
        out[f"layers.{l}.mlp.down_proj.weight"] = (h, i)
        out[f"layers.{l}.input_layernorm.weight"] = (h,)
        out[f"layers.{l}.post_attention_layernorm.weight"] = (h,)
    out["norm.weight"] = (h,)
    return out


def make_weights(cfg: Config, seed: int = 0, layers: int | None = None, std: float = 0.02,
                 jitter_gains: bool = False, as_bits: bool = False) -> dict[str, np.ndarray]:
    """Every weight of the stack by upstream name: f32 arrays (bf16-valued for bf16 configs), or
    with `as_bits` the uint16 bf16 bits of the bf16 configs' projections."""
    L = cfg.layers if layers is None else layers
    shapes = weight_shapes(cfg, L)
    rng = np.random.default_rng(seed)
    gain_rng = np.random.default_rng(seed + 1000)
    out: dict[str, np.ndarray] = {}
    for l in range(L):
        for w in WEIGHT_ORDER:
            name = f"layers.{l}.{w}.weight"
            v = rng.standard_normal(shapes[name], dtype=np.float32) * np.float32(std)
            if cfg.dtype == "bf16":
                v = bf16_bits(v) if as_bits else bf16_round(v)
            out[name] = v
        for g in ("input_layernorm", "post_attention_layernorm"):
            name = f"layers.{l}.{g}.weight"
            out[name] = _gain(cfg.hidden, gain_rng if jitter_gains else None)
    out["norm.weight"] = _gain(cfg.hidden, gain_rng if jitter_gains else None)
    return out


def _gain(n: int, rng) -> np.ndarray:
    if rng is None:
        return np.ones(n, np.float32)
    return (1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)


def make_inputs(rows: int, hidden: int, seed: int = 1, bf16: bool = False) -> np.ndarray:
    """N(0, 1) input embeddings [rows][hidden] (bf16-valued when `bf16`)."""
    x = np.random.default_rng(seed).standard_normal((rows, hidden), dtype=np.float32)
    return bf16_round(x) if bf16 else x


def as_f32(weights: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Weights with any bf16 bits widened to f32."""
    return {k: (bf16_to_f32(v) if v.dtype == np.uint16 else v) for k, v in weights.items()}

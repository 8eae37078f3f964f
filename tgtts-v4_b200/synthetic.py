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
# VoxCPM2's base LM (crates/graph/src/decode.rs:946-947's known answer: 2048 wide, 6144 inner,
# 16 heads of 128 over 2 key-value heads, 28 layers): the shape a tgtts-v4 deployment runs.
VOXCPM2_LM = Config("voxcpm2_lm", hidden=2048, inner=6144, heads=16, kv_heads=2, head_dim=128, layers=28,
                    dtype="bf16")
CONFIGS = {"tiny": TINY, "0p5b": S05B, "voxcpm2_lm": VOXCPM2_LM}


def shape_of(cfg: Config, capacity: int, layers: int | None = None):
    """The package's Shape for `cfg` with a cache of `capacity` positions."""
    from . import Shape

    return Shape(hidden=cfg.hidden, inner=cfg.inner, heads=cfg.heads, kv_heads=cfg.kv_heads,
                 head_dim=cfg.head_dim, layers=cfg.layers if layers is None else layers,
                 capacity=capacity, eps=cfg.eps, rope_theta=cfg.rope_theta,
                 residual_scale=cfg.residual_scale)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The bf16 bits of f32 values, rounded to nearest even (finite values: the low 16 bits are
    rounded into the high 16, ties to the even result). The sum is taken in u32: where it wraps
    (only negative NaNs), its high 16 bits are those of the exact sum modulo 2^16, the same bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += u
    r += np.uint32(0x7FFF)
    r >>= 16
    return r.astype(np.uint16)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    u = bits.astype(np.uint32)
    u <<= 16
    return u.view(np.float32)


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


# ---- VoxCPM2's local stacks (crates/graph/src/local) ---------------------------------------------
#
# VoxCPM2's local DiT and local encoder are 1024 wide with 4096 inner, 16 heads of 128 over the base
# LM's 2 key-value heads, patches of 4 frames of 64 channels (crates/graph/src/patch.rs:482-525).
# Their layer count comes from the checkpoint's config.json, which is not here: LOCAL_VOXCPM2
# takes 8. LOCAL_SMALL is a small stack of the same form for parity tests.

@dataclass(frozen=True)
class LocalConfig:
    name: str
    hidden: int
    inner: int
    heads: int
    kv_heads: int
    head_dim: int
    layers: int
    feat_dim: int
    patch_size: int
    eps: float = 1e-5
    rope_theta: float = 10000.0


LOCAL_SMALL = LocalConfig("local_small", hidden=256, inner=512, heads=4, kv_heads=2, head_dim=64,
                          layers=2, feat_dim=16, patch_size=4)
LOCAL_VOXCPM2 = LocalConfig("voxcpm2_local", hidden=1024, inner=4096, heads=16, kv_heads=2,
                            head_dim=128, layers=8, feat_dim=64, patch_size=4)
LOCAL_CONFIGS = {"local_small": LOCAL_SMALL, "voxcpm2_local": LOCAL_VOXCPM2}


def local_shape(cfg: LocalConfig, layers: int | None = None):
    """The package's Shape of a local stack (the sampler and the encoder set its capacity)."""
    from . import Shape

    return Shape(hidden=cfg.hidden, inner=cfg.inner, heads=cfg.heads, kv_heads=cfg.kv_heads,
                 head_dim=cfg.head_dim, layers=cfg.layers if layers is None else layers, capacity=1,
                 eps=cfg.eps, rope_theta=cfg.rope_theta)


def _local_stack_weights(cfg: LocalConfig, prefix: str, rng, gain_rng, std: float, layers: int) -> dict:
    h, i, d = cfg.hidden, cfg.inner, cfg.head_dim
    shapes = {"self_attn.q_proj": (cfg.heads * d, h), "self_attn.k_proj": (cfg.kv_heads * d, h),
              "self_attn.v_proj": (cfg.kv_heads * d, h), "self_attn.o_proj": (h, cfg.heads * d),
              "mlp.gate_proj": (i, h), "mlp.up_proj": (i, h), "mlp.down_proj": (h, i)}
    out = {}
    for l in range(layers):
        for w in WEIGHT_ORDER:
            out[f"{prefix}layers.{l}.{w}.weight"] = rng.standard_normal(shapes[w], dtype=np.float32) * np.float32(std)
        for g in ("input_layernorm", "post_attention_layernorm"):
            out[f"{prefix}layers.{l}.{g}.weight"] = _gain(h, gain_rng)
    out[f"{prefix}norm.weight"] = _gain(h, gain_rng)
    return out


def make_sampler_weights(cfg: LocalConfig, seed: int = 0, layers: int | None = None,
                         std: float = 0.02) -> dict[str, np.ndarray]:
    """Every tensor of the sampler (load_sampler's names, crates/graph/src/local/dit.rs:325-370),
    f32: the stack's projections, in_proj, cond_proj, out_proj and the two timestep MLPs N(0, std),
    their biases N(0, std), gains 1 + 0.1 N(0, 1); drawn in that order from generators seeded
    `seed` and `seed + 1000`."""
    L = cfg.layers if layers is None else layers
    rng, gain_rng = np.random.default_rng(seed), np.random.default_rng(seed + 1000)
    p = "feat_decoder.estimator."
    out = _local_stack_weights(cfg, p + "decoder.", rng, gain_rng, std, L)
    h, f = cfg.hidden, cfg.feat_dim
    for name, shape in (("in_proj", (h, f)), ("cond_proj", (h, f)), ("out_proj", (f, h))):
        out[f"{p}{name}.weight"] = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        out[f"{p}{name}.bias"] = rng.standard_normal(shape[0], dtype=np.float32) * np.float32(std)
    for mlp in ("time_mlp", "delta_time_mlp"):
        for i in (1, 2):
            out[f"{p}{mlp}.linear_{i}.weight"] = rng.standard_normal((h, h), dtype=np.float32) * np.float32(std)
            out[f"{p}{mlp}.linear_{i}.bias"] = rng.standard_normal(h, dtype=np.float32) * np.float32(std)
    return out


def make_encoder_weights(cfg: LocalConfig, seed: int = 0, layers: int | None = None,
                         std: float = 0.02) -> dict[str, np.ndarray]:
    """Every tensor of the local encoder (load_encoder's names, encoder.rs:129-157), f32: as
    make_sampler_weights, with the learned token N(0, 1)."""
    L = cfg.layers if layers is None else layers
    rng, gain_rng = np.random.default_rng(seed), np.random.default_rng(seed + 1000)
    p = "feat_encoder."
    out = _local_stack_weights(cfg, p + "encoder.", rng, gain_rng, std, L)
    h, f = cfg.hidden, cfg.feat_dim
    out[p + "in_proj.weight"] = rng.standard_normal((h, f), dtype=np.float32) * np.float32(std)
    out[p + "in_proj.bias"] = rng.standard_normal(h, dtype=np.float32) * np.float32(std)
    out[p + "special_token"] = rng.standard_normal(h, dtype=np.float32)
    return out


# The temperatures and guidance scales the reference's local tests cycle through
# (crates/graph/tests/local.rs:118-121), and voxcpm's defaults first.
SAMPLING_PAIRS = ([1.0, 2.0], [1.0, 2.0], [1.0, 2.0], [0.8, 1.5], [1.2, 3.0], [1.0, 2.5])


def make_sampler_inputs(cfg: LocalConfig, rows: int, seed: int = 1):
    """Each row's mu ([rows][2][hidden], U(-1.7, 1.7) rounded to f16: about a normed hidden state's
    scale, as the reference's cases draw them), the patch before and the noise ([rows][feat]
    [patch] N(0, 1)), and its sampling pair."""
    rng = np.random.default_rng(seed)
    mu = rng.uniform(-1.7, 1.7, (rows, 2, cfg.hidden)).astype(np.float16)
    cond = rng.standard_normal((rows, cfg.feat_dim, cfg.patch_size), dtype=np.float32)
    noise = rng.standard_normal((rows, cfg.feat_dim, cfg.patch_size), dtype=np.float32)
    sampling = np.array([SAMPLING_PAIRS[r % len(SAMPLING_PAIRS)] for r in range(rows)], np.float32)
    return mu, cond, noise, sampling

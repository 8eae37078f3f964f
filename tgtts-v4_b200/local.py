"""VoxCPM2's local stacks on the GPU: the patch sampler with its local DiT and the local encoder
(crates/graph/src/local/{mod,dit,encoder}.rs).

Each is a bidirectional MiniCPM-4 stack over the few tokens of one patch per sequence, f16 weights
and activations with f32 sums, recorded once as one program (a CUDA graph of the local kernels,
`tgtts-v4_b200/csrc/local.cu`) and run whole. A row's results are the same bits whatever rows run
beside it (local/mod.rs:9-11).

- `PatchConfig`, `StackConfig`, `DitConfig`: what VoxCPM2's config.json says of the local stacks
  (local/mod.rs:120-170); `PatchConfig.stack` derives a stack's `Shape` as upstream does.
- `Tuning`: the column parts of the q/k/v, output and down projections' sums (local/mod.rs:187-214),
  which decide the order of the sums and nothing else.
- `schedule`, `euler_steps`: the sampler's times (dit.rs:39-81).
- `Sampler` (dit.rs:273-323) and `Encoder` (encoder.rs:160-215).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace
from typing import Mapping, Optional

import numpy as np

from . import (F16, F32, BF16, Context, Error, LmConfig, Shape, ShapeError, TgLocalTuning,
               _FP, check, library)

MU_TOKENS = 2  # dit.rs:35: the condition tokens leading the DiT's sequence
SAMPLER_PREFIX = "feat_decoder.estimator."
ENCODER_PREFIX = "feat_encoder."
LAYER_WEIGHTS = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                 "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                 "mlp.down_proj.weight", "input_layernorm.weight", "post_attention_layernorm.weight")


@dataclass
class StackConfig:
    """`encoder_config`, or the stack of `dit_config` (local/mod.rs:132-141)."""

    hidden_dim: int
    ffn_dim: int
    num_heads: int
    num_layers: int
    kv_channels: Optional[int] = None


@dataclass
class DitConfig:
    stack: StackConfig
    mean_mode: bool = False
    dit_mean_mode: bool = False


@dataclass
class PatchConfig:
    """What VoxCPM2's config.json says of the local stacks (local/mod.rs:120-130)."""

    lm_config: LmConfig
    patch_size: int
    feat_dim: int
    encoder_config: StackConfig
    dit_config: DitConfig

    @classmethod
    def from_dict(cls, d: Mapping) -> "PatchConfig":
        def stack(s):
            return StackConfig(s["hidden_dim"], s["ffn_dim"], s["num_heads"], s["num_layers"],
                               s.get("kv_channels"))

        dit = d["dit_config"]
        return cls(LmConfig.from_dict(d["lm_config"]), d["patch_size"], d["feat_dim"],
                   stack(d["encoder_config"]),
                   DitConfig(stack(dit), bool(dit.get("mean_mode", False)),
                             bool(dit.get("dit_mean_mode", False))))

    def stack(self, stack: StackConfig, tokens: int) -> Shape:
        """PatchConfig::stack (local/mod.rs:153-170): head count and width are the stack's, the
        rest the base LM's; sequences of `tokens` tokens."""
        config = replace(self.lm_config, hidden_size=stack.hidden_dim,
                         intermediate_size=stack.ffn_dim, num_attention_heads=stack.num_heads,
                         num_hidden_layers=stack.num_layers, kv_channels=stack.kv_channels,
                         residual_scale=1.0)
        return Shape.new(config, stack.num_layers, tokens)


@dataclass
class Tuning:
    """The column parts of the q/k/v, output and down projections' sums (0: the default, 4, 8
    and 8, or the most that cut the width into multiples of 64)."""

    qkv_parts: int = 0
    o_parts: int = 0
    down_parts: int = 0

    def _c(self) -> TgLocalTuning:
        return TgLocalTuning(self.qkv_parts, self.o_parts, self.down_parts)


def schedule(timesteps: int) -> np.ndarray:
    """dit.rs:41-54: the timesteps + 1 times the sampler steps through, f32."""
    out = np.zeros(timesteps + 1, np.float32)
    check(library().tg_cfm_schedule(timesteps, out.ctypes.data_as(_FP)))
    return out


def euler_steps(timesteps: int) -> list[tuple[float, float]]:
    """dit.rs:59-76: the (time, step length) of each step the DiT runs at."""
    n = ctypes.c_size_t()
    check(library().tg_cfm_euler_steps(timesteps, None, None, 0, ctypes.byref(n)))
    t = np.zeros(max(n.value, 1), np.float32)
    dt = np.zeros_like(t)
    check(library().tg_cfm_euler_steps(timesteps, t.ctypes.data_as(_FP), dt.ctypes.data_as(_FP),
                                       n.value, ctypes.byref(n)))
    return [(float(a), float(b)) for a, b in zip(t[:n.value], dt[:n.value])]


def stack_weight_names(layers: int, prefix: str) -> list[str]:
    names = [f"{prefix}layers.{l}.{w}" for l in range(layers) for w in LAYER_WEIGHTS]
    return names + [f"{prefix}norm.weight"]


def sampler_weight_names(layers: int) -> list[str]:
    """Every tensor load_sampler reads (dit.rs:325-370)."""
    p = SAMPLER_PREFIX
    names = stack_weight_names(layers, p + "decoder.")
    for lin in ("in_proj", "cond_proj", "out_proj"):
        names += [f"{p}{lin}.weight", f"{p}{lin}.bias"]
    for mlp in ("time_mlp", "delta_time_mlp"):
        for i in (1, 2):
            names += [f"{p}{mlp}.linear_{i}.weight", f"{p}{mlp}.linear_{i}.bias"]
    return names


def encoder_weight_names(layers: int) -> list[str]:
    """Every tensor load_encoder reads (encoder.rs:129-157)."""
    p = ENCODER_PREFIX
    return stack_weight_names(layers, p + "encoder.") + [
        p + "special_token", p + "in_proj.weight", p + "in_proj.bias"]


def tiled(w: np.ndarray) -> np.ndarray:
    """W [n][k] (n a multiple of 128, k of 64) as f16 in the tiled layout the local projections read
    (TG_KERNEL_LOCAL_PARTIAL): each 128 rows x 64 columns one contiguous 16 KiB block, blocks in
    row-block then column-block order, a block's rows 128 bytes apart with row r's 16-byte chunk c
    at chunk c ^ (r % 8) (the 128-byte swizzle). The layout plays the part of local::tiled
    (local/mod.rs:737-755): each block's share of W is one stream."""
    w = np.asarray(w, np.float16)
    n, k = w.shape
    if n % 128 or k % 64:
        raise ShapeError(f"a {n} x {k} weight is not whole 128 x 64 blocks")
    x = w.reshape(n // 128, 16, 8, k // 64, 8, 8).transpose(0, 3, 1, 2, 4, 5)  # t, b, r/8, r%8, c, e
    out = np.empty_like(x)
    for lo in range(8):
        out[:, :, :, lo, [c ^ lo for c in range(8)], :] = x[:, :, :, lo, :, :]
    return out.reshape(-1)


def _src(values: np.ndarray):
    a = np.ascontiguousarray(values)
    if a.dtype == np.float16:
        return a, F16
    if a.dtype == np.uint16:  # bf16 bits, as the decoder takes them
        return a, BF16
    return np.ascontiguousarray(a, dtype=np.float32), F32


class _Program:
    """What the sampler and the encoder share: a handle, its timings and labels."""

    _prefix = ""

    def _fn(self, name):
        return getattr(library(), f"tg_{self._prefix}_{name}")

    def load(self, weights: Mapping[str, np.ndarray]) -> None:
        """Every tensor by its upstream name, from f32, f16 or bf16-bit (uint16) arrays."""
        for name in self.weight_names():
            if name not in weights:
                raise Error(f"checkpoint: no tensor {name}")
            self.load_tensor(name, weights[name])

    def load_tensor(self, name: str, values: np.ndarray) -> None:
        a, src = _src(values)
        check(self._fn("load")(self.handle, name.encode(), a.ctypes.data, a.size, src))

    def load_checkpoint(self, path) -> None:
        """load_sampler / load_encoder from a safetensors file (crates/graph/src/checkpoint.rs):
        every tensor by its upstream name, read a tensor at a time, rounded to f16."""
        from .checkpoint import Checkpoint

        with Checkpoint(path) as ck:
            for name in self.weight_names():
                if ck.shape(name) is None:
                    raise Error(f"checkpoint: no tensor {name}")
                self.load_tensor(name, ck.tensor(name))

    def wait(self, timeout_ns: int = 0) -> None:
        check(self._fn("wait")(self.handle, timeout_ns))

    def elapsed_ns(self) -> float:
        ns = ctypes.c_double()
        check(self._fn("elapsed_ns")(self.handle, ctypes.byref(ns)))
        return ns.value

    def labels(self) -> list[str]:
        n = ctypes.c_size_t()
        check(self._fn("timings")(self.handle, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(256)
        out = []
        for i in range(n.value):
            check(self._fn("dispatch_label")(self.handle, i, buf, 256))
            out.append(buf.value.decode())
        return out

    def timings(self) -> list[tuple[str, float]]:
        """Each dispatch's label and GPU time (ns) in the last run, when created timed."""
        labels = self.labels()
        ns = (ctypes.c_double * len(labels))()
        check(self._fn("timings")(self.handle, ns, len(labels), None))
        return list(zip(labels, list(ns)))

    @property
    def weight_bytes(self) -> int:
        return int(self._fn("weight_bytes")(self.handle))

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._fn("destroy")(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Sampler(_Program):
    """VoxCPM2's patch sampler on the GPU (Sampler, dit.rs:273-323): `timesteps` Euler steps of
    the local DiT over `rows` rows, each a request of its own, every weight zero until loaded."""

    _prefix = "sampler"

    def __init__(self, ctx: Context, shape: Shape, feat_dim: int, patch_size: int, timesteps: int,
                 rows: int, tuning: Optional[Tuning] = None, timed: bool = False):
        self.ctx, self.shape, self.rows = ctx, shape, rows
        self.feat_dim, self.patch_size, self.timesteps = feat_dim, patch_size, timesteps
        s, self._keep = shape._c()
        h = ctypes.c_void_p()
        t = (tuning or Tuning())._c()
        check(library().tg_sampler_create(ctx.handle, ctypes.byref(s), feat_dim, patch_size,
                                          timesteps, rows, ctypes.byref(t), int(timed),
                                          ctypes.byref(h)))
        self.handle = h

    @classmethod
    def from_config(cls, ctx: Context, config: PatchConfig, timesteps: int, rows: int,
                    tuning: Optional[Tuning] = None, timed: bool = False) -> "Sampler":
        """Sampler::new (dit.rs:280-295): refuses the DiT's mean mode, as voxcpm does."""
        dit = config.dit_config
        if dit.mean_mode or dit.dit_mean_mode:
            raise ShapeError("the DiT's mean mode")
        tokens = MU_TOKENS + 1 + 2 * config.patch_size
        shape = config.stack(dit.stack, tokens)
        return cls(ctx, shape, config.feat_dim, config.patch_size, timesteps, rows, tuning, timed)

    def weight_names(self) -> list[str]:
        return sampler_weight_names(self.shape.layers)

    def steps(self) -> list[tuple[float, float]]:
        n = ctypes.c_size_t()
        check(library().tg_sampler_steps(self.handle, None, None, 0, ctypes.byref(n)))
        t = np.zeros(max(n.value, 1), np.float32)
        dt = np.zeros_like(t)
        check(library().tg_sampler_steps(self.handle, t.ctypes.data_as(_FP), dt.ctypes.data_as(_FP),
                                         n.value, ctypes.byref(n)))
        return [(float(a), float(b)) for a, b in zip(t[:n.value], dt[:n.value])]

    def sample(self, mu: np.ndarray, cond: np.ndarray, noise: np.ndarray,
               sampling: np.ndarray) -> np.ndarray:
        """Sampler::sample (dit.rs:298-313): mu [rows][2][hidden] (f16, or values rounded to
        it), cond and noise [rows][feat_dim][patch_size] f32, sampling [rows][2] (temperature,
        guidance scale) -> each row's patch, [rows][feat_dim][patch_size] f32."""
        H, R = self.shape.hidden, self.rows
        mu = np.ascontiguousarray(np.asarray(mu, np.float16).reshape(R, MU_TOKENS, H))
        cond = np.ascontiguousarray(np.asarray(cond, np.float32).reshape(R, self.feat_dim, self.patch_size))
        noise = np.ascontiguousarray(np.asarray(noise, np.float32).reshape(cond.shape))
        sampling = np.ascontiguousarray(np.asarray(sampling, np.float32).reshape(R, 2))
        out = np.empty_like(cond)
        check(library().tg_sampler_sample(self.handle, mu.ctypes.data, cond.ctypes.data_as(_FP),
                                          noise.ctypes.data_as(_FP), sampling.ctypes.data_as(_FP),
                                          out.ctypes.data_as(_FP)))
        return out

    def sample_device(self, mu_ptr: int, cond_ptr: int, noise_ptr: int, sampling_ptr: int,
                      patch_ptr: int) -> None:
        """The same from device pointers, enqueued on the context's stream, not waited for."""
        check(library().tg_sampler_sample_device(self.handle, mu_ptr, cond_ptr, noise_ptr,
                                                 sampling_ptr, patch_ptr))


class Encoder(_Program):
    """VoxCPM2's local encoder on the GPU (Encoder, encoder.rs:160-215): each of `rows` rows'
    patch embedded, every weight zero until loaded."""

    _prefix = "encoder"

    def __init__(self, ctx: Context, shape: Shape, feat_dim: int, patch_size: int, rows: int,
                 tuning: Optional[Tuning] = None, timed: bool = False):
        self.ctx, self.shape, self.rows = ctx, shape, rows
        self.feat_dim, self.patch_size = feat_dim, patch_size
        s, self._keep = shape._c()
        h = ctypes.c_void_p()
        t = (tuning or Tuning())._c()
        check(library().tg_encoder_create(ctx.handle, ctypes.byref(s), feat_dim, patch_size, rows,
                                          ctypes.byref(t), int(timed), ctypes.byref(h)))
        self.handle = h

    @classmethod
    def from_config(cls, ctx: Context, config: PatchConfig, rows: int,
                    tuning: Optional[Tuning] = None, timed: bool = False) -> "Encoder":
        shape = config.stack(config.encoder_config, 1 + config.patch_size)
        return cls(ctx, shape, config.feat_dim, config.patch_size, rows, tuning, timed)

    def weight_names(self) -> list[str]:
        return encoder_weight_names(self.shape.layers)

    def encode(self, patches: np.ndarray) -> np.ndarray:
        """Encoder::encode: patches [rows][feat_dim][patch_size] f32 -> each row's embedding,
        [rows][hidden] f16."""
        p = np.ascontiguousarray(np.asarray(patches, np.float32).reshape(
            self.rows, self.feat_dim, self.patch_size))
        out = np.empty((self.rows, self.shape.hidden), np.float16)
        check(library().tg_encoder_encode(self.handle, p.ctypes.data_as(_FP), out.ctypes.data))
        return out

    def encode_device(self, patches_ptr: int, out_ptr: int) -> None:
        check(library().tg_encoder_encode_device(self.handle, patches_ptr, out_ptr))

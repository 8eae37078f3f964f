"""TEST INFRASTRUCTURE ONLY: the CPU oracle the parity tests, `__graft_entry__.smoke()` and the
CPU-baseline legs of `bench.py` check the CUDA path against. The product (libtgcuda.so and the
tgtts-v4_b200 package) never imports, links or calls anything here.

`OracleStack` holds one stack's f32 weights and KV caches and runs the C restatement
(minicpm4_ref.c) of tgtts-v4's decode step (crates/graph/src/decode.rs:618-735) and prefill
(crates/graph/src/prefill.rs:318-411). `ref_numpy` is an independent numpy restatement used to
cross-check it. Pinned against the reference's known answers (the testkit rms_layernorm golden,
the RoPE table answers, zero weights giving zero, the sequential-K GEMM); whole-stack parity
against the reference itself is unpinned (its backbone goldens need the external VoxCPM2
checkpoint, and it cannot run here).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import Mapping, Optional, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "libtgoracle.so"
SPARE = 0xFFFFFFFF


def build() -> Path:
    """Builds build/libtgoracle.so with gcc (oracle/Makefile)."""
    res = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"building the oracle failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


class _Shape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("hidden", "inner", "heads", "kv_heads", "head_dim", "layers", "capacity", "slots")] + [
        ("eps", ctypes.c_float), ("residual_scale", ctypes.c_float), ("rope", ctypes.c_int32),
        ("cos", ctypes.POINTER(ctypes.c_float)), ("sin", ctypes.POINTER(ctypes.c_float))]


_FP = ctypes.POINTER(ctypes.c_float)


class _Layer(ctypes.Structure):
    _fields_ = [(n, _FP) for n in ("input_norm", "qkv", "o", "post_norm", "gate_up", "down",
                                   "k_cache", "v_cache")]


_lib = None


def library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(LIB_PATH))
        U32P = ctypes.POINTER(ctypes.c_uint32)
        lib.tgo_rope_tables.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                        ctypes.POINTER(ctypes.c_double), _FP, _FP]
        lib.tgo_rope_tables.restype = None
        lib.tgo_rmsnorm.argtypes = [_FP, _FP, ctypes.c_int32, ctypes.c_float, _FP]
        lib.tgo_rmsnorm.restype = None
        lib.tgo_decode_step.argtypes = [ctypes.POINTER(_Shape), ctypes.POINTER(_Layer), _FP,
                                        ctypes.c_int32, U32P, U32P, _FP, _FP, ctypes.c_int32]
        lib.tgo_decode_step.restype = ctypes.c_int32
        lib.tgo_prefill.argtypes = [ctypes.POINTER(_Shape), ctypes.POINTER(_Layer), _FP,
                                    ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, _FP, _FP,
                                    ctypes.c_int32]
        lib.tgo_prefill.restype = ctypes.c_int32
        lib.tgo_gemm_abt.argtypes = [_FP, _FP, _FP, ctypes.c_int32, ctypes.c_int32,
                                     ctypes.c_int32, ctypes.c_int32]
        lib.tgo_gemm_abt.restype = None
        lib.tgo_gemv_linear.argtypes = [_FP, _FP, _FP, _FP, _FP] + [ctypes.c_int32] * 7 + [ctypes.c_float]
        lib.tgo_gemv_linear.restype = None
        _lib = lib
    return _lib


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_FP)


def rope_tables(head_dim: int, capacity: int, theta: float,
                factors: Optional[Sequence[float]] = None) -> tuple[np.ndarray, np.ndarray]:
    cos = np.zeros((capacity, head_dim // 2), np.float32)
    sin = np.zeros_like(cos)
    f = None if factors is None else (ctypes.c_double * len(factors))(*factors)
    library().tgo_rope_tables(head_dim, capacity, theta, f, _fp(cos), _fp(sin))
    return cos, sin


def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty_like(x)
    library().tgo_rmsnorm(_fp(x), _fp(g), x.size, eps, _fp(out))
    return out


def gemm_abt(a: np.ndarray, b: np.ndarray, threads: int = 0) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    c = np.empty((a.shape[0], b.shape[0]), np.float32)
    library().tgo_gemm_abt(_fp(a), _fp(b), _fp(c), a.shape[0], b.shape[0], a.shape[1],
                           threads or os.cpu_count() or 1)
    return c


def gemv_linear(x0: np.ndarray, x1: Optional[np.ndarray], w: np.ndarray, bias: np.ndarray, act: int = 0,
                levels: float = 9.0, offset: int = 0, stride: Optional[int] = None) -> np.ndarray:
    """tgo_gemv_linear: out [rows][stride] with act(W [x0; x1] + bias) at columns offset.."""
    x0 = np.ascontiguousarray(x0, np.float32)
    rows, k0 = x0.shape
    x1 = np.zeros((rows, 0), np.float32) if x1 is None else np.ascontiguousarray(x1, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    n = w.shape[0]
    stride = offset + n if stride is None else stride
    out = np.zeros((rows, stride), np.float32)
    library().tgo_gemv_linear(_fp(x0), _fp(x1) if x1.size else None, _fp(w),
                              _fp(np.ascontiguousarray(bias, np.float32)), _fp(out), rows, n, k0, x1.shape[1],
                              offset, stride, act, ctypes.c_float(levels))
    return out


class OracleStack:
    """One stack's f32 weights (bf16-valued for bf16 configs) and KV caches of `slots` slots, run
    on the CPU by the C restatement."""

    def __init__(self, shape, weights: Mapping[str, np.ndarray], slots: int = 1,
                 threads: Optional[int] = None):
        self.shape = shape
        self.slots = slots
        self.threads = threads or os.cpu_count() or 1
        s = shape
        self.cos, self.sin = rope_tables(s.head_dim, s.capacity, s.rope_theta, s.rope_factors)
        self._c = _Shape(s.hidden, s.inner, s.heads, s.kv_heads, s.head_dim, s.layers, s.capacity,
                         slots, s.eps, s.residual_scale, int(s.rope), _fp(self.cos), _fp(self.sin))
        f32 = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        self.arrays = []
        layers = (_Layer * s.layers)()
        cache = (slots, s.kv_heads, s.capacity, s.head_dim)
        self.k_cache = [np.zeros(cache, np.float32) for _ in range(s.layers)]
        self.v_cache = [np.zeros(cache, np.float32) for _ in range(s.layers)]
        for l in range(s.layers):
            w = lambda n: f32(weights[f"layers.{l}.{n}.weight"])  # noqa: E731
            qkv = np.concatenate([w("self_attn.q_proj"), w("self_attn.k_proj"), w("self_attn.v_proj")])
            gate_up = np.concatenate([w("mlp.gate_proj"), w("mlp.up_proj")])
            parts = [w("input_layernorm"), qkv, w("self_attn.o_proj"), w("post_attention_layernorm"),
                     gate_up, w("mlp.down_proj")]
            self.arrays.extend(parts)
            layers[l] = _Layer(*[_fp(p) for p in parts], _fp(self.k_cache[l]), _fp(self.v_cache[l]))
        self.final = f32(weights["norm.weight"])
        self._layers = layers

    def decode_step(self, rows: Sequence[Optional[tuple[int, int]]], x: np.ndarray) -> np.ndarray:
        """One step over rows (position, slot) or None (spare), x [rows][hidden]."""
        n = len(rows)
        pos = np.array([SPARE if r is None else r[0] for r in rows], np.uint32)
        slot = np.array([0 if r is None else r[1] for r in rows], np.uint32)
        x = np.ascontiguousarray(x, np.float32).reshape(n, self.shape.hidden)
        out = np.empty_like(x)
        U32P = ctypes.POINTER(ctypes.c_uint32)
        st = library().tgo_decode_step(ctypes.byref(self._c), self._layers, _fp(self.final), n,
                                       pos.ctypes.data_as(U32P), slot.ctypes.data_as(U32P), _fp(x),
                                       _fp(out), self.threads)
        if st:
            raise ValueError("oracle: shape refused")
        return out

    def prefill(self, start: int, x: np.ndarray, slot: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32).reshape(-1, self.shape.hidden)
        out = np.empty_like(x)
        st = library().tgo_prefill(ctypes.byref(self._c), self._layers, _fp(self.final), start,
                                   x.shape[0], slot, _fp(x), _fp(out), self.threads)
        if st:
            raise ValueError("oracle: shape refused")
        return out


# ---- VoxCPM2's local stacks (local_ref.c) ---------------------------------------------------------

class _LocalShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("hidden", "inner", "heads", "kv_heads", "head_dim", "layers", "tokens")] + [
        ("eps", ctypes.c_float), ("cos", _FP), ("sin", _FP)]


class _LocalLayer(ctypes.Structure):
    _fields_ = [(n, _FP) for n in ("input_norm", "qkv", "o", "post_norm", "gate", "up", "down")]


def _local_library() -> ctypes.CDLL:
    lib = library()
    if not getattr(lib, "_local_typed", False):
        I32 = ctypes.c_int32
        SP, LP, DP = ctypes.POINTER(_LocalShape), ctypes.POINTER(_LocalLayer), ctypes.POINTER(ctypes.c_double)
        lib.tgo_local_set_threads.argtypes = [I32]
        lib.tgo_round_f16.argtypes = [_FP, ctypes.c_int64]
        lib.tgo_local_stack.argtypes = [SP, LP, _FP, I32, _FP, _FP]
        lib.tgo_schedule.argtypes = [I32, _FP]
        lib.tgo_euler_steps.argtypes = [I32, _FP, _FP]
        lib.tgo_euler_steps.restype = I32
        lib.tgo_time_tokens.argtypes = [I32] + [_FP] * 8 + [I32, _FP, DP]
        lib.tgo_sampler.argtypes = [SP, LP, _FP] + [_FP] * 8 + [I32, I32, I32, I32, _FP, _FP, _FP, _FP, _FP]
        lib.tgo_encoder.argtypes = [SP, LP, _FP, _FP, _FP, _FP, I32, I32, I32, _FP, _FP]
        for f in ("tgo_local_set_threads", "tgo_round_f16", "tgo_local_stack", "tgo_schedule",
                  "tgo_time_tokens", "tgo_sampler", "tgo_encoder"):
            getattr(lib, f).restype = None
        lib._local_typed = True
    return lib


def round_f16(x: np.ndarray) -> np.ndarray:
    """The f32 values of x rounded to f16 (RNE), by the oracle's own conversion."""
    a = np.array(x, np.float32, copy=True, order="C")
    _local_library().tgo_round_f16(_fp(a), a.size)
    return a


def cfm_schedule(timesteps: int) -> np.ndarray:
    out = np.zeros(timesteps + 1, np.float32)
    _local_library().tgo_schedule(timesteps, _fp(out))
    return out


def cfm_euler_steps(timesteps: int) -> list[tuple[float, float]]:
    t = np.zeros(timesteps + 1, np.float32)
    dt = np.zeros_like(t)
    n = _local_library().tgo_euler_steps(timesteps, _fp(t), _fp(dt))
    return [(float(a), float(b)) for a, b in zip(t[:n], dt[:n])]


class OracleLocal:
    """A local stack (the sampler's DiT or the local encoder) on the CPU: f32 copies of its weights
    rounded to f16, as the GPU holds them, run by local_ref.c. `prefix` is the stack's name prefix
    ("feat_decoder.estimator." or "feat_encoder.")."""

    def __init__(self, shape, weights: Mapping[str, np.ndarray], prefix: str, tokens: int,
                 threads: Optional[int] = None):
        lib = _local_library()
        lib.tgo_local_set_threads(threads or os.cpu_count() or 1)
        s = shape
        self.shape, self.prefix, self.tokens = s, prefix, tokens
        self.cos, self.sin = rope_tables(s.head_dim, tokens, s.rope_theta, s.rope_factors)
        self._c = _LocalShape(s.hidden, s.inner, s.heads, s.kv_heads, s.head_dim, s.layers, tokens,
                              s.eps, _fp(self.cos), _fp(self.sin))
        self.w = {k: round_f16(np.asarray(v, np.float32)) for k, v in weights.items()
                  if k.startswith(prefix)}
        stack = prefix + ("decoder." if prefix.startswith("feat_decoder") else "encoder.")
        self.layers = (_LocalLayer * s.layers)()
        self._keep = []
        for l in range(s.layers):
            g = lambda n: self.w[f"{stack}layers.{l}.{n}.weight"]  # noqa: E731
            qkv = np.ascontiguousarray(np.concatenate(
                [g("self_attn.q_proj"), g("self_attn.k_proj"), g("self_attn.v_proj")]))
            arrs = [g("input_layernorm"), qkv, g("self_attn.o_proj"), g("post_attention_layernorm"),
                    g("mlp.gate_proj"), g("mlp.up_proj"), g("mlp.down_proj")]
            arrs = [np.ascontiguousarray(a, np.float32) for a in arrs]
            self._keep += arrs
            self.layers[l] = _LocalLayer(*[_fp(a) for a in arrs])
        self.final = np.ascontiguousarray(self.w[f"{stack}norm.weight"])

    def stack(self, x: np.ndarray, seqs: int) -> np.ndarray:
        """tgo_local_stack: x [seqs tokens][hidden] (f16 values) -> the tokens after the final norm."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        _local_library().tgo_local_stack(ctypes.byref(self._c), self.layers, _fp(self.final), seqs,
                                         _fp(x), _fp(out))
        return out

    def time_tokens(self, times: Sequence[float]) -> np.ndarray:
        """dit.rs:372-422 in f64, then rounded to f16 (as f32 values)."""
        p, H = self.prefix, self.shape.hidden
        ws = [np.ascontiguousarray(self.w[f"{p}{m}.linear_{i}.{kind}"], np.float32)
              for m in ("time_mlp", "delta_time_mlp") for i in (1, 2) for kind in ("weight", "bias")]
        t = np.ascontiguousarray(times, np.float32)
        out = np.zeros((len(t), H), np.float64)
        _local_library().tgo_time_tokens(H, *[_fp(a) for a in ws], len(t), _fp(t),
                                         out.ctypes.data_as(ctypes.POINTER(ctypes.c_double)))
        return out.astype(np.float16).astype(np.float32)

    def sample(self, mu: np.ndarray, cond: np.ndarray, noise: np.ndarray, sampling: np.ndarray,
               timesteps: int, feat: int, patch: int) -> np.ndarray:
        """tgo_sampler: each row's patch, [rows][feat][patch]."""
        p = self.prefix
        steps = cfm_euler_steps(timesteps)
        times = self.time_tokens([t for t, _ in steps]) if steps else np.zeros((1, self.shape.hidden), np.float32)
        dts = np.ascontiguousarray([dt for _, dt in steps] or [0.0], np.float32)
        rows = mu.shape[0]
        f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        mu, cond, noise, sampling = f(round_f16(mu)), f(cond), f(noise), f(sampling)
        out = np.zeros((rows, feat, patch), np.float32)
        lin = [f(self.w[f"{p}{n}.{k}"]) for n in ("in_proj", "cond_proj", "out_proj") for k in ("weight", "bias")]
        _local_library().tgo_sampler(ctypes.byref(self._c), self.layers, _fp(self.final), *[_fp(a) for a in lin],
                                     _fp(f(times)), _fp(dts), len(steps), rows, feat, patch, _fp(mu),
                                     _fp(cond), _fp(noise), _fp(sampling), _fp(out))
        return out

    def encode(self, patches: np.ndarray, feat: int, patch: int) -> np.ndarray:
        """tgo_encoder: each row's embedding, [rows][hidden] (f16 values)."""
        p = self.prefix
        f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        patches = f(patches)
        rows = patches.shape[0]
        out = np.zeros((rows, self.shape.hidden), np.float32)
        _local_library().tgo_encoder(ctypes.byref(self._c), self.layers, _fp(self.final), _fp(f(self.w[p + "in_proj.weight"])),
                                     _fp(f(self.w[p + "in_proj.bias"])), _fp(f(self.w[p + "special_token"])), rows,
                                     feat, patch, _fp(patches), _fp(out))
        return out

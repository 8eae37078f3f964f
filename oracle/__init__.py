"""TEST INFRASTRUCTURE ONLY: the CPU oracle the parity tests, `__graft_entry__.smoke()` and the
CPU-baseline legs of `bench.py` check the CUDA path against. The product (libtgcuda.so and the
tgtts-v4_b200 package) never imports, links or calls anything here.

`OracleStack` holds one stack's f32 weights and KV caches and runs the C restatement
(minicpm4_ref.c) of tgtts-v4's decode step (crates/graph/src/decode.rs:618-735) and prefill
(crates/graph/src/prefill.rs:318-411). `ref_numpy` is an independent numpy restatement used to
cross-check it.
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

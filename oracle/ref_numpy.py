"""TEST INFRASTRUCTURE ONLY: an independent numpy restatement of the MiniCPM-4 stack, in f64, used
to cross-check the C oracle (minicpm4_ref.c) on small shapes. It follows the same reference
lines: crates/graph/src/decode.rs:618-735 (the step), kernels/glsl/norm.glsl:10-53 (RMSNorm),
gemv_qkv_rope.comp:82-104 (RoPE on row pairs), attention_split.comp + attention_combine.comp
(softmax over positions 0..pos, GQA head -> kv head = head / group), gemv_gate_up.comp:44-50
(SiLU), prefill.rs:318-411 (a run of positions, causal over the slot).
"""

from __future__ import annotations

import numpy as np


def rope_tables(head_dim: int, capacity: int, theta: float, factors=None):
    """decode.rs:146-168 in f32: inv = 1 / theta^(2i/d), rate = 1 / factor, f = t * rate * inv."""
    half = head_dim // 2
    i = np.arange(half)
    inv = (np.float32(1.0) / np.power(np.float32(theta), (2 * i).astype(np.float32) / np.float32(head_dim),
                                      dtype=np.float32)).astype(np.float32)
    fac = np.ones(half, np.float64) if factors is None else np.asarray(factors, np.float64)
    rate = (np.float32(1.0) / fac.astype(np.float32)).astype(np.float32)
    t = np.arange(capacity, dtype=np.float32)[:, None]
    f = (t * rate[None, :]).astype(np.float32) * inv[None, :]
    # cos and sin of the f32 angle taken in f64 and rounded once, as a correctly rounded f32
    # cosf/sinf gives them (numpy's own f32 sin is not correctly rounded).
    f = f.astype(np.float32).astype(np.float64)
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def rmsnorm(x, g, eps):
    x = np.asarray(x, np.float64)
    scale = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * scale * np.asarray(g, np.float64)


class NumpyStack:
    def __init__(self, shape, weights, slots=1):
        self.s = shape
        self.w = {k: np.asarray(v, np.float64) for k, v in weights.items()}
        cos, sin = rope_tables(shape.head_dim, shape.capacity, shape.rope_theta, shape.rope_factors)
        self.cos, self.sin = cos.astype(np.float64), sin.astype(np.float64)
        c = (slots, shape.kv_heads, shape.capacity, shape.head_dim)
        self.k = [np.zeros(c) for _ in range(shape.layers)]
        self.v = [np.zeros(c) for _ in range(shape.layers)]

    def _layer(self, l, x, places):
        s, W = self.s, lambda n: self.w[f"layers.{l}.{n}.weight"]
        hd, half, H = s.head_dim, s.head_dim // 2, s.heads
        xn = rmsnorm(x, W("input_layernorm"), s.eps)
        q = xn @ W("self_attn.q_proj").T
        k = xn @ W("self_attn.k_proj").T
        v = xn @ W("self_attn.v_proj").T
        n = x.shape[0]
        q = q.reshape(n, H, hd)
        k = k.reshape(n, s.kv_heads, hd)
        v = v.reshape(n, s.kv_heads, hd)
        for b, (pos, slot) in enumerate(places):
            if pos is None:
                continue
            if s.rope:
                co, si = self.cos[pos], self.sin[pos]
                for t in (q, k):
                    a, c = t[b, :, :half].copy(), t[b, :, half:].copy()
                    t[b, :, :half] = a * co - c * si
                    t[b, :, half:] = c * co + a * si
            self.k[l][slot, :, pos] = k[b]
            self.v[l][slot, :, pos] = v[b]
        att = np.zeros((n, H, hd))
        group = H // s.kv_heads
        for b, (pos, slot) in enumerate(places):
            if pos is None:
                continue
            for h in range(H):
                kv = h // group
                sc = self.k[l][slot, kv, : pos + 1] @ q[b, h] / np.sqrt(hd)
                p = np.exp(sc - sc.max())
                att[b, h] = (p / p.sum()) @ self.v[l][slot, kv, : pos + 1]
        mid = x + s.residual_scale * (att.reshape(n, -1) @ W("self_attn.o_proj").T)
        mn = rmsnorm(mid, W("post_attention_layernorm"), s.eps)
        g = mn @ W("mlp.gate_proj").T
        u = mn @ W("mlp.up_proj").T
        return mid + s.residual_scale * ((g / (1 + np.exp(-g)) * u) @ W("mlp.down_proj").T)

    def run(self, places, x):
        """places: (position, slot) or (None, None) per row; all rows' k and v of a layer are
        written before any row attends."""
        h = np.asarray(x, np.float64)
        for l in range(self.s.layers):
            h = self._layer(l, h, places)
        out = rmsnorm(h, self.w["norm.weight"], self.s.eps)
        for b, (pos, _) in enumerate(places):
            if pos is None:
                out[b] = 0
        return out

    def decode_step(self, rows, x):
        return self.run([(None, None) if r is None else r for r in rows], x)

    def prefill(self, start, x, slot=0):
        x = np.asarray(x).reshape(-1, self.s.hidden)
        return self.run([(start + i, slot) for i in range(x.shape[0])], x)


# ---- VoxCPM2's local stacks (crates/graph/src/local), cross-checking local_ref.c -----------------

def f16(x):
    return np.asarray(x, np.float64).astype(np.float16).astype(np.float64)


def local_stack(shape, w, stack_prefix, tokens, x):
    """local/mod.rs:573-680 in f64 with the f16 roundings of the kernels (local_*.comp): x
    [seqs tokens][hidden] -> the tokens after the final norm. `w` holds f16-valued weights."""
    s = shape
    hd, half, H = s.head_dim, s.head_dim // 2, s.hidden
    cos, sin = rope_tables(hd, tokens, s.rope_theta, s.rope_factors)
    cos, sin = cos.astype(np.float64), sin.astype(np.float64)
    g = lambda n: np.asarray(w[stack_prefix + n], np.float64)  # noqa: E731
    M = x.shape[0]
    pos = np.arange(M) % tokens

    def norm(v, gain):
        return f16(rmsnorm(v, gain, s.eps))

    cur = np.asarray(x, np.float64)
    normed = norm(cur, g("layers.0.input_layernorm.weight"))
    group = s.heads // s.kv_heads
    for l in range(s.layers):
        L = lambda n: g(f"layers.{l}.{n}.weight")  # noqa: E731
        def rot(v):  # [M][heads][hd]
            a, b = v[..., :half], v[..., half:]
            c, sn = cos[pos][:, None, :], sin[pos][:, None, :]
            return np.concatenate([a * c - b * sn, b * c + a * sn], axis=-1)
        q = f16(rot((normed @ L("self_attn.q_proj").T).reshape(M, s.heads, hd)))
        k = f16(rot((normed @ L("self_attn.k_proj").T).reshape(M, s.kv_heads, hd)))
        v = f16((normed @ L("self_attn.v_proj").T).reshape(M, s.kv_heads, hd))
        att = np.zeros((M, s.heads, hd))
        for m0 in range(0, M, tokens):
            sl = slice(m0, m0 + tokens)
            for h in range(s.heads):
                kv = h // group
                sc = q[sl, h] @ k[sl, kv].T / np.sqrt(hd)
                e = np.exp(sc - sc.max(axis=1, keepdims=True))
                att[sl, h] = (e @ v[sl, kv]) / e.sum(axis=1, keepdims=True)
        att = f16(att.reshape(M, -1))
        mid = f16(cur + att @ L("self_attn.o_proj").T)
        normed = norm(mid, L("post_attention_layernorm"))
        gate, up = normed @ L("mlp.gate_proj").T, normed @ L("mlp.up_proj").T
        mlp = f16(gate / (1.0 + np.exp(-gate)) * up)
        cur = f16(mid + mlp @ L("mlp.down_proj").T)
        gain = g(f"layers.{l + 1}.input_layernorm.weight") if l + 1 < s.layers else g("norm.weight")
        normed = norm(cur, gain)
    return normed

"""VoxCPM2's LM side of a patch on the GPU (crates/graph/src/lm_side.rs:337-495): from the local
encoder's output for the last patch to what the next patch is sampled with, for a batch of rows,
each a request at its own position and slot of both LMs' caches.

    embed       = enc_to_lm_proj(enc)
    base_out    = the base LM's decode step over embed (RoPE)
    levels      = fsq_layer.in_proj(base_out), the scalar quantizer's rounding
    lm_hidden   = fsq_layer.out_proj(levels)
    residual_in = fusion_concat_proj([lm_hidden; embed])
    mu[:dit]    = lm_to_dit_proj(lm_hidden)
    stop_logits = stop_head(SiLU(stop_proj(lm_hidden)))        (stop_head has no bias upstream)
    res_out     = the residual LM's decode step over residual_in (no RoPE)
    mu[dit:]    = res_to_dit_proj(res_out)

The two stacks are Decoders over the same rows and slots; the linear layers are gemv_linear
dispatches (TG_KERNEL_GEMV_LINEAR) recorded once into three programs. The whole step is enqueued on
the context's stream without a wait until its outputs are read. Intermediates are f32 (the
reference's are f16)."""

from __future__ import annotations

import dataclasses
from typing import Mapping, Optional, Sequence

import numpy as np

HEADS = ("enc_to_lm_proj", "fsq_layer.in_proj", "fsq_layer.out_proj", "fusion_concat_proj",
         "lm_to_dit_proj", "res_to_dit_proj", "stop_proj", "stop_head")


@dataclasses.dataclass
class LmSideShape:
    """LmSideShape (lm_side.rs:59-91): the two stacks' shapes and the widths between them."""

    base: object       # the package's Shape, with RoPE
    residual: object   # the package's Shape, without RoPE (residual_lm_no_rope)
    encoder: int       # the local encoder's width, the step's input
    dit: int           # the local DiT's width, half the condition's
    latent: int        # the scalar quantizer's bottleneck
    levels: int        # scalar_quantization_scale

    def head_shapes(self) -> dict[str, tuple[int, int]]:
        h = self.base.hidden
        return {"enc_to_lm_proj": (h, self.encoder), "fsq_layer.in_proj": (self.latent, h),
                "fsq_layer.out_proj": (h, self.latent), "fusion_concat_proj": (h, 2 * h),
                "lm_to_dit_proj": (self.dit, h), "res_to_dit_proj": (self.dit, h),
                "stop_proj": (h, h), "stop_head": (2, h)}


class LmSide:
    def __init__(self, pkg, ctx, shape: LmSideShape, rows: int = 1, slots: Optional[int] = None,
                 dtype: str = "f32"):
        b, r = shape.base, shape.residual
        if (r.hidden, r.capacity, r.head_dim) != (b.hidden, b.capacity, b.head_dim):
            raise pkg.ShapeError("a residual LM that does not meet the base LM (lm_side.rs:342-348)")
        self.pkg, self.ctx, self.shape, self.rows, self.dtype = pkg, ctx, shape, rows, dtype
        slots = rows if slots is None else slots
        self.base = pkg.Decoder(ctx, b, rows=rows, slots=slots, dtype=dtype)
        self.residual = pkg.Decoder(ctx, r, rows=rows, slots=slots, dtype=dtype)
        H, es = b.hidden, 2 if dtype == "bf16" else 4
        f = lambda n: pkg.Memory(ctx, max(16, rows * n * 4))  # noqa: E731
        self.enc, self.embed, self.base_out = f(shape.encoder), f(H), f(H)
        self.levels_m, self.lm_hidden, self.residual_in = f(shape.latent), f(H), f(H)
        self.res_out, self.stop_hidden = f(H), f(H)
        self.mu, self.stop = f(2 * shape.dit), f(2)
        self.w, self.bias = {}, {}
        for name, (n, k) in shape.head_shapes().items():
            self.w[name] = pkg.Memory(ctx, n * k * es)
            self.bias[name] = pkg.Memory(ctx, max(16, n * 4))
            self.bias[name].fill(0)
        self.programs = self._record()

    def _linear(self, name, x0, x1, k0, k1, out, stride, offset=0, act=0):
        n, k = self.shape.head_shapes()[name]
        assert k == k0 + k1
        p = self.pkg.params(self.shape.base, self.dtype, rows=self.rows, n=n, k=k0, k1=k1, offset=offset,
                            stride=stride, act=act, levels=float(self.shape.levels))
        es = 2 if self.dtype == "bf16" else 4
        R = self.rows
        return ("gemv_linear", p, [(x0, 0, R * k0 * 4), (x1, 0, max(16, R * k1 * 4)), (self.w[name], 0, n * k * es),
                                   (self.bias[name], 0, n * 4), (out, 0, R * stride * 4)], name)

    def _record(self):
        s, H = self.shape, self.shape.base.hidden
        L = self._linear
        first = [L("enc_to_lm_proj", self.enc, self.enc, s.encoder, 0, self.embed, H)]
        between = [
            L("fsq_layer.in_proj", self.base_out, self.base_out, H, 0, self.levels_m, s.latent, act=2),
            L("fsq_layer.out_proj", self.levels_m, self.levels_m, s.latent, 0, self.lm_hidden, H),
            L("fusion_concat_proj", self.lm_hidden, self.embed, H, H, self.residual_in, H),
            L("lm_to_dit_proj", self.lm_hidden, self.lm_hidden, H, 0, self.mu, 2 * s.dit),
            L("stop_proj", self.lm_hidden, self.lm_hidden, H, 0, self.stop_hidden, H, act=1),
            L("stop_head", self.stop_hidden, self.stop_hidden, H, 0, self.stop, 2),
        ]
        last = [L("res_to_dit_proj", self.res_out, self.res_out, H, 0, self.mu, 2 * s.dit, offset=s.dit)]
        return [self.pkg.Program(self.ctx, d) for d in (first, between, last)]

    def load(self, weights: Mapping[str, np.ndarray]) -> None:
        """load_lm_side (lm_side.rs:501-541): both stacks under "base_lm." and "residual_lm.", and
        each head's weight and bias (stop_head's bias zero when the checkpoint has none)."""
        self.base.load(weights, prefix="base_lm.")
        self.residual.load(weights, prefix="residual_lm.")
        for name, (n, k) in self.shape.head_shapes().items():
            w = np.ascontiguousarray(weights[f"{name}.weight"])
            if w.shape != (n, k):
                raise self.pkg.ShapeError(f"{name}.weight: shape {w.shape}, not {(n, k)}")
            if self.dtype == "bf16" and w.dtype != np.uint16:
                from . import synthetic

                w = synthetic.bf16_bits(w)
            elif self.dtype == "f32":
                w = np.ascontiguousarray(w, np.float32)
            self.w[name].write(w)
            b = weights.get(f"{name}.bias")
            self.bias[name].write(np.zeros(n, np.float32) if b is None else np.ascontiguousarray(b, np.float32))

    def step(self, rows: Sequence[Optional[tuple[int, int]]], enc: np.ndarray):
        """One patch's LM side for the batch: rows (position, slot) or None (spare), enc
        [rows][encoder] f32 -> (mu [rows][2 dit], stop_logits [rows][2], levels [rows][latent])."""
        R = self.rows
        if len(rows) != R:
            raise self.pkg.ShapeError(f"{len(rows)} rows for a batch of {R}")
        words = self.pkg.Batch(R, self.base.batch.slots).placement(
            [None if r is None else self.pkg.Row(*r) for r in rows], self.shape.base.capacity)
        self.enc.write(np.ascontiguousarray(enc, np.float32))
        self.programs[0].start()
        self.base.step_device(words, self.embed.device_ptr, self.base_out.device_ptr)
        self.programs[1].start()
        self.residual.step_device(words, self.residual_in.device_ptr, self.res_out.device_ptr)
        self.programs[2].start()
        self.programs[2].wait()
        s = self.shape
        return (self.mu.read(np.float32, R * 2 * s.dit).reshape(R, 2 * s.dit),
                self.stop.read(np.float32, R * 2).reshape(R, 2),
                self.levels_m.read(np.float32, R * s.latent).reshape(R, s.latent))

    def close(self):
        for p in self.programs:
            p.close()
        self.base.close()
        self.residual.close()


def oracle_step(oracle, shape: LmSideShape, stacks, weights, rows, enc):
    """The same patch on the CPU: the oracle's two stacks and its gemv_linear (test
    infrastructure)."""
    base, residual = stacks
    f = lambda n: np.ascontiguousarray(weights[n], np.float32)  # noqa: E731
    b = lambda n: np.ascontiguousarray(weights.get(f"{n}.bias", np.zeros(f(f"{n}.weight").shape[0], np.float32)), np.float32)  # noqa: E731
    lin = lambda n, x0, x1=None, act=0: oracle.gemv_linear(x0, x1, f(f"{n}.weight"), b(n), act=act, levels=float(shape.levels))  # noqa: E731
    embed = lin("enc_to_lm_proj", enc)
    base_out = base.decode_step(rows, embed)
    levels = lin("fsq_layer.in_proj", base_out, act=2)
    lm_hidden = lin("fsq_layer.out_proj", levels)
    residual_in = lin("fusion_concat_proj", lm_hidden, embed)
    stop = lin("stop_head", lin("stop_proj", lm_hidden, act=1))
    res_out = residual.decode_step(rows, residual_in)
    mu = np.concatenate([lin("lm_to_dit_proj", lm_hidden), lin("res_to_dit_proj", res_out)], 1)
    return mu, stop, levels


class LogitsHead:
    """An output projection over a stack's final hidden states: logits [rows][vocab] = W h + bias,
    one gemv_linear dispatch (TG_KERNEL_GEMV_LINEAR) recorded once. The decode stack itself ends at
    the final norm (crates/graph/src/decode.rs:716-723) and VoxCPM2's only logits are the LM side's
    stop head; this is the optional vocabulary head a plain LM adds, on the same kernel."""

    def __init__(self, pkg, ctx, hidden: int, vocab: int, rows: int = 1, dtype: str = "bf16"):
        self.pkg, self.ctx, self.hidden, self.vocab, self.rows, self.dtype = pkg, ctx, hidden, vocab, rows, dtype
        es = 2 if dtype == "bf16" else 4
        self.x = pkg.Memory(ctx, rows * hidden * 4)
        self.out = pkg.Memory(ctx, rows * vocab * 4)
        self.w = pkg.Memory(ctx, vocab * hidden * es)
        self.b = pkg.Memory(ctx, max(16, vocab * 4))
        self.b.fill(0)
        shape = pkg.Shape(hidden=hidden, inner=hidden, heads=1, kv_heads=1, head_dim=64, layers=1, capacity=64)
        self.params = pkg.params(shape, dtype, rows=rows, n=vocab, k=hidden, k1=0, offset=0, stride=vocab, act=0)
        self.dispatch = ("gemv_linear", self.params,
                         [(self.x, 0, rows * hidden * 4), (self.x, 0, 16), (self.w, 0, vocab * hidden * es),
                          (self.b, 0, vocab * 4), (self.out, 0, rows * vocab * 4)], "logits")
        self.program = pkg.Program(ctx, [self.dispatch])

    def load(self, weight: np.ndarray, bias: Optional[np.ndarray] = None) -> None:
        w = np.ascontiguousarray(weight)
        if w.shape != (self.vocab, self.hidden):
            raise self.pkg.ShapeError(f"logits weight: shape {w.shape}, not {(self.vocab, self.hidden)}")
        if self.dtype == "bf16" and w.dtype != np.uint16:
            from . import synthetic

            w = synthetic.bf16_bits(w)
        elif self.dtype == "f32":
            w = np.ascontiguousarray(w, np.float32)
        self.w.write(w)
        self.b.write(np.zeros(self.vocab, np.float32) if bias is None else np.ascontiguousarray(bias, np.float32))

    def __call__(self, h: np.ndarray) -> np.ndarray:
        """h [rows][hidden] f32 -> logits [rows][vocab] f32."""
        self.x.write(np.ascontiguousarray(h, np.float32).reshape(self.rows, self.hidden))
        self.program.run()
        return self.out.read(np.float32, self.rows * self.vocab).reshape(self.rows, self.vocab)

"""The decode-attention entry point that allocates nothing (tg_attention_decode_noalloc), for
callers that own all device memory themselves or record CUDA graphs and so cannot let a library
allocate: its output must match the attention_split + attention_combine dispatches that take a
scratch buffer from the caller, on two calls in a row (the second over the first's leftovers in
the shared fixed array). Collected last, so that a run stopping at the first failure has run every
other test before it."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(pkg, ctx, rows=4, cap=256, dtype="bf16", seed=0):
    shape = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=cap)
    rng = np.random.default_rng(seed)
    hd, heads, kv = shape.head_dim, shape.heads, shape.kv_heads
    q = rng.standard_normal((rows, heads, hd), dtype=np.float32)
    cache = (rows, kv, cap, hd)
    k = rng.standard_normal(cache, dtype=np.float32)
    v = rng.standard_normal(cache, dtype=np.float32)
    if dtype == "bf16":
        from tgtts_v4_b200 import synthetic as syn

        k, v = syn.bf16_bits(k), syn.bf16_bits(v)
    mem = {}
    for name, a in (("q", q), ("k", k), ("v", v)):
        mem[name] = pkg.Memory(ctx, a.nbytes)
        mem[name].write(a)
    return shape, mem


def _reference(pkg, ctx, shape, mem, p, words, rows):
    """The existing path: the two kernel-table dispatches with caller-owned scratch."""
    chunks = shape.capacity // 64
    po = pkg.Memory(ctx, rows * shape.heads * chunks * shape.head_dim * 4)
    pml = pkg.Memory(ctx, rows * shape.heads * chunks * 2 * 4)
    at = pkg.Memory(ctx, words.nbytes)
    at.write(words)
    out = pkg.Memory(ctx, rows * shape.heads * shape.head_dim * 4)
    out.write(np.zeros(rows * shape.heads * shape.head_dim, np.float32))
    qb, cb = mem["q"].nbytes, mem["k"].nbytes
    pkg.dispatch_once(ctx, "attention_split", p, [(mem["q"], 0, qb), (mem["k"], 0, cb), (mem["v"], 0, cb),
                                                  (at, 0, words.nbytes), (po, 0, po.nbytes), (pml, 0, pml.nbytes)])
    pkg.dispatch_once(ctx, "attention_combine", p, [(at, 0, words.nbytes), (po, 0, po.nbytes),
                                                    (pml, 0, pml.nbytes), (out, 0, out.nbytes)])
    return out.read(np.float32, rows * shape.heads * shape.head_dim)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_no_alloc_attention_matches_the_scratch_taking_path_twice(pkg, ctx, dtype):
    rows = 4
    shape, mem = _setup(pkg, ctx, rows=rows, dtype=dtype)
    p = pkg.params(shape, dtype, rows=rows, slots=rows)
    n = rows * shape.heads * shape.head_dim
    for call, positions in enumerate(([5, 100, 0xFFFFFFFF, 255], [200, 0, 63, 64])):
        words = np.array(positions + list(range(rows)), np.uint32)
        want = _reference(pkg, ctx, shape, mem, p, words, rows)
        at = pkg.Memory(ctx, words.nbytes)
        at.write(words)
        out = pkg.Memory(ctx, n * 4)
        out.write(np.zeros(n, np.float32))
        pkg.attention_decode_noalloc(p, mem["q"].device_ptr, mem["k"].device_ptr, mem["v"].device_ptr,
                                     at.device_ptr, out.device_ptr, ctx.stream)
        ctx.synchronize()
        got = out.read(np.float32, n)
        # The same kernels over the same inputs: equal within the decode tolerance (f32 2e-4),
        # and in fact bit for bit.
        assert np.max(np.abs(got - want)) <= 2e-4, call
        assert np.array_equal(got, want), call


def test_no_alloc_attention_refuses_what_its_array_cannot_hold(pkg, ctx):
    shape = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=2048)
    rows = 64
    p = pkg.params(shape, "bf16", rows=rows, slots=rows)
    # Buffers of the full size the shape reaches, so that nothing could run out of them.
    q = pkg.Memory(ctx, rows * 16 * 64 * 4)
    cache = rows * 2 * 2048 * 64 * 2
    k, v = pkg.Memory(ctx, cache), pkg.Memory(ctx, cache)
    at = pkg.Memory(ctx, 2 * rows * 4)
    at.fill(0xFFFFFFFF)
    out = pkg.Memory(ctx, rows * 16 * 64 * 4)
    # 64 rows x 16 heads x 32 chunks x 66 floats = 8.6 MB of partials, past the 4 MiB array.
    with pytest.raises(pkg.ShapeError, match="scratch"):
        pkg.attention_decode_noalloc(p, q.device_ptr, k.device_ptr, v.device_ptr, at.device_ptr,
                                     out.device_ptr, ctx.stream)
    # No heads at all is a shape it cannot run either, refused before anything is enqueued.
    p0 = pkg.params(shape, "bf16", rows=rows, slots=rows)
    p0.heads = 0
    with pytest.raises(pkg.ShapeError):
        pkg.attention_decode_noalloc(p0, q.device_ptr, k.device_ptr, v.device_ptr, at.device_ptr,
                                     out.device_ptr, ctx.stream)

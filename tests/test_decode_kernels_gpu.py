"""The decode step's projection kernels one at a time (gemv_residual, gemv_gate_up, gemv_qkv_rope),
dispatched through the C ABI, against f64 references with bounds derived from f32 arithmetic, as
the reference's device tests hold its kernels (crates/vulkan/tests/glsl.rs:170-186, :276-358 for
the GEMV with residual, :370-458 gate/up after the norm, :460-615 q/k/v with RoPE and the cache
write). Each test also shows that its bound catches a planted defect (the residual scale, the
norm's gain, the direction of the rotation), computed on the CPU.

Bounds, with u = 2^-24 and a sum of k products in f32 within k u of the sum of their magnitudes:
  RMSNorm: the mean of k squares within (k + 1) u, the reciprocal root within 4 u more (two
    ulp), two products: each normed value within (k / 2 + 7) u of its own magnitude;
  a projection of normed values: E = (1.5 k + 8) u sum |w| |xn|;
  SiLU(g) up (|d SiLU / dg| <= 1.1): 1.1 E_g |up| + |SiLU(g)| E_up + E_g E_up + 8 u |out|;
  a RoPE pair: E_a + E_c + 3 u (|a| + |c|); a bf16 store adds 2^-8 of the value."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

U = 2.0**-24
SPARE = 0xFFFFFFFF


def _mem(pkg, ctx, a):
    a = np.ascontiguousarray(a)
    m = pkg.Memory(ctx, max(a.nbytes, 16))
    m.write(a)
    return m


def _weights(syn, rng, shape, dtype, scale=0.05):
    w = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
    if dtype == "bf16":
        bits = syn.bf16_bits(w)
        return bits, syn.bf16_to_f32(bits).astype(np.float64)
    return w, w.astype(np.float64)


def _normed(x, g, eps):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * g.astype(np.float64)


def _projection_bound(w, xn, k):
    return (1.5 * k + 8) * U * (np.abs(xn) @ np.abs(w).T)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows", [1, 5])
def test_gemv_residual_against_f64(pkg, ctx, syn, dtype, rows):
    rng = np.random.default_rng(20 + rows)
    n, k, s = 1024, 4096, 0.35
    wt, w = _weights(syn, rng, (n, k), dtype)
    x = rng.standard_normal((rows, k), dtype=np.float32)
    res = rng.standard_normal((rows, n), dtype=np.float32)
    shape = pkg.Shape(hidden=n, inner=k, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=64,
                      residual_scale=s)
    p = pkg.params(shape, dtype, rows=rows, n=n, k=k)
    mo = pkg.Memory(ctx, rows * n * 4)
    pkg.dispatch_once(ctx, "gemv_residual", p, [(_mem(pkg, ctx, x), 0, x.nbytes), (_mem(pkg, ctx, wt), 0, wt.nbytes),
                                                (_mem(pkg, ctx, res), 0, res.nbytes), (mo, 0, rows * n * 4)])
    got = mo.read(np.float32, rows * n).reshape(rows, n)
    dot = x.astype(np.float64) @ w.T
    want = res.astype(np.float64) + np.float32(s).astype(np.float64) * dot
    bound = s * (k + 2) * U * (np.abs(x.astype(np.float64)) @ np.abs(w).T) + 2 * U * np.abs(want) + 1e-30
    assert np.all(np.abs(got - want) <= bound), float(np.max(np.abs(got - want) / bound))
    # Planted: the residual branch without its scale.
    unscaled = res.astype(np.float64) + dot
    assert np.mean(np.abs(unscaled - want) > bound) > 0.9


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("rows", [1, 3])
def test_gemv_gate_up_against_f64(pkg, ctx, syn, dtype, rows):
    rng = np.random.default_rng(30 + rows)
    h, inner, eps = 1024, 512, 1e-5
    gate_t, gate = _weights(syn, rng, (inner, h), dtype)
    up_t, up = _weights(syn, rng, (inner, h), dtype)
    # Joined as the decoder joins them: gate rows i..i+127, then up rows i..i+127.
    joined = np.empty((2 * inner, h), gate_t.dtype)
    for i0 in range(0, inner, 128):
        joined[2 * i0:2 * i0 + 128] = gate_t[i0:i0 + 128]
        joined[2 * i0 + 128:2 * i0 + 256] = up_t[i0:i0 + 128]
    x = rng.standard_normal((rows, h), dtype=np.float32) * 3
    g = (1 + 0.25 * rng.standard_normal(h)).astype(np.float32)
    shape = pkg.Shape(hidden=h, inner=inner, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=64, eps=eps)
    p = pkg.params(shape, dtype, rows=rows)
    mo = pkg.Memory(ctx, rows * inner * 4)
    pkg.dispatch_once(ctx, "gemv_gate_up", p, [(_mem(pkg, ctx, x), 0, x.nbytes), (_mem(pkg, ctx, g), 0, g.nbytes),
                                               (_mem(pkg, ctx, joined), 0, joined.nbytes), (mo, 0, rows * inner * 4)])
    got = mo.read(np.float32, rows * inner).reshape(rows, inner)

    def reference(xn):
        a, b = xn @ gate.T, xn @ up.T
        return a / (1 + np.exp(-a)) * b, a, b

    xn = _normed(x, g, np.float32(eps))
    want, a, b = reference(xn)
    e_a, e_b = _projection_bound(gate, xn, h), _projection_bound(up, xn, h)
    silu = a / (1 + np.exp(-a))
    bound = 1.1 * e_a * np.abs(b) + np.abs(silu) * e_b + e_a * e_b + 8 * U * np.abs(want) + 1e-30
    assert np.all(np.abs(got - want) <= bound), float(np.max(np.abs(got - want) / bound))
    # Planted: the norm's gain left out.
    no_gain, _, _ = reference(_normed(x, np.ones_like(g), np.float32(eps)))
    assert np.mean(np.abs(no_gain - want) > bound) > 0.9


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_gemv_qkv_rope_against_f64(pkg, ctx, syn, dtype):
    rng = np.random.default_rng(40)
    h, heads, kvh, hd, cap, eps = 1024, 16, 2, 64, 128, 1e-5
    half, width, slots = hd // 2, (heads + 2 * kvh) * hd, 3
    wt, w = _weights(syn, rng, (width, h), dtype)
    x = rng.standard_normal((3, h), dtype=np.float32)
    g = (1 + 0.25 * rng.standard_normal(h)).astype(np.float32)
    shape = pkg.Shape(hidden=h, inner=1024, heads=heads, kv_heads=kvh, head_dim=hd, layers=1, capacity=cap, eps=eps)
    cos, sin = shape.rope_tables()
    # Rows: position 37 in slot 2, position 100 in slot 0, and a spare row.
    rows = [(37, 2), (100, 0), None]
    words = np.array([37, 100, SPARE, 2, 0, 1], np.uint32)
    esz = 2 if dtype == "bf16" else 4
    cache_vals = slots * kvh * cap * hd
    sentinel = np.full(3 * heads * hd, 7.0, np.float32)
    mq = _mem(pkg, ctx, sentinel)
    mk, mv = pkg.Memory(ctx, cache_vals * esz), pkg.Memory(ctx, cache_vals * esz)
    p = pkg.params(shape, dtype, rows=3, slots=slots)
    pkg.dispatch_once(ctx, "gemv_qkv_rope", p, [
        (_mem(pkg, ctx, x), 0, x.nbytes), (_mem(pkg, ctx, g), 0, g.nbytes), (_mem(pkg, ctx, wt), 0, wt.nbytes),
        (_mem(pkg, ctx, cos), 0, cos.nbytes), (_mem(pkg, ctx, sin), 0, sin.nbytes), (_mem(pkg, ctx, words), 0, words.nbytes),
        (mq, 0, sentinel.nbytes), (mk, 0, cache_vals * esz), (mv, 0, cache_vals * esz)])
    q = mq.read(np.float32, sentinel.size).reshape(3, heads, hd)
    if dtype == "bf16":
        kc = syn.bf16_to_f32(mk.read(np.uint16, cache_vals)).reshape(slots, kvh, cap, hd)
        vc = syn.bf16_to_f32(mv.read(np.uint16, cache_vals)).reshape(slots, kvh, cap, hd)
    else:
        kc = mk.read(np.float32, cache_vals).reshape(slots, kvh, cap, hd)
        vc = mv.read(np.float32, cache_vals).reshape(slots, kvh, cap, hd)
    store = 2.0**-8 if dtype == "bf16" else 0.0

    def rotate(r, pos, sign=1.0):
        a, c = r[..., :half], r[..., half:]
        co, si = cos[pos].astype(np.float64), sign * sin[pos].astype(np.float64)
        return np.concatenate([a * co - c * si, c * co + a * si], axis=-1)

    for b, row in enumerate(rows):
        if row is None:
            assert np.all(q[b] == 7.0)  # a spare row stores nothing
            continue
        pos, slot = row
        xn = _normed(x[b:b + 1], g, np.float32(eps))[0]
        r = (w @ xn).reshape(heads + 2 * kvh, hd)
        e = _projection_bound(w, xn[None], h)[0].reshape(heads + 2 * kvh, hd)
        e_pair = e[:, :half] + e[:, half:]
        rot_bound = np.concatenate([e_pair, e_pair], axis=-1) + 3 * U * np.concatenate(
            [np.abs(r[:, :half]) + np.abs(r[:, half:])] * 2, axis=-1)
        want = np.concatenate([rotate(r[:heads + kvh], pos), r[heads + kvh:]])
        bound = rot_bound + 1e-30
        got_q = q[b].astype(np.float64)
        assert np.all(np.abs(got_q - want[:heads]) <= bound[:heads]), \
            float(np.max(np.abs(got_q - want[:heads]) / bound[:heads]))
        for kv in range(kvh):
            for got, at in ((kc[slot, kv, pos], heads + kv), (vc[slot, kv, pos], heads + kvh + kv)):
                bnd = 1.01 * bound[at] + store * np.abs(want[at])
                assert np.all(np.abs(got - want[at]) <= bnd), float(np.max(np.abs(got - want[at]) / bnd))
        # Planted: the rotation taken the other way.
        wrong = rotate(r[:heads], pos, sign=-1.0)
        assert np.mean(np.abs(wrong - want[:heads]) > bound[:heads]) > 0.5
    # Nothing else of the caches was written: only (slot 2, position 37) and (slot 0, position 100).
    written = np.zeros((slots, cap), bool)
    written[2, 37] = written[0, 100] = True
    assert np.all(kc.transpose(0, 2, 1, 3)[~written] == 0) and np.all(vc.transpose(0, 2, 1, 3)[~written] == 0)


@pytest.mark.parametrize("family", ["f32", "bf16", "bf16 persistent", "bf16 tensor"])
def test_nan_in_the_cache_past_each_row_changes_no_bit(pkg, ctx, syn, family):
    """Keys and values past a row's position are masked, never read into a sum: the reference's
    attention test plants NaN there (crates/vulkan/tests/glsl.rs:617-749). Here every kernel family
    (CUDA-core split, the persistent step, the tensor decoder's mma.sync split) steps once over a
    prefilled cache, then again over the same cache with NaN at every position past each row's,
    and gives the same bits."""
    dtype = family.split()[0]
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    rows = 16 if family.endswith("tensor") else 1
    cap, layers = 256, 2
    shape = syn.shape_of(cfg, capacity=cap, layers=layers)
    w = syn.make_weights(cfg, seed=0, layers=layers, jitter_gains=True, as_bits=dtype == "bf16")
    dec = pkg.Decoder(ctx, shape, rows=rows, slots=rows, dtype=dtype)
    if family.endswith("persistent"):
        dec.retuned(True)
    assert dec.tensor == family.endswith("tensor")
    dec.load(w)
    rng = np.random.default_rng(50)
    lens = [9 + 13 * s for s in range(rows)]  # each row's position: 9 .. 204
    pre = pkg.Prefill(dec, max_rows=256)
    for s, n in enumerate(lens):
        pre.run(0, rng.standard_normal((n, cfg.hidden), dtype=np.float32), slot=s)
    per_slot = dec.prefix_bytes(cap)
    kept = pkg.Memory(ctx, per_slot * rows)
    for s in range(rows):
        dec.copy_out(s, cap, kept, s * per_slot)
    x = rng.standard_normal((rows, cfg.hidden), dtype=np.float32)
    placement = [pkg.Row(lens[s], s) for s in range(rows)]
    want = dec.step_rows(placement, x)
    assert np.all(np.isfinite(want))
    # The kept caches again, with NaN at positions past each row's (the step writes the row's own).
    etype, nan = (np.uint16, 0x7FC0) if dtype == "bf16" else (np.uint32, 0x7FC00000)
    caches = kept.read(etype, per_slot * rows // np.dtype(etype).itemsize)
    caches = caches.reshape(rows, layers, 2, shape.kv_heads, cap, shape.head_dim)
    for s in range(rows):
        caches[s, :, :, :, lens[s] + 1:, :] = nan
    planted = pkg.Memory(ctx, per_slot * rows)
    planted.write(caches)
    for s in range(rows):
        dec.copy_in(s, cap, planted, s * per_slot)
    got = dec.step_rows(placement, x)
    np.testing.assert_array_equal(got, want)
    dec.close()

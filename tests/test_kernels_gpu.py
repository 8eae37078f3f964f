"""Single kernels of the table on the GPU, dispatched through the C ABI (tg_dispatch_once),
against f64 references; and the dispatch checks that refuse a binding too small for its params."""

import numpy as np
import pytest

from conftest import distance

pytestmark = pytest.mark.gpu


def _mem(pkg, ctx, a):
    a = np.ascontiguousarray(a)
    m = pkg.Memory(ctx, max(a.nbytes, 16))
    m.write(a)
    return m


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 1280, 1024), (384, 1024, 4096), (200, 192, 256),
                                   (128, 128, 128), (512, 8192, 1024)])
def test_tcgen05_gemm_matches_f64(pkg, ctx, syn, m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((n, k), dtype=np.float32) * 0.02
    ab, bb = syn.bf16_bits(a), syn.bf16_bits(b)
    ma, mb = _mem(pkg, ctx, ab), _mem(pkg, ctx, bb)
    mc = pkg.Memory(ctx, m * n * 4)
    shape = pkg.Shape(hidden=256, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "bf16", rows=m, m=m, n=n, k=k)
    pkg.dispatch_once(ctx, "gemm", p, [(ma, 0, ab.nbytes), (mb, 0, bb.nbytes), (mc, 0, m * n * 4)])
    got = mc.read(np.float32, m * n).reshape(m, n)
    af, bf = syn.bf16_to_f32(ab).astype(np.float64), syn.bf16_to_f32(bb).astype(np.float64)
    want = af @ bf.T
    # An f32 sum of k products is within k unit roundoffs of the sum of their magnitudes.
    bound = k * 2.0**-24 * (np.abs(af) @ np.abs(bf).T) + 1e-30
    assert np.all(np.abs(got - want) <= bound), float(np.max(np.abs(got - want) / bound))
    # A defect the bound catches: one k-step of 16 left out.
    short = af[:, 16:] @ bf[:, 16:].T
    assert np.mean(np.abs(short - want) > bound) > 0.5


@pytest.mark.parametrize("m,n,k,parts,flags", [(128, 1024, 1024, 8, 3), (64, 1024, 4096, 8, 3), (200, 256, 512, 2, 0),
                                                (128, 512, 1024, 4, 1)])
def test_gemm_in_parts_then_add_norm_rows(pkg, ctx, syn, m, n, k, parts, flags):
    """A GEMM in parts of K stores, for each part, exactly what the whole GEMM computes over that
    part's columns alone; add_norm_rows (a warp to a row, or with flags bit 1 a block) adds the
    parts in part order (f32, bit for bit as numpy's left-to-right sum) before the residual and the
    norm."""
    rng = np.random.default_rng(m + n + parts)
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((n, k), dtype=np.float32) * 0.02
    ab, bb = syn.bf16_bits(a), syn.bf16_bits(b)
    ma, mb = _mem(pkg, ctx, ab), _mem(pkg, ctx, bb)
    shape = pkg.Shape(hidden=n, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    mc = pkg.Memory(ctx, parts * m * n * 4)
    p = pkg.params(shape, "bf16", rows=m, m=m, n=n, k=k, parts=parts, flags=flags)
    pkg.dispatch_once(ctx, "gemm", p, [(ma, 0, ab.nbytes), (mb, 0, bb.nbytes), (mc, 0, parts * m * n * 4)])
    got = mc.read(np.float32, parts * m * n).reshape(parts, m, n)
    w = k // parts
    for j in sorted({0, parts - 1, parts // 2}):
        a_j, b_j = np.ascontiguousarray(ab[:, j * w:(j + 1) * w]), np.ascontiguousarray(bb[:, j * w:(j + 1) * w])
        one = pkg.Memory(ctx, m * n * 4)
        q = pkg.params(shape, "bf16", rows=m, m=m, n=n, k=w, flags=flags)
        pkg.dispatch_once(ctx, "gemm", q, [(_mem(pkg, ctx, a_j), 0, a_j.nbytes), (_mem(pkg, ctx, b_j), 0, b_j.nbytes),
                                           (one, 0, m * n * 4)])
        np.testing.assert_array_equal(got[j], one.read(np.float32, m * n).reshape(m, n), err_msg=f"part {j}")
    # Too few bytes for the parts, and a K the parts do not divide, are refused.
    with pytest.raises(pkg.ShapeError):
        pkg.dispatch_once(ctx, "gemm", p, [(ma, 0, ab.nbytes), (mb, 0, bb.nbytes), (mc, 0, m * n * 4)])
    bad = pkg.params(shape, "bf16", rows=m, m=m, n=n, k=k, parts=3 if k % 192 else 5, flags=flags)
    with pytest.raises(pkg.ShapeError):
        pkg.dispatch_once(ctx, "gemm", bad, [(ma, 0, ab.nbytes), (mb, 0, bb.nbytes), (mc, 0, parts * m * n * 4)])

    res = rng.standard_normal((m, n), dtype=np.float32)
    gain = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    words = _mem(pkg, ctx, np.zeros(m, np.uint32))
    msum, mnorm = pkg.Memory(ctx, m * n * 4), pkg.Memory(ctx, m * n * 2)
    pa = pkg.params(shape, "bf16", rows=m, parts=parts, flags=flags & 2)
    pkg.dispatch_once(ctx, "add_norm_rows", pa, [(words, 0, m * 4), (mc, 0, parts * m * n * 4), (_mem(pkg, ctx, res), 0, res.nbytes),
                                                 (_mem(pkg, ctx, gain), 0, gain.nbytes), (msum, 0, m * n * 4),
                                                 (mnorm, 0, m * n * 2)])
    c = got[0].copy()
    for j in range(1, parts):
        c = c + got[j]
    np.testing.assert_array_equal(msum.read(np.float32, m * n).reshape(m, n), res + c)
    s64 = (res + c).astype(np.float64)
    want = s64 / np.sqrt(np.mean(s64 * s64, axis=1, keepdims=True) + shape.eps) * gain
    assert distance(syn.bf16_to_f32(mnorm.read(np.uint16, m * n).reshape(m, n)), want)[1] < 1e-2
    with pytest.raises(pkg.ShapeError):  # at most 16 parts
        pkg.dispatch_once(ctx, "add_norm_rows", pkg.params(shape, "bf16", rows=m, parts=17),
                          [(words, 0, m * 4), (mc, 0, parts * m * n * 4), (msum, 0, m * n * 4), (msum, 0, m * n * 4),
                           (msum, 0, m * n * 4), (mnorm, 0, m * n * 2)])


def test_simt_gemm_f32(pkg, ctx):
    rng = np.random.default_rng(1)
    m, n, k = 100, 72, 48
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((n, k), dtype=np.float32)
    ma, mb, mc = _mem(pkg, ctx, a), _mem(pkg, ctx, b), pkg.Memory(ctx, m * n * 4)
    shape = pkg.Shape(hidden=256, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "f32", rows=m, m=m, n=n, k=k)
    pkg.dispatch_once(ctx, "gemm", p, [(ma, 0, a.nbytes), (mb, 0, b.nbytes), (mc, 0, m * n * 4)])
    got = mc.read(np.float32, m * n).reshape(m, n)
    np.testing.assert_allclose(got, a.astype(np.float64) @ b.T.astype(np.float64), atol=1e-4)


def test_a_binding_smaller_than_its_reach_is_refused(pkg, ctx):
    shape = pkg.Shape(hidden=256, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "f32", rows=2)
    x, g, out = pkg.Memory(ctx, 2 * 256 * 4), pkg.Memory(ctx, 256 * 4), pkg.Memory(ctx, 256 * 4)
    with pytest.raises(pkg.ShapeError):
        pkg.dispatch_once(ctx, "rmsnorm", p, [(x, 0, 2 * 256 * 4), (g, 0, 256 * 4), (out, 0, 256 * 4)])
    with pytest.raises(pkg.InvalidError):
        pkg.dispatch_once(ctx, "rmsnorm", p, [(x, 0, 2 * 256 * 4), (g, 0, 256 * 4)])


def test_rmsnorm_kernel(pkg, ctx):
    import oracle

    rng = np.random.default_rng(2)
    rows, h = 5, 1024
    x = rng.standard_normal((rows, h), dtype=np.float32) * 3
    g = (1 + 0.25 * rng.standard_normal(h)).astype(np.float32)
    mx, mg, mo = _mem(pkg, ctx, x), _mem(pkg, ctx, g), pkg.Memory(ctx, x.nbytes)
    shape = pkg.Shape(hidden=h, inner=1024, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "f32", rows=rows)
    pkg.dispatch_once(ctx, "rmsnorm", p, [(mx, 0, x.nbytes), (mg, 0, g.nbytes), (mo, 0, x.nbytes)])
    got = mo.read(np.float32, rows * h).reshape(rows, h)
    want = np.stack([oracle.rmsnorm(x[i], g, 1e-5) for i in range(rows)])
    assert distance(got, want)[0] < 1e-5


def test_stream_read_reads_every_word(pkg, ctx):
    words = np.arange(1 << 20, dtype=np.uint32) * np.uint32(2654435761)
    m = _mem(pkg, ctx, words)
    out = pkg.Memory(ctx, 148 * 8 * 4 * 4)
    shape = pkg.Shape(hidden=256, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "f32", rows=0, k=words.size, n=ctx.sm_count * 8)
    pkg.dispatch_once(ctx, "stream_read", p, [(m, 0, words.nbytes), (out, 0, ctx.sm_count * 8 * 4)])
    got = out.read(np.uint32, ctx.sm_count * 8)
    assert np.bitwise_xor.reduce(got) == np.bitwise_xor.reduce(words)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_decode_attention_split_and_combine_against_f64(pkg, ctx, syn, dtype):
    """attention_split + attention_combine (attention_split.comp, attention_combine.comp) over
    rows at chunk edges and a spare row: the same bits on a second run, and softmax attention in
    f64 for a live row within 1e-5 (glsl.rs:617-649 holds its attention to a bound of that order)."""
    rows, cap = 5, 256
    shape = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=cap)
    rng = np.random.default_rng(9)
    hd, heads, kv = 64, 16, 2
    q = rng.standard_normal((rows, heads, hd), dtype=np.float32)
    k = rng.standard_normal((rows, kv, cap, hd), dtype=np.float32)
    v = rng.standard_normal((rows, kv, cap, hd), dtype=np.float32)
    if dtype == "bf16":
        k, v = syn.bf16_bits(k), syn.bf16_bits(v)
    words = np.array([0, 63, 64, 0xFFFFFFFF, 255] + list(range(rows)), np.uint32)
    mq, mk, mv, mat = _mem(pkg, ctx, q), _mem(pkg, ctx, k), _mem(pkg, ctx, v), _mem(pkg, ctx, words)
    chunks = cap // 64
    po = pkg.Memory(ctx, rows * heads * chunks * hd * 4)
    pml = pkg.Memory(ctx, rows * heads * chunks * 2 * 4)
    n = rows * heads * hd
    outs = []
    for _ in range(2):
        a = pkg.Memory(ctx, n * 4)
        a.write(np.zeros(n, np.float32))
        p = pkg.params(shape, dtype, rows=rows, slots=rows)
        common = [(mq, 0, q.nbytes), (mk, 0, k.nbytes), (mv, 0, v.nbytes), (mat, 0, words.nbytes),
                  (po, 0, po.nbytes), (pml, 0, pml.nbytes)]
        pkg.dispatch_once(ctx, "attention_split", p, common)
        pkg.dispatch_once(ctx, "attention_combine", p, [(mat, 0, words.nbytes), (po, 0, po.nbytes),
                                                        (pml, 0, pml.nbytes), (a, 0, n * 4)])
        outs.append(a.read(np.float32, n))
    assert np.array_equal(outs[0], outs[1])
    # Against softmax attention in f64 for live rows at chunk edges: row 2 at position 64 (the first
    # position of the second chunk), row 1 at 63 (the last of the first), slot = row.
    kf = syn.bf16_to_f32(k) if dtype == "bf16" else k
    vf = syn.bf16_to_f32(v) if dtype == "bf16" else v
    got = outs[0].reshape(rows, heads, hd)
    for r, pos in ((2, 64), (1, 63), (4, 255)):
        for h in (0, 9):
            s = kf[r, h // 8, :pos + 1].astype(np.float64) @ q[r, h].astype(np.float64) / 8.0
            e = np.exp(s - s.max())
            want = (e / e.sum()) @ vf[r, h // 8, :pos + 1].astype(np.float64)
            assert np.max(np.abs(got[r, h] - want)) < 1e-5, (r, pos, h)


@pytest.mark.parametrize("m,inner,k,flags", [(200, 256, 256, 0), (512, 4096, 1024, 0), (128, 4096, 1024, 2),
                                             (40, 256, 256, 2)])
def test_gemm_silu_epilogue_equals_gemm_then_silu_mul_rows(pkg, ctx, syn, m, inner, k, flags):
    """The fused epilogue takes SiLU(gate) up of the same f32 accumulators the plain GEMM stores, so
    it matches gemm + silu_mul_rows bit for bit, in 256-column tiles and in narrow ones (flags bit
    1: each tile's gate and up rows loaded as two boxes of 32); gate and up rows are interleaved in
    blocks of 128."""
    rng = np.random.default_rng(m + inner)
    a = rng.standard_normal((m, k), dtype=np.float32)
    gate = rng.standard_normal((inner, k), dtype=np.float32) * 0.05
    up = rng.standard_normal((inner, k), dtype=np.float32) * 0.05
    w = np.concatenate([np.concatenate([gate[i:i + 128], up[i:i + 128]]) for i in range(0, inner, 128)])
    ab, wb = syn.bf16_bits(a), syn.bf16_bits(w)
    ma, mw = _mem(pkg, ctx, ab), _mem(pkg, ctx, wb)
    shape = pkg.Shape(hidden=256, inner=inner, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "bf16", rows=m, m=m, n=2 * inner, k=k)
    fused = pkg.Memory(ctx, m * inner * 2)
    pf = pkg.params(shape, "bf16", rows=m, m=m, n=2 * inner, k=k, flags=flags)
    pkg.dispatch_once(ctx, "gemm_silu", pf, [(ma, 0, ab.nbytes), (mw, 0, wb.nbytes), (fused, 0, m * inner * 2)])
    c = pkg.Memory(ctx, m * 2 * inner * 4)
    pkg.dispatch_once(ctx, "gemm", p, [(ma, 0, ab.nbytes), (mw, 0, wb.nbytes), (c, 0, m * 2 * inner * 4)])
    words = _mem(pkg, ctx, np.zeros(m, np.uint32))
    split = pkg.Memory(ctx, m * inner * 2)
    pkg.dispatch_once(ctx, "silu_mul_rows", p, [(words, 0, m * 4), (c, 0, m * 2 * inner * 4),
                                                (split, 0, m * inner * 2)])
    got = fused.read(np.uint16, m * inner).reshape(m, inner)
    np.testing.assert_array_equal(got, split.read(np.uint16, m * inner).reshape(m, inner))
    af = syn.bf16_to_f32(ab).astype(np.float64)
    g64 = af @ syn.bf16_to_f32(syn.bf16_bits(gate)).astype(np.float64).T
    u64 = af @ syn.bf16_to_f32(syn.bf16_bits(up)).astype(np.float64).T
    want = g64 / (1.0 + np.exp(-g64)) * u64
    assert distance(syn.bf16_to_f32(got), want)[1] < 1e-2


@pytest.mark.parametrize("m,flags", [(256, 0), (64, 2)])
def test_gemm_silu_output_16_byte_aligned_gives_the_same_bits(pkg, ctx, syn, m, flags):
    """The bf16 epilogues store a lane's 32 bytes of a row as one 256-bit store only at a 32-byte
    aligned address; an output binding that is 16- but not 32-byte aligned (the runtime asks for 16)
    takes two 16-byte stores and gives the same bits, in CTA pairs (256 rows) and narrow tiles."""
    inner, k = 256, 128
    rng = np.random.default_rng(m + 7)
    a = syn.bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    w = syn.bf16_bits(rng.standard_normal((2 * inner, k), dtype=np.float32) * 0.05)
    ma, mw = _mem(pkg, ctx, a), _mem(pkg, ctx, w)
    shape = pkg.Shape(hidden=256, inner=inner, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "bf16", rows=m, m=m, n=2 * inner, k=k, flags=flags)
    nb = m * inner * 2
    out0, out16 = pkg.Memory(ctx, nb), pkg.Memory(ctx, nb + 16)
    pkg.dispatch_once(ctx, "gemm_silu", p, [(ma, 0, a.nbytes), (mw, 0, w.nbytes), (out0, 0, nb)])
    pkg.dispatch_once(ctx, "gemm_silu", p, [(ma, 0, a.nbytes), (mw, 0, w.nbytes), (out16, 16, nb)])
    np.testing.assert_array_equal(out16.read(np.uint16, m * inner, offset=16), out0.read(np.uint16, m * inner))


def test_gemm_silu_refuses_a_width_it_does_not_tile(pkg, ctx):
    shape = pkg.Shape(hidden=256, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    p = pkg.params(shape, "bf16", rows=128, m=128, n=384, k=64)
    a, b, out = pkg.Memory(ctx, 128 * 64 * 2), pkg.Memory(ctx, 384 * 64 * 2), pkg.Memory(ctx, 128 * 192 * 2)
    with pytest.raises(pkg.ShapeError):
        pkg.dispatch_once(ctx, "gemm_silu", p, [(a, 0, a.nbytes), (b, 0, b.nbytes), (out, 0, out.nbytes)])


def test_gemm_qkv_rope_equals_gemm_then_rope_rows(pkg, ctx, syn):
    """RoPE and the cache append in the q/k/v GEMM's epilogue give the same bits as the GEMM's f32
    rows through rope_rows: q rows, and the caches at each row's position and slot."""
    H, heads, kvh, hd, cap, slots, m = 1024, 16, 2, 64, 256, 3, 384
    W = (heads + 2 * kvh) * hd
    shape = pkg.Shape(hidden=H, inner=4096, heads=heads, kv_heads=kvh, head_dim=hd, layers=1, capacity=cap)
    rng = np.random.default_rng(12)
    a = syn.bf16_bits(rng.standard_normal((m, H), dtype=np.float32))
    w = syn.bf16_bits(rng.standard_normal((W, H), dtype=np.float32) * 0.03)
    words = np.full(2 * m, 0xFFFFFFFF, np.uint32)
    for first, n, start, slot in ((0, 200, 17, 2), (256, 100, 0, 0)):
        words[first:first + n] = np.arange(start, start + n)
        words[m + first:m + first + n] = slot
    cs, sn = shape.rope_tables()
    ma, mw, mwd, mc, ms = (_mem(pkg, ctx, x) for x in (a, w, words, cs, sn))
    p = pkg.params(shape, "bf16", rows=m, slots=slots, m=m, n=W, k=H)
    cache = slots * kvh * cap * hd * 2
    qb = m * heads * hd * 2
    got, want = [], []
    for fused in (True, False):
        q, kc, vc = pkg.Memory(ctx, qb), pkg.Memory(ctx, cache), pkg.Memory(ctx, cache)
        if fused:
            pkg.dispatch_once(ctx, "gemm_qkv_rope", p, [(ma, 0, a.nbytes), (mw, 0, w.nbytes), (mwd, 0, words.nbytes),
                                                        (mc, 0, cs.nbytes), (ms, 0, sn.nbytes), (q, 0, qb),
                                                        (kc, 0, cache), (vc, 0, cache)])
        else:
            c = pkg.Memory(ctx, m * W * 4)
            pkg.dispatch_once(ctx, "gemm", p, [(ma, 0, a.nbytes), (mw, 0, w.nbytes), (c, 0, m * W * 4)])
            pkg.dispatch_once(ctx, "rope_rows", p, [(mwd, 0, words.nbytes), (c, 0, m * W * 4), (mc, 0, cs.nbytes),
                                                    (ms, 0, sn.nbytes), (q, 0, qb), (kc, 0, cache), (vc, 0, cache)])
        out = (q.read(np.uint16, qb // 2), kc.read(np.uint16, cache // 2), vc.read(np.uint16, cache // 2))
        (got if fused else want).append(out)
    live = np.repeat(words[:m] != 0xFFFFFFFF, heads * hd)
    np.testing.assert_array_equal(got[0][0][live], want[0][0][live])
    np.testing.assert_array_equal(got[0][1], want[0][1])
    np.testing.assert_array_equal(got[0][2], want[0][2])
    assert np.any(got[0][1] != 0) and np.any(got[0][2] != 0)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_gemv_linear_against_the_oracle_and_alone(pkg, ctx, syn, dtype):
    """gemv_linear.comp on the GPU: W [x0; x1] + bias through each activation, written at an
    offset of longer rows, within f32 rounding of the CPU oracle; each batch row the same bits
    computed alone."""
    import oracle

    rng = np.random.default_rng(21)
    rows, k0, k1, n, offset, stride = 5, 1024, 256, 200, 24, 256
    x0 = rng.standard_normal((rows, k0), dtype=np.float32)
    x1 = rng.standard_normal((rows, k1), dtype=np.float32)
    w = rng.standard_normal((n, k0 + k1), dtype=np.float32) * 0.03
    if dtype == "bf16":
        wb = syn.bf16_bits(w)
        w = syn.bf16_to_f32(wb)
    else:
        wb = w
    bias = rng.standard_normal(n).astype(np.float32)
    shape = pkg.Shape(hidden=256, inner=256, heads=4, kv_heads=1, head_dim=64, layers=1, capacity=64)
    mx0, mx1, mw, mb = (_mem(pkg, ctx, a) for a in (x0, x1, wb, bias))

    def run(act, r, xa, xb):
        p = pkg.params(shape, dtype, rows=r, n=n, k=k0, k1=k1, offset=offset, stride=stride, act=act, levels=9.0)
        out = pkg.Memory(ctx, r * stride * 4)
        out.fill(0)
        pkg.dispatch_once(ctx, "gemv_linear", p, [(xa, 0, r * k0 * 4), (xb, 0, r * k1 * 4), (mw, 0, wb.nbytes),
                                                  (mb, 0, bias.nbytes), (out, 0, r * stride * 4)])
        return out.read(np.float32, r * stride).reshape(r, stride)

    for act in (0, 1, 2):
        got = run(act, rows, mx0, mx1)
        want = oracle.gemv_linear(x0, x1, w, bias, act=act, levels=9.0, offset=offset, stride=stride)
        assert np.all(got[:, :offset] == 0) and np.all(got[:, offset + n:] == 0)
        if act == 2:
            lin = oracle.gemv_linear(x0, x1, w, bias, act=0)
            t9 = np.abs(np.tanh(lin.astype(np.float64)) * 9)
            safe = np.abs(t9 % 1 - 0.5) > 1e-3  # away from a rounding boundary
            assert np.array_equal(got[:, offset:offset + n][safe], want[:, offset:offset + n][safe])
        else:
            np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5)
        for b in (0, 3):
            alone = run(act, 1, _mem(pkg, ctx, x0[b:b + 1]), _mem(pkg, ctx, x1[b:b + 1]))
            np.testing.assert_array_equal(alone[0], got[b])
    bad = pkg.params(shape, dtype, rows=rows, n=n, k=k0, k1=k1, offset=100, stride=256, act=0, levels=9.0)
    with pytest.raises(pkg.ShapeError):
        pkg.dispatch_once(ctx, "gemv_linear", bad, [(mx0, 0, x0.nbytes), (mx1, 0, x1.nbytes), (mw, 0, wb.nbytes),
                                                    (mb, 0, bias.nbytes), (pkg.Memory(ctx, rows * 256 * 4), 0, rows * 256 * 4)])

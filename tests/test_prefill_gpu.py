"""The prefill on the GPU against the oracle: runs in pieces, several runs at once, zero weights,
and the refusals (crates/graph/tests/prefill.rs:278-363)."""

import numpy as np
import pytest

import oracle
from conftest import distance

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_prefill_in_pieces_matches_one_run_and_the_oracle(pkg, ctx, syn, dtype):
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    shape = syn.shape_of(cfg, capacity=512, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2, jitter_gains=True)
    x = syn.make_inputs(300, cfg.hidden, seed=2, bf16=dtype == "bf16")
    dec = pkg.Decoder(ctx, shape, rows=1, dtype=dtype)
    dec.load(w)
    whole = pkg.Prefill(dec, max_rows=384).run(0, x)
    small = pkg.Prefill(dec, max_rows=128)
    pieces = small.run(0, x)  # three pieces of at most 128
    assert small.max_rows() == 128
    ref = oracle.OracleStack(shape, w)
    want = ref.prefill(0, x)
    tol = 2e-4 if dtype == "f32" else 2e-2
    for got in (whole, pieces):
        m, _, cos = distance(got, want)
        assert m <= tol and cos >= 0.9999, (m, cos)
    # The cache after the run in pieces holds the oracle's keys and values.
    kc = dec.read_cache(1, 0, "k", 0, 300)
    assert distance(kc, ref.k_cache[1][0, :, :300])[0] <= (1e-4 if dtype == "f32" else 2e-2)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_runs_prefilled_together_match_each_run_alone(pkg, ctx, syn, dtype):
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    shape = syn.shape_of(cfg, capacity=256, layers=2)
    w = syn.make_weights(cfg, seed=1, layers=2)
    runs = [(0, 70, 0), (0, 130, 1), (5, 33, 2)]
    x = syn.make_inputs(sum(r[1] for r in runs), cfg.hidden, seed=5, bf16=dtype == "bf16")
    dec = pkg.Decoder(ctx, shape, rows=3, slots=3, dtype=dtype)
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=512)
    # The third run goes on from a 5-position prefix in its slot.
    pre.run(0, syn.make_inputs(5, cfg.hidden, seed=6), slot=2)
    together = pre.run_batch(runs, x)
    alone_dec = pkg.Decoder(ctx, shape, rows=1, slots=3, dtype=dtype)
    alone_dec.load(w)
    alone_pre = pkg.Prefill(alone_dec, max_rows=512)
    alone_pre.run(0, syn.make_inputs(5, cfg.hidden, seed=6), slot=2)
    row = 0
    for start, n, slot in runs:
        alone = alone_pre.run(start, x[row:row + n], slot=slot)
        assert np.array_equal(together[row:row + n], alone), (start, n, slot)
        row += n


def test_zero_weights_give_zero(pkg, ctx, syn):
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=128, layers=2)
    w = {k: np.zeros_like(v) for k, v in syn.make_weights(cfg, layers=2).items()}
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
    dec.load(w)
    out = pkg.Prefill(dec, max_rows=128).run(0, np.ones((40, cfg.hidden), np.float32))
    assert np.all(out == 0)


def test_refused_runs(pkg, ctx, syn):
    cfg = syn.TINY
    shape = syn.shape_of(cfg, capacity=64, layers=1)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="f32")
    pre = pkg.Prefill(dec, max_rows=128)
    with pytest.raises(pkg.ShapeError):
        pre.run(60, np.zeros((8, cfg.hidden), np.float32))  # past the capacity
    with pytest.raises(pkg.ShapeError):
        pre.run(0, np.zeros((8, cfg.hidden), np.float32), slot=1)  # no such slot
    with pytest.raises(pkg.ShapeError):
        pre.run(0, np.zeros(cfg.hidden + 1, np.float32))


def test_config2_full_stack_prefill_512_and_decode(pkg, ctx, syn):
    """BASELINE config 2 at full depth: 24 layers, a 512-position bf16 prefill, then decode steps."""
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=1024)
    w = syn.make_weights(cfg, seed=0)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=512)
    ref = oracle.OracleStack(shape, w)
    x = syn.make_inputs(512, cfg.hidden, seed=1, bf16=True)
    got, want = pre.run(0, x), ref.prefill(0, x)
    m, _, cos = distance(got, want)
    assert m <= 2e-2 and cos >= 0.9999, (m, cos)
    # Each step fed its own output, as config 1 runs: the stack amplifies any difference over the
    # steps (tests/test_oracle.py), so this holds over the first eight.
    h, hr = got[-1], want[-1]
    for t in range(8):
        h = dec.step(512 + t, h)[0]
        hr = ref.decode_step([(512 + t, 0)], hr[None])[0]
        m, _, cos = distance(h, hr)
        assert m <= 2e-2 and cos >= 0.9999, (t, m, cos)


def test_tcgen05_attention_matches_the_mma_sync_kernel_within_rounding(pkg, ctx, syn):
    """The prefill attention on tcgen05 (bf16, head_dim 64) against the mma.sync kernel of the
    kernel table on the same q and cache: runs of 128-aligned rows, causal, spare rows between."""
    import numpy as np

    from conftest import distance

    shape = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=512)
    rows, heads, hd, kvh, cap, slots = 512, 16, 64, 2, 512, 3
    rng = np.random.default_rng(8)
    q = syn.bf16_bits(rng.standard_normal((rows, heads, hd), dtype=np.float32))
    k = syn.bf16_bits(rng.standard_normal((slots, kvh, cap, hd), dtype=np.float32))
    v = syn.bf16_bits(rng.standard_normal((slots, kvh, cap, hd), dtype=np.float32))
    # Runs: 200 rows of slot 1 from position 37, 128 rows of slot 0 from 0, 100 rows of slot 2 from 400.
    words = np.full(2 * rows, 0xFFFFFFFF, np.uint32)
    for first, n, start, slot in ((0, 200, 37, 1), (256, 128, 0, 0), (384, 100, 400, 2)):
        words[first:first + n] = np.arange(start, start + n)
        words[rows + first:rows + first + n] = slot
    def mem(a):
        m = pkg.Memory(ctx, a.nbytes)
        m.write(np.ascontiguousarray(a))
        return m

    mw, mq, mk, mv = mem(words), mem(q), mem(k), mem(v)
    p = pkg.params(shape, "bf16", rows=rows, slots=slots)
    outs = []
    for kernel in ("attention_rows", "attention_rows_tc"):
        o = pkg.Memory(ctx, rows * heads * hd * 2)
        o.fill(0)
        pkg.dispatch_once(ctx, kernel, p, [(mw, 0, words.nbytes), (mq, 0, q.nbytes), (mk, 0, k.nbytes),
                                           (mv, 0, v.nbytes), (o, 0, rows * heads * hd * 2)])
        outs.append(syn.bf16_to_f32(o.read(np.uint16, rows * heads * hd)).reshape(rows, heads, hd))
    live = words[:rows] != 0xFFFFFFFF
    m, rel, cos = distance(outs[1][live], outs[0][live])
    assert rel < 1e-2 and cos > 0.9999, (m, rel, cos)
    assert np.all(outs[1][~live] == 0)  # spare rows are not written


def test_tcgen05_attention_moves_its_reference_on_later_tiles(pkg, ctx, syn):
    """Keys that grow with their position (x (1 + p / 32)) make each later 128-key tile's largest
    score pass the row's reference by ~14 (base 2, scaled) against the 8 that lets it stay, for
    rows with unit queries: their reference moves on every tile, O is rescaled in TMEM and the
    tile's pass runs again; rows with queries 0.02 as large, in the same warps, keep theirs. Against
    the mma.sync kernel within rounding, as above."""
    import numpy as np

    from conftest import distance

    shape = pkg.Shape(hidden=1024, inner=4096, heads=16, kv_heads=2, head_dim=64, layers=1, capacity=512)
    rows, heads, hd, kvh, cap, slots = 512, 16, 64, 2, 512, 2
    rng = np.random.default_rng(21)
    row_scale = np.where(np.arange(rows) % 2 == 0, 1.0, 0.02).astype(np.float32)
    q = syn.bf16_bits(rng.standard_normal((rows, heads, hd), dtype=np.float32) * row_scale[:, None, None])
    grow = (1.0 + np.arange(cap, dtype=np.float32) / 32.0)[None, None, :, None]
    k = syn.bf16_bits(rng.standard_normal((slots, kvh, cap, hd), dtype=np.float32) * grow)
    v = syn.bf16_bits(rng.standard_normal((slots, kvh, cap, hd), dtype=np.float32))
    # Runs: 384 rows of slot 1 from position 0, 100 rows of slot 0 from 300.
    words = np.full(2 * rows, 0xFFFFFFFF, np.uint32)
    for first, n, start, slot in ((0, 384, 0, 1), (384, 100, 300, 0)):
        words[first:first + n] = np.arange(start, start + n)
        words[rows + first:rows + first + n] = slot

    def mem(a):
        m = pkg.Memory(ctx, a.nbytes)
        m.write(np.ascontiguousarray(a))
        return m

    mw, mq, mk, mv = mem(words), mem(q), mem(k), mem(v)
    p = pkg.params(shape, "bf16", rows=rows, slots=slots)
    outs = []
    for kernel in ("attention_rows", "attention_rows_tc"):
        o = pkg.Memory(ctx, rows * heads * hd * 2)
        o.fill(0)
        pkg.dispatch_once(ctx, kernel, p, [(mw, 0, words.nbytes), (mq, 0, q.nbytes), (mk, 0, k.nbytes),
                                           (mv, 0, v.nbytes), (o, 0, rows * heads * hd * 2)])
        outs.append(syn.bf16_to_f32(o.read(np.uint16, rows * heads * hd)).reshape(rows, heads, hd))
    live = words[:rows] != 0xFFFFFFFF
    assert np.all(np.isfinite(outs[1][live]))
    m, rel, cos = distance(outs[1][live], outs[0][live])
    assert rel < 1e-2 and cos > 0.9999, (m, rel, cos)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_nan_in_the_cache_past_a_run_changes_no_bit(pkg, ctx, syn, dtype):
    """attention_rows.comp reads the keys past a tile's last position as zero (:77-83), so what a
    slot held past the run (a request that came out NaN there before, or any stale value) cannot
    reach the run's outputs: a prompt prefilled into a slot that is NaN everywhere gives the same
    bits as into a clean one. 300 positions leave the last 128-key tile 84 positions past the run;
    bf16 runs the tcgen05 kernel, f32 the CUDA-core one."""
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    cap = 512
    shape = syn.shape_of(cfg, capacity=cap, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2, jitter_gains=True, as_bits=dtype == "bf16")
    dec = pkg.Decoder(ctx, shape, rows=1, slots=2, dtype=dtype)
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=384)
    x = syn.make_inputs(300, cfg.hidden, seed=2, bf16=dtype == "bf16")
    want = pre.run(0, x, slot=0)
    assert np.all(np.isfinite(want))
    nan = pkg.Memory(ctx, dec.prefix_bytes(cap))
    nan.fill(0x7FC07FC0 if dtype == "bf16" else 0x7FC00000)
    dec.copy_in(1, cap, nan)
    got = pre.run(0, x, slot=1)
    np.testing.assert_array_equal(got, want)
    # The next decode step reads the same cache from either slot.
    step = x[-1:]
    a = dec.step_rows([pkg.Row(300, 0)], step)
    b = dec.step_rows([pkg.Row(300, 1)], step)
    np.testing.assert_array_equal(a, b)

"""The decode step on the GPU against the CPU oracle, and its batch invariance: a request decoded
beside others comes out bit for bit as it does alone (crates/graph/src/decode.rs:8-11,
crates/graph/tests/decode.rs:229-256)."""

import numpy as np
import pytest

import oracle
from conftest import distance

pytestmark = pytest.mark.gpu

# BASELINE: bf16 weights with f32 accumulation match burn's CPU f32 model within max-abs 2e-2
# and cosine >= 0.9999. The f32 stack is held far tighter.
BF16_MAX_ABS, BF16_COS = 2e-2, 0.9999
F32_MAX_ABS = 2e-4


def _within(got, want, dtype):
    m, rel, cos = distance(got, want)
    if dtype == "f32":
        assert m <= F32_MAX_ABS, (m, rel, cos)
    else:
        assert m <= BF16_MAX_ABS and cos >= BF16_COS, (m, rel, cos)


def test_config1_prefill_then_feedback_decode_matches_the_oracle(pkg, ctx, syn):
    """the tiny f32 stack, a 32-position prefill of N(0,1) embeddings (seed 1),
    then 16 decode steps each fed the previous step's output."""
    cfg = syn.TINY
    shape = syn.shape_of(cfg, capacity=64)
    w = syn.make_weights(cfg, seed=0)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="f32")
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=128)
    ref = oracle.OracleStack(shape, w)
    x = syn.make_inputs(32, cfg.hidden, seed=1)
    got, want = pre.run(0, x), ref.prefill(0, x)
    _within(got, want, "f32")
    h, hr = got[-1], want[-1]
    for t in range(16):
        if t % 2:
            h = dec.step(32 + t, h)[0]
        else:  # Decoder::step's parts (decode.rs:833-837)
            dec.set_input(32 + t, h)
            dec.start()
            dec.wait()
            h = dec.output()[0]
        hr = ref.decode_step([(32 + t, 0)], hr[None])[0]
        _within(h, hr, "f32")
    # The cache holds what the oracle's does.
    for l in (0, 3):
        for kind, oc in (("k", ref.k_cache), ("v", ref.v_cache)):
            got_c = dec.read_cache(l, 0, kind, 0, 48)
            assert distance(got_c, oc[l][0, :, :48])[0] < 1e-4


@pytest.mark.parametrize("layers", [2, 24])
def test_bf16_stack_matches_the_oracle(pkg, ctx, syn, layers):
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=256, layers=layers)
    w = syn.make_weights(cfg, seed=0, layers=layers, jitter_gains=True)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=128)
    ref = oracle.OracleStack(shape, w)
    x = syn.make_inputs(96, cfg.hidden, seed=1, bf16=True)
    got, want = pre.run(0, x), ref.prefill(0, x)
    _within(got, want, "bf16")
    h, hr = got[-1], want[-1]
    for t in range(8):
        h = dec.step(96 + t, h)[0]
        hr = ref.decode_step([(96 + t, 0)], hr[None])[0]
        _within(h, hr, "bf16")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_a_row_comes_out_bit_for_bit_as_it_does_alone(pkg, ctx, syn, dtype):
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    layers = 2
    shape = syn.shape_of(cfg, capacity=128, layers=layers)
    w = syn.make_weights(cfg, seed=0, layers=layers, jitter_gains=True)
    rng = np.random.default_rng(11)
    steps = 5
    xs = rng.standard_normal((steps, 64, cfg.hidden), dtype=np.float32)
    # Each request's positions: request r starts at position 3r % 40.
    start = [(3 * r) % 40 for r in range(64)]

    def run(rows, slots, requests, tensor=False):
        dec = pkg.Decoder(ctx, shape, rows=rows, slots=slots, dtype=dtype)
        if dec.tensor != tensor:
            dec.with_tensor(tensor)
        dec.load(w)
        outs = []
        for t in range(steps):
            placement = [None] * rows
            x = np.zeros((rows, cfg.hidden), np.float32)
            for i, r in enumerate(requests):
                placement[i] = pkg.Row(start[r] + t, i)
                x[i] = xs[t, r]
            outs.append(dec.step_rows(placement, x)[: len(requests)])
        dec.close()
        return np.stack(outs)  # [steps][requests][hidden]

    alone = {r: run(1, 1, [r])[:, 0] for r in (0, 5, 17, 63)}
    # Alone again on the persistent step: the same bits as on the kernels.
    for r in (0, 17):
        dec = pkg.Decoder(ctx, shape, rows=1, slots=1, dtype=dtype).retuned(True)
        dec.load(w)
        for t in range(steps):
            assert np.array_equal(dec.step_rows([pkg.Row(start[r] + t, 0)], xs[t, r][None])[0], alone[r][t])
        dec.close()
    for rows in (3, 8, 64):
        requests = list(range(rows)) if rows == 64 else [0, 5, 17][:rows] + list(range(20, 20 + rows - 3))
        batched = run(rows, rows, requests)
        for i, r in enumerate(requests):
            if r in alone:
                assert np.array_equal(batched[:, i], alone[r]), (rows, r)
    if dtype == "bf16":
        # The tcgen05 projections (a 64-row decoder's own): alone and beside 63 others alike.
        alone_tc = {r: run(64, 64, [r], tensor=True)[:, 0] for r in (0, 17, 63)}
        batched = run(64, 64, list(range(64)), tensor=True)
        for r, want in alone_tc.items():
            assert np.array_equal(batched[:, r], want), ("tensor", r)


def test_spare_rows_write_nothing_and_slots_are_kept_apart(pkg, ctx, syn):
    cfg = syn.TINY
    shape = syn.shape_of(cfg, capacity=64, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2)
    dec = pkg.Decoder(ctx, shape, rows=3, slots=4, dtype="f32")
    dec.load(w)
    ref = oracle.OracleStack(shape, w, slots=4)
    rng = np.random.default_rng(3)
    for t in range(4):
        x = rng.standard_normal((3, cfg.hidden), dtype=np.float32)
        rows = [pkg.Row(t, 2), None, pkg.Row(t + 7, 0)]
        got = dec.step_rows(rows, x)
        want = ref.decode_step([(t, 2), None, (t + 7, 0)], x)
        assert distance(got[[0, 2]], want[[0, 2]])[0] < F32_MAX_ABS
    # Slots 1 and 3 were never written; slot 0 only from position 7.
    assert np.all(dec.read_cache(0, 1, "k", 0, 64) == 0)
    assert np.all(dec.read_cache(1, 3, "v", 0, 64) == 0)
    assert np.all(dec.read_cache(0, 0, "k", 0, 7) == 0)
    with pytest.raises(pkg.ShapeError):
        dec.step_rows([pkg.Row(1, 2), pkg.Row(2, 2), None], np.zeros((3, cfg.hidden), np.float32))


def test_copy_slot_moves_a_prefix_between_slots(pkg, ctx, syn):
    cfg = syn.TINY
    shape = syn.shape_of(cfg, capacity=64, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2)
    dec = pkg.Decoder(ctx, shape, rows=2, slots=2, dtype="f32")
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=128)
    x = syn.make_inputs(20, cfg.hidden, seed=4)
    pre.run(0, x, slot=0)
    dec.copy_slot(0, 1, 20)
    for l in range(2):
        for kind in "kv":
            assert np.array_equal(dec.read_cache(l, 1, kind, 0, 20), dec.read_cache(l, 0, kind, 0, 20))
    # Decoding on from the copied prefix in slot 1 gives what slot 0 gives.
    h = np.random.default_rng(0).standard_normal((2, cfg.hidden), dtype=np.float32)
    h[1] = h[0]
    out = dec.step_rows([pkg.Row(20, 0), pkg.Row(20, 1)], h)
    assert np.array_equal(out[0], out[1])


@pytest.mark.parametrize("family", ["f32", "bf16", "bf16 persistent", "bf16 tensor"])
def test_a_cache_of_a_multiple_of_32_positions(pkg, ctx, syn, family):
    """A capacity is a multiple of CHUNK = 32 (decode.rs:28, :480), so the last 64-position
    attention chunk of a 160-position cache is half full: a prefill to position 140, then decode
    steps to the last position (159), against the oracle, in every kernel family."""
    dtype = family.split()[0]
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    rows = 16 if family.endswith("tensor") else 1
    cap, layers = 160, 2
    shape = syn.shape_of(cfg, capacity=cap, layers=layers)
    w = syn.make_weights(cfg, seed=0, layers=layers, jitter_gains=True)
    dec = pkg.Decoder(ctx, shape, rows=rows, slots=rows, dtype=dtype)
    if family.endswith("persistent"):
        dec.retuned(True)
    assert dec.tensor == family.endswith("tensor")
    dec.load(w)
    ref = oracle.OracleStack(shape, w)
    x = syn.make_inputs(140, cfg.hidden, seed=3, bf16=dtype == "bf16")
    got, want = pkg.Prefill(dec, max_rows=256).run(0, x), ref.prefill(0, x)
    _within(got, want, dtype)
    h, hr = got[-1], want[-1]
    for t in range(140, cap):
        xs = np.zeros((rows, cfg.hidden), np.float32)
        xs[0] = h
        h = dec.step_rows([pkg.Row(t, 0)] + [None] * (rows - 1), xs)[0]
        hr = ref.decode_step([(t, 0)], hr[None])[0]
        _within(h, hr, dtype)
    dec.close()


def test_refusals(pkg, ctx, syn):
    cfg = syn.TINY
    bad = syn.shape_of(cfg, capacity=100)  # not a multiple of 32 (decode.rs:28 CHUNK, :480)
    with pytest.raises(pkg.ShapeError):
        pkg.Decoder(ctx, bad, rows=1, dtype="f32")
    shape = syn.shape_of(cfg, capacity=64, layers=1)
    with pytest.raises(pkg.ShapeError):
        pkg.Decoder(ctx, shape, rows=3, slots=2, dtype="f32")
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="f32")
    with pytest.raises(pkg.InvalidError):
        dec.load_tensor("layers.0.self_attn.x_proj.weight", np.zeros(4, np.float32))
    with pytest.raises(pkg.ShapeError):
        dec.load_tensor("layers.0.self_attn.q_proj.weight", np.zeros(4, np.float32))
    with pytest.raises(pkg.ShapeError):
        dec.step(64, np.zeros(cfg.hidden, np.float32))


def test_timed_steps_label_six_dispatches_a_layer(pkg, ctx, syn):
    # crates/graph/src/decode.rs:935-951: six dispatches a layer and the final norm.
    cfg = syn.TINY
    shape = syn.shape_of(cfg, capacity=64)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="f32", timed=True)
    dec.load(syn.make_weights(cfg, seed=0))
    dec.step(0, np.ones(cfg.hidden, np.float32))
    t = dec.timings()
    assert len(t) == 6 * cfg.layers + 1
    assert [l for l, _ in t[:6]] == ["qkv_rope", "attention_split", "attention_combine", "o_proj",
                                     "gate_up", "down_proj"]
    assert t[-1][0] == "final_norm" and all(ns > 0 for _, ns in t)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_the_persistent_step_gives_the_kernel_steps_bits(pkg, ctx, syn, dtype):
    """One persistent launch per step and six kernels a layer (Decoder::retuned) take the same sums
    in the same order: every live row comes out bit for bit the same, spare rows included."""
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    shape = syn.shape_of(cfg, capacity=256, layers=3)
    w = syn.make_weights(cfg, seed=0, layers=3, jitter_gains=True)
    outs, caches = {}, {}
    for persistent in (True, False):
        dec = pkg.Decoder(ctx, shape, rows=2, slots=2, dtype=dtype)
        dec.load(w)
        dec.retuned(persistent)
        assert dec.persistent == persistent
        pkg.Prefill(dec, max_rows=128).run(0, syn.make_inputs(70, cfg.hidden, seed=3), slot=1)
        rng = np.random.default_rng(4)
        res = []
        for t in range(5):
            x = rng.standard_normal((2, cfg.hidden), dtype=np.float32)
            rows = [pkg.Row(t, 0), pkg.Row(70 + t, 1)] if t < 4 else [None, pkg.Row(74, 1)]
            res.append(dec.step_rows(rows, x))
        outs[persistent] = res
        caches[persistent] = [dec.read_cache(l, s_, k, 0, 75) for l in range(3) for s_ in range(2) for k in "kv"]
        dec.close()
    for t, (a, b) in enumerate(zip(outs[True], outs[False])):
        assert np.array_equal(a[1], b[1]), t
        if t < 4:
            assert np.array_equal(a[0], b[0]), t
    for a, b in zip(caches[True], caches[False]):
        assert np.array_equal(a, b)


def test_the_persistent_step_takes_small_batches_only(pkg, ctx, syn):
    shape = syn.shape_of(syn.S05B, capacity=1024, layers=1)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
    assert dec.persistent  # the default for bf16 decoders of one or two rows
    assert dec.labels() == ["decode_step"]
    assert dec.retuned(True).persistent
    assert not dec.retuned(False).persistent and len(dec.labels()) == 7
    with pytest.raises(pkg.ShapeError):
        pkg.Decoder(ctx, shape, rows=3, slots=3, dtype="bf16").retuned(True)


def test_a_checkpoint_file_loads_the_same_bits_as_the_arrays(pkg, ctx, syn, tmp_path):
    """Decoder::load from a safetensors file (checkpoint.rs) under a prefix: the same step, bit for
    bit, as loading the arrays themselves."""
    from tgtts_v4_b200 import checkpoint

    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=128, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2, jitter_gains=True, as_bits=True)
    path = tmp_path / "stack.safetensors"
    checkpoint.save(path, {"base_lm." + k: v for k, v in w.items()})
    x = syn.make_inputs(1, cfg.hidden, seed=4)
    outs = []
    for how in ("arrays", "file"):
        dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
        if how == "arrays":
            dec.load(w)
        else:
            dec.load_checkpoint(path, prefix="base_lm.")
        outs.append(dec.step(5, x))
        dec.close()
    np.testing.assert_array_equal(outs[0], outs[1])
    with pytest.raises(pkg.Error):
        pkg.Decoder(ctx, shape, rows=1, dtype="bf16").load_checkpoint(path, prefix="residual_lm.")

"""The LM side of a patch (crates/graph/src/lm_side.rs:337-495) on the GPU against the same
composition on the CPU oracle: the two stacks (the residual one without RoPE) and the linear
layers between them, over a few patches at two rows; and a row's bits alone."""

import numpy as np
import pytest

import oracle
from conftest import distance

pytestmark = pytest.mark.gpu


def _setup(pkg, syn):
    from tgtts_v4_b200.lm_side import LmSideShape

    cfg = syn.TINY
    base = syn.shape_of(cfg, capacity=128, layers=2)
    residual = syn.shape_of(cfg, capacity=128, layers=1)
    residual.rope = False
    shape = LmSideShape(base=base, residual=residual, encoder=128, dit=64, latent=32, levels=9)
    rng = np.random.default_rng(4)
    w = {}
    for prefix, layers, seed in (("base_lm.", 2, 0), ("residual_lm.", 1, 1)):
        for k, v in syn.make_weights(cfg, seed=seed, layers=layers, jitter_gains=True).items():
            w[prefix + k] = v
    for name, (n, k) in shape.head_shapes().items():
        w[f"{name}.weight"] = rng.standard_normal((n, k), dtype=np.float32) * np.float32(1 / np.sqrt(k))
        if name != "stop_head":
            w[f"{name}.bias"] = rng.standard_normal(n, dtype=np.float32) * np.float32(0.05)
    return cfg, shape, w


def test_lm_side_matches_the_oracle_composition(pkg, ctx, syn):
    from tgtts_v4_b200.lm_side import LmSide, oracle_step

    cfg, shape, w = _setup(pkg, syn)
    side = LmSide(pkg, ctx, shape, rows=2, dtype="f32")
    side.load(w)
    strip = lambda p: {k[len(p):]: v for k, v in w.items() if k.startswith(p)}  # noqa: E731
    stacks = (oracle.OracleStack(shape.base, strip("base_lm."), slots=2),
              oracle.OracleStack(shape.residual, strip("residual_lm."), slots=2))
    rng = np.random.default_rng(5)
    for t in range(4):
        enc = rng.standard_normal((2, shape.encoder), dtype=np.float32)
        rows = [(t, 0), (t + 3, 1)]
        mu, stop, levels = side.step(rows, enc)
        mu_r, stop_r, levels_r = oracle_step(oracle, shape, stacks, w, rows, enc)
        np.testing.assert_array_equal(levels, levels_r)  # the quantizer's levels, exactly
        assert np.all(np.abs(levels * 9 - np.round(levels * 9)) < 1e-4)
        assert distance(mu, mu_r)[0] < 2e-4 and distance(stop, stop_r)[0] < 2e-4, (t, distance(mu, mu_r))
    side.close()


def test_a_row_of_the_lm_side_is_the_same_bits_alone(pkg, ctx, syn):
    from tgtts_v4_b200.lm_side import LmSide

    cfg, shape, w = _setup(pkg, syn)
    both = LmSide(pkg, ctx, shape, rows=2, dtype="f32")
    alone = LmSide(pkg, ctx, shape, rows=1, dtype="f32")
    both.load(w)
    alone.load(w)
    rng = np.random.default_rng(6)
    for t in range(3):
        enc = rng.standard_normal((2, shape.encoder), dtype=np.float32)
        mu, stop, _ = both.step([(t, 0), (t + 7, 1)], enc)
        mu1, stop1, _ = alone.step([(t + 7, 0)], enc[1:])
        np.testing.assert_array_equal(mu1[0], mu[1])
        np.testing.assert_array_equal(stop1[0], stop[1])
    both.close()
    alone.close()


@pytest.mark.parametrize("rows", [1, 4])
def test_a_32000_word_logits_head_matches_the_oracle(pkg, ctx, syn, rows):
    """The optional vocabulary head (gemv_linear over the final hidden states) at V = 32000, the
    synthetic size it is timed at, bf16 weights: within f32 rounding of the oracle, and
    a row alone the same bits as among others."""
    import oracle
    from tgtts_v4_b200.lm_side import LogitsHead

    H, V = 1024, 32000
    rng = np.random.default_rng(31)
    w = syn.bf16_round(rng.standard_normal((V, H), dtype=np.float32) * 0.02)
    h = rng.standard_normal((rows, H), dtype=np.float32)
    head = LogitsHead(pkg, ctx, H, V, rows=rows)
    head.load(w)
    got = head(h)
    want = oracle.gemv_linear(h, None, w, np.zeros(V, np.float32))
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=2e-5)
    if rows > 1:
        one = LogitsHead(pkg, ctx, H, V, rows=1)
        one.load(w)
        np.testing.assert_array_equal(one(h[2:3])[0], got[2])

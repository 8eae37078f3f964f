"""The backbone at VoxCPM2's own base-LM shape (hidden 2048, FFN 6144, 16 heads of 128 over 2 KV
heads; crates/graph/src/decode.rs:946-947), which BASELINE's configs (head_dim 64) do not reach:
the prefill (mma.sync attention for head_dim 128), the batch-1 decode (CUDA-core GEMVs) and a
16-row decoder (tcgen05 projections, CUDA-core attention for head_dim 128), each against the
oracle, and a row among others bit for bit as alone."""

import numpy as np
import pytest

import oracle
from conftest import distance

pytestmark = pytest.mark.gpu

MAX_ABS, MIN_COS = 2e-2, 0.9999


def _within(got, want):
    m, rel, cos = distance(got, want)
    assert m <= MAX_ABS and cos >= MIN_COS, (m, rel, cos)


@pytest.fixture(scope="module")
def stack(pkg, ctx, syn):
    cfg = syn.VOXCPM2_LM
    shape = syn.shape_of(cfg, capacity=256, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2, jitter_gains=True)
    return cfg, shape, w


def test_prefill_and_batch1_decode_match_the_oracle(pkg, ctx, syn, stack):
    cfg, shape, w = stack
    ref = oracle.OracleStack(shape, w, slots=1)
    dec = pkg.Decoder(ctx, shape, rows=1, dtype="bf16")
    assert not dec.tensor
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=128)
    x = syn.make_inputs(100, cfg.hidden, seed=1, bf16=True)
    got, want = pre.run(0, x), ref.prefill(0, x)
    _within(got, want)
    h, hr = got[-1], want[-1]
    for t in range(4):
        h = dec.step(100 + t, h)[0]
        hr = ref.decode_step([(100 + t, 0)], hr[None])[0]
        _within(h, hr)


def test_a_16_row_decoder_matches_the_oracle_and_a_row_alone(pkg, ctx, syn, stack):
    cfg, shape, w = stack
    dec = pkg.Decoder(ctx, shape, rows=16, slots=16, dtype="bf16")
    assert dec.tensor
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=256)
    ref = oracle.OracleStack(shape, w, slots=1)
    x = syn.make_inputs(40, cfg.hidden, seed=2, bf16=True)
    hp = pre.run(0, x, slot=3)[-1]
    hr = ref.prefill(0, x)[-1]
    # Another request in slot 9, beside it.
    y = syn.make_inputs(24, cfg.hidden, seed=3, bf16=True)
    hy = pre.run(0, y, slot=9)[-1]
    both = dec.step_rows_n([pkg.Row(40, 3), pkg.Row(24, 9)], np.stack([hp, hy]))
    _within(both[0], ref.decode_step([(40, 0)], hr[None])[0])
    # The same step of slot 3 alone (position 40 again overwrites the same cache entry).
    alone = dec.step_rows_n([pkg.Row(40, 3)], hp[None])
    np.testing.assert_array_equal(alone[0], both[0])


def test_continuous_batching_at_this_shape_is_batch_invariant(pkg, ctx, syn, stack):
    """A 16-slot server (tcgen05 projections; the 6144-column down projection as the GEMV in every
    bucket): 6 requests admitted together and later, each re-run alone, the same bits at every
    step; one against the oracle."""
    from test_server_gpu import _serve

    cfg, shape, w = stack
    dec = pkg.Decoder(ctx, shape, rows=16, slots=16, dtype="bf16")
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=256)
    server = pkg.Server(dec, pre)
    rng = np.random.default_rng(7)
    requests, prompts, admit = [], [], []
    for i in range(6):
        n, steps = int(rng.integers(1, 60)), int(rng.integers(2, 12))
        requests.append((i * 2, n, steps))
        prompts.append(syn.make_inputs(n, cfg.hidden, seed=100 + i, bf16=True))
        admit.append(0 if i < 4 else 3)
    batched = _serve(pkg, server, requests, prompts, admit)
    for i in (0, 5):
        alone = _serve(pkg, server, [requests[i]], [prompts[i]], [0])
        for t, (a, b) in enumerate(zip(alone[0], batched[i])):
            np.testing.assert_array_equal(a, b, err_msg=f"request {i} step {t}")
    ref = oracle.OracleStack(shape, w)
    slot, n, steps = requests[1]
    h = ref.prefill(0, prompts[1])[-1]
    for t in range(steps):
        h = ref.decode_step([(n + t, 0)], h[None])[0]
        _within(batched[1][t], h)
    server.close()


def test_the_local_encoder_at_voxcpm2_width(pkg, ctx, syn):
    """VoxCPM2's local encoder widths (1024, 16 heads of 128), 2 layers: 20 patches within the
    tolerance of the oracle, 16 at once the same bits as one at a time."""
    from tgtts_v4_b200 import local

    cfg = syn.LOCAL_VOXCPM2
    shape = syn.local_shape(cfg, 2)
    w = syn.make_encoder_weights(cfg, seed=4, layers=2)
    patches = np.random.default_rng(9).standard_normal((20, cfg.feat_dim, cfg.patch_size)).astype(np.float32)
    want = oracle.OracleLocal(shape, w, "feat_encoder.", 1 + cfg.patch_size).encode(patches, cfg.feat_dim, cfg.patch_size)

    def run(rows):
        e = local.Encoder(ctx, shape, cfg.feat_dim, cfg.patch_size, rows)
        e.load(w)
        out = []
        for c0 in range(0, len(patches), rows):
            idx = list(range(c0, min(c0 + rows, len(patches))))
            out.append(e.encode(patches[idx + [0] * (rows - len(idx))])[:len(idx)].astype(np.float32))
        e.close()
        return np.concatenate(out)

    alone = run(1)
    _within(alone, want)
    np.testing.assert_array_equal(run(16), alone)

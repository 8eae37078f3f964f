"""VoxCPM2's local stacks on the B200 against the CPU oracle (oracle/local_ref.c), modelled on the
reference's own local tests (crates/graph/tests/local.rs): the sampler in one Euler step and in ten,
the encoder, each at several tunings; every case run alone and among others, where it must come
out bit for bit as alone; and the defects those tests plant (the conditions left out, a step short,
the frames reversed), which must fail the same tolerance.

The tolerance is BASELINE's: max |d| <= 2e-2 and cosine >= 0.9999, with the relative RMS reported.
"""

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9999


def distance(got, want):
    g, w = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    d = np.abs(g - w)
    cos = float(g @ w / (np.linalg.norm(g) * np.linalg.norm(w)))
    return float(d.max()), float(np.sqrt((d ** 2).mean() / (w ** 2).mean())), cos


def within(got, want):
    m, rel, cos = distance(got, want)
    return m <= MAX_ABS and cos >= MIN_COS


@pytest.fixture(scope="module")
def local(pkg):
    from tgtts_v4_b200 import local as mod

    return mod


def make_sampler(pkg, local, ctx, syn, cfg, rows, timesteps, weights, tuning=None, layers=None):
    shape = syn.local_shape(cfg, layers)
    s = local.Sampler(ctx, shape, cfg.feat_dim, cfg.patch_size, timesteps, rows, tuning)
    s.load(weights)
    return s


def sample_rows(s, mu, cond, noise, sampling):
    """The cases `rows` at a time, the last run padded with the first case (local.rs:206-229)."""
    n, R = len(mu), s.rows
    out = []
    for c0 in range(0, n, R):
        idx = list(range(c0, min(c0 + R, n)))
        pad = idx + [0] * (R - len(idx))
        got = s.sample(mu[pad], cond[pad], noise[pad], sampling[pad])
        out.append(got[:len(idx)])
    return np.concatenate(out)


TUNINGS = [None, (1, 1, 1), (2, 4, 2), (4, 2, 8)]


@pytest.mark.parametrize("tuning", TUNINGS)
def test_one_euler_step_samples_as_the_oracle_and_alone_among_others(pkg, local, ctx, syn, tuning):
    cfg = syn.LOCAL_SMALL
    w = syn.make_sampler_weights(cfg, seed=0)
    mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, 16, seed=1)
    t = None if tuning is None else local.Tuning(*tuning)
    ref = oracle.OracleLocal(syn.local_shape(cfg), w, "feat_decoder.estimator.", 11)
    want = ref.sample(mu, cond, noise, sampling, 2, cfg.feat_dim, cfg.patch_size)
    alone = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, 1, 2, w, t), mu, cond, noise, sampling)
    m, rel, cos = distance(alone, want)
    assert m <= MAX_ABS and cos >= MIN_COS, (m, rel, cos)
    for rows in (3, 16):
        got = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, rows, 2, w, t), mu, cond, noise, sampling)
        np.testing.assert_array_equal(got, alone, err_msg=f"{rows} rows")
    # Defect: the conditions left out (local.rs:381-395).
    got = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, 16, 2, w, t), np.zeros_like(mu), cond, noise, sampling)
    assert not within(got, want)


def test_ten_steps_sample_as_the_oracle_and_alone_among_others(pkg, local, ctx, syn):
    cfg = syn.LOCAL_SMALL
    w = syn.make_sampler_weights(cfg, seed=7)
    mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, 16, seed=8)
    ref = oracle.OracleLocal(syn.local_shape(cfg), w, "feat_decoder.estimator.", 11)
    want = ref.sample(mu, cond, noise, sampling, 10, cfg.feat_dim, cfg.patch_size)
    s1 = make_sampler(pkg, local, ctx, syn, cfg, 1, 10, w)
    assert s1.steps() == oracle.cfm_euler_steps(10)
    alone = sample_rows(s1, mu, cond, noise, sampling)
    m, rel, cos = distance(alone, want)
    assert m <= MAX_ABS and cos >= MIN_COS, (m, rel, cos)
    for rows in (5, 16):
        got = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, rows, 10, w), mu, cond, noise, sampling)
        np.testing.assert_array_equal(got, alone, err_msg=f"{rows} rows")
    # Defect: a step short (local.rs:430-436).
    short = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, 16, 9, w), mu, cond, noise, sampling)
    assert not within(short, want)


def test_a_voxcpm2_wide_sampler_samples_as_the_oracle_and_alone(pkg, local, ctx, syn):
    # 1024 wide, 16 heads of 128, 4096 inner, 2 layers: 16 rows are 352 tokens, two token chunks
    # in every projection.
    cfg = syn.LOCAL_VOXCPM2
    w = syn.make_sampler_weights(cfg, seed=11, layers=2)
    mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, 16, seed=12)
    ref = oracle.OracleLocal(syn.local_shape(cfg, 2), w, "feat_decoder.estimator.", 11)
    want = ref.sample(mu[:2], cond[:2], noise[:2], sampling[:2], 2, cfg.feat_dim, cfg.patch_size)
    alone = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, 1, 2, w, layers=2), mu, cond, noise, sampling)
    m, rel, cos = distance(alone[:2], want)
    assert m <= MAX_ABS and cos >= MIN_COS, (m, rel, cos)
    got = sample_rows(make_sampler(pkg, local, ctx, syn, cfg, 16, 2, w, layers=2), mu, cond, noise, sampling)
    np.testing.assert_array_equal(got, alone)


def test_a_sampler_loads_a_checkpoint_file_as_the_arrays(pkg, local, ctx, syn, tmp_path):
    # load_sampler from safetensors (f32 and bf16 tensors): the same patches as the arrays.
    from tgtts_v4_b200 import checkpoint

    cfg = syn.LOCAL_SMALL
    w = syn.make_sampler_weights(cfg, seed=9)
    bf16 = [n for n in w if n.endswith("mlp.down_proj.weight")]
    path = tmp_path / "sampler.safetensors"
    checkpoint.save(path, {n: (syn.bf16_bits(v) if n in bf16 else v) for n, v in w.items()})
    w_bf16 = {n: (syn.bf16_round(v) if n in bf16 else v) for n, v in w.items()}
    mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, 2, seed=10)
    a = make_sampler(pkg, local, ctx, syn, cfg, 2, 2, w_bf16)
    b = local.Sampler(ctx, syn.local_shape(cfg), cfg.feat_dim, cfg.patch_size, 2, 2)
    b.load_checkpoint(path)
    np.testing.assert_array_equal(b.sample(mu, cond, noise, sampling), a.sample(mu, cond, noise, sampling))


def make_encoder(pkg, local, ctx, syn, cfg, rows, weights, tuning=None, layers=None):
    e = local.Encoder(ctx, syn.local_shape(cfg, layers), cfg.feat_dim, cfg.patch_size, rows, tuning)
    e.load(weights)
    return e


def encode_rows(e, patches):
    n, R = len(patches), e.rows
    out = []
    for c0 in range(0, n, R):
        idx = list(range(c0, min(c0 + R, n)))
        got = e.encode(patches[idx + [0] * (R - len(idx))])
        out.append(got[:len(idx)].astype(np.float32))
    return np.concatenate(out)


@pytest.mark.parametrize("tuning", TUNINGS[:3])
def test_the_encoder_embeds_as_the_oracle_and_alone_among_others(pkg, local, ctx, syn, tuning):
    cfg = syn.LOCAL_SMALL
    w = syn.make_encoder_weights(cfg, seed=5)
    # Sharper attention than the N(0, 0.02) draw gives, so that the frames' places (RoPE) matter.
    for l in range(cfg.layers):
        for n in ("q_proj", "k_proj"):
            w[f"feat_encoder.encoder.layers.{l}.self_attn.{n}.weight"] *= np.float32(8.0)
    patches = np.random.default_rng(6).standard_normal((20, cfg.feat_dim, cfg.patch_size)).astype(np.float32)
    t = None if tuning is None else local.Tuning(*tuning)
    ref = oracle.OracleLocal(syn.local_shape(cfg), w, "feat_encoder.", 1 + cfg.patch_size)
    want = ref.encode(patches, cfg.feat_dim, cfg.patch_size)
    alone = encode_rows(make_encoder(pkg, local, ctx, syn, cfg, 1, w, t), patches)
    m, rel, cos = distance(alone, want)
    assert m <= MAX_ABS and cos >= MIN_COS, (m, rel, cos)
    for rows in (7, 16):
        np.testing.assert_array_equal(encode_rows(make_encoder(pkg, local, ctx, syn, cfg, rows, w, t), patches), alone)
    # Defect: the frames in another order, which only RoPE tells apart (local.rs:540-556).
    got = encode_rows(make_encoder(pkg, local, ctx, syn, cfg, 16, w, t), patches[:, :, ::-1].copy())
    assert not within(got, want)


def test_a_patch_that_comes_out_nan_is_not_finite(pkg, local, ctx, syn):
    """generator.rs:418-421: a sampled patch that is NaN or infinite is Error::NotFinite; the rows
    beside it are sampled as before, and so is the next sample."""
    cfg = syn.LOCAL_SMALL
    w = syn.make_sampler_weights(cfg, seed=0)
    mu, cond, noise, sampling = syn.make_sampler_inputs(cfg, 3, seed=1)
    s = make_sampler(pkg, local, ctx, syn, cfg, 3, 2, w)
    want = s.sample(mu, cond, noise, sampling)
    assert np.all(np.isfinite(want))
    bad = np.array(mu, np.float32)
    bad[1].flat[5] = np.nan
    with pytest.raises(pkg.NotFiniteError, match="row 1"):
        s.sample(bad, cond, noise, sampling)
    np.testing.assert_array_equal(s.sample(mu, cond, noise, sampling), want)


def test_the_local_kernels_refuse_what_they_do_not_take(pkg, local, ctx, syn):
    cfg = syn.LOCAL_SMALL
    bad = syn.local_shape(cfg)
    bad.hidden = 200  # local/mod.rs:375-385: the width a multiple of 256
    with pytest.raises(pkg.ShapeError):
        local.Sampler(ctx, bad, cfg.feat_dim, cfg.patch_size, 2, 1)
    with pytest.raises(pkg.ShapeError):
        local.Encoder(ctx, syn.local_shape(cfg), 12, cfg.patch_size, 1)  # channels a multiple of 8
    with pytest.raises(pkg.ShapeError):
        local.Sampler(ctx, syn.local_shape(cfg), cfg.feat_dim, cfg.patch_size, 2, 0)
    s = make_sampler(pkg, local, ctx, syn, cfg, 1, 2, syn.make_sampler_weights(cfg, seed=0))
    with pytest.raises(pkg.Error):
        s.load_tensor("feat_decoder.estimator.decoder.layers.9.mlp.up_proj.weight", np.zeros(4, np.float32))
    with pytest.raises(pkg.ShapeError):
        s.load_tensor("feat_decoder.estimator.out_proj.bias", np.zeros(3, np.float32))


def test_the_partial_projection_sums_each_part_of_the_columns(pkg, local, ctx):
    # TG_KERNEL_LOCAL_PARTIAL alone, against f64 sums of each part: token counts across a chunk
    # boundary (300 tokens are two chunks of 160), parts of 64 and 256 columns; the tokens
    # k-block-major, W tiled.
    rng = np.random.default_rng(0)
    for M, N, K, parts in ((1, 128, 256, 4), (22, 256, 512, 2), (300, 384, 256, 1), (37, 128, 1024, 4)):
        x = rng.standard_normal((M, K)).astype(np.float16)
        w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
        mx, mw = pkg.Memory(ctx, x.nbytes), pkg.Memory(ctx, w.nbytes)
        mp = pkg.Memory(ctx, parts * M * N * 4)
        mx.write(np.ascontiguousarray(x.reshape(M, K // 64, 64).transpose(1, 0, 2))), mw.write(local.tiled(w))
        p = pkg.TgParams(dtype=pkg.F16, m=M, n=N, k=K, parts=parts, rows=1, slots=1)
        pkg.dispatch_once(ctx, "local_partial", p, [(mx, 0, x.nbytes), (mw, 0, w.nbytes), (mp, 0, parts * M * N * 4)])
        got = mp.read(np.float32, parts * M * N).reshape(parts, M, N)
        kc = K // parts
        for j in range(parts):
            want = x[:, j * kc:(j + 1) * kc].astype(np.float64) @ w[:, j * kc:(j + 1) * kc].astype(np.float64).T
            np.testing.assert_allclose(got[j], want, rtol=1e-5, atol=1e-5 * np.abs(want).max())

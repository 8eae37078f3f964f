"""VoxCPM2's local stacks on the CPU: the oracle (oracle/local_ref.c) against the reference's rules
for the sampler's times (crates/graph/src/local/dit.rs:39-81) and against an independent numpy
restatement of the stack; the library's host functions against the oracle; the weight names."""

import numpy as np
import pytest

import oracle
from oracle import ref_numpy


def test_the_schedule_runs_from_one_to_zero_swayed_towards_one():
    # dit.rs:41-54: linspace(1, 0) then t + cos(pi t / 2) - 1 + t.
    for steps in (1, 2, 10, 25):
        s = oracle.cfm_schedule(steps)
        assert len(s) == steps + 1
        assert s[0] == pytest.approx(1.0, abs=1e-6) and s[-1] == 0.0
        assert np.all(np.diff(s) < 0)
        lin = np.linspace(1.0, 0.0, steps + 1)
        want = lin + (np.cos(np.pi / 2 * lin) - 1.0 + lin)
        np.testing.assert_allclose(s, want, atol=2e-6)


def test_the_first_four_percent_of_the_steps_but_at_least_one_run_nothing():
    # dit.rs:56-76: "Two steps, the first of which stays where it starts: one run of the DiT"
    # (crates/graph/tests/local.rs:372-374); ten steps run the DiT nine times.
    assert len(oracle.cfm_euler_steps(2)) == 1
    assert len(oracle.cfm_euler_steps(10)) == 9
    assert len(oracle.cfm_euler_steps(50)) == 48  # 51 times: int(51 * 0.04) = 2 stay
    for steps in (2, 10, 50):
        span = oracle.cfm_schedule(steps)
        run = oracle.cfm_euler_steps(steps)
        skipped = span[0] - run[0][0]
        # The steps run cover the rest of the way from 1 to 0.
        assert skipped + sum(dt for _, dt in run) == pytest.approx(1.0, abs=1e-5)
        for (t, dt), (t2, _) in zip(run, run[1:]):
            assert t - dt == pytest.approx(t2, abs=1e-6)


def test_the_library_steps_as_the_oracle(pkg):
    from tgtts_v4_b200 import local

    for steps in (1, 2, 10, 37):
        np.testing.assert_array_equal(local.schedule(steps), oracle.cfm_schedule(steps))
        assert local.euler_steps(steps) == oracle.cfm_euler_steps(steps)


def _small(syn, layers=2):
    cfg = syn.LOCAL_SMALL
    return cfg, syn.local_shape(cfg, layers)


@pytest.mark.parametrize("prefix,stack", [("feat_decoder.estimator.", "decoder."), ("feat_encoder.", "encoder.")])
def test_the_stack_oracle_matches_a_numpy_restatement(syn, prefix, stack):
    cfg, shape = _small(syn)
    w = (syn.make_sampler_weights if prefix.startswith("feat_decoder") else syn.make_encoder_weights)(cfg, seed=3)
    tokens = 11 if prefix.startswith("feat_decoder") else 5
    ref = oracle.OracleLocal(shape, w, prefix, tokens, threads=4)
    x = oracle.round_f16(np.random.default_rng(5).standard_normal((3 * tokens, cfg.hidden)).astype(np.float32))
    got = ref.stack(x, 3)
    w16 = {k: oracle.round_f16(v) for k, v in w.items()}
    want = ref_numpy.local_stack(shape, w16, prefix + stack, tokens, x)
    # Both round to f16 at the same points; a value whose f32 sum lands on the other side of an
    # f16 tie is off by one f16 step, which the next layers carry.
    d = np.abs(got - want)
    assert d.max() < 2e-2, d.max()
    assert np.sqrt((d ** 2).mean() / (want ** 2).mean()) < 2e-3


def test_a_sequence_comes_out_of_the_oracle_as_it_would_alone(syn):
    cfg, shape = _small(syn)
    w = syn.make_encoder_weights(cfg, seed=4)
    ref = oracle.OracleLocal(shape, w, "feat_encoder.", 5, threads=4)
    x = oracle.round_f16(np.random.default_rng(6).standard_normal((4 * 5, cfg.hidden)).astype(np.float32))
    together = ref.stack(x, 4)
    for s in range(4):
        np.testing.assert_array_equal(ref.stack(x[5 * s:5 * s + 5], 1), together[5 * s:5 * s + 5])


def test_the_time_tokens_are_the_mlps_in_f64(syn):
    # dit.rs:386-422: SinusoidalPosEmb(1000 t) in f32, linear_2(SiLU(linear_1(.))) in f64, time's
    # plus the delta MLP's at 0, rounded to f16.
    cfg, shape = _small(syn)
    w = syn.make_sampler_weights(cfg, seed=2)
    ref = oracle.OracleLocal(shape, w, "feat_decoder.estimator.", 11)
    H, half = cfg.hidden, cfg.hidden // 2
    p = "feat_decoder.estimator."
    w16 = {k: oracle.round_f16(v).astype(np.float64) for k, v in w.items()}

    def emb(t):
        rate = np.float32(-(np.log(10000.0) / (half - 1)))
        a = (np.float32(t) * np.float32(1000.0)) * np.exp(np.arange(half, dtype=np.float32) * rate).astype(np.float32)
        a = a.astype(np.float32).astype(np.float64)
        return np.concatenate([np.sin(a), np.cos(a)])

    def mlp(m, x):
        h = w16[f"{p}{m}.linear_1.weight"] @ x + w16[f"{p}{m}.linear_1.bias"]
        h = h / (1.0 + np.exp(-h))
        return w16[f"{p}{m}.linear_2.weight"] @ h + w16[f"{p}{m}.linear_2.bias"]

    times = [t for t, _ in oracle.cfm_euler_steps(10)]
    got = ref.time_tokens(times)
    for i, t in enumerate(times):
        want = (mlp("time_mlp", emb(t)) + mlp("delta_time_mlp", emb(0.0))).astype(np.float16).astype(np.float32)
        # The angles' sines and cosines come from libm's f32 functions in the oracle: within an
        # ulp of numpy's, which moves a token by at most an f16 step.
        np.testing.assert_allclose(got[i], want, atol=2e-3, rtol=2e-3)


def test_the_weight_names_are_upstreams(pkg):
    from tgtts_v4_b200 import local

    names = local.sampler_weight_names(2)
    assert "feat_decoder.estimator.decoder.layers.1.mlp.down_proj.weight" in names
    assert "feat_decoder.estimator.decoder.norm.weight" in names
    assert "feat_decoder.estimator.time_mlp.linear_2.bias" in names
    assert "feat_decoder.estimator.delta_time_mlp.linear_1.weight" in names
    assert len(names) == 2 * 9 + 1 + 6 + 8
    enc = local.encoder_weight_names(1)
    assert enc[-3:] == ["feat_encoder.special_token", "feat_encoder.in_proj.weight", "feat_encoder.in_proj.bias"]


def test_the_patch_config_derives_the_stack_as_upstream(pkg):
    # local/mod.rs:153-170: heads and width from the stack, the rest from the base LM.
    from tgtts_v4_b200 import local

    lm = {"hidden_size": 2048, "intermediate_size": 6144, "num_attention_heads": 16, "num_key_value_heads": 2,
          "num_hidden_layers": 28, "rms_norm_eps": 1e-5, "rope_theta": 10000, "kv_channels": 128,
          "max_position_embeddings": 32768, "use_mup": False,
          "rope_scaling": {"type": "longrope", "short_factor": [1.0] * 64, "long_factor": [1.0] * 64,
                           "original_max_position_embeddings": 32768}}
    stack = {"hidden_dim": 1024, "ffn_dim": 4096, "num_heads": 16, "num_layers": 4, "kv_channels": 128}
    cfg = local.PatchConfig.from_dict({"lm_config": lm, "patch_size": 4, "feat_dim": 64, "encoder_config": stack,
                                       "dit_config": dict(stack, mean_mode=False)})
    s = cfg.stack(cfg.dit_config.stack, 11)
    assert (s.hidden, s.inner, s.heads, s.kv_heads, s.head_dim, s.layers, s.capacity) == (1024, 4096, 16, 2, 128, 4, 11)
    assert s.residual_scale == 1.0
    mean = local.PatchConfig.from_dict({"lm_config": lm, "patch_size": 4, "feat_dim": 64, "encoder_config": stack,
                                        "dit_config": dict(stack, mean_mode=True)})
    assert mean.dit_config.mean_mode
    # Sampler::new refuses the DiT's mean mode (dit.rs:189-192), before it reaches the GPU.
    with pytest.raises(pkg.ShapeError):
        local.Sampler.from_config(None, mean, timesteps=10, rows=1)
    assert cfg.stack(cfg.encoder_config, 5).capacity == 5


def test_the_tiled_layout_puts_each_value_where_the_kernels_read_it(pkg):
    from tgtts_v4_b200 import local

    # local_tiled_offset: block (t, b) at (t k / 64 + b) 16 KiB, row r's chunk c at
    # (r / 8) 1024 + (r % 8) 128 + (c ^ (r % 8)) 16.
    n, k = 256, 192
    w = np.arange(n * k, dtype=np.float32).reshape(n, k) % 2039
    t = local.tiled(w)
    for row, col in ((0, 0), (5, 17), (127, 63), (128, 64), (200, 191), (9, 100)):
        tb, r, b, c = row // 128, row % 128, col // 64, (col % 64) // 8
        off = ((tb * (k // 64) + b) * 16384 + (r // 8) * 1024 + (r % 8) * 128 + ((c ^ (r % 8)) << 4)) // 2 + col % 8
        assert t[off] == np.float16(w[row, col]), (row, col)

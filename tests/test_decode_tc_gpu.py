"""The batched decoder's tcgen05 projections (bf16 decoders of 16 rows or more), in both forms - the
prefill's GEMMs over bf16 activations (the default) and split-K clusters over hi/lo activations:
against the CPU oracle within BASELINE's bf16 tolerance, and bit-identical rows in every row bucket,
so a request decoded beside 127 others comes out as it does alone (crates/graph/src/decode.rs:8-11)."""

import numpy as np
import pytest

import oracle
from conftest import distance

pytestmark = pytest.mark.gpu

BF16_MAX_ABS, BF16_COS = 2e-2, 0.9999


def _filled(pkg, ctx, syn, rows, layers, capacity, seed, split_k=False):
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=capacity, layers=layers)
    w = syn.make_weights(cfg, seed=0, layers=layers, jitter_gains=True, as_bits=True)
    dec = pkg.Decoder(ctx, shape, rows=rows, slots=rows, dtype="bf16")
    dec.with_tensor(True, split_k=split_k)  # the default is the GEMMs
    assert dec.tensor and dec.split_k == split_k
    dec.load(w)
    pre = pkg.Prefill(dec, max_rows=1024)
    rng = np.random.default_rng(seed)
    lens = [int(v) for v in rng.integers(1, capacity // 2, rows)]
    prompts = [rng.standard_normal((n, cfg.hidden), dtype=np.float32) for n in lens]
    # All prompts at once, as the server admits them (runs of up to 1024 rows a launch, each
    # starting on a multiple of 128 rows).
    runs, xs, used = [], [], 0
    for s, (n, x) in enumerate(zip(lens, prompts)):
        if used + n + 128 > 1024:
            pre.run_batch(runs, np.concatenate(xs))
            runs, xs, used = [], [], 0
        runs.append((0, n, s))
        xs.append(x)
        used += (n + 127) // 128 * 128
    pre.run_batch(runs, np.concatenate(xs))
    return cfg, shape, w, dec, pre, lens, prompts


@pytest.mark.parametrize("split_k", [False, True], ids=["gemm", "split_k"])
@pytest.mark.parametrize("rows,capacity", [(16, 256), (64, 256), (128, 256), (64, 1280)])
def test_tensor_decoder_rows_are_the_same_bits_in_every_bucket(pkg, ctx, syn, rows, capacity, split_k):
    """Contexts up to half the capacity: at 1280 the attention joins up to three blocks of 256
    positions a row, whichever arrives last."""
    cfg, shape, w, dec, pre, lens, _ = _filled(pkg, ctx, syn, rows, layers=2, capacity=capacity, seed=rows,
                                               split_k=split_k)
    assert dec.tensor
    rng = np.random.default_rng(1)
    x = rng.standard_normal((rows, cfg.hidden), dtype=np.float32)
    rws = [pkg.Row(lens[s], s) for s in range(rows)]
    full = dec.step_rows(rws, x)
    for n in sorted({1, 2, 3, 7, 16, rows // 2 + 1, rows}):
        got = dec.step_rows_n(rws[:n], x[:n])
        np.testing.assert_array_equal(got, full[:n], err_msg=f"{n} rows")
    for b in (0, rows // 3, rows - 1):
        alone = dec.step_rows_n([rws[b]], x[b:b + 1])
        np.testing.assert_array_equal(alone[0], full[b], err_msg=f"row {b} alone")


@pytest.mark.parametrize("rows,layers,capacity,split_k", [(64, 2, 192, False), (128, 24, 192, False),
                                                        (64, 2, 1280, False), (64, 2, 192, True),
                                                        (128, 24, 192, True)])
def test_tensor_decoder_matches_the_oracle(pkg, ctx, syn, rows, layers, capacity, split_k):
    cfg, shape, w, dec, pre, lens, prompts = _filled(pkg, ctx, syn, rows, layers=layers, capacity=capacity, seed=3,
                                                     split_k=split_k)
    check = [0, rows // 2, rows - 1]
    ref = oracle.OracleStack(shape, syn.as_f32(w), slots=len(check))
    for j, s in enumerate(check):
        ref.prefill(0, prompts[s], slot=j)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((rows, cfg.hidden), dtype=np.float32)
    rws = [pkg.Row(lens[s], s) for s in range(rows)]
    for t in range(3):
        got = dec.step_rows(rws, x)
        want = ref.decode_step([(lens[s] + t, j) for j, s in enumerate(check)], x[check])
        for j, s in enumerate(check):
            m, rel, cos = distance(got[s], want[j])
            assert m <= BF16_MAX_ABS and cos >= BF16_COS, (t, s, m, rel, cos)
        x = got
        rws = [pkg.Row(lens[s] + t + 1, s) for s in range(rows)]


@pytest.mark.parametrize("split_k", [False, True], ids=["gemm", "split_k"])
def test_tensor_and_gemv_decoders_agree(pkg, ctx, syn, split_k):
    """The kernel families compute the same step to within their roundings: the split-K form
    carries 16 bits of each activation, close to the GEMVs' f32 (within 1e-2); the GEMM form rounds
    the projections' inputs to bf16 as the prefill does (within BASELINE's bf16 tolerance)."""
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=128, layers=2)
    w = syn.make_weights(cfg, seed=0, layers=2, jitter_gains=True, as_bits=True)
    big = pkg.Decoder(ctx, shape, rows=16, slots=16, dtype="bf16")
    big.with_tensor(True, split_k=split_k)
    small = pkg.Decoder(ctx, shape, rows=1, slots=16, dtype="bf16")
    assert big.tensor and big.split_k == split_k and not small.tensor
    rng = np.random.default_rng(5)
    prompt = rng.standard_normal((40, cfg.hidden), dtype=np.float32)
    x = rng.standard_normal((1, cfg.hidden), dtype=np.float32)
    outs = []
    for dec in (big, small):
        dec.load(w)
        pkg.Prefill(dec, max_rows=128).run(0, prompt, slot=3)
        outs.append(dec.step_rows_n([pkg.Row(40, 3)], x)[0])
    m, rel, cos = distance(outs[0], outs[1])
    if split_k:
        assert m < 1e-2 and cos > 0.99999, (m, rel, cos)
    else:
        assert m <= BF16_MAX_ABS and cos >= BF16_COS, (m, rel, cos)


def test_the_default_family_by_rows(pkg, ctx, syn):
    """bf16 decoders of 16 rows or more run the prefill's GEMMs (faster than split-K clusters on
    B200 at every size from 16 rows), of fewer rows the GEMVs."""
    shape = syn.shape_of(syn.S05B, capacity=128, layers=1)
    for rows, tensor, split_k in ((1, False, False), (15, False, False), (16, True, False), (64, True, False),
                                  (128, True, False)):
        dec = pkg.Decoder(ctx, shape, rows=rows, slots=rows, dtype="bf16")
        assert (dec.tensor, dec.split_k) == (tensor, split_k), rows
        dec.close()

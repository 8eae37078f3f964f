"""Continuous batching on the GPU (crates/graph/src/generator.rs:99-352): row
buckets, requests admitted between steps by prefill, and the invariant that makes it safe — a
request decoded beside others comes out bit for bit as it does alone (crates/graph/src/decode.rs:8-11,
crates/graph/tests/generator.rs)."""

import numpy as np
import pytest

import oracle
from conftest import distance

pytestmark = pytest.mark.gpu


def _stack(pkg, ctx, syn, dtype, rows, capacity, layers=None):
    cfg = syn.TINY if dtype == "f32" else syn.S05B
    shape = syn.shape_of(cfg, capacity=capacity, layers=layers)
    w = syn.make_weights(cfg, seed=0, layers=layers, jitter_gains=True, as_bits=dtype == "bf16")
    dec = pkg.Decoder(ctx, shape, rows=rows, slots=rows, dtype=dtype)
    dec.load(w)
    return cfg, shape, w, dec


@pytest.mark.parametrize("dtype,layers", [("f32", None), ("bf16", 2)])
def test_a_row_is_the_same_bits_in_every_bucket(pkg, ctx, syn, dtype, layers):
    cfg, shape, w, dec = _stack(pkg, ctx, syn, dtype, rows=8, capacity=128, layers=layers)
    pre = pkg.Prefill(dec, max_rows=256)
    rng = np.random.default_rng(4)
    lens = [5, 17, 64, 3, 40, 9, 30, 12]
    for slot, n in enumerate(lens):
        pre.run(0, rng.standard_normal((n, cfg.hidden), dtype=np.float32), slot=slot)
    x = rng.standard_normal((8, cfg.hidden), dtype=np.float32)
    rows = [pkg.Row(lens[s], s) for s in range(8)]
    full = dec.step_rows(rows, x)
    for n in (1, 2, 3, 5, 8):
        got = dec.step_rows_n(rows[:n], x[:n])
        np.testing.assert_array_equal(got, full[:n])
    for b in range(8):
        alone = dec.step_rows_n([rows[b]], x[b:b + 1])
        np.testing.assert_array_equal(alone[0], full[b])
    with pytest.raises(pkg.ShapeError):
        dec.step_rows_n(rows + rows[:1], np.zeros((9, cfg.hidden), np.float32))


def _serve(pkg, server, requests, prompts, admit_at):
    """Runs `requests` ((slot, len, steps), prompt rows in `prompts`), admitting request i at step
    admit_at[i] (once its slot is free), until all are done; each request's outputs by step."""
    outs = {i: [] for i in range(len(requests))}
    owner = {}
    pending = list(range(len(requests)))
    step = 0
    while pending or owner:
        ready = [i for i in pending if admit_at[i] <= step and requests[i][0] not in owner]
        if ready:
            server.start([requests[i] for i in ready], np.concatenate([prompts[i] for i in ready]))
            for i in ready:
                owner[requests[i][0]] = i
                pending.remove(i)
        slots, out = server.step()
        for r, slot in enumerate(slots):
            outs[owner[slot]].append(out[r].copy())
        for slot in list(owner):
            held, _, left = server.request(slot)
            if held and left == 0:
                server.finish(slot)
                del owner[slot]
        step += 1
        assert step < 10000
    return outs


@pytest.mark.parametrize("dtype,layers", [("f32", None), ("bf16", 2)])
def test_continuous_batching_is_batch_invariant_and_matches_the_oracle(pkg, ctx, syn, dtype, layers):
    cfg, shape, w, dec = _stack(pkg, ctx, syn, dtype, rows=8, capacity=192, layers=layers)
    pre = pkg.Prefill(dec, max_rows=256)
    server = pkg.Server(dec, pre)
    rng = np.random.default_rng(5)
    # 14 requests over 8 slots: the first 8 at once, then each later one as its slot frees.
    requests, prompts, admit = [], [], []
    for i in range(14):
        slot = i % 8
        n = int(rng.integers(1, 70))
        steps = int(rng.integers(1, 30))
        requests.append((slot, n, steps))
        prompts.append(rng.standard_normal((n, cfg.hidden), dtype=np.float32))
        admit.append(0 if i < 8 else int(rng.integers(0, 20)))
    batched = _serve(pkg, server, requests, prompts, admit)
    for i, r in enumerate(requests):
        assert len(batched[i]) == r[2]
    # Each of 5 requests again, alone in the same server: the same bits at every step.
    for i in (0, 3, 8, 11, 13):
        alone = _serve(pkg, server, [requests[i]], [prompts[i]], [0])
        for t, (a, b) in enumerate(zip(alone[0], batched[i])):
            np.testing.assert_array_equal(a, b, err_msg=f"request {i} step {t}")
    # And one request against the CPU oracle, prompt then fed-back steps.
    ref = oracle.OracleStack(shape, syn.as_f32(w))
    i = 3
    slot, n, steps = requests[i]
    h = ref.prefill(0, prompts[i])[-1]
    tol = 2e-4 if dtype == "f32" else 2e-2
    for t in range(steps):
        h = ref.decode_step([(n + t, 0)], h[None])[0]
        m, rel, cos = distance(batched[i][t], h)
        assert m <= tol and cos >= 0.9999, (t, m, rel, cos)
    server.close()


def test_server_refusals(pkg, ctx, syn):
    cfg, shape, w, dec = _stack(pkg, ctx, syn, "f32", rows=4, capacity=64)
    pre = pkg.Prefill(dec, max_rows=128)
    server = pkg.Server(dec, pre)
    x = np.zeros((10, cfg.hidden), np.float32)
    with pytest.raises(pkg.ShapeError):
        server.start([(4, 10, 1)], x)  # no slot 4
    with pytest.raises(pkg.ShapeError):
        server.start([(0, 10, 55)], x)  # past the capacity
    with pytest.raises(pkg.ShapeError):
        server.start([(1, 5, 1), (1, 5, 1)], x)  # one slot twice
    slots, out = server.step()
    assert slots == [] and out.shape == (0, cfg.hidden)
    with pytest.raises(pkg.InvalidError):
        server.finish(2)
    wide = pkg.Decoder(ctx, shape, rows=2, slots=4, dtype="f32")
    with pytest.raises(pkg.ShapeError):
        pkg.Server(wide, pkg.Prefill(wide, max_rows=128))


@pytest.mark.parametrize("dtype,layers", [("f32", None), ("bf16", 2)])
def test_a_kept_prefix_gives_the_same_bits_as_the_whole_prompt(pkg, ctx, syn, dtype, layers):
    """prompt.rs's prompt cache on the backbone: a request whose prompt begins with a kept prefix
    copies its keys and values in and prefills only the rest, and comes out bit for bit as the
    same request prefilled whole; the cache keeps to its budget."""
    from tgtts_v4_b200.prompt_cache import PromptCache

    cfg, shape, w, dec = _stack(pkg, ctx, syn, dtype, rows=4, capacity=512, layers=layers)
    pre = pkg.Prefill(dec, max_rows=512)
    server = pkg.Server(dec, pre)
    cache = PromptCache(dec, budget=dec.prefix_bytes(300))
    rng = np.random.default_rng(9)
    voice = rng.standard_normal((260, cfg.hidden), dtype=np.float32)
    tail = rng.standard_normal((40, cfg.hidden), dtype=np.float32)
    prompt = np.concatenate([voice, tail])
    steps = 6

    def run(slot, start):
        server.start([(slot, len(prompt), steps, start)], prompt[start:])
        outs = []
        for _ in range(steps):
            slots, out = server.step()
            outs.append(out[slots.index(slot)].copy())
        server.finish(slot)
        return outs

    whole = run(0, 0)
    # The voice alone, kept from its slot after its prefill.
    server.start([(1, len(voice), 1)], voice)
    server.step()
    server.finish(1)
    assert cache.keep(1, voice)
    assert not cache.keep(1, voice[:100])  # already covered
    start = cache.restore(2, prompt)
    assert start == 260
    cached = run(2, start)
    for t in range(steps):
        np.testing.assert_array_equal(cached[t], whole[t], err_msg=f"step {t}")
    # The caches themselves match over the prompt's positions.
    for layer in (0, shape.layers - 1):
        np.testing.assert_array_equal(dec.read_cache(layer, 2, "k", 0, 300), dec.read_cache(layer, 0, "k", 0, 300))
    # A second prefix past the budget drops the first.
    other = rng.standard_normal((200, cfg.hidden), dtype=np.float32)
    server.start([(3, 200, 1)], other)
    server.step()
    server.finish(3)
    assert cache.keep(3, other)
    assert cache.restore(0, prompt) == 0 and cache.bytes <= cache.budget
    server.close()

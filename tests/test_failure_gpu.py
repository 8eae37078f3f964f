"""Failure detection in the two forms the reference has it, driven without a GPU fault:

- the host's wait gives up at its deadline (Submission::wait, crates/vulkan/src/context.rs:119-136)
  and leaves the run pending, to be waited for again before the recording is reused
  (crates/vulkan/src/recording.rs:631-642, :747-760): a 1 us deadline on a 24-layer step returns
  TG_ETIMEOUT, a second wait succeeds, and the step's outputs are the bits of a step waited for
  normally;
- a kernel's own bounded waits (an mbarrier no one arrives on, a global word no one writes) give
  up at their limit, report TG_EKERNEL through the context's error word, and the context then
  runs a step with the same bits as before.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _decoder(pkg, ctx, syn, rows=1):
    cfg = syn.S05B
    shape = syn.shape_of(cfg, capacity=1024)
    dec = pkg.Decoder(ctx, shape, rows=rows, dtype="bf16")
    dec.load(syn.make_weights(cfg, seed=0, as_bits=True))
    return cfg, dec


def test_a_wait_past_its_deadline_times_out_and_the_run_stays_pending(pkg, ctx, syn):
    cfg, dec = _decoder(pkg, ctx, syn)
    x = syn.make_inputs(1, cfg.hidden, seed=4)
    want = dec.step(0, x)
    dec.set_input(0, x)
    dec.start()
    with pytest.raises(pkg.TimeoutError):
        dec.wait(1000)  # 1 us: a 24-layer step takes hundreds
    dec.wait(0)  # the same run, waited for to its end
    np.testing.assert_array_equal(dec.output(), want)
    # A start after a wait that gave up first waits for the pending run, then launches the next.
    dec.start()
    with pytest.raises(pkg.TimeoutError):
        dec.wait(1000)
    dec.start()
    dec.wait(0)
    np.testing.assert_array_equal(dec.output(), want)
    # The context's own wait gives up the same way.
    dec.start()
    with pytest.raises(pkg.TimeoutError):
        ctx.synchronize(1000)
    ctx.synchronize()
    dec.wait(0)
    np.testing.assert_array_equal(dec.output(), want)
    dec.close()


def test_a_kernel_wait_that_runs_out_reports_an_error_and_the_context_stays_usable(pkg, ctx, syn):
    cfg, dec = _decoder(pkg, ctx, syn)
    x = syn.make_inputs(1, cfg.hidden, seed=5)
    want = dec.step(3, x)
    with pytest.raises(pkg.KernelError, match="bounded wait"):
        ctx.selftest_wait(1_000_000)  # 1 ms
    # The error word was taken by that wait: the next ones report nothing.
    ctx.synchronize()
    np.testing.assert_array_equal(dec.step(3, x), want)
    with pytest.raises(pkg.KernelError):
        ctx.selftest_wait(20_000)
    np.testing.assert_array_equal(dec.step(3, x), want)
    with pytest.raises(pkg.InvalidError):
        ctx.selftest_wait(10)  # below the 1 us floor: refused before a launch
    dec.close()

"""Failure detection of the persistent decode step, driven without a GPU fault.

Every wait of the step kernel is bounded. Two drills, set from the host, make a wait run out
on purpose: one CTA leaves at grid barrier k without arriving (as a CTA that died would), or one
CTA requests none of its expert tiles in a layer (its own ring waits run out). Nothing faults,
traps or hangs: the waits give up after a short limit (20 ms here), the CTA that saw the timeout
poisons the grid barrier, every other CTA leaves at its next barrier, and the call returns
BT_ERR_TIMEOUT after about one limit -- not one limit per remaining barrier. The engine stays
usable: the next steps give the oracle's bits.
"""
import time

import numpy as np
import pytest

import bigtea_b200 as bt
from bigtea_b200 import _lib
from oracle import pyoracle as orc
from tests.conftest import bits

pytestmark = pytest.mark.gpu

LIMIT_US = 20000


def _expect_timeout(runner, cache, tok, n0):
    t0 = time.perf_counter()
    with pytest.raises(bt.BtError) as ex:
        runner.forward_cached(cache, [tok], cache.len())
    dt = time.perf_counter() - t0
    assert ex.value.status == _lib.BT_ERR_TIMEOUT
    assert cache.len() == n0  # the failed step appended nothing
    return dt


@pytest.mark.parametrize("drill,values", [
    ("fault_barrier", (1, 5, 13)),  # QKV->ATTN of layer 0, a mid-layer barrier, the one after the head
    ("fault_copy", (1, 2)),         # expert tiles of layer 0 and layer 1
])
def test_a_failed_wait_ends_the_step_once_and_leaves_the_engine_usable(tiny_cfg, tiny_weights, drill, values):
    e = bt.Engine(tiny_cfg, tiny_weights)
    model = orc.Model(tiny_cfg, tiny_weights)
    try:
        cache = bt.KvCache(e, max_positions=256)
        runner = bt.StreamingRunner(e)
        prompt = np.random.default_rng(61).integers(0, tiny_cfg.n_vocab, 20)
        runner.forward_cached(cache, prompt, 0)
        model.forward(prompt, 0)
        n0 = cache.len()
        # a normal step first, so the timing below has no first-launch cost in it
        tok = 5
        assert np.array_equal(bits(runner.forward_cached(cache, [tok], n0)), bits(model.forward([tok], n0)))
        n0 = cache.len()
        e.set_option("wait_limit_us", LIMIT_US)
        e.set_option("fault_cta", 2)  # a CTA that owns expert units at this size
        # one failed step untimed first: the first pass through the failure path carries one-time
        # costs on a fresh box
        e.set_option(drill, values[-1])
        _expect_timeout(runner, cache, 7, n0)
        for v in values:
            e.set_option(drill, v)
            dt = _expect_timeout(runner, cache, 7, n0)
            # about one limit; without the poisoned barrier every remaining barrier (up to 12
            # of the 13 in this 2-layer step) would wait out its own limit
            assert dt < 6 * LIMIT_US * 1e-6, dt
        e.set_option(drill, 0)
        e.set_option("wait_limit_us", 0)
        for tok in (7, 9):
            got = runner.forward_cached(cache, [tok], cache.len())
            want = model.forward([tok], model.len())
            assert np.array_equal(bits(got), bits(want))
        first = orc.argmax(want)
        toks = runner.generate_greedy(cache, [first], 3)
        assert list(toks[:, 0]) == model.greedy(first, 3)
        cache.close()
    finally:
        model.close()
        e.close()

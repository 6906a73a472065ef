"""GPU: an engine whose experts live in pinned host memory behind a small HBM expert cache gives
the same bits as the oracle (and so as a resident engine): prefill, single-token steps, a
batched step with the experts grouped, and the greedy loop, under both policies. The cache is
far smaller than the experts, so hits, misses, evictions (LRU) and bypasses (frequency gated)
all occur."""
import numpy as np
import pytest

import bigtea_b200 as bt
from oracle import pyoracle as orc
from tests.conftest import bits
from tests.test_gpu_parity import assert_logits, compare_kv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("policy", ["lru", "freq"])
@pytest.mark.parametrize("on_device,persistent", [(1, 1), (1, 0), (0, 1)])
def test_expert_cache_matches_oracle(policy, on_device, persistent):
    """The policy on the device -- inside the persistent step (CTA 0 looks up, every CTA copies
    missed slots) or as lookup and copy kernels between the per-phase kernels -- or on the host
    (per-phase kernels): the oracle's bits every way."""
    cfg = bt.config("tiny", router_zipf=1.1, max_positions=512)
    W = bt.synth_model(cfg, seed=7)
    e = bt.Engine(cfg, W)
    e.set_option("xcache_device", on_device)
    e.set_option("persistent", persistent)
    per_expert = sum(len(W[f"blk.0.{n}.weight"][2]) for n in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"))
    per_expert //= cfg.n_expert
    e.enable_expert_cache(10 * (per_expert + 4096), policy)  # about 10 of the 32 (layer, expert) pairs
    st0 = e.expert_cache_stats()
    assert 8 <= st0["capacity_slots"] <= 12
    model = orc.Model(cfg, W)
    cache = bt.KvCache(e, max_positions=512)
    runner = bt.StreamingRunner(e)
    prompt = np.random.default_rng(31).integers(0, cfg.n_vocab, 21)
    assert_logits(runner.forward_cached(cache, prompt, 0), model.forward(prompt, 0))
    tok = 4
    for _ in range(5):
        assert_logits(runner.forward_cached(cache, [tok], cache.len()), model.forward([tok], model.len()))
        gi, _ = e.debug_topk(1, 0)
        assert np.array_equal(gi, model.topk(1, 0)[0])
        tok = (tok * 13 + 1) % cfg.n_vocab
    toks = runner.generate_greedy(cache, [tok], 6)
    assert list(toks[:, 0]) == model.greedy(tok, 6)
    compare_kv(cache, model, cfg)
    st = e.expert_cache_stats()
    assert st["hits"] > 0 and st["misses"] > 0
    assert st["evictions"] + st["bypasses"] > 0
    assert st["bytes_copied"] >= st["admissions"] * per_expert
    with pytest.raises(bt.BtError):
        e.tensor_bytes("blk.0.ffn_gate_exps.weight", len(W["blk.0.ffn_gate_exps.weight"][2]))
    cache.close()
    e.close()


def test_expert_cache_batched_step_matches_oracle():
    """Twelve sequences in one step (grouped experts, more distinct experts than cache slots)."""
    cfg = bt.config("tiny", router_zipf=1.1, max_positions=1024)
    W = bt.synth_model(cfg, seed=7)
    e = bt.Engine(cfg, W)
    e.enable_expert_cache(2 << 20, "freq")  # about 9 slots against 12 x 4 selections per layer
    rng = np.random.default_rng(44)
    ctxs = [int(c) for c in rng.integers(20, 300, 12)]
    kw = cfg.n_head_kv * cfg.head_dim
    cache = bt.KvCache(e, max_positions=1024, max_seqs=len(ctxs))
    kv = []
    for s, n in enumerate(ctxs):
        layers = []
        for il in range(cfg.n_layer):
            k = (0.5 * rng.standard_normal(n * kw)).astype(np.float16)
            v = rng.standard_normal(n * kw).astype(np.float16)
            cache.restore_layer(il, k, v, seq=s)
            layers.append((k, v))
        cache.set_positions(n, s)
        kv.append(layers)
    toks = [int(t) for t in rng.integers(0, cfg.n_vocab, len(ctxs))]
    got = bt.StreamingRunner(e).forward_batch(cache, list(range(len(ctxs))), [[t] for t in toks], ctxs)
    for s, n in enumerate(ctxs):
        model = orc.Model(cfg, W)
        for il in range(cfg.n_layer):
            model.write_kv_layer(il, kv[s][il][0], kv[s][il][1])
        model.set_len(n)
        want = model.forward([toks[s]], n)
        assert np.array_equal(bits(got[s]), bits(want))
    cache.close()
    e.close()


@pytest.mark.parametrize("policy", ["lru", "freq"])
def test_device_and_host_policies_decide_alike_in_an_engine(policy):
    """The same prefill and decode steps under the device policy and the host policy: the same
    hit, miss, eviction, admission and bypass counts and copied bytes."""
    cfg = bt.config("tiny", router_zipf=1.1, max_positions=512)
    W = bt.synth_model(cfg, seed=9)
    stats = {}
    for on_device in (1, 0):
        e = bt.Engine(cfg, W)
        e.set_option("xcache_device", on_device)  # (1: the persistent step's lookups)
        e.enable_expert_cache(2 << 20, policy)  # about 9 slots
        cache = bt.KvCache(e, max_positions=256, max_seqs=3)
        runner = bt.StreamingRunner(e)
        rng = np.random.default_rng(5)
        runner.forward_batch(cache, [0, 1, 2], [rng.integers(0, cfg.n_vocab, n) for n in (17, 9, 30)], [0, 0, 0])
        runner.generate_greedy(cache, [3, 5, 7], 8, seqs=[0, 1, 2])
        stats[on_device] = e.expert_cache_stats()
        cache.close()
        e.close()
    assert stats[1] == stats[0]
    assert stats[1]["misses"] > 0 and stats[1]["evictions"] + stats[1]["bypasses"] > 0


def _trace(steps, n_layer, n_expert, n_sel, seed):
    """seeded skewed selections with repeats inside a layer's group (several tokens)"""
    rng = np.random.default_rng(seed)
    p = (rng.permutation(n_expert) + 1.0) ** -1.1
    return rng.choice(n_expert, size=(steps, n_layer, n_sel), p=p / p.sum()).astype(np.int32)


@pytest.mark.parametrize("policy", ["lru", "freq"])
@pytest.mark.parametrize("capacity,n_sel", [(6, 12), (16, 8), (60, 8), (200, 24)])
def test_device_policy_equals_host_policy(policy, capacity, n_sel):
    """bt_expert_cache_simulate_device runs the lookup kernel over a trace: every count equals
    the host policy's (which a CPU test pins to a Python restatement), including the cases where
    every slot is pinned by the layer and experts are served from bounce slots."""
    trace = _trace(50, 6, 48, n_sel, seed=capacity + n_sel)
    host = bt.runner.simulate_expert_cache(policy, capacity, trace, n_expert=48)
    dev = bt.runner.simulate_expert_cache(policy, capacity, trace, device=True, n_expert=48)
    assert dev == host
    assert host["misses"] > 0 and host["evictions"] + host["bypasses"] > 0

"""The device sampler (bt_sample, Sampler::sample of core/arch/src/sample.rs:474-680) against the
oracle's restatement, bit for bit: the same token and the same sampler state after every step.

Covers each stage the reference has (logit bias, ignore_eos, infill suppression, the three
penalties, DRY with breakers, top_n_sigma, top_k, typical_p, top_p, min_p, XTC, temperature and
dynamic temperature, mirostat, adaptive-p), reordered and empty chains, ties among logits, several
sequences per call, the engine's own device logits (no host copy) and the full 151,936-entry
vocabulary with no top_k.
"""
import zlib

import numpy as np
import pytest

import bigtea_b200 as bt
from oracle import pyoracle as orc

pytestmark = pytest.mark.gpu

CASES = {
    "greedy": {},
    "llamacpp": dict(base="llamacpp", seed=11),
    "hot_top_k": dict(temperature=1.7, top_k=50, seed=3),
    "top_p_full_vocab": dict(temperature=0.9, top_p=0.9, seed=5),
    "min_p_full_vocab": dict(temperature=1.0, min_p=0.02, seed=6),
    "typical": dict(temperature=0.8, top_k=1500, typical_p=0.7, seed=8),
    "top_n_sigma": dict(temperature=1.0, top_n_sigma=1.5, seed=9),
    "xtc": dict(temperature=1.0, top_k=64, xtc_probability=0.7, xtc_threshold=0.02, seed=10),
    "dynatemp": dict(temperature=0.9, top_k=200, dynatemp_range=0.5, dynatemp_exponent=1.3, seed=12),
    "mirostat": dict(temperature=0.0, mirostat=2, mirostat_tau=4.0, mirostat_eta=0.2, top_k=300, seed=13),
    "adaptive": dict(temperature=1.0, top_k=80, adaptive_p=0.4, adaptive_decay=0.9, seed=14),
    "penalties_dry_bias": dict(temperature=0.7, top_k=100, repeat_penalty=1.3, frequency_penalty=0.2,
                               presence_penalty=0.4, repeat_last_n=32, dry_multiplier=0.9, dry_base=1.75,
                               dry_allowed_length=2, dry_breakers=[5], bias_ids=[3, 17, 3],
                               bias_values=[4.0, -2.0, 1.5], suppress_ids=[0], ignore_eos=1, eos=2, seed=15),
    "penalised_argmax": dict(temperature=0.0, repeat_penalty=1.5, repeat_last_n=16, bias_ids=[9],
                             bias_values=[0.5]),
    "reordered_chain": dict(temperature=2.0, top_p=0.5, top_k=400, chain=[5, 2], seed=16),
    "empty_chain": dict(temperature=1.0, top_k=30, chain=[], seed=17),
}


def _oracle_cfg(kw):
    kw = dict(kw)
    base = kw.pop("base", "default")
    return orc.sampler_config(base, **kw)


def _run_case(engine, kw, logits_fn, n_seqs, steps, rng):
    kw2 = dict(kw)
    base = kw2.pop("base", "default")
    dev = bt.Sampler(engine, n_seqs, base=base, **kw2)
    cfg, keep = _oracle_cfg(kw)
    ost = [orc.sampler_state(cfg) for _ in range(n_seqs)]
    V = engine.cfg.n_vocab
    hists = [list(rng.integers(0, 40, int(rng.integers(0, 50)))) for _ in range(n_seqs)]
    for step in range(steps):
        logits = logits_fn(step)
        got = dev.sample(logits, hists)
        for i in range(n_seqs):
            want = orc.sample(cfg, ost[i], logits[i], hists[i])
            assert int(got[i]) == want, (kw, step, i)
            s = dev.states[i]
            assert s.rng == ost[i].rng
            for f in ("mu", "ap_weighted", "ap_total"):
                assert np.float32(getattr(s, f)).view(np.uint32) == np.float32(getattr(ost[i], f)).view(np.uint32), f
            assert 0 <= int(got[i]) < V
            hists[i].append(int(got[i]))


@pytest.fixture(scope="module")
def engine(tiny_cfg, tiny_weights):
    e = bt.Engine(tiny_cfg, tiny_weights)
    yield e
    e.close()


@pytest.fixture(scope="module")
def wide_engine():
    cfg = bt.config("tiny", n_vocab=151936)
    e = bt.Engine.synthetic(cfg, seed=5)
    yield e
    e.close()


@pytest.mark.parametrize("name", sorted(CASES))
def test_sampler_matches_oracle(engine, name):
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    V = engine.cfg.n_vocab
    n = 3

    def logits(step):
        x = (rng.standard_normal((n, V)) * rng.choice([1.0, 3.0])).astype(np.float32)
        x[1, rng.integers(0, V, 40)] = x[1].max()  # ties at the top
        x[2, 5:20] = x[2, 4]
        return x

    _run_case(engine, CASES[name], logits, n, 4, rng)


@pytest.mark.parametrize("name", ["llamacpp", "top_p_full_vocab", "top_n_sigma", "penalties_dry_bias", "mirostat"])
def test_sampler_full_vocabulary(wide_engine, name):
    rng = np.random.default_rng(7)
    V = wide_engine.cfg.n_vocab

    def logits(step):
        return (rng.standard_normal((2, V)) * 2.5).astype(np.float32)

    _run_case(wide_engine, CASES[name], logits, 2, 2, rng)


def test_sampler_reads_the_engines_own_logits(tiny_cfg, tiny_weights, engine):
    """bt_forward without a host buffer, then bt_sample on the logits left on the device"""
    rng = np.random.default_rng(3)
    cache = bt.KvCache(engine, max_positions=256, max_seqs=2)
    runner = bt.StreamingRunner(engine)
    prompts = [list(rng.integers(0, tiny_cfg.n_vocab, 9)), list(rng.integers(0, tiny_cfg.n_vocab, 5))]
    held = {}

    def logits(step):
        if step == 0:
            x = runner.forward_batch(cache, [0, 1], prompts, [0, 0])
        else:
            x = runner.forward_batch(cache, [0, 1], [[held[0]], [held[1]]], [cache.len(0), cache.len(1)])
        return np.array(x, np.float32).reshape(2, -1)

    kw = CASES["llamacpp"]
    kw2 = dict(kw)
    base = kw2.pop("base")
    dev = bt.Sampler(engine, 2, base=base, **kw2)
    cfg, keep = _oracle_cfg(kw)
    ost = [orc.sampler_state(cfg) for _ in range(2)]
    for step in range(3):
        lg = logits(step)
        got = dev.sample(None, prompts)
        for i in range(2):
            assert int(got[i]) == orc.sample(cfg, ost[i], lg[i], prompts[i])
            held[i] = int(got[i])
            prompts[i] = prompts[i] + [held[i]]
    cache.close()


def test_sampler_errors(engine, wide_engine):
    with pytest.raises(bt.BtError):  # no forward has left logits on this engine's device yet
        bt.Sampler(wide_engine, 1, temperature=1.0).sample(None)
    V = engine.cfg.n_vocab
    lg = np.zeros((1, V), np.float32)
    with pytest.raises(bt.BtError):  # an unknown stage
        bt.Sampler(engine, 1, temperature=1.0, chain=[7]).sample(lg)
    s = bt.Sampler(engine, 1, temperature=1.0, typical_p=0.5)  # typical_p over 1000 tokens: fits
    assert 0 <= int(s.sample(lg)[0]) < V
    wide = np.zeros((1, wide_engine.cfg.n_vocab), np.float32)
    with pytest.raises(bt.BtError):  # typical_p over the whole 151,936-token vocabulary
        bt.Sampler(wide_engine, 1, temperature=1.0, typical_p=0.5).sample(wide)
    # the engine stays usable after the refusal
    assert 0 <= int(bt.Sampler(wide_engine, 1, temperature=1.0, top_k=5, seed=1).sample(wide)[0]) < wide.shape[1]

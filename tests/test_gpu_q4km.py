"""GPU parity on the headline weight mix: the Q4_K_M stand-in of the 48-layer benchmark model.

The benchmark model carries Q6_K `attn_v` and `ffn_down_exps` on even layers (the rest Q4_K),
and its batch-1 steps run the persistent step kernel at G = 8 query heads per KV head. These
tests run that mix through every path the benchmark uses, against the CPU oracle, bit for bit:

- a 4-layer slice of the benchmark shape (hidden 2048, 32/4 heads, 128 experts top-8, expert
  width 768, vocab 151936): prefill through the batched kernels (128-token steps, grouped
  experts, Q6_K down and attn_v), then batch-1 steps through the persistent kernel (G = 8) and
  through the per-phase kernels, past three attention chunks; and a batched single-token step
  of twelve sequences at contexts up to 1500 (grouped experts, warp-pair attention);
- the same on the small shape with the same mix.

Reference: core/arch/src/stream.rs:2265-2474 (q/k/v), 1168-1176 (expert math), 1232-1284
(expert sum), 905-1067 (the block path).
"""
import numpy as np
import pytest

import bigtea_b200 as bt
from bigtea_b200.models import q4km_layer_types
from oracle import pyoracle as orc
from tests.conftest import bits

pytestmark = pytest.mark.gpu


def assert_logits(got, want):
    assert np.abs(got - want).max() <= 1e-2
    assert np.array_equal(bits(got), bits(want))


def compare_kv(cache, model, cfg, seq=0):
    assert cache.len(seq) == model.len()
    for il in range(cfg.n_layer):
        k, v = cache.layer_bytes(il, seq)
        ko, vo = model.kv_layer(il)
        assert np.array_equal(k, ko.view(np.uint8)), f"layer {il} keys"
        assert np.array_equal(v, vo.view(np.uint8)), f"layer {il} values"


@pytest.fixture(scope="module", params=["cfg1_4l", "tiny_q4km"])
def q4km(request):
    if request.param == "cfg1_4l":
        cfg = bt.config("cfg1", n_layer=4, layer_types=q4km_layer_types(4), max_positions=2048)
    else:
        cfg = bt.config("tiny", layer_types=q4km_layer_types(2), max_positions=2048)
    assert cfg.layer_types[0][2] == bt._lib.TYPE_Q6_K and cfg.layer_types[0][6] == bt._lib.TYPE_Q6_K
    return cfg, bt.synth_model(cfg, seed=88)


@pytest.mark.parametrize("persistent", [1, 0])
def test_q4km_prefill_then_single_token_steps(q4km, persistent):
    """Prefill 300 tokens (grouped batched kernels), then greedy and direct single-token steps
    (the persistent kernel, or the per-phase kernels), into a fourth attention chunk."""
    cfg, W = q4km
    e = bt.Engine(cfg, W)
    e.set_option("persistent", persistent)
    model = orc.Model(cfg, W)
    try:
        cache = bt.KvCache(e, max_positions=1024)
        runner = bt.StreamingRunner(e)
        prompt = np.random.default_rng(3).integers(0, cfg.n_vocab, 300)
        want = model.forward(prompt, 0)
        assert_logits(runner.forward_cached(cache, prompt, 0), want)
        for il in range(cfg.n_layer):
            for t in (260, 299):  # the debug hook keeps the last step (256..299)
                gi, gw = e.debug_topk(il, t)
                oi, ow = model.topk(il, t)
                assert np.array_equal(gi, oi) and np.array_equal(bits(gw), bits(ow))
        first = orc.argmax(want)
        toks = runner.generate_greedy(cache, [first], 12)
        assert list(toks[:, 0]) == model.greedy(first, 12)
        tok = int(toks[-1, 0])
        for _ in range(3):
            got = runner.forward_cached(cache, [tok], cache.len())
            want = model.forward([tok], model.len())
            assert_logits(got, want)
            for il in range(cfg.n_layer):
                gi, gw = e.debug_topk(il, 0)
                oi, ow = model.topk(il, 0)
                assert np.array_equal(gi, oi) and np.array_equal(bits(gw), bits(ow))
            assert np.array_equal(bits(e.debug_hidden(0)), bits(model.hidden(0)))
            tok = orc.argmax(want)
        compare_kv(cache, model, cfg)
        cache.close()
    finally:
        model.close()
        e.close()


def test_q4km_long_context_batched_step(q4km):
    """One single-token step of twelve sequences over seeded caches of up to 1500 positions:
    warp-pair attention with the head merge, grouped experts (Q6_K down on even layers)."""
    cfg, W = q4km
    e = bt.Engine(cfg, W)
    rng = np.random.default_rng(17)
    ctxs = [int(c) for c in rng.integers(100, 1500, 12)]
    kw = cfg.n_head_kv * cfg.head_dim
    try:
        cache = bt.KvCache(e, max_positions=2048, max_seqs=len(ctxs))
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
            m = orc.Model(cfg, W)
            for il in range(cfg.n_layer):
                m.write_kv_layer(il, kv[s][il][0], kv[s][il][1])
            m.set_len(n)
            assert_logits(got[s], m.forward([toks[s]], n))
            compare_kv(cache, m, cfg, seq=s)
            m.close()
        cache.close()
    finally:
        e.close()


def test_q4km_persistent_g8_at_long_context(q4km):
    """Batch-1 steps of the persistent kernel over a seeded 1900-position cache (15 attention
    chunks, the head merge in dimension slices) against the oracle."""
    cfg, W = q4km
    e = bt.Engine(cfg, W)
    rng = np.random.default_rng(23)
    n = 1900
    kw = cfg.n_head_kv * cfg.head_dim
    model = orc.Model(cfg, W)
    try:
        cache = bt.KvCache(e, max_positions=2048)
        for il in range(cfg.n_layer):
            k = (0.5 * rng.standard_normal(n * kw)).astype(np.float16)
            v = rng.standard_normal(n * kw).astype(np.float16)
            cache.restore_layer(il, k, v)
            model.write_kv_layer(il, k, v)
        cache.set_positions(n)
        model.set_len(n)
        runner = bt.StreamingRunner(e)
        tok = int(rng.integers(0, cfg.n_vocab))
        want = model.forward([tok], n)
        assert_logits(runner.forward_cached(cache, [tok], n), want)
        first = orc.argmax(want)
        toks = runner.generate_greedy(cache, [first], 6)
        assert list(toks[:, 0]) == model.greedy(first, 6)
        compare_kv(cache, model, cfg)
        cache.close()
    finally:
        model.close()
        e.close()


def test_expert_stream_kernel_matches_per_layer_kernels(q4km):
    """bt_bench_experts kernel 1 (every layer's experts in one persistent kernel, a producer warp
    streaming the tiles) gives the per-layer expert kernels' sums bit for bit, with the Q6_K down
    layers of the mix, at 1, 3 and 4 tokens a layer; the engine stays usable afterwards."""
    cfg, W = q4km
    e = bt.Engine(cfg, W)
    try:
        for T in (1, 3, 4):
            ms0, b0, o0 = e.bench_experts(T, n_iters=2, seed=40 + T, kernel=0, out=True)
            ms1, b1, o1 = e.bench_experts(T, n_iters=2, seed=40 + T, kernel=1, out=True)
            assert ms0 > 0 and ms1 > 0 and b0 == b1
            assert np.abs(o1).max() > 0
            assert np.array_equal(bits(o0), bits(o1)), f"T={T}"
        model = orc.Model(cfg, W)
        cache = bt.KvCache(e, max_positions=64)
        prompt = [3, 1, 4, 1, 5]
        assert_logits(bt.StreamingRunner(e).forward_cached(cache, prompt, 0), model.forward(prompt, 0))
        cache.close()
        model.close()
    finally:
        e.close()


@pytest.mark.parametrize("n_tok", [13, 64, 200])
def test_token_group_gemv_matches_token_chunks(q4km, n_tok):
    """The batched dp4a GEMV over few tiles (the Q6_K attn_v of even layers) splits its tokens
    into groups (option token_groups): prefill logits and cache bytes equal the token-chunk
    launches' bit for bit, and the oracle's, with a ragged last group."""
    cfg, W = q4km
    prompt = np.random.default_rng(50 + n_tok).integers(0, cfg.n_vocab, n_tok)
    outs = []
    for groups in (1, 0):
        e = bt.Engine(cfg, W)
        e.set_option("token_groups", groups)
        try:
            cache = bt.KvCache(e, max_positions=256)
            logits = bt.StreamingRunner(e).forward_cached(cache, prompt, 0)
            kv = [cache.layer_bytes(il) for il in range(cfg.n_layer)]
            outs.append((logits, kv))
            cache.close()
        finally:
            e.close()
    assert np.array_equal(bits(outs[0][0]), bits(outs[1][0]))
    for (k0, v0), (k1, v1) in zip(outs[0][1], outs[1][1]):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
    model = orc.Model(cfg, W)
    try:
        assert_logits(outs[0][0], model.forward(prompt, 0))
    finally:
        model.close()

"""GPU parity: every kernel of the decode layer against the CPU oracle, through the C ABI.

The bar: K-quant dequant, KV-cache bytes and top-k expert ids bit-exact; logits within 1e-2
max-abs after the final norm (the tolerance the path's specification states) -- and, because
both sides implement one arithmetic contract, bit-exact as well, which is asserted too.
"""
import numpy as np
import pytest

import bigtea_b200 as bt
from bigtea_b200 import _lib
from oracle import pyoracle as orc
from tests.conftest import bits

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2


def assert_logits(got, want):
    assert np.abs(got - want).max() <= LOGIT_TOL
    assert np.array_equal(bits(got), bits(want))


# ------------------------------------------------------------------ dequant
def test_dequant_bit_exact_on_golden(golden):
    for ty, key in ((_lib.TYPE_Q4_K, "q4k"), (_lib.TYPE_Q6_K, "q6k")):
        b = golden[key + "_bytes"].reshape(-1)
        want = golden[key + "_values"]
        assert np.array_equal(bits(bt.dequantize(ty, b, want.size)), bits(want))


@pytest.mark.parametrize("ty", [_lib.TYPE_Q4_K, _lib.TYPE_Q6_K])
def test_dequant_bit_exact_on_synthetic(ty):
    w = bt.models.synth_tensor("deq.weight", ty, (2048, 97), 0.0, seed=4)
    n = 2048 * 97
    assert np.array_equal(bits(bt.dequantize(ty, w, n)), bits(orc.dequant(ty, w, n)))


# ------------------------------------------------------------------ GEMV
@pytest.mark.parametrize("ty", [_lib.TYPE_Q4_K, _lib.TYPE_Q6_K])
@pytest.mark.parametrize("rows,cols,T", [(37, 256, 1), (768, 2048, 1), (2048, 768, 3), (2048, 4096, 8),
                                          (130, 512, 9), (1, 2048, 2)])
def test_gemv_bit_exact(ty, rows, cols, T):
    w = bt.models.synth_tensor(f"gemv.{rows}.{cols}", ty, (cols, rows), 0.0, seed=rows + cols)
    x = np.random.default_rng(rows).standard_normal((T, cols)).astype(np.float32)
    x[0, :256] = 0.0  # an all-zero activation block (d = 0)
    got = bt.gemv(ty, w, rows, cols, x)
    want = orc.gemv(ty, w, rows, cols, x)
    assert np.array_equal(bits(got), bits(want))


# ------------------------------------------------------------------ whole forward
@pytest.fixture(scope="module")
def tiny_engine(tiny_cfg, tiny_weights):
    e = bt.Engine(tiny_cfg, tiny_weights)
    yield e
    e.close()


def compare_kv(cache, model, cfg, seq=0):
    n = cache.len(seq)
    assert n == model.len()
    for il in range(cfg.n_layer):
        k, v = cache.layer_bytes(il, seq)
        ko, vo = model.kv_layer(il)
        assert np.array_equal(k, ko.view(np.uint8)), f"layer {il} keys"
        assert np.array_equal(v, vo.view(np.uint8)), f"layer {il} values"


def test_forward_prefill_and_decode_match_oracle(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, cfg.n_vocab, 20)
    model = orc.Model(cfg, tiny_weights)
    cache = bt.KvCache(tiny_engine, max_positions=512)
    runner = bt.StreamingRunner(tiny_engine)
    got = runner.forward_cached(cache, prompt, 0)
    want = model.forward(prompt, 0)
    assert_logits(got, want)
    for il in range(cfg.n_layer):
        for t in (0, 7, 19):
            gi, gw = tiny_engine.debug_topk(il, t)
            oi, ow = model.topk(il, t)
            assert np.array_equal(gi, oi) and np.array_equal(bits(gw), bits(ow))
    assert np.array_equal(bits(tiny_engine.debug_hidden(19)), bits(model.hidden(19)))
    compare_kv(cache, model, cfg)
    tok = int(np.argmax(want))
    for step in range(6):
        got = runner.forward_cached(cache, [tok], cache.len())
        want = model.forward([tok], model.len())
        assert_logits(got, want)
        gi, _ = tiny_engine.debug_topk(1, 0)
        oi, _ = model.topk(1, 0)
        assert np.array_equal(gi, oi)
        tok = orc.argmax(want)
    compare_kv(cache, model, cfg)
    assert cache.is_consistent()


@pytest.mark.parametrize("persistent", [1, 0])
@pytest.mark.parametrize("source", ["tensors", "synthetic"])
def test_router_bias_matches_oracle(persistent, source):
    """A log-Zipf router bias, from the tensor set (blk.N.ffn_gate_inp.bias) or set on a
    synthetic engine: logits, top-k ids and weights of a prefill and greedy steps bit-exact."""
    cfg = bt.config("tiny", router_zipf=1.1)
    W = bt.synth_model(cfg, seed=7)
    e = bt.Engine(cfg, W) if source == "tensors" else bt.Engine.synthetic(cfg, seed=7)
    e.set_option("persistent", persistent)
    model = orc.Model(cfg, W)
    cache = bt.KvCache(e, max_positions=256)
    runner = bt.StreamingRunner(e)
    prompt = np.random.default_rng(29).integers(0, cfg.n_vocab, 13)
    assert_logits(runner.forward_cached(cache, prompt, 0), model.forward(prompt, 0))
    for il in range(cfg.n_layer):
        for t in (0, 12):
            gi, gw = e.debug_topk(il, t)
            oi, ow = model.topk(il, t)
            assert np.array_equal(gi, oi) and np.array_equal(bits(gw), bits(ow))
    tok = 3
    for _ in range(4):
        assert_logits(runner.forward_cached(cache, [tok], cache.len()), model.forward([tok], model.len()))
        gi, _ = e.debug_topk(1, 0)
        assert np.array_equal(gi, model.topk(1, 0)[0])
        tok = (tok * 11 + 5) % cfg.n_vocab
    toks = runner.generate_greedy(cache, [tok], 5)
    assert list(toks[:, 0]) == model.greedy(tok, 5)
    compare_kv(cache, model, cfg)
    cache.close()
    e.close()


def test_long_context_uses_several_attention_chunks(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    prompt = np.random.default_rng(22).integers(0, cfg.n_vocab, 600)
    model = orc.Model(cfg, tiny_weights)
    cache = bt.KvCache(tiny_engine, max_positions=1024)
    runner = bt.StreamingRunner(tiny_engine)
    assert_logits(runner.forward_cached(cache, prompt, 0), model.forward(prompt, 0))
    tok = 5
    for _ in range(3):
        assert_logits(runner.forward_cached(cache, [tok], cache.len()), model.forward([tok], model.len()))
        tok = (tok * 7 + 3) % cfg.n_vocab
    compare_kv(cache, model, cfg)


def test_greedy_graph_loop_matches_oracle(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    prompt = np.random.default_rng(23).integers(0, cfg.n_vocab, 17)
    model = orc.Model(cfg, tiny_weights)
    cache = bt.KvCache(tiny_engine, max_positions=512)
    runner = bt.StreamingRunner(tiny_engine)
    first = orc.argmax(model.forward(prompt, 0))
    runner.forward_cached(cache, prompt, 0)
    toks, logits = runner.generate_greedy(cache, [first], 12, want_logits=True)
    want = model.greedy(first, 12)
    assert list(toks[:, 0]) == want
    compare_kv(cache, model, cfg)
    # the last step's logits are the oracle's for the same position
    last = model.forward([want[-1]], model.len())
    nxt = runner.forward_cached(cache, [want[-1]], cache.len())
    assert_logits(nxt, last)


def test_batched_sequences_match_single_sequence_runs(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    rng = np.random.default_rng(24)
    prompts = [rng.integers(0, cfg.n_vocab, n) for n in (5, 1, 12)]
    cache = bt.KvCache(tiny_engine, max_positions=256, max_seqs=4)
    runner = bt.StreamingRunner(tiny_engine)
    got = runner.forward_batch(cache, [2, 0, 3], prompts, [0, 0, 0])
    for i, p in enumerate(prompts):
        model = orc.Model(cfg, tiny_weights)
        assert_logits(got[i], model.forward(p, 0))
    # one decode step for all three, then against the oracle continued per sequence
    nxt = [int(np.argmax(g)) for g in got]
    got2 = runner.forward_batch(cache, [2, 0, 3], [[t] for t in nxt], [5, 1, 12])
    for i, (p, s) in enumerate(zip(prompts, [2, 0, 3])):
        model = orc.Model(cfg, tiny_weights)
        model.forward(p, 0)
        assert_logits(got2[i], model.forward([nxt[i]], len(p)))
        compare_kv(cache, model, cfg, seq=s)


def test_batched_greedy_matches_per_sequence_oracle(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    rng = np.random.default_rng(25)
    prompts = [rng.integers(0, cfg.n_vocab, n) for n in (3, 9)]
    cache = bt.KvCache(tiny_engine, max_positions=128, max_seqs=2)
    runner = bt.StreamingRunner(tiny_engine)
    lg = runner.forward_batch(cache, [0, 1], prompts, [0, 0])
    first = [orc.argmax(x) for x in lg]
    toks = runner.generate_greedy(cache, first, 8, seqs=[0, 1])
    for i, p in enumerate(prompts):
        model = orc.Model(cfg, tiny_weights)
        model.forward(p, 0)
        assert list(toks[:, i]) == model.greedy(first[i], 8)


# ------------------------------------------------------------------ KvCache semantics on the device pool (kv.rs tests)
def test_kv_truncate_shift_and_restore(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    rng = np.random.default_rng(26)
    prompt = rng.integers(0, cfg.n_vocab, 40)
    cache = bt.KvCache(tiny_engine, max_positions=256)
    runner = bt.StreamingRunner(tiny_engine)
    runner.forward_cached(cache, prompt, 0)
    k0, v0 = cache.layer_bytes(0)
    per = cfg.n_head_kv * cfg.head_dim * 2
    # shift_out(keep=4, drop=10): positions 0..3 stay, 14.. slide down to 4..
    cache.shift_out(4, 10)
    assert cache.len() == 30 and cache.is_consistent()
    k1, v1 = cache.layer_bytes(0)
    assert np.array_equal(k1[:4 * per], k0[:4 * per])
    assert np.array_equal(k1[4 * per:], k0[14 * per:])
    assert np.array_equal(v1[4 * per:], v0[14 * per:])
    # a decode step over the shifted cache equals the oracle given the same cache
    model = orc.Model(cfg, tiny_weights)
    for il in range(cfg.n_layer):
        k, v = cache.layer_bytes(il)
        model.write_kv_layer(il, k, v)
    model.set_len(30)
    assert_logits(runner.forward_cached(cache, [11], 30), model.forward([11], 30))
    # shifting more than there is clamps; shifting nothing is a no-op
    cache.shift_out(28, 100)
    assert cache.len() == 28
    before = cache.keys(0)
    cache.shift_out(0, 0)
    cache.shift_out(50, 3)
    assert np.array_equal(cache.keys(0), before)
    # truncate_to keeps a prefix; a larger n is a no-op
    cache.truncate_to(10)
    assert cache.len() == 10 and np.array_equal(cache.keys(0), before[:10 * per])
    cache.truncate_to(99)
    assert cache.len() == 10
    # restore_layer + set_positions (the prompt cache path); a ragged length is refused
    for il in range(cfg.n_layer):
        cache.restore_layer(il, *(x[:10 * per] for x in model.kv_layer(il, 10)))
    cache.set_positions(10)
    assert cache.is_consistent()
    with pytest.raises(bt.BtError):
        cache.restore_layer(0, np.zeros(per + 2, np.uint8), np.zeros(per + 2, np.uint8))
    cache.clear()
    assert cache.is_empty() and cache.bytes() == 0


def test_errors_leave_the_engine_usable(tiny_cfg, tiny_weights, tiny_engine):
    cfg = tiny_cfg
    cache = bt.KvCache(tiny_engine, max_positions=64)
    runner = bt.StreamingRunner(tiny_engine)
    with pytest.raises(bt.BtError) as e:
        runner.forward_cached(cache, [cfg.n_vocab + 5], 0)
    assert e.value.status == _lib.BT_ERR_INVALID
    with pytest.raises(bt.BtError) as e:
        runner.forward_cached(cache, [1, 2], 3)
    assert e.value.status == _lib.BT_ERR_KV
    with pytest.raises(bt.BtError):
        runner.forward_cached(cache, list(range(65)), 0)
    model = orc.Model(cfg, tiny_weights)
    assert_logits(runner.forward_cached(cache, [1, 2, 3], 0), model.forward([1, 2, 3], 0))


# ------------------------------------------------------------------ the reference's CPU-runnable workload
def test_cfg0_prefill_128_then_64_greedy_steps():
    """qwen3moe, 2 layers at Qwen3-30B-A3B dims, Q4_K weights with Q6_K embedding/output:
    128-token prefill of uniform-random ids, then 64 greedy steps (the reference's cfg0)."""
    cfg = bt.config("cfg0")
    W = bt.synth_model(cfg, seed=2024)
    prompt = np.random.default_rng(2024).integers(0, cfg.n_vocab, 128)
    model = orc.Model(cfg, W)
    want0 = model.forward(prompt, 0)
    e = bt.Engine(cfg, W)
    try:
        cache = bt.KvCache(e, max_positions=256)
        runner = bt.StreamingRunner(e)
        got0 = runner.forward_cached(cache, prompt, 0)
        assert_logits(got0, want0)
        for il in range(cfg.n_layer):
            for t in (3, 64, 100, 127):  # the debug hooks keep the last step: the whole prompt
                gi, gw = e.debug_topk(il, t)
                oi, ow = model.topk(il, t)
                assert np.array_equal(gi, oi) and np.array_equal(bits(gw), bits(ow))
        with pytest.raises(bt.BtError):
            e.debug_topk(0, 128)
        first = orc.argmax(want0)
        toks = runner.generate_greedy(cache, [first], 64)
        want = model.greedy(first, 64)
        assert list(toks[:, 0]) == want
        compare_kv(cache, model, cfg)
        # the same 64 steps twice more from the prefilled cache: the grid barrier's ordering of
        # each phase's inputs is exercised 64 x 15 times per run, so a missed ordering would show
        # as a repeatable mismatch rather than a rare one
        for _ in range(2):
            cache.truncate_to(128)
            toks = runner.generate_greedy(cache, [first], 64)
            assert list(toks[:, 0]) == want
            compare_kv(cache, model, cfg)
    finally:
        e.close()


# ------------------------------------------------------------------ the persistent step against the per-phase kernels
@pytest.mark.parametrize("shape", ["tiny", "tiny_sh"])
def test_persistent_and_per_phase_steps_agree(tiny_cfg, tiny_weights, shape):
    """Single-token steps run as one cooperative kernel by default; the per-phase kernels
    are the other implementation of the same contract. Both must equal the oracle (with and
    without a shared expert)."""
    if shape == "tiny":
        cfg, weights = tiny_cfg, tiny_weights
    else:
        cfg = bt.config("tiny_sh", max_positions=1024)
        weights = bt.synth_model(cfg, seed=8)
    prompt = np.random.default_rng(31).integers(0, cfg.n_vocab, 300)  # three attention chunks
    runs = {}
    for persistent in (1, 0):
        e = bt.Engine(cfg, weights)
        e.set_option("persistent", persistent)
        cache = bt.KvCache(e, max_positions=512, max_seqs=3)
        runner = bt.StreamingRunner(e)
        runner.forward_batch(cache, [0, 2], [prompt, prompt[:50]], [0, 0])
        toks = runner.generate_greedy(cache, [7, 9], 5, seqs=[0, 2])
        lg = runner.forward_batch(cache, [0, 2], [[11], [12]], [305, 55])
        runs[persistent] = (toks, lg, [cache.layer_bytes(il, 0) for il in range(cfg.n_layer)])
        e.close()
    assert np.array_equal(runs[0][0], runs[1][0])
    assert np.array_equal(bits(runs[0][1]), bits(runs[1][1]))
    for a, b in zip(runs[0][2], runs[1][2]):
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    model = orc.Model(cfg, weights)
    model.forward(prompt, 0)
    assert list(runs[1][0][:, 0]) == model.greedy(7, 5)


@pytest.mark.parametrize("persistent,ctxs", [
    (1, (2900, 450, 1700)),
    (0, (2900, 450, 1700, 3000, 300, 1290)),
    (0, tuple(int(c) for c in np.random.default_rng(5).integers(130, 2200, 40))),
])
def test_long_context_batched_step_matches_oracle(tiny_cfg, tiny_weights, persistent, ctxs):
    """One single-token step of several sequences whose cached contexts span many attention
    chunks (seeded cache contents): the step's logits and its KV append against the oracle run
    per sequence. Three sequences run as the persistent kernel, six as the per-phase kernels,
    forty as the per-phase kernels with the experts grouped (more than 8 tokens in the step)."""
    cfg = bt.config("tiny", max_positions=4096)
    rng = np.random.default_rng(41 + persistent)
    kw = cfg.n_head_kv * cfg.head_dim
    e = bt.Engine(cfg, tiny_weights)
    e.set_option("persistent", persistent)
    cache = bt.KvCache(e, max_positions=4096, max_seqs=len(ctxs))
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
    runner = bt.StreamingRunner(e)
    got = runner.forward_batch(cache, list(range(len(ctxs))), [[t] for t in toks], list(ctxs))
    for s, n in enumerate(ctxs):
        model = orc.Model(cfg, tiny_weights)
        for il in range(cfg.n_layer):
            model.write_kv_layer(il, kv[s][il][0], kv[s][il][1])
        model.set_len(n)
        assert_logits(got[s], model.forward([toks[s]], n))
        compare_kv(cache, model, cfg, seq=s)
    cache.close()
    e.close()


@pytest.mark.parametrize("n_head", [4, 12, 16])  # GQA groups of 2, 6 and 8 query heads
def test_batched_step_gqa_groups_match_oracle(n_head):
    """A batched single-token step (per-phase attention, grouped experts) for each group size the
    attention kernel is built for: paired heads (2, 8 per kv head -> 1, 4 per thread) and the
    one-head-at-a-time path (6 -> 3 per thread)."""
    cfg = bt.config("tiny", n_head=n_head, max_positions=2048)
    W = bt.synth_model(cfg, seed=5)
    e = bt.Engine(cfg, W)
    rng = np.random.default_rng(n_head)
    ctxs = [int(c) for c in rng.integers(50, 700, 10)]
    kw = cfg.n_head_kv * cfg.head_dim
    cache = bt.KvCache(e, max_positions=2048, max_seqs=len(ctxs))
    kv = []
    for s_, n in enumerate(ctxs):
        layers = []
        for il in range(cfg.n_layer):
            k = (0.5 * rng.standard_normal(n * kw)).astype(np.float16)
            v = rng.standard_normal(n * kw).astype(np.float16)
            cache.restore_layer(il, k, v, seq=s_)
            layers.append((k, v))
        cache.set_positions(n, s_)
        kv.append(layers)
    toks = [int(t) for t in rng.integers(0, cfg.n_vocab, len(ctxs))]
    got = bt.StreamingRunner(e).forward_batch(cache, list(range(len(ctxs))), [[t] for t in toks], ctxs)
    for s_, n in enumerate(ctxs):
        model = orc.Model(cfg, W)
        for il in range(cfg.n_layer):
            model.write_kv_layer(il, kv[s_][il][0], kv[s_][il][1])
        model.set_len(n)
        assert_logits(got[s_], model.forward([toks[s_]], n))
        compare_kv(cache, model, cfg, seq=s_)
    cache.close()
    e.close()


@pytest.mark.parametrize("source,persistent", [("tensors", 1), ("tensors", 0), ("synthetic", 1)])
def test_shared_expert_matches_oracle(source, persistent):
    """A model with a shared expert (DeepSeek-style, added unweighted to the routed sum): a
    prefill, single-token steps (the persistent kernel, whose down units carry the shared
    expert as one more expert, or the per-phase kernels), the greedy loop and a 12-sequence
    batched step (grouped experts) give the oracle's bits."""
    cfg = bt.config("tiny_sh", max_positions=1024)
    W = bt.synth_model(cfg, seed=7)
    e = bt.Engine(cfg, W) if source == "tensors" else bt.Engine.synthetic(cfg, seed=7)
    e.set_option("persistent", persistent)
    model = orc.Model(cfg, W)
    cache = bt.KvCache(e, max_positions=512)
    runner = bt.StreamingRunner(e)
    prompt = np.random.default_rng(33).integers(0, cfg.n_vocab, 19)
    assert_logits(runner.forward_cached(cache, prompt, 0), model.forward(prompt, 0))
    tok = 9
    for _ in range(3):
        assert_logits(runner.forward_cached(cache, [tok], cache.len()), model.forward([tok], model.len()))
        tok = (tok * 17 + 2) % cfg.n_vocab
    toks = runner.generate_greedy(cache, [tok], 4)
    assert list(toks[:, 0]) == model.greedy(tok, 4)
    compare_kv(cache, model, cfg)
    cache.close()
    rng = np.random.default_rng(34)
    ctxs = [int(c) for c in rng.integers(20, 400, 12)]
    kw = cfg.n_head_kv * cfg.head_dim
    cache = bt.KvCache(e, max_positions=512, max_seqs=len(ctxs))
    kv = []
    for s_, n in enumerate(ctxs):
        layers = []
        for il in range(cfg.n_layer):
            k = (0.5 * rng.standard_normal(n * kw)).astype(np.float16)
            v = rng.standard_normal(n * kw).astype(np.float16)
            cache.restore_layer(il, k, v, seq=s_)
            layers.append((k, v))
        cache.set_positions(n, s_)
        kv.append(layers)
    toks = [int(t) for t in rng.integers(0, cfg.n_vocab, len(ctxs))]
    got = runner.forward_batch(cache, list(range(len(ctxs))), [[t] for t in toks], ctxs)
    for s_, n in enumerate(ctxs):
        m2 = orc.Model(cfg, W)
        for il in range(cfg.n_layer):
            m2.write_kv_layer(il, kv[s_][il][0], kv[s_][il][1])
        m2.set_len(n)
        assert_logits(got[s_], m2.forward([toks[s_]], n))
    cache.close()
    e.close()


def test_warp_attention_matches_cta_attention_and_oracle(tiny_cfg, tiny_weights):
    """Batched attention with one warp per 128-key chunk gives the per-CTA kernel's bits and the
    oracle's: 40 sequences whose contexts cover one-chunk finalisation, partial 32-key pieces,
    a last page of one key and up to 63 chunks (the combine): enough chunk groups that every
    CTA walks several and its warps prefetch across their items."""
    cfg = bt.config("tiny", max_positions=8192)
    rng = np.random.default_rng(57)
    ctxs = [1, 15, 16, 17, 31, 32, 33, 127, 128, 129, 255, 256, 257, 511, 700] + \
        [int(c) for c in rng.integers(1, 8000, 25)]
    kw = cfg.n_head_kv * cfg.head_dim
    kv = [[((0.5 * rng.standard_normal(n * kw)).astype(np.float16), rng.standard_normal(n * kw).astype(np.float16))
           for _ in range(cfg.n_layer)] for n in ctxs]
    toks = [int(t) for t in rng.integers(0, cfg.n_vocab, len(ctxs))]
    outs = {}
    for mode in (1, 0):
        e = bt.Engine(cfg, tiny_weights)
        e.set_option("attn_warp", mode)
        cache = bt.KvCache(e, max_positions=8192, max_seqs=len(ctxs))
        for s_, n in enumerate(ctxs):
            for il in range(cfg.n_layer):
                cache.restore_layer(il, kv[s_][il][0], kv[s_][il][1], seq=s_)
            cache.set_positions(n, s_)
        runner = bt.StreamingRunner(e)
        outs[mode] = runner.forward_batch(cache, list(range(len(ctxs))), [[t] for t in toks], ctxs)
        cache.close()
        e.close()
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    for s_ in (0, 3, 7, 9, 14, 15, 20):
        m2 = orc.Model(cfg, tiny_weights)
        for il in range(cfg.n_layer):
            m2.write_kv_layer(il, kv[s_][il][0], kv[s_][il][1])
        m2.set_len(ctxs[s_])
        assert_logits(outs[1][s_], m2.forward([toks[s_]], ctxs[s_]))


def test_tensor_core_gemv_matches_dp4a_and_oracle():
    """The batched GEMVs on tcgen05 give the dp4a kernels' bits and the oracle's: q/k/v at
    K = 512 (32-token units) and attn_output at K = 4096 (32 heads of 128: 16-token units), on a
    4-CTA grid so every CTA streams many (token chunk, row block) units, and gate/up many chunks,
    through its weight ring (prefetch across units and chunks)."""
    cfg = bt.config("tiny", n_head=32, n_head_kv=4)
    W = bt.synth_model(cfg, seed=11)
    rng = np.random.default_rng(56)
    prompt = rng.integers(0, cfg.n_vocab, 100)
    outs = {}
    for mode in ("mma", "dp4a"):
        e = bt.Engine(cfg, W)
        if mode == "mma":
            e.set_option("mma_min_units", 1)
            e.set_option("mma_grid", 4)
        else:
            e.set_option("mma", 0)
        cache = bt.KvCache(e, max_positions=256, max_seqs=40)
        runner = bt.StreamingRunner(e)
        lg = runner.forward_batch(cache, [0], [prompt], [0])
        steps = runner.forward_batch(cache, list(range(1, 40)), [[int(t)] for t in prompt[:39]], [0] * 39)
        outs[mode] = (lg, steps, cache.layer_bytes(1, 0))
        cache.close()
        e.close()
    assert np.array_equal(bits(outs["mma"][0]), bits(outs["dp4a"][0]))
    assert np.array_equal(bits(outs["mma"][1]), bits(outs["dp4a"][1]))
    assert np.array_equal(outs["mma"][2][0], outs["dp4a"][2][0])
    assert np.array_equal(outs["mma"][2][1], outs["dp4a"][2][1])
    model = orc.Model(cfg, W)
    assert_logits(outs["mma"][0][0], model.forward(list(prompt), 0))
    for i in (0, 17, 38):
        m1 = orc.Model(cfg, W)
        assert_logits(outs["mma"][1][i], m1.forward([int(prompt[i])], 0))


@pytest.mark.parametrize("grid", [4, 0])
def test_tensor_core_q6k_gemv_and_head_match_dp4a_and_oracle(grid):
    """Q6_K on tcgen05 (two MMAs per 32-value K step against zero-padded halves of the
    activations, one per 16-value sub-block): q/k/v all Q6_K (K = 512), and the Q6_K output head
    with its argmax keys at more than 8 outputs, give the dp4a kernels' bits and the oracle's --
    a 100-token prefill, a 40-sequence step, then 3 greedy steps of the 40 sequences (the head's
    keys pick the tokens). grid 4: every CTA streams many (token chunk, row block) units."""
    types = [[bt._lib.TYPE_Q6_K] * 3 + [bt._lib.TYPE_Q4_K] * 4] * 2
    cfg = bt.config("tiny", n_head=32, n_head_kv=4, n_vocab=1024, layer_types=types)
    W = bt.synth_model(cfg, seed=12)
    rng = np.random.default_rng(57)
    prompt = rng.integers(0, cfg.n_vocab, 100)
    outs = {}
    for mode in ("mma", "dp4a"):
        e = bt.Engine(cfg, W)
        if mode == "mma":
            e.set_option("mma_min_units", 1)
            e.set_option("mma_grid", grid)
        else:
            e.set_option("mma", 0)
        cache = bt.KvCache(e, max_positions=256, max_seqs=41)
        runner = bt.StreamingRunner(e)
        lg = runner.forward_batch(cache, [0], [prompt], [0])
        steps = runner.forward_batch(cache, list(range(1, 41)), [[int(t)] for t in prompt[:40]], [0] * 40)
        first = [int(np.argmax(steps[i])) for i in range(40)]
        toks = runner.generate_greedy(cache, first, 3, seqs=list(range(1, 41)))
        outs[mode] = (lg, steps, toks, cache.layer_bytes(1, 0))
        cache.close()
        e.close()
    assert np.array_equal(bits(outs["mma"][0]), bits(outs["dp4a"][0]))
    assert np.array_equal(bits(outs["mma"][1]), bits(outs["dp4a"][1]))
    assert np.array_equal(outs["mma"][2], outs["dp4a"][2])
    assert np.array_equal(outs["mma"][3][0], outs["dp4a"][3][0])
    assert np.array_equal(outs["mma"][3][1], outs["dp4a"][3][1])
    model = orc.Model(cfg, W)
    assert_logits(outs["mma"][0][0], model.forward(list(prompt), 0))
    model.close()
    for i in (0, 21, 39):
        m1 = orc.Model(cfg, W)
        want = m1.forward([int(prompt[i])], 0)
        assert_logits(outs["mma"][1][i], want)
        assert list(outs["mma"][2][:, i]) == m1.greedy(orc.argmax(want), 3)
        m1.close()


def test_tensor_core_gateup_matches_dp4a_kernel(tiny_cfg, tiny_weights):
    """The grouped gate/up on tcgen05 (int8 MMA per K-quant sub-block, integer-exact) and the
    dp4a grouped kernel give the same bits: a 70-token prefill step and a 24-sequence step."""
    rng = np.random.default_rng(55)
    prompt = rng.integers(0, tiny_cfg.n_vocab, 70)
    outs = {}
    for mma in (1, 0):
        e = bt.Engine(tiny_cfg, tiny_weights)
        e.set_option("mma", mma)
        cache = bt.KvCache(e, max_positions=512, max_seqs=24)
        runner = bt.StreamingRunner(e)
        lg = runner.forward_batch(cache, [0], [prompt], [0])
        steps = runner.forward_batch(cache, list(range(1, 24)), [[int(t)] for t in prompt[:23]], [0] * 23)
        outs[mma] = (lg, steps, cache.layer_bytes(1, 0))
        cache.close()
        e.close()
    assert np.array_equal(bits(outs[0][0]), bits(outs[1][0]))
    assert np.array_equal(bits(outs[0][1]), bits(outs[1][1]))
    assert np.array_equal(outs[0][2][0], outs[1][2][0]) and np.array_equal(outs[0][2][1], outs[1][2][1])



def test_isolated_expert_timing_reports_the_selected_bytes(tiny_cfg, tiny_weights):
    """bt_bench_experts: the routed experts' kernels over every layer at 1 and 24 tokens a layer
    report a positive device time and the distinct selected experts' bytes (K distinct experts at
    one token: exactly K per layer), and leave the engine usable."""
    e = bt.Engine(tiny_cfg, tiny_weights)
    per_expert = sum(bt.gguf.tensor_nbytes(tiny_cfg.layer_types[0][i], tiny_cfg.n_embd * tiny_cfg.n_ff_exp)
                     for i in (4, 5, 6))
    ms1, b1 = e.bench_experts(1, n_iters=3)
    assert ms1 > 0 and b1 == tiny_cfg.n_layer * tiny_cfg.n_expert_used * per_expert
    ms24, b24 = e.bench_experts(24, n_iters=3)
    assert ms24 > 0 and b1 < b24 <= tiny_cfg.n_layer * tiny_cfg.n_expert * per_expert
    model = orc.Model(tiny_cfg, tiny_weights)
    cache = bt.KvCache(e, max_positions=64)
    prompt = [3, 1, 4, 1, 5]
    assert_logits(bt.StreamingRunner(e).forward_cached(cache, prompt, 0), model.forward(prompt, 0))
    cache.close()
    model.close()
    e.close()


@pytest.mark.parametrize("down_type", ["q4", "q6"])
def test_tensor_core_down_at_wide_experts(down_type):
    """The grouped down on tcgen05 at an expert width of 2048 (8 superblocks per row, as the
    DeepSeek-style shape has) gives the dp4a kernel's bits and the oracle's: a 40-token prefill
    step and a 20-sequence step, with Q4_K or Q6_K down matrices."""
    dt = bt._lib.TYPE_Q4_K if down_type == "q4" else bt._lib.TYPE_Q6_K
    types = [[bt._lib.TYPE_Q4_K] * 6 + [dt]] * 2
    cfg = bt.config("tiny", n_ff_exp=2048, layer_types=types)
    W = bt.synth_model(cfg, seed=13)
    prompt = np.random.default_rng(58).integers(0, cfg.n_vocab, 40)
    outs = {}
    for mma in (1, 0):
        e = bt.Engine(cfg, W)
        e.set_option("mma", mma)
        cache = bt.KvCache(e, max_positions=128, max_seqs=21)
        runner = bt.StreamingRunner(e)
        lg = runner.forward_batch(cache, [0], [prompt], [0])
        steps = runner.forward_batch(cache, list(range(1, 21)), [[int(t)] for t in prompt[:20]], [0] * 20)
        outs[mma] = (lg, steps)
        cache.close()
        e.close()
    assert np.array_equal(bits(outs[1][0]), bits(outs[0][0]))
    assert np.array_equal(bits(outs[1][1]), bits(outs[0][1]))
    model = orc.Model(cfg, W)
    try:
        assert_logits(outs[1][0][0], model.forward(list(prompt), 0))
    finally:
        model.close()


def test_forward_into_page_locked_logits(tiny_cfg, tiny_weights):
    """bt_forward into a bt_host_alloc buffer (the logits copied straight into it) gives the bits a
    pageable buffer gets, for single-token and batched calls, and a wrong-shaped buffer is refused."""
    e = bt.Engine(tiny_cfg, tiny_weights)
    try:
        outs = []
        for pinned in (False, True):
            cache = bt.KvCache(e, max_positions=128, max_seqs=12)
            runner = bt.StreamingRunner(e)
            buf1 = bt.pinned_empty((1, tiny_cfg.n_vocab)) if pinned else None
            bufb = bt.pinned_empty((12, tiny_cfg.n_vocab)) if pinned else None
            a = runner.forward_cached(cache, [3, 1, 4, 1, 5], 0, out=buf1).copy()
            b = runner.forward_cached(cache, [9], 5, out=buf1).copy()
            c = runner.forward_batch(cache, list(range(1, 12)), [[t] for t in range(11)], [0] * 11,
                                     out=None if bufb is None else bufb[:11]).copy()
            outs.append((a, b, c))
            cache.close()
        for x, y in zip(outs[0], outs[1]):
            assert np.array_equal(bits(x), bits(y))
        with pytest.raises(ValueError):
            bt.StreamingRunner(e).forward_cached(None, [1], 0, out=bt.pinned_empty((2, tiny_cfg.n_vocab)))
    finally:
        e.close()

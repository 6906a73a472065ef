"""CPU tests of the oracle: pinned against gguf-py golden vectors, hand-built known answers,
independent numpy restatements, and the reference's own routing / sampling tests."""
import math

import numpy as np
import pytest

from oracle import pyoracle as orc
from tests.conftest import bits

QK = 256


# ------------------------------------------------------------------ K-quant dequant
def test_dequant_matches_gguf_py_golden(golden):
    for ty, key in ((orc.OR_Q4_K, "q4k"), (orc.OR_Q6_K, "q6k")):
        b = golden[key + "_bytes"]
        want = golden[key + "_values"]
        got = orc.dequant(ty, b.reshape(-1), want.size)
        assert np.array_equal(bits(got), bits(want)), key


def _pack_q4k(d, dmin, sc, m, q):
    """Build one block_q4_K from its fields (the inverse of get_scale_min_k4)."""
    b = np.zeros(144, np.uint8)
    b[0:2] = np.array([d], np.float16).view(np.uint8)
    b[2:4] = np.array([dmin], np.float16).view(np.uint8)
    s = np.zeros(12, np.uint8)
    for j in range(4):
        s[j] = (sc[j] & 63) | ((sc[j + 4] >> 4) << 6)
        s[j + 4] = (m[j] & 63) | ((m[j + 4] >> 4) << 6)
        s[j + 8] = (sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4)
    b[4:16] = s
    for g in range(4):
        for l in range(32):
            b[16 + 32 * g + l] = q[64 * g + l] | (q[64 * g + 32 + l] << 4)
    return b


def test_q4k_known_answer():
    # x = d*sc*q - dmin*m with exactly representable values
    sc = np.array([1, 2, 3, 63, 17, 32, 48, 5])
    m = np.array([0, 1, 63, 2, 40, 7, 9, 33])
    q = np.arange(256) % 16
    blk = _pack_q4k(0.5, 0.25, sc, m, q)
    got = orc.dequant(orc.OR_Q4_K, blk, 256)
    want = np.array([0.5 * sc[i // 32] * q[i] - 0.25 * m[i // 32] for i in range(256)], np.float32)
    assert np.array_equal(got, want)


def test_q6k_known_answer():
    rng = np.random.default_rng(3)
    L = rng.integers(0, 64, 256)
    sc = rng.integers(-128, 128, 16).astype(np.int8)
    b = np.zeros(210, np.uint8)
    for n in range(2):
        for l in range(32):
            L1, L2, L3, L4 = L[128 * n + l], L[128 * n + 32 + l], L[128 * n + 64 + l], L[128 * n + 96 + l]
            b[64 * n + l] = (L1 & 0xF) | ((L3 & 0xF) << 4)
            b[64 * n + 32 + l] = (L2 & 0xF) | ((L4 & 0xF) << 4)
            b[128 + 32 * n + l] = (L1 >> 4) | ((L2 >> 4) << 2) | ((L3 >> 4) << 4) | ((L4 >> 4) << 6)
    b[192:208] = sc.view(np.uint8)
    b[208:210] = np.array([0.125], np.float16).view(np.uint8)
    got = orc.dequant(orc.OR_Q6_K, b, 256)
    want = np.array([np.float32(0.125 * sc[i // 16]) * np.float32(L[i] - 32) for i in range(256)], np.float32)
    assert np.array_equal(got, want)


def test_partial_block_is_refused():
    with pytest.raises(ValueError):
        orc.dequant(orc.OR_Q4_K, np.zeros(144, np.uint8), 200)


# ------------------------------------------------------------------ Q8_K activations
def q8k_numpy(x):
    """Independent restatement of ggml's quantize_row_q8_K (C3)."""
    out = []
    for b in range(x.size // QK):
        xb = x[QK * b:QK * (b + 1)].astype(np.float32)
        ax = np.abs(xb)
        if ax.max() == 0:
            out.append((np.float32(0), np.zeros(QK, np.int8)))
            continue
        mx = xb[int(np.argmax(ax))]  # first occurrence of the largest |x|
        iscale = np.float32(-127.0) / mx
        q = np.minimum(127, np.rint(iscale * xb).astype(np.int32)).astype(np.int8)
        out.append((np.float32(1.0) / iscale, q))
    return out


def test_q8k_matches_numpy_restatement():
    rng = np.random.default_rng(11)
    x = rng.standard_normal(4 * QK).astype(np.float32)
    x[QK:2 * QK] = 0.0
    x[2 * QK + 5] = 3.0
    x[2 * QK + 9] = -3.0  # a tie in |x|: the first one sets the sign of the scale
    d, qs, bs = orc.quantize_q8k(x)
    for b, (dw, qw) in enumerate(q8k_numpy(x)):
        assert bits(d[b]) == bits(dw)
        assert np.array_equal(qs[b], qw)
        assert np.array_equal(bs[b], qw.astype(np.int32).reshape(16, 16).sum(1))
    assert d[2] < 0  # max taken from the positive first occurrence, iscale = -127/3


# ------------------------------------------------------------------ GEMV contract
def q4k_fields(blk):
    d = np.frombuffer(blk[0:2].tobytes(), np.float16)[0].astype(np.float32)
    dmin = np.frombuffer(blk[2:4].tobytes(), np.float16)[0].astype(np.float32)
    s = blk[4:16].astype(np.int32)
    sc, m = np.zeros(8, np.int32), np.zeros(8, np.int32)
    for j in range(8):
        if j < 4:
            sc[j], m[j] = s[j] & 63, s[j + 4] & 63
        else:
            sc[j] = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4)
            m[j] = (s[j + 4] >> 4) | ((s[j] >> 6) << 4)
    qs = blk[16:144]
    q = np.zeros(256, np.int32)
    for g in range(4):
        q[64 * g:64 * g + 32] = qs[32 * g:32 * g + 32] & 0xF
        q[64 * g + 32:64 * g + 64] = qs[32 * g:32 * g + 32] >> 4
    return d, dmin, sc, m, q


def gemv_q4k_numpy(w, rows, cols, x):
    """Independent numpy restatement of contract C4 for Q4_K."""
    nsb = cols // QK
    acts = q8k_numpy(x)
    y = np.zeros(rows, np.float32)
    for r in range(rows):
        acc = np.float32(0.0)
        for b in range(nsb):
            blk = w[(r * nsb + b) * 144:(r * nsb + b + 1) * 144]
            d, dmin, sc, m, q = q4k_fields(blk)
            dx, a = acts[b]
            a = a.astype(np.int32)
            sumi = int(sum(sc[j] * int(np.dot(q[32 * j:32 * j + 32], a[32 * j:32 * j + 32])) for j in range(8)))
            summ = int(sum(m[j] * int(a[32 * j:32 * j + 32].sum()) for j in range(8)))
            sb = np.float32(np.float32(sumi) * np.float32(d * dx)) - np.float32(np.float32(summ) * np.float32(dmin * dx))
            acc = np.float32(acc + sb)
        y[r] = acc
    return y


def test_gemv_q4k_matches_numpy_restatement():
    import bigtea_b200 as bt

    rows, cols = 6, 768
    w = bt.models.synth_tensor("probe.w", bt.models.TYPE_Q4_K, (cols, rows), 0.0, seed=5)
    x = np.random.default_rng(2).standard_normal(cols).astype(np.float32)
    got = orc.gemv(orc.OR_Q4_K, w, rows, cols, x)[0]
    want = gemv_q4k_numpy(w, rows, cols, x)
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("ty", [orc.OR_Q4_K, orc.OR_Q6_K])
def test_gemv_tracks_float64_dot(ty):
    import bigtea_b200 as bt

    rows, cols = 64, 2048
    w = bt.models.synth_tensor("probe.w2", ty, (cols, rows), 0.0, seed=9)
    x = np.random.default_rng(4).standard_normal(cols).astype(np.float32)
    got = orc.gemv(ty, w, rows, cols, x)[0].astype(np.float64)
    wf = orc.dequant(ty, w, rows * cols).reshape(rows, cols).astype(np.float64)
    want = wf @ x.astype(np.float64)
    # Q8_K activations carry about 0.4% relative error per block
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-2


# ------------------------------------------------------------------ scalar contract pieces
@pytest.mark.parametrize("ty", [12, 14])
def test_simd_kquant_dots_equal_the_plain_dots(ty):
    """or_gemv's AVX2 integer dots (unsigned weights times signed Q8_K values, widened and
    scaled in int32) give the plain C dots' bits: the integer sums are exact and the float
    combination is the same code. Wide value ranges, several shapes, a zero activation block."""
    import ctypes as C
    L = orc.lib()
    L.or_gemv_scalar_dots.restype = C.c_int
    L.or_gemv_scalar_dots.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.POINTER(C.c_float),
                                      C.POINTER(C.c_float)]
    rng = np.random.default_rng(90 + ty)
    for rows, cols, seed in ((768, 2048, 1), (2048, 768, 2), (37, 4096, 3), (5, 256, 4)):
        w = orc.synth_tensor("x", ty, (cols, rows), 0.0, seed, sigma=0.3)
        for trial in range(3):
            x = (rng.standard_normal(cols) * (10 ** rng.uniform(-3, 3))).astype(np.float32)
            if trial == 2:
                x[:256] = 0.0
            y1 = orc.gemv(ty, w, rows, cols, x).reshape(-1)
            y2 = np.empty(rows, np.float32)
            assert L.or_gemv_scalar_dots(ty, w.ctypes.data, rows, cols, x.ctypes.data_as(C.POINTER(C.c_float)),
                                         y2.ctypes.data_as(C.POINTER(C.c_float))) == 0
            assert np.array_equal(bits(y1), bits(y2)), (rows, cols, trial)


def test_exp_error_bound():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-87, 88.7, 20000), rng.uniform(-2, 2, 20000), [0.0, -1e-30, 1e-30]])
    worst = 0.0
    for x in xs.astype(np.float32):
        got, ref = orc.exp(float(x)), math.exp(float(x))
        worst = max(worst, abs(got - ref) / float(np.spacing(np.float32(ref))))
    assert worst <= 2.0
    assert orc.exp(0.0) == 1.0
    assert orc.exp(float("-inf")) == 0.0
    assert math.isinf(orc.exp(100.0))


def test_f16_rounding_is_round_to_nearest_even():
    rng = np.random.default_rng(1)
    raw = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    raw = raw[np.isfinite(raw)]
    with np.errstate(over="ignore"):
        want = raw.astype(np.float16).view(np.uint16)
    got = np.array([orc.f32_to_f16(float(v)) for v in raw], np.uint16)
    assert np.array_equal(got, want)


def test_softmax_sums_to_one_and_tracks_float64():
    x = np.random.default_rng(3).standard_normal(128).astype(np.float32)
    p = orc.softmax(x)
    ref = np.exp(x.astype(np.float64) - x.max())
    ref /= ref.sum()
    assert abs(p.sum() - 1) < 1e-5
    assert np.abs(p - ref).max() < 1e-6


# ------------------------------------------------------------------ route() and argmax (stream.rs:3067-3105, sample.rs:928)
def test_routing_picks_the_highest_scoring_experts():
    ids, _ = orc.route([0.1, 0.5, 0.2, 0.9], 2)
    assert list(ids) == [3, 1]


def test_routing_weights_are_renormalised_over_the_selection():
    _, w = orc.route([0.1, 0.5, 0.2, 0.9], 2)
    assert abs(w.sum() - 1.0) < 1e-6


def test_zero_probabilities_do_not_divide_by_zero():
    ids, w = orc.route([0.0, 0.0, 0.0, 0.0], 2)
    assert len(ids) == 2 and np.all(np.isfinite(w))
    assert list(ids) == [0, 1]  # stable sort keeps the original order of ties


def test_routing_ties_keep_the_lower_index_first():
    ids, _ = orc.route([0.25, 0.5, 0.25, 0.5, 0.1], 3)
    assert list(ids) == [1, 3, 0]


def test_argmax_last_maximum_wins():
    assert orc.argmax([1.0, 3.0, 2.0, 3.0, 0.5]) == 3
    assert orc.argmax([0.0, -0.0]) == 0  # total_cmp: -0.0 < +0.0
    assert orc.argmax([-0.0, 0.0]) == 1


# ------------------------------------------------------------------ attention (C8) against float64
def test_attention_head_tracks_float64():
    rng = np.random.default_rng(8)
    D, nk = 128, 700  # three chunks, the last one partial
    q = rng.standard_normal(D).astype(np.float32)
    k = rng.standard_normal((nk, D)).astype(np.float16)
    v = rng.standard_normal((nk, D)).astype(np.float16)
    scale = 1 / math.sqrt(D)
    got = orc.attn_head(q, k.view(np.uint16), v.view(np.uint16), nk, scale)
    qh = q.astype(np.float16).astype(np.float64)
    s = (k.astype(np.float64) @ qh) * scale
    p = np.exp(s - s.max())
    want = (p / p.sum()) @ v.astype(np.float64)
    assert np.abs(got - want).max() < 1e-5


# ------------------------------------------------------------------ whole model
def _f64_forward(cfg, W, tokens):
    """A float64 numpy restatement of the qwen3moe forward (no Q8_K, no f16 cache rounding
    except where the cache stores f16) for a whole prompt; logits of the last token."""
    E, H, HK, D = cfg.n_embd, cfg.n_head, cfg.n_head_kv, cfg.head_dim
    F, K = cfg.n_ff_exp, cfg.n_expert_used

    def deq(name, rows, cols):
        ty, ne, data = W[name]
        if ty == 0:
            return np.frombuffer(data.tobytes(), np.float32).astype(np.float64).reshape(rows, cols)
        return orc.dequant(ty, data, rows * cols).astype(np.float64).reshape(rows, cols)

    def vec(name):
        return np.frombuffer(W[name][2].tobytes(), np.float32).astype(np.float64)

    def rms(x, w):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + cfg.rms_eps) * w

    T = len(tokens)
    emb = deq("token_embd.weight", cfg.n_vocab, E)
    x = emb[tokens]
    pos = np.arange(T)
    inv = cfg.rope_freq_base ** (-np.arange(0, D, 2) / D)
    ang = pos[:, None] * inv[None, :]
    cos, sin = np.cos(ang), np.sin(ang)

    def rope(h):  # h [T, n, D]
        a, b = h[..., :D // 2], h[..., D // 2:]
        c, s = cos[:, None, :], sin[:, None, :]
        return np.concatenate([a * c - b * s, a * s + b * c], -1)

    for il in range(cfg.n_layer):
        p = f"blk.{il}."
        xn = rms(x, vec(p + "attn_norm.weight"))
        q = (xn @ deq(p + "attn_q.weight", H * D, E).T).reshape(T, H, D)
        k = (xn @ deq(p + "attn_k.weight", HK * D, E).T).reshape(T, HK, D)
        v = (xn @ deq(p + "attn_v.weight", HK * D, E).T).reshape(T, HK, D)
        q = rope(rms(q, vec(p + "attn_q_norm.weight")))
        k = rope(rms(k, vec(p + "attn_k_norm.weight")))
        att = np.zeros((T, H, D))
        for h in range(H):
            g = h // (H // HK)
            s = q[:, h] @ k[:, g].T / math.sqrt(D)
            s = np.where(np.tril(np.ones((T, T))) > 0, s, -np.inf)
            pm = np.exp(s - s.max(-1, keepdims=True))
            att[:, h] = (pm / pm.sum(-1, keepdims=True)) @ v[:, g]
        x = x + att.reshape(T, H * D) @ deq(p + "attn_output.weight", E, H * D).T
        fn = rms(x, vec(p + "ffn_norm.weight"))
        logits = fn @ deq(p + "ffn_gate_inp.weight", cfg.n_expert, E).T
        if p + "ffn_gate_inp.bias" in W:
            logits = logits + vec(p + "ffn_gate_inp.bias")
        pr = np.exp(logits - logits.max(-1, keepdims=True))
        pr /= pr.sum(-1, keepdims=True)
        out = np.zeros_like(x)
        for t in range(T):
            sel = np.argsort(-pr[t], kind="stable")[:K]
            w = pr[t, sel] / pr[t, sel].sum()
            for e, we in zip(sel, w):
                ty, ne, data = W[p + "ffn_gate_exps.weight"]
                per = len(data) // cfg.n_expert
                gw = orc.dequant(ty, data[e * per:(e + 1) * per], F * E).astype(np.float64).reshape(F, E)
                ty, ne, data = W[p + "ffn_up_exps.weight"]
                uw = orc.dequant(ty, data[e * per:(e + 1) * per], F * E).astype(np.float64).reshape(F, E)
                ty, ne, data = W[p + "ffn_down_exps.weight"]
                per_d = len(data) // cfg.n_expert
                dw = orc.dequant(ty, data[e * per_d:(e + 1) * per_d], E * F).astype(np.float64).reshape(E, F)
                g_ = gw @ fn[t]
                a = g_ / (1 + np.exp(-g_)) * (uw @ fn[t])
                out[t] += we * (dw @ a)
            if p + "ffn_gate_shexp.weight" in W:  # the shared expert, unweighted
                FS = cfg.n_ff_shexp
                g_ = deq(p + "ffn_gate_shexp.weight", FS, E) @ fn[t]
                a = g_ / (1 + np.exp(-g_)) * (deq(p + "ffn_up_shexp.weight", FS, E) @ fn[t])
                out[t] += deq(p + "ffn_down_shexp.weight", E, FS) @ a
        x = x + out
    xn = rms(x[-1], vec("output_norm.weight"))
    return xn @ deq("output.weight", cfg.n_vocab, E).T


def test_forward_tracks_float64_restatement(tiny_cfg, tiny_weights):
    tokens = np.random.default_rng(5).integers(0, tiny_cfg.n_vocab, 12)
    m = orc.Model(tiny_cfg, tiny_weights)
    got = m.forward(tokens, 0).astype(np.float64)
    want = _f64_forward(tiny_cfg, tiny_weights, tokens)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel < 0.05, rel  # Q8_K activations and the f16 cache are the only differences


def test_router_bias_forward_tracks_float64_restatement_and_skews_routing():
    import bigtea_b200 as bt

    cfg = bt.config("tiny", router_zipf=1.1)
    W = bt.synth_model(cfg, seed=7)
    b0 = np.frombuffer(W["blk.0.ffn_gate_inp.bias"][2].tobytes(), np.float32)
    assert np.array_equal(b0, bt.models.zipf_router_bias(cfg.n_expert, 0, 7, 1.1))
    assert sorted(np.round(np.exp(-b0 / 1.1)).astype(int)) == list(range(1, cfg.n_expert + 1))
    tokens = np.random.default_rng(8).integers(0, cfg.n_vocab, 40)
    m = orc.Model(cfg, W)
    got = m.forward(tokens, 0).astype(np.float64)
    want = _f64_forward(cfg, W, tokens)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 0.05
    # the experts the bias favours are the ones picked most: rank-1 expert in most top-k sets
    top = int(np.argmax(b0))
    hits = sum(top in m.topk(0, t)[0] for t in range(len(tokens)))
    assert hits >= len(tokens) // 2, hits


def test_shared_expert_forward_tracks_float64_restatement():
    import bigtea_b200 as bt

    cfg = bt.config("tiny_sh")
    W = bt.synth_model(cfg, seed=7)
    assert W["blk.1.ffn_down_shexp.weight"][1] == (cfg.n_ff_shexp, cfg.n_embd)
    tokens = np.random.default_rng(12).integers(0, cfg.n_vocab, 10)
    got = orc.Model(cfg, W).forward(tokens, 0).astype(np.float64)
    want = _f64_forward(cfg, W, tokens)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 0.05
    # and the shared expert matters: without it the logits move
    W2 = {k: v for k, v in W.items() if "shexp" not in k}
    cfg2 = bt.config("tiny_sh", n_ff_shexp=0)
    other = orc.Model(cfg2, W2).forward(tokens, 0).astype(np.float64)
    assert np.abs(other - got).max() > 1e-3


def test_block_prefill_and_token_steps_share_layer0_kv(tiny_cfg, tiny_weights):
    tokens = np.random.default_rng(6).integers(0, tiny_cfg.n_vocab, 9)
    a = orc.Model(tiny_cfg, tiny_weights)
    a.forward(tokens, 0)
    b = orc.Model(tiny_cfg, tiny_weights)
    for i, t in enumerate(tokens):
        b.forward([t], i)
    ka, va = a.kv_layer(0)
    kb, vb = b.kv_layer(0)
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_forward_refuses_a_wrong_position(tiny_cfg, tiny_weights):
    m = orc.Model(tiny_cfg, tiny_weights)
    with pytest.raises(ValueError):
        m.forward([1, 2], 3)


@pytest.mark.parametrize("ty,ne,mean", [(orc.OR_Q4_K, (2048, 96), 0.0), (orc.OR_Q6_K, (768, 40), 0.0),
                                        (orc.OR_F32, (2048,), 1.0), (orc.OR_F32, (1000, 3), 0.0),
                                        (orc.OR_F16, (300,), 0.5)])
def test_oracle_synthetic_weights_equal_the_libraries(ty, ne, mean):
    """The CPU arm builds its model with the oracle's generator (it never loads the product
    library); the bytes must be the product generator's for the same seed and tensor name."""
    import bigtea_b200 as bt

    name = f"blk.3.synth_check_{ty}.weight"
    got = orc.synth_tensor(name, ty, ne, mean, seed=77)
    want = bt.models.synth_tensor(name, ty, ne, mean, seed=77)
    assert got.dtype == np.uint8 and np.array_equal(got, want)


@pytest.mark.parametrize("name", ["cfg0", "cfg1"])
def test_cpu_arm_workloads_equal_the_products(name):
    """The CPU arm's description of the benchmark models (oracle/workloads.py) has the product's
    hyper-parameters and exactly its tensor list, types, dims and means."""
    import bigtea_b200 as bt
    from oracle import workloads

    w = workloads.workload(name)
    c = bt.config(name)
    for f in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_expert", "n_expert_used", "n_ff_exp",
              "n_vocab", "rms_eps", "rope_freq_base", "expert_workers", "max_positions", "embd_type", "out_type",
              "layer_types"):
        assert getattr(w, f) == getattr(c, f), f
    assert w.tensor_specs() == c.tensor_specs()

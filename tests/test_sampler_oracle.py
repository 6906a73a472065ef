"""The sampler oracle (oracle/sample.c) against the reference's own sampler tests and a second,
independent restatement.

- The cases of core/arch/src/sample.rs:1072-1380 (`mod tests`), restated on the oracle's stage
  functions and Sampler::sample, with the reference's inputs and assertions.
- SplitMix64 against its published first outputs from state 0.
- S5 ln and S6 pow against float64 libm within a few ulp.
- A Python restatement of Sampler::sample (sample.rs:474-680), written separately from the C one
  and sharing only the exp/ln/pow primitives, on random logits, histories and configurations:
  the two must return the same token and the same sampler state, bit for bit.
"""
import ctypes as C
import math
import os

import numpy as np
import pytest

from oracle import pyoracle as orc

F = np.float32
LOGITS = [0.0, 2.0, -1.0, 5.0, 1.0]  # sample.rs:1074-1076: token 3 best, 1 second


def run(cfg_kw, logits, n, history=(), base="default"):
    cfg, keep = orc.sampler_config(base, **cfg_kw)
    st = orc.sampler_state(cfg)
    return [orc.sample(cfg, st, logits, history) for _ in range(n)]


# ----------------------------------------------------------------- the reference's tests
def test_the_default_is_exactly_the_old_greedy_behaviour():
    assert run({}, LOGITS, 10) == [3] * 10


def test_the_same_seed_reproduces_the_same_sequence():
    a = run(dict(temperature=1.0, seed=42), LOGITS, 32)
    assert a == run(dict(temperature=1.0, seed=42), LOGITS, 32)
    assert a != run(dict(temperature=1.0, seed=43), LOGITS, 32)


def test_top_k_one_is_greedy_however_hot_the_temperature():
    assert run(dict(temperature=5.0, top_k=1), LOGITS, 32) == [3] * 32


def test_temperature_widens_the_distribution():
    cold = run(dict(temperature=0.1, seed=7), LOGITS, 400).count(3)
    hot = run(dict(temperature=3.0, seed=7), LOGITS, 400).count(3)
    assert cold > 380 and hot < cold


def test_top_p_keeps_a_prefix_and_min_p_scales_with_confidence():
    c = orc.stage("top_p", [(0, 0.6), (1, 0.3), (2, 0.07), (3, 0.03)], 0.9)
    assert len(c) == 2 and abs(sum(x[1] for x in c) - 1.0) < 1e-5
    assert len(orc.stage("min_p", [(0, 0.9), (1, 0.06), (2, 0.04)], 0.1)) == 1
    assert len(orc.stage("min_p", [(0, 0.3), (1, 0.28), (2, 0.24), (3, 0.18)], 0.1)) == 4


def test_a_filter_never_empties_the_candidate_list():
    c = orc.stage("top_p", [(9, 1.0)], 0.0)
    assert c == [(9, 1.0)]
    assert len(orc.stage("min_p", [(9, 0.5), (1, 0.5)], 1.5)) == 1


def test_the_repeat_penalty_pushes_a_token_down_whatever_its_sign():
    c = orc.stage_penalties([(0, 4.0), (1, -4.0)], [0, 1], 2.0, 0.0, 0.0, 64)
    assert c[0][1] == 2.0 and c[1][1] == -8.0


def test_ordering_temperature_before_top_p_changes_the_result():
    lg = [4.0, 3.0, 2.0, 1.0, 0.0]
    after = set(run(dict(temperature=2.0, top_p=0.5, chain=[orc.STAGE_TOP_P, orc.STAGE_TEMPERATURE], seed=5), lg, 200))
    before = set(run(dict(temperature=2.0, top_p=0.5, chain=[orc.STAGE_TEMPERATURE, orc.STAGE_TOP_P], seed=5), lg, 200))
    assert after != before


def test_an_empty_chain_still_samples_rather_than_panicking():
    assert run(dict(temperature=1.0, chain=[], seed=3), [1.0, 2.0, 3.0], 1)[0] < 3


def test_dry_penalises_the_token_that_continues_a_repeat():
    c = orc.stage_dry([(1, 0.0), (2, 0.0), (3, 0.0), (4, 0.0)], [1, 2, 3, 1, 2], 1.0, 2.0, 2, 0)
    assert c[2][1] == -1.0 and c[0][1] == 0.0 and c[3][1] == 0.0


def test_dry_grows_with_the_length_of_the_repeat():
    assert orc.stage_dry([(3, 0.0)], [1, 2, 3, 1, 2], 1.0, 3.0, 2, 0)[0][1] == -1.0
    assert orc.stage_dry([(4, 0.0)], [8, 1, 2, 3, 4, 9, 1, 2, 3], 1.0, 3.0, 2, 0)[0][1] == -3.0
    assert orc.stage_dry([(4, 0.0)], [9, 1, 2, 3, 4, 9, 1, 2, 3], 1.0, 3.0, 2, 0)[0][1] == -9.0


def test_dry_respects_allowed_length_and_being_off():
    assert orc.stage_dry([(3, 0.0)], [1, 2, 3, 1, 2], 1.0, 2.0, 3, 0)[0][1] == 0.0
    assert orc.stage_dry([(3, 0.0)], [1, 2, 3, 1, 2], 0.0, 2.0, 2, 0)[0][1] == 0.0


def test_a_sequence_breaker_stops_a_match_spanning_it():
    assert orc.stage_dry([(3, 0.0)], [1, 2, 3, 1, 2], 1.0, 2.0, 2, 0, [2])[0][1] == 0.0


def test_dry_takes_the_largest_penalty_not_the_sum():
    assert orc.stage_dry([(3, 0.0)], [1, 2, 3, 1, 2, 3, 1, 2], 1.0, 2.0, 2, 0)[0][1] >= -8.0


def test_top_n_sigma_cuts_by_logit_spread():
    c = orc.stage("top_n_sigma", [(0, 10.0), (1, 9.8), (2, 9.6), (3, 9.4), (4, -5.0)], 1.0)
    assert len(c) == 4 and all(x[0] != 4 for x in c)
    assert len(orc.stage("top_n_sigma", [(0, 10.0), (4, -5.0)], 0.0)) == 2


def test_xtc_removes_the_likely_tokens_not_the_unlikely_ones():
    c = orc.stage("xtc", [(0, 0.5), (1, 0.3), (2, 0.15), (3, 0.05)], 1.0, 0.1, 0.0)
    assert c[0][0] == 2 and len(c) == 2


def test_xtc_does_nothing_when_the_roll_fails_or_only_one_token_qualifies():
    before = [(0, 0.9), (1, 0.05), (2, 0.05)]
    f32 = [(i, float(F(v))) for i, v in before]
    assert orc.stage("xtc", before, 0.5, 0.1, 0.9) == f32
    assert orc.stage("xtc", before, 1.0, 0.1, 0.0) == f32


def test_dynamic_temperature_is_high_when_the_model_is_unsure():
    hot = orc.dynamic_temperature([(0, 0.25), (1, 0.25), (2, 0.25), (3, 0.25)], 1.0, 0.5, 1.0)
    cold = orc.dynamic_temperature([(0, 0.97), (1, 0.01), (2, 0.01), (3, 0.01)], 1.0, 0.5, 1.0)
    assert hot > cold and abs(hot - 1.5) < 1e-3 and cold < 0.8


# ----------------------------------------------------------------- known answers and primitives
def test_splitmix64_published_outputs():
    """Vigna's SplitMix64 from state 0 gives 0xe220a8397b1dcdaf, 0x6e789e6aa1b965f4,
    0x06c45d188009454f; next_f32 keeps the top 24 bits."""
    st = orc.SamplerState()
    st.rng = 0
    got = [orc.lib().or_sampler_next_f32(st) for _ in range(3)]
    want = [(z >> 40) / 2.0**24 for z in (0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F)]
    assert got == want
    cfg, _ = orc.sampler_config(seed=0)
    assert orc.sampler_state(cfg).rng == 0x9E3779B97F4A7C15  # Sampler::new: seed + the golden gamma


def _ulps(a, b):
    return abs(np.float32(a).view(np.int32).astype(np.int64) - np.float32(b).view(np.int32).astype(np.int64))


def test_ln_and_pow_agree_with_libm_within_a_few_ulp():
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.uniform(1e-30, 1.0, 2000), rng.uniform(0.5, 2.0, 2000),
                         np.exp(rng.uniform(-80, 80, 2000)), [1e-45, 1e-40, 1.0, 2.0, 0.5]]).astype(np.float32)
    worst = 0
    for x in xs:
        want = np.float32(math.log(float(x)))
        got = orc.ln(float(x))
        if abs(float(want)) > 1e-3:
            worst = max(worst, _ulps(got, want))
        else:
            assert abs(got - float(want)) < 2e-7
    assert worst <= 2, worst
    assert orc.ln(0.0) == -math.inf and math.isnan(orc.ln(-1.0)) and orc.ln(1.0) == 0.0
    for x, y in zip(rng.uniform(1e-6, 1.0, 2000).astype(np.float32), rng.uniform(0.1, 10.0, 2000).astype(np.float32)):
        want = float(x) ** float(y)
        if want > 1e-30:
            assert abs(orc.pow_(float(x), float(y)) - want) <= 4e-6 * want
    assert orc.pow_(2.0, -10.0) == 2.0**-10 and orc.pow_(0.0, 2.0) == 0.0 and orc.pow_(1.0, 7.5) == 1.0


# ----------------------------------------------------------------- a second restatement
def _key(v):
    u = int(np.float32(v).view(np.uint32))
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def _exp(x):
    return F(orc.exp(float(x)))


def _ln(x):
    return F(orc.ln(float(x)))


def _pow(x, y):
    return F(orc.pow_(float(x), float(y)))


def _sum(vals):
    t = F(0.0)
    for v in vals:
        t = F(t + v)
    return t


def _fmax(a, b):
    """f32::max: NaN gives way to the other operand"""
    return F(np.fmax(F(a), F(b)))


def _clamp(v, lo, hi):
    v = F(v)
    if v < lo:
        v = F(lo)
    if v > hi:
        v = F(hi)
    return v


class PySampler:
    """Sampler (sample.rs:306-680) over lists of (id, np.float32), with the restatement's tie
    rules, each statement in float32."""

    def __init__(self, c):
        self.c = c
        self.rng = (c["seed"] + 0x9E3779B97F4A7C15) & (2**64 - 1)
        decay = _clamp(c["adaptive_decay"], 0.0, 0.99)
        self.apw = F(_fmax(c["adaptive_p"], 0.0) / F(F(1.0) - decay))
        self.apt = F(F(1.0) / F(F(1.0) - decay))
        self.mu = F(F(2.0) * F(c["mirostat_tau"]))

    def next(self):
        M = 2**64 - 1
        self.rng = (self.rng + 0x9E3779B97F4A7C15) & M
        z = self.rng
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        z ^= z >> 31
        return F((z >> 40) / 16777216.0)

    @staticmethod
    def softmax(c):
        if not c:
            return c
        mx = c[0][1]
        e = [(i, _exp(F(v - mx))) for i, v in c]
        tot = _sum(v for _, v in e)
        return [(i, F(v / tot)) for i, v in e] if tot > 0 else e

    @staticmethod
    def renorm(c):
        tot = _sum(v for _, v in c)
        return [(i, F(v / tot)) for i, v in c] if tot > 0 else c

    @staticmethod
    def temperature(c, t):
        if abs(F(F(t) - F(1.0))) <= np.finfo(np.float32).eps:
            return c
        inv = F(F(1.0) / _fmax(t, 1e-6))
        c = [(i, _pow(v, inv)) for i, v in c]
        return PySampler.renorm(c)

    @staticmethod
    def entropy(c):
        return F(-_sum(F(v * _ln(v)) for _, v in c if v > 0))

    def draw(self, c):
        r = self.next()
        acc = F(0.0)
        for k, (i, p) in enumerate(c):
            acc = F(acc + p)
            if r < acc:
                return k
        return len(c) - 1

    def sample(self, logits, hist):
        c = self.c
        greedy = (c["temperature"] <= 0 and c["repeat_penalty"] == 1 and c["frequency_penalty"] == 0
                  and c["presence_penalty"] == 0 and not c["bias"] and c["mirostat"] == 0
                  and not c["ignore_eos"] and not c["suppress"]
                  and c["dry_multiplier"] == 0 and c["adaptive_p"] < 0)
        lg = [F(x) for x in logits]
        if greedy:
            return max(range(len(lg)), key=lambda i: (_key(lg[i]), i))
        v = list(lg)
        for i, b in c["bias"]:
            v[i] = F(v[i] + F(b))
        if c["ignore_eos"] and 0 <= c["eos"] < len(v):
            v[c["eos"]] = F(-np.inf)
        for i in c["suppress"]:
            v[i] = F(-np.inf)
        # penalties (sample.rs:967-1008)
        if c["repeat_last_n"] and hist:
            w = hist[-c["repeat_last_n"]:]
            for t in sorted(set(w)):
                n = w.count(t)
                if c["repeat_penalty"] != 1:
                    rp = F(c["repeat_penalty"])
                    v[t] = F(v[t] / rp) if v[t] > 0 else F(v[t] * rp)
                v[t] = F(v[t] - F(F(F(n) * F(c["frequency_penalty"])) + F(c["presence_penalty"])))
        # DRY (sample.rs:682-753)
        if c["dry_multiplier"] > 0 and len(hist) >= 2:
            w = hist if c["dry_last_n"] == 0 or c["dry_last_n"] >= len(hist) else hist[-c["dry_last_n"]:]
            br = set(c["breakers"])
            n = len(w)
            if n >= 2 and w[-1] not in br:
                pen = {}
                for i in range(n - 1):
                    if w[i] != w[-1]:
                        continue
                    ln_ = 1
                    while ln_ <= i and ln_ < n and w[i - ln_] == w[n - 1 - ln_] and w[i - ln_] not in br:
                        ln_ += 1
                    if ln_ < c["dry_allowed"]:
                        continue
                    a, k, r = F(c["dry_base"]), ln_ - c["dry_allowed"], F(1.0)
                    while True:
                        if k & 1:
                            r = F(r * a)
                        k >>= 1
                        if not k:
                            break
                        a = F(a * a)
                    p = F(F(c["dry_multiplier"]) * r)
                    if p > pen.get(w[i + 1], F(0.0)):
                        pen[w[i + 1]] = p
                for t, p in pen.items():
                    v[t] = F(v[t] - p)
        if c["temperature"] <= 0 and c["mirostat"] == 0 and c["adaptive_p"] < 0:
            return max(range(len(v)), key=lambda i: (_key(v[i]), i))
        cand = sorted(((i, v[i]) for i in range(len(v))), key=lambda t: (-_key(t[1]), t[0]))
        if c["top_n_sigma"] > 0 and len(cand) >= 2:  # sample.rs:820-857
            mx = F(-np.inf)
            for _, x in cand:
                mx = F(np.fmax(mx, x))
            fin = [x for _, x in cand if np.isfinite(x)]
            if np.isfinite(mx) and len(fin) >= 2:
                mean = F(_sum(fin) / F(len(fin)))
                var = F(_sum(F(F(x - mean) * F(x - mean)) for x in fin) / F(len(fin)))
                sigma = F(np.sqrt(var))
                if sigma > 0:
                    fl = F(mx - F(F(c["top_n_sigma"]) * sigma))
                    cand = [t for t in cand if t[1] >= fl]
        if c["top_k"] > 0:
            cand = cand[:c["top_k"]]
        cand = self.softmax(cand)
        if c["mirostat"] > 0:
            cut = _pow(F(2.0), F(-self.mu))
            kept = max(sum(1 for _, p in cand if p >= cut), 1)
            cand = self.temperature(cand[:kept], c["temperature"] if c["temperature"] > 0 else 1.0)
            k = self.draw(cand)
            p = cand[k][1]
            obs = F(-F(_ln(_fmax(p, 1e-30)) * F(1.44269502162933349609375)))
            self.mu = F(self.mu - F(F(c["mirostat_eta"]) * F(obs - F(c["mirostat_tau"]))))
            self.mu = _clamp(self.mu, 0.0, 100.0)
            return cand[k][0]
        for s in c["chain"]:
            if s == orc.STAGE_TOP_K and c["top_k"] > 0:
                cand = cand[:c["top_k"]]
            elif s == orc.STAGE_TOP_P and c["top_p"] < 1:
                acc, keep = F(0.0), len(cand)
                for k, (_, p) in enumerate(cand):
                    acc = F(acc + p)
                    if acc >= F(c["top_p"]):
                        keep = k + 1
                        break
                cand = self.renorm(cand[:max(keep, 1)])
            elif s == orc.STAGE_MIN_P and c["min_p"] > 0 and cand:
                fl = F(F(c["min_p"]) * cand[0][1])
                keep = 0
                while keep < len(cand) and cand[keep][1] >= fl:
                    keep += 1
                cand = self.renorm(cand[:max(keep, 1)])
            elif s == orc.STAGE_TYPICAL_P and c["typical_p"] < 1 and len(cand) >= 2:
                h = self.entropy(cand)
                sc = sorted(range(len(cand)),
                            key=lambda k: (_key(abs(F(-_ln(_fmax(cand[k][1], 1e-30)) - h))), k))
                cum, keep = F(0.0), 0
                for k in sc:
                    cum = F(cum + cand[k][1])
                    keep += 1
                    if cum >= F(c["typical_p"]):
                        break
                cand = [cand[k] for k in sorted(sc[:keep], key=lambda k: (-_key(cand[k][1]), k))]
            elif s == orc.STAGE_XTC and c["xtc_probability"] > 0:
                roll = self.next()
                if roll < F(c["xtc_probability"]) and len(cand) >= 2:
                    above = 0
                    while above < len(cand) and cand[above][1] >= F(c["xtc_threshold"]):
                        above += 1
                    if above >= 2:
                        cand = cand[above - 1:]
            elif s == orc.STAGE_TEMPERATURE:
                t = F(c["temperature"])
                if c["dynatemp_range"] > 0 and len(cand) >= 2:  # sample.rs:878-915
                    lo = _fmax(F(t - F(c["dynatemp_range"])), 0.0)
                    hi = F(t + F(c["dynatemp_range"]))
                    h = self.entropy(cand)
                    hmax = _ln(F(len(cand)))
                    if hmax > 0:
                        nrm = _clamp(F(h / hmax), 0.0, 1.0)
                        t = F(lo + F(F(hi - lo) * _pow(nrm, _fmax(c["dynatemp_exponent"], 1e-6))))
                cand = self.temperature(cand, t)
        if c["adaptive_p"] >= 0:  # sample.rs:374-419
            target = _clamp(c["adaptive_p"], 0.0, 1.0)
            mean = target if self.apt == 0 else F(self.apw / self.apt)
            adapted = _clamp(F(F(2.0) * target) - mean, 0.0, 1.0)
            orig = [p for _, p in cand]
            t = []
            for i, p in cand:
                d = abs(F(F(p - adapted) / F(0.3)))
                t.append((i, F(F(5.0) - F(F(F(F(10.0) * d) * d) / F(F(1.0) + d)))))
            cand = self.softmax(t)
            k = max(self.draw(cand), 0)
            decay = _clamp(c["adaptive_decay"], 0.0, 0.99)
            self.apw = F(orig[k] + F(decay * self.apw))
            self.apt = F(F(1.0) + F(decay * self.apt))
            return cand[k][0]
        return cand[self.draw(cand)][0]


def _random_case(rng):
    nv = int(rng.choice([5, 37, 300, 2000]))
    logits = (rng.standard_normal(nv) * rng.choice([0.5, 2.0, 6.0])).astype(np.float32)
    if rng.random() < 0.3:  # ties
        logits[rng.integers(0, nv, nv // 3)] = logits[0]
    if rng.random() < 0.15:  # infinities and NaN among the logits
        logits[rng.integers(0, nv, 2)] = rng.choice([np.inf, -np.inf, np.nan])
    hist = [int(t) for t in rng.integers(0, min(nv, 12), int(rng.integers(0, 40)))]
    chain = list(rng.permutation(6)[: int(rng.integers(0, 7))]) if rng.random() < 0.4 else [0, 1, 2, 3, 4, 5]
    c = dict(temperature=float(rng.choice([0.0, 0.3, 0.8, 1.0, 1.7])), top_k=int(rng.choice([0, 1, 5, 40])),
             top_p=float(rng.choice([1.0, 0.95, 0.5])), min_p=float(rng.choice([0.0, 0.05, 0.2])),
             typical_p=float(rng.choice([1.0, 0.9, 0.5])), xtc_probability=float(rng.choice([0.0, 0.5])),
             xtc_threshold=float(rng.choice([0.1, 0.05])), repeat_penalty=float(rng.choice([1.0, 1.1, 1.5])),
             frequency_penalty=float(rng.choice([0.0, 0.2])), presence_penalty=float(rng.choice([0.0, 0.3])),
             repeat_last_n=int(rng.choice([0, 8, 64])), dry_multiplier=float(rng.choice([0.0, 0.8])),
             dry_base=1.75, dry_allowed=int(rng.choice([1, 2])), dry_last_n=int(rng.choice([0, 16])),
             mirostat=int(rng.choice([0, 0, 0, 2])), mirostat_tau=5.0, mirostat_eta=0.1,
             adaptive_p=float(rng.choice([-1.0, -1.0, 0.3, 0.7])), adaptive_decay=float(rng.choice([0.95, 0.5])), seed=int(rng.integers(0, 2**63)), chain=chain,
             bias=[(int(rng.integers(0, nv)), float(rng.choice([-5.0, 2.5])))] if rng.random() < 0.3 else [],
             breakers=[int(rng.integers(0, 12))] if rng.random() < 0.3 else [],
             top_n_sigma=float(rng.choice([0.0, 0.0, 1.0, 2.5])),
             dynatemp_range=float(rng.choice([0.0, 0.0, 0.4])), dynatemp_exponent=float(rng.choice([1.0, 1.7])),
             ignore_eos=int(rng.random() < 0.2), eos=int(rng.integers(0, nv)),
             suppress=[int(rng.integers(0, nv))] if rng.random() < 0.2 else [])
    return logits, hist, c


@pytest.mark.filterwarnings("ignore:invalid value")
@pytest.mark.parametrize("seed", range(10))
def test_c_and_python_restatements_agree(seed):
    rng = np.random.default_rng(100 + seed)
    for _ in range(40):
        logits, hist, c = _random_case(rng)
        kw = {k: c[k] for k in ("temperature", "top_k", "top_p", "min_p", "typical_p", "xtc_probability",
                                "xtc_threshold", "repeat_penalty", "frequency_penalty", "presence_penalty",
                                "repeat_last_n", "dry_multiplier", "dry_base", "mirostat", "mirostat_tau",
                                "mirostat_eta", "adaptive_p", "adaptive_decay", "seed", "chain", "top_n_sigma",
                                "dynatemp_range", "dynatemp_exponent", "ignore_eos", "eos")}
        kw.update(dry_allowed_length=c["dry_allowed"], dry_penalty_last_n=c["dry_last_n"],
                  bias_ids=[b[0] for b in c["bias"]], bias_values=[b[1] for b in c["bias"]],
                  dry_breakers=c["breakers"], suppress_ids=c["suppress"])
        cfg, keep = orc.sampler_config(**kw)
        st = orc.sampler_state(cfg)
        py = PySampler(c)
        for step in range(4):
            want = py.sample(logits, hist)
            got = orc.sample(cfg, st, logits, hist)
            assert got == want, (c, step)
            assert st.rng == py.rng
            for a, b in ((st.mu, py.mu), (st.ap_weighted, py.apw), (st.ap_total, py.apt)):
                assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)
            hist = hist + [got]


def test_sampler_structs_agree_with_the_header():
    """bt_sampler_config / bt_sampler_state: the header, the product's ctypes mirror and the
    oracle's struct have the same fields in the same order (the oracle's functions take the
    product's structs' bytes in the GPU tests' comparisons)."""
    import re

    from bigtea_b200 import _lib

    text = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                             "bigtea_decode.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    for cname, prod, orac in (("bt_sampler_config", _lib.SamplerConfig, orc.SamplerConfig),
                              ("bt_sampler_state", _lib.SamplerState, orc.SamplerState)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), text, flags=re.S).group(1)
        names = []
        for stmt in body.split(";"):
            stmt = " ".join(stmt.replace("*", " ").split())
            if stmt:
                first, *rest = stmt.split(",")
                names += [first.split()[-1]] + [r.strip() for r in rest]
        assert [f[0] for f in prod._fields_] == names
        assert [f[0] for f in orac._fields_] == names
        assert C.sizeof(prod) == C.sizeof(orac)


def test_product_sampler_defaults_and_init_match_the_oracle():
    """bt_sampler_config_default / _llamacpp and bt_sampler_init are host code in the product
    library: the same fields and the same initial state as the oracle's Sampler::new."""
    from bigtea_b200 import _lib

    for base in ("default", "llamacpp"):
        p = _lib.SamplerConfig()
        (_lib.lib.bt_sampler_config_llamacpp if base == "llamacpp" else _lib.lib.bt_sampler_config_default)(C.byref(p))
        o, _ = orc.sampler_config(base)
        for name, _t in _lib.SamplerConfig._fields_:
            a, b = getattr(p, name), getattr(o, name)
            if isinstance(a, (int, float)):
                assert np.float32(a).tobytes() == np.float32(b).tobytes() if isinstance(a, float) else a == b, name
            else:
                assert not a and not b, name  # the list pointers: NULL
    rng = np.random.default_rng(4)
    for _ in range(200):
        kw = dict(seed=int(rng.integers(0, 2**64, dtype=np.uint64)), mirostat_tau=float(rng.uniform(0, 10)),
                  adaptive_p=float(rng.choice([-1.0, 0.0, 0.3, 1.5, np.nan])),
                  adaptive_decay=float(rng.choice([0.0, 0.5, 0.95, 0.999, 2.0, -1.0])))
        o, _ = orc.sampler_config(**kw)
        p = _lib.SamplerConfig()
        _lib.lib.bt_sampler_config_default(C.byref(p))
        for k, v in kw.items():
            setattr(p, k, v)
        ps, os_ = _lib.SamplerState(), orc.sampler_state(o)
        assert _lib.lib.bt_sampler_init(C.byref(p), C.byref(ps)) == 0
        assert ps.rng == os_.rng
        for f in ("mu", "ap_weighted", "ap_total"):
            assert np.float32(getattr(ps, f)).tobytes() == np.float32(getattr(os_, f)).tobytes(), (kw, f)


def test_stage_names_and_the_default_chain():
    """sample.rs:1193-1220 (the_default_chain_is_llamacpp_s_order, stage_names_match_llamacpp_s_spelling)
    on the product's host side, and a chain given by name reaching the C struct"""
    from bigtea_b200 import runner

    assert runner.DEFAULT_CHAIN == [runner.STAGES[n] for n in ("top_k", "typical_p", "top_p", "min_p", "xtc",
                                                               "temperature")]
    assert runner.parse_stage("top_k") == 0 and runner.parse_stage("typ_p") == 1 and runner.parse_stage("min_p") == 3
    assert runner.parse_stage(" TEMPERATURE ") == 5
    assert runner.parse_stage("top_q") is None
    assert runner.parse_chain("temp;top_p") == [5, 2]
    with pytest.raises(ValueError):
        runner.parse_chain("top_k;top_q")
    s = runner.Sampler(None, 2, temperature=1.0, chain="top_p;temperature", seed=9)
    assert s.cfg.n_chain == 2 and [s.cfg.chain[i] for i in range(2)] == [2, 5]
    o, _ = orc.sampler_config(temperature=1.0, seed=9)
    assert all(st.rng == orc.sampler_state(o).rng for st in s.states)


def test_oracle_reproduces_the_sampler_golden_vectors():
    """tests/golden/sampler_golden.npz (made by gen_sampler_golden.py): every token and state"""
    import json

    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "sampler_golden.npz"))
    for c, (base, kw) in enumerate(json.loads(str(g["configs"]))):
        cfg, _keep = orc.sampler_config(base, **kw)
        st = orc.sampler_state(cfg)
        hist = [int(x) for x in g["history0"]]
        for s in range(g["tokens"].shape[1]):
            t = orc.sample(cfg, st, g["logits"][s], hist)
            assert t == int(g["tokens"][c, s]), (base, kw, s)
            got = [st.rng] + [int(np.float32(getattr(st, f)).view(np.uint32)) for f in ("mu", "ap_weighted", "ap_total")]
            assert got == [int(x) for x in g["states"][c, s]], (base, kw, s)
            hist.append(t)

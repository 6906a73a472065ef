"""Generate tests/golden/sampler_golden.npz: tokens and sampler states of the oracle's
restatement of Sampler::sample (core/arch/src/sample.rs:474-680) on seeded logits.

The restatement itself is pinned by the reference's own sampler tests and by a second,
independent restatement (tests/test_sampler_oracle.py); this file freezes its outputs so that a
later change to oracle/sample.c that moves a draw is seen. Run from the repository root:
    python tests/golden/gen_sampler_golden.py
"""
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import pyoracle as orc  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_golden.npz")
V, STEPS = 1000, 6
CONFIGS = [
    ("llamacpp", {"seed": 1}),
    ("default", {"temperature": 1.0, "seed": 2}),
    ("default", {"temperature": 0.7, "top_p": 0.8, "seed": 3}),
    ("default", {"temperature": 1.2, "top_k": 100, "typical_p": 0.6, "min_p": 0.01, "seed": 4}),
    ("default", {"temperature": 1.0, "top_n_sigma": 1.0, "xtc_probability": 0.5, "xtc_threshold": 0.05, "seed": 5}),
    ("default", {"temperature": 0.9, "dynatemp_range": 0.4, "dynatemp_exponent": 1.5, "top_k": 50, "seed": 6}),
    ("default", {"mirostat": 2, "mirostat_tau": 3.0, "seed": 7}),
    ("default", {"temperature": 1.0, "top_k": 60, "adaptive_p": 0.3, "seed": 8}),
    ("default", {"temperature": 0.8, "top_k": 80, "repeat_penalty": 1.2, "frequency_penalty": 0.1,
                 "presence_penalty": 0.2, "dry_multiplier": 0.8, "dry_breakers": [7], "bias_ids": [3],
                 "bias_values": [2.0], "suppress_ids": [0], "seed": 9}),
    ("default", {"temperature": 2.0, "top_p": 0.5, "chain": [5, 2], "seed": 10}),
]


def main():
    rng = np.random.default_rng(2024)
    logits = (rng.standard_normal((STEPS, V)) * 2.0).astype(np.float32)
    history0 = rng.integers(0, 30, 40).astype(np.uint32)
    tokens = np.zeros((len(CONFIGS), STEPS), np.uint32)
    states = np.zeros((len(CONFIGS), STEPS, 4), np.uint64)
    for c, (base, kw) in enumerate(CONFIGS):
        cfg, _keep = orc.sampler_config(base, **kw)
        st = orc.sampler_state(cfg)
        hist = list(history0)
        for s in range(STEPS):
            t = orc.sample(cfg, st, logits[s], hist)
            tokens[c, s] = t
            states[c, s] = [st.rng] + [int(np.float32(getattr(st, f)).view(np.uint32))
                                       for f in ("mu", "ap_weighted", "ap_total")]
            hist.append(t)
    np.savez_compressed(OUT, logits=logits, history0=history0, tokens=tokens, states=states,
                        configs=np.array(json.dumps(CONFIGS)))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()

"""How far the arithmetic contract lies from ggml's CPU arithmetic (TEST INFRASTRUCTURE).

Runs the reference's CPU-runnable workload (cfg0: 2 layers at the Qwen3-30B-A3B shape, seeded
weights, a 128-token prefill of uniform ids, then `steps` greedy steps) through oracle models of
different numerics, teacher-forced with the first model's greedy tokens so that every step
compares logits for the same history:

- the contract (what the device computes, bit for bit) against ggml-cpu's generic algorithms
  (NUM_GGML), and ggml against a second build of the same code (NUM_FMA: its multiply-adds
  contracted into fmaf, as a GNU-C build would do) -- the yardstick;
- the same with routing forced equal (each model takes route()'s expert choice from the contract
  run), which removes the discontinuity of a different expert set and leaves the arithmetic;
- each op's departure alone: the contract with one op switched to ggml's algorithm.

    python -m oracle.ggml_distance [steps]

prints the table quoted in the design notes. tests/test_ggml_bound.py asserts on the same
measurements.
"""
from __future__ import annotations

import sys

import numpy as np

from oracle import pyoracle as orc
from oracle import workloads

OPS = {"rms_norm (double sum)": orc.NUM_NORM, "K-quant dot (generic lanes)": orc.NUM_QDOT,
       "router F32 dot (double sum)": orc.NUM_FDOT, "soft_max (libm expf, double sum)": orc.NUM_SOFTMAX,
       "silu (libm expf)": orc.NUM_SILU, "flash_attn_ext (serial, f16 acc)": orc.NUM_ATTN,
       "flash_attn_ext (serial, f32 acc)": orc.NUM_ATTN_F32V}


def cfg0_model(seed: int = 2024):
    cfg = workloads.workload("cfg0")
    W = orc.synth_model(cfg.tensor_specs(), seed=seed)
    prompt = np.random.default_rng(seed).integers(0, cfg.n_vocab, 128)
    return cfg, W, prompt


def run(cfg, W, prompt, modes: dict, forced: dict, steps: int):
    """Teacher-forced decode of every model in `modes` (name -> numerics); the first name drives
    the tokens; `forced` maps a name to the name whose routing it takes. Returns the logits of
    each of the steps + 1 positions per model and the routing differences against the first model
    as (step, layer, name, the first model's 8th-9th probability gap)."""
    ms = {n: orc.Model(cfg, W, numerics=v) for n, v in modes.items()}
    try:
        for n, src in forced.items():
            ms[n].route_from(ms[src])
        order = [n for n in ms if n not in forced] + [n for n in ms if n in forced]
        ref = order[0]
        lg = {n: ms[n].forward(prompt, 0) for n in order}
        hist, flips = [dict(lg)], []
        for step in range(steps):
            t = len(prompt) - 1 if step == 0 else 0
            for il in range(cfg.n_layer):
                ids0 = set(ms[ref].topk(il, t)[0].tolist())
                for n in order[1:]:
                    if set(ms[n].topk(il, t)[0].tolist()) != ids0:
                        flips.append((step, il, n, ms[ref].route_gap(il, t)))
            tok = orc.argmax(lg[ref])
            lg = {n: ms[n].forward([tok], ms[n].len()) for n in order}
            hist.append(dict(lg))
        return hist, flips
    finally:
        for m in ms.values():
            m.close()


def distance(hist, a: str, b: str) -> dict:
    """max-abs and relative L2 of the logits over all positions, and the positions whose argmax
    differs with the first model's top-2 logit gap there"""
    mx = max(float(np.abs(h[a] - h[b]).max()) for h in hist)
    rl = max(float(np.linalg.norm(h[a] - h[b]) / np.linalg.norm(h[b])) for h in hist)
    diffs = []
    for i, h in enumerate(hist):
        if orc.argmax(h[a]) != orc.argmax(h[b]):
            top = np.sort(h[a])[-2:]
            diffs.append((i, float(top[1] - top[0])))
    return {"max_abs": mx, "rel_l2": rl, "argmax_diff": diffs}


def measure(steps: int = 64, per_op: bool = True) -> dict:
    cfg, W, prompt = cfg0_model()
    G = orc.NUM_GGML
    out = {}
    hist, flips = run(cfg, W, prompt, {"contract": 0, "ggml": G, "ggml_fma": G | orc.NUM_FMA}, {}, steps)
    out["free"] = {"contract_vs_ggml": distance(hist, "contract", "ggml"),
                   "ggml_vs_ggml_fma": distance(hist, "ggml", "ggml_fma"),
                   "route_flips": [f for f in flips if f[2] == "ggml"]}
    hist, _ = run(cfg, W, prompt, {"contract": 0, "ggml": G, "ggml_fma": G | orc.NUM_FMA},
                  {"ggml": "contract", "ggml_fma": "contract"}, steps)
    out["forced"] = {"contract_vs_ggml": distance(hist, "contract", "ggml"),
                     "ggml_vs_ggml_fma": distance(hist, "ggml", "ggml_fma")}
    if per_op:
        modes = {"contract": 0, **OPS}
        hist, _ = run(cfg, W, prompt, modes, {k: "contract" for k in OPS}, steps)
        out["per_op"] = {k: distance(hist, "contract", k) for k in OPS}
    return out


def _fmt(d):
    return (f"max-abs {d['max_abs']:.4f}, rel-L2 {d['rel_l2']:.2e}, argmax differences {len(d['argmax_diff'])}"
            + (f" (top-2 logit gaps {', '.join(f'{g:.1e}' for _, g in d['argmax_diff'])})" if d["argmax_diff"] else ""))


if __name__ == "__main__":
    steps = int(sys.argv[1]) if len(sys.argv) > 1 else 64
    r = measure(steps)
    print(f"cfg0, 128-token prefill + {steps} teacher-forced greedy steps ({steps + 1} logit vectors)")
    print("routing free:")
    print("  contract vs ggml      :", _fmt(r["free"]["contract_vs_ggml"]))
    print("  ggml vs ggml (fma)    :", _fmt(r["free"]["ggml_vs_ggml_fma"]))
    fl = r["free"]["route_flips"]
    print(f"  top-k set differences contract vs ggml: {len(fl)} of {2 * (steps + 1)} (layer, position); "
          f"8th-9th probability gaps at them: max {max((f[3] for f in fl), default=0):.2e}")
    print("routing forced equal:")
    print("  contract vs ggml      :", _fmt(r["forced"]["contract_vs_ggml"]))
    print("  ggml vs ggml (fma)    :", _fmt(r["forced"]["ggml_vs_ggml_fma"]))
    print("one departure at a time (contract with that op switched to ggml's, routing forced):")
    for k, d in r["per_op"].items():
        print(f"  {k:34s}: {_fmt(d)}")

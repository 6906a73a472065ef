#!/usr/bin/env python
"""Decode-throughput benchmark of the B200 decode-step layer (one JSON line on rank 0).

Workload (N=1): the full 48-layer Qwen3-30B-A3B shape (hidden 2048, 32/4 heads, head_dim 128,
128 experts top-8, expert FFN 768, vocab 151936) with synthetic N(0, 0.02) weights in a
Q4_K_M stand-in mix, all resident in HBM; batch-1 greedy decode after an 8192-token prefill
of uniform-random token ids into the f16 paged KV cache. A step = one decode token.

  value      device tok/s: K graph-replayed decode steps timed with CUDA events
  e2e        tok/s through bt_forward with host token in / host logits out every step
  roofline   the expert FFN (gate/up + down kernels) against the measured HBM copy peak
  cpu_baseline  the CPU oracle decoding from the same weights and cache on the host cores
  parity     the first measured decode step's logits against the CPU oracle from the same
             weights and cache, bit for bit (a mismatch fails the run)
  expert_gemv  the routed experts' arithmetic alone over every layer (bt_bench_experts): the
             per-layer kernels at batch 1 and at the batched leg's batch, and the multi-layer
             stream kernel at batch 1 (checked bit for bit against the per-layer kernels): HBM
             GB/s of the distinct expert weights
  expert_cache  experts moved to pinned host memory behind an HBM cache (the policy on the
             device, inside the persistent step), a fresh sequence: 128-token prefill then 128
             batch-1 decode steps of seeded uniform ids; LRU and frequency-gated admission, each
             from a cold cache: decode tok/s and hit rate, for the log-Zipf router bias at the cfg4
             ratio of cache to experts (6.26 GiB), the same bias with a third of that cache, no
             bias at 6.26 GiB, and a routing trace whose working set exceeds the cache
  batched    64 concurrent sequences, contexts seeded uniform in [512, 16384], paged f16 KV
             with seeded contents, a log-Zipf(1.1) router bias per layer (expert popularity
             over a seeded rank permutation); device tok/s of K graph-replayed steps

N>1 (torchrun): replicas -- every rank runs the same batch-1 decode on its own GPU (weak
scaling; no collective on the batch-1 path); rank 0 reports the sum of tok/s with the step
time taken as the max over ranks. The batched workload then runs expert parallel: each rank
holds its own batch of sequences and keeps only 1/N of the experts in HBM, computing them for
every rank's tokens, the rows exchanged over NCCL (weak scaling: global batch = N x batch);
rank 0 checks one expert-parallel step against a one-GPU engine holding every expert.

--impl reference: the reference's CPU implementation of the path is not buildable here (Rust,
no toolchain; ggml absent), so this arm times the CPU oracle restatement (`kind: "port"`) on
the same config with all host threads.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (bs1, bs64) Qwen3-30B-A3B shape; expert-GEMV HBM GB/s vs peak"
QWEN3_30B = dict(n_embd=2048, n_head=32, n_head_kv=4, head_dim=128, n_expert=128, n_expert_used=8, n_ff_exp=768,
                 n_vocab=151936)


def shape_name(cfg):
    if cfg.name in ("cfg0", "cfg1"):
        return f"Qwen3-30B-A3B shape, {cfg.n_layer} layers" + (", Q4_K_M stand-in" if cfg.name == "cfg1" else ", Q4_K")
    return (f"{cfg.n_layer} layers, hidden {cfg.n_embd}, {cfg.n_head}/{cfg.n_head_kv} heads, {cfg.n_expert} experts "
            f"top-{cfg.n_expert_used}" + (f" + a shared expert of {cfg.n_ff_shexp}" if cfg.n_ff_shexp else "")
            + f", expert width {cfg.n_ff_exp}, vocab {cfg.n_vocab}")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def expert_bytes(cfg, per_expert=False):
    """Algorithmic bytes of the expert FFN per token, averaged over layers: top-k experts x
    (gate + up + down) in each layer's K-quant types (per_expert: one expert's bytes)."""
    from bigtea_b200.gguf import tensor_nbytes

    E, F, K = cfg.n_embd, cfg.n_ff_exp, cfg.n_expert_used
    if per_expert:
        return float(np.mean([tensor_nbytes(t[4], E * F) + tensor_nbytes(t[5], E * F) + tensor_nbytes(t[6], F * E)
                              for t in cfg.layer_types]))
    gu, dn = [], []
    for t in cfg.layer_types:
        gu.append(K * (tensor_nbytes(t[4], E * F) + tensor_nbytes(t[5], E * F)))
        dn.append(K * tensor_nbytes(t[6], F * E))
    return float(np.mean(gu)), float(np.mean(dn))


def workload_config(config_name, cfg, shape, ctx, world):
    """The `config` dict of both arms' JSON lines (identical for the same workload and N)."""
    resident = sum(_kq_bytes(ty, int(np.prod(ne))) for _, ty, ne, _ in cfg.tensor_specs())
    return {"workload": f"{config_name}: {shape}, batch 1 greedy decode at context {ctx}", "batch": 1,
            "context": ctx, "parallelism": "replicas" if world > 1 else "single GPU",
            "l2": f"inputs larger than L2: {decode_bytes_per_token(cfg, ctx) / 1e9:.2f} GB of weights and KV read "
                  f"per step ({resident / 1e9:.1f} GB of weights resident)"}


def _kq_bytes(ty, n):
    return n * 4 if ty == 0 else n * 2 if ty == 1 else n // 256 * (144 if ty == 12 else 210)


def decode_bytes_per_token(cfg, ctx):
    """Algorithmic bytes one batch-1 decode token reads at context ctx: the attention weights,
    norms and router of every layer, the K selected experts' gate/up/down, the output head, and
    the K/V of ctx + 1 positions (the new one included); the embedding row is negligible."""
    tot = 0
    for name, ty, ne, _ in cfg.tensor_specs():
        n = 1
        for d in ne:
            n *= d
        if name == "token_embd.weight":
            continue
        b = _kq_bytes(ty, n)
        if "_exps." in name:
            b = b // cfg.n_expert * cfg.n_expert_used
        tot += b
    return tot + cfg.n_layer * 2 * cfg.n_head_kv * cfg.head_dim * 2 * (ctx + 1)


def host_info(threads):
    """CPU model, the threads used, and the host's STREAM-style copy bandwidth (read + write)."""
    from oracle import pyoracle as orc

    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    gbs = orc.lib().or_copy_gbs(1 << 30, threads, 3)
    return {"cpu_model": model, "cores": threads, "host_copy_gbs": round(gbs, 1)}


def cpu_baseline_from_engine(engine, cache, cfg, ctx, n_tokens, threads, tok0):
    """The CPU oracle decoding n_tokens from the same weights (copied back from HBM) and the same
    first ctx cache positions, starting with token tok0 at position ctx. Returns the tok/s and the
    logits of that first step, which the caller compares with the GPU's for the same position."""
    from oracle import pyoracle as orc
    from bigtea_b200.gguf import tensor_nbytes

    W = {}
    for name, ty, ne, _ in cfg.tensor_specs():
        n = 1
        for d in ne:
            n *= d
        W[name] = (ty, ne, engine.tensor_bytes(name, tensor_nbytes(ty, n)))
    model = orc.Model(cfg, W)
    for il in range(cfg.n_layer):
        k, v = cache.layer_bytes(il, 0, ctx)
        model.write_kv_layer(il, k, v)
    model.set_len(ctx)
    orc.lib().or_set_threads(threads)
    tok = tok0
    t0 = time.perf_counter()
    first = None
    for i in range(n_tokens):
        lg = model.forward([tok], model.len())
        if first is None:
            first = lg
        tok = orc.argmax(lg)
    dt = time.perf_counter() - t0
    model.close()
    return n_tokens / dt, first


def run_ours(args, rank, world, local_rank):
    import bigtea_b200 as bt

    longest = max(args.ctx, args.ctx2_max if args.batch2 else 0)
    over = {"max_positions": longest + 2 * (args.steps + args.warmup) + args.steps // 4 + args.prof_steps + 64}
    if args.layers:
        over["n_layer"] = args.layers
        over["layer_types"] = bt.config(args.config).layer_types[:args.layers]
    cfg = bt.config(args.config, **over)
    t_setup = time.perf_counter()
    engine = bt.Engine.synthetic(cfg, seed=args.seed, device=local_rank)
    if args.prefetch:
        engine.set_option("prefetch", 1)
    if args.no_pdl:
        engine.set_option("pdl", 0)
    cache = bt.KvCache(engine, max_positions=cfg.max_positions)
    runner = bt.StreamingRunner(engine)
    rng = np.random.default_rng(args.seed + 1)
    t0 = time.perf_counter()
    if args.fill == "prefill":
        prompt = rng.integers(0, cfg.n_vocab, args.ctx)
        logits = runner.forward_cached(cache, prompt, 0)
        tok = int(np.argmax(logits))
    else:  # seeded f16 values: the decode cost does not depend on the cache contents
        kw = cfg.n_head_kv * cfg.head_dim
        for il in range(cfg.n_layer):
            k = rng.standard_normal(args.ctx * kw).astype(np.float16)
            v = rng.standard_normal(args.ctx * kw).astype(np.float16)
            cache.restore_layer(il, k, v)
        cache.set_positions(args.ctx)
        tok = int(rng.integers(0, cfg.n_vocab))
    prefill_s = time.perf_counter() - t0
    # the first decode position: one bt_forward step (the persistent kernel at batch 1) whose
    # logits the CPU oracle reproduces below from the same weights and the same first ctx cache
    # positions -- the parity check of the measured path
    tok0 = tok
    logits0 = runner.forward_cached(cache, [tok0], args.ctx)
    tok = int(np.argmax(logits0))
    # warm-up (also captures the step graph), then K timed graph replays
    runner.generate_greedy(cache, [tok], args.warmup)
    sync_ranks(world)
    # clocks sampled from the batch-1 timed steps through the batched leg's timed steps (the
    # batch-1 region alone is a fraction of a second)
    clk = ClockSampler(local_rank).__enter__()
    toks = runner.generate_greedy(cache, [tok], args.steps)
    dev_ms = runner.last_device_ms()
    ms = max_over_ranks(dev_ms, world)
    value = world * args.steps / (ms / 1e3)

    # e2e: bt_forward with a host token in and host logits out every step, after its own
    # untimed warm-up calls (the first direct launches after the graph replays cost a few ms)
    e2e_steps = max(16, args.steps)
    nxt = int(toks[-1, 0])
    lg_out = bt.pinned_empty((1, cfg.n_vocab))  # the caller's page-locked logits buffer
    for _ in range(max(3, args.warmup)):
        lg = runner.forward_cached(cache, [nxt], cache.len(), out=lg_out)
        nxt = int(np.argmax(lg))
    sync_ranks(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        lg = runner.forward_cached(cache, [nxt], cache.len(), out=lg_out)
        nxt = int(np.argmax(lg))
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = world * e2e_steps / e2e_s

    # per-kernel device times (serialised launches) for the roofline
    prof = runner.profile_decode(cache, [nxt], args.prof_steps) if args.prof_steps else {}
    if not args.batch2:
        clk.__exit__(None, None, None)
    gu_bytes, dn_bytes = expert_bytes(cfg)
    persistent = "decode_step" in prof

    # the routed experts' kernels alone (bt_bench_experts): every layer in turn, a seeded selection
    # of K distinct experts per token, at batch 1 (1.02 GB of distinct expert weights a pass over
    # the 48 layers) and at the batched leg's batch; HBM GB/s of the distinct weights read
    expert_gemv = None
    if args.expert_iters:
        peak_gbs, _ = peaks()
        expert_gemv = {"what": "the routed experts' gate/up and down kernels alone, every layer in turn (one CUDA "
                               "graph), seeded selections of K distinct experts per token; bytes = the distinct "
                               "selected experts' weights of a pass", "peak_gbs": peak_gbs}
        for T in sorted({1, args.batch2 or 64}):
            ms_x, nb_x = engine.bench_experts(T, n_iters=args.expert_iters, seed=args.seed)
            gbs = nb_x / (ms_x / 1e3) / 1e9
            expert_gemv[f"batch{T}"] = {"ms_per_pass": round(ms_x, 4), "gb_per_pass": round(nb_x / 1e9, 3),
                                        "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak_gbs, 4),
                                        "path": "per-token kernels" if T <= 8 else "grouped kernels (tcgen05 gate/up)"}
        # the same arithmetic as one persistent kernel over every layer, given the selections up
        # front: the weight stream runs on across the gate/up -> down dependency of each layer
        ms_s, nb_s, out_s = engine.bench_experts(1, n_iters=args.expert_iters, seed=args.seed, kernel=1, out=True)
        _, _, out_k = engine.bench_experts(1, n_iters=1, seed=args.seed, kernel=0, out=True)
        gbs = nb_s / (ms_s / 1e3) / 1e9
        expert_gemv["batch1_stream"] = {
            "ms_per_pass": round(ms_s, 4), "gb_per_pass": round(nb_s / 1e9, 3), "achieved_gbs": round(gbs, 1),
            "frac": round(gbs / peak_gbs, 4),
            "path": "one persistent kernel over the layers: a producer warp per CTA streams the selected experts' "
                    "tiles through a CTA-wide TMA ring; layer s's gate/up and layer s-1's down share a stage",
            "bit_exact_vs_per_layer_kernels": bool(np.array_equal(out_s.view(np.uint32), out_k.view(np.uint32)))}

    # the batched workload: batch2 concurrent sequences, per-sequence contexts seeded uniform in
    # [ctx2_min, ctx2_max], paged f16 KV
    batched = None
    if args.batch2:
        B = args.batch2
        rng2 = np.random.default_rng(args.seed + 2)
        ctxs = rng2.integers(args.ctx2_min, args.ctx2_max + 1, B)
        cache2 = bt.KvCache(engine, max_positions=int(ctxs.max()) + 2 * (args.steps + args.warmup) + 8,
                            max_seqs=B)
        # seeded f16 values in every cached position (a zero-filled pool is not a fair workload:
        # pages that hold only zeros can cost the memory system almost nothing to read); one
        # random buffer per layer, its prefixes shared by the sequences
        kw = cfg.n_head_kv * cfg.head_dim
        cmax = int(ctxs.max())
        # N > 1: rank 0 also builds a one-GPU engine with every expert resident and the first NREF
        # sequences' caches, to check the expert-parallel step's logits against it
        NREF = min(4, B)
        ref_engine = ref_cache = None
        if world > 1 and rank == 0 and args.ep_check:
            ref_engine = bt.Engine.synthetic(cfg, seed=args.seed, device=local_rank)
            ref_cache = bt.KvCache(ref_engine, max_positions=int(ctxs[:NREF].max()) + 8, max_seqs=NREF)
        for il in range(cfg.n_layer):
            k = rng2.standard_normal(cmax * kw).astype(np.float16)
            v = rng2.standard_normal(cmax * kw).astype(np.float16)
            for sq, c in enumerate(ctxs):
                cache2.restore_layer(il, k[:int(c) * kw], v[:int(c) * kw], seq=sq)
                if ref_cache is not None and sq < NREF:
                    ref_cache.restore_layer(il, k[:int(c) * kw], v[:int(c) * kw], seq=sq)
        for sq, c in enumerate(ctxs):
            cache2.set_positions(int(c), sq)
            if ref_cache is not None and sq < NREF:
                ref_cache.set_positions(int(c), sq)
        first2 = rng2.integers(0, cfg.n_vocab, B)
        if args.zipf > 0:  # skewed routing: a log-Zipf router bias per layer
            for il in range(cfg.n_layer):
                bias = bt.models.zipf_router_bias(cfg.n_expert, il, args.seed, args.zipf)
                engine.set_router_bias(il, bias)
                if ref_engine is not None:
                    ref_engine.set_router_bias(il, bias)
        ep_parity = None
        if world > 1:
            # expert parallelism: each rank computes NE/world experts for every rank's tokens
            engine.enable_ep_torch()
            # one single-token step of every sequence (a collective: every rank runs it); rank 0
            # compares its first NREF sequences with the one-GPU engine
            lg_ep = runner.forward_batch(cache2, list(range(B)), [[int(t)] for t in first2], [int(c) for c in ctxs])
            if ref_engine is not None:
                lg_ref = bt.StreamingRunner(ref_engine).forward_batch(
                    ref_cache, list(range(NREF)), [[int(t)] for t in first2[:NREF]], [int(c) for c in ctxs[:NREF]])
                same = bool(np.array_equal(lg_ep[:NREF].view(np.uint32), lg_ref.view(np.uint32)))
                ep_parity = {"status": "bit-exact" if same else "MISMATCH",
                             "max_abs": float(np.abs(lg_ep[:NREF] - lg_ref).max()),
                             "what": f"rank 0's first {NREF} sequences: logits of one expert-parallel step against "
                                     "a one-GPU engine holding every expert"}
                ref_cache.close()
                ref_engine.close()
            first2 = np.argmax(lg_ep, axis=1)
        runner.generate_greedy(cache2, first2, args.warmup)
        sync_ranks(world)
        runner.generate_greedy(cache2, first2, args.steps)
        clk.__exit__(None, None, None)
        ms2 = max_over_ranks(runner.last_device_ms(), world)
        # distinct experts a layer's last step selected (this rank's tokens)
        distinct = [len({int(i) for t in range(B) for i in engine.debug_topk(il, t)[0]}) for il in range(cfg.n_layer)]
        batched = {"value": round(world * B * args.steps / (ms2 / 1e3), 1), "unit": "tok/s", "batch": B,
                   "ms_per_step": round(ms2 / args.steps, 3),
                   "context": f"per sequence, seeded uniform in [{args.ctx2_min}, {args.ctx2_max}], "
                              f"mean {float(ctxs.mean()):.0f}",
                   "kv": "paged f16, 16-token blocks, seeded random contents",
                   "routing": (f"log-Zipf({args.zipf}) router bias per layer over a seeded permutation of the "
                               f"expert ranks" if args.zipf > 0 else "the synthetic router (no popularity bias)"),
                   "distinct_experts_per_layer": round(float(np.mean(distinct)), 1),
                   "path": "per-phase kernels (single-token steps of more than 4 sequences)",
                   "parallelism": (f"expert parallel over {world} GPUs: {B} sequences per rank, experts split "
                                   f"{cfg.n_expert // world} per rank (only those resident in each GPU's HBM), "
                                   f"rows exchanged by NCCL send/recv (Q8_K rows to the owners, f32 rows back)" if world > 1
                                   else "single GPU"),
                   "comm_nranks": world, "ep_parity": ep_parity}
        cache2.close()

    # per-phase kernels: the expert kernels' times; the persistent step: its gate/up and down
    # phases (slowest CTA, from the in-kernel timeline)
    gu = prof.get("expert_gateup", prof.get("ph5_gateup_work", (1, 0.0)))
    dn = prof.get("expert_down", prof.get("ph6_down_work", (1, 0.0)))
    exp_ms = gu[1] / max(gu[0], 1) + dn[1] / max(dn[0], 1)
    achieved = (gu_bytes + dn_bytes) / (exp_ms / 1e3) / 1e9 if exp_ms > 0 else None
    peak, peak_kind = peaks()
    per_step_launches = 1 if persistent else 1 + cfg.n_layer * 7 + 1 + 1

    # the device sampler (bt_sample) on the logits the last step left in HBM: one sequence,
    # llama.cpp's default chain over the whole vocabulary; host wall time per call
    sampler_leg = None
    if rank == 0 and world == 1:
        try:
            smp = bt.Sampler(engine, 1, base="llamacpp", seed=args.seed)
            hist = [list(range(64))]
            for _ in range(3):
                smp.sample(None, hist)
            n_draws = 50
            t_s = time.perf_counter()
            for _ in range(n_draws):
                smp.sample(None, hist)
            sampler_leg = {"ms_per_draw": round((time.perf_counter() - t_s) / n_draws * 1e3, 4),
                           "what": "bt_sample wall time per call: 1 sequence, llama.cpp defaults (top_k 40, top_p "
                                   "0.95, min_p 0.05, temperature 0.8, repeat penalty 1.1 over 64 tokens), "
                                   f"{cfg.n_vocab} logits already in HBM, 3 launches (prepare, radix sort, chain)"}
        except Exception as ex:  # a refusal is reported, never fatal to the bench line
            sampler_leg = {"error": str(ex)[:300]}

    result = None
    xcache = None
    if rank == 0:
        cpu, parity = None, {"status": "not checked (--no-cpu)"}
        if world > 1:
            # the CPU leg runs at N = 1 only: it copies every expert back from HBM, and the
            # expert-parallel leg has left each rank only its share (ep_parity checks that leg)
            parity = {"status": "not checked at N > 1 (the batch-1 parity runs at N = 1; batched.ep_parity "
                                "checks the expert-parallel step)"}
        elif not args.no_cpu:
            threads = os.cpu_count() or 1
            cpu_tps, first = cpu_baseline_from_engine(engine, cache, cfg, args.ctx, args.cpu_tokens, threads, tok0)
            host = host_info(threads)
            bpt = decode_bytes_per_token(cfg, args.ctx)
            cpu = {"value": round(cpu_tps, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                   "sample": f"{args.cpu_tokens} greedy decode tokens of the same {cfg.n_layer}-layer model from the "
                             f"same ctx-{args.ctx} KV cache (weights and cache copied back from HBM)",
                   "cpu_model": host["cpu_model"], "host_copy_gbs": host["host_copy_gbs"],
                   "bytes_per_token": bpt,
                   "host_ceiling_tok_s": round(host["host_copy_gbs"] * 1e9 / bpt, 2),
                   "ceiling_note": "host copy GB/s (read + write bytes) / algorithmic bytes a decode token reads"}
            diff = np.abs(first.astype(np.float64) - logits0.astype(np.float64))
            exact = bool(np.array_equal(first.view(np.uint32), logits0.view(np.uint32)))
            parity = {"status": "bit-exact" if exact else "MISMATCH", "max_abs": float(diff.max()),
                      "tolerance": 1e-2, "argmax_equal": int(np.argmax(first)) == int(np.argmax(logits0)),
                      "what": f"logits of the first decode step (position {args.ctx}, the persistent step kernel) "
                              "against the CPU oracle from the same weights and cache"}
        kernel_table = {k: {"launches": v[0], "avg_us": round(1e3 * v[1] / max(v[0], 1), 2)} for k, v in prof.items()}
        bpt_all = decode_bytes_per_token(cfg, args.ctx)
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_K/q6_K weights, int8 dot, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, uniform-random token ids)",
            "config": workload_config(args.config, cfg, shape_name(cfg), args.ctx, world),
            "setup": {"context_fill": f"{args.ctx}-token prefill of uniform-random ids" if args.fill == "prefill"
                      else "seeded f16 cache fill", "prefill_seconds": round(prefill_s, 2),
                      "setup_seconds": round(time.perf_counter() - t_setup, 1)},
            "parity": parity,
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * 7 + 1,
                    "d2h_bytes_per_step": 4 * cfg.n_vocab + 4},
            "gpu_launches": per_step_launches * args.steps,
            "roofline": {"bound": "hbm", "kernel": "expert FFN (gate/up + down)",
                         "achieved": round(achieved, 1) if achieved else None, "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4) if achieved else None, "peak_kind": peak_kind,
                         "bytes_per_token_layer": gu_bytes + dn_bytes, "traffic": None,
                         "traffic_note": "the expert FFN is two phases of the one persistent step kernel and ncu "
                                         "counts DRAM bytes per kernel: see step.traffic for the whole kernel"},
            "step": {"kernel": "decode_step_kernel (the whole batch-1 step)", "bytes_per_step": bpt_all,
                     "achieved_gbs": round(bpt_all / (ms / args.steps / 1e3) / 1e9, 1),
                     "frac": round(bpt_all / (ms / args.steps / 1e3) / 1e9 / peak, 4)},
            "kernels_us": kernel_table,
            "expert_gemv": expert_gemv,
            "batched": batched,
            "expert_cache": None,
            "sampler": sampler_leg,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
    # the out-of-HBM case at this model's scale: experts in pinned host memory behind an HBM
    # cache, batch-1 greedy decode, each policy from a cold cache, in three workloads: the
    # log-Zipf router bias with the cfg4 ratio of cache to experts (args.xcache_gib; the biased
    # working set about fits), the same bias with a cache a third that size, and no bias at the
    # cfg4 ratio (every expert in use: the working set is three times the cache)
    if args.xcache_gib > 0 and world == 1:
        xcache = {"steps": args.xcache_steps, "batch": 1,
                  "experts_bytes": int(cfg.n_layer * cfg.n_expert * expert_bytes(cfg, per_expert=True)),
                  "timing": (f"decode steps after a {args.xcache_prompt}-token prefill of seeded uniform ids: wall "
                             "clock of bt_forward per token (host token in, logits out; the cache policy on the "
                             "device inside the persistent step: CTA 0 looks each layer's experts up, every CTA "
                             "fills missed slots from pinned host memory); hit rate over the decode steps")}
        rngx = np.random.default_rng(args.seed + 3)
        prompt_x = rngx.integers(0, cfg.n_vocab, args.xcache_prompt)
        toks_x = rngx.integers(0, cfg.n_vocab, args.xcache_steps)
        cases = [("zipf", args.xcache_gib), ("zipf_small_cache", args.xcache_gib / 3), ("unbiased", args.xcache_gib),
                 ("zipf_trace", args.xcache_gib)]
        zs = args.zipf if args.zipf > 0 else 1.1
        try:
            for name, gib in cases:
                biased = name.startswith("zipf") and name != "zipf_trace" and args.zipf > 0
                for il in range(cfg.n_layer):
                    engine.set_router_bias(il, bt.models.zipf_router_bias(cfg.n_expert, il, args.seed, args.zipf)
                                           if biased else None)
                case = {"cache_bytes": int(gib * (1 << 30)),
                        "routing": (f"log-Zipf({args.zipf}) router bias per layer" if biased else
                                    f"a routing trace: each decode step's K experts per layer drawn from Zipf({zs}) "
                                    "over a seeded per-layer rank permutation, forced by a router bias (+30 on the "
                                    "drawn experts)" if name == "zipf_trace" else "unbiased")}
                trace = None
                if name == "zipf_trace":  # per step and layer, K distinct experts drawn from Zipf(zs)
                    rt = np.random.default_rng(args.seed + 4)
                    K_, NE_ = cfg.n_expert_used, cfg.n_expert
                    pz = np.arange(1, NE_ + 1, dtype=np.float64) ** -zs
                    pz /= pz.sum()
                    perms = [np.random.default_rng([args.seed, il, 0x2F1B]).permutation(NE_) for il in range(cfg.n_layer)]
                    trace = [[perms[il][rt.choice(NE_, K_, replace=False, p=pz)] for il in range(cfg.n_layer)]
                             for _ in range(args.xcache_steps)]
                for policy in ("lru", "freq"):
                    engine.enable_expert_cache(case["cache_bytes"], policy)
                    cache_x = bt.KvCache(engine, max_positions=args.xcache_prompt + args.xcache_steps + 8)
                    runner.forward_cached(cache_x, prompt_x, 0)  # prefill: warms the cache
                    st0 = engine.expert_cache_stats()
                    t0 = time.perf_counter()
                    wall_bias = 0.0
                    for si, tk in enumerate(toks_x):  # one token a step, seeded uniform ids
                        if trace is not None:
                            tb = time.perf_counter()
                            for il in range(cfg.n_layer):
                                b = np.zeros(cfg.n_expert, np.float32)
                                b[trace[si][il]] = 30.0
                                engine.set_router_bias(il, b)
                            wall_bias += time.perf_counter() - tb
                        runner.forward_cached(cache_x, [int(tk)], cache_x.len())
                    wall = time.perf_counter() - t0 - wall_bias
                    st = engine.expert_cache_stats()
                    cache_x.close()
                    d = {k: st[k] - st0[k] for k in ("hits", "misses", "evictions", "bypasses", "bytes_copied")}
                    case[policy] = {"tok_s": round(args.xcache_steps / wall, 2),
                                    "hit_rate": round(d["hits"] / max(d["hits"] + d["misses"], 1), 4),
                                    "evictions": d["evictions"], "bypasses": d["bypasses"],
                                    "gb_copied": round(d["bytes_copied"] / 1e9, 2), "wall_s": round(wall, 2),
                                    "prefill_hit_rate": round(st0["hit_rate"], 4)}
                    case["slots"] = st["capacity_slots"]
                xcache[name] = case
        except bt.BtError as err:  # e.g. pinned host memory refused
            xcache["unavailable"] = str(err)
    if result is not None:
        result["expert_cache"] = xcache
    cache.close()
    engine.close()
    return result


def run_reference(args, rank, world):
    """The CPU restatement of the reference's decode path on the host cores, same workload and
    config dict as the GPU arm. The model comes from the oracle's own seeded generator and
    workload description (oracle/workloads.py), so this arm never loads the product library."""
    if rank != 0:
        return None
    from oracle import pyoracle as orc
    from oracle import workloads

    try:
        cfg = workloads.workload(args.config, max_positions=args.ctx + args.steps + args.warmup + 8)
    except KeyError as err:
        return {"impl": "reference", "unavailable": f"no CPU-arm description of {args.config}: {err}"}
    threads = os.cpu_count() or 1
    W = orc.synth_model(cfg.tensor_specs(), seed=args.seed)
    model = orc.Model(cfg, W)
    # the decode cost does not depend on the cache contents: seeded f16 values stand in for
    # the prefilled context
    rng = np.random.default_rng(args.seed)
    kw = cfg.n_head_kv * cfg.head_dim
    for il in range(cfg.n_layer):
        k = rng.standard_normal(args.ctx * kw).astype(np.float16)
        v = rng.standard_normal(args.ctx * kw).astype(np.float16)
        model.write_kv_layer(il, k, v)
    model.set_len(args.ctx)
    orc.lib().or_set_threads(threads)
    tok = 1
    for _ in range(args.warmup):
        tok = orc.argmax(model.forward([tok], model.len()))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        tok = orc.argmax(model.forward([tok], model.len()))
    dt = time.perf_counter() - t0
    tps = args.steps / dt
    host = host_info(threads)
    bpt = decode_bytes_per_token(cfg, args.ctx)
    return {
        "impl": "reference", "metric": METRIC, "value": round(tps, 3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4_K/q6_K weights, int8 dot, f32 accumulate", "data": "synthetic",
        "config": workload_config(args.config, cfg, cfg.shape_name(), args.ctx, world),
        "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} decode tokens at context {args.ctx} (seeded f16 cache)",
                         "cpu_model": host["cpu_model"], "host_copy_gbs": host["host_copy_gbs"],
                         "bytes_per_token": bpt, "host_ceiling_tok_s": round(host["host_copy_gbs"] * 1e9 / bpt, 2),
                         "ceiling_note": "host copy GB/s (read + write bytes) / algorithmic bytes a decode token "
                                         "reads"},
        "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


_dist = None


def sync_ranks(world):
    if world > 1:
        import torch

        torch.cuda.synchronize()
        _dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch

    t = torch.tensor([float(x)], device="cuda")
    _dist.all_reduce(t, op=_dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="cfg1")
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--prof-steps", type=int, default=4)
    ap.add_argument("--cpu-tokens", type=int, default=3)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--fill", default="prefill", choices=["prefill", "random"],
                    help="build the context by a real prefill, or fill the cache with seeded f16 values")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (profiling runs)")
    ap.add_argument("--prefetch", action="store_true", help="enable the L2 bulk prefetch of upcoming inputs")
    ap.add_argument("--no-pdl", action="store_true", help="disable programmatic dependent launch")
    ap.add_argument("--batch2", type=int, default=64, help="sequences of the batched workload (0 skips it)")
    ap.add_argument("--ctx2-min", type=int, default=512)
    ap.add_argument("--ctx2-max", type=int, default=16384)
    ap.add_argument("--xcache-gib", type=float, default=6.26,
                    help="HBM expert-cache size of the out-of-HBM leg (0 skips it); the default keeps the "
                         "cfg4 ratio of cache to experts (120 GB of ~311 GB)")
    ap.add_argument("--xcache-steps", type=int, default=128)
    ap.add_argument("--expert-iters", type=int, default=20, help="passes of the isolated expert-kernel timing "
                    "(0 skips it)")
    ap.add_argument("--ep-check", type=int, default=1, help="N > 1: rank 0 checks one expert-parallel step against a "
                    "one-GPU engine (needs the model twice in rank 0's HBM)")
    ap.add_argument("--xcache-prompt", type=int, default=128)
    ap.add_argument("--zipf", type=float, default=1.1, help="router-bias Zipf exponent of the batched workload "
                    "(0: unbiased)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    global _dist
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        _dist = dist
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    else:
        out = run_ours(args, rank, world, local_rank)
    if world > 1:
        _dist.barrier()
        _dist.destroy_process_group()
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
        if out.get("parity", {}).get("status") == "MISMATCH":
            print("bench: the measured step's logits differ from the CPU oracle's", file=sys.stderr)
            sys.exit(3)
        if ((out.get("batched") or {}).get("ep_parity") or {}).get("status") == "MISMATCH":
            print("bench: the expert-parallel step's logits differ from the one-GPU engine's", file=sys.stderr)
            sys.exit(3)
        if ((out.get("expert_gemv") or {}).get("batch1_stream") or {}).get("bit_exact_vs_per_layer_kernels") is False:
            print("bench: the expert stream kernel's sums differ from the per-layer kernels'", file=sys.stderr)
            sys.exit(3)


if __name__ == "__main__":
    main()

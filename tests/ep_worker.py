"""One rank of the expert-parallel parity test (launched by tests/test_gpu_ep.py under torchrun).

Each rank builds the same tiny synthetic model on its own GPU, joins the expert-parallel group
(the NCCL unique id travels over a gloo process group) and runs `rank_workload`: batched steps
whose sequence count and contexts depend on the rank, so the ranks send each other different
numbers of rows. Its results go to <out>/rank<r>.npz; the test compares them with a
single-GPU engine running the same workload.
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def rank_workload(bt, engine, cfg, rank: int) -> dict:
    """The steps of one rank: one single-token step of every sequence, a mixed step (two short
    prompts beside single tokens), four greedy graph-replayed steps, one more single-token step.
    Every call is one engine step (at most 64 tokens under expert parallelism), the same count on
    every rank."""
    n_seq = 3 + 4 * (rank % 3)
    rng = np.random.default_rng(100 + rank)
    ctxs = [int(c) for c in rng.integers(100, 1500, n_seq)]
    kw = cfg.n_head_kv * cfg.head_dim
    cache = bt.KvCache(engine, max_positions=2048, max_seqs=n_seq)
    for s, n in enumerate(ctxs):
        for il in range(cfg.n_layer):
            k = (0.5 * rng.standard_normal(n * kw)).astype(np.float16)
            v = rng.standard_normal(n * kw).astype(np.float16)
            cache.restore_layer(il, k, v, seq=s)
        cache.set_positions(n, s)
    runner = bt.StreamingRunner(engine)
    seqs = list(range(n_seq))
    out = {}
    toks = [int(t) for t in rng.integers(0, cfg.n_vocab, n_seq)]
    out["step1"] = runner.forward_batch(cache, seqs, [[t] for t in toks], [cache.len(s) for s in seqs])
    lists = [[int(t) for t in rng.integers(0, cfg.n_vocab, 5)], [int(t) for t in rng.integers(0, cfg.n_vocab, 3)]]
    lists += [[int(t)] for t in rng.integers(0, cfg.n_vocab, n_seq - 2)]
    out["step2"] = runner.forward_batch(cache, seqs, lists, [cache.len(s) for s in seqs])
    first = [int(t) for t in np.argmax(out["step2"], axis=1)]
    out["greedy"] = runner.generate_greedy(cache, first, 4, seqs=seqs).astype(np.int64)
    last = [int(t) for t in out["greedy"][-1]]
    out["step3"] = runner.forward_batch(cache, seqs, [[t] for t in last], [cache.len(s) for s in seqs])
    k0, v0 = cache.layer_bytes(cfg.n_layer - 1, 0)
    out["kv_k"], out["kv_v"] = np.asarray(k0), np.asarray(v0)
    cache.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    import torch
    import torch.distributed as dist

    import bigtea_b200 as bt

    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    cfg = bt.config("tiny", max_positions=2048)
    engine = bt.Engine(cfg, bt.synth_model(cfg, seed=7), device=local)
    engine.set_option("ep_timeout_ms", 30000)
    before = engine.stats()["weight_bytes"]
    engine.enable_ep_torch()
    after = engine.stats()["weight_bytes"]
    res = rank_workload(bt, engine, cfg, rank)
    res["weight_bytes"] = np.array([before, after], np.int64)
    np.savez(os.path.join(args.out, f"rank{rank}.npz"), **res)
    engine.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

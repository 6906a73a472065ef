"""The expert-parallel exchange protocol, restated in Python and run over 2 gloo ranks on the CPU.

With n ranks, rank r owns the experts [r * NE / n, (r + 1) * NE / n). Per layer of a step of T
tokens with K selected experts each (S = TB * K slots per rank, TB the step capacity):

1. pack (`ep_pack_kernel`): slot tk = t * K + k of the local step goes to the rank that owns its
   expert, at the same slot position tk of that rank's block: send_meta[owner * S + tk] = expert,
   every other rank's entry -1; send_rows[owner * S + tk] = the token's normalised row;
2. dispatch: block q of every rank's send buffers goes to rank q (NCCL grouped send/recv);
3. the owner runs its experts on the received slots (recv block q, slot tk: an expert id or -1)
   and writes each result row at the same position (dpart[q * S + tk]);
4. combine exchange: block q of dpart goes back to rank q;
5. combine (`down_combine_kernel`): token t's slot k reads the row at
   ret[(expert / per) * S + t * K + k] and the K rows are added with their route weights in the
   reference's order -- expert_ffn_single's chunks of ceil(K / workers) for a single-token step
   (core/arch/src/stream.rs:1232-1284), expert_ffn_block's sequential sum otherwise (1051-1058).

The test runs this protocol across two gloo processes (all_to_all over CPU tensors) with a
stand-in expert function, each rank with its own tokens and step size, and compares every rank's
result with the same computation done in one process without an exchange, bit for bit. It
checks the indexing of the protocol; the GPU test (tests/test_gpu_ep.py) checks the kernels.
"""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

NE, K, E, TB, WORKERS = 16, 4, 64, 8, 4


def expert(e: int, row: np.ndarray) -> np.ndarray:
    """a stand-in expert FFN: deterministic, different per expert, f32"""
    return (np.float32(1.0 + 0.125 * e) * row + np.float32(0.01 * e)).astype(np.float32)


def combine(o: np.ndarray, w: np.ndarray, single: bool) -> np.ndarray:
    """the reference's expert sum of K rows o[k] with weights w[k] (f32, in order)"""
    s = np.zeros(o.shape[1], np.float32)
    if single:
        workers = max(1, min(WORKERS, K))
        chunk = (K + workers - 1) // workers
        for s0 in range(0, K, chunk):
            tot = (o[s0] * w[s0]).astype(np.float32)
            for i in range(s0 + 1, min(K, s0 + chunk)):
                tot = (tot + (o[i] * w[i]).astype(np.float32)).astype(np.float32)
            s = tot if workers <= 1 else (s + tot).astype(np.float32)
    else:
        for i in range(K):
            s = (s + (o[i] * w[i]).astype(np.float32)).astype(np.float32)
    return s


def local_step(sel, wts, fn, single):
    """one rank's step without an exchange: every expert evaluated where the token lives"""
    T = sel.shape[0]
    out = np.empty((T, E), np.float32)
    for t in range(T):
        o = np.stack([expert(int(sel[t, k]), fn[t]) for k in range(K)])
        out[t] = combine(o, wts[t], single)
    return out


def workload(rank: int, T: int):
    rng = np.random.default_rng(100 + rank)
    sel = np.stack([np.sort(rng.choice(NE, K, replace=False)) for _ in range(T)]).astype(np.int32)
    wts = rng.dirichlet(np.ones(K), T).astype(np.float32)
    fn = rng.standard_normal((T, E)).astype(np.float32)
    return sel, wts, fn


def ep_step(rank, n, sel, wts, fn, single, dist):
    """the protocol: pack, dispatch, owner compute, combine exchange, combine"""
    S, per, T = TB * K, NE // n, sel.shape[0]
    send_meta = np.full((n, S), -1, np.int32)
    send_rows = np.zeros((n, S, E), np.float32)
    for tk in range(T * K):
        e = int(sel[tk // K, tk % K])
        owner = e // per
        send_meta[owner, tk] = e
        send_rows[owner, tk] = fn[tk // K]
    recv_meta = torch.empty((n, S), dtype=torch.int32)
    recv_rows = torch.empty((n, S, E), dtype=torch.float32)
    dist.all_to_all_single(recv_meta, torch.from_numpy(send_meta))
    dist.all_to_all_single(recv_rows, torch.from_numpy(send_rows))
    recv_meta, recv_rows = recv_meta.numpy(), recv_rows.numpy()
    dpart = np.zeros((n, S, E), np.float32)
    for q in range(n):
        for tk in range(S):
            e = int(recv_meta[q, tk])
            if e >= 0:
                assert rank * per <= e < (rank + 1) * per, "a slot reached a rank that does not own its expert"
                dpart[q, tk] = expert(e, recv_rows[q, tk])
    ret = torch.empty((n, S, E), dtype=torch.float32)
    dist.all_to_all_single(ret, torch.from_numpy(dpart))
    ret = ret.numpy()
    out = np.empty((T, E), np.float32)
    for t in range(T):
        o = np.stack([ret[int(sel[t, k]) // per, t * K + k] for k in range(K)])
        out[t] = combine(o, wts[t], single)
    return out


def _rank(rank, n, port, outdir):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=n,
                            timeout=datetime.timedelta(seconds=60))
    try:
        ok = True
        for T, single in ((TB, False), (3 + rank, False), (1, True)):  # full, ragged per rank, single-token
            sel, wts, fn = workload(rank * 10 + T, T)
            got = ep_step(rank, n, sel, wts, fn, single, dist)
            want = local_step(sel, wts, fn, single)
            ok &= bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
        with open(os.path.join(outdir, f"ok{rank}"), "w") as f:
            f.write("1" if ok else "0")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [2])
def test_pack_dispatch_combine_equals_one_process(tmp_path, n):
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_rank, args=(n, port, str(tmp_path)), nprocs=n, join=True, start_method="spawn")
    for r in range(n):
        assert (tmp_path / f"ok{r}").read_text() == "1", f"rank {r}"

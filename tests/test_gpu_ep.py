"""Expert parallelism on 2 or more GPUs: every rank's logits, greedy tokens and KV bytes equal a
single-GPU engine's on the same workload, bit for bit (the expert FFN of each (token, slot)
row runs on the rank owning the expert and comes back in the reference's summation order), and
every rank holds only its own 1/n of the routed experts' weights in HBM.

Runs the ranks as child processes (tests/ep_worker.py under torchrun, bounded by `timeout`);
skipped with fewer than two GPUs."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import bigtea_b200 as bt
from tests.conftest import bits
from tests.ep_worker import rank_workload

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    torch = pytest.importorskip("torch")
    return torch.cuda.device_count()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n", [2, 4, 8])
def test_expert_parallel_matches_single_gpu(tmp_path, n):
    if _gpus() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=ROOT)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(n), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "ep_worker.py"), "--out", str(tmp_path)]
    r = subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    cfg = bt.config("tiny", max_positions=2048)
    engine = bt.Engine(cfg, bt.synth_model(cfg, seed=7))
    for rank in range(n):
        got = np.load(tmp_path / f"rank{rank}.npz")
        want = rank_workload(bt, engine, cfg, rank)
        for key in ("step1", "step2", "step3"):
            assert np.array_equal(bits(got[key]), bits(want[key])), (rank, key)
        assert np.array_equal(got["greedy"], want["greedy"]), rank
        assert np.array_equal(got["kv_k"], want["kv_k"]) and np.array_equal(got["kv_v"], want["kv_v"]), rank
        # each rank keeps only its 1/n of the routed experts in HBM
        before, after = (int(x) for x in got["weight_bytes"])
        expert = sum(bt.gguf.tensor_nbytes(ty, int(np.prod(ne))) for name, ty, ne, _ in cfg.tensor_specs()
                     if name.endswith("_exps.weight"))
        assert before - after == expert - expert // n, (rank, before, after, expert)
    engine.close()

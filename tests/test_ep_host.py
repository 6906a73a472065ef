"""Host side of expert parallelism, without a GPU: the NCCL unique id shared over a 2-rank gloo
group, and argument checks of bt_engine_enable_ep."""
import ctypes as C
import datetime
import os

import pytest

from bigtea_b200 import _lib

torch = pytest.importorskip("torch")


def _share(rank, world, port, out):
    import torch.distributed as dist

    from bigtea_b200.runner import share_ep_unique_id

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                           timeout=datetime.timedelta(seconds=30))
    uid = share_ep_unique_id()
    with open(os.path.join(out, f"uid{rank}"), "wb") as f:
        f.write(uid)
    dist.barrier()
    dist.destroy_process_group()


def test_unique_id_is_shared_by_every_rank(tmp_path):
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_share, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    a = (tmp_path / "uid0").read_bytes()
    b = (tmp_path / "uid1").read_bytes()
    assert len(a) == 128 and a == b and any(a)


def test_enable_ep_rejects_bad_arguments():
    uid = (C.c_uint8 * 128)()
    assert _lib.lib.bt_engine_enable_ep(None, uid, 128, 0, 2) == _lib.BT_ERR_INVALID
    assert _lib.lib.bt_ep_unique_id(None, 128) == _lib.BT_ERR_INVALID
    assert _lib.lib.bt_ep_unique_id(uid, 64) == _lib.BT_ERR_INVALID

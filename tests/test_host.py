"""CPU tests of the host side: the C ABI loads and exports what the header declares, the
synthetic weights are seeded and well-formed, the GGUF writer produces files llama.cpp's
gguf-py reads, and the error paths return statuses instead of aborting."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import bigtea_b200 as bt
from bigtea_b200 import _lib
from oracle import pyoracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for hdr in os.listdir(os.path.join(ROOT, "include")):
        if hdr.endswith(".h"):
            text = open(os.path.join(ROOT, "include", hdr)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(bt_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    declared = declared_functions()
    assert len(declared) >= 25
    raw = C.CDLL(bt.build.LIB if hasattr(bt, "build") else _lib._build.LIB)
    missing = [n for n in sorted(declared) if not hasattr(raw, n)]
    assert not missing, missing
    # and the Python binding covers exactly the header
    assert declared == set(_lib.SIGNATURES)


def test_abi_version():
    assert _lib.lib.bt_abi_version() == _lib.ABI_VERSION


def test_tensor_id_is_fnv1a():
    def fnv(s):
        h = 1469598103934665603
        for ch in s.encode():
            h ^= ch
            h = (h * 1099511628211) % 2 ** 64
        return h

    for name in ("token_embd.weight", "blk.7.ffn_down_exps.weight"):
        assert bt.models.tensor_id(name) == fnv(name)


def test_synthetic_weights_are_seeded():
    a = bt.models.synth_tensor("x.weight", _lib.TYPE_Q4_K, (512, 8), 0.0, seed=1)
    b = bt.models.synth_tensor("x.weight", _lib.TYPE_Q4_K, (512, 8), 0.0, seed=1)
    c = bt.models.synth_tensor("x.weight", _lib.TYPE_Q4_K, (512, 8), 0.0, seed=2)
    assert np.array_equal(a, b) and not np.array_equal(a, c)


@pytest.mark.parametrize("ty", [_lib.TYPE_Q4_K, _lib.TYPE_Q6_K, _lib.TYPE_F32])
def test_synthetic_weights_are_gaussian(ty):
    w = bt.models.synth_tensor("stats.weight", ty, (2048, 64), 0.0, seed=3, sigma=0.02)
    x = orc.dequant(ty, w, 2048 * 64)
    assert abs(x.mean()) < 1e-3 and abs(x.std() - 0.02) < 1e-3


def test_norm_weights_center_on_one():
    w = bt.models.synth_tensor("blk.0.attn_norm.weight", _lib.TYPE_F32, (2048,), 1.0, seed=3)
    x = w.view(np.float32)
    assert abs(x.mean() - 1.0) < 2e-3


def test_gguf_roundtrip_through_gguf_py(tmp_path, tiny_cfg, tiny_weights):
    gguf = pytest.importorskip("gguf")
    path = str(tmp_path / "tiny.gguf")
    bt.write_gguf(path, tiny_cfg, tiny_weights)
    r = gguf.GGUFReader(path)
    names = {t.name: t for t in r.tensors}
    assert set(names) == set(tiny_weights)
    for name, (ty, ne, data) in tiny_weights.items():
        t = names[name]
        assert int(t.tensor_type) == ty
        assert list(map(int, t.shape)) == list(ne)
        assert np.array_equal(np.asarray(t.data).view(np.uint8).reshape(-1), data)
    arch = r.fields["general.architecture"]
    assert bytes(arch.parts[arch.data[0]]).decode() == "qwen3moe"
    # and our own reader recovers the config and bytes
    cfg2, t2 = bt.read_gguf(path, max_positions=tiny_cfg.max_positions)
    assert cfg2.n_expert == tiny_cfg.n_expert and cfg2.layer_types == tiny_cfg.layer_types
    assert all(np.array_equal(np.asarray(t2[n][2]), tiny_weights[n][2]) for n in tiny_weights)


def test_q4km_standin_mix():
    cfg = bt.config("cfg1")
    assert cfg.layer_types[0][2] == _lib.TYPE_Q6_K and cfg.layer_types[1][2] == _lib.TYPE_Q4_K
    assert cfg.layer_types[0][6] == _lib.TYPE_Q6_K and cfg.layer_types[1][6] == _lib.TYPE_Q4_K


def test_unsupported_shapes_are_refused_before_any_device_call(tiny_cfg):
    d = bt.config("tiny", head_dim=64).desc()
    h = C.c_void_p()
    st = _lib.lib.bt_engine_create(C.byref(d), None, 0, 0, C.byref(h))
    assert st == _lib.BT_ERR_UNSUPPORTED and not h.value
    assert b"head_dim" in _lib.lib.bt_last_error()


def test_missing_device_is_an_error_not_an_abort(tiny_cfg):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    d = tiny_cfg.desc()
    h = C.c_void_p()
    st = _lib.lib.bt_engine_create(C.byref(d), None, 0, 0, C.byref(h))
    assert st == _lib.BT_ERR_CUDA and not h.value


def test_partial_kquant_block_is_refused_by_the_dequant_hook():
    out = np.empty(200, np.float32)
    st = _lib.lib.bt_debug_dequant(_lib.TYPE_Q4_K, _lib.ptr(np.zeros(144, np.uint8)), 200,
                                   _lib.ptr(out, C.c_float))
    assert st == _lib.BT_ERR_INVALID

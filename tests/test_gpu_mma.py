"""GPU: the tensor-core path's building block, one tcgen05.mma kind::i8 contraction through the
operand layouts and descriptors the grouped expert kernel uses, against an exact integer
matmul (integer products and sums: the result is exact, so equality is the bar)."""
import ctypes as C

import numpy as np
import pytest

from bigtea_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k", [(8, 32), (16, 32), (16, 256), (32, 64), (16, 512)])
def test_i8_mma_is_exact(n, k):
    rng = np.random.default_rng(n * 1000 + k)
    a = rng.integers(0, 256, (128, k), dtype=np.uint8)
    b = rng.integers(-128, 128, (n, k), dtype=np.int8)
    d = np.empty((128, n), np.int32)
    rc = _lib.lib.bt_op_i8_mma(a.ctypes.data, b.ctypes.data, n, k, _lib.ptr(d, C.c_int32))
    assert rc == 0, _lib.lib.bt_last_error()
    want = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(d.astype(np.int64), want)


def test_i8_mma_rejects_bad_shapes():
    a = np.zeros((128, 32), np.uint8)
    b = np.zeros((16, 32), np.int8)
    d = np.zeros((128, 16), np.int32)
    assert _lib.lib.bt_op_i8_mma(a.ctypes.data, b.ctypes.data, 12, 32, _lib.ptr(d, C.c_int32)) == _lib.BT_ERR_INVALID
    assert _lib.lib.bt_op_i8_mma(a.ctypes.data, b.ctypes.data, 16, 48, _lib.ptr(d, C.c_int32)) == _lib.BT_ERR_INVALID

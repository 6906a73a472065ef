"""GPU tests of the allocation-free GEMV entry point, bt_op_gemv_noalloc, against bt_op_gemv.

The file name sorts last, so the tests run after every other test has used the device; they
also pass on their own (`pytest tests/test_zz_no_alloc.py -m gpu`). Caller-owned device
buffers come from torch."""
import numpy as np
import pytest

from bigtea_b200 import _lib
from bigtea_b200.runner import gemv

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

BLOCK_BYTES = {_lib.TYPE_Q4_K: 144, _lib.TYPE_Q6_K: 210}


def _synth(ggml_type, rows, cols, seed):
    w = np.empty(rows * (cols // 256) * BLOCK_BYTES[ggml_type], np.uint8)
    rc = _lib.lib.bt_synth_tensor(ggml_type, rows, cols, seed, 99, 0.0, 0.02, w.ctypes.data)
    assert rc == 0, _lib.lib.bt_last_error()
    return w


def _noalloc(ggml_type, w_dev, rows, cols, x_dev, y_dev):
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.lib.bt_op_gemv_noalloc(ggml_type, w_dev.data_ptr(), rows, cols, x_dev.data_ptr(), x_dev.shape[0],
                                       y_dev.data_ptr(), stream)


# (type, rows, cols, tokens): an expert gate matrix, a Q6_K down matrix, attn_output with more
# tokens than one launch carries (8), and the q|k|v-sized Q4_K matrix
CASES = [
    (_lib.TYPE_Q4_K, 768, 2048, 1),
    (_lib.TYPE_Q6_K, 2048, 768, 3),
    (_lib.TYPE_Q4_K, 2048, 4096, 9),
    (_lib.TYPE_Q4_K, 5120, 2048, 2),
]


def test_noalloc_matches_bt_op_gemv_calls_in_a_row():
    torch.cuda.init()
    rng = np.random.default_rng(11)
    inputs = []
    for i, (ty, rows, cols, T) in enumerate(CASES):
        w = _synth(ty, rows, cols, seed=100 + i)
        x = rng.standard_normal((T, cols)).astype(np.float32)
        inputs.append((ty, rows, cols, w, x, gemv(ty, w, rows, cols, x)))
    dev = [(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()) for (_, _, _, w, x, _) in inputs]
    outs = [torch.empty((x.shape[0], rows), dtype=torch.float32, device="cuda") for (_, rows, _, _, x, _) in inputs]
    torch.cuda.synchronize()
    # first pass: includes this device's one-time set-up
    for (ty, rows, cols, _, _, ref), (w_dev, x_dev), y_dev in zip(inputs, dev, outs):
        assert _noalloc(ty, w_dev, rows, cols, x_dev, y_dev) == 0, _lib.lib.bt_last_error()
        np.testing.assert_array_equal(y_dev.cpu().numpy(), ref)
    # two more passes back to back, in reverse order, with the outputs cleared in between; the
    # device's free memory does not move across the calls themselves (measured after torch's
    # own kernels for the clearing and the copies have been loaded)
    for _ in range(2):
        for y_dev in outs:
            y_dev.fill_(float("nan"))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for (ty, rows, cols, _, _, ref), (w_dev, x_dev), y_dev in reversed(list(zip(inputs, dev, outs))):
            assert _noalloc(ty, w_dev, rows, cols, x_dev, y_dev) == 0, _lib.lib.bt_last_error()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before
        for (_, _, _, _, _, ref), y_dev in zip(inputs, outs):
            np.testing.assert_array_equal(y_dev.cpu().numpy(), ref)


def test_noalloc_rejects_a_matrix_larger_than_its_scratch():
    # the 151936 x 2048 Q6_K output head: 255 MB tiled, far above the 16 MiB scratch; rejected
    # before anything touches the (tiny) buffers
    small = torch.zeros(256, dtype=torch.float32, device="cuda")
    rc = _lib.lib.bt_op_gemv_noalloc(_lib.TYPE_Q6_K, small.data_ptr(), 151936, 2048, small.data_ptr(), 1,
                                     small.data_ptr(), None)
    assert rc == _lib.BT_ERR_INVALID
    assert b"BT_NOALLOC_SCRATCH_BYTES" in _lib.lib.bt_last_error()
    # bad arguments are statuses too
    assert _lib.lib.bt_op_gemv_noalloc(_lib.TYPE_Q4_K, None, 16, 256, small.data_ptr(), 1, small.data_ptr(),
                                       None) == _lib.BT_ERR_INVALID
    assert _lib.lib.bt_op_gemv_noalloc(_lib.TYPE_F32, small.data_ptr(), 16, 256, small.data_ptr(), 1,
                                       small.data_ptr(), None) == _lib.BT_ERR_UNSUPPORTED
    assert _lib.lib.bt_op_gemv_noalloc(_lib.TYPE_Q4_K, small.data_ptr(), 16, 200, small.data_ptr(), 1,
                                       small.data_ptr(), None) == _lib.BT_ERR_UNSUPPORTED


def test_noalloc_on_its_own_stream_with_a_partial_last_chunk():
    """17 tokens (two full launches of 8 and a 1-token tail) on a stream that is not torch's
    current one, for a Q6_K shape the other test does not use: the call orders itself on the
    given stream, and the tail chunk's offsets are right."""
    ty, rows, cols, T = _lib.TYPE_Q6_K, 1536, 2048, 17
    rng = np.random.default_rng(12)
    w = _synth(ty, rows, cols, seed=300)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    ref = gemv(ty, w, rows, cols, x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        w_dev = torch.from_numpy(w).to("cuda", non_blocking=False)
        x_dev = torch.from_numpy(x).to("cuda", non_blocking=False)
        y_dev = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
    rc = _lib.lib.bt_op_gemv_noalloc(ty, w_dev.data_ptr(), rows, cols, x_dev.data_ptr(), T, y_dev.data_ptr(),
                                     s.cuda_stream)
    assert rc == 0, _lib.lib.bt_last_error()
    s.synchronize()
    np.testing.assert_array_equal(y_dev.cpu().numpy(), ref)

"""ctypes binding of include/bigtea_decode.h (the C ABI of libbigtea_decode.so).

The library is required: importing this module loads it and raises if it is missing or
does not export the ABI. There is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

BT_OK, BT_ERR_INVALID, BT_ERR_CUDA, BT_ERR_OOM, BT_ERR_MISSING_TENSOR, BT_ERR_KV, BT_ERR_TIMEOUT, BT_ERR_UNSUPPORTED = range(8)
STATUS_NAMES = {
    1: "BT_ERR_INVALID", 2: "BT_ERR_CUDA", 3: "BT_ERR_OOM", 4: "BT_ERR_MISSING_TENSOR",
    5: "BT_ERR_KV", 6: "BT_ERR_TIMEOUT", 7: "BT_ERR_UNSUPPORTED",
}
TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 12, 14
KV_F16 = 1
ABI_VERSION = 2


class BtError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class ModelDesc(C.Structure):
    _fields_ = [
        ("n_layer", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32), ("n_head_kv", C.c_uint32),
        ("head_dim", C.c_uint32), ("n_expert", C.c_uint32), ("n_expert_used", C.c_uint32),
        ("n_ff_exp", C.c_uint32), ("n_vocab", C.c_uint32), ("n_rot", C.c_uint32),
        ("rms_eps", C.c_float), ("rope_freq_base", C.c_float),
        ("expert_workers", C.c_uint32), ("max_positions", C.c_uint32), ("n_ff_shexp", C.c_uint32),
    ]


class TensorView(C.Structure):
    _fields_ = [
        ("name", C.c_char_p), ("type", C.c_uint32), ("n_dims", C.c_uint32), ("ne", C.c_uint64 * 4),
        ("data", C.c_void_p), ("nbytes", C.c_uint64),
    ]


class Stats(C.Structure):
    _fields_ = [
        ("forward_calls", C.c_uint64), ("tokens", C.c_uint64), ("forward_seconds", C.c_double),
        ("weight_bytes", C.c_uint64), ("graph_replays", C.c_uint64),
    ]


class XCacheStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("hits", "misses", "evictions", "admissions", "bypasses", "bytes_copied",
                                          "capacity_slots", "slot_bytes")]


XCACHE_LRU, XCACHE_FREQ = 0, 1


class KernelTime(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("launches", C.c_uint64), ("total_ms", C.c_double)]


class SamplerConfig(C.Structure):
    """bt_sampler_config: SamplerConfig (core/arch/src/sample.rs:84-180)"""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float), ("min_p", C.c_float),
                ("typical_p", C.c_float), ("top_n_sigma", C.c_float), ("xtc_probability", C.c_float),
                ("xtc_threshold", C.c_float), ("dynatemp_range", C.c_float), ("dynatemp_exponent", C.c_float),
                ("repeat_penalty", C.c_float), ("frequency_penalty", C.c_float), ("presence_penalty", C.c_float),
                ("repeat_last_n", C.c_uint32), ("dry_multiplier", C.c_float), ("dry_base", C.c_float),
                ("dry_allowed_length", C.c_uint32), ("dry_penalty_last_n", C.c_uint32), ("mirostat", C.c_uint32),
                ("mirostat_tau", C.c_float), ("mirostat_eta", C.c_float), ("adaptive_p", C.c_float),
                ("adaptive_decay", C.c_float), ("ignore_eos", C.c_int32), ("eos", C.c_int32),
                ("chain", C.POINTER(C.c_int32)), ("n_chain", C.c_uint32),
                ("bias_ids", C.POINTER(C.c_uint32)), ("bias_values", C.POINTER(C.c_float)), ("n_bias", C.c_uint32),
                ("suppress_ids", C.POINTER(C.c_uint32)), ("n_suppress", C.c_uint32),
                ("dry_breakers", C.POINTER(C.c_uint32)), ("n_dry_breakers", C.c_uint32), ("seed", C.c_uint64)]


class SamplerState(C.Structure):
    """bt_sampler_state: the state a Sampler carries between tokens (sample.rs:306-321)"""
    _fields_ = [("rng", C.c_uint64), ("mu", C.c_float), ("ap_weighted", C.c_float), ("ap_total", C.c_float)]


_P = C.c_void_p
_U32P = C.POINTER(C.c_uint32)
_F32P = C.POINTER(C.c_float)
_I32P = C.POINTER(C.c_int32)

# name -> (restype, argtypes); every function the header declares
SIGNATURES = {
    "bt_last_error": (C.c_char_p, []),
    "bt_abi_version": (C.c_int, []),
    "bt_engine_create": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(TensorView), C.c_size_t, C.c_int, C.POINTER(_P)]),
    "bt_engine_create_synthetic": (C.c_int, [C.POINTER(ModelDesc), _U32P, C.c_uint32, C.c_uint32, C.c_uint64,
                                             C.c_float, C.c_int, C.POINTER(_P)]),
    "bt_engine_destroy": (None, [_P]),
    "bt_engine_stats": (C.c_int, [_P, C.POINTER(Stats)]),
    "bt_engine_tensor_bytes": (C.c_int, [_P, C.c_char_p, _P, C.c_uint64]),
    "bt_kv_create": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(_P)]),
    "bt_kv_destroy": (None, [_P]),
    "bt_kv_len": (C.c_int, [_P, C.c_uint32, _U32P]),
    "bt_kv_clear": (C.c_int, [_P, C.c_uint32]),
    "bt_kv_truncate": (C.c_int, [_P, C.c_uint32, C.c_uint32]),
    "bt_kv_shift_out": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint32]),
    "bt_kv_set_positions": (C.c_int, [_P, C.c_uint32, C.c_uint32]),
    "bt_kv_bytes": (C.c_int, [_P, C.POINTER(C.c_uint64)]),
    "bt_kv_is_consistent": (C.c_int, [_P, C.c_uint32, C.POINTER(C.c_int)]),
    "bt_kv_export_layer": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, _P, C.c_uint64]),
    "bt_kv_import_layer": (C.c_int, [_P, C.c_uint32, C.c_uint32, _P, _P, C.c_uint64]),
    # (array arguments as plain addresses: the per-token call is latency-bound, and building
    # typed ctypes pointers costs more host time than the rest of the wrapper)
    "bt_forward": (C.c_int, [_P, _P, _P, _P, _P, _P, C.c_uint32, _P]),
    "bt_generate_greedy": (C.c_int, [_P, _P, _U32P, _U32P, C.c_uint32, C.c_uint32, _U32P, _F32P]),
    "bt_last_device_ms": (C.c_int, [_P, C.POINTER(C.c_double)]),
    "bt_sampler_config_default": (None, [C.POINTER(SamplerConfig)]),
    "bt_sampler_config_llamacpp": (None, [C.POINTER(SamplerConfig)]),
    "bt_sampler_init": (C.c_int, [C.POINTER(SamplerConfig), C.POINTER(SamplerState)]),
    "bt_sample": (C.c_int, [_P, C.POINTER(SamplerConfig), C.POINTER(SamplerState), C.c_uint32, _F32P, _U32P, _U32P,
                            _U32P]),
    "bt_host_alloc": (C.c_int, [C.c_uint64, C.POINTER(C.c_void_p)]),
    "bt_host_free": (C.c_int, [_P]),
    "bt_bench_experts": (C.c_int, [_P, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint32, C.POINTER(C.c_double),
                                   C.POINTER(C.c_uint64), C.POINTER(C.c_float)]),
    "bt_profile_decode": (C.c_int, [_P, _P, _U32P, _U32P, C.c_uint32, C.c_uint32, C.POINTER(KernelTime),
                                    C.c_uint32, _U32P]),
    "bt_set_option": (C.c_int, [_P, C.c_char_p, C.c_int]),
    "bt_debug_dequant": (C.c_int, [C.c_uint32, _P, C.c_uint64, _F32P]),
    "bt_debug_topk": (C.c_int, [_P, C.c_uint32, C.c_uint32, _I32P, _F32P]),
    "bt_debug_hidden": (C.c_int, [_P, C.c_uint32, _F32P]),
    "bt_op_gemv": (C.c_int, [C.c_uint32, _P, C.c_uint32, C.c_uint32, _F32P, C.c_uint32, _F32P]),
    "bt_ep_unique_id": (C.c_int, [_P, C.c_size_t]),
    "bt_engine_set_router_bias": (C.c_int, [_P, C.c_uint32, _F32P, C.c_uint32]),
    "bt_op_i8_mma": (C.c_int, [_P, _P, C.c_uint32, C.c_uint32, _I32P]),
    "bt_engine_enable_expert_cache": (C.c_int, [_P, C.c_uint64, C.c_int]),
    "bt_expert_cache_stats": (C.c_int, [_P, C.POINTER(XCacheStats)]),
    "bt_expert_cache_simulate": (C.c_int, [C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _I32P,
                                           C.c_uint32, C.POINTER(XCacheStats)]),
    "bt_expert_cache_simulate_device": (C.c_int, [C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, _I32P,
                                           C.c_uint32, C.POINTER(XCacheStats)]),
    "bt_engine_enable_ep": (C.c_int, [_P, _P, C.c_size_t, C.c_int, C.c_int]),
    # device pointers and a cudaStream_t, passed as integers
    "bt_op_gemv_noalloc": (C.c_int, [C.c_uint32, _P, C.c_uint32, C.c_uint32, _P, C.c_uint32, _P, _P]),
    "bt_synth_tensor": (C.c_int, [C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float,
                                  C.c_float, _P]),
    "bt_tensor_id": (C.c_uint64, [C.c_char_p]),
}


def _load() -> C.CDLL:
    path = _build.LIB
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python -m bigtea_b200.build` (nvcc, sm_100a). "
            "This package has no CPU fallback.")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError = the ABI is incomplete: fail loudly
        fn.restype = res
        fn.argtypes = args
    if lib.bt_abi_version() != ABI_VERSION:
        raise ImportError("libbigtea_decode.so ABI version mismatch")
    return lib


lib = _load()


def check(status: int) -> None:
    if status != BT_OK:
        raise BtError(status, lib.bt_last_error().decode(errors="replace"))


def ptr(a, ctype=None):
    """ctypes pointer to a numpy array's data."""
    p = a.ctypes.data_as(C.c_void_p)
    return C.cast(p, C.POINTER(ctype)) if ctype is not None else p

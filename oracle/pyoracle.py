"""ctypes wrapper of oracle/liboracle.so -- the CPU parity checker (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module; the product
(bigtea_b200) never does. `build()` compiles the library with oracle/Makefile.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

OR_F32, OR_F16, OR_Q4_K, OR_Q6_K = 0, 1, 12, 14
ATTN_CHUNK = 128  # keys per attention chunk in the arithmetic contract (C8)


class Q8KBlock(C.Structure):
    _fields_ = [("d", C.c_float), ("qs", C.c_int8 * 256), ("bsums", C.c_int16 * 16)]


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_expert",
                                        "n_expert_used", "n_ff_exp", "n_vocab", "n_rot")] + \
               [("rms_eps", C.c_float), ("rope_base", C.c_float), ("expert_workers", C.c_int),
                ("attn_chunk", C.c_int), ("max_positions", C.c_int), ("numerics", C.c_int)]


# numerics of an oracle model: 0 = the device's arithmetic contract; else a set of bits, each op
# whose bit is set computing with ggml-cpu's generic algorithm (NUM_GGML: all of them)
NUM_CONTRACT, NUM_NORM, NUM_QDOT, NUM_FDOT, NUM_SOFTMAX, NUM_SILU, NUM_ATTN, NUM_ATTN_F32V, NUM_FMA = \
    0, 1, 2, 4, 8, 16, 32, 64, 128
NUM_GGML = 63
NUM_GGML_F32V = NUM_GGML & ~NUM_ATTN | NUM_ATTN_F32V


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_int), ("ne", C.c_int64 * 4), ("data", C.c_void_p)]


class SamplerConfig(C.Structure):
    """SamplerConfig (core/arch/src/sample.rs:84-180); the layout of bt_sampler_config"""
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
    _fields_ = [("rng", C.c_uint64), ("mu", C.c_float), ("ap_weighted", C.c_float), ("ap_total", C.c_float)]


STAGE_TOP_K, STAGE_TYPICAL_P, STAGE_TOP_P, STAGE_MIN_P, STAGE_XTC, STAGE_TEMPERATURE = range(6)


def build() -> str:
    src = [os.path.join(HERE, f) for f in ("oracle.c", "sample.c", "oracle.h", "Makefile")]
    if not os.path.exists(LIB) or any(os.path.getmtime(s) > os.path.getmtime(LIB) for s in src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB)
        P, F, I = C.c_void_p, C.POINTER(C.c_float), C.c_int
        sig = {
            "or_f32_to_f16": (C.c_uint16, [C.c_float]),
            "or_f16_to_f32": (C.c_float, [C.c_uint16]),
            "or_exp": (C.c_float, [C.c_float]),
            "or_silu": (C.c_float, [C.c_float]),
            "or_row_bytes": (C.c_int64, [I, C.c_int64]),
            "or_dequant": (I, [I, P, C.c_int64, F]),
            "or_quantize_q8k": (None, [F, C.c_int64, C.POINTER(Q8KBlock)]),
            "or_gemv": (I, [I, P, C.c_int64, C.c_int64, F, F]),
            "or_rmsnorm": (None, [F, F, I, C.c_float, F]),
            "or_rope_table": (None, [I, I, C.c_float, F]),
            "or_softmax": (None, [F, I, F]),
            "or_route": (None, [F, I, I, C.POINTER(C.c_int32), F]),
            "or_attn_head": (None, [F, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), C.c_int64, I, I, C.c_float, I, F]),
            "or_argmax": (C.c_uint32, [F, C.c_int64]),
            "or_model_new": (P, [C.POINTER(Config), C.POINTER(Tensor), I]),
            "or_model_free": (None, [P]),
            "or_last_error": (C.c_char_p, []),
            "or_kv_new": (P, [P]),
            "or_kv_free": (None, [P]),
            "or_kv_len": (I, [P]),
            "or_kv_set_len": (None, [P, I]),
            "or_kv_read": (None, [P, I, I, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16)]),
            "or_kv_write": (None, [P, I, I, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16)]),
            "or_forward": (I, [P, P, C.POINTER(C.c_int32), I, I, F]),
            "or_debug_topk": (I, [P, I, I, C.POINTER(C.c_int32), F]),
            "or_debug_hidden": (I, [P, I, F]),
            "or_set_threads": (I, [I]),
            "or_tensor_id": (C.c_uint64, [C.c_char_p]),
            "or_synth_tensor": (I, [I, C.c_int64, C.c_int64, C.c_uint64, C.c_uint64, C.c_float, C.c_float, P]),
            "or_copy_gbs": (C.c_double, [C.c_int64, I, I]),
            "or_model_route_from": (None, [P, P]),
            "or_debug_route_gap": (I, [P, I, I, F]),
            "or_ggml_rmsnorm": (None, [F, F, I, C.c_float, F]),
            "or_ggml_gemv": (I, [I, P, C.c_int64, C.c_int64, F, F]),
            "or_ggml_softmax": (None, [F, I, F]),
            "or_ggml_attn_head": (None, [F, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), C.c_int64, I, I, C.c_float,
                                         I, F]),
            "or_ln": (C.c_float, [C.c_float]),
            "or_pow": (C.c_float, [C.c_float, C.c_float]),
            "or_sampler_config_default": (None, [C.POINTER(SamplerConfig)]),
            "or_sampler_config_llamacpp": (None, [C.POINTER(SamplerConfig)]),
            "or_sampler_init": (None, [C.POINTER(SamplerConfig), C.POINTER(SamplerState)]),
            "or_sampler_next_f32": (C.c_float, [C.POINTER(SamplerState)]),
            "or_sample": (C.c_int64, [C.POINTER(SamplerConfig), C.POINTER(SamplerState), F, C.c_int64, C.POINTER(C.c_uint32),
                                      C.c_int64]),
            "or_stage_top_p": (C.c_int64, [C.POINTER(C.c_uint32), F, C.c_int64, C.c_float]),
            "or_stage_min_p": (C.c_int64, [C.POINTER(C.c_uint32), F, C.c_int64, C.c_float]),
            "or_stage_typical_p": (C.c_int64, [C.POINTER(C.c_uint32), F, C.c_int64, C.c_float]),
            "or_stage_top_n_sigma": (C.c_int64, [C.POINTER(C.c_uint32), F, C.c_int64, C.c_float]),
            "or_stage_xtc": (C.c_int64, [C.POINTER(C.c_uint32), F, C.c_int64, C.c_float, C.c_float, C.c_float]),
            "or_stage_temperature": (None, [F, C.c_int64, C.c_float]),
            "or_dynamic_temperature": (C.c_float, [F, C.c_int64, C.c_float, C.c_float, C.c_float]),
            "or_stage_penalties": (None, [C.POINTER(C.c_uint32), F, C.c_int64, C.POINTER(C.c_uint32), C.c_int64, C.c_float, C.c_float, C.c_float,
                                          C.c_uint32]),
            "or_stage_dry": (None, [C.POINTER(C.c_uint32), F, C.c_int64, C.POINTER(C.c_uint32), C.c_int64, C.c_float, C.c_float, C.c_uint32,
                                    C.c_uint32, C.POINTER(C.c_uint32), C.c_uint32]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(L, n)
            fn.restype = r
            fn.argtypes = a
        _lib = L
    return _lib


def _f(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def dequant(ggml_type: int, data: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    data = np.ascontiguousarray(data).view(np.uint8)
    if lib().or_dequant(ggml_type, data.ctypes.data_as(C.c_void_p), n, _f(out)):
        raise ValueError("or_dequant rejected the input")
    return out


def quantize_q8k(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    nb = x.size // 256
    blocks = (Q8KBlock * nb)()
    lib().or_quantize_q8k(_f(x), x.size, blocks)
    d = np.array([b.d for b in blocks], np.float32)
    qs = np.array([list(b.qs) for b in blocks], np.int8)
    bs = np.array([list(b.bsums) for b in blocks], np.int16)
    return d, qs, bs


def gemv(ggml_type: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    w = np.ascontiguousarray(w).view(np.uint8)
    y = np.empty((x.shape[0], rows), np.float32)
    for t in range(x.shape[0]):
        xt = np.ascontiguousarray(x[t])
        yt = np.empty(rows, np.float32)
        if lib().or_gemv(ggml_type, w.ctypes.data_as(C.c_void_p), rows, cols, _f(xt), _f(yt)):
            raise ValueError("or_gemv rejected the input")
        y[t] = yt
    return y


def row_bytes(ggml_type: int, n: int) -> int:
    return int(lib().or_row_bytes(ggml_type, n))


def synth_tensor(name: str, ggml_type: int, ne: tuple, mean: float, seed: int, sigma: float = 0.02) -> np.ndarray:
    """The seeded synthetic tensor `name` (ggml dims `ne`, innermost first) as GGUF bytes."""
    n = 1
    for d in ne:
        n *= d
    cols = ne[0]
    nbytes = (n // cols) * row_bytes(ggml_type, cols) if ggml_type in (OR_Q4_K, OR_Q6_K) else n * (4 if ggml_type == OR_F32 else 2)
    buf = np.empty(nbytes, np.uint8)
    if lib().or_synth_tensor(ggml_type, n // cols, cols, seed, lib().or_tensor_id(name.encode()), mean, sigma,
                             buf.ctypes.data_as(C.c_void_p)):
        raise ValueError(f"or_synth_tensor rejected {name}")
    return buf


def synth_model(specs, seed: int, sigma: float = 0.02) -> dict:
    """name -> (type, dims, bytes) for (name, type, dims, mean) specs, without the product library."""
    return {name: (ty, ne, synth_tensor(name, ty, ne, mean, seed, sigma)) for name, ty, ne, mean in specs}


def exp(x: float) -> float:
    return lib().or_exp(x)


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def softmax(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().or_softmax(_f(x), x.size, _f(out))
    return out


def route(probs, k):
    p = np.ascontiguousarray(probs, np.float32)
    ids = np.empty(k, np.int32)
    w = np.empty(k, np.float32)
    lib().or_route(_f(p), p.size, k, ids.ctypes.data_as(C.POINTER(C.c_int32)), _f(w))
    return ids, w


def ggml_rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().or_ggml_rmsnorm(_f(x), _f(w), x.size, eps, _f(out))
    return out


def ggml_gemv(ggml_type: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w).view(np.uint8)
    y = np.empty(rows, np.float32)
    if lib().or_ggml_gemv(ggml_type, w.ctypes.data_as(C.c_void_p), rows, cols, _f(x), _f(y)):
        raise ValueError("or_ggml_gemv rejected the input")
    return y


def ggml_softmax(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().or_ggml_softmax(_f(x), x.size, _f(out))
    return out


def ggml_attn_head(q, k16, v16, nk, scale, f32_acc=False):
    q = np.ascontiguousarray(q, np.float32)
    k16 = np.ascontiguousarray(k16, np.uint16)
    v16 = np.ascontiguousarray(v16, np.uint16)
    out = np.empty(q.size, np.float32)
    u16 = C.POINTER(C.c_uint16)
    lib().or_ggml_attn_head(_f(q), k16.ctypes.data_as(u16), v16.ctypes.data_as(u16), k16.shape[1], nk, q.size, scale,
                            int(f32_acc), _f(out))
    return out


def argmax(logits) -> int:
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().or_argmax(_f(x), x.size))


def rmsnorm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().or_rmsnorm(_f(x), _f(w), x.size, eps, _f(out))
    return out


def rope_table(n_pos, n_rot, base):
    out = np.empty((n_pos, n_rot), np.float32)
    lib().or_rope_table(n_pos, n_rot, base, _f(out))
    return out


def attn_head(q, k16, v16, nk, scale, chunk=128):
    """one query head over f16 keys/values [nk, head_dim] (uint16 bit patterns)"""
    q = np.ascontiguousarray(q, np.float32)
    k16 = np.ascontiguousarray(k16, np.uint16)
    v16 = np.ascontiguousarray(v16, np.uint16)
    out = np.empty(q.size, np.float32)
    u16 = C.POINTER(C.c_uint16)
    lib().or_attn_head(_f(q), k16.ctypes.data_as(u16), v16.ctypes.data_as(u16), k16.shape[1], nk, q.size, scale,
                       chunk, _f(out))
    return out


class Model:
    """The whole qwen3moe decode path on the CPU: forward_cached over a contiguous f16 cache."""

    def __init__(self, cfg, tensors: dict, numerics: int = NUM_CONTRACT):
        c = Config(cfg.n_layer, cfg.n_embd, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.n_expert,
                   cfg.n_expert_used, cfg.n_ff_exp, cfg.n_vocab, cfg.head_dim, cfg.rms_eps, cfg.rope_freq_base,
                   cfg.expert_workers, ATTN_CHUNK, cfg.max_positions, numerics)
        self.cfg = cfg
        self._keep = []
        arr = (Tensor * len(tensors))()
        for i, (name, (ty, ne, data)) in enumerate(tensors.items()):
            nb = name.encode()
            data = np.ascontiguousarray(data)
            self._keep += [nb, data]
            arr[i].name = nb
            arr[i].type = ty
            for j in range(4):
                arr[i].ne[j] = ne[j] if j < len(ne) else 1
            arr[i].data = data.ctypes.data_as(C.c_void_p)
        self._arr = arr
        self.h = lib().or_model_new(C.byref(c), arr, len(tensors))
        if not self.h:
            raise ValueError(lib().or_last_error().decode())
        self.kv = lib().or_kv_new(self.h)

    def close(self):
        if self.h:
            lib().or_kv_free(self.kv)
            lib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, pos_start: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(self.cfg.n_vocab, np.float32)
        if lib().or_forward(self.h, self.kv, t.ctypes.data_as(C.POINTER(C.c_int32)), t.size, pos_start, _f(out)):
            raise ValueError(lib().or_last_error().decode())
        return out

    def len(self) -> int:
        return lib().or_kv_len(self.kv)

    def set_len(self, n: int):
        lib().or_kv_set_len(self.kv, n)

    def kv_layer(self, layer: int, n_pos: int | None = None):
        n = self.len() if n_pos is None else n_pos
        kw = self.cfg.n_head_kv * self.cfg.head_dim
        k = np.empty(n * kw, np.uint16)
        v = np.empty(n * kw, np.uint16)
        u16 = C.POINTER(C.c_uint16)
        lib().or_kv_read(self.kv, layer, n, k.ctypes.data_as(u16), v.ctypes.data_as(u16))
        return k, v

    def write_kv_layer(self, layer: int, k: np.ndarray, v: np.ndarray):
        kw = self.cfg.n_head_kv * self.cfg.head_dim
        k = np.ascontiguousarray(k).view(np.uint16)
        v = np.ascontiguousarray(v).view(np.uint16)
        u16 = C.POINTER(C.c_uint16)
        lib().or_kv_write(self.kv, layer, k.size // kw, k.ctypes.data_as(u16), v.ctypes.data_as(u16))

    def topk(self, layer: int, t: int):
        K = self.cfg.n_expert_used
        ids = np.empty(K, np.int32)
        w = np.empty(K, np.float32)
        if lib().or_debug_topk(self.h, layer, t, ids.ctypes.data_as(C.POINTER(C.c_int32)), _f(w)):
            raise ValueError("no top-k capture")
        return ids, w

    def route_from(self, other):
        """take route()'s expert choice from `other`'s last forward (None: route itself)"""
        self._route_src = other
        lib().or_model_route_from(self.h, other.h if other is not None else None)

    def route_gap(self, layer: int, t: int) -> float:
        g = C.c_float()
        if lib().or_debug_route_gap(self.h, layer, t, C.byref(g)):
            raise ValueError("no route capture")
        return g.value

    def hidden(self, t: int) -> np.ndarray:
        out = np.empty(self.cfg.n_embd, np.float32)
        if lib().or_debug_hidden(self.h, t, _f(out)):
            raise ValueError("no hidden capture")
        return out

    def greedy(self, first_token: int, n_steps: int) -> list:
        """the chaos-run temp-0 loop: feed the argmax back n_steps times"""
        toks = []
        tok = first_token
        for _ in range(n_steps):
            logits = self.forward([tok], self.len())
            tok = argmax(logits)
            toks.append(tok)
        return toks


# ---------------------------------------------------------------- the token sampler (sample.c)
_LISTS = {"chain": (C.c_int32, np.int32), "bias_ids": (C.c_uint32, np.uint32),
          "bias_values": (C.c_float, np.float32), "suppress_ids": (C.c_uint32, np.uint32),
          "dry_breakers": (C.c_uint32, np.uint32)}
_COUNTS = {"chain": "n_chain", "bias_ids": "n_bias", "suppress_ids": "n_suppress", "dry_breakers": "n_dry_breakers"}


def sampler_config(base: str = "default", **kw):
    """(SamplerConfig, keep-alive arrays): SamplerConfig::default() or llamacpp_defaults() with the
    fields in `kw` replaced. List fields (chain, bias_ids, bias_values, suppress_ids, dry_breakers)
    take sequences; `chain=None` means the default chain."""
    c = SamplerConfig()
    (lib().or_sampler_config_llamacpp if base == "llamacpp" else lib().or_sampler_config_default)(C.byref(c))
    keep = []
    for k, v in kw.items():
        if k in _LISTS:
            if v is None:
                continue
            ct, nt = _LISTS[k]
            a = np.ascontiguousarray(np.asarray(v, dtype=nt))
            keep.append(a)
            setattr(c, k, a.ctypes.data_as(C.POINTER(ct)) if a.size else C.cast(C.pointer(ct()), C.POINTER(ct)))
            if k in _COUNTS:
                setattr(c, _COUNTS[k], int(a.size))
        else:
            setattr(c, k, v)
    return c, keep


def sampler_state(cfg) -> SamplerState:
    st = SamplerState()
    lib().or_sampler_init(C.byref(cfg), C.byref(st))
    return st


def sample(cfg, st: SamplerState, logits, history=()) -> int:
    """Sampler::sample (sample.rs:474-680); advances `st` as the reference's Sampler does"""
    lg = np.ascontiguousarray(np.asarray(logits, dtype=np.float32))
    h = np.ascontiguousarray(np.asarray(history, dtype=np.uint32))
    r = lib().or_sample(C.byref(cfg), C.byref(st), _f(lg), lg.size, h.ctypes.data_as(C.POINTER(C.c_uint32)), h.size)
    if r < 0:
        raise ValueError(lib().or_last_error().decode())
    return int(r)


def _cand(c):
    ids = np.ascontiguousarray(np.array([x[0] for x in c], dtype=np.uint32))
    vals = np.ascontiguousarray(np.array([x[1] for x in c], dtype=np.float32))
    return ids, vals


def _u32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def stage(name: str, cands, *args):
    """run one stage function on a list of (id, value) pairs; returns the new list"""
    ids, vals = _cand(cands)
    fn = getattr(lib(), "or_stage_" + name)
    n = fn(_u32p(ids), _f(vals), ids.size, *args)
    return [(int(i), float(v)) for i, v in zip(ids[:n], vals[:n])]


def stage_temperature(cands, t: float):
    ids, vals = _cand(cands)
    lib().or_stage_temperature(_f(vals), vals.size, t)
    return [(int(i), float(v)) for i, v in zip(ids, vals)]


def dynamic_temperature(cands, t: float, rng: float, ex: float) -> float:
    _, vals = _cand(cands)
    return float(lib().or_dynamic_temperature(_f(vals), vals.size, t, rng, ex))


def stage_penalties(cands, history, repeat, frequency, presence, last_n):
    ids, vals = _cand(cands)
    h = np.ascontiguousarray(np.asarray(history, dtype=np.uint32))
    lib().or_stage_penalties(_u32p(ids), _f(vals), ids.size, _u32p(h), h.size, repeat, frequency, presence, last_n)
    return [(int(i), float(v)) for i, v in zip(ids, vals)]


def stage_dry(cands, history, multiplier, base, allowed, last_n, breakers=()):
    ids, vals = _cand(cands)
    h = np.ascontiguousarray(np.asarray(history, dtype=np.uint32))
    b = np.ascontiguousarray(np.asarray(breakers, dtype=np.uint32))
    lib().or_stage_dry(_u32p(ids), _f(vals), ids.size, _u32p(h), h.size, multiplier, base, allowed, last_n,
                       _u32p(b), b.size)
    return [(int(i), float(v)) for i, v in zip(ids, vals)]


def ln(x: float) -> float:
    return float(lib().or_ln(x))


def pow_(x: float, y: float) -> float:
    return float(lib().or_pow(x, y))

"""Host-side mirror of the reference's decode interface over the C ABI.

`StreamingRunner.forward_cached(cache, tokens, pos_start)` and `KvCache` keep the names,
argument meaning and error behaviour of core/arch/src/stream.rs:1933-1975 and
core/arch/src/kv.rs:114-338, so callers (and tests) read like the reference's. Everything
runs on the GPU through libbigtea_decode.so; there is no host compute path.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _lib
from ._lib import BtError, check, lib
from .models import Qwen3MoeConfig, synth_model, tensor_views


class Engine:
    """StreamingRunner::new + load_resident: the model resident in HBM on one GPU."""

    def __init__(self, cfg: Qwen3MoeConfig, tensors: dict | None = None, *, seed: int | None = None,
                 sigma: float = 0.02, device: int = 0):
        self.cfg = cfg
        self.h = C.c_void_p()
        self._caches = weakref.WeakSet()
        d = cfg.desc()
        if tensors is not None:
            arr, _keep = tensor_views(tensors)
            check(lib.bt_engine_create(C.byref(d), arr, len(tensors), device, C.byref(self.h)))
        else:
            if seed is None:
                raise ValueError("give tensors or a synthetic seed")
            types = cfg.flat_layer_types()
            check(lib.bt_engine_create_synthetic(C.byref(d), _lib.ptr(types, C.c_uint32), cfg.embd_type,
                                                 cfg.out_type, seed, sigma, device, C.byref(self.h)))
            if cfg.router_zipf > 0:  # the same bias synth_model puts in the tensor set
                from .models import zipf_router_bias

                for il in range(cfg.n_layer):
                    self.set_router_bias(il, zipf_router_bias(cfg.n_expert, il, seed, cfg.router_zipf))

    @classmethod
    def synthetic(cls, cfg: Qwen3MoeConfig, seed: int, sigma: float = 0.02, device: int = 0) -> "Engine":
        return cls(cfg, seed=seed, sigma=sigma, device=device)

    def close(self):
        # a KV pool belongs to its engine: release the pools first
        for c in list(self._caches):
            c.close()
        if self.h:
            lib.bt_engine_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def stats(self) -> dict:
        s = _lib.Stats()
        check(lib.bt_engine_stats(self.h, C.byref(s)))
        return {k: getattr(s, k) for k, _ in s._fields_}

    def tensor_bytes(self, name: str, nbytes: int) -> np.ndarray:
        out = np.empty(nbytes, dtype=np.uint8)
        check(lib.bt_engine_tensor_bytes(self.h, name.encode(), _lib.ptr(out), nbytes))
        return out

    def enable_expert_cache(self, cache_bytes: int, policy: str = "freq"):
        """Move the experts to pinned host memory and serve them through an HBM cache of
        cache_bytes ("lru" or "freq": the reference's frequency-gated admission)."""
        pol = {"lru": _lib.XCACHE_LRU, "freq": _lib.XCACHE_FREQ}[policy]
        check(lib.bt_engine_enable_expert_cache(self.h, int(cache_bytes), pol))

    def expert_cache_stats(self) -> dict:
        s = _lib.XCacheStats()
        check(lib.bt_expert_cache_stats(self.h, C.byref(s)))
        d = {k: getattr(s, k) for k, _ in s._fields_}
        n = d["hits"] + d["misses"]
        d["hit_rate"] = d["hits"] / n if n else 0.0
        return d

    def set_router_bias(self, layer: int, bias):
        """Set (or, with None, remove) layer's router bias: one F32 value per expert, added to
        the router logits before the softmax."""
        if bias is None:
            check(lib.bt_engine_set_router_bias(self.h, layer, None, 0))
            return
        b = np.ascontiguousarray(bias, dtype=np.float32)
        check(lib.bt_engine_set_router_bias(self.h, layer, _lib.ptr(b, C.c_float), b.size))

    def bench_experts(self, T: int, n_iters: int = 20, seed: int = 1, kernel: int = 0, out: bool = False):
        """(ms per pass over every layer, weight bytes per pass) of the routed experts' arithmetic
        alone at T tokens a layer (bt_bench_experts): kernel 0 the decode step's per-layer
        kernels, kernel 1 the multi-layer stream kernel. With out=True a third element is the last
        layer's expert sum, [T][n_embd] f32."""
        ms, nb = C.c_double(), C.c_uint64()
        o = np.empty((T, self.cfg.n_embd), np.float32) if out else None
        check(lib.bt_bench_experts(self.h, T, n_iters, seed, kernel, C.byref(ms), C.byref(nb),
                                   _lib.ptr(o, C.c_float) if out else None))
        return (ms.value, nb.value, o) if out else (ms.value, nb.value)

    def set_option(self, name: str, value: int):
        check(lib.bt_set_option(self.h, name.encode(), int(value)))

    def enable_ep(self, unique_id: bytes, rank: int, n_ranks: int):
        """Join an expert-parallel group of n_ranks engines, one per GPU and process: this rank
        computes experts [rank*NE/n, (rank+1)*NE/n) for every rank's tokens, with the rows
        exchanged over NCCL. Collective: all ranks call it with the same unique_id (from
        ep_unique_id() on one rank), then run the same sequence of steps."""
        buf = (C.c_uint8 * len(unique_id)).from_buffer_copy(unique_id)
        check(lib.bt_engine_enable_ep(self.h, buf, len(unique_id), int(rank), int(n_ranks)))

    def enable_ep_torch(self, group=None):
        """enable_ep over an initialised torch.distributed process group (any backend): rank 0's
        unique id is shared through the group, then every rank joins."""
        import torch.distributed as dist

        self.enable_ep(share_ep_unique_id(group), dist.get_rank(group), dist.get_world_size(group))

    def debug_topk(self, layer: int, token: int):
        K = self.cfg.n_expert_used
        ids = np.empty(K, np.int32)
        w = np.empty(K, np.float32)
        check(lib.bt_debug_topk(self.h, layer, token, _lib.ptr(ids, C.c_int32), _lib.ptr(w, C.c_float)))
        return ids, w

    def debug_hidden(self, token: int) -> np.ndarray:
        out = np.empty(self.cfg.n_embd, np.float32)
        check(lib.bt_debug_hidden(self.h, token, _lib.ptr(out, C.c_float)))
        return out


class KvCache:
    """KvCache over a paged device pool. Sequence 0 is the reference's single cache; the
    others serve batched decode. Byte layouts follow kv.rs: [pos][n_kv_heads*head_dim] f16."""

    def __init__(self, engine: Engine, max_positions: int, max_seqs: int = 1):
        self.engine = engine
        self.h = C.c_void_p()
        self.max_positions = max_positions
        self.max_seqs = max_seqs
        check(lib.bt_kv_create(engine.h, _lib.KV_F16, max_seqs, max_positions, 16, C.byref(self.h)))
        engine._caches.add(self)

    def close(self):
        if self.h and self.engine.h:
            lib.bt_kv_destroy(self.h)
        self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def per_position(self) -> int:
        c = self.engine.cfg
        return c.n_head_kv * c.head_dim

    def len(self, seq: int = 0) -> int:
        n = C.c_uint32()
        check(lib.bt_kv_len(self.h, seq, C.byref(n)))
        return n.value

    def is_empty(self, seq: int = 0) -> bool:
        return self.len(seq) == 0

    def bytes(self) -> int:
        n = C.c_uint64()
        check(lib.bt_kv_bytes(self.h, C.byref(n)))
        return n.value

    def clear(self, seq: int = 0):
        check(lib.bt_kv_clear(self.h, seq))

    def truncate_to(self, n: int, seq: int = 0):
        check(lib.bt_kv_truncate(self.h, seq, n))

    def shift_out(self, keep: int, drop: int, seq: int = 0):
        check(lib.bt_kv_shift_out(self.h, seq, keep, drop))

    def set_positions(self, n: int, seq: int = 0):
        check(lib.bt_kv_set_positions(self.h, seq, n))

    def is_consistent(self, seq: int = 0) -> bool:
        ok = C.c_int()
        check(lib.bt_kv_is_consistent(self.h, seq, C.byref(ok)))
        return bool(ok.value)

    def _export(self, layer: int, seq: int, n_pos: int):
        nb = n_pos * self.per_position * 2
        k = np.empty(nb, np.uint8)
        v = np.empty(nb, np.uint8)
        check(lib.bt_kv_export_layer(self.h, seq, layer, _lib.ptr(k), _lib.ptr(v), nb))
        return k, v

    def keys(self, layer: int, seq: int = 0, n_pos: int | None = None) -> np.ndarray:
        return self._export(layer, seq, self.len(seq) if n_pos is None else n_pos)[0]

    def values(self, layer: int, seq: int = 0, n_pos: int | None = None) -> np.ndarray:
        return self._export(layer, seq, self.len(seq) if n_pos is None else n_pos)[1]

    def layer_bytes(self, layer: int, seq: int = 0, n_pos: int | None = None):
        return self._export(layer, seq, self.len(seq) if n_pos is None else n_pos)

    def restore_layer(self, layer: int, k: np.ndarray, v: np.ndarray, seq: int = 0):
        k = np.ascontiguousarray(k).view(np.uint8)
        v = np.ascontiguousarray(v).view(np.uint8)
        if k.nbytes != v.nbytes:
            raise BtError(_lib.BT_ERR_KV, "k and v differ in size")
        check(lib.bt_kv_import_layer(self.h, seq, layer, _lib.ptr(k), _lib.ptr(v), k.nbytes))


def simulate_expert_cache(policy: str, capacity: int, trace: np.ndarray, device: bool = False,
                          n_expert: int | None = None) -> dict:
    """The expert-cache policy alone on a selection trace [steps, layers, n_sel]: on the host
    (bt_expert_cache_simulate), or through the device lookup kernel (device=True)."""
    tr = np.ascontiguousarray(trace, dtype=np.int32)
    steps, n_layer, n_sel = tr.shape
    s = _lib.XCacheStats()
    pol = {"lru": _lib.XCACHE_LRU, "freq": _lib.XCACHE_FREQ}[policy]
    fn = lib.bt_expert_cache_simulate_device if device else lib.bt_expert_cache_simulate
    ne = n_expert if n_expert is not None else int(tr.max()) + 1
    check(fn(pol, capacity, n_layer, ne, n_sel, _lib.ptr(tr, C.c_int32), steps, C.byref(s)))
    return {k: getattr(s, k) for k, _ in s._fields_}


def ep_unique_id() -> bytes:
    """An NCCL unique id for Engine.enable_ep (made on one rank, shared with the others)."""
    buf = (C.c_uint8 * 128)()
    check(lib.bt_ep_unique_id(buf, 128))
    return bytes(buf)


def share_ep_unique_id(group=None) -> bytes:
    """Rank 0 of the torch.distributed group makes the unique id; every rank returns it."""
    import torch.distributed as dist

    obj = [ep_unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def pinned_empty(shape, dtype=np.float32) -> np.ndarray:
    """An uninitialised array in page-locked host memory (bt_host_alloc), freed with the array:
    bt_forward copies logits straight into such an output buffer."""
    dt = np.dtype(dtype)
    n = int(np.prod(shape)) * dt.itemsize
    p = C.c_void_p()
    check(lib.bt_host_alloc(max(n, 1), C.byref(p)))
    buf = (C.c_uint8 * max(n, 1)).from_address(p.value)
    arr = np.frombuffer(buf, dtype=dt, count=int(np.prod(shape))).reshape(shape)
    weakref.finalize(buf, lib.bt_host_free, C.c_void_p(p.value))
    return arr


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint32))


class StreamingRunner:
    """forward_cached over the device engine (stream.rs:1933-1975)."""

    def __init__(self, engine: Engine):
        self.engine = engine

    def forward_cached(self, cache: KvCache, tokens, pos_start: int, seq: int = 0, out=None) -> np.ndarray:
        """One step of `tokens` at `pos_start` for sequence `seq`: logits of the last position
        (into `out`, shape (1, n_vocab) float32, when given; page-locked from pinned_empty saves
        a host copy)."""
        return self.forward_batch(cache, [seq], [list(tokens)], [pos_start], out=out)[0]

    def forward_batch(self, cache: KvCache, seqs, token_lists, pos_starts, out=None) -> np.ndarray:
        V = self.engine.cfg.n_vocab
        ns = len(seqs)
        if ns == 1:  # the per-token decode loop: one sequence, no list flattening
            toks = np.array(token_lists[0], dtype=np.uint32).reshape(-1)
            n = np.array([toks.size], np.uint32)
        else:
            toks = _u32([t for tl in token_lists for t in tl])
            n = _u32([len(tl) for tl in token_lists])
        s = np.array(seqs, dtype=np.uint32)
        ps = np.array(pos_starts, dtype=np.uint32)
        if out is None:
            out = np.empty((ns, V), np.float32)
        elif out.shape != (ns, V) or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {(ns, V)}")
        check(lib.bt_forward(self.engine.h, cache.h, s.ctypes.data, toks.ctypes.data, n.ctypes.data, ps.ctypes.data,
                             ns, out.ctypes.data))
        return out

    def generate_greedy(self, cache: KvCache, first_tokens, n_steps: int, seqs=None, want_logits: bool = False):
        """The chaos-run temp-0 loop on the device; returns tokens [n_steps, n_seqs]."""
        first = _u32(first_tokens)
        seqs = _u32(range(len(first)) if seqs is None else seqs)
        out = np.empty((n_steps, len(first)), np.uint32)
        logits = np.empty((len(first), self.engine.cfg.n_vocab), np.float32) if want_logits else None
        check(lib.bt_generate_greedy(self.engine.h, cache.h, _lib.ptr(seqs, C.c_uint32), _lib.ptr(first, C.c_uint32),
                                     len(first), n_steps, _lib.ptr(out, C.c_uint32),
                                     _lib.ptr(logits, C.c_float) if want_logits else None))
        return (out, logits) if want_logits else out

    def last_device_ms(self) -> float:
        ms = C.c_double()
        check(lib.bt_last_device_ms(self.engine.h, C.byref(ms)))
        return ms.value

    def profile_decode(self, cache: KvCache, first_tokens, n_steps: int, seqs=None) -> dict:
        first = _u32(first_tokens)
        seqs = _u32(range(len(first)) if seqs is None else seqs)
        cap = 128
        arr = (_lib.KernelTime * cap)()
        n = C.c_uint32()
        check(lib.bt_profile_decode(self.engine.h, cache.h, _lib.ptr(seqs, C.c_uint32), _lib.ptr(first, C.c_uint32),
                                    len(first), n_steps, arr, cap, C.byref(n)))
        return {arr[i].name.decode(): (arr[i].launches, arr[i].total_ms) for i in range(min(n.value, cap))}


_SAMPLER_LISTS = {"chain": (C.c_int32, np.int32, "n_chain"), "bias_ids": (C.c_uint32, np.uint32, "n_bias"),
                  "bias_values": (C.c_float, np.float32, None), "suppress_ids": (C.c_uint32, np.uint32, "n_suppress"),
                  "dry_breakers": (C.c_uint32, np.uint32, "n_dry_breakers")}
STAGES = {"top_k": 0, "typical_p": 1, "top_p": 2, "min_p": 3, "xtc": 4, "temperature": 5}
DEFAULT_CHAIN = [0, 1, 2, 3, 4, 5]  # SamplerStage::default_chain (sample.rs:70-79)
_STAGE_SPELLINGS = {"top_k": 0, "topk": 0, "typ_p": 1, "typical": 1, "typical_p": 1, "typ": 1, "top_p": 2, "topp": 2,
                    "min_p": 3, "minp": 3, "xtc": 4, "temperature": 5, "temp": 5}


def parse_stage(name: str):
    """SamplerStage::parse (sample.rs:56-67): llama.cpp's spellings, trimmed, any case; None for
    anything else, so that a caller can refuse the whole chain."""
    return _STAGE_SPELLINGS.get(name.strip().lower())


def parse_chain(names: str):
    """a `--samplers`-style list separated by ';' or ','; ValueError on an unknown stage"""
    out = []
    for part in names.replace(",", ";").split(";"):
        if not part.strip():
            continue
        st = parse_stage(part)
        if st is None:
            raise ValueError(f"unknown sampler stage {part.strip()!r}")
        out.append(st)
    return out


class Sampler:
    """Sampler (core/arch/src/sample.rs:306-680) for a batch of sequences, on the device.

    `config` fields are SamplerConfig's (`base="llamacpp"` starts from llamacpp_defaults());
    `chain` takes stage numbers, llama.cpp's names (SamplerStage::parse) or one string of them
    separated by ';'. One state per sequence, advanced as the reference's Sampler is; `sample`
    returns one token per sequence. Construction is host work; `sample` runs on the device."""

    def __init__(self, engine: Engine, n_seqs: int = 1, base: str = "default", **config):
        self.engine = engine
        self.cfg = _lib.SamplerConfig()
        (lib.bt_sampler_config_llamacpp if base == "llamacpp" else lib.bt_sampler_config_default)(C.byref(self.cfg))
        self._keep = []
        for k, v in config.items():
            if k in _SAMPLER_LISTS:
                if v is None:
                    continue
                ct, nt, count = _SAMPLER_LISTS[k]
                if k == "chain":
                    if isinstance(v, str):
                        v = parse_chain(v)
                    else:
                        v = [x if not isinstance(x, str) else parse_stage(x) for x in v]
                        if any(x is None for x in v):
                            raise ValueError("unknown sampler stage in the chain")
                a = np.ascontiguousarray(np.asarray(v, dtype=nt))
                if a.size == 0:
                    a = np.zeros(1, nt)[:0]
                self._keep.append(a)
                setattr(self.cfg, k, C.cast(a.ctypes.data, C.POINTER(ct)))
                if count:
                    setattr(self.cfg, count, int(a.size))
            else:
                setattr(self.cfg, k, v)
        self.states = (_lib.SamplerState * n_seqs)()
        for i in range(n_seqs):
            check(lib.bt_sampler_init(C.byref(self.cfg), C.byref(self.states[i])))

    def sample(self, logits=None, histories=None) -> np.ndarray:
        """One token per sequence. `logits` None samples the engine's logits of its last forward
        (no copy to the host); else a host array [n_seqs, n_vocab]. `histories`: one token list
        per sequence (the tokens so far), or None."""
        n = len(self.states)
        if logits is not None:
            logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(n, -1)
        hl = np.array([len(h) for h in histories] if histories is not None else [0] * n, np.uint32)
        hist = (np.concatenate([_u32(h) for h in histories]) if histories is not None and hl.sum()
                else np.zeros(1, np.uint32))
        out = np.empty(n, np.uint32)
        check(lib.bt_sample(self.engine.h, C.byref(self.cfg), self.states, n,
                            _lib.ptr(logits, C.c_float) if logits is not None else None,
                            _lib.ptr(hist, C.c_uint32), _lib.ptr(hl, C.c_uint32), _lib.ptr(out, C.c_uint32)))
        return out


def dequantize(ggml_type: int, data: np.ndarray, n: int) -> np.ndarray:
    """dequantize() (core/ggml/src/lib.rs:233-290) through the device kernels."""
    out = np.empty(n, np.float32)
    data = np.ascontiguousarray(data).view(np.uint8)
    check(lib.bt_debug_dequant(ggml_type, _lib.ptr(data), n, _lib.ptr(out, C.c_float)))
    return out


def gemv(ggml_type: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """One quantised mul_mat on the device: y[t, r] = W[r, :] . x[t, :]."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    T = x.shape[0]
    y = np.empty((T, rows), np.float32)
    w = np.ascontiguousarray(w).view(np.uint8)
    check(lib.bt_op_gemv(ggml_type, _lib.ptr(w), rows, cols, _lib.ptr(x, C.c_float), T, _lib.ptr(y, C.c_float)))
    return y

"""qwen3moe shapes, the tensor set of the decode layer, and seeded synthetic weights.

Hyper-parameters follow Qwen3Config::from_model (core/arch/src/qwen3.rs:565-844): the GGUF
keys `qwen3moe.embedding_length`, `.attention.head_count(_kv)`, `.attention.key_length`,
`.expert_count`, `.expert_used_count`, `.expert_feed_forward_length`, `.rope.freq_base`,
`.attention.layer_norm_rms_epsilon`, `.block_count`, `.vocab_size`. Tensor names are the ones
Qwen3Model::required_tensors lists for an MoE block (qwen3.rs:1003-1123).

Synthetic weights are N(mean, sigma) values (an Irwin-Hall(4) approximation) quantised by
this package's own K-quant quantiser; the bytes come from bt_synth_tensor on the host and are
identical to what bt_engine_create_synthetic generates on the device.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field, replace

import numpy as np

from . import _lib
from ._lib import TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, check, lib
from .gguf import GGUFReader, GGUFWriter, tensor_nbytes

# order of the per-layer type list (bt_engine_create_synthetic)
LAYER_QUANT_TENSORS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate_exps", "ffn_up_exps",
                       "ffn_down_exps")


@dataclass
class Qwen3MoeConfig:
    n_layer: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_expert: int
    n_expert_used: int
    n_ff_exp: int
    n_vocab: int
    rms_eps: float = 1e-6
    rope_freq_base: float = 1e6
    expert_workers: int = 4
    max_positions: int = 4096
    embd_type: int = TYPE_Q6_K
    out_type: int = TYPE_Q6_K
    layer_types: list = field(default_factory=list)  # per layer: 7 ggml types (LAYER_QUANT_TENSORS)
    name: str = "qwen3moe"
    # > 0: each layer carries an F32 router bias ffn_gate_inp.bias = log-Zipf(router_zipf)
    # expert popularity over a seeded per-layer permutation of the expert ranks (zipf_router_bias)
    router_zipf: float = 0.0
    # > 0: one shared expert of this width per layer (ffn_{gate,up,down}_shexp, the routed
    # experts' types), added unweighted to the routed sum (DeepSeek-style models)
    n_ff_shexp: int = 0

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = [[TYPE_Q4_K] * 7 for _ in range(self.n_layer)]

    @property
    def n_rot(self) -> int:
        return self.head_dim

    def desc(self) -> _lib.ModelDesc:
        return _lib.ModelDesc(self.n_layer, self.n_embd, self.n_head, self.n_head_kv, self.head_dim,
                              self.n_expert, self.n_expert_used, self.n_ff_exp, self.n_vocab, self.n_rot,
                              self.rms_eps, self.rope_freq_base, self.expert_workers, self.max_positions,
                              self.n_ff_shexp)

    def tensor_specs(self):
        """(name, ggml type, ggml dims innermost-first, mean) for every tensor."""
        E, QW, KW = self.n_embd, self.n_head * self.head_dim, self.n_head_kv * self.head_dim
        F, NE, V, D = self.n_ff_exp, self.n_expert, self.n_vocab, self.head_dim
        out = [("token_embd.weight", self.embd_type, (E, V), 0.0),
               ("output_norm.weight", TYPE_F32, (E,), 1.0),
               ("output.weight", self.out_type, (E, V), 0.0)]
        for il in range(self.n_layer):
            t = self.layer_types[il]
            p = f"blk.{il}."
            out += [(p + "attn_norm.weight", TYPE_F32, (E,), 1.0),
                    (p + "attn_q.weight", t[0], (E, QW), 0.0),
                    (p + "attn_k.weight", t[1], (E, KW), 0.0),
                    (p + "attn_v.weight", t[2], (E, KW), 0.0),
                    (p + "attn_q_norm.weight", TYPE_F32, (D,), 1.0),
                    (p + "attn_k_norm.weight", TYPE_F32, (D,), 1.0),
                    (p + "attn_output.weight", t[3], (QW, E), 0.0),
                    (p + "ffn_norm.weight", TYPE_F32, (E,), 1.0),
                    (p + "ffn_gate_inp.weight", TYPE_F32, (E, NE), 0.0),
                    (p + "ffn_gate_exps.weight", t[4], (E, F, NE), 0.0),
                    (p + "ffn_up_exps.weight", t[5], (E, F, NE), 0.0),
                    (p + "ffn_down_exps.weight", t[6], (F, E, NE), 0.0)]
            if self.router_zipf > 0:
                out.append((p + "ffn_gate_inp.bias", TYPE_F32, (NE,), 0.0))
            if self.n_ff_shexp:
                FS = self.n_ff_shexp
                out += [(p + "ffn_gate_shexp.weight", t[4], (E, FS), 0.0),
                        (p + "ffn_up_shexp.weight", t[5], (E, FS), 0.0),
                        (p + "ffn_down_shexp.weight", t[6], (FS, E), 0.0)]
        return out

    def weight_bytes(self) -> int:
        tot = 0
        for _, ty, ne, _ in self.tensor_specs():
            n = 1
            for d in ne:
                n *= d
            tot += tensor_nbytes(ty, n)
        return tot

    def flat_layer_types(self) -> np.ndarray:
        return np.asarray(self.layer_types, dtype=np.uint32).reshape(-1)

    @classmethod
    def from_gguf(cls, r: GGUFReader, max_positions: int = 4096) -> "Qwen3MoeConfig":
        a = r.arch_value
        n_embd = int(a("embedding_length"))
        n_head = int(a("attention.head_count"))
        t = r.tensors
        n_layer = int(a("block_count"))
        types = [[t[f"blk.{il}.{n}.weight"].type for n in LAYER_QUANT_TENSORS] for il in range(n_layer)]
        out = t.get("output.weight", t["token_embd.weight"])
        return cls(n_layer=n_layer, n_embd=n_embd, n_head=n_head,
                   n_head_kv=int(a("attention.head_count_kv", n_head)),
                   head_dim=int(a("attention.key_length", n_embd // n_head)),
                   n_expert=int(a("expert_count")), n_expert_used=int(a("expert_used_count")),
                   n_ff_exp=int(a("expert_feed_forward_length")),
                   n_vocab=int(a("vocab_size", t["token_embd.weight"].ne[1])),
                   rms_eps=float(a("attention.layer_norm_rms_epsilon", 1e-6)),
                   rope_freq_base=float(a("rope.freq_base", 10000.0)),
                   max_positions=max_positions, embd_type=t["token_embd.weight"].type, out_type=out.type,
                   layer_types=types, name=r.arch(),
                   n_ff_shexp=int(a("expert_shared_feed_forward_length", 0)) if "blk.0.ffn_gate_shexp.weight" in t else 0,
                   router_zipf=0.0)


def q4km_layer_types(n_layer: int):
    """A documented stand-in for llama.cpp's Q4_K_M mix: attn_v and ffn_down_exps in Q6_K on
    every other layer (even indices), everything else Q4_K."""
    out = []
    for il in range(n_layer):
        t = [TYPE_Q4_K] * 7
        if il % 2 == 0:
            t[2] = TYPE_Q6_K
            t[6] = TYPE_Q6_K
        out.append(t)
    return out


QWEN3_30B_A3B = dict(n_embd=2048, n_head=32, n_head_kv=4, head_dim=128, n_expert=128, n_expert_used=8,
                     n_ff_exp=768, n_vocab=151936, rms_eps=1e-6, rope_freq_base=1e6)

CONFIGS = {
    # a small shape for fast parity tests: GQA 4, 16 experts, top-4
    "tiny": Qwen3MoeConfig(n_layer=2, n_embd=512, n_head=8, n_head_kv=2, head_dim=128, n_expert=16,
                           n_expert_used=4, n_ff_exp=256, n_vocab=1000, max_positions=1024, name="tiny"),
    # the reference's CPU-runnable case: qwen3moe, 2 layers, Qwen3-30B-A3B dims, Q4_K + Q6_K embd/output
    "cfg0": Qwen3MoeConfig(n_layer=2, max_positions=1024, name="cfg0", **QWEN3_30B_A3B),
    # the full 48-layer Qwen3-30B-A3B shape, Q4_K_M stand-in
    "cfg1": Qwen3MoeConfig(n_layer=48, max_positions=8192 + 512, layer_types=q4km_layer_types(48),
                           name="cfg1", **QWEN3_30B_A3B),
    # DeepSeek-style: 43 layers, hidden 4096, 32 heads / 8 KV heads, 256 routed experts top-6
    # plus one shared expert, expert width 2048, vocab 129280; Q4_K experts, Q6_K attention
    "cfg3": Qwen3MoeConfig(n_layer=43, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_expert=256,
                           n_expert_used=6, n_ff_exp=2048, n_vocab=129280, n_ff_shexp=2048,
                           max_positions=4096 + 512, layer_types=[[TYPE_Q6_K] * 4 + [TYPE_Q4_K] * 3] * 43,
                           name="cfg3"),
    # small shapes with a shared expert for parity tests
    "tiny_sh": Qwen3MoeConfig(n_layer=2, n_embd=512, n_head=8, n_head_kv=2, head_dim=128, n_expert=16,
                              n_expert_used=4, n_ff_exp=256, n_vocab=1000, max_positions=1024, n_ff_shexp=512,
                              name="tiny_sh"),
}


def config(name: str, **over) -> Qwen3MoeConfig:
    c = CONFIGS[name]
    c = replace(c, layer_types=[list(x) for x in c.layer_types])
    return replace(c, **over) if over else c


def tensor_id(name: str) -> int:
    return int(lib.bt_tensor_id(name.encode()))


def synth_tensor(name: str, ggml_type: int, ne: tuple, mean: float, seed: int, sigma: float = 0.02) -> np.ndarray:
    n = 1
    for d in ne:
        n *= d
    buf = np.empty(tensor_nbytes(ggml_type, n), dtype=np.uint8)
    rows, cols = n // ne[0], ne[0]
    check(lib.bt_synth_tensor(ggml_type, rows, cols, seed, tensor_id(name), mean, sigma, _lib.ptr(buf)))
    return buf


def zipf_router_bias(n_expert: int, layer: int, seed: int, s: float) -> np.ndarray:
    """A router bias giving expert e of a layer the log-popularity of Zipf(s) at its rank:
    bias[e] = -s * ln(rank(e)), the ranks 1..n_expert a seeded permutation per layer."""
    rank = np.random.default_rng([seed, layer, 0x2F1B]).permutation(n_expert) + 1
    return (-s * np.log(rank.astype(np.float64))).astype(np.float32)


def synth_model(cfg: Qwen3MoeConfig, seed: int, sigma: float = 0.02) -> dict:
    """name -> (ggml type, dims, uint8 bytes) for every tensor of `cfg`."""
    out = {}
    for name, ty, ne, mean in cfg.tensor_specs():
        if name.endswith("ffn_gate_inp.bias"):
            layer = int(name.split(".")[1])
            out[name] = (ty, ne, zipf_router_bias(cfg.n_expert, layer, seed, cfg.router_zipf).view(np.uint8))
        else:
            out[name] = (ty, ne, synth_tensor(name, ty, ne, mean, seed, sigma))
    return out


def write_gguf(path: str, cfg: Qwen3MoeConfig, tensors: dict) -> None:
    w = GGUFWriter(path)
    arch = "qwen3moe"
    w.add("general.architecture", arch)
    w.add("general.name", f"synthetic-{cfg.name}")
    w.add("general.alignment", 32)
    for k, v in [("block_count", cfg.n_layer), ("embedding_length", cfg.n_embd),
                 ("attention.head_count", cfg.n_head), ("attention.head_count_kv", cfg.n_head_kv),
                 ("attention.key_length", cfg.head_dim), ("attention.value_length", cfg.head_dim),
                 ("expert_count", cfg.n_expert), ("expert_used_count", cfg.n_expert_used),
                 ("expert_feed_forward_length", cfg.n_ff_exp), ("vocab_size", cfg.n_vocab),
                 ("context_length", cfg.max_positions)]:
        w.add(f"{arch}.{k}", int(v))
    if cfg.n_ff_shexp:
        w.add(f"{arch}.expert_shared_feed_forward_length", int(cfg.n_ff_shexp))
    w.add(f"{arch}.rope.freq_base", float(cfg.rope_freq_base))
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", float(cfg.rms_eps))
    for name, (ty, ne, data) in tensors.items():
        w.add_tensor(name, ne, ty, data)
    w.write()


def read_gguf(path: str, max_positions: int = 4096):
    r = GGUFReader(path)
    cfg = Qwen3MoeConfig.from_gguf(r, max_positions=max_positions)
    tensors = {n: (t.type, t.ne, t.data) for n, t in r.tensors.items()}
    return cfg, tensors


def tensor_views(tensors: dict):
    """A ctypes TensorView array over `tensors` (kept alive by the returned tuple)."""
    names = []
    arr = (_lib.TensorView * len(tensors))()
    for i, (name, (ty, ne, data)) in enumerate(tensors.items()):
        nb = name.encode()
        names.append(nb)
        v = arr[i]
        v.name = nb
        v.type = ty
        v.n_dims = len(ne)
        for k in range(4):
            v.ne[k] = ne[k] if k < len(ne) else 1
        data = np.ascontiguousarray(data)
        v.data = data.ctypes.data_as(C.c_void_p)
        v.nbytes = data.nbytes
    return arr, names

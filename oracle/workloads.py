"""The benchmark workloads' model shapes, restated for the CPU arm (TEST INFRASTRUCTURE).

The CPU reference arm of bench.py builds its model from this description and the oracle's
seeded generator, so it never loads the product library. The shapes are the reference's
qwen3moe hyper-parameters (Qwen3Config::from_model, core/arch/src/qwen3.rs:565-844) at the
Qwen3-30B-A3B size, and the tensor list is Qwen3Model::required_tensors for an MoE block
(qwen3.rs:1003-1123). tests/test_oracle.py checks that every field and every tensor spec equals
the product's own description (bigtea_b200.models).
"""
from __future__ import annotations

from dataclasses import dataclass, field

OR_F32, OR_Q4_K, OR_Q6_K = 0, 12, 14


def q4km_layer_types(n_layer: int):
    """The Q4_K_M stand-in: attn_v and ffn_down_exps in Q6_K on even layers, the rest Q4_K (7 types
    per layer: attn_q, attn_k, attn_v, attn_output, ffn_gate_exps, ffn_up_exps, ffn_down_exps)."""
    return [[OR_Q4_K, OR_Q4_K, OR_Q6_K if il % 2 == 0 else OR_Q4_K, OR_Q4_K, OR_Q4_K, OR_Q4_K,
             OR_Q6_K if il % 2 == 0 else OR_Q4_K] for il in range(n_layer)]


@dataclass
class Workload:
    name: str
    n_layer: int
    n_embd: int = 2048
    n_head: int = 32
    n_head_kv: int = 4
    head_dim: int = 128
    n_expert: int = 128
    n_expert_used: int = 8
    n_ff_exp: int = 768
    n_vocab: int = 151936
    rms_eps: float = 1e-6
    rope_freq_base: float = 1e6
    expert_workers: int = 4
    max_positions: int = 4096
    embd_type: int = OR_Q6_K
    out_type: int = OR_Q6_K
    layer_types: list = field(default_factory=list)

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = [[OR_Q4_K] * 7 for _ in range(self.n_layer)]

    def tensor_specs(self):
        """(name, ggml type, ggml dims innermost-first, mean) for every tensor."""
        E, QW, KW = self.n_embd, self.n_head * self.head_dim, self.n_head_kv * self.head_dim
        F, NE, V, D = self.n_ff_exp, self.n_expert, self.n_vocab, self.head_dim
        out = [("token_embd.weight", self.embd_type, (E, V), 0.0),
               ("output_norm.weight", OR_F32, (E,), 1.0),
               ("output.weight", self.out_type, (E, V), 0.0)]
        for il, t in enumerate(self.layer_types):
            p = f"blk.{il}."
            out += [(p + "attn_norm.weight", OR_F32, (E,), 1.0),
                    (p + "attn_q.weight", t[0], (E, QW), 0.0),
                    (p + "attn_k.weight", t[1], (E, KW), 0.0),
                    (p + "attn_v.weight", t[2], (E, KW), 0.0),
                    (p + "attn_q_norm.weight", OR_F32, (D,), 1.0),
                    (p + "attn_k_norm.weight", OR_F32, (D,), 1.0),
                    (p + "attn_output.weight", t[3], (QW, E), 0.0),
                    (p + "ffn_norm.weight", OR_F32, (E,), 1.0),
                    (p + "ffn_gate_inp.weight", OR_F32, (E, NE), 0.0),
                    (p + "ffn_gate_exps.weight", t[4], (E, F, NE), 0.0),
                    (p + "ffn_up_exps.weight", t[5], (E, F, NE), 0.0),
                    (p + "ffn_down_exps.weight", t[6], (F, E, NE), 0.0)]
        return out

    def shape_name(self) -> str:
        mix = ", Q4_K_M stand-in" if any(OR_Q6_K in t for t in self.layer_types) else ", Q4_K"
        return f"Qwen3-30B-A3B shape, {self.n_layer} layers" + mix


def workload(name: str, **over) -> Workload:
    if name == "cfg0":
        w = Workload(name="cfg0", n_layer=2, max_positions=1024)
    elif name == "cfg1":
        w = Workload(name="cfg1", n_layer=48, max_positions=8192 + 512, layer_types=q4km_layer_types(48))
    else:
        raise KeyError(f"no CPU-arm workload {name}")
    for k, v in over.items():
        setattr(w, k, v)
    return w

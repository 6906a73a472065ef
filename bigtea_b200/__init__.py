"""bigtea_b200 -- the B200 decode-step layer of a GGUF mixture-of-experts model.

A drop-in for Chaos's qwen3moe decode path (core/arch/src/stream.rs forward_cached): f16
paged KV append, GQA flash-decode, fused router top-k and the Q4_K/Q6_K expert FFN, as
sm_100a kernels behind the C ABI in include/bigtea_decode.h. Importing the package loads
libbigtea_decode.so and fails if it is missing: there is no CPU fallback.
"""
from ._lib import BtError, lib  # noqa: F401  (loads the library: fails loudly if absent)
from .models import CONFIGS, Qwen3MoeConfig, config, synth_model, write_gguf, read_gguf  # noqa: F401
from .runner import Engine, KvCache, Sampler, StreamingRunner, dequantize, ep_unique_id, gemv, pinned_empty  # noqa: F401

__all__ = ["Engine", "KvCache", "Sampler", "StreamingRunner", "Qwen3MoeConfig", "CONFIGS", "config", "synth_model",
           "write_gguf", "read_gguf", "dequantize", "gemv", "ep_unique_id", "BtError"]

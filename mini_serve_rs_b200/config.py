"""Model configurations (the fields of src/backends/qwen2.rs:9-54 the step reads)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional


@dataclass
class ModelConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_position_embeddings: int
    head_dim: Optional[int] = None
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    qk_norm: bool = True
    attention_bias: bool = False
    tie_word_embeddings: bool = True

    def hd(self) -> int:
        return self.head_dim or self.hidden_size // self.num_attention_heads


def qwen3_0_6b() -> ModelConfig:
    return ModelConfig(151936, 1024, 3072, 28, 16, 8, 40960, 128, 1e6, 1e-6, True, False, True)


def qwen2_5_7b() -> ModelConfig:
    return ModelConfig(152064, 3584, 18944, 28, 28, 4, 32768, 128, 1e6, 1e-6, False, True, False)


def weight_shapes(cfg) -> Dict[str, tuple]:
    """Hugging Face tensor names and shapes of a Qwen2/Qwen3 checkpoint."""
    d, h = cfg.hd(), cfg.hidden_size
    out = {"model.embed_tokens.weight": (cfg.vocab_size, h), "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        out["lm_head.weight"] = (cfg.vocab_size, h)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = (h,)
        out[p + "post_attention_layernorm.weight"] = (h,)
        out[p + "self_attn.q_proj.weight"] = (cfg.num_attention_heads * d, h)
        out[p + "self_attn.k_proj.weight"] = (cfg.num_key_value_heads * d, h)
        out[p + "self_attn.v_proj.weight"] = (cfg.num_key_value_heads * d, h)
        out[p + "self_attn.o_proj.weight"] = (h, cfg.num_attention_heads * d)
        if cfg.attention_bias:
            for n, k in (("q", cfg.num_attention_heads), ("k", cfg.num_key_value_heads),
                         ("v", cfg.num_key_value_heads)):
                out[p + f"self_attn.{n}_proj.bias"] = (k * d,)
        if cfg.qk_norm:
            out[p + "self_attn.q_norm.weight"] = (d,)
            out[p + "self_attn.k_norm.weight"] = (d,)
        out[p + "mlp.gate_proj.weight"] = (cfg.intermediate_size, h)
        out[p + "mlp.up_proj.weight"] = (cfg.intermediate_size, h)
        out[p + "mlp.down_proj.weight"] = (h, cfg.intermediate_size)
    return out


def host_random_weights(cfg, seed: int, std: float = 0.02, norm_std: float = 0.0):
    """Seeded random-init weights on the host, regenerable on any machine:
    one numpy PCG64 stream walked in sorted-name order; matrices and biases
    N(0, std) in f32, norm weights 1 (+ N(0, norm_std)).  The committed
    transformers golden vectors were computed from weights drawn this way."""
    import numpy as np
    import torch
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name in sorted(weight_shapes(cfg)):
        shape = weight_shapes(cfg)[name]
        if name.endswith("norm.weight"):
            w = np.ones(shape, np.float32)
            if norm_std:
                w = w + rng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)
        else:
            w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
        out[name] = torch.from_numpy(w.astype(np.float32))
    return out


def iter_random_device_weights(cfg, seed: int, device: str = "cuda", std: float = 0.02):
    """As random_device_weights, one tensor at a time (so a 7B model never
    holds a full f32 copy on the device)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    shapes = weight_shapes(cfg)
    for name in sorted(shapes):
        if name.endswith("norm.weight"):
            yield name, torch.ones(shapes[name], dtype=torch.float32, device=device)
        else:
            yield name, torch.randn(shapes[name], generator=g, dtype=torch.float32, device=device) * std


def random_device_weights(cfg, seed: int, device: str = "cuda", std: float = 0.02):
    """Seeded random-init weights generated directly on the GPU (benchmarks):
    matrices and biases ~ N(0, std), norm weights 1."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for name in sorted(weight_shapes(cfg)):
        shape = weight_shapes(cfg)[name]
        if name.endswith("norm.weight"):
            out[name] = torch.ones(shape, dtype=torch.float32, device=device)
        else:
            out[name] = torch.randn(shape, generator=g, dtype=torch.float32, device=device) * std
    return out

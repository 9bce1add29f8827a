"""Case definitions and seeded inputs shared by gen_golden.py and the tests.

Inputs are regenerated from numpy PCG64 seeds (bit-identical on any
machine), so only the outputs are stored in golden.npz.
"""
from __future__ import annotations

import numpy as np

from oracle.qwen_ref import Config

# --- model cases -------------------------------------------------------------
# "sin_tiny" is the configuration and weight construction of the reference's
# tests/test_pretrained_numerics.rs:73-108 (VarMap-built, so no QK-norm, no
# bias, tied lm_head) with its three prompts (:103-107).
SIN_TINY = Config(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=128,
                  head_dim=8, rope_theta=1e6, rms_norm_eps=1e-6, qk_norm=False,
                  attention_bias=False, tie_word_embeddings=True)

# Qwen3-architecture miniature with the real head_dim (128) and GQA ratio (2).
QWEN3_SMALL = Config(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=4096,
                     head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6, qk_norm=True,
                     attention_bias=False, tie_word_embeddings=True)

# Qwen2.5-architecture miniature: q/k/v bias, untied lm_head, GQA ratio 7.
QWEN2_SMALL = Config(vocab_size=512, hidden_size=1792, intermediate_size=512, num_hidden_layers=2,
                     num_attention_heads=14, num_key_value_heads=2, max_position_embeddings=4096,
                     head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6, qk_norm=False,
                     attention_bias=True, tie_word_embeddings=False)


# Qwen2.5-7B's attention shape (hidden 3584, 28 query / 4 KV heads x 128, q/k/v
# bias, untied lm_head) on two layers with a small vocabulary and MLP: shards
# one KV head per rank at TP=4, as the 7B model does.
QWEN2_KV4 = Config(vocab_size=512, hidden_size=3584, intermediate_size=1024, num_hidden_layers=2,
                   num_attention_heads=28, num_key_value_heads=4, max_position_embeddings=4096,
                   head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6, qk_norm=False,
                   attention_bias=True, tie_word_embeddings=False)


def _prompt(seed: int, n: int, vocab: int):
    rng = np.random.Generator(np.random.PCG64(seed))
    return [int(t) for t in rng.integers(0, vocab, n)]


MODEL_CASES = [
    {"name": "sin_tiny", "cfg": SIN_TINY, "weights": "sin",
     "prompts": [[1, 2, 3], list(range(1, 18)), list(range(1, 34))], "decode_steps": 3},
    {"name": "qwen3_small", "cfg": QWEN3_SMALL, "weights": "random", "seed": 1234, "norm_std": 0.1,
     "prompts": [_prompt(11, 17, 1024), _prompt(12, 64, 1024), _prompt(13, 33, 1024)],
     "decode_steps": 8},
    {"name": "qwen2_small", "cfg": QWEN2_SMALL, "weights": "random", "seed": 4321,
     "prompts": [_prompt(21, 16, 512), _prompt(22, 31, 512)], "decode_steps": 6},
    {"name": "qwen2_kv4", "cfg": QWEN2_KV4, "weights": "random", "seed": 7007,
     "prompts": [_prompt(31, 20, 512), _prompt(32, 37, 512), _prompt(33, 50, 512)], "decode_steps": 6},
]

# --- kernel cases (scripts/validate_cuda_kernels.py:132-251) -----------------
RMSNORM_CASES = [(1, 128), (4, 128), (17, 128), (1, 1024), (4, 1024), (17, 1024)]
ATTN_SEQ_LENS = (1, 15, 16, 17, 31, 32, 33, 64, 128)
ATTN_FRAGMENTED_TABLE = [29, 3, 18, 0, 25, 11, 7, 14]
ATTN_RAGGED_LENS = (1, 15, 16, 17, 31, 32, 33)
ATTN_RAGGED_TABLES = [[7, 0, 0, 0], [7, 0, 0, 0], [7, 0, 0, 0], [7, 19, 0, 0],
                      [7, 12, 0, 0], [7, 12, 0, 0], [7, 12, 28, 0]]
ATTN_POOL_BLOCKS = 32
ATTN_HEADS, ATTN_KV_HEADS, ATTN_DIM = 16, 8, 128


def rmsnorm_inputs(rows: int, dim: int):
    rng = np.random.Generator(np.random.PCG64(1000 + rows * 7 + dim))
    x = rng.standard_normal((rows, dim), dtype=np.float32)
    w = rng.standard_normal(dim, dtype=np.float32)
    return x, w


def attn_inputs():
    """(q for the single-sequence cases [len(ATTN_SEQ_LENS), Hq, D], k_pool,
    v_pool [32, 8, 16, 128], q for the ragged batch [7, Hq, D]) in f32."""
    rng = np.random.Generator(np.random.PCG64(42))
    kp = rng.standard_normal((ATTN_POOL_BLOCKS, ATTN_KV_HEADS, 16, ATTN_DIM), dtype=np.float32)
    vp = rng.standard_normal((ATTN_POOL_BLOCKS, ATTN_KV_HEADS, 16, ATTN_DIM), dtype=np.float32)
    q1 = rng.standard_normal((len(ATTN_SEQ_LENS), ATTN_HEADS, ATTN_DIM), dtype=np.float32)
    qr = rng.standard_normal((len(ATTN_RAGGED_LENS), ATTN_HEADS, ATTN_DIM), dtype=np.float32)
    return q1, kp, vp, qr

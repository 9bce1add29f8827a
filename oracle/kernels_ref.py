"""fp32 CPU references for the individual kernels (test infrastructure only)."""
from __future__ import annotations

import math
from typing import Optional, Sequence

import numpy as np
import torch

from .qwen_ref import rms_norm, rotate_half, softmax_last


def paged_gqa_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                        block_tables: torch.Tensor, ctx_lens: Sequence[int], scale: float,
                        block_size: int = 16, row_table: Optional[Sequence[int]] = None) -> torch.Tensor:
    """Paged GQA attention of one query row per entry, in fp32.

    Gathers each row's pages as scripts/validate_cuda_kernels.py:29-46 does,
    then runs decode_attention_gqa_zero_copy (src/backends/qwen2.rs:182-203):
    q [R, Hq, D]; k_pool/v_pool [blocks, Hkv, bs, D]; block_tables [rows, mb].
    Returns fp32 [R, Hq, D].
    """
    R, hq, d = q.shape
    hkv = k_pool.shape[1]
    g = hq // hkv
    out = torch.zeros(R, hq, d, dtype=torch.float32)
    for r in range(R):
        L = int(ctx_lens[r])
        trow = r if row_table is None else int(row_table[r])
        pages = block_tables[trow, : (L + block_size - 1) // block_size].long()
        ks = k_pool[pages].permute(1, 0, 2, 3).reshape(hkv, -1, d)[:, :L].to(torch.float32)
        vs = v_pool[pages].permute(1, 0, 2, 3).reshape(hkv, -1, d)[:, :L].to(torch.float32)
        qr = q[r].to(torch.float32)
        for h in range(hkv):
            s = torch.matmul(qr[h * g:(h + 1) * g], ks[h].t()) * scale
            out[r, h * g:(h + 1) * g] = torch.matmul(softmax_last(s), vs[h])
    return out


def add_rmsnorm(x: torch.Tensor, r: Optional[torch.Tensor], w: torch.Tensor, eps: float):
    """Residual add then RMSNorm in the tensors' dtype, as the reference's
    decoder layer does (qwen2.rs:420-427 then 68-75).  Returns (resid, normed)."""
    resid = x if r is None else (x + r)
    return resid, rms_norm(resid, w, eps)


def qk_norm_rope(qkv: torch.Tensor, positions: Sequence[int], cos: torch.Tensor, sin: torch.Tensor,
                 num_heads: int, num_kv_heads: int, head_dim: int,
                 q_norm_w: Optional[torch.Tensor], k_norm_w: Optional[torch.Tensor],
                 bias: Optional[torch.Tensor], eps: float):
    """Per-token restatement of qwen2.rs:287-311 (bias, QK-norm, rotate-half
    RoPE) on a packed [T, (Hq + 2 Hkv) * D] projection.  Returns q, k, v
    [T, H*, D] in the input dtype."""
    T = qkv.shape[0]
    x = qkv if bias is None else qkv + bias
    q = x[:, : num_heads * head_dim].reshape(T, num_heads, head_dim)
    k = x[:, num_heads * head_dim:(num_heads + num_kv_heads) * head_dim].reshape(T, num_kv_heads, head_dim)
    v = x[:, (num_heads + num_kv_heads) * head_dim:].reshape(T, num_kv_heads, head_dim)
    if q_norm_w is not None:
        q = rms_norm(q, q_norm_w, eps)
    if k_norm_w is not None:
        k = rms_norm(k, k_norm_w, eps)
    pos = torch.as_tensor(list(positions), dtype=torch.long)
    c = torch.cat([cos[pos], cos[pos]], dim=-1).reshape(T, 1, head_dim)
    s = torch.cat([sin[pos], sin[pos]], dim=-1).reshape(T, 1, head_dim)
    q = q * c + rotate_half(q) * s
    k = k * c + rotate_half(k) * s
    return q, k, v


def silu_mul(gate_up: torch.Tensor, inter: int) -> torch.Tensor:
    """qwen2.rs:171-173 on a fused [T, 2I] gate|up projection."""
    g = gate_up[:, :inter]
    u = gate_up[:, inter:]
    dtype = gate_up.dtype
    gf = g.to(torch.float32)
    act = (gf / (1.0 + torch.exp(-gf))).to(dtype)
    return act * u


# ---- the kernels' 16-bit arithmetic: f32 inside, each stored value rounded once ----
# (Candle's half-precision path rounds after every op instead; the kernels
# keep f32 until the store, which puts them within half a unit in the last
# place of the f32 reference's value from the same inputs.)


def add_rmsnorm_once(x: torch.Tensor, r: Optional[torch.Tensor], w: torch.Tensor, eps: float):
    """K4 in the inputs' dtype: (round(x + r), round((x + r) / norm * w)) with
    the sum and the norm in f32."""
    dt = x.dtype
    s = x.to(torch.float32) + (0.0 if r is None else r.to(torch.float32))
    norm = torch.sqrt((s * s).mean(dim=-1, keepdim=True) + eps)
    return s.to(dt), (s / norm * w.to(torch.float32)).to(dt)


def qk_norm_rope_once(qkv: torch.Tensor, positions: Sequence[int], cos32: torch.Tensor, sin32: torch.Tensor,
                      num_heads: int, num_kv_heads: int, head_dim: int,
                      q_norm_w: Optional[torch.Tensor], k_norm_w: Optional[torch.Tensor],
                      bias: Optional[torch.Tensor], eps: float):
    """K5 in qkv's dtype: bias, QK-norm and RoPE (f32 tables) in f32, q/k/v
    rounded once."""
    dt = qkv.dtype
    f = lambda t: None if t is None else t.to(torch.float32)
    q, k, v = qk_norm_rope(qkv.to(torch.float32), positions, cos32.to(torch.float32), sin32.to(torch.float32),
                           num_heads, num_kv_heads, head_dim, f(q_norm_w), f(k_norm_w), f(bias), eps)
    return q.to(dt), k.to(dt), v.to(dt)


def silu_mul_once(gate_up: torch.Tensor, inter: int) -> torch.Tensor:
    """K6 in gate_up's dtype: silu(g) * u in f32, rounded once."""
    gf = gate_up[:, :inter].to(torch.float32)
    uf = gate_up[:, inter:].to(torch.float32)
    return (gf / (1.0 + torch.exp(-gf)) * uf).to(gate_up.dtype)


def ulp16(ref: torch.Tensor, dtype) -> torch.Tensor:
    """Spacing of `dtype` (bf16 / f16) at |ref|, per element."""
    mant = 7 if dtype == torch.bfloat16 else 10
    e = torch.floor(torch.log2(ref.abs().to(torch.float32).clamp(min=2.0 ** -14)))
    return torch.pow(2.0, e - mant)


def argmax_rows(logits: torch.Tensor) -> np.ndarray:
    """Row-wise first-index argmax (candle.rs:747-751)."""
    return torch.argmax(logits.to(torch.float32), dim=-1).to(torch.int32).numpy()


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)

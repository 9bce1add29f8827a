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


def argmax_rows(logits: torch.Tensor) -> np.ndarray:
    """Row-wise first-index argmax (candle.rs:747-751)."""
    return torch.argmax(logits.to(torch.float32), dim=-1).to(torch.int32).numpy()


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)

"""Numpy restatement of the ragged-batch metadata (test infrastructure only).

The reference builds, per step, the decode inputs on the host
(``src/backends/candle.rs:603-630``: input id = last output token,
position = prompt + outputs - 1) and the per-step RoPE positions
(``src/backends/qwen2.rs:649-655``); its K/V land in the slot
``block_table[pos // 16] * 16 + pos % 16`` of the prototype kernels' paged
layout (``docs/colab_cuda_kernels/mini_serve_kernels.cu:219-223``).  These
functions produce the same integers for a packed batch.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np


def pack(seqs: Sequence[Tuple[int, int, Sequence[int]]], block_size: int = 16,
         max_blocks_per_seq: int | None = None):
    """seqs: (num_tokens, start_pos, block_ids) per sequence in step order.

    Returns dict of int arrays: cu_seqlens [n+1] i32, positions [T] i32,
    slot_mapping [T] i64, row_ctx [T] i32 (= pos + 1), seq_of_token [T] i32,
    block_tables [n, max_blocks] i32 (zero padded), last_index [n] i32.
    """
    n = len(seqs)
    counts = np.array([s[0] for s in seqs], dtype=np.int64)
    cu = np.zeros(n + 1, dtype=np.int32)
    cu[1:] = np.cumsum(counts).astype(np.int32)
    T = int(cu[-1])
    mb = max_blocks_per_seq or max((len(s[2]) for s in seqs), default=1)
    tables = np.zeros((n, mb), dtype=np.int32)
    positions = np.zeros(T, dtype=np.int32)
    slots = np.zeros(T, dtype=np.int64)
    owner = np.zeros(T, dtype=np.int32)
    for i, (cnt, start, blocks) in enumerate(seqs):
        tables[i, :len(blocks)] = np.asarray(blocks, dtype=np.int32)
        pos = np.arange(start, start + cnt, dtype=np.int64)
        b = np.asarray(blocks, dtype=np.int64)
        if cnt and (pos[-1] // block_size) >= len(b):
            raise ValueError("block table too short for position %d" % pos[-1])
        positions[cu[i]:cu[i + 1]] = pos
        slots[cu[i]:cu[i + 1]] = b[pos // block_size] * block_size + pos % block_size
        owner[cu[i]:cu[i + 1]] = i
    return {"cu_seqlens": cu, "positions": positions, "slot_mapping": slots,
            "row_ctx": (positions + 1).astype(np.int32), "seq_of_token": owner,
            "block_tables": tables, "last_index": (cu[1:] - 1).astype(np.int32)}


def step_inputs(prompt_len: int, outputs: List[int], is_prefilled: bool, cached: int = 0):
    """Tokens the reference runs for one sequence in one step
    (candle.rs:430-551 prefill, 602-630 decode): returns (num_tokens, start_pos)."""
    if not is_prefilled:
        if cached >= prompt_len:  # exact prefix hit replays the last prompt token
            return 1, prompt_len - 1
        return prompt_len - cached, cached
    return 1, prompt_len + len(outputs) - 1

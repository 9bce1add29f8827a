"""Helpers shared by the GPU tests (tests only)."""
import ctypes as C

import numpy as np
import pytest
import torch

from mini_serve_rs_b200 import engine as E


def need_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")


# Device tensors handed to a launch stay referenced until the next sync_ok():
# a temporary like ptr(x.to(DEV)) would otherwise return its memory to the
# caching allocator while the kernel still reads it.
_KEEP = []


def ptr(t):
    if t is None:
        return C.c_void_p(0)
    _KEEP.append(t)
    return C.c_void_p(t.data_ptr())


def dt_code(t):
    return E.torch_dtype_code(t)


def max_abs(a, b):
    return float((a.to(torch.float32) - b.to(torch.float32)).abs().max().item())


def sync_ok(rc, what="launch"):
    torch.cuda.synchronize()
    _KEEP.clear()
    assert rc == 0, f"{what} returned {rc}"


def attention(q, k_pool, v_pool, block_tables, ctx, out, *, row_table=None, part=0, max_ctx=None):
    """Call ms_launch_paged_attention on torch CUDA tensors."""
    lib = E.lib()
    rows, hq, d = q.shape
    hkv = k_pool.shape[1]
    mctx = int(max_ctx if max_ctx is not None else int(ctx.max().item()))
    ws_bytes = lib.ms_attention_workspace_bytes(rows, hq, mctx, part, 16)
    if part <= 0:
        # mirror the launcher's own choice so the workspace is large enough
        ws_bytes = max(ws_bytes, rows * hq * ((mctx + 15) // 16) * (d * 4 + 8) + 256)
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)
    rc = lib.ms_launch_paged_attention(ptr(q), ptr(k_pool), ptr(v_pool), ptr(block_tables), block_tables.shape[1],
                                       ptr(row_table), ptr(ctx), rows, mctx, ptr(out), hq, hkv, d, 16,
                                       1.0 / np.sqrt(d), part, ptr(ws), ws.numel(), dt_code(q), None)
    sync_ok(rc, "ms_launch_paged_attention")

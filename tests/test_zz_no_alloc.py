"""The attention entry point that allocates nothing, against the one that does.

launch_paged_gqa_decode_tiled_bf16_noalloc exists for callers that may not
call cudaMalloc: a server whose allocator already holds the HBM budget for its
KV pages, or a hot path that cannot take the device-wide synchronisation an
allocation or free brings.  It keeps its split-K scratch in a fixed 16 MiB
buffer compiled into the library.  These checks call both entry points through
the C ABI on the same inputs, twice in a row with different inputs (the shared
buffer keeps the previous call's contents), and check that a batch needing
more than the fixed buffer is refused before anything runs.  This file is
collected last so that a stop-at-first-failure run has already run every
other test; it also passes alone in a fresh process.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from mini_serve_rs_b200 import engine as E

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
CUDA_ERROR_MEMORY_ALLOCATION = 2


def _case(seed, batch, max_blocks, pool):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    rng = np.random.Generator(np.random.PCG64(seed))
    ctx = rng.integers(1, max_blocks * 16 + 1, batch).astype(np.int32)
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((batch, max_blocks), np.int32)
    off = 0
    for b in range(batch):
        n = (int(ctx[b]) + 15) // 16
        tables[b, :n] = perm[off:off + n]
        off += n
    kp = torch.randn(pool, 8, 16, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
    vp = torch.randn(pool, 8, 16, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(batch, 16, 128, generator=gen, device=DEV, dtype=torch.bfloat16)
    return q, kp, vp, torch.from_numpy(tables).to(DEV), torch.from_numpy(ctx).to(DEV)


def _run(fn, q, kp, vp, tables, ctx):
    out = torch.full_like(q, float("nan"))
    p = lambda t: C.c_void_p(t.data_ptr())
    rc = fn(p(q), p(kp), p(vp), p(tables), p(ctx), p(out), q.shape[0], 16, 8, tables.shape[1],
            1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    assert rc == 0, rc
    return out


def test_no_alloc_attention_matches_allocating_entry_point_twice():
    assert torch.cuda.is_available()
    lib = E.lib()
    # two different calls back to back: config-2 shapes, then a smaller ragged batch
    for seed, batch, max_blocks, pool in ((11, 256, 256, 40000), (12, 37, 40, 2000)):
        q, kp, vp, tables, ctx = _case(seed, batch, max_blocks, pool)
        got = _run(lib.launch_paged_gqa_decode_tiled_bf16_noalloc, q, kp, vp, tables, ctx)
        want = _run(lib.launch_paged_gqa_decode_tiled_bf16, q, kp, vp, tables, ctx)
        assert torch.isfinite(got).all()
        # same tolerance the bf16 attention tests use
        assert (got.float() - want.float()).abs().max().item() <= 2e-2


def test_no_alloc_attention_refuses_batches_beyond_its_scratch():
    lib = E.lib()
    # 2048 sequences x 16 heads x 4 partitions x 520 B is far above 16 MiB; the
    # call must fail before touching any pointer
    rc = lib.launch_paged_gqa_decode_tiled_bf16_noalloc(None, None, None, None, None, None, 2048, 16, 8, 256,
                                                        1.0 / math.sqrt(128))
    assert rc == CUDA_ERROR_MEMORY_ALLOCATION
    assert lib.launch_paged_gqa_decode_tiled_bf16_noalloc(None, None, None, None, None, None, 0, 16, 8, 8, 1.0) != 0

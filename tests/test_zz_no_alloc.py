"""The attention entry point that allocates nothing, against the one that does.

launch_paged_gqa_decode_tiled_bf16_noalloc exists for callers that may not
call cudaMalloc: a server whose allocator already holds the HBM budget for its
KV pages, or a hot path that cannot take the device-wide synchronisation an
allocation or free brings.  It keeps its split-K scratch in a fixed 16 MiB
buffer compiled into the library.  These checks call both entry points through
the C ABI on the same inputs, twice in a row with different inputs (the shared
buffer keeps the previous call's contents): the two choose the same partition
and run the same kernel, so their outputs must be bit-identical, and both are
checked against an fp32 dense reference.  They also cover a batch that needs
no scratch at all, the largest batch that fits the buffer, the first one that
does not (refused before anything runs), and that only the first call on the
device changes the free device memory.  This file is collected last so that a
stop-at-first-failure run has already run every other test; it also passes
alone in a fresh process.
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
SCRATCH = 16 << 20
MiB = 1 << 20


def _partition(batch, max_blocks, kv_heads=8):
    """The launchers' split-K partition (pages) for this call shape: ~16 CTAs
    per SM over 148 SMs, at least 8 and at most 64 pages, a multiple of 4."""
    work = max(1, batch * max_blocks // 2) * kv_heads
    pb = -(-work // (148 * 16))
    pb = min(max(pb, 8), 64)
    return -(-pb // 4) * 4


def _scratch_need(batch, max_blocks, heads=16):
    parts = -(-max_blocks // _partition(batch, max_blocks))
    return 0 if parts <= 1 else batch * heads * parts * (128 * 4 + 8) + 256


def _case(seed, batch, max_blocks, pool, shared_pages=False):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    rng = np.random.Generator(np.random.PCG64(seed))
    ctx = rng.integers(1, max_blocks * 16 + 1, batch).astype(np.int32)
    tables = np.zeros((batch, max_blocks), np.int32)
    if shared_pages:  # rows may share pages (the kernel only reads them)
        tables[:] = (np.arange(batch)[:, None] * 131 + np.arange(max_blocks)[None, :] * 7) % pool
    else:
        perm = rng.permutation(pool).astype(np.int32)
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


def _fp32_reference(q, kp, vp, tables, ctx, rows):
    """Dense fp32 attention of the listed rows (16 query heads over 8 KV heads)."""
    out = {}
    for b in rows:
        n = int(ctx[b])
        pages = tables[b, :(n + 15) // 16].long()
        k = kp[pages].float().permute(1, 0, 2, 3).reshape(8, -1, 128)[:, :n]
        v = vp[pages].float().permute(1, 0, 2, 3).reshape(8, -1, 128)[:, :n]
        qq = q[b].float().reshape(8, 2, 128)
        s = torch.einsum("hgd,hnd->hgn", qq, k) / math.sqrt(128)
        out[b] = torch.einsum("hgn,hnd->hgd", torch.softmax(s, dim=-1), v).reshape(16, 128)
    return out


def test_no_alloc_attention_matches_allocating_entry_point_twice():
    assert torch.cuda.is_available()
    lib = E.lib()
    E.kernel_status(0)  # clear what earlier launches left
    # the allocating launcher first: its kernels and its own workspace are in place
    # before the free memory is read around the no-allocation calls
    cases = [(11, 256, 256, 40000), (12, 37, 40, 2000)]  # config-2 shapes, then a smaller ragged batch
    data = [_case(*c) for c in cases]
    want = [_run(lib.launch_paged_gqa_decode_tiled_bf16, *d) for d in data]
    for (seed, batch, mb, _), d in zip(cases, data):
        assert 0 < _scratch_need(batch, mb) <= SCRATCH
    free0 = torch.cuda.mem_get_info(0)[0]
    got0 = _run(lib.launch_paged_gqa_decode_tiled_bf16_noalloc, *data[0])
    free1 = torch.cuda.mem_get_info(0)[0]
    got1 = _run(lib.launch_paged_gqa_decode_tiled_bf16_noalloc, *data[1])
    free2 = torch.cuda.mem_get_info(0)[0]
    print(f"free device memory: first call {(free0 - free1) / MiB:.1f} MiB, second call {(free1 - free2) / MiB:.1f} MiB")
    # the first call on the device may load the buffer's module (16 MiB); later calls take nothing
    assert free0 - free1 <= SCRATCH + 4 * MiB
    assert free1 == free2
    for got, ref, d in ((got0, want[0], data[0]), (got1, want[1], data[1])):
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref)  # same partition, same kernel: bit-identical
        q, kp, vp, tables, ctx = d
        rows = range(0, q.shape[0], max(1, q.shape[0] // 24))
        for b, r in _fp32_reference(q, kp, vp, tables, ctx, rows).items():
            assert (got[b].float() - r).abs().max().item() <= 2e-2  # the bf16 attention tolerance
    assert E.kernel_status(0) == 0


def test_no_alloc_attention_without_split_and_at_the_scratch_limit():
    lib = E.lib()
    # one partition per row: no scratch used at all
    d = _case(13, 5, 4, 64)
    assert _scratch_need(5, 4) == 0
    assert torch.equal(_run(lib.launch_paged_gqa_decode_tiled_bf16_noalloc, *d),
                       _run(lib.launch_paged_gqa_decode_tiled_bf16, *d))
    # the largest batch at 4096-token capacity whose scratch fits the 16 MiB
    mb = 256
    batch = max(b for b in range(1, 1024) if _scratch_need(b, mb) <= SCRATCH)
    assert _scratch_need(batch, mb) > SCRATCH - 64 * 1024  # within 64 KiB of the limit
    d = _case(14, batch, mb, 4096, shared_pages=True)
    got = _run(lib.launch_paged_gqa_decode_tiled_bf16_noalloc, *d)
    assert torch.isfinite(got).all()
    assert torch.equal(got, _run(lib.launch_paged_gqa_decode_tiled_bf16, *d))
    # one more row needs more than the buffer: refused before any pointer is read
    rc = lib.launch_paged_gqa_decode_tiled_bf16_noalloc(None, None, None, None, None, None, batch + 1, 16, 8, mb,
                                                        1.0 / math.sqrt(128))
    assert rc == CUDA_ERROR_MEMORY_ALLOCATION
    assert E.kernel_status(0) == 0


def test_no_alloc_attention_refuses_batches_beyond_its_scratch():
    lib = E.lib()
    # 2048 sequences x 16 heads x 4 partitions x 520 B is far above 16 MiB; the
    # call must fail before touching any pointer
    rc = lib.launch_paged_gqa_decode_tiled_bf16_noalloc(None, None, None, None, None, None, 2048, 16, 8, 256,
                                                        1.0 / math.sqrt(128))
    assert rc == CUDA_ERROR_MEMORY_ALLOCATION
    assert lib.launch_paged_gqa_decode_tiled_bf16_noalloc(None, None, None, None, None, None, 0, 16, 8, 8, 1.0) != 0

"""K3p ragged causal prefill attention against an fp32 reference.

Restates the prefill branch of qwen2.rs:329-345 (causal mask of :476-503 with
the offset columns of a cached prefix) on the paged pool.  Pool pages outside
the written keys hold NaN so that any read of a stale key would show up.
Tolerance: 2e-2 max-abs for bf16 / f16 against fp32."""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from mini_serve_rs_b200 import engine as E
from tests.gpu_util import max_abs, need_gpu, ptr, sync_ok

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    need_gpu()


def _tiles(lib, chunks, hq, hkv):
    row0, ntok, start, trow = [], [], [], []
    r = 0
    for i, (st, n) in enumerate(chunks):
        row0.append(r), ntok.append(n), start.append(st), trow.append(i)
        r += n
    arr = lambda xs: (C.c_int32 * len(xs))(*xs)
    cap = sum(n for _, n in chunks)
    out = (C.c_int32 * (4 * cap))()
    n = lib.ms_prefill_tiles(arr(row0), arr(ntok), arr(start), arr(trow), len(chunks), hq, hkv, out, cap)
    assert n > 0
    return torch.tensor(list(out)[:4 * n], dtype=torch.int32, device=DEV), n


def _case(group, head_dim, dt, chunks, seed, pool=256, hkv=2):
    lib = E.lib()
    gen = torch.Generator().manual_seed(seed)
    hq = hkv * group
    T = sum(n for _, n in chunks)
    mb = max((st + n + 15) // 16 for st, n in chunks)
    perm = torch.randperm(pool, generator=gen)
    tables = torch.zeros(len(chunks), mb, dtype=torch.int32)
    kp = torch.full((pool, hkv, 16, head_dim), float("nan"), dtype=torch.float32)
    vp = torch.full((pool, hkv, 16, head_dim), float("nan"), dtype=torch.float32)
    keys, vals = [], []
    off = 0
    for i, (st, n) in enumerate(chunks):
        L = st + n
        nb = (L + 15) // 16
        tables[i, :nb] = perm[off:off + nb].to(torch.int32)
        off += nb
        k = torch.randn(L, hkv, head_dim, generator=gen)
        v = torch.randn(L, hkv, head_dim, generator=gen)
        pos = torch.arange(L)
        pages = tables[i, (pos // 16)].long()
        kp[pages, :, pos % 16] = k
        vp[pages, :, pos % 16] = v
        keys.append(k.to(dt).float())
        vals.append(v.to(dt).float())
    q = torch.randn(T, hq, head_dim, generator=gen).to(dt)
    # fp32 reference: row at position p of chunk i attends to keys 0..p
    want = torch.zeros(T, hq, head_dim)
    r = 0
    scale = 1.0 / math.sqrt(head_dim)
    for i, (st, n) in enumerate(chunks):
        kk, vv = keys[i], vals[i]
        for j in range(n):
            p = st + j
            for h in range(hq):
                s = (kk[:p + 1, h // group] @ q[r + j, h].float()) * scale
                want[r + j, h] = torch.softmax(s, dim=0) @ vv[:p + 1, h // group]
        r += n
    qd, kd, vd, td = q.to(DEV), kp.to(dt).to(DEV), vp.to(dt).to(DEV), tables.to(DEV)
    tiles, nt = _tiles(lib, chunks, hq, hkv)
    out = torch.full((T, hq, head_dim), float("nan"), dtype=dt, device=DEV)
    sync_ok(lib.ms_launch_paged_prefill(ptr(qd), ptr(kd), ptr(vd), ptr(td), mb, ptr(tiles), nt, ptr(out), hq, hkv,
                                        head_dim, 16, scale, E.torch_dtype_code(q), None), "prefill")
    assert torch.isfinite(out).all()
    return max_abs(out.cpu(), want)


@pytest.mark.parametrize("group,head_dim,dt", [(2, 128, torch.bfloat16), (1, 128, torch.bfloat16),
                                               (4, 128, torch.float16), (7, 128, torch.bfloat16),
                                               (8, 128, torch.bfloat16), (2, 64, torch.bfloat16),
                                               (7, 64, torch.float16)])
def test_prefill_matches_fp32_causal_reference(group, head_dim, dt):
    # fresh prompts, cached prefixes (offset columns), page-boundary lengths, one token
    chunks = [(0, 17), (16, 33), (37, 5), (0, 1), (100, 64), (0, 129)]
    assert _case(group, head_dim, dt, chunks, seed=group * 10 + head_dim) <= 2e-2


def test_prefill_long_chunk_with_prefix():
    assert _case(2, 128, torch.bfloat16, [(1000, 300), (0, 700)], seed=5, pool=256) <= 2e-2


def _case_large(group, head_dim, dt, chunks, seed, hkv=2):
    """As _case at bench scale: pages in a random permutation of a NaN-filled
    pool, fp32 reference computed with torch on the GPU (masked softmax per
    chunk and kv head)."""
    lib = E.lib()
    gen = torch.Generator(device=DEV).manual_seed(seed)
    hq = hkv * group
    T = sum(n for _, n in chunks)
    mb = max((st + n + 15) // 16 for st, n in chunks)
    pool = sum((st + n + 15) // 16 for st, n in chunks) + 7
    perm = torch.randperm(pool, device=DEV, generator=gen)
    tables = torch.zeros(len(chunks), mb, dtype=torch.int32, device=DEV)
    kp = torch.full((pool, hkv, 16, head_dim), float("nan"), dtype=dt, device=DEV)
    vp = torch.full_like(kp, float("nan"))
    q = torch.randn(T, hq, head_dim, generator=gen, device=DEV).to(dt)
    want = torch.empty(T, hq, head_dim, device=DEV)
    scale = 1.0 / math.sqrt(head_dim)
    off = r = 0
    for i, (st, n) in enumerate(chunks):
        L = st + n
        nb = (L + 15) // 16
        tables[i, :nb] = perm[off:off + nb].to(torch.int32)
        off += nb
        k = torch.randn(L, hkv, head_dim, generator=gen, device=DEV).to(dt)
        v = torch.randn(L, hkv, head_dim, generator=gen, device=DEV).to(dt)
        pos = torch.arange(L, device=DEV)
        pages = tables[i, pos // 16].long()
        kp[pages, :, pos % 16] = k
        vp[pages, :, pos % 16] = v
        qpos = st + torch.arange(n, device=DEV)
        mask = torch.arange(L, device=DEV)[None, :] > qpos[:, None]  # (n, L): key after the row's position
        for h in range(hkv):
            qh = q[r:r + n, h * group:(h + 1) * group].float()                 # (n, G, D)
            s = torch.einsum("ngd,ld->ngl", qh, k[:, h].float()) * scale
            s = s.masked_fill(mask[:, None, :], float("-inf"))
            want[r:r + n, h * group:(h + 1) * group] = torch.einsum("ngl,ld->ngd", torch.softmax(s, -1),
                                                                    v[:, h].float())
        r += n
    tiles, nt = _tiles(lib, chunks, hq, hkv)
    out = torch.full((T, hq, head_dim), float("nan"), dtype=dt, device=DEV)
    sync_ok(lib.ms_launch_paged_prefill(ptr(q), ptr(kp), ptr(vp), ptr(tables), mb, ptr(tiles), nt, ptr(out), hq,
                                        hkv, head_dim, 16, scale, E.torch_dtype_code(q), None), "prefill")
    assert torch.isfinite(out).all()
    return float((out.float() - want).abs().max())


@pytest.mark.parametrize("group,head_dim,dt", [(2, 128, torch.bfloat16), (7, 128, torch.bfloat16),
                                               (1, 64, torch.float16)])
def test_prefill_4096_token_prompts_against_torch_fp32(group, head_dim, dt):
    # a full 4096-token prompt, cached prefixes at offsets that are not multiples of 128 (or 16),
    # a chunk that starts past a page boundary: up to 257 key pages, ~36 tiles per sequence
    chunks = [(0, 4096), (513, 1536), (3001, 999), (16, 240)]
    assert _case_large(group, head_dim, dt, chunks, seed=group + head_dim) <= 2e-2

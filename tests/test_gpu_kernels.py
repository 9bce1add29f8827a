"""Kernel-level parity on the B200: each sm_100a kernel against the golden
vectors (reference validator functions) and the CPU oracle on the same seeded
inputs.  Tolerances: f32 atol 1e-5 / rtol 1e-4 and f16 5e-3 (the reference
validator's, scripts/validate_cuda_kernels.py:126-129); bf16 vs the fp32
reference 2e-2 max-abs for attention, the add + RMSNorm
and the QK-norm + RoPE outputs -- those two compute in f32 and round each
output once, so they are also held to one bf16 unit in the last place of the
once-rounded restatement; bit-exact for integer outputs."""
import math

import numpy as np
import pytest
import torch

from mini_serve_rs_b200 import engine as E
from oracle import kernels_ref
from oracle.packer_ref import pack
from oracle.qwen_ref import rms_norm, rope_tables
from tests.golden.golden_cases import (ATTN_FRAGMENTED_TABLE, ATTN_RAGGED_LENS, ATTN_RAGGED_TABLES,
                                       ATTN_SEQ_LENS, QWEN3_SMALL, RMSNORM_CASES, attn_inputs,
                                       rmsnorm_inputs)
from tests.golden.load import golden
from tests.gpu_util import attention, max_abs, need_gpu, ptr, sync_ok

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    need_gpu()
    torch.manual_seed(0)


# ---- RMSNorm ---------------------------------------------------------------------

@pytest.mark.parametrize("dt_name,dt,atol,rtol,fn", [
    ("f32", torch.float32, 1e-5, 1e-4, "launch_rmsnorm_f32"),
    ("f16", torch.float16, 5e-3, 5e-3, "launch_rmsnorm_f16")])
def test_rmsnorm_prototype_launchers_match_reference_validator(dt_name, dt, atol, rtol, fn):
    lib = E.lib()
    g = golden()
    for rows, dim in RMSNORM_CASES:
        x, w = rmsnorm_inputs(rows, dim)
        xt = torch.from_numpy(x).to(dt).to(DEV)
        wt = torch.from_numpy(w).to(dt).to(DEV)
        out = torch.empty_like(xt)
        sync_ok(getattr(lib, fn)(ptr(xt), ptr(wt), ptr(out), rows, dim, 1e-6), fn)
        want = torch.from_numpy(g[f"rmsnorm/{dt_name}/{rows}x{dim}"]).to(DEV)
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out.float(), want, atol=atol, rtol=rtol)


def test_add_rmsnorm_bf16_config3_shape():
    """T=8192 packed tokens, hidden 1024, bf16, x and residual
    ~ N(0,1), weights ~ 1 + N(0, 0.1)."""
    lib = E.lib()
    gen = torch.Generator().manual_seed(3)
    T, H = 8192, 1024
    x = torch.randn(T, H, generator=gen).to(torch.bfloat16)
    r = torch.randn(T, H, generator=gen).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=gen)).to(torch.bfloat16)
    xd, rd, wd = x.to(DEV), r.to(DEV), w.to(DEV)
    resid = torch.empty_like(xd)
    normed = torch.empty_like(xd)
    sync_ok(lib.ms_launch_add_rmsnorm(ptr(xd), ptr(rd), None, ptr(wd), ptr(resid), ptr(normed), T, H, 1e-6,
                                      E.MS_DTYPE_BF16, None))
    # residual: one bf16 rounding of the f32 sum, exactly as the reference's bf16 add
    want_resid, want_once = kernels_ref.add_rmsnorm_once(x, r, w, 1e-6)
    assert torch.equal(resid.cpu(), want_resid)
    # f32 inside, rounded once: within one bf16 ulp of the once-rounded restatement
    assert ((normed.cpu().float() - want_once.float()).abs() <= kernels_ref.ulp16(want_once, torch.bfloat16)).all()
    # against the fp32 reference path: the north-star bar, absolute
    _, want_f32 = kernels_ref.add_rmsnorm(x.float(), r.float(), w.float(), 1e-6)
    err = (normed.cpu().float() - want_f32).abs().max().item()
    print(f"K4 bf16 vs fp32: max-abs {err:.5f} (max |y| {want_f32.abs().max().item():.2f})")
    assert err <= 2e-2


def test_add_rmsnorm_row_gather_and_f32():
    lib = E.lib()
    gen = torch.Generator().manual_seed(4)
    T, H = 37, 256
    x = torch.randn(T, H, generator=gen)
    r = torch.randn(T, H, generator=gen)
    w = 1 + 0.1 * torch.randn(H, generator=gen)
    idx = torch.tensor([36, 0, 5, 5, 17], dtype=torch.int32)
    out = torch.empty(len(idx), H, device=DEV)
    sync_ok(lib.ms_launch_add_rmsnorm(ptr(x.to(DEV)), ptr(r.to(DEV)), ptr(idx.to(DEV)), ptr(w.to(DEV)), None,
                                      ptr(out), len(idx), H, 1e-6, E.MS_DTYPE_F32, None))
    _, want = kernels_ref.add_rmsnorm(x[idx.long()], r[idx.long()], w, 1e-6)
    torch.testing.assert_close(out.cpu(), want, atol=1e-5, rtol=1e-5)


# ---- paged GQA attention -----------------------------------------------------------

@pytest.mark.parametrize("dt_name,dt,atol,rtol,fn", [
    ("f32", torch.float32, 1e-5, 1e-4, "launch_paged_gqa_decode_tiled_f32"),
    ("f16", torch.float16, 5e-3, 5e-3, "launch_paged_gqa_decode_tiled_f16")])
def test_paged_attention_prototype_launchers_match_reference_validator(dt_name, dt, atol, rtol, fn):
    """The validator's cases (validate_cuda_kernels.py:162-251): boundary lengths
    over the fragmented table [29,3,18,0,25,11,7,14], then a ragged batch of 7
    sequences sharing physical pages 7 and 12."""
    lib = E.lib()
    g = golden()
    q1, kp, vp, qr = attn_inputs()
    kpd, vpd = torch.from_numpy(kp).to(dt).to(DEV), torch.from_numpy(vp).to(dt).to(DEV)
    table = torch.tensor([ATTN_FRAGMENTED_TABLE], dtype=torch.int32, device=DEV)
    scale = 1.0 / math.sqrt(128)
    for li, L in enumerate(ATTN_SEQ_LENS):
        q = torch.from_numpy(q1[li:li + 1]).to(dt).to(DEV)
        out = torch.empty_like(q)
        lens = torch.tensor([L], dtype=torch.int32, device=DEV)
        sync_ok(getattr(lib, fn)(ptr(q), ptr(kpd), ptr(vpd), ptr(table), ptr(lens), ptr(out), 1, 16, 8, 8, scale))
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out.float().cpu(), torch.from_numpy(g[f"paged_gqa/{dt_name}/len{L}"]),
                                   atol=atol, rtol=rtol)
    q = torch.from_numpy(qr).to(dt).to(DEV)
    out = torch.empty_like(q)
    tables = torch.tensor(ATTN_RAGGED_TABLES, dtype=torch.int32, device=DEV)
    lens = torch.tensor(ATTN_RAGGED_LENS, dtype=torch.int32, device=DEV)
    sync_ok(getattr(lib, fn)(ptr(q), ptr(kpd), ptr(vpd), ptr(tables), ptr(lens), ptr(out), 7, 16, 8, 4, scale))
    torch.testing.assert_close(out.float().cpu(), torch.from_numpy(g[f"paged_gqa/{dt_name}/ragged"]),
                               atol=atol, rtol=rtol)


def test_paged_attention_bf16_prototype_launcher_vs_fp32():
    lib = E.lib()
    q1, kp, vp, qr = attn_inputs()
    kb, vb = torch.from_numpy(kp).bfloat16(), torch.from_numpy(vp).bfloat16()
    q = torch.from_numpy(qr).bfloat16()
    tables = torch.tensor(ATTN_RAGGED_TABLES, dtype=torch.int32)
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=DEV)
    sync_ok(lib.launch_paged_gqa_decode_tiled_bf16(
        ptr(q.to(DEV)), ptr(kb.to(DEV)), ptr(vb.to(DEV)), ptr(tables.to(DEV)),
        ptr(torch.tensor(ATTN_RAGGED_LENS, dtype=torch.int32, device=DEV)), ptr(out), 7, 16, 8, 4,
        1.0 / math.sqrt(128)))
    want = kernels_ref.paged_gqa_attention(q.float(), kb.float(), vb.float(), tables, ATTN_RAGGED_LENS,
                                           1.0 / math.sqrt(128))
    assert max_abs(out.cpu(), want) <= 2e-2


@pytest.mark.parametrize("group,head_dim,dt", [(1, 128, torch.bfloat16), (2, 128, torch.float32),
                                               (4, 128, torch.bfloat16), (7, 128, torch.bfloat16),
                                               (8, 128, torch.float32), (2, 64, torch.bfloat16),
                                               (7, 64, torch.float32)])
def test_paged_attention_group_sizes_and_partitions(group, head_dim, dt):
    """Every compiled (group, head_dim) variant, with ragged lengths around page
    and partition boundaries and several forced partition sizes, against the
    fp32 oracle; results must not depend on the partition size."""
    gen = torch.Generator().manual_seed(100 + group * 7 + head_dim)
    hkv, pool = 2, 96
    hq = hkv * group
    lens = [1, 15, 16, 17, 33, 64, 65, 200, 511, 777]
    R = len(lens)
    kp = torch.randn(pool, hkv, 16, head_dim, generator=gen).to(dt)
    vp = torch.randn(pool, hkv, 16, head_dim, generator=gen).to(dt)
    q = torch.randn(R, hq, head_dim, generator=gen).to(dt)
    mb = (max(lens) + 15) // 16
    tables = torch.stack([torch.randperm(pool, generator=gen)[:mb] for _ in range(R)]).to(torch.int32)
    ctx = torch.tensor(lens, dtype=torch.int32)
    want = kernels_ref.paged_gqa_attention(q.float(), kp.float(), vp.float(), tables, lens,
                                           1.0 / math.sqrt(head_dim))
    tol = 2e-2 if dt == torch.bfloat16 else 2e-5
    outs = []
    for part in (0, 1, 4, 8, 64):
        out = torch.empty(q.shape, dtype=dt, device=DEV)
        attention(q.to(DEV), kp.to(DEV), vp.to(DEV), tables.to(DEV), ctx.to(DEV), out, part=part)
        assert max_abs(out.cpu(), want) <= tol, (part, max_abs(out.cpu(), want))
        outs.append(out.float().cpu())
    for o in outs[1:]:
        assert (o - outs[0]).abs().max().item() <= (1e-2 if dt == torch.bfloat16 else 1e-5)


def test_paged_attention_config2_full_size():
    """256 sequences, one query each, context ~ U[1, 4096],
    16/8 heads x 128, bf16, block tables a seeded random permutation of a
    70k-page pool, q/k/v ~ N(0,1), scale 1/sqrt(128); against an fp32 dense
    reference of the same op."""
    gen = torch.Generator(device=DEV).manual_seed(2)
    cg = torch.Generator().manual_seed(2)
    B, hq, hkv, D, pool = 256, 16, 8, 128, 70000
    ctx = torch.randint(1, 4097, (B,), generator=cg, dtype=torch.int32)
    mb = 256
    perm = torch.randperm(pool, generator=cg)
    nblk = (ctx + 15) // 16
    tables = torch.zeros(B, mb, dtype=torch.int32)
    off = 0
    for b in range(B):
        n = int(nblk[b])
        tables[b, :n] = perm[off:off + n].to(torch.int32)
        off += n
    kp = torch.randn(pool, hkv, 16, D, generator=gen, device=DEV, dtype=torch.bfloat16)
    vp = torch.randn(pool, hkv, 16, D, generator=gen, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(B, hq, D, generator=gen, device=DEV, dtype=torch.bfloat16)
    out = torch.empty_like(q)
    td, cd = tables.to(DEV), ctx.to(DEV)
    attention(q, kp, vp, td, cd, out)
    # fp32 dense reference, one sequence at a time on the device
    scale = 1.0 / math.sqrt(D)
    worst = 0.0
    for b in range(B):
        L = int(ctx[b])
        pages = td[b, :int(nblk[b])].long()
        k = kp[pages].permute(1, 0, 2, 3).reshape(hkv, -1, D)[:, :L].float()
        v = vp[pages].permute(1, 0, 2, 3).reshape(hkv, -1, D)[:, :L].float()
        qq = q[b].float().reshape(hkv, hq // hkv, D)
        p = torch.softmax(torch.einsum("hgd,hld->hgl", qq, k) * scale, dim=-1)
        ref = torch.einsum("hgl,hld->hgd", p, v).reshape(hq, D)
        worst = max(worst, (out[b].float() - ref).abs().max().item())
    assert worst <= 2e-2, worst
    # the prototype-compatible entry point gives the same answer
    out2 = torch.empty_like(q)
    sync_ok(E.lib().launch_paged_gqa_decode_tiled_bf16(ptr(q), ptr(kp), ptr(vp), ptr(td), ptr(cd), ptr(out2), B,
                                                       hq, hkv, mb, scale))
    assert max_abs(out2, out) <= 1e-2


# ---- QK-norm + RoPE + paged append -------------------------------------------------

def _config3_batch(gen):
    """8 prefill chunks of length U[256, 768] at consecutive positions starting
    at U[0, 8192 - len), the rest single decode tokens at U[0, 8192)."""
    T = 8192
    pos = []
    for _ in range(8):
        n = int(torch.randint(256, 769, (1,), generator=gen))
        s = int(torch.randint(0, 8192 - n, (1,), generator=gen))
        pos.extend(range(s, s + n))
    while len(pos) < T:
        pos.append(int(torch.randint(0, 8192, (1,), generator=gen)))
    return torch.tensor(pos[:T], dtype=torch.int32)


@pytest.mark.parametrize("dt,qk_norm,bias,hq,hkv", [(torch.bfloat16, True, False, 16, 8),
                                                    (torch.float32, True, False, 16, 8),
                                                    (torch.bfloat16, False, True, 16, 8),
                                                    (torch.bfloat16, False, True, 7, 1),
                                                    (torch.bfloat16, True, False, 14, 2)])
def test_qk_norm_rope_append_config3(dt, qk_norm, bias, hq, hkv):
    """BASELINE config 3's QK-norm + RoPE (theta 1e6) on 16/8 heads x 128 over a
    packed T=8192 batch; K and V must land in exactly their slot.  Also the head
    counts one tensor-parallel rank of Qwen2.5-7B holds (7/1 at TP=4 with q/k/v
    bias, 14/2 at TP=2), where a warp holds pair items of two kinds of head."""
    lib = E.lib()
    gen = torch.Generator().manual_seed(33)
    T, D = 8192, 128
    pos = _config3_batch(gen)
    qkv = torch.randn(T, (hq + 2 * hkv) * D, generator=gen).to(dt)
    qn = (1 + 0.1 * torch.randn(D, generator=gen)).to(dt) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, generator=gen)).to(dt) if qk_norm else None
    b = (0.1 * torch.randn((hq + 2 * hkv) * D, generator=gen)).to(dt) if bias else None
    cos, sin = rope_tables(QWEN3_SMALL, torch.float32, max_pos=8192)  # f32 tables in every mode
    pool = 640
    slots = torch.randperm(pool * 16, generator=gen)[:T].to(torch.int64)
    kp = torch.zeros(pool, hkv, 16, D, dtype=dt, device=DEV)
    vp = torch.zeros_like(kp)
    qo = torch.empty(T, hq, D, dtype=dt, device=DEV)
    dev = lambda t: None if t is None else t.to(DEV)
    sync_ok(lib.ms_launch_qk_norm_rope_append(ptr(qkv.to(DEV)), ptr(dev(b)), ptr(dev(qn)), ptr(dev(kn)),
                                              ptr(cos.to(DEV)), ptr(sin.to(DEV)), ptr(pos.to(DEV)),
                                              ptr(slots.to(DEV)), ptr(qo), ptr(kp), ptr(vp), T, hq, hkv, D, 16,
                                              1e-6, E.dt_code(qkv) if hasattr(E, "dt_code") else
                                              E.torch_dtype_code(qkv), None))
    wq, wk, wv = kernels_ref.qk_norm_rope_once(qkv, pos.tolist(), cos, sin, hq, hkv, D, qn, kn, b, 1e-6)
    blk, off = (slots // 16).long(), (slots % 16).long()
    got_k = kp.cpu()[blk, :, off]  # [T, hkv, D]
    got_v = vp.cpu()[blk, :, off]
    # f32 inside, one rounding per output: within one unit in the last place
    if dt == torch.bfloat16:
        for got, want in ((qo.cpu(), wq), (got_k, wk)):
            assert ((got.float() - want.float()).abs() <= kernels_ref.ulp16(want, dt)).all()
    else:
        assert max_abs(qo.cpu(), wq) <= 1e-5
        assert max_abs(got_k, wk) <= 1e-5
    assert torch.equal(got_v, wv)  # V is a copy (+ bias, rounded once): exact
    # untouched slots stay zero
    mask = torch.ones(pool * 16, dtype=torch.bool)
    mask[slots] = False
    assert kp.cpu().permute(0, 2, 1, 3).reshape(pool * 16, hkv, D)[mask].abs().max().item() == 0
    if dt == torch.bfloat16:  # against the fp32 restatement
        fq, fk, _ = kernels_ref.qk_norm_rope(qkv.float(), pos.tolist(), cos, sin, hq, hkv, D,
                                             None if qn is None else qn.float(),
                                             None if kn is None else kn.float(), None if b is None else b.float(),
                                             1e-6)
        # the north-star bar against the fp32 reference, absolute
        for name, a, w_ in (("q", qo.cpu().float(), fq), ("k", got_k.float(), fk)):
            err = (a - w_).abs().max().item()
            print(f"K5 bf16 {name} vs fp32: max-abs {err:.5f} (max |y| {w_.abs().max().item():.2f})")
            assert err <= 2e-2


# ---- packer ---------------------------------------------------------------------------

def test_pack_matches_oracle_bit_exact():
    lib = E.lib()
    rng = np.random.Generator(np.random.PCG64(5))
    nseq, mb, rows = 300, 40, 512
    ntok = rng.integers(1, 4, nseq)
    ntok[rng.integers(0, nseq, 6)] = rng.integers(100, 600, 6)
    start = np.array([rng.integers(0, mb * 16 - n + 1) for n in ntok])
    seq_row = rng.permutation(rows)[:nseq].astype(np.int32)
    tables = np.zeros((rows, mb), np.int32)
    dr, di, dbk = [], [], []
    seqs = []
    for i in range(nseq):
        need = (start[i] + ntok[i] + 15) // 16
        blocks = rng.integers(0, 100000, need).astype(np.int32)
        seqs.append((int(ntok[i]), int(start[i]), blocks.tolist()))
        for j, bk in enumerate(blocks):
            dr.append(seq_row[i]); di.append(j); dbk.append(bk)
    want = pack(seqs, 16, mb)
    T = int(want["cu_seqlens"][-1])
    t = lambda a, dt=torch.int32: torch.as_tensor(np.asarray(a), dtype=dt, device=DEV)
    bt = t(tables)
    cu, posd, rt, rc = t(np.zeros(nseq + 1)), t(np.zeros(T)), t(np.zeros(T)), t(np.zeros(T))
    sl = t(np.zeros(T), torch.int64)
    sync_ok(lib.ms_launch_pack(ptr(t(seq_row)), ptr(t(ntok)), ptr(t(start)), nseq, ptr(t(dr)), ptr(t(di)),
                               ptr(t(dbk)), len(dr), ptr(bt), mb, 16, ptr(cu), ptr(posd), ptr(sl), ptr(rt), ptr(rc),
                               None))
    assert np.array_equal(cu.cpu().numpy(), want["cu_seqlens"])
    assert np.array_equal(posd.cpu().numpy(), want["positions"])
    assert np.array_equal(sl.cpu().numpy(), want["slot_mapping"])
    assert np.array_equal(rc.cpu().numpy(), want["row_ctx"])
    assert np.array_equal(rt.cpu().numpy(), seq_row[want["seq_of_token"]])
    btn = bt.cpu().numpy()
    for i in range(nseq):
        n = len(seqs[i][2])
        assert np.array_equal(btn[seq_row[i], :n], want["block_tables"][i, :n])


# ---- SiLU-mul, argmax ------------------------------------------------------------------

@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_silu_mul(dt):
    gen = torch.Generator().manual_seed(6)
    T, I = 300, 3072
    gu = torch.randn(T, 2 * I, generator=gen).to(dt)
    out = torch.empty(T, I, dtype=dt, device=DEV)
    sync_ok(E.lib().ms_launch_silu_mul(ptr(gu.to(DEV)), ptr(out), T, I, E.torch_dtype_code(gu), None))
    want = kernels_ref.silu_mul_once(gu, I)
    if dt == torch.bfloat16:  # f32 inside, rounded once
        assert ((out.cpu().float() - want.float()).abs() <= kernels_ref.ulp16(want, dt)).all()
    else:
        assert max_abs(out.cpu(), want) <= 1e-5


def test_argmax_first_index_on_ties():
    V = 151936
    gen = torch.Generator().manual_seed(8)
    lg = torch.randn(9, V, generator=gen)
    lg[1, 100] = lg[1, 5000] = 50.0  # tie: first index wins
    lg[2, :] = 0.0
    lg[3, V - 1] = 99.0
    out = torch.empty(9, dtype=torch.int32, device=DEV)
    sync_ok(E.lib().ms_launch_argmax(ptr(lg.to(DEV)), 9, V, ptr(out), None))
    assert out.cpu().tolist() == kernels_ref.argmax_rows(lg).tolist()
    assert out[1].item() == 100 and out[2].item() == 0 and out[3].item() == V - 1


def test_paged_attention_ignores_nan_in_stale_page_slots():
    """Pool slots past each row's context hold NaN (as never-written pages
    may); decode attention must not read them into its result."""
    gen = torch.Generator().manual_seed(77)
    pool, hkv, D = 64, 8, 128
    lens = [1, 15, 16, 17, 40, 100]
    kp = torch.full((pool, hkv, 16, D), float("nan"))
    vp = torch.full((pool, hkv, 16, D), float("nan"))
    tables = torch.zeros(len(lens), 8, dtype=torch.int32)
    perm = torch.randperm(pool, generator=gen)
    off = 0
    for i, L in enumerate(lens):
        nb = (L + 15) // 16
        tables[i, :nb] = perm[off:off + nb].to(torch.int32)
        off += nb
        pos = torch.arange(L)
        pages = tables[i, pos // 16].long()
        kp[pages, :, pos % 16] = torch.randn(L, hkv, D, generator=gen)
        vp[pages, :, pos % 16] = torch.randn(L, hkv, D, generator=gen)
    q = torch.randn(len(lens), 16, D, generator=gen).bfloat16()
    kb, vb = kp.bfloat16(), vp.bfloat16()
    want = kernels_ref.paged_gqa_attention(q.float(), torch.nan_to_num(kb.float()), torch.nan_to_num(vb.float()),
                                           tables, lens, 1.0 / math.sqrt(D))
    out = torch.empty(q.shape, dtype=torch.bfloat16, device=DEV)
    attention(q.to(DEV), kb.to(DEV), vb.to(DEV), tables.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV),
              out, part=4)
    assert torch.isfinite(out).all()
    assert max_abs(out.cpu(), want) <= 2e-2

"""Time the reference's prototype paged-attention kernel against this library's
on BASELINE config 2 (test infrastructure: runs the reference's own kernel as
a comparison point, never as part of the product).

The prototype (docs/colab_cuda_kernels/mini_serve_kernels.cu:191-296) is
built from the reference tree by oracle/Makefile into
oracle/_ref/libmini_serve_kernels.so.  It supports f32/f16, so both kernels
run on the same inputs in f16 (ours also in bf16, the serving type); outputs
are cross-checked and the median of CUDA-event-timed launches is reported.

    python oracle/compare_prototype.py [--steps 10] [--out gpurun_out/proto.json]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from mini_serve_rs_b200 import engine as E  # noqa: E402

PROTO = ROOT / "oracle" / "_ref" / "libmini_serve_kernels.so"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--out", type=Path, default=None)
    args = ap.parse_args()
    if not PROTO.exists():
        raise SystemExit(f"{PROTO} missing: build it with `make -C oracle` where the reference tree exists")
    proto = C.CDLL(str(PROTO))
    ours = E.lib()
    for lib, name in ((proto, "launch_paged_gqa_decode_tiled_f16"), (ours, "launch_paged_gqa_decode_tiled_f16"),
                      (ours, "launch_paged_gqa_decode_tiled_bf16")):
        fn = getattr(lib, name)
        fn.argtypes = [C.c_void_p] * 6 + [C.c_int] * 4 + [C.c_float]
        fn.restype = C.c_int

    dev = "cuda:0"
    rng = np.random.Generator(np.random.PCG64(2))
    B, hq, hkv, D, pool, mb = 256, 16, 8, 128, 40000, 256
    ctx = rng.integers(1, 4097, B).astype(np.int32)
    nblk = (ctx + 15) // 16
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((B, mb), np.int32)
    off = 0
    for b in range(B):
        tables[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += nblk[b]
    g = torch.Generator(device=dev).manual_seed(2)
    k = torch.randn(pool, hkv, 16, D, generator=g, device=dev, dtype=torch.float16)
    v = torch.randn(pool, hkv, 16, D, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(B, hq, D, generator=g, device=dev, dtype=torch.float16)
    td = torch.from_numpy(tables).to(dev)
    cd = torch.from_numpy(ctx).to(dev)
    scale = 1.0 / math.sqrt(D)
    p = lambda t: C.c_void_p(t.data_ptr())
    algo = int(ctx.sum()) * hkv * D * 2 * 2 + 2 * B * hq * D * 2 + int(nblk.sum()) * 4 + B * 4

    def timed(fn, qq, kk, vv):
        out = torch.empty_like(qq)
        for _ in range(2):
            assert fn(p(qq), p(kk), p(vv), p(td), p(cd), p(out), B, hq, hkv, mb, scale) == 0
        torch.cuda.synchronize()
        ts = []
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            assert fn(p(qq), p(kk), p(vv), p(td), p(cd), p(out), B, hq, hkv, mb, scale) == 0
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        return ts[len(ts) // 2], out

    t_proto, o_proto = timed(proto.launch_paged_gqa_decode_tiled_f16, q, k, v)
    t_f16, o_f16 = timed(ours.launch_paged_gqa_decode_tiled_f16, q, k, v)
    kb, vb, qb = k.to(torch.bfloat16), v.to(torch.bfloat16), q.to(torch.bfloat16)
    del k, v
    t_bf16, o_bf16 = timed(ours.launch_paged_gqa_decode_tiled_bf16, qb, kb, vb)
    res = {
        "workload": "BASELINE config 2: 256 rows, ctx U[1,4096], 16/8 heads x 128, 40k-page pool",
        "algorithmic_bytes": algo,
        "prototype_f16_ms": t_proto, "prototype_f16_gbs": algo / t_proto / 1e6,
        "ours_f16_ms": t_f16, "ours_f16_gbs": algo / t_f16 / 1e6,
        "ours_bf16_ms": t_bf16, "ours_bf16_gbs": algo / t_bf16 / 1e6,
        "speedup_f16": t_proto / t_f16,
        "max_abs_ours_f16_vs_prototype": float((o_f16.float() - o_proto.float()).abs().max()),
        "max_abs_ours_bf16_vs_prototype_f16": float((o_bf16.float() - o_proto.float()).abs().max()),
    }
    print(json.dumps(res))
    if args.out:
        args.out.write_text(json.dumps(res, indent=1) + "\n")


if __name__ == "__main__":
    main()

"""Benchmark: ragged decode tokens/s of the Qwen3-0.6B-architecture forward step
on B200, with the paged-attention kernel's HBM GB/s against the roofline.

Workload (N=1 and per rank): one continuous-batching decode step of a
Qwen3-0.6B-architecture model (28 layers, hidden 1024, 16/8 heads x 128,
vocab 151936, bf16, seeded random-init weights) over 256 sequences whose
contexts are uniform in [1, 4096] (BASELINE config 2's shapes; the KV pages
hold seeded N(0,1) data and the block ids are a seeded random permutation of
the pool).  A "step" = one token for each of the 256 sequences.  Inputs (60 GB
of KV) are far larger than L2, so no flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: one process per GPU (torchrun), each rank an independent
data-parallel replica with its own 256 sequences (weak scaling, no data-path
collective); rank 0 prints the whole-job aggregate.  With N >= 2 the line
also carries a "tp" record: BASELINE config 5 (Qwen2.5-7B architecture) under
tensor parallelism by KV head on the same ranks (TP=2 at N=2, TP=4 at N=4, two
TP=4 replicas at N=8) -- first the committed transformers golden case on every
rank (fused peer-memory and NCCL all-reduce), then decode steps timed with each
all-reduce path, with the all-reduce share of the step.

CPU leg (N=1 line's cpu_baseline, and --impl reference): the oracle's
torch-CPU f32 restatement of the reference's batched decode at batches 8, 32,
64 and 256 (the GPU arm's), all host threads; the value is the largest batch
that fits host memory.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "ragged decode tokens/s per GPU (Qwen3-0.6B arch); attn HBM GB/s as % of peak"
UNIT = "tokens/s"
BATCH = 256
MAX_CTX = 4096
SEED = 20261201


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config5", action="store_true",
                    help="BASELINE config 5: Qwen2.5-7B arch, 256 seqs x ctx U[1024,32768], tensor parallel")
    ap.add_argument("--tp", type=int, default=2, help="tensor-parallel size for --config5")
    ap.add_argument("--tp-max-ctx", type=int, default=None,
                    help="cap config 5's context range (default: the full U[1024, 32768 - steps])")
    ap.add_argument("--no-tp", action="store_true",
                    help="with N >= 2: skip the tensor-parallel record (golden parity + config-5 decode)")
    ap.add_argument("--config4", action="store_true",
                    help="BASELINE config 4: serving trace (1024 Poisson arrivals at 64 req/s), one replica per GPU")
    ap.add_argument("--requests", type=int, default=1024, help="requests in the --config4 trace")
    ap.add_argument("--token-budget", type=int, default=2048, help="packed tokens per step for --config4")
    ap.add_argument("--max-active", type=int, default=512, help="concurrent requests per replica for --config4")
    ap.add_argument("--http", action="store_true",
                    help="--config4 through the HTTP/SSE driver: each replica serves /v1/completions and a "
                         "client process replays the trace (examples/bench.rs metrics)")
    ap.add_argument("--http-frontend", choices=["process", "thread"], default="process",
                    help="with --http: the aiohttp front-end in its own process (default) or on a thread of "
                         "the engine process")
    ap.add_argument("--kernel", choices=["attention", "norm_rope", "sample", "prefill"], default=None,
                    help="time one kernel in isolation (BASELINE config 2 for attention) instead of the step")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


def contexts(batch: int, seed: int):
    import numpy as np
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.integers(1, MAX_CTX + 1, batch)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []  # (arrival time, csv line)
        self.t_start = self.t_stop = 0.0

    def __enter__(self):
        import time
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        # nvidia-smi takes a moment to start: wait (at most 5 s) for its first sample, so that a
        # timed region shorter than that is still covered; samples before this point are dropped
        deadline = time.time() + 5.0
        while self.proc is not None and not self.lines and time.time() < deadline:
            time.sleep(0.01)
        self.t_start = time.time()
        return self

    def begin(self):
        """Mark the start of the timed region (after a barrier that follows __enter__)."""
        import time
        self.t_start = time.time()

    def _read(self):
        import time
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def __exit__(self, *a):
        import time
        self.t_stop = time.time()
        if self.proc:
            # a timed region can be shorter than the 100 ms interval: wait for the next sample,
            # used only if none arrived inside the region
            n = len(self.lines)
            deadline = time.time() + 1.0
            while len(self.lines) == n and time.time() < deadline:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        inside = [ln for t, ln in self.lines if self.t_start <= t <= self.t_stop]
        if not inside:
            inside = [ln for t, ln in self.lines if t > self.t_stop][:1]
        for ln in inside:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU leg: the reference's CPU path restated (oracle), on a bounded sample

def cpu_batches(avail_bytes: int):
    """Decode batches for the CPU leg: 8, 32, 64 and the GPU arm's 256, keeping
    only those whose f32 KV caches (prompt + a few steps, 28 layers x 8 KV
    heads x 128 x K and V) fit in 60 % of the host's available memory."""
    cfg_kv = 28 * 2 * 8 * 128 * 4
    ctx = contexts(BATCH, SEED)
    out = []
    for b in (8, 32, 64, BATCH):
        need = int(sum(int(c) + 8 for c in ctx[:b])) * cfg_kv
        if need <= 0.6 * avail_bytes:
            out.append(b)
    return out or [8]


def cpu_sample(batches, steps: int, warmup: int):
    """Time the torch-CPU f32 restatement of the reference's batched decode
    (qwen2.rs:630-764, per-sequence contiguous KV caches) on the first B
    sequences of this workload for each B in `batches`, all host threads.
    The cached contexts hold seeded N(0,1) K/V (copied from one random block:
    the values do not change the work).  Returns (tokens/s at the largest B,
    cores, sample description, {B: tokens/s})."""
    import numpy as np
    import torch

    from oracle.qwen_ref import QwenRef, SeqState, qwen3_0_6b, random_weights

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    cfg = qwen3_0_6b()
    model = QwenRef(cfg, random_weights(cfg, SEED))
    all_ctx = [int(c) for c in contexts(BATCH, SEED)]
    gen = torch.Generator().manual_seed(SEED)
    hkv, d = cfg.num_key_value_heads, cfg.hd()
    block_k = torch.randn(hkv, MAX_CTX, d, generator=gen)
    block_v = torch.randn(hkv, MAX_CTX, d, generator=gen)
    rates = {}
    for nseq in batches:
        ctx = all_ctx[:nseq]
        states = []
        for c in ctx:
            st = SeqState(cfg, c + warmup + steps + 2)
            st.preallocate(hkv, d)
            for layer in range(cfg.num_hidden_layers):
                st.k[layer][:, :c - 1].copy_(block_k[:, :c - 1])
                st.v[layer][:, :c - 1].copy_(block_v[:, :c - 1])
                st.n[layer] = c - 1
            states.append(st)
        ids = [int(t) for t in np.random.Generator(np.random.PCG64(SEED)).integers(0, cfg.vocab_size, nseq)]
        pos = [c - 1 for c in ctx]
        t_total = 0.0
        for s_ in range(warmup + steps):
            t0 = time.perf_counter()
            logits = model.step_decode_batch(states, ids, pos)
            ids = [int(x) for x in torch.argmax(logits, dim=-1)]
            dt = time.perf_counter() - t0
            if s_ >= warmup:
                t_total += dt
            pos = [p + 1 for p in pos]
        rates[nseq] = nseq * steps / t_total
        del states
    top = max(rates)
    ctx = all_ctx[:top]
    desc = (f"{top} of the {BATCH} sequences (contexts {min(ctx)}..{max(ctx)}, mean {sum(ctx) / top:.0f}), "
            f"{steps} timed decode steps after {warmup} warm-up, f32 torch-CPU restatement of "
            f"qwen2.rs step_decode_batch; tokens/s by batch: "
            + ", ".join(f"B={b}: {r:.1f}" for b, r in sorted(rates.items())))
    return rates[top], cores, desc, rates


def host_available_bytes() -> int:
    try:
        import psutil
        return int(psutil.virtual_memory().available)
    except ImportError:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    return 16 << 30


# ---------------------------------------------------------------------------
# our arm

def cudart():
    import ctypes
    lib = ctypes.CDLL("libcudart.so.12")
    lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    lib.cudaMemcpy.restype = ctypes.c_int
    return lib


def fill_pool(eng, cfg, pool_blocks, device, seed, kv_heads=None):
    """Seeded N(0,1) bf16 K/V in every page: one random 64 MB chunk copied over
    each layer's K and V pool (the contents do not change the kernel's traffic;
    the chunk stays in L2, so the fill is bound by HBM writes alone)."""
    import torch
    rt = cudart()
    layer_bytes = pool_blocks * (kv_heads or cfg.num_key_value_heads) * 16 * cfg.hd() * 2
    chunk = min(layer_bytes, 64 << 20)
    g = torch.Generator(device=f"cuda:{device}").manual_seed(seed)
    src = torch.randn(chunk // 2, generator=g, dtype=torch.bfloat16, device=f"cuda:{device}")
    torch.cuda.synchronize()
    for layer in range(cfg.num_hidden_layers):
        for which in (0, 1):
            base = eng.pool_ptr(layer, which)
            off = 0
            while off < layer_bytes:
                n = min(chunk, layer_bytes - off)
                rc = rt.cudaMemcpy(base + off, src.data_ptr(), n, 3)  # device to device
                if rc != 0:
                    raise RuntimeError(f"cudaMemcpy failed: {rc}")
                off += n
    torch.cuda.synchronize()  # D2D cudaMemcpy may return early; the engine stream does not wait on it
    del src


def run_decode(args, rank, world, local, cfg, ctx, seed, tp_rank=0, tp_size=1, comm=None):
    """Build one engine (one rank of a replica), admit len(ctx) sequences whose
    contexts are already cached (synthetic N(0,1) K/V), then time decode steps:
    `value` with decode inputs fed back on the device, `e2e` through ms_step with
    host token arrays.  seed is per replica (all TP ranks of a replica agree)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from mini_serve_rs_b200 import engine as E
    from mini_serve_rs_b200.config import iter_random_device_weights

    torch.cuda.set_device(local)
    B, K, W = len(ctx), args.steps, args.warmup
    KP = min(K, 10)
    extra = decode_extra(args, tp_size)
    need = [(int(c) + extra + 15) // 16 for c in ctx]
    pool_blocks = int(sum(need) * 1.02) + 64
    mbps = (max(int(c) for c in ctx) + extra + 15) // 16 + 1
    eng = E.Engine(cfg, device=local, pool_blocks=pool_blocks, max_seqs=B, max_tokens_per_step=max(B, 256),
                   max_blocks_per_seq=mbps, dtype=E.MS_DTYPE_BF16, tp_rank=tp_rank, tp_size=tp_size,
                   nccl_comm=comm)
    eng.load_weights(iter_random_device_weights(cfg, SEED, device=f"cuda:{local}"))
    fill_pool(eng, cfg, pool_blocks, local, seed + 17 * tp_rank, kv_heads=cfg.num_key_value_heads // tp_size)
    rng = np.random.Generator(np.random.PCG64(seed))
    perm = rng.permutation(pool_blocks).astype(np.int32)
    ids = np.arange(1, B + 1, dtype=np.uint64)
    off = 0
    for i in range(B):
        prompt = rng.integers(0, cfg.vocab_size, int(ctx[i])).astype(np.uint32)
        # the whole prompt is cached (synthetic KV); step 1 replays its last token
        eng.admit(int(ids[i]), prompt, perm[off:off + need[i]], num_cached=int(ctx[i]))
        off += need[i]
    stream = torch.cuda.ExternalStream(eng.stream_ptr())

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(W):
        eng.step_launch(ids, None, None, E.MS_STEP_TOKENS_FROM_DEVICE)
        toks, _ = eng.step_wait()
    torch.cuda.synchronize()

    # ---- value: device-resident inputs (decode tokens fed back on the device);
    # pure-decode steps replay a captured CUDA graph (captured during warm-up)
    launches0 = eng.profile()[0]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:  # started before the barrier: its start-up skews no rank
        barrier()
        torch.cuda.synchronize()
        clk.begin()
        e0.record(stream)
        for _ in range(K):
            eng.step_launch(ids, None, None, E.MS_STEP_TOKENS_FROM_DEVICE)
            toks, _ = eng.step_wait()
        e1.record(stream)
        e1.synchronize()
    ms = e0.elapsed_time(e1)
    gpu_launches = eng.profile()[0] - launches0
    graphs = eng.graph_stats()
    torch.cuda.synchronize()
    barrier()

    # ---- attention kernel time inside the step: KP more steps with CUDA
    # events around every paged-attention launch (eager: events need launches)
    eng.profile()  # reset the event log
    eng.set_profiling(True)
    for _ in range(KP):
        eng.step_launch(ids, None, None, E.MS_STEP_TOKENS_FROM_DEVICE)
        toks, _ = eng.step_wait()
    _, alaunch, attn_ms, attn_bytes = eng.profile()
    ar_calls, ar_ms = eng.profile_allreduce()
    eng.set_profiling(False)
    torch.cuda.synchronize()
    barrier()

    # ---- tensor parallelism: the same steps with the all-reduces through
    # NCCL + K4 instead of the fused peer-memory kernel (every rank switches)
    nccl = None
    fused = eng.tp_fused()
    if tp_size > 1 and fused:
        eng.set_tp_fused(False)
        barrier()
        torch.cuda.synchronize()
        n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0.record(stream)
        for _ in range(K):
            eng.step_launch(ids, None, None, E.MS_STEP_TOKENS_FROM_DEVICE)
            toks, _ = eng.step_wait()
        n1.record(stream)
        n1.synchronize()
        nccl_ms = n0.elapsed_time(n1)
        eng.profile()
        eng.set_profiling(True)
        for _ in range(KP):
            eng.step_launch(ids, None, None, E.MS_STEP_TOKENS_FROM_DEVICE)
            toks, _ = eng.step_wait()
        eng.profile()
        nccl_calls, nccl_ar_ms = eng.profile_allreduce()
        eng.set_profiling(False)
        eng.set_tp_fused(True)
        nccl = {"ms": nccl_ms, "ar_calls": nccl_calls, "ar_ms": nccl_ar_ms}
        torch.cuda.synchronize()
        barrier()

    # ---- e2e: through the public step call with host token arrays
    # step 1 replayed the last cached prompt token; every later step added one
    done = W + K + KP + (K + KP if nccl else 0)
    pos = np.array([int(c) + done - 1 for c in ctx], dtype=np.int32)
    host_toks = np.asarray(toks, dtype=np.uint32)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0 = eng.graph_stats()
    f0.record(stream)
    for _ in range(K):
        host_toks, _ = eng.step(ids, host_toks, pos)
        pos += 1
    f1.record(stream)
    f1.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    g1 = eng.graph_stats()
    barrier()

    t = torch.tensor([ms, ms_e2e, nccl["ms"] if nccl else 0.0], dtype=torch.float64, device=f"cuda:{local}")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_e2e = float(t[0]), float(t[1])
    if nccl:
        nccl["ms"] = float(t[2])
    res = {
        "ms": ms, "ms_e2e": ms_e2e, "gpu_launches": gpu_launches, "clocks": clk.summary(),
        "attn_launches": alaunch, "attn_ms": attn_ms, "attn_bytes": attn_bytes,
        "ar_calls": ar_calls, "ar_ms": ar_ms, "nccl": nccl,
        "h2d": (4 + 7 * B) * 4, "d2h": B * 4 + 4, "ctx_mean": float(np.mean(ctx)),
        "graphs": {"captured": graphs[0], "replayed": graphs[1],
                   "e2e_captured": g1[0] - g0[0], "e2e_replayed": g1[1] - g0[1]}, "kp": KP, "tp_fused": eng.tp_fused(),
        "memory": eng.memory(),
    }
    eng.close()
    return res


def decode_extra(args, tp_size: int = 1) -> int:
    """Decode steps run_decode takes beyond each sequence's admitted context
    (warm-up, timed, profiled and e2e steps; under TP also the NCCL pass)."""
    K, KP = args.steps, min(args.steps, 10)
    return args.warmup + 2 * K + KP + 2 + (K + KP if tp_size > 1 else 0)


def run_ours(args, rank, world, local):
    from mini_serve_rs_b200.config import qwen3_0_6b
    return run_decode(args, rank, world, local, qwen3_0_6b(), contexts(args.batch, SEED + rank), SEED + rank)


def attention_config2(device: int, seed: int = 2, pool: int = 40000):
    """BASELINE config 2's isolated op: 256 rows, ctx ~ U[1,4096], 16/8 heads x
    128, bf16, block tables a seeded random permutation of the page pool."""
    import numpy as np
    import torch
    dev = f"cuda:{device}"
    rng = np.random.Generator(np.random.PCG64(seed))
    B, hq, hkv, D = BATCH, 16, 8, 128
    ctx = rng.integers(1, MAX_CTX + 1, B).astype(np.int32)
    nblk = (ctx + 15) // 16
    perm = rng.permutation(pool).astype(np.int32)
    tables = np.zeros((B, 256), np.int32)
    off = 0
    for b in range(B):
        tables[b, :nblk[b]] = perm[off:off + nblk[b]]
        off += nblk[b]
    g = torch.Generator(device=dev).manual_seed(seed)
    kp = torch.randn(pool, hkv, 16, D, generator=g, device=dev, dtype=torch.bfloat16)
    vp = torch.randn(pool, hkv, 16, D, generator=g, device=dev, dtype=torch.bfloat16)
    q = torch.randn(B, hq, D, generator=g, device=dev, dtype=torch.bfloat16)
    return {"q": q, "k": kp, "v": vp, "tables": torch.from_numpy(tables).to(dev),
            "ctx": torch.from_numpy(ctx).to(dev), "sum_ctx": int(ctx.sum()), "sum_blocks": int(nblk.sum())}


def run_attention_kernel(args, local):
    """Time ms_launch_paged_attention alone on config 2 (CUDA events on the
    launching stream; inputs 4.6 GB >> L2)."""
    import ctypes as C
    import torch
    from mini_serve_rs_b200 import engine as E
    torch.cuda.set_device(local)
    d = attention_config2(local)
    lib = E.lib()
    B, hq, hkv, D = BATCH, 16, 8, 128
    part = 0
    ws_bytes = B * hq * 256 * (D * 4 + 8) + 256
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=f"cuda:{local}")
    out = torch.empty_like(d["q"])
    st = torch.cuda.current_stream()
    p = lambda t: C.c_void_p(t.data_ptr())

    def launch():
        rc = lib.ms_launch_paged_attention(p(d["q"]), p(d["k"]), p(d["v"]), p(d["tables"]), 256, None, p(d["ctx"]),
                                           B, MAX_CTX, p(out), hq, hkv, D, 16, 1.0 / math.sqrt(D), part, p(ws),
                                           ws_bytes, E.MS_DTYPE_BF16, C.c_void_p(st.cuda_stream))
        assert rc == 0, rc

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        launch()
        e1.record(st)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    ms = times[len(times) // 2]
    algo = d["sum_ctx"] * hkv * D * 2 * 2 + 2 * B * hq * D * 2 + d["sum_blocks"] * 4 + B * 4
    peak, kind = peaks()
    gbs = algo / (ms / 1000) / 1e9
    print(json.dumps({"kernel": "paged_attention (K3 + combine)", "workload": "BASELINE config 2 isolated op",
                      "ms_median": ms, "ms_all": times, "algorithmic_bytes": algo, "achieved_gbs": gbs,
                      "peak_gbs": peak, "frac": gbs / peak, "peak_source": kind}), flush=True)


def config4_trace(n_req: int, vocab: int, seed: int = 4):
    """BASELINE config 4, seeded: Poisson arrivals at 64 req/s; prompt length
    lognormal (median 512, sigma 1.0) clipped to [16, 8192]; output length
    U[32, 1024]; 30 % of prompts are a shared 1024-token prefix + their own
    suffix (total clipped to 8192); token ids U[0, V)."""
    import numpy as np
    from mini_serve_rs_b200.serving import Request
    rng = np.random.Generator(np.random.PCG64(seed))
    shared = rng.integers(0, vocab, 1024).tolist()
    t = 0.0
    reqs = []
    for i in range(n_req):
        t += float(rng.exponential(1.0 / 64.0))
        n = int(np.clip(np.round(rng.lognormal(np.log(512.0), 1.0)), 16, 8192))
        own = rng.integers(0, vocab, n).tolist()
        prompt = (shared + own)[:8192] if rng.random() < 0.3 else own
        reqs.append(Request(rid=i + 1, prompt=prompt, max_tokens=int(rng.integers(32, 1025)), arrival=t))
    return reqs


def run_config4(args, rank, world, local):
    """One replica per GPU (one process each).  A dispatcher thread on rank 0
    routes every request at its arrival time to the replica with the lowest
    router.rs score, (queue + active + 1) x max(avg latency, 1 ms), among
    those with capacity (mini_serve_rs_b200/router.py); replicas publish their
    metrics through a TCPStore after every step.  Each replica runs the
    continuous-batching loop (serving.ServingLoop) in real time; rank 0
    reports aggregate and per-GPU token rates and TTFT.  With --http the trace
    client deals requests round-robin over the replicas' HTTP servers."""
    import time as _time

    import torch
    import torch.distributed as dist
    from mini_serve_rs_b200 import engine as E
    from mini_serve_rs_b200.config import iter_random_device_weights, qwen3_0_6b
    from mini_serve_rs_b200.router import Dispatcher, ReplicaLink, router_stores, summarize_routing
    from mini_serve_rs_b200.serving import ServingLoop, summarize
    torch.cuda.set_device(local)
    cfg = qwen3_0_6b()
    page_bytes = cfg.num_hidden_layers * 2 * cfg.num_key_value_heads * 16 * cfg.hd() * 2
    pool_blocks = int(100e9 // page_bytes)
    max_active = args.max_active
    eng = E.Engine(cfg, device=local, pool_blocks=pool_blocks, max_seqs=max_active,
                   max_tokens_per_step=args.token_budget + max_active, max_blocks_per_seq=(8192 + 1024) // 16 + 1,
                   dtype=E.MS_DTYPE_BF16)
    eng.load_weights(iter_random_device_weights(cfg, SEED, device=f"cuda:{local}"))
    pages = E.Pages(pool_blocks, 16, max_chunks=pool_blocks // 2)
    trace = config4_trace(args.requests, cfg.vocab_size)
    # warm-up: a few requests outside the trace (first-launch costs, library heuristics)
    warm = ServingLoop(eng, pages, max_active, args.token_budget)
    from mini_serve_rs_b200.serving import Request
    warm.run([Request(rid=10_000_000 + k, prompt=list(range(100 + 37 * k)), max_tokens=8) for k in range(4)])
    pages.close()
    pages = E.Pages(pool_blocks, 16, max_chunks=pool_blocks // 2)
    routing = None
    if args.http:
        from mini_serve_rs_b200.http_driver import (BackgroundHttp, HttpFrontendProcess, ServingServer,
                                                    run_trace_process, summarize_http)
        reqs = [r for r in trace if (r.rid - 1) % world == rank]
        srv = ServingServer(eng, pages, model="qwen3-0.6b-arch", max_active=max_active,
                            token_budget=args.token_budget).start()
        http = (HttpFrontendProcess if args.http_frontend == "process" else BackgroundHttp)(srv).start()
        if world > 1:
            dist.barrier()
        with ClockSampler(local) as clk:
            results, elapsed = run_trace_process(http.url, "qwen3-0.6b-arch", reqs, timeout_s=900.0)
        http.stop()
        srv.stop()
        summ = summarize_http(results, elapsed)
        summ["steps"] = srv.steps
    else:
        master, store, dstore = router_stores(rank, world)
        loop = ServingLoop(eng, pages, max_active, args.token_budget)
        disp = Dispatcher(dstore, world, trace) if rank == 0 else None
        if world > 1:
            dist.barrier()
        if disp:
            disp.start(t0=_time.time() + 0.2)
        with ClockSampler(local) as clk:
            elapsed = loop.run_routed(ReplicaLink(store, rank), {r.rid: r for r in trace}, timeout_s=900.0)
        if disp:
            disp.join(60)
            routing = summarize_routing(disp.choices, world)
            routing["unrouted"] = len(disp.failed)
        summ = summarize(loop.finished, elapsed)
        summ["steps"] = loop.steps
        summ["engine_s"], summ["host_step_s"] = loop.engine_s, loop.host_s
        if world > 1:
            dist.barrier()  # the store's host (rank 0) outlives every client
        del store, dstore, master
    summ["prefix"] = pages.stats()
    summ["clocks"] = clk.summary()
    summ["gpu_launches"] = eng.profile()[0]
    eng.close()
    alls = [summ]
    if world > 1:
        alls = [None] * world
        dist.all_gather_object(alls, summ)
    if rank == 0:
        tokens = sum(x["tokens"] for x in alls)
        span = max(x["elapsed_s"] for x in alls)
        agg = tokens / span
        # TTFT percentiles over every request of the trace
        ttfts = sorted(t for x in alls for t in x.get("ttft_ms_all", []))

        def pct(q):
            return ttfts[min(len(ttfts) - 1, int(q * len(ttfts)))] if ttfts else None

        print(json.dumps({
            "metric": "serving trace decode tokens/s (BASELINE config 4)" + (" via HTTP/SSE" if args.http else ""),
            "value": agg, "unit": UNIT,
            "n_gpus": world, "higher_is_better": True, "scaling": "weak", "dtype": "bf16",
            "data": "synthetic seeded trace (random-init Qwen3-0.6B-arch weights)",
            "config": {"workload": "BASELINE config 4", "requests": args.requests, "arrival_rate_per_s": 64,
                       "prompt": "lognormal median 512 sigma 1.0 clipped [16,8192], 30% shared 1024-token prefix",
                       "output": "uniform[32,1024]", "token_budget": args.token_budget, "max_active": max_active,
                       "sampling": "greedy",
                       "routing": ("round-robin over replicas (HTTP trace client)" if args.http else
                                   "router.rs latency-aware score, dispatcher on rank 0"),
                       "driver": (f"POST /v1/completions stream=true, HTTP front-end: {args.http_frontend}, "
                                  "trace client in its own process" if args.http else "ServingLoop in process")},
            "note": "arrival-bound: the trace offers 64 req/s whatever N is, so tokens/s grows with N only while "
                    "one replica cannot keep up with the arrivals",
            "tokens_per_s_per_gpu": agg / world, "tokens": tokens, "elapsed_s": span,
            "ttft_ms_p50": pct(0.5), "ttft_ms_p90": pct(0.9), "ttft_ms_p99": pct(0.99),
            "routing": routing,
            "per_rank": [{k: v for k, v in x.items() if k != "ttft_ms_all"} for x in alls]}), flush=True)


def tp_group_comm(rank, world, local, tp):
    """NCCL communicator of this rank's tensor-parallel group (ranks
    [g*tp, (g+1)*tp)); the unique id travels over the torch process group."""
    import torch.distributed as dist
    from mini_serve_rs_b200 import engine as E
    group, tp_rank = rank // tp, rank % tp
    uid = E.nccl_unique_id() if tp_rank == 0 else None
    uids = [None] * world
    dist.all_gather_object(uids, uid)
    return group, tp_rank, E.nccl_comm_init(tp, uids[group * tp], tp_rank, local)


def tp_parity_cfg():
    """The committed golden case "qwen2_kv4": Qwen2.5-7B's attention shape
    (hidden 3584, 28 query / 4 KV heads x 128, q/k/v bias, untied lm_head) on
    two layers, vocabulary 512, MLP 1024, weights host_random_weights(seed 7007)."""
    from mini_serve_rs_b200.config import ModelConfig
    return ModelConfig(512, 3584, 1024, 2, 28, 4, 4096, 128, 1e6, 1e-6, False, True, False)


def tp_parity(local, tp_rank, tp, comm):
    """One tensor-parallel group runs the golden case in f32 -- three prompts
    prefilled in one packed step, then six decode steps fed the golden greedy
    tokens -- first with the fused peer-memory all-reduce, then through NCCL.
    Every step's logits are compared with the committed transformers outputs
    (tests/golden/golden.npz, max-abs 2e-4, the f32 tolerance of the GPU
    parity tests) and its greedy tokens must be equal."""
    import numpy as np
    from mini_serve_rs_b200 import engine as E
    from mini_serve_rs_b200.config import host_random_weights
    cfg = tp_parity_cfg()
    with np.load(ROOT / "tests" / "golden" / "golden.npz") as z:
        g = {k: z[k] for k in z.files if k.startswith("qwen2_kv4/")}
    prompts = [g[f"qwen2_kv4/p{i}/prompt"].tolist() for i in range(3)]
    steps = g["qwen2_kv4/p0/tokens"].shape[0] - 1
    eng = E.Engine(cfg, device=local, pool_blocks=64, max_seqs=4, max_tokens_per_step=256, max_blocks_per_seq=16,
                   dtype=E.MS_DTYPE_F32, tp_rank=tp_rank, tp_size=tp, nccl_comm=comm)
    eng.load_weights(host_random_weights(cfg, 7007))
    out = {}
    modes = [True, False] if eng.tp_fused() else [False]
    for fused in modes:
        if eng.tp_fused() != fused:
            eng.set_tp_fused(fused)
        ids = [1, 2, 3]
        for k, (sid, p) in enumerate(zip(ids, prompts)):
            eng.admit(sid, p, list(range(16 * k, 16 * k + 8)))
        worst, bad = 0.0, 0
        toks, _ = eng.step(ids, flags=E.MS_STEP_KEEP_LOGITS)
        for s in range(steps + 1):
            lg = eng.logits(len(ids))
            for i in range(len(ids)):
                worst = max(worst, float(np.abs(lg[i] - g[f"qwen2_kv4/p{i}/logits"][s]).max()))
                bad += int(toks[i]) != int(g[f"qwen2_kv4/p{i}/tokens"][s])
            if s == steps:
                break
            inputs = [int(g[f"qwen2_kv4/p{i}/tokens"][s]) for i in range(len(ids))]
            toks, _ = eng.step(ids, inputs, [len(p) + s for p in prompts], flags=E.MS_STEP_KEEP_LOGITS)
        for sid in ids:
            eng.release(sid)
        out["fused" if fused else "nccl"] = {"max_abs_logits": worst, "token_mismatches": bad,
                                             "ok": worst <= 2e-4 and bad == 0}
    eng.close()
    return out


def tp_decode_record(args, r, tp, world, cfg, ctx_desc):
    """The config-5 numbers of one run_decode result (rank 0's view; times
    are already the max over ranks)."""
    replicas = world // tp
    K, KP = args.steps, r["kp"]
    value = replicas * args.batch * K / (r["ms"] / 1000.0)
    per_launch_ms = r["attn_ms"] / max(1, r["attn_launches"])
    per_launch_bytes = r["attn_bytes"] / max(1, r["attn_launches"])
    achieved = per_launch_bytes / (per_launch_ms / 1000.0) / 1e9
    peak, kind = peaks()
    step_ms = r["ms"] / K
    rec = {
        "value": value, "unit": UNIT, "ms_per_step": step_ms, "tokens_per_s_per_gpu": value / world,
        "e2e": {"value": replicas * args.batch * K / (r["ms_e2e"] / 1000.0), "unit": UNIT,
                "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
        "config": ctx_desc,
        "attention": {"kernel": "paged_attention_tc_kernel (per rank: its KV heads)", "achieved_gbs": achieved,
                      "peak_gbs": peak, "frac": achieved / peak, "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({kind})",
                      "ms_per_launch": per_launch_ms, "share_of_step": (r["attn_ms"] / KP) / step_ms},
        "allreduce": {"path": ("fused peer-memory all-reduce + residual add + RMSNorm (NVLink, CUDA IPC)"
                               if r["tp_fused"] else "NCCL all-reduce + K4"),
                      "calls_per_step": r["ar_calls"] / max(1, KP), "ms_per_step": r["ar_ms"] / max(1, KP),
                      "share_of_step": (r["ar_ms"] / max(1, KP)) / step_ms},
        "gpu_launches": r["gpu_launches"], "clocks": r["clocks"], "memory_bytes": r["memory"],
    }
    if r.get("nccl"):
        n = r["nccl"]
        rec["nccl_allreduce"] = {"ms_per_step": n["ms"] / K, "value": replicas * args.batch * K / (n["ms"] / 1000.0),
                                 "allreduce_ms_per_step": n["ar_ms"] / max(1, KP),
                                 "allreduce_share_of_step": (n["ar_ms"] / max(1, KP)) / (n["ms"] / K)}
    return rec


def config5_contexts(args, tp, group, max_ctx=None):
    """Per-replica config-5 contexts: U[1024, min(max_ctx, 32768 - extra)]."""
    import numpy as np
    from mini_serve_rs_b200.config import qwen2_5_7b
    cfg = qwen2_5_7b()
    hi = cfg.max_position_embeddings - decode_extra(args, tp)
    if max_ctx:
        hi = min(hi, max_ctx)
    rng = np.random.Generator(np.random.PCG64(SEED + group))
    return cfg, rng.integers(1024, hi + 1, args.batch), hi


def run_tp(args, rank, world, local):
    """The tensor-parallel record added to the headline line when N >= 2:
    TP=2 at N=2, TP=4 at N=4, two TP=4 replicas at N=8.  First the golden
    parity case on every rank (fused and NCCL all-reduce), then BASELINE
    config 5's decode (Qwen2.5-7B arch, 256 sequences per replica, contexts
    U[1024, 32768 - steps], bf16), timed with the fused all-reduce and again
    with NCCL on the same engines."""
    import torch
    import torch.distributed as dist
    from mini_serve_rs_b200 import engine as E
    tp = 2 if world == 2 or world % 4 else 4
    if world % tp:
        return {"skipped": f"{world} ranks do not split into tensor-parallel groups of {tp}"}
    torch.cuda.empty_cache()
    group, tp_rank, comm = tp_group_comm(rank, world, local, tp)
    try:
        par = tp_parity(local, tp_rank, tp, comm)
    except Exception as e:  # a failure is reported, and every rank still takes the same collective steps
        par = {"error": repr(e)}
    pars = [None] * world
    dist.all_gather_object(pars, par)
    parity_ok = all("error" not in p and all(v["ok"] for v in p.values()) and "fused" in p for p in pars)
    cfg, ctx, hi = config5_contexts(args, tp, group, args.tp_max_ctx)
    r = run_decode(args, rank, world, local, cfg, ctx, SEED + group, tp_rank, tp, comm)
    E.nccl_comm_destroy(comm)
    desc = {"workload": "BASELINE config 5 decode (Qwen2.5-7B arch, TP by KV head)", "tp": tp,
            "replicas": world // tp, "seqs_per_replica": args.batch, "ctx": f"uniform[1024,{hi}]",
            "ctx_mean": r["ctx_mean"], "steps": args.steps}
    rec = tp_decode_record(args, r, tp, world, cfg, desc)
    worst = max((v["max_abs_logits"] for p in pars if "error" not in p for v in p.values()), default=None)
    rec = {"parity": parity_ok,
           "parity_check": {"case": "tests/golden/golden.npz qwen2_kv4 (transformers, f32): 3 prompts, "
                                    "prefill + 6 decode steps on every rank, logits max-abs <= 2e-4, tokens equal",
                            "paths": sorted({k for p in pars for k in p}), "max_abs_logits": worst,
                            "per_rank": pars},
           **rec}
    return rec


def run_config5(args, rank, world, local):
    """BASELINE config 5 decode: Qwen2.5-7B architecture, tensor parallel by KV
    head over `--tp` GPUs per replica (world / tp replicas), 256 sequences per
    replica with contexts U[1024, 32768 - steps] (the model's 32768 positions
    bound the last decode step), bf16.  Prints its own JSON line."""
    from mini_serve_rs_b200 import engine as E
    tp = args.tp
    if world < 2 or world % tp != 0:
        raise SystemExit("--config5 runs under torchrun with a multiple of --tp ranks (TP=1 does not fit 248 GB of KV)")
    group, tp_rank, comm = tp_group_comm(rank, world, local, tp)
    cfg, ctx, hi = config5_contexts(args, tp, group, args.tp_max_ctx)
    r = run_decode(args, rank, world, local, cfg, ctx, SEED + group, tp_rank, tp, comm)
    E.nccl_comm_destroy(comm)
    if rank == 0:
        desc = {"workload": "BASELINE config 5", "seqs_per_replica": args.batch, "ctx": f"uniform[1024,{hi}]",
                "ctx_mean": r["ctx_mean"]}
        rec = tp_decode_record(args, r, tp, world, cfg, desc)
        print(json.dumps({"metric": "decode tokens/s (Qwen2.5-7B arch, TP by KV head)", "n_gpus": world, "tp": tp,
                          "replicas": world // tp, "steps": args.steps, "warmup": args.warmup, "dtype": "bf16",
                          "data": "synthetic (seeded random-init weights, N(0,1) KV)",
                          "cuda_graphs": r["graphs"], **rec}), flush=True)


def run_norm_rope_kernels(args, local):
    """a packed T=8192 bf16 batch (8 prefill chunks of
    U[256,768] tokens, the rest single decode tokens): K4 fused residual-add +
    RMSNorm over hidden 1024, then K5 QK-norm + RoPE (theta 1e6, 16/8 heads x
    128, positions per sequence in [0, 8192)) fused with the paged K/V append.
    Before every timed launch L2 is flushed by READING a 256 MB buffer, so it
    holds clean lines (a write-based flush leaves dirty lines whose write-back
    would be charged to the timed kernel); median of K."""
    import ctypes as C
    import numpy as np
    import torch
    from mini_serve_rs_b200 import engine as E
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    lib = E.lib()
    T, H, hq, hkv, D = 8192, 1024, 16, 8, 128
    rng = np.random.Generator(np.random.PCG64(3))
    pos = []
    for _ in range(8):
        n = int(rng.integers(256, 769))
        st = int(rng.integers(0, 8192 - n))
        pos.extend(range(st, st + n))
    while len(pos) < T:
        pos.append(int(rng.integers(0, 8192)))
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(T, H, generator=g, device=dev, dtype=torch.bfloat16)
    r = torch.randn(T, H, generator=g, device=dev, dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    resid, normed = torch.empty_like(x), torch.empty_like(x)
    qkv = torch.randn(T, (hq + 2 * hkv) * D, generator=g, device=dev, dtype=torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    half = D // 2
    inv = torch.tensor([1.0 / (1e6 ** (i / D)) for i in range(0, D, 2)], dtype=torch.float32)
    fr = torch.arange(8192, dtype=torch.float32).reshape(-1, 1) * inv.reshape(1, -1)
    cos, sin = fr.cos().to(dev), fr.sin().to(dev)  # f32 tables (K5 computes in f32 in every mode)
    posd = torch.tensor(pos, dtype=torch.int32, device=dev)
    pool = 640
    slots = torch.from_numpy(rng.permutation(pool * 16)[:T].astype(np.int64)).to(dev)
    kp = torch.zeros(pool, hkv, 16, D, device=dev, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    qo = torch.empty(T, hq, D, device=dev, dtype=torch.bfloat16)
    scribble = torch.ones(32 << 20, dtype=torch.int64, device=dev)  # 256 MB
    p = lambda t: C.c_void_p(t.data_ptr())
    st = torch.cuda.current_stream()
    ptr_st = C.c_void_p(st.cuda_stream)

    def k4():
        assert lib.ms_launch_add_rmsnorm(p(x), p(r), None, p(w), p(resid), p(normed), T, H, 1e-6,
                                         E.MS_DTYPE_BF16, ptr_st) == 0

    def k5():
        assert lib.ms_launch_qk_norm_rope_append(p(qkv), None, p(qn), p(kn), p(cos), p(sin), p(posd), p(slots),
                                                 p(qo), p(kp), p(vp), T, hq, hkv, D, 16, 1e-6, E.MS_DTYPE_BF16,
                                                 ptr_st) == 0

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        ts = []
        for _ in range(args.steps):
            scribble.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        return ts[len(ts) // 2]

    peak, kind = peaks()
    k4_bytes = T * H * 2 * 4 + H * 2
    k5_qk = T * (hq + hkv) * D * 2 * 2
    k5_bytes = T * (hq + 2 * hkv) * D * 2 * 2 + T * 12 + 2 * D * 2  # tables excluded (L2-resident lookups)
    t4, t5 = timed(k4), timed(k5)
    print(json.dumps({"workload": "BASELINE config 3 (T=8192 packed, bf16)", "l2": "256 MB read-only flush before each launch",
                      "k4_add_rmsnorm": {"ms": t4, "bytes": k4_bytes, "gbs": k4_bytes / t4 / 1e6,
                                         "frac": k4_bytes / t4 / 1e6 / peak},
                      "k5_qk_norm_rope_append": {"ms": t5, "bytes": k5_bytes, "qk_only_bytes": k5_qk,
                                                 "gbs": k5_bytes / t5 / 1e6, "frac": k5_bytes / t5 / 1e6 / peak},
                      "peak_gbs": peak, "peak_source": kind}), flush=True)


def run_sample_kernel(args, local):
    """K6b on-device sampling for a decode batch: 256 rows of f32 logits over
    the Qwen3 vocabulary (151936), temperature 0.8, with top-p 0.9 (race pass
    + nucleus checks) and without (one race pass).  Median of K CUDA-event
    intervals of one launch each; the argmax kernel over the same rows for
    scale."""
    import ctypes as C
    import torch
    from mini_serve_rs_b200 import engine as E
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    lib = E.lib()
    rows, V = 256, 151936
    g = torch.Generator(device=dev).manual_seed(5)
    lg = torch.randn(rows, V, generator=g, device=dev) * 3
    t = torch.full((rows,), 0.8, device=dev)
    p9 = torch.full((rows,), 0.9, device=dev)
    sd = torch.arange(rows, device=dev, dtype=torch.int64)
    out = torch.zeros(rows, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream()
    ptr = lambda x: C.c_void_p(x.data_ptr())
    sp = C.c_void_p(st.cuda_stream)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        ts = []
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        return ts[len(ts) // 2]

    topp = timed(lambda: lib.ms_launch_sample(ptr(lg), rows, V, ptr(t), ptr(p9), ptr(sd), ptr(out), sp))
    plain = timed(lambda: lib.ms_launch_sample(ptr(lg), rows, V, ptr(t), None, ptr(sd), ptr(out), sp))
    amax = timed(lambda: lib.ms_launch_argmax(ptr(lg), rows, V, ptr(out), sp))
    peak, kind = peaks()
    nbytes = rows * V * 4  # the logits, read once (155 MB, above the 126 MB L2)
    print(json.dumps({"workload": "256 rows x 151936 f32 logits (Qwen3 vocabulary), temperature 0.8",
                      "logits_bytes": nbytes, "ms_top_p_0.9": topp, "ms_temperature_only": plain,
                      "ms_argmax": amax, "top_p_frac_of_hbm_read_once": nbytes / topp / 1e6 / peak,
                      "peak_gbs": peak, "peak_source": kind}), flush=True)


def run_prefill_kernel(args, local, seqs: int = 4, length: int = 4096):
    """K3p causal prefill attention over the paged pool: `seqs` prompts of
    `length` tokens from position 0 (Qwen3-0.6B heads: 16 q / 8 kv x 128,
    bf16), packed as one ragged batch.  Algorithmic FLOPs = sum over tokens of
    4 * Hq * D * (keys attended) (QK^T and PV, causal).  Median of K launches,
    CUDA events; compared with the measured dense bf16 peak."""
    import ctypes as C
    import numpy as np
    import torch
    from mini_serve_rs_b200 import engine as E
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    lib = E.lib()
    hq, hkv, D = 16, 8, 128
    T = seqs * length
    pages = T // 16
    g = torch.Generator(device=dev).manual_seed(9)
    kp = torch.randn(pages, hkv, 16, D, generator=g, device=dev).to(torch.bfloat16)
    vp = torch.randn(pages, hkv, 16, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(T, hq, D, generator=g, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    mbps = length // 16
    tables = torch.arange(pages, dtype=torch.int32, device=dev).reshape(seqs, mbps)
    row0 = np.arange(seqs, dtype=np.int32) * length
    ntok = np.full(seqs, length, np.int32)
    start = np.zeros(seqs, np.int32)
    trow = np.arange(seqs, dtype=np.int32)
    cap = T
    tiles = np.zeros(4 * cap, np.int32)
    ip = lambda a: a.ctypes.data_as(C.POINTER(C.c_int32))
    nt = lib.ms_prefill_tiles(ip(row0), ip(ntok), ip(start), ip(trow), seqs, hq, hkv, ip(tiles), cap)
    assert nt > 0
    tiles_d = torch.from_numpy(tiles[:4 * nt].copy()).to(dev)
    st = torch.cuda.current_stream()
    P = lambda t: C.c_void_p(t.data_ptr())

    def launch():
        rc = lib.ms_launch_paged_prefill(P(q), P(kp), P(vp), P(tables), mbps, P(tiles_d), nt, P(out), hq, hkv, D, 16,
                                         1.0 / (D ** 0.5), E.MS_DTYPE_BF16, C.c_void_p(st.cuda_stream))
        assert rc == 0

    for _ in range(args.warmup):
        launch()
    ts = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        launch()
        e1.record(st)
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ts.sort()
    ms = ts[len(ts) // 2]
    flops = seqs * 4.0 * hq * D * (length * (length + 1) / 2)
    peaks_d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks_d.get("bf16_tflops", 1590.0))
    tf = flops / (ms / 1000.0) / 1e12
    print(json.dumps({"workload": f"{seqs} prompts x {length} tokens, causal, 16/8 heads x 128, bf16",
                      "tiles": nt, "ms": ms, "tflops": tf, "peak_tflops": peak, "frac": tf / peak,
                      "peak_source": "MEASURED_PEAKS.json bf16_tflops" if peaks_d else "fallback"}), flush=True)


def traffic_per_launch(algorithmic_bytes: float):
    """dram bytes (read + write) per attention launch: the committed ncu ratio of
    dram bytes to algorithmic bytes (profiles/k3_attention_traffic.json, from a
    capture of the config-2 launch) times this launch's algorithmic bytes."""
    p = ROOT / "profiles" / "k3_attention_traffic.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_algorithmic_byte"]) * algorithmic_bytes
        except (KeyError, ValueError):
            return None
    return None


def main():
    args = parse()
    rank, world, local = dist_env()
    n = world if world > 1 else args.gpus
    cfg_desc = {"workload": "Qwen3-0.6B-arch decode step, 256 seqs x ctx U[1,4096] (BASELINE config 2 shapes "
                            "through the full 28-layer model)",
                "model": "qwen3-0.6b-arch", "global_batch": args.batch * n, "seqs_per_gpu": args.batch,
                "ctx": "uniform[1,4096] at admission, +1 per step", "block_size": 16,
                "parallelism": f"dp{n} (independent replicas)", "l2": "inputs (60 GB KV/GPU) >> L2, no flush"}

    if args.kernel == "attention":
        run_attention_kernel(args, local)
        return
    if args.kernel == "norm_rope":
        run_norm_rope_kernels(args, local)
        return
    if args.kernel == "sample":
        run_sample_kernel(args, local)
        return
    if args.kernel == "prefill":
        run_prefill_kernel(args, local)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        steps = max(1, min(args.steps, 2))
        warm = max(1, min(args.warmup, 1))
        batches = cpu_batches(host_available_bytes())
        tps, cores, desc, rates = cpu_sample(batches, steps, warm)
        top = max(rates)
        line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": n,
                "steps": steps, "warmup": warm, "ms_per_step": top / tps * 1000, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg_desc,
                "batch": top, "tokens_per_s_by_batch": rates,
                "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc},
                "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device(f"cuda:{local}"))
    if args.config5:
        run_config5(args, rank, world, local)
        dist.barrier()
        dist.destroy_process_group()
        return
    if args.config4:
        run_config4(args, rank, world, local)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    r = run_ours(args, rank, world, local)
    tp_rec = None
    if world > 1 and not args.no_tp:
        tp_rec = run_tp(args, rank, world, local)
    if rank == 0:
        B, K = args.batch, args.steps
        value = n * B * K / (r["ms"] / 1000.0)
        e2e = n * B * K / (r["ms_e2e"] / 1000.0)
        peak, peak_kind = peaks()
        per_launch_ms = r["attn_ms"] / max(1, r["attn_launches"])
        per_launch_bytes = r["attn_bytes"] / max(1, r["attn_launches"])
        achieved = per_launch_bytes / (per_launch_ms / 1000.0) / 1e9
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n, "steps": K, "warmup": args.warmup,
                "ms_per_step": r["ms"] / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded random-init weights, N(0,1) KV)", "config": cfg_desc,
                "tokens_per_s_per_gpu": value / n,
                "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"],
                        "ms_per_step": r["ms_e2e"] / K, "tokens_per_s_per_gpu": e2e / n},
                "gpu_launches": r["gpu_launches"], "clocks": r["clocks"],
                "roofline": {"kernel": "paged_attention_kernel (K3 split-K GQA decode + combine)", "bound": "hbm",
                             "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                             "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                             "traffic": traffic_per_launch(per_launch_bytes), "algorithmic_bytes_per_launch": per_launch_bytes,
                             "ms_per_launch": per_launch_ms, "launches": r["attn_launches"],
                             "share_of_step": (r["attn_ms"] / r["kp"]) / (r["ms"] / K)},
                "cuda_graphs": r["graphs"], "memory_bytes": r["memory"]}
        if world <= 1 and not args.no_cpu_baseline:
            tps, cores, desc, _ = cpu_sample(cpu_batches(host_available_bytes()), 2, 1)
            line["cpu_baseline"] = {"value": tps, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc}
        if tp_rec is not None:
            line["tp"] = tp_rec
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

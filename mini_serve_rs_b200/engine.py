"""ctypes binding of include/ms_engine.h (libms_engine.so, sm_100a).

The library is required: importing this module without the built .so raises
immediately, so no code path can silently fall back to a CPU implementation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Dict, Iterable, Optional, Sequence

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libms_engine.so"

MS_OK, MS_E_INVALID, MS_E_PRESSURE, MS_E_DEVICE, MS_E_INJECTED, MS_E_QUARANTINED, MS_E_TOKEN_LIMIT, \
    MS_E_NOT_FOUND = range(8)
MS_DTYPE_F32, MS_DTYPE_BF16, MS_DTYPE_F16 = 0, 1, 2
MS_STEP_TOKENS_FROM_DEVICE = 1
MS_STEP_KEEP_LOGITS = 2
MS_FLAG_PREFILLED = 1
MS_FLAG_NO_TOKEN = 2


class MsModelCfg(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32),
                ("num_layers", C.c_int32), ("num_heads", C.c_int32), ("num_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("max_position_embeddings", C.c_int32), ("rope_theta", C.c_double),
                ("rms_norm_eps", C.c_double), ("qk_norm", C.c_int32), ("attn_bias", C.c_int32),
                ("tie_word_embeddings", C.c_int32), ("dtype", C.c_int32)]


class MsEngineOpts(C.Structure):
    _fields_ = [("device", C.c_int32), ("tp_rank", C.c_int32), ("tp_size", C.c_int32), ("nccl_comm", C.c_void_p),
                ("pool_blocks", C.c_int64), ("block_size", C.c_int32), ("max_seqs", C.c_int32),
                ("max_tokens_per_step", C.c_int32), ("max_blocks_per_seq", C.c_int32)]


class MsStepDesc(C.Structure):
    _fields_ = [("num_seqs", C.c_int32), ("seq_ids", C.POINTER(C.c_uint64)),
                ("input_tokens", C.POINTER(C.c_uint32)), ("positions", C.POINTER(C.c_int32)),
                ("flags", C.c_uint32), ("temperature", C.POINTER(C.c_float)), ("top_p", C.POINTER(C.c_float)),
                ("seeds", C.POINTER(C.c_uint64)), ("token_budget", C.c_int32)]


class MsPagesStats(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("total_blocks", "free_blocks", "cached_chunks", "cache_only_blocks",
                                         "hits", "misses", "tokens_saved", "evictions", "rejections",
                                         "reserved_blocks", "peak_reserved_blocks", "reservation_rejections")]


_P = C.c_void_p
_I32 = C.c_int32
_SIGS = {
    "ms_engine_create": ([C.POINTER(MsModelCfg), C.POINTER(MsEngineOpts), C.POINTER(_P)], C.c_int),
    "ms_engine_destroy": ([_P], C.c_int),
    "ms_engine_load_weight": ([_P, C.c_char_p, _P, C.c_int64, _I32, _I32], C.c_int),
    "ms_engine_finalize": ([_P], C.c_int),
    "ms_engine_memory": ([_P, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_int64)], C.c_int),
    "ms_seq_admit": ([_P, C.c_uint64, C.POINTER(C.c_uint32), _I32, C.POINTER(_I32), _I32, _I32], C.c_int),
    "ms_seq_append_block": ([_P, C.c_uint64, _I32], C.c_int),
    "ms_seq_release": ([_P, C.c_uint64], C.c_int),
    "ms_seq_cached_tokens": ([_P, C.c_uint64, C.POINTER(_I32)], C.c_int),
    "ms_step": ([_P, C.POINTER(MsStepDesc), C.POINTER(C.c_uint32), C.POINTER(C.c_uint8)], C.c_int),
    "ms_step_launch": ([_P, C.POINTER(MsStepDesc)], C.c_int),
    "ms_step_wait": ([_P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint8)], C.c_int),
    "ms_engine_stream": ([_P, C.POINTER(_P)], C.c_int),
    "ms_engine_set_profiling": ([_P, _I32], C.c_int),
    "ms_engine_profile": ([_P, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(C.c_double),
                           C.POINTER(C.c_double)], C.c_int),
    "ms_engine_profile_allreduce": ([_P, C.POINTER(C.c_int64), C.POINTER(C.c_double)], C.c_int),
    "ms_engine_set_graphs": ([_P, _I32], C.c_int),
    "ms_engine_tp_fused": ([_P, C.POINTER(_I32)], C.c_int),
    "ms_engine_set_tp_fused": ([_P, _I32], C.c_int),
    "ms_engine_graph_stats": ([_P, C.POINTER(C.c_int64), C.POINTER(C.c_int64), C.POINTER(_I32)], C.c_int),
    "ms_nccl_get_unique_id": ([C.c_char_p, _I32], C.c_int),
    "ms_nccl_comm_init": ([C.POINTER(_P), _I32, C.c_char_p, _I32, _I32], C.c_int),
    "ms_nccl_comm_destroy": ([_P], C.c_int),
    "ms_is_healthy": ([_P], C.c_int),
    "ms_mark_unhealthy": ([_P], C.c_int),
    "ms_inject_fault": ([_P, _I32], C.c_int),
    "ms_last_error": ([_P, C.c_char_p, _I32], C.c_int),
    "ms_debug_dump_tables": ([_P, C.POINTER(_I32), C.POINTER(_I32), C.POINTER(_I32), C.POINTER(C.c_int64),
                              C.POINTER(_I32)], C.c_int),
    "ms_debug_logits": ([_P, C.POINTER(C.c_float), C.c_int64], C.c_int),
    "ms_debug_pool_ptr": ([_P, _I32, _I32, C.POINTER(_P)], C.c_int),
    "ms_debug_buffer": ([_P, C.c_char_p, _P, C.c_int64], C.c_int),
    "ms_debug_stop_after_layer": ([_P, _I32], C.c_int),
    "ms_launch_pack": ([_P, _P, _P, _I32, _P, _P, _P, _I32, _P, _I32, _I32, _P, _P, _P, _P, _P, _P], C.c_int),
    "ms_launch_add_rmsnorm": ([_P, _P, _P, _P, _P, _P, _I32, _I32, C.c_float, _I32, _P], C.c_int),
    "ms_launch_qk_norm_rope_append": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I32, _I32, _I32, _I32, _I32,
                                       C.c_float, _I32, _P], C.c_int),
    "ms_attention_workspace_bytes": ([_I32, _I32, _I32, _I32, _I32], C.c_int64),
    "ms_launch_paged_attention": ([_P, _P, _P, _P, _I32, _P, _P, _I32, _I32, _P, _I32, _I32, _I32, _I32, C.c_float,
                                   _I32, _P, C.c_int64, _I32, _P], C.c_int),
    "ms_launch_paged_prefill": ([_P, _P, _P, _P, _I32, _P, _I32, _P, _I32, _I32, _I32, _I32, C.c_float, _I32, _P],
                                C.c_int),
    "ms_prefill_tiles": ([C.POINTER(_I32)] * 4 + [_I32, _I32, _I32, C.POINTER(_I32), _I32], C.c_int),
    "ms_launch_silu_mul": ([_P, _P, _I32, _I32, _I32, _P], C.c_int),
    "ms_launch_argmax": ([_P, _I32, _I32, _P, _P], C.c_int),
    "ms_launch_sample": ([_P, _I32, _I32, _P, _P, _P, _P, _P], C.c_int),
    "ms_kernel_status": ([_I32, C.POINTER(C.c_uint32)], C.c_int),
    "ms_test_set_attention_wait_limit": ([_I32], C.c_int),
    "ms_pages_create": ([C.c_int64, _I32, _I32, C.POINTER(_P)], C.c_int),
    "ms_pages_destroy": ([_P], C.c_int),
    "ms_pages_admit": ([_P, C.c_uint64, _P, _I32, _P, _I32, C.POINTER(_I32), C.POINTER(_I32)], C.c_int),
    "ms_pages_allocate_block": ([_P, C.c_uint64, C.POINTER(_I32)], C.c_int),
    "ms_pages_release": ([_P, C.c_uint64, C.POINTER(_I32)], C.c_int),
    "ms_pages_publish": ([_P, C.c_uint64, _P, _I32, C.POINTER(_I32)], C.c_int),
    "ms_pages_lookup": ([_P, _P, _I32, C.POINTER(_I32)], C.c_int),
    "ms_pages_reserve": ([_P, C.c_uint64, C.c_int64, C.c_int64], C.c_int),
    "ms_pages_stats_get": ([_P, C.POINTER(MsPagesStats)], C.c_int),
    "ms_prefix_chunk_hashes": ([_P, _I32, _I32, _P, _I32], C.c_int),
    "launch_rmsnorm_f32": ([_P, _P, _P, C.c_int, C.c_int, C.c_float], C.c_int),
    "launch_rmsnorm_f16": ([_P, _P, _P, C.c_int, C.c_int, C.c_float], C.c_int),
    "launch_rmsnorm_bf16": ([_P, _P, _P, C.c_int, C.c_int, C.c_float], C.c_int),
    "launch_paged_gqa_decode_tiled_f32": ([_P] * 6 + [C.c_int] * 4 + [C.c_float], C.c_int),
    "launch_paged_gqa_decode_tiled_f16": ([_P] * 6 + [C.c_int] * 4 + [C.c_float], C.c_int),
    "launch_paged_gqa_decode_tiled_bf16": ([_P] * 6 + [C.c_int] * 4 + [C.c_float], C.c_int),
    "launch_paged_gqa_decode_tiled_bf16_noalloc": ([_P] * 6 + [C.c_int] * 4 + [C.c_float], C.c_int),
}


def load_library(path: Optional[os.PathLike] = None) -> C.CDLL:
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `python -m mini_serve_rs_b200.build` "
                           "(this package has no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (args, res) in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


_LIB: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load_library()
    return _LIB


def exported_symbols() -> Iterable[str]:
    return tuple(_SIGS)


# ---- errors (src/core/errors.rs:8-17) -------------------------------------------


class EngineError(RuntimeError):
    code = -1


class CachePressure(EngineError):
    code = MS_E_PRESSURE


class BackendError(EngineError):
    code = MS_E_DEVICE


class NoHealthyWorkers(EngineError):
    code = MS_E_QUARANTINED


class TokenLimitExceeded(EngineError):
    code = MS_E_TOKEN_LIMIT


def error_for(code: int, msg: str) -> EngineError:
    if code == MS_E_PRESSURE:
        return CachePressure(msg)
    if code == MS_E_QUARANTINED:
        return NoHealthyWorkers(msg)
    if code == MS_E_TOKEN_LIMIT:
        return TokenLimitExceeded(msg)
    e = BackendError(msg)
    e.code = code
    return e


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def _i32p(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_int32))


def torch_dtype_code(t) -> int:
    import torch
    return {torch.float32: MS_DTYPE_F32, torch.bfloat16: MS_DTYPE_BF16, torch.float16: MS_DTYPE_F16}[t.dtype]


class Engine:
    """One engine per GPU: weights, paged KV pool and the step (ms_engine_*)."""

    def __init__(self, cfg, *, device: int = 0, pool_blocks: int, max_seqs: int = 256,
                 max_tokens_per_step: int = 8192, max_blocks_per_seq: int | None = None,
                 dtype: int = MS_DTYPE_BF16, tp_rank: int = 0, tp_size: int = 1, nccl_comm: int | None = None):
        """cfg: any object with the fields of oracle-style Config (vocab_size,
        hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
        num_key_value_heads, head_dim or hd(), max_position_embeddings,
        rope_theta, rms_norm_eps, qk_norm, attention_bias, tie_word_embeddings)."""
        self.lib = lib()
        self.cfg = cfg
        hd = cfg.hd() if hasattr(cfg, "hd") else cfg.head_dim
        self.c_cfg = MsModelCfg(cfg.vocab_size, cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers,
                                cfg.num_attention_heads, cfg.num_key_value_heads, hd, cfg.max_position_embeddings,
                                float(cfg.rope_theta), float(cfg.rms_norm_eps), int(cfg.qk_norm),
                                int(cfg.attention_bias), int(cfg.tie_word_embeddings), dtype)
        if max_blocks_per_seq is None:
            max_blocks_per_seq = (cfg.max_position_embeddings + 15) // 16
        self.opts = MsEngineOpts(device, tp_rank, tp_size, nccl_comm, pool_blocks, 16, max_seqs, max_tokens_per_step,
                                 max_blocks_per_seq)
        self.dtype = dtype
        self.max_seqs = max_seqs
        self.max_blocks_per_seq = max_blocks_per_seq
        h = C.c_void_p()
        rc = self.lib.ms_engine_create(C.byref(self.c_cfg), C.byref(self.opts), C.byref(h))
        if rc != MS_OK:
            raise error_for(rc, "ms_engine_create: " + self._err(None))
        self.h = h
        self._out_tok = np.zeros(max_seqs, np.uint32)
        self._out_flags = np.zeros(max_seqs, np.uint8)

    # -- plumbing
    def _err(self, h=...) -> str:
        buf = C.create_string_buffer(1024)
        self.lib.ms_last_error(self.h if h is ... else h, buf, 1024)
        return buf.value.decode(errors="replace")

    def _check(self, rc: int, what: str):
        if rc != MS_OK:
            raise error_for(rc, f"{what}: {self._err()}")

    def close(self):
        if getattr(self, "h", None):
            self.lib.ms_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- weights
    def load_weights(self, weights):
        """weights: dict or iterable of (name, torch tensor) on the CPU or on this
        engine's device; full (unsharded) tensors under tensor parallelism."""
        import torch
        items = weights.items() if hasattr(weights, "items") else weights
        for name, t in items:
            t = t.contiguous()
            on_dev = 1 if t.is_cuda else 0
            if not on_dev and t.dtype not in (torch.float32, torch.bfloat16, torch.float16):
                t = t.to(torch.float32)
            self._check(self.lib.ms_engine_load_weight(self.h, name.encode(), C.c_void_p(t.data_ptr()), t.numel(),
                                                       torch_dtype_code(t), on_dev), f"load {name}")
        self._check(self.lib.ms_engine_finalize(self.h), "finalize")

    def memory(self):
        w, p, s = C.c_int64(), C.c_int64(), C.c_int64()
        self._check(self.lib.ms_engine_memory(self.h, C.byref(w), C.byref(p), C.byref(s)), "memory")
        return {"weights": w.value, "pool": p.value, "workspace": s.value}

    # -- sequences
    def admit(self, seq_id: int, prompt: Sequence[int], blocks: Sequence[int], num_cached: int = 0):
        pr = np.ascontiguousarray(prompt, dtype=np.uint32)
        bl = np.ascontiguousarray(blocks, dtype=np.int32)
        self._check(self.lib.ms_seq_admit(self.h, seq_id, _u32p(pr), len(pr), _i32p(bl), len(bl), num_cached),
                    "admit")

    def append_block(self, seq_id: int, block: int):
        self._check(self.lib.ms_seq_append_block(self.h, seq_id, block), "append_block")

    def release(self, seq_id: int):
        self._check(self.lib.ms_seq_release(self.h, seq_id), "release")

    def cached_tokens(self, seq_id: int) -> int:
        v = C.c_int32()
        self._check(self.lib.ms_seq_cached_tokens(self.h, seq_id, C.byref(v)), "cached_tokens")
        return v.value

    # -- step
    def _desc(self, seq_ids, input_tokens, positions, flags, temperature=None, top_p=None, seeds=None,
              token_budget=0):
        ids = np.ascontiguousarray(seq_ids, dtype=np.uint64)
        toks = None if input_tokens is None else np.ascontiguousarray(input_tokens, dtype=np.uint32)
        pos = None if positions is None else np.ascontiguousarray(positions, dtype=np.int32)
        n = len(ids)

        def per_seq(v, dt):  # scalar or per-sequence array -> contiguous [n]
            if v is None:
                return None
            return np.ascontiguousarray(np.broadcast_to(np.asarray(v, dtype=dt), (n,)), dtype=dt)

        temp = per_seq(temperature, np.float32)
        tp = per_seq(top_p, np.float32)
        sd = per_seq(seeds, np.uint64)
        fp = lambda a: None if a is None else a.ctypes.data_as(C.POINTER(C.c_float))
        d = MsStepDesc(n, ids.ctypes.data_as(C.POINTER(C.c_uint64)),
                       None if toks is None else _u32p(toks), None if pos is None else _i32p(pos), flags,
                       fp(temp), fp(tp), None if sd is None else sd.ctypes.data_as(C.POINTER(C.c_uint64)),
                       int(token_budget))
        return d, (ids, toks, pos, temp, tp, sd)

    def step(self, seq_ids, input_tokens=None, positions=None, flags: int = 0, temperature=None, top_p=None,
             seeds=None, token_budget: int = 0):
        """One step; temperature / top_p / seeds (scalars or per-sequence) select
        on-device sampling for rows with temperature >= 1e-7 (greedy otherwise);
        token_budget > 0 chunks prefills (rows flagged MS_FLAG_NO_TOKEN)."""
        d, keep = self._desc(seq_ids, input_tokens, positions, flags, temperature, top_p, seeds, token_budget)
        n = len(keep[0])
        rc = self.lib.ms_step(self.h, C.byref(d), _u32p(self._out_tok),
                              self._out_flags.ctypes.data_as(C.POINTER(C.c_uint8)))
        self._check(rc, "step")
        return self._out_tok[:n].copy(), self._out_flags[:n].copy()

    def step_launch(self, seq_ids, input_tokens=None, positions=None, flags: int = 0, temperature=None,
                    top_p=None, seeds=None, token_budget: int = 0):
        d, keep = self._desc(seq_ids, input_tokens, positions, flags, temperature, top_p, seeds, token_budget)
        self._pending_n = len(keep[0])
        self._check(self.lib.ms_step_launch(self.h, C.byref(d)), "step_launch")

    def step_wait(self):
        rc = self.lib.ms_step_wait(self.h, _u32p(self._out_tok), self._out_flags.ctypes.data_as(C.POINTER(C.c_uint8)))
        self._check(rc, "step_wait")
        n = self._pending_n
        return self._out_tok[:n].copy(), self._out_flags[:n].copy()

    def stream_ptr(self) -> int:
        s = C.c_void_p()
        self._check(self.lib.ms_engine_stream(self.h, C.byref(s)), "stream")
        return s.value or 0

    # -- instrumentation
    def set_profiling(self, on: bool):
        self._check(self.lib.ms_engine_set_profiling(self.h, 1 if on else 0), "set_profiling")

    def profile(self):
        """(kernel_launches, attention launches, attention ms, attention algorithmic bytes)."""
        kl, al, ms, by = C.c_int64(), C.c_int64(), C.c_double(), C.c_double()
        self._check(self.lib.ms_engine_profile(self.h, C.byref(kl), C.byref(al), C.byref(ms), C.byref(by)),
                    "profile")
        return kl.value, al.value, ms.value, by.value

    def profile_allreduce(self):
        """(all-reduce sections bracketed, their summed ms) under tensor parallelism."""
        n, ms = C.c_int64(), C.c_double()
        self._check(self.lib.ms_engine_profile_allreduce(self.h, C.byref(n), C.byref(ms)), "profile_allreduce")
        return n.value, ms.value

    def tp_fused(self) -> bool:
        """True when TP all-reduces run as the fused peer-memory kernel."""
        v = _I32()
        self._check(self.lib.ms_engine_tp_fused(self.h, C.byref(v)), "tp_fused")
        return bool(v.value)

    def set_tp_fused(self, on: bool):
        """Fused peer-memory all-reduce (True, where set up) or NCCL (False) for
        later steps; every rank of the group switches at the same step."""
        self._check(self.lib.ms_engine_set_tp_fused(self.h, 1 if on else 0), "set_tp_fused")

    def set_graphs(self, on: bool):
        """Replay pure-decode steps from captured CUDA graphs (default on)."""
        self._check(self.lib.ms_engine_set_graphs(self.h, 1 if on else 0), "set_graphs")

    def graph_stats(self):
        """(graphs captured, steps replayed, graphs cached)."""
        c, r, n = C.c_int64(), C.c_int64(), _I32()
        self._check(self.lib.ms_engine_graph_stats(self.h, C.byref(c), C.byref(r), C.byref(n)), "graph_stats")
        return c.value, r.value, n.value

    # -- health
    def is_healthy(self) -> bool:
        return bool(self.lib.ms_is_healthy(self.h))

    def mark_unhealthy(self):
        self._check(self.lib.ms_mark_unhealthy(self.h), "mark_unhealthy")

    def inject_fault(self):
        self._check(self.lib.ms_inject_fault(self.h, 1), "inject_fault")

    # -- debugging
    def dump_tables(self, num_seqs: int):
        n = C.c_int32()
        self._check(self.lib.ms_debug_dump_tables(self.h, C.byref(n), None, None, None, None), "dump")
        T = n.value
        cu = np.zeros(num_seqs + 1, np.int32)
        pos = np.zeros(T, np.int32)
        slots = np.zeros(T, np.int64)
        bt = np.zeros((num_seqs, self.max_blocks_per_seq), np.int32)
        self._check(self.lib.ms_debug_dump_tables(self.h, C.byref(n), _i32p(cu), _i32p(pos),
                                                  slots.ctypes.data_as(C.POINTER(C.c_int64)), _i32p(bt)), "dump")
        return {"cu_seqlens": cu, "positions": pos, "slot_mapping": slots, "block_tables": bt}

    def logits(self, num_seqs: int) -> np.ndarray:
        out = np.zeros((num_seqs, self.cfg.vocab_size), np.float32)
        self._check(self.lib.ms_debug_logits(self.h, out.ctypes.data_as(C.POINTER(C.c_float)), out.size), "logits")
        return out

    def buffer(self, name: str, shape, dtype) -> np.ndarray:
        """Activation buffer of the last step (see ms_debug_buffer); dtype is a
        numpy dtype (np.float32, np.int32, or np.uint16 for raw bf16 bits)."""
        out = np.zeros(shape, dtype)
        self._check(self.lib.ms_debug_buffer(self.h, name.encode(), out.ctypes.data_as(C.c_void_p), out.nbytes),
                    f"buffer {name}")
        return out

    def stop_after_layer(self, layer: int):
        """Later steps end after `layer`'s MLP (-1: off); see ms_debug_stop_after_layer."""
        self._check(self.lib.ms_debug_stop_after_layer(self.h, layer), "stop_after_layer")

    def pool_ptr(self, layer: int, which: int) -> int:
        p = C.c_void_p()
        self._check(self.lib.ms_debug_pool_ptr(self.h, layer, which, C.byref(p)), "pool_ptr")
        return p.value


# ---- NCCL communicator helpers (tensor parallelism) ------------------------------


class Pages:
    """Host-side paged prefix cache + block manager (ms_pages_*): the
    scheduler's KVCache with prefix-cache page sharing.  No GPU needed."""

    def __init__(self, total_blocks: int, block_size: int = 16, max_chunks: int = 512):
        self.lib = lib()
        h = C.c_void_p()
        rc = self.lib.ms_pages_create(total_blocks, block_size, max_chunks, C.byref(h))
        if rc != MS_OK:
            raise error_for(rc, "ms_pages_create")
        self.h = h
        self.block_size = block_size

    @staticmethod
    def _toks(prompt):
        return np.ascontiguousarray(prompt, dtype=np.uint32)

    def admit(self, seq_id: int, prompt):
        """(block ids, cached tokens) for a new request; raises CachePressure."""
        pr = self._toks(prompt)
        cap = max(1, -(-max(len(pr), 1) // self.block_size))
        out = np.zeros(cap, np.int32)
        n, cached = _I32(), _I32()
        rc = self.lib.ms_pages_admit(self.h, seq_id, pr.ctypes.data, len(pr), out.ctypes.data, cap,
                                     C.byref(n), C.byref(cached))
        if rc != MS_OK:
            raise error_for(rc, "ms_pages_admit")
        return out[:n.value].tolist(), cached.value

    def reserve(self, seq_id: int, prompt_len: int, max_tokens: int):
        """Charge the request's worst-case pages against the pool (idempotent per
        id); raises CachePressure when they do not fit, TokenLimitExceeded for a
        zero-length prompt or zero max_tokens."""
        rc = self.lib.ms_pages_reserve(self.h, seq_id, prompt_len, max_tokens)
        if rc != MS_OK:
            raise error_for(rc, "Tensor memory budget exhausted" if rc == MS_E_PRESSURE else "ms_pages_reserve")

    def allocate_block(self, seq_id: int) -> int:
        b = _I32()
        rc = self.lib.ms_pages_allocate_block(self.h, seq_id, C.byref(b))
        if rc != MS_OK:
            raise error_for(rc, "ms_pages_allocate_block")
        return b.value

    def release(self, seq_id: int) -> int:
        n = _I32()
        self.lib.ms_pages_release(self.h, seq_id, C.byref(n))
        return n.value

    def publish(self, seq_id: int, prompt) -> int:
        pr = self._toks(prompt)
        n = _I32()
        rc = self.lib.ms_pages_publish(self.h, seq_id, pr.ctypes.data, len(pr), C.byref(n))
        if rc != MS_OK:
            raise error_for(rc, "ms_pages_publish")
        return n.value

    def lookup(self, prompt) -> int:
        pr = self._toks(prompt)
        n = _I32()
        rc = self.lib.ms_pages_lookup(self.h, pr.ctypes.data, len(pr), C.byref(n))
        if rc != MS_OK:
            raise error_for(rc, "ms_pages_lookup")
        return n.value

    def stats(self) -> dict:
        st = MsPagesStats()
        self.lib.ms_pages_stats_get(self.h, C.byref(st))
        return {n: getattr(st, n) for n, _ in MsPagesStats._fields_}

    def close(self):
        if getattr(self, "h", None):
            self.lib.ms_pages_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def chunk_hashes(tokens, chunk_size: int = 16):
    """The reference's chain keys (hex strings) computed by the library."""
    tk = np.ascontiguousarray(tokens, dtype=np.uint32)
    cap = max(1, len(tk) // chunk_size)
    out = np.zeros(cap * 32, np.uint8)
    n = lib().ms_prefix_chunk_hashes(tk.ctypes.data, len(tk), chunk_size, out.ctypes.data, cap)
    if n < 0:
        raise ValueError("ms_prefix_chunk_hashes")
    return [bytes(out[32 * i:32 * i + 32]).hex() for i in range(n)]


def kernel_status(device: int = 0) -> int:
    """Status bits of kernels launched without an engine on `device` since the
    last call (ms_kernel_status); clears them."""
    v = C.c_uint32()
    rc = lib().ms_kernel_status(device, C.byref(v))
    if rc != MS_OK:
        raise error_for(rc, "ms_kernel_status")
    return v.value


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    rc = lib().ms_nccl_get_unique_id(buf, 128)
    if rc != MS_OK:
        raise error_for(rc, "ms_nccl_get_unique_id failed (NCCL not loadable?)")
    return buf.raw


def nccl_comm_init(nranks: int, unique_id: bytes, rank: int, device: int) -> int:
    comm = C.c_void_p()
    rc = lib().ms_nccl_comm_init(C.byref(comm), nranks, unique_id, rank, device)
    if rc != MS_OK:
        raise error_for(rc, "ms_nccl_comm_init failed")
    return comm.value


def nccl_comm_destroy(comm: int):
    lib().ms_nccl_comm_destroy(comm)

"""Torch-CPU restatement of the reference model math (test infrastructure only).

Restates ``src/backends/qwen2.rs`` (Candle) op for op, including where the
reference rounds to the model dtype, and the prefill/decode order of
``CandleBackend::step_batch`` (``src/backends/candle.rs:377-698``).  Runs in
f32 (the reference's CPU dtype, ``candle.rs:184-187``) unless a dtype is given.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch


@dataclass
class Config:
    """Fields of ``qwen2.rs:9-54`` read by the forward step."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_position_embeddings: int
    head_dim: Optional[int] = None
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    qk_norm: bool = True
    attention_bias: bool = False
    tie_word_embeddings: bool = True

    def hd(self) -> int:
        # qwen2.rs:49-53
        return self.head_dim or self.hidden_size // self.num_attention_heads


def qwen3_0_6b() -> Config:
    """Qwen3-0.6B architecture (the BASELINE configs 1-4)."""
    return Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                  num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                  max_position_embeddings=40960, head_dim=128, rope_theta=1e6,
                  rms_norm_eps=1e-6, qk_norm=True, attention_bias=False,
                  tie_word_embeddings=True)


def qwen2_5_7b() -> Config:
    """Qwen2.5-7B architecture."""
    return Config(vocab_size=152064, hidden_size=3584, intermediate_size=18944,
                  num_hidden_layers=28, num_attention_heads=28, num_key_value_heads=4,
                  max_position_embeddings=32768, head_dim=128, rope_theta=1e6,
                  rms_norm_eps=1e-6, qk_norm=False, attention_bias=True,
                  tie_word_embeddings=False)


def weight_shapes(cfg: Config) -> Dict[str, tuple]:
    """Hugging Face tensor names and shapes the reference's VarBuilder reads
    (qwen2.rs:157-159, 234-260, 396-405, 455-465, 592-596)."""
    d = cfg.hd()
    h = cfg.hidden_size
    out = {"model.embed_tokens.weight": (cfg.vocab_size, h), "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        out["lm_head.weight"] = (cfg.vocab_size, h)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = (h,)
        out[p + "post_attention_layernorm.weight"] = (h,)
        out[p + "self_attn.q_proj.weight"] = (cfg.num_attention_heads * d, h)
        out[p + "self_attn.k_proj.weight"] = (cfg.num_key_value_heads * d, h)
        out[p + "self_attn.v_proj.weight"] = (cfg.num_key_value_heads * d, h)
        out[p + "self_attn.o_proj.weight"] = (h, cfg.num_attention_heads * d)
        if cfg.attention_bias:
            out[p + "self_attn.q_proj.bias"] = (cfg.num_attention_heads * d,)
            out[p + "self_attn.k_proj.bias"] = (cfg.num_key_value_heads * d,)
            out[p + "self_attn.v_proj.bias"] = (cfg.num_key_value_heads * d,)
        if cfg.qk_norm:
            out[p + "self_attn.q_norm.weight"] = (d,)
            out[p + "self_attn.k_norm.weight"] = (d,)
        out[p + "mlp.gate_proj.weight"] = (cfg.intermediate_size, h)
        out[p + "mlp.up_proj.weight"] = (cfg.intermediate_size, h)
        out[p + "mlp.down_proj.weight"] = (h, cfg.intermediate_size)
    return out


def sin_fixture_weights(cfg: Config) -> Dict[str, torch.Tensor]:
    """Deterministic nonzero weights of tests/test_pretrained_numerics.rs:88-100:
    rank-1 tensors are 1; others are sin((i + offset) * 0.17) * 0.1 with
    offset = sum of the name's bytes, i over the row-major flattening."""
    out = {}
    for name, shape in weight_shapes(cfg).items():
        n = int(np.prod(shape))
        if len(shape) == 1:
            out[name] = torch.ones(shape, dtype=torch.float32)
        else:
            off = sum(name.encode())
            i = np.arange(n, dtype=np.int64) + off
            # f32 multiply then f32 sin, as the Rust expression does
            vals = np.sin((i.astype(np.float32) * np.float32(0.17)).astype(np.float32))
            out[name] = torch.from_numpy((vals * np.float32(0.1)).astype(np.float32)).reshape(shape)
    return out


def random_weights(cfg: Config, seed: int, std: float = 0.02,
                   norm_std: float = 0.0) -> Dict[str, torch.Tensor]:
    """Seeded N(0, std) matrices and biases; norm weights 1 (+ N(0, norm_std)),
    generated in sorted-name order from one numpy PCG64 stream so any machine
    regenerates them bit-identically."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name in sorted(weight_shapes(cfg)):
        shape = weight_shapes(cfg)[name]
        if name.endswith("norm.weight"):
            w = np.ones(shape, np.float32)
            if norm_std:
                w = w + rng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)
            out[name] = torch.from_numpy(w.astype(np.float32))
        else:
            out[name] = torch.from_numpy(
                (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32))
    return out


# --------------------------------------------------------------------------
# layers


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """qwen2.rs:68-75: f32 variance, divide by sqrt(var + eps), cast back to
    the input dtype, then multiply by the weight in that dtype."""
    dtype = x.dtype
    xf = x.to(torch.float32)
    var = (xf * xf).mean(dim=-1, keepdim=True)
    norm = torch.sqrt(var + eps)
    return (xf / norm).to(dtype) * w.to(dtype)


def inv_freq(cfg: Config) -> np.ndarray:
    """qwen2.rs:94-97: theta.powf(i/dim) in f64, cast to f32, then 1/x in f32."""
    dim = cfg.hd()
    vals = [np.float32(1.0) / np.float32(cfg.rope_theta ** (i / dim)) for i in range(0, dim, 2)]
    return np.array(vals, dtype=np.float32)


def rope_tables(cfg: Config, dtype=torch.float32, max_pos: Optional[int] = None):
    """qwen2.rs:91-108: freqs = t (f32) x inv_freq (f32); sin/cos in f32, cast
    to the model dtype.  Returns (cos, sin) of shape [max_pos, dim/2]."""
    n = max_pos or cfg.max_position_embeddings
    t = torch.arange(n, dtype=torch.float32).reshape(n, 1)
    f = torch.from_numpy(inv_freq(cfg)).reshape(1, -1)
    freqs = t * f  # k = 1 matmul: one f32 product per entry
    return freqs.cos().to(dtype), freqs.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """qwen2.rs:125-130."""
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """qwen2.rs:132-142 with cos/sin already selected per position:
    x [..., t, d], cos/sin [t, d/2] (broadcast over leading dims)."""
    c = torch.cat([cos, cos], dim=-1)
    s = torch.cat([sin, sin], dim=-1)
    return x * c + rotate_half(x) * s


def silu(x: torch.Tensor) -> torch.Tensor:
    dtype = x.dtype
    xf = x.to(torch.float32)
    return (xf / (1.0 + torch.exp(-xf))).to(dtype)


def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None) -> torch.Tensor:
    """candle_nn::Linear: x @ w.T (+ b)."""
    y = torch.matmul(x, w.t())
    if b is not None:
        y = y + b
    return y


def softmax_last(x: torch.Tensor) -> torch.Tensor:
    """candle_nn::ops::softmax over the last dim (max-subtracted, computed in
    the tensor's dtype)."""
    m = x.max(dim=-1, keepdim=True).values
    e = torch.exp(x - m)
    return e / e.sum(dim=-1, keepdim=True)


def decode_attention_gqa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                         num_kv_heads: int, groups: int, scale: float) -> torch.Tensor:
    """qwen2.rs:182-203: q [Hq, D], k/v [Hkv, L, D] -> [Hq, D]."""
    outs = []
    for h in range(num_kv_heads):
        qg = q[h * groups:(h + 1) * groups]
        scores = torch.matmul(qg, k[h].t()) * scale
        outs.append(torch.matmul(softmax_last(scores), v[h]))
    return torch.cat(outs, dim=0)


# --------------------------------------------------------------------------
# model with per-request contiguous KV (candle_nn::kv_cache::KvCache)


class SeqState:
    """One request's model clone: per-layer K/V buffers [Hkv, capacity, D]
    filled in place and read through narrowed views, as
    candle_nn::kv_cache::KvCache does (qwen2.rs:219, 349-361, 604-618)."""

    def __init__(self, cfg: Config, capacity: int):
        self.capacity = capacity
        self.k: List[Optional[torch.Tensor]] = [None] * cfg.num_hidden_layers
        self.v: List[Optional[torch.Tensor]] = [None] * cfg.num_hidden_layers
        self.n: List[int] = [0] * cfg.num_hidden_layers

    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor):
        """k, v: [Hkv, t, D]; returns views of the cached [Hkv, len, D]."""
        t = k.shape[1]
        if self.k[layer] is None:
            shape = (k.shape[0], self.capacity, k.shape[2])
            self.k[layer] = torch.empty(shape, dtype=k.dtype)
            self.v[layer] = torch.empty(shape, dtype=v.dtype)
        n = self.n[layer]
        if n + t > self.capacity:
            raise RuntimeError("kv cache capacity exceeded")
        self.k[layer][:, n:n + t] = k
        self.v[layer][:, n:n + t] = v
        self.n[layer] = n + t
        return self.k[layer][:, :n + t], self.v[layer][:, :n + t]

    def length(self) -> int:
        return self.n[0]

    def fill_random(self, length: int, gen: torch.Generator, dtype=torch.float32):
        """Synthetic cached context of `length` tokens with N(0,1) K/V."""
        for layer in range(len(self.k)):
            if self.k[layer] is None:
                raise RuntimeError("call append once per layer (or use preallocate) first")
            self.k[layer][:, :length] = torch.randn(self.k[layer][:, :length].shape, generator=gen, dtype=dtype)
            self.v[layer][:, :length] = torch.randn(self.v[layer][:, :length].shape, generator=gen, dtype=dtype)
            self.n[layer] = length

    def preallocate(self, num_kv_heads: int, head_dim: int, dtype=torch.float32):
        for layer in range(len(self.k)):
            self.k[layer] = torch.empty((num_kv_heads, self.capacity, head_dim), dtype=dtype)
            self.v[layer] = torch.empty((num_kv_heads, self.capacity, head_dim), dtype=dtype)


class QwenRef:
    """ModelForCausalLM of qwen2.rs:583-764 over explicit per-request state."""

    def __init__(self, cfg: Config, weights: Dict[str, torch.Tensor], dtype=torch.float32):
        self.cfg = cfg
        self.dtype = dtype
        self.w = {k: v.to(dtype) for k, v in weights.items()}
        self.cos, self.sin = rope_tables(cfg, dtype, max_pos=min(cfg.max_position_embeddings, 65536))
        self.lm_head = self.w.get("lm_head.weight", self.w["model.embed_tokens.weight"])
        # per-layer activations, filled by forward() when set to a dict:
        # ("attn", l) attention output before o_proj, ("x_norm", l) the
        # post-attention RMSNorm, ("x_resid", l) the residual after attention,
        # "last_norm" the final norm of the last position
        self.capture: Optional[Dict] = None

    # ---- one decoder layer, q_len tokens of a single request (qwen2.rs:279-347, 414-428)
    def _attn(self, l: int, xs: torch.Tensor, state: SeqState, offset: int) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        p = f"model.layers.{l}.self_attn."
        t = xs.shape[0]
        d, hq, hkv = cfg.hd(), cfg.num_attention_heads, cfg.num_key_value_heads
        q = linear(xs, w[p + "q_proj.weight"], w.get(p + "q_proj.bias")).reshape(t, hq, d)
        k = linear(xs, w[p + "k_proj.weight"], w.get(p + "k_proj.bias")).reshape(t, hkv, d)
        v = linear(xs, w[p + "v_proj.weight"], w.get(p + "v_proj.bias")).reshape(t, hkv, d)
        v = v.transpose(0, 1)
        if cfg.qk_norm:
            q = rms_norm(q, w[p + "q_norm.weight"], cfg.rms_norm_eps)
            k = rms_norm(k, w[p + "k_norm.weight"], cfg.rms_norm_eps)
        q = q.transpose(0, 1)  # [hq, t, d]
        k = k.transpose(0, 1)
        cos = self.cos[offset:offset + t]
        sin = self.sin[offset:offset + t]
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        kk, vv = state.append(l, k, v)
        scale = 1.0 / math.sqrt(d)
        g = hq // hkv
        if t == 1:
            out = decode_attention_gqa(q[:, 0], kk, vv, hkv, g, scale).reshape(1, hq * d)
        else:
            kr = kk.repeat_interleave(g, dim=0)
            vr = vv.repeat_interleave(g, dim=0)
            att = torch.matmul(q, kr.transpose(1, 2)) * scale  # [hq, t, t+off]
            mask = torch.zeros(t, offset + t, dtype=att.dtype)
            i = torch.arange(t).reshape(t, 1)
            j = torch.arange(t).reshape(1, t)
            mask[:, offset:] = torch.where(i < j, torch.tensor(float("-inf")), torch.tensor(0.0)).to(att.dtype)
            att = softmax_last(att + mask)
            out = torch.matmul(att, vr).transpose(0, 1).reshape(t, hq * d)
        if self.capture is not None:
            self.capture[("attn", l)] = out
        return linear(out, w[p + "o_proj.weight"])

    def _mlp(self, l: int, xs: torch.Tensor) -> torch.Tensor:
        """qwen2.rs:169-174."""
        w = self.w
        p = f"model.layers.{l}.mlp."
        lhs = silu(linear(xs, w[p + "gate_proj.weight"]))
        rhs = linear(xs, w[p + "up_proj.weight"])
        return linear(lhs * rhs, w[p + "down_proj.weight"])

    def _layer(self, l: int, xs: torch.Tensor, state: SeqState, offset: int) -> torch.Tensor:
        """qwen2.rs:414-428."""
        w, eps = self.w, self.cfg.rms_norm_eps
        p = f"model.layers.{l}."
        residual = xs
        h = rms_norm(xs, w[p + "input_layernorm.weight"], eps)
        h = self._attn(l, h, state, offset)
        xs = h + residual
        residual = xs
        h = rms_norm(xs, w[p + "post_attention_layernorm.weight"], eps)
        if self.capture is not None:
            self.capture[("x_resid", l)] = xs
            self.capture[("x_norm", l)] = h
        h = self._mlp(l, h)
        return residual + h

    def forward(self, ids: Sequence[int], state: SeqState, offset: int) -> torch.Tensor:
        """ModelForCausalLM::forward (qwen2.rs:620-626): logits of the last
        position, f32 [vocab]."""
        xs = self.w["model.embed_tokens.weight"][torch.as_tensor(list(ids), dtype=torch.long)]
        for l in range(self.cfg.num_hidden_layers):
            xs = self._layer(l, xs, state, offset)
        xs = rms_norm(xs, self.w["model.norm.weight"], self.cfg.rms_norm_eps)
        if self.capture is not None:
            self.capture["last_norm"] = xs[-1]
        return linear(xs[-1:], self.lm_head)[0].to(torch.float32)

    def step_decode_batch(self, states: List[SeqState], ids: Sequence[int],
                          positions: Sequence[int]) -> torch.Tensor:
        """qwen2.rs:630-764: batched norms/projections/MLP, per-sequence
        append + zero-copy GQA.  Returns f32 logits [B, vocab]."""
        b = len(states)
        if b == 1:
            return self.forward([ids[0]], states[0], positions[0]).reshape(1, -1)
        cfg, w, eps = self.cfg, self.w, self.cfg.rms_norm_eps
        d, hq, hkv = cfg.hd(), cfg.num_attention_heads, cfg.num_key_value_heads
        g = hq // hkv
        scale = 1.0 / math.sqrt(d)
        xs = w["model.embed_tokens.weight"][torch.as_tensor(list(ids), dtype=torch.long)]
        pos = torch.as_tensor(list(positions), dtype=torch.long)
        cos = self.cos[pos]  # [b, d/2]
        sin = self.sin[pos]
        for l in range(cfg.num_hidden_layers):
            p = f"model.layers.{l}."
            residual = xs
            h = rms_norm(xs, w[p + "input_layernorm.weight"], eps)
            q = linear(h, w[p + "self_attn.q_proj.weight"], w.get(p + "self_attn.q_proj.bias")).reshape(b, hq, d)
            k = linear(h, w[p + "self_attn.k_proj.weight"], w.get(p + "self_attn.k_proj.bias")).reshape(b, hkv, d)
            v = linear(h, w[p + "self_attn.v_proj.weight"], w.get(p + "self_attn.v_proj.bias")).reshape(b, hkv, d)
            if cfg.qk_norm:
                q = rms_norm(q, w[p + "self_attn.q_norm.weight"], eps)
                k = rms_norm(k, w[p + "self_attn.k_norm.weight"], eps)
            c = torch.cat([cos, cos], dim=-1).reshape(b, 1, d)
            s = torch.cat([sin, sin], dim=-1).reshape(b, 1, d)
            q = q * c + rotate_half(q) * s
            k = k * c + rotate_half(k) * s
            outs = []
            for i in range(b):
                kk, vv = states[i].append(l, k[i].reshape(hkv, 1, d), v[i].reshape(hkv, 1, d))
                outs.append(decode_attention_gqa(q[i], kk, vv, hkv, g, scale))
            attn = torch.stack(outs, dim=0).reshape(b, hq * d)
            xs_mid = residual + linear(attn, w[p + "self_attn.o_proj.weight"])
            h = rms_norm(xs_mid, w[p + "post_attention_layernorm.weight"], eps)
            xs = xs_mid + self._mlp(l, h)
        xs = rms_norm(xs, w["model.norm.weight"], eps)
        return linear(xs, self.lm_head).to(torch.float32)


def argmax_first(logits: torch.Tensor) -> int:
    """Greedy sampling (candle.rs:747-751): argmax of f32 logits; ties resolve
    to the first index."""
    return int(torch.argmax(logits.to(torch.float32)).item())


# --------------------------------------------------------------------------
# CandleBackend::step_batch restated (no prefix cache, greedy)


@dataclass
class RefSequence:
    """The fields of ActiveSequence (src/core/types.rs:231-254) step_batch reads."""

    request_id: str
    prompt_tokens: List[int]
    max_tokens: int
    output_tokens: List[int] = field(default_factory=list)
    is_prefilled: bool = False
    kv_blocks: List[int] = field(default_factory=list)


class RefBackend:
    """candle.rs:377-698 with greedy sampling: prefill each new sequence alone,
    then one batched decode over the rest; per-request model state is created
    on first sight with capacity prompt + max_tokens (candle.rs:405-418) and
    dropped when the sequence finishes (candle.rs:678-685)."""

    def __init__(self, model: QwenRef, eos_ids: Sequence[int] = ()):
        self.model = model
        self.states: Dict[str, SeqState] = {}
        self.eos = set(eos_ids)
        self.last_logits: Dict[str, torch.Tensor] = {}

    def cancel_sequence(self, request_id: str):
        self.states.pop(request_id, None)

    def step_batch(self, seqs: List[RefSequence]) -> List[int]:
        if not seqs:
            return []
        for s in seqs:
            if s.request_id not in self.states:
                self.states[s.request_id] = SeqState(self.model.cfg, len(s.prompt_tokens) + s.max_tokens)
        results: List[Optional[int]] = [None] * len(seqs)
        for i, s in enumerate(seqs):
            if not s.is_prefilled:
                s.is_prefilled = True
                logits = self.model.forward(s.prompt_tokens, self.states[s.request_id], 0)
                self.last_logits[s.request_id] = logits
                results[i] = argmax_first(logits)
        dec = [i for i in range(len(seqs)) if results[i] is None]
        if dec:
            ids = [seqs[i].output_tokens[-1] if seqs[i].output_tokens else 1 for i in dec]
            pos = [len(seqs[i].prompt_tokens) + len(seqs[i].output_tokens) - 1
                   if seqs[i].output_tokens else 0 for i in dec]
            logits = self.model.step_decode_batch([self.states[seqs[i].request_id] for i in dec], ids, pos)
            for k, i in enumerate(dec):
                self.last_logits[seqs[i].request_id] = logits[k]
                results[i] = argmax_first(logits[k])
        for i, s in enumerate(seqs):
            if results[i] in self.eos or len(s.output_tokens) + 1 >= s.max_tokens:
                self.states.pop(s.request_id, None)
        return [int(r) for r in results]

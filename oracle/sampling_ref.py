"""CPU restatement of token sampling (test infrastructure only).

Two functions:

* `candle_probs` restates the distribution the reference samples from.  The
  reference's sample_token (src/backends/candle.rs:737-763) hands f32 logits
  to candle_transformers::generation::LogitsProcessor (candle-transformers
  0.11.0, Cargo.lock:390-391; that crate's source is not in the reference
  tree).  Its published algorithm is restated here:
  - LogitsProcessor::new maps temperature < 1e-7 to ArgMax;
  - top_p is Some only for 0 < top_p < 1 (candle.rs:754-758);
  - scaled logits are logits * (1 / temperature) in f32 (candle's Tensor / f64
    is an affine multiply);
  - softmax over the last dim in f32 (max subtracted, exp, sum, divide);
  - sample_topp sorts probabilities descending (a stable sort of the indices,
    so ties stay in index order).  It walks that order with an f32 running sum
    and zeroes every probability met once the sum has reached top_p;
  - the token is drawn from the remaining (unnormalised) weights.
  The reference seeds its generator from the wall clock (candle.rs:576-580,
  648-652), so only this distribution can be compared, not its draws.

* `sample_like_kernel` restates the device kernel (ms_sample.cu) exactly.  It
  has the same integer weights, the same nucleus and the same race scores
  z - log(-log(U)) over the same SplitMix64 stream, so the GPU and this
  function agree on the drawn token for a given seed.  The only exceptions are
  rows where CUDA's expf/logf (and the kernel's fast outer log, 3 ulp) and
  numpy's differ at a decision point: two race scores within about 1e-6 of
  each other, or a mass sum exactly at the target.
"""
from __future__ import annotations

import numpy as np

FIX = 2.0 ** 40
_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _f32(v) -> float:
    return float(np.float32(v))


def greedy(temperature: float) -> bool:
    return not (_f32(temperature) >= 1e-7)


def _nucleus(top_p) -> bool:
    return top_p is not None and 0.0 < _f32(top_p) < 1.0


def scaled(logits, temperature: float) -> np.ndarray:
    """z = logits * f32(1 / f64(temperature)), rounded in f32."""
    x = np.asarray(logits, np.float32)
    return (x * np.float32(1.0 / _f32(temperature))).astype(np.float32)


def candle_probs(logits, temperature: float, top_p: float | None):
    """Weights LogitsProcessor draws from (unnormalised, zeros outside the nucleus)."""
    z = scaled(logits, temperature)
    e = np.exp(z - z.max()).astype(np.float32)
    prs = (e / e.sum(dtype=np.float32)).astype(np.float32)
    if not _nucleus(top_p):
        return prs
    order = np.argsort(-prs, kind="stable")
    out = prs.copy()
    cum = np.float32(0.0)
    p = np.float32(top_p)
    for i in order:
        if cum >= p:
            out[i] = 0.0
        else:
            cum = np.float32(cum + prs[i])
    return out


def splitmix64_uniform(seed: int, idx: np.ndarray) -> np.ndarray:
    """(top 24 bits of SplitMix64(seed + (i + 1) * golden)) + 0.5, over 2^24: in (0, 1)."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (idx.astype(np.uint64) + np.uint64(1)) * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    top = (z >> np.uint64(40)).astype(np.float32)
    return ((top + np.float32(0.5)) * np.float32(1.0 / 16777216.0)).astype(np.float32)


def kernel_weights(logits, temperature: float):
    """e = exp(z - max z) in f32 and the integer weights trunc(e * 2^40)."""
    z = scaled(logits, temperature)
    e = np.exp((z - z.max()).astype(np.float32)).astype(np.float32)
    w = np.where(e > 0, np.floor(e.astype(np.float64) * FIX), 0).astype(np.uint64)
    return e, w


def kept_mask(logits, temperature: float, top_p: float | None) -> np.ndarray:
    """Tokens the kernel keeps: the shortest prefix of (e descending, index
    ascending) whose fixed-point mass reaches ceil(top_p * W)."""
    e, w = kernel_weights(logits, temperature)
    if not _nucleus(top_p):
        return e > 0
    W = int(w.sum(dtype=np.uint64))
    target = np.uint64(np.ceil(_f32(top_p) * float(W)))
    order = np.lexsort((np.arange(len(e)), -e.astype(np.float64)))
    cum = np.cumsum(w[order], dtype=np.uint64)
    m = int(np.argmax(cum >= target))  # first prefix reaching the target
    keep = np.zeros(len(e), bool)
    keep[order[:m + 1]] = True
    return keep & (w > 0)


def sample_like_kernel(logits, temperature: float, top_p: float | None, seed: int) -> int | None:
    """The token ms_sample.cu draws, or None for greedy rows (argmax left in place)."""
    if greedy(temperature):
        return None
    z = scaled(logits, temperature)
    keep = kept_mask(logits, temperature, top_p)
    u = splitmix64_uniform(seed, np.arange(len(z)))
    E = (-np.log(u)).astype(np.float32)
    race = (z - np.log(E).astype(np.float32)).astype(np.float32)
    score = np.where(keep, race, np.float32(-np.inf))
    return int(np.argmax(score))  # first index among equal maxima


def explains_mismatch(logits, temperature: float, top_p: float | None, seed: int, got: int,
                      ulps: float = 16.0) -> bool:
    """True when a kernel draw `got` that differs from sample_like_kernel can
    only come from the last-bit differences between the device's expf / logf
    and numpy's exp / log (the restatement cannot reproduce those bits):

    * both tokens are in the restated nucleus and their race scores are within
      `ulps` f32 ulps of each other (a near tie of the race), or
    * `got` sits at the edge of the restated nucleus: the fixed-point mass
      ranked up to it is within 1e-5 of ceil(top_p * W), so a weight a few
      ulps off moves the edge."""
    want = sample_like_kernel(logits, temperature, top_p, seed)
    if want is None or got == want or not (0 <= got < len(logits)):
        return got == want
    z = scaled(logits, temperature)
    u = splitmix64_uniform(seed, np.arange(len(z)))
    race = (z - np.log((-np.log(u)).astype(np.float32)).astype(np.float32)).astype(np.float32)
    keep = kept_mask(logits, temperature, top_p)
    tol = ulps * float(np.spacing(np.float32(max(abs(race[got]), abs(race[want])))))
    if keep[got] and abs(float(race[got]) - float(race[want])) <= tol:
        return True
    if _nucleus(top_p):
        e, w = kernel_weights(logits, temperature)
        W = float(w.sum(dtype=np.uint64))
        target = np.ceil(_f32(top_p) * W)
        order = np.lexsort((np.arange(len(e)), -e.astype(np.float64)))
        cum = np.cumsum(w[order], dtype=np.uint64).astype(np.float64)
        rank = int(np.nonzero(order == got)[0][0])
        before = cum[rank - 1] if rank > 0 else 0.0
        return min(abs(before - target), abs(cum[rank] - target)) <= 1e-5 * W
    return False

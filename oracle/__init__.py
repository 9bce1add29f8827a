"""CPU oracle for the continuous-batching forward step -- TEST INFRASTRUCTURE ONLY.

Nothing in this package is part of the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may
import it, and only as the checker (or, in ``bench.py --impl reference``, as
the timed restatement of the reference's CPU path).  The product path in
``mini_serve_rs_b200`` never calls into this package.

Contents (each function cites the reference file:line it restates; all paths
are relative to the Harsha-Karimikonda/mini-serve-rs project root):

* ``qwen_ref``      -- torch-CPU restatement of ``src/backends/qwen2.rs`` (model
                       math, contiguous per-request KV caches) and of the
                       prefill-then-batched-decode order of
                       ``src/backends/candle.rs:377-698`` with greedy sampling.
* ``kv_cache_ref``  -- restatement of ``src/cache/kv_cache.rs`` (LIFO free stack).
* ``scheduler_ref`` -- restatement of the admission / growth / eviction order of
                       ``src/scheduler/scheduler.rs:298-559``.
* ``packer_ref``    -- numpy restatement of the ragged-batch metadata
                       (cu_seqlens, positions, slot_mapping, block tables).
* ``kernels_ref``   -- fp32 references for paged GQA attention, RMSNorm,
                       QK-norm + RoPE, SiLU-mul, argmax.

Pinning: ``tests/golden/`` holds vectors produced by (a) Hugging Face
``transformers`` Qwen2/Qwen3 on CPU f32 -- the library the reference itself
uses as its independent golden generator
(``tests/fixtures/generation/generate_reference.py``) -- and (b) the torch
reference functions of ``scripts/validate_cuda_kernels.py:21-46``, imported
from the reference tree.  The scripts that made them sit beside the fixtures.
Candle-internal choices no reference test pins (softmax max-subtraction,
argmax tie-break, libm sin/cos ulps) are restated, not pinned.
"""

"""CPU oracle for the Qwen3 attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference engine's own algorithms for the
three hot-path operations (paged decode attention, varlen causal prefill
attention, KV-cache slot scatter) plus the QK-RMSNorm / RoPE input transforms.
Every function cites the reference file:line it follows (paths are relative to
the uphome/Qwen3-engine-from-scratch repository root).

Who may use it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / ``--impl reference`` legs, and there only as the checker or the
timed CPU baseline.  The product path (``qwen3_engine_from_scratch_b200``)
never imports anything from here and fails loudly when its CUDA library is
missing.

Parity pin: ``tests/golden/*.npz`` hold outputs of the reference's own PyTorch
functions (``qwen3/paged_attention.py:paged_attention``,
``qwen3/attention.py:Qwen3Attention._standard_attention``,
``qwen3/PagedKVcache.py:PagedKVCache.update``,
``qwen3/kernels/paged_attention.py`` scatter semantics, ``qwen3/norm.py``,
``qwen3/rope.py``), produced by ``tests/golden/make_golden.py`` with the
reference imported in the build container.  ``tests/test_oracle_golden.py``
checks this oracle against them.
"""

from .attention import (  # noqa: F401
    bf16_round,
    bf16_bits,
    from_bf16_bits,
    rms_norm,
    rope_cos_sin,
    apply_rope,
    kv_scatter_rows,
    kv_scatter_slots,
    paged_decode,
    varlen_prefill,
    prefill_batched,
    decode_bytes,
    prefill_flops,
)
from .synth import det_normal, det_uniform_int, det_permutation  # noqa: F401

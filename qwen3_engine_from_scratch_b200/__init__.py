"""B200-native (sm_100a) attention hot path for the Qwen3 inference engine.

Hand-written CUDA kernels behind the C ABI in ``include/qwen3_b200_attn.h``:

* paged decode attention (split-K flash-decoding, TMA-staged pages, mma.sync
  with the GQA heads on the N side, splits merged by the last one to finish);
* varlen causal prefill attention (tcgen05 MMAs with TMEM accumulators, TMA
  tiles, persistent CTAs), also over the paged cache (chunked prefill);
* KV-cache slot scatter (row-addressed and slot_mapping-addressed);
* the fused QK-RMSNorm + RoPE + KV write prologue and the fused token sampler.

``ops`` holds the reference-facing functions (same names and arguments as the
reference engine's kernel wrappers), ``paged_kv`` the host-side pool / request
handles, ``shim`` the drop-in binding into the reference engine, and
``dist`` the multi-GPU request sharding and ``graph_runner`` the per-bucket
CUDA-graph pool of the decode step.
"""

from .ops import (  # noqa: F401
    paged_attention_decode_triton,
    triton_paged_attention_decode,
    triton_paged_attention_decode_batch,
    update_kv_batch_triton,
    flash_attention_prefill,
    flash_attention_prefill_batched,
    paged_decode,
    paged_decode_kv_write,
    kv_scatter_rows,
    kv_scatter_slots,
    kv_scatter_span,
    paged_cache_update,
    qk_norm_rope_kv_write,
    paged_prefill,
    sample_tokens,
    device_status,
    clear_device_status,
    check_device_status,
    decode_workspace_bytes,
)
from .paged_kv import KVCachePool, PagedKVCache  # noqa: F401
from .graph_runner import GraphRunner, kv_pool_blocks  # noqa: F401

__version__ = "0.1.0"

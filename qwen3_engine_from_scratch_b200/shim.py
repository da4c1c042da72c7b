"""Drop-in binding of the B200 kernels into the reference engine's modules.

The reference imports its kernel entry points by name
(qwen3/attention.py:26-28, qwen3/PagedKVcache.py:16) and selects them with
environment switches read on every call:

* decode:  ``QWEN3_PAGED_ATTN == "triton"`` (default; qwen3/attention.py:101-104,
  144-147; qwen3/model.py:87-90) calls ``triton_paged_attention_decode[_batch]``;
* prefill: ``QWEN3_FLASH_ATTN != "pytorch"`` (qwen3/attention.py:113-116,
  162-165; qwen3/model.py:143-146) calls ``flash_attention_prefill_batched``;
* the decode write goes through ``update_kv_batch_triton`` imported into
  qwen3/PagedKVcache.py;
* the prefill write is the method ``PagedKVCache.update``
  (qwen3/PagedKVcache.py:177-214, called per request at qwen3/attention.py:112
  and :161); it is rebound on the class to ``ops.paged_cache_update`` (same
  page allocation, then one scatter launch from the handle's ``seq_len``).
  Inputs outside the kernel's contract (CPU tensors, dtypes other than bf16)
  keep the reference's own method.

``install()`` rebinds those module-level names to the B200 implementations, so
the reference's own switches route to them and the reference's ``GraphRunner``
(or this package's, bound in its place) captures them unchanged.  Setting ``QWEN3_FLASH_ATTN=b200`` before importing this module
installs it automatically.  ``QWEN3_PAGED_ATTN`` must stay ``triton`` (its
default): the reference compares it with ``==`` and any other value silently
routes decode to its PyTorch fallback.  ``uninstall()`` restores the originals.
"""

from __future__ import annotations

import importlib
import os

import torch

from . import graph_runner, ops

_UPDATE_KEY = ("qwen3.PagedKVcache", "PagedKVCache.update")


def _paged_cache_update(self, layer_idx, k_new, v_new):
    """Bound in place of the reference's ``PagedKVCache.update``."""
    if (k_new.is_cuda and v_new.is_cuda and k_new.dtype == torch.bfloat16
            and v_new.dtype == torch.bfloat16):
        return ops.paged_cache_update(self, layer_idx, k_new, v_new)
    return _saved[_UPDATE_KEY](self, layer_idx, k_new, v_new)


# (module, attribute or Class.attribute) -> replacement
_BINDINGS = {
    ("qwen3.attention", "triton_paged_attention_decode"): ops.triton_paged_attention_decode,
    ("qwen3.attention", "triton_paged_attention_decode_batch"): ops.triton_paged_attention_decode_batch,
    ("qwen3.attention", "flash_attention_prefill_batched"): ops.flash_attention_prefill_batched,
    ("qwen3.PagedKVcache", "update_kv_batch_triton"): ops.update_kv_batch_triton,
    _UPDATE_KEY: _paged_cache_update,
    ("qwen3.kernels.paged_attention", "paged_attention_decode_triton"): ops.paged_attention_decode_triton,
    ("qwen3.kernels.paged_attention", "triton_paged_attention_decode"): ops.triton_paged_attention_decode,
    ("qwen3.kernels.paged_attention", "triton_paged_attention_decode_batch"): ops.triton_paged_attention_decode_batch,
    ("qwen3.kernels.paged_attention", "update_kv_batch_triton"): ops.update_kv_batch_triton,
    ("qwen3.kernels.flash_attention_varlen", "flash_attention_prefill"): ops.flash_attention_prefill,
    ("qwen3.kernels.flash_attention_varlen", "flash_attention_prefill_batched"): ops.flash_attention_prefill_batched,
    # fused sampler (qwen3/sampling.py:234-270); callers that did `from qwen3.sampling
    # import sample_tokens` before install() keep the reference's function
    ("qwen3.sampling", "sample_tokens"): ops.sample_tokens,
    ("qwen3", "sample_tokens"): ops.sample_tokens,
    # decode-step graph pool (qwen3/graph_runner.py:26-200), same constructor and replay;
    # as above, only callers that import the name after install() get it
    ("qwen3.graph_runner", "GraphRunner"): graph_runner.GraphRunner,
}

_saved: dict = {}


def _owner(mod_name: str, attr: str):
    """(object holding the attribute, attribute name) for ``attr`` or ``Class.attr``."""
    obj = importlib.import_module(mod_name)
    *path, name = attr.split(".")
    for p in path:
        obj = getattr(obj, p)
    return obj, name


def install() -> list[str]:
    """Rebind the reference's kernel names to the B200 ops; returns what was bound."""
    bound = []
    for (mod_name, attr), fn in _BINDINGS.items():
        owner, name = _owner(mod_name, attr)
        if (mod_name, attr) not in _saved:
            _saved[(mod_name, attr)] = getattr(owner, name)
        setattr(owner, name, fn)
        bound.append(f"{mod_name}.{attr}")
    if os.environ.get("QWEN3_PAGED_ATTN", "triton") != "triton":
        raise RuntimeError("QWEN3_PAGED_ATTN must be 'triton' (the reference's gate) for the "
                           "B200 decode kernel to be selected")
    return bound


def uninstall() -> None:
    for (mod_name, attr), fn in list(_saved.items()):
        owner, name = _owner(mod_name, attr)
        setattr(owner, name, fn)
    _saved.clear()


if os.environ.get("QWEN3_FLASH_ATTN") == "b200":
    try:
        install()
    except ModuleNotFoundError:
        pass  # the reference engine is not importable in this process

"""B200-native (sm_100a) paged-KV attention path for InferKernelLab.

Public API -- drop-in replacements for the reference's attention/append
operators plus host mirrors of its cache, scheduler and runtime:

* ``paged_decode_attention`` -- split-KV paged decode (MHA/GQA/MQA);
* ``append_kv`` -- reshape-and-cache through ``slot_mapping``, bit-exact;
* ``rope_append_kv`` -- rotary embedding of q/k fused with the K/V append;
* ``paged_decode_attention_append`` -- a decode step's append (+ rotary) fused
  into the attention launch;
* ``paged_prefill_attention`` / ``paged_prefill_attention_varlen`` -- ragged
  causal prefill over the paged cache;
* ``build_slot_mapping`` -- device-built slots + ``cu_seqlens`` for a batch;
* ``PagedKVCache``, ``BlockAllocator``, ``TokenBudgetScheduler``,
  ``InferenceRuntime`` -- the reference's host-side contract;
* ``PrefixCache`` -- prefix sharing: refcounted blocks indexed by prompt content.

Backend names for the reference runners: ``BACKEND_NAME`` (attention) and
``APPEND_BACKEND_NAME`` (append).  The kernels live in
``_lib/libb200_paged_attn.so`` (C ABI in ``include/b200_paged_attn.h``);
build it with ``python -m inferkernellab_b200.build``.
"""

from .cache import BlockAllocator, CacheLayout, PagedKVCache
from .ops import (
    add_rmsnorm,
    append_kv,
    b200_available,
    build_slot_mapping,
    check_device_errors,
    paged_decode_attention,
    paged_decode_attention_append,
    paged_prefill_attention,
    paged_prefill_attention_varlen,
    rope_append_kv,
    silu_mul,
)
from .prefix_cache import PrefixCache
from .runtime import InferenceRuntime, RuntimeStats
from .scheduler import InferenceRequest, ScheduleBatch, TokenBudgetScheduler

BACKEND_NAME = "b200_paged"
APPEND_BACKEND_NAME = "b200"

# Reference-style aliases (reference names: append_kv_triton, paged_decode_attention_triton).
paged_decode_attention_b200 = paged_decode_attention
append_kv_b200 = append_kv
paged_prefill_attention_b200 = paged_prefill_attention

__all__ = [
    "APPEND_BACKEND_NAME",
    "BACKEND_NAME",
    "BlockAllocator",
    "CacheLayout",
    "InferenceRequest",
    "InferenceRuntime",
    "PagedKVCache",
    "PrefixCache",
    "RuntimeStats",
    "ScheduleBatch",
    "TokenBudgetScheduler",
    "add_rmsnorm",
    "append_kv",
    "append_kv_b200",
    "b200_available",
    "build_slot_mapping",
    "check_device_errors",
    "paged_decode_attention",
    "paged_decode_attention_append",
    "paged_decode_attention_b200",
    "paged_prefill_attention",
    "paged_prefill_attention_b200",
    "paged_prefill_attention_varlen",
    "rope_append_kv",
    "silu_mul",
]

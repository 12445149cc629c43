"""B200-native (sm_100a) paged-attention decode path of llm-serving-runtime.

Public entry points
  paged_attention_decode(query, key_cache, value_cache, block_tables,
                         context_lens, scale, slot_mapping=None, key=None, value=None)
      the north-star call: fused KV append + paged decode attention
  kv_append(...)                      the KV-append kernel alone
  prefix_sharing.PrefixGroups         shared prompt prefixes -> cascade decode
                                      (paged_attention_decode(..., prefix_groups=))
  shared_blocks.BlockRefAllocator     refcounted KV blocks: prefix-cache snapshots and
                                      hits share blocks instead of copying them
  reference_api                       drop-in for runtime/phase2/paged_attention_triton.py
  kv_block_pool.write_tokens_batch_into
                                      the reference pool's write_tokens_batch on the append kernel
  integration.install()               patch the reference runtime in place (decode, append,
                                      and multi-token steps through its cache and HF hook)

The kernels live in lib/libpa_b200.so (C ABI: include/paged_attention_b200.h).
"""

from .paged_attention import (  # noqa: F401
    DeviceErrorFlags,
    decode_workspace,
    describe_device_errors,
    kv_append,
    paged_attention_decode,
    read_device_errors,
)
from .prefix_sharing import PrefixGroups, find_shared_prefixes  # noqa: F401

__version__ = "1.0.0"

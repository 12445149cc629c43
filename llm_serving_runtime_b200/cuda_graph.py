"""CUDA-graph capture of a decode step's attention work (append + decode per layer).

The reference's CudaGraphDecodeManager (runtime/phase2/cuda_graph_decode.py:38-245)
captures whole decode steps bucketed by (batch, pow2 max_blocks) and falls
back to eager when capture fails (the Triton path's host syncs invalidate it,
docs/adr/0012-cuda-graph-decode.md).  The sm_100a kernels here read lengths,
block tables and slots on the device and size their grids from host shapes
only, so one capture per bucket replays correctly for every later step: the
lengths grow, the tables change, the graph stays valid.

``DecodeStepGraph`` owns static input buffers (per-layer query / new K / new V,
shared block tables, context lengths and slot mapping) and per-layer outputs,
captures ``layers`` x (pa_kv_append + pa_decode) once, and replays it.
Callers either write the static buffers in place (what a model's projections
would do) or pass tensors to ``step`` to have them copied in.
"""

from __future__ import annotations

import torch

from .paged_attention import paged_attention_decode

__all__ = ["DecodeStepGraph", "bucket_max_blocks"]


def bucket_max_blocks(max_blocks: int) -> int:
    """Power-of-two bucket of a block-table width (cuda_graph_decode.py:54-58)."""
    q = 1
    while q < max_blocks:
        q *= 2
    return q


class DecodeStepGraph:
    def __init__(self, key_caches, value_caches, *, batch: int, max_blocks: int, num_q_heads: int,
                 q_len: int = 1, scale: float, warmup: int = 1, prefix_groups=None):
        if len(key_caches) != len(value_caches) or not key_caches:
            raise ValueError("one key and one value cache view per layer")
        kc0 = key_caches[0]
        self.device = kc0.device
        self.key_caches = list(key_caches)
        self.value_caches = list(value_caches)
        _, Hkv, _, D = kc0.shape
        dt = kc0.dtype
        L = len(key_caches)
        self.scale = float(scale)
        # shared-prefix groups (cascade); their tensors are read at replay, so
        # they may be rewritten in place between steps (same host bounds)
        self.prefix_groups = prefix_groups
        self.batch, self.max_blocks, self.q_len = batch, max_blocks, q_len
        dev = self.device
        self.query = [torch.zeros(batch, num_q_heads, q_len, D, dtype=dt, device=dev) for _ in range(L)]
        self.new_key = [torch.zeros(batch, Hkv, q_len, D, dtype=dt, device=dev) for _ in range(L)]
        self.new_value = [torch.zeros(batch, Hkv, q_len, D, dtype=dt, device=dev) for _ in range(L)]
        self.out = [torch.empty(batch, num_q_heads, q_len, D, dtype=dt, device=dev) for _ in range(L)]
        self.block_tables = torch.zeros(batch, max_blocks, dtype=torch.int32, device=dev)
        self.context_lens = torch.zeros(batch, dtype=torch.int32, device=dev)
        # padding slots (-1) until real ones are written: warm-up and capture append nothing
        self.slot_mapping = torch.full((batch * q_len,), -1, dtype=torch.int64, device=dev)
        self.graph = torch.cuda.CUDAGraph()
        for _ in range(warmup):  # sizes the workspace and the kernels' attributes eagerly
            self._body()
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(self.graph):
            self._body()

    def _body(self):
        for layer in range(len(self.key_caches)):
            paged_attention_decode(
                self.query[layer], self.key_caches[layer], self.value_caches[layer], self.block_tables,
                self.context_lens, self.scale, self.slot_mapping, self.new_key[layer], self.new_value[layer],
                out=self.out[layer], prefix_groups=self.prefix_groups,
            )

    def replay(self) -> list[torch.Tensor]:
        self.graph.replay()
        return self.out

    def step(self, *, block_tables, context_lens, slot_mapping, queries, new_keys, new_values) -> list[torch.Tensor]:
        """Copy one step's inputs into the static buffers and replay."""
        b, mb = block_tables.shape
        if b != self.batch or mb > self.max_blocks:
            raise ValueError("step does not fit this graph's (batch, max_blocks) bucket")
        self.block_tables.zero_()
        self.block_tables[:, :mb].copy_(block_tables)
        self.context_lens.copy_(context_lens)
        self.slot_mapping.copy_(slot_mapping)
        for layer in range(len(self.key_caches)):
            self.query[layer].copy_(queries[layer])
            self.new_key[layer].copy_(new_keys[layer])
            self.new_value[layer].copy_(new_values[layer])
        return self.replay()

"""One layer's decode step as a single CUDA-graph replay.

A serving loop runs, per layer and step, the append of the new tokens' K/V
followed by the decode over the updated cache.  :class:`DecodeStep` captures
those two calls (five kernels) once and replays them, so a step costs one
graph launch instead of the Python and launch overhead of each call.  The
cache, block table, lengths and RoPE tables are bound when the step is built
(their contents may change between replays, their storage may not); the
per-step inputs go through static buffers.

Validation inside the graph is deferred: a replay never reads the error word
on the host.  ``step(..., check=True)`` (or ``iris_kernel.check_errors()``
later) raises what the kernels recorded; a batch the append check rejects is
not written.
"""
from __future__ import annotations

import torch

from . import _runtime
from .fused_attention import fused_int4_paged_decode_attention
from .fused_kv import fused_rope_int4_paged_append


class DecodeStep:
    def __init__(self, k_data, v_data, k_scale, v_scale, block_table, seq_lens, cos_cache, sin_cache, *,
                 num_q_heads: int, new_tokens: int, rotary_dim: int, page_size: int = 16, group_size: int = 32,
                 softmax_scale: float | None = None):
        dev = k_data.device
        batch = block_table.shape[0]
        num_kv_heads, head_dim = k_data.shape[2], k_data.shape[3] * 2
        self.cache = (k_data, v_data, k_scale, v_scale)
        self.block_table, self.seq_lens = block_table, seq_lens
        self.cos, self.sin = cos_cache, sin_cache
        self.kw_append = dict(rotary_dim=rotary_dim, group_size=group_size, page_size=page_size)
        self.kw_decode = dict(page_size=page_size, group_size=group_size, softmax_scale=softmax_scale)
        self.query = torch.zeros((batch, num_q_heads, head_dim), dtype=torch.float16, device=dev)
        self.key = torch.zeros((new_tokens, num_kv_heads, head_dim), dtype=torch.float16, device=dev)
        self.value = torch.zeros_like(self.key)
        self.positions = torch.zeros(new_tokens, dtype=torch.int32, device=dev)
        self.slots = torch.full((new_tokens,), -1, dtype=torch.int32, device=dev)  # warm-up writes nothing
        self.output = torch.empty_like(self.query)
        self.graph = torch.cuda.CUDAGraph()
        mode = _runtime.validation_mode()
        _runtime.set_validation_mode("deferred")
        try:
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                self._calls()  # first calls outside the capture (launch shapes, scratch buffers)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(self.graph, stream=side):
                self._calls()
            torch.cuda.synchronize(dev)
        finally:
            _runtime.set_validation_mode(mode)

    def _calls(self):
        fused_rope_int4_paged_append(self.key, self.value, self.positions, self.slots, self.cos, self.sin,
                                     *self.cache, **self.kw_append)
        fused_int4_paged_decode_attention(self.query, *self.cache, self.block_table, self.seq_lens, self.output,
                                          **self.kw_decode)

    def __call__(self, query, key, value, positions, slots, *, check: bool = False) -> torch.Tensor:
        """Append ``key/value [T, Hkv, D]`` at ``positions``/``slots [T]`` and
        decode ``query [B, Hq, D]``; returns the step's output (a static
        buffer, overwritten by the next replay)."""
        self.query.copy_(query, non_blocking=True)
        self.key.copy_(key, non_blocking=True)
        self.value.copy_(value, non_blocking=True)
        self.positions.copy_(positions, non_blocking=True)
        self.slots.copy_(slots, non_blocking=True)
        self.graph.replay()
        if check:
            _runtime.check_errors(self.query.device)
        return self.output

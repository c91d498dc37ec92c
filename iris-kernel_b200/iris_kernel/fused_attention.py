"""Read path: INT4 paged decode attention.

Drop-in for ``iris_kernel.fused_attention.fused_int4_paged_decode_attention``
of Hunter2030ZeRo/Iris-Kernel (src/iris_kernel/fused_attention.py:437-525):
same signature, layouts, output allocation and exception types.  The work
runs in the sm_100a kernels behind ``iris_b200_int4_paged_decode``
(csrc/decode.cu): split-KV over all SMs plus an in-call combine.

``decode_partial`` is the log-sum-exp form used by split-context multi-GPU
decode (``iris_kernel.parallel``); it has no counterpart in the reference.
"""
from __future__ import annotations

import torch

from . import _lib, _runtime


def _validate_common_decode_inputs(query, block_table, seq_lens, *, num_pages, num_kv_heads, page_size):
    """Host-side checks of fused_attention.py:373-434 minus the data-dependent
    ones (positive lengths, table length, page ids), which the kernels check
    on the device (see ``_runtime``)."""
    if not _runtime.cuda_available():
        raise RuntimeError("Iris fused kernels require CUDA")
    if query.device.type != "cuda":
        raise ValueError("query must be a CUDA tensor")
    if query.ndim != 3:
        raise ValueError("query must have shape [B, Hq, D]")
    if query.dtype != torch.float16:
        raise TypeError("query must use FP16(torch.float16)")
    if page_size != 16:
        raise NotImplementedError("decode fast path currently supports page_size=16")
    batch, num_query_heads, head_dim = query.shape
    if head_dim not in (64, 128):
        raise NotImplementedError("decode fast path currently supports head_dim in {64, 128}")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if num_query_heads // num_kv_heads > 16:
        raise NotImplementedError("decode fast path supports at most 16 query heads per KV head")
    if block_table.ndim != 2 or block_table.shape[0] != batch:
        raise ValueError("block_table must have shape [B, max_pages_per_sequence]")
    if seq_lens.shape != (batch,):
        raise ValueError("seq_lens must have shape [B]")
    if block_table.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise TypeError("block_table and seq_lens must use torch.int32")
    device = query.device
    if block_table.device != device or seq_lens.device != device:
        raise ValueError("block_table and seq_lens must be on the query device")
    _runtime.require_sm100(device)
    return batch, num_query_heads, head_dim


def _check_cache(query, k_data, v_data, k_scale, v_scale, page_size, group_size):
    if group_size != 32:
        raise NotImplementedError("decode fast path currently supports group_size=32")
    if k_data.ndim != 4 or tuple(v_data.shape) != tuple(k_data.shape):
        raise ValueError("k_data/v_data must have identical rank-4 shapes")
    num_pages, cache_page_size, num_kv_heads, packed_dim = k_data.shape
    head_dim = query.shape[-1]
    if cache_page_size != page_size or packed_dim * 2 != head_dim:
        raise ValueError("packed cache shape does not match query/page_size")
    return num_pages, num_kv_heads, head_dim


def _check_scales(query, k_data, v_data, k_scale, v_scale, num_pages, num_kv_heads, head_dim, page_size, group_size):
    expected = (num_pages, page_size, num_kv_heads, head_dim // group_size)
    if tuple(k_scale.shape) != expected:
        raise ValueError(f"k_scale must have shape {expected}")
    if tuple(v_scale.shape) != expected:
        raise ValueError(f"v_scale must have shape {expected}")
    if k_data.dtype != torch.uint8 or v_data.dtype != torch.uint8:
        raise TypeError("k_data/v_data must use UINT8(torch.uint8)")
    if k_scale.dtype != torch.float16 or v_scale.dtype != torch.float16:
        raise TypeError("k_scale/v_scale must use FP16(torch.float16)")
    for name, t in (("k_data", k_data), ("v_data", v_data), ("k_scale", k_scale), ("v_scale", v_scale)):
        if t.device != query.device:
            raise ValueError(f"{name} must be on {query.device}")
    if num_pages == 0:
        raise IndexError("block_table contains an invalid physical page id")
    for name, t in (("query", query), ("k_data", k_data), ("v_data", v_data), ("k_scale", k_scale),
                    ("v_scale", v_scale)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")


_OUT_SLOT = 8  # position of the output pointer in the decode entry point's arguments
_FP16_OUT_SLOT = 6  # the same in the FP16 decode entry point's arguments


def _launch(query, k_data, v_data, k_scale, v_scale, block_table, seq_lens, out, out_lse, mode, softmax_scale,
            page_size, fast_key=None):
    device = query.device
    batch, hq, head_dim = query.shape
    num_pages, _, hkv, _ = k_data.shape
    if block_table.stride(1) != 1 and block_table.shape[1] > 1:
        raise ValueError("block_table rows must be contiguous")
    scale = head_dim ** -0.5 if softmax_scale is None or softmax_scale == 0.0 else float(softmax_scale)
    with torch.cuda.device(device):
        stream = _runtime.stream_ptr(device)
        word = _runtime.error_word(device)
        if not seq_lens.is_contiguous():
            seq_lens = seq_lens.contiguous()
            fast_key = None  # a fresh copy per call: nothing to reuse
        ws_bytes = _runtime.workspace_bytes(_lib.lib.iris_b200_decode_workspace_bytes, batch, hq, hkv, head_dim,
                                            device.index or 0)
        ws = _runtime.scratch(device, stream, "decode", ws_bytes)
        args = [query.data_ptr(), k_data.data_ptr(), v_data.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(),
                block_table.data_ptr(), block_table.stride(0), seq_lens.data_ptr(), out.data_ptr(),
                out_lse.data_ptr() if out_lse is not None else None, mode, batch, hq, hkv, head_dim, num_pages,
                page_size, block_table.shape[1], scale, ws.data_ptr(), ws.numel(), word.data_ptr(), stream]
        fn = _lib.lib.iris_b200_int4_paged_decode
        _lib.check_status(fn(*args), "iris_b200_int4_paged_decode")
        if fast_key is not None:
            _runtime.fast_store(fast_key, _runtime.FastEntry([(fn, args, _OUT_SLOT, "iris_b200_int4_paged_decode")],
                                                             device.index, stream, (ws, word)))
        if _runtime.validation_mode() == "sync":
            _runtime.raise_for_bits(_runtime.read_and_clear(word))


def fused_int4_paged_decode_attention(
    query: torch.Tensor,
    k_data: torch.Tensor,
    v_data: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    output: torch.Tensor | None = None,
    *,
    page_size: int = 16,
    group_size: int = 32,
    softmax_scale: float | None = None,
) -> torch.Tensor:
    """
    Fused decode attention over Iris INT4 paged K/V.

    Direct path: packed load -> signed nibble unpack -> group dequantization
    -> QK -> online softmax -> PV, FP32 accumulation, fp16 output.  No FP16
    K/V is materialised in global memory.  ``softmax_scale`` None (or 0.0, as
    in the reference kernel) means head_dim ** -0.5.
    """
    sig = _runtime.tensor_sig
    key = ("int4_decode", sig(query), sig(k_data), sig(v_data), sig(k_scale), sig(v_scale), sig(block_table),
           sig(seq_lens), None if output is None else sig(output), page_size, group_size, softmax_scale)
    ent = _runtime.fast_lookup(key)
    if ent is not None:  # the same signature passed every host check before
        if output is None:
            output = torch.empty_like(query)
        _runtime.fast_run(ent, output.data_ptr())
        return output
    num_pages, num_kv_heads, head_dim = _check_cache(query, k_data, v_data, k_scale, v_scale, page_size, group_size)
    _validate_common_decode_inputs(query, block_table, seq_lens, num_pages=num_pages, num_kv_heads=num_kv_heads,
                                   page_size=page_size)
    _check_scales(query, k_data, v_data, k_scale, v_scale, num_pages, num_kv_heads, head_dim, page_size, group_size)
    if output is None:
        output = torch.empty_like(query)
    elif output.shape != query.shape or output.dtype != query.dtype:
        raise ValueError("output must match query shape and dtype")
    elif output.device != query.device:
        raise ValueError("output must be on the same device as query")
    if not output.is_contiguous():
        raise ValueError("output must be contiguous")
    if query.shape[0] == 0:
        return output
    _launch(query, k_data, v_data, k_scale, v_scale, block_table, seq_lens, output, None, _lib.DECODE_OUT_FP16,
            softmax_scale, page_size, fast_key=key)
    return output


def decode_partial(query, k_data, v_data, k_scale, v_scale, block_table, seq_lens, *, page_size: int = 16,
                   group_size: int = 32, softmax_scale: float | None = None, out: torch.Tensor | None = None,
                   lse: torch.Tensor | None = None):
    """Decode attention in log-sum-exp form: returns ``(o, lse)`` with
    ``o [B, Hq, D]`` fp32 normalised over the given tokens and ``lse [B, Hq]``
    fp32 = log2(sum_l 2^(x_l)), x_l = softmax_scale * log2(e) * q.k_l.
    ``block_table`` may be a column slice (row stride > width) so that a
    caller can attend over a page-aligned sub-range of each sequence.
    ``out`` / ``lse`` (contiguous fp32 views, e.g. into an all-gather send
    buffer) receive the result in place when given."""
    num_pages, num_kv_heads, head_dim = _check_cache(query, k_data, v_data, k_scale, v_scale, page_size, group_size)
    _validate_common_decode_inputs(query, block_table, seq_lens, num_pages=num_pages, num_kv_heads=num_kv_heads,
                                   page_size=page_size)
    _check_scales(query, k_data, v_data, k_scale, v_scale, num_pages, num_kv_heads, head_dim, page_size, group_size)
    if out is None:
        out = torch.empty(query.shape, dtype=torch.float32, device=query.device)
    if lse is None:
        lse = torch.empty(query.shape[:2], dtype=torch.float32, device=query.device)
    for t, shape in ((out, query.shape), (lse, query.shape[:2])):
        if t.shape != shape or t.dtype != torch.float32 or not t.is_contiguous() or t.device != query.device:
            raise ValueError(f"partial outputs must be contiguous float32 {tuple(shape)} on the query's device")
    if query.shape[0]:
        _launch(query, k_data, v_data, k_scale, v_scale, block_table, seq_lens, out, lse, _lib.DECODE_OUT_LSE,
                softmax_scale, page_size)
    return out, lse


def merge_lse_partials(parts_o: torch.Tensor, parts_lse: torch.Tensor, output: torch.Tensor | None = None):
    """Merge ``parts_o [P, B, Hq, D]`` / ``parts_lse [P, B, Hq]`` (as returned
    by :func:`decode_partial` for disjoint token ranges) into fp16 output."""
    if parts_o.dtype != torch.float32 or parts_lse.dtype != torch.float32:
        raise TypeError("partials must be float32")
    if parts_o.ndim != 4 or parts_lse.shape != parts_o.shape[:3]:
        raise ValueError("parts_o must be [P, B, Hq, D] and parts_lse [P, B, Hq]")
    P, B, Hq, D = parts_o.shape
    if output is None:
        output = torch.empty((B, Hq, D), dtype=torch.float16, device=parts_o.device)
    parts_o = parts_o.contiguous()
    parts_lse = parts_lse.contiguous()
    with torch.cuda.device(parts_o.device):
        _lib.check_status(
            _lib.lib.iris_b200_merge_lse_partials(parts_o.data_ptr(), parts_lse.data_ptr(), P, B * Hq, D,
                                                  output.data_ptr(), _runtime.stream_ptr(parts_o.device)),
            "iris_b200_merge_lse_partials")
    return output


def merge_lse_packed(parts: torch.Tensor, num_parts: int, batch: int, num_q_heads: int, head_dim: int,
                     output: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partials packed as one all-gather produces them: ``parts`` is a
    flat fp32 buffer of ``num_parts`` blocks of ``batch*Hq*(D+1)`` floats,
    each ``O [batch, Hq, D]`` then ``lse [batch, Hq]``.  Rows whose lse is
    -inf in a block are ignored for that block."""
    rows = batch * num_q_heads
    if parts.dtype != torch.float32 or not parts.is_contiguous():
        raise TypeError("parts must be a contiguous float32 buffer")
    if parts.numel() != num_parts * rows * (head_dim + 1):
        raise ValueError("parts must hold num_parts * batch * Hq * (D + 1) floats")
    if output is None:
        output = torch.empty((batch, num_q_heads, head_dim), dtype=torch.float16, device=parts.device)
    with torch.cuda.device(parts.device):
        _lib.check_status(
            _lib.lib.iris_b200_merge_lse_packed(parts.data_ptr(), num_parts, rows, head_dim, output.data_ptr(),
                                                _runtime.stream_ptr(parts.device)),
            "iris_b200_merge_lse_packed")
    return output


def fused_fp16_paged_decode_attention(
    query: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    output: torch.Tensor | None = None,
    *,
    page_size: int = 16,
    softmax_scale: float | None = None,
) -> torch.Tensor:
    """Matched FP16 paged decode-attention baseline (reference
    fused_attention.py:528-582: same signature, checks and exception types)
    over ``k_cache / v_cache [pages, 16, Hkv, D]`` fp16, with the INT4
    decode's schedule; semantics of torch_eager_fp16_paged_decode_attention."""
    sig = _runtime.tensor_sig
    key = ("fp16_decode", sig(query), sig(k_cache), sig(v_cache), sig(block_table), sig(seq_lens),
           None if output is None else sig(output), page_size, softmax_scale)
    ent = _runtime.fast_lookup(key)
    if ent is not None:  # the same signature passed every host check before
        if output is None:
            output = torch.empty_like(query)
        _runtime.fast_run(ent, output.data_ptr())
        return output
    if k_cache.ndim != 4 or tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError("k_cache/v_cache must have identical rank-4 shapes")
    num_pages, cache_page_size, num_kv_heads, cache_dim = k_cache.shape
    _, _, head_dim = query.shape
    if cache_page_size != page_size or cache_dim != head_dim:
        raise ValueError("FP16 cache shape does not match query/page_size")
    _validate_common_decode_inputs(query, block_table, seq_lens, num_pages=num_pages, num_kv_heads=num_kv_heads,
                                   page_size=page_size)
    if k_cache.dtype != torch.float16 or v_cache.dtype != torch.float16:
        raise TypeError("k_cache/v_cache must use FP16")
    if k_cache.device != query.device or v_cache.device != query.device:
        raise ValueError("k_cache/v_cache must be on the query device")
    if output is None:
        output = torch.empty_like(query)
    elif output.shape != query.shape or output.dtype != query.dtype:
        raise ValueError("output must match query shape and dtype")
    elif output.device != query.device:
        raise ValueError("output must be on the same device as query")
    for name, t in (("query", query), ("k_cache", k_cache), ("v_cache", v_cache), ("output", output)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    if num_pages == 0:
        raise IndexError("block_table contains an invalid physical page id")
    if query.shape[0] == 0:
        return output
    if block_table.stride(1) != 1 and block_table.shape[1] > 1:
        raise ValueError("block_table rows must be contiguous")
    device = query.device
    batch, hq, _ = query.shape
    scale = head_dim ** -0.5 if softmax_scale is None or softmax_scale == 0.0 else float(softmax_scale)
    with torch.cuda.device(device):
        stream = _runtime.stream_ptr(device)
        word = _runtime.error_word(device)
        if not seq_lens.is_contiguous():
            seq_lens = seq_lens.contiguous()
            key = None  # a fresh copy per call: nothing to reuse
        ws_bytes = _runtime.workspace_bytes(_lib.lib.iris_b200_fp16_decode_workspace_bytes, batch, hq,
                                            num_kv_heads, head_dim, device.index or 0)
        ws = _runtime.scratch(device, stream, "decode_fp16", ws_bytes)
        args = [query.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr(),
                block_table.stride(0), seq_lens.data_ptr(), output.data_ptr(), None, _lib.DECODE_OUT_FP16, batch, hq,
                num_kv_heads, head_dim, num_pages, page_size, block_table.shape[1], scale, ws.data_ptr(), ws.numel(),
                word.data_ptr(), stream]
        fn = _lib.lib.iris_b200_fp16_paged_decode
        _lib.check_status(fn(*args), "iris_b200_fp16_paged_decode")
        if key is not None:
            _runtime.fast_store(key, _runtime.FastEntry([(fn, args, _FP16_OUT_SLOT, "iris_b200_fp16_paged_decode")],
                                                        device.index, stream, (ws, word)))
        if _runtime.validation_mode() == "sync":
            _runtime.raise_for_bits(_runtime.read_and_clear(word))
    return output

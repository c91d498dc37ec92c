"""Write path: fused RoPE(K) + INT4 quantise + pack + paged append.

Drop-in for ``iris_kernel.fused_kv.fused_rope_int4_paged_append`` of
Hunter2030ZeRo/Iris-Kernel (src/iris_kernel/fused_kv.py:600-780): same
signature, tensor layouts and exception types.  The work runs in the sm_100a
kernel ``iris_b200_rope_int4_paged_append`` (csrc/append.cu) and is
bit-exact with the reference's eager path (torch_eager_kv.py:110-337).
"""
from __future__ import annotations

import torch

from . import _lib, _runtime


def _check_append_args(key, value, positions, slot_mapping, cos_cache, sin_cache, k_data, v_data, k_scale, v_scale,
                       *, rotary_dim, group_size, page_size):
    """Host-side argument checks, in the order of fused_kv.py:616-739."""
    if key.device.type != "cuda":
        raise ValueError("key/value must be CUDA tensors")
    if key.shape != value.shape:
        raise ValueError("key and value must have identical shapes")
    if key.ndim != 3:
        raise ValueError("key/value must have shape [T, Hkv, D]")
    if key.dtype != torch.float16:
        raise TypeError("key must use FP16(torch.float16)")
    if value.dtype != torch.float16:
        raise TypeError("value must use FP16(torch.float16)")
    num_tokens, num_kv_heads, head_dim = key.shape
    if head_dim % 64 != 0:
        raise NotImplementedError("fused append requires head_dim divisible by 64")
    if head_dim > 512:
        raise NotImplementedError("fused append supports head_dim <= 512")
    if group_size != 32:
        raise NotImplementedError("fused append supports group_size=32")
    if rotary_dim != head_dim:
        raise NotImplementedError("fused append requires rotary_dim == head_dim")
    if rotary_dim % 2 != 0:
        raise ValueError("rotary_dim must be even")
    if page_size <= 0:
        raise ValueError("page_size must be positive")
    if positions.shape != (num_tokens,):
        raise ValueError("positions must have shape [T]")
    if slot_mapping.shape != (num_tokens,):
        raise ValueError("slot_mapping must have shape [T]")
    device = key.device
    for name, t in (("value", value), ("positions", positions), ("slot_mapping", slot_mapping),
                    ("cos_cache", cos_cache), ("sin_cache", sin_cache), ("k_data", k_data), ("v_data", v_data),
                    ("k_scale", k_scale), ("v_scale", v_scale)):
        if t.device != device:
            raise ValueError(f"{name} must be on {device}")
    if positions.dtype != torch.int32:
        raise TypeError("positions must use torch.int32")
    if slot_mapping.dtype != torch.int32:
        raise TypeError("slot_mapping must use torch.int32")
    half = rotary_dim // 2
    if cos_cache.ndim != 2:
        raise ValueError("cos_cache must have shape [max_position, rotary_dim // 2]")
    if sin_cache.shape != cos_cache.shape:
        raise ValueError("sin_cache must match cos_cache")
    if cos_cache.shape[-1] != half:
        raise ValueError(f"RoPE cache width must be {half}")
    if cos_cache.dtype != torch.float16:
        raise TypeError("cos_cache must use FP16(torch.float16)")
    if sin_cache.dtype != torch.float16:
        raise TypeError("sin_cache must use FP16(torch.float16)")
    if k_data.ndim != 4:
        raise ValueError("k_data/v_data must be rank-4 tensors")
    num_pages = k_data.shape[0]
    data_shape = (num_pages, page_size, num_kv_heads, head_dim // 2)
    scale_shape = (num_pages, page_size, num_kv_heads, head_dim // group_size)
    if tuple(k_data.shape) != data_shape:
        raise ValueError(f"k_data must have shape {data_shape}")
    if tuple(v_data.shape) != data_shape:
        raise ValueError(f"v_data must have shape {data_shape}")
    if tuple(k_scale.shape) != scale_shape:
        raise ValueError(f"k_scale must have shape {scale_shape}")
    if tuple(v_scale.shape) != scale_shape:
        raise ValueError(f"v_scale must have shape {scale_shape}")
    if k_data.dtype != torch.uint8:
        raise TypeError("k_data must use UINT8(torch.uint8)")
    if v_data.dtype != torch.uint8:
        raise TypeError("v_data must use UINT8(torch.uint8)")
    if k_scale.dtype != torch.float16:
        raise TypeError("k_scale must use FP16(torch.float16)")
    if v_scale.dtype != torch.float16:
        raise TypeError("v_scale must use FP16(torch.float16)")
    for name, t in (("key", key), ("value", value), ("positions", positions), ("slot_mapping", slot_mapping),
                    ("cos_cache", cos_cache), ("sin_cache", sin_cache), ("k_data", k_data), ("v_data", v_data),
                    ("k_scale", k_scale), ("v_scale", v_scale)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    return num_tokens, num_kv_heads, head_dim, num_pages


def fused_rope_int4_paged_append(
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    slot_mapping: torch.Tensor,
    cos_cache: torch.Tensor,
    sin_cache: torch.Tensor,
    k_data: torch.Tensor,
    v_data: torch.Tensor,
    k_scale: torch.Tensor,
    v_scale: torch.Tensor,
    *,
    rotary_dim: int,
    group_size: int = 32,
    page_size: int,
) -> None:
    """RoPE(K), group-32 INT4 quantisation of K and V, low-nibble-first
    packing and paged append, in place.  Tokens with ``slot_mapping < 0`` are
    skipped; untouched slots stay byte-identical."""
    sig = _runtime.tensor_sig
    sig_key = ("int4_append", sig(key), sig(value), sig(positions), sig(slot_mapping), sig(cos_cache), sig(sin_cache),
           sig(k_data), sig(v_data), sig(k_scale), sig(v_scale), rotary_dim, group_size, page_size)
    ent = _runtime.fast_lookup(sig_key)
    if ent is not None:  # the same signature passed every host check before
        _runtime.fast_run(ent)
        return
    if not _runtime.cuda_available():
        raise RuntimeError("Iris fused kernels require CUDA")
    num_tokens, num_kv_heads, head_dim, num_pages = _check_append_args(
        key, value, positions, slot_mapping, cos_cache, sin_cache, k_data, v_data, k_scale, v_scale,
        rotary_dim=rotary_dim, group_size=group_size, page_size=page_size)
    device = key.device
    _runtime.require_sm100(device)
    if num_tokens == 0:
        return
    with torch.cuda.device(device):
        stream = _runtime.stream_ptr(device)
        word = _runtime.error_word(device)
        calls, keep = [], [word]
        if num_tokens > _lib.APPEND_INLINE_CHECK_TOKENS:  # smaller batches are checked by the append itself
            ws_bytes = _lib.lib.iris_b200_append_check_workspace_bytes(num_pages, page_size)
            ws = _runtime.scratch(device, stream, "append_check", max(ws_bytes, 4))
            keep.append(ws)
            calls.append((_lib.lib.iris_b200_append_check,
                          [positions.data_ptr(), slot_mapping.data_ptr(), num_tokens, cos_cache.shape[0], num_pages,
                           page_size, ws.data_ptr(), ws.numel(), word.data_ptr(), stream], -1,
                          "iris_b200_append_check"))
        # the append kernel writes nothing if the check recorded an error, so
        # one host read after the launches keeps "raise before writing"
        calls.append((_lib.lib.iris_b200_rope_int4_paged_append,
                      [key.data_ptr(), value.data_ptr(), positions.data_ptr(), slot_mapping.data_ptr(),
                       cos_cache.data_ptr(), sin_cache.data_ptr(), k_data.data_ptr(), v_data.data_ptr(),
                       k_scale.data_ptr(), v_scale.data_ptr(), num_tokens, num_kv_heads, head_dim,
                       cos_cache.shape[0], num_pages, page_size, word.data_ptr(), stream], -1,
                      "iris_b200_rope_int4_paged_append"))
        for fn, args, _, what in calls:
            _lib.check_status(fn(*args), what)
        _runtime.fast_store(sig_key, _runtime.FastEntry(calls, device.index, stream, keep))
        if _runtime.validation_mode() == "sync":
            _runtime.raise_for_bits(_runtime.read_and_clear(word))


def fused_quantize_pack_int4(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> None:
    """Group-32 INT4 quantisation + low-nibble-first packing of ``x [T, H, D]``
    fp16 into ``packed [T, H, D/2]`` uint8 and ``scales [T, H, D/32]`` fp16,
    in place.  Drop-in for fused_kv.py:362-416 of the reference (same checks,
    messages and exception types); bit-exact with its eager
    ``quantize_int4_groupwise`` + ``pack_int4``.  Tensors must be contiguous."""
    if not _runtime.cuda_available():
        raise RuntimeError("Iris fused kernels require CUDA")
    if x.device.type != "cuda":
        raise ValueError("x must be a CUDA tensor")
    if x.ndim != 3:
        raise ValueError("x must have shape [T, H_kv, D]")
    if x.dtype != torch.float16:
        raise TypeError("INT4 fast path currently requires FP16 input")
    _, _, head_dim = x.shape
    if head_dim % 64 != 0:
        raise NotImplementedError("INT4 fast path currently requires head_dim divisible by 64")
    expected_packed = (x.shape[0], x.shape[1], head_dim // 2)
    expected_scales = (x.shape[0], x.shape[1], head_dim // 32)
    if tuple(packed.shape) != expected_packed:
        raise ValueError(f"packed tensor must have shape {expected_packed}")
    if tuple(scales.shape) != expected_scales:
        raise ValueError(f"scales must have shape {expected_scales}")
    if packed.dtype != torch.uint8:
        raise TypeError("packed tensor must use UINT8(torch.uint8)")
    if scales.dtype != torch.float16:
        raise TypeError("scales must use FP16(torch.float16)")
    if packed.device != x.device:
        raise ValueError("packed tensor must be on the same device as x")
    if scales.device != x.device:
        raise ValueError("scales must be on the same device as x")
    for name, t in (("x", x), ("packed", packed), ("scales", scales)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    _runtime.require_sm100(x.device)
    rows = x.shape[0] * x.shape[1]
    if rows == 0:
        return
    with torch.cuda.device(x.device):
        _lib.check_status(
            _lib.lib.iris_b200_int4_quantize_pack(x.data_ptr(), packed.data_ptr(), scales.data_ptr(), rows, head_dim,
                                                  _runtime.stream_ptr(x.device)),
            "iris_b200_int4_quantize_pack")


def fused_rope_fp16_append(
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    slot_mapping: torch.Tensor,
    cos_cache: torch.Tensor,
    sin_cache: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    rotary_dim: int,
    page_size: int,
) -> None:
    """FP16 paged append (reference fused_kv.py:153-297: same signature, checks
    and exception types): RoPE(K) over ``rotary_dim`` dims with fp16 rounding
    after every operation, K tail and V copied, into ``k_cache / v_cache
    [pages, page_size, Hkv, D]`` fp16.  Validation runs on the device (no
    host round trip before the write); a rejected batch writes nothing."""
    if not _runtime.cuda_available():
        raise RuntimeError("Iris fused kernels require CUDA")
    if key.device.type != "cuda":
        raise ValueError("key/value must be CUDA tensors")
    if key.shape != value.shape:
        raise ValueError("key and value must have identical shapes")
    if key.ndim != 3:
        raise ValueError("key/value must have shape [T, Hkv, D]")
    if key.dtype != torch.float16:
        raise TypeError("Stage A currently supports FP16 input")
    if value.dtype != torch.float16:
        raise TypeError("Stage A currently supports FP16 input")
    num_tokens, num_kv_heads, head_dim = key.shape
    if rotary_dim > head_dim:
        raise ValueError("rotary_dim cannot exceed head_dim")
    if rotary_dim % 2 != 0:
        raise ValueError("rotary_dim must be even")
    if page_size <= 0:
        raise ValueError("page_size must be positive")
    if positions.shape != (num_tokens,):
        raise ValueError("positions must have shape [T]")
    if slot_mapping.shape != (num_tokens,):
        raise ValueError("slot_mapping must have shape [T]")
    if tuple(k_cache.shape[1:]) != (page_size, num_kv_heads, head_dim):
        raise ValueError("invalid k_cache shape")
    if tuple(v_cache.shape) != tuple(k_cache.shape):
        raise ValueError("k_cache and v_cache must have identical shapes")
    if k_cache.dtype != torch.float16:
        raise TypeError("Stage A cache must use FP16")
    if v_cache.dtype != torch.float16:
        raise TypeError("Stage A cache must use FP16")
    device = key.device
    for name, t in (("value", value), ("positions", positions), ("slot_mapping", slot_mapping),
                    ("cos_cache", cos_cache), ("sin_cache", sin_cache), ("k_cache", k_cache), ("v_cache", v_cache)):
        if t.device != device:
            raise ValueError(f"{name} must be on {device}")
    if positions.dtype != torch.int32:
        raise TypeError("positions must use torch.int32")
    if slot_mapping.dtype != torch.int32:
        raise TypeError("slot_mapping must use torch.int32")
    half = rotary_dim // 2
    if cos_cache.ndim != 2:
        raise ValueError("cos_cache must have shape [max_position, rotary_dim // 2]")
    if sin_cache.shape != cos_cache.shape:
        raise ValueError("sin_cache must match cos_cache")
    if cos_cache.shape[-1] != half:
        raise ValueError(f"RoPE cache width must be {half}")
    if cos_cache.dtype != torch.float16:
        raise TypeError("Stage A RoPE cache must use FP16")
    if sin_cache.dtype != torch.float16:
        raise TypeError("Stage A RoPE cache must use FP16")
    for name, t in (("key", key), ("value", value), ("positions", positions), ("slot_mapping", slot_mapping),
                    ("cos_cache", cos_cache), ("sin_cache", sin_cache), ("k_cache", k_cache), ("v_cache", v_cache)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    _runtime.require_sm100(device)
    if num_tokens == 0:
        return
    num_pages = k_cache.shape[0]
    with torch.cuda.device(device):
        stream = _runtime.stream_ptr(device)
        word = _runtime.error_word(device)
        if num_tokens > _lib.APPEND_INLINE_CHECK_TOKENS:  # smaller batches are checked by the append itself
            ws_bytes = _lib.lib.iris_b200_append_check_workspace_bytes(num_pages, page_size)
            ws = _runtime.scratch(device, stream, "append_check", max(ws_bytes, 4))
            _lib.check_status(
                _lib.lib.iris_b200_append_check(positions.data_ptr(), slot_mapping.data_ptr(), num_tokens,
                                                cos_cache.shape[0], num_pages, page_size, ws.data_ptr(),
                                                ws.numel(), word.data_ptr(), stream),
                "iris_b200_append_check")
        _lib.check_status(
            _lib.lib.iris_b200_rope_fp16_paged_append(
                key.data_ptr(), value.data_ptr(), positions.data_ptr(), slot_mapping.data_ptr(),
                cos_cache.data_ptr(), sin_cache.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), num_tokens,
                num_kv_heads, head_dim, rotary_dim, cos_cache.shape[0], num_pages, page_size, word.data_ptr(),
                stream),
            "iris_b200_rope_fp16_paged_append")
        if _runtime.validation_mode() == "sync":
            _runtime.raise_for_bits(_runtime.read_and_clear(word))

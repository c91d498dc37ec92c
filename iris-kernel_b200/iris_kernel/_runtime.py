"""Per-device state shared by the wrappers: the device error word and the
validation mode.

The reference validates on the host with device->host synchronisations
(``torch.unique`` / ``any()`` in fused_kv.py:741-759, one ``.item()`` per
sequence in fused_attention.py:415-429).  Here the kernels check the data on
the device and OR ``IRIS_ERR_*`` bits into an int32 error word:

* ``"sync"`` (default): after launching, the wrapper reads the word once and
  raises the reference's exception type.  The append's check kernel runs
  before the append kernel, which writes nothing when the check recorded an
  error (the cache is untouched on error, as in the reference); the decode
  kernels skip bad pages while running and the wrapper raises afterwards.
* ``"deferred"``: no host synchronisation at all (CUDA-graph friendly); call
  :func:`check_errors` whenever convenient to raise for any recorded error.
  A rejected append batch writes nothing, and while a slot / position /
  duplicate error is pending on the device (until :func:`check_errors`
  clears it) every later append on that device is refused as well, so a bad
  batch never leads to a partly written cache.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib

_MODES = ("sync", "deferred")
_state = threading.local()
_words: dict[int, torch.Tensor] = {}
_words_lock = threading.Lock()


def set_validation_mode(mode: str) -> None:
    if mode not in _MODES:
        raise ValueError(f"validation mode must be one of {_MODES}")
    _state.mode = mode


_cuda_seen = False


def cuda_available() -> bool:
    """``torch.cuda.is_available()``, remembered once it is true (the torch
    call reads the environment and asks the driver on every call, ~5 us)."""
    global _cuda_seen
    if not _cuda_seen:
        _cuda_seen = torch.cuda.is_available()
    return _cuda_seen


def validation_mode() -> str:
    return getattr(_state, "mode", "sync")


def error_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _words_lock:
        w = _words.get(idx)
        if w is None:
            w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
            _words[idx] = w
    return w


# bit -> (exception type, message), in the order the reference checks
_APPEND_ERRORS = (
    (_lib.ERR_DUP_SLOT, ValueError, "duplicate physical KV-cache slots are not allowed"),
    (_lib.ERR_SLOT_RANGE, IndexError, "slot_mapping points outside allocated KV cache"),
    (_lib.ERR_POS_NEGATIVE, IndexError, "positions must be non-negative"),
    (_lib.ERR_POS_RANGE, IndexError, "positions point outside RoPE cache"),
)
_DECODE_ERRORS = (
    (_lib.ERR_SEQ_LEN, ValueError, "all sequence lengths must be positive"),
    (_lib.ERR_BLOCK_TABLE, ValueError, "block_table does not contain enough pages"),
    (_lib.ERR_PAGE_ID, IndexError, "block_table contains an invalid physical page id"),
)
_ALL_ERRORS = _APPEND_ERRORS + _DECODE_ERRORS + (
    (_lib.ERR_PIPELINE_TIMEOUT, RuntimeError, "a decode pipeline wait timed out"),)


def raise_for_bits(bits: int) -> None:
    for bit, exc, msg in _ALL_ERRORS:
        if bits & bit:
            raise exc(msg)
    if bits:
        raise RuntimeError(f"iris_kernel: unknown device error bits 0x{bits:x}")


def read_and_clear(word: torch.Tensor) -> int:
    bits = int(word.item())
    if bits:
        word.zero_()
    return bits


def check_errors(device: torch.device | int | None = None) -> None:
    """Raise (and clear) any error the kernels recorded on ``device``."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        device = torch.device("cuda", device)
    raise_for_bits(read_and_clear(error_word(device)))


_capability: dict = {}


def require_sm100(device: torch.device) -> None:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    cap = _capability.get(idx)
    if cap is None:
        cap = _capability[idx] = torch.cuda.get_device_capability(idx)
    if cap[0] != 10:
        raise RuntimeError(f"iris_kernel is built for sm_100a (B200); device capability is {cap}")


_scratch: dict = {}


def scratch(device: torch.device, stream: int, kind: str, nbytes: int) -> torch.Tensor:
    """A device byte buffer of at least ``nbytes`` for one launcher on one
    stream, kept between calls (the kernels rewrite what they read, so its
    contents do not matter); one per stream so that calls in flight at the
    same time never share it."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream, kind)
    with _words_lock:
        buf = _scratch.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=torch.device("cuda", idx))
            _scratch[key] = buf
    return buf


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """The current torch CUDA stream of ``device`` as a raw handle (through
    torch's raw-stream query when it has one: no Stream object per call)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


_ws_sizes: dict = {}


def workspace_bytes(fn, *shape) -> int:
    """Workspace size from a library query, remembered per (query, shape)."""
    key = (fn.__name__, shape)
    n = _ws_sizes.get(key)
    if n is None:
        n = fn(*shape)
        if len(_ws_sizes) < 4096:
            _ws_sizes[key] = n
    return n


# ---------------------------------------------------------------- fast path
# A wrapper call whose tensors (device address, shape, strides, dtype) and
# keyword arguments equal those of an earlier call that passed every host
# check needs no new checks: the host checks depend on nothing else (the
# data-dependent ones run on the device).  The prepared C-ABI arguments of
# such calls are kept per (signature, stream), so a repeated call (a decode
# loop over the same cache) is one dictionary lookup and one C call.  Device
# addresses identify the device too (unified virtual addressing).

_FAST_MAX = 512


def _prepared(fn, args):
    """``fn`` as a bare function pointer plus ``args`` converted once to its
    ctypes argument types: a repeat call then skips ctypes' per-argument
    conversion (about 1.5 us of the ~3 us a 23-argument call costs)."""
    bare = ctypes.CFUNCTYPE(fn.restype)(ctypes.cast(fn, ctypes.c_void_p).value)
    return bare, [t(a) for t, a in zip(fn.argtypes, args)]


class FastEntry:
    __slots__ = ("calls", "device", "stream", "keep")

    def __init__(self, calls, device, stream, keep):
        # [(bare C function, converted arguments, output slot or -1, what)]
        self.calls = [(*_prepared(fn, args), slot, what) for fn, args, slot, what in calls]
        self.device = device  # CUDA device index
        self.stream = stream  # raw stream the arguments were prepared for
        self.keep = keep      # tensors the arguments point into (kept alive)


_fast: dict = {}


def tensor_sig(t):
    return (t.data_ptr(), t.shape, t.stride(), t.dtype, t.is_cuda)


def fast_lookup(key):
    """The entry prepared for ``key`` on the current stream of its device,
    or None."""
    ent = _fast.get(key)
    if ent is None:
        return None
    if _raw_stream is not None:
        stream = _raw_stream(ent.device)
    else:
        stream = torch.cuda.current_stream(ent.device).cuda_stream
    return ent if stream == ent.stream else None


def fast_store(key, ent):
    if len(_fast) >= _FAST_MAX:
        _fast.clear()
    _fast[key] = ent


def fast_run(ent, out_ptr=None):
    """Launch a prepared entry (``out_ptr`` fills the output slot) and apply
    the validation mode, as the full wrapper would."""
    cur = torch.cuda.current_device()
    if cur != ent.device:
        torch.cuda.set_device(ent.device)
    try:
        for fn, args, slot, what in ent.calls:
            if slot >= 0:
                args = list(args)
                args[slot] = ctypes.c_void_p(out_ptr)
            _lib.check_status(fn(*args), what)
    finally:
        if cur != ent.device:
            torch.cuda.set_device(cur)
    if validation_mode() == "sync":
        raise_for_bits(read_and_clear(_words[ent.device]))


def fast_clear():
    _fast.clear()

"""B200 paged-attention backend: the reference's Triton entry points on sm_100a CUDA.

Free functions with the reference's call signatures
(mini_vllm/attention/paged_attention_gpu.py):

* ``paged_cache_write(key, value, key_cache, value_cache, slot_mapping, block_size)``
  replaces ``triton_cache_write`` (:90-154);
* ``paged_decode_attention(query, key_cache, value_cache, block_table,
  kv_len_after, block_size, scale=None)`` replaces ``triton_decode_attention``
  (:252-321), with the optional ``scale`` defaulting to ``head_dim ** -0.5``
  as at :304.

``triton_cache_write`` / ``triton_decode_attention`` are aliases of the two so
an import of the reference names keeps working; nothing here uses Triton.
Both call libmvb200.so through ctypes with raw pointers and strides and launch
on ``torch.cuda.current_stream()``.

Error behaviour follows the reference:

* argument checks the reference makes with ``assert`` raise ``AssertionError``
  (the exception also derives from ``ValueError``, the type the torch oracle
  ``write_to_paged_cache`` raises for the same checks, cache_write.py:82-140);
* ``kv_len_after < 1`` raises ``ValueError`` (:296-300);
* a duplicate write slot raises ``AssertionError`` mentioning "Duplicate"
  (:126-135);
* a slot outside ``[0, num_blocks * block_size)`` other than -1 raises
  ``IndexError`` (the oracle's rule, cache_write.py:61-66);
* a block table too short for ``kv_len`` raises ``IndexError`` (the gather's
  rule, cache_read.py:62-67).

The device-side conditions are detected by the kernels, which OR a bit into a
per-device error word.  With ``strict=True`` (the default) every call reads
that word back — one host sync, as the reference's own checks cost — and
raises; with ``strict=False`` the word accumulates until
``check_device_errors`` is called, so a timed loop has no host sync.
"""

from __future__ import annotations

import threading
from typing import Any, Dict, List, Optional, Tuple

import torch

from .. import _native
from ..cache.pool import KVCachePool
from .backend import AttentionBackend

_DTYPE_CODES = {
    torch.float32: _native.DTYPE_F32,
    torch.float16: _native.DTYPE_F16,
    torch.bfloat16: _native.DTYPE_BF16,
}
_VARIANTS = {"auto": _native.DECODE_AUTO, "fma": _native.DECODE_FMA, "mma": _native.DECODE_MMA,
             "stream": _native.DECODE_STREAM, "sched": _native.DECODE_SCHED}
_VARIANT_NAMES = {v: k for k, v in _VARIANTS.items()}


class ArgumentError(AssertionError, ValueError):
    """A rejected argument: an ``AssertionError`` like the Triton entry points
    raise, and a ``ValueError`` like the torch oracle raises."""


def _require(cond: bool, msg) -> None:
    """Raise ArgumentError unless `cond`; `msg` is a string or a zero-argument
    callable producing one (so the hot path formats nothing)."""
    if not cond:
        raise ArgumentError(msg() if callable(msg) else msg)


# ---------------------------------------------------------------------------
# per-device state: error word, duplicate-slot claim arrays, split-K workspace
# ---------------------------------------------------------------------------
class _DeviceState:
    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.err_ptr = self.err.data_ptr()
        self._claims: Dict[int, Tuple[torch.Tensor, int]] = {}
        self._workspaces: Dict[str, torch.Tensor] = {}
        self._counters: Dict[int, torch.Tensor] = {}

    def next_claims(self, total_slots: int) -> Tuple[torch.Tensor, int]:
        """Claim array for a pool of ``total_slots`` and a fresh epoch (never 0)."""
        entry = self._claims.get(total_slots)
        if entry is None:
            arr = torch.zeros(total_slots, dtype=torch.int32, device=self.device)
            epoch = 1
        else:
            arr, epoch = entry
            epoch += 1
            if epoch >= 0xFFFFFFFF:
                arr.zero_()
                epoch = 1
        self._claims[total_slots] = (arr, epoch)
        return arr, epoch

    def gather_counter(self, stream: int) -> int:
        """Device address of the gather's two work-counter words for one stream
        (zero when allocated; every gather leaves them zero)."""
        buf = self._counters.get(stream)
        if buf is None:
            buf = torch.zeros(2, dtype=torch.int32, device=self.device)
            self._counters[stream] = buf
        return buf.data_ptr()

    def workspace(self, nbytes: int, variant: str, stream: int = 0) -> torch.Tensor:
        """Decode workspace of one kernel variant (the stream, scheduled and
        split-K kernels each keep their own buffer), zero-filled when allocated.
        The stream and scheduled kernels' hold arrival counters (and the
        scheduled kernel's its schedule), so each stream gets its own."""
        key = (variant, stream) if variant in ("sched", "stream") else "split"
        buf = self._workspaces.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
            self._workspaces[key] = buf
        return buf


_states: Dict[int, _DeviceState] = {}
_states_lock = threading.Lock()


def _state(device) -> _DeviceState:
    """Per-device state; `device` is a torch.device or a CUDA device index."""
    if isinstance(device, int):
        idx = device
    else:
        idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _states.get(idx)
    if st is None:
        with _states_lock:
            st = _states.get(idx)
            if st is None:
                st = _DeviceState(torch.device("cuda", idx))
                _states[idx] = st
    return st


try:  # the raw handle without building a torch.cuda.Stream object per call
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream_handle(device) -> int:
    """Current stream of `device` (a torch.device or a CUDA device index)."""
    if isinstance(device, int):
        idx = device
    else:
        idx = device.index if device.index is not None else torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _host_status(status: int, what: str) -> None:
    if status == _native.OK:
        return
    msg = f"{what}: {_native.status_string(status)} (status {status})"
    if status in (_native.ERR_HEAD_DIM, _native.ERR_BLOCK_SIZE, _native.ERR_HEADS,
                  _native.ERR_INVALID_ARG, _native.ERR_DTYPE):
        raise ArgumentError(msg)
    raise RuntimeError(msg)


def _take_flags(state: _DeviceState) -> int:
    flags = int(state.err.item())
    if flags:
        state.err.zero_()
    return flags


def check_device_errors(device: Optional[torch.device] = None) -> None:
    """Raise for device-side errors accumulated by ``strict=False`` calls."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    flags = _take_flags(_state(dev))
    if flags:
        _raise_flags(flags, None)


def _raise_flags(flags: int, detail: Optional[Dict[str, Any]]) -> None:
    d = detail or {}
    if flags & _native.DEV_KV_LEN:
        kvl = d.get("kv_len_after")
        got = f", got min={int(kvl.min().item())}" if kvl is not None else ""
        raise ValueError(f"kv_len_after must be >= 1 for all decode sequences{got}")
    if flags & _native.DEV_SLOT_RANGE:
        slots = d.get("slot_mapping")
        total = d.get("total_slots")
        msg = "slot_mapping entry out of range"
        if slots is not None and total is not None:
            bad = ((slots < -1) | (slots >= total)).nonzero()
            if bad.numel():
                t = int(bad[0, 0].item())
                msg = (f"slot_mapping[{t}] = {int(slots[t].item())} out of range [0, {total}) "
                       f"(block_size={d.get('block_size')}, num_blocks={d.get('num_blocks')})")
        raise IndexError(msg)
    if flags & _native.DEV_TABLE_SHORT:
        raise IndexError(
            "block_table length insufficient to cover kv_len_after tokens "
            f"(max_blocks_per_seq={d.get('max_blocks')}, block_size={d.get('block_size')})"
        )
    if flags & _native.DEV_BLOCK_ID:
        raise IndexError(
            f"block_table entry out of range [0, {d.get('num_blocks')}) within a sequence's "
            "kv_len (a -1 pad or a stale id where a block is required)"
        )
    if flags & _native.DEV_DUP_SLOT:
        raise AssertionError(
            "Duplicate slots in slot_mapping: parallel writes to one slot race, "
            "so duplicate slots are forbidden."
        )
    if flags & _native.DEV_POSITION:
        rows = d.get("table_rows")
        raise IndexError(f"rope position out of range of the cos/sin table ({rows} rows)")
    if flags & _native.DEV_TIMEOUT:
        raise RuntimeError("paged decode: a bounded pipeline wait timed out on the device "
                           "(a decode schedule used by that call must be built again)")
    if flags & _native.DEV_SCHEDULE:
        raise RuntimeError("paged decode: the decode schedule did not fit its workspace")
    raise RuntimeError(f"unknown device error flags 0x{flags:x}")


# ---------------------------------------------------------------------------
# KV write
# ---------------------------------------------------------------------------
def _diagnose_write(key, value, key_cache, value_cache, slot_mapping, block_size) -> None:
    """Raise the error of the first failed check of ``paged_cache_write``, in
    the order the checks are documented (the call's fast path tests them all
    at once)."""
    _require(key.dim() == 3,
             lambda: f"key must be [num_tokens, num_kv_heads, head_dim], got {tuple(key.shape)}")
    _require(key.shape == value.shape, lambda: f"key {tuple(key.shape)} != value {tuple(value.shape)}")
    _require(key_cache.dim() == 4, lambda: f"key_cache must be 4-D, got {tuple(key_cache.shape)}")
    _require(key_cache.shape == value_cache.shape,
             lambda: f"key_cache shape {tuple(key_cache.shape)} != value_cache shape {tuple(value_cache.shape)}")
    num_tokens, num_kv_heads, head_dim = key.shape
    num_blocks = key_cache.shape[0]
    _require(slot_mapping.dim() == 1 and slot_mapping.shape[0] == num_tokens,
             lambda: f"slot_mapping length {tuple(slot_mapping.shape)} != num_tokens {num_tokens}")
    _require(num_kv_heads == key_cache.shape[1],
             lambda: f"key num_kv_heads {num_kv_heads} != key_cache num_kv_heads {key_cache.shape[1]}")
    _require(head_dim == key_cache.shape[3],
             lambda: f"key head_dim {head_dim} != key_cache head_dim {key_cache.shape[3]}")
    _require(block_size > 0, lambda: f"block_size must be > 0, got {block_size}")
    _require(block_size == key_cache.shape[2],
             lambda: f"block_size {block_size} != cache dim2 {key_cache.shape[2]}")
    _require(key.dtype == key_cache.dtype,
             lambda: f"key dtype {key.dtype} != cache dtype {key_cache.dtype}")
    _require(value.dtype == value_cache.dtype,
             lambda: f"value dtype {value.dtype} != value_cache dtype {value_cache.dtype}")
    _require(key_cache.dtype in _DTYPE_CODES, lambda: f"unsupported cache dtype {key_cache.dtype}")
    _require(key.device == key_cache.device,
             lambda: f"key device {key.device} != cache device {key_cache.device}")
    _require(value.device == value_cache.device,
             lambda: f"value device {value.device} != value_cache device {value_cache.device}")
    _require(key.device.type == "cuda", lambda: f"key.device must be cuda, got {key.device}")
    _require(value_cache.device == key_cache.device,
             lambda: f"value_cache device {value_cache.device} != key_cache device {key_cache.device}")
    _require(key_cache.is_contiguous() and value_cache.is_contiguous(),
             "key_cache and value_cache must be contiguous [num_blocks, num_kv_heads, block_size, head_dim]")
    raise ArgumentError("invalid paged_cache_write arguments")


def paged_cache_write(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
    *,
    strict: bool = True,
    check_duplicates: bool = True,
) -> None:
    """Scatter-write per-token K/V into one layer's paged cache (in place).

    Same bytes as ``write_to_paged_cache`` (mini_vllm/cache/cache_write.py:25-74)
    for every input without duplicate slots; the checks mirror
    ``triton_cache_write`` (paged_attention_gpu.py:109-135).  ``value`` may be
    a strided view (e.g. of a fused QKV output): its strides are passed to the
    kernel instead of making it contiguous.

    ``check_duplicates`` stamps every slot with a per-call epoch to detect two
    tokens writing one slot.  A CUDA graph replays its launch arguments, epoch
    included, so code that captures this call in a graph passes
    ``check_duplicates=False`` (out-of-range slots are still flagged).
    """
    fast = _native.fast()
    if fast is not None and key.is_cuda:  # direct binding: the common case in one C++ call
        state = _state(key.get_device())
        status = fast.kv_write(key, value, key_cache, value_cache, slot_mapping, block_size,
                                         check_duplicates, state.err_ptr)
        if status == _native.OK:
            if strict:
                flags = _take_flags(state)
                if flags:
                    _raise_flags(flags, {"slot_mapping": slot_mapping,
                                         "total_slots": key_cache.shape[0] * block_size,
                                         "block_size": block_size, "num_blocks": key_cache.shape[0]})
            return
        # anything else (a conversion to make, an argument to reject, a failed
        # call to report) takes the full path below
    if not (key.dim() == 3 and key.shape == value.shape and key_cache.dim() == 4
            and key_cache.shape == value_cache.shape and slot_mapping.dim() == 1
            and slot_mapping.shape[0] == key.shape[0] and key.shape[1] == key_cache.shape[1]
            and key.shape[2] == key_cache.shape[3] and block_size > 0 and block_size == key_cache.shape[2]
            and key.dtype == key_cache.dtype and value.dtype == value_cache.dtype
            and key_cache.dtype in _DTYPE_CODES and key.is_cuda
            and key.get_device() == key_cache.get_device() and value.get_device() == value_cache.get_device()
            and value_cache.get_device() == key_cache.get_device()
            and key_cache.is_contiguous() and value_cache.is_contiguous()):
        _diagnose_write(key, value, key_cache, value_cache, slot_mapping, block_size)
    num_tokens, num_kv_heads, head_dim = key.shape
    num_blocks = key_cache.shape[0]
    if num_tokens == 0:
        return
    if key.stride(2) != 1:
        key = key.contiguous()
    if value.stride(2) != 1:
        value = value.contiguous()
    if slot_mapping.dtype != torch.int64 or slot_mapping.get_device() != key.get_device() or not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.to(device=key.device, dtype=torch.int64).contiguous()

    dev_idx = key.get_device()
    state = _state(dev_idx)
    total_slots = num_blocks * block_size
    if check_duplicates:
        claims, epoch = state.next_claims(total_slots)
        claims_ptr = claims.data_ptr()
    else:
        claims_ptr, epoch = None, 0
    status = _native.lib().mvb_kv_cache_write(
        key.data_ptr(), key.stride(0), key.stride(1),
        value.data_ptr(), value.stride(0), value.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(),
        slot_mapping.data_ptr(), num_tokens, num_kv_heads, head_dim, block_size, num_blocks,
        _DTYPE_CODES[key_cache.dtype], claims_ptr, epoch,
        state.err.data_ptr(), _stream_handle(dev_idx),
    )
    _host_status(status, "kv cache write")
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"slot_mapping": slot_mapping, "total_slots": total_slots,
                                 "block_size": block_size, "num_blocks": num_blocks})


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------
def _diagnose_decode(query, key_cache, value_cache, block_table, kv_len_after, block_size) -> None:
    """Raise the error of the first failed check of ``paged_decode_attention``,
    in the documented order (the call's fast path tests them all at once)."""
    _require(query.dim() == 3,
             lambda: f"query must be [total_decode, num_heads, head_dim], got {tuple(query.shape)}")
    total_decode, num_q_heads, head_dim = query.shape
    _require(key_cache.dim() == 4 and key_cache.shape == value_cache.shape,
             lambda: f"key_cache {tuple(key_cache.shape)} / value_cache {tuple(value_cache.shape)} mismatch")
    num_blocks, num_kv_heads = key_cache.shape[0], key_cache.shape[1]
    _require(head_dim in (64, 128), lambda: f"head_dim {head_dim} not supported (only 64, 128)")
    _require(block_size > 0 and (block_size & (block_size - 1)) == 0,
             f"block_size {block_size} must be a power of 2")
    _require(key_cache.shape[2] == block_size,
             lambda: f"block_size {block_size} != cache dim2 {key_cache.shape[2]}")
    _require(key_cache.shape[3] == head_dim,
             lambda: f"cache head_dim {key_cache.shape[3]} != query head_dim {head_dim}")
    _require(num_q_heads % num_kv_heads == 0,
             lambda: f"num_q_heads {num_q_heads} not divisible by num_kv_heads {num_kv_heads}")
    _require(query.dtype in _DTYPE_CODES, lambda: f"query dtype {query.dtype} must be bf16, f16 or f32")
    _require(key_cache.dtype == query.dtype and value_cache.dtype == query.dtype,
             lambda: f"cache dtype {key_cache.dtype} != query dtype {query.dtype}")
    _require(key_cache.is_contiguous() and value_cache.is_contiguous(), "caches must be contiguous")
    _require(block_table.dim() == 2 and block_table.shape[0] == total_decode,
             lambda: f"block_table rows {tuple(block_table.shape)} != total_decode {total_decode}")
    _require(kv_len_after.shape == (total_decode,),
             lambda: f"kv_len_after shape {tuple(kv_len_after.shape)} != ({total_decode},)")
    _require(query.device.type == "cuda", lambda: f"query.device must be cuda, got {query.device}")
    _require(key_cache.device == query.device and value_cache.device == query.device,
             "query and caches must share one device")
    raise ArgumentError("invalid paged_decode_attention arguments")


_plan_cache: Dict[tuple, Dict[str, Any]] = {}


def _cached_plan(device_index: int, *args) -> Dict[str, Any]:
    """decode_plan memoised per device and shape (the plan is a pure function of
    them), so the per-step host path makes one library call, not two."""
    key = (device_index,) + args
    plan = _plan_cache.get(key)
    if plan is None:
        if len(_plan_cache) > 256:
            _plan_cache.clear()
        plan = decode_plan(*args)
        _plan_cache[key] = plan
    return plan


def decode_plan(
    num_seqs: int,
    num_heads: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    num_blocks: int,
    max_blocks_per_seq: int,
    dtype: torch.dtype,
    variant: str = "auto",
    partition_tokens: Optional[int] = None,
    cache_ptr: int = 0,
) -> Dict[str, Any]:
    """The library's launch plan for a decode of this shape (no GPU work)."""
    import ctypes

    v, pt, np_, nl = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    ws = ctypes.c_int64()
    status = _native.lib().mvb_paged_decode_plan(
        num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks, max_blocks_per_seq,
        _DTYPE_CODES[dtype], _VARIANTS[variant], int(partition_tokens or 0), cache_ptr or None,
        ctypes.byref(v), ctypes.byref(pt), ctypes.byref(np_), ctypes.byref(ws), ctypes.byref(nl),
    )
    _host_status(status, "paged decode plan")
    return {"variant": _VARIANT_NAMES[v.value], "partition_tokens": pt.value,
            "num_partitions": np_.value, "workspace_bytes": ws.value, "launches": nl.value}


def _decode_fast(query, key_cache, value_cache, block_table, kv_len_after, block_size, scale, out, variant,
                 partition_tokens, strict, after_write, schedule=None) -> Optional[torch.Tensor]:
    """The common case of a decode in one C++ call (the direct binding), or
    None when the full path of paged_decode_attention must run instead (no
    binding, a conversion to make, an argument to reject, a failed call)."""
    fast = _native.fast()
    if fast is None or not query.is_cuda:
        return None
    state = _state(query.get_device())
    flags = _native.DECODE_AFTER_WRITE if after_write else 0
    ws = None
    if schedule is not None and schedule.variant is not None:
        if variant not in ("auto", schedule.variant):
            return None
        variant = schedule.variant  # the kernel the schedule was built for
        flags |= _native.DECODE_SCHEDULE_READY
        ws = schedule.workspace
    status, res = fast.decode(query, key_cache, value_cache, block_table, kv_len_after, block_size,
                              -1.0 if scale is None else float(scale), out,
                              _VARIANTS.get(variant, -1) | flags,
                              int(partition_tokens or 0), state.err_ptr, ws)
    if status != _native.OK:
        return None
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"kv_len_after": kv_len_after, "max_blocks": block_table.shape[1],
                                 "block_size": block_size, "num_blocks": key_cache.shape[0]})
    return res


class DecodeSchedule:
    """The per-step set-up of the decode kernel the plan picks (``variant``:
    ``"stream"`` or ``"sched"``; ``None`` for kernels that need none) and the
    device workspace it lives in: the step's tile ranges and the pool row of
    each KV tile.

    kv_len and the block tables are the same for every layer of a model step,
    so one schedule, built once per step by ``build_decode_schedule``, serves
    every layer's ``paged_decode_attention(..., schedule=...)``.  It depends on
    the contents of ``kv_len_after`` and ``block_tables`` and on the shapes it
    was built for; build it again whenever those change, and after a call that
    raised a device timeout (which may leave its counters dirty).
    """

    __slots__ = ("workspace", "key", "variant")

    def __init__(self, workspace: Optional[torch.Tensor], key: tuple, variant: Optional[str] = "sched") -> None:
        self.workspace = workspace
        self.key = key
        self.variant = variant


def build_decode_schedule(
    kv_len_after: torch.Tensor,
    block_tables: torch.Tensor,
    num_heads: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    num_blocks: int,
    dtype: torch.dtype,
    *,
    schedule: Optional[DecodeSchedule] = None,
    after_write: bool = False,
    strict: bool = True,
    variant: str = "auto",
) -> DecodeSchedule:
    """Build the per-step decode schedule of a batch
    (``mvb_paged_decode_schedule``, one launch on the current stream) for
    decodes of the given shape with ``variant`` (the plan's kernel: the stream
    and scheduled kernels have a per-step set-up, the others none), with
    ``block_tables`` ``[num_seqs, max_blocks_per_seq]`` (``-1`` padded).
    ``schedule`` reuses an earlier schedule's workspace when it is large
    enough.  ``after_write``: the kernel launched just before on the current
    stream is ``paged_cache_write`` (the schedule is then computed while it
    runs)."""
    _require(kv_len_after.dim() == 1 and kv_len_after.is_cuda,
             lambda: f"kv_len_after must be a 1-D CUDA tensor, got {tuple(kv_len_after.shape)}")
    if kv_len_after.dtype != torch.int32 or not kv_len_after.is_contiguous():
        kv_len_after = kv_len_after.to(torch.int32).contiguous()
    num_seqs = kv_len_after.shape[0]
    dev_idx = kv_len_after.get_device()
    _require(block_tables.dim() == 2 and block_tables.shape[0] == num_seqs,
             lambda: f"block_tables must be [num_seqs={num_seqs}, max_blocks], got {tuple(block_tables.shape)}")
    if block_tables.dtype != torch.int64 or block_tables.get_device() != dev_idx or block_tables.stride(1) != 1:
        block_tables = block_tables.to(device=kv_len_after.device, dtype=torch.int64).contiguous()
    max_blocks_per_seq = block_tables.shape[1]
    _require(variant in _VARIANTS, lambda: f"variant must be one of {sorted(_VARIANTS)}, got {variant!r}")
    plan = _cached_plan(dev_idx, num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks,
                        max_blocks_per_seq, dtype, variant, None, 16)
    nbytes = plan["workspace_bytes"]
    key = (dev_idx, num_seqs, num_heads, num_kv_heads, head_dim, block_size, num_blocks, max_blocks_per_seq, dtype,
           plan["variant"])
    if plan["variant"] not in ("stream", "sched"):
        return DecodeSchedule(None, key, None)  # the plan's kernel has no per-step set-up
    if schedule is not None and schedule.workspace.get_device() == dev_idx and schedule.workspace.numel() >= nbytes:
        ws = schedule.workspace
    else:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=kv_len_after.device)
    state = _state(dev_idx)
    status = _native.lib().mvb_paged_decode_schedule(
        kv_len_after.data_ptr(), block_tables.data_ptr(), block_tables.stride(0), num_seqs, num_heads,
        num_kv_heads, head_dim, block_size, num_blocks,
        max_blocks_per_seq, _DTYPE_CODES[dtype], _VARIANTS[variant], _native.DECODE_AFTER_WRITE if after_write else 0,
        ws.data_ptr(), ws.numel(), state.err_ptr, _stream_handle(dev_idx))
    _host_status(status, "paged decode schedule")
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"kv_len_after": kv_len_after, "max_blocks": max_blocks_per_seq,
                                 "block_size": block_size, "num_blocks": num_blocks})
    if schedule is not None and schedule.workspace is ws:
        schedule.key = key
        schedule.variant = plan["variant"]
        return schedule
    return DecodeSchedule(ws, key, plan["variant"])


def paged_decode_attention(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: torch.Tensor,
    kv_len_after: torch.Tensor,
    block_size: int,
    scale: Optional[float] = None,
    *,
    out: Optional[torch.Tensor] = None,
    variant: str = "auto",
    partition_tokens: Optional[int] = None,
    strict: bool = True,
    after_write: bool = False,
    schedule: Optional[DecodeSchedule] = None,
) -> torch.Tensor:
    """Paged decode attention (one query token per sequence) on the B200 kernels.

    Args (as ``triton_decode_attention``, paged_attention_gpu.py:252-321):
        query: ``[total_decode, num_q_heads, head_dim]`` bf16 / f16 / f32.
        key_cache, value_cache: ``[num_blocks, num_kv_heads, block_size, head_dim]``.
        block_table: ``[total_decode, max_blocks_per_seq]`` int64, ``-1`` padded.
        kv_len_after: ``[total_decode]`` int32 — tokens to attend per sequence.
        block_size: tokens per block (power of two).
        scale: softmax scale, default ``head_dim ** -0.5``.
    Keyword-only extensions: ``out`` (write in place), ``variant``
    (``"auto" | "sched" | "stream" | "mma" | "fma"``; ``"auto"`` is
    ``"stream"`` for bf16/f16 caches with block sizes that are multiples of 16
    and batches it serves, else ``"sched"`` where that applies, else ``"fma"``;
    with ``schedule`` it is ``"sched"``),
    ``partition_tokens`` (split-K partition length of the ``"mma"`` / ``"fma"``
    kernels; ``None`` lets the library choose), ``strict``, ``after_write``
    (the kernel launched just before this call on the current stream is
    ``paged_cache_write``: the kernel then reads query, block table, kv_len
    and schedule while the write is still running and waits only before its
    cache loads; leave it False when any other kernel may run in between and
    signal its dependents early), ``schedule`` (a ``DecodeSchedule`` of this
    batch from ``build_decode_schedule``: the ``"sched"`` kernel then skips its
    own schedule launch; without it every call builds the schedule first).

    Returns ``[total_decode, num_q_heads, head_dim]`` in the query's dtype.
    """
    if schedule is not None and schedule.variant is not None and variant == "auto":
        variant = schedule.variant
    res = _decode_fast(query, key_cache, value_cache, block_table, kv_len_after, block_size, scale, out,
                       variant, partition_tokens, strict, after_write, schedule)
    if res is not None:
        return res
    # anything else takes the full path below
    if not (query.dim() == 3 and key_cache.dim() == 4 and key_cache.shape == value_cache.shape
            and query.shape[2] in (64, 128) and block_size > 0 and (block_size & (block_size - 1)) == 0
            and key_cache.shape[2] == block_size and key_cache.shape[3] == query.shape[2]
            and key_cache.shape[1] > 0 and query.shape[1] % key_cache.shape[1] == 0
            and query.dtype in _DTYPE_CODES and key_cache.dtype == query.dtype
            and value_cache.dtype == query.dtype and key_cache.is_contiguous() and value_cache.is_contiguous()
            and block_table.dim() == 2 and block_table.shape[0] == query.shape[0]
            and kv_len_after.shape == (query.shape[0],) and query.is_cuda
            and key_cache.get_device() == query.get_device() and value_cache.get_device() == query.get_device()):
        _diagnose_decode(query, key_cache, value_cache, block_table, kv_len_after, block_size)
    total_decode, num_q_heads, head_dim = query.shape
    num_blocks, num_kv_heads = key_cache.shape[0], key_cache.shape[1]
    if scale is None:
        scale = head_dim ** -0.5

    if out is None:
        out = torch.empty((total_decode, num_q_heads, head_dim), dtype=query.dtype, device=query.device)
    else:
        _require(out.shape == query.shape and out.dtype == query.dtype and out.get_device() == query.get_device(),
                 "out must match query's shape, dtype and device")
        _require(out.stride(2) == 1, "out's last dimension must be contiguous")
    if total_decode == 0:
        return out

    if query.stride(2) != 1 or query.data_ptr() % 16 or (query.stride(0) * query.element_size()) % 16 \
            or (query.stride(1) * query.element_size()) % 16:
        query = query.contiguous()
    if block_table.dtype != torch.int64 or block_table.get_device() != query.get_device() or block_table.stride(1) != 1:
        block_table = block_table.to(device=query.device, dtype=torch.int64).contiguous()
    if kv_len_after.dtype != torch.int32 or kv_len_after.get_device() != query.get_device() or not kv_len_after.is_contiguous():
        kv_len_after = kv_len_after.to(device=query.device, dtype=torch.int32).contiguous()

    dev_idx = query.get_device()
    state = _state(dev_idx)
    max_blocks = block_table.shape[1]
    # the plan only inspects the cache pointer's 16-byte alignment
    plan = _cached_plan(dev_idx, total_decode, num_q_heads, num_kv_heads, head_dim, block_size,
                        num_blocks, max_blocks, query.dtype, variant, partition_tokens,
                        16 if key_cache.data_ptr() % 16 == 0 else 8)
    ws_bytes = plan["workspace_bytes"]
    flags = _native.DECODE_AFTER_WRITE if after_write else 0
    if schedule is not None and schedule.variant is not None:
        _require(plan["variant"] == schedule.variant,
                 lambda: f"the schedule was built for the {schedule.variant!r} kernel, the plan is {plan['variant']!r}")
        _require(schedule.workspace.get_device() == dev_idx and schedule.workspace.numel() >= ws_bytes,
                 "the schedule was built for another device or a smaller shape")
        ws_ptr, ws_bytes = schedule.workspace.data_ptr(), schedule.workspace.numel()
        flags |= _native.DECODE_SCHEDULE_READY
    else:
        ws_ptr = state.workspace(ws_bytes, plan["variant"], _stream_handle(dev_idx)).data_ptr() \
            if ws_bytes > 0 else None
    status = _native.lib().mvb_paged_decode(
        query.data_ptr(), query.stride(0), query.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(),
        block_table.data_ptr(), block_table.stride(0), max_blocks,
        kv_len_after.data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        total_decode, num_q_heads, num_kv_heads, head_dim, block_size, num_blocks,
        float(scale), _DTYPE_CODES[query.dtype],
        _VARIANTS[variant] | flags, int(partition_tokens or 0),
        ws_ptr, ws_bytes, state.err.data_ptr(), _stream_handle(dev_idx),
    )
    _host_status(status, "paged decode")
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"kv_len_after": kv_len_after, "max_blocks": max_blocks,
                                 "block_size": block_size, "num_blocks": num_blocks})
    return out


# ---------------------------------------------------------------------------
# gather (prefill prefix read)
# ---------------------------------------------------------------------------
def _host_ints(values) -> List[int]:
    if isinstance(values, torch.Tensor):
        return [int(v) for v in values.reshape(-1).tolist()]
    return [int(v) for v in values]


def paged_prefill_attention(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_rows,
    cached_len: torch.Tensor,
    query_len: torch.Tensor,
    block_size: int,
    *,
    key: Optional[torch.Tensor] = None,
    value: Optional[torch.Tensor] = None,
    scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None,
    strict: bool = True,
) -> torch.Tensor:
    """Causal prefill attention of a batch of chunks read in place from the
    paged pool (``mvb_paged_prefill``, one launch for the batch, no host
    synchronisation).

    Chunk ``i`` holds ``query_len[i]`` query tokens, one after another in
    ``query`` ``[total_q, num_heads, head_dim]``; its sequence's block table is
    ``block_table[seq_rows[i]]`` and ``cached_len[i]`` of its tokens are in the
    cache before it.  Its token ``t`` attends positions
    ``[0, cached_len[i] + t]``: the cached prefix from the pool, the chunk from
    ``key`` / ``value`` (``[total_q, num_kv_heads, head_dim]``) when given, else
    from the pool (written there first, as the reference's runner does).  The
    same result as AttentionBackendGPU.prefill_attention
    (paged_attention_gpu.py:577-661) without its per-sequence gather, concat,
    GQA repeat and SDPA.  ``seq_rows`` / ``cached_len`` / ``query_len`` may be
    lists or tensors (int64 on the device is the zero-copy form).
    Returns ``[total_q, num_heads, head_dim]`` in the query's dtype.
    """
    _require(query.dim() == 3 and query.is_cuda, lambda: f"query must be a 3-D CUDA tensor, got {tuple(query.shape)}")
    _require(key_cache.dim() == 4 and key_cache.shape == value_cache.shape,
             lambda: f"key_cache {tuple(key_cache.shape)} / value_cache {tuple(value_cache.shape)} mismatch")
    _require(query.dtype in (torch.bfloat16, torch.float16) and key_cache.dtype == query.dtype
             and value_cache.dtype == query.dtype,
             lambda: f"prefill needs bf16 or f16 query and caches of that dtype, got {query.dtype} / {key_cache.dtype}")
    _require(key_cache.is_contiguous() and value_cache.is_contiguous(), "caches must be contiguous")
    total_q, num_heads, head_dim = query.shape
    num_blocks, num_kv_heads, bs, d2 = key_cache.shape
    _require(bs == block_size and d2 == head_dim, lambda: f"cache {tuple(key_cache.shape)} does not match "
                                                          f"block_size {block_size} / head_dim {head_dim}")
    _require(num_heads % num_kv_heads == 0, lambda: f"{num_heads} query heads over {num_kv_heads} KV heads")
    _require((key is None) == (value is None), "give both key and value, or neither")
    dev = query.device
    dev_idx = query.get_device()

    def as_dev64(x):
        if isinstance(x, torch.Tensor):
            return x.to(device=dev, dtype=torch.int64).contiguous()
        return torch.tensor(list(x), dtype=torch.int64).to(dev)

    rows, cached, qlen = as_dev64(seq_rows), as_dev64(cached_len), as_dev64(query_len)
    n = rows.numel()
    _require(cached.numel() == n and qlen.numel() == n,
             lambda: f"{n} sequences but {cached.numel()} cached lengths and {qlen.numel()} query lengths")
    if out is None:
        out = torch.empty_like(query)
    else:
        _require(out.shape == query.shape and out.dtype == query.dtype and out.get_device() == dev_idx
                 and out.stride(2) == 1, "out must match query's shape, dtype and device, last dim contiguous")
    if n == 0 or total_q == 0:
        return out
    if query.stride(2) != 1:
        query = query.contiguous()
    if key is not None:
        _require(key.shape == (total_q, num_kv_heads, head_dim) and value.shape == key.shape,
                 lambda: f"key / value must be [{total_q}, {num_kv_heads}, {head_dim}]")
        if key.stride(2) != 1 or (key.stride(0) * key.element_size()) % 16 or (key.stride(1) * key.element_size()) % 16 \
                or key.data_ptr() % 16:
            key = key.contiguous()
        if value.stride(2) != 1 or (value.stride(0) * value.element_size()) % 16 \
                or (value.stride(1) * value.element_size()) % 16 or value.data_ptr() % 16:
            value = value.contiguous()
    if block_table.dtype != torch.int64 or block_table.get_device() != dev_idx or block_table.stride(1) != 1:
        block_table = block_table.to(device=dev, dtype=torch.int64).contiguous()
    state = _state(dev_idx)
    scale = head_dim ** -0.5 if scale is None else float(scale)
    status = _native.lib().mvb_paged_prefill(
        query.data_ptr(), query.stride(0), query.stride(1),
        key.data_ptr() if key is not None else None, key.stride(0) if key is not None else 0,
        key.stride(1) if key is not None else 0,
        value.data_ptr() if value is not None else None, value.stride(0) if value is not None else 0,
        value.stride(1) if value is not None else 0,
        key_cache.data_ptr(), value_cache.data_ptr(), block_table.data_ptr(), block_table.shape[0],
        block_table.stride(0), block_table.shape[1], rows.data_ptr(), cached.data_ptr(), qlen.data_ptr(), n,
        total_q, out.data_ptr(), out.stride(0), out.stride(1), num_heads, num_kv_heads, head_dim, block_size,
        num_blocks, scale, _DTYPE_CODES[query.dtype], state.err_ptr, _stream_handle(dev_idx))
    _host_status(status, "paged prefill")
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"max_blocks": block_table.shape[1], "block_size": block_size,
                                 "num_blocks": num_blocks})
    return out


def paged_gather(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_rows,
    num_tokens,
    block_size: int,
    *,
    strict: bool = True,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Logical -> physical gather of the first ``num_tokens[i]`` cached tokens
    of each sequence ``block_table[seq_rows[i]]`` into contiguous
    ``[sum(num_tokens), num_kv_heads, head_dim]`` K and V, sequences one after
    another (``mvb_paged_gather``, one launch for the batch).

    The batched form of ``gather_paged_kv`` (mini_vllm/cache/cache_read.py:19-84).
    A table too short for a sequence's tokens raises ``IndexError`` as there;
    a ``-1`` or out-of-range block id inside them raises ``IndexError`` too.
    """
    _require(key_cache.dim() == 4 and key_cache.shape == value_cache.shape,
             lambda: f"key_cache {tuple(key_cache.shape)} / value_cache {tuple(value_cache.shape)} mismatch")
    _require(key_cache.dtype == value_cache.dtype and key_cache.dtype in _DTYPE_CODES,
             lambda: f"cache dtypes {key_cache.dtype} / {value_cache.dtype} must match and be bf16, f16 or f32")
    _require(key_cache.is_contiguous() and value_cache.is_contiguous(), "caches must be contiguous")
    _require(key_cache.is_cuda and value_cache.get_device() == key_cache.get_device(),
             "key_cache and value_cache must be on one CUDA device")
    num_blocks, num_kv_heads, bs, head_dim = key_cache.shape
    _require(block_size == bs, lambda: f"block_size {block_size} != cache dim2 {bs}")
    _require((head_dim * key_cache.element_size()) % 16 == 0,
             lambda: f"head_dim {head_dim} rows must be a multiple of 16 bytes")
    rows, counts = _host_ints(seq_rows), _host_ints(num_tokens)
    _require(len(rows) == len(counts), lambda: f"{len(rows)} sequences but {len(counts)} token counts")
    if any(n < 0 for n in counts):
        raise ValueError(f"token counts must be >= 0, got {counts}")
    _require(block_table.dim() == 2, lambda: f"block_table must be 2-D, got {tuple(block_table.shape)}")
    n_rows, max_blocks = block_table.shape
    for r in rows:
        if not 0 <= r < n_rows:
            raise IndexError(f"sequence index {r} out of range for a block table of {n_rows} rows")
    total = sum(counts)
    dev = key_cache.device
    out_k = torch.empty((total, num_kv_heads, head_dim), dtype=key_cache.dtype, device=dev)
    out_v = torch.empty((total, num_kv_heads, head_dim), dtype=key_cache.dtype, device=dev)
    if total == 0:
        return out_k, out_v
    for n in counts:
        if n > max_blocks * block_size:
            raise IndexError(
                f"block_table length {max_blocks} insufficient to cover {n} tokens (block_size={block_size})"
            )
    if block_table.dtype != torch.int64 or block_table.get_device() != key_cache.get_device() \
            or block_table.stride(1) != 1:
        block_table = block_table.to(device=dev, dtype=torch.int64).contiguous()
    offsets = [0]
    for n in counts:
        offsets.append(offsets[-1] + n)
    meta = torch.tensor(rows + offsets, dtype=torch.int64).to(dev)  # one small copy: rows, then offsets
    dev_idx = key_cache.get_device()
    state = _state(dev_idx)
    stream = _stream_handle(dev_idx)
    status = _native.lib().mvb_paged_gather(
        key_cache.data_ptr(), value_cache.data_ptr(), block_table.data_ptr(), n_rows, block_table.stride(0),
        max_blocks, meta.data_ptr(), meta.data_ptr() + 8 * len(rows), out_k.data_ptr(), out_v.data_ptr(),
        len(rows), total, num_kv_heads, head_dim, block_size, num_blocks, _DTYPE_CODES[key_cache.dtype],
        state.gather_counter(stream or 0), state.err_ptr, stream,
    )
    _host_status(status, "paged gather")
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"max_blocks": max_blocks, "block_size": block_size, "num_blocks": num_blocks})
    return out_k, out_v


def gather_prefix_kv(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table: torch.Tensor,
    cached_len_before,
    seq_indices,
    block_size: int,
    *,
    strict: bool = True,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """The cached prefixes of the prefill sequences, concatenated:
    ``[sum(cached_len_before), num_kv_heads, head_dim]`` K and V.

    Same signature and result as the Triton ``gather_prefix_kv``
    (paged_attention_gpu.py:391-433), with no host loop over tokens; rows of
    ``block_table`` are the global sequence indices ``seq_indices``."""
    return paged_gather(key_cache, value_cache, block_table, seq_indices, cached_len_before, block_size,
                        strict=strict)


def gather_paged_kv(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_table,
    num_tokens: int,
    block_size: int,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``gather_paged_kv`` (mini_vllm/cache/cache_read.py:19-84) on the GPU: the
    first ``num_tokens`` tokens of one sequence whose physical blocks are
    ``block_table`` (a list of ids in logical order)."""
    ids = _host_ints(block_table)
    if num_tokens > len(ids) * block_size:
        raise IndexError(
            f"block_table length {len(ids)} insufficient to cover {num_tokens} tokens (block_size={block_size})"
        )
    table = torch.tensor([ids or [0]], dtype=torch.int64)
    return paged_gather(key_cache, value_cache, table, [0], [int(num_tokens)], block_size)


# ---------------------------------------------------------------------------
# rotary embedding fused with the KV write
# ---------------------------------------------------------------------------
def rope_tables(head_dim: int, theta: float = 1000000.0, max_seq_len: int = 32768,
                dtype: torch.dtype = torch.float32, device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """The cos / sin cache ``[max_seq_len, head_dim]`` of the reference's
    RotaryEmbedding (mini_vllm/model/rotary.py:15-33): inverse frequencies
    theta^(-2i/D), outer product with the positions, duplicated halves, cos/sin
    in float32, then cast to ``dtype``.  The same torch operations in the same
    order, so the tables are bit-identical to the reference's on the same
    device."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=device) / head_dim))
    pos = torch.arange(max_seq_len, dtype=torch.float32, device=device)
    freqs = torch.einsum("i,j->ij", pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rope_cache_write(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    positions: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
    *,
    query_out: Optional[torch.Tensor] = None,
    return_key: bool = False,
    strict: bool = True,
    check_duplicates: bool = True,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """RoPE of the step's query and key rows fused with the paged KV write, in one launch.

    Bit for bit the reference's ``q = rope(q, positions); k = rope(k, positions);
    write_kv_cache(k, v, slot_mapping)`` (mini_vllm/model_runner/qwen_runner.py:
    163-170) with ``rope`` = ``RotaryEmbedding.__call__`` (rotary.py:47-85) over
    the tables ``cos`` / ``sin`` (see ``rope_tables``).  Returns the rotated
    query (into ``query_out`` when given, which may be ``query`` itself) and,
    with ``return_key``, the rotated keys (which the prefill path appends after
    the cached prefix).  Slots follow ``paged_cache_write``; a position outside
    the tables raises ``IndexError``.
    """
    _require(query.dim() == 3 and key.dim() == 3 and key.shape == value.shape,
             lambda: f"query {tuple(query.shape)} / key {tuple(key.shape)} / value {tuple(value.shape)}")
    num_tokens, num_heads, head_dim = query.shape
    _require(key.shape[0] == num_tokens and key.shape[2] == head_dim,
             lambda: f"key {tuple(key.shape)} does not match query {tuple(query.shape)}")
    num_kv_heads = key.shape[1]
    _require(key_cache.dim() == 4 and key_cache.shape == value_cache.shape
             and key_cache.shape[1] == num_kv_heads and key_cache.shape[3] == head_dim,
             lambda: f"caches {tuple(key_cache.shape)} / {tuple(value_cache.shape)} do not match key "
                     f"{tuple(key.shape)}")
    _require(block_size > 0 and key_cache.shape[2] == block_size,
             lambda: f"block_size {block_size} != cache dim2 {key_cache.shape[2]}")
    _require(head_dim % 2 == 0, lambda: f"head_dim {head_dim} must be even")
    dt = query.dtype
    _require(dt in _DTYPE_CODES and key.dtype == dt and value.dtype == dt and key_cache.dtype == dt
             and value_cache.dtype == dt and cos.dtype == dt and sin.dtype == dt,
             "query, key, value, caches and cos/sin tables must share one dtype (bf16, f16 or f32)")
    _require(cos.dim() == 2 and cos.shape == sin.shape and cos.shape[1] == head_dim,
             lambda: f"cos/sin tables {tuple(cos.shape)} / {tuple(sin.shape)} must be [rows, {head_dim}]")
    _require(positions.dim() == 1 and positions.shape[0] == num_tokens,
             lambda: f"positions {tuple(positions.shape)} != ({num_tokens},)")
    _require(slot_mapping.dim() == 1 and slot_mapping.shape[0] == num_tokens,
             lambda: f"slot_mapping {tuple(slot_mapping.shape)} != ({num_tokens},)")
    _require(query.is_cuda, lambda: f"query.device must be cuda, got {query.device}")
    dev_idx = query.get_device()
    _require(all(t.get_device() == dev_idx for t in (key, value, key_cache, value_cache, cos, sin)),
             "query, key, value, caches and tables must be on one CUDA device")
    _require(key_cache.is_contiguous() and value_cache.is_contiguous(), "caches must be contiguous")
    if query_out is None:
        query_out = torch.empty((num_tokens, num_heads, head_dim), dtype=dt, device=query.device)
    else:
        _require(query_out.shape == query.shape and query_out.dtype == dt and query_out.get_device() == dev_idx
                 and query_out.stride(2) == 1, "query_out must match query and have a contiguous last dim")
    key_out = torch.empty((num_tokens, num_kv_heads, head_dim), dtype=dt, device=query.device) if return_key \
        else None
    if num_tokens == 0:
        return query_out, key_out
    if query.stride(2) != 1:
        query = query.contiguous()
    if key.stride(2) != 1:
        key = key.contiguous()
    if value.stride(2) != 1:
        value = value.contiguous()
    cos, sin = cos.contiguous(), sin.contiguous()
    if positions.dtype != torch.int64 or positions.get_device() != dev_idx or not positions.is_contiguous():
        positions = positions.to(device=query.device, dtype=torch.int64).contiguous()
    if slot_mapping.dtype != torch.int64 or slot_mapping.get_device() != dev_idx or not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.to(device=query.device, dtype=torch.int64).contiguous()
    state = _state(dev_idx)
    num_blocks = key_cache.shape[0]
    if check_duplicates:
        claims, epoch = state.next_claims(num_blocks * block_size)
        claims_ptr = claims.data_ptr()
    else:
        claims_ptr, epoch = None, 0
    status = _native.lib().mvb_rope_kv_cache_write(
        query.data_ptr(), query.stride(0), query.stride(1), query_out.data_ptr(), query_out.stride(0),
        query_out.stride(1), key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(), value.stride(0),
        value.stride(1), positions.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
        key_cache.data_ptr(), value_cache.data_ptr(), slot_mapping.data_ptr(),
        key_out.data_ptr() if key_out is not None else None, num_tokens, num_heads, num_kv_heads, head_dim,
        block_size, num_blocks, _DTYPE_CODES[dt], claims_ptr, epoch, state.err_ptr, _stream_handle(dev_idx),
    )
    _host_status(status, "rope + kv cache write")
    if strict:
        flags = _take_flags(state)
        if flags:
            _raise_flags(flags, {"slot_mapping": slot_mapping, "total_slots": num_blocks * block_size,
                                 "block_size": block_size, "num_blocks": num_blocks, "table_rows": cos.shape[0]})
    return query_out, key_out


# Reference names, for code that imports them from the Triton module.
triton_cache_write = paged_cache_write
triton_decode_attention = paged_decode_attention


# ---------------------------------------------------------------------------
# backend class
# ---------------------------------------------------------------------------
class AttentionBackendB200(AttentionBackend):
    """``AttentionBackend`` on the B200 kernels (mirror of AttentionBackendGPU,
    paged_attention_gpu.py:454-661).

    * ``write_kv_cache`` → ``paged_cache_write`` (CUDA scatter kernel);
    * ``decode_attention`` → ``paged_decode_attention`` (TMA + tensor-core
      kernel for bf16/f16, FMA kernel otherwise, split-K for long contexts);
    * ``prefill_attention`` → torch gather of the paged prefix by index
      tensors plus SDPA (no Triton; the reference's C3 path, :577-661).
    """

    def __init__(self, config: Any, *, strict: bool = True, decode_variant: str = "auto",
                 partition_tokens: Optional[int] = None, overlap_after_write: bool = False) -> None:
        hd = getattr(config, "head_dim", 0)
        if hd not in (64, 128):
            raise RuntimeError(
                f"AttentionBackendB200: head_dim={hd} not supported (only 64, 128)."
            )
        if decode_variant not in _VARIANTS:
            raise ValueError(f"decode_variant must be one of {sorted(_VARIANTS)}, got {decode_variant!r}")
        if not torch.cuda.is_available():
            raise RuntimeError("attention_backend='b200' requires CUDA, but CUDA is not available.")
        _native.lib()  # fail here, not at the first step, when the library is missing
        self._config = config
        self._pool: Optional[KVCachePool] = None
        self._block_size = 0
        self.strict = strict
        self.decode_variant = decode_variant
        self.partition_tokens = partition_tokens
        # With overlap_after_write, a decode that directly follows this
        # backend's KV write of the same layer on the same stream starts its
        # set-up while the write runs (``after_write``).  The caller promises
        # that nothing launched between the two calls signals its dependents
        # early and writes the decode's inputs (plain torch kernels do not).
        self.overlap_after_write = overlap_after_write
        self._last_write: Optional[Tuple[int, int]] = None
        # The decode schedule of the current step (variants "stream" and
        # "sched"): built at
        # layer 0 of every step and whenever the metadata object, its
        # tensors or the shapes change; every other layer reuses it.
        self._schedule: Optional[DecodeSchedule] = None
        self._schedule_key: Optional[tuple] = None
        self._schedule_src: tuple = (None, None, None, None, None, None)

    def begin_step(self) -> None:
        """Forget the current step's decode schedule, so the next decode builds
        a new one.  Layer 0 and a new metadata object already do this; a
        caller that rewrites the metadata tensors in place between the layers
        of a step calls it after doing so."""
        self._schedule_key = None

    def allocate_pool(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int,
                      head_dim: int, dtype: torch.dtype, device: torch.device) -> KVCachePool:
        validate_block_size(block_size)
        pool = KVCachePool.allocate(num_layers, num_blocks, block_size, num_kv_heads, head_dim,
                                    dtype, device)
        self._pool = pool
        self._block_size = block_size
        return pool

    def write_kv_cache(self, layer_idx: int, key: torch.Tensor, value: torch.Tensor,
                       slot_mapping: torch.Tensor) -> None:
        pool = self._pool
        assert pool is not None, "allocate_pool must be called first"
        self._last_write = None
        paged_cache_write(key, value, pool.key_caches[layer_idx], pool.value_caches[layer_idx],
                          slot_mapping, pool.block_size, strict=self.strict)
        if self.overlap_after_write and key.shape[0] > 0:
            self._last_write = (layer_idx, _stream_handle(key.get_device()))

    def decode_attention(self, layer_idx: int, query: torch.Tensor, attn_metadata: Any,
                         pool: Any, *, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The reference method (backend.py:63-77); ``out=`` (an extension) lets
        a runner decode straight into its ``attn_out[num_prefill:]`` slice
        instead of allocating and copying (qwen_runner.py:173-190)."""
        last, self._last_write = self._last_write, None  # only the very next decode may overlap
        if query.shape[0] == 0:
            return query
        group = None
        for g in attn_metadata.groups:
            if g.attention_type == "decode_gpu":
                group = g
                break
        if group is None:
            return query
        after = last is not None and query.is_cuda and last == (layer_idx, _stream_handle(query.get_device()))
        kc, vc = pool.key_caches[layer_idx], pool.value_caches[layer_idx]
        bt, kvl = attn_metadata.decode_block_tables, group.kv_len_after
        schedule = self._step_schedule(layer_idx, query, kc, bt, kvl, attn_metadata, pool.block_size, after)
        if schedule is not None and self._schedule_built_now:
            after = False  # the decode now follows the schedule launch, not the write
        # the common case straight to the binding (per-step host time); else the full path
        res = _decode_fast(query, kc, vc, bt, kvl, pool.block_size, None, out, self.decode_variant,
                           self.partition_tokens, self.strict, after, schedule)
        if res is not None:
            return res
        return paged_decode_attention(query, kc, vc, bt, kvl, pool.block_size, out=out, variant=self.decode_variant,
                                      partition_tokens=self.partition_tokens, strict=self.strict, after_write=after,
                                      schedule=schedule)

    _schedule_built_now = False

    def _step_schedule(self, layer_idx, query, kc, bt, kvl, attn_metadata, block_size, after) -> Optional[DecodeSchedule]:
        """The decode schedule of this step for the "stream" or "sched"
        kernel, built when needed (None when the decode runs another
        kernel)."""
        self._schedule_built_now = False
        if (layer_idx != 0 and self._schedule_key is not None and attn_metadata is self._schedule_src[0]
                and bt is self._schedule_src[1] and kvl is self._schedule_src[2]):
            # the same metadata object and tensors as the layer that built it
            # (the full key below also covers shapes and pools; a caller that
            # rewrites these tensors in place calls begin_step)
            if kc.shape == self._schedule_src[3] and query.shape == self._schedule_src[4] and \
                    query.dtype == self._schedule_src[5]:
                return self._schedule
        if self.decode_variant not in ("auto", "sched", "stream") or not (query.is_cuda and kvl.is_cuda and bt.is_cuda):
            return None
        if query.dtype not in (torch.bfloat16, torch.float16) or block_size % 16 or kc.dtype != query.dtype:
            return None
        key = (id(attn_metadata), bt.data_ptr(), kvl.data_ptr(), tuple(bt.shape), tuple(query.shape[1:]),
               tuple(kc.shape), query.dtype, kvl.dtype)
        if layer_idx != 0 and key == self._schedule_key and self._schedule is not None:
            return self._schedule
        plan = _cached_plan(query.get_device(), query.shape[0], query.shape[1], kc.shape[1], query.shape[2],
                            block_size, kc.shape[0], bt.shape[1], query.dtype, self.decode_variant,
                            self.partition_tokens, 16 if kc.data_ptr() % 16 == 0 else 8)
        if plan["variant"] not in ("sched", "stream"):
            return None
        self._schedule_key = None
        self._schedule = build_decode_schedule(kvl, bt, query.shape[1], kc.shape[1], query.shape[2], block_size,
                                               kc.shape[0], query.dtype, schedule=self._schedule,
                                               after_write=after, strict=False, variant=plan["variant"])
        self._schedule_key = key
        self._schedule_src = (attn_metadata, bt, kvl, kc.shape, query.shape, query.dtype)
        self._schedule_built_now = True
        return self._schedule

    def prefill_attention(self, layer_idx: int, query: torch.Tensor, key: Optional[torch.Tensor],
                          value: Optional[torch.Tensor], attn_metadata: Any, pool: Any) -> torch.Tensor:
        """Causal prefill attention over each sequence's cached prefix and its new
        chunk (mirror of AttentionBackendGPU.prefill_attention,
        paged_attention_gpu.py:577-661).

        One ``paged_prefill_attention`` launch for every prefill group of the
        step: each query tile reads its cached prefix in place from the pool and
        runs causal attention on the tensor cores, with no host synchronisation.
        With the chunk's ``key`` / ``value`` given, the chunk's positions come from
        them, as the Triton backend appends them; with ``None``, the whole
        context is read from the cache (the new tokens are written before
        attention), as AttentionBackendRef does (paged_attention_ref.py:166-240).
        """
        if query.shape[0] == 0:
            return query
        kc, vc = pool.key_caches[layer_idx], pool.value_caches[layer_idx]
        groups = [g for g in attn_metadata.groups if g.attention_type in ("prefill_gpu", "prefill_ref")]
        if not groups:
            return query
        if query.dtype not in (torch.bfloat16, torch.float16) or query.shape[2] not in (64, 128):
            return self._prefill_general(layer_idx, query, key, value, attn_metadata, pool)
        dev = query.device
        rows = torch.cat([torch.as_tensor(g.seq_indices, dtype=torch.int64).to(dev) for g in groups])
        cached = torch.cat([g.cached_len_before.to(device=dev, dtype=torch.int64).reshape(-1) for g in groups])
        qlen = torch.cat([g.query_len.to(device=dev, dtype=torch.int64).reshape(-1) for g in groups])
        with_chunk = key is not None and value is not None
        return paged_prefill_attention(query, kc, vc, attn_metadata.prefill_block_tables, rows, cached, qlen,
                                       pool.block_size, key=key if with_chunk else None,
                                       value=value if with_chunk else None, strict=self.strict)


    def _prefill_general(self, layer_idx, query, key, value, attn_metadata, pool) -> torch.Tensor:
        """Prefill for shapes the paged prefill kernel does not take (fp32, head
        dims other than 64 / 128): one paged_gather launch per group reads the
        cached context, then torch SDPA per sequence with the offset causal mask
        (the structure of paged_attention_gpu.py:577-661)."""
        num_heads, head_dim = query.shape[1], query.shape[2]
        reps = num_heads // pool.num_kv_heads
        scale = head_dim ** -0.5
        kc, vc = pool.key_caches[layer_idx], pool.value_caches[layer_idx]
        with_chunk = key is not None and value is not None
        parts = []
        offset = 0
        for group in attn_metadata.groups:
            if group.attention_type not in ("prefill_gpu", "prefill_ref"):
                continue
            seqs = _host_ints(group.seq_indices)
            cached = _host_ints(group.cached_len_before)
            qlens = _host_ints(group.query_len)
            counts = cached if with_chunk else [c + n for c, n in zip(cached, qlens)]
            ks, vs = paged_gather(kc, vc, attn_metadata.prefill_block_tables, seqs, counts, pool.block_size,
                                  strict=self.strict)
            src = 0
            for c, q_len, n in zip(cached, qlens, counts):
                kv_len = c + q_len
                k, v = ks[src:src + n], vs[src:src + n]
                if with_chunk:
                    k = torch.cat([k, key[offset:offset + q_len]], dim=0)
                    v = torch.cat([v, value[offset:offset + q_len]], dim=0)
                k = k.repeat_interleave(reps, dim=1)
                v = v.repeat_interleave(reps, dim=1)
                qpos = torch.arange(c, kv_len, device=query.device)
                kpos = torch.arange(kv_len, device=query.device)
                mask = kpos.unsqueeze(0) <= qpos.unsqueeze(1)
                q = query[offset:offset + q_len]
                o = torch.nn.functional.scaled_dot_product_attention(
                    q.permute(1, 0, 2).unsqueeze(0), k.permute(1, 0, 2).unsqueeze(0),
                    v.permute(1, 0, 2).unsqueeze(0), attn_mask=mask, is_causal=False, scale=scale,
                )
                parts.append(o.squeeze(0).permute(1, 0, 2))
                offset += q_len
                src += n
        if not parts:
            return query
        return torch.cat(parts, dim=0)


def validate_block_size(block_size: int) -> None:
    """The pool rule of ``AttentionBackendGPU.allocate_pool`` (:502-506)."""
    if block_size <= 0 or (block_size & (block_size - 1)) != 0:
        raise RuntimeError(f"AttentionBackendB200: block_size={block_size} must be a positive power of 2.")

"""Stream-ordered host <-> device staging for a serving loop.

A decode step of a serving loop moves its inputs from pinned host memory to
the device and its output back, on side streams ordered by events, so the
copies overlap the neighbouring steps' attention.  Written with torch's
``Tensor.copy_``, ``Stream.wait_event``, ``Event.record`` and
``torch.cuda.set_stream``, that choreography costs a microsecond or more of
host time per call, several calls per step; on a slow host it becomes the
bound of the loop.  These helpers issue the same CUDA calls directly on the
raw stream and event handles (one binding call per copy, wait list or record)
and never switch torch's current stream.

They need the direct binding (``lib/_mvb_torch.so``, built by
``__graft_entry__.build()``) and raise ``RuntimeError`` without it.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _native


def _binding():
    fast = _native.fast()
    if fast is None:
        raise RuntimeError("mini_vllm_b200.staging needs lib/_mvb_torch.so: build it with __graft_entry__.build()")
    return fast


def _event_handle(event: Optional[torch.cuda.Event]) -> int:
    return 0 if event is None else int(event.cuda_event)


def stream_copy(dst: torch.Tensor, src: torch.Tensor, stream: torch.cuda.Stream, *,
                wait: Optional[torch.cuda.Event] = None, record: Optional[torch.cuda.Event] = None) -> None:
    """On ``stream``: wait for ``wait`` (if given and ever recorded), copy
    ``src`` into ``dst``, then record ``record`` (if given).

    One of the two tensors is on the GPU and the other in host memory (pinned,
    for the copy to be asynchronous); both are contiguous with the same byte
    size.  Like ``dst.copy_(src, non_blocking=True)`` on a side stream, the
    caller keeps both tensors alive until the copy is done (``record`` tells).
    """
    if dst.is_cuda == src.is_cuda:
        raise ValueError("stream_copy copies between host and device memory: exactly one tensor must be on the GPU")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("stream_copy needs contiguous tensors")
    dev = dst.device if dst.is_cuda else src.device
    if stream.device != dev:
        raise ValueError(f"stream_copy: the device tensor is on {dev} but the stream belongs to {stream.device}")
    nbytes = dst.numel() * dst.element_size()
    if nbytes != src.numel() * src.element_size():
        raise ValueError(f"stream_copy size mismatch: {nbytes} vs {src.numel() * src.element_size()} bytes")
    fast = _binding()
    rec = _event_handle(record)
    if record is not None and rec == 0:  # torch creates an event on its first record
        record.record(stream)
        rec = int(record.cuda_event)
    st = fast.stream_copy(dst.data_ptr(), src.data_ptr(), nbytes, 0 if dst.is_cuda else 1, stream.cuda_stream,
                          _event_handle(wait), rec)
    if st != 0:
        raise RuntimeError(f"stream_copy failed: CUDA error {st}")


def wait_events(stream: torch.cuda.Stream, *events: Optional[torch.cuda.Event]) -> None:
    """``stream`` waits for each event (events never recorded are skipped, as
    torch's ``Stream.wait_event`` does)."""
    st = _binding().stream_wait_events(stream.cuda_stream, [_event_handle(e) for e in events])
    if st != 0:
        raise RuntimeError(f"wait_events failed: CUDA error {st}")


def record(event: torch.cuda.Event, stream: torch.cuda.Stream) -> None:
    """Record ``event`` on ``stream``."""
    handle = int(event.cuda_event)
    if handle == 0:  # not created yet: torch creates it on this first record
        event.record(stream)
        return
    st = _binding().event_record(handle, stream.cuda_stream)
    if st != 0:
        raise RuntimeError(f"record failed: CUDA error {st}")


class CopyPlan:
    """A fixed ``stream_copy`` — the same tensors, stream and events every
    step, as a serving loop's preallocated staging buffers are — checked once;
    ``run()`` then issues it (wait, copy, record on the stream) in one binding
    call with the handles resolved, skipping the per-call checks.  The plan
    keeps its tensors and events alive."""

    __slots__ = ("_dst", "_src", "_stream", "_wait", "_record", "_args", "_wait_h", "_rec_h")

    def __init__(self, dst: torch.Tensor, src: torch.Tensor, stream: torch.cuda.Stream, *,
                 wait: Optional[torch.cuda.Event] = None, record: Optional[torch.cuda.Event] = None) -> None:
        if dst.is_cuda == src.is_cuda:
            raise ValueError("CopyPlan copies between host and device memory: exactly one tensor must be on the GPU")
        if not (dst.is_contiguous() and src.is_contiguous()):
            raise ValueError("CopyPlan needs contiguous tensors")
        dev = dst.device if dst.is_cuda else src.device
        if stream.device != dev:
            raise ValueError(f"CopyPlan: the device tensor is on {dev} but the stream belongs to {stream.device}")
        nbytes = dst.numel() * dst.element_size()
        if nbytes != src.numel() * src.element_size():
            raise ValueError(f"CopyPlan size mismatch: {nbytes} vs {src.numel() * src.element_size()} bytes")
        _binding()
        self._dst, self._src, self._stream, self._wait, self._record = dst, src, stream, wait, record
        self._args = (dst.data_ptr(), src.data_ptr(), nbytes, 0 if dst.is_cuda else 1, stream.cuda_stream)
        self._wait_h = 0
        self._rec_h = 0

    def run(self) -> None:
        """Wait for ``wait`` (once it has been recorded), copy, record ``record``."""
        if self._wait_h == 0 and self._wait is not None:
            self._wait_h = _event_handle(self._wait)  # 0 until torch creates it on a first record
        if self._rec_h == 0 and self._record is not None:
            self._rec_h = _event_handle(self._record)
            if self._rec_h == 0:  # torch creates an event on its first record
                self._record.record(self._stream)
                self._rec_h = int(self._record.cuda_event)
        st = _native.fast().stream_copy(*self._args, self._wait_h, self._rec_h)
        if st != 0:
            raise RuntimeError(f"CopyPlan.run failed: CUDA error {st}")

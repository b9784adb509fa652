"""Per-device runtime state for the wavefront kernels: workspace, error word,
stream handles and tensor checks.

PyTorch supplies device memory and the current CUDA stream; every compute step
is a libwfd_b200 launch.  The workspace (segment table, prefix, arrival
counters, split-K partials) is allocated once per device, zero-filled once, and
grown only outside CUDA-graph capture (the kernels leave it zeroed again).  A grown
workspace keeps the previous buffer allocated: graphs captured against it still
point at it, and the allocator must not hand it to anything else.
"""
from __future__ import annotations

import threading

import torch

from . import _abi

_state_lock = threading.Lock()
_ws: dict[int, tuple[torch.Tensor, int, int]] = {}   # device -> (buffer, max_items, head_dim)
_ws_retired: dict[int, list[torch.Tensor]] = {}       # device -> buffers replaced by a larger one
_err: dict[int, torch.Tensor] = {}


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return _abi.WFD_DTYPE_BF16
    if dt == torch.float32:
        return _abi.WFD_DTYPE_F32
    raise TypeError(f"wavefront kernels take bfloat16 or float32 tensors, got {dt}")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("wavefront kernels run on CUDA tensors only (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _capturing() -> bool:
    return torch.cuda.is_current_stream_capturing()


def workspace(device: torch.device, max_items: int, head_dim: int) -> tuple[torch.Tensor, int]:
    """Workspace large enough for `max_items` segments at `head_dim`."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _state_lock:
        cur = _ws.get(idx)
        if cur is not None and cur[1] >= max_items and cur[2] >= head_dim:
            return cur[0], cur[0].numel()
        if _capturing():
            raise RuntimeError("wavefront workspace must be reserved before CUDA-graph capture "
                               "(call reserve_workspace with the largest item count first)")
        lib = _abi.load()
        n_items = max(max_items, cur[1] if cur else 0, 1024)
        dh = max(head_dim, cur[2] if cur else 0, 128)
        with torch.cuda.device(idx):
            nbytes = int(lib.wfd_workspace_bytes(n_items, dh, 0))
            if nbytes <= 0:
                raise _abi.WfdError("wfd_workspace_bytes", -1, "could not size workspace")
            buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
            _abi.check(lib.wfd_workspace_init(buf.data_ptr(), nbytes, stream_ptr(device)), "wfd_workspace_init")
        if cur is not None:
            _ws_retired.setdefault(idx, []).append(cur[0])
        _ws[idx] = (buf, n_items, dh)
        return buf, nbytes


def reserve_workspace(device: torch.device, max_items: int, head_dim: int = 128) -> None:
    workspace(torch.device(device), max_items, head_dim)


def error_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _state_lock:
        e = _err.get(idx)
        if e is None:
            if _capturing():
                raise RuntimeError("wavefront error word must exist before CUDA-graph capture")
            e = torch.zeros(1, dtype=torch.int32, device=device)
            _err[idx] = e
        return e


def read_device_error(device: torch.device | None = None) -> int:
    """Synchronise and return (then clear) the device error word; raise on error."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    e = error_word(device)
    import ctypes
    h = ctypes.c_int32(0)
    status = _abi.load().wfd_read_error(e.data_ptr(), ctypes.addressof(h), stream_ptr(device))
    if status not in (_abi.WFD_OK,):
        raise _abi.WfdError("device error word", status, f"{_abi.status_string(status)}; bits=0x{h.value:x}")
    return h.value


def set_batch_invariant(on: bool) -> bool:
    """Turn the library's batch-invariant attention on or off; returns the old mode."""
    lib = _abi.load()
    old = bool(lib.wfd_get_batch_invariant())
    _abi.check(lib.wfd_set_batch_invariant(1 if on else 0), "wfd_set_batch_invariant")
    return old


class batch_invariant:
    """Context manager: batch-invariant attention inside the block."""

    def __init__(self, on: bool = True):
        self.on = on
        self.old = False

    def __enter__(self):
        self.old = set_batch_invariant(self.on)
        return self

    def __exit__(self, *exc):
        set_batch_invariant(self.old)



def test_fail_waits(on: bool) -> None:
    """Test hook: every CTA of the tcgen05 attention kernel gives up right after
    issuing its first K/V copies, as when a bounded wait runs out, and reports a
    timeout (launches built while it is on)."""
    _abi.check(_abi.load().wfd_test_fail_waits(1 if on else 0), "wfd_test_fail_waits")

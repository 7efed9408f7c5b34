"""ctypes binding of the C ABI in ``include/mt_b200.h`` (``lib/libmtb200.so``).

The product path has no fallback: if the library is missing or the device is
not an sm_100 GPU, the ops raise instead of silently running something else.
"""

from __future__ import annotations

import ctypes
import os
import threading
import time
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmtb200.so"

MT_F32, MT_F16, MT_BF16 = 0, 1, 2
_DTYPE_CODE = {torch.float32: MT_F32, torch.float16: MT_F16, torch.bfloat16: MT_BF16}

c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_float = ctypes.c_float
c_vp = ctypes.c_void_p
c_i64p = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/mt_b200.h
PROTOTYPES: dict[str, tuple[object, list[object]]] = {
    "mt_status_string": (ctypes.c_char_p, [c_int]),
    "mt_version": (c_int, []),
    "mt_built_arch": (c_int, []),
    "mt_last_error": (ctypes.c_char_p, []),
    "mt_rms_norm_fwd": (c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_i64, c_i64, c_float, c_vp]),
    "mt_rms_norm_bwd_workspace_bytes": (c_i64, [c_i64, c_i64]),
    "mt_rms_norm_bwd": (
        c_int,
        [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_i64, c_i64, c_i64, c_vp],
    ),
    "mt_rms_norm_bwd_noalloc": (
        c_int,
        [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_i64, c_i64, c_vp],
    ),
    "mt_add_rms_norm_fwd": (
        c_int,
        [c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_i64, c_i64, c_float, c_vp],
    ),
    "mt_add_rms_norm_bwd": (
        c_int,
        [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_i64, c_i64,
         c_i64, c_vp],
    ),
    "mt_add_rms_norm_bwd_dual": (
        c_int,
        [c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_int, c_vp, c_int, c_vp, c_int, c_vp, c_vp, c_int, c_vp, c_i64,
         c_i64, c_i64, c_vp],
    ),
    "mt_swiglu_gemm_fwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "mt_swiglu_gemm_bwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "mt_qkv_rope_gemm": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64,
                                 c_vp, c_vp]),
    "mt_launch_count": (c_i64, []),
    "mt_set_timing_events": (c_int, [c_vp, c_vp]),
    "mt_rope": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64p, c_i64p, c_i64p,
         c_i64p, c_i64p, c_i64p, c_int, c_vp],
    ),
    "mt_swiglu_fwd": (c_int, [c_vp, c_vp, c_vp, c_int, c_i64, c_vp]),
    "mt_swiglu_bwd": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_vp]),
    "mt_swiglu_packed_fwd": (c_int, [c_vp, c_vp, c_int, c_i64, c_i64, c_vp]),
    "mt_swiglu_packed_bwd": (c_int, [c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_vp]),
    "mt_adamw_step": (c_int, [c_vp, c_int, c_i64, c_int, c_float, c_float, c_float, c_float, c_float, c_float,
                              c_float, c_vp, c_vp]),
    "mt_debug_wait_timeout": (c_int, [c_i64, c_int, c_vp, c_vp]),
    "mt_attention_fwd_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64, c_i64]),
    "mt_attention_fwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64p, c_i64p, c_i64p, c_i64p,
         c_float, c_vp, c_i64, c_vp, c_vp],
    ),
    "mt_attention_bwd_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64, c_i64]),
    "mt_attention_bwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64p,
         c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, c_float, c_vp, c_i64, c_vp, c_vp],
    ),
    "mt_attention_rope_bwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64p,
         c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, c_i64p, c_float, c_vp, c_vp, c_i64, c_vp, c_i64, c_vp,
         c_vp],
    ),
    "mt_fused_ce_workspace_bytes": (c_i64, [c_i64, c_i64]),
    "mt_fused_ce_fwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp],
    ),
    "mt_fused_ce_bwd_workspace_bytes": (c_i64, [c_i64, c_i64, c_i64]),
    "mt_fused_ce_bwd": (
        c_int,
        [c_vp, c_vp, c_vp, c_int, c_i64, c_int, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_int, c_vp, c_int, c_vp,
         c_i64, c_vp, c_vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class B200KernelError(RuntimeError):
    """A C-ABI call returned a nonzero mt_status."""


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load ``libmtb200.so`` once and attach the prototypes; raise if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path is not None else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"B200 kernel library not found at {p}; build it with `python -m mega_trading_b200.build` "
                "(there is no fallback implementation)"
            )
        lib = ctypes.CDLL(os.fspath(p))
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(status: int, name: str) -> None:
    if status != 0:
        lib = load()
        text = lib.mt_status_string(status).decode()
        detail = lib.mt_last_error().decode()
        raise B200KernelError(f"{name} failed: {text} (status {status}){': ' + detail if detail else ''}")


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[t]
    except KeyError as exc:
        raise RuntimeError(f"unsupported dtype {t}") from exc


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def i64_array(values) -> ctypes.Array:
    arr = (ctypes.c_int64 * len(values))(*[int(v) for v in values])
    return arr


# Per-device uint32 status word for the bounded device waits.
_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def read_status(device: torch.device) -> int:
    """Return and clear the device status word (synchronises the device)."""
    t = status_word(device)
    v = int(t.item())
    if v:
        t.zero_()
    return v


# kernel ids of the status word's high half (the kKernelId constants in csrc/)
KERNEL_NAMES = {1: "attention forward", 2: "attention backward", 3: "fused cross-entropy", 4: "fused cross-entropy",
                6: "projection GEMM", 15: "wait probe"}


def describe_status(code: int) -> str:
    """Text for a nonzero device status word: which kernel gave up and where."""
    kid, site = code >> 16, code & 0xFFFF
    if site == 0xEEEE:
        return f"{KERNEL_NAMES.get(kid, f'kernel {kid}')}: a target label is out of range [0, vocab)"
    if site == 0xFFFF:
        return f"{KERNEL_NAMES.get(kid, f'kernel {kid}')}: dynamic shared memory not 1024-byte aligned"
    return f"{KERNEL_NAMES.get(kid, f'kernel {kid}')}: bounded device wait {site} gave up (status {code:#x})"


def check_status(device: torch.device) -> None:
    """Raise :class:`B200KernelError` if a kernel on ``device`` reported an error through the
    status word since the last check (synchronises the device; clears the word)."""
    v = read_status(device)
    if v:
        raise B200KernelError(f"device error reported by the sm_100a kernels: {describe_status(v)}")


class StatusMonitor:
    """Deferred check of the device status word that never stalls the launch queue.

    ``poll()`` (once per training step) queues an asynchronous copy of the word
    into pinned host memory behind the step's kernels, then inspects every earlier
    copy that the device has finished; it blocks only when more than ``depth``
    copies are outstanding.  A nonzero word raises :class:`B200KernelError` at the
    first poll after the device wrote it (at most ``depth`` steps late)."""

    def __init__(self, device: torch.device, depth: int = 2) -> None:
        self.device = device
        self.depth = max(1, int(depth))
        self.pending: list[tuple[torch.Tensor, torch.cuda.Event]] = []
        self.blocked_s = 0.0  # host seconds spent waiting for the device in poll()

    def _inspect(self, host: torch.Tensor) -> None:
        v = int(host[0])
        if v:
            self.pending.clear()
            status_word(self.device).zero_()
            raise B200KernelError(f"device error reported by the sm_100a kernels: {describe_status(v)}")

    def poll(self) -> None:
        host = torch.zeros(1, dtype=torch.int32).pin_memory()
        host.copy_(status_word(self.device), non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.pending.append((host, ev))
        while self.pending and (self.pending[0][1].query() or len(self.pending) > self.depth):
            h, e = self.pending.pop(0)
            t0 = time.perf_counter()
            e.synchronize()
            self.blocked_s += time.perf_counter() - t0
            self._inspect(h)

    def flush(self) -> None:
        """Wait for every queued copy and raise if any holds an error."""
        while self.pending:
            h, e = self.pending.pop(0)
            e.synchronize()
            self._inspect(h)


def require_cuda_sm100(t: torch.Tensor, op: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"{op} requires CUDA tensors (the B200 path has no CPU fallback)")
    major, minor = torch.cuda.get_device_capability(t.device)
    if major != 10 or minor != 0:
        raise RuntimeError(f"{op} requires an sm_100 (B200) GPU, found sm_{major}{minor}")


def launch_count() -> int:
    """Kernels the library has launched in this process (its own counter,
    ``mt_launch_count``); bench.py reports the difference over the timed region."""
    return int(load().mt_launch_count())


class KernelTimer:
    """Optional CUDA-event timing of named C-ABI calls on their launch stream."""

    def __init__(self) -> None:
        self.enabled = False
        self.events: dict[str, list[tuple[torch.cuda.Event, torch.cuda.Event]]] = {}

    def reset(self) -> None:
        self.events = {}

    def start(self, name: str, device: torch.device, main_kernel: bool = False):
        """Events around the whole call; with ``main_kernel`` also events the library records
        around the call's main kernel (mt_set_timing_events), kept as ``name + "_kernel"``."""
        if not self.enabled:
            return None
        stream = torch.cuda.current_stream(device)
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        inner = None
        if main_kernel:
            inner = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for e in inner:  # create the driver events; the library re-records them
                e.record(stream)
            _check_hook(load().mt_set_timing_events(inner[0].cuda_event, inner[1].cuda_event))
        return (name, ev, device, inner)

    def stop(self, token) -> None:
        if token is None:
            return
        name, ev, device, inner = token
        if inner is not None:
            _check_hook(load().mt_set_timing_events(None, None))
            self.events.setdefault(name + "_kernel", []).append(inner)
        end = torch.cuda.Event(enable_timing=True)
        end.record(torch.cuda.current_stream(device))
        self.events.setdefault(name, []).append((ev, end))

    def summary(self) -> dict[str, tuple[int, float]]:
        """name -> (launches, mean milliseconds); synchronises the device."""
        torch.cuda.synchronize()
        out = {}
        for name, pairs in self.events.items():
            total = sum(a.elapsed_time(b) for a, b in pairs)
            out[name] = (len(pairs), total / max(len(pairs), 1))
        return out


def _check_hook(st: int) -> None:
    if st != 0:
        raise B200KernelError(f"mt_set_timing_events failed (status {st})")


timer = KernelTimer()

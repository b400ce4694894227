"""ctypes binding of libflashgmm_sm100.so (C ABI in include/flashgmm.h).

Tensors cross the boundary as raw device pointers (``data_ptr()``), element
strides and torch's current CUDA stream handle, exactly as a cgo / JNI / N-API
binding of the same header would pass them.  There is no CPU fallback: if the
library is missing or the device is not sm_100 the call raises.
"""

from __future__ import annotations

import ctypes
import functools
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libflashgmm_sm100.so")

FGMM_VARIANT_ISO = 0
FGMM_VARIANT_DIAG = 1
FGMM_VARIANT_FULL = 2
FGMM_FLAG_ACCUMULATE = 1
FGMM_FLAG_FORCE_GENERAL = 2
FGMM_X_F32 = 0
FGMM_X_BF16 = 1

_ERRORS = {1: "invalid argument", 2: "workspace", 3: "unsupported shape",
           4: "CUDA error", 5: "unsupported device", 6: "device-side failure"}
FGMM_STATUS_RANGE = 0x10000
ERR_DEVICE_STATUS = 6   # raised by estep(check=True); not a C ABI return code

_lib = None
_lock = threading.Lock()

_c_i64 = ctypes.c_int64
_c_i32 = ctypes.c_int32
_c_ptr = ctypes.c_void_p


class FlashGMMError(RuntimeError):
    """A nonzero status returned by the C ABI."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{_ERRORS.get(code, code)}] {msg}")
        self.code = code


def load():
    """Load the shared library once; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python flash-gmm_b200/build_lib.py` "
                "(nvcc, sm_100a). There is no fallback implementation.")
        lib = ctypes.CDLL(LIB_PATH)
        est = [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr,
               _c_i64, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
               _c_ptr, ctypes.c_size_t, ctypes.c_uint, _c_ptr]
        for name in ("fgmm_estep_iso", "fgmm_estep_diag", "fgmm_estep_full"):
            f = getattr(lib, name)
            f.argtypes = est
            f.restype = ctypes.c_int
        lib.fgmm_estep_x.argtypes = [ctypes.c_int, ctypes.c_int] + est
        lib.fgmm_estep_x.restype = ctypes.c_int
        lib.fgmm_workspace_bytes.argtypes = [ctypes.c_int, _c_i64, _c_i32, _c_i32]
        lib.fgmm_workspace_bytes.restype = ctypes.c_size_t
        lib.fgmm_last_error.argtypes = []
        lib.fgmm_last_error.restype = ctypes.c_char_p
        lib.fgmm_version.argtypes = []
        lib.fgmm_version.restype = ctypes.c_int
        lib.fgmm_launch_count.argtypes = []
        lib.fgmm_launch_count.restype = ctypes.c_uint64
        lib.fgmm_set_profile_events.argtypes = [_c_ptr, _c_ptr]
        lib.fgmm_set_profile_events.restype = None
        lib.fgmm_generate_iso_rows.argtypes = [_c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32,
                                               _c_ptr, _c_i32, ctypes.c_uint64, _c_ptr]
        lib.fgmm_generate_iso_rows.restype = ctypes.c_int
        _lib = lib
        return lib


def _check(code: int):
    if code != 0:
        raise FlashGMMError(code, load().fgmm_last_error().decode(errors="replace"))


def workspace_bytes(variant: int, N: int, K: int, D: int) -> int:
    return int(load().fgmm_workspace_bytes(variant, N, K, D))


# Per-(device, stream) workspace cache: grows monotonically, reused across
# calls so a steady-state E-step loop performs no allocation.  Guarded by
# _lock (callers may run on several Python threads).  A buffer is only ever
# used in the order of its stream; when it is replaced by a larger one, the
# old buffer is marked as used by that stream (record_stream), so the caching
# allocator does not hand its memory out before the stream's queued work on
# it has finished.
_ws_cache: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    stream = torch.cuda.current_stream(device)
    key = (device.index, stream.cuda_stream)
    with _lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None:
                buf.record_stream(stream)
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
        return buf


def _f32(t: torch.Tensor, device) -> torch.Tensor:
    t = t.to(device=device)
    return t if t.dtype == torch.float32 else t.float()


def estep(variant: int, X: torch.Tensor, mu: torch.Tensor, cov: torch.Tensor,
          log_pi: torch.Tensor, *, out=None, accumulate: bool = False,
          force_general: bool = False, check: bool = False):
    """One E-step through the C ABI on torch's current stream.

    ``out`` may supply (logZ, Nk, mu_acc, sig) buffers (required when
    ``accumulate`` is set); otherwise fresh tensors are allocated, as the
    reference does on every call (flash_gmm_diag_h100.py:24-25).

    ``check=True`` waits for the call and reads the workspace's device status
    word (include/flashgmm.h): a device-side failure -- a scaled value of X
    outside fp16's range, or a bounded wait that timed out, after which the
    statistics are NaN -- raises FlashGMMError.  Without it the call stays
    asynchronous and such a failure shows only as NaN statistics.
    """
    lib = load()
    dev = X.device
    N, D = X.shape
    K = mu.shape[0]
    x_bf16 = X.dtype == torch.bfloat16   # passed as is (FGMM_X_BF16), widened exactly on read
    if not x_bf16:
        X = _f32(X, dev)
    mu = _f32(mu, dev)
    cov = _f32(cov, dev).contiguous()
    log_pi = _f32(log_pi, dev).contiguous()
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs the out= buffers to add into")
        sig_shape = (K,) if variant == FGMM_VARIANT_ISO else \
            (K, D) if variant == FGMM_VARIANT_DIAG else (K, D, D)
        out = (torch.empty(N, device=dev, dtype=torch.float32),
               torch.empty(K, device=dev, dtype=torch.float32),
               torch.empty(K, D, device=dev, dtype=torch.float32),
               torch.empty(sig_shape, device=dev, dtype=torch.float32))
    logZ, Nk, mu_acc, sig = out
    for t in out:
        if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
            raise ValueError("output buffers must be contiguous float32 CUDA tensors")
    nbytes = workspace_bytes(variant, N, K, D)
    ws = _workspace(dev, nbytes)
    flags = (FGMM_FLAG_ACCUMULATE if accumulate else 0) | \
        (FGMM_FLAG_FORCE_GENERAL if force_general else 0)
    fn = (lib.fgmm_estep_iso, lib.fgmm_estep_diag, lib.fgmm_estep_full)[variant]
    if x_bf16:
        fn = functools.partial(lib.fgmm_estep_x, variant, FGMM_X_BF16)
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        _check(fn(X.data_ptr(), X.stride(0), X.stride(1), mu.data_ptr(), mu.stride(0),
                  mu.stride(1), cov.data_ptr(), log_pi.data_ptr(), N, K, D,
                  logZ.data_ptr(), Nk.data_ptr(), mu_acc.data_ptr(), sig.data_ptr(),
                  ws.data_ptr(), ws.numel(), flags, stream))
        if check:
            status = int(ws[:4].view(torch.int32).item())  # synchronises with the stream
            if status != 0:
                what = ("a scaled value of X is outside fp16's range" if status == FGMM_STATUS_RANGE
                        else f"device status word 0x{status:x} (a bounded wait timed out)")
                raise FlashGMMError(ERR_DEVICE_STATUS, what + "; the statistics are NaN")
    return logZ, Nk, mu_acc, sig


def generate_iso_rows(X: torch.Tensor, centres: torch.Tensor, seed: int, row0: int = 0,
                      row_ids: torch.Tensor | None = None):
    """Fill X (nrows, D) with rows of the streaming mixture (see flashgmm.h)."""
    lib = load()
    assert X.is_cuda and X.is_contiguous() and X.dtype == torch.float32
    centres = centres.to(device=X.device, dtype=torch.float32).contiguous()
    ids = 0
    if row_ids is not None:
        row_ids = row_ids.to(device=X.device, dtype=torch.int64).contiguous()
        ids = row_ids.data_ptr()
    stream = torch.cuda.current_stream(X.device).cuda_stream
    with torch.cuda.device(X.device):
        _check(lib.fgmm_generate_iso_rows(X.data_ptr(), ids, row0, X.shape[0], X.shape[1],
                                          centres.data_ptr(), centres.shape[0],
                                          seed & 0xFFFFFFFFFFFFFFFF, stream))
    return X


def launch_count() -> int:
    """Kernels the library has launched in this process so far."""
    return int(load().fgmm_launch_count())


def set_profile_events(start: "torch.cuda.Event | None", stop: "torch.cuda.Event | None"):
    """Have later E-step calls on this thread record ``start``/``stop`` around
    their dominant kernel (pass None, None to stop)."""
    lib = load()
    if start is None:
        lib.fgmm_set_profile_events(None, None)
    else:
        lib.fgmm_set_profile_events(start.cuda_event, stop.cuda_event)

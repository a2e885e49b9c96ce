"""ctypes binding of libb2o.so (the C ABI declared in include/b2o.h).

The engine has no CPU fallback: every compute entry point here raises when the
shared library is missing or when no CUDA device is present.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libb2o.so"

F32 = 0
BF16 = 1
F16 = 2

c_void_p = C.c_void_p
c_int = C.c_int
c_int64 = C.c_int64
c_float = C.c_float


class AdamwTensor(C.Structure):
    _fields_ = [
        ("param", c_void_p),
        ("rem", c_void_p),
        ("grad", c_void_p),
        ("exp_avg", c_void_p),
        ("exp_avg_sq", c_void_p),
        ("ema", c_void_p),
        ("numel", c_int64),
        ("group", C.c_int32),
        ("_pad", C.c_int32),
        ("step_out", c_void_p),
    ]


class AdamwGroup(C.Structure):
    _fields_ = [
        ("lr", c_float),
        ("beta1", c_float),
        ("beta2", c_float),
        ("eps", c_float),
        ("weight_decay", c_float),
        ("lr_wd", c_float),
        ("step", c_float),
        ("cautious", C.c_int32),
        ("grad_scale", c_void_p),
    ]


class NormuonBatch(C.Structure):
    """b2o_normuon_batch: one shape batch of a multi-batch front/apply call."""
    _fields_ = [
        ("S", C.c_int32),
        ("r", C.c_int32),
        ("c", C.c_int32),
        ("shape_scale", C.c_float),
        ("grads", c_void_p),
        ("bufs", c_void_p),
        ("u", c_void_p),
        ("partial", c_void_p),
        ("o", c_void_p),
        ("rowsq", c_void_p),
        ("params", c_void_p),
        ("rems", c_void_p),
        ("emas", c_void_p),
        ("vrows", c_void_p),
        ("scratch", c_void_p),
        ("prescale", c_void_p),
        ("xscale", c_void_p),
        ("flags", c_void_p),
        ("x0_half", C.c_int32),
        ("_pad", C.c_int32),
    ]


class OrthoGroup(C.Structure):
    _fields_ = [
        ("u", c_void_p),
        ("partial", c_void_p),
        ("out", c_void_p),
        ("rowsq", c_void_p),
        ("S", C.c_int32),
        ("r", C.c_int32),
        ("c", C.c_int32),
        ("_pad", C.c_int32),
        ("xscale", c_void_p),
    ]


# name -> (restype, argtypes); mirrors include/b2o.h one to one
SIGNATURES = {
    "b2o_version": (c_int, []),
    "b2o_last_error": (c_int, [C.c_char_p, c_int]),
    "b2o_launch_count": (c_int64, []),
    "b2o_check_device_error": (c_int, [c_void_p]),
    "b2o_num_sms": (c_int, []),
    "b2o_launch_graphs": (c_int, [c_int]),
    "b2o_launch_graph_stats": (c_int, [C.POINTER(c_int64), C.POINTER(c_int64), C.POINTER(c_int64)]),
    "b2o_gemm_timing": (c_int, [c_int]),
    "b2o_gemm_timing_read": (c_int, [C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(c_int64)]),
    "b2o_adamw_step": (c_int, [C.POINTER(AdamwTensor), c_int, C.POINTER(AdamwGroup), c_int, c_int, c_int,
                               c_float, c_void_p]),
    "b2o_ema_update": (c_int, [C.POINTER(c_void_p), C.POINTER(c_void_p), C.POINTER(c_int64), c_int, c_int,
                               c_float, c_void_p]),
    "b2o_ema_copy_to_params": (c_int, [C.POINTER(c_void_p), C.POINTER(c_void_p), C.POINTER(c_int64), c_int,
                                       c_int, c_void_p]),
    "b2o_normuon_front_parts": (c_int, [c_int64]),
    "b2o_normuon_front": (c_int, [C.POINTER(c_void_p), C.POINTER(c_void_p), c_int, c_int, c_int, c_int, c_float,
                                  c_float, c_int, c_void_p, c_void_p, c_void_p]),
    "b2o_ortho_workspace_bytes": (c_int64, [c_int, c_int, c_int]),
    "b2o_orthogonalize": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, C.POINTER(c_float), c_int,
                                  C.POINTER(c_int), c_int, c_float, c_float, c_void_p, c_int64, c_void_p,
                                  c_void_p, c_void_p]),
    "b2o_ortho_workspace_bytes_multi": (c_int64, [C.POINTER(OrthoGroup), c_int]),
    "b2o_orthogonalize_multi": (c_int, [C.POINTER(OrthoGroup), c_int, c_int, C.POINTER(c_float), c_int,
                                        C.POINTER(c_int), c_int, c_float, c_float, c_void_p, c_int64, c_void_p]),
    "b2o_normuon_apply_scratch_floats": (c_int64, [c_int, c_int]),
    "b2o_normuon_apply": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, C.POINTER(c_void_p),
                                  C.POINTER(c_void_p), C.POINTER(c_void_p), C.POINTER(c_void_p), c_int, c_float,
                                  c_float, c_float, c_int, c_int, c_float, c_float, c_float, c_void_p, c_void_p]),
    "b2o_normuon_apply_static_max_floats": (c_int64, []),
    "b2o_normuon_apply_static": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, C.POINTER(c_void_p),
                                         C.POINTER(c_void_p), C.POINTER(c_void_p), C.POINTER(c_void_p), c_int,
                                         c_float, c_float, c_float, c_int, c_int, c_float, c_float, c_float,
                                         c_void_p]),
    "b2o_gemm_bf16": (c_int, [c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_int64, c_int, c_void_p,
                              c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int,
                              c_int, c_float, c_float, c_float, c_void_p, c_void_p, c_void_p]),
    "b2o_gemm": (c_int, [c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_int64, c_int, c_void_p,
                         c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_int, c_int, c_int, c_int,
                         c_int, c_int, c_float, c_float, c_float, c_void_p, c_void_p, c_void_p]),
    "b2o_gemm_bf16_simt": (c_int, [c_void_p, c_int64, c_int64, c_int, c_void_p, c_int64, c_int64, c_int,
                                   c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_int,
                                   c_int, c_int, c_float, c_float, c_float, c_void_p, c_void_p, c_void_p]),
    "b2o_normuon_front_multi": (c_int, [C.POINTER(NormuonBatch), c_int, c_int, c_float, c_float, c_int, c_void_p,
                                        c_void_p]),
    "b2o_normuon_prescale": (c_int, [C.POINTER(NormuonBatch), c_int, c_int, c_float, c_float, c_int, c_void_p,
                                     c_float, c_float, c_void_p]),
    "b2o_clip_scratch_floats": (c_int64, [C.POINTER(c_int64), c_int]),
    "b2o_clip_grad_norm": (c_int, [C.POINTER(c_void_p), C.POINTER(c_int64), C.POINTER(c_int), c_int, c_float,
                                   c_void_p, c_void_p, c_void_p]),
    "b2o_clip_scale": (c_int, [C.POINTER(c_void_p), C.POINTER(c_int64), C.POINTER(c_int), c_int, c_void_p,
                               c_void_p]),
    "b2o_normuon_apply_multi": (c_int, [C.POINTER(NormuonBatch), c_int, c_int, c_float, c_float, c_float, c_int,
                                        c_int, c_float, c_float, c_void_p]),
    "b2o_ipc_export": (c_int, [c_void_p, c_void_p, C.POINTER(C.c_uint64)]),
    "b2o_ipc_import": (c_int, [c_void_p, C.POINTER(c_void_p)]),
    "b2o_ipc_close": (c_int, [c_void_p]),
    "b2o_copy_async": (c_int, [C.POINTER(c_void_p), C.POINTER(c_void_p), C.POINTER(c_int64), c_int, c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Loads libb2o.so (building it first if this tree has nvcc and no .so)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            from . import build as _build
            _build.build()
        lib = C.CDLL(str(p))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    buf = C.create_string_buffer(1024)
    lib.b2o_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"libb2o {what} failed (status {rc}): {last_error()}")


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: the B200 engine runs on CUDA tensors only (got {t.device}); "
                           "there is no CPU fallback")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr_array(ptrs) -> C.Array:
    return (c_void_p * len(ptrs))(*[int(x) if x else None for x in ptrs])


def addr(arr) -> int | None:
    """Address of a ctypes array (for pointer fields of a struct), or None."""
    return C.addressof(arr) if arr is not None else None


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {dt}; the engine handles float32 and bfloat16")


def launch_count() -> int:
    return int(load().b2o_launch_count())


def device_error(stream: int | None = None) -> int:
    """Synchronises the stream and returns/clears the device error word."""
    lib = load()
    return int(lib.b2o_check_device_error(stream if stream is not None else stream_ptr()))


def launch_graphs(enable: bool) -> bool:
    """Turns the orthogonaliser's launch graphs on or off; returns the previous setting."""
    return bool(load().b2o_launch_graphs(1 if enable else 0))


def launch_graph_stats() -> dict:
    """Launch graphs captured, replayed and failed (failed argument sets launch directly)."""
    c, r, f = c_int64(), c_int64(), c_int64()
    load().b2o_launch_graph_stats(C.byref(c), C.byref(r), C.byref(f))
    return {"captures": c.value, "replays": r.value, "failures": f.value}


def gemm_timing(enable: bool) -> None:
    load().b2o_gemm_timing(1 if enable else 0)


def gemm_timing_read():
    """(device ms, algorithmic FLOPs, launches) of the tensor-core GEMM launches since the last read."""
    ms, fl, n = C.c_double(), C.c_double(), c_int64()
    load().b2o_gemm_timing_read(C.byref(ms), C.byref(fl), C.byref(n))
    return ms.value, fl.value, n.value


IPC_HANDLE_BYTES = 64


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(64-byte CUDA IPC handle of the allocation holding ptr, ptr's offset in it)."""
    lib = load()
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    off = C.c_uint64(0)
    check(lib.b2o_ipc_export(ptr, buf, C.byref(off)), "ipc_export")
    return buf.raw, off.value


def ipc_import(handle: bytes) -> int:
    """Maps another process's allocation into this one; returns its base pointer."""
    lib = load()
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("IPC handle must be 64 bytes")
    base = c_void_p(0)
    check(lib.b2o_ipc_import(C.create_string_buffer(handle, IPC_HANDLE_BYTES), C.byref(base)), "ipc_import")
    return base.value


def ipc_close(base: int) -> None:
    check(load().b2o_ipc_close(base), "ipc_close")


def copy_args(copies):
    """ctypes arguments of b2o_copy_async for [(dst_ptr, src_ptr, nbytes), ...]."""
    n = len(copies)
    dst = ptr_array([d for d, _, _ in copies])
    src = ptr_array([s for _, s, _ in copies])
    nb = (c_int64 * max(1, n))(*[b for _, _, b in copies])
    return dst, src, nb, n


def copy_async_args(args, stream: int) -> None:
    """Enqueues the copies prepared by copy_args on stream."""
    dst, src, nb, n = args
    check(load().b2o_copy_async(dst, src, nb, n, stream), "copy_async")


def copy_async(copies, stream: int) -> None:
    """Enqueues device-to-device copies [(dst_ptr, src_ptr, nbytes), ...] on stream."""
    copy_async_args(copy_args(copies), stream)

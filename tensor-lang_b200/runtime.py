"""ctypes binding of libtlb200.so (the C ABI declared in include/tlb200.h).

Replaces the reference's device layer: PyCUDA (``pycuda.autoinit``,
``driver.mem_alloc``, ``memcpy_htod``/``memcpy_dtoh``; tensorlang/compiler.py
lines 1472-1503) and the per-program ``ctypes.cdll.LoadLibrary`` of a
freshly nvcc-compiled ``kernel.so`` (compiler.py:1429-1476).

There is no CPU fallback: if the library or a CUDA device is missing, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_uint, c_uint64, c_void_p
from pathlib import Path

import numpy as np

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libtlb200.so"
# compiled fused-region cubins, keyed by a hash of their source; TL_JIT_DIR
# moves the cache (an empty directory gives a cold first run)
JIT_DIR = Path(os.environ.get("TL_JIT_DIR", str(PKG_DIR / "_jit")))

TL_ERR_INVALID_ARG = 1001
TL_ERR_ALIGNMENT = 1002
TL_ERR_JIT = 1003
TL_ERR_NO_NCCL = 1004
TL_ERR_NCCL = 1005
TL_ERR_TIMEOUT = 1006
TL_ERR_UNSUPPORTED = 1008

RED_SUM, RED_MEAN, RED_MAX, RED_MIN, RED_ARGMAX, RED_ARGMIN = range(6)
EPI_NONE, EPI_RELU = 0, 1


class TLCudaError(RuntimeError):
    """A libtlb200 entry point returned a non-zero status."""

    def __init__(self, code: int, msg: str, where: str = ""):
        super().__init__(f"{where}: [{code}] {msg}" if where else f"[{code}] {msg}")
        self.code = code


# (name, restype, argtypes) of every exported entry point
_SIGS = [
    ("tl_init", c_int, [c_int]),
    ("tl_device_count", c_int, [ctypes.POINTER(c_int)]),
    ("tl_device_info", c_int, [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                               ctypes.POINTER(c_int), ctypes.POINTER(c_size_t)]),
    ("tl_error_string", c_char_p, [c_int]),
    ("tl_default_stream", c_void_p, []),
    ("tl_malloc", c_int, [ctypes.POINTER(c_void_p), c_size_t, c_void_p]),
    ("tl_free", c_int, [c_void_p, c_void_p]),
    ("tl_host_alloc", c_int, [ctypes.POINTER(c_void_p), c_size_t]),
    ("tl_host_free", c_int, [c_void_p]),
    ("tl_memcpy_h2d", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("tl_memcpy_d2h", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("tl_memcpy_d2d", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("tl_memset", c_int, [c_void_p, c_int, c_size_t, c_void_p]),
    ("tl_stream_create", c_int, [ctypes.POINTER(c_void_p)]),
    ("tl_stream_create_priority", c_int, [ctypes.POINTER(c_void_p), c_int]),
    ("tl_stream_destroy", c_int, [c_void_p]),
    ("tl_stream_sync", c_int, [c_void_p]),
    ("tl_device_sync", c_int, []),
    ("tl_event_create", c_int, [ctypes.POINTER(c_void_p)]),
    ("tl_event_destroy", c_int, [c_void_p]),
    ("tl_event_record", c_int, [c_void_p, c_void_p]),
    ("tl_event_elapsed_ms", c_int, [c_void_p, c_void_p, ctypes.POINTER(c_float)]),
    ("tl_stream_wait_event", c_int, [c_void_p, c_void_p]),
    ("tl_graph_begin", c_int, [c_void_p]),
    ("tl_graph_end", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    ("tl_graph_last_stats", c_int, [ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    ("tl_graph_launch", c_int, [c_void_p, c_void_p]),
    ("tl_graph_destroy", c_int, [c_void_p]),
    ("tl_launch_counter", c_int, [ctypes.POINTER(c_uint64), c_int]),
    ("tl_jit_compile", c_int, [c_char_p, c_char_p, c_char_p, c_char_p, ctypes.POINTER(c_void_p)]),
    ("tl_jit_log", c_char_p, []),
    ("tl_jit_launch", c_int, [c_void_p, c_uint, c_uint, c_uint, ctypes.POINTER(c_void_p), c_void_p]),
    ("tl_reduce_rows", c_int, [c_int, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    ("tl_reduce_cols_scratch_bytes", c_size_t, [c_int, c_int64, c_int64]),
    ("tl_reduce_cols", c_int, [c_int, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p]),
    ("tl_reduce_cols_noalloc", c_int, [c_int, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    ("tl_reduce_full_scratch_bytes", c_size_t, [c_int, c_int64]),
    ("tl_reduce_full", c_int, [c_int, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    ("tl_softmax_rows", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    ("tl_norm_cols_scratch_bytes", c_size_t, [c_int64, c_int64]),
    ("tl_layer_norm_rows", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p]),
    ("tl_layer_norm_cols", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_void_p]),
    ("tl_batch_norm", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float,
                              c_void_p]),
    ("tl_loss_scratch_bytes", c_size_t, [c_int64]),
    ("tl_mse_loss", c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    ("tl_cross_entropy", c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p,
                                 c_void_p]),
    ("tl_softmax_backward_rows", c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int,
                                         c_void_p]),
    ("tl_ce_softmax_backward", c_int, [c_void_p, c_void_p, c_int, c_void_p, c_float, c_void_p,
                                       c_void_p, c_int64, c_int64, c_int, c_void_p]),
    ("tl_layer_norm_backward_rows", c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                            c_float, c_int, c_void_p]),
    ("tl_transpose2d", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    ("tl_slice2d", c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                           c_void_p]),
    ("tl_concat_rows", c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    ("tl_gemm", c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                        c_int64, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p]),
    ("tl_gemm_masked", c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64,
                               c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int,
                               c_void_p, c_int64, c_void_p]),
    ("tl_gemm_pairs", c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64,
                              c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p,
                              c_int, c_int, c_void_p, c_int64, c_void_p]),
    ("tl_gemm_pair_bytes", c_int64, [c_int64, c_int64, c_int]),
    ("tl_gemm_tc_plan", c_int, [c_int64, c_int64, c_int64, ctypes.POINTER(c_int)]),
    ("tl_gemm_pair_prepare", c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int,
                                     c_void_p, c_int, c_void_p]),
    ("tl_gemm_pair_colsum_scratch_bytes", ctypes.c_size_t, [c_int64, c_int64]),
    ("tl_gemm_pair_prepare_colsum", c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p, c_int,
                                            c_void_p, c_int, c_void_p, c_void_p, ctypes.c_size_t,
                                            c_void_p]),
    ("tl_gemm_uses_pairs", c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_int64, c_int64]),
    ("tl_gemm_path", c_int, [c_int, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                             c_int64, c_void_p, c_int64]),
    ("tl_gemm_force_simt", c_int, [c_int]),
    ("tl_gemm_set_scheme", c_int, [c_int, ctypes.POINTER(c_int)]),
    ("tl_gemm_set_cta_pair", c_int, [c_int, ctypes.POINTER(c_int)]),
    ("tl_gemm_set_tile_schedule", c_int, [c_int, ctypes.POINTER(c_int)]),
    ("tl_gemm_set_store_path", c_int, [c_int, ctypes.POINTER(c_int)]),
    ("tl_head_ce_ok", c_int, [c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_int64]),
    ("tl_head_ce", c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p, c_int,
                           c_void_p, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_int64, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p]),
    ("tl_device_error", c_int, [ctypes.POINTER(c_int), c_int]),
    ("tl_nccl_unique_id", c_int, [ctypes.c_char_p]),
    ("tl_nccl_comm_init", c_int, [ctypes.POINTER(c_void_p), c_int, ctypes.c_char_p, c_int, c_int]),
    ("tl_nccl_allreduce_sum", c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    ("tl_nccl_wait", c_int, [c_void_p, c_void_p, c_int]),
    ("tl_nccl_comm_destroy", c_int, [c_void_p]),
    ("tl_nccl_comm_abort", c_int, [c_void_p]),
]

EXPORTED = [s[0] for s in _SIGS]

_lib = None
_lib_lock = threading.Lock()


def load_library(path: os.PathLike | None = None) -> ctypes.CDLL:
    """Load libtlb200.so (built by ``__graft_entry__.build()``); raise if absent."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"{p} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
        lib = ctypes.CDLL(str(p))
        for name, res, args in _SIGS:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load_library()


def check(status: int, where: str = "") -> None:
    if status:
        l = lib()
        msg = l.tl_error_string(status).decode()
        if status == TL_ERR_JIT:
            log = l.tl_jit_log()
            if log:
                msg += "\n" + log.decode(errors="replace")
        raise TLCudaError(status, msg, where)


# ---------------------------------------------------------------------------
# device, buffers
# ---------------------------------------------------------------------------

class Device:
    """One CUDA device with the library's stream and memory pool."""

    _instances: dict = {}

    def __init__(self, index: int = 0):
        L = lib()
        n = c_int(0)
        L.tl_device_count(ctypes.byref(n))
        if n.value <= index:
            raise RuntimeError(f"no CUDA device {index} (found {n.value}); libtlb200 has no CPU path")
        check(L.tl_init(index), "tl_init")
        self.index = index
        self.stream = c_void_p(L.tl_default_stream())
        sms, maj, mnr, mem = c_int(), c_int(), c_int(), c_size_t()
        check(L.tl_device_info(index, ctypes.byref(sms), ctypes.byref(maj), ctypes.byref(mnr),
                               ctypes.byref(mem)))
        self.sm_count, self.cc = sms.value, (maj.value, mnr.value)
        self.total_mem = mem.value

    @classmethod
    def get(cls, index: int = 0) -> "Device":
        if index not in cls._instances:
            cls._instances[index] = Device(index)
        dev = cls._instances[index]
        check(lib().tl_init(index), "tl_init")  # makes it current
        return dev

    def sync(self):
        check(lib().tl_stream_sync(self.stream), "tl_stream_sync")


class DeviceBuffer:
    """A float32 device allocation from the stream-ordered pool."""

    __slots__ = ("ptr", "nbytes", "shape", "dev", "_owned")

    def __init__(self, dev: Device, shape, zero: bool = False):
        self.dev = dev
        self.shape = tuple(int(d) for d in shape)
        n = int(np.prod(self.shape)) if self.shape else 1
        self.nbytes = max(4 * n, 4)
        p = c_void_p()
        check(lib().tl_malloc(ctypes.byref(p), self.nbytes, dev.stream), "tl_malloc")
        self.ptr = p.value
        self._owned = True
        if zero:
            self.zero()

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @classmethod
    def view(cls, parent: "DeviceBuffer", offset_elems: int, shape) -> "DeviceBuffer":
        """A non-owning float32 view into ``parent`` starting at ``offset_elems``."""
        v = cls.__new__(cls)
        v.dev = parent.dev
        v.shape = tuple(int(d) for d in shape)
        n = int(np.prod(v.shape)) if v.shape else 1
        v.nbytes = max(4 * n, 4)
        if offset_elems + n > parent.size:
            raise ValueError("view exceeds its parent buffer")
        v.ptr = parent.ptr + 4 * int(offset_elems)
        v._owned = False
        return v

    def zero(self):
        check(lib().tl_memset(self.ptr, 0, self.nbytes, self.dev.stream), "tl_memset")

    def upload(self, arr: np.ndarray):
        a = np.ascontiguousarray(arr, dtype=np.float32)
        if a.nbytes != self.size * 4:
            raise ValueError(f"upload of {a.shape} into buffer of shape {self.shape}")
        check(lib().tl_memcpy_h2d(self.ptr, a.ctypes.data, a.nbytes, self.dev.stream), "h2d")
        self.dev.sync()  # the host array may be freed once we return

    def download(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=np.float32)
        check(lib().tl_memcpy_d2h(out.ctypes.data, self.ptr, out.nbytes, self.dev.stream), "d2h")
        self.dev.sync()
        return out

    def copy_from(self, other: "DeviceBuffer"):
        check(lib().tl_memcpy_d2d(self.ptr, other.ptr, min(self.nbytes, other.nbytes),
                                  self.dev.stream), "d2d")

    def free(self):
        if self._owned and self.ptr:
            lib().tl_free(self.ptr, self.dev.stream)
        self.ptr = None
        self._owned = False

    def __del__(self):
        try:
            if self._owned and self.ptr and _lib is not None:
                _lib.tl_free(self.ptr, self.dev.stream)
        except Exception:
            pass


class PinnedHost:
    """Page-locked host staging buffer (for timed host<->device copies)."""

    def __init__(self, nbytes: int):
        p = c_void_p()
        check(lib().tl_host_alloc(ctypes.byref(p), nbytes), "tl_host_alloc")
        self.ptr, self.nbytes = p.value, nbytes

    def array(self, shape) -> np.ndarray:
        n = int(np.prod(shape))
        buf = (ctypes.c_float * n).from_address(self.ptr)
        return np.frombuffer(buf, dtype=np.float32, count=n).reshape(shape)

    def free(self):
        if self.ptr:
            lib().tl_host_free(self.ptr)
            self.ptr = None


class Event:
    def __init__(self):
        p = c_void_p()
        check(lib().tl_event_create(ctypes.byref(p)), "event")
        self.ptr = p.value

    def record(self, stream):
        check(lib().tl_event_record(self.ptr, stream), "event_record")

    def elapsed_ms(self, end: "Event") -> float:
        ms = c_float()
        check(lib().tl_event_elapsed_ms(self.ptr, end.ptr, ctypes.byref(ms)), "elapsed")
        return float(ms.value)

    def __del__(self):
        try:
            if _lib is not None and self.ptr:
                _lib.tl_event_destroy(self.ptr)
        except Exception:
            pass


def launch_count(reset: bool = False) -> int:
    c = c_uint64()
    lib().tl_launch_counter(ctypes.byref(c), 1 if reset else 0)
    return int(c.value)

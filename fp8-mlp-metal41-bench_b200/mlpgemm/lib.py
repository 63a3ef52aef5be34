"""ctypes binding of libgemm.so (the C ABI declared in include/mlpgemm.h).

The library is the product: there is no fallback.  If libgemm.so is missing
or cannot be loaded, every entry point here raises GemmError.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("GEMM_LIB", os.path.join(PKG_ROOT, "libgemm.so"))

GEMM_OK, GEMM_ERR_ARGS, GEMM_ERR_INIT, GEMM_ERR_MISMATCH, GEMM_ERR_CUDA, GEMM_ERR_TIMEOUT = range(6)

# Every symbol the header declares (tests check the library exports them all).
EXPORTS = [
    "gemm_init", "gemm_device_count", "gemm_device_info", "gemm_last_error", "gemm_version",
    "gemm_dtype_name", "gemm_kernel_name", "gemm_num_tiles", "gemm_tile_name",
    "gemm_tile_index", "gemm_tile_supported", "gemm_default_tile", "gemm_check_layout",
    "gemm_workspace_size", "gemm_alloc", "gemm_free", "gemm_memset", "gemm_h2d", "gemm_d2h",
    "gemm_host_alloc", "gemm_host_free", "gemm_run", "gemm_sync", "gemm_time",
    "gemm_time_e2e", "gemm_time_e2e_pipelined", "gemm_launches_per_run", "gemm_peak_probe",
    "gemm_read_probe",
    "gemm_run_noalloc",
    "gemm_quantize",
    "gemm_run_gather", "gemm_gather_supported", "gemm_peer_alloc", "gemm_peer_open", "gemm_peer_close",
]

MAX_PEERS = 7            # GEMM_MAX_PEERS
PEER_HANDLE_BYTES = 64   # GEMM_PEER_HANDLE_BYTES

# quantiser formats (GEMM_Q_* in include/mlpgemm.h)
Q_E4M3_REF, Q_E4M3, Q_E2M1, Q_MXFP4, Q_MXFP8 = 0, 1, 2, 3, 4


class GemmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def build() -> str:
    """Compile libgemm.so in-tree with the package Makefile (nvcc, sm_100a)."""
    subprocess.run(["make", "-s", "-C", PKG_ROOT], check=True)
    return LIB_PATH


def _declare(L):
    c_int, c_size, vp, c_char_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p
    vpp = ctypes.POINTER(ctypes.c_void_p)
    sig = {
        "gemm_init": (c_int, [c_int]),
        "gemm_device_count": (c_int, []),
        "gemm_device_info": (c_int, [c_int, c_char_p, c_int, c_char_p, c_int, ctypes.POINTER(c_int)]),
        "gemm_last_error": (c_char_p, []),
        "gemm_version": (c_char_p, []),
        "gemm_dtype_name": (c_char_p, [c_int]),
        "gemm_kernel_name": (c_char_p, [c_int]),
        "gemm_num_tiles": (c_int, []),
        "gemm_tile_name": (c_char_p, [c_int]),
        "gemm_tile_index": (c_int, [c_char_p]),
        "gemm_tile_supported": (c_int, [c_int, c_int, c_int, c_int, c_int]),
        "gemm_default_tile": (c_int, [c_int, c_int, c_int, c_int]),
        "gemm_check_layout": (c_int, [c_int, c_int, c_int, c_int]),
        "gemm_workspace_size": (c_size, [c_int, c_int, c_int, c_int, c_int]),
        "gemm_alloc": (vp, [c_int, c_size]),
        "gemm_free": (c_int, [c_int, vp]),
        "gemm_memset": (c_int, [c_int, vp, c_int, c_size]),
        "gemm_h2d": (c_int, [c_int, vp, vp, c_size]),
        "gemm_d2h": (c_int, [c_int, vp, vp, c_size]),
        "gemm_host_alloc": (vp, [c_size]),
        "gemm_host_free": (c_int, [vp]),
        "gemm_run": (c_int, [c_int, c_int, c_int, vp, vp, vp, c_int, c_int, c_int, vp, vp, vp,
                             c_size, vp]),
        "gemm_sync": (c_int, [c_int, vp]),
        "gemm_time": (c_int, [c_int, c_int, c_int, vp, vpp, vp, c_int, c_int, c_int, vp, vpp,
                              c_int, vp, c_size, c_int, c_int, vp, c_size,
                              ctypes.POINTER(ctypes.c_float)]),
        "gemm_time_e2e": (c_int, [c_int, c_int, c_int, vp, vp, vp, vp, vp, c_int, c_int, c_int,
                                  vp, vp, vp, vp, c_size, c_int, c_int,
                                  ctypes.POINTER(ctypes.c_float)]),
        "gemm_time_e2e_pipelined": (c_int, [c_int, c_int, c_int, vp, vp, vp, vp, vp, vp, vp, c_int, c_int,
                                            c_int, vp, vp, vp, vp, vp, c_size, c_int, c_int,
                                            ctypes.POINTER(ctypes.c_float)]),
        "gemm_launches_per_run": (c_int, [c_int, c_int, c_int, c_int, c_int]),
        "gemm_peak_probe": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(ctypes.c_double)]),
        "gemm_read_probe": (c_int, [c_int, vp, c_size, c_int, c_int, vp, c_size,
                                    ctypes.POINTER(ctypes.c_float)]),
        "gemm_run_noalloc": (c_int, [c_int, c_int, c_int, vp, vp, vp, c_int, c_int, c_int, vp, vp,
                                     vp]),
        "gemm_quantize": (c_int, [c_int, c_int, vp, vp, vp, ctypes.c_long, ctypes.c_long, vp]),
        "gemm_run_gather": (c_int, [c_int, c_int, c_int, vp, vp, vp, c_int, c_int, c_int, vp, vp, vp,
                                    c_size, vpp, c_int, vp]),
        "gemm_gather_supported": (c_int, [c_int, c_int]),
        "gemm_peer_alloc": (c_int, [c_int, c_size, vpp, vp]),
        "gemm_peer_open": (c_int, [c_int, vp, vpp]),
        "gemm_peer_close": (c_int, [c_int, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> ctypes.CDLL:
    """Load libgemm.so (once).  Raises GemmError(GEMM_ERR_INIT) if it is absent."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise GemmError(GEMM_ERR_INIT,
                                f"{LIB_PATH} not found: build it with `make -C {PKG_ROOT}`")
            try:
                L = ctypes.CDLL(LIB_PATH)
            except OSError as e:
                raise GemmError(GEMM_ERR_INIT, f"cannot load {LIB_PATH}: {e}") from e
            _declare(L)
            _lib = L
    return _lib


def last_error() -> str:
    return lib().gemm_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    if rc != GEMM_OK:
        raise GemmError(rc, f"{what}: {last_error()}" if what else last_error())


def _s(b: bytes) -> str:
    return b.decode() if b is not None else ""


# ---- thin wrappers -------------------------------------------------------------
def init(device: int = 0) -> None:
    check(lib().gemm_init(device), f"gemm_init({device})")


def device_count() -> int:
    return lib().gemm_device_count()


def device_info(device: int = 0):
    name = ctypes.create_string_buffer(256)
    arch = ctypes.create_string_buffer(64)
    sms = ctypes.c_int(0)
    check(lib().gemm_device_info(device, name, 256, arch, 64, ctypes.byref(sms)), "device info")
    return name.value.decode(), arch.value.decode(), sms.value


def version() -> str:
    return _s(lib().gemm_version())


def tile_names() -> list[str]:
    L = lib()
    return [_s(L.gemm_tile_name(i)) for i in range(L.gemm_num_tiles())]


def tile_index(name: str) -> int:
    return lib().gemm_tile_index(name.encode())


def tile_supported(dtype: int, tile: int, N: int, K: int, M: int) -> bool:
    return bool(lib().gemm_tile_supported(dtype, tile, N, K, M))


def default_tile(dtype: int, N: int, K: int, M: int) -> int:
    return lib().gemm_default_tile(dtype, N, K, M)


def workspace_size(dtype: int, tile: int, N: int, K: int, M: int) -> int:
    return lib().gemm_workspace_size(dtype, tile, N, K, M)


def launches_per_run(dtype: int, tile: int, N: int, K: int, M: int) -> int:
    return lib().gemm_launches_per_run(dtype, tile, N, K, M)


class DeviceBuffer:
    """Device memory from gemm_alloc (freed on close / garbage collection)."""

    def __init__(self, device: int, nbytes: int):
        self.device = device
        self.nbytes = int(nbytes)
        p = lib().gemm_alloc(device, max(self.nbytes, 1))
        if not p:
            raise GemmError(GEMM_ERR_CUDA, f"gemm_alloc({nbytes}): {last_error()}")
        self.ptr = p

    def upload(self, arr) -> "DeviceBuffer":
        import numpy as np
        a = np.ascontiguousarray(arr)
        assert a.nbytes <= self.nbytes, (a.nbytes, self.nbytes)
        check(lib().gemm_h2d(self.device, self.ptr, a.ctypes.data_as(ctypes.c_void_p), a.nbytes), "h2d")
        return self

    def download(self, arr):
        import numpy as np
        assert arr.flags["C_CONTIGUOUS"] and arr.nbytes <= self.nbytes
        check(lib().gemm_d2h(self.device, arr.ctypes.data_as(ctypes.c_void_p), self.ptr, arr.nbytes),
              "d2h")
        return arr

    def zero(self) -> "DeviceBuffer":
        check(lib().gemm_memset(self.device, self.ptr, 0, self.nbytes), "memset")
        return self

    def close(self):
        if getattr(self, "ptr", None):
            try:
                lib().gemm_free(self.device, self.ptr)
            finally:
                self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def as_ptr(x):
    """Device pointer of a DeviceBuffer, a torch tensor, an int or None."""
    if x is None:
        return None
    if isinstance(x, DeviceBuffer):
        return x.ptr
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    return int(x)


def run(device, dtype, tile, X, W, Y, N, K, M, xscale=None, wscale=None, workspace=None,
        workspace_bytes=0, stream=None) -> None:
    check(lib().gemm_run(device, dtype, tile, as_ptr(X), as_ptr(W), as_ptr(Y), N, K, M,
                         as_ptr(xscale), as_ptr(wscale), as_ptr(workspace), int(workspace_bytes),
                         as_ptr(stream)), "gemm_run")


def run_noalloc(device, dtype, ksplit, X, W, Y, N, K, M, xscale=None, wscale=None,
                stream=None) -> None:
    """Thin-row GEMM whose split-K scratch is the library's fixed device array
    (no allocation by the library or the caller; see gemm_run_noalloc)."""
    check(lib().gemm_run_noalloc(device, dtype, ksplit, as_ptr(X), as_ptr(W), as_ptr(Y), N, K, M,
                                 as_ptr(xscale), as_ptr(wscale), as_ptr(stream)),
          "gemm_run_noalloc")


def run_gather(device, dtype, tile, X, W, Y, N, K, M, xscale=None, wscale=None, workspace=None,
               workspace_bytes=0, peers=(), stream=None) -> None:
    """gemm_run whose epilogue also stores Y at the same offset from every
    pointer of `peers` (other GPUs' Y buffers mapped with peer_open)."""
    arr = (ctypes.c_void_p * max(1, len(peers)))(*[as_ptr(q) for q in peers])
    check(lib().gemm_run_gather(device, dtype, tile, as_ptr(X), as_ptr(W), as_ptr(Y), N, K, M,
                                as_ptr(xscale), as_ptr(wscale), as_ptr(workspace), int(workspace_bytes),
                                arr, len(peers), as_ptr(stream)), "gemm_run_gather")


def gather_supported(dtype: int, tile: int) -> bool:
    return bool(lib().gemm_gather_supported(dtype, tile))


def peer_alloc(device: int, nbytes: int):
    """(device pointer, IPC handle bytes) of a buffer other processes can map."""
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
    check(lib().gemm_peer_alloc(device, int(nbytes), ctypes.byref(ptr), h), "gemm_peer_alloc")
    return int(ptr.value), bytes(h.raw)


def peer_open(device: int, handle: bytes) -> int:
    assert len(handle) == PEER_HANDLE_BYTES
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(bytes(handle), PEER_HANDLE_BYTES)
    check(lib().gemm_peer_open(device, h, ctypes.byref(ptr)), "gemm_peer_open")
    return int(ptr.value)


def peer_close(device: int, ptr: int) -> None:
    check(lib().gemm_peer_close(device, ctypes.c_void_p(ptr)), "gemm_peer_close")


def free(device: int, ptr: int) -> None:
    check(lib().gemm_free(device, ctypes.c_void_p(ptr)), "gemm_free")


def sync(device: int = 0, stream=None) -> None:
    check(lib().gemm_sync(device, as_ptr(stream)), "gemm_sync")


def time(device, dtype, tile, X, Ws, Y, N, K, M, xscale=None, wscales=None, workspace=None,
         workspace_bytes=0, warmup=5, iters=100, flush=None, flush_bytes=0):
    """Per-iteration CUDA-event times (ms) of `iters` back-to-back GEMMs."""
    Ws = list(Ws) if isinstance(Ws, (list, tuple)) else [Ws]
    nrot = len(Ws)
    warr = (ctypes.c_void_p * nrot)(*[as_ptr(w) for w in Ws])
    if wscales is None:
        sarr = None
    else:
        wscales = list(wscales) if isinstance(wscales, (list, tuple)) else [wscales]
        assert len(wscales) == nrot
        sarr = (ctypes.c_void_p * nrot)(*[as_ptr(s) for s in wscales])
    out = (ctypes.c_float * iters)()
    check(lib().gemm_time(device, dtype, tile, as_ptr(X), warr, as_ptr(Y), N, K, M, as_ptr(xscale),
                          sarr, nrot, as_ptr(workspace), int(workspace_bytes), warmup, iters,
                          as_ptr(flush), int(flush_bytes), out), "gemm_time")
    return list(out)


def time_e2e(device, dtype, tile, hX, dX, dW, dY, hY, N, K, M, hxscale=None, dxscale=None,
             dwscale=None, workspace=None, workspace_bytes=0, warmup=3, iters=10):
    out = (ctypes.c_float * iters)()
    check(lib().gemm_time_e2e(device, dtype, tile, as_ptr(hX), as_ptr(dX), as_ptr(dW), as_ptr(dY),
                              as_ptr(hY), N, K, M, as_ptr(hxscale), as_ptr(dxscale),
                              as_ptr(dwscale), as_ptr(workspace), int(workspace_bytes), warmup,
                              iters, out), "gemm_time_e2e")
    return list(out)


def time_e2e_pipelined(device, dtype, tile, hX, dX, dW, dY, hY, N, K, M, hxscale=None, dxscale=(None, None),
                       dwscale=None, workspace=None, workspace_bytes=0, warmup=3, iters=10) -> float:
    """Total ms of `iters` end-to-end steps overlapped two deep; dX, dY (and
    dxscale) are pairs of device buffers used in turn."""
    out = ctypes.c_float(0.0)
    check(lib().gemm_time_e2e_pipelined(device, dtype, tile, as_ptr(hX), as_ptr(dX[0]), as_ptr(dX[1]),
                                        as_ptr(dW), as_ptr(dY[0]), as_ptr(dY[1]), as_ptr(hY), N, K, M,
                                        as_ptr(hxscale), as_ptr(dxscale[0]), as_ptr(dxscale[1]),
                                        as_ptr(dwscale), as_ptr(workspace), int(workspace_bytes), warmup,
                                        iters, ctypes.byref(out)), "gemm_time_e2e_pipelined")
    return out.value


def peak_probe(device: int, kind: int, reps: int = 4096, iters: int = 10) -> float:
    v = ctypes.c_double(0.0)
    check(lib().gemm_peak_probe(device, kind, reps, iters, ctypes.byref(v)), "gemm_peak_probe")
    return v.value


def read_probe(device: int, buf, nbytes: int, warmup: int = 3, iters: int = 20, flush=None,
               flush_bytes: int = 0) -> list:
    """CUDA-event times (ms) of a plain streaming read of `nbytes` of `buf`."""
    out = (ctypes.c_float * iters)()
    check(lib().gemm_read_probe(device, as_ptr(buf), int(nbytes), warmup, iters, as_ptr(flush),
                                int(flush_bytes), out), "gemm_read_probe")
    return list(out)


def quantize(device, fmt, src, dst, scales=None, rows=1, cols=1, stream=None) -> None:
    """f32 [rows, cols] on the device -> a GEMM_Q_* format in `dst` (+ UE8M0 `scales`)."""
    check(lib().gemm_quantize(device, fmt, as_ptr(src), as_ptr(dst), as_ptr(scales), int(rows), int(cols),
                              as_ptr(stream)), "gemm_quantize")

"""B200 (sm_100a) MXFP8 x BF16 GEMM and MXFP8 codec.

Python binding of ``libmpk.so`` (C ABI in ``include/mpk.h``) through ctypes.
The function names follow the reference project's C++ API
(chcoliang/mix_precision_kernel ``include/gemm_kernels.h:12-16`` and
``include/mxfp8_utils.h:34-47``) with the same argument order and meaning:

    gemm_fp8_tensorcore(A_data, A_scales, B, C_data, C_scales, D_data, D_scales, M, N, K, stream)
    mxfp8_quantize_gpu(input, data, scales, M, K, stream)
    mxfp8_dequantize_gpu(data, scales, output, M, K, stream)
    mxfp8_quantize_host(input, data, scales, M, K)
    mxfp8_dequantize_host(data, scales, output, M, K)

Arguments are torch CUDA tensors (or raw device addresses as ints) for the GPU
functions and numpy arrays for the host functions.  Where the reference calls
``exit()`` on a CUDA error, these raise :class:`MpkError`.  There is no CPU
fallback: if ``libmpk.so`` is missing the import of any GPU function fails.
"""
from __future__ import annotations

import ctypes
import os
import threading

__all__ = [
    "MpkError", "lib", "library_path",
    "gemm_fp8_tensorcore", "mxfp8_quantize_gpu", "mxfp8_dequantize_gpu",
    "mxfp8_quantize_host", "mxfp8_dequantize_host",
    "gemm_fp8_tensorcore_ws", "gemm_workspace_size", "release_workspace_pool",
    "mxfp8_dequantize_bf16_gpu", "mxfp8_quantize_bf16_gpu", "gemm_fp8_tensorcore_gather", "peer_barrier",
    "mxfp8_quantize_cols_gpu", "mxfp8_quantize_bf16_cols_gpu", "quantize_cols",
    "ipc_export", "ipc_import", "ipc_close",
    "gemm_fp8_tensorcore_noalloc", "NOALLOC_SCRATCH_BYTES",
    "gemm", "quantize", "dequantize", "device_status", "set_wait_timeout_ns", "wait_selftest",
    "set_gemm_schedule", "gemm_schedule", "gemm_plan", "SCHEDULE_AUTO", "SCHEDULE_TILES", "SCHEDULE_STREAM_K",
    "gemm_path", "PATH_PREPASS", "PATH_ONCHIP",
    "MX_BLOCK", "nblk",
]

MX_BLOCK = 32
_PKG = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_PKG, "_lib", "libmpk.so")
_lock = threading.Lock()
_lib = None

MPK_SUCCESS = 0
MPK_ERR_INVALID_VALUE = 1001
MPK_ERR_UNSUPPORTED = 1002
MPK_ERR_MISALIGNED = 1003
MPK_ERR_DEVICE_TIMEOUT = 1004
MPK_ERR_ARCH = 1005
MPK_ERR_DRIVER = 1006

# GEMM work schedules (MPK_SCHEDULE_* in include/mpk.h)
SCHEDULE_AUTO = 0
SCHEDULE_TILES = 1
SCHEDULE_STREAM_K = 2
# Kernel paths of the default GEMM entry point (MPK_PATH_* in include/mpk.h)
PATH_PREPASS = 0
PATH_ONCHIP = 1


class MpkError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"mpk status {status}: {message}")
        self.status = status


def nblk(cols: int) -> int:
    return (cols + MX_BLOCK - 1) // MX_BLOCK


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load libmpk.so (built in-tree by ``mix_precision_kernel_b200.build``)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise ImportError(
                    f"{_LIB_PATH} is missing: build it with `python -m mix_precision_kernel_b200.build`")
            L = ctypes.CDLL(_LIB_PATH)
            vp, ci, u8p = ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p
            L.mpk_gemm_mxfp8_bf16.argtypes = [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, vp]
            L.mpk_gemm_mxfp8_bf16_ws.argtypes = [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, vp,
                                                 ctypes.c_size_t, vp]
            L.mpk_gemm_workspace_size.argtypes = [ci, ci, ci, ctypes.POINTER(ctypes.c_size_t)]
            L.mpk_release_workspace_pool.argtypes = []
            L.mpk_gemm_mxfp8_bf16_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, vp]
            L.mpk_mxfp8_quantize.argtypes = [vp, vp, vp, ci, ci, vp]
            L.mpk_mxfp8_dequantize.argtypes = [vp, vp, vp, ci, ci, vp]
            L.mpk_mxfp8_dequantize_bf16.argtypes = [vp, vp, vp, ci, ci, vp]
            L.mpk_mxfp8_quantize_bf16.argtypes = [vp, vp, vp, ci, ci, vp]
            L.mpk_mxfp8_quantize_cols.argtypes = [vp, vp, vp, ci, ci, vp]
            L.mpk_mxfp8_quantize_bf16_cols.argtypes = [vp, vp, vp, ci, ci, vp]
            L.mpk_gemm_mxfp8_bf16_gather.argtypes = [vp, vp, vp, vp, vp, ci, ci, ci, ctypes.c_int64,
                                                     ctypes.c_int64, ci, ci, vp, vp, ci, vp, ctypes.c_size_t,
                                                     vp]
            L.mpk_peer_barrier.argtypes = [vp, ci, ci, ctypes.c_uint32, vp]
            L.mpk_ipc_export.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
            L.mpk_ipc_import.argtypes = [vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]
            L.mpk_ipc_close.argtypes = [vp]
            L.mpk_mxfp8_quantize_host.argtypes = [vp, u8p, u8p, ci, ci]
            L.mpk_mxfp8_dequantize_host.argtypes = [u8p, u8p, vp, ci, ci]
            L.mpk_device_status.argtypes = [ctypes.POINTER(ci)]
            L.mpk_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
            L.mpk_wait_selftest.argtypes = [ctypes.c_uint64, vp]
            L.mpk_status_string.argtypes = [ci]
            L.mpk_status_string.restype = ctypes.c_char_p
            L.mpk_last_error.argtypes = []
            L.mpk_last_error.restype = ctypes.c_char_p
            L.mpk_last_error_string.argtypes = []
            L.mpk_last_error_string.restype = ctypes.c_char_p
            L.mpk_set_gemm_schedule.argtypes = [ci]
            L.mpk_gemm_schedule.argtypes = []
            ip = ctypes.POINTER(ci)
            L.mpk_gemm_plan.argtypes = [ci, ci, ci, ip, ip, ip]
            L.mpk_gemm_path.argtypes = [vp, vp, ci, ci, ci, ip]
            for f in ("mpk_gemm_mxfp8_bf16", "mpk_gemm_mxfp8_bf16_ws", "mpk_gemm_workspace_size",
                      "mpk_release_workspace_pool", "mpk_mxfp8_quantize", "mpk_mxfp8_dequantize",
                      "mpk_mxfp8_dequantize_bf16", "mpk_gemm_mxfp8_bf16_noalloc",
                      "mpk_mxfp8_quantize_bf16", "mpk_gemm_mxfp8_bf16_gather", "mpk_peer_barrier",
                      "mpk_mxfp8_quantize_cols", "mpk_mxfp8_quantize_bf16_cols",
                      "mpk_ipc_export", "mpk_ipc_import", "mpk_ipc_close",
                      "mpk_mxfp8_quantize_host", "mpk_mxfp8_dequantize_host", "mpk_device_status",
                      "mpk_set_wait_timeout_ns", "mpk_wait_selftest", "mpk_version",
                      "mpk_set_gemm_schedule", "mpk_gemm_schedule", "mpk_gemm_plan", "mpk_gemm_path"):
                getattr(L, f).restype = ci
            _lib = L
    return _lib


def _check(status: int) -> None:
    if status != MPK_SUCCESS:
        L = lib()
        detail = (L.mpk_last_error_string() or b"").decode(errors="replace")
        msg = L.mpk_status_string(status).decode(errors="replace")
        raise MpkError(status, f"{msg}; {detail}" if detail else msg)


def _addr(t) -> int | None:
    """Device address of a torch tensor, an int address, or None."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(stream, *tensors) -> int | None:
    if stream is None:
        for t in tensors:
            if t is not None and not isinstance(t, int) and getattr(t, "is_cuda", False):
                import torch
                return torch.cuda.current_stream(t.device).cuda_stream
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _np_ptr(a):
    import numpy as np
    assert isinstance(a, np.ndarray) and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---------------------------------------------------------------------------
# Reference-named entry points
# ---------------------------------------------------------------------------

def gemm_fp8_tensorcore(A_data, A_scales, B, C_data, C_scales, D_data, D_scales,
                        M: int, N: int, K: int, stream=None) -> None:
    """D = A*B + C (MXFP8 A, BF16 B [K][N], MXFP8 C/D along N).  C may be None."""
    s = _stream(stream, A_data, D_data)
    _check(lib().mpk_gemm_mxfp8_bf16(_addr(A_data), _addr(A_scales), _addr(B), _addr(C_data),
                                     _addr(C_scales), _addr(D_data), _addr(D_scales), M, N, K, s))


def gemm_workspace_size(M: int, N: int, K: int) -> int:
    n = ctypes.c_size_t(0)
    _check(lib().mpk_gemm_workspace_size(M, N, K, ctypes.byref(n)))
    return n.value


def _nbytes(buf, nbytes):
    """Size of a workspace given as a tensor, or as a raw address plus its size."""
    if buf is None:
        return 0
    if isinstance(buf, int):
        if nbytes is None:
            raise ValueError("a workspace given as a raw address needs workspace_bytes")
        return int(nbytes)
    return buf.numel() * buf.element_size()


def gemm_fp8_tensorcore_ws(A_data, A_scales, B, C_data, C_scales, D_data, D_scales,
                           M: int, N: int, K: int, workspace, stream=None,
                           workspace_bytes: int | None = None) -> None:
    """gemm_fp8_tensorcore with the A operand dequantized into a caller workspace
    (a uint8 CUDA tensor of at least gemm_workspace_size(M, N, K) bytes, or a raw
    device address with workspace_bytes), or, with workspace=None, converted on chip
    by the GEMM kernel itself."""
    s = _stream(stream, A_data, D_data)
    nbytes = _nbytes(workspace, workspace_bytes)
    _check(lib().mpk_gemm_mxfp8_bf16_ws(_addr(A_data), _addr(A_scales), _addr(B), _addr(C_data),
                                        _addr(C_scales), _addr(D_data), _addr(D_scales), M, N, K,
                                        _addr(workspace), nbytes, s))


NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024  # MPK_NOALLOC_SCRATCH_BYTES in include/mpk.h


def gemm_fp8_tensorcore_noalloc(A_data, A_scales, B, C_data, C_scales, D_data, D_scales,
                                M: int, N: int, K: int, stream=None) -> None:
    """gemm_fp8_tensorcore for callers that may not allocate device memory: the A
    workspace is the library's fixed per-device array (M*K*2 <= NOALLOC_SCRATCH_BYTES).
    Calls that can overlap on one device share that array and race; issue them on
    one stream or order them."""
    s = _stream(stream, A_data, D_data)
    _check(lib().mpk_gemm_mxfp8_bf16_noalloc(_addr(A_data), _addr(A_scales), _addr(B), _addr(C_data),
                                             _addr(C_scales), _addr(D_data), _addr(D_scales), M, N, K, s))


def gemm_fp8_tensorcore_gather(A_data, A_scales, B, C_data, C_scales, M: int, N: int, K: int,
                               row_offset: int, M_total: int, D_dest, Ds_dest, workspace,
                               stream=None, workspace_bytes: int | None = None,
                               col_offset: int = 0, N_total: int | None = None) -> None:
    """Fused GEMM + all-gather: element (r, c) of this slab's D goes to
    (row_offset + r, col_offset + c) of every destination (device addresses;
    D_dest[0] is this GPU's full M_total x N_total D).  The other GPUs' parts are
    present after peer_barrier on every GPU."""
    n = len(D_dest)
    assert n == len(Ds_dest) and 1 <= n <= 8
    dd = (ctypes.c_void_p * n)(*[_addr(x) for x in D_dest])
    ds = (ctypes.c_void_p * n)(*[_addr(x) for x in Ds_dest])
    s = _stream(stream, A_data)
    nbytes = _nbytes(workspace, workspace_bytes)
    _check(lib().mpk_gemm_mxfp8_bf16_gather(_addr(A_data), _addr(A_scales), _addr(B), _addr(C_data),
                                            _addr(C_scales), M, N, K, row_offset, col_offset, M_total,
                                            N if N_total is None else N_total, dd, ds, n,
                                            _addr(workspace), nbytes, s))


def peer_barrier(flags, rank: int, world: int, epoch: int, stream=None) -> None:
    """Stream-ordered barrier over the GPUs' flag arrays (device addresses, rank order)."""
    arr = (ctypes.c_void_p * world)(*[_addr(x) for x in flags])
    _check(lib().mpk_peer_barrier(arr, rank, world, epoch, _stream(stream)))


def ipc_export(t) -> tuple[bytes, int, int]:
    """(handle, offset, allocation bytes) describing the device allocation of t."""
    h = ctypes.create_string_buffer(64)
    off, size = ctypes.c_uint64(0), ctypes.c_uint64(0)
    _check(lib().mpk_ipc_export(_addr(t), h, ctypes.byref(off), ctypes.byref(size)))
    return h.raw, off.value, size.value


def ipc_import(handle: bytes, offset: int, alloc_bytes: int) -> int:
    """Map another process's exported buffer for the current device; returns its address."""
    p = ctypes.c_void_p(0)
    _check(lib().mpk_ipc_import(ctypes.c_char_p(handle), offset, alloc_bytes, ctypes.byref(p)))
    return p.value


def ipc_close(addr: int) -> None:
    _check(lib().mpk_ipc_close(addr))


def release_workspace_pool() -> None:
    """Return the current device's pooled GEMM workspace to the driver."""
    _check(lib().mpk_release_workspace_pool())


def mxfp8_quantize_gpu(input, data, scales, M: int, K: int, stream=None) -> None:
    s = _stream(stream, input, data)
    _check(lib().mpk_mxfp8_quantize(_addr(input), _addr(data), _addr(scales), M, K, s))


def mxfp8_dequantize_gpu(data, scales, output, M: int, K: int, stream=None) -> None:
    s = _stream(stream, data, output)
    _check(lib().mpk_mxfp8_dequantize(_addr(data), _addr(scales), _addr(output), M, K, s))


def mxfp8_quantize_bf16_gpu(input, data, scales, M: int, K: int, stream=None) -> None:
    """BF16 [M, K] -> MXFP8 along K (each value widened exactly to FP32 first)."""
    s = _stream(stream, input, data)
    _check(lib().mpk_mxfp8_quantize_bf16(_addr(input), _addr(data), _addr(scales), M, K, s))


def mxfp8_quantize_cols_gpu(input, data, scales, M: int, K: int, stream=None) -> None:
    """float32 [M, K] -> MXFP8 with blocks of 32 rows per column: data [M, K], scales
    [ceil(M/32), K]."""
    s = _stream(stream, input, data)
    _check(lib().mpk_mxfp8_quantize_cols(_addr(input), _addr(data), _addr(scales), M, K, s))


def mxfp8_quantize_bf16_cols_gpu(input, data, scales, M: int, K: int, stream=None) -> None:
    """BF16 [M, K] -> MXFP8 with blocks of 32 rows per column (values widened exactly)."""
    s = _stream(stream, input, data)
    _check(lib().mpk_mxfp8_quantize_bf16_cols(_addr(input), _addr(data), _addr(scales), M, K, s))


def quantize_cols(x, stream=None):
    """float32 or bfloat16 CUDA tensor [M, K] -> (codes uint8 [M, K], scales uint8
    [ceil(M/32), K]), blocks of 32 rows per column."""
    import torch
    assert x.is_cuda and x.dim() == 2 and x.is_contiguous() and x.dtype in (torch.float32, torch.bfloat16)
    M, K = x.shape
    d = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((nblk(M), K), dtype=torch.uint8, device=x.device)
    (mxfp8_quantize_cols_gpu if x.dtype == torch.float32 else mxfp8_quantize_bf16_cols_gpu)(x, d, s, M, K, stream)
    return d, s


def mxfp8_dequantize_bf16_gpu(data, scales, output, M: int, K: int, stream=None) -> None:
    """MXFP8 -> BF16 (the GEMM's A pre-pass); output is a bfloat16 CUDA tensor [M, K]."""
    s = _stream(stream, data, output)
    _check(lib().mpk_mxfp8_dequantize_bf16(_addr(data), _addr(scales), _addr(output), M, K, s))


def mxfp8_quantize_host(input, data, scales, M: int, K: int) -> None:
    _check(lib().mpk_mxfp8_quantize_host(_np_ptr(input), _np_ptr(data), _np_ptr(scales), M, K))


def mxfp8_dequantize_host(data, scales, output, M: int, K: int) -> None:
    _check(lib().mpk_mxfp8_dequantize_host(_np_ptr(data), _np_ptr(scales), _np_ptr(output), M, K))


def device_status() -> int:
    """Synchronize the current device, then read and clear its device status word."""
    v = ctypes.c_int(0)
    st = lib().mpk_device_status(ctypes.byref(v))
    if st not in (MPK_SUCCESS, MPK_ERR_DEVICE_TIMEOUT):
        _check(st)
    return v.value


def set_wait_timeout_ns(ns: int) -> None:
    _check(lib().mpk_set_wait_timeout_ns(int(ns)))


def wait_selftest(timeout_ns: int, stream=None) -> None:
    _check(lib().mpk_wait_selftest(int(timeout_ns), _stream(stream)))


def set_gemm_schedule(schedule: int) -> int:
    """Sets the process-wide GEMM work schedule (SCHEDULE_AUTO, SCHEDULE_TILES or
    SCHEDULE_STREAM_K); returns the previous one."""
    L = lib()
    prev = L.mpk_gemm_schedule()
    _check(L.mpk_set_gemm_schedule(int(schedule)))
    return prev


def gemm_schedule() -> int:
    return lib().mpk_gemm_schedule()


def gemm_path(A_data, B, M: int, N: int, K: int) -> int:
    """PATH_PREPASS or PATH_ONCHIP: the kernel path gemm_fp8_tensorcore takes for these
    operands (tensors or device addresses) under the current schedule."""
    path = ctypes.c_int(-1)
    _check(lib().mpk_gemm_path(_addr(A_data), _addr(B), M, N, K, ctypes.byref(path)))
    return path.value


def gemm_plan(M: int, N: int, K: int) -> tuple[int, int, int]:
    """(tiles, stream-K tiles, stream-K SM pairs) of an M x N x K product on the
    current device under the current schedule."""
    t, st, sp = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _check(lib().mpk_gemm_plan(M, N, K, ctypes.byref(t), ctypes.byref(st), ctypes.byref(sp)))
    return t.value, st.value, sp.value


# ---------------------------------------------------------------------------
# Allocating conveniences (torch tensors)
# ---------------------------------------------------------------------------

def quantize(x, stream=None):
    """float32 CUDA tensor [M, K] -> (codes uint8 [M, K], scales uint8 [M, ceil(K/32)])."""
    import torch
    assert x.dtype == torch.float32 and x.is_cuda and x.dim() == 2 and x.is_contiguous()
    M, K = x.shape
    d = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    s = torch.empty((M, nblk(K)), dtype=torch.uint8, device=x.device)
    mxfp8_quantize_gpu(x, d, s, M, K, stream)
    return d, s


def dequantize(d, s, stream=None):
    import torch
    assert d.dtype == torch.uint8 and d.is_cuda and d.dim() == 2 and d.is_contiguous()
    M, K = d.shape
    out = torch.empty((M, K), dtype=torch.float32, device=d.device)
    mxfp8_dequantize_gpu(d, s, out, M, K, stream)
    return out


def gemm(A_data, A_scales, B, C_data=None, C_scales=None, stream=None):
    """Allocating form of :func:`gemm_fp8_tensorcore`; B is a bf16 CUDA tensor [K, N]."""
    import torch
    M, K = A_data.shape
    K2, N = B.shape
    assert K == K2 and B.dtype == torch.bfloat16 and B.is_contiguous()
    D = torch.empty((M, N), dtype=torch.uint8, device=A_data.device)
    Ds = torch.empty((M, nblk(N)), dtype=torch.uint8, device=A_data.device)
    gemm_fp8_tensorcore(A_data, A_scales, B, C_data, C_scales, D, Ds, M, N, K, stream)
    return D, Ds

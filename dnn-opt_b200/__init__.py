"""Python mirror of the dnnopt B200 C ABI (include/dnnopt_b200.h).

Thin ctypes bindings over ``lib/libdnnopt_b200.so`` with the reference's
argument order and meaning (include/dnnopt/gemm/gemm.h of DNN-Opt): row-major
``C = alpha * A * B + beta * C``.  Every call returns a ``dnnopt_status`` int;
:func:`check` raises :class:`DnnoptError` on failure.

Arguments that are matrices accept a numpy array (host memory, synchronous
copy in/out by the library), a torch CUDA tensor (device memory) or a raw
integer address.  The library is required: importing this module fails loudly
when the shared object is missing (build it with ``make -C dnn-opt_b200``).
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libdnnopt_b200.so")
BLAS_PATH = os.path.join(_HERE, "lib", "libdnnopt_blas.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "dnnopt_b200.h")

SUCCESS = 0
INVALID_VALUE = 1
NOT_SUPPORTED = 2
CUDA_ERROR = 3
ALLOC_FAILED = 4
NO_DEVICE = 5
KERNEL_TIMEOUT = 6
INJECTED_FAULT = 7
EXCEEDS_SCRATCH = 8

# dnnopt_plan_describe kinds
KIND_F32, KIND_BF16F32, KIND_F32_BF16ROUND, KIND_F32_S8QUANT = 0, 1, 2, 3
KIND_S8S32, KIND_E4M3BF16, KIND_REFE4M3_E5M2, KIND_REFE5M2_E5M2 = 4, 5, 6, 7


class DnnoptError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})")


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int), ("N", ctypes.c_int), ("K", ctypes.c_int),
        ("lda", ctypes.c_int), ("ldb", ctypes.c_int), ("ldc", ctypes.c_int),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
        ("trans_a", ctypes.c_int), ("trans_b", ctypes.c_int),
    ]


def desc(M, N, K, lda, ldb, ldc, alpha=1.0, beta=0.0, trans_a=0, trans_b=0) -> GemmDesc:
    return GemmDesc(M, N, K, lda, ldb, ldc, alpha, beta, int(trans_a), int(trans_b))


MAX_RANKS = 8


class AllGatherDesc(ctypes.Structure):
    _fields_ = [
        ("world", ctypes.c_int), ("rank", ctypes.c_int),
        ("out", ctypes.c_void_p * MAX_RANKS),
        ("flags", ctypes.c_void_p * MAX_RANKS),
        ("seq", ctypes.c_void_p),
        ("out_stride", ctypes.c_size_t),
    ]


if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C dnn-opt_b200` "
                      "(there is no CPU fallback)")

lib = ctypes.CDLL(LIB_PATH)

_I, _F, _P = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
_HOST_SIG = [_I, _I, _I, _F, _P, _I, _P, _I, _F, _P, _I]
for _name in ("dnnopt_gemm_fp32", "dnnopt_gemm_bf16", "dnnopt_gemm_bf16_bf16bf16f32",
              "dnnopt_gemm_int8", "dnnopt_gemm_fp8_e4m3", "dnnopt_gemm_fp8_e5m2",
              "dnnopt_gemm_fp8"):
    getattr(lib, _name).argtypes = _HOST_SIG
    getattr(lib, _name).restype = _I
lib.dnnopt_gemm_int8_int8int8int32.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _I]
lib.dnnopt_gemm_e4m3_bf16.argtypes = [_I, _I, _I, _P, _I, _P, _I, _P, _P, _I]
lib.dnnopt_gemm_f32_desc.argtypes = [ctypes.POINTER(GemmDesc), _P, _P, _P]
lib.dnnopt_saxpy.argtypes = [_I, _F, _P, _I, _P, _I]
_I64P, _FP = ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_float)
_COLMAJOR_SIG = [ctypes.c_char_p, ctypes.c_char_p, _I64P, _I64P, _I64P, _FP, _P, _I64P, _P, _I64P,
                 _FP, _P, _I64P, _P]
class Conv3DParams(ctypes.Structure):
    """dnnopt_conv3d_params: N, IC, ID, IH, IW, OC, KD, KH, KW, strides d/h/w, pads d/h/w."""
    _fields_ = [(n, ctypes.c_int) for n in ("N", "IC", "ID", "IH", "IW", "OC", "KD", "KH", "KW",
                                             "stride_d", "stride_h", "stride_w",
                                             "pad_d", "pad_h", "pad_w")]


CONV3D_FP32, CONV3D_BF16, CONV3D_INT8 = 0, 1, 2
POSTOP_NONE, POSTOP_RELU, POSTOP_RELU6 = 0, 1, 2
lib.dnnopt_conv3d.argtypes = [_I, ctypes.POINTER(Conv3DParams), _P, _P, _P, _P, _I]
lib.dnnopt_cuda_conv3d.argtypes = [_I, ctypes.POINTER(Conv3DParams), _P, _P, _P, _P, _I, _P]
lib.dnnopt_sgemm_colmajor.argtypes = _COLMAJOR_SIG
lib.dnnopt_cuda_sgemm_colmajor.argtypes = _COLMAJOR_SIG + [_P]
for _name in ("dnnopt_cuda_gemm_f32", "dnnopt_cuda_gemm_bf16f32", "dnnopt_cuda_gemm_f32_bf16round",
              "dnnopt_cuda_gemm_f32_s8quant", "dnnopt_cuda_gemm_s8s32",
              "dnnopt_cuda_gemm_refe4m3_e5m2", "dnnopt_cuda_gemm_refe5m2_e5m2",
              "dnnopt_cuda_gemm_f32_noalloc"):
    getattr(lib, _name).argtypes = [ctypes.POINTER(GemmDesc), _P, _P, _P, _P]
    getattr(lib, _name).restype = _I
lib.dnnopt_cuda_gemm_e4m3bf16.argtypes = [ctypes.POINTER(GemmDesc), _P, _P, _P, _P, _P]
lib.dnnopt_has_fp8_support.restype = _I
lib.dnnopt_gemm_get_num_threads.restype = _I
lib.dnnopt_gemm_set_num_threads.argtypes = [_I]
lib.dnnopt_gemm_set_num_threads.restype = None
lib.dnnopt_set_stream.argtypes = [_P]
lib.dnnopt_get_last_error.restype = _I
lib.dnnopt_status_string.argtypes = [_I]
lib.dnnopt_status_string.restype = ctypes.c_char_p
lib.dnnopt_launch_count.restype = ctypes.c_uint64
lib.dnnopt_plan_describe.argtypes = [_I, ctypes.POINTER(GemmDesc), ctypes.c_char_p, _I]
lib.dnnopt_autotune_enable.argtypes = [_I]
lib.dnnopt_autotune_save.argtypes = [ctypes.c_char_p]
lib.dnnopt_autotune_load.argtypes = [ctypes.c_char_p]
lib.dnnopt_debug_inject_fault.argtypes = [_I, _I]
lib.dnnopt_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]
lib.dnnopt_peer_free.argtypes = [_P]
lib.dnnopt_ipc_handle.argtypes = [_P, ctypes.c_char_p]
lib.dnnopt_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
lib.dnnopt_ipc_close.argtypes = [_P]
lib.dnnopt_cuda_gemm_e4m3bf16_allgather.argtypes = [ctypes.POINTER(GemmDesc), _P, _P, _P,
                                                    ctypes.POINTER(AllGatherDesc), _P]
lib.dnnopt_cuda_peer_wait.argtypes = [_P, _I, ctypes.c_uint, ctypes.c_uint, _P]
lib.dnnopt_stream_status.argtypes = [_P]


def ptr(x) -> int | None:
    """Address of a numpy array, torch tensor, or raw integer (None -> NULL)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)!r}")


def status_string(status: int) -> str:
    return lib.dnnopt_status_string(status).decode()


def check(status: int, what: str = "dnnopt call") -> None:
    if status != SUCCESS:
        raise DnnoptError(status, what)


def declared_functions(header: str = HEADER_PATH) -> list[str]:
    """Names of every function declared in include/dnnopt_b200.h."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dnnopt_[a-z0-9_]+)\s*\(", text)))


# ---- reference-signature entry points (host or device pointers) -------------
def gemm_fp32(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_fp32(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta, ptr(C), ldc)


def gemm_bf16(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_bf16(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta, ptr(C), ldc)


def gemm_bf16_bf16bf16f32(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_bf16_bf16bf16f32(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta,
                                            ptr(C), ldc)


def gemm_int8(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_int8(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta, ptr(C), ldc)


def gemm_int8_int8int8int32(M, N, K, A, lda, B, ldb, C, ldc) -> int:
    return lib.dnnopt_gemm_int8_int8int8int32(M, N, K, ptr(A), lda, ptr(B), ldb, ptr(C), ldc)


def gemm_fp8_e4m3(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_fp8_e4m3(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta, ptr(C), ldc)


def gemm_fp8_e5m2(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_fp8_e5m2(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta, ptr(C), ldc)


def gemm_fp8(M, N, K, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    return lib.dnnopt_gemm_fp8(M, N, K, alpha, ptr(A), lda, ptr(B), ldb, beta, ptr(C), ldc)


def gemm_e4m3_bf16(M, N, K, A, lda, W, ldw, scale, C, ldc) -> int:
    return lib.dnnopt_gemm_e4m3_bf16(M, N, K, ptr(A), lda, ptr(W), ldw, ptr(scale), ptr(C), ldc)


def gemm_f32_desc(d: GemmDesc, A, B, C) -> int:
    return lib.dnnopt_gemm_f32_desc(ctypes.byref(d), ptr(A), ptr(B), ptr(C))


def saxpy(N, alpha, X, incX, Y, incY) -> int:
    return lib.dnnopt_saxpy(N, alpha, ptr(X), incX, ptr(Y), incY)


def _colmajor_args(transa, transb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, bias):
    i64, f32 = ctypes.c_int64, ctypes.c_float
    return (transa.encode() if isinstance(transa, str) else transa,
            transb.encode() if isinstance(transb, str) else transb,
            ctypes.byref(i64(M)), ctypes.byref(i64(N)), ctypes.byref(i64(K)), ctypes.byref(f32(alpha)),
            ptr(A), ctypes.byref(i64(lda)), ptr(B), ctypes.byref(i64(ldb)), ctypes.byref(f32(beta)),
            ptr(C), ctypes.byref(i64(ldc)), ptr(bias))


def sgemm_colmajor(transa, transb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, bias=None) -> int:
    """The oneDNN integration's dnnopt_sgemm: column-major, optional bias[i]."""
    return lib.dnnopt_sgemm_colmajor(*_colmajor_args(transa, transb, M, N, K, alpha, A, lda, B, ldb,
                                                     beta, C, ldc, bias))


def conv3d(precision, params, inp, flt, bias, out, post_op=0) -> int:
    """params: Conv3DParams or the 15 ints in its field order."""
    p = params if isinstance(params, Conv3DParams) else Conv3DParams(*params)
    return lib.dnnopt_conv3d(precision, ctypes.byref(p), ptr(inp), ptr(flt), ptr(bias), ptr(out), post_op)


def has_fp8_support() -> bool:
    return bool(lib.dnnopt_has_fp8_support())


# ---- device-pointer entry points (asynchronous on `stream`) -----------------
def cuda_gemm(kind: str, d: GemmDesc, A, B, C, stream=None, scale=None) -> int:
    """kind: f32 | bf16f32 | f32_bf16round | f32_s8quant | s8s32 | e4m3bf16 |
    refe4m3_e5m2 | refe5m2_e5m2 | f32_noalloc."""
    s = ptr(stream) if not hasattr(stream, "cuda_stream") else stream.cuda_stream
    fn = getattr(lib, f"dnnopt_cuda_gemm_{kind}")
    if kind == "e4m3bf16":
        return fn(ctypes.byref(d), ptr(A), ptr(B), ptr(scale), ptr(C), s)
    return fn(ctypes.byref(d), ptr(A), ptr(B), ptr(C), s)


def cuda_sgemm_colmajor(transa, transb, M, N, K, alpha, A, lda, B, ldb, beta, C, ldc, bias=None,
                        stream=None) -> int:
    return lib.dnnopt_cuda_sgemm_colmajor(*_colmajor_args(transa, transb, M, N, K, alpha, A, lda, B,
                                                          ldb, beta, C, ldc, bias), _stream(stream))


def cuda_conv3d(precision, params, inp, flt, bias, out, post_op=0, stream=None) -> int:
    p = params if isinstance(params, Conv3DParams) else Conv3DParams(*params)
    return lib.dnnopt_cuda_conv3d(precision, ctypes.byref(p), ptr(inp), ptr(flt), ptr(bias), ptr(out),
                                  post_op, _stream(stream))


def _stream(stream):
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else ptr(stream)


# ---- multi-GPU (one process per GPU) ----------------------------------------
def peer_alloc(nbytes: int) -> int:
    p = ctypes.c_void_p()
    check(lib.dnnopt_peer_alloc(nbytes, ctypes.byref(p)), "peer_alloc")
    return int(p.value)


def peer_free(address: int) -> None:
    check(lib.dnnopt_peer_free(address), "peer_free")


def ipc_handle(address: int) -> bytes:
    buf = ctypes.create_string_buffer(64)
    check(lib.dnnopt_ipc_handle(address, buf), "ipc_handle")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    if len(handle) != 64:
        raise ValueError("CUDA IPC handles are 64 bytes")
    p = ctypes.c_void_p()
    check(lib.dnnopt_ipc_open(handle, ctypes.byref(p)), "ipc_open")
    return int(p.value)


def ipc_close(address: int) -> None:
    check(lib.dnnopt_ipc_close(address), "ipc_close")


def cuda_gemm_e4m3bf16_allgather(d: GemmDesc, A, W, scale, ag: AllGatherDesc, stream=None) -> int:
    return lib.dnnopt_cuda_gemm_e4m3bf16_allgather(ctypes.byref(d), ptr(A), ptr(W), ptr(scale),
                                                   ctypes.byref(ag), _stream(stream))


def cuda_peer_wait(flags, world: int, epoch: int, timeout_us: int, stream=None) -> int:
    return lib.dnnopt_cuda_peer_wait(ptr(flags), world, epoch, timeout_us, _stream(stream))


def stream_status(stream=None) -> int:
    return lib.dnnopt_stream_status(_stream(stream))


def plan_describe(kind: int, d: GemmDesc) -> str:
    buf = ctypes.create_string_buffer(256)
    check(lib.dnnopt_plan_describe(kind, ctypes.byref(d), buf, 256), "plan_describe")
    return buf.value.decode()


def launch_count() -> int:
    return int(lib.dnnopt_launch_count())


def set_stream(stream) -> int:
    s = stream.cuda_stream if hasattr(stream, "cuda_stream") else ptr(stream)
    return lib.dnnopt_set_stream(s)

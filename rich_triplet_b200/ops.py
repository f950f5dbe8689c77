"""Per-call GPU operators: the CUDA counterpart of the reference's metal_ops.

    metal_gemv_q4k_t(a, q4k)  -> cuda_gemv_q4k_t(a, q4k)   (src/metal_ops.rs:799-860)
    metal_gemv_bf16_t(a, bf16) -> cuda_gemv_bf16_t(a, bf16) (src/metal_ops.rs:887-960)

Like the Metal versions, each call uploads the weight once (cached by buffer
address and length, src/metal_ops.rs:811-815), copies the activation in,
runs one GEMV and copies the result out.  Shape mismatches raise ValueError
where the reference's assert_eq! panics; device failures raise RtError.
"""

import ctypes
import threading

import numpy as np

from . import _lib
from ._lib import RT_DEVICE, RT_FMT_BF16, RT_FMT_Q4K, RT_HOST, RtError, check, lib
from .model import MatBf16, Q4KMat


class Context:
    """One device, one stream (rt_ctx)."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        rc = lib().rt_init(device, ctypes.byref(h))
        if rc != _lib.RT_OK:
            raise RtError(rc, f"rt_init(device={device}) failed (no CUDA device?)")
        self.h = h
        self.device = device

    @property
    def stream_ptr(self):
        return lib().rt_stream(self.h)

    def sync(self):
        check(lib().rt_sync(self.h), self.h)

    def last_error(self):
        return lib().rt_last_error(self.h).decode()

    def close(self):
        if self.h:
            lib().rt_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceWeight:
    """A weight matrix resident in HBM (rt_w)."""

    def __init__(self, ctx, handle, fmt, rows, cols):
        self.ctx, self.h, self.fmt, self.rows, self.cols = ctx, handle, fmt, rows, cols

    @classmethod
    def upload(cls, ctx, fmt, host, rows, cols):
        host = np.ascontiguousarray(host)
        h = ctypes.c_void_p()
        check(lib().rt_weight_upload(ctx.h, fmt, host.ctypes.data, host.nbytes, rows, cols, ctypes.byref(h)), ctx.h)
        return cls(ctx, h, fmt, rows, cols)

    @property
    def nbytes(self):
        b = ctypes.c_uint64()
        lib().rt_weight_info(self.h, None, None, None, ctypes.byref(b))
        return b.value

    @property
    def device_ptr(self):
        return lib().rt_weight_device_ptr(self.h)

    def download(self):
        dt = np.uint16 if self.fmt == RT_FMT_BF16 else np.uint8
        n = self.nbytes // np.dtype(dt).itemsize
        out = np.empty(n, dtype=dt)
        check(lib().rt_weight_download(self.ctx.h, self.h, out.ctypes.data, out.nbytes), self.ctx.h)
        return out

    def free(self):
        if self.h:
            lib().rt_weight_free(self.ctx.h, self.h)
            self.h = None

    def __del__(self):
        try:
            if self.ctx is not None and self.ctx.h:
                self.free()
        except Exception:
            pass


_tls = threading.local()


def default_context():
    """Thread-local context, created on first use (METAL_CTX, src/metal_ops.rs:404-428)."""
    ctx = getattr(_tls, "ctx", None)
    if ctx is None:
        ctx = Context(0)
        _tls.ctx = ctx
        _tls.cache = {}
    return ctx


def _cached_weight(ctx, fmt, buf, rows, cols):
    key = (fmt, buf.ctypes.data, buf.nbytes, rows, cols)
    w = _tls.cache.get(key)
    if w is None:
        w = DeviceWeight.upload(ctx, fmt, buf, rows, cols)
        _tls.cache[key] = (w, buf)  # keep the host buffer alive with its device copy
        return w
    return w[0]


def _as_row(a, k, name):
    a = np.ascontiguousarray(a, dtype=np.float32)
    if a.ndim == 2:
        if a.shape[0] != 1:
            raise ValueError(f"{name}: only M=1 supported")
        a = a[0]
    if a.shape[0] != k:
        raise ValueError(f"{name}: a.cols {a.shape[0]} != weight cols {k}")
    return np.ascontiguousarray(a)


def cuda_gemv_q4k_t(a, q4k: Q4KMat):
    """C[1, N] = A[1, K] @ dequant(Q4K[N, K])^T on the GPU, f32 accumulation."""
    ctx = default_context()
    x = _as_row(a, q4k.cols, "cuda_gemv_q4k_t")
    w = _cached_weight(ctx, RT_FMT_Q4K, q4k.blocks, q4k.rows, q4k.cols)
    y = np.empty(q4k.rows, dtype=np.float32)
    check(lib().rt_gemv_q4k(ctx.h, w.h, x.ctypes.data, y.ctypes.data, RT_HOST), ctx.h)
    return y.reshape(1, -1)


def cuda_gemv_bf16_t(a, bf16: MatBf16):
    """C[1, N] = A[1, K] @ BF16[N, K]^T on the GPU, f32 accumulation."""
    ctx = default_context()
    x = _as_row(a, bf16.cols, "cuda_gemv_bf16_t")
    w = _cached_weight(ctx, RT_FMT_BF16, bf16.data, bf16.rows, bf16.cols)
    y = np.empty(bf16.rows, dtype=np.float32)
    check(lib().rt_gemv_bf16(ctx.h, w.h, x.ctypes.data, y.ctypes.data, RT_HOST), ctx.h)
    return y.reshape(1, -1)


def bf16_bits(a):
    """f32 -> bf16 bits (uint16), round to nearest even."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)


def cuda_matmul_q4k_t(a, q4k: Q4KMat):
    """C[M, N] = A[M, K] @ dequant(Q4K[N, K])^T on the tensor cores, f32
    accumulation (Q4KMat::matmul_q4k_t, src/autograd2.rs:1437-1457).  `a` is
    bf16 bits (uint16) or f32, which is rounded to bf16 first."""
    ctx = default_context()
    a = np.ascontiguousarray(a)
    if a.ndim != 2 or a.shape[1] != q4k.cols:
        raise ValueError(f"cuda_matmul_q4k_t: a shape {a.shape} does not match weight cols {q4k.cols}")
    bits = a if a.dtype == np.uint16 else bf16_bits(a)
    w = _cached_weight(ctx, RT_FMT_Q4K, q4k.blocks, q4k.rows, q4k.cols)
    c = np.empty((a.shape[0], q4k.rows), dtype=np.float32)
    check(lib().rt_gemm_q4k(ctx.h, w.h, bits.ctypes.data, a.shape[0], c.ctypes.data, RT_HOST), ctx.h)
    return c


def cuda_matmul_bf16_t(a, bf16: MatBf16):
    """C[M, N] = A[M, K] @ BF16[N, K]^T on the tensor cores (MatBf16::matmul_by_t, M > 1)."""
    ctx = default_context()
    a = np.ascontiguousarray(a)
    if a.ndim != 2 or a.shape[1] != bf16.cols:
        raise ValueError(f"cuda_matmul_bf16_t: a shape {a.shape} does not match weight cols {bf16.cols}")
    bits = a if a.dtype == np.uint16 else bf16_bits(a)
    w = _cached_weight(ctx, RT_FMT_BF16, bf16.data, bf16.rows, bf16.cols)
    c = np.empty((a.shape[0], bf16.rows), dtype=np.float32)
    check(lib().rt_gemm_bf16(ctx.h, w.h, bits.ctypes.data, a.shape[0], c.ctypes.data, RT_HOST), ctx.h)
    return c


def gemm_device(ctx, w: DeviceWeight, a_ptr, m, c_ptr):
    """Enqueue C[m, N] = A[m, K] @ W^T on device pointers (A bf16; W Q4_K or BF16)."""
    fn = lib().rt_gemm_q4k if w.fmt == RT_FMT_Q4K else lib().rt_gemm_bf16
    check(fn(ctx.h, w.h, a_ptr, m, c_ptr, RT_DEVICE), ctx.h)


def gemv_device(ctx, w: DeviceWeight, x_ptr, y_ptr):
    """Enqueue one GEMV on device pointers (no synchronisation)."""
    fn = lib().rt_gemv_q4k if w.fmt == RT_FMT_Q4K else lib().rt_gemv_bf16
    check(fn(ctx.h, w.h, x_ptr, y_ptr, RT_DEVICE), ctx.h)


def gemv_bench(ctx, weights, x_ptr, y_ptr, launches=256, ctas_per_sm=2, reps=3):
    """Mean device time (us) per GEMV over a CUDA graph of `launches` chained
    GEMVs rotating over `weights` (same format and shape); see rt_gemv_bench."""
    arr = (ctypes.c_void_p * len(weights))(*[w.h for w in weights])
    us = ctypes.c_float()
    check(lib().rt_gemv_bench(ctx.h, weights[0].fmt, arr, len(weights), x_ptr, y_ptr, launches, ctas_per_sm, reps,
                              ctypes.byref(us)), ctx.h)
    return us.value


def convert_q4_0_to_q4k(ctx, q4_0_bytes, rows, cols):
    """GGUF Q4_0 -> Q4_K on the GPU, bit-exact with decode_q4_0_to_q4mat +
    Q4KMat::from_q4mat (src/gguf_loader.rs:282-350, src/autograd2.rs:1291-1320)."""
    src = np.ascontiguousarray(q4_0_bytes, dtype=np.uint8)
    h = ctypes.c_void_p()
    check(lib().rt_convert_q4_0_to_q4k(ctx.h, src.ctypes.data, rows, cols, RT_HOST, ctypes.byref(h)), ctx.h)
    return DeviceWeight(ctx, h, RT_FMT_Q4K, rows, cols)


def convert_q6k_to_bf16(ctx, q6k_bytes, rows, cols):
    """GGUF Q6_K -> BF16 on the GPU, bit-exact with decode_q6k_to_f32 +
    f32s_to_bf16_and_drop (src/gguf_loader.rs:482-533, src/transformer4.rs:1084-1097)."""
    src = np.ascontiguousarray(q6k_bytes, dtype=np.uint8)
    h = ctypes.c_void_p()
    check(lib().rt_convert_q6k_to_bf16(ctx.h, src.ctypes.data, rows, cols, RT_HOST, ctypes.byref(h)), ctx.h)
    return DeviceWeight(ctx, h, RT_FMT_BF16, rows, cols)

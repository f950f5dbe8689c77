"""B200-native (sm_100a) rebuild of rich-triplet's Q4_K decode hot path.

The product is librtcuda.so (C ABI: include/rt_cuda.h); this package is the
host-side mirror of the reference crate's operator surface:

    ops.cuda_gemv_q4k_t / cuda_gemv_bf16_t   <- metal_ops::metal_gemv_*_t
    decode.CudaDecodeContext                  <- metal_decode::MetalDecodeContext
    model.Config4 / Q4KMat / MatBf16          <- transformer4::Config4, autograd2 types
"""

from ._lib import RtError, build, lib  # noqa: F401

__version__ = "0.1.0"

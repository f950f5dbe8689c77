"""QLinear on the GPU: the reference's inference-only linear layer
(src/qlinear.rs:26-132, used by its FLUX and T5 stacks) over a weight held in
HBM.

The weight is [out_features, in_features] (PyTorch's Linear.weight layout) in
one of the formats the reference's QLinear loads; forward is x[T, in] ->
x . W^T + bias, through rt_qlinear_forward: one row runs the GEMV (f32-level
accuracy), several rows the product over fp16 rows of x (relative error about
1e-4): the multi-row GEMV for a Q4_K weight and up to 16 rows, else the
tensor-core GEMM.  Q4_K (matmul_q4k_t_exact) and BF16 (matmul_by_t) weights are
supported; the f32 format of the reference (its small VAE layers) is not on
this path and is refused.
"""

import ctypes

import numpy as np

from ._lib import RT_DEVICE, RT_FMT_BF16, RT_FMT_Q4K, RT_HOST, check, lib
from .model import MatBf16, Q4KMat
from .ops import Context, DeviceWeight


class QLinear:
    """QLinear (src/qlinear.rs:26-37): in_features, out_features, one weight
    (here a DeviceWeight in HBM) and an optional bias of out_features."""

    def __init__(self, ctx: Context = None, weight: DeviceWeight = None, in_features=0, out_features=0, bias=()):
        self.ctx = ctx
        self.weight = weight
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        b = np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        if b.size and b.size != self.out_features:
            raise ValueError(f"QLinear: bias of {b.size}, out_features {self.out_features}")
        self.bias = b

    @classmethod
    def from_q4k(cls, ctx: Context, weight: Q4KMat, out_features, in_features, bias=()):
        """QLinear::from_q4k (src/qlinear.rs:71-73): uploads the Q4_K blocks."""
        if weight.rows != out_features or weight.cols != in_features:
            raise ValueError(f"QLinear.from_q4k: weight [{weight.rows}, {weight.cols}], "
                             f"expected [{out_features}, {in_features}]")
        w = DeviceWeight.upload(ctx, RT_FMT_Q4K, weight.blocks, out_features, in_features)
        return cls(ctx, w, in_features, out_features, bias)

    @classmethod
    def from_bf16(cls, ctx: Context, weight: MatBf16, bias=()):
        """QLinear::from_bf16 (src/qlinear.rs:67-69)."""
        w = DeviceWeight.upload(ctx, RT_FMT_BF16, weight.data, weight.rows, weight.cols)
        return cls(ctx, w, weight.cols, weight.rows, bias)

    @classmethod
    def from_f32(cls, *args, **kwargs):
        """QLinear::from_f32 (src/qlinear.rs:63-65) keeps an f32 weight for small
        layers; the GPU path takes Q4_K and BF16 weights only."""
        raise NotImplementedError("QLinear on the GPU takes Q4_K or BF16 weights (from_q4k / from_bf16)")

    def loaded(self):
        """QLinear::loaded (src/qlinear.rs:76-78)."""
        return self.weight is not None and self.weight.h is not None

    def forward(self, x):
        """QLinear::forward (src/qlinear.rs:83-111): x [T, in] f32 -> [T, out],
        plus the bias if there is one."""
        if not self.loaded():
            raise ValueError("QLinear.forward: no weight loaded")
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x.reshape(1, -1)
        if x.ndim != 2 or x.shape[1] != self.in_features:
            raise ValueError(f"QLinear: input width {x.shape[-1]} != in_features {self.in_features}")
        t = x.shape[0]
        y = np.empty((t, self.out_features), dtype=np.float32)
        b = self.bias.ctypes.data if self.bias.size else None
        check(lib().rt_qlinear_forward(self.ctx.h, self.weight.h, x.ctypes.data, t, b, y.ctypes.data, RT_HOST),
              self.ctx.h)
        return y

    def forward_device(self, x_ptr, t, y_ptr, bias_ptr=None):
        """The same on device pointers (x [t, in], y [t, out], bias [out] or
        None), enqueued on the context stream."""
        if not self.loaded():
            raise ValueError("QLinear.forward_device: no weight loaded")
        check(lib().rt_qlinear_forward(self.ctx.h, self.weight.h, ctypes.c_void_p(x_ptr), int(t),
                                       ctypes.c_void_p(bias_ptr) if bias_ptr else None, ctypes.c_void_p(y_ptr),
                                       RT_DEVICE), self.ctx.h)

    def size_bytes(self):
        """QLinear::size_bytes (src/qlinear.rs:114-122): bytes of the weight."""
        return self.weight.nbytes if self.loaded() else 0

    def free_weight(self):
        """QLinear::free_weight (src/qlinear.rs:125-131): release the weight."""
        if self.weight is not None:
            self.weight.free()
        self.weight = None

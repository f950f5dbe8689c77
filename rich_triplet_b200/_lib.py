"""ctypes binding of librtcuda.so (the C ABI declared in include/rt_cuda.h).

The library is built in-tree (rich_triplet_b200/librtcuda.so) by build();
loading fails loudly when it is missing -- there is no CPU fallback.
"""

import ctypes
import os
import subprocess
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librtcuda.so")
CSRC = os.path.join(_HERE, "csrc")

RT_OK = 0
RT_E_INVAL = -1
RT_E_CUDA = -2
RT_E_NOMEM = -3
RT_E_SHAPE = -4
RT_E_FORMAT = -5
RT_E_IO = -6
RT_E_STATE = -7
RT_E_TIMEOUT = -8

RT_FMT_F32 = 0
RT_FMT_Q4_0 = 2
RT_FMT_Q4K = 12
RT_FMT_Q6K = 14
RT_FMT_BF16 = 30

RT_HOST = 0
RT_DEVICE = 1

_STATUS_NAMES = {0: "RT_OK", -1: "RT_E_INVAL", -2: "RT_E_CUDA", -3: "RT_E_NOMEM", -4: "RT_E_SHAPE",
                 -5: "RT_E_FORMAT", -6: "RT_E_IO", -7: "RT_E_STATE", -8: "RT_E_TIMEOUT"}


class RtError(RuntimeError):
    """A C-ABI call returned a negative RT_E_* status."""

    def __init__(self, code, msg):
        self.code = code
        super().__init__(f"{_STATUS_NAMES.get(code, code)}: {msg}")


def build(verbose=False):
    """Compile librtcuda.so for sm_100a with nvcc (no GPU needed)."""
    cmd = ["make", "-C", CSRC, "-j8"]
    if not verbose:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)


class RtGemma3Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads",
                                              "num_key_value_heads", "head_dim", "intermediate_size",
                                              "sliding_window")] + \
               [(n, ctypes.c_float) for n in ("rope_theta_local", "rope_theta_global", "rope_freq_scale_local",
                                              "rope_freq_scale_global", "rms_norm_eps", "query_pre_attn_scalar")]


class RtGemma3Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("q", "k", "v", "o", "gate", "up", "down")] + \
               [(n, ctypes.c_void_p) for n in ("attn_norm", "post_attn_norm", "pre_ffn_norm", "post_ffn_norm",
                                               "q_norm", "k_norm")]


class RtQwen35Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("vocab_size", "hidden_size", "num_hidden_layers", "num_attention_heads",
                                              "num_key_value_heads", "head_dim", "linear_num_key_heads",
                                              "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim",
                                              "linear_conv_kernel_dim", "intermediate_size",
                                              "full_attention_interval", "rope_dim")] + \
               [("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


class RtQwen35Layer(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("gate", "up", "down", "input_norm", "post_attn_norm", "in_qkv", "in_z",
                                               "in_a", "in_b", "out_proj", "conv1d_weight", "a_log", "dt_bias",
                                               "norm_weight", "q", "k", "v", "o", "q_norm", "k_norm")]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_pp = ctypes.POINTER(ctypes.c_void_p)

SIGNATURES = {
    "rt_init": (ctypes.c_int, [ctypes.c_int, _pp]),
    "rt_destroy": (None, [_vp]),
    "rt_last_error": (ctypes.c_char_p, [_vp]),
    "rt_version": (ctypes.c_char_p, []),
    "rt_stream": (_vp, [_vp]),
    "rt_sync": (ctypes.c_int, [_vp]),
    "rt_weight_upload": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _u64, _i64, _i64, _pp]),
    "rt_weight_download": (ctypes.c_int, [_vp, _vp, _vp, _u64]),
    "rt_weight_info": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(_i64),
                                      ctypes.POINTER(_i64), ctypes.POINTER(_u64)]),
    "rt_weight_device_ptr": (_vp, [_vp]),
    "rt_weight_free": (None, [_vp, _vp]),
    "rt_gemv_q4k": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int]),
    "rt_gemv_bf16": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int]),
    "rt_gemv_bf16_argmax_static": (
        ctypes.c_int,
        [_vp, ctypes.c_int64, ctypes.c_int, _vp, _vp, _vp, _vp, ctypes.c_char_p, ctypes.c_size_t],
    ),
    "rt_gemm_q4k": (ctypes.c_int, [_vp, _vp, _vp, _i64, _vp, ctypes.c_int]),
    "rt_batch_create": (ctypes.c_int, [_vp, _i32, _i32, _pp]),
    "rt_batch_destroy": (None, [_vp]),
    "rt_batch_set": (ctypes.c_int, [_vp, _vp, _vp]),
    "rt_batch_step": (ctypes.c_int, [_vp, _vp, _vp]),
    "rt_batch_generate": (ctypes.c_int, [_vp, _i32, ctypes.c_int]),
    "rt_batch_synth_kv": (ctypes.c_int, [_vp, _u64, _i32]),
    "rt_batch_info": (ctypes.c_int, [_vp, ctypes.POINTER(_u64), ctypes.POINTER(_i32)]),
    "rt_gemm_bf16": (ctypes.c_int, [_vp, _vp, _vp, _i64, _vp, ctypes.c_int]),
    "rt_gemm_plan": (ctypes.c_int, [_i64, _i64, _i32, _i32, _i32, ctypes.POINTER(_i32)]),
    "rt_qlinear_forward": (ctypes.c_int, [_vp, _vp, _vp, _i64, _vp, _vp, ctypes.c_int]),
    "rt_gemv_bench": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(_vp), ctypes.c_int, _vp, _vp, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]),
    "rt_convert_q4_0_to_q4k": (ctypes.c_int, [_vp, _vp, _i64, _i64, ctypes.c_int, _pp]),
    "rt_convert_q6k_to_bf16": (ctypes.c_int, [_vp, _vp, _i64, _i64, ctypes.c_int, _pp]),
    "rt_decoder_create": (ctypes.c_int, [_vp, ctypes.POINTER(RtGemma3Cfg), ctypes.POINTER(RtGemma3Layer), _vp,
                                         _vp, _i32, _pp]),
    "rt_decoder_destroy": (None, [_vp]),
    "rt_decoder_load_kv": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32]),
    "rt_decoder_read_kv": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32]),
    "rt_decoder_step": (ctypes.c_int, [_vp, _i32, _i32, _vp]),
    "rt_qwen35_create": (ctypes.c_int, [_vp, ctypes.POINTER(RtQwen35Cfg), ctypes.POINTER(RtQwen35Layer), _vp, _vp, _i32,
                                        _pp]),
    "rt_qwen35_destroy": (None, [_vp]),
    "rt_qwen35_reset": (ctypes.c_int, [_vp]),
    "rt_qwen35_step": (ctypes.c_int, [_vp, _i32, _i32, _vp]),
    "rt_qwen35_logits_device": (ctypes.c_int, [_vp, _pp]),
    "rt_decoder_prefill": (ctypes.c_int, [_vp, _vp, _i32, _i32, _vp]),
    "rt_decoder_prefill_gemm": (ctypes.c_int, [_vp, _vp, _i32, _i32, _vp]),
    "rt_decoder_step_batch": (ctypes.c_int, [_vp, _vp, _i32, _i32, _vp]),
    "rt_decoder_generate": (ctypes.c_int, [_vp, _i32, _i32, _i32, _vp, ctypes.c_int]),
    "rt_decoder_enqueue_q4k_gemvs": (ctypes.c_int, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_u64)]),
    "rt_decoder_memory": (ctypes.c_int, [_vp, ctypes.POINTER(_u64)]),
    "rt_decoder_launches_per_step": (ctypes.c_int, [_vp, ctypes.POINTER(_i32)]),
    "rt_decoder_read_activation": (ctypes.c_int, [_vp, _i32, _vp, _i64]),
    "rt_synth_q4k": (None, [_u64, _u64, _i64, _i64, _vp]),
    "rt_nccl_unique_id": (ctypes.c_int, [_vp]),
    "rt_tp_create": (ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    "rt_batch_vocab_slice": (ctypes.c_int, [_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "rt_tp_peer_handle": (ctypes.c_int, [_vp, _vp]),
    "rt_tp_peer_open": (ctypes.c_int, [_vp, _vp]),
    "rt_test_peer_allreduce_lonely": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int),
                                                     ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)]),
    "rt_synth_q4k_slice": (None, [_u64, _u64, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "rt_synth_normal_f32": (None, [_u64, _u64, _i64, ctypes.c_float, ctypes.c_float, _vp]),
    "rt_synth_normal_bf16": (None, [_u64, _u64, _i64, ctypes.c_float, ctypes.c_float, _vp]),
    "rt_synth_tokens": (None, [_u64, _u64, _i64, _i32, _vp]),
    "rt_synth_bytes": (None, [_u64, _u64, _i64, _vp]),
}

_lock = threading.Lock()
_lib = None


def lib():
    """The loaded librtcuda.so.  Raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: run rich_triplet_b200.build() (nvcc, sm_100a) first; "
                                   "the package has no CPU fallback")
            h = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
        return _lib


def check(rc, ctx=None):
    if rc != RT_OK:
        msg = lib().rt_last_error(ctx).decode() if ctx else ""
        raise RtError(rc, msg)
    return rc

"""ctypes prototypes for include/willamette_b200.h.

Loads project_willamette_b200/_lib/libwillamette_b200.so (built in-tree by
``python -m project_willamette_b200.build``).  A missing library is an
error: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import enum
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libwillamette_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "willamette_b200.h")


class WLStatus(enum.IntEnum):
    OK = 0
    UNSUPPORTED_TENSOR_TYPE = 1
    GGUF_PARSE = 2
    NOT_IMPLEMENTED = 3
    INVALID_ARGUMENT = 4
    CUDA = 5
    NO_DEVICE = 6
    DEVICE_TIMEOUT = 7
    COMM = 8
    INVALID_MAGIC = 9
    UNSUPPORTED_VERSION = 10
    UNSUPPORTED_ARCHITECTURE = 11
    MISSING_METADATA = 12
    TENSOR_OUT_OF_BOUNDS = 13


class WlTensorView(C.Structure):
    _fields_ = [
        ("name", C.c_char_p),
        ("shape", C.POINTER(C.c_uint64)),
        ("n_dims", C.c_uint32),
        ("ggml_type", C.c_uint32),
        ("data", C.POINTER(C.c_uint8)),
        ("data_len", C.c_size_t),
        ("scale_data", C.POINTER(C.c_uint8)),
        ("scale_len", C.c_size_t),
    ]


class WlI2sDevWeight(C.Structure):
    _fields_ = [
        ("packed", C.c_void_p),
        ("w_scale", C.c_float),
        ("out_dim", C.c_uint32),
        ("y", C.c_void_p),
        ("acc", C.c_void_p),
        ("flags", C.c_uint32),
    ]


WL_I2S_NO_CODE3 = 1


class I2sKernel(enum.IntEnum):
    """The reference's dispatch choice (src/model/dispatch.rs:47-71 Kernel)."""
    SCALAR = 0       # bitlinear_i2s_matvec_f32_scalar
    NEON = 1         # aarch64: no GPU arm (WL_ERR_NOT_IMPLEMENTED)
    SSE2_I8 = 2      # the x86 default (int8 activations)
    SCALAR_LUT = 3   # SSE2 hosts without SSSE3
    SSE2_F32 = 4     # x86 under --cfg willamette_sse2_f32


class WlI2sStreamOp(C.Structure):
    _fields_ = [
        ("packed", C.c_void_p),
        ("w_scale", C.c_float),
        ("in_dim", C.c_uint32),
        ("out_dim", C.c_uint32),
        ("x", C.c_void_p),
        ("y", C.c_void_p),
        ("acc", C.c_void_p),
        ("flags", C.c_uint32),
        ("row_off", C.c_uint32),
    ]


WL_TP_HANDLE_BYTES = 64


class WlBitnetConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "n_embd", "n_heads", "n_kv_heads",
                                          "head_dim", "n_ff", "vocab", "n_rot", "max_seq")] + \
               [("eps", C.c_float), ("freq_base", C.c_float), ("exact", C.c_uint32),
                ("persistent", C.c_uint32), ("kv_f16", C.c_uint32)]


class WlBitnetWeights(C.Structure):
    _fields_ = [("w", C.POINTER(C.c_void_p)), ("w_scale", C.POINTER(C.c_float)),
                ("norms", C.POINTER(C.c_float)), ("output_norm", C.POINTER(C.c_float)),
                ("token_embd", C.c_void_p)]

class WlLlamaWeights(C.Structure):
    _fields_ = [("w", C.POINTER(C.c_void_p)), ("attn_norm", C.POINTER(C.c_float)),
                ("ffn_norm", C.POINTER(C.c_float)), ("output_norm", C.POINTER(C.c_float)),
                ("token_embd", C.c_void_p)]


_vp = C.c_void_p
_sz = C.c_size_t
_u32 = C.c_uint32
_i = C.c_int
_fp = C.POINTER(C.c_float)
_tv = C.POINTER(WlTensorView)

PROTOTYPES = {
    "wl_version": ([], C.c_char_p),
    "wl_last_error": ([], C.c_char_p),
    "wl_last_error_tensor_type": ([], _u32),
    "wl_init": ([_i], _i),
    "wl_release_weights": ([], _i),
    "wl_device_status": ([C.POINTER(_u32)], _i),
    "wl_set_wait_limit_ns": ([C.c_uint64], _i),
    "wl_dev_rms_norm_f32": ([_vp, _vp, _u32, C.c_float, _vp, _vp], _i),
    "wl_dev_softmax_f32": ([_vp, _u32, _vp], _i),
    "wl_bitlinear_i2s_matvec_f32_kernel": ([_tv, _fp, _sz, _fp, _sz, _u32], _i),
    "wl_dev_i2s_matvec_f32act": ([_vp, C.c_float, _u32, _u32, _vp, _vp, _u32, _vp], _i),
    "wl_dev_wait_flag": ([_vp, _u32, _vp], _i),
    "wl_bitlinear_i2s_matvec_f32": ([_tv, _fp, _sz, _fp, _sz], _i),
    "wl_bitlinear_i2s_matvec_f32_dbg": ([_tv, _fp, _sz, _fp, _sz, C.POINTER(C.c_int32), _fp,
                                         C.POINTER(C.c_int8)], _i),
    "wl_bitlinear_i2s_gemm_f32": ([_tv, _fp, _sz, _fp, C.POINTER(C.c_int32)], _i),
    "wl_linear_matvec_f32": ([_tv, _fp, _sz, _fp, _sz], _i),
    "wl_compute_logits": ([_fp, _sz, _tv, _u32, _u32, _fp, _sz], _i),
    "wl_argmax": ([_fp, _sz, C.POINTER(C.c_int64)], _i),
    "wl_lm_head_greedy": ([_fp, _sz, _tv, _u32, _u32, C.POINTER(_u32), _fp], _i),
    "wl_dev_quantize_absmax_i8": ([_vp, _u32, _u32, _vp, _vp, _vp], _i),
    "wl_dev_i2s_matvec": ([C.POINTER(WlI2sDevWeight), _u32, _u32, _vp, _vp, _vp], _i),
    "wl_dev_i2s_matvec_f32": ([_vp, C.c_float, _u32, _u32, _vp, _vp, _vp, _vp, _vp], _i),
    "wl_dev_i2s_matvec_fused_f32": ([C.POINTER(WlI2sDevWeight), _u32, _u32, _vp, _vp], _i),
    "wl_dev_i2s_scan_code3": ([_vp, _sz, _vp, _vp], _i),
    "wl_i2s_gemm_workspace_bytes": ([_u32, _u32], _sz),
    "wl_dev_i2s_gemm_f32": ([_vp, C.c_float, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _u32, _vp], _i),
    "wl_i2s_expanded_bytes": ([_u32, _u32], _sz),
    "wl_dev_i2s_expand": ([_vp, _u32, _u32, _vp, _vp], _i),
    "wl_dev_i2s_gemm_s8_f32": ([_vp, C.c_float, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp], _i),
    "wl_i2s_stream_plan_create": ([C.POINTER(WlI2sStreamOp), _u32, C.POINTER(_vp)], _i),
    "wl_dev_i2s_stream_run": ([_vp, _vp], _i),
    "wl_i2s_stream_plan_destroy": ([_vp], _i),
    "wl_dev_i2s_matvec_f32_noalloc": ([_vp, C.c_float, _u32, _u32, _vp, _vp, _vp], _i),
    "wl_q6k_packed_bytes": ([_u32, _u32], _sz),
    "wl_dev_q6k_repack": ([_vp, _u32, _u32, _vp, _vp], _i),
    "wl_q6k_scratch_bytes": ([_u32], _sz),
    "wl_dev_q6k_lm_head": ([_vp, _u32, _u32, _vp, _u32, _vp, _vp, _vp, _vp], _i),
    "wl_q8_0_packed_bytes": ([_u32, _u32], _sz),
    "wl_dev_q8_0_repack": ([_vp, _u32, _u32, _vp, _vp], _i),
    "wl_dev_q8_0_matvec": ([_vp, _u32, _u32, _vp, _vp, _vp], _i),
    "wl_bitnet_create": ([C.POINTER(WlBitnetConfig), C.POINTER(WlBitnetWeights), C.POINTER(_vp)],
                         _i),
    "wl_bitnet_create_tp": ([C.POINTER(WlBitnetConfig), C.POINTER(WlBitnetWeights), _vp,
                             C.POINTER(_vp)], _i),
    "wl_bitnet_tp_sym_bytes": ([C.POINTER(WlBitnetConfig)], _sz),
    "wl_bitnet_destroy": ([_vp], _i),
    "wl_bitnet_reset": ([_vp], _i),
    "wl_bitnet_position": ([_vp], _u32),
    "wl_bitnet_uses_persistent_kernel": ([_vp], _i),
    "wl_bitnet_forward": ([_vp, _u32, _u32, _fp], _i),
    "wl_bitnet_prefill": ([_vp, C.POINTER(_u32), _u32], _i),
    "wl_bitnet_decode": ([_vp, _u32, C.POINTER(_u32), _fp, _fp], _i),
    "wl_bitnet_generate": ([_vp, C.POINTER(_u32), _u32, _u32, C.POINTER(_u32), _fp], _i),
    "wl_llama_batch_create": ([C.POINTER(WlBitnetConfig), C.POINTER(WlLlamaWeights), _u32,
                               C.POINTER(_vp)], _i),
    "wl_llama_batch_destroy": ([_vp], _i),
    "wl_llama_batch_reset": ([_vp], _i),
    "wl_llama_batch_position": ([_vp, _u32], _u32),
    "wl_llama_batch_attention_splits": ([_vp], _u32),
    "wl_llama_batch_set_tokens_per_cta": ([_vp, _u32], _i),
    "wl_llama_batch_prefill": ([_vp, C.POINTER(_u32), C.POINTER(_u32)], _i),
    "wl_llama_batch_decode": ([_vp, _u32, C.POINTER(_u32), _fp, _fp], _i),
    "wl_llama_batch_generate": ([_vp, C.POINTER(_u32), C.POINTER(_u32), _u32, C.POINTER(_u32),
                                 _fp], _i),
    "wl_gguf_open": ([_vp, _sz, C.POINTER(_vp)], _i),
    "wl_gguf_close": ([_vp], _i),
    "wl_gguf_version": ([_vp], _u32),
    "wl_gguf_alignment": ([_vp], C.c_uint64),
    "wl_gguf_tensor_count": ([_vp], C.c_uint64),
    "wl_gguf_tensor": ([_vp, C.c_uint64, _tv], _i),
    "wl_gguf_find_tensor": ([_vp, C.c_char_p, _tv], _i),
    "wl_gguf_get_u64": ([_vp, C.c_char_p, C.POINTER(C.c_uint64)], _i),
    "wl_gguf_get_f32": ([_vp, C.c_char_p, _fp], _i),
    "wl_gguf_get_str": ([_vp, C.c_char_p, C.POINTER(C.c_char_p)], _i),
    "wl_gguf_array_len": ([_vp, C.c_char_p], C.c_uint64),
    "wl_gguf_model_config": ([_vp, C.POINTER(WlBitnetConfig), C.POINTER(_u32)], _i),
    "wl_bitnet_create_from_gguf": ([_vp, _u32, _u32, _u32, C.POINTER(_vp)], _i),
    "wl_llama_batch_create_from_gguf": ([_vp, _u32, _u32, _u32, C.POINTER(_vp)], _i),
    "wl_tp_create": ([_i, _i, _sz, C.POINTER(_vp), C.POINTER(C.c_uint8)], _i),
    "wl_tp_connect": ([_vp, C.POINTER(C.c_uint8)], _i),
    "wl_tp_buffer": ([_vp, _sz], _vp),
    "wl_tp_destroy": ([_vp], _i),
    "wl_tp_wait": ([_vp, _vp], _i),
    "wl_tp_i2s_matvec_fused_f32": ([_vp, C.POINTER(WlI2sDevWeight), C.POINTER(_u32), _u32, _u32,
                                    _vp, _i, _vp], _i),
    "wl_tp_i2s_stream_run": ([_vp, _vp, _vp], _i),
    "wl_tp_q6k_lm_head_greedy": ([_vp, _vp, _u32, _u32, _u32, _vp, _u32, _vp, _vp, _vp], _i),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m project_willamette_b200.build` "
                "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in PROTOTYPES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def header_functions() -> list[str]:
    """Names of the functions include/willamette_b200.h declares."""
    import re
    src = open(HEADER_PATH).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(wl_[a-z0-9_]+)\s*\(", src)))

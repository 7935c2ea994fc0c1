"""ctypes binding of libb200fp8.so (the C ABI declared in include/b200fp8.h).

The library is built in-tree (``make -C airi-summer-kernel-evo_b200``) and loaded from
this package directory.  There is no fallback: if the shared object is missing or fails
to load, every op raises.  The CPU oracle under ``oracle/`` is test infrastructure and is
never reached from here.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb200fp8.so")

B2F_OK = 0
B2F_ERR_ARG = 1
B2F_ERR_UNSUPPORTED = 2
B2F_ERR_CUDA = 3
B2F_ERR_TIMEOUT = 4
B2F_ERR_NCCL = 5

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_E4M3 = 2
DTYPE_F16 = 3

ACT_NONE = 0
ACT_RELU = 1
ACT_GELU_TANH = 2
ACT_LEAKY_RELU = 3
ACT_SILU = 4

GEMM_STORE = 0
GEMM_ROWSUM = 1

NORM_RMS = 0
NORM_LAYER = 1
SCALE_STATIC, SCALE_DYNAMIC, SCALE_DYNAMIC_STATS, SCALE_DYNAMIC_APPLY = 0, 1, 2, 3
NORM_SCHEDULE_AUTO, NORM_SCHEDULE_ROWGROUP = 0, 1


class B2FError(RuntimeError):
    """Raised when a b2f_* entry point returns a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"b200fp8 error {code}: {message}")
        self.code = code


class GemmArgs(ctypes.Structure):
    """Mirror of ``b2f_gemm_args`` (include/b200fp8.h)."""

    _fields_ = [
        ("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int),
        ("a", ctypes.c_void_p), ("lda", ctypes.c_longlong),
        ("b", ctypes.c_void_p), ("ldb", ctypes.c_longlong),
        ("alpha", ctypes.c_float), ("alpha_ptr", ctypes.c_void_p),
        ("col_scale", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("pre_mul", ctypes.c_float), ("pre_add", ctypes.c_float),
        ("act", ctypes.c_int), ("act_param", ctypes.c_float),
        ("post_mul", ctypes.c_float),
        ("residual", ctypes.c_void_p), ("residual_dtype", ctypes.c_int),
        ("residual_ld", ctypes.c_longlong), ("residual_scale", ctypes.c_float),
        ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int),
        ("out_ld", ctypes.c_longlong), ("out_scale", ctypes.c_float),
        ("amax", ctypes.c_void_p),
        ("mode", ctypes.c_int),
        ("tile_n", ctypes.c_int),
        ("splits", ctypes.c_int),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_longlong),
        ("gate", ctypes.c_void_p), ("gate_dtype", ctypes.c_int),
        ("gate_ld", ctypes.c_longlong),
    ]


class NormArgs(ctypes.Structure):
    """Mirror of ``b2f_norm_args`` (include/b200fp8.h)."""

    _fields_ = [
        ("rows", ctypes.c_int), ("cols", ctypes.c_int),
        ("x", ctypes.c_void_p), ("x_dtype", ctypes.c_int), ("x_scale", ctypes.c_float),
        ("x_ld", ctypes.c_longlong),
        ("residual", ctypes.c_void_p), ("residual_dtype", ctypes.c_int),
        ("residual_ld", ctypes.c_longlong),
        ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("weight_dtype", ctypes.c_int), ("weight_offset", ctypes.c_float),
        ("kind", ctypes.c_int), ("eps", ctypes.c_float),
        ("h_out", ctypes.c_void_p), ("h_dtype", ctypes.c_int), ("h_ld", ctypes.c_longlong),
        ("y_out", ctypes.c_void_p), ("y_ld", ctypes.c_longlong),
        ("q_out", ctypes.c_void_p), ("q_ld", ctypes.c_longlong),
        ("q_scale", ctypes.c_float), ("dynamic_scale", ctypes.c_int),
        ("amax", ctypes.c_void_p), ("scale_out", ctypes.c_void_p),
        ("schedule", ctypes.c_int), ("row_stats", ctypes.c_void_p),
    ]


class LnRowsArgs(ctypes.Structure):
    """Mirror of ``b2f_lnrows_args`` (include/b200fp8.h)."""

    _fields_ = [
        ("rows", ctypes.c_int), ("cols", ctypes.c_longlong),
        ("x", ctypes.c_void_p), ("x_dtype", ctypes.c_int), ("x_ld", ctypes.c_longlong),
        ("x_scale", ctypes.c_float), ("weight", ctypes.c_void_p), ("bias", ctypes.c_void_p),
        ("eps", ctypes.c_float), ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int),
        ("out_ld", ctypes.c_longlong), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_longlong),
    ]


class QuantArgs(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int), ("cols", ctypes.c_int),
        ("x", ctypes.c_void_p), ("x_dtype", ctypes.c_int), ("x_ld", ctypes.c_longlong),
        ("q", ctypes.c_void_p), ("q_ld", ctypes.c_longlong),
        ("dynamic", ctypes.c_int), ("scale", ctypes.c_float),
        ("amax", ctypes.c_void_p), ("scale_out", ctypes.c_void_p),
        ("scale_mul", ctypes.c_void_p), ("scale_prod_out", ctypes.c_void_p),
    ]


class AttnArgs(ctypes.Structure):
    """Mirror of ``b2f_attn_args`` (include/b200fp8.h)."""

    _fields_ = [
        ("batch", ctypes.c_int), ("seq", ctypes.c_int), ("hq", ctypes.c_int),
        ("hkv", ctypes.c_int), ("head_dim", ctypes.c_int), ("causal", ctypes.c_int),
        ("q", ctypes.c_void_p), ("q_ld", ctypes.c_longlong), ("q_scale", ctypes.c_float),
        ("k", ctypes.c_void_p), ("k_ld", ctypes.c_longlong), ("k_scale", ctypes.c_float),
        ("v", ctypes.c_void_p), ("v_ld", ctypes.c_longlong), ("v_scale", ctypes.c_float),
        ("sm_scale", ctypes.c_float),
        ("gate", ctypes.c_void_p), ("gate_dtype", ctypes.c_int), ("gate_ld", ctypes.c_longlong),
        ("gate_head_stride", ctypes.c_longlong), ("gate_scale", ctypes.c_float),
        ("ctx", ctypes.c_void_p), ("ctx_ld", ctypes.c_longlong), ("ctx_scale", ctypes.c_float),
        ("v_dtype", ctypes.c_int),
    ]


class Gpt2BlockArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("seq", ctypes.c_int), ("d_model", ctypes.c_int),
        ("heads", ctypes.c_int), ("mlp", ctypes.c_int),
        ("hidden", ctypes.c_void_p), ("hidden_dtype", ctypes.c_int),
        ("hidden_ld", ctypes.c_longlong), ("hidden_scale", ctypes.c_float),
        ("qkv_w", ctypes.c_void_p), ("qkv_s", ctypes.c_float), ("qkv_b", ctypes.c_void_p),
        ("out_w", ctypes.c_void_p), ("out_s", ctypes.c_float), ("out_b", ctypes.c_void_p),
        ("fc_w", ctypes.c_void_p), ("fc_s", ctypes.c_float), ("fc_b", ctypes.c_void_p),
        ("proj_w", ctypes.c_void_p), ("proj_s", ctypes.c_float), ("proj_b", ctypes.c_void_p),
        ("ln1_w", ctypes.c_void_p), ("ln1_b", ctypes.c_void_p), ("ln2_w", ctypes.c_void_p),
        ("ln2_b", ctypes.c_void_p), ("eps", ctypes.c_float),
        ("norm_scale", ctypes.c_float), ("qkv_scale", ctypes.c_float),
        ("ctx_scale", ctypes.c_float), ("mlp_scale", ctypes.c_float),
        ("causal", ctypes.c_int), ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
        ("residual_dtype", ctypes.c_int), ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int),
        ("out_ld", ctypes.c_longlong), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_longlong),
    ]


class QwenBlockArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("seq", ctypes.c_int), ("hidden", ctypes.c_int),
        ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("rotary_dim", ctypes.c_int), ("interleaved", ctypes.c_int),
        ("hidden_in", ctypes.c_void_p), ("hidden_dtype", ctypes.c_int),
        ("hidden_ld", ctypes.c_longlong), ("hidden_scale", ctypes.c_float),
        ("qgkv_w", ctypes.c_void_p), ("qgkv_col_scale", ctypes.c_void_p),
        ("o_w", ctypes.c_void_p), ("o_s", ctypes.c_float),
        ("in_norm_w", ctypes.c_void_p), ("q_norm_w", ctypes.c_void_p),
        ("k_norm_w", ctypes.c_void_p), ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p), ("eps", ctypes.c_float), ("norm_scale", ctypes.c_float),
        ("qkv_scale", ctypes.c_float), ("ctx_scale", ctypes.c_float),
        ("add_residual", ctypes.c_int), ("post_norm_w", ctypes.c_void_p),
        ("mlp_gu_w", ctypes.c_void_p), ("mlp_gu_col_scale", ctypes.c_void_p),
        ("inter", ctypes.c_int), ("mlp_down_w", ctypes.c_void_p),
        ("mlp_down_s", ctypes.c_float), ("mlp_proj_scale", ctypes.c_float),
        ("mlp_act_scale", ctypes.c_float), ("residual_dtype", ctypes.c_int),
        ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int), ("out_ld", ctypes.c_longlong),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_longlong),
    ]


class RopeArgs(ctypes.Structure):
    """Mirror of ``b2f_rope_args`` (include/b200fp8.h)."""

    _fields_ = [
        ("rows", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("in", ctypes.c_void_p), ("in_ld", ctypes.c_longlong),
        ("in_head_stride", ctypes.c_longlong), ("in_scale", ctypes.c_float),
        ("weight", ctypes.c_void_p), ("weight_offset", ctypes.c_float), ("eps", ctypes.c_float),
        ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("rotary_dim", ctypes.c_int),
        ("seq", ctypes.c_int),
        ("out", ctypes.c_void_p), ("out_ld", ctypes.c_longlong), ("out_scale", ctypes.c_float),
    ]


class HeadPrepArgs(ctypes.Structure):
    """Mirror of ``b2f_head_prep_args`` (include/b200fp8.h)."""

    _fields_ = [
        ("q_off", ctypes.c_int), ("q_head_stride", ctypes.c_int), ("q_heads", ctypes.c_int),
        ("k_off", ctypes.c_int), ("k_heads", ctypes.c_int),
        ("v_off", ctypes.c_int), ("v_heads", ctypes.c_int),
        ("q_out", ctypes.c_void_p), ("q_ld", ctypes.c_longlong),
        ("k_out", ctypes.c_void_p), ("k_ld", ctypes.c_longlong),
        ("v_out", ctypes.c_void_p), ("v_ld", ctypes.c_longlong), ("v_dtype", ctypes.c_int),
        ("q_norm_w", ctypes.c_void_p), ("k_norm_w", ctypes.c_void_p),
        ("weight_offset", ctypes.c_float), ("eps", ctypes.c_float),
        ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p), ("seq", ctypes.c_int),
        ("out_scale", ctypes.c_float),
    ]


class Op(ctypes.Structure):
    """Mirror of ``b2f_op``."""

    _fields_ = [
        ("name", ctypes.c_char_p),
        ("abi_version", ctypes.c_int),
        ("fn", ctypes.c_void_p),
        ("signature", ctypes.c_char_p),
    ]


# Every symbol include/b200fp8.h declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "b2f_version", "b2f_last_error", "b2f_num_sms", "b2f_status_read",
    "b2f_debug_bounded_wait", "b2f_gemm_args_init", "b2f_gemm_fp8", "b2f_gemm_pair_capacity",
    "b2f_gemm_workspace_bytes", "b2f_gemm_fp8_static", "b2f_gemm_fp8_head_prep",
    "b2f_norm_args_init", "b2f_norm_quant", "b2f_norm_plan", "b2f_attn_args_init", "b2f_attention_fp8",
    "b2f_head_norm_rope", "b2f_attn_prep", "b2f_fp8_to_bf16", "b2f_fp8_to_f16", "b2f_swiglu_fp8",
    "b2f_quant_args_init", "b2f_quantize_fp8",
    "b2f_lnrows_args_init", "b2f_layer_norm_rows_workspace_bytes", "b2f_layer_norm_rows",
    "b2f_gpt2_block_args_init", "b2f_gpt2_block_workspace_bytes", "b2f_gpt2_block",
    "b2f_qwen_block_args_init", "b2f_qwen_block_workspace_bytes", "b2f_qwen_block",
    "b2f_registry_lookup", "b2f_registry_size", "b2f_registry_at",
)

_lib = None


def _declare(lib: ctypes.CDLL) -> None:
    vp = ctypes.c_void_p
    lib.b2f_version.restype = ctypes.c_int
    lib.b2f_last_error.restype = ctypes.c_char_p
    lib.b2f_num_sms.restype = ctypes.c_int
    lib.b2f_status_read.argtypes = [ctypes.c_int]
    lib.b2f_status_read.restype = ctypes.c_int
    lib.b2f_debug_bounded_wait.argtypes = [ctypes.c_ulonglong, vp]
    lib.b2f_debug_bounded_wait.restype = ctypes.c_int
    lib.b2f_gemm_args_init.argtypes = [ctypes.POINTER(GemmArgs)]
    lib.b2f_gemm_args_init.restype = None
    lib.b2f_gemm_fp8.argtypes = [ctypes.POINTER(GemmArgs), vp]
    lib.b2f_gemm_fp8.restype = ctypes.c_int
    lib.b2f_gemm_pair_capacity.restype = ctypes.c_int
    lib.b2f_gemm_fp8_static.argtypes = [ctypes.POINTER(GemmArgs), vp]
    lib.b2f_gemm_fp8_head_prep.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(HeadPrepArgs), vp]
    lib.b2f_gemm_fp8_head_prep.restype = ctypes.c_int
    lib.b2f_gemm_fp8_static.restype = ctypes.c_int
    lib.b2f_gemm_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
    lib.b2f_gemm_workspace_bytes.restype = ctypes.c_longlong
    lib.b2f_norm_args_init.argtypes = [ctypes.POINTER(NormArgs)]
    lib.b2f_norm_args_init.restype = None
    lib.b2f_norm_quant.argtypes = [ctypes.POINTER(NormArgs), vp]
    lib.b2f_norm_quant.restype = ctypes.c_int
    lib.b2f_quant_args_init.argtypes = [ctypes.POINTER(QuantArgs)]
    lib.b2f_quant_args_init.restype = None
    lib.b2f_quantize_fp8.argtypes = [ctypes.POINTER(QuantArgs), vp]
    lib.b2f_quantize_fp8.restype = ctypes.c_int
    for nm, st in (("gpt2", Gpt2BlockArgs), ("qwen", QwenBlockArgs)):
        getattr(lib, f"b2f_{nm}_block_args_init").argtypes = [ctypes.POINTER(st)]
        getattr(lib, f"b2f_{nm}_block_args_init").restype = None
        getattr(lib, f"b2f_{nm}_block_workspace_bytes").argtypes = [ctypes.POINTER(st)]
        getattr(lib, f"b2f_{nm}_block_workspace_bytes").restype = ctypes.c_longlong
        getattr(lib, f"b2f_{nm}_block").argtypes = [ctypes.POINTER(st), vp]
        getattr(lib, f"b2f_{nm}_block").restype = ctypes.c_int
    lib.b2f_lnrows_args_init.argtypes = [ctypes.POINTER(LnRowsArgs)]
    lib.b2f_lnrows_args_init.restype = None
    lib.b2f_layer_norm_rows_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_longlong]
    lib.b2f_layer_norm_rows_workspace_bytes.restype = ctypes.c_longlong
    lib.b2f_layer_norm_rows.argtypes = [ctypes.POINTER(LnRowsArgs), vp]
    lib.b2f_layer_norm_rows.restype = ctypes.c_int
    lib.b2f_norm_plan.argtypes = [ctypes.POINTER(NormArgs)]
    lib.b2f_norm_plan.restype = ctypes.c_int
    lib.b2f_attn_args_init.argtypes = [ctypes.POINTER(AttnArgs)]
    lib.b2f_attn_args_init.restype = None
    lib.b2f_attention_fp8.argtypes = [ctypes.POINTER(AttnArgs), vp]
    lib.b2f_attention_fp8.restype = ctypes.c_int
    lib.b2f_head_norm_rope.argtypes = [ctypes.POINTER(RopeArgs), vp]
    lib.b2f_head_norm_rope.restype = ctypes.c_int
    lib.b2f_attn_prep.argtypes = [ctypes.POINTER(RopeArgs), ctypes.POINTER(RopeArgs), vp,
                                  ctypes.c_longlong, vp, ctypes.c_longlong, ctypes.c_int,
                                  ctypes.c_int, vp]
    lib.b2f_attn_prep.restype = ctypes.c_int
    lib.b2f_fp8_to_bf16.argtypes = [vp, ctypes.c_longlong, vp, ctypes.c_longlong, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_float, vp]
    lib.b2f_fp8_to_bf16.restype = ctypes.c_int
    lib.b2f_fp8_to_f16.argtypes = lib.b2f_fp8_to_bf16.argtypes
    lib.b2f_fp8_to_f16.restype = ctypes.c_int
    lib.b2f_swiglu_fp8.argtypes = [vp, ctypes.c_longlong, vp, ctypes.c_longlong, vp,
                                   ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                   ctypes.c_float, vp]
    lib.b2f_swiglu_fp8.restype = ctypes.c_int
    lib.b2f_registry_lookup.argtypes = [ctypes.c_char_p]
    lib.b2f_registry_lookup.restype = ctypes.POINTER(Op)
    lib.b2f_registry_size.restype = ctypes.c_int
    lib.b2f_registry_at.argtypes = [ctypes.c_int]
    lib.b2f_registry_at.restype = ctypes.POINTER(Op)


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libb200fp8.so not built at {LIB_PATH}; run `make -C airi-summer-kernel-evo_b200`"
                " or __graft_entry__.build()")
        handle = ctypes.CDLL(LIB_PATH)
        _declare(handle)
        _lib = handle
    return _lib


def check(code: int) -> None:
    if code != B2F_OK:
        msg = lib().b2f_last_error().decode(errors="replace")
        raise B2FError(code, msg)


def device_status(reset: bool = False) -> int:
    """Device status word (0 = ok; B2F_DEV_* codes after a bounded wait expired)."""
    return int(lib().b2f_status_read(1 if reset else 0))

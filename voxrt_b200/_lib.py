"""ctypes binding of libvxg.so, the in-tree sm_100a kernel library. There is no CPU fallback: if the library is
missing or cannot load, every call raises."""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvxg.so")

VXG_OK, VXG_ERR_ARG, VXG_ERR_CUDA, VXG_ERR_TIMEOUT, VXG_ERR_OOM, VXG_ERR_UNSUPPORTED = range(6)
STATUS_NAMES = {0: "OK", 1: "ERR_ARG", 2: "ERR_CUDA", 3: "ERR_TIMEOUT", 4: "ERR_OOM", 5: "ERR_UNSUPPORTED"}

_P, _I, _F, _Z = C.c_void_p, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes): every symbol include/vxg.h declares
SIGNATURES = {
    "vxg_last_error": (C.c_char_p, []),
    "vxg_version": (C.c_char_p, []),
    "vxg_device_status": (_I, [C.POINTER(_I)]),
    "vxg_ternary_codes_bytes": (_Z, [_I, _I]),
    "vxg_ternary_scales_count": (_Z, [_I, _I, _I]),
    "vxg_ternary_out_pad": (_I, [_I]),
    "vxg_ternary_repack": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "vxg_gemm_ternary_i8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P]),
    "vxg_ternary_i8_bytes": (_Z, [_I, _I]),
    "vxg_ternary_repack_i8": (_I, [_P, _P, _I, _I, _I, _P, _P]),
    "vxg_gemm_ternary_i8w": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P]),
    "vxg_gemm_ternary_silu_q": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "vxg_gemm_ternary_silu_q_w": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P]),
    "vxg_gemm_ternary_qkv_quant": (_I, [_P, _P, _P, _P, _I, _I, _I, _I] + [_P] * 10),
    "vxg_glu_source_row": (_I, [_I, _I]),
    "vxg_gemm_ternary_glu": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P]),
    "vxg_quantize_rows": (_I, [_P, _I, _I, _I, _P, _P, _P]),
    "vxg_ln_quant": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P]),
    "vxg_fold_bn": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _P]),
    "vxg_conv_workspace_bytes": (_Z, [_I, _I]),
    "vxg_conv_glu_dw_silu_quant": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _I, _P, _P, _P, _P, _Z, _P]),
    "vxg_conv_glu_dw_silu_quant_static": (_I, [_P, _I, _P, _P, _I, _P, _P, _I, _I, _P, _P, _P, _P]),
    "vxg_sub_out_frames": (_I, [_I]),
    "vxg_subsampling_workspace_bytes": (_Z, [_P, _I, _I]),
    "vxg_subsampling": (_I, [_P, _P, _I, _I] + [_P] * 12 + [_I, _P, _P, _Z, _P]),
    "vxg_linear_f32": (_I, [_P, _I, _I, _P, _P, _I, _I, _P, _P]),
    "vxg_encoder_create": (_I, [_P, _I, C.POINTER(_P)]),
    "vxg_encoder_destroy": (None, [_P]),
    "vxg_encoder_out_frames": (_I, [_I]),
    "vxg_encoder_forward_feats": (_I, [_P, _P, _I, _P, _Z, C.POINTER(_I)]),
    "vxg_encoder_forward_batch": (_I, [_P, _P, _P, _I, _P, _P]),
    "vxg_encoder_forward_device": (_I, [_P, _P, _P, _I, _P, _P, _P]),
    "vxg_encoder_forward_layers_device": (_I, [_P, _P, _P, _I, _P, _P]),
    "vxg_encoder_set_profiling": (_I, [_P, _I]),
    "vxg_encoder_profile": (_I, [_P, C.POINTER(C.c_double), C.POINTER(_I), C.POINTER(C.c_double)]),
    "vxg_kernel_launches": (C.c_ulonglong, []),
    "vxg_attention_workspace_bytes": (_Z, [_I, _I, _I, _I]),
    "vxg_attention_i8": (_I, [_P, _I, _P, _I, _P, _P, _I, _P, _P, _I, _I, _F, _P, _P, _P, _P, _Z, _P]),
    "vxg_tdt_create": (_I, [_P, C.POINTER(_P)]),
    "vxg_tdt_destroy": (None, [_P]),
    "vxg_tdt_project_device": (_I, [_P, _P, _I, _P, _P]),
    "vxg_tdt_greedy": (_I, [_P, _P, _I, _P, _Z, C.POINTER(_Z)]),
    "vxg_tdt_greedy_batch": (_I, [_P, _I, _P, _P, _P, _P, _P, _I]),
    "vxg_tdt_pred_step": (_I, [_P, _I, _P, _P, _P, _P, _P]),
    "vxg_tdt_joint": (_I, [_P, _P, _P, _P]),
    "vxg_tdt_greedy_device": (_I, [_P, _I, _P, _P, _P, _P, _P, _P]),
    "vxg_tdt_pred_step_device": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P]),
    "vxg_tdt_joint_device": (_I, [_P, _I, _P, _P, _P, _P]),
    "vxg_encoder_subsample_device": (_I, [_P, _P, _P, _I, _P, _P, _P]),
    "vxg_frontend_info": (_I, [_P, _P, _P]),
    "vxg_vad_create": (_I, [_P, _P]),
    "vxg_vad_create_from_model": (_I, [_P, _I, _P]),
    "vxg_vad_destroy": (None, [_P]),
    "vxg_vad_info": (_I, [_P, _P, _P, _P, _P]),
    "vxg_vad_probs_device": (_I, [_P, _P, _P, _I, _P, _P]),
    "vxg_segment_cfg_default": (None, [_P]),
    "vxg_segment": (_I, [_P, _I, _P, _P, _Z, _P]),
    "vxg_longform_cfg_default": (None, [_P]),
    "vxg_longform_create": (_I, [_P, _P, _P, _P, _P, _P]),
    "vxg_longform_create_with_vad": (_I, [_P, _P, _P, _P]),
    "vxg_longform_destroy": (None, [_P]),
    "vxg_longform_push": (_I, [_P, _P, C.c_longlong, _P, _Z, _P]),
    "vxg_longform_flush": (_I, [_P, _P, _Z, _P]),
    "vxg_longform_ranges": (_I, [_P, _P, _Z, _P]),
    "vxg_longform_emissions": (_I, [_P, _P, _Z, _P]),
    "vxg_longform_stats": (_I, [_P, _P, _P, _P]),
    "vxg_transcribe_long": (_I, [_P, _P, _P, _P, _P, C.c_longlong, _P, _P, _Z, _P, _P, _Z, _P]),
    "vxg_math_host": (_I, [_I, _P, _Z, _P]),
    "vxg_math_device": (_I, [_I, _P, _Z, _P, _P]),
    "vxg_mel_filterbank": (_I, [_I, _I, _I, _P]),
    "vxg_frontend_frames": (_I, [C.c_longlong]),
    "vxg_frontend_create": (_I, [_I, _I, _I, C.POINTER(_P)]),
    "vxg_frontend_destroy": (None, [_P]),
    "vxg_frontend_device": (_I, [_P, _P, _P, _I, _I, _P, _P, _P]),
    "vxg_model_open": (_I, [C.c_char_p, C.POINTER(_P)]),
    "vxg_model_close": (None, [_P]),
    "vxg_model_validate": (_I, [_P, C.c_char_p, _Z]),
    "vxg_model_config": (_I, [_P, _P]),
    "vxg_model_tensor": (_I, [_P, C.c_char_p, C.POINTER(_I), C.POINTER(C.c_int64), C.POINTER(_I),
                              C.POINTER(_P), C.POINTER(_Z)]),
    "vxg_model_tensor_f32": (_I, [_P, C.c_char_p, _P, _Z]),
    "vxg_encoder_create_from_model": (_I, [_P, _I, _I, C.POINTER(_P)]),
    "vxg_tdt_create_from_model": (_I, [_P, _I, C.POINTER(_P)]),
}


class VxgError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"vxg {STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def lib():
    """Load libvxg.so (building it first if this checkout has nvcc and no library yet)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import build as _build

            _build.build()
        _lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(_lib, name)
            f.restype = res
            f.argtypes = args
    return _lib


def check(status: int):
    if status != VXG_OK:
        raise VxgError(status, lib().vxg_last_error().decode(errors="replace"))


def device_status() -> int:
    """Synchronise the current device and return (and clear) its kernel status word (0 = fine)."""
    code = C.c_int(0)
    check(lib().vxg_device_status(C.byref(code)))
    return code.value


def check_device():
    code = device_status()
    if code:
        raise VxgError(VXG_ERR_TIMEOUT, f"a kernel reported device status 0x{code:x} (bounded wait expired)")

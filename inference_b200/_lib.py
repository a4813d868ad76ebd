"""ctypes binding of libq3_sm100a.so (the C ABI in include/q3_sm100a.h).

The library must exist: there is no fallback path.  Build it with
``python -m inference_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libq3_sm100a.so")

Q3_OK = 0
STATUS = {0: "Q3_OK", 1: "Q3_ERR_INVALID", 2: "Q3_ERR_CUDA", 3: "Q3_ERR_UNSUPPORTED", 4: "Q3_ERR_OOM",
          5: "Q3_ERR_DEVICE", 6: "Q3_ERR_NCCL"}

# Every exported symbol declared in include/q3_sm100a.h, with ctypes signatures.
_vp, _sz, _u16p, _u32p, _i32p = C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p
_szp = C.POINTER(C.c_size_t)
SIGNATURES = {
    "q3_last_error": (C.c_char_p, []),
    "q3_version": (C.c_int, []),
    "q3_embedding": (C.c_int, [_u16p, _sz, _sz, C.c_uint32, _u16p, _vp]),
    "q3_gemv": (C.c_int, [_u16p, _u16p, _u16p, _sz, _sz, _vp]),
    "q3_gemm": (C.c_int, [_u16p, _u16p, _u16p, _sz, _sz, _sz, _vp]),
    "q3_nvfp4_packed_bytes": (_sz, [_sz, _sz]),
    "q3_nvfp4_packed_offset": (_sz, [_sz, _sz, C.c_int, _sz, _sz, C.c_int]),
    "q3_quantize_nvfp4": (C.c_int, [_u16p, _sz, _sz, _vp, _vp, _vp]),
    "q3_dequant_nvfp4": (C.c_int, [_vp, _vp, _sz, _sz, _u16p, _vp]),
    "q3_gemv_nvfp4": (C.c_int, [_u16p, _vp, _vp, _u16p, _sz, _sz, _vp]),
    "q3_quantize_e4m3": (C.c_int, [_u16p, _sz, _sz, _sz, _sz, _vp, _vp, _vp]),
    "q3_gemv_e4m3": (C.c_int, [_u16p, _vp, _vp, _u16p, _sz, _sz, _vp]),
    "q3_e4m3_packed_bytes": (_sz, [_sz, _sz]),
    "q3_e4m3_packed_offset": (_sz, [_sz, _sz, C.c_int, _sz, _sz]),
    "q3_pack_e4m3": (C.c_int, [_vp, _sz, _sz, _vp, _vp]),
    "q3_rmsnorm": (C.c_int, [_u16p, _u16p, _u16p, _sz, C.c_float, _vp]),
    "q3_rmsnorm_add": (C.c_int, [_u16p, _u16p, _u16p, _u16p, _sz, C.c_float, _vp]),
    "q3_rope": (C.c_int, [_u16p, _vp, _vp, _sz, _sz, _sz, _vp]),
    "q3_qk_norm_rope": (C.c_int, [_u16p, _u16p, _u16p, _u16p, _vp, _vp, _sz, _sz, _sz, _sz, C.c_float, _vp]),
    "q3_attention_workspace_bytes": (_sz, [_sz, _sz, _sz]),
    "q3_attention": (C.c_int, [_u16p, _u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, _vp, _sz, _vp]),
    "q3_attention_paged": (C.c_int, [_u16p, _u16p, _u16p, _i32p, _u16p, _sz, _sz, _sz, _sz, _sz, _vp, _sz, _vp]),
    "q3_add": (C.c_int, [_u16p, _u16p, _u16p, _sz, _vp]),
    "q3_silu_mul": (C.c_int, [_u16p, _u16p, _u16p, _sz, _vp]),
    "q3_argmax": (C.c_int, [_u16p, _sz, _u32p, _vp]),
    "q3_argmax_noalloc": (C.c_int, [_u16p, _sz, _u32p, _vp]),
    "q3_rope_tables": (C.c_int, [_sz, _sz, C.c_float, _vp, _vp]),
    "q3_fill_normal": (C.c_int, [_u16p, C.c_uint64, C.c_uint64, _sz, _sz, _sz, _sz, _sz, _sz, _vp]),
    "q3_prompt_ids": (None, [_u32p, _sz, C.c_uint64, C.c_uint32]),
    "q3_engine_create": (C.c_int, [_vp, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "q3_engine_destroy": (C.c_int, [_vp]),
    "q3_engine_init_synthetic": (C.c_int, [_vp, C.c_uint64]),
    "q3_engine_set_weight": (C.c_int, [_vp, C.c_char_p, _u16p, _sz, _sz]),
    "q3_engine_reset": (C.c_int, [_vp]),
    "q3_engine_set_tokens": (C.c_int, [_vp, _u32p, _sz]),
    "q3_engine_prefill": (C.c_int, [_vp, _sz]),
    "q3_engine_step": (C.c_int, [_vp, _sz]),
    "q3_engine_sync": (C.c_int, [_vp]),
    "q3_engine_forward": (C.c_int, [_vp, C.c_uint32, C.POINTER(C.c_uint32)]),
    "q3_engine_generate": (C.c_int, [_vp, _u32p, _sz, _sz, C.c_int, _u32p, C.POINTER(C.c_size_t)]),
    "q3_engine_set_position": (C.c_int, [_vp, _sz]),
    "q3_engine_set_tuning": (C.c_int, [_vp, C.c_uint32]),
    "q3_engine_tuning": (C.c_int, [_vp, C.POINTER(C.c_uint32)]),
    "q3_engine_trace": (C.c_int, [_vp, C.c_int, _vp, _sz, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "q3_engine_position": (C.c_int, [_vp, C.POINTER(C.c_size_t)]),
    "q3_engine_logits": (C.c_int, [_vp, _u16p]),
    "q3_engine_argmax_history": (C.c_int, [_vp, _u32p, _sz]),
    "q3_engine_kv_slot": (C.c_int, [_vp, _sz, _sz, _u16p, _u16p]),
    "q3_engine_fill_kv": (C.c_int, [_vp, _sz, C.c_uint64]),
    "q3_engine_kv_read": (C.c_int, [_vp, _sz, _sz, _sz, _u16p, _u16p]),
    "q3_engine_kv_write": (C.c_int, [_vp, _sz, _sz, _sz, _u16p, _u16p]),
    "q3_engine_stream": (C.c_int, [_vp, C.POINTER(C.c_void_p)]),
    "q3_engine_weight_bytes": (_sz, [_vp]),
    "q3_engine_kv_bytes_per_position": (_sz, [_vp]),
    "q3_engine_profile_step": (C.c_int, [_vp, C.c_int, C.POINTER(C.c_double), C.POINTER(C.c_size_t),
                                         C.POINTER(C.c_double)]),
    "q3_nccl_unique_id": (C.c_int, [_vp]),
    "q3_engine_load_safetensors": (C.c_int, [_vp, C.c_char_p, _szp]),
    "q3_safetensors_list": (C.c_int, [C.c_char_p, C.c_char_p, _sz, _szp]),
    "q3_engine_peer_handle": (C.c_int, [_vp, _vp]),
    "q3_engine_attach_peers": (C.c_int, [_vp, _vp, _sz]),
    "q3_engine_attach_nccl": (C.c_int, [_vp, _vp]),
    "q3_engine_set_comm_timeout": (C.c_int, [_vp, C.c_double]),
    "q3_tokenizer_load": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "q3_tokenizer_destroy": (C.c_int, [_vp]),
    "q3_tokenizer_encode": (C.c_int, [_vp, C.c_char_p, _sz, _u32p, _sz, _szp]),
    "q3_tokenizer_decode": (C.c_int, [_vp, _u32p, _sz, _vp, _sz, _szp]),
    "q3_chat_template": (C.c_int, [C.c_char_p, _sz, _vp, _sz, _szp]),
    "q3_engine_generate_text": (C.c_int, [_vp, _vp, C.c_char_p, _sz, C.POINTER(C.c_void_p), _szp]),
    "q3_string_free": (None, [_vp]),
    "q3_batch_create": (C.c_int, [_vp, C.c_uint32, C.c_uint32, C.POINTER(C.c_void_p)]),
    "q3_batch_destroy": (C.c_int, [_vp]),
    "q3_batch_add": (C.c_int, [_vp, _u32p, _sz, _sz, C.POINTER(C.c_uint32)]),
    "q3_batch_fork": (C.c_int, [_vp, C.c_uint32, C.POINTER(C.c_uint32)]),
    "q3_batch_append": (C.c_int, [_vp, C.c_uint32, _u32p, _sz]),
    "q3_batch_release": (C.c_int, [_vp, C.c_uint32]),
    "q3_batch_step": (C.c_int, [_vp, _sz]),
    "q3_batch_tokens": (C.c_int, [_vp, C.c_uint32, _u32p, _sz, _szp]),
    "q3_batch_logits": (C.c_int, [_vp, C.c_uint32, _u16p]),
    "q3_batch_info": (C.c_int, [_vp, C.c_uint32, _szp, _szp]),
}


class Q3Error(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


_LIB = None


def lib() -> C.CDLL:
    """Load the library (once).  Raises if it was not built: no fallback."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m inference_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(status: int) -> None:
    if status != Q3_OK:
        raise Q3Error(status, lib().q3_last_error().decode(errors="replace"))


class ModelConfig(C.Structure):
    """q3_model_config (include/q3_sm100a.h)."""

    _fields_ = [("hidden", C.c_uint32), ("inter", C.c_uint32), ("layers", C.c_uint32), ("q_heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("vocab", C.c_uint32), ("tied", C.c_uint32),
                ("eps", C.c_float), ("theta", C.c_float), ("capacity", C.c_uint32), ("eos", C.c_uint32),
                ("weight_format", C.c_uint32)]


WEIGHT_FORMATS = {"bf16": 0, "fp8": 1, "nvfp4": 2}  # Q3_WEIGHTS_BF16, Q3_WEIGHTS_FP8_E4M3, Q3_WEIGHTS_NVFP4

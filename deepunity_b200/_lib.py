"""ctypes binding of libdeepunity_cuda.so (include/deepunity_cuda.h).

The library is built in-tree by ``deepunity_b200.build`` (``__graft_entry__.build``).
There is no fallback: if the shared library is missing or fails to load, every
entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdeepunity_cuda.so")

DU_OK, DU_EINVAL, DU_ECUDA, DU_ENOMEM, DU_EBUSY, DU_ENCCL, DU_ENOTFOUND, DU_ESTATE, DU_EIO = range(9)
QUANT_FP16, QUANT_INT8, QUANT_INT4 = 0, 1, 2
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
FLAG_NO_PERSISTENT = 1
FLAG_PERSISTENT = 2
ARCH_QK_NORM, ARCH_SANDWICH, ARCH_GELU, ARCH_ATTN_GATE = 1, 2, 4, 8


class DUError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[du error {code}] {msg}")
        self.code = code


class ModelConfig(C.Structure):
    """du_model_config (include/deepunity_cuda.h)."""
    _fields_ = [("hidden_size", C.c_int32), ("intermediate_size", C.c_int32), ("num_layers", C.c_int32),
                ("num_heads_q", C.c_int32), ("num_heads_kv", C.c_int32), ("head_dim", C.c_int32),
                ("vocab_size", C.c_int32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("embed_scale", C.c_float), ("quant", C.c_int32), ("group_size", C.c_int32),
                ("kv_capacity", C.c_int32), ("max_batch", C.c_int32), ("tp_rank", C.c_int32),
                ("tp_size", C.c_int32), ("tie_embedding", C.c_int32), ("flags", C.c_int32),
                ("kv_quant", C.c_int32), ("arch_flags", C.c_int32), ("sliding_window", C.c_int32),
                ("sliding_pattern", C.c_int32), ("rope_theta_local", C.c_float), ("attn_scale", C.c_float),
                ("rope_rot_dim", C.c_int32), ("reserved", C.c_int32 * 1)]


# name -> (restype, argtypes); every symbol of include/deepunity_cuda.h
P, I, I64, F, U64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64
SIGNATURES = {
    "du_last_error": (C.c_char_p, []),
    "du_version": (C.c_char_p, []),
    "du_init": (I, [I]),
    "du_model_create": (I, [C.POINTER(ModelConfig), C.POINTER(P)]),
    "du_model_load_tensor": (I, [P, C.c_char_p, P, C.c_size_t]),
    "du_model_init_random": (I, [P, U64, F]),
    "du_nccl_unique_id": (I, [P]),
    "du_tp_init": (I, [P, P, I]),
    "du_tp_comm_handle": (I, [P, P]),
    "du_tp_comm_open": (I, [P, P, I]),
    "du_tp_shard_window": (I, [C.POINTER(ModelConfig), C.c_char_p, C.POINTER(C.c_int64)]),
    "du_forward": (I, [P, P, I, I, I, I, P, P]),
    "du_decode_step": (I, [P, P, I, P]),
    "du_decode_loop": (I, [P, P, I, I, P]),
    "du_read_logits": (I, [P, P, I]),
    "du_reset_cache": (I, [P]),
    "du_cache_len": (I, [P, I, C.POINTER(C.c_int)]),
    "du_model_stream": (I, [P, C.POINTER(P)]),
    "du_model_weight_bytes": (I, [P, C.POINTER(C.c_uint64)]),
    "du_model_destroy": (I, [P]),
    "du_model_graph_info": (I, [P, I, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "du_model_kernel_times": (I, [P, I, I, C.POINTER(C.c_float)]),
    "du_model_stage_times": (I, [P, C.POINTER(C.c_float), I, C.POINTER(C.c_int)]),
    "du_gemv_q8": (I, [P, P, I, P, P, I, I, I, I, P]),
    "du_gemv_q4": (I, [P, P, I, P, P, I, I, I, I, P]),
    "du_gemv_f16": (I, [P, P, I, P, I, I, I, P]),
    "du_flash_decode": (I, [P, P, P, P, P, I, I, I, I, I, F, P]),
    "du_kv_write_int8": (I, [P, I, I, I, I, P, P, P]),
    "du_flash_decode_window": (I, [P, P, P, P, P, I, I, I, I, I, F, I, P]),
    "du_model_load_folder": (I, [P, C.c_char_p, C.POINTER(I)]),
    "du_model_save_cache": (I, [P, I, C.c_char_p]),
    "du_model_load_cache": (I, [P, I, C.c_char_p, C.POINTER(I)]),
    "du_model_save_kv": (I, [P, I, C.c_char_p, U64, P, I]),
    "du_model_load_kv": (I, [P, I, C.c_char_p, U64, C.POINTER(I)]),
    "du_kv_file_peek": (I, [C.c_char_p, C.POINTER(I), C.POINTER(U64), C.POINTER(I), C.POINTER(I), C.POINTER(I), P, I,
                            C.POINTER(I)]),
    "du_flash_decode_kv8": (I, [P, P, P, P, P, P, P, I, I, I, I, I, F, P]),
    "du_flash_decode_noalloc": (I, [P, P, P, P, P, I, I, I, I, I, F, P]),
    "du_quantize_int8": (I, [P, I64, I64, P, P, P]),
    "du_quantize_int4": (I, [P, I64, I64, I, P, P, P]),
    "du_rmsnorm": (I, [P, P, P, I, I, F, P]),
    "du_tp_wait_selftest": (I, [C.c_uint, C.POINTER(C.c_int)]),
    "du_dequant": (I, [P, P, P, I, I, I, I64, I, I, P]),
    "du_sample": (I, [P, P, I, I, I, F, I, F, F, P, P]),
    "du_decode_step_sample": (I, [P, P, I, F, I, F, F, P, P]),
    "du_decode_step_sample_ex": (I, [P, P, I, F, I, F, F, F, F, P, P]),
    "du_apply_penalties": (I, [P, I, I, I, P, I, F, F, P]),
    "du_mark_seen": (I, [P, I, I, I, P, P]),
}

_lib = None


def lib():
    """Loads the library (raises if it is missing: there is no CPU fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m deepunity_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().du_last_error().decode(errors="replace")


def check(rc: int):
    if rc != DU_OK:
        raise DUError(rc, last_error())
    return rc


def call(name: str, *args):
    return check(getattr(lib(), name)(*args))

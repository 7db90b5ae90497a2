"""ctypes binding of ``libfgemma.so`` (the C ABI declared in include/fgemma.h).

Loading fails loudly: there is no fallback implementation behind this
module. Build the library with ``python -m ai_b200.build`` (or
``__graft_entry__.build()``) before importing code that needs it.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfgemma.so"

FG_OK = 0
FG_EINVAL = -1
FG_ENOMEM = -2
FG_ECUDA = -3
FG_ETIMEOUT = -4
FG_ESTATE = -5
FG_ENODEV = -6

PREC_SPLIT = 0  # fp32-level: split-fp16 where the weights allow, else split-TF32
PREC_TF32 = 1
PREC_SPLIT_TF32 = 2  # fp32-level, every product split-TF32

ACT_NONE = 0
ACT_RELU = 1
ACT_GELU = 2

DT_F32 = 0
DT_BF16 = 1
DT_F16 = 2

MAX_DENSE = 4

# Phases of fg_model_read_profile (include/fgemma.h FG_PHASE_*).
PHASES = ["embed", "gemm_qkv", "qk_norm_rope", "attention", "gemm_o", "residual",
          "gemm_gate_up", "gemm_down", "pool_head", "widen"]

# fg_model_set_weight_residency modes
WEIGHTS_F32 = 0
WEIGHTS_BF16 = 1

# Every symbol include/fgemma.h declares, with (restype, argtypes).
_i64 = C.c_int64
_fp = C.POINTER(C.c_float)
_vp = C.c_void_p


class Epilogue(C.Structure):
    """fg_epilogue: tensor.Fused (tensor/matmul_fused.go:17-23)."""

    _fields_ = [
        ("bias", _vp),
        ("row_scale", _vp),
        ("act", C.c_int),
        ("mul", _vp),
        ("ldm", _i64),
        ("residual", _vp),
        ("ldr", _i64),
    ]


class Config(C.Structure):
    """fg_config: the encoder's hyper-parameters (models/gemma/config.go:19-37)."""

    _fields_ = [
        ("hidden_size", C.c_int),
        ("intermediate_size", C.c_int),
        ("num_layers", C.c_int),
        ("num_heads", C.c_int),
        ("num_kv_heads", C.c_int),
        ("head_dim", C.c_int),
        ("vocab_size", C.c_int),
        ("window", C.c_int),
        ("rms_norm_eps", C.c_float),
        ("attn_scale", C.c_float),
        ("max_tokens", C.c_int),
        ("sliding", C.POINTER(C.c_int)),
        ("rope_base", C.POINTER(C.c_double)),
        ("num_dense", C.c_int),
        ("dense_in", C.c_int * MAX_DENSE),
        ("dense_out", C.c_int * MAX_DENSE),
        ("dense_tanh", C.c_int * MAX_DENSE),
        ("l2_normalize", C.c_int),
        ("variant", C.c_int),
        ("layer_head_dim", C.POINTER(C.c_int)),
        ("layer_kv_heads", C.POINTER(C.c_int)),
        ("ple_dim", C.c_int),
        ("embedding_dim", C.c_int),
    ]


SIGNATURES = {
    "fg_device_count": (C.c_int, []),
    "fg_last_error": (C.c_char_p, []),
    "fg_malloc": (C.c_int, [C.c_int, _i64, C.POINTER(_vp)]),
    "fg_free": (C.c_int, [C.c_int, _vp]),
    "fg_memcpy_h2d": (C.c_int, [C.c_int, _vp, _vp, _i64]),
    "fg_memcpy_d2h": (C.c_int, [C.c_int, _vp, _vp, _i64]),
    "fg_synchronize": (C.c_int, [C.c_int]),
    "fg_set_wait_limit": (C.c_int, [C.c_int, _i64]),
    "fg_model_create": (C.c_int, [C.POINTER(Config), C.c_int, C.POINTER(_vp)]),
    "fg_model_set_weight": (C.c_int, [_vp, C.c_char_p, C.c_int, C.POINTER(_i64), C.c_int, _vp]),
    "fg_model_finalize": (C.c_int, [_vp, _i64]),
    "fg_model_set_weight_residency": (C.c_int, [_vp, C.c_int]),
    "fg_model_weight_bytes": (C.c_int64, [_vp]),
    "fg_embed_ids": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp]),
    "fg_embed_ids_device": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, _vp, _vp]),
    "fg_embed_many": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, _i64, C.c_int, C.c_int, _vp]),
    "fg_plan_batches": (C.c_int, [_vp, C.c_int, _i64, _vp, _vp]),
    "fg_embed_many_multi": (C.c_int, [C.POINTER(_vp), C.c_int, _vp, _vp, C.c_int, C.c_int, _i64, C.c_int,
                                      C.c_int, _vp]),
    "fg_plan_split": (C.c_int, [_vp, C.c_int, C.c_int, _vp, _vp]),
    "fg_sequence_cost": (C.c_double, [C.c_int]),
    "fg_model_check": (C.c_int, [_vp]),
    "fg_model_destroy": (None, [_vp]),
    "fg_model_set_profiling": (C.c_int, [_vp, C.c_int]),
    "fg_model_read_profile": (C.c_int, [_vp, C.POINTER(C.c_double), C.POINTER(C.c_int64),
                                        C.POINTER(C.c_double), C.c_int]),
    "fg_matmul": (C.c_int, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, C.c_int, _vp, _i64,
                            C.POINTER(Epilogue), C.c_int, _vp]),
    "fg_matmul_noalloc": (C.c_int, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, C.c_int, _vp, _i64,
                                    C.POINTER(Epilogue), C.c_int, _vp]),
    "fg_row_sum_squares": (C.c_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "fg_rmsnorm": (C.c_int, [_vp, _i64, _i64, _vp, C.c_float, _vp, _vp]),
    "fg_rope": (C.c_int, [_vp, _i64, C.c_int, C.c_int, C.c_double, _vp, _vp, _vp]),
    "fg_attention": (C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                               C.c_int, _vp, C.c_int, C.c_float, _vp, C.c_int, _vp]),
    "fg_normalize_rows": (C.c_int, [_i64, _i64, _vp, _i64, _vp, _i64, _vp]),
    "fg_similarities": (C.c_int, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _i64, C.c_int, _vp]),
    "fg_nearest": (C.c_int, [_i64, _i64, _i64, _vp, _i64, _vp, _i64, _vp, _vp, C.c_int, _vp]),
    "fg_kmeans": (C.c_int, [_i64, _i64, _vp, _i64, C.c_int, C.c_int, C.c_uint64, _vp, _vp, _vp, _vp,
                            C.POINTER(C.c_int), C.c_int, _vp]),
}


class FGError(RuntimeError):
    """A libfgemma call returned a negative status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{msg} (status {code})")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Loads libfgemma.so once; raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m ai_b200.build` "
                "(there is no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int) -> None:
    """Raises FGError for a negative status, with the library's message."""
    if rc != FG_OK:
        msg = lib().fg_last_error().decode(errors="replace")
        raise FGError(rc, msg)

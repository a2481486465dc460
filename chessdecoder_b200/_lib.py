"""ctypes binding of libcdk.so (declarations in include/cdk.h).

The library is loaded from the package directory.  There is no fallback: if
it is missing or fails to load, every op raises, so a GPU run can never
silently take a PyTorch or CPU path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcdk.so"

_vp, _i64, _i32, _f32 = C.c_void_p, C.c_int64, C.c_int32, C.c_float
_int = C.c_int


class CdkGemmEpilogue(C.Structure):
    _fields_ = [
        ("kind", C.c_int32),
        ("seq_len", C.c_int32),
        ("rope_cols", C.c_int32),
        ("reserved", C.c_int32),
        ("out", _vp),
        ("ldo", _i64),
        ("bias", _vp),
        ("resid", _vp),
        ("ldr", _i64),
        ("out2", _vp),
        ("ldo2", _i64),
        ("aux", _vp),
        ("ldaux", _i64),
        ("half_n", _i64),
        ("rope", _vp),
    ]


# name -> (restype, argtypes); mirrors include/cdk.h
SIGNATURES = {
    "cdk_version": (_int, []),
    "cdk_get_error": (_int, [C.POINTER(C.c_int), _int]),
    "cdk_gemm_bf16": (_int, [_vp, _i64, _int, _vp, _i64, _int, _i64, _i64, _i64, C.POINTER(CdkGemmEpilogue), _int,
                             _vp]),
    "cdk_gemm_pair_clusters": (_int, []),
    "cdk_gemm_fp8": (_int, [_vp, _i64, _int, _int, _vp, _i64, _int, _int, _i64, _i64, _i64, _vp, _vp,
                            C.POINTER(CdkGemmEpilogue), _int, _vp]),
    "cdk_fp8_cast": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _int, _vp, _i64, _vp, _i64, _vp, _vp]),
    "cdk_fp8_amax": (_int, [_vp, _int, _i64, _i64, _i64, _vp, _vp]),
    "cdk_fp8_scales": (_int, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "cdk_moe_route_workspace": (_i64, [_i64, _i32, _i32]),
    "cdk_moe_route": (_int, [_vp, _i64, _i32, _i32, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "cdk_moe_dispatch": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _vp]),
    "cdk_moe_combine": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "cdk_moe_combine_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _vp]),
    "cdk_moe_route_bwd": (_int, [_vp, _vp, _vp, _i64, _i32, _vp, _i64, _vp]),
    "cdk_moe_gather_sum": (_int, [_vp, _vp, _vp, _i64, _i64, _int, _vp]),
    "cdk_attn_bwd_workspace": (_i64, [_i64, _i64, _i64]),
    "cdk_attn_bwd_ws": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _i64, _vp]),
    "cdk_attn_bwd_q8": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp,
                               _vp]),
    "cdk_attn_prefix_meta": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "cdk_attn_meta_elems": (_i64, [_i64, _i64]),
    "cdk_attn_fwd": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
    "cdk_attn_bwd": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "cdk_rmsnorm_fwd": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "cdk_rmsnorm_fwd_q8": (_int, [_vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "cdk_rmsnorm_bwd_q8": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _vp, _vp, _vp, _i64, _i64, _vp]),
    "cdk_rmsnorm_bwd": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "cdk_fourier_features": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _vp, _i64, _vp, _vp, _vp]),
    "cdk_embed_fwd": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _vp]),
    "cdk_embed_bwd": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _vp]),
    "cdk_fourier_bwd": (_int, [_vp, _vp, _i32, _vp, _i64, _vp, _vp]),
    "cdk_softmax_ce": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _f32, _vp, _i64, _vp, _vp, _vp, _vp]),
    "cdk_soft_bucket_ce": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _f32, _vp, _i64, _vp, _vp]),
    "cdk_value_tail": (_int, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _f32, _vp, _vp, _vp, _i64, _vp,
                              _vp, _vp, _vp]),
    "cdk_gather_rows_bf16": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
    "cdk_scatter_add_rows_f32": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _i64, _vp]),
    "cdk_cast_f32_bf16": (_int, [_vp, _vp, _i64, _vp]),
    "cdk_add_f32": (_int, [_vp, _vp, _vp, _i64, _vp]),
    "cdk_scale_f32": (_int, [_vp, _i64, _f32, _vp]),
    "cdk_swiglu_bwd": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "cdk_swiglu_bwd_q8": (_int, [_vp, _i64, _vp, _i64, _vp, _i64, _int, _vp, _vp, _i64, _i64, _vp]),
    "cdk_gemm_f32": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _i64, _i64, _i64, _vp, _int, _vp]),
    "cdk_sumsq": (_int, [_vp, _i64, _vp, _i64, _vp]),
    "cdk_adamw": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _f32, _f32, _f32, _f32, _f32, _f32, _i64, _f32,
                         _vp]),
    "cdk_adamw_clip_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _f32, _f32, _f32, _f32, _f32, _i64,
                                      _f32, _vp]),
    "cdk_grpo_token": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _f32, _f32, _f32, _vp, _vp, _i64, _vp,
                              _vp, _vp]),
    "cdk_vocab_create": (_vp, [_vp, _vp, _i64, _vp, _vp]),
    "cdk_vocab_destroy": (None, [_vp]),
    "cdk_tokenize_games": (_int, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int,
                                  _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "cdk_kv_append": (_int, [_vp, _i64, _int, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _i64,
                             _int, _vp]),
    "cdk_decode_attn": (_int, [_vp, _i64, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _int, _vp, _vp, _vp,
                               _i64, _vp, _i64, _f32, _vp]),
    "cdk_decode_mark": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _vp]),
    "cdk_decode_slots": (_int, [_vp, _i64, _vp, _vp]),
    "cdk_swiglu_f32": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "cdk_head_select": (_int, [_vp, _i64, _i64, _i64, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp]),
    "cdk_mish_bf16": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _vp]),
}

_lib = None


def load() -> C.CDLL:
    """Loads libcdk.so once and binds every entry point; raises if it cannot."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m chessdecoder_b200.build_ext` "
                           "(the CUDA kernels are the only implementation; there is no fallback)")
    lib = C.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)

"""ctypes binding of libmb200.so (declared in include/mb200.h).

The library is loaded from the package directory only. If it is missing the
import fails loudly: there is no CPU or PyTorch fallback for any kernel.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmb200.so"

MB_OK = 0
MB_ERR = {-1: "BAD_ARG", -2: "UNKNOWN_KERNEL", -3: "CUDA", -4: "NCCL", -5: "TIMEOUT", -6: "NOT_INIT"}
DTYPE = {"f32": 0, "f16": 1, "i32": 2, "u32": 3, "bf16": 4}
ROLE_INPUT, ROLE_OUTPUT = 0, 1
DEVICE_PTR = 1


class MbBuf(C.Structure):
    _fields_ = [("binding", C.c_int), ("role", C.c_int), ("dtype", C.c_int), ("flags", C.c_int),
                ("ptr", C.c_void_p), ("bytes", C.c_size_t)]


class _ScalarV(C.Union):
    _fields_ = [("u", C.c_uint32), ("i", C.c_int32), ("f", C.c_float)]


class MbScalar(C.Structure):
    _fields_ = [("binding", C.c_int), ("dtype", C.c_int), ("v", _ScalarV)]


class MbTiming(C.Structure):
    _fields_ = [("min_ms", C.c_double), ("median_ms", C.c_double), ("mean_ms", C.c_double),
                ("iters", C.c_int), ("smem_bytes", C.c_int), ("threads_per_cta", C.c_int),
                ("launches_per_iter", C.c_int), ("h2d_ms", C.c_double), ("d2h_ms", C.c_double),
                ("profile_ms", C.c_double)]


class MbDevice(C.Structure):
    _fields_ = [("name", C.c_char * 128), ("type", C.c_char * 32), ("bucket", C.c_char * 32),
                ("sm_count", C.c_int), ("cc_major", C.c_int), ("cc_minor", C.c_int),
                ("cpu_cores", C.c_int), ("hbm_bytes", C.c_uint64), ("ram_bytes", C.c_uint64),
                ("l2_bytes", C.c_int), ("smem_per_block_optin", C.c_int)]


class MbDecoderConfig(C.Structure):
    _fields_ = [("d_model", C.c_int), ("n_heads", C.c_int), ("n_kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("rope_base", C.c_float),
                ("eps", C.c_float)]


class MbError(RuntimeError):
    def __init__(self, fn: str, rc: int, msg: str):
        super().__init__(f"{fn} failed: MB_ERR_{MB_ERR.get(rc, rc)}: {msg}")
        self.rc = rc


# name -> (restype, argtypes) for every symbol include/mb200.h declares.
_P, _I64, _I, _U32P = C.c_void_p, C.c_int64, C.c_int, C.POINTER(C.c_uint32)
SIGNATURES = {
    "mb_init": (C.c_int, [_I, _I, _I, C.c_char_p, _I]),
    "mb_shutdown": (None, []),
    "mb_last_error": (C.c_char_p, []),
    "mb_device_info": (C.c_int, [C.POINTER(MbDevice)]),
    "mb_kernel_names": (C.c_char_p, []),
    "mb_run": (C.c_int, [C.c_char_p, C.POINTER(MbBuf), _I, C.POINTER(MbScalar), _I, C.c_char_p,
                         _I, _I, C.POINTER(MbTiming)]),
    "mb_device_status": (C.c_int, [_U32P]),
    "mb_clear_device_status": (C.c_int, []),
    "mb_selftest_bounded_wait": (C.c_int, [_I, _P]),
    "mb_transpose_2d_f32": (C.c_int, [_P, _P, _I64, _I64, _P]),
    "mb_transpose_batched_bf16": (C.c_int, [_P, _P, _I64, _I64, _I64, _P]),
    "mb_transpose_batched_f32": (C.c_int, [_P, _P, _I64, _I64, _I64, _P]),
    "mb_gemm_bf16": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _I, _P]),
    "mb_sqr_mm_f32_workspace_bytes": (C.c_size_t, [_I64, _I64, _I64]),
    "mb_sqr_mm_f32": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, C.c_size_t, _P]),
    "mb_llama_attention_workspace_bytes": (C.c_size_t, [_I64, _I64, _I64, _I64]),
    "mb_llama_attention_bf16": (C.c_int, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, C.c_float, _P,
                                           C.c_size_t, _P]),
    "mb_mha_attention_workspace_bytes": (C.c_size_t, [_I64, _I64]),
    "mb_mha_attention_bf16": (C.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _P, C.c_size_t, _P]),
    "mb_transformer_block_workspace_bytes": (C.c_size_t, [_I64, _I64, _I64, _I64]),
    "mb_transformer_block_bf16": (C.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64,
                                            C.c_float, _P, C.c_size_t, _P]),
    "mb_batch_mm_f32_workspace_bytes": (C.c_size_t, [_I64, _I64, _I64, _I64]),
    "mb_batch_mm_f32": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _I64, _P, C.c_size_t, _P]),
    "mb_conv2d_nhwc_bf16": (C.c_int, [_P, _P, _P] + [_I] * 9 + [_P]),
    "mb_conv2d_nhwc_f32_workspace_bytes": (C.c_size_t, [_I] * 9),
    "mb_conv2d_nhwc_f32": (C.c_int, [_P, _P, _P] + [_I] * 9 + [_P, C.c_size_t, _P]),
    "mb_llama_decoder_f32_workspace_bytes": (C.c_size_t, [_I] * 6),
    "mb_llama_decoder_f32": (C.c_int, [_P] * 6 + [_I] * 6 + [C.c_float, C.c_float, _I, _P,
                                                            C.c_size_t, _P]),
    "mb_attention_decode_workspace_bytes": (C.c_size_t, [_I, _I, _I, _I]),
    "mb_attention_decode_bf16": (C.c_int, [_P, _I, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _P, _I,
                                           _P, C.c_size_t, _P]),
    "mb_attention_prefill_bf16": (C.c_int, [_P, _I, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I,
                                            _P, _I, _P]),
    "mb_decoder_layer_create": (C.c_int, [C.POINTER(MbDecoderConfig), _P, _P, _P, _P, _I, _I,
                                          C.POINTER(C.c_void_p)]),
    "mb_decoder_layer_destroy": (None, [_P]),
    "mb_decoder_layer_workspace_bytes": (C.c_size_t, [_P, _I, _I, _I]),
    "mb_decoder_layer_forward": (C.c_int, [_P, _P, _P, _I, _I, _P, _P, _I, _P, _P, _P, _I, _I, _P,
                                           C.c_size_t, _P]),
    "mb_decoder_layer_forward_ex": (C.c_int, [_P, _P, _P, _P, _P, _I, _I, _P, _P, _I, _P, _P, _P,
                                              _I, _I, _P, C.c_size_t, _P]),
    "mb_decoder_layer_forward_chain": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _I,
                                                 _P, _P, _P, _I, _I, _P, C.c_size_t, _P]),
    "mb_tp_allreduce_bf16": (C.c_int, [_P, C.c_size_t, _P]),
    "mb_rms_norm_linear_workspace_bytes": (C.c_size_t, [_I64]),
    "mb_rms_norm_linear_bf16": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, C.c_float, _P,
                                          C.c_size_t, _P]),
    "mb_fused_add_rms_norm_bf16": (C.c_int, [_P, _P, _P, _I64, _I64, C.c_float, _P]),
    "mb_rope_bf16": (C.c_int, [_P, _P, _I64, _I64, C.c_float, _P]),
    "mb_swiglu_packed_bytes": (C.c_size_t, [_I64, _I64]),
    "mb_swiglu_pack_bf16": (C.c_int, [_P, _P, _P, _I64, _I64, _P]),
    "mb_swiglu_bf16": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _P]),
    "mb_sdpa_workspace_bytes": (C.c_size_t, [_I64]),
    "mb_sdpa_bf16": (C.c_int, [_P, _P, _P, _P, _I64, _I64, _P, C.c_size_t, _P]),
    "mb_sqr_mm_f32_noalloc_max_workspace_bytes": (C.c_size_t, []),
    "mb_sqr_mm_f32_noalloc": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _P]),
}

_lib = None


def lib() -> C.CDLL:
    """Load libmb200.so once (RTLD_GLOBAL off) and bind every declared symbol."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m metalbench_b200.build` "
                "(there is no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().mb_last_error() or b"").decode()


def check(fn: str, rc: int) -> None:
    if rc != MB_OK:
        raise MbError(fn, rc, last_error())


def call(name: str, *args) -> None:
    check(name, getattr(lib(), name)(*args))

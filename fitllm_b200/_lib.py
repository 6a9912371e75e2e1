"""ctypes binding of libfitq.so (include/fitq.h).

The library is the only compute path: if it cannot be loaded, every op raises
FitqError.  There is no CPU or library fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("FITQ_LIB", _HERE / "_lib" / "libfitq.so"))

FITQ_OK = 0
ERRORS = {
    1: "FITQ_ERR_ARG", 2: "FITQ_ERR_SHAPE", 3: "FITQ_ERR_ALIGN", 4: "FITQ_ERR_UNSUPPORTED",
    5: "FITQ_ERR_WORKSPACE", 6: "FITQ_ERR_CUDA", 7: "FITQ_ERR_TIMEOUT", 8: "FITQ_ERR_NO_DEVICE",
}
DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2

# Every symbol include/fitq.h declares, with (restype, argtypes).
P, I32, I64, F32, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


class Nf4WeightC(ctypes.Structure):
    """struct fitq_nf4_weight"""
    _fields_ = [
        ("packed", P), ("absmax_code", P), ("nested_absmax", P), ("nested_quant_map", P),
        ("absmax_f32", P), ("quant_map", P), ("offset", F32), ("n_out", I64), ("k_in", I64),
    ]


WP = ctypes.POINTER(Nf4WeightC)


class GemvJobC(ctypes.Structure):
    """struct fitq_gemv_job"""
    _fields_ = [
        ("w", WP), ("lora_a", P), ("lora_b", P), ("rank", I32), ("scale", F32), ("bias", P),
        ("y", P), ("y_add", P),
    ]


JP = ctypes.POINTER(GemvJobC)

SIGNATURES = {
    "fitq_version": (ctypes.c_char_p, []),
    "fitq_last_error": (ctypes.c_char_p, []),
    "fitq_get_device_status": (I32, [I32, P]),
    "fitq_selftest_wait_timeout": (I32, [ctypes.c_uint64, P, P]),
    "fitq_nf4_dequant": (I32, [WP, P, I32, I32, P]),
    "fitq_nf4_quantize_workspace": (SZ, [I64, I64]),
    "fitq_nf4_quantize": (I32, [P, I64, I64, P, P, P, P, P, P, P, SZ, P]),
    "fitq_qlora_fwd_workspace": (SZ, [I64, I64, I64, I32]),
    "fitq_qlora_fwd": (I32, [WP, P, I64, P, P, I32, F32, P, P, P, P, P, SZ, P]),
    "fitq_qlora_bwd_workspace": (SZ, [I64, I64, I64, I32]),
    "fitq_qlora_bwd": (I32, [WP, P, P, I64, P, P, I32, F32, P, P, I32, P, P, I32, P, SZ, P]),
    "fitq_nf4_gemv_workspace": (SZ, [I64, I64, I64, I32]),
    "fitq_nf4_gemv": (I32, [WP, P, I64, P, P, I32, F32, P, P, P, P, SZ, P]),
    "fitq_gemm_bf16_tn": (I32, [P, P, P, P, I64, I64, I64, P]),
    "fitq_adamw_step": (I32, [P, P, P, P, I64, F32, F32, F32, F32, F32, I32, P, P]),
    "fitq_grad_norm_workspace": (SZ, [I64]),
    "fitq_grad_clip_coef": (I32, [P, I64, F32, P, P, SZ, P]),
    "fitq_timing_enable": (I32, [I32]),
    "fitq_timing_read": (I32, [P, P, I32]),
    "fitq_launch_count": (ctypes.c_longlong, []),
    "fitq_nf4_gemv_noalloc": (I32, [WP, P, I64, P, P, I32, F32, P, P, P, P]),
    "fitq_lora_merge": (I32, [P, I32, I64, I64, P, P, I32, F32, P]),
    "fitq_nf4_gateup_swiglu_workspace": (SZ, [I64, I64, I64]),
    "fitq_nf4_gateup_swiglu": (I32, [WP, WP, P, I64, P, P, P, P, SZ, P]),
    "fitq_nf4_down_dswiglu_workspace": (SZ, [I64, I64, I64]),
    "fitq_nf4_down_dswiglu": (I32, [WP, P, I64, P, P, P, P, P, SZ, P]),
    "fitq_rmsnorm_fwd": (I32, [P, P, P, I64, I64, F32, P]),
    "fitq_rmsnorm_bwd": (I32, [P, P, P, P, I64, I64, F32, P]),
    "fitq_rope": (I32, [P, P, P, P, I64, I32, I32, I64, I32, P]),
    "fitq_swiglu_fwd": (I32, [P, P, P, I64, P]),
    "fitq_swiglu_bwd": (I32, [P, P, P, P, P, I64, P]),
    "fitq_rope_append": (I32, [P, P, P, P, P, P, P, P, I64, I32, I32, I32, I32, I32, I32, P]),
    "fitq_nf4_gemv_grouped_workspace": (SZ, [JP, I32, I64]),
    "fitq_nf4_gemv_grouped": (I32, [JP, I32, P, I64, P, SZ, P]),
    "fitq_nf4_gemv_swiglu_workspace": (SZ, [JP, I64]),
    "fitq_nf4_gemv_swiglu": (I32, [JP, P, I64, P, P, SZ, P]),
    "fitq_cross_entropy_workspace": (SZ, [I64]),
    "fitq_cross_entropy": (I32, [P, P, I64, I64, I64, F32, P, P, SZ, P]),
    "fitq_verify_attention_workspace": (SZ, [I64, I32, I32, I32, I32]),
    "fitq_verify_attention": (I32, [P, P, P, P, I64, I32, I32, I32, I32, I32, I32, P, SZ, P]),
    "fitq_attention_fwd": (I32, [P, P, P, P, P, I64, I64, I32, I32, I32, P]),
    "fitq_attention_bwd_workspace": (SZ, [I64, I64, I32]),
    "fitq_attention_bwd": (I32, [P, P, P, P, P, P, P, P, P, I64, I64, I32, I32, I32, P, SZ, P]),
}


class FitqError(RuntimeError):
    def __init__(self, code: int, where: str, detail: str = ""):
        self.code = code
        name = ERRORS.get(code, f"code {code}")
        super().__init__(f"{where}: {name}" + (f" ({detail})" if detail else ""))


_lib = None
_lock = threading.Lock()


def load():
    """Load libfitq.so once; raise FitqError if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise FitqError(-1, "libfitq", f"{LIB_PATH} not built: run python -m fitllm_b200.build")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int, where: str) -> None:
    if rc != FITQ_OK:
        detail = load().fitq_last_error().decode(errors="replace")
        raise FitqError(rc, where, detail)


def version() -> str:
    return load().fitq_version().decode()


def ptr(t) -> int | None:
    """Device pointer of a tensor, or None."""
    return None if t is None else t.data_ptr()

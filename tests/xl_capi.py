"""ctypes binding of libxl_engine.so for the tests (the C ABI of include/xl_engine.h)."""
import ctypes as C
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "xingling-cpp_b200", "libxl_engine.so")
HEADER = os.path.join(ROOT, "include", "xl_engine.h")

VP, I, F, SZ = C.c_void_p, C.c_int, C.c_float, C.c_size_t

_SIGS = {
    "xl_last_error": ([], C.c_char_p),
    "xl_op_norm_gemv": ([I, VP, VP, VP, VP, VP, I, I, VP], I),
    "xl_rope_table": ([F, I, VP], I),
    "xl_op_attn_decode_workspace_bytes": ([I, I], SZ),
    "xl_op_attn_decode": ([VP, VP, VP, VP, VP, VP, I, I, VP, VP], I),
    "xl_op_attn_decode_noalloc": ([VP, VP, VP, VP, VP, VP, I, I, VP], I),
    "xl_op_lm_head_workspace_bytes": ([], SZ),
    "xl_op_lm_head": ([VP, VP, VP, VP, VP, F, I, I, C.POINTER(C.c_int), VP, VP], I),
    "xl_op_sample_workspace_bytes": ([I], SZ),
    "xl_op_sample": ([VP, I, F, F, F, C.POINTER(C.c_int), VP, VP], I),
    "xl_op_linear": ([I, VP, VP, VP, VP, VP, VP, VP, I, I, I, VP], I),
    "xl_op_split_lo": ([VP, VP, SZ, VP], I),
    "xl_op_rmsnorm": ([VP, VP, VP, I, I, VP], I),
    "xl_op_embedding": ([VP, VP, VP, I, I, VP], I),
    "xl_op_attn_prefill": ([VP, VP, VP, VP, VP, I, I, I, VP], I),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = C.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            fn = getattr(_lib, name)
            fn.argtypes = args
            fn.restype = res
    return _lib


def declared_functions() -> list[str]:
    """Every function the public header declares with XL_API."""
    text = open(HEADER).read()
    return re.findall(r"XL_API\s+[\w\s\*]+?\b(xl_\w+)\s*\(", text)


def check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(f"xl status {rc}: {lib().xl_last_error().decode()}")


def ptr(t) -> int:
    return t.data_ptr() if t is not None else None


def stream():
    import torch

    return C.c_void_p(torch.cuda.current_stream().cuda_stream)

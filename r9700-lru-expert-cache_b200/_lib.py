"""ctypes bindings of the two in-tree C-ABI libraries (declared in include/*.h).

The product path has no fallback: if a library is missing or does not load, the ops raise.
Prototypes here are the ones the reference's own Python binds (r4d_mxfp4_moe.py.lru.diff
L179-206 for librlu; draft_w4_lmhead.py:118-127; tests/k3/test_fp8sk.py:13-34), plus the
B200 entries.
"""
from __future__ import annotations

import ctypes
import functools
import os

HERE = os.path.dirname(os.path.abspath(__file__))

c_int, c_long, c_ll, c_vp = ctypes.c_int, ctypes.c_long, ctypes.c_longlong, ctypes.c_void_p

# name -> (restype, argtypes)
RLU_PROTOS = {
    "r4d_lru_manage": (c_int, [c_vp] + [c_int] * 5 + [c_vp] * 8 + [c_vp]),
    "r4d_lru_fused": (c_int, [c_vp] + [c_int] * 5 + [c_vp] * 8 + [c_int] * 3 + [c_vp] * 7),
    "r4d_lru_gather": (c_int, [c_vp, c_vp, c_long] * 6 + [c_vp, c_vp, c_int, c_int, c_vp]),
    "r4d_lru_host_device_pointer": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
}

LMHEAD_PROTOS = {
    "b200_silu_mul_quant": (c_int, [c_vp, c_int, c_int, c_ll, c_int, c_vp, c_vp, c_vp, c_int, c_vp]),
    "b200_per_token_group_quant_fp8": (c_int, [c_vp, c_int, c_int, c_ll, c_int, c_int, c_vp, c_vp, c_vp]),
    "b200_per_token_quant_fp8": (c_int, [c_vp, c_int, c_int, c_ll, c_int, c_vp, c_vp, c_vp, c_vp]),
    "b200_lmhead_workspace_bytes": (c_ll, []),
    "b200_lmhead_error": (c_int, [c_int]),
    "b200_fp8_lmhead": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_int, c_ll, c_vp, c_ll,
                                c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_ll, c_vp]),
    "b200_fp8_lmhead_static_scratch": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_int, c_ll, c_vp,
                                               c_ll, c_vp, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "b200_fp8_lmhead_combined": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_int, c_ll, c_vp, c_ll,
                                         c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_ll,
                                         c_vp, c_int, c_int, c_vp, c_int, c_vp]),
    "b200_w4_lmhead_combined": (c_int, [c_int, c_vp, c_int, c_int, c_int, c_vp, c_vp, c_int, c_int, c_ll,
                                        c_vp, c_ll, c_vp, c_vp, c_vp, c_vp, c_ll,
                                        c_vp, c_int, c_int, c_vp, c_int, c_vp]),
    "b200_pack_row_stats": (c_int, [c_vp, c_vp, c_vp, c_int, c_vp, c_vp]),
    "b200_combine_row_stats": (c_int, [c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    "b200_p2p_combine_bytes": (c_ll, [c_int, c_int]),
    "b200_p2p_combine_row_stats": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_vp, c_int, c_int, c_vp, c_vp,
                                           c_vp, c_vp, c_vp]),
    "fp8hip_gemm_w8a8_launch": (c_int, [c_vp] * 5 + [c_int] * 3 + [c_vp]),
    "hcq_gemm_fp8blk_nt_m16": (c_int, [c_vp] * 5 + [c_int] * 6 + [c_vp]),
    "hcq_gemm_fp8blk_nt_m16_max_m": (c_int, []),
    "hcq_stream_probe": (c_int, [c_vp, c_ll, c_int, c_vp, c_vp]),
    "b200_w4_lmhead": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_int, c_int, c_ll, c_vp,
                               c_ll, c_vp, c_vp, c_vp, c_vp, c_ll, c_vp]),
    "b200_w4_lmhead_sym": (c_int, [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_int, c_int, c_ll, c_vp,
                                   c_ll, c_vp, c_vp, c_vp, c_vp, c_ll, c_vp]),
    "b200_sigmoid_gate_mul": (c_int, [c_vp, c_vp, c_vp, c_int, c_int, c_ll, c_int, c_vp]),
    "b200_gemv_sigmoid_gate_mul": (c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_ll, c_ll,
                                           c_int, c_vp]),
    "b200_moe_sum": (c_int, [c_vp, c_vp, c_int, c_int, c_int, c_ll, c_int, c_vp]),
    "r4d_gemm_w4a16_nt_m64": (None, [c_long] * 4 + [c_int] * 8 + [c_long]),
    "r4d_gemm_w4a16_nt_m64_last_error": (c_int, []),
    "r4d_gemm_w4a16_nt_m64_max_m": (c_int, []),
    "r4d_gemm_w4a16_nt_m64_group": (c_int, []),
    "r4d_gemm_moe_mxfp4a8_nt_b16": (None, [c_long] * 10 + [c_int] * 8 + [c_long]),
    "r4d_gemm_moe_mxfp4a8_nt_b16_last_error": (c_int, []),
    "r4d_gemm_moe_mxfp4a8_nt_b16_block": (c_int, []),
    "r4d_gemm_moe_mxfp4a8_nt_b16_group": (c_int, []),
    "b200_moe_gemm_hot_cold": (c_int, [c_vp] * 8 + [c_int] + [c_vp] * 3 + [c_int, c_vp] + [c_int] * 4 + [c_vp]),
    "b200_moe_gemm_smem_bytes": (c_int, [c_int]),
    "b200_moe_gemm_error": (c_int, [c_int]),
}

LIB_FILES = {"librlu.so": RLU_PROTOS, "libb200lmhead.so": LMHEAD_PROTOS}


class NativeLibraryError(RuntimeError):
    pass


def lib_path(name: str) -> str:
    env = {"librlu.so": "R4D_LRU_LIB", "libb200lmhead.so": "B200_LMHEAD_LIB"}[name]
    return os.environ.get(env) or os.path.join(HERE, name)


@functools.lru_cache(maxsize=None)
def load(name: str) -> ctypes.CDLL:
    """dlopen an in-tree library and bind every prototype; raises if anything is missing."""
    path = lib_path(name)
    if not os.path.exists(path):
        raise NativeLibraryError(
            f"{path} is missing: build it with `python {os.path.join(HERE, 'build.py')}`")
    try:
        lib = ctypes.CDLL(path)
    except OSError as e:
        raise NativeLibraryError(f"cannot load {path}: {e}") from e
    for sym, (res, args) in LIB_FILES[name].items():
        try:
            fn = getattr(lib, sym)
        except AttributeError as e:
            raise NativeLibraryError(f"{path} does not export {sym}") from e
        fn.restype = res
        fn.argtypes = args
    return lib


def rlu() -> ctypes.CDLL:
    return load("librlu.so")


def lmhead() -> ctypes.CDLL:
    return load("libb200lmhead.so")


def ptr(t) -> c_vp:
    return c_vp(0 if t is None else t.data_ptr())


def stream_ptr(stream=None) -> c_vp:
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return c_vp(s.cuda_stream)


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed rc={rc}")


_CHECK = os.environ.get("B200_LMHEAD_CHECK", "0") == "1"


def debug_check(what: str) -> None:
    """With B200_LMHEAD_CHECK=1 in the environment: wait for the stream and raise if a bounded
    device wait of the lm_head kernels ran out (the device error word). Off by default, since
    it synchronizes; without it such a call's row statistics come out NaN / -1 instead."""
    if not _CHECK:
        return
    import torch
    torch.cuda.current_stream().synchronize()
    err = int(lmhead().b200_lmhead_error(0))
    if err != 0:
        raise RuntimeError(f"{what}: device error word {err} (1: a pipeline wait ran out, "
                           "2: a peer's statistics did not arrive); clear it with b200_lmhead_error(1)")


def require_cuda(what: str, *tensors) -> None:
    """The product path runs on the GPU only: refuse host tensors instead of launching a
    kernel on host pointers."""
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{what}: expected CUDA tensors (got a {t.device} tensor)")

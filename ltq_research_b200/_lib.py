"""Loader of the in-tree CUDA library ``libltq_b200.so`` (C ABI: include/ltq_b200.h).

There is no fallback: if the library is missing, or a call is made without a CUDA device, the call raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libltq_b200.so"
_LIB = None
_LOCK = threading.Lock()

P = ctypes.c_void_p
I = ctypes.c_int
SZ = ctypes.c_size_t
LL = ctypes.c_longlong

# name -> (restype, argtypes); mirrors include/ltq_b200.h
SIGNATURES = {
    "ltq_b200_version": (ctypes.c_char_p, []),
    # reference ctypes binding, src/tcq_proto.py:529: 15 pointers, 18 ints, pointer, int, pointer
    "tcq_viterbi": (I, [P] * 15 + [I] * 18 + [P, I, P]),
    "ltq_viterbi_tb_workspace_bytes": (SZ, [I] * 8),
    "ltq_viterbi_tb": (I, [P, P, I, P, P, P, P, P, P] + [I] * 5 + [P] + [I] * 10 + [P, SZ, P]),
    # matrix-level kernels
    "ltq_fwht256": (I, [P, I, ctypes.c_longlong, P, ctypes.c_longlong, P, I, I, I, P]),
    "ltq_scale_fit": (I, [P, ctypes.c_longlong, I, I, ctypes.c_float, ctypes.c_float, I, P, P, P, P, P]),
    "ltq_ldlq_gather": (I, [P, ctypes.c_longlong, P, I, P, P]),
    "ltq_ldlq_feedback": (I, [P, ctypes.c_longlong, I, I, P, P, P, P, ctypes.c_longlong, P, ctypes.c_longlong, P,
                              ctypes.c_longlong, P, P, ctypes.c_longlong, P]),
    "ltq_ldlq_block_workspace_bytes": (SZ, [I] * 6),
    "ltq_ldlq_bcat_elems": (SZ, [I]),
    "ltq_bf16x6_split": (I, [P, LL, I, I, I, I, P, LL, P]),
    "ltq_bf16x6_split_batched": (I, [P, LL, LL, I, I, I, I, I, I, P, LL, LL, P]),
    "ltq_trtri256_lower": (I, [P, LL, I, P, LL, P]),
    "ltq_chol256_diag": (I, [P, LL, I, P, P, LL, P, P]),
    "lut_subs_quant": (I, [P, P, P, P, I, ctypes.c_float, ctypes.c_float, I, P]),
    "ltq_int8_rings": (I, [P, P, LL, I, P]),
    "ltq_matvec_slice": (I, [P, I, I, I, I, I, I, P, I, P, P, P, P, LL, P, P, P]),
    "ltq_ldlq_bcat": (I, [P, LL, I, P, P]),
    "ltq_ldlq_bcat_t": (I, [P, LL, I, P, P]),
    "ltq_gemm_bf16_tn": (I, [P, LL, P, LL, P, LL, I, I, I, ctypes.c_float, ctypes.c_float, P, P]),
    "ltq_gemm_bf16x6_tn": (I, [P, LL, P, LL, P, LL, I, I, I, ctypes.c_float, ctypes.c_float, P, P]),
    "ltq_gemm_wait_selftest": (I, [I, ctypes.c_uint, P, P, P]),
    "ltq_chol_solve": (I, [P, LL, I, P, P, P, P, P]),
    "ltq_gemm_bf16x3p_tn": (I, [P, LL, LL, P, LL, LL, P, LL, LL, I, I, I, I, I, ctypes.c_float, ctypes.c_float, P, P]),
    "ltq_bf16x3_split": (I, [P, LL, LL, I, I, I, I, I, I, P, LL, LL, P]),
    "ltq_ldlq_inter3": (I, [P, LL, P, LL, P, LL, P, LL, I, P, LL, P, LL, P, P]),
    "ltq_ldlq_inter": (I, [P, LL, P, LL, P, LL, P, LL, I, P, LL, P, LL, P, P]),
    "ltq_ldlq_block": (I, [P, LL, P, LL, P, P, LL, P, LL, P, LL, P, P, LL, I, P, P, I, I, P] + [I] * 6 + [P, SZ, P]),
    # .ltq packing and spec decode
    "ltq_slice_bytes": (SZ, [I] * 6),
    "ltq_pack_slice": (I, [P, P, LL] + [I] * 6 + [P, SZ, P]),
    "ltq_decode_slice": (I, [P] + [I] * 6 + [P, I, P, P, P, LL, P, LL, P, P]),
    # allocation-free variant (scratch inside the library): same arguments without the workspace
    "ltq_viterbi_tb_noalloc_capacity": (SZ, []),
    "ltq_viterbi_tb_noalloc": (I, [P, P, I, P, P, P, P, P, P] + [I] * 5 + [P] + [I] * 10 + [P]),
}


class LtqLibraryError(RuntimeError):
    pass


# kernels launched by one successful call (a constant, or a function of the call's arguments)
KERNELS_PER_CALL = {
    "tcq_viterbi": 2,
    "ltq_viterbi_tb": lambda a: 2 * int(a[22]),
    "ltq_viterbi_tb_noalloc": lambda a: 2 * int(a[22]),
    "ltq_fwht256": 1, "ltq_scale_fit": 1, "ltq_ldlq_gather": 1, "ltq_ldlq_feedback": 1, "ltq_ldlq_block": 2,
    "ltq_ldlq_bcat": 1, "ltq_ldlq_bcat_t": 1, "ltq_gemm_bf16_tn": 1, "ltq_gemm_bf16x6_tn": 1, "ltq_gemm_bf16x3p_tn": 1, "ltq_gemm_wait_selftest": 1, "ltq_chol_solve": lambda a: 2 * (int(a[2]) // 256), "ltq_bf16x3_split": 1,
    "ltq_ldlq_inter": 1, "ltq_ldlq_inter3": 1, "ltq_bf16x6_split": 1, "ltq_bf16x6_split_batched": 1,
    "ltq_trtri256_lower": 1, "ltq_chol256_diag": 1, "lut_subs_quant": 1, "ltq_int8_rings": 1, "ltq_matvec_slice": 1,
    "ltq_pack_slice": 1, "ltq_decode_slice": 1,
}


class _CountingLib:
    """The ctypes library with a count of the kernels its calls launched (``kernels``), per process."""

    def __init__(self, cdll: ctypes.CDLL):
        self._cdll = cdll
        self.kernels = 0
        self._lock = threading.Lock()

    def __getattr__(self, name):
        fn = getattr(self._cdll, name)
        k = KERNELS_PER_CALL.get(name)
        if k is None:
            return fn

        def call(*a):
            rc = fn(*a)
            if rc == 0:
                n = k(a) if callable(k) else k
                with self._lock:
                    self.kernels += n
            return rc
        call.__name__ = name
        self.__dict__[name] = call
        return call


def kernels_launched() -> int:
    """Kernels launched so far by this process through the library (successful calls only)."""
    return lib().kernels


def lib() -> "_CountingLib":
    """The loaded library (ctypes functions, plus a launch count); raises LtqLibraryError when it has not been
    built."""
    global _LIB
    if _LIB is None:
        with _LOCK:
            if _LIB is None:
                if not LIB_PATH.exists():
                    raise LtqLibraryError(f"{LIB_PATH} is missing: build it with `python -m ltq_research_b200.build`")
                L = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _LIB = _CountingLib(L)
    return _LIB


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    """Every tensor must live on one CUDA device; there is no CPU path."""
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("ltq_research_b200: inputs must be CUDA tensors (there is no CPU implementation)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError("ltq_research_b200: all inputs must be on the same CUDA device")
    if dev is None:
        raise RuntimeError("ltq_research_b200: no CUDA tensor given")
    return dev


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()

"""Loader of the oracle's C model of tensor-core accumulation (oracle/tcgemm.c).
TEST INFRASTRUCTURE ONLY.  Built by `make -C oracle` (run here on first use if missing)."""
import ctypes
import subprocess
from pathlib import Path

import torch

_DIR = Path(__file__).resolve().parent
_SO = _DIR / "_build" / "libtcgemm.so"
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not _SO.exists():
            subprocess.run(["make", "-C", str(_DIR)], check=True, capture_output=True)
        _lib = ctypes.CDLL(str(_SO))
        _lib.tc_fp8_acc.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p]
        _lib.tc_fp8_acc.restype = None
        _lib.tc_bf16_acc.argtypes = [ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 6 + [ctypes.c_void_p]
        _lib.tc_bf16_acc.restype = None
    return _lib


def acc(q, w8, k0, k1):
    """fp32 [M, N] accumulators of q [M, K] . w8 [N, K]^T (e4m3) over K in [k0, k1)."""
    q = q.contiguous()
    w8 = w8.contiguous()
    m, n = q.shape[0], w8.shape[0]
    out = torch.empty(m, n, dtype=torch.float32)
    lib().tc_fp8_acc(q.view(torch.uint8).data_ptr(), w8.view(torch.uint8).data_ptr(), m, n, q.shape[1],
                     w8.shape[1], k0, k1, out.data_ptr())
    return out


def acc_bf16(a, w, k0, k1):
    """fp32 [M, N] accumulators of a [M, K] . w [N, K]^T (bf16, kind::f16) over K in [k0, k1)."""
    a = a.to(torch.bfloat16).contiguous()
    w = w.to(torch.bfloat16).contiguous()
    m, n = a.shape[0], w.shape[0]
    out = torch.empty(m, n, dtype=torch.float32)
    lib().tc_bf16_acc(a.view(torch.int16).data_ptr(), w.view(torch.int16).data_ptr(), m, n, a.shape[1], w.shape[1],
                      k0, k1, out.data_ptr())
    return out

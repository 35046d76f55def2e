"""Loader of the oracle's C models: tensor-core accumulation (oracle/tcgemm.c), the
attention kernel's softmax arithmetic (oracle/attn.c) and the bf16 linear's GELU
epilogues (oracle/act.c).
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
        _lib.tc_acc_scalar.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int] * 6 + \
            [ctypes.c_void_p]
        _lib.tc_acc_scalar.restype = None
        _lib.tc_vector_path.restype = ctypes.c_int
        _lib.ffo_exp2_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.attn_softmax_block.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _lib.attn_fold.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.attn_finish.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
        for name in ("ffo_gelu_tanh_array", "ffo_gelu_erf_array"):
            getattr(_lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_long]
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


def acc_scalar(kind, a, w, k0, k1):
    """The scalar model (kind 0: e4m3, 1: bf16) that the vectorised one is checked against."""
    dt = torch.uint8 if kind == 0 else torch.int16
    a = a.contiguous()
    w = w.contiguous()
    out = torch.empty(a.shape[0], w.shape[0], dtype=torch.float32)
    lib().tc_acc_scalar(kind, a.view(dt).data_ptr(), w.view(dt).data_ptr(), a.shape[0], w.shape[0], a.shape[1],
                        w.shape[1], k0, k1, out.data_ptr())
    return out


def exp2(x):
    """exp2_poly of fp32 values (the attention kernel's exponential)."""
    x = x.float().contiguous()
    y = torch.empty_like(x)
    lib().ffo_exp2_array(x.data_ptr(), y.data_ptr(), x.numel())
    return y


def gelu(x, form):
    """The bf16 linear epilogue's GELU of fp32 values, form "tanh" or "erf" (oracle/act.c)."""
    x = x.float().contiguous()
    y = torch.empty_like(x)
    fn = lib().ffo_gelu_tanh_array if form == "tanh" else lib().ffo_gelu_erf_array
    fn(x.data_ptr(), y.data_ptr(), x.numel())
    return y


def attention_head(q, k, v, qpos, lo, scale_log2):
    """One query head of the attention kernel, restated (oracle/attn.c).
    q [R, 128], k / v [T, 128] bf16; qpos / lo int [R]; returns bf16 [R, 128]."""
    r_n, t_n = q.shape[0], k.shape[0]
    qpos = qpos.to(torch.int32).contiguous()
    lo = lo.to(torch.int32).contiguous()
    s_all = acc_bf16(q, k, 0, 128)                      # [R, T]: 8 MMA steps of 16 over d
    jb_lo = int(lo.min()) // 64
    jb_hi = min(int(qpos.max()), t_n - 1) // 64
    m = torch.full((r_n,), float("-inf"))
    l = torch.zeros(r_n, 4)
    o = torch.zeros(r_n, 128)
    alpha = torch.empty(r_n)
    p = torch.empty(r_n, 64, dtype=torch.int16)
    L = lib()
    for jb in range(jb_lo, jb_hi + 1):
        k0 = jb * 64
        n = min(64, t_n - k0)
        sb = torch.zeros(r_n, 64)
        sb[:, :n] = s_all[:, k0:k0 + n]
        L.attn_softmax_block(sb.data_ptr(), r_n, qpos.data_ptr(), lo.data_ptr(), t_n, k0, float(scale_log2),
                             m.data_ptr(), l.data_ptr(), p.data_ptr(), alpha.data_ptr())
        vt = torch.zeros(128, 64, dtype=torch.bfloat16)
        vt[:, :n] = v[k0:k0 + n].t()
        big_o = acc_bf16(p.view(torch.bfloat16), vt, 0, 64)  # [R, 128]: 4 MMA steps of 16 over keys
        L.attn_fold(o.data_ptr(), big_o.data_ptr(), alpha.data_ptr(), r_n)
    out = torch.empty(r_n, 128, dtype=torch.int16)
    L.attn_finish(o.data_ptr(), l.data_ptr(), r_n, out.data_ptr())
    return out.view(torch.bfloat16)

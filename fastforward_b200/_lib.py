"""ctypes binding of libffb200.so (the C ABI declared in include/ffb200.h).

The library is loaded from this package directory.  There is no fallback: if the
shared library is missing or no CUDA device is present, every op raises.
"""
import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint32, c_void_p, c_char_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libffb200.so")

OK, EINVAL, EUNSUPPORTED, ECUDA, ETIMEOUT = 0, -1, -2, -3, -4
QUANT_NONE, QUANT_STATIC, QUANT_ROWWISE, QUANT_ROWSCALE = 0, 1, 2, 3
EPI_BF16, EPI_F32_PARTIAL, EPI_SWIGLU = 0, 1, 2
EPI_BIAS, EPI_BIAS_RES, EPI_BIAS_GELU_TANH, EPI_BIAS_GELU_ERF = 10, 11, 12, 13  # ffb_bf16_gemm
TILE_STREAM = 1  # ffb_fp8_gemm feature_tile: the weight-stationary schedule
PRO_QUANT, PRO_ADD_RMSNORM = 1, 2


class Prologue(ctypes.Structure):
    """`ffb_gemm_prologue` (include/ffb200.h): the producer fused into the front of a GEMM."""
    _fields_ = [("kind", c_int), ("x", c_void_p), ("b", c_void_p), ("b32", c_void_p), ("splits", c_int),
                ("add", c_int), ("deep", c_void_p), ("start", c_int), ("nv", c_int), ("norm_w", c_void_p),
                ("eps", c_float), ("residual", c_void_p), ("quant_mode", c_int), ("inv_scale", c_float),
                ("sync", c_void_p)]

P, I, F = c_void_p, c_int, c_float
MAX_PEERS = 8


class PeerSync(ctypes.Structure):
    """`ffb_peer_sync` (include/ffb200.h): a rank's cross-GPU handshake state."""
    _fields_ = [("flags", c_void_p * MAX_PEERS), ("local", c_void_p), ("rank", c_int), ("world", c_int),
                ("nslots", c_int)]


# name -> argtypes, in the order of include/ffb200.h
SIGNATURES = {
    "ffb_version": [],
    "ffb_set_pdl": [I],
    "ffb_last_error": [c_char_p, c_size_t],
    "ffb_device_error": [P, I],
    "ffb_embed_gather": [P, P, c_int64, P, I, I, P, I, I, P],
    "ffb_rmsnorm": [P, P, F, P, I, F, P, P, I, I, P],
    "ffb_add_rmsnorm": [P, P, P, I, P, I, I, P, F, P, P, I, F, P, P, I, I, P],
    "ffb_qk_norm_rope": [P, P, I, I, P, P, F, P, P, P, P, P, I, I, I, P],
    "ffb_attention": [P, P, P, P, I, P, I, I, I, I, F, P],
    "ffb_attention_segmented": [P, P, P, P, I, P, P, I, I, I, I, F, P],
    "ffb_attention_fp8": [P, P, P, P, F, P, I, I, I, F, P],
    "ffb_attention_rowwise": [P, P, P, P, P, P, I, I, I, F, P],
    "ffb_attention_rowwise_sync_bytes": [I, I],
    "ffb_gather_rows": [P, P, P, I, I, P],
    "ffb_quantize_fp8": [P, I, F, P, P, I, I, P],
    "ffb_quantize_weight_fp8": [P, I, P, P, P, I, I, P],
    "ffb_quantize_weight_fp8_noalloc": [P, I, P, P, I, I, P],
    "ffb_fp8_gemm": [P, P, I, P, P, I, I, P, P, I, I, I, I, I, P],
    "ffb_fp8_gemm_stream_ctas": [I, I, I, I, I],
    "ffb_fp8_gemm_qk_rope": [P, P, I, P, P, I, P, P, F, P, P, P, P, P, I, I, I, I, P],
    "ffb_fp8_gemm_swiglu_fp8": [P, P, I, P, P, I, F, P, I, I, I, P],
    "ffb_fp8_gemm_fused": [P, P, P, I, P, P, I, I, P, P, I, I, I, I, I, P],
    "ffb_fp8_gemm_qk_rope_fused": [P, P, P, I, P, P, I, P, P, F, P, P, P, P, P, I, I, I, I, P],
    "ffb_pack_gateup": [P, P, I, I, I, P],
    "ffb_swiglu": [P, P, I, P, I, I, P],
    "ffb_readout": [P, P, P, I, P, F, P, I, I, P, P, I, P],
    "ffb_pack_int4": [P, P, P, I, I, P],
    "ffb_w4a16_gemm": [P, P, P, I, P, P, I, I, I, I, I, P],
    "ffb_pack_rgb": [P, P, I, I, P],
    "ffb_pack_rgb_batch": [P, P, I, I, I, P],
    "ffb_peer_alloc": [c_size_t, P, P],
    "ffb_peer_open": [P, P],
    "ffb_peer_close": [P],
    "ffb_peer_free": [P],
    "ffb_add_rmsnorm_peers": [P, P, P, P, I, I, P, F, P, P, I, F, P, P, I, I, P],
    "ffb_quantize_fp8_peers": [P, P, P, P, P, I, I, P],
    "ffb_bf16_gemm": [P, P, P, P, I, P, I, I, P, P, I, I, I, P],
    "ffb_bf16_gemm_plan": [I, I, I, P],
    "ffb_layernorm": [P, P, P, F, P, I, I, P],
    "ffb_add_layernorm": [P, P, P, P, F, P, P, I, I, P],
    "ffb_vision_rope": [P, P, P, I, I, I, I, P, P, P, P],
    "ffb_attention_full": [P, P, P, P, I, I, I, F, P],
}


class FFBError(RuntimeError):
    """A libffb200 call failed (CUDA error or device-side timeout)."""


class FFBUnsupported(FFBError, NotImplementedError):
    """The kernels do not implement the requested configuration."""


_lib = None


def lib():
    """The loaded library (loaded on first use)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FFBError(f"{LIB_PATH.name} is not built; run `python -m fastforward_b200.build`")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = c_char_p if name == "ffb_version" else c_int
        _lib = handle
    return _lib


def last_error():
    buf = ctypes.create_string_buffer(512)
    lib().ffb_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(rc):
    if rc == OK:
        return
    msg = last_error()
    if rc == EINVAL:
        raise ValueError(msg)
    if rc == EUNSUPPORTED:
        raise FFBUnsupported(msg)
    raise FFBError(f"[{rc}] {msg}")


def call(name, *args):
    """Calls `name` and raises on a non-zero return code."""
    check(getattr(lib(), name)(*args))


def ptr(t):
    """Device pointer of a tensor, or None (NULL) for None."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libffb200 ops take CUDA tensors only (no CPU fallback)")
    return t.data_ptr()


def stream_ptr(device=None):
    return torch.cuda.current_stream(device).cuda_stream


def device_error(clear=False):
    w = c_uint32(0)
    call("ffb_device_error", ctypes.addressof(w), int(clear))
    return w.value


def stream_ctas(m, n, k, epilogue, splits=1):
    """CTAs of ffb_fp8_gemm's weight-stationary schedule for this GEMM, 0 if it does not
    apply (host query)."""
    return int(lib().ffb_fp8_gemm_stream_ctas(int(m), int(n), int(k), int(epilogue), int(splits)))


def bf16_gemm_plan(m, n, k):
    """(feature tile, K splits, counters needed) that ffb_bf16_gemm plans for m x n x k."""
    plan = (ctypes.c_int * 3)()
    call("ffb_bf16_gemm_plan", int(m), int(n), int(k), ctypes.addressof(plan))
    return plan[0], plan[1], plan[2]


def set_pdl(enable):
    return lib().ffb_set_pdl(int(enable))


def require_cuda():
    if not torch.cuda.is_available():
        raise FFBError("a CUDA device is required: this path has no CPU fallback")

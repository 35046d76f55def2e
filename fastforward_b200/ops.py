"""Fused ops with the reference's Python signatures, backed by libffb200 (sm_100a).

Each function mirrors one of FastForward's Triton-backed ops (argument meaning, output
shapes and dtypes, duck-typed norm modules with `.weight` / `.variance_epsilon`), so
code written against the reference runs unchanged:

    add_rms            _legacy/lower_kernels.py:24-32
    fast_norm          _legacy/sub10_runtime.py:37-41
    qk_pair            _legacy/broad_kernels.py:63-74
    attention_direct   _legacy/limit_kernels.py:36-45
    swiglu             _legacy/search_kernels.py:18-23
    lm_readout         _legacy/limit_kernels.py:60-66
    StaticFP8Linear    _legacy/limit_kernels.py:117-135
    RuntimeScaleLinear _family/depth_fp8.py:22-26
    FP8Linear          _legacy/fp8_private.py:21-38
    Int4               _family/night_runtime.py:15-42 (symmetric group-128 scheme)
    pack_rgb           _legacy/sub10_runtime.py:21-29
    pack_rectangle     _family/depth_runtime.py:18-25
    add_layernorm      _legacy/lower_kernels.py:130-136
    vision_rope        _legacy/search_kernels.py:127-134
    vision_linear / vision_attention: the HF vision blocks' nn.Linear (+ residual / GELU)
                       and SDPA (_legacy/vision_graph_runtime.py:16-27)

Outputs are allocated with torch on the input's device (stream-ordered, graph-safe
through the caching allocator).  Argument errors raise ValueError (the reference uses
assert); CUDA failures raise FFBError.  There is no CPU path.
"""
import torch

from . import _lib as L
from ._lib import call, ptr, stream_ptr

BF16 = torch.bfloat16
E4M3 = torch.float8_e4m3fn


def _need(cond, msg):
    if not cond:
        raise ValueError(msg)


def _bf16_cuda(*ts):
    for t in ts:
        _need(t.is_cuda, "CUDA tensors required (no CPU fallback)")
        _need(t.dtype == BF16, f"bf16 required, got {t.dtype}")


def add_rms(a, b, deep, module, start=0, nv=0):
    """residual = bf16(a + b) (+ deep on rows [start, start+nv)); out = RMSNorm(residual)."""
    _need(a.shape == b.shape and a.is_contiguous() and b.is_contiguous(), "a, b: same shape, contiguous")
    _bf16_cuda(a, b, module.weight)
    h = a.shape[-1]
    if deep is not None:
        _need(deep.shape == (nv, h) and deep.is_contiguous(), "deep must be [nv, H] contiguous")
    residual = torch.empty_like(a)
    out = torch.empty_like(a)
    t = a.numel() // h
    call("ffb_add_rmsnorm", ptr(a), ptr(b), None, 0, ptr(deep), int(start), int(nv), ptr(module.weight),
         float(module.variance_epsilon), ptr(residual), ptr(out), L.QUANT_NONE, 0.0, None, None, t, h,
         stream_ptr(a.device))
    return residual, out


def fast_norm(x, module):
    """RMSNorm of each row (bf16 rounding as `rms_one`)."""
    _need(x.is_contiguous(), "x must be contiguous")
    _bf16_cuda(x, module.weight)
    out = torch.empty_like(x)
    h = x.shape[-1]
    call("ffb_rmsnorm", ptr(x), ptr(module.weight), float(module.variance_epsilon), ptr(out), L.QUANT_NONE, 0.0,
         None, None, x.numel() // h, h, stream_ptr(x.device))
    return out


def qk_pair(q, k, qn, kn, cos, sin, rows=4, warps=4, half=False, pad=1, fusion=False):
    """Per-head RMSNorm + rotate-half RoPE.  q [1,T,HQ,D], k [1,T,HK,D] (views into the
    packed qkv rows); cos/sin [1,T,D].  Returns yq [1,HQ,T,D], yk [1,HK,T,D] (head-major).
    `rows`, `warps`, `pad`, `fusion` are Triton launch knobs of the reference (ignored);
    `half=True` selects the half-split kernel there, which computes the same values."""
    _need(q.shape[0] == k.shape[0] == 1 and q.shape[1] == k.shape[1], "batch 1, same T")
    _need(q.stride(1) == k.stride(1) and q.stride(-1) == k.stride(-1) == 1, "q, k: same row stride, unit last")
    _bf16_cuda(q, k, qn.weight, kn.weight, cos, sin)
    _, t, hq, d = q.shape
    hk = k.shape[2]
    _need(d == 128, "head_dim 128 only")
    _need(q.stride(2) == d and k.stride(2) == d, "heads must be contiguous inside a row")
    _need(abs(qn.variance_epsilon - kn.variance_epsilon) < 1e-12, "q_norm and k_norm must share eps")
    stride = q.stride(1)
    packed = (k.data_ptr() == q.data_ptr() + hq * d * q.element_size() and stride >= (hq + 2 * hk) * d)
    if packed:
        base, row_stride = q, stride
    else:  # pack q|k|0 rows so the kernel sees one row layout
        base = torch.cat([q.reshape(t, hq * d), k.reshape(t, hk * d), torch.zeros(t, hk * d, dtype=BF16,
                          device=q.device)], -1)
        row_stride = base.shape[-1]
    yq = torch.empty((1, hq, t, d), device=q.device, dtype=BF16)
    yk = torch.empty((1, hk, t, d), device=q.device, dtype=BF16)
    c = cos.reshape(t, d).contiguous()
    s = sin.reshape(t, d).contiguous()
    call("ffb_qk_norm_rope", base.data_ptr(), None, 0, int(row_stride), ptr(qn.weight), ptr(kn.weight),
         float(qn.variance_epsilon), ptr(c), ptr(s), ptr(yq), ptr(yk), None, t, hq, hk, stream_ptr(q.device))
    return yq, yk


def attention_direct(q, k, v, scale, bm=16, bn=64, warps=4, positions=None, triangular=True):
    """Causal GQA attention.  q [1,HQ,S,D] contiguous, k [1,HK,T,D] contiguous, v [1,HK,T,D]
    (any strides with unit last); positions [S] int64 selects the query positions (tail).
    Returns y [1,S,HQ,D] bf16.  `bm`, `bn`, `warps`, `triangular` are launch knobs of the
    reference that do not change the result (ignored)."""
    _need(q.is_contiguous() and k.is_contiguous() and q.shape[0] == k.shape[0] == v.shape[0] == 1, "layout")
    _, hq, s, d = q.shape
    _, hk, t, kd = k.shape
    _need(kd == d == 128 and tuple(v.shape) == (1, hk, t, d) and v.stride(-1) == 1 and hq % hk == 0, "shapes")
    _bf16_cuda(q, k, v)
    vv = v if v.is_contiguous() else v.contiguous()
    pos = None
    if positions is not None:
        _need(tuple(positions.shape) == (s,) and positions.is_contiguous(), "positions must be [S] contiguous")
        pos = positions.to(torch.int64)
    else:
        _need(s == t, "causal attention over all rows needs S == T (pass positions for selected rows)")
    y = torch.empty((1, s, hq, d), device=q.device, dtype=BF16)
    call("ffb_attention", ptr(q), ptr(k), ptr(vv), ptr(pos), 0, ptr(y), s, t, hq, hk, float(scale),
         stream_ptr(q.device))
    return y


def swiglu(gate, up, block=1024, warps=4):
    """y = bf16(bf16(silu(gate)) * up) on strided [.., I] views (same strides)."""
    _need(gate.shape == up.shape and gate.stride() == up.stride(), "gate, up: same shape and strides")
    _need(gate.stride(-1) == 1, "unit last stride")
    _bf16_cuda(gate, up)
    i = gate.shape[-1]
    m = gate.numel() // i
    row_stride = gate.stride(-2) if gate.dim() > 1 else i
    if gate.dim() > 2:
        _need(all(gate.stride(j) == gate.stride(j + 1) * gate.shape[j + 1] for j in range(gate.dim() - 2)),
              "leading dims must be collapsible")
    y = torch.empty(gate.shape, device=gate.device, dtype=BF16)
    call("ffb_swiglu", ptr(gate), ptr(up), int(row_stride), ptr(y), m, i, stream_ptr(gate.device))
    return y


def lm_readout(x, norm, weight):
    """Final RMSNorm of one row, then dots with the option rows: fp32 [1, n]."""
    _need(x.numel() == x.shape[-1] == weight.shape[1] and x.is_contiguous() and weight.is_contiguous(), "shapes")
    _bf16_cuda(x, weight, norm.weight)
    n = weight.shape[0]
    _need(1 <= n <= 8, "1..8 option rows")
    y = torch.empty((1, n), device=x.device, dtype=torch.float32)
    call("ffb_readout", ptr(x), None, None, 0, ptr(norm.weight), float(norm.variance_epsilon), ptr(weight), n, n,
         ptr(y), None, x.shape[-1], stream_ptr(x.device))
    return y


def readout_logsoftmax(x, norm, weight, k):
    """lm_readout followed by log-softmax over the first k options: (logits [k], logprobs [k])."""
    _bf16_cuda(x, weight, norm.weight)
    n = weight.shape[0]
    xc = x.contiguous()
    z = torch.empty(n, device=x.device, dtype=torch.float32)
    lp = torch.empty(k, device=x.device, dtype=torch.float32)
    call("ffb_readout", ptr(xc), None, None, 0, ptr(norm.weight), float(norm.variance_epsilon),
         ptr(weight), n, int(k), ptr(z), ptr(lp), x.shape[-1], stream_ptr(x.device))
    return z[:k], lp


# ---------------------------------------------------------------------------- FP8 linears

def quantize_weight(w, per_channel):
    """bf16 [N,K] -> (e4m3 [N,K], fp32 scale [N] or [1]) on the GPU, bit-exact to the
    reference's torch expression."""
    _bf16_cuda(w)
    w = w.contiguous()
    n, k = w.shape
    w8 = torch.empty((n, k), device=w.device, dtype=E4M3)
    scale = torch.empty(n if per_channel else 1, device=w.device, dtype=torch.float32)
    ws = torch.empty(n, device=w.device, dtype=torch.float32)
    call("ffb_quantize_weight_fp8", ptr(w), int(per_channel), ptr(w8), ptr(scale), ptr(ws), n, k,
         stream_ptr(w.device))
    return w8, scale


def quantize_activation(x, mode, inverse_scale=1.0):
    """bf16 [..., K] -> (e4m3 [pad16(M), K] with zero pad rows, fp32 row scales or None)."""
    _bf16_cuda(x)
    flat = x.reshape(-1, x.shape[-1]).contiguous()
    m, k = flat.shape
    pad = (m + 15) // 16 * 16
    q = torch.zeros((pad, k), device=x.device, dtype=E4M3)
    scale = None
    if mode == L.QUANT_ROWWISE:
        scale = torch.full((pad,), 1e-12 / 448.0, device=x.device, dtype=torch.float32)
    call("ffb_quantize_fp8", ptr(flat), int(mode), float(inverse_scale), ptr(q), ptr(scale), m, k,
         stream_ptr(x.device))
    return q, scale


def fp8_gemm(a8, a_scale, w8, w_scale, m, out_dtype=BF16, token_tile=0):
    """bf16 [m, N] = (a8 . w8^T) * a_scale * w_scale on tcgen05 (plain bf16 epilogue)."""
    n, k = w8.shape
    out = torch.empty((m, n), device=a8.device, dtype=BF16)
    call("ffb_fp8_gemm", ptr(a8), ptr(a_scale), int(a_scale.numel() > 1), ptr(w8), ptr(w_scale),
         int(w_scale.numel() > 1), L.EPI_BF16, ptr(out), None, 1, int(token_tile), m, n, k, stream_ptr(a8.device))
    return out


class StaticFP8Linear:
    """Per-tensor FP8 weight + static activation scale (`inverse_scale` = 448 / bound)."""

    def __init__(self, weight, inverse_scale=16.0):
        w = weight.detach()
        if w.dtype != BF16:
            w = w.to(BF16)
        self.weight, self.weight_scale = quantize_weight(w, per_channel=False)
        self.inverse_scale = inverse_scale
        self.input_scale = torch.tensor([1.0 / inverse_scale], device=w.device, dtype=torch.float32)
        self.fast_accum = True  # accepted for parity; tcgen05 always accumulates in fp32

    def __call__(self, x):
        q, _ = quantize_activation(x, L.QUANT_STATIC, self.inverse_scale)
        m = x.reshape(-1, x.shape[-1]).shape[0]
        return fp8_gemm(q, self.input_scale, self.weight, self.weight_scale, m)


class RuntimeScaleLinear(StaticFP8Linear):
    """The reference's runtime-scale variant: identical arithmetic, the scale is a runtime
    value (`inverse_scale` may be reassigned between calls, `input_scale` refilled)."""

    def __call__(self, x):
        q, _ = quantize_activation(x, L.QUANT_STATIC, self.inverse_scale)
        m = x.reshape(-1, x.shape[-1]).shape[0]
        return fp8_gemm(q, self.input_scale, self.weight, self.weight_scale, m)


class FP8Linear:
    """Per-output-channel FP8 weights x per-token dynamic activation scales."""

    def __init__(self, weight):
        _need(weight.is_cuda and weight.ndim == 2 and weight.shape[0] % 16 == weight.shape[1] % 16 == 0,
              "weight: CUDA [N,K], N and K multiples of 16")
        self.weight, w_scale = quantize_weight(weight.detach().to(BF16), per_channel=True)
        self.scale = w_scale.reshape(1, -1)

    def __call__(self, x):
        _need(x.is_cuda and x.dtype == BF16, "x: CUDA bf16")
        q, s = quantize_activation(x, L.QUANT_ROWWISE)
        m = x.reshape(-1, x.shape[-1]).shape[0]
        y = fp8_gemm(q, s, self.weight, self.scale.reshape(-1), m)
        return y.reshape(*x.shape[:-1], self.weight.shape[0])


# ---------------------------------------------------------------------------- W4A16

def pack_int4(w):
    """bf16 [N,K] -> (packed uint8 [N, K/2], bf16 scales [N, K/128]) symmetric group 128."""
    _bf16_cuda(w)
    w = w.contiguous()
    n, k = w.shape
    _need(k % 128 == 0, "K must be a multiple of 128")
    packed = torch.empty((n, k // 2), device=w.device, dtype=torch.uint8)
    scales = torch.empty((n, k // 128), device=w.device, dtype=BF16)
    call("ffb_pack_int4", ptr(w), ptr(packed), ptr(scales), n, k, stream_ptr(w.device))
    return packed, scales


class Int4:
    """W4A16 linear (symmetric int4, group 128, bf16 scales) on tcgen05 bf16 MMAs."""

    def __init__(self, w, oracle=False):
        n, k = w.shape
        _need(n % 128 == 0 and k % 128 == 0, "N and K must be multiples of 128")
        self.packed, self.scales = pack_int4(w.detach().to(BF16))
        self.shape = (n, k)
        self.group = 128

    def __call__(self, x):
        _bf16_cuda(x)
        flat = x.reshape(-1, x.shape[-1]).contiguous()
        m, k = flat.shape
        n = self.shape[0]
        out = torch.empty((m, n), device=x.device, dtype=BF16)
        call("ffb_w4a16_gemm", ptr(flat), ptr(self.packed), ptr(self.scales), L.EPI_BF16, ptr(out), None, 1, 0, m,
             n, k, stream_ptr(x.device))
        return out.reshape(*x.shape[:-1], n)


# ---------------------------------------------------------------------------- input packing

def _pack(rgb, pixels):
    _need(rgb.is_cuda and rgb.dtype == torch.uint8, "rgb: CUDA uint8 canvas")
    _need(rgb.dim() in (3, 4) and rgb.shape[-1] == 3 and rgb.is_contiguous(),
          "rgb must be a contiguous [H, W, 3] or [n, H, W, 3] canvas")
    n = rgb.shape[0] if rgb.dim() == 4 else 1
    h, w = rgb.shape[-3], rgb.shape[-2]
    _need(h % 32 == 0 and w % 32 == 0, f"canvas {h}x{w}: sides must be multiples of 32")
    rows = n * (h // 16) * (w // 16)
    if pixels is None:
        pixels = torch.empty((rows, 1536), device=rgb.device, dtype=BF16)
    _need(pixels.shape == (rows, 1536) and pixels.dtype == BF16 and pixels.is_contiguous() and pixels.is_cuda,
          f"pixels must be a contiguous CUDA bf16 [{rows}, 1536] tensor")
    call("ffb_pack_rgb_batch", ptr(rgb), ptr(pixels), n, h, w, stream_ptr(rgb.device))
    return pixels


def pack_rgb(rgb, side=None, pixels=None):
    """Square canvas [S, S, 3] uint8 -> patch rows [(S/16)^2, 1536] bf16 (the reference's
    `pack_rgb[grid](rgb, pixels, S, N, 1024)`, `_legacy/sub10_runtime.py:21-29`).  A
    [n, S, S, 3] batch gives n canvases' rows one after the other."""
    if side is not None:
        _need(rgb.shape[-3] == rgb.shape[-2] == side, f"canvas is not {side}x{side}")
    return _pack(rgb, pixels)


def pack_rectangle(rgb, width=None, pixels=None):
    """Canvas [H, W, 3] uint8 (H, W multiples of 32) -> [(H/16)(W/16), 1536] bf16
    (`pack_rectangle`, `_family/depth_runtime.py:18-25`)."""
    if width is not None:
        _need(rgb.shape[-2] == width, f"canvas width is not {width}")
    return _pack(rgb, pixels)


# ---------------------------------------------------------------------------- vision tower

_VISION_EPI = {"bias": L.EPI_BIAS, "res": L.EPI_BIAS_RES, "gelu_tanh": L.EPI_BIAS_GELU_TANH,
               "gelu_erf": L.EPI_BIAS_GELU_ERF}


def vision_linear(x, weight, bias=None, epilogue="bias", res=None, out=None, feature_tile=0, splits=None):
    """bf16 linear of the vision tower on tcgen05: epilogue "bias" = bf16(x W^T + b), "res" =
    bf16(res + that), "gelu_tanh" / "gelu_erf" = bf16(gelu(that)) (nn.Linear + the residual
    add or activation that follows it in the HF vision blocks and mergers).  feature_tile /
    splits: 0 / None = the library's plan."""
    _need(epilogue in _VISION_EPI, f"unknown epilogue {epilogue!r}")
    _bf16_cuda(x, weight)
    _need(x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1], "x [M, K], weight [N, K]")
    _need(x.is_contiguous() and weight.is_contiguous(), "contiguous operands")
    m, k = x.shape
    n = weight.shape[0]
    if bias is not None:
        _bf16_cuda(bias)
        _need(bias.shape == (n,) and bias.is_contiguous(), "bias [N]")
    if epilogue == "res":
        _need(res is not None and res.shape == (m, n) and res.is_contiguous(), "res [M, N] contiguous")
        _bf16_cuda(res)
    out = torch.empty(m, n, dtype=BF16, device=x.device) if out is None else out
    tile, plan_splits, _ = L.bf16_gemm_plan(m, n, k)
    tile = int(feature_tile) or tile
    splits = plan_splits if splits is None else int(splits)
    ws = counters = None
    if splits > 1:
        ws = torch.empty(splits, m, n, dtype=torch.float32, device=x.device)
        counters = torch.zeros(-(-m // 128) * -(-n // tile), dtype=torch.int32, device=x.device)
    call("ffb_bf16_gemm", ptr(x), ptr(weight), ptr(bias), ptr(res), _VISION_EPI[epilogue], ptr(out), tile, splits,
         ptr(ws), ptr(counters), m, n, k, stream_ptr(x.device))
    return out


def add_layernorm(a, b, module):
    """residual = bf16(a + b), out = LayerNorm(residual) (`_legacy/lower_kernels.py:130-136`);
    with b None only the LayerNorm (residual is a).  `module` has .weight, .bias, .eps."""
    _need(a.is_contiguous() and (b is None or (b.shape == a.shape and b.is_contiguous())), "a, b contiguous")
    _bf16_cuda(a, module.weight, module.bias)
    d = a.shape[-1]
    out = torch.empty_like(a)
    residual = torch.empty_like(a) if b is not None else a
    call("ffb_add_layernorm", ptr(a), ptr(b), ptr(module.weight), ptr(module.bias), float(module.eps),
         ptr(residual) if b is not None else None, ptr(out), a.numel() // d, d, stream_ptr(a.device))
    return residual, out


def vision_rope(q, k, cos, sin, block=512):
    """The reference's `vision_rope` (`_legacy/search_kernels.py:127-134`): q, k [n, h, d]
    (any row stride), cos, sin [n, d] fp32; returns yq, yk [n, h, d] in q's dtype."""
    _need(q.shape == k.shape and q.dim() == 3, "q, k [n, h, d]")
    _bf16_cuda(q, k)
    n, h, d = q.shape
    qkv = torch.zeros(n, 3, h, d, dtype=BF16, device=q.device)
    qkv[:, 0] = q
    qkv[:, 1] = k
    yq = torch.empty(h, n, d, dtype=BF16, device=q.device)
    yk = torch.empty_like(yq)
    yv = torch.empty_like(yq)
    cos, sin = cos.float().contiguous(), sin.float().contiguous()  # held until the launch is enqueued
    call("ffb_vision_rope", ptr(qkv), ptr(cos), ptr(sin), n, h, d, d, ptr(yq), ptr(yk), ptr(yv), stream_ptr(q.device))
    return yq.transpose(0, 1).contiguous(), yk.transpose(0, 1).contiguous()


def vision_attention(q, k, v, d, scale):
    """Non-causal attention over one image's patches: q, k, v [H, T, 128] bf16 (head dim d
    zero-padded to 128); returns [T, H * d] bf16 (the vision blocks' SDPA)."""
    _bf16_cuda(q, k, v)
    _need(q.shape == k.shape == v.shape and q.dim() == 3 and q.shape[2] == 128, "q, k, v [H, T, 128]")
    _need(q.is_contiguous() and k.is_contiguous() and v.is_contiguous(), "contiguous q, k, v")
    h, t, _ = q.shape
    out = torch.empty(t, h * d, dtype=BF16, device=q.device)
    call("ffb_attention_full", ptr(q), ptr(k), ptr(v), ptr(out), t, h, int(d), float(scale), stream_ptr(q.device))
    return out

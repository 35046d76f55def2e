"""Generates tests/golden/reference_ops.pt: outputs of the REFERENCE's own code for the ops
on the prefill + choice-scoring path, on small seeded inputs, to pin the oracle (and the
CUDA kernels) to the reference.

Usage (in a container that has the FastForward source tree; nothing here runs on the GPU
box):

    python tests/golden/make_golden.py <path of the FastForward checkout>

What runs: the reference's Triton kernels (`_legacy/lower_kernels.add_rms`,
`_legacy/sub10_runtime.fast_norm`, `_legacy/broad_kernels.qk_pair`,
`_legacy/limit_kernels.attention_direct` / `lm_readout`, `_legacy/search_kernels.swiglu`,
`_family/depth_fp8.quantize_runtime`, `_legacy/fp8_private.quantize_rows`,
`_legacy/sub10_runtime.pack_rgb`, `_family/depth_runtime.pack_rectangle`,
`_legacy/search_kernels.vision_rope`) under Triton's
CPU interpreter (TRITON_INTERPRET=1), the reference's torch code (`StaticFP8Linear`,
`FP8Linear`, `RuntimeScaleLinear` through CPU `torch._scaled_mm`, `Int4`), and
transformers' Qwen3-VL `get_rope_index` / `Qwen3VLTextRotaryEmbedding`.

The interpreter is made faithful to the GPU where it is not, by patching it (not the
reference):
  * fp32 -> bf16 and fp32 -> e4m3 casts round to nearest even (the interpreter truncates;
    GPU Triton rounds);
  * `tl.dot` on bf16 operands multiplies the values (the interpreter multiplies the raw
    16-bit words) with a float64 accumulation rounded to fp32;
  * fp32 `tl.sum` is evaluated exactly (float64) and rounded once to fp32.  This is the
    one deliberate deviation from the GPU reference, shared by the oracle and the CUDA
    kernels: the reference's fp32 reduction order is unspecified, an exact sum is not.
    The fixtures of add_rms / fast_norm / qk_pair / lm_readout are therefore the
    reference's rounding points under an exact fp32 reduction, not the bytes of its GPU
    tree sum;
  * `libdevice.exp` / `libdevice.div_rn` (CUDA-only) map to `tl.exp` / `tl.div_rn`.
`sub10_runtime` and `night_runtime` import an un-vendored module
(`_legacy/decision_pilot_contract.py:11-13`); it is replaced by an empty stand-in, which
none of the functions used here touch.
"""
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = Path(__file__).resolve().with_name("reference_ops.pt")
BF16 = torch.bfloat16


# ----------------------------------------------------------------------------- interpreter
def _patch_interpreter():
    import triton.language as tl
    from triton.runtime import interpreter as itp

    orig_convert = itp._convert_float

    def convert(data, src, dst, rounding_mode):
        if src == tl.float32 and dst == tl.bfloat16:
            t = torch.from_numpy(np.ascontiguousarray(data).view(np.float32).copy())
            return t.to(BF16).view(torch.int16).numpy().view(np.uint16).reshape(data.shape)
        if src == tl.float32 and dst in (tl.float8e4nv,):
            t = torch.from_numpy(np.ascontiguousarray(data).view(np.float32).copy())
            return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy().reshape(data.shape)
        return orig_convert(data, src, dst, rounding_mode)

    itp._convert_float = convert

    orig_cast = itp.InterpreterBuilder.cast_impl

    def cast_impl(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if s == tl.float32 and d == tl.float8e4nv:
            data = convert(src.data, s, d, None).view(itp._get_np_dtype(dst_type))
            return itp.TensorHandle(data, d)
        return orig_cast(self, src, dst_type)

    itp.InterpreterBuilder.cast_impl = cast_impl
    itp.InterpreterBuilder.create_fp_trunc = lambda self, src, dst_type: self.cast_impl(src, dst_type)

    orig_dot = itp.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            def f32(h):
                if h.dtype.scalar == tl.bfloat16:
                    return (h.data.astype(np.uint32) << 16).view(np.float32)
                return h.data.astype(np.float32)
            acc = np.matmul(f32(a).astype(np.float64), f32(b).astype(np.float64)) + d.data.astype(np.float64)
            return itp.TensorHandle(acc.astype(np.float32), d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    itp.InterpreterBuilder.create_dot = create_dot

    orig_sum = itp.ReduceOps.sum

    def exact_sum(self, input):
        data = input.handle.data
        if data.dtype == np.float32:
            s = np.sum(data.astype(np.float64), axis=self.axis, keepdims=self.keep_dims).astype(np.float32)
            return self.to_tensor(s, input.dtype)
        return orig_sum(self, input)

    itp.ReduceOps.sum = exact_sum


class _Libdevice:
    """Stand-in for CUDA's libdevice namespace inside interpreted kernels; resolved at call
    time, when the interpreter has patched `triton.language`."""

    def __getattr__(self, name):
        import triton.language as tl
        return {"exp": tl.exp, "div_rn": tl.div_rn}[name]


def _import_reference(root):
    sys.path.insert(0, str(Path(root) / "src"))
    stub = types.ModuleType("fastforward_accel._legacy.decision_pilot_contract")
    stub.__file__ = "<stand-in>"

    class _Unused:
        def __init__(self, *a, **k):
            pass

    def _attr(name):
        if name.startswith("__"):
            raise AttributeError(name)
        return _Unused

    stub.__getattr__ = _attr
    sys.modules[stub.__name__] = stub
    from fastforward_accel._legacy import lower_kernels, limit_kernels, broad_kernels, search_kernels, fp8_private
    from fastforward_accel._legacy import sub10_runtime
    from fastforward_accel._family import depth_fp8, night_runtime, depth_runtime
    search_kernels.libdevice = _Libdevice()
    limit_kernels.libdevice = _Libdevice()
    return types.SimpleNamespace(lower=lower_kernels, limit=limit_kernels, broad=broad_kernels,
                                 search=search_kernels, fp8p=fp8_private, sub10=sub10_runtime, depth=depth_fp8,
                                 night=night_runtime, depth_rt=depth_runtime)


class _ClaimsCuda(torch.Tensor):
    """CPU tensor that answers `is_cuda` with True, so the reference's device asserts in
    `FP8Linear` let its (device-independent) torch code run on the CPU."""

    @property
    def is_cuda(self):
        return True


def _norm(w, eps=1e-6):
    return types.SimpleNamespace(weight=w, variance_epsilon=eps)


def _randn(g, *shape, std=1.0):
    return (torch.randn(*shape, generator=g) * std).to(BF16)


def main(root):
    _patch_interpreter()
    R = _import_reference(root)
    g = torch.Generator().manual_seed(2024)
    out = {}

    # add_rms with deepstack rows (lower_kernels.py:24-32)
    for H in (2048, 2560):
        T, start, nv = 6, 1, 3
        a, b = _randn(g, 1, T, H), _randn(g, 1, T, H)
        deep = _randn(g, nv, H)
        w = (1 + 0.1 * torch.randn(H, generator=g)).to(BF16)
        res, y = R.lower.add_rms(a, b, deep, _norm(w), start, nv)
        out[f"add_rms_{H}"] = dict(a=a, b=b, deep=deep, w=w, start=start, nv=nv, eps=1e-6, residual=res, out=y)

    # fast_norm / rms_one (sub10_runtime.py:31-41)
    x = _randn(g, 1, 5, 2560)
    w = (1 + 0.1 * torch.randn(2560, generator=g)).to(BF16)
    out["fast_norm"] = dict(x=x, w=w, eps=1e-6, out=R.sub10.fast_norm(x, _norm(w)))

    # qk_pair (broad_kernels.py:63-74): q/k are strided views of the packed qkv row
    T, HQ, HK, D = 7, 4, 2, 128
    qkv = _randn(g, 1, T, (HQ + 2 * HK) * D)
    q = qkv[..., :HQ * D].view(1, T, HQ, D)
    k = qkv[..., HQ * D:(HQ + HK) * D].view(1, T, HK, D)
    qn = (1 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    kn = (1 + 0.1 * torch.randn(D, generator=g)).to(BF16)
    pos = torch.arange(T, dtype=torch.float32)
    ang = pos[:, None] * (5e6 ** (-torch.arange(0, D, 2).float() / D))[None, :]
    emb = torch.cat((ang, ang), -1)
    cos, sin = emb.cos().to(BF16)[None], emb.sin().to(BF16)[None]
    yq, yk = R.broad.qk_pair(q, k, _norm(qn), _norm(kn), cos, sin)
    out["qk_pair"] = dict(qkv=qkv, HQ=HQ, HK=HK, q_norm=qn, k_norm=kn, cos=cos, sin=sin, eps=1e-6, yq=yq, yk=yk)

    # attention_direct (limit_kernels.py:36-45), causal and with selected positions
    S, HQ, HK, D = 70, 4, 2, 128
    qa = _randn(g, 1, HQ, S, D)
    ka = _randn(g, 1, HK, S, D)
    va = _randn(g, 1, HK, S, D)
    scale = D ** -0.5
    ya = R.limit.attention_direct(qa, ka, va, scale)
    sel = torch.tensor([69, 33])
    ys = R.limit.attention_direct(qa[:, :, sel].contiguous(), ka, va, scale, positions=sel)
    out["attention"] = dict(q=qa, k=ka, v=va, scale=scale, out=ya, positions=sel, out_selected=ys)

    # lm_readout (limit_kernels.py:60-66)
    H = 2560
    xr = _randn(g, 1, H)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).to(BF16)
    head = _randn(g, 8, H, std=0.02)
    out["lm_readout"] = dict(x=xr, norm=nw, head=head, eps=1e-6, out=R.limit.lm_readout(xr, _norm(nw), head))

    # swiglu on the two halves of a packed gate/up row (search_kernels.py:18-23)
    I = 320
    gu = _randn(g, 9, 2 * I, std=2.0)
    out["swiglu"] = dict(gu=gu, I=I, out=R.search.swiglu(gu[:, :I], gu[:, I:]))

    # static activation quant (depth_fp8.py:8-19): rows padded to 16
    xq = _randn(g, 13, 256, std=3.0)
    inv = 448.0 / 9.0
    q8, m = R.depth.quantize_runtime(xq, types.SimpleNamespace(inverse_scale=inv))
    out["quant_static"] = dict(x=xq, inverse_scale=inv, q8=q8.view(torch.uint8), m=m)

    # per-token activation quant (fp8_private.py:11-18), launched as FP8Linear does
    import triton
    xr2 = _randn(g, 13, 300, std=2.0)
    pad = triton.cdiv(13, 16) * 16
    q8r = torch.empty((pad, 300), dtype=torch.float8_e4m3fn)
    sr = torch.empty((pad, 1), dtype=torch.float32)
    R.fp8p.quantize_rows[(pad,)](xr2, q8r, sr, 13, 300, triton.next_power_of_2(300), num_warps=4)
    out["quant_rows"] = dict(x=xr2, q8=q8r.view(torch.uint8), scale=sr)

    # weight quantisation: per tensor (limit_kernels.py:122-127) and per channel
    # (fp8_private.py:22-27)
    wq = _randn(g, 64, 256, std=0.02)
    st = R.limit.StaticFP8Linear(wq, inverse_scale=448.0 / 9.0)
    pc = R.fp8p.FP8Linear(wq.as_subclass(_ClaimsCuda))
    out["weight_quant"] = dict(w=wq, w8_tensor=st.weight.view(torch.uint8), scale_tensor=st.weight_scale,
                               w8_channel=torch.Tensor(pc.weight).view(torch.uint8),
                               scale_channel=torch.Tensor(pc.scale))

    # the static-scale FP8 linear end to end on the CPU (depth_fp8.py:22-26)
    try:
        rs = R.depth.RuntimeScaleLinear(wq, inverse_scale=448.0 / 9.0)
        xs = _randn(g, 5, 256, std=2.0)
        out["runtime_scale_linear"] = dict(x=xs, w=wq, inverse_scale=448.0 / 9.0, out=rs(xs))
    except Exception as e:  # CPU torch._scaled_mm not available in this torch build
        print("runtime_scale_linear skipped:", e)

    # the reference's asymmetric int4 (night_runtime.py:15-30); the device packing call is
    # replaced by identity (only the quantisation arithmetic is recorded)
    w4 = _randn(g, 16, 256, std=0.02)
    real_ops = torch.ops

    class _Aten:
        def __getattr__(self, name):
            if name == "_convert_weight_to_int4pack":
                return lambda p, n: p
            return getattr(real_ops.aten, name)

    class _Torch:
        ops = types.SimpleNamespace(aten=_Aten())

        def __getattr__(self, name):
            return getattr(torch, name)

    R.night.torch = _Torch()
    try:
        i4 = R.night.Int4(w4, oracle=True)
    finally:
        R.night.torch = torch
    out["int4_asym"] = dict(w=w4, scales=i4.scales, deq=i4.oracle)

    # Qwen3-VL M-RoPE positions and tables (transformers)
    from transformers.models.qwen3_vl import modeling_qwen3_vl as hf
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    fake = types.SimpleNamespace(config=types.SimpleNamespace(vision_config=types.SimpleNamespace(
        spatial_merge_size=2)))
    fake.get_vision_position_ids = types.MethodType(hf.Qwen3VLModel.get_vision_position_ids, fake) \
        if hasattr(hf.Qwen3VLModel, "get_vision_position_ids") else None
    cfg = Qwen3VLTextConfig(head_dim=128, hidden_size=2560, num_attention_heads=32, num_key_value_heads=8,
                            rope_parameters=dict(rope_type="default", rope_theta=5_000_000.0,
                                                 mrope_section=[24, 20, 20], mrope_interleaved=True))
    rot = hf.Qwen3VLTextRotaryEmbedding(cfg)
    cases = []
    for n_tokens, start, gh, gw in ((80, 5, 8, 12), (320, 0, 32, 32), (40, 3, 12, 6)):
        nv = (gh // 2) * (gw // 2)
        ids = torch.full((1, n_tokens), 7, dtype=torch.long)
        types_ = torch.zeros((1, n_tokens), dtype=torch.int32)
        types_[0, start:start + nv] = 1
        pos, _ = hf.Qwen3VLModel.get_rope_index(fake, ids, types_, image_grid_thw=torch.tensor([[1, gh, gw]]))
        x = torch.zeros(1, n_tokens, 128, dtype=BF16)
        c, s = rot(x, pos)
        cases.append(dict(n_tokens=n_tokens, image_start=start, grid_h=gh, grid_w=gw, position_ids=pos[:, 0],
                          cos=c[0], sin=s[0]))
    out["mrope"] = cases

    # input packing: pack_rgb (sub10_runtime.py:21-29) and pack_rectangle
    # (depth_runtime.py:18-25), launched as the reference launches them (1024 per program)
    import triton
    gp = torch.Generator().manual_seed(77)
    packs = []
    for kind, (H, W) in (("square", (64, 64)), ("square", (96, 96)), ("rectangle", (64, 160)),
                         ("rectangle", (96, 32))):
        rgb = torch.randint(0, 256, (H, W, 3), generator=gp, dtype=torch.uint8)
        rgb.view(-1)[:256] = torch.arange(256, dtype=torch.uint8)  # every byte value
        pixels = torch.empty(((H // 16) * (W // 16), 1536), dtype=BF16)
        grid = (triton.cdiv(pixels.numel(), 1024),)
        if kind == "square":
            R.sub10.pack_rgb[grid](rgb, pixels, W, pixels.numel(), 1024, enable_fp_fusion=False)
        else:
            R.depth_rt.pack_rectangle[grid](rgb, pixels, W, pixels.numel(), 1024, enable_fp_fusion=False)
        packs.append(dict(kind=kind, height=H, width=W, rgb=rgb, pixels=pixels))
    out["pack_rgb"] = packs

    # vision_rope (search_kernels.py:111-134): q/k strided views of the packed qkv rows, as
    # NativeNormVision.core passes them (scaled_qwen_runtime.py:47-48)
    gv = torch.Generator().manual_seed(91)
    n, hv, dv = 24, 2, 64
    qkv_v = _randn(gv, n, 3, hv, dv)
    qv, kv = qkv_v[:, 0], qkv_v[:, 1]
    ang = torch.rand((n, dv // 2), generator=gv) * 20.0
    emb = torch.cat([ang, ang], dim=-1)
    cv, sv = emb.cos(), emb.sin()
    yq, yk = R.search.vision_rope(qv, kv, cv, sv)
    out["vision_rope"] = dict(q=qv.contiguous(), k=kv.contiguous(), cos=cv, sin=sv, yq=yq, yk=yk)

    out["_note"] = "outputs of the reference's own code; see make_golden.py"
    torch.save(out, OUT)
    print(OUT, sorted(k for k in out if not k.startswith("_")))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])

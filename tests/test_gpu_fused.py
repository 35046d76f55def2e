"""Fused GEMM prologues (ffb_fp8_gemm_fused, ffb_fp8_gemm_qk_rope_fused) against the
separate launches they replace (ffb_quantize_fp8 / ffb_add_rmsnorm / ffb_rmsnorm, then
ffb_fp8_gemm / ffb_fp8_gemm_qk_rope), through the C ABI: every output byte identical --
the FP8 operand, the per-row scales, the residual rows and the GEMM result -- on two calls
in a row that share the grid-barrier words.  The engine's fused forward is then compared
with its unfused forward (bit-identical logits and residual streams)."""
import ctypes

import pytest
import torch

from fastforward_b200 import _lib as L
from fastforward_b200._lib import call, ptr
from tests._util import assert_bytes_equal

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = "cuda"


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _randn(shape, seed, std=1.0, dtype=BF16):
    return (torch.randn(shape, generator=_g(seed)) * std).to(dtype).to(DEV)


def _s():
    return torch.cuda.current_stream().cuda_stream


def _weights(N, K, seed):
    w = _randn((N, K), seed, 0.02)
    w8 = torch.empty((N, K), dtype=torch.uint8, device=DEV)
    sc = torch.empty(N, dtype=torch.float32, device=DEV)
    ws = torch.empty(N, dtype=torch.float32, device=DEV)
    call("ffb_quantize_weight_fp8", ptr(w), 1, ptr(w8), ptr(sc), ptr(ws), N, K, _s())
    return w8, sc


def _act_scale(M, rowwise, bound=6.0):
    """(per-row scale buffer or the static per-tensor scale, inverse multiplier)"""
    if rowwise:
        return torch.zeros(M, dtype=torch.float32, device=DEV), 0.0
    return torch.full((1,), bound / 448.0, dtype=torch.float32, device=DEV), 448.0 / bound


def _outputs(M, N, epi, splits):
    if epi == L.EPI_F32_PARTIAL:
        return None, torch.zeros((splits, M, N), dtype=torch.float32, device=DEV)
    n_out = N // 2 if epi == L.EPI_SWIGLU else N
    return torch.zeros((M, n_out), dtype=BF16, device=DEV), None


def _gemm(a8, sa, rowwise, w8, wsc, epi, out, ws, splits, bn, M, N, K, pro=None):
    args = (ptr(a8), ptr(sa), int(rowwise), ptr(w8), ptr(wsc), 1, epi, ptr(out), ptr(ws), splits, bn, M, N, K, _s())
    if pro is None:
        call("ffb_fp8_gemm", *args)
    else:
        call("ffb_fp8_gemm_fused", ctypes.addressof(pro), *args)


def _result(out, ws):
    return out if out is not None else ws


@pytest.mark.parametrize("M,K,N,epi,bn,splits", [
    (320, 4096, 2560, L.EPI_F32_PARTIAL, 256, 4),     # o_proj of the 4B model
    (320, 9728, 2560, L.EPI_F32_PARTIAL, 256, 4),     # down_proj of the 4B model
    (1, 9728, 2560, L.EPI_BF16, 128, 1),              # the tail's one-row down_proj
    (300, 2048, 19456, L.EPI_SWIGLU, 256, 1),         # ragged rows, 148-CTA grid
    (77, 4096, 2560, L.EPI_F32_PARTIAL, 128, 3),      # ragged rows, one token tile
    (1030, 5120, 1024, L.EPI_BF16, 128, 1),           # more rows than CTAs x batch
])
@pytest.mark.parametrize("rowwise", [True, False])
def test_quant_prologue_matches_separate_launches(M, K, N, epi, bn, splits, rowwise):
    x = _randn((M, K), 11)
    w8, wsc = _weights(N, K, 12)
    sync = torch.zeros(2, dtype=torch.int32, device=DEV)
    qmode = L.QUANT_ROWWISE if rowwise else L.QUANT_STATIC
    # separate launches
    a8_ref = torch.zeros((M, K), dtype=torch.uint8, device=DEV)
    sa_ref, inv = _act_scale(M, rowwise)
    call("ffb_quantize_fp8", ptr(x), qmode, inv, ptr(a8_ref), ptr(sa_ref) if rowwise else None, M, K, _s())
    out_ref, ws_ref = _outputs(M, N, epi, splits)
    _gemm(a8_ref, sa_ref, rowwise, w8, wsc, epi, out_ref, ws_ref, splits, bn, M, N, K)
    for rep in range(2):  # two calls in a row on the same barrier words
        a8 = torch.full((M, K), 0x7F, dtype=torch.uint8, device=DEV)
        sa, _ = _act_scale(M, rowwise)
        out, ws = _outputs(M, N, epi, splits)
        pro = L.Prologue(kind=L.PRO_QUANT, x=ptr(x), quant_mode=qmode, inv_scale=inv, sync=ptr(sync))
        _gemm(a8, sa, rowwise, w8, wsc, epi, out, ws, splits, bn, M, N, K, pro)
        torch.cuda.synchronize()
        assert_bytes_equal(a8, a8_ref, f"a8 (call {rep})")
        if rowwise:
            assert_bytes_equal(sa, sa_ref, f"row scales (call {rep})")
        assert_bytes_equal(_result(out, ws), _result(out_ref, ws_ref), f"gemm output (call {rep})")
    assert L.device_error() == 0
    assert sync[0].item() == 0  # every barrier completed (arrival count back to zero)


@pytest.mark.parametrize("M,K,N,epi,bn,splits,add", [
    (320, 2560, 19456, L.EPI_SWIGLU, 256, 1, "b32x4"),   # gate/up after the split-K o_proj
    (320, 2560, 2560, L.EPI_F32_PARTIAL, 256, 2, "b32x3+deep"),
    (96, 2048, 12288, L.EPI_SWIGLU, 256, 1, "bf16"),
    (1, 2560, 19456, L.EPI_SWIGLU, 256, 1, "b32x1"),     # the tail's one row
    (200, 5120, 1024, L.EPI_BF16, 128, 1, "none"),        # plain RMSNorm (layer-0 input)
])
@pytest.mark.parametrize("rowwise", [True, False])
def test_add_rmsnorm_prologue_matches_separate_launches(M, K, N, epi, bn, splits, add, rowwise):
    a = _randn((M, K), 21)
    w = (1 + 0.1 * torch.randn(K, generator=_g(22))).to(BF16).to(DEV)
    w8, wsc = _weights(N, K, 23)
    sync = torch.zeros(2, dtype=torch.int32, device=DEV)
    qmode = L.QUANT_ROWWISE if rowwise else L.QUANT_STATIC
    b = b32 = deep = None
    nsp, start, nv = 0, 0, 0
    if add.startswith("b32"):
        nsp = int(add[4])
        b32 = _randn((nsp, M, K), 24, 0.5, torch.float32)
        if add.endswith("+deep"):
            start, nv = 7, min(64, M - 7)
            deep = _randn((nv, K), 25)
    elif add == "bf16":
        b = _randn((M, K), 26)
    eps = 1e-6
    # separate launches
    a8_ref = torch.zeros((M, K), dtype=torch.uint8, device=DEV)
    sa_ref, inv = _act_scale(M, rowwise, bound=4.0)
    res_ref = torch.zeros((M, K), dtype=BF16, device=DEV)
    if add == "none":
        call("ffb_rmsnorm", ptr(a), ptr(w), eps, None, qmode, inv, ptr(a8_ref), ptr(sa_ref) if rowwise else None, M, K,
             _s())
    else:
        call("ffb_add_rmsnorm", ptr(a), ptr(b), ptr(b32), nsp, ptr(deep), start, nv, ptr(w), eps, ptr(res_ref), None,
             qmode, inv, ptr(a8_ref), ptr(sa_ref) if rowwise else None, M, K, _s())
    out_ref, ws_ref = _outputs(M, N, epi, splits)
    _gemm(a8_ref, sa_ref, rowwise, w8, wsc, epi, out_ref, ws_ref, splits, bn, M, N, K)
    for rep in range(2):
        a8 = torch.full((M, K), 0x7F, dtype=torch.uint8, device=DEV)
        sa, _ = _act_scale(M, rowwise, bound=4.0)
        res = torch.zeros((M, K), dtype=BF16, device=DEV)
        out, ws = _outputs(M, N, epi, splits)
        pro = L.Prologue(kind=L.PRO_ADD_RMSNORM, x=ptr(a), norm_w=ptr(w), eps=eps, quant_mode=qmode, inv_scale=inv,
                         sync=ptr(sync))
        if add != "none":
            pro.add, pro.b, pro.b32, pro.splits, pro.residual = 1, ptr(b), ptr(b32), nsp, ptr(res)
            if deep is not None:
                pro.deep, pro.start, pro.nv = ptr(deep), start, nv
        _gemm(a8, sa, rowwise, w8, wsc, epi, out, ws, splits, bn, M, N, K, pro)
        torch.cuda.synchronize()
        assert_bytes_equal(a8, a8_ref, f"a8 (call {rep})")
        if rowwise:
            assert_bytes_equal(sa, sa_ref, f"row scales (call {rep})")
        if add != "none":
            assert_bytes_equal(res, res_ref, f"residual (call {rep})")
        assert_bytes_equal(_result(out, ws), _result(out_ref, ws_ref), f"gemm output (call {rep})")
    assert L.device_error() == 0


@pytest.mark.parametrize("T,H,HQ,HK", [(320, 2560, 32, 8), (100, 2048, 16, 8)])
def test_qk_rope_with_prologue_matches_separate_launches(T, H, HQ, HK):
    N = (HQ + 2 * HK) * 128
    a = _randn((T, H), 31)
    b32 = _randn((4, T, H), 32, 0.5, torch.float32)
    w = (1 + 0.1 * torch.randn(H, generator=_g(33))).to(BF16).to(DEV)
    w8, wsc = _weights(N, H, 34)
    qn = (1 + 0.1 * torch.randn(128, generator=_g(35))).to(BF16).to(DEV)
    kn = (1 + 0.1 * torch.randn(128, generator=_g(36))).to(BF16).to(DEV)
    ang = torch.randn((T, 64), generator=_g(37))
    cos = torch.cat([ang.cos(), ang.cos()], 1).to(BF16).to(DEV)
    sin = torch.cat([ang.sin(), ang.sin()], 1).to(BF16).to(DEV)
    sync = torch.zeros(2, dtype=torch.int32, device=DEV)

    def heads():
        return [torch.zeros((h, T, 128), dtype=BF16, device=DEV) for h in (HQ, HK, HK)]

    def rope(a8, sa, ys, pro=None):
        args = (ptr(a8), ptr(sa), 1, ptr(w8), ptr(wsc), 1, ptr(qn), ptr(kn), 1e-6, ptr(cos), ptr(sin),
                ptr(ys[0]), ptr(ys[1]), ptr(ys[2]), T, HQ, HK, H, _s())
        if pro is None:
            call("ffb_fp8_gemm_qk_rope", *args)
        else:
            call("ffb_fp8_gemm_qk_rope_fused", ctypes.addressof(pro), *args)

    a8_ref = torch.zeros((T, H), dtype=torch.uint8, device=DEV)
    sa_ref = torch.zeros(T, dtype=torch.float32, device=DEV)
    res_ref = torch.zeros((T, H), dtype=BF16, device=DEV)
    call("ffb_add_rmsnorm", ptr(a), None, ptr(b32), 4, None, 0, 0, ptr(w), 1e-6, ptr(res_ref), None,
         L.QUANT_ROWWISE, 0.0, ptr(a8_ref), ptr(sa_ref), T, H, _s())
    y_ref = heads()
    rope(a8_ref, sa_ref, y_ref)
    for rep in range(2):
        a8 = torch.zeros((T, H), dtype=torch.uint8, device=DEV)
        sa = torch.zeros(T, dtype=torch.float32, device=DEV)
        res = torch.zeros((T, H), dtype=BF16, device=DEV)
        ys = heads()
        pro = L.Prologue(kind=L.PRO_ADD_RMSNORM, x=ptr(a), b32=ptr(b32), splits=4, add=1, residual=ptr(res),
                         norm_w=ptr(w), eps=1e-6, quant_mode=L.QUANT_ROWWISE, sync=ptr(sync))
        rope(a8, sa, ys, pro)
        torch.cuda.synchronize()
        assert_bytes_equal(res, res_ref, "residual")
        assert_bytes_equal(a8, a8_ref, "a8")
        for name, y, yr in zip("qkv", ys, y_ref):
            assert_bytes_equal(y, yr, f"{name} heads (call {rep})")
    assert L.device_error() == 0


def test_prologue_argument_errors():
    sync = torch.zeros(2, dtype=torch.int32, device=DEV)
    x = torch.zeros((4, 256), dtype=BF16, device=DEV)
    a8 = torch.zeros((4, 256), dtype=torch.uint8, device=DEV)
    sa = torch.zeros(4, dtype=torch.float32, device=DEV)
    w8 = torch.zeros((256, 256), dtype=torch.uint8, device=DEV)
    wsc = torch.ones(256, dtype=torch.float32, device=DEV)
    out = torch.zeros((4, 256), dtype=BF16, device=DEV)
    pro = L.Prologue(kind=L.PRO_QUANT, x=ptr(x), quant_mode=L.QUANT_ROWWISE, sync=ptr(sync))
    with pytest.raises(ValueError, match="a_per_row"):
        _gemm(a8, sa, False, w8, wsc, L.EPI_BF16, out, None, 1, 128, 4, 256, 256, pro)
    pro.sync = None
    with pytest.raises(ValueError, match="sync"):
        _gemm(a8, sa, True, w8, wsc, L.EPI_BF16, out, None, 1, 128, 4, 256, 256, pro)
    pro = L.Prologue(kind=L.PRO_ADD_RMSNORM, x=ptr(x), norm_w=ptr(wsc), add=1, quant_mode=L.QUANT_ROWWISE,
                     sync=ptr(sync))
    with pytest.raises(ValueError, match="needs b or b32"):
        _gemm(a8, sa, True, w8, wsc, L.EPI_BF16, out, None, 1, 128, 4, 256, 256, pro)


@pytest.mark.parametrize("mode", ["rowwise", "static"])
def test_engine_fused_forward_is_bit_identical_to_unfused(mode):
    from fastforward_b200.config import MODELS, Layout
    from fastforward_b200.engine import Engine, PackedModel
    from tests._model import small_case
    dims, src, req, layout = small_case(MODELS["2B"], 3, Layout(0, 16, 16, 40, k=4), vocab=4096)
    dev = torch.device(DEV)
    pm = PackedModel(dims, src, mode=mode, device=dev)
    T = layout.bucket
    args = (req["ids"][:T].to(dev), req["visual"].to(dev), [x.to(dev) for x in req["deep"]], req["pick"], layout.k,
            layout.image_start, layout.grid_h, layout.grid_w)
    outs = []
    for fuse in ("none", "tail", "all"):
        # the same K splits in all three: token-major o / down plans (the weight-stationary
        # schedule has no fused-prologue form, so fuse="all" plans token-major GEMMs)
        eng = Engine(pm, fuse=fuse, autotune=False, stream_od=False)
        hs, z, lp = eng.trace(*args, T=T)
        outs.append((hs, z, lp))
        # the captured graph replays the same forward
        ent = eng.capture(T, layout.image_start, layout.nv, layout.grid_h, layout.grid_w, layout.k, len(req["deep"]))
        z2, lp2 = eng.replay(ent, args[0], args[1], args[2], args[3])
        assert_bytes_equal(z2, z, f"graph replay logits (fuse={fuse})")
    h0, z0, l0 = outs[0]
    for (h1, z1, l1), fuse in zip(outs[1:], ("tail", "all")):
        assert len(h0) == len(h1)
        for j, (a, b) in enumerate(zip(h0, h1)):
            assert_bytes_equal(b, a, f"residual entering layer {j} (fuse={fuse})")
        assert_bytes_equal(z1, z0, f"logits (fuse={fuse})")
        assert_bytes_equal(l1, l0, f"log-probs (fuse={fuse})")
    assert L.device_error() == 0


def _all_bf16_upto(a):
    """Every bf16 value v with |v| <= a (both signs, zero once), as a float32 tensor."""
    bits = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(BF16).float()
    pos = bits[bits <= a]
    return torch.cat([pos, -pos[1:]])


@pytest.mark.parametrize("rows_amax", [(3.71875, 0.0123, 448.0, 1.0), (97.5, 2.0 ** -10, 0.00549, 200.0)])
def test_rowwise_quant_exhaustive_bf16(rows_amax):
    """Each row holds every bf16 value up to its maximum, so the quotients x/s fall next to
    e4m3 rounding midpoints, on them (power-of-two scales) and in the e4m3 subnormal range:
    the prologue's reciprocal-with-check cast must give the IEEE-division bytes everywhere."""
    import oracle
    rows = [_all_bf16_upto(a) for a in rows_amax]
    K = max(r.numel() for r in rows)
    K = (K + 127) // 128 * 128
    assert K <= 36864
    x = torch.zeros((len(rows), K))
    for i, r in enumerate(rows):
        x[i, :r.numel()] = r
    x = x.to(BF16)
    M, N = x.shape[0], 128
    xd = x.to(DEV)
    w8 = torch.zeros((N, K), dtype=torch.uint8, device=DEV)
    wsc = torch.ones(N, dtype=torch.float32, device=DEV)
    sync = torch.zeros(2, dtype=torch.int32, device=DEV)
    a8 = torch.zeros((M, K), dtype=torch.uint8, device=DEV)
    sa = torch.zeros(M, dtype=torch.float32, device=DEV)
    out = torch.zeros((M, N), dtype=BF16, device=DEV)
    pro = L.Prologue(kind=L.PRO_QUANT, x=ptr(xd), quant_mode=L.QUANT_ROWWISE, sync=ptr(sync))
    _gemm(a8, sa, True, w8, wsc, L.EPI_BF16, out, None, 1, 128, M, N, K, pro)
    torch.cuda.synchronize()
    q, s = oracle.quantize_rows(x)
    assert_bytes_equal(sa, s[:M], "row scales")
    assert_bytes_equal(a8, q[:M].view(torch.uint8), "e4m3 bytes")
    assert L.device_error() == 0


@pytest.mark.parametrize("amax", [3.71875, 0.0123, 448.0, 1.0, 97.5, 2.0 ** -10, 0.00549, 200.0])
def test_quantizer_rowwise_exhaustive_bf16(amax):
    """ffb_quantize_fp8 (ROWWISE) over every bf16 value up to a row maximum: the vectorised
    kernel (K = 8192, each row = the maximum + a slice of the values) and the scalar one
    (one row of all of them) give the oracle's IEEE-division bytes."""
    import oracle
    vals = _all_bf16_upto(amax)
    K = 8192
    per = K - 1
    nrows = (vals.numel() + per - 1) // per
    x = torch.zeros((nrows, K))
    for i in range(nrows):
        part = vals[i * per:(i + 1) * per]
        x[i, 0] = amax
        x[i, 1:1 + part.numel()] = part
    K1 = (vals.numel() + 127) // 128 * 128
    x1 = torch.zeros((1, K1))
    x1[0, :vals.numel()] = vals
    for xx in (x, x1):
        xx = xx.to(BF16)
        M, Kx = xx.shape
        xd = xx.to(DEV)
        q8 = torch.zeros((M, Kx), dtype=torch.uint8, device=DEV)
        qs = torch.zeros(M, device=DEV)
        call("ffb_quantize_fp8", ptr(xd), L.QUANT_ROWWISE, 0.0, ptr(q8), ptr(qs), M, Kx, _s())
        torch.cuda.synchronize()
        q, s = oracle.quantize_rows(xx)
        assert_bytes_equal(qs, s[:M], f"row scales (K={Kx})")  # the oracle pads the rows
        assert_bytes_equal(q8, q[:M].view(torch.uint8), f"e4m3 bytes (K={Kx})")
    assert L.device_error() == 0

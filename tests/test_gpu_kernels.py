"""Per-kernel parity of libffb200 (called through its C ABI) against the CPU oracle.

Bars: FP8 quantisation and int4 packing bit-exact; norm / RoPE / readout kernels within
1 bf16 ulp on a small fraction of elements (the GPU's rsqrt/exp are hardware
approximations, the oracle's are correctly rounded); GEMM outputs within one bf16
rounding of the oracle's exact FP8 dot products; attention within bf16 tolerance.
"""
import math

import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200 import ops
from fastforward_b200._lib import call, ptr
from tests._util import assert_bf16_near, assert_bytes_equal

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
E4M3 = torch.float8_e4m3fn
DEV = "cuda"


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _randn(shape, seed, std=1.0):
    return (torch.randn(shape, generator=_g(seed)) * std).to(BF16)


def _sp():
    return torch.cuda.current_stream().cuda_stream


_ALIVE = []


def _keep(t):
    """Holds a device temporary until the test's kernels are done (a tensor created inline in
    an argument list would be freed, and its memory handed to the next argument, before the
    call runs)."""
    _ALIVE.append(t)
    return t


@pytest.fixture(autouse=True)
def _release_temporaries():
    yield
    torch.cuda.synchronize()
    _ALIVE.clear()


class Norm:
    def __init__(self, w, eps=1e-6):
        self.weight = w
        self.variance_epsilon = eps


# ---------------------------------------------------------------------------- norms

@pytest.mark.parametrize("T,H", [(1, 2048), (64, 2560), (333, 4096), (17, 5120)])
def test_rmsnorm(T, H):
    x = _randn((T, H), 1)
    w = (1 + 0.1 * torch.randn(H, generator=_g(2))).to(BF16)
    got = ops.fast_norm(x.to(DEV), Norm(w.to(DEV)))
    # order-independent statistics (exact fp64 sum of squares, IEEE sqrt/divide): bit-exact
    assert_bytes_equal(got, oracle.rms_one(x, w, 1e-6), "rmsnorm")


@pytest.mark.parametrize("T,H,start,nv", [(64, 2048, 8, 16), (320, 2560, 0, 256), (5, 5120, 0, 0)])
def test_add_rmsnorm_deep(T, H, start, nv):
    a, b = _randn((T, H), 3), _randn((T, H), 4)
    deep = _randn((nv, H), 5) if nv else None
    w = (1 + 0.1 * torch.randn(H, generator=_g(6))).to(BF16)
    r, y = ops.add_rms(a.to(DEV), b.to(DEV), deep.to(DEV) if deep is not None else None, Norm(w.to(DEV)),
                       start, nv)
    rr, yy = oracle.add_rms(a, b, deep, w, 1e-6, start, nv)
    assert_bytes_equal(r, rr, "residual")          # pure adds: bit-exact
    assert_bytes_equal(y, yy, "normed")


@pytest.mark.parametrize("S", [1, 2, 4, 5, 8])
def test_add_rmsnorm_partial_planes_in_plane_order(S):
    """The split-K planes are summed in plane order from 0 (fp32), then rounded to bf16 --
    bit-exact for every split count (the kernel loads up to 4 planes at once, more plane by
    plane)."""
    T, H = 24, 2560
    a = _randn((T, H), 17)
    parts = torch.randn((S, T, H), generator=_g(18)) * 0.5
    w = (1 + 0.1 * torch.randn(H, generator=_g(19))).to(BF16)
    res = torch.empty((T, H), device=DEV, dtype=BF16)
    out = torch.empty((T, H), device=DEV, dtype=BF16)
    a_d, p_d, w_d = a.to(DEV), parts.to(DEV), w.to(DEV)  # referenced until the kernel has run
    call("ffb_add_rmsnorm", ptr(a_d), None, ptr(p_d), S, None, 0, 0, ptr(w_d), 1e-6, ptr(res), ptr(out),
         L.QUANT_NONE, 0.0, None, None, T, H, _sp())
    torch.cuda.synchronize()
    acc = torch.zeros((T, H))
    for s in range(S):
        acc = acc + parts[s]
    rr, yy = oracle.add_rms(a, acc.to(BF16), None, w, 1e-6)
    assert_bytes_equal(res, rr, f"residual, {S} planes")
    assert_bytes_equal(out, yy, f"normed, {S} planes")


@pytest.mark.parametrize("mode", [L.QUANT_ROWWISE, L.QUANT_STATIC])
def test_add_rmsnorm_partials_and_fused_quant(mode):
    T, H, S = 40, 2560, 3
    a = _randn((T, H), 7)
    parts = torch.randn((S, T, H), generator=_g(8)) * 0.5
    w = torch.ones(H, dtype=BF16)
    a_d, p_d, w_d = a.to(DEV), parts.to(DEV), w.to(DEV)
    res = torch.empty((T, H), device=DEV, dtype=BF16)
    out = torch.empty((T, H), device=DEV, dtype=BF16)
    q8 = torch.empty((T, H), device=DEV, dtype=E4M3)
    qs = torch.empty(T, device=DEV, dtype=torch.float32)
    inv = 37.5
    call("ffb_add_rmsnorm", ptr(a_d), None, ptr(p_d), S, None, 0, 0, ptr(w_d), 1e-6, ptr(res), ptr(out), mode, inv,
         ptr(q8), ptr(qs), T, H, _sp())
    b = parts.sum(0).to(BF16)  # fixed-order fp32 sum, rounded like the linear's bf16 output
    rr, yy = oracle.add_rms(a, b, None, w, 1e-6)
    assert_bf16_near(res, rr, max_frac=0.002, what="residual from partials")
    # normalisation of the kernel's own residual is bit-exact
    assert_bytes_equal(out, oracle.rms_one(res.cpu(), w, 1e-6), "normed")
    # the fused quantiser must be bit-exact on the kernel's own bf16 output
    if mode == L.QUANT_ROWWISE:
        q_ref, s_ref = oracle.quantize_rows(out.cpu())
        assert_bytes_equal(q8, q_ref[:T], "fused rowwise q8")
        assert torch.equal(qs.cpu(), s_ref[:T])
    else:
        assert_bytes_equal(q8, oracle.quantize_static(out.cpu(), inv)[:T], "fused static q8")


# ---------------------------------------------------------------------------- FP8 quantisers

@pytest.mark.parametrize("M,K", [(1, 2048), (320, 2560), (77, 9728)])
def test_quantize_activation_bit_exact(M, K):
    x = _randn((M, K), 9, std=3.0)
    q, s = ops.quantize_activation(x.to(DEV), L.QUANT_ROWWISE)
    q_ref, s_ref = oracle.quantize_rows(x)
    assert_bytes_equal(q, q_ref, "rowwise q8")
    assert torch.equal(s.cpu(), s_ref)
    inv = 448.0 / 9.3
    q, _ = ops.quantize_activation(x.to(DEV), L.QUANT_STATIC, inv)
    assert_bytes_equal(q, oracle.quantize_static(x, inv), "static q8")


def test_rowwise_quant_every_bf16_value():
    """The rowwise quantiser's IEEE quotients: every finite bf16 value, quantised under row
    maxima of several magnitudes, gives the bytes of the oracle's correctly rounded divide."""
    allv = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(BF16).float()
    allv = allv[torch.isfinite(allv)]
    rows = []
    for mx in (1.0, 3.71875, 448.0, 1e-3, 12345.0, 0.0302734375):
        v = allv[allv.abs() <= mx]
        idx = torch.linspace(0, v.numel() - 1, 16384).round().long()  # spread over the whole range
        row = v[idx].clone()
        row[-1] = mx  # the row maximum
        rows.append(row)
    x = torch.stack(rows).to(BF16)
    M, K = x.shape
    q8 = torch.empty((M, K), device=DEV, dtype=E4M3)
    sc = torch.empty(M, device=DEV)
    call("ffb_quantize_fp8", ptr(_keep(x.to(DEV))), L.QUANT_ROWWISE, 0.0, ptr(q8), ptr(sc), M, K, _sp())
    want, want_s = oracle.quantize_rows(x)
    assert torch.equal(sc.cpu(), want_s[:M])
    assert_bytes_equal(q8, want[:M], "rowwise quant over every bf16 value")


@pytest.mark.parametrize("N,K", [(256, 2048), (6144, 2560), (128, 9728)])
def test_quantize_weight_bit_exact(N, K):
    w = _randn((N, K), 10, std=0.02)
    w8, s = ops.quantize_weight(w.to(DEV), per_channel=True)
    w8r, sr = oracle.quantize_weight_channel(w)
    assert_bytes_equal(w8, w8r, "per-channel W8")
    assert torch.equal(s.cpu(), sr)
    w8, s = ops.quantize_weight(w.to(DEV), per_channel=False)
    w8r, sr = oracle.quantize_weight_tensor(w)
    assert_bytes_equal(w8, w8r, "per-tensor W8")
    assert torch.equal(s.cpu(), sr)


# ---------------------------------------------------------------------------- GEMM

def _gemm_case(M, N, K, seed, splits=1):
    """Inputs and the oracle's fp32 result under its tensor-core accumulation model."""
    x = _randn((M, K), seed)
    w = _randn((N, K), seed + 1, std=0.02)
    q, sa = oracle.quantize_rows(x)
    w8, sw = oracle.quantize_weight_channel(w)
    ref32 = oracle.qwen_path._fp8_linear(q, sa, w8, sw, splits)[:M]
    return q, sa, w8, sw, ref32


@pytest.mark.parametrize("M,N,K,bn", [
    (320, 6144, 2560, 0), (320, 2560, 4096, 128), (1, 2560, 9728, 256), (16, 256, 256, 128),
    (100, 384, 1024, 0), (576, 1280, 2560, 256), (64, 128, 128, 0), (333, 512, 2048, 128),
    (1024, 256, 512, 256), (33, 256, 2048, 128), (200, 256, 768, 256), (90, 256, 640, 0)])
def test_fp8_gemm_bf16(M, N, K, bn):
    q, sa, w8, sw, ref32 = _gemm_case(M, N, K, 11)
    out = torch.empty((M, N), device=DEV, dtype=BF16)
    call("ffb_fp8_gemm", ptr(_keep(q.to(DEV))), ptr(_keep(sa.to(DEV))), 1, ptr(_keep(w8.to(DEV))), ptr(_keep(sw.to(DEV))), 1, L.EPI_BF16,
         ptr(out), None, 1, bn, M, N, K, _sp())
    torch.cuda.synchronize()
    # the oracle's tensor-core accumulation model (fp32 sum of exact K=32 partial dots) makes
    # the bf16 output bit-exact
    assert_bytes_equal(out, ref32.to(BF16), f"gemm {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K,splits", [(320, 2560, 9728, 4), (1, 2560, 4096, 7), (320, 6144, 2560, 3),
                                          (129, 1280, 1024, 8)])
def test_fp8_gemm_split_k(M, N, K, splits):
    q, sa, w8, sw, ref32 = _gemm_case(M, N, K, 12, splits)
    ws = torch.empty((splits, M, N), device=DEV, dtype=torch.float32)
    call("ffb_fp8_gemm", ptr(_keep(q.to(DEV))), ptr(_keep(sa.to(DEV))), 1, ptr(_keep(w8.to(DEV))), ptr(_keep(sw.to(DEV))), 1,
         L.EPI_F32_PARTIAL, None, ptr(ws), splits, 0, M, N, K, _sp())
    parts = ws.cpu()
    got = parts[0].clone()
    for s_ in range(1, splits):  # the consumers add the splits in order
        got = got + parts[s_]
    assert torch.equal(got, ref32), (got - ref32).abs().max()


def test_fp8_gemm_static_scales():
    M, N, K = 96, 768, 2048
    x = _randn((M, K), 13)
    w = _randn((N, K), 14, std=0.02)
    inv = 448.0 / x.float().abs().max().item()
    w8, ws_ = oracle.quantize_weight_tensor(w)
    want = oracle.fp8_linear_static(x, w8, ws_, inv)
    lin = ops.RuntimeScaleLinear.__new__(ops.RuntimeScaleLinear)
    lin.weight, lin.weight_scale = w8.to(DEV), ws_.to(DEV)
    lin.inverse_scale = inv
    lin.input_scale = torch.tensor([1.0 / inv], device=DEV)
    got = lin(x.to(DEV))
    assert_bytes_equal(got, want, "static fp8 linear")


@pytest.mark.parametrize("M,I", [(320, 512), (1, 768), (57, 512), (300, 9728)])
def test_fp8_gemm_swiglu_epilogue(M, I):
    K = 2560
    x = _randn((M, K), 15)
    w = _randn((2 * I, K), 16, std=0.02)
    q, sa = oracle.quantize_rows(x)
    w8, sw = oracle.quantize_weight_channel(w)
    gu = oracle.fp8_linear_rowwise(x, w8, sw)
    want = oracle.swiglu(gu[:, :I], gu[:, I:])
    w_d = w.to(DEV)
    packed = torch.empty_like(w_d)
    call("ffb_pack_gateup", ptr(w_d), ptr(packed), I, K, 2, _sp())
    w8p, swp = ops.quantize_weight(packed, per_channel=True)
    out = torch.empty((M, I), device=DEV, dtype=BF16)
    call("ffb_fp8_gemm", ptr(_keep(q.to(DEV))), ptr(_keep(sa.to(DEV))), 1, ptr(w8p), ptr(swp), 1, L.EPI_SWIGLU, ptr(out), None, 1,
         0, M, 2 * I, K, _sp())
    assert_bytes_equal(out, want, "swiglu epilogue")


@pytest.mark.parametrize("M,I,a_per_row", [(320, 9728, 0), (57, 512, 0), (1, 768, 0), (200, 1024, 1)])
def test_fp8_gemm_swiglu_fp8_is_swiglu_then_static_quant(M, I, a_per_row):
    """The fused SwiGLU + static FP8 output (`ffb_fp8_gemm_swiglu_fp8`) writes exactly the
    bytes of the SwiGLU epilogue followed by `ffb_quantize_fp8` (STATIC), with rows of the
    last token tile clipped; the oracle's static quantiser of the same SwiGLU output agrees."""
    K = 2560
    x = _randn((M, K), 25)
    w = _randn((2 * I, K), 26, std=0.02)
    if a_per_row:
        q, sa = oracle.quantize_rows(x)
    else:
        inv_in = 448.0 / 6.0
        q, sa = oracle.quantize_static(x, inv_in), torch.tensor([1.0 / inv_in])
    w_d = w.to(DEV)
    packed = torch.empty_like(w_d)
    call("ffb_pack_gateup", ptr(w_d), ptr(packed), I, K, 2, _sp())
    w8p, swp = ops.quantize_weight(packed, per_channel=True)
    q_d, sa_d = _keep(q.to(DEV)), _keep(sa.to(DEV))
    act = torch.empty((M, I), device=DEV, dtype=BF16)
    call("ffb_fp8_gemm", ptr(q_d), ptr(sa_d), a_per_row, ptr(w8p), ptr(swp), 1, L.EPI_SWIGLU, ptr(act), None, 1, 0, M,
         2 * I, K, _sp())
    inv = 448.0 / 0.35
    want8 = torch.empty((M, I), device=DEV, dtype=E4M3)
    call("ffb_quantize_fp8", ptr(act), L.QUANT_STATIC, inv, ptr(want8), None, M, I, _sp())
    got8 = torch.full((M + 1, I), 0x7F, device=DEV, dtype=torch.uint8)  # a guard row after the output
    call("ffb_fp8_gemm_swiglu_fp8", ptr(q_d), ptr(sa_d), a_per_row, ptr(w8p), ptr(swp), 1, inv, ptr(got8), M, 2 * I,
         K, _sp())
    torch.cuda.synchronize()
    assert_bytes_equal(got8[:M], want8, "fused swiglu + static quant")
    assert bool((got8[M] == 0x7F).all()), "wrote past the last row"
    assert_bytes_equal(got8[:M], oracle.quantize_static(act.cpu(), inv)[:M], "oracle static quantiser")
    with pytest.raises(ValueError):
        call("ffb_fp8_gemm_swiglu_fp8", ptr(q_d), ptr(sa_d), a_per_row, ptr(w8p), ptr(swp), 1, 0.0, ptr(got8), M,
             2 * I, K, _sp())


@pytest.mark.parametrize("T,HQ,HK,segments", [(320, 32, 8, None), (100, 16, 8, None), (512, 8, 2, (200, 130, 64))])
def test_attention_fp8_is_attention_then_static_quant(T, HQ, HK, segments):
    """`ffb_attention_fp8` writes exactly the bytes of the causal attention (segmented when
    several requests share the sequence) followed by `ffb_quantize_fp8` (STATIC)."""
    g = _g(41)
    q = torch.randn((HQ, T, 128), generator=g).to(BF16).to(DEV)
    k = torch.randn((HK, T, 128), generator=g).to(BF16).to(DEV)
    v = torch.randn((HK, T, 128), generator=g).to(BF16).to(DEV)
    lo = None
    if segments:
        rows = [-(-n // 64) * 64 for n in segments]
        assert sum(rows) == T
        offs = [sum(rows[:i]) for i in range(len(rows))]
        lo = torch.repeat_interleave(torch.tensor(offs, dtype=torch.int32), torch.tensor(rows)).to(DEV)
    out = torch.empty((T, HQ * 128), device=DEV, dtype=BF16)
    call("ffb_attention_segmented", ptr(q), ptr(k), ptr(v), None, 0, ptr(lo), ptr(out), T, T, HQ, HK, 128 ** -0.5,
         _sp())
    inv = 448.0 / 3.0
    want8 = torch.empty((T, HQ * 128), device=DEV, dtype=E4M3)
    call("ffb_quantize_fp8", ptr(out), L.QUANT_STATIC, inv, ptr(want8), None, T, HQ * 128, _sp())
    got8 = torch.full((T + 1, HQ * 128), 0x7F, device=DEV, dtype=torch.uint8)
    call("ffb_attention_fp8", ptr(q), ptr(k), ptr(v), ptr(lo), inv, ptr(got8), T, HQ, HK, 128 ** -0.5, _sp())
    torch.cuda.synchronize()
    assert_bytes_equal(got8[:T], want8, "fused attention + static quant")
    assert bool((got8[T] == 0x7F).all()), "wrote past the last row"
    assert L.device_error() == 0
    with pytest.raises(ValueError):
        call("ffb_attention_fp8", ptr(q), ptr(k), ptr(v), None, 0.0, ptr(got8), T, HQ, HK, 128 ** -0.5, _sp())


@pytest.mark.parametrize("T,HQ,HK", [(320, 32, 8), (100, 16, 8), (576, 16, 8), (1, 8, 2)])
def test_attention_rowwise_is_attention_then_rowwise_quant(T, HQ, HK):
    """`ffb_attention_rowwise` writes exactly the bytes (e4m3 rows and per-row scales) of the
    causal attention followed by `ffb_quantize_fp8` (ROWWISE): each row's maximum is combined
    over its HQ head CTAs in-kernel.  Three calls on one sync buffer (its counters carry the
    generation over), different inputs each time."""
    g = _g(43)
    sync = torch.zeros((L.lib().ffb_attention_rowwise_sync_bytes(T, HQ) + 15) // 16 * 2, device=DEV,
                       dtype=torch.int64)
    for rep in range(3):
        q = (torch.randn((HQ, T, 128), generator=g) * (1 + rep)).to(BF16).to(DEV)
        k = torch.randn((HK, T, 128), generator=g).to(BF16).to(DEV)
        v = (torch.randn((HK, T, 128), generator=g) * (3 - rep)).to(BF16).to(DEV)
        out = torch.empty((T, HQ * 128), device=DEV, dtype=BF16)
        call("ffb_attention", ptr(q), ptr(k), ptr(v), None, 0, ptr(out), T, T, HQ, HK, 128 ** -0.5, _sp())
        want8 = torch.empty((T, HQ * 128), device=DEV, dtype=E4M3)
        want_s = torch.empty(T, device=DEV, dtype=torch.float32)
        call("ffb_quantize_fp8", ptr(out), L.QUANT_ROWWISE, 0.0, ptr(want8), ptr(want_s), T, HQ * 128, _sp())
        got8 = torch.full((T + 1, HQ * 128), 0x7F, device=DEV, dtype=torch.uint8)
        got_s = torch.full((T + 1,), -1.0, device=DEV, dtype=torch.float32)
        call("ffb_attention_rowwise", ptr(q), ptr(k), ptr(v), ptr(got8), ptr(got_s), ptr(sync), T, HQ, HK,
             128 ** -0.5, _sp())
        torch.cuda.synchronize()
        assert_bytes_equal(got8[:T], want8, "fused attention + rowwise quant")
        assert torch.equal(got_s[:T], want_s), "row scales"
        assert bool((got8[T] == 0x7F).all()) and got_s[T].item() == -1.0, "wrote past the last row"
        assert L.device_error() == 0


def test_attention_rowwise_refuses_grids_larger_than_the_sms():
    """The row maxima meet across the CTAs of a query tile, so the whole grid must be resident:
    more CTAs than SMs is refused before any launch."""
    T, HQ = 2048, 32
    sync = torch.zeros(T * HQ, device=DEV, dtype=torch.int64)
    x = torch.zeros((HQ, T, 128), device=DEV, dtype=BF16)
    with pytest.raises(L.FFBUnsupported, match="resident"):
        call("ffb_attention_rowwise", ptr(x), ptr(x), ptr(x), ptr(x), ptr(sync), ptr(sync), T, HQ, 8, 0.1, _sp())


def test_swiglu_epilogue_every_bf16_gate():
    """The SwiGLU epilogues look the activation bf16(g / (1 + exp(-g))) up by the bf16 gate's
    bits; the table must equal the formula evaluated on the device (the standalone swiglu
    kernel: expf + IEEE divide) for every finite bf16 gate.  Each GEMM column computes
    acc = 1 (one-hot rows) times a per-channel scale equal to the gate value under test."""
    n = 65536
    g = torch.arange(n, dtype=torch.int32).to(torch.int16).view(BF16)  # every bf16 bit pattern
    gf = g.float()
    M, K = 16, 128
    a8 = torch.zeros((M, K), dtype=torch.float32)
    a8[:, 0] = 1.0
    a8 = a8.to(torch.float8_e4m3fn).to(DEV)
    sa = torch.ones(M, device=DEV)
    w8 = torch.zeros((2 * n, K), dtype=torch.float32)
    w8[:, 0] = 1.0
    w8 = w8.to(torch.float8_e4m3fn).to(DEV)
    sw = torch.ones((n // 128, 2, 128), dtype=torch.float32)  # tile t: gate channels, then up
    sw[:, 0, :] = gf.view(n // 128, 128)
    sw = sw.reshape(-1).to(DEV)
    out = torch.empty((M, n), device=DEV, dtype=BF16)
    call("ffb_fp8_gemm", ptr(a8), ptr(sa), 1, ptr(w8), ptr(sw), 1, L.EPI_SWIGLU, ptr(out), None, 1, 0, M, 2 * n, K, _sp())
    direct = ops.swiglu(g.view(1, n).to(DEV), torch.ones((1, n), device=DEV, dtype=BF16))
    torch.cuda.synchronize()
    fin = torch.isfinite(gf)
    got = out[0].cpu().view(torch.int16)[fin]
    assert torch.equal(got, out[M - 1].cpu().view(torch.int16)[fin])
    assert torch.equal(got, direct[0].cpu().view(torch.int16)[fin]), "table != device formula"
    ref = oracle.swiglu(g.view(1, n), torch.ones((1, n), dtype=BF16))[0].view(torch.int16)[fin]
    print(f"\nlooked-up SiLU vs the oracle (CPU exp): {(got != ref).sum().item()} of {int(fin.sum())} bf16 gates differ")


@pytest.mark.parametrize("T,HQ,HK,K", [(320, 32, 8, 2560), (77, 16, 8, 2048), (1, 8, 8, 512)])
def test_fp8_gemm_qk_rope_fused(T, HQ, HK, K):
    """qkv projection with the per-head norm + RoPE in its epilogue, against the oracle's
    FP8 linear (tensor-core accumulation model) rounded to bf16 followed by `qk_pair`:
    bit-exact."""
    from fastforward_b200.mrope import position_ids, cos_sin
    x = _randn((T, K), 70)
    w = _randn(((HQ + 2 * HK) * 128, K), 71, std=0.02)
    q8, sa = oracle.quantize_rows(x)
    w8, sw = oracle.quantize_weight_channel(w)
    pos = position_ids(max(T, 64), 0, 8, 8)[:, :T] if T < 64 else position_ids(T, 0, 16, 16)
    cos, sin = cos_sin(pos)
    qn = (1 + 0.1 * torch.randn(128, generator=_g(72))).to(BF16)
    kn = (1 + 0.1 * torch.randn(128, generator=_g(73))).to(BF16)
    yq = torch.empty((HQ, T, 128), device=DEV, dtype=BF16)
    yk = torch.empty((HK, T, 128), device=DEV, dtype=BF16)
    yv = torch.empty((HK, T, 128), device=DEV, dtype=BF16)
    call("ffb_fp8_gemm_qk_rope", ptr(_keep(q8.to(DEV))), ptr(_keep(sa.to(DEV))), 1, ptr(_keep(w8.to(DEV))),
         ptr(_keep(sw.to(DEV))), 1, ptr(_keep(qn.to(DEV))), ptr(_keep(kn.to(DEV))), 1e-6,
         ptr(_keep(cos.contiguous().to(DEV))), ptr(_keep(sin.contiguous().to(DEV))), ptr(yq), ptr(yk), ptr(yv),
         T, HQ, HK, K, _sp())
    torch.cuda.synchronize()
    qkv = oracle.fp8_linear_rowwise(x, w8, sw)
    rq, rk = oracle.qk_pair(qkv[:, :HQ * 128].reshape(T, HQ, 128), qkv[:, HQ * 128:(HQ + HK) * 128].reshape(T, HK, 128),
                            qn, kn, cos, sin)
    assert_bytes_equal(yq, rq, "Q")
    assert_bytes_equal(yk, rk, "K")
    assert_bytes_equal(yv, qkv[:, (HQ + HK) * 128:].reshape(T, HK, 128).transpose(0, 1), "V")


# ---------------------------------------------------------------------------- QK norm + RoPE, attention

def _rope_inputs(T, HQ, HK, seed):
    from fastforward_b200.mrope import position_ids, cos_sin
    qkv = _randn((T, (HQ + 2 * HK) * 128), seed)
    grid = 16 if T >= 64 else 4
    pos = position_ids(T, 0, grid, grid)
    cos, sin = cos_sin(pos)
    qn = (1 + 0.1 * torch.randn(128, generator=_g(seed + 1))).to(BF16)
    kn = (1 + 0.1 * torch.randn(128, generator=_g(seed + 2))).to(BF16)
    return qkv, cos, sin, qn, kn


@pytest.mark.parametrize("T,HQ,HK", [(320, 32, 8), (7, 16, 8), (1024, 64, 8)])
def test_qk_norm_rope(T, HQ, HK):
    qkv, cos, sin, qn, kn = _rope_inputs(T, HQ, HK, 20)
    yq = torch.empty((HQ, T, 128), device=DEV, dtype=BF16)
    yk = torch.empty((HK, T, 128), device=DEV, dtype=BF16)
    yv = torch.empty((HK, T, 128), device=DEV, dtype=BF16)
    call("ffb_qk_norm_rope", ptr(_keep(qkv.to(DEV))), None, 0, qkv.shape[1], ptr(_keep(qn.to(DEV))), ptr(_keep(kn.to(DEV))), 1e-6,
         ptr(_keep(cos.to(DEV))), ptr(_keep(sin.to(DEV))), ptr(yq), ptr(yk), ptr(yv), T, HQ, HK, _sp())
    q = qkv[:, :HQ * 128].reshape(T, HQ, 128)
    k = qkv[:, HQ * 128:(HQ + HK) * 128].reshape(T, HK, 128)
    rq, rk = oracle.qk_pair(q, k, qn, kn, cos, sin)
    assert_bytes_equal(yq, rq, "Q")
    assert_bytes_equal(yk, rk, "K")
    assert_bytes_equal(yv, qkv[:, (HQ + HK) * 128:].reshape(T, HK, 128).transpose(0, 1), "V copy")


def test_qk_pair_mirror_signature():
    T, HQ, HK = 64, 16, 8
    qkv, cos, sin, qn, kn = _rope_inputs(T, HQ, HK, 21)
    x = qkv.to(DEV)[None]
    q = x[..., :HQ * 128].view(1, T, HQ, 128)
    k = x[..., HQ * 128:(HQ + HK) * 128].view(1, T, HK, 128)
    yq, yk = ops.qk_pair(q, k, Norm(qn.to(DEV)), Norm(kn.to(DEV)), cos.to(DEV)[None], sin.to(DEV)[None], 4, 4, False)
    rq, rk = oracle.qk_pair(qkv[:, :HQ * 128].reshape(T, HQ, 128), qkv[:, HQ * 128:(HQ + HK) * 128].reshape(T, HK, 128),
                            qn, kn, cos, sin)
    assert yq.shape == (1, HQ, T, 128) and yk.shape == (1, HK, T, 128)
    assert_bytes_equal(yq[0], rq, "Q")
    assert_bytes_equal(yk[0], rk, "K")


@pytest.mark.parametrize("T,HQ,HK", [(320, 32, 8), (100, 16, 8), (1024, 64, 8), (13, 8, 8), (576, 32, 8)])
def test_attention_causal(T, HQ, HK):
    """Bit-exact against the oracle's restatement of the kernel's arithmetic
    (`oracle.attention_tc`), and within rounding of the reference restatement
    (`oracle.attention_direct`, exact products)."""
    q, k, v = _randn((HQ, T, 128), 30), _randn((HK, T, 128), 31), _randn((HK, T, 128), 32)
    got = ops.attention_direct(q.to(DEV)[None], k.to(DEV)[None], v.to(DEV)[None], 128 ** -0.5)
    assert_bytes_equal(got[0], oracle.attention_tc(q, k, v, 128 ** -0.5), f"attention T={T}")
    want = oracle.attention_direct(q, k, v, 128 ** -0.5)
    torch.testing.assert_close(got[0].cpu().float(), want.float(), atol=2e-2, rtol=2e-2)
    from tests._util import bf16_ulp_diff
    d = bf16_ulp_diff(got[0].cpu(), want)
    print(f"\nattention T={T}: {(d == 0).float().mean().item():.2%} equal to the exact-product restatement, "
          f"max {d.max().item()} ulp")


@pytest.mark.parametrize("T,pick", [(320, 319), (320, 200), (77, 0), (1024, 700)])
def test_attention_selected_gather(T, pick):
    """The tail's selected query row (gathered from the full projection) is bit-identical to
    the same row of the causal prefill and to the oracle."""
    HQ, HK = 32, 8
    q, k, v = _randn((HQ, T, 128), 33), _randn((HK, T, 128), 34), _randn((HK, T, 128), 35)
    pos = torch.tensor([pick], dtype=torch.long)
    out = torch.empty((1, HQ * 128), device=DEV, dtype=BF16)
    call("ffb_attention", ptr(_keep(q.to(DEV))), ptr(_keep(k.to(DEV))), ptr(_keep(v.to(DEV))), ptr(_keep(pos.to(DEV))), 1, ptr(out), 1, T, HQ, HK,
         128 ** -0.5, _sp())
    want = oracle.attention_tc(q[:, pick:pick + 1], k, v, 128 ** -0.5, positions=pos)
    assert_bytes_equal(out.reshape(1, HQ, 128), want, "selected row")
    full = ops.attention_direct(q.to(DEV)[None], k.to(DEV)[None], v.to(DEV)[None], 128 ** -0.5)
    assert_bytes_equal(out.reshape(HQ, 128), full[0, pick], "selected row == causal row")


def test_attention_selected_rows_ungathered():
    """Selected rows whose Q is already gathered ([HQ, S, 128], q_gather = 0), several rows."""
    HQ, HK, T = 16, 8, 300
    q, k, v = _randn((HQ, T, 128), 36), _randn((HK, T, 128), 37), _randn((HK, T, 128), 38)
    sel = torch.tensor([299, 5, 130, 64], dtype=torch.long)
    got = ops.attention_direct(q[:, sel].contiguous().to(DEV)[None], k.to(DEV)[None], v.to(DEV)[None], 128 ** -0.5,
                               positions=sel.to(DEV))
    want = oracle.attention_tc(q[:, sel], k, v, 128 ** -0.5, positions=sel)
    assert_bytes_equal(got[0], want, "selected rows")


# ---------------------------------------------------------------------------- misc

def test_swiglu_standalone():
    M, I = 64, 1536
    gu = _randn((M, 2 * I), 40, std=2.0)
    g, u = gu.to(DEV).chunk(2, -1)
    got = ops.swiglu(g, u)
    assert_bf16_near(got, oracle.swiglu(gu[:, :I], gu[:, I:]), what="swiglu")


@pytest.mark.parametrize("H,k", [(2560, 4), (5120, 8), (2048, 2)])
def test_readout_logsoftmax(H, k):
    res, mlp = _randn((H,), 41), _randn((H,), 42)
    w = (1 + 0.1 * torch.randn(H, generator=_g(43))).to(BF16)
    head = _randn((8, H), 44, std=0.02)
    z = torch.empty(8, device=DEV)
    lp = torch.empty(8, device=DEV)
    call("ffb_readout", ptr(_keep(res.to(DEV))), ptr(_keep(mlp.to(DEV))), None, 0, ptr(_keep(w.to(DEV))), 1e-6, ptr(_keep(head.to(DEV))), 8, k,
         ptr(z), ptr(lp), H, _sp())
    chosen = (res.float() + mlp.float()).to(BF16)
    zr = oracle.lm_readout(chosen, w, head, 1e-6)
    assert torch.equal(z.cpu(), zr), (z.cpu(), zr)
    torch.testing.assert_close(lp[:k].cpu(), oracle.log_softmax(z[:k].cpu()), atol=1e-5, rtol=1e-5)


def test_embed_gather_exact():
    V, H, T = 1000, 2048, 96
    table = _randn((V, H), 50, std=0.02)
    ids = torch.randint(0, V, (T,), generator=_g(51))
    vis = _randn((36, H), 52)
    h = torch.empty((T, H), device=DEV, dtype=BF16)
    call("ffb_embed_gather", ptr(_keep(ids.to(DEV))), ptr(_keep(table.to(DEV))), V, ptr(_keep(vis.to(DEV))), 10, 36, ptr(h), T, H, _sp())
    assert_bytes_equal(h, oracle.embed_rows(table, ids, vis, 10), "embed")


@pytest.mark.parametrize("N,K", [(256, 2560), (128, 9728)])
def test_pack_int4_bit_exact(N, K):
    w = _randn((N, K), 60, std=0.02)
    packed, scales = ops.pack_int4(w.to(DEV))
    q, s = oracle.int4_sym_quantize(w)
    assert_bytes_equal(scales, s, "int4 scales")
    assert_bytes_equal(packed, oracle.int4_sym_pack(q), "int4 nibbles")


def test_device_error_word_clear():
    assert L.device_error(clear=True) == 0

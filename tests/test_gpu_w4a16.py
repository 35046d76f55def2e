"""W4A16 GEMM (int4 symmetric group-128 weights dequantised to bf16 in shared memory,
tcgen05 kind::f16) against the oracle: the packed weights are bit-exact, and the product
matches the exact (float64) sum of x * bf16(q * s) to within one bf16 rounding, the
tensor core's fp32 accumulation moving a result across a bf16 rounding boundary on a small
share of outputs."""
import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200 import ops
from fastforward_b200._lib import call, ptr
from tests._util import assert_bf16_near

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
BF16 = torch.bfloat16


def _randn(shape, seed, std=1.0):
    return (torch.randn(shape, generator=torch.Generator().manual_seed(seed)) * std).to(BF16)


def _packed(w):
    packed, scales = ops.pack_int4(w.to(DEV))
    q, s = oracle.int4_sym_quantize(w)
    assert torch.equal(scales.cpu().view(torch.int16), s.view(torch.int16))
    return packed, scales, oracle.int4_sym_dequantize(q, s)


def _exact(x, deq):
    return torch.matmul(x.double(), deq.double().t()).float()


def _sp():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("M,N,K,bn", [(320, 6144, 2560, 256), (576, 2560, 4096, 128), (1, 2560, 9728, 256),
                                      (100, 384, 1024, 128), (77, 256, 512, 0), (130, 1280, 2560, 0)])
def test_w4a16_bf16(M, N, K, bn):
    x, w = _randn((M, K), 21), _randn((N, K), 22, std=0.02)
    packed, scales, deq = _packed(w)
    xd = x.to(DEV)
    out = torch.empty((M, N), device=DEV, dtype=BF16)
    call("ffb_w4a16_gemm", ptr(xd), ptr(packed), ptr(scales), L.EPI_BF16, ptr(out), None, 1, bn, M, N, K, _sp())
    torch.cuda.synchronize()
    # outputs are O(1); the fp32 accumulation differs from the exact sum by ~1e-5, which
    # is many ulps only for results that cancel to near zero
    assert_bf16_near(out, _exact(x, deq).to(BF16), max_ulp=1, max_frac=0.01, what="w4a16", atol=1e-4)
    assert L.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(320, 6144, 2560), (77, 256, 512), (1, 2560, 4096)])
def test_w4a16_bf16_bit_exact_vs_tensor_core_model(M, N, K):
    """The oracle's model of the kind::f16 accumulation (oracle/tcgemm.c) makes the bf16
    output bit-exact."""
    x, w = _randn((M, K), 29), _randn((N, K), 30, std=0.02)
    packed, scales, deq = _packed(w)
    xd = x.to(DEV)
    out = torch.empty((M, N), device=DEV, dtype=BF16)
    call("ffb_w4a16_gemm", ptr(xd), ptr(packed), ptr(scales), L.EPI_BF16, ptr(out), None, 1, 0, M, N, K, _sp())
    torch.cuda.synchronize()
    want = oracle.qwen_path._bf16_linear(x, deq, 1).to(BF16)
    assert torch.equal(out.cpu().view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("M,N,K,splits", [(320, 2560, 9728, 4), (576, 2560, 4096, 3), (1, 2560, 9728, 7)])
def test_w4a16_split_k(M, N, K, splits):
    x, w = _randn((M, K), 23), _randn((N, K), 24, std=0.02)
    packed, scales, deq = _packed(w)
    xd = x.to(DEV)
    ws = torch.empty((splits, M, N), device=DEV, dtype=torch.float32)
    call("ffb_w4a16_gemm", ptr(xd), ptr(packed), ptr(scales), L.EPI_F32_PARTIAL, None, ptr(ws), splits, 0, M, N, K,
         _sp())
    torch.cuda.synchronize()
    nkb = K // 64
    for s in range(splits):  # each split holds the sum over its 64-wide K blocks
        k0, k1 = s * nkb // splits * 64, (s + 1) * nkb // splits * 64
        want = torch.matmul(x[:, k0:k1].double(), deq[:, k0:k1].double().t())
        torch.testing.assert_close(ws[s].cpu().double(), want, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("M,I", [(320, 512), (576, 9728), (1, 768)])
def test_w4a16_swiglu_epilogue(M, I):
    K = 2560
    x, w = _randn((M, K), 25), _randn((2 * I, K), 26, std=0.02)
    wd = w.to(DEV)
    wp = torch.empty_like(wd)
    call("ffb_pack_gateup", ptr(wd), ptr(wp), I, K, 2, _sp())
    packed, scales, deq = _packed(wp.cpu())
    xd = x.to(DEV)
    out = torch.empty((M, I), device=DEV, dtype=BF16)
    call("ffb_w4a16_gemm", ptr(xd), ptr(packed), ptr(scales), L.EPI_SWIGLU, ptr(out), None, 1, 0, M, 2 * I, K, _sp())
    # the same product through the plain bf16 epilogue: the SwiGLU epilogue must equal the
    # reference's swiglu applied to those gate / up values, bit for bit
    z = torch.empty((M, 2 * I), device=DEV, dtype=BF16)
    call("ffb_w4a16_gemm", ptr(xd), ptr(packed), ptr(scales), L.EPI_BF16, ptr(z), None, 1, 256, M, 2 * I, K, _sp())
    torch.cuda.synchronize()
    z = z.cpu().reshape(M, I // 128, 2, 128)  # undo the 128-channel gate/up interleave
    gate, up = z[:, :, 0, :].reshape(M, I), z[:, :, 1, :].reshape(M, I)
    assert torch.equal(out.cpu().view(torch.int16), oracle.swiglu(gate, up).view(torch.int16))
    # and against the exact product: a gate/up flip of one bf16 ulp moves a few outputs
    ze = _exact(x, deq).reshape(M, I // 128, 2, 128)
    want = oracle.swiglu(ze[:, :, 0, :].reshape(M, I).to(BF16), ze[:, :, 1, :].reshape(M, I).to(BF16))
    assert_bf16_near(out, want, max_ulp=2, max_frac=0.02, what="w4a16 swiglu vs exact", atol=0.1)


def test_int4_mirror_matches_entry_point():
    x, w = _randn((40, 1024), 27), _randn((384, 1024), 28, std=0.02)
    lin = ops.Int4(w.to(DEV))
    got = lin(x.to(DEV).reshape(1, 40, 1024))
    assert got.shape == (1, 40, 384)
    _, _, deq = _packed(w)
    assert_bf16_near(got.reshape(40, 384), _exact(x, deq).to(BF16), max_ulp=1, max_frac=0.01, what="Int4",
                     atol=1e-4)


def test_w4a16_rejects_bad_group_size():
    with pytest.raises(ValueError, match="group size 128"):
        call("ffb_w4a16_gemm", 16, 16, 16, L.EPI_BF16, 16, None, 1, 0, 16, 128, 96, None)


def test_engine_int4_tail_matches_oracle():
    """Depth-2 model in W4A16 mode (layer 0 full, layer 1 the pick-row tail)."""
    from fastforward_b200.config import MODELS
    from fastforward_b200.engine import Engine, PackedModel
    from fastforward_b200.mrope import position_ids
    from tests._model import small_case
    dims, src, req, layout = small_case(MODELS["4B"], 2, vocab=4096)
    eng = Engine(PackedModel(dims, src, mode="int4", device=DEV))
    T = layout.bucket
    z, _ = eng.forward(req["ids"][:T].to(DEV), req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]],
                       req["pick"], req["k"], layout.image_start, layout.grid_h, layout.grid_w, T=T)
    om = oracle.quantized_model(dims, src, "int4", splits={k: p.splits for k, p in eng.plans[T].items()})
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    def score():
        return oracle.prefill_score(om, req["ids"][:T], req["visual"], req["deep"], pos, req["pick"], req["k"],
                                    mode="int4", image_start=layout.image_start)[0]
    zr = score()
    old = oracle.set_attention_block(32)  # the oracle's own attention-rounding noise floor
    try:
        floor = (score() - zr).abs().max().item()
    finally:
        oracle.set_attention_block(old)
    err = (z.cpu() - zr).abs().max().item()
    assert err <= max(2e-2, floor), (z, zr, floor)
    assert oracle.response_argmax(z.cpu()) == oracle.response_argmax(zr)

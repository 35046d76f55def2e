"""The weight-stationary FP8 GEMM schedule (weights on the MMA's M side, one weight tile,
token range and K range per CTA; `csrc/gemm_fp8_stream.cu`): every epilogue writes exactly
the bytes of the token-major kernel and of the oracle's tensor-core accumulation model,
for token counts that are and are not multiples of 16, K that ends inside a 128-byte
block, K splits, and both scale schemes."""
import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200 import ops
from fastforward_b200._lib import call, ptr
from tests._util import assert_bytes_equal

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
E4M3 = torch.float8_e4m3fn
DEV = "cuda"
STREAM = 1  # FFB_TILE_STREAM


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _randn(shape, seed, std=1.0):
    return (torch.randn(shape, generator=_g(seed)) * std).to(BF16)


def _s():
    return torch.cuda.current_stream().cuda_stream


def _operands(M, N, K, seed, rowwise=True):
    x = _randn((M, K), seed)
    w = _randn((N, K), seed + 1, std=0.02)
    if rowwise:
        q, sa = oracle.quantize_rows(x)
        w8, sw = oracle.quantize_weight_channel(w)
    else:
        inv = 448.0 / 6.0
        q, sa = oracle.quantize_static(x, inv), torch.tensor([1.0 / inv])
        w8, sw = oracle.quantize_weight_tensor(w)
    return x, w, q[:M].contiguous(), sa[:M].contiguous() if sa.numel() > 1 else sa, w8, sw


@pytest.mark.parametrize("M,N,K,rowwise", [
    (320, 6144, 2560, True), (320, 2560, 4096, True), (1, 2560, 9728, True), (13, 384, 1040, True),
    (235, 1280, 2048, False), (384, 512, 640, True), (57, 128, 256, True), (300, 4096, 2560, False)])
def test_stream_bf16_equals_token_major_and_oracle(M, N, K, rowwise):
    _, _, q, sa, w8, sw = _operands(M, N, K, 100 + M, rowwise)
    qd, sad, w8d, swd = q.to(DEV), sa.to(DEV), w8.to(DEV), sw.to(DEV)
    outs = {}
    for tile in (STREAM, 128):
        out = torch.full((M + 1, N), -7.0, device=DEV, dtype=BF16)  # a guard row after the output
        call("ffb_fp8_gemm", ptr(qd), ptr(sad), int(rowwise), ptr(w8d), ptr(swd), int(rowwise), L.EPI_BF16, ptr(out),
             None, 1, tile, M, N, K, _s())
        outs[tile] = out
    torch.cuda.synchronize()
    assert_bytes_equal(outs[STREAM][:M], outs[128][:M], f"stream vs token-major {M}x{N}x{K}")
    assert bool((outs[STREAM][M] == -7.0).all()), "wrote past the last row"
    ref = oracle.qwen_path._fp8_linear(q, sa, w8, sw, 1)[:M].to(BF16)
    assert_bytes_equal(outs[STREAM][:M], ref, "stream vs oracle")


@pytest.mark.parametrize("M,I,rowwise", [(320, 4096, True), (235, 6144, True), (1, 768, True), (300, 512, False),
                                         (64, 12288, True)])
def test_stream_swiglu_equals_token_major(M, I, rowwise):
    K = 2560
    x, w, q, sa, _, _ = _operands(M, 2 * I, K, 200 + M, rowwise)
    w_d = w.to(DEV)
    packed = torch.empty_like(w_d)
    call("ffb_pack_gateup", ptr(w_d), ptr(packed), I, K, 2, _s())
    w8p, swp = ops.quantize_weight(packed, per_channel=rowwise)
    qd, sad = q.to(DEV), sa.to(DEV)
    outs = {}
    for tile in (STREAM, 256):
        out = torch.empty((M, I), device=DEV, dtype=BF16)
        call("ffb_fp8_gemm", ptr(qd), ptr(sad), int(rowwise), ptr(w8p), ptr(swp), int(rowwise), L.EPI_SWIGLU, ptr(out),
             None, 1, tile, M, 2 * I, K, _s())
        outs[tile] = out
    torch.cuda.synchronize()
    assert_bytes_equal(outs[STREAM], outs[256], f"swiglu stream vs token-major M={M} I={I}")


@pytest.mark.parametrize("M,N,K,splits", [(320, 2560, 9728, 3), (320, 2560, 4096, 3), (1, 2560, 4096, 7),
                                          (129, 1280, 1024, 4), (320, 6144, 2560, 1)])
def test_stream_split_k_partials_equal_token_major(M, N, K, splits):
    """fp32 K-split partial planes: the same K ranges as the token-major split, so every
    plane is byte-identical; their in-order sum is the oracle's split model."""
    _, _, q, sa, w8, sw = _operands(M, N, K, 300 + M)
    qd, sad, w8d, swd = q.to(DEV), sa.to(DEV), w8.to(DEV), sw.to(DEV)
    planes = {}
    for tile in (STREAM, 128):
        ws = torch.full((splits + 1, M, N), -7.0, device=DEV)  # a guard plane after the output
        call("ffb_fp8_gemm", ptr(qd), ptr(sad), 1, ptr(w8d), ptr(swd), 1, L.EPI_F32_PARTIAL, None, ptr(ws), splits,
             tile, M, N, K, _s())
        planes[tile] = ws
    torch.cuda.synchronize()
    assert_bytes_equal(planes[STREAM][:splits], planes[128][:splits], f"partials {M}x{N}x{K}/{splits}")
    assert bool((planes[STREAM][splits] == -7.0).all()), "wrote past the last plane"
    got = planes[STREAM][0].cpu().clone()
    for s_ in range(1, splits):
        got = got + planes[STREAM][s_].cpu()
    assert torch.equal(got, oracle.qwen_path._fp8_linear(q, sa, w8, sw, splits)[:M])


def test_stream_plan_query_and_rejections():
    M, N, K = 320, 2560, 9728
    assert L.stream_ctas(M, N, K, L.EPI_F32_PARTIAL, 3) > 0
    assert L.stream_ctas(M, N, K, L.EPI_BF16, 3) == 0            # a K split needs fp32 partials
    assert L.stream_ctas(M, N, K, L.EPI_F32_PARTIAL, 8) == 0     # 20 tiles x 8 splits > SMs
    assert L.stream_ctas(320, 19456, 2560, L.EPI_SWIGLU, 1) == 0  # 76 pair tiles: 320 tokens in one CTA
    q = torch.zeros((M, K), device=DEV, dtype=torch.uint8)
    w = torch.zeros((N, K), device=DEV, dtype=torch.uint8)
    sa = torch.ones(M, device=DEV)
    sw = torch.ones(N, device=DEV)
    ws = torch.empty((8, M, N), device=DEV)
    with pytest.raises(ValueError, match="weight-stationary"):
        call("ffb_fp8_gemm", ptr(q), ptr(sa), 1, ptr(w), ptr(sw), 1, L.EPI_F32_PARTIAL, None, ptr(ws), 8, STREAM, M, N,
             K, _s())
    assert L.device_error() == 0

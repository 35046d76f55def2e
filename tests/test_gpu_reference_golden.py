"""The CUDA kernels, called through the reference-signature mirrors in
`fastforward_b200.ops`, on the inputs stored with the reference's own outputs in
tests/golden/reference_ops.pt (made by tests/golden/make_golden.py): bit-exact wherever
the arithmetic is order-independent; attention within its rounding noise."""
import types
from pathlib import Path

import pytest
import torch

from fastforward_b200 import _lib as L
from fastforward_b200 import ops
from tests._util import bf16_ulp_diff

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_ops.pt"


@pytest.fixture(scope="module")
def ref():
    return torch.load(GOLDEN, weights_only=False)


def _norm(w, eps):
    return types.SimpleNamespace(weight=w.to(DEV), variance_epsilon=eps)


def _eq(got, want, what):
    got = got.cpu()
    if got.dtype == torch.bfloat16:
        got, want = got.view(torch.int16), want.view(torch.int16)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    n = int((got != want).sum())
    assert n == 0, f"{what}: {n} of {got.numel()} elements differ from the reference"


@pytest.mark.parametrize("h", [2048, 2560])
def test_add_rms(ref, h):
    c = ref[f"add_rms_{h}"]
    r, y = ops.add_rms(c["a"].to(DEV), c["b"].to(DEV), c["deep"].to(DEV), _norm(c["w"], c["eps"]), c["start"],
                       c["nv"])
    _eq(r, c["residual"], "residual")
    _eq(y, c["out"], "normed")


def test_fast_norm(ref):
    c = ref["fast_norm"]
    _eq(ops.fast_norm(c["x"].to(DEV), _norm(c["w"], c["eps"])), c["out"], "rms_one")


def test_qk_pair(ref):
    c = ref["qk_pair"]
    qkv = c["qkv"].to(DEV)
    t, hq, hk = qkv.shape[1], c["HQ"], c["HK"]
    q = qkv[..., :hq * 128].view(1, t, hq, 128)
    k = qkv[..., hq * 128:(hq + hk) * 128].view(1, t, hk, 128)
    yq, yk = ops.qk_pair(q, k, _norm(c["q_norm"], c["eps"]), _norm(c["k_norm"], c["eps"]), c["cos"].to(DEV),
                         c["sin"].to(DEV))
    _eq(yq, c["yq"], "yq")
    _eq(yk, c["yk"], "yk")


def test_attention(ref):
    c = ref["attention"]
    q, k, v = c["q"].to(DEV), c["k"].to(DEV), c["v"].to(DEV)
    for got, want in ((ops.attention_direct(q, k, v, c["scale"]), c["out"]),
                      (ops.attention_direct(q[:, :, c["positions"]].contiguous(), k, v, c["scale"],
                                            positions=c["positions"].to(DEV)), c["out_selected"])):
        # hardware exp2 and MMA summation order: a few bf16 ulps on a small share of elements
        d = bf16_ulp_diff(got.cpu(), want)
        assert d.max().item() <= 4 and (d > 0).float().mean().item() <= 0.1, (d.max().item(),
                                                                            (d > 0).float().mean().item())


def test_lm_readout(ref):
    c = ref["lm_readout"]
    _eq(ops.lm_readout(c["x"].to(DEV), _norm(c["norm"], c["eps"]), c["head"].to(DEV)), c["out"], "readout")


def test_swiglu(ref):
    c = ref["swiglu"]
    gu, i = c["gu"].to(DEV), c["I"]
    _eq(ops.swiglu(gu[:, :i], gu[:, i:]), c["out"], "swiglu")


def test_activation_quant(ref):
    c = ref["quant_static"]
    q8, _ = ops.quantize_activation(c["x"].to(DEV), L.QUANT_STATIC, c["inverse_scale"])
    _eq(q8.view(torch.uint8), c["q8"], "static e4m3")
    c = ref["quant_rows"]
    q8, s = ops.quantize_activation(c["x"].to(DEV), L.QUANT_ROWWISE)
    _eq(q8.view(torch.uint8), c["q8"], "row e4m3")
    _eq(s, c["scale"].reshape(-1), "row scales")


def test_weight_quant(ref):
    c = ref["weight_quant"]
    w8, s = ops.quantize_weight(c["w"].to(DEV), per_channel=False)
    _eq(w8.view(torch.uint8), c["w8_tensor"], "per-tensor e4m3")
    _eq(s, c["scale_tensor"].reshape(-1), "per-tensor scale")
    w8, s = ops.quantize_weight(c["w"].to(DEV), per_channel=True)
    _eq(w8.view(torch.uint8), c["w8_channel"], "per-channel e4m3")
    _eq(s, c["scale_channel"].reshape(-1), "per-channel scales")


def test_static_fp8_linear(ref):
    c = ref.get("runtime_scale_linear")
    if c is None:
        pytest.skip("fixture made without CPU torch._scaled_mm")
    w = c["w"]
    n = w.shape[0]
    # the GEMM tiles 128 output features: zero rows pad the weight (the per-tensor scale,
    # set by the largest |w|, is unchanged) and the extra outputs are dropped
    wp = torch.cat([w, torch.zeros(-n % 128, w.shape[1], dtype=w.dtype)])
    lin = ops.RuntimeScaleLinear(wp.to(DEV), inverse_scale=c["inverse_scale"])
    got = lin(c["x"].to(DEV)).cpu()[:, :n]
    # the reference ran torch._scaled_mm on the CPU (fp32 sums); the tensor core
    # truncates per 32-wide K step, which can move a bf16 result by one ulp
    d = bf16_ulp_diff(got, c["out"])
    assert d.max().item() <= 1, d.max().item()

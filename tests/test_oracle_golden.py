"""The oracle pinned to the reference: every function on the path reproduces, bit for bit,
the output of the reference's own code (Triton kernels under the CPU interpreter, torch
code, transformers' M-RoPE) stored in tests/golden/reference_ops.pt by
tests/golden/make_golden.py.  Also checks the product's host-side M-RoPE tables."""
from pathlib import Path

import pytest
import torch

import oracle
from oracle import qwen_path as Q

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_ops.pt"


@pytest.fixture(scope="module")
def ref():
    return torch.load(GOLDEN, weights_only=False)


def _eq(got, want, what):
    if got.dtype == torch.bfloat16:
        got, want = got.view(torch.int16), want.view(torch.int16)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    n = int((got != want).sum())
    assert n == 0, f"{what}: {n} of {got.numel()} elements differ from the reference"


@pytest.mark.parametrize("h", [2048, 2560])
def test_add_rms(ref, h):
    c = ref[f"add_rms_{h}"]
    r, y = oracle.add_rms(c["a"][0], c["b"][0], c["deep"], c["w"], c["eps"], c["start"], c["nv"])
    _eq(r, c["residual"][0], "residual")
    _eq(y, c["out"][0], "normed")


def test_fast_norm(ref):
    c = ref["fast_norm"]
    _eq(oracle.rms_one(c["x"][0], c["w"], c["eps"]), c["out"][0], "rms_one")


def test_qk_pair(ref):
    c = ref["qk_pair"]
    t, hq, hk = c["qkv"].shape[1], c["HQ"], c["HK"]
    q = c["qkv"][0, :, :hq * 128].reshape(t, hq, 128)
    k = c["qkv"][0, :, hq * 128:(hq + hk) * 128].reshape(t, hk, 128)
    yq, yk = oracle.qk_pair(q, k, c["q_norm"], c["k_norm"], c["cos"][0], c["sin"][0])
    _eq(yq, c["yq"][0], "yq")
    _eq(yk, c["yk"][0], "yk")


def test_attention_causal_and_selected(ref):
    c = ref["attention"]
    _eq(oracle.attention_direct(c["q"][0], c["k"][0], c["v"][0], c["scale"]), c["out"][0], "causal")
    sel = c["positions"]
    got = oracle.attention_direct(c["q"][0][:, sel], c["k"][0], c["v"][0], c["scale"], positions=sel)
    _eq(got, c["out_selected"][0], "selected rows")


def test_lm_readout(ref):
    c = ref["lm_readout"]
    _eq(oracle.lm_readout(c["x"][0], c["norm"], c["head"], c["eps"]), c["out"][0], "readout")


def test_swiglu(ref):
    c = ref["swiglu"]
    i = c["I"]
    _eq(oracle.swiglu(c["gu"][:, :i], c["gu"][:, i:]), c["out"], "swiglu")


def test_static_activation_quant(ref):
    c = ref["quant_static"]
    _eq(oracle.quantize_static(c["x"], c["inverse_scale"]).view(torch.uint8), c["q8"], "static e4m3 (padded rows)")


def test_rowwise_activation_quant(ref):
    c = ref["quant_rows"]
    q8, s = oracle.quantize_rows(c["x"])
    _eq(q8.view(torch.uint8), c["q8"], "row e4m3 (padded rows)")
    _eq(s.reshape(-1), c["scale"].reshape(-1), "row scales")


def test_weight_quant(ref):
    c = ref["weight_quant"]
    w8, s = oracle.quantize_weight_tensor(c["w"])
    _eq(w8.view(torch.uint8), c["w8_tensor"], "per-tensor e4m3")
    _eq(s.reshape(-1), c["scale_tensor"].reshape(-1), "per-tensor scale")
    w8, s = oracle.quantize_weight_channel(c["w"])
    _eq(w8.view(torch.uint8), c["w8_channel"], "per-channel e4m3")
    _eq(s.reshape(-1), c["scale_channel"].reshape(-1), "per-channel scales")


def test_static_fp8_linear_end_to_end(ref):
    c = ref.get("runtime_scale_linear")
    if c is None:
        pytest.skip("the generating torch had no CPU torch._scaled_mm")
    w8, ws = oracle.quantize_weight_tensor(c["w"])
    old = Q.set_accumulation("exact")  # the reference ran torch._scaled_mm on the CPU
    try:
        y = oracle.fp8_linear_static(c["x"], w8, ws, c["inverse_scale"])
    finally:
        Q.set_accumulation(old)
    _eq(y, c["out"], "RuntimeScaleLinear output")


def test_int4_asymmetric(ref):
    c = ref["int4_asym"]
    _, s, z, deq = oracle.int4_asym_quantize(c["w"])
    _eq(s.t().contiguous(), c["scales"][..., 0], "int4 scales")
    _eq(z.t().contiguous(), c["scales"][..., 1], "int4 zeros")
    _eq(deq, c["deq"], "int4 dequantised weight")


def test_mrope_oracle_and_host_tables(ref):
    from fastforward_b200 import mrope
    for m in ref["mrope"]:
        args = (m["n_tokens"], m["image_start"], m["grid_h"], m["grid_w"])
        pos = oracle.mrope_position_ids(*args)
        _eq(pos, m["position_ids"], f"oracle positions {args}")
        cos, sin = oracle.mrope_cos_sin(pos)
        _eq(cos, m["cos"], f"oracle cos {args}")
        _eq(sin, m["sin"], f"oracle sin {args}")
        # the product's host-side tables (uploaded once per graph key)
        hp = mrope.position_ids(*args)
        _eq(hp, m["position_ids"], f"host positions {args}")
        hc, hs = mrope.cos_sin(hp)
        _eq(hc, m["cos"], f"host cos {args}")
        _eq(hs, m["sin"], f"host sin {args}")

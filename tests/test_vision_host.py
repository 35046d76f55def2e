"""Host side of the vision tower (no GPU): the product's geometry tables equal the oracle's
(which is pinned to transformers' own vision code), the synthetic parameters have the
checkpoint shapes, the GELU restatement of the linear's epilogue is accurate, the oracle's
kernel-arithmetic tower agrees with its module-semantics tower, and the C ABI rejects bad
vision arguments before any CUDA call."""
import pytest
import torch

import oracle
from oracle import _tc
from fastforward_b200 import _lib as L
from fastforward_b200.checkpoint import vision_param_shapes
from fastforward_b200.config import VISION_MODELS, VisionDims
from fastforward_b200.synthetic import make_vision_bf16
from fastforward_b200.vision import VisionTower, position_table, rotary_cos_sin

BF16 = torch.bfloat16


@pytest.mark.parametrize("grid", [(32, 32), (16, 24), (8, 64), (2, 2)])
def test_geometry_equals_oracle(grid):
    gh, gw = grid
    table = (torch.randn(2304, 64) * 0.02).to(BF16)
    pos = position_table(table, gh, gw)
    ref_pos = oracle.vision_pos_embed(table, gh, gw)
    assert torch.equal(pos.view(torch.int16), ref_pos.view(torch.int16))
    for d in (64, 72):
        cos, sin = rotary_cos_sin(gh, gw, d)
        rc, rs = oracle.vision_rot_cos_sin(gh, gw, d)
        assert torch.equal(cos, rc) and torch.equal(sin, rs)


def test_synthetic_vision_parameters_have_checkpoint_shapes():
    v = VisionDims(64, 2, 128, 96, 2, (0,), num_pos=16)
    p = make_vision_bf16(v, seed=3)
    shapes = vision_param_shapes(v)
    assert set(p) == set(shapes)
    for name, shape in shapes.items():
        assert tuple(p[name].shape) == tuple(shape) and p[name].dtype == BF16, name
    assert torch.equal(make_vision_bf16(v, seed=3)["blocks.1.attn.qkv.weight"], p["blocks.1.attn.qkv.weight"])


def test_launch_count():
    assert VisionTower.launches(VISION_MODELS["4B"]) == 1 + 8 * 24 + 3 * 4


@pytest.mark.parametrize("form,approx", [("tanh", "tanh"), ("erf", "none")])
def test_gelu_epilogue_accuracy(form, approx):
    """The epilogue's GELU (own tanh / Abramowitz-Stegun erf over exp2_poly) rounds to the
    same bf16 as the exact function on every bf16 input of |x| < 3, and stays within 5e-7
    absolute everywhere."""
    x = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16).view(BF16).float()
    x = x[torch.isfinite(x) & (x.abs() < 64)]
    y = _tc.gelu(x, form)
    exact = torch.nn.functional.gelu(x.double(), approximate=approx)
    assert (y.double() - exact).abs().max().item() < 5e-7
    small = x.abs() < 3
    assert torch.equal(y[small].to(BF16), exact[small].to(BF16))


def test_layer_norm_restatement_matches_float64():
    g = torch.Generator().manual_seed(0)
    x = (torch.randn(7, 1152, generator=g) * 3 + 0.5).to(BF16)
    w = (1 + torch.randn(1152, generator=g) * 0.1).to(BF16)
    b = (torch.randn(1152, generator=g) * 0.02).to(BF16)
    y = oracle.layer_norm_k(x, w, b, 1e-6)
    ref = torch.nn.functional.layer_norm(x.double(), (1152,), w.double(), b.double(), 1e-6)
    assert (y.double() - ref).abs().max().item() <= 2 ** -7 * ref.abs().max().item()


def test_kernel_arithmetic_tower_close_to_module_semantics():
    """`vision_tower_k` (the kernels' rounding points) against `vision_tower` in fp32 (the HF
    modules' semantics) on a small two-block tower: the bf16 roundings between kernels
    move the outputs by a few bf16 ulps only."""
    v = VisionDims(128, 2, 256, 128, 2, (0,), num_pos=64)
    p = make_vision_bf16(v, seed=1)
    g = torch.Generator().manual_seed(2)
    pixels = (torch.rand(64, 1536, generator=g) * 2 - 1).to(BF16)
    mk, dk = oracle.vision_tower_k(p, v, pixels, 8, 8)
    mf, df = oracle.vision_tower({k: t.float() for k, t in p.items()}, v, pixels.float(), 8, 8)
    for a, b in [(mk, mf)] + list(zip(dk, df)):
        err = (a.float() - b).abs().max().item()
        assert err <= 0.02 * b.abs().max().item(), err


def test_vision_entries_reject_bad_arguments():
    with pytest.raises(ValueError, match="multiples of 8"):
        L.call("ffb_bf16_gemm", 16, 16, None, None, L.EPI_BIAS, 16, 0, 1, None, None, 16, 20, 64, None)
    with pytest.raises(ValueError, match="epilogue"):
        L.call("ffb_bf16_gemm", 16, 16, None, None, 99, 16, 0, 1, None, None, 16, 16, 64, None)
    with pytest.raises(ValueError, match="BIAS_RES"):
        L.call("ffb_bf16_gemm", 16, 16, None, None, L.EPI_BIAS_RES, 16, 0, 1, None, None, 16, 16, 64, None)
    with pytest.raises(ValueError, match="feature tile"):
        L.call("ffb_bf16_gemm", 16, 16, None, None, L.EPI_BIAS, 16, 96, 1, None, None, 16, 16, 64, None)
    with pytest.raises(ValueError, match="splits"):
        L.call("ffb_bf16_gemm", 16, 16, None, None, L.EPI_BIAS, 16, 0, 2, None, None, 16, 16, 640, None)
    with pytest.raises(ValueError, match="splits"):
        L.call("ffb_bf16_gemm", 16, 16, None, None, L.EPI_BIAS, 16, 0, 3, None, None, 16, 16, 128, None)
    with pytest.raises(ValueError, match="head dim"):
        L.call("ffb_attention_full", 16, 16, 16, 16, 64, 4, 12, 0.1, None)
    with pytest.raises(ValueError, match="multiple of 8"):
        L.call("ffb_layernorm", 16, 16, 16, 1e-6, 16, 4, 100, None)
    with pytest.raises(ValueError, match="residual"):
        L.call("ffb_add_layernorm", 16, 16, 16, 16, 1e-6, None, 16, 4, 128, None)
    with pytest.raises(ValueError, match="bad shape"):
        L.call("ffb_vision_rope", 16, 16, 16, 4, 2, 9, 128, 16, 16, 16, None)


def test_linear_plans():
    """The plan minimises the fitted time model (no GPU here: the library assumes 148 SMs):
    qkv / fc1 unsplit 256-wide tiles; proj 256-wide split 2 ways, fc2 and the mergers' K=4096
    linears split 4 ways (cluster split-K: no counters); a many-tile K=64 shape 128-wide."""
    assert L.bf16_gemm_plan(1024, 3072, 1024) == (256, 1, 0)
    assert L.bf16_gemm_plan(1024, 4096, 1024) == (256, 1, 0)
    assert L.bf16_gemm_plan(1024, 1024, 1024) == (256, 2, 0)
    assert L.bf16_gemm_plan(1024, 1024, 4096) == (256, 4, 0)
    assert L.bf16_gemm_plan(256, 4096, 4096) == (256, 4, 0)
    assert L.bf16_gemm_plan(256, 2560, 4096) == (256, 4, 0)
    assert L.bf16_gemm_plan(4096, 4096, 64) == (128, 1, 0)
    with pytest.raises(ValueError, match="bad shape"):
        L.bf16_gemm_plan(0, 4096, 64)


def test_read_canvas_formats(tmp_path):
    """Canvases come as arrays, .npy files or binary PPM (P6) files; anything else, or sides
    that are not multiples of 32, is rejected."""
    import numpy as np
    from fastforward_b200.vision import read_canvas, synthetic_text_ids
    a = np.random.default_rng(0).integers(0, 256, (64, 96, 3), dtype=np.uint8)
    np.save(tmp_path / "c.npy", a)
    (tmp_path / "c.ppm").write_bytes(b"P6\n# comment\n96 64\n255\n" + a.tobytes())
    for src in (a, torch.from_numpy(a), tmp_path / "c.npy", tmp_path / "c.ppm"):
        assert torch.equal(read_canvas(src), torch.from_numpy(a))
    (tmp_path / "x.png").write_bytes(b"\x89PNG not decoded here")
    with pytest.raises(ValueError, match="npy or binary PPM"):
        read_canvas(tmp_path / "x.png")
    with pytest.raises(ValueError, match="multiples of 32"):
        read_canvas(a[:48])
    p1, s1 = synthetic_text_ids("q", ["a", "b"], 4, 8, 1000)
    p2, s2 = synthetic_text_ids("q", ["a", "b"], 4, 8, 1000)
    assert torch.equal(p1, p2) and torch.equal(s1, s2) and p1.shape == (4,) and s1.shape == (8,)

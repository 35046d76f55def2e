"""Static-FP8 calibration profiles (host logic and the oracle, no GPU): the reference's
bound rule (`_legacy/limit_runtime.py:88-91`), the profile keys (`_family/night_runtime.py:
48-54, 72-76`) and the oracle's calibration over a small model."""
import math

import pytest
import torch

import oracle
from fastforward_b200.config import MODELS, Layout
from fastforward_b200.engine import PROFILE_ROLE, PackedModel, static_bound
from fastforward_b200.mrope import position_ids
from tests._model import small_case


def test_static_bound_rule():
    # 448 / (1.0 * 1.5) = 298.7 -> inverse 2^8 = 256 -> bound 1.75
    assert static_bound(1.0) == 448.0 / 256
    assert static_bound(0.0) == 448.0 / 2.0 ** math.floor(math.log2(448.0 / 1.5e-12))
    g = torch.Generator().manual_seed(0)
    for m in torch.exp(torch.randn(2000, generator=g, dtype=torch.float64) * 4).tolist():
        for margin in (1.0, 1.5, 2.0):
            b = static_bound(m, margin)
            assert b == oracle.static_bound(m, margin)
            inv = 448.0 / b
            assert inv == 2.0 ** round(math.log2(inv))          # a power of two
            assert 224.0 < inv * m * margin <= 448.0              # the largest such power


def test_profile_keys_follow_the_reference():
    assert [PROFILE_ROLE[r] for r in ("qkv", "o", "gateup", "down")] == ["qkv", "output", "gateup", "down"]
    assert oracle.qwen_path.PROFILE_ROLE == PROFILE_ROLE


def test_profile_needs_static_mode():
    with pytest.raises(ValueError):
        PackedModel(MODELS["2B"], {"layers": []}, mode="rowwise", device="cpu", profile={"0:qkv": 1.0})


def test_oracle_calibration_small_model():
    """The bf16 calibration forward observes every linear of every layer, each bound puts
    the observed maximum into (224, 448] / margin of the e4m3 range, and the static model
    built from the profile carries inverse 448/bound and input scale fp32(bound/448)."""
    dims, src, req, layout = small_case(MODELS["2B"], 2, layout=Layout(0, 8, 8, 32, k=4), vocab=1024)
    T = layout.bucket
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    r = dict(ids=req["ids"][:T], visual=req["visual"], deepstack=req["deep"], position_ids=pos, pick=req["pick"],
             k=req["k"], image_start=layout.image_start)
    prof, seen = oracle.calibration_profile(oracle.quantized_model(dims, src, "bf16"), [r])
    assert set(prof) == {f"{j}:{n}" for j in range(2) for n in ("qkv", "output", "gateup", "down")}
    for key, bound in prof.items():
        assert 224.0 < (448.0 / bound) * seen[key] * 1.5 <= 448.0, key
    om = oracle.quantized_model(dims, src, "static", profile=prof)
    lin = om["layers"][1]["down"]
    assert lin["inv"] == 448.0 / prof["1:down"]
    assert lin["a_scale"].item() == torch.tensor(prof["1:down"] / 448.0, dtype=torch.float32).item()
    z, lp = oracle.prefill_score(om, mode="static", **r)
    assert torch.isfinite(z).all() and torch.isfinite(lp).all()

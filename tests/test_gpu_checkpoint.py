"""A checkpoint bundle on the GPU: `Accelerator` built from a bundle whose `model` is a
Hugging Face Qwen3-VL directory (written by `checkpoint.save_language_model`) answers
exactly as an engine built from the same weights in memory -- the loader changes nothing
the kernels see."""
import json
import threading
from dataclasses import replace

import pytest
import torch

from fastforward_b200 import checkpoint as C
from fastforward_b200.api import Accelerator, sha256
from fastforward_b200.config import MODELS, Layout
from fastforward_b200.engine import Engine, PackedModel
from fastforward_b200.synthetic import make_model_bf16, make_request

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


@pytest.mark.parametrize("mode", ["fp8", "fp8_rowwise", "int4"])
def test_checkpoint_bundle_matches_in_memory_weights(tmp_path, mode):
    """fp8 = the reference's static-scale scheme with the bundle's calibration profile
    (`profile_path`, `variant`); fp8_rowwise and int4 need none."""
    dims = replace(MODELS["2B"], vocab=4096, layers=2)
    src = make_model_bf16(dims, seed=4)
    lay = Layout(5, 8, 12, 40, k=3)
    r = make_request(dims, lay, seed=9)
    n = lay.n_tokens
    extra, profile = {}, None
    if mode == "fp8":
        from fastforward_b200.engine import calibrate_profile
        T = 128
        cal = make_request(dims, lay, seed=10, device=DEV)
        profile, _ = calibrate_profile(dims, src,
                                       [dict(ids=cal["ids"][:T], visual=cal["visual"], deep=cal["deep"], pick=n - 1,
                                             k=lay.k, image_start=lay.image_start, grid_h=lay.grid_h,
                                             grid_w=lay.grid_w, T=T)], device=DEV)
        prof = tmp_path / "profiles.json"
        prof.write_text(json.dumps({"profiles": {"aspect320": profile}}))
        extra = dict(profile_path=str(prof), profile_sha256=sha256(prof), variant="aspect320")
    C.save_language_model(tmp_path / "model", dims, src, shards=2)
    ck = tmp_path / "repair.pt"
    torch.save({"state_dict": {"down": torch.randn(32, dims.hidden), "up": torch.zeros(dims.hidden, 32),
                               "bias": torch.zeros(dims.hidden)}}, ck)
    bundle = tmp_path / "bundle.json"
    bundle.write_text(json.dumps(dict(
        schema_version=1, task="visual_choice", architecture="qwen3_vl_family", model=str(tmp_path / "model"),
        expected_dimensions=[2, dims.hidden, 24], checkpoint=str(ck), checkpoint_sha256=sha256(ck),
        execution_mode=mode, buckets=[64, 128, 256], **extra)))
    acc = Accelerator(bundle)
    assert acc.dims.layers == 2 and acc.encoder is None
    got = acc.prefill_score(r["ids"][:n], r["visual"], r["deep"], lay.k, lay.image_start, lay.grid_h, lay.grid_w)
    # the same weights, packed from memory
    pm = PackedModel(dims, src, mode={"fp8": "static", "fp8_rowwise": "rowwise", "int4": "int4"}[mode], device=DEV,
                     profile=profile)
    ref = Accelerator.__new__(Accelerator)
    ref.engine, ref.dims, ref.device, ref.lock, ref.buckets = Engine(pm), dims, DEV, threading.RLock(), (64, 128, 256)
    want = ref.prefill_score(r["ids"][:n], r["visual"], r["deep"], lay.k, lay.image_start, lay.grid_h, lay.grid_w)
    assert got == want
    with pytest.raises(RuntimeError, match="encoder"):
        img = tmp_path / "x.png"
        img.write_bytes(b"\x89PNG")
        acc.predict(img, "Which?", ["a", "b"])

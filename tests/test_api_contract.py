"""The public surface's contract, as the reference's tests/test_contract.py pins it:
request validation, the response dict (first maximum wins, probabilities sum to one,
non-finite logits raise), and the Accelerator's argument errors -- all on the CPU."""
import json
import math

import pytest

from fastforward_b200.api import Accelerator, response, validate_request


def test_reference_import_name_resolves_to_this_surface():
    """`fastforward_accel.Accelerator(config, backend="fast")` -- the reference's import
    name -- is this package's surface, so the reference's callers run unchanged."""
    import fastforward_accel
    assert fastforward_accel.Accelerator is Accelerator
    assert fastforward_accel.validate_request is validate_request
    assert fastforward_accel.response is response


def test_request_validation(tmp_path):
    image = tmp_path / "input.png"
    image.touch()
    validate_request(image, "Question", ["A", "B"])
    for choices in (["A"], ["A", ""], ["A"] * 9, "AB"):
        with pytest.raises(ValueError):
            validate_request(image, "Question", choices)
    with pytest.raises(ValueError, match="nonempty question"):
        validate_request(image, "  ", ["A", "B"])
    with pytest.raises(FileNotFoundError):
        validate_request(tmp_path / "missing.png", "Question", ["A", "B"])


def test_response():
    r = response([1.0, 1.0], ["a", "b"], "x")
    assert r["answer"] == {"letter": "A", "text": "a"}  # ties: the first maximum wins
    assert r["id"] == "x"
    assert math.isclose(sum(r["probabilities"]), 1.0)
    r = response([0.5, 2.0, -1.0], ["a", "b", "c"], "y", logprobs=[-1.7, -0.2, -3.2])
    assert r["answer"]["letter"] == "B" and r["logprobs"] == [-1.7, -0.2, -3.2]
    with pytest.raises(RuntimeError):
        response([float("nan"), 0.0], ["a", "b"], "x")
    with pytest.raises(RuntimeError):
        response([1.0], ["a", "b"], "x")


def _bundle(tmp_path, **kw):
    c = dict(schema_version=1, task="visual_choice", architecture="qwen3_vl_family",
             synthetic=dict(model="2B", layers=1, seed=0))
    c.update(kw)
    p = tmp_path / "bundle.json"
    p.write_text(json.dumps(c))
    return p


def test_accelerator_argument_errors(tmp_path):
    with pytest.raises(ValueError, match="schema"):
        Accelerator(_bundle(tmp_path, schema_version=2))
    with pytest.raises(ValueError, match="backend"):
        Accelerator(_bundle(tmp_path), backend="native-cpu")
    with pytest.raises(FileNotFoundError):
        Accelerator(_bundle(tmp_path, synthetic=None, model=str(tmp_path / "no-model"),
                            checkpoint=str(tmp_path / "no-ckpt"), checkpoint_sha256="0"))


def test_accelerator_has_no_cpu_fallback(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CPU fallback is disabled"):
        Accelerator(_bundle(tmp_path))


def test_static_profile_bundle_fields(tmp_path):
    """Static-FP8 bundles name their calibration profile as the reference's bundles do
    (`_family/family_api.py:27-31`): path, sha256 and variant."""
    from fastforward_b200.api import sha256
    prof = tmp_path / "profile.json"
    prof.write_text(json.dumps({"profiles": {"v1": {"0:qkv": 3.5, "0:output": 1.75}}}))
    c = dict(profile_path=str(prof), profile_sha256=sha256(prof), variant="v1")
    assert Accelerator._read_profile(c) == {"0:qkv": 3.5, "0:output": 1.75}
    assert Accelerator._read_profile({}) is None
    with pytest.raises(ValueError):
        Accelerator._read_profile(dict(c, profile_sha256="0" * 64))
    with pytest.raises(ValueError):
        Accelerator._read_profile(dict(c, variant="v2"))
    with pytest.raises(FileNotFoundError):
        Accelerator._read_profile(dict(c, profile_path=str(tmp_path / "missing.json")))


def test_prefill_score_batch_validates_before_the_device():
    """The batched entry rejects a bad request (choice count, visual rows vs grid) before
    anything reaches the engine."""
    import threading
    import torch
    acc = Accelerator.__new__(Accelerator)
    acc.lock = threading.RLock()
    acc.engine = None  # never reached
    good = dict(ids=torch.zeros(8, dtype=torch.long), visual=torch.zeros((16, 8)), deep=[], k=4, image_start=0,
                grid_h=8, grid_w=8)
    with pytest.raises(ValueError, match="two to eight"):
        acc.prefill_score_batch([good, dict(good, k=9)])
    with pytest.raises(ValueError, match="merged image grid"):
        acc.prefill_score_batch([dict(good, grid_h=6)])

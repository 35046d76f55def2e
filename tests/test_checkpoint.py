"""Checkpoint bundles on the host: the Hugging Face Qwen3-VL checkpoint reader
(`fastforward_b200.checkpoint`) against checkpoints written by transformers itself, the
writer/reader round trip (single file and sharded), the bundle's asset checks (the
reference's `api.py:56-66`, `_family/family_api.py:19-23`) -- no GPU."""
import json

import pytest
import torch

from fastforward_b200 import checkpoint as C
from fastforward_b200.api import Accelerator, sha256
from fastforward_b200.config import Dims, MODELS
from fastforward_b200.synthetic import make_model_bf16

BF16 = torch.bfloat16
TINY = dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
            intermediate_size=512, vocab_size=1024)
OPT = (11, 12, 13, 14, 15, 16, 17, 18)


def _hf_checkpoint(path, tied):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Qwen3VLConfig(
        text_config=dict(TINY, tie_word_embeddings=tied), tie_word_embeddings=tied,
        vision_config=dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=2, out_hidden_size=256,
                           deepstack_visual_indexes=[0, 1]))
    torch.manual_seed(0)
    m = transformers.Qwen3VLForConditionalGeneration(cfg).to(BF16)
    with torch.no_grad():  # non-trivial norm weights, so a swapped norm would show
        for n, p in m.named_parameters():
            if "norm" in n:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    m.save_pretrained(str(path), safe_serialization=True)
    return {k: v.detach().clone() for k, v in m.state_dict().items()}


def test_expected_vision_depth_is_checked(tmp_path):
    """A bundle's expected_dimensions (layers, hidden, vision blocks) must match the
    checkpoint's vision depth too (`scaled_qwen_runtime.py:69`)."""
    _hf_checkpoint(tmp_path, True)
    C.load_language_model(tmp_path, option_ids=OPT, expected_dimensions=[2, 256, 2])
    with pytest.raises(C.CheckpointError, match="vision blocks"):
        C.load_language_model(tmp_path, option_ids=OPT, expected_dimensions=[2, 256, 24])


@pytest.mark.parametrize("tied", [True, False])
def test_reads_checkpoints_written_by_transformers(tmp_path, tied):
    sd = _hf_checkpoint(tmp_path, tied)
    dims, m = C.load_language_model(tmp_path, option_ids=OPT)
    assert (dims.layers, dims.hidden, dims.hq, dims.hk, dims.inter, dims.d, dims.vocab) == (2, 256, 4, 2, 512, 128, 1024)
    assert dims.deepstack == 2 and dims.sections == (24, 20, 20) and dims.name == "custom"
    lm = "model.language_model."
    assert torch.equal(m["embed"], sd[lm + "embed_tokens.weight"])
    head_src = sd[lm + "embed_tokens.weight"] if tied else sd["lm_head.weight"]
    assert torch.equal(m["head"], head_src[list(OPT)])
    assert torch.equal(m["final_norm"], sd[lm + "norm.weight"])
    for j, lay in enumerate(m["layers"]):
        p = f"{lm}layers.{j}."
        assert torch.equal(lay["qkv"], torch.cat([sd[p + f"self_attn.{x}_proj.weight"] for x in "qkv"]))
        assert torch.equal(lay["gateup"], torch.cat([sd[p + "mlp.gate_proj.weight"], sd[p + "mlp.up_proj.weight"]]))
        assert torch.equal(lay["o"], sd[p + "self_attn.o_proj.weight"])
        assert torch.equal(lay["down"], sd[p + "mlp.down_proj.weight"])
        for mine, theirs in (("in_norm", "input_layernorm"), ("post_norm", "post_attention_layernorm"),
                             ("q_norm", "self_attn.q_norm"), ("k_norm", "self_attn.k_norm")):
            assert torch.equal(lay[mine], sd[p + theirs + ".weight"]), mine
    d1, m1 = C.load_language_model(tmp_path, option_ids=OPT, layers=1)
    assert len(m1["layers"]) == 1 and torch.equal(m1["layers"][0]["qkv"], m["layers"][0]["qkv"])


@pytest.mark.parametrize("shards,tied", [(1, True), (3, False)])
def test_save_load_round_trip(tmp_path, shards, tied):
    from dataclasses import replace
    dims = replace(MODELS["2B"], hidden=256, hq=2, hk=1, inter=384, vocab=512, layers=2, tied=tied)
    src = make_model_bf16(dims, seed=3)
    C.save_language_model(tmp_path, dims, src, shards=shards)
    assert (tmp_path / "model.safetensors.index.json").exists() == (shards > 1)
    d2, m = C.load_language_model(tmp_path)
    assert (d2.layers, d2.hidden, d2.hq, d2.hk, d2.inter, d2.vocab, d2.tied) == \
        (dims.layers, dims.hidden, dims.hq, dims.hk, dims.inter, dims.vocab, tied)
    assert d2.theta == dims.theta and d2.sections == dims.sections and d2.deepstack == dims.deepstack
    for key in ("embed", "head", "final_norm"):
        assert torch.equal(m[key], src[key]), key
    for a, b in zip(m["layers"], src["layers"]):
        assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)


def test_dims_of_the_shipped_families():
    for name, dims in MODELS.items():
        cfg = dict(model_type="qwen3_vl", tie_word_embeddings=dims.tied,
                   text_config=dict(hidden_size=dims.hidden, num_hidden_layers=dims.layers,
                                    num_attention_heads=dims.hq, num_key_value_heads=dims.hk, head_dim=128,
                                    intermediate_size=dims.inter, vocab_size=dims.vocab, rms_norm_eps=1e-6,
                                    rope_theta=5_000_000, rope_scaling=dict(mrope_section=[24, 20, 20])),
                   vision_config=dict(deepstack_visual_indexes=[5, 11, 17]))
        assert C.dims_from_config(cfg) == dims, name


def test_checkpoint_errors(tmp_path):
    from dataclasses import replace
    dims = replace(MODELS["2B"], hidden=256, hq=2, hk=1, inter=384, vocab=512, layers=2)
    src = make_model_bf16(dims, seed=3)
    C.save_language_model(tmp_path, dims, src)
    with pytest.raises(C.CheckpointError, match="expected"):
        C.load_language_model(tmp_path, expected_dimensions=[36, 2560, 24])
    C.load_language_model(tmp_path, expected_dimensions=[2, 256, 24])
    with pytest.raises(C.CheckpointError, match="option"):
        C.load_language_model(tmp_path, option_ids=(1, 2, 3))
    cfg = json.loads((tmp_path / "config.json").read_text())
    cfg["text_config"]["intermediate_size"] = 512  # shapes no longer match the tensors
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(C.CheckpointError, match="shape"):
        C.load_language_model(tmp_path)
    with pytest.raises(C.CheckpointError, match="config.json"):
        C.load_language_model(tmp_path / "nowhere")


def test_option_ids_from_tokenizer(tmp_path):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    vocab = {"[UNK]": 0, **{" " + a: 100 + i for i, a in enumerate("ABCDEFGH")}}
    Tokenizer(WordLevel(vocab, unk_token="[UNK]")).save(str(tmp_path / "tokenizer.json"))
    assert C.option_token_ids(tmp_path) == tuple(range(100, 108))
    assert C.option_token_ids(tmp_path / "none") is None


def _assets(tmp_path, up=0.0):
    model = tmp_path / "model"
    model.mkdir()
    ck = tmp_path / "repair.pt"
    torch.save({"state_dict": {"down": torch.randn(32, 256), "up": torch.full((256, 32), up),
                               "bias": torch.zeros(256)}}, ck)
    return dict(model=str(model), checkpoint=str(ck), checkpoint_sha256=sha256(ck))


def test_bundle_asset_checks(tmp_path):
    c = _assets(tmp_path)
    Accelerator._check_assets(c)
    with pytest.raises(ValueError, match="SHA256"):
        Accelerator._check_assets(dict(c, checkpoint_sha256="0" * 64))
    with pytest.raises(FileNotFoundError):
        Accelerator._check_assets(dict(c, model=str(tmp_path / "missing")))
    sub = tmp_path / "nonzero"
    sub.mkdir()
    bad = _assets(sub, up=0.5)
    with pytest.raises(ValueError, match="not zero"):
        Accelerator._check_assets(bad)
    assert Accelerator._checkpoint_mode({}) == "static"
    assert Accelerator._checkpoint_mode({"execution_mode": "int4"}) == "int4"
    assert Accelerator._checkpoint_mode({"execution_mode": "fp8_rowwise"}) == "rowwise"
    with pytest.raises(ValueError):
        Accelerator._checkpoint_mode({"execution_mode": "bf16"})


def test_reads_the_vision_tower_written_by_transformers(tmp_path):
    """The vision tower's tensors come back under their checkpoint names with the config's
    shapes, and the vision oracle run on them reproduces transformers' own vision forward."""
    transformers = pytest.importorskip("transformers")
    import numpy as np
    import oracle
    cfg = transformers.Qwen3VLConfig(
        text_config=dict(TINY), vision_config=dict(depth=2, hidden_size=64, intermediate_size=128, num_heads=2,
                                                   out_hidden_size=256, deepstack_visual_indexes=[1]))
    torch.manual_seed(3)
    m = transformers.Qwen3VLForConditionalGeneration(cfg).to(BF16)
    m.save_pretrained(str(tmp_path), safe_serialization=True)
    vd, params = C.load_vision_tower(tmp_path)
    assert (vd.hidden, vd.heads, vd.inter, vd.out_hidden, vd.depth, vd.deepstack) == (64, 2, 128, 256, 2, (1,))
    sd = m.state_dict()
    assert set(params) == {k[len(C.VISUAL):] for k in sd if k.startswith(C.VISUAL)}
    for name, x in params.items():
        assert torch.equal(x, sd[C.VISUAL + name]), name
    rgb = np.random.default_rng(0).integers(0, 256, (64, 64, 3), dtype=np.uint8)
    pixels = oracle.pack_rgb(rgb).float()
    visual = m.model.visual.float()
    with torch.no_grad():
        want = visual(pixels, grid_thw=torch.tensor([[1, 4, 4]]))
        got, deep = oracle.vision_tower({k: v.float() for k, v in params.items()},
                                        oracle.VisionDims.from_config(cfg.vision_config), pixels, 4, 4)
    torch.testing.assert_close(got, want.pooler_output, atol=2e-5, rtol=2e-5)
    torch.testing.assert_close(deep[0], want.deepstack_features[0], atol=2e-5, rtol=2e-5)
    (tmp_path / "model.safetensors").unlink()
    with pytest.raises(C.CheckpointError):
        C.load_vision_tower(tmp_path)


def test_vision_shapes_of_the_shipped_families():
    from fastforward_b200.config import VISION_MODELS
    for name, v in VISION_MODELS.items():
        assert v.out_hidden == MODELS[name].hidden and v.head_dim in (64, 72) and v.depth in (24, 27)
        shapes = C.vision_param_shapes(v)
        assert shapes["deepstack_merger_list.2.linear_fc2.weight"] == (v.out_hidden, 4 * v.hidden)
        assert len([k for k in shapes if k.startswith("blocks.")]) == 12 * v.depth

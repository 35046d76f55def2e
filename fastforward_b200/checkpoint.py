"""Real Qwen3-VL checkpoints: the language decoder's weights from a Hugging Face model
directory (config.json + safetensors, single file or sharded with an index) into the bf16
layout `PackedModel` packs to FP8 / int4.

The reference loads the whole model with `Qwen3VLForConditionalGeneration.from_pretrained`
(`scaled_qwen_runtime.py:61-63`), checks `expected_dimensions` (`:67`), reads the option
rows of `lm_head` (`:68`) and, in `pack_release` (`_family/depth_runtime.py:99-117`),
concatenates q/k/v and gate/up per layer before quantising them.  Here only the tensors the
decoder path needs are read (lazily, tensor by tensor, from the safetensors files: the
vision tower's weights are never loaded), in the same concatenations.

`save_language_model` writes the inverse (the Hugging Face names and a config.json), so a
synthetic model can be exported and re-read; the tests use it to check the round trip.
"""
import json
from pathlib import Path

import torch

from .config import MODELS, OPTION_IDS, Dims

BF16 = torch.bfloat16
LM = "model.language_model."
OPTION_LETTERS = "ABCDEFGH"


class CheckpointError(ValueError):
    """The model directory does not hold a supported Qwen3-VL checkpoint."""


# ---------------------------------------------------------------------------- config

def _rope(tc):
    """(theta, mrope sections) from a text config in either transformers layout
    (`rope_theta` + `rope_scaling`, or `rope_parameters`)."""
    rp = tc.get("rope_parameters") or {}
    rs = tc.get("rope_scaling") or {}
    theta = tc.get("rope_theta", rp.get("rope_theta", 5_000_000.0))
    sections = rs.get("mrope_section") or rp.get("mrope_section") or (24, 20, 20)
    return float(theta), tuple(int(x) for x in sections)


def dims_from_config(config):
    """`Dims` of the language decoder described by a Qwen3-VL config.json (dict or path)."""
    if not isinstance(config, dict):
        config = json.loads(Path(config).read_text())
    if config.get("model_type") not in ("qwen3_vl", None):
        raise CheckpointError(f"model_type {config.get('model_type')!r} is not qwen3_vl")
    tc = config.get("text_config", config)
    try:
        layers, hidden = int(tc["num_hidden_layers"]), int(tc["hidden_size"])
        hq, hk = int(tc["num_attention_heads"]), int(tc["num_key_value_heads"])
        inter, vocab = int(tc["intermediate_size"]), int(tc["vocab_size"])
    except KeyError as e:
        raise CheckpointError(f"text config lacks {e}") from None
    d = int(tc.get("head_dim", hidden // hq))
    theta, sections = _rope(tc)
    if sum(sections) * 2 != d:
        raise CheckpointError(f"mrope sections {sections} do not cover head_dim {d}")
    vc = config.get("vision_config") or {}
    deepstack = len(vc.get("deepstack_visual_indexes", (0, 1, 2)))
    tied = bool(config.get("tie_word_embeddings", tc.get("tie_word_embeddings", False)))
    name = next((k for k, v in MODELS.items()
                 if (v.layers, v.hidden, v.hq, v.hk, v.inter, v.d) == (layers, hidden, hq, hk, inter, d)), "custom")
    return Dims(name, layers, hidden, hq, hk, inter, d=d, vocab=vocab, tied=tied,
                eps=float(tc.get("rms_norm_eps", 1e-6)), theta=theta, sections=sections, deepstack=deepstack)


# ---------------------------------------------------------------------------- tensors

class _Tensors:
    """Lazy name -> tensor access over the safetensors files of a model directory."""

    def __init__(self, model_dir):
        from safetensors import safe_open
        d = Path(model_dir)
        index = d / "model.safetensors.index.json"
        if index.exists():
            wm = json.loads(index.read_text())["weight_map"]
            files = sorted(set(wm.values()))
        else:
            files = sorted(p.name for p in d.glob("*.safetensors"))
            if not files:
                raise CheckpointError(f"no safetensors files in {d}")
            wm = None
        self.handles = {f: safe_open(str(d / f), framework="pt") for f in files}
        if wm is None:
            wm = {k: f for f, h in self.handles.items() for k in h.keys()}
        self.where = wm

    def __contains__(self, name):
        return name in self.where

    def get(self, name):
        if name not in self.where:
            raise CheckpointError(f"checkpoint lacks {name}")
        return self.handles[self.where[name]].get_tensor(name)


def option_token_ids(model_dir):
    """Token ids of " A" .. " H" from the model directory's tokenizer (the reference's
    `option_ids`, `scaled_qwen_runtime.py:70-72`); None when the directory has no
    tokenizer.json."""
    f = Path(model_dir) / "tokenizer.json"
    if not f.exists():
        return None
    from tokenizers import Tokenizer
    tok = Tokenizer.from_file(str(f))
    ids = []
    for a in OPTION_LETTERS:
        enc = tok.encode(" " + a, add_special_tokens=False).ids
        ids.append(enc[0])
    return tuple(ids)


def load_language_model(model_dir, *, device="cpu", layers=None, option_ids=None, expected_dimensions=None):
    """(dims, bf16 model) of the checkpoint in `model_dir`, in `PackedModel`'s layout:
    embed [V, H], head [8, H] (the lm_head rows of the option tokens), final_norm [H], and
    per layer qkv = cat(q, k, v), o, gateup = cat(gate, up), down, in_norm, post_norm,
    q_norm, k_norm (`_family/depth_runtime.py:103-104`).

    option_ids: the eight option token ids (default: from tokenizer.json, else the
    built-in ids).  expected_dimensions: the bundle's (layers, hidden, ...) check
    (`scaled_qwen_runtime.py:67`).  layers: load only the first n decoder layers."""
    d = Path(model_dir)
    if not (d / "config.json").exists():
        raise CheckpointError(f"{d} has no config.json")
    dims = dims_from_config(d / "config.json")
    if expected_dimensions is not None and tuple(expected_dimensions[:2]) != (dims.layers, dims.hidden):
        raise CheckpointError(f"expected (layers, hidden) {tuple(expected_dimensions[:2])}, "
                              f"checkpoint has {(dims.layers, dims.hidden)}")
    if expected_dimensions is not None and len(expected_dimensions) > 2:
        # the third entry is the vision tower's depth, as the reference asserts
        # (`scaled_qwen_runtime.py:69`); checked whenever the config states one (a
        # language-only checkpoint written by `save_language_model` does not)
        vc = json.loads((d / "config.json").read_text()).get("vision_config") or {}
        if "depth" in vc and int(expected_dimensions[2]) != int(vc["depth"]):
            raise CheckpointError(f"expected {int(expected_dimensions[2])} vision blocks, "
                                  f"checkpoint has {int(vc['depth'])}")
    t = _Tensors(d)
    dev = torch.device(device)

    def w(name, shape):
        x = t.get(name)
        if tuple(x.shape) != tuple(shape):
            raise CheckpointError(f"{name}: shape {tuple(x.shape)}, expected {tuple(shape)}")
        return x.to(dev, BF16).contiguous()

    h, hd = dims.hidden, dims.d
    embed = w(LM + "embed_tokens.weight", (dims.vocab, h))
    ids = option_ids if option_ids is not None else (option_token_ids(d) or OPTION_IDS)
    ids = torch.tensor(ids, dtype=torch.long)
    if len(ids) != 8 or int(ids.max()) >= dims.vocab:
        raise CheckpointError("need eight option token ids inside the vocabulary")
    head_full = "lm_head.weight"
    if head_full in t:  # untied head (or a tied one stored explicitly): its option rows only
        head = t.get(head_full)
        if tuple(head.shape) != (dims.vocab, h):
            raise CheckpointError(f"lm_head: shape {tuple(head.shape)}")
        head = head[ids].to(dev, BF16).contiguous()
    else:
        head = embed[ids.to(dev)].contiguous()
    out_layers = []
    n = dims.layers if layers is None else min(int(layers), dims.layers)
    for j in range(n):
        p = f"{LM}layers.{j}."
        q = w(p + "self_attn.q_proj.weight", (dims.hq * hd, h))
        k = w(p + "self_attn.k_proj.weight", (dims.hk * hd, h))
        v = w(p + "self_attn.v_proj.weight", (dims.hk * hd, h))
        gate = w(p + "mlp.gate_proj.weight", (dims.inter, h))
        up = w(p + "mlp.up_proj.weight", (dims.inter, h))
        out_layers.append(dict(
            qkv=torch.cat([q, k, v]), o=w(p + "self_attn.o_proj.weight", (h, dims.hq * hd)),
            gateup=torch.cat([gate, up]), down=w(p + "mlp.down_proj.weight", (h, dims.inter)),
            in_norm=w(p + "input_layernorm.weight", (h,)), post_norm=w(p + "post_attention_layernorm.weight", (h,)),
            q_norm=w(p + "self_attn.q_norm.weight", (hd,)), k_norm=w(p + "self_attn.k_norm.weight", (hd,))))
        del q, k, v, gate, up
    model = dict(embed=embed, head=head, final_norm=w(LM + "norm.weight", (h,)), layers=out_layers)
    return dims, model


VISUAL = "model.visual."


def vision_dims_from_config(config):
    """`VisionDims` of the vision tower described by a Qwen3-VL config.json (dict or path)."""
    from .config import VisionDims
    if not isinstance(config, dict):
        config = json.loads(Path(config).read_text())
    vc = config.get("vision_config")
    if not vc:
        raise CheckpointError("config has no vision_config")
    tc = config.get("text_config", {})
    try:
        return VisionDims(int(vc["hidden_size"]), int(vc["num_heads"]), int(vc["intermediate_size"]),
                          int(vc.get("out_hidden_size", tc.get("hidden_size", 0))), int(vc["depth"]),
                          tuple(int(i) for i in vc.get("deepstack_visual_indexes", ())),
                          int(vc.get("num_position_embeddings", 2304)), int(vc.get("patch_size", 16)),
                          int(vc.get("temporal_patch_size", 2)), int(vc.get("spatial_merge_size", 2)),
                          act=str(vc.get("hidden_act", "gelu_pytorch_tanh")))
    except KeyError as e:
        raise CheckpointError(f"vision config lacks {e}") from None


def vision_param_shapes(v):
    """Checkpoint name (without `model.visual.`) -> shape of every vision-tower tensor."""
    C, I, O, m2 = v.hidden, v.inter, v.out_hidden, v.merge * v.merge
    shapes = {"patch_embed.proj.weight": (C, 3, v.temporal, v.patch, v.patch), "patch_embed.proj.bias": (C,),
              "pos_embed.weight": (v.num_pos, C)}
    for j in range(v.depth):
        b = f"blocks.{j}."
        shapes.update({b + "norm1.weight": (C,), b + "norm1.bias": (C,), b + "norm2.weight": (C,),
                       b + "norm2.bias": (C,), b + "attn.qkv.weight": (3 * C, C), b + "attn.qkv.bias": (3 * C,),
                       b + "attn.proj.weight": (C, C), b + "attn.proj.bias": (C,),
                       b + "mlp.linear_fc1.weight": (I, C), b + "mlp.linear_fc1.bias": (I,),
                       b + "mlp.linear_fc2.weight": (C, I), b + "mlp.linear_fc2.bias": (C,)})
    mergers = [("merger.", C)] + [(f"deepstack_merger_list.{i}.", C * m2) for i in range(len(v.deepstack))]
    for prefix, norm in mergers:
        shapes.update({prefix + "norm.weight": (norm,), prefix + "norm.bias": (norm,),
                       prefix + "linear_fc1.weight": (C * m2, C * m2), prefix + "linear_fc1.bias": (C * m2,),
                       prefix + "linear_fc2.weight": (O, C * m2), prefix + "linear_fc2.bias": (O,)})
    return shapes


def load_vision_tower(model_dir, *, device="cpu", dtype=BF16):
    """(VisionDims, {name: tensor}) of the vision tower in `model_dir`: every tensor under
    `model.visual.` read lazily and checked against the config's shapes (the names are
    the checkpoint's without the prefix)."""
    d = Path(model_dir)
    if not (d / "config.json").exists():
        raise CheckpointError(f"{d} has no config.json")
    v = vision_dims_from_config(d / "config.json")
    t = _Tensors(d)
    params = {}
    for name, shape in vision_param_shapes(v).items():
        x = t.get(VISUAL + name)
        if tuple(x.shape) != tuple(shape):
            raise CheckpointError(f"{VISUAL + name}: shape {tuple(x.shape)}, expected {tuple(shape)}")
        params[name] = x.to(device, dtype).contiguous()
    return v, params


def save_language_model(model_dir, dims, model, *, option_ids=OPTION_IDS, shards=1):
    """Writes `model` (the layout `load_language_model` returns, with every decoder layer)
    as a Hugging Face Qwen3-VL language-model checkpoint: config.json and `shards`
    safetensors files (an index when shards > 1).  The head is stored as a full lm_head
    whose option rows are `model["head"]` (other rows zero) unless dims.tied."""
    from safetensors.torch import save_file
    d = Path(model_dir)
    d.mkdir(parents=True, exist_ok=True)
    h, hd = dims.hidden, dims.d
    tensors = {LM + "embed_tokens.weight": model["embed"], LM + "norm.weight": model["final_norm"]}
    if not dims.tied:
        full = torch.zeros((dims.vocab, h), dtype=BF16)
        full[torch.tensor(option_ids)] = model["head"].cpu()
        tensors["lm_head.weight"] = full
    nq, nk = dims.hq * hd, dims.hk * hd
    for j, lay in enumerate(model["layers"]):
        p = f"{LM}layers.{j}."
        q, k, v = lay["qkv"].split([nq, nk, nk])
        gate, up = lay["gateup"].split([dims.inter, dims.inter])
        tensors.update({p + "self_attn.q_proj.weight": q, p + "self_attn.k_proj.weight": k,
                        p + "self_attn.v_proj.weight": v, p + "self_attn.o_proj.weight": lay["o"],
                        p + "mlp.gate_proj.weight": gate, p + "mlp.up_proj.weight": up,
                        p + "mlp.down_proj.weight": lay["down"], p + "input_layernorm.weight": lay["in_norm"],
                        p + "post_attention_layernorm.weight": lay["post_norm"],
                        p + "self_attn.q_norm.weight": lay["q_norm"], p + "self_attn.k_norm.weight": lay["k_norm"]})
    tensors = {k: v.detach().to("cpu", BF16).contiguous() for k, v in tensors.items()}
    names = sorted(tensors)
    if shards <= 1:
        save_file(tensors, str(d / "model.safetensors"), metadata={"format": "pt"})
    else:
        per = -(-len(names) // shards)
        wm = {}
        for i in range(shards):
            part = names[i * per:(i + 1) * per]
            fname = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
            save_file({k: tensors[k] for k in part}, str(d / fname), metadata={"format": "pt"})
            wm.update({k: fname for k in part})
        (d / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}, indent=1))
    cfg = dict(model_type="qwen3_vl", architectures=["Qwen3VLForConditionalGeneration"],
               tie_word_embeddings=dims.tied,
               text_config=dict(model_type="qwen3_vl_text", hidden_size=h, num_hidden_layers=len(model["layers"]),
                                num_attention_heads=dims.hq, num_key_value_heads=dims.hk, head_dim=hd,
                                intermediate_size=dims.inter, vocab_size=dims.vocab, rms_norm_eps=dims.eps,
                                rope_theta=dims.theta,
                                rope_scaling=dict(rope_type="default", mrope_interleaved=True,
                                                  mrope_section=list(dims.sections)),
                                tie_word_embeddings=dims.tied),
               vision_config=dict(deepstack_visual_indexes=list(range(dims.deepstack))))
    (d / "config.json").write_text(json.dumps(cfg, indent=1))
    return d

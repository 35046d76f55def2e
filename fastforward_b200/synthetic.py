"""Seeded synthetic weights and requests (no checkpoints or datasets exist on this box).

Weights follow the benchmark recipe: every projection and the embedding table are
N(0, 0.02) drawn from `torch.Generator(device).manual_seed(seed)` in a fixed order,
cast to bf16; every RMSNorm weight is 1.0.  Requests: visual embeddings and the three
deepstack tensors N(0, 1), text ids uniform in [0, vocab), bucket padding id 0 (the
reference zero-pads `ids` up to the bucket, `_family/night_runtime.py:122`).
"""
import torch

from .config import OPTION_IDS

BF16 = torch.bfloat16


def _randn(shape, g, device, std):
    return (torch.randn(shape, generator=g, device=device) * std).to(BF16)


def make_layer_bf16(dims, g, device, std=0.02):
    """One decoder layer's bf16 weights in the packed orientation the runtime uses:
    qkv = cat(q, k, v) [(HQ+2HK)*D, H]; o [H, HQ*D]; gateup = cat(gate, up) [2I, H];
    down [H, I] (`_family/depth_runtime.py:99-117` packs the same concatenations)."""
    h, d = dims.hidden, dims.d
    q = _randn((dims.hq * d, h), g, device, std)
    k = _randn((dims.hk * d, h), g, device, std)
    v = _randn((dims.hk * d, h), g, device, std)
    o = _randn((h, dims.hq * d), g, device, std)
    gate = _randn((dims.inter, h), g, device, std)
    up = _randn((dims.inter, h), g, device, std)
    down = _randn((h, dims.inter), g, device, std)
    one = lambda n: torch.ones(n, dtype=BF16, device=device)
    return dict(qkv=torch.cat([q, k, v]), o=o, gateup=torch.cat([gate, up]), down=down,
                in_norm=one(h), post_norm=one(h), q_norm=one(d), k_norm=one(d))


def make_model_bf16(dims, seed=0, device="cpu", layers=None):
    """Full bf16 synthetic model: embed [V, H], head [8, H] (tied rows of embed for the
    2B/4B families), final_norm, and `layers` (default all) decoder layers."""
    g = torch.Generator(device=device).manual_seed(seed)
    embed = _randn((dims.vocab, dims.hidden), g, device, 0.02)
    n_layers = dims.layers if layers is None else layers
    out_layers = [make_layer_bf16(dims, g, device) for _ in range(n_layers)]
    ids = torch.tensor(OPTION_IDS, device=device)
    head = embed[ids].contiguous() if dims.tied else _randn((8, dims.hidden), g, device, 0.02)
    return dict(embed=embed, head=head, final_norm=torch.ones(dims.hidden, dtype=BF16, device=device),
                layers=out_layers)


def make_request(dims, layout, seed=1, device="cpu", deepstack=True):
    """One synthetic request for `layout`: ids [bucket] int64 (zero padded), visual [nv, H],
    deepstack list of 3 x [nv, H] (or []), pick, k."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    bucket = layout.bucket
    n = layout.n_tokens
    ids = torch.zeros(bucket, dtype=torch.long)
    ids[:n] = torch.randint(0, dims.vocab, (n,), generator=g)
    visual = torch.randn((layout.nv, dims.hidden), generator=g).to(BF16)
    deep = [torch.randn((layout.nv, dims.hidden), generator=g).to(BF16)
            for _ in range(dims.deepstack)] if deepstack else []
    return dict(ids=ids.to(device), visual=visual.to(device), deep=[x.to(device) for x in deep],
                pick=layout.pick, k=layout.k, image_start=layout.image_start)


def make_vision_bf16(vdims, seed=0, device="cpu", std=0.02):
    """Seeded bf16 vision-tower parameters by checkpoint name (without `model.visual.`), in
    the order of `checkpoint.vision_param_shapes`: linear and patch-embedding weights,
    biases and the position table N(0, std); LayerNorm weights 1 + N(0, 0.1) and biases
    N(0, std), so that every term of the norms is exercised."""
    from .checkpoint import vision_param_shapes
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shape in vision_param_shapes(vdims).items():
        if name.endswith("norm1.weight") or name.endswith("norm2.weight") or name.endswith("norm.weight"):
            out[name] = (1.0 + torch.randn(shape, generator=g, device=device) * 0.1).to(BF16)
        else:
            out[name] = _randn(shape, g, device, std)
    return out

"""The vision-tower oracle (`oracle/vision.py`) pinned to the code the reference calls: the
transformers Qwen3-VL vision model (fp32, tiny seeded configs, every output: merged rows and
deepstack features) and the reference's own `_vision_rope` Triton kernel (its outputs under
the CPU interpreter, tests/golden/reference_ops.pt).  No GPU."""
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_ops.pt"


def _model(depth, hidden, heads, inter, out_hidden, num_pos, deepstack, seed):
    pytest.importorskip("transformers")
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionModel
    cfg = Qwen3VLVisionConfig(depth=depth, hidden_size=hidden, intermediate_size=inter, num_heads=heads,
                              out_hidden_size=out_hidden, num_position_embeddings=num_pos,
                              deepstack_visual_indexes=list(deepstack), hidden_act="gelu_pytorch_tanh")
    torch.manual_seed(seed)
    m = Qwen3VLVisionModel(cfg).float().eval()
    with torch.no_grad():  # non-trivial norms and biases, so a swapped parameter would show
        for n, p in m.named_parameters():
            if "norm" in n and n.endswith("weight"):
                p.copy_(1 + 0.2 * torch.randn_like(p))
            elif n.endswith("bias"):
                p.copy_(0.1 * torch.randn_like(p))
            elif n == "pos_embed.weight":
                p.copy_(torch.randn_like(p))
    return cfg, m


@pytest.mark.parametrize("case", [
    # depth, hidden, heads, inter, out, G^2, deepstack, canvas (H, W)
    (3, 128, 2, 256, 192, 64, (0, 2), (64, 96)),
    (2, 256, 4, 512, 320, 2304, (1,), (128, 64)),   # the shipped 48 x 48 position table
])
def test_vision_tower_matches_transformers(case):
    depth, hidden, heads, inter, out_hidden, num_pos, deep_idx, (H, W) = case
    cfg, m = _model(depth, hidden, heads, inter, out_hidden, num_pos, deep_idx, seed=depth)
    rgb = np.random.default_rng(H + W).integers(0, 256, (H, W, 3), dtype=np.uint8)
    pixels = oracle.pack_rgb(rgb).float()  # the reference's packed patch rows
    gh, gw = H // 16, W // 16
    with torch.no_grad():
        ref = m(pixels, grid_thw=torch.tensor([[1, gh, gw]]))
        params = {n: p.detach().clone() for n, p in m.named_parameters()}
        dims = oracle.VisionDims.from_config(cfg)
        out, deep = oracle.vision_tower(params, dims, pixels, gh, gw)
    torch.testing.assert_close(out, ref.pooler_output, atol=2e-5, rtol=2e-5)
    assert len(deep) == len(ref.deepstack_features) == len(deep_idx)
    for a, b in zip(deep, ref.deepstack_features):
        torch.testing.assert_close(a, b, atol=2e-5, rtol=2e-5)


def test_vision_geometry_matches_transformers():
    """Position embeddings (bilinear in the table's dtype) from a bf16 table, and the fp32
    rotary tables (the model's inverse frequencies stay fp32 when it is loaded in bf16)."""
    cfg, m = _model(1, 128, 2, 256, 192, 2304, (0,), seed=5)
    m.pos_embed.to(torch.bfloat16)
    for gh, gw in ((16, 16), (8, 20), (32, 12)):
        grid = torch.tensor([[1, gh, gw]])
        want_pos = m.fast_pos_embed_interpolate(grid)
        rot = m.rot_pos_emb(grid).reshape(gh * gw, -1)
        emb = torch.cat([rot, rot], dim=-1)
        pos, cos, sin = oracle.vision_geometry(m.pos_embed.weight.detach(), gh, gw, 128 // 2)
        assert torch.equal(pos, want_pos.detach()), (gh, gw)
        assert torch.equal(cos, emb.cos()) and torch.equal(sin, emb.sin())


def test_vision_rope_matches_reference_kernel():
    c = torch.load(GOLDEN, weights_only=False)["vision_rope"]
    yq, yk = oracle.vision_rope(c["q"], c["k"], c["cos"], c["sin"])
    assert torch.equal(yq.view(torch.int16), c["yq"].view(torch.int16))
    assert torch.equal(yk.view(torch.int16), c["yk"].view(torch.int16))

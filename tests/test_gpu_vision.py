"""The vision tower's kernels on the B200 against the oracle's restatement of their
arithmetic (`oracle.vision` kernel-arithmetic functions): the bf16 tcgen05 linear with each
epilogue, LayerNorm (plain and with the residual add), the vision rotary (also against the
reference's own `vision_rope` output), the non-causal attention, and the whole tower --
patch embedding, blocks, deepstack and final mergers -- bit for bit, eager and through its
CUDA graph.  The module-semantics oracle (`oracle.vision_tower`, pinned to transformers'
vision model) bounds the distance to the reference's fp32 arithmetic."""
from pathlib import Path

import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200 import ops
from fastforward_b200.config import VISION_MODELS, VisionDims
from fastforward_b200.synthetic import make_vision_bf16
from fastforward_b200.vision import VisionTower

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
BF16 = torch.bfloat16
GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_ops.pt"


def _bits_equal(a, b):
    return torch.equal(a.cpu().contiguous().view(torch.int16), b.cpu().contiguous().view(torch.int16))


def _rand(shape, g, std=1.0):
    return (torch.randn(shape, generator=g) * std).to(BF16)


# ---------------------------------------------------------------------------- linear

@pytest.mark.parametrize("epilogue", ["bias", "res", "gelu_tanh", "gelu_erf"])
@pytest.mark.parametrize("m,n,k,tile,splits", [(300, 136, 200, 0, 1), (128, 256, 64, 256, 1), (1, 64, 1536, 64, 1),
                                               (517, 1152, 1152, 128, 1), (256, 4304, 72, 0, 1),
                                               (300, 136, 1000, 64, 3), (1024, 1024, 4096, 128, 2),
                                               (200, 520, 4304, 256, 4), (1024, 1024, 4096, 256, 4),
                                               (256, 2560, 4096, 256, 2), (1, 64, 1536, 256, 2),
                                               (130, 264, 520, 256, 4)])
def test_bf16_linear_bit_exact(epilogue, m, n, k, tile, splits):
    """Every epilogue, ragged M / N / K (zero-filled K tail, clipped stores), each feature
    tile, K splits (last-arriver reduction in split order; 256-wide tiles split 2 or 4 ways
    run as thread-block clusters reducing over distributed shared memory): identical bytes
    to the tensor-core accumulation model + the restated epilogue."""
    g = torch.Generator().manual_seed(m * 7 + n + k)
    x, w = _rand((m, k), g), _rand((n, k), g, k ** -0.5)
    b = _rand((n,), g, 0.5)
    res = _rand((m, n), g) if epilogue == "res" else None
    out = ops.vision_linear(x.to(DEV), w.to(DEV), b.to(DEV), epilogue, res.to(DEV) if res is not None else None,
                            feature_tile=tile, splits=splits)
    torch.cuda.synchronize()
    ref = oracle.linear_k(x, w, b, epilogue, res, splits=splits)
    assert _bits_equal(out, ref), (out.cpu().float() - ref.float()).abs().max()


def test_bf16_linear_residual_in_place_and_no_bias():
    """res may alias out (the blocks' h = h + proj(o)); a NULL bias adds nothing."""
    g = torch.Generator().manual_seed(5)
    x, w, h = _rand((384, 512), g), _rand((1024, 512), g, 0.05), _rand((384, 1024), g)
    hd = h.to(DEV)
    ops.vision_linear(x.to(DEV), w.to(DEV), None, "res", hd, out=hd, splits=1)
    torch.cuda.synchronize()
    assert _bits_equal(hd, oracle.linear_k(x, w, None, "res", h))
    hd = h.to(DEV)
    ops.vision_linear(x.to(DEV), w.to(DEV), None, "res", hd, out=hd, splits=2)
    torch.cuda.synchronize()
    assert _bits_equal(hd, oracle.linear_k(x, w, None, "res", h, splits=2))
    for sp in (2, 4):  # the cluster split-K kernel, in place
        hd = h.to(DEV)
        ops.vision_linear(x.to(DEV), w.to(DEV), None, "res", hd, out=hd, feature_tile=256, splits=sp)
        torch.cuda.synchronize()
        assert _bits_equal(hd, oracle.linear_k(x, w, None, "res", h, splits=sp))


def test_bf16_linear_tile_choice_does_not_change_bytes():
    g = torch.Generator().manual_seed(6)
    x, w, b = _rand((700, 1024), g), _rand((3072, 1024), g, 0.03), _rand((3072,), g)
    outs = [ops.vision_linear(x.to(DEV), w.to(DEV), b.to(DEV), "bias", feature_tile=t, splits=1) for t in (64, 128, 256)]
    torch.cuda.synchronize()
    assert _bits_equal(outs[0], outs[1]) and _bits_equal(outs[0], outs[2])


# ---------------------------------------------------------------------------- row kernels

@pytest.mark.parametrize("rows,c", [(37, 1024), (5, 1152), (64, 4096), (3, 4608), (9, 72)])
def test_layernorm_bit_exact(rows, c):
    g = torch.Generator().manual_seed(rows + c)
    x = (torch.randn(rows, c, generator=g) * 2 + 0.3).to(BF16)
    add = _rand((rows, c), g)
    w, b = (1 + torch.randn(c, generator=g) * 0.1).to(BF16), _rand((c,), g, 0.05)

    class M:
        weight, bias, eps = w.to(DEV), b.to(DEV), 1e-6
    _, y = ops.add_layernorm(x.to(DEV), None, M)
    r, y2 = ops.add_layernorm(x.to(DEV), add.to(DEV), M)
    torch.cuda.synchronize()
    assert _bits_equal(y, oracle.layer_norm_k(x, w, b, 1e-6))
    assert _bits_equal(r, (x.float() + add.float()).to(BF16))
    assert _bits_equal(y2, oracle.layer_norm_k(x, w, b, 1e-6, add=add))


def test_vision_rope_reference_golden():
    """The reference's own `vision_rope` output (its Triton kernel, recorded by
    tests/golden/make_golden.py) reproduced bit for bit."""
    r = torch.load(GOLDEN)["vision_rope"]
    yq, yk = ops.vision_rope(r["q"].to(DEV), r["k"].to(DEV), r["cos"].to(DEV), r["sin"].to(DEV))
    torch.cuda.synchronize()
    assert _bits_equal(yq, r["yq"]) and _bits_equal(yk, r["yk"])


@pytest.mark.parametrize("n_p,heads,d", [(1024, 16, 64), (256, 16, 72), (100, 4, 64)])
def test_vision_rope_heads_layout(n_p, heads, d):
    """qkv rows -> head-major q, k (rotated), v in [H, P, 128]; the padding columns past d
    are not touched (the tower zeroes them once)."""
    from fastforward_b200.vision import rotary_cos_sin
    g = torch.Generator().manual_seed(n_p + d)
    qkv = _rand((n_p, 3 * heads * d), g)
    side = int(n_p ** 0.5) if int(n_p ** 0.5) ** 2 == n_p else None
    gh, gw = (side, side) if side else (10, 10)
    cos, sin = rotary_cos_sin(gh, gw, d)
    out = [torch.full((heads, n_p, 128), 7.0, dtype=BF16, device=DEV) for _ in range(3)]
    qkv_d, cos_d, sin_d = qkv.to(DEV), cos.to(DEV), sin.to(DEV)  # alive until the kernel has run
    L.call("ffb_vision_rope", L.ptr(qkv_d), L.ptr(cos_d), L.ptr(sin_d), n_p, heads, d, 128, *[L.ptr(t) for t in out],
           L.stream_ptr())
    torch.cuda.synchronize()
    ref = oracle.vision._rope_heads(qkv, cos, sin, heads, d)
    for a, b in zip(out, ref):
        assert _bits_equal(a[:, :, :d], b[:, :, :d])
        assert bool((a[:, :, d:] == 7.0).all()), "columns past d are left as they are"


# ---------------------------------------------------------------------------- attention

@pytest.mark.parametrize("t,heads,d", [(1024, 16, 64), (256, 16, 72), (100, 3, 64), (64, 2, 128)])
def test_attention_full_bit_exact(t, heads, d):
    """Non-causal attention over all T keys: bit-identical to the restated kernel arithmetic
    and within bf16 rounding of an fp32 softmax."""
    g = torch.Generator().manual_seed(t + d)
    q, k, v = (torch.zeros(heads, t, 128, dtype=BF16) for _ in range(3))
    for z in (q, k, v):
        z[:, :, :d] = _rand((heads, t, d), g)
    out = ops.vision_attention(q.to(DEV), k.to(DEV), v.to(DEV), d, d ** -0.5)
    torch.cuda.synchronize()
    ref = oracle.attention_full_k(q, k, v, d, d ** -0.5)
    assert _bits_equal(out, ref)
    s = torch.softmax((q[:, :, :d].float() @ k[:, :, :d].float().transpose(1, 2)) * d ** -0.5, dim=-1)
    f32 = (s @ v[:, :, :d].float()).transpose(0, 1).reshape(t, heads * d)
    assert (out.cpu().float() - f32).abs().max().item() < 2e-2


# ---------------------------------------------------------------------------- the tower

def _tower_case(vdims, grid, seed=0):
    p = make_vision_bf16(vdims, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    pixels = (torch.rand(grid[0] * grid[1], 1536, generator=g) * 2 - 1).to(BF16)
    return p, pixels


def _splits(vt, grid):
    return {sh: sp for sh, (_, sp, _) in vt.bufs[grid[0] * grid[1]].plans.items()}


def _check_tower(vt, p, vdims, pixels, grid, graph):
    run = vt.replay if graph else vt.forward
    merged, deep = run(pixels.to(DEV), *grid)
    torch.cuda.synchronize()
    merged, deep = merged.cpu().clone(), [d.cpu().clone() for d in deep]
    rm, rd = oracle.vision_tower_k(p, vdims, pixels, *grid, splits=_splits(vt, grid))
    assert len(deep) == len(rd) == len(vdims.deepstack)
    assert _bits_equal(merged, rm), (merged.float() - rm.float()).abs().max()
    for a, b in zip(deep, rd):
        assert _bits_equal(a, b), (a.float() - b.float()).abs().max()
    return merged, deep


@pytest.mark.parametrize("name", ["4B", "8B"])
def test_vision_tower_two_blocks_bit_exact(name):
    """The real families' widths (head dim 64 for 2B/4B, 72 for 8B/32B) at two blocks, both
    deepstack mergers on, a 16 x 24 patch grid: eager and graph replay equal the kernel
    arithmetic bit for bit, and stay close to the fp32 module semantics."""
    v0 = VISION_MODELS[name]
    v = VisionDims(v0.hidden, v0.heads, v0.inter, v0.out_hidden, 2, (0, 1))
    p, pixels = _tower_case(v, (16, 24))
    vt = VisionTower(v, p, device=DEV)
    m_eager, _ = _check_tower(vt, p, v, pixels, (16, 24), graph=False)
    m_graph, _ = _check_tower(vt, p, v, pixels, (16, 24), graph=True)
    assert _bits_equal(m_eager, m_graph)
    mf, _ = oracle.vision_tower({k: t.float() for k, t in p.items()}, v, pixels.float(), 16, 24)
    assert (m_graph.float() - mf).abs().max().item() <= 0.03 * mf.abs().max().item()


@pytest.mark.parametrize("grid", [(4, 4), (2, 8), (6, 2)])
def test_vision_tower_tiny_canvases(grid):
    """Canvases of a few patches (16, 16 and 12 patch rows: 4, 4 and 3 merged rows): every
    kernel runs with far fewer rows than one 128-row tile, bit-identical to the oracle."""
    v = VisionDims(1024, 16, 4096, 2560, 2, (0, 1))
    p, pixels = _tower_case(v, grid, seed=11)
    vt = VisionTower(v, p, device=DEV)
    _check_tower(vt, p, v, pixels, grid, graph=True)


def test_vision_tower_full_depth_4b_bit_exact():
    """The 4B vision tower at full depth (24 blocks, deepstack at 5 / 11 / 17) on the
    benchmarked 32 x 32 patch grid (a 512 x 512 canvas, 256 merged rows), through the CUDA
    graph: bit-identical to the oracle's kernel arithmetic."""
    v = VISION_MODELS["4B"]
    p, pixels = _tower_case(v, (32, 32), seed=4)
    vt = VisionTower(v, p, device=DEV)
    merged, deep = _check_tower(vt, p, v, pixels, (32, 32), graph=True)
    assert merged.shape == (256, v.out_hidden) and all(d.shape == (256, v.out_hidden) for d in deep)
    assert torch.isfinite(merged.float()).all()


def test_vision_tower_encodes_a_canvas():
    """uint8 canvas -> ffb_pack_rgb -> tower graph: equals the tower on the oracle's packed
    patch rows."""
    v = VisionDims(1024, 16, 4096, 2560, 1, (0,))
    p = make_vision_bf16(v, seed=9)
    g = torch.Generator().manual_seed(10)
    rgb = torch.randint(0, 256, (256, 384, 3), generator=g, dtype=torch.uint8)
    vt = VisionTower(v, p, device=DEV)
    merged, deep = vt.encode(rgb.to(DEV))
    torch.cuda.synchronize()
    rm, rd = oracle.vision_tower_k(p, v, oracle.pack_rgb(rgb), 16, 24, splits=_splits(vt, (16, 24)))
    assert _bits_equal(merged, rm) and _bits_equal(deep[0], rd[0])


# ---------------------------------------------------------------------------- predict

def test_predict_runs_the_vision_tower_end_to_end(tmp_path):
    """`Accelerator.predict(canvas, question, choices)` on a synthetic bundle with the
    vision tower on: canvas -> ffb_pack_rgb -> the tower's graph -> the language prefill +
    scoring graph.  The logits equal, bit for bit, the oracle's vision tower (kernel
    arithmetic) feeding the oracle's language path on the same ids."""
    import json
    import numpy as np
    from dataclasses import replace
    from fastforward_b200.api import Accelerator
    from fastforward_b200.config import MODELS
    from fastforward_b200.mrope import position_ids
    from fastforward_b200.synthetic import make_model_bf16
    g = torch.Generator().manual_seed(21)
    rgb = torch.randint(0, 256, (256, 256, 3), generator=g, dtype=torch.uint8)
    img = tmp_path / "canvas.npy"
    np.save(img, rgb.numpy())
    syn = dict(model="2B", layers=2, seed=3, vision=dict(seed=5, depth=3),
               layout=dict(image_start=4, grid_h=16, grid_w=16, n_text=32))
    bundle = tmp_path / "bundle.json"
    bundle.write_text(json.dumps(dict(schema_version=1, task="visual_choice", architecture="qwen3_vl_family",
                                      synthetic=syn)))
    acc = Accelerator(bundle)
    cands = ["cat", "dog", "bird", "fish"]
    out = acc.predict(img, "What is shown?", cands)
    r = acc.encoder(str(img), "What is shown?", cands)
    assert r.visual.shape == (64, 2048) and len(r.deep) == 3 and r.image_start == 4

    v = acc.vision.v
    p = make_vision_bf16(v, seed=5, device=DEV)
    p = {k: t.cpu() for k, t in p.items()}
    merged, deep = oracle.vision_tower_k(p, v, oracle.pack_rgb(rgb), 16, 16, splits=_splits(acc.vision, (16, 16)))
    assert _bits_equal(r.visual, merged) and all(_bits_equal(a, b) for a, b in zip(r.deep, deep))
    dims = MODELS["2B"]
    src = make_model_bf16(dims, seed=3, device=DEV, layers=2)
    src = {k: ([{n: t.cpu() for n, t in lay.items()} for lay in src[k]] if k == "layers" else src[k].cpu())
           for k in src}
    T = next(b for b in acc.buckets if b >= r.ids.shape[0])
    splits = {k: pl.splits for k, pl in acc.engine.plans[T].items()}
    om = oracle.quantized_model(dims, src, "rowwise", splits=splits)
    ids = torch.zeros(T, dtype=torch.long)
    ids[:r.ids.shape[0]] = r.ids
    pos = position_ids(T, r.image_start, 16, 16)
    zr, _ = oracle.prefill_score(om, ids, merged, deep, pos, r.ids.shape[0] - 1, 4, image_start=r.image_start)
    assert torch.equal(torch.tensor(out["logits"], dtype=torch.float32).view(torch.int32), zr.view(torch.int32)), \
        (out["logits"], zr)
    assert out["answer"]["text"] == cands[int(torch.argmax(zr))]

"""CPU oracle for the Qwen3-VL vision tower in front of the language path (TEST
INFRASTRUCTURE: only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU legs use it).

Restates what the reference runs for a still image (`scaled_qwen_runtime.py:42-55`,
`NativeNormVision.core`; geometry from `_legacy/vision_graph_runtime.py:11-15`):

    h = patch_embed(pixels) + pos                  patch rows [P, 1536] -> [P, C]
    per block j:
        x = LayerNorm1(h); q, k, v = split(x W_qkv^T + b_qkv) into heads of d = C / heads
        q, k = vision_rope(q, k, cos, sin)         `_legacy/search_kernels.py:111-125`
        h = h + proj(softmax(q k^T / sqrt(d)) v)   non-causal, over the image's P patches
        h = h + fc2(gelu_tanh(fc1(LayerNorm2(h))))
        deepstack block j: deep += merger_j(h)     (post-shuffle LayerNorm over 4C)
    out = merger(h)                                LayerNorm over C, then 4 patches -> one row

The geometry is restated from the published algorithm of the transformers Qwen3-VL vision
model (transformers 5.5.0 here; the reference pins 4.57.1), which the reference calls
(`fast_pos_embed_interpolate`, `rot_pos_emb`):
  * position embedding: a G x G table (G^2 = num_position_embeddings) sampled bilinearly at
    linspace(0, G-1, h) x linspace(0, G-1, w), then put in 2x2 merge-group order;
  * rotary: per patch (row, col) in merge-group order, angle tables row * f and col * f with
    f = theta^(-2i/(d/2)), i < d/4, theta 1e4; cos/sin of cat(row part, col part) twice.

The patch rows are those of `oracle.pack_rgb` (channel-major 3 x 2 x 16 x 16 per patch),
which is the layout the patch embedding's Conv3d weight flattens to.  Parameters are a dict
with the checkpoint names under `model.visual.` (see `vision_params_from_state_dict`).
"""
import math

import torch

__all__ = ["vision_geometry", "vision_pos_embed", "vision_rot_cos_sin", "vision_rope", "vision_tower",
           "vision_params_from_state_dict", "VisionDims", "layer_norm_k", "linear_k", "attention_full_k",
           "vision_tower_k"]


class VisionDims:
    """Shape of a vision tower (the fields the forward needs)."""

    def __init__(self, hidden, heads, inter, out_hidden, depth, deepstack, num_pos, patch=16, temporal=2,
                 merge=2, eps=1e-6, theta=10000.0, act="gelu_pytorch_tanh"):
        self.hidden, self.heads, self.inter, self.out_hidden = hidden, heads, inter, out_hidden
        self.depth, self.deepstack, self.num_pos = depth, tuple(deepstack), num_pos
        self.patch, self.temporal, self.merge, self.eps, self.theta = patch, temporal, merge, eps, theta
        if act not in ("gelu_pytorch_tanh", "gelu"):
            raise ValueError(f"unsupported vision activation {act!r}")
        self.act = act

    @property
    def head_dim(self):
        return self.hidden // self.heads

    @classmethod
    def from_config(cls, vc):
        """From a transformers vision config (object or dict)."""
        g = (lambda k, d=None: vc.get(k, d)) if isinstance(vc, dict) else (lambda k, d=None: getattr(vc, k, d))
        return cls(g("hidden_size"), g("num_heads"), g("intermediate_size"), g("out_hidden_size"), g("depth"),
                   g("deepstack_visual_indexes", ()), g("num_position_embeddings"), g("patch_size", 16),
                   g("temporal_patch_size", 2), g("spatial_merge_size", 2), act=g("hidden_act", "gelu_pytorch_tanh"))


def _merge_order(grid_h, grid_w, merge=2):
    """(row, col) of every patch in the order the patch rows come: merge groups row-major,
    each group's patches row-major."""
    rows, cols = [], []
    for gy in range(grid_h // merge):
        for gx in range(grid_w // merge):
            for my in range(merge):
                for mx in range(merge):
                    rows.append(gy * merge + my)
                    cols.append(gx * merge + mx)
    return torch.tensor(rows), torch.tensor(cols)


def vision_pos_embed(table, grid_h, grid_w, merge=2):
    """Bilinear sample of the [G*G, C] position table at the h x w patch grid, in merge
    order; computed in the table's dtype as the model does (weights cast to it, four
    weighted rows summed in corner order)."""
    G = int(round(math.sqrt(table.shape[0])))
    assert G * G == table.shape[0]
    hs = torch.linspace(0, G - 1, grid_h)
    ws = torch.linspace(0, G - 1, grid_w)
    h0, w0 = hs.int(), ws.int()
    h1, w1 = (h0 + 1).clamp(max=G - 1), (w0 + 1).clamp(max=G - 1)
    dh, dw = hs - h0, ws - w0
    corners = [(h0, w0, (1 - dh)[:, None] * (1 - dw)[None, :]), (h0, w1, (1 - dh)[:, None] * dw[None, :]),
               (h1, w0, dh[:, None] * (1 - dw)[None, :]), (h1, w1, dh[:, None] * dw[None, :])]
    total = None
    for hi, wi, wt in corners:
        idx = (hi[:, None] * G + wi[None, :]).reshape(-1)
        term = table[idx] * wt.reshape(-1, 1).to(table.dtype)
        total = term if total is None else total + term
    rows, cols = _merge_order(grid_h, grid_w, merge)
    return total[rows * grid_w + cols]


def vision_rot_cos_sin(grid_h, grid_w, head_dim, theta=10000.0, merge=2):
    """cos, sin [P, head_dim] fp32 of the 2D rotary embedding, patches in merge order."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, 2, dtype=torch.float32) / half))
    rows, cols = _merge_order(grid_h, grid_w, merge)
    table = torch.outer(torch.arange(max(grid_h, grid_w), dtype=torch.float32), inv)
    emb = torch.cat([table[rows], table[cols]], dim=-1)
    emb = torch.cat([emb, emb], dim=-1)
    return emb.cos(), emb.sin()


def vision_geometry(table, grid_h, grid_w, head_dim, theta=10000.0, merge=2):
    """(pos [P, C], cos, sin) of one image geometry (`vision_graph_runtime.py:11-15`)."""
    return (vision_pos_embed(table, grid_h, grid_w, merge),) + vision_rot_cos_sin(grid_h, grid_w, head_dim, theta,
                                                                                  merge)


def vision_rope(q, k, cos, sin):
    """The reference's `_vision_rope` (`_legacy/search_kernels.py:111-125`): q, k [P, H, d]
    (any float dtype), cos/sin [P, d] fp32.  y[c] = x[c]*cos[c] + r[c]*sin[c] with
    r = (-x[c + d/2] for c < d/2, x[c - d/2] otherwise), each product and the sum rounded
    to fp32 separately (no fused multiply-add), stored in the input's dtype (round to
    nearest even)."""
    d = q.shape[-1]
    out = []
    for x in (q, k):
        xf = x.float()
        rot = torch.cat([-xf[..., d // 2:], xf[..., :d // 2]], dim=-1)
        c, s = cos.float()[:, None, :], sin.float()[:, None, :]
        y = (xf * c) + (rot * s)
        out.append(y.to(x.dtype))
    return out[0], out[1]


def _ln(x, w, b, eps):
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


def _act(x, dims):
    """The blocks' MLP activation: tanh-approximated GELU for the shipped configs."""
    return torch.nn.functional.gelu(x, approximate="tanh" if dims.act == "gelu_pytorch_tanh" else "none")


def _merger(p, prefix, h, dims, post_shuffle):
    C4 = dims.hidden * dims.merge * dims.merge
    if post_shuffle:
        x = _ln(h.reshape(-1, C4), p[prefix + "norm.weight"], p[prefix + "norm.bias"], dims.eps)
    else:
        x = _ln(h, p[prefix + "norm.weight"], p[prefix + "norm.bias"], dims.eps).reshape(-1, C4)
    x = torch.nn.functional.linear(x, p[prefix + "linear_fc1.weight"], p[prefix + "linear_fc1.bias"])
    x = torch.nn.functional.gelu(x)  # exact (erf) GELU in the mergers
    return torch.nn.functional.linear(x, p[prefix + "linear_fc2.weight"], p[prefix + "linear_fc2.bias"])


def vision_tower(p, dims, pixels, grid_h, grid_w, dtype=torch.float32):
    """(merged [P/4, out_hidden], [deepstack features]) of one still image.

    p: parameters by checkpoint name without the `model.visual.` prefix; pixels [P, 1536]
    patch rows (oracle.pack_rgb); grid_h, grid_w: patch grid (canvas / 16).  Everything
    runs in `dtype` (fp32 for the pinning tests)."""
    p = {k: v.to(dtype) for k, v in p.items()}
    P = grid_h * grid_w
    assert pixels.shape == (P, 3 * dims.temporal * dims.patch * dims.patch)
    w_pe = p["patch_embed.proj.weight"].reshape(dims.hidden, -1)
    h = torch.nn.functional.linear(pixels.to(dtype), w_pe, p["patch_embed.proj.bias"])
    pos, cos, sin = vision_geometry(p["pos_embed.weight"], grid_h, grid_w, dims.head_dim, dims.theta, dims.merge)
    h = h + pos
    H, d = dims.heads, dims.head_dim
    deep = []
    for j in range(dims.depth):
        b = f"blocks.{j}."
        x = _ln(h, p[b + "norm1.weight"], p[b + "norm1.bias"], dims.eps)
        qkv = torch.nn.functional.linear(x, p[b + "attn.qkv.weight"], p[b + "attn.qkv.bias"]).reshape(P, 3, H, d)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        q, k = vision_rope(q, k, cos, sin)
        att = torch.softmax((q.transpose(0, 1) @ k.transpose(0, 1).transpose(1, 2)) * (d ** -0.5), dim=-1)
        o = (att @ v.transpose(0, 1)).transpose(0, 1).reshape(P, H * d)
        h = h + torch.nn.functional.linear(o, p[b + "attn.proj.weight"], p[b + "attn.proj.bias"])
        x = _ln(h, p[b + "norm2.weight"], p[b + "norm2.bias"], dims.eps)
        x = _act(torch.nn.functional.linear(x, p[b + "mlp.linear_fc1.weight"], p[b + "mlp.linear_fc1.bias"]), dims)
        h = h + torch.nn.functional.linear(x, p[b + "mlp.linear_fc2.weight"], p[b + "mlp.linear_fc2.bias"])
        if j in dims.deepstack:
            i = dims.deepstack.index(j)
            deep.append(_merger(p, f"deepstack_merger_list.{i}.", h, dims, post_shuffle=True))
    return _merger(p, "merger.", h, dims, post_shuffle=False), deep


def vision_params_from_state_dict(sd, prefix="model.visual."):
    """The vision tower's parameters out of a full-model state dict (checkpoint names)."""
    return {k[len(prefix):]: v for k, v in sd.items() if k.startswith(prefix)}


# ----------------------------------------------------------------------------- kernel arithmetic
# The same forward with the rounding points and operation orders of the CUDA kernels
# (fastforward_b200/csrc/gemm_bf16.cu, vision.cu, attention_tc.cu), for bit-exact checks of
# the GPU path: every linear accumulates as the tensor core does (`_tc.acc_bf16`, kind::f16)
# and rounds its bf16 output once after the bias add; the residual adds, LayerNorms and GELUs
# are the kernels' own (below); the attention is the language path's kernel arithmetic with
# every key visible.  It differs from `vision_tower` (the HF modules' semantics) only by
# rounding.

def layer_norm_k(x, w, b, eps, add=None):
    """LayerNorm of the kernel `ffb_layernorm`: float64 sums S1 = sum x, S2 = sum x^2;
    mean = fp32(S1 / C), rstd = fp32(1 / sqrt(max(S2 / C - (S1 / C)^2, 0) + eps)) in float64;
    y = bf16(((x - mean) * rstd) * w + b) in fp32 operations.  x [R, C] bf16.  With `add`
    (`ffb_add_layernorm`, the reference's `add_layernorm`, `_legacy/lower_kernels.py:115-136`)
    the row is x = bf16(x + add) first."""
    if add is not None:
        x = (x.float() + add.float()).to(torch.bfloat16)
    xf = x.float()
    xd = xf.double()
    c = x.shape[-1]
    mean_d = xd.sum(-1) / c
    var_d = ((xd * xd).sum(-1) / c - mean_d * mean_d).clamp(min=0.0)
    mean = mean_d.float()
    eps_d = float(torch.tensor(eps, dtype=torch.float32))
    rstd = (1.0 / torch.sqrt(var_d + eps_d)).float()
    y = ((xf - mean[:, None]) * rstd[:, None]) * w.float() + b.float()
    return y.to(torch.bfloat16)


def linear_k(x, w, b, epilogue="bias", res=None, splits=1):
    """The bf16 linear `ffb_bf16_gemm`: v = fp32(acc + b) with acc the tensor core's fp32
    accumulator of x [M, K] . w [N, K]^T -- with a K split, the splits' accumulators over
    their ranges of 64-element K blocks summed in split order -- ; epilogue "bias": bf16(v);
    "res": bf16(res + bf16(v)); "gelu_tanh" / "gelu_erf": bf16(gelu(bf16(v))) with the
    kernel's GELU (oracle/act.c).  bf16 in, bf16 out."""
    from . import _tc
    k = x.shape[1]
    nkb = -(-k // 64)
    acc = None
    for j in range(splits):
        k0, k1 = j * nkb // splits * 64, min((j + 1) * nkb // splits * 64, k)
        part = _tc.acc_bf16(x, w, k0, k1)
        acc = part if acc is None else acc + part
    v = acc + (b.float() if b is not None else 0.0)
    if epilogue == "bias":
        y = v
    elif epilogue == "res":
        y = res.float() + v.to(torch.bfloat16).float()
    elif epilogue in ("gelu_tanh", "gelu_erf"):
        y = _tc.gelu(v.to(torch.bfloat16).float(), epilogue[5:])
    else:
        raise ValueError(epilogue)
    return y.to(torch.bfloat16)


def attention_full_k(q, k, v, d, scale):
    """Non-causal attention of `ffb_attention_full`: q, k, v [H, T, 128] bf16 (head dim d
    zero-padded to 128); returns [T, H * d] bf16."""
    from .qwen_path import attention_tc
    h, t, _ = q.shape
    out = attention_tc(q, k, v, scale, positions=torch.full((t,), t - 1, dtype=torch.long))
    return out[:, :, :d].reshape(t, h * d)


def _rope_heads(qkv, cos, sin, heads, d, dp=128):
    """Rotary on q, k of qkv [P, 3 H d] and the head-major zero-padded layout [H, P, dp]
    (`ffb_vision_rope`)."""
    p_n = qkv.shape[0]
    x = qkv.reshape(p_n, 3, heads, d)
    q, k = vision_rope(x[:, 0], x[:, 1], cos, sin)
    out = []
    for t in (q, k, x[:, 2]):
        z = torch.zeros(heads, p_n, dp, dtype=torch.bfloat16)
        z[:, :, :d] = t.transpose(0, 1)
        out.append(z)
    return out


def _merger_k(p, prefix, h, dims, post_shuffle, sp):
    c4 = dims.hidden * dims.merge * dims.merge
    if post_shuffle:
        x = layer_norm_k(h.reshape(-1, c4), p[prefix + "norm.weight"], p[prefix + "norm.bias"], dims.eps)
    else:
        x = layer_norm_k(h, p[prefix + "norm.weight"], p[prefix + "norm.bias"], dims.eps).reshape(-1, c4)
    w1, w2 = p[prefix + "linear_fc1.weight"], p[prefix + "linear_fc2.weight"]
    x = linear_k(x, w1, p[prefix + "linear_fc1.bias"], "gelu_erf", splits=sp(x, w1))
    return linear_k(x, w2, p[prefix + "linear_fc2.bias"], splits=sp(x, w2))


def vision_tower_k(p, dims, pixels, grid_h, grid_w, splits=None):
    """`vision_tower` with the CUDA kernels' arithmetic (bf16 activations between kernels).
    p: bf16 parameters by checkpoint name (without `model.visual.`); pixels [P, 1536] bf16;
    splits: {(M, N, K): K splits} of the linears (the GPU's plans; default none split).
    Returns (merged [P/4, out_hidden], [deepstack features]) bf16."""
    p = {k: v.to(torch.bfloat16) for k, v in p.items()}
    plan = splits or {}

    def sp(x, w):
        return plan.get((x.shape[0], w.shape[0], x.shape[1]), 1)
    n_p = grid_h * grid_w
    heads, d = dims.heads, dims.head_dim
    pos, cos, sin = vision_geometry(p["pos_embed.weight"], grid_h, grid_w, d, dims.theta, dims.merge)
    act = "gelu_tanh" if dims.act == "gelu_pytorch_tanh" else "gelu_erf"
    pixels = pixels.to(torch.bfloat16)
    w_pe = p["patch_embed.proj.weight"].reshape(dims.hidden, -1)
    h = linear_k(pixels, w_pe, p["patch_embed.proj.bias"], "res", pos, splits=sp(pixels, w_pe))
    deep = []
    for j in range(dims.depth):
        b = f"blocks.{j}."
        x = layer_norm_k(h, p[b + "norm1.weight"], p[b + "norm1.bias"], dims.eps)
        w = p[b + "attn.qkv.weight"]
        qkv = linear_k(x, w, p[b + "attn.qkv.bias"], splits=sp(x, w))
        q, k, v = _rope_heads(qkv, cos, sin, heads, d)
        o = attention_full_k(q, k, v, d, d ** -0.5)
        w = p[b + "attn.proj.weight"]
        h = linear_k(o, w, p[b + "attn.proj.bias"], "res", h, splits=sp(o, w))
        x = layer_norm_k(h, p[b + "norm2.weight"], p[b + "norm2.bias"], dims.eps)
        w = p[b + "mlp.linear_fc1.weight"]
        x = linear_k(x, w, p[b + "mlp.linear_fc1.bias"], act, splits=sp(x, w))
        w = p[b + "mlp.linear_fc2.weight"]
        h = linear_k(x, w, p[b + "mlp.linear_fc2.bias"], "res", h, splits=sp(x, w))
        if j in dims.deepstack:
            i = dims.deepstack.index(j)
            deep.append(_merger_k(p, f"deepstack_merger_list.{i}.", h, dims, True, sp))
    return _merger_k(p, "merger.", h, dims, False, sp), deep

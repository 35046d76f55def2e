"""The Qwen3-VL vision tower on the B200: patch embedding, ViT blocks, deepstack and final
mergers, every step a libffb200 kernel (bf16 tcgen05 linears with fused bias / residual /
GELU epilogues, LayerNorm, the 2-D vision rotary, non-causal tcgen05 attention), replayed
as one CUDA graph per image geometry.

It replaces the reference's vision wrappers (`_legacy/vision_graph_runtime.py:16-27`,
`VisionGraph.core`, and `scaled_qwen_runtime.py:42-55`, `NativeNormVision.core`): HF
modules + SDPA + the Triton vision RoPE, captured per geometry.  Per block:

    x = LayerNorm1(h); qkv = x W_qkv^T + b            ffb_layernorm, ffb_bf16_gemm
    q, k = rope(q, k) (head-major, d padded to 128)    ffb_vision_rope
    o = softmax(q k^T / sqrt(d)) v  (all patches)      ffb_attention_full
    h = h + o W_proj^T + b                              ffb_bf16_gemm (residual epilogue)
    h = h + gelu_tanh(LayerNorm2(h) W1^T + b1) W2^T + b2   two ffb_bf16_gemm, GELU / residual
    deepstack block j: LayerNorm over 4C of 2x2 patch groups -> fc1 + GELU(erf) -> fc2

then the final merger (LayerNorm over C per patch, 2x2 groups, fc1 + GELU, fc2).  The
geometry (bilinearly sampled position table in merge-group order, rotary cos / sin) is
computed once per (grid_h, grid_w) on the host, as the reference caches it per grid
(`VisionGraph.geo`), and the position add rides the patch embedding's residual epilogue.
"""
import math
import threading

import torch

from . import _lib as L
from ._lib import call, ptr, stream_ptr

BF16 = torch.bfloat16
HEAD_PAD = 128  # the attention kernel's head dimension; d < 128 is zero-padded


# ---------------------------------------------------------------------------- geometry

def merge_order(grid_h, grid_w, merge=2):
    """(row, col) of each patch in the order the patch rows come: 2x2 merge groups row-major,
    the group's patches row-major inside it (the order `ffb_pack_rgb` writes)."""
    gy = torch.arange(grid_h // merge).repeat_interleave(grid_w // merge)
    gx = torch.arange(grid_w // merge).repeat(grid_h // merge)
    my = torch.arange(merge).repeat_interleave(merge)
    mx = torch.arange(merge).repeat(merge)
    rows = (gy[:, None] * merge + my[None, :]).reshape(-1)
    cols = (gx[:, None] * merge + mx[None, :]).reshape(-1)
    return rows, cols


def position_table(table, grid_h, grid_w, merge=2):
    """[P, C] position embedding of a grid_h x grid_w patch grid, in merge order: the G x G
    learned table sampled bilinearly at linspace(0, G - 1, n) along each axis, in the
    table's dtype (corner weights cast to it, the four corner terms added in the order
    (h0,w0), (h0,w1), (h1,w0), (h1,w1)) -- the arithmetic of transformers'
    `fast_pos_embed_interpolate`, which the reference calls."""
    g = int(round(math.sqrt(table.shape[0])))
    if g * g != table.shape[0]:
        raise ValueError(f"position table of {table.shape[0]} rows is not square")
    ys = torch.linspace(0, g - 1, grid_h)
    xs = torch.linspace(0, g - 1, grid_w)
    y0, x0 = ys.int(), xs.int()
    y1, x1 = (y0 + 1).clamp(max=g - 1), (x0 + 1).clamp(max=g - 1)
    fy, fx = ys - y0, xs - x0
    acc = None
    for yi, xi, wy, wx in ((y0, x0, 1 - fy, 1 - fx), (y0, x1, 1 - fy, fx), (y1, x0, fy, 1 - fx), (y1, x1, fy, fx)):
        idx = (yi[:, None] * g + xi[None, :]).reshape(-1)
        wt = (wy[:, None] * wx[None, :]).reshape(-1, 1).to(table.dtype)
        term = table[idx] * wt
        acc = term if acc is None else acc + term
    rows, cols = merge_order(grid_h, grid_w, merge)
    return acc[rows * grid_w + cols].contiguous()


def rotary_cos_sin(grid_h, grid_w, head_dim, theta=10000.0, merge=2):
    """cos, sin [P, head_dim] fp32 of the 2-D rotary, patches in merge order: frequencies
    theta^(-2i / (d/2)) for i < d/4; angles (row f, col f) concatenated, then repeated
    (transformers' `rot_pos_emb` + cat(emb, emb), as `VisionGraph.geo` builds them)."""
    half = head_dim // 2
    freq = 1.0 / (theta ** (torch.arange(0, half, 2, dtype=torch.float32) / half))
    rows, cols = merge_order(grid_h, grid_w, merge)
    ang = torch.outer(torch.arange(max(grid_h, grid_w), dtype=torch.float32), freq)
    emb = torch.cat([ang[rows], ang[cols]], dim=-1)
    emb = torch.cat([emb, emb], dim=-1)
    return emb.cos().contiguous(), emb.sin().contiguous()


# ---------------------------------------------------------------------------- the tower

class _Buffers:
    def __init__(self, v, n_p, device):
        c, m2 = v.hidden, v.merge * v.merge
        z = lambda *s: torch.zeros(s, dtype=BF16, device=device)
        self.pixels = z(n_p, 3 * v.temporal * v.patch * v.patch)
        self.h, self.x, self.o = z(n_p, c), z(n_p, c), z(n_p, c)
        self.qkv = z(n_p, 3 * c)
        self.q, self.k, self.v = (z(v.heads, n_p, HEAD_PAD) for _ in range(3))
        self.f = z(n_p, v.inter)
        self.mln = z(n_p // m2, c * m2)
        self.mfc = z(n_p // m2, c * m2)
        self.merged = z(n_p // m2, v.out_hidden)
        self.deep = [z(n_p // m2, v.out_hidden) for _ in v.deepstack]
        # the linears' plans (feature tile, K splits, counters) and one split-K scratch for the
        # plans that reduce through fp32 planes (they run one after another on the stream; each
        # leaves its counters zero); the cluster split-K plans (counters 0) need none
        g = n_p // m2
        shapes = [(n_p, c, 3 * v.temporal * v.patch * v.patch), (n_p, 3 * c, c), (n_p, c, c), (n_p, v.inter, c),
                  (n_p, c, v.inter), (g, c * m2, c * m2), (g, v.out_hidden, c * m2)]
        self.plans = {sh: L.bf16_gemm_plan(*sh) for sh in shapes}
        ws = max((sp * m * n for (m, n, _), (_, sp, c_n) in self.plans.items() if sp > 1 and c_n > 0), default=4)
        cnt = max((c_n for (_, sp, c_n) in self.plans.values() if sp > 1), default=1)
        cnt = max(cnt, 1)
        self.ws = torch.zeros(ws, dtype=torch.float32, device=device)
        self.counters = torch.zeros(cnt, dtype=torch.int32, device=device)


class VisionTower:
    """One model's vision tower on one device.  `params`: tensors by checkpoint name without
    the `model.visual.` prefix (`checkpoint.load_vision_tower`, or seeded synthetic ones);
    kept on the device as bf16.  Calls are serialised by a lock; buffers, geometry and
    graphs are cached per image geometry."""

    def __init__(self, vdims, params, device=None):
        L.require_cuda()
        self.v = v = vdims
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        d = v.head_dim
        if v.hidden % v.heads or d % 8 or d > HEAD_PAD:
            raise ValueError(f"head dim {d} unsupported (a multiple of 8, at most {HEAD_PAD})")
        if v.hidden % 8 or v.inter % 8 or v.out_hidden % 8:
            raise ValueError("hidden, intermediate and output sizes must be multiples of 8")
        if v.act not in ("gelu_pytorch_tanh", "gelu"):
            raise ValueError(f"unsupported vision activation {v.act!r}")
        self.act = "gelu_tanh" if v.act == "gelu_pytorch_tanh" else "gelu_erf"
        dev = self.device

        def w(name):
            if name not in params:
                raise KeyError(f"vision parameter {name!r} missing")
            return params[name].to(device=dev, dtype=BF16).contiguous()

        self.patch_w = w("patch_embed.proj.weight").reshape(v.hidden, -1).contiguous()
        self.patch_b = w("patch_embed.proj.bias")
        self.pos_table = params["pos_embed.weight"].detach().to("cpu", BF16)
        self.blocks = []
        for j in range(v.depth):
            b = f"blocks.{j}."
            self.blocks.append({k: w(b + n) for k, n in (
                ("n1w", "norm1.weight"), ("n1b", "norm1.bias"), ("qkv_w", "attn.qkv.weight"), ("qkv_b", "attn.qkv.bias"),
                ("proj_w", "attn.proj.weight"), ("proj_b", "attn.proj.bias"), ("n2w", "norm2.weight"),
                ("n2b", "norm2.bias"), ("fc1_w", "mlp.linear_fc1.weight"), ("fc1_b", "mlp.linear_fc1.bias"),
                ("fc2_w", "mlp.linear_fc2.weight"), ("fc2_b", "mlp.linear_fc2.bias"))})

        def merger(prefix):
            return {k: w(prefix + n) for k, n in (("nw", "norm.weight"), ("nb", "norm.bias"),
                                                  ("fc1_w", "linear_fc1.weight"), ("fc1_b", "linear_fc1.bias"),
                                                  ("fc2_w", "linear_fc2.weight"), ("fc2_b", "linear_fc2.bias"))}
        self.merger = merger("merger.")
        self.deep_mergers = [merger(f"deepstack_merger_list.{i}.") for i in range(len(v.deepstack))]
        self.lock = threading.RLock()
        self.geoms, self.bufs, self.graphs = {}, {}, {}

    # ------------------------------------------------------------------ caches
    def geometry(self, grid_h, grid_w):
        """(pos [P, C] bf16, cos, sin [P, d] fp32) on the device, cached per grid."""
        key = (grid_h, grid_w)
        if key not in self.geoms:
            m = self.v.merge
            if grid_h % m or grid_w % m or grid_h <= 0 or grid_w <= 0:
                raise ValueError(f"patch grid {grid_h}x{grid_w} must be positive multiples of {m}")
            pos = position_table(self.pos_table, grid_h, grid_w, m)
            cos, sin = rotary_cos_sin(grid_h, grid_w, self.v.head_dim, self.v.theta, m)
            self.geoms[key] = tuple(t.to(self.device) for t in (pos, cos, sin))
        return self.geoms[key]

    def buffers(self, n_p):
        if n_p not in self.bufs:
            self.bufs[n_p] = _Buffers(self.v, n_p, self.device)
        return self.bufs[n_p]

    # ------------------------------------------------------------------ launches
    def _linear(self, x, wt, bias, epi, out, res=None):
        m, k = x.shape
        n = wt.shape[0]
        buf = self.bufs[self._n_p]
        tile, splits, _ = buf.plans[(m, n, k)]
        call("ffb_bf16_gemm", ptr(x), ptr(wt), ptr(bias), ptr(res), epi, ptr(out), tile, splits, ptr(buf.ws),
             ptr(buf.counters), m, n, k, self._s)

    def _norm(self, x, wt, bias, out, rows, c):
        call("ffb_layernorm", ptr(x), ptr(wt), ptr(bias), float(self.v.eps), ptr(out), rows, c, self._s)

    def _merge(self, mg, h, n_p, out, post_shuffle):
        v, buf = self.v, self.bufs[n_p]
        c4 = v.hidden * v.merge * v.merge
        if post_shuffle:  # LayerNorm over each 2x2 group's 4C values
            self._norm(h, mg["nw"], mg["nb"], buf.mln, n_p // (v.merge * v.merge), c4)
        else:             # LayerNorm over each patch's C values, then the groups
            self._norm(h, mg["nw"], mg["nb"], buf.mln, n_p, v.hidden)
        self._linear(buf.mln.view(-1, c4), mg["fc1_w"], mg["fc1_b"], L.EPI_BIAS_GELU_ERF, buf.mfc)
        self._linear(buf.mfc, mg["fc2_w"], mg["fc2_b"], L.EPI_BIAS, out)

    def enqueue(self, grid_h, grid_w):
        """Launches the tower on the current stream over the patch rows already in
        `buffers(P).pixels`; results in `.merged` and `.deep`."""
        v = self.v
        n_p = grid_h * grid_w
        pos, cos, sin = self.geometry(grid_h, grid_w)
        buf = self.buffers(n_p)
        self._s = stream_ptr(self.device)
        self._n_p = n_p
        c, d, heads = v.hidden, v.head_dim, v.heads
        act = L.EPI_BIAS_GELU_TANH if self.act == "gelu_tanh" else L.EPI_BIAS_GELU_ERF
        self._linear(buf.pixels, self.patch_w, self.patch_b, L.EPI_BIAS_RES, buf.h, res=pos)
        scale = d ** -0.5
        for j, blk in enumerate(self.blocks):
            self._norm(buf.h, blk["n1w"], blk["n1b"], buf.x, n_p, c)
            self._linear(buf.x, blk["qkv_w"], blk["qkv_b"], L.EPI_BIAS, buf.qkv)
            call("ffb_vision_rope", ptr(buf.qkv), ptr(cos), ptr(sin), n_p, heads, d, HEAD_PAD, ptr(buf.q), ptr(buf.k),
                 ptr(buf.v), self._s)
            call("ffb_attention_full", ptr(buf.q), ptr(buf.k), ptr(buf.v), ptr(buf.o), n_p, heads, d, float(scale),
                 self._s)
            self._linear(buf.o, blk["proj_w"], blk["proj_b"], L.EPI_BIAS_RES, buf.h, res=buf.h)
            self._norm(buf.h, blk["n2w"], blk["n2b"], buf.x, n_p, c)
            self._linear(buf.x, blk["fc1_w"], blk["fc1_b"], act, buf.f)
            self._linear(buf.f, blk["fc2_w"], blk["fc2_b"], L.EPI_BIAS_RES, buf.h, res=buf.h)
            if j in v.deepstack:
                i = v.deepstack.index(j)
                self._merge(self.deep_mergers[i], buf.h, n_p, buf.deep[i], post_shuffle=True)
        self._merge(self.merger, buf.h, n_p, buf.merged, post_shuffle=False)
        return buf

    @staticmethod
    def launches(vdims):
        """Kernel launches of one forward (the graph's node count)."""
        return 1 + 8 * vdims.depth + 3 * (len(vdims.deepstack) + 1)

    # ------------------------------------------------------------------ entry points
    def forward(self, pixels, grid_h, grid_w):
        """Eager forward of one image: pixels [grid_h * grid_w, 1536] bf16 patch rows (merge
        order, as `ops.pack_rgb` writes them).  Returns (merged [P/4, out_hidden],
        [deepstack features]) -- views of the geometry's buffers, valid until the next call
        with the same geometry."""
        with self.lock, torch.cuda.device(self.device):
            buf = self.buffers(grid_h * grid_w)
            buf.pixels.copy_(pixels)
            self.enqueue(grid_h, grid_w)
            return buf.merged, list(buf.deep)

    def capture(self, grid_h, grid_w):
        """The CUDA graph of one geometry (built on first use, as `VisionGraph.build`)."""
        key = (grid_h, grid_w)
        with self.lock, torch.cuda.device(self.device):
            if key not in self.graphs:
                self.geometry(grid_h, grid_w)
                self.buffers(grid_h * grid_w)
                side = torch.cuda.Stream(self.device)
                side.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(side):
                    self.enqueue(grid_h, grid_w)  # warm-up: dynamic shared memory attributes
                torch.cuda.current_stream(self.device).wait_stream(side)
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=side):
                    self.enqueue(grid_h, grid_w)
                self.graphs[key] = g
            return self.graphs[key]

    def replay(self, pixels, grid_h, grid_w):
        """forward() through the geometry's CUDA graph."""
        with self.lock, torch.cuda.device(self.device):
            g = self.capture(grid_h, grid_w)
            buf = self.bufs[grid_h * grid_w]
            buf.pixels.copy_(pixels)
            g.replay()
            return buf.merged, list(buf.deep)

    def encode(self, rgb):
        """Image canvas rgb [H, W, 3] uint8 on the device (sides multiples of 32) -> the
        tower's outputs, through `ffb_pack_rgb` and the graph of its geometry."""
        from .ops import pack_rectangle
        h, w = int(rgb.shape[0]), int(rgb.shape[1])
        grid_h, grid_w = h // self.v.patch, w // self.v.patch
        with self.lock, torch.cuda.device(self.device):
            g = self.capture(grid_h, grid_w)
            buf = self.bufs[grid_h * grid_w]
            pack_rectangle(rgb, pixels=buf.pixels)
            g.replay()
            return buf.merged, list(buf.deep)


# ---------------------------------------------------------------------------- request encoder

def read_canvas(image):
    """uint8 [H, W, 3] canvas from an array or tensor, a `.npy` file, or a binary PPM (P6,
    maxval 255) file.  Canvas sides must already be multiples of 32: decoding compressed
    formats and resizing into the canvas (the reference's cv2 step, `_family/depth_runtime.py:
    54-76`) happen before this package."""
    import numpy as np
    from pathlib import Path
    if isinstance(image, torch.Tensor):
        a = image
    elif isinstance(image, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(image))
    else:
        path = Path(image)
        raw = path.read_bytes()
        if raw[:6] == b"\x93NUMPY":
            a = torch.from_numpy(np.ascontiguousarray(np.load(path, allow_pickle=False)))
        elif raw[:2] == b"P6":
            fields, pos = [], 2
            while len(fields) < 3:  # width, height, maxval; whitespace and '#' comments between
                while raw[pos:pos + 1].isspace():
                    pos += 1
                if raw[pos:pos + 1] == b"#":
                    pos = raw.index(b"\n", pos) + 1
                    continue
                end = pos
                while not raw[end:end + 1].isspace():
                    end += 1
                fields.append(int(raw[pos:end]))
                pos = end
            w, h, maxval = fields
            if maxval != 255:
                raise ValueError(f"PPM maxval {maxval}: only 8-bit canvases are supported")
            pos += 1
            a = torch.frombuffer(bytearray(raw[pos:pos + h * w * 3]), dtype=torch.uint8).reshape(h, w, 3)
        else:
            raise ValueError(f"{path.name}: expected an uint8 canvas as .npy or binary PPM (P6)")
    if a.dtype != torch.uint8 or a.dim() != 3 or a.shape[2] != 3:
        raise ValueError(f"canvas must be uint8 [H, W, 3], got {tuple(a.shape)} {a.dtype}")
    if a.shape[0] % 32 or a.shape[1] % 32:
        raise ValueError(f"canvas {a.shape[0]}x{a.shape[1]}: sides must be multiples of 32")
    return a.contiguous()


def synthetic_text_ids(question, candidates, n_prefix, n_suffix, vocab):
    """Deterministic stand-in for the tokenizer (absent here): prefix and suffix ids drawn
    from a generator seeded by the question and choices."""
    import hashlib
    h = hashlib.sha256(question.encode() + b"\x00" + "\x00".join(candidates).encode()).digest()
    g = torch.Generator().manual_seed(int.from_bytes(h[:8], "little") & ((1 << 62) - 1))
    ids = torch.randint(0, vocab, (n_prefix + n_suffix,), generator=g)
    return ids[:n_prefix], ids[n_prefix:]


class VisionEncoder:
    """image canvas + question + choices -> `api.Request` through this package's vision
    tower: the canvas is packed into patch rows and run through the tower's CUDA graph;
    the merged rows are the request's visual rows and the deepstack mergers' outputs its
    deepstack rows.  Text ids come from `tokenize(question, candidates) -> (prefix ids,
    suffix ids)`; without one (no tokenizer ships with this package) they are the
    deterministic synthetic ids of the bundle's layout (`n_prefix` before the image,
    `n_suffix` after it)."""

    def __init__(self, tower, vocab, tokenize=None, n_prefix=0, n_suffix=64):
        self.tower = tower
        self.vocab = vocab
        self.tokenize = tokenize
        self.n_prefix, self.n_suffix = n_prefix, n_suffix

    def __call__(self, image, question, candidates):
        from .api import Request
        rgb = read_canvas(image).to(self.tower.device)
        merged, deep = self.tower.encode(rgb)
        grid_h, grid_w = rgb.shape[0] // self.tower.v.patch, rgb.shape[1] // self.tower.v.patch
        if self.tokenize is not None:
            pre, suf = self.tokenize(question, list(candidates))
            pre, suf = torch.as_tensor(pre, dtype=torch.long), torch.as_tensor(suf, dtype=torch.long)
        else:
            pre, suf = synthetic_text_ids(question, list(candidates), self.n_prefix, self.n_suffix, self.vocab)
        nv = merged.shape[0]
        ids = torch.cat([pre, torch.zeros(nv, dtype=torch.long), suf])
        # the tower's buffers are reused by its next image: the request keeps copies
        return Request(ids=ids, visual=merged.clone(), deep=[d.clone() for d in deep], image_start=int(pre.shape[0]),
                       grid_h=grid_h, grid_w=grid_w, k=len(candidates))

"""Prefill + choice-scoring engine: packed weights in HBM, fused launch sequence, graphs.

Layer order, deepstack placement and the pick-row tail follow the reference runtime
(`scaled_qwen_runtime.py:143-176` `prefix`/`attention`/`mlp`, `_family/night_runtime.py:
92-105` `tail`, `:106-125` `graph`).  Per decoder layer the engine enqueues
(rowwise-FP8 mode):

    qkv GEMM  -> QK-norm + M-RoPE (+ split-K reduce) -> attention -> quant(O)
    -> o GEMM -> add+RMSNorm (+ split-K reduce, + fused quant of the MLP input)
    -> gate/up GEMM with fused SwiGLU epilogue -> quant(act) -> down GEMM
    -> add+RMSNorm (+ deepstack rows, + fused quant of the next layer's input)

The last layer runs K/V over all T rows but Q, o_proj and the MLP on the pick row only,
then the readout kernel adds the MLP row, applies the final norm, dots the option rows
and takes the log-softmax over the k choices.  `Engine.capture` records the whole
sequence into one CUDA graph per request geometry (bucket, image window, k), replayed
with the request's ids / visual rows / deepstack rows / pick copied into static buffers.
"""
import ctypes
import math
from dataclasses import dataclass, field

import torch

from . import _lib as L
from ._lib import call, ptr
from .config import MODELS, Dims
from .mrope import position_ids, cos_sin

BF16 = torch.bfloat16
E4M3 = torch.float8_e4m3fn
SMS = 148
ROLES = ("qkv", "o", "gateup", "down")
# Calibration-profile key of each role: "{layer}:{role}" with the reference's role names
# (`_family/night_runtime.py:72-76`, `pack_release`).
PROFILE_ROLE = {"qkv": "qkv", "o": "output", "gateup": "gateup", "down": "down"}
FP8_MAX = 448.0
# Static activation bound used when no profile is given: StaticFP8Linear's default
# inverse scale 16 (`_legacy/limit_kernels.py:120`), i.e. bound 448 / 16.
DEFAULT_STATIC_BOUND = FP8_MAX / 16.0


def static_bound(maximum, margin=1.5):
    """Calibrated static activation bound from an observed max|x|, as the reference's
    calibration (`_legacy/limit_runtime.py:88-91`): inverse = 2^floor(log2(448 /
    (max(maximum, 1e-12) * margin))), bound = 448 / inverse (exact: inverse is a power of two)."""
    inverse = 2.0 ** math.floor(math.log2(FP8_MAX / (max(float(maximum), 1e-12) * margin)))
    return FP8_MAX / inverse


# ---------------------------------------------------------------------------- packing

def _pack_fp8(w, per_channel):
    n, k = w.shape
    w8 = torch.empty((n, k), device=w.device, dtype=E4M3)
    scale = torch.empty(n if per_channel else 1, device=w.device, dtype=torch.float32)
    ws = torch.empty(n, device=w.device, dtype=torch.float32)
    call("ffb_quantize_weight_fp8", ptr(w), int(per_channel), ptr(w8), ptr(scale), ptr(ws), n, k,
         torch.cuda.current_stream(w.device).cuda_stream)
    return w8, scale


def _interleave_gateup(t, inter, elem_bytes):
    """[2I, K] (gate rows then up rows) -> tile order of the SwiGLU epilogue."""
    out = torch.empty_like(t)
    k = t.shape[1] if t.dim() == 2 else 1
    call("ffb_pack_gateup", ptr(t), ptr(out), inter, k, elem_bytes, torch.cuda.current_stream(t.device).cuda_stream)
    return out


@dataclass
class PackedLayer:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    lin: dict = field(default_factory=dict)   # role -> dict(w8, scale) | dict(packed, scales)
    inv: dict = field(default_factory=dict)   # role -> static inverse activation scale 448/bound
    ascale: dict = field(default_factory=dict)  # role -> fp32 [1] device tensor bound/448


class PackedModel:
    """A model's weights in the layouts the kernels read.

    mode "rowwise": FP8 e4m3 weights with per-output-channel scales, per-token activation
    scales (`_legacy/fp8_private.py`); "static": per-tensor weight
    scale + static per-tensor activation scale (`_family/depth_fp8.py`, the reference's
    shipped scheme); "int4": W4A16 symmetric group 128.

    `profile` (static mode) maps "{layer}:{role}" (roles qkv, output, gateup, down) to the
    activation bound of that linear, as the reference's calibration profiles do: the
    activation is quantised with inverse scale 448/bound and the GEMM multiplies by the
    fp32 input scale bound/448 (`_family/night_runtime.py:48-54`).  Without a profile every
    bound is 448/16 (StaticFP8Linear's default).  `calibrate_profile` measures one.
    The gate/up weight rows (and their scales) are stored interleaved per 128 channels for
    the fused SwiGLU epilogue.

    tp = (rank, world) keeps only this rank's tensor-parallel shard of every linear
    (`fastforward_b200.tp`): each weight is packed whole, then sliced, and `dims` becomes the
    per-rank shape (heads and SwiGLU channels divided by the world size).
    """

    def __init__(self, dims, bf16_model, mode="rowwise", device="cuda", free_source=False, tp=None, profile=None):
        assert mode in ("rowwise", "static", "int4")
        if profile is not None and mode != "static":
            raise ValueError("a calibration profile applies to mode 'static' only")
        from . import tp as tpmod
        self.full_dims = dims
        self.tp = tp
        self.dims = tpmod.local_dims(dims, tp[1]) if tp else dims
        self.mode = mode
        self.device = torch.device(device)
        self.embed = bf16_model["embed"].to(self.device, BF16).contiguous()
        self.head = bf16_model["head"].to(self.device, BF16).contiguous()
        self.final_norm = bf16_model["final_norm"].to(self.device, BF16).contiguous()
        self.layers = []
        src_layers = bf16_model["layers"]
        for j in range(len(src_layers)):
            src = src_layers[j]
            lay = PackedLayer(*(src[n].to(self.device, BF16).contiguous()
                                for n in ("in_norm", "post_norm", "q_norm", "k_norm")))
            for role in ("qkv", "o", "gateup", "down"):
                w = src[role].to(self.device, BF16).contiguous()
                if role == "gateup":
                    w = _interleave_gateup(w, dims.inter, 2)
                if mode == "int4":
                    packed = torch.empty((w.shape[0], w.shape[1] // 2), device=self.device, dtype=torch.uint8)
                    scales = torch.empty((w.shape[0], w.shape[1] // 128), device=self.device, dtype=BF16)
                    call("ffb_pack_int4", ptr(w), ptr(packed), ptr(scales), w.shape[0], w.shape[1],
                         torch.cuda.current_stream(self.device).cuda_stream)
                    lay.lin[role] = dict(packed=packed, scales=scales)
                else:
                    w8, scale = _pack_fp8(w, per_channel=(mode == "rowwise"))
                    lay.lin[role] = dict(w8=w8, scale=scale)
                if tp:
                    lay.lin[role] = tpmod.shard_packed(role, lay.lin[role], dims, tp[0], tp[1])
                lay.inv[role] = 1.0
                if mode == "static":
                    lay.ascale[role] = torch.empty(1, device=self.device, dtype=torch.float32)
                del w
            self.layers.append(lay)
            if free_source:
                src_layers[j] = None
        if mode == "static":
            self.set_profile(profile)
        torch.cuda.synchronize(self.device)

    def set_profile(self, profile):
        """Sets every static activation bound from `profile` ("{layer}:{role}" -> bound;
        None = the default bound), as the reference's `select(variant)` does
        (`_family/night_runtime.py:48-54`).  Graphs captured before keep the old inverse
        scales: `Engine.set_profile` drops them."""
        if self.mode != "static":
            raise ValueError("a calibration profile applies to mode 'static' only")
        for j, lay in enumerate(self.layers):
            for role in ROLES:
                key = f"{j}:{PROFILE_ROLE[role]}"
                if profile is None:
                    bound = DEFAULT_STATIC_BOUND
                elif key in profile:
                    bound = float(profile[key])
                else:
                    raise ValueError(f"calibration profile has no bound for {key}")
                if not (math.isfinite(bound) and bound > 0):
                    raise ValueError(f"bad static activation bound {bound} for {key}")
                lay.inv[role] = FP8_MAX / bound
                lay.ascale[role].fill_(bound / FP8_MAX)

    @property
    def depth(self):
        return len(self.layers)

    def weight_bytes(self):
        total = 0
        for lay in self.layers:
            for d in lay.lin.values():
                total += sum(t.numel() * t.element_size() for t in d.values())
        return total


# ---------------------------------------------------------------------------- planning

def pick_feature_tile(n):
    """Output features per GEMM tile: 256 (the MMA's cost is nearly flat in N) when N allows."""
    return 256 if n % 256 == 0 else 128


# Largest K-split of a plan: the consumers of the fp32 partials (add+RMSNorm, standalone or
# as a fused GEMM prologue) sum at most this many.
MAX_PLAN_SPLITS = 8


def plan_splits(m, n, k, bn=None, allow_split=True, sms=SMS):
    """K-split count that minimises (waves x k-blocks per CTA) plus a small per-split cost
    for the fp32 partial tiles the consumer has to read back."""
    bn = bn or pick_feature_tile(n)
    base = (n // bn) * math.ceil(m / 128)
    nkb = math.ceil(k / 128)
    if not allow_split:
        return 1
    best, best_cost = 1, None
    for s in range(1, min(nkb, MAX_PLAN_SPLITS) + 1):
        waves = math.ceil(base * s / sms)
        cost = waves * (math.ceil(nkb / s) + 1.5) + (0.0 if s == 1 else 0.4 * s * m * n / (2048 * 320))
        if best_cost is None or cost < best_cost - 1e-9:
            best, best_cost = s, cost
    return best


def weight_stationary_plan(m, n, k, swiglu=False, max_splits=MAX_PLAN_SPLITS):
    """(splits, epilogue) of the weight-stationary schedule (`ffb_fp8_gemm` feature_tile
    TILE_STREAM) for an m x n x k GEMM, or None when it does not apply.  A CTA's mainloop
    costs about the same per 128-byte K block whatever its token count (one tcgen05.mma
    chain, ~70 ns per instruction, 4 per K block), so fewer K blocks per CTA is what counts;
    the cost model -- K blocks per CTA x (16 KB weight tile + 2 KB per 16 tokens), plus a
    charge per split for the fp32 partial planes the consumer sums -- ranks the feasible
    plans of the 4B / 8B shapes the same way (o / down: 3 splits, the most that one wave of
    <= 256-token CTAs allows).  A split plan writes fp32 partials (EPI_F32_PARTIAL); one
    split writes bf16 (or SwiGLU) directly."""
    nkb = math.ceil(k / 128)
    units = math.ceil(m / 16)
    tiles = n // (256 if swiglu else 128)
    best = None
    for s in (1,) if swiglu else range(1, min(nkb, max_splits) + 1):
        epi = L.EPI_SWIGLU if swiglu else (L.EPI_BF16 if s == 1 else L.EPI_F32_PARTIAL)
        ctas = L.stream_ctas(m, n, k, epi, s)
        if not ctas:
            continue
        per_tile = ctas // (tiles * s)
        n_max = math.ceil(units / per_tile)
        cost = math.ceil(nkb / s) * ((32 if swiglu else 16) + 2 * n_max) + (0 if s == 1 else 24 * s)
        if best is None or cost < best[0]:
            best = (cost, s, epi)
    return None if best is None else best[1:]


@dataclass
class GemmPlan:
    m: int
    n: int
    k: int
    bn: int
    splits: int
    epilogue: int


# ---------------------------------------------------------------------------- engine

class Buffers:
    """Activation buffers for one token count T (all device memory, allocated once)."""

    def __init__(self, dims, T, ws_elems, device, mode):
        h, d, hq, hk, i = dims.hidden, dims.d, dims.hq, dims.hk, dims.inter
        z = lambda *s, dt=BF16: torch.zeros(s, device=device, dtype=dt)
        self.ids = z(T, dt=torch.long)
        self.pick = z(1, dt=torch.long)
        self.hA, self.hB = z(T, h), z(T, h)
        self.x8 = z(T, h, dt=E4M3)
        self.xs = z(T, dt=torch.float32)
        self.qkv = z(T, dims.qkv_out)
        self.yq, self.yk, self.yv = z(hq, T, d), z(hk, T, d), z(hk, T, d)
        self.attn = z(T, hq * d)
        self.o8 = z(T, hq * d, dt=E4M3)
        self.os = z(T, dt=torch.float32)
        # ffb_attention_rowwise's row maxima + tile counters (zero once; they carry over)
        self.qsync = z((L.lib().ffb_attention_rowwise_sync_bytes(T, hq) + 7) // 8, dt=torch.int64)
        self.lin_out = z(T, h)
        self.post8 = z(T, h, dt=E4M3)
        self.posts = z(T, dt=torch.float32)
        self.act = z(T, i)
        self.act8 = z(T, i, dt=E4M3)
        self.acts = z(T, dt=torch.float32)
        self.ws = z(max(ws_elems, 1), dt=torch.float32)
        self.hp = z(1, h)
        self.res1 = z(1, h)
        self.mlp1 = z(1, h)
        self.sync = z(2, dt=torch.int32)  # grid-barrier words of the fused GEMM prologues
        self.logits = z(8, dt=torch.float32)
        self.logprobs = z(8, dt=torch.float32)
        if mode == "int4":
            self.xb = z(T, h)          # bf16 GEMM inputs for W4A16
            self.postb = z(T, h)


class BatchBuffers(Buffers):
    """Buffers of a batched forward: T concatenated rows of R requests (`Engine.forward_batch`)."""

    def __init__(self, dims, T, R, ws_elems, device, mode):
        super().__init__(dims, T, ws_elems, device, mode)
        h = dims.hidden
        z = lambda *s, dt=BF16: torch.zeros(s, device=device, dtype=dt)
        self.R = R
        self.pick = z(R, dt=torch.long)           # the pick rows in the concatenated sequence
        self.hp, self.res1, self.mlp1 = z(R, h), z(R, h), z(R, h)
        self.logits = z(R, 8, dt=torch.float32)
        self.logprobs = z(R, 8, dt=torch.float32)
        self.key_lo = z(T, dt=torch.int32)        # first row of each row's request
        self.tail_lo = z(R, dt=torch.int32)       # first row of each pick row's request
        self.cos = z(T, dims.d)
        self.sin = z(T, dims.d)
        # deepstack rows of the batch: -0.0 outside the requests' visual rows (x + -0.0 == x
        # for every x, so those rows are untouched, bit for bit)
        self.deep = [torch.full((T, h), -0.0, device=device, dtype=BF16) for _ in range(dims.deepstack)]


class Engine:
    """Runs prefill + choice scoring for one packed model on one device."""

    def __init__(self, model: PackedModel, pdl=True, autotune=True, tp_group=None, fuse="tail", stream_od=True,
                 attn_q8=False, peer=False):
        """tp_group: the torch.distributed (NCCL) group of a tensor-parallel model
        (`PackedModel(tp=...)`); o_proj and down_proj partial sums are all-reduced in it.
        fuse (FP8 modes): where an activation quantiser or an add+RMSNorm runs as the fused
        prologue of the GEMM that consumes it (`ffb_fp8_gemm_fused`) instead of a launch of
        its own -- "tail": in the one-row tail only (where the row work is a few hundred
        elements and the launch is the whole cost); "all" (or True): everywhere, five
        launches per layer instead of nine; "none" (or False): nowhere.  Every choice
        computes the same bytes.  At T = 320 the separate row kernels are faster than the
        prologues (which run the same row work on fewer warps per row, then meet at a grid
        barrier), hence the default.  attn_q8 (per-token scales): the attention kernel writes
        the o projection's FP8 input and scales itself (`ffb_attention_rowwise`) whenever its
        grid is resident at once -- the same bytes as attention + `ffb_quantize_fp8`.  Off by
        default: measured in CUDA-graph chains on a B200 (4B, T = 320) it takes 22.5 us where
        attention + the separate quantiser take 19.2 us, because every head CTA of a query
        tile must stay resident until the tile's last head arrives, which holds back the
        next kernel's CTAs; the whole request went from 3.45 to 3.58 ms with it on."""
        L.require_cuda()
        self.m = model
        self.d = model.dims
        self.world = model.tp[1] if model.tp else 1
        self.group = tp_group
        if self.world > 1 and tp_group is None:
            raise ValueError("a tensor-parallel model needs its process group")
        self.device = model.device
        self.graphs = {}
        self.tables = {}
        self.buffers = {}
        self.plans = {}
        self.autotune_enabled = autotune and model.mode != "int4"
        self.tuned = {}
        mode_ = {True: "all", False: "none"}.get(fuse, fuse)
        if mode_ not in ("none", "tail", "all"):
            raise ValueError(f"fuse must be 'none', 'tail' or 'all', not {fuse!r}")
        # int4 has no FP8 prologue; tensor-parallel rowwise quantisers need a collective
        # between the slice scales and the cast, so no quantiser runs as a GEMM prologue
        self.fuse = "none" if (model.mode == "int4" or self.world > 1) else mode_
        # static scales: attention and the gate/up launch also write the FP8 input of the
        # linear after them (`ffb_attention_fp8`, `ffb_fp8_gemm_swiglu_fp8`), so neither
        # activation quantiser has a launch of its own
        self.static_q8 = model.mode == "static" and self.fuse != "none"
        # per-token scales: attention writes the o projection's FP8 input and scales itself
        # (`ffb_attention_rowwise`) when its grid fits the SMs at once (single GPU: with tensor
        # parallelism the scale is a maximum over the ranks)
        self.attn_q8 = attn_q8 and model.mode == "rowwise" and self.world == 1 and self.fuse != "all"
        self.sms = torch.cuda.get_device_properties(model.device).multi_processor_count
        # tensor parallel, peer=True: the full layers' reductions read the ranks' partials and
        # activation maxima from peer memory inside the consuming kernel
        # (`ffb_add_rmsnorm_peers`, `ffb_quantize_fp8_peers`) when every rank could map every
        # other's buffers.  Bit-identical to the NCCL path, but measured slower on 2 B200s at
        # the 32B shapes (T = 1024: 119 us against 86 us for all-reduce + add+RMSNorm, 37 us
        # against 20 us for the scale exchange; the peer plane is read over NVLink at ~230
        # GB/s), so NCCL stays the default.
        self.peer = self._open_peers() if (peer and self.world > 1) else None
        # o_proj / down_proj on the weight-stationary schedule (K splits chosen by its cost
        # model, measured 1% faster per 4B request than token-major split-K tiles)
        self.stream_od = stream_od
        L.set_pdl(pdl)

    def _open_peers(self):
        """PeerBuffers for the group, or None on every rank when any rank cannot map them
        (the decision is collective, so the ranks never mix the two reduction paths)."""
        import torch.distributed as dist
        from .config import BUCKETS
        from .peer import PeerBuffers
        pb, ok = None, 1
        try:
            pb = PeerBuffers(self.group, self.m.tp[0], self.world, max(BUCKETS), self.d.hidden, self.device)
        except Exception:
            ok = 0
        flag = torch.tensor([ok], dtype=torch.int32, device=self.device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        if int(flag.item()) == 0:
            if pb is not None:
                pb.close()
            return None
        return pb

    def close_peers(self):
        """Releases the peer mappings (call on every rank before destroying the group)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _red_target(self, b):
        """Where the next row-parallel GEMM writes its fp32 partial: this rank's peer plane
        (alternating between two) or the NCCL workspace."""
        if self.peer is None:
            return b.ws
        from .peer import DevicePtr
        return DevicePtr(self.peer.own_plane[self._pc & 1])

    def _add_rmsnorm_reduced(self, plan, b, ws, a, deep, start, nv, w, eps, residual, out, qmode, inv, q8, qs, T, H):
        """residual = a + (the ranks' summed partial), out / q8 = its RMSNorm: through peer
        memory in one kernel, or NCCL all-reduce + ffb_add_rmsnorm."""
        if self.peer is not None:
            call("ffb_add_rmsnorm_peers", ptr(a), ctypes.addressof(self.peer.planes[self._pc & 1]),
                 ctypes.addressof(self.peer.sync), ptr(deep), start, nv, ptr(w), eps, ptr(residual), ptr(out), qmode,
                 inv, ptr(q8), ptr(qs), T, H, self._s)
            self._pc += 1
            return
        self._tp_reduce(plan, ws)
        xb, x32, xs = self._split_args(plan, None, ws)
        call("ffb_add_rmsnorm", ptr(a), xb, x32, xs, ptr(deep), start, nv, ptr(w), eps, ptr(residual), ptr(out),
             qmode, inv, ptr(q8), ptr(qs), T, H, self._s)

    # ------------------------------------------------------------------ plans / buffers
    def _plans(self, T):
        if T not in self.plans:
            self.plans[T] = self._make_plans(T, 1)
        return self.plans[T]

    def _make_plans(self, T, tail_rows):
        """GEMM plans of a forward over T rows whose tail scores `tail_rows` pick rows.

        Up to STREAM_MAX_ROWS rows the gate/up GEMM (and o / down when `stream_od`) runs the
        weight-stationary schedule when it applies (`weight_stationary_plan`: weights on the
        MMA's M side, one weight tile, token range and K range per CTA); the qkv GEMM picks
        it by itself.  Otherwise token-major tiles with the cost model's K split."""
        d = self.d
        pl = {}
        for tag, m in (("full", T), ("tail", tail_rows)):
            for role, n, k in (("qkv", d.qkv_out, d.hidden), ("o", d.hidden, d.hq * d.d),
                               ("gateup", 2 * d.inter, d.hidden), ("down", d.hidden, d.inter)):
                if tag == "tail" and role == "qkv":
                    continue
                swiglu = role == "gateup"
                bn = 128 if role == "qkv" else (256 if swiglu else pick_feature_tile(n))
                s = plan_splits(m, n, k, bn, allow_split=not swiglu and role != "qkv")
                epi = L.EPI_SWIGLU if swiglu else (L.EPI_F32_PARTIAL if s > 1 else L.EPI_BF16)
                if self.world > 1 and role in ("o", "down"):  # fp32 partial for the all-reduce
                    s, epi = 1, L.EPI_F32_PARTIAL
                elif (tag == "full" and self.fuse != "all" and m <= self.STREAM_MAX_ROWS and self.m.mode != "int4"
                      and (swiglu or (role in ("o", "down") and self.stream_od))):
                    # (FP8 only; the fused-prologue GEMMs of the tail and of fuse="all" are token-major)
                    ws_plan = weight_stationary_plan(m, n, k, swiglu)
                    if ws_plan is not None:
                        s, epi = ws_plan
                        bn = L.TILE_STREAM
                pl[(tag, role)] = GemmPlan(m, n, k, bn, s, epi)
        return pl

    # largest row count given the weight-stationary schedule (token-major tiles are full above)
    STREAM_MAX_ROWS = 512

    def buffers_for(self, T):
        if T not in self.buffers:
            pl = self._plans(T)
            # workspace sized for any split count the tuner may pick (<= MAX_SPLITS)
            ws = max(self.MAX_SPLITS * p.m * p.n for p in pl.values())
            self.buffers[T] = Buffers(self.d, T, ws, self.device, self.m.mode)
            if self.autotune_enabled:
                self._autotune(T)
        return self.buffers[T]

    MAX_SPLITS = MAX_PLAN_SPLITS

    def _autotune(self, T, reps=5):
        """Times the feature-tile choices (128 / 256 outputs per tile) of every GEMM of the
        forward on this device (zero-filled inputs, the layer-0 weights) and keeps the
        fastest.  Runs once per T, outside any timed region.  The K-split count stays the
        cost model's (`plan_splits`): it decides how the fp32 partial sums are added, so a
        timing-dependent choice would make the results depend on timing noise; the feature
        tile does not change any output element's accumulation."""
        b = self.buffers[T]
        pl = self.plans[T]
        lay = self.m.layers[0]
        s = torch.cuda.current_stream(self.device)
        self._s = s.cuda_stream
        ins = {"qkv": (b.x8, b.xs, b.qkv), "o": (b.o8, b.os, b.lin_out), "gateup": (b.post8, b.posts, b.act),
               "down": (b.act8, b.acts, b.lin_out)}
        for key, p in list(pl.items()):
            tag, role = key
            if role == "qkv" or p.epilogue == L.EPI_SWIGLU or p.bn == L.TILE_STREAM:
                continue  # fixed tiles: one head per tile / gate-up pairs per tile / token stream
            if self.world > 1 and role in ("o", "down"):
                continue  # one fp32 partial per rank, all-reduced
            a8, sc, out = ins[role]
            if self.m.mode == "static":
                sc = lay.ascale[role]
            bns = [x for x in (256, 128) if p.n % x == 0]
            best = None
            for bn in bns:
                cand = GemmPlan(p.m, p.n, p.k, bn, p.splits, p.epilogue)
                for _ in range(2):
                    self._gemm(cand, a8, sc, lay.lin[role], out, b.ws, self.m.mode == "rowwise")
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                for _ in range(reps):
                    self._gemm(cand, a8, sc, lay.lin[role], out, b.ws, self.m.mode == "rowwise")
                e1.record(s)
                e1.synchronize()
                us = e0.elapsed_time(e1) / reps * 1e3
                if best is None or us < best[0]:
                    best = (us, cand)
            pl[key] = best[1]
            self.tuned[(T,) + key] = dict(us=best[0], bn=best[1].bn, splits=best[1].splits)

    def rope_tables(self, T, image_start, grid_h, grid_w):
        key = (T, image_start, grid_h, grid_w)
        if key not in self.tables:
            pos = position_ids(T, image_start, grid_h, grid_w)
            c, s = cos_sin(pos, self.d.d, self.d.theta, self.d.sections)
            self.tables[key] = (c.to(self.device).contiguous(), s.to(self.device).contiguous())
        return self.tables[key]

    # ------------------------------------------------------------------ kernels
    def _gemm(self, plan, a8, ascale, lin, out, ws, per_row):
        call("ffb_fp8_gemm", ptr(a8), ptr(ascale), int(per_row), ptr(lin["w8"]), ptr(lin["scale"]),
             int(lin["scale"].numel() > 1), plan.epilogue, ptr(out) if plan.epilogue != L.EPI_F32_PARTIAL else None,
             ptr(ws) if plan.epilogue == L.EPI_F32_PARTIAL else None, plan.splits, plan.bn, plan.m, plan.n, plan.k,
             self._s)

    def _gemm_swiglu_q8(self, plan, a8, ascale, lin, out_inv, out8):
        """gate/up GEMM + SwiGLU + the down projection's static FP8 quantisation in one launch;
        byte-identical to the SwiGLU epilogue followed by `ffb_quantize_fp8` (STATIC)."""
        call("ffb_fp8_gemm_swiglu_fp8", ptr(a8), ptr(ascale), 0, ptr(lin["w8"]), ptr(lin["scale"]),
             int(lin["scale"].numel() > 1), float(out_inv), ptr(out8), plan.m, plan.n, plan.k, self._s)

    def _pro_quant(self, x, qmode, inv, b):
        """Prologue quantising bf16 rows x (the former ffb_quantize_fp8 launch)."""
        return L.Prologue(kind=L.PRO_QUANT, x=ptr(x), quant_mode=qmode, inv_scale=float(inv), sync=ptr(b.sync))

    def _pro_norm(self, a, bsum, deep, start, nv, w, qmode, inv, residual, b):
        """Prologue add(+partials, +deepstack) + RMSNorm + quantisation (the former
        ffb_add_rmsnorm / ffb_rmsnorm launch); bsum = (b, b32, splits) or None (no add)."""
        p = L.Prologue(kind=L.PRO_ADD_RMSNORM, x=ptr(a), norm_w=ptr(w), eps=float(self.d.eps), quant_mode=qmode,
                       inv_scale=float(inv), sync=ptr(b.sync))
        if bsum is not None:
            p.add = 1
            p.b, p.b32, p.splits = bsum
            p.residual = ptr(residual)
            if deep is not None:
                p.deep, p.start, p.nv = ptr(deep), int(start), int(nv)
        return p

    def _gemm_fused(self, pro, plan, a8, ascale, lin, out, ws, per_row):
        call("ffb_fp8_gemm_fused", ctypes.addressof(pro), ptr(a8), ptr(ascale), int(per_row), ptr(lin["w8"]),
             ptr(lin["scale"]), int(lin["scale"].numel() > 1), plan.epilogue,
             ptr(out) if plan.epilogue != L.EPI_F32_PARTIAL else None,
             ptr(ws) if plan.epilogue == L.EPI_F32_PARTIAL else None, plan.splits, plan.bn, plan.m, plan.n, plan.k,
             self._s)

    def _qkv_fused(self, pro, b, lay, cos, sin, T, rowwise):
        d = self.d
        lin = lay.lin["qkv"]
        call("ffb_fp8_gemm_qk_rope_fused", ctypes.addressof(pro), ptr(b.x8), ptr(b.xs if rowwise else lay.ascale["qkv"]),
             int(rowwise), ptr(lin["w8"]), ptr(lin["scale"]), int(lin["scale"].numel() > 1), ptr(lay.q_norm),
             ptr(lay.k_norm), float(d.eps), ptr(cos), ptr(sin), ptr(b.yq), ptr(b.yk), ptr(b.yv), T, d.hq, d.hk,
             d.hidden, self._s)

    def _w4(self, plan, x, lin, out, ws):
        call("ffb_w4a16_gemm", ptr(x), ptr(lin["packed"]), ptr(lin["scales"]), plan.epilogue,
             ptr(out) if plan.epilogue != L.EPI_F32_PARTIAL else None,
             ptr(ws) if plan.epilogue == L.EPI_F32_PARTIAL else None, plan.splits, plan.bn, plan.m, plan.n, plan.k,
             self._s)

    def _qkv(self, plan, b, lay, cos, sin, T, int4, rowwise):
        """qkv projection + per-head QK-norm + M-RoPE -> head-major Q/K/V in b.yq/yk/yv."""
        d = self.d
        if int4:
            self._w4(plan, b.xb, lay.lin["qkv"], b.qkv, b.ws)
            qb, q32, qs = self._split_args(plan, b.qkv, b.ws)
            call("ffb_qk_norm_rope", qb, q32, qs, d.qkv_out, ptr(lay.q_norm), ptr(lay.k_norm), float(d.eps),
                 ptr(cos), ptr(sin), ptr(b.yq), ptr(b.yk), ptr(b.yv), T, d.hq, d.hk, self._s)
            return
        lin = lay.lin["qkv"]
        call("ffb_fp8_gemm_qk_rope", ptr(b.x8), ptr(b.xs if rowwise else lay.ascale["qkv"]), int(rowwise), ptr(lin["w8"]), ptr(lin["scale"]),
             int(lin["scale"].numel() > 1), ptr(lay.q_norm), ptr(lay.k_norm), float(d.eps), ptr(cos), ptr(sin),
             ptr(b.yq), ptr(b.yk), ptr(b.yv), T, d.hq, d.hk, d.hidden, self._s)

    def _quant_rows_tp(self, x, q8, qs, rows, K):
        """Rowwise quantisation of a row-parallel linear's input x [rows, K] (this rank's
        slice of each row): the slice's scales, all-reduced (MAX) over the tensor-parallel
        group -- the whole row's scale, max(max|x_row|, 1e-12) / 448 being monotonic in the
        maximum -- then the slice quantised with them (FFB_QUANT_ROWSCALE), so every rank
        holds exactly the unsharded activation bytes.  One [rows] fp32 all-reduce on the
        compute stream (captured in the graph with the kernels)."""
        call("ffb_quantize_fp8", ptr(x), L.QUANT_ROWWISE, 0.0, ptr(q8), ptr(qs), rows, K, self._s)
        import torch.distributed as dist
        dist.all_reduce(qs[:rows], op=dist.ReduceOp.MAX, group=self.group)
        call("ffb_quantize_fp8", ptr(x), L.QUANT_ROWSCALE, 0.0, ptr(q8), ptr(qs), rows, K, self._s)

    def _quant_in(self, x, qmode, inv, q8, qs, rows, K, full=False):
        """The activation quantiser in front of o_proj / down_proj (rank-complete rows under
        tensor parallelism: in the full layers through peer memory when available)."""
        if self.world > 1 and qmode == L.QUANT_ROWWISE and full and self.peer is not None:
            call("ffb_quantize_fp8_peers", ptr(x), ctypes.addressof(self.peer.amax[self._qc & 1]),
                 ctypes.addressof(self.peer.sync), ptr(q8), ptr(qs), rows, K, self._s)
            self._qc += 1
        elif self.world > 1 and qmode == L.QUANT_ROWWISE:
            self._quant_rows_tp(x, q8, qs, rows, K)
        else:
            call("ffb_quantize_fp8", ptr(x), qmode, inv, ptr(q8), ptr(qs), rows, K, self._s)

    def _tp_reduce(self, plan, ws):
        """Sums this rank's fp32 partial [m, n] (in ws) over the tensor-parallel group, in
        place, on the current stream (captured into the graph with the kernels)."""
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(ws[:plan.m * plan.n], group=self.group)

    def _split_args(self, plan, bf16_out, ws):
        """(b, b32, splits) arguments of a consumer of this GEMM's output."""
        if plan.epilogue == L.EPI_F32_PARTIAL:
            return None, ptr(ws), plan.splits
        return ptr(bf16_out), None, 0

    def enqueue(self, T, image_start, nv, grid_h, grid_w, k, visual, deep, b=None, on_layer=None, observe=None):
        """Enqueue the whole forward for the request held in the T-row static buffers.

        visual: [>= nv, H] bf16 device rows scattered to [image_start, image_start + nv);
        deep: list of [nv, H] bf16 device tensors (deepstack rows added after layers 0..).
        on_layer(j, h): optional hook called with the residual stream entering layer j
        (debug tracing; it must only enqueue stream-ordered work).
        observe (rowwise mode): fp32 [depth, 4] device tensor that keeps, per layer and role
        (ROLES order), the largest per-token activation scale max|x|/448 entering that
        linear (calibration).
        Results land in b.logits [8] / b.logprobs [:k]."""
        if self.fuse == "all":
            return self._enqueue_fused(T, image_start, nv, grid_h, grid_w, k, visual, deep, b, on_layer, observe)
        d, m = self.d, self.m
        b = b or self.buffers_for(T)
        pl = self._plans(T)
        self._s = torch.cuda.current_stream(self.device).cuda_stream
        self._pc = self._qc = 0  # peer planes / maxima: each forward starts on buffer 0 (an even count of uses)
        cos, sin = self.rope_tables(T, image_start, grid_h, grid_w)
        H, D, HQ, HK, I = d.hidden, d.d, d.hq, d.hk, d.inter
        eps = float(d.eps)
        rowwise = m.mode == "rowwise"
        int4 = m.mode == "int4"
        qmode = L.QUANT_ROWWISE if rowwise else L.QUANT_STATIC
        scale = D ** -0.5
        lay0 = m.layers[0]
        if observe is not None and not rowwise:
            raise ValueError("activation observation needs the rowwise (per-token scale) forward")

        def sa(lay_, role, rowbuf):  # the GEMM's activation scale: per-token or static
            return rowbuf if rowwise else lay_.ascale[role]

        def obs(j, role, scales, rows):
            if observe is not None:
                r = ROLES.index(role)
                observe[j, r] = torch.maximum(observe[j, r], scales[:rows].amax())

        call("ffb_embed_gather", ptr(b.ids), ptr(m.embed), d.vocab, ptr(visual), image_start,
             nv if visual is not None else 0, ptr(b.hA), T, H, self._s)
        if int4:
            call("ffb_rmsnorm", ptr(b.hA), ptr(lay0.in_norm), eps, ptr(b.xb), L.QUANT_NONE, 0.0, None, None, T, H,
                 self._s)
        else:
            call("ffb_rmsnorm", ptr(b.hA), ptr(lay0.in_norm), eps, None, qmode, lay0.inv["qkv"], ptr(b.x8),
                 ptr(b.xs), T, H, self._s)
            obs(0, "qkv", b.xs, T)
        h_cur, h_mid = b.hA, b.hB
        depth = m.depth
        for j in range(depth - 1):
            if on_layer is not None:
                on_layer(j, h_cur)
            lay = m.layers[j]
            nxt = m.layers[j + 1]
            # ---- attention block
            self._qkv(pl[("full", "qkv")], b, lay, cos, sin, T, int4, rowwise)
            attn_q8 = self.attn_uses_q8(T)
            if self.static_q8:  # attention writes the o projection's FP8 input itself
                call("ffb_attention_fp8", ptr(b.yq), ptr(b.yk), ptr(b.yv), None, float(lay.inv["o"]), ptr(b.o8),
                     T, HQ, HK, scale, self._s)
            elif attn_q8:  # ... with per-token scales
                call("ffb_attention_rowwise", ptr(b.yq), ptr(b.yk), ptr(b.yv), ptr(b.o8), ptr(b.os), ptr(b.qsync),
                     T, HQ, HK, scale, self._s)
            else:
                call("ffb_attention", ptr(b.yq), ptr(b.yk), ptr(b.yv), None, 0, ptr(b.attn), T, T, HQ, HK, scale,
                     self._s)
            p = pl[("full", "o")]
            red = self._red_target(b) if self.world > 1 else b.ws  # the fp32 partial's home
            if int4:
                self._w4(p, b.attn, lay.lin["o"], b.lin_out, red)
            else:
                if not self.static_q8:
                    if not attn_q8:
                        self._quant_in(b.attn, qmode, lay.inv["o"], b.o8, b.os, T, HQ * D, full=True)
                    obs(j, "o", b.os, T)
                self._gemm(p, b.o8, sa(lay, "o", b.os), lay.lin["o"], b.lin_out, red, rowwise)
            if self.world > 1:
                if int4:
                    self._add_rmsnorm_reduced(p, b, red, h_cur, None, 0, 0, lay.post_norm, eps, h_mid, b.postb,
                                              L.QUANT_NONE, 0.0, None, None, T, H)
                else:
                    self._add_rmsnorm_reduced(p, b, red, h_cur, None, 0, 0, lay.post_norm, eps, h_mid, None, qmode,
                                              lay.inv["gateup"], b.post8, b.posts, T, H)
                    obs(j, "gateup", b.posts, T)
            else:
                ob, o32, os_ = self._split_args(p, b.lin_out, b.ws)
                if int4:
                    call("ffb_add_rmsnorm", ptr(h_cur), ob, o32, os_, None, 0, 0, ptr(lay.post_norm), eps, ptr(h_mid),
                         ptr(b.postb), L.QUANT_NONE, 0.0, None, None, T, H, self._s)
                else:
                    call("ffb_add_rmsnorm", ptr(h_cur), ob, o32, os_, None, 0, 0, ptr(lay.post_norm), eps, ptr(h_mid),
                         None, qmode, lay.inv["gateup"], ptr(b.post8), ptr(b.posts), T, H, self._s)
                    obs(j, "gateup", b.posts, T)
            # ---- MLP block
            p = pl[("full", "gateup")]
            if int4:
                self._w4(p, b.postb, lay.lin["gateup"], b.act, b.ws)
            elif self.static_q8:
                self._gemm_swiglu_q8(p, b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"], lay.inv["down"],
                                     b.act8)
            else:
                self._gemm(p, b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"], b.act, b.ws, rowwise)
            p = pl[("full", "down")]
            red = self._red_target(b) if self.world > 1 else b.ws
            if int4:
                self._w4(p, b.act, lay.lin["down"], b.lin_out, red)
            else:
                if not self.static_q8:
                    self._quant_in(b.act, qmode, lay.inv["down"], b.act8, b.acts, T, I, full=True)
                    obs(j, "down", b.acts, T)
                self._gemm(p, b.act8, sa(lay, "down", b.acts), lay.lin["down"], b.lin_out, red, rowwise)
            dp = deep[j] if (deep is not None and j < len(deep)) else None
            dnv = nv if dp is not None else 0
            if self.world > 1:
                if int4:
                    self._add_rmsnorm_reduced(p, b, red, h_mid, dp, image_start, dnv, nxt.in_norm, eps, h_cur, b.xb,
                                              L.QUANT_NONE, 0.0, None, None, T, H)
                else:
                    self._add_rmsnorm_reduced(p, b, red, h_mid, dp, image_start, dnv, nxt.in_norm, eps, h_cur, None,
                                              qmode, nxt.inv["qkv"], b.x8, b.xs, T, H)
                    obs(j + 1, "qkv", b.xs, T)
            else:
                db, d32, ds = self._split_args(p, b.lin_out, b.ws)
                if int4:
                    call("ffb_add_rmsnorm", ptr(h_mid), db, d32, ds, ptr(dp), image_start, dnv, ptr(nxt.in_norm), eps,
                         ptr(h_cur), ptr(b.xb), L.QUANT_NONE, 0.0, None, None, T, H, self._s)
                else:
                    call("ffb_add_rmsnorm", ptr(h_mid), db, d32, ds, ptr(dp), image_start, dnv, ptr(nxt.in_norm), eps,
                         ptr(h_cur), None, qmode, nxt.inv["qkv"], ptr(b.x8), ptr(b.xs), T, H, self._s)
                    obs(j + 1, "qkv", b.xs, T)
        # ---- tail: last layer on the pick row (night_runtime.py:92-105)
        if on_layer is not None:
            on_layer(depth - 1, h_cur)
        lay = m.layers[depth - 1]
        self._qkv(pl[("full", "qkv")], b, lay, cos, sin, T, int4, rowwise)
        if self.fuse == "tail":
            return self._tail_fused(b, h_cur, k, obs, sa, qmode)
        call("ffb_attention", ptr(b.yq), ptr(b.yk), ptr(b.yv), ptr(b.pick), 1, ptr(b.attn), 1, T, HQ, HK, scale,
             self._s)
        p = pl[("tail", "o")]
        if int4:
            self._w4(p, b.attn, lay.lin["o"], b.lin_out, b.ws)
        else:
            self._quant_in(b.attn, qmode, lay.inv["o"], b.o8, b.os, 1, HQ * D)
            obs(depth - 1, "o", b.os, 1)
            self._gemm(p, b.o8, sa(lay, "o", b.os), lay.lin["o"], b.lin_out, b.ws, rowwise)
        self._tp_reduce(p, b.ws)
        ob, o32, os_ = self._split_args(p, b.lin_out, b.ws)
        call("ffb_gather_rows", ptr(h_cur), ptr(b.pick), ptr(b.hp), 1, H * 2, self._s)
        if int4:
            call("ffb_add_rmsnorm", ptr(b.hp), ob, o32, os_, None, 0, 0, ptr(lay.post_norm), eps, ptr(b.res1),
                 ptr(b.postb), L.QUANT_NONE, 0.0, None, None, 1, H, self._s)
        else:
            call("ffb_add_rmsnorm", ptr(b.hp), ob, o32, os_, None, 0, 0, ptr(lay.post_norm), eps, ptr(b.res1),
                 None, qmode, lay.inv["gateup"], ptr(b.post8), ptr(b.posts), 1, H, self._s)
            obs(depth - 1, "gateup", b.posts, 1)
        p = pl[("tail", "gateup")]
        if int4:
            self._w4(p, b.postb, lay.lin["gateup"], b.act, b.ws)
        else:
            self._gemm(p, b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"], b.act, b.ws, rowwise)
        p = pl[("tail", "down")]
        if int4:
            self._w4(p, b.act, lay.lin["down"], b.mlp1, b.ws)
        else:
            self._quant_in(b.act, qmode, lay.inv["down"], b.act8, b.acts, 1, I)
            obs(depth - 1, "down", b.acts, 1)
            self._gemm(p, b.act8, sa(lay, "down", b.acts), lay.lin["down"], b.mlp1, b.ws, rowwise)
        self._tp_reduce(p, b.ws)
        mb, m32, ms = self._split_args(p, b.mlp1, b.ws)
        call("ffb_readout", ptr(b.res1), mb, m32, ms, ptr(m.final_norm), eps, ptr(m.head), m.head.shape[0], int(k),
             ptr(b.logits), ptr(b.logprobs), H, self._s)
        return b

    def _enqueue_fused(self, T, image_start, nv, grid_h, grid_w, k, visual, deep, b, on_layer, observe):
        """`enqueue` with every row kernel of a decoder layer fused into the GEMM after it:
        per layer qkv(+add/RMSNorm prologue, QK-norm/RoPE epilogue), attention,
        o(+quant prologue), gate/up(+add/RMSNorm prologue, SwiGLU epilogue),
        down(+quant prologue); the add+RMSNorm of the down output is the next layer's qkv
        prologue (the first layer's is the plain RMSNorm of the embeddings)."""
        d, m = self.d, self.m
        b = b or self.buffers_for(T)
        pl = self._plans(T)
        self._s = torch.cuda.current_stream(self.device).cuda_stream
        cos, sin = self.rope_tables(T, image_start, grid_h, grid_w)
        H, D, HQ, HK, I = d.hidden, d.d, d.hq, d.hk, d.inter
        eps = float(d.eps)
        rowwise = m.mode == "rowwise"
        qmode = L.QUANT_ROWWISE if rowwise else L.QUANT_STATIC
        scale = D ** -0.5
        if observe is not None and not rowwise:
            raise ValueError("activation observation needs the rowwise (per-token scale) forward")

        def sa(lay_, role, rowbuf):
            return rowbuf if rowwise else lay_.ascale[role]

        def obs(j, role, scales, rows):
            if observe is not None:
                r = ROLES.index(role)
                observe[j, r] = torch.maximum(observe[j, r], scales[:rows].amax())

        call("ffb_embed_gather", ptr(b.ids), ptr(m.embed), d.vocab, ptr(visual), image_start,
             nv if visual is not None else 0, ptr(b.hA), T, H, self._s)
        h_cur, h_mid = b.hA, b.hB
        depth = m.depth
        # the qkv prologue of layer 0: RMSNorm of the embeddings
        pro = self._pro_norm(h_cur, None, None, 0, 0, m.layers[0].in_norm, qmode, m.layers[0].inv["qkv"], None, b)
        for j in range(depth):
            lay = m.layers[j]
            self._qkv_fused(pro, b, lay, cos, sin, T, rowwise)
            obs(j, "qkv", b.xs, T)
            if on_layer is not None:  # the residual entering layer j (written by the prologue above)
                on_layer(j, h_cur)
            if j == depth - 1:
                break
            nxt = m.layers[j + 1]
            call("ffb_attention", ptr(b.yq), ptr(b.yk), ptr(b.yv), None, 0, ptr(b.attn), T, T, HQ, HK, scale,
                 self._s)
            p = pl[("full", "o")]
            self._gemm_fused(self._pro_quant(b.attn, qmode, lay.inv["o"], b), p, b.o8, sa(lay, "o", b.os),
                             lay.lin["o"], b.lin_out, b.ws, rowwise)
            obs(j, "o", b.os, T)
            self._tp_reduce(p, b.ws)
            pro = self._pro_norm(h_cur, self._split_args(p, b.lin_out, b.ws), None, 0, 0, lay.post_norm, qmode,
                                 lay.inv["gateup"], h_mid, b)
            self._gemm_fused(pro, pl[("full", "gateup")], b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"],
                             b.act, b.ws, rowwise)
            obs(j, "gateup", b.posts, T)
            p = pl[("full", "down")]
            self._gemm_fused(self._pro_quant(b.act, qmode, lay.inv["down"], b), p, b.act8, sa(lay, "down", b.acts),
                             lay.lin["down"], b.lin_out, b.ws, rowwise)
            obs(j, "down", b.acts, T)
            self._tp_reduce(p, b.ws)
            dp = deep[j] if (deep is not None and j < len(deep)) else None
            pro = self._pro_norm(h_mid, self._split_args(p, b.lin_out, b.ws), dp, image_start,
                                 nv if dp is not None else 0, nxt.in_norm, qmode, nxt.inv["qkv"], h_cur, b)
        # ---- tail: last layer on the pick row (night_runtime.py:92-105); its qkv ran above
        return self._tail_fused(b, h_cur, k, obs, sa, qmode)

    def _tail_fused(self, b, h_cur, k, obs, sa, qmode):
        """The last layer after its full-T qkv (`_family/night_runtime.py:92-105`): attention,
        o_proj, MLP and readout on the pick row, with the one-row quantisers and the
        add+RMSNorm as fused GEMM prologues."""
        d, m = self.d, self.m
        T = b.ids.shape[0]
        pl = self._plans(T)
        H, D, HQ, HK = d.hidden, d.d, d.hq, d.hk
        rowwise = m.mode == "rowwise"
        depth = m.depth
        lay = m.layers[depth - 1]
        call("ffb_attention", ptr(b.yq), ptr(b.yk), ptr(b.yv), ptr(b.pick), 1, ptr(b.attn), 1, T, HQ, HK, D ** -0.5,
             self._s)
        p = pl[("tail", "o")]
        self._gemm_fused(self._pro_quant(b.attn, qmode, lay.inv["o"], b), p, b.o8, sa(lay, "o", b.os), lay.lin["o"],
                         b.lin_out, b.ws, rowwise)
        obs(depth - 1, "o", b.os, 1)
        self._tp_reduce(p, b.ws)
        ob, o32, os_ = self._split_args(p, b.lin_out, b.ws)
        call("ffb_gather_rows", ptr(h_cur), ptr(b.pick), ptr(b.hp), 1, H * 2, self._s)
        pro = self._pro_norm(b.hp, (ob, o32, os_), None, 0, 0, lay.post_norm, qmode, lay.inv["gateup"], b.res1, b)
        self._gemm_fused(pro, pl[("tail", "gateup")], b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"], b.act,
                         b.ws, rowwise)
        obs(depth - 1, "gateup", b.posts, 1)
        p = pl[("tail", "down")]
        self._gemm_fused(self._pro_quant(b.act, qmode, lay.inv["down"], b), p, b.act8, sa(lay, "down", b.acts),
                         lay.lin["down"], b.mlp1, b.ws, rowwise)
        obs(depth - 1, "down", b.acts, 1)
        self._tp_reduce(p, b.ws)
        mb, m32, ms = self._split_args(p, b.mlp1, b.ws)
        call("ffb_readout", ptr(b.res1), mb, m32, ms, ptr(m.final_norm), float(d.eps), ptr(m.head), m.head.shape[0],
             int(k), ptr(b.logits), ptr(b.logprobs), H, self._s)
        return b

    # ------------------------------------------------------------------ batched prefill
    def forward_batch(self, requests):
        """Prefill + choice scoring of several independent requests in ONE forward pass.

        Their tokens are concatenated, each request padded with id 0 to a multiple of 64 rows
        (request i at rows [off_i, off_i + n_i), off_i a multiple of 64, so its 64-key
        softmax blocks are the ones of its own forward); every GEMM and
        row kernel runs once over all rows -- the weights stream from HBM once per batch
        instead of once per request -- attention keeps each request to its own keys
        (`ffb_attention_segmented`) and the tail scores every request's pick row.  The
        reference serialises requests (README.md:53); per request the arithmetic is the
        single-request forward's, except that the K-split of o_proj / down_proj follows the
        batch's row count (fp32 partials summed in another grouping) and the tail's down_proj
        is unsplit.
        requests: list of dicts with ids [n] int64, visual [nv, H] bf16 or None, deep (list
        of [nv, H]), pick (row within the request; default n - 1), k, image_start, grid_h,
        grid_w -- device or host tensors.  Launched eagerly on the current stream.  Returns
        [(logits [k], logprobs [k])] as device tensors (views of the batch buffers, valid
        until the next batch)."""
        d, m = self.d, self.m
        if m.mode == "int4":
            raise NotImplementedError("batched prefill runs the FP8 modes")
        if self.world > 1:
            raise NotImplementedError("batched prefill runs on one GPU (replicas)")
        R = len(requests)
        if R == 0:
            return []
        ns = [int(r["ids"].shape[0]) for r in requests]
        rows = [-(-n // 64) * 64 for n in ns]       # rows per request, padding included
        offs = [sum(rows[:i]) for i in range(R)]
        T = sum(rows)
        picks, ks = [], []
        for r, n, off in zip(requests, ns, offs):
            pk = n - 1 if r.get("pick") is None else int(r["pick"])
            if not 0 <= pk < n:
                raise ValueError(f"pick {pk} outside the request's {n} rows")
            k = int(r["k"])
            if not 2 <= k <= 8:
                raise ValueError("Provide two to eight choices")
            picks.append(off + pk)
            ks.append(k)
        if (T, R) not in self.plans:
            pl = self._make_plans(T, R)
            tp = pl[("tail", "down")]
            pl[("tail", "down")] = GemmPlan(tp.m, tp.n, tp.k, tp.bn, 1, L.EPI_BF16)  # one bf16 row per request
            self.plans[(T, R)] = pl
        pl = self.plans[(T, R)]
        # buffers for up to T_alloc rows (a multiple of 256), used for the first T: head-major
        # Q/K/V take the head stride T from the kernels' arguments, row-major ones the prefix
        t_alloc = -(-T // 256) * 256
        key = ("batch", t_alloc, R)
        if key not in self.buffers:
            ws = self.MAX_SPLITS * t_alloc * max(d.hidden, d.qkv_out)
            for b_old in [k_ for k_ in self.buffers if isinstance(k_, tuple) and k_[0] == "batch"]:
                del self.buffers[b_old]  # one batch geometry resident at a time
            self.buffers[key] = BatchBuffers(d, t_alloc, R, ws, self.device, m.mode)
        b = self.buffers[key]
        self._s = torch.cuda.current_stream(self.device).cuda_stream
        dev = self.device
        H, D, HQ, HK, I = d.hidden, d.d, d.hq, d.hk, d.inter
        eps = float(d.eps)
        rowwise = m.mode == "rowwise"
        qmode = L.QUANT_ROWWISE if rowwise else L.QUANT_STATIC
        scale = D ** -0.5
        lo = torch.repeat_interleave(torch.tensor(offs, dtype=torch.int32), torch.tensor(rows))
        b.key_lo[:T].copy_(lo, non_blocking=True)
        b.tail_lo.copy_(torch.tensor(offs, dtype=torch.int32), non_blocking=True)
        b.pick.copy_(torch.tensor(picks, dtype=torch.long), non_blocking=True)
        for x in b.deep:
            x.fill_(-0.0)
        b.ids[:T].zero_()
        for r, n, nr, off in zip(requests, ns, rows, offs):
            b.ids[off:off + n].copy_(r["ids"], non_blocking=True)
            c, s_ = self.rope_tables(nr, int(r["image_start"]), int(r["grid_h"]), int(r["grid_w"]))
            b.cos[off:off + nr].copy_(c)
            b.sin[off:off + nr].copy_(s_)
            vis = r.get("visual")
            nv = int(vis.shape[0]) if vis is not None else 0
            if nv:
                st = off + int(r["image_start"])
                for x, src in zip(b.deep, r.get("deep") or []):
                    x[st:st + nv].copy_(src, non_blocking=True)
                vis = vis.to(dev, non_blocking=True)
            call("ffb_embed_gather", ptr(b.ids) + 8 * off, ptr(m.embed), d.vocab, ptr(vis) if nv else None,
                 int(r["image_start"]), nv, ptr(b.hA) + 2 * H * off, nr, H, self._s)
        cos, sin = b.cos, b.sin
        lay0 = m.layers[0]
        call("ffb_rmsnorm", ptr(b.hA), ptr(lay0.in_norm), eps, None, qmode, lay0.inv["qkv"], ptr(b.x8), ptr(b.xs), T,
             H, self._s)
        sa = lambda lay_, role, rowbuf: rowbuf if rowwise else lay_.ascale[role]
        h_cur, h_mid = b.hA, b.hB
        depth = m.depth
        for j in range(depth - 1):
            lay, nxt = m.layers[j], m.layers[j + 1]
            self._qkv(pl[("full", "qkv")], b, lay, cos, sin, T, False, rowwise)
            if self.static_q8:
                call("ffb_attention_fp8", ptr(b.yq), ptr(b.yk), ptr(b.yv), ptr(b.key_lo), float(lay.inv["o"]),
                     ptr(b.o8), T, HQ, HK, scale, self._s)
            else:
                call("ffb_attention_segmented", ptr(b.yq), ptr(b.yk), ptr(b.yv), None, 0, ptr(b.key_lo), ptr(b.attn),
                     T, T, HQ, HK, scale, self._s)
                call("ffb_quantize_fp8", ptr(b.attn), qmode, lay.inv["o"], ptr(b.o8), ptr(b.os), T, HQ * D, self._s)
            p = pl[("full", "o")]
            self._gemm(p, b.o8, sa(lay, "o", b.os), lay.lin["o"], b.lin_out, b.ws, rowwise)
            ob, o32, os_ = self._split_args(p, b.lin_out, b.ws)
            call("ffb_add_rmsnorm", ptr(h_cur), ob, o32, os_, None, 0, 0, ptr(lay.post_norm), eps, ptr(h_mid), None,
                 qmode, lay.inv["gateup"], ptr(b.post8), ptr(b.posts), T, H, self._s)
            if self.static_q8:
                self._gemm_swiglu_q8(pl[("full", "gateup")], b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"],
                                     lay.inv["down"], b.act8)
            else:
                self._gemm(pl[("full", "gateup")], b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"], b.act,
                           b.ws, rowwise)
                call("ffb_quantize_fp8", ptr(b.act), qmode, lay.inv["down"], ptr(b.act8), ptr(b.acts), T, I, self._s)
            p = pl[("full", "down")]
            self._gemm(p, b.act8, sa(lay, "down", b.acts), lay.lin["down"], b.lin_out, b.ws, rowwise)
            db, d32, ds = self._split_args(p, b.lin_out, b.ws)
            dp = b.deep[j] if j < len(b.deep) else None
            call("ffb_add_rmsnorm", ptr(h_mid), db, d32, ds, ptr(dp), 0, T if dp is not None else 0,
                 ptr(nxt.in_norm), eps, ptr(h_cur), None, qmode, nxt.inv["qkv"], ptr(b.x8), ptr(b.xs), T, H, self._s)
        # ---- tail: the last layer's K/V over all rows, the rest on the R pick rows
        lay = m.layers[depth - 1]
        self._qkv(pl[("full", "qkv")], b, lay, cos, sin, T, False, rowwise)
        call("ffb_attention_segmented", ptr(b.yq), ptr(b.yk), ptr(b.yv), ptr(b.pick), 1, ptr(b.tail_lo), ptr(b.attn),
             R, T, HQ, HK, scale, self._s)
        p = pl[("tail", "o")]
        call("ffb_quantize_fp8", ptr(b.attn), qmode, lay.inv["o"], ptr(b.o8), ptr(b.os), R, HQ * D, self._s)
        self._gemm(p, b.o8, sa(lay, "o", b.os), lay.lin["o"], b.lin_out, b.ws, rowwise)
        ob, o32, os_ = self._split_args(p, b.lin_out, b.ws)
        call("ffb_gather_rows", ptr(h_cur), ptr(b.pick), ptr(b.hp), R, H * 2, self._s)
        call("ffb_add_rmsnorm", ptr(b.hp), ob, o32, os_, None, 0, 0, ptr(lay.post_norm), eps, ptr(b.res1), None, qmode,
             lay.inv["gateup"], ptr(b.post8), ptr(b.posts), R, H, self._s)
        self._gemm(pl[("tail", "gateup")], b.post8, sa(lay, "gateup", b.posts), lay.lin["gateup"], b.act, b.ws,
                   rowwise)
        p = pl[("tail", "down")]
        call("ffb_quantize_fp8", ptr(b.act), qmode, lay.inv["down"], ptr(b.act8), ptr(b.acts), R, I, self._s)
        self._gemm(p, b.act8, sa(lay, "down", b.acts), lay.lin["down"], b.mlp1, b.ws, rowwise)
        for i, k in enumerate(ks):
            call("ffb_readout", ptr(b.res1) + 2 * H * i, ptr(b.mlp1) + 2 * H * i, None, 0, ptr(m.final_norm), eps,
                 ptr(m.head), m.head.shape[0], int(k), ptr(b.logits) + 32 * i, ptr(b.logprobs) + 32 * i, H, self._s)
        return [(b.logits[i, :k], b.logprobs[i, :k]) for i, k in enumerate(ks)]

    def launches_per_batch(self, R):
        """Kernel launches of `forward_batch` for R requests (embed and readout per request)."""
        per_layer = 7 if self.static_q8 else 9
        return R + 1 + per_layer * (self.m.depth - 1) + 1 + 1 + 2 + 1 + 1 + 2 + R

    def attn_uses_q8(self, T):
        """Whether the T-row forward's attention writes the o projection's rowwise FP8 input
        (`ffb_attention_rowwise`: its ceil(T/128) x HQ CTAs must fit the SMs at once)."""
        return self.attn_q8 and -(-T // 128) * self.d.hq <= self.sms

    def launches_per_forward(self, T=None):
        """Kernel launches `enqueue` issues for T rows (for the bench's gpu_launches count)."""
        tail = 6 if self.fuse != "none" else 9  # attention, (quant,) o, gather, (add+norm,) gate/up, (quant,) down, readout
        if self.fuse == "all":  # embed, 5 per layer, the last layer's qkv, tail
            return 1 + 5 * (self.m.depth - 1) + 1 + tail
        per_layer = 7 if self.static_q8 else (9 if self.m.mode != "int4" else 8)
        if T is not None and not self.static_q8 and self.attn_uses_q8(T):
            per_layer -= 1
        if self.m.mode == "int4":
            tail = 8
        return 2 + per_layer * (self.m.depth - 1) + 1 + tail

    # ------------------------------------------------------------------ request I/O
    def stage(self, T, ids, visual, pick):
        """Copy one request into the T-row static buffers (device tensors or host tensors)."""
        b = self.buffers_for(T)
        n = ids.shape[0]
        if n < T:
            b.ids.zero_()
        b.ids[:n].copy_(ids, non_blocking=True)
        if isinstance(pick, torch.Tensor):
            b.pick.copy_(pick.reshape(1), non_blocking=True)
        else:
            b.pick.fill_(int(pick))
        return b

    def forward(self, ids, visual, deep, pick, k, image_start, grid_h, grid_w, T=None, observe=None):
        """Eager forward (no graph): returns (logits [k], logprobs [k]) on the device."""
        T = T or ids.shape[0]
        b = self.stage(T, ids, visual, pick)
        vis = visual.contiguous() if visual is not None else None
        nv = visual.shape[0] if visual is not None else 0
        self.enqueue(T, image_start, nv, grid_h, grid_w, k, vis, deep, b, observe=observe)
        return b.logits[:k], b.logprobs[:k]

    def calibrate(self, requests, margin=1.5):
        """Static-FP8 calibration profile, by the reference's procedure
        (`_legacy/limit_runtime.py:78-97`): run the calibration requests, keep the largest
        |x| entering each linear, and give each linear the bound `static_bound(max, margin)`.

        The observed forward is this engine's rowwise-FP8 forward (mode "rowwise"): each
        token's scale is max|x_row|/448 in fp32, so 448 x the largest scale, rounded to bf16,
        is the largest |x| exactly.  (The reference observes its bf16-weight forward; the two
        activations differ by the FP8 rounding of the weights, which moves a power-of-two
        bound only when a maximum lies within that rounding of a bound boundary.)  With a
        tensor-parallel model the maxima are reduced (MAX) over the group, so every rank gets
        the same profile.

        requests: iterable of dicts with `forward`'s arguments (ids, visual, deep, pick, k,
        image_start, grid_h, grid_w, T).  Returns (profile {"{layer}:{role}": bound},
        maxima {"{layer}:{role}": max|x|})."""
        if self.m.mode != "rowwise":
            raise ValueError("calibration runs the rowwise-FP8 forward of the model")
        observe = torch.zeros((self.m.depth, len(ROLES)), device=self.device, dtype=torch.float32)
        n = 0
        for r in requests:
            self.forward(observe=observe, **r)
            n += 1
        if n == 0:
            raise ValueError("calibration needs at least one request")
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(observe, op=dist.ReduceOp.MAX, group=self.group)
        maxima = (observe.double() * FP8_MAX).to(BF16).float().cpu()
        profile, seen = {}, {}
        for j in range(self.m.depth):
            for r, role in enumerate(ROLES):
                key = f"{j}:{PROFILE_ROLE[role]}"
                seen[key] = float(maxima[j, r])
                profile[key] = static_bound(seen[key], margin)
        return profile, seen

    def set_profile(self, profile):
        """New static activation bounds (`PackedModel.set_profile`); drops captured graphs,
        whose kernels hold the old inverse scales."""
        torch.cuda.synchronize(self.device)
        self.m.set_profile(profile)
        self.graphs.clear()

    def trace(self, ids, visual, deep, pick, k, image_start, grid_h, grid_w, T=None):
        """Eager forward that also returns the residual stream entering every layer
        (list of [T, H] bf16 copies) -- for per-layer parity checks."""
        T = T or ids.shape[0]
        b = self.stage(T, ids, visual, pick)
        vis = visual.contiguous() if visual is not None else None
        nv = visual.shape[0] if visual is not None else 0
        hs = []
        self.enqueue(T, image_start, nv, grid_h, grid_w, k, vis, deep, b, on_layer=lambda j, h: hs.append(h.clone()))
        return hs, b.logits[:k].clone(), b.logprobs[:k].clone()

    def capture(self, T, image_start, nv, grid_h, grid_w, k, n_deep):
        """Capture the forward for one geometry into a CUDA graph with static inputs."""
        key = (T, image_start, nv, grid_h, grid_w, k, n_deep)
        if key in self.graphs:
            return self.graphs[key]
        d = self.d
        b = self.buffers_for(T)
        vis = torch.zeros((max(nv, 1), d.hidden), device=self.device, dtype=BF16)
        deep = [torch.zeros((max(nv, 1), d.hidden), device=self.device, dtype=BF16) for _ in range(n_deep)]
        vin = vis if nv > 0 else None
        self.rope_tables(T, image_start, grid_h, grid_w)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside the graph
                self.enqueue(T, image_start, nv, grid_h, grid_w, k, vin, deep, b)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.enqueue(T, image_start, nv, grid_h, grid_w, k, vin, deep, b)
        entry = dict(graph=g, buffers=b, visual=vis, deep=deep, k=k, nv=nv)
        self.graphs[key] = entry
        return entry

    def replay(self, entry, ids, visual, deep, pick):
        """Copy a request into the graph's static inputs and replay it (stream-ordered)."""
        b = entry["buffers"]
        n = ids.shape[0]
        T = b.ids.shape[0]
        if n < T:
            b.ids[n:].zero_()
        b.ids[:n].copy_(ids, non_blocking=True)
        nv = entry["nv"]
        if nv > 0:
            entry["visual"][:nv].copy_(visual, non_blocking=True)
        for dst, src in zip(entry["deep"], deep or []):
            dst[:nv].copy_(src, non_blocking=True)
        if isinstance(pick, torch.Tensor):
            b.pick.copy_(pick.reshape(1), non_blocking=True)
        else:
            b.pick.fill_(int(pick))
        entry["graph"].replay()
        k = entry["k"]
        return b.logits[:k], b.logprobs[:k]


def calibrate_profile(dims, bf16_model, requests, margin=1.5, device="cuda", tp=None, tp_group=None):
    """Calibration profile of a bf16 source model for mode "static": packs it rowwise
    (per-channel FP8), runs `Engine.calibrate` over `requests` and frees the packed copy.
    Returns (profile, maxima) as `Engine.calibrate`."""
    pm = PackedModel(dims, bf16_model, "rowwise", device, tp=tp)
    eng = Engine(pm, autotune=False, tp_group=tp_group)
    try:
        return eng.calibrate(requests, margin)
    finally:
        eng.close_peers()
        del eng, pm
        torch.cuda.empty_cache()

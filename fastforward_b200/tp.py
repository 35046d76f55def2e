"""Tensor parallelism for the large (32B-shaped) model: one process per GPU, NCCL over
NVLink for the two reductions of each decoder layer.

Partitioning at TP = N, rank r (the 64 query / 8 KV heads and the 25600 SwiGLU channels
of the 32B shape divide by N = 2, 4, 8):
  qkv      column-split by heads: query heads [r*HQ/N, (r+1)*HQ/N) and the matching KV
           heads [r*HK/N, (r+1)*HK/N); attention is local;
  o_proj   row-split over this rank's heads' HQ/N * 128 inputs -> fp32 partial [T, H],
           summed across ranks (all-reduce) before the residual add + RMSNorm;
  gate/up  column-split over channels [r*I/N, (r+1)*I/N) (the SwiGLU epilogue stays local);
  down     row-split over the same channels -> fp32 partial, all-reduced.
Embedding, deepstack, the norms and the readout are replicated.  Weights are quantised
whole and then sliced, so every rank's FP8 (or int4) bytes and per-channel scales equal
the unsharded model's.  Per-token activation scales of the o_proj / down_proj inputs are
the whole row's: each rank quantises its slice with the MAX over the ranks' slice scales (a
[T] fp32 all-reduce before the cast, `Engine._quant_rows_tp`), so the activation bytes are
the unsharded ones too and each rank's partial is one K split of the unsharded linear.

The packed weight layouts sliced here are those of `engine.PackedModel`: qkv rows
[q heads; k heads; v heads]; gate/up rows interleaved per 128 channels (so a rank's
channels are one contiguous block of 256-row tiles); o / down [H, K] K-major.
"""
from dataclasses import replace


def check_divisible(dims, world):
    if world < 1:
        raise ValueError("world size must be >= 1")
    if dims.hq % world or dims.hk % world:
        raise ValueError(f"{dims.name}: {dims.hq} query / {dims.hk} KV heads do not split over {world} ranks")
    if dims.inter % (128 * world):
        raise ValueError(f"{dims.name}: {dims.inter} SwiGLU channels do not split into 128-channel tiles "
                         f"over {world} ranks")


def local_dims(dims, world):
    """The per-rank shape: heads and SwiGLU channels divided by the world size."""
    check_divisible(dims, world)
    return replace(dims, hq=dims.hq // world, hk=dims.hk // world, inter=dims.inter // world)


def qkv_rows(dims, rank, world):
    """Row ranges (start, stop) of the packed qkv weight that rank `rank` keeps."""
    d, hq, hk = dims.d, dims.hq // world, dims.hk // world
    q0 = rank * hq * d
    k0 = dims.hq * d + rank * hk * d
    v0 = (dims.hq + dims.hk) * d + rank * hk * d
    return [(q0, q0 + hq * d), (k0, k0 + hk * d), (v0, v0 + hk * d)]


def gateup_rows(dims, rank, world):
    """Row range of the 128-channel-interleaved gate/up weight that rank `rank` keeps."""
    per = dims.inter // world  # channels per rank, a multiple of 128
    return [(2 * rank * per, 2 * (rank + 1) * per)]


def o_cols(dims, rank, world):
    """K range (columns) of o_proj [H, HQ*128] that rank `rank` keeps."""
    w = dims.hq * dims.d // world
    return rank * w, (rank + 1) * w


def down_cols(dims, rank, world):
    """K range (columns) of down_proj [H, I] that rank `rank` keeps."""
    w = dims.inter // world
    return rank * w, (rank + 1) * w


def take_rows(t, ranges):
    import torch
    return torch.cat([t[a:b] for a, b in ranges]).contiguous()


def shard_packed(role, packed, dims, rank, world):
    """Slices one packed linear (dict of FP8 `w8` + `scale`, or int4 `packed` + `scales`) of
    the full model down to rank `rank`'s part."""
    out = {}
    if role in ("qkv", "gateup"):
        ranges = qkv_rows(dims, rank, world) if role == "qkv" else gateup_rows(dims, rank, world)
        for k, v in packed.items():
            if k == "scale" and v.numel() == 1:  # per-tensor scale
                out[k] = v
            else:
                out[k] = take_rows(v, ranges)
        return out
    k0, k1 = o_cols(dims, rank, world) if role == "o" else down_cols(dims, rank, world)
    for k, v in packed.items():
        if k == "w8":
            out[k] = v[:, k0:k1].contiguous()
        elif k == "packed":  # two nibbles per byte along K
            out[k] = v[:, k0 // 2:k1 // 2].contiguous()
        elif k == "scales":  # int4 group scales [N, K/128]
            out[k] = v[:, k0 // 128:k1 // 128].contiguous()
        else:  # FP8 per-output-channel (or per-tensor) scale: all H outputs stay
            out[k] = v
    return out

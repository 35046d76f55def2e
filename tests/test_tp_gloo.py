"""Tensor-parallel host logic on the CPU: the shard layout of `fastforward_b200.tp` and the
row-parallel (K-split) linears, run as `gloo` ranks.  Each rank quantises its slice of the
activation rows with the whole row's scale (its slice scales MAX-all-reduced first, as
`Engine._quant_rows_tp` does) and all-reduces its fp32 partial.  The result must equal,
bit for bit, the oracle's tensor-parallel linear and the unsharded linear computed with a
`world`-way K split -- the sharded path computes the unsharded bytes."""
import os
import socket
from dataclasses import replace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from fastforward_b200 import tp
from fastforward_b200.config import MODELS

BF16 = torch.bfloat16
# a small 32B-like shape: head_dim 128, 8 query / 2 KV heads, 512 SwiGLU channels
DIMS = replace(MODELS["32B"], hidden=512, hq=8, hk=2, inter=512, layers=2, vocab=512)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(seed=3):
    g = torch.Generator().manual_seed(seed)
    o = (torch.randn(DIMS.hidden, DIMS.hq * DIMS.d, generator=g) * 0.02).to(BF16)
    down = (torch.randn(DIMS.hidden, DIMS.inter, generator=g) * 0.02).to(BF16)
    x_attn = torch.randn(40, DIMS.hq * DIMS.d, generator=g).to(BF16)
    x_act = torch.randn(40, DIMS.inter, generator=g).to(BF16)
    return o, down, x_attn, x_act


def _rank_main(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        o, down, x_attn, x_act = _weights()
        results = {}
        for role, w, x in (("o", o, x_attn), ("down", down, x_act)):
            w8, sc = oracle.quantize_weight_channel(w)  # quantised whole, then sliced
            shard = tp.shard_packed(role, {"w8": w8, "scale": sc}, DIMS, rank, world)
            k0, k1 = tp.o_cols(DIMS, rank, world) if role == "o" else tp.down_cols(DIMS, rank, world)
            _, sa = oracle.quantize_rows(x[:, k0:k1])  # this rank's slice scales ...
            dist.all_reduce(sa, op=dist.ReduceOp.MAX)  # ... made the whole row's
            xs = x[:, k0:k1].float()
            q = (xs.double() / sa.double()[:xs.shape[0], None]).float().clamp(-448, 448).to(torch.float8_e4m3fn)
            part = oracle.qwen_path._fp8_linear(q, sa[:x.shape[0]], shard["w8"], shard["scale"], 1)[:x.shape[0]]
            part = part.contiguous()
            dist.all_reduce(part)  # the all-reduce of the engine (NCCL on the GPU)
            results[role] = part.to(BF16)
        if rank == 0:
            torch.save(results, out)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_linears_over_gloo(tmp_path, world):
    out = str(tmp_path / "tp.pt")
    mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    got = torch.load(out)
    o, down, x_attn, x_act = _weights()
    for role, w, x in (("o", o, x_attn), ("down", down, x_act)):
        w8, sc = oracle.quantize_weight_channel(w)
        lin = {"w8": w8, "w_scale": sc}
        want = oracle.qwen_path._tp_linear(x, lin, "rowwise", world)
        unsharded = oracle.fp8_linear_rowwise(x, w8, sc, splits=world)  # whole-row scales, K split `world` ways
        assert torch.equal(want.view(torch.int16), unsharded.view(torch.int16)), role
        if world == 2:  # a + b == b + a: the all-reduce's summation order cannot matter
            assert torch.equal(got[role].view(torch.int16), want.view(torch.int16)), role
        else:  # a 4-way fp32 sum in the collective's order: within one bf16 rounding
            torch.testing.assert_close(got[role].float(), want.float(), atol=0, rtol=2 ** -7)


def test_local_dims_and_divisibility():
    d32 = MODELS["32B"]
    for world in (2, 4, 8):
        ld = tp.local_dims(d32, world)
        assert (ld.hq, ld.hk, ld.inter) == (64 // world, 8 // world, 25600 // world)
    with pytest.raises(ValueError):
        tp.local_dims(d32, 16)  # 8 KV heads do not split 16 ways
    with pytest.raises(ValueError):
        tp.local_dims(MODELS["2B"], 16)


def test_shards_reassemble_the_full_layer():
    """Row shards of qkv / gate-up and column shards of o / down cover the packed layer
    exactly once."""
    world = 2
    qkv = torch.arange(DIMS.qkv_out * 4, dtype=torch.float32).reshape(DIMS.qkv_out, 4)
    parts = [tp.shard_packed("qkv", {"w8": qkv, "scale": qkv[:, 0].clone()}, DIMS, r, world) for r in range(world)]
    rows = torch.cat([p["w8"] for p in parts])
    assert sorted(rows[:, 0].tolist()) == sorted(qkv[:, 0].tolist())
    assert torch.equal(parts[0]["scale"], parts[0]["w8"][:, 0])
    # rank r's q heads come first, then its k and v heads
    d = DIMS.d
    assert torch.equal(parts[1]["w8"][:d * DIMS.hq // world], qkv[d * DIMS.hq // world:d * DIMS.hq])
    gu = torch.arange(2 * DIMS.inter * 2, dtype=torch.float32).reshape(2 * DIMS.inter, 2)
    parts = [tp.shard_packed("gateup", {"w8": gu, "scale": torch.ones(1)}, DIMS, r, world) for r in range(world)]
    assert torch.equal(torch.cat([p["w8"] for p in parts]), gu)
    assert parts[0]["scale"].numel() == 1
    o = torch.arange(DIMS.hidden * DIMS.hq * d, dtype=torch.float32).reshape(DIMS.hidden, DIMS.hq * d)
    parts = [tp.shard_packed("o", {"w8": o, "scale": torch.ones(DIMS.hidden)}, DIMS, r, world) for r in range(world)]
    assert torch.equal(torch.cat([p["w8"] for p in parts], 1), o)
    assert parts[1]["scale"].shape == (DIMS.hidden,)

"""Tensor-parallel engine on 2 GPUs: a 32B-shaped model of two layers (one full layer and
the pick-row tail) sharded over two ranks, once with the full layers' reductions read from
peer memory inside the consuming kernels (`ffb_add_rmsnorm_peers`, `ffb_quantize_fp8_peers`)
and once through NCCL.  The logits must equal, bit for bit, the oracle's tensor-parallel
path (whole-row activation scales, fp32 partials summed across ranks -- for two ranks the
unsharded linear with a two-way K split), both reduction paths must agree, and the
CUDA-graph replays -- which hold the handshakes or the NCCL calls -- must equal the eager
forwards bit for bit.  Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    from fastforward_b200.config import MODELS, Layout
    from tests._model import small_case
    return small_case(MODELS["32B"], 2, layout=Layout(0, 16, 16, 64, k=4), vocab=4096)


def _rank_main(rank, world, port, out):
    from datetime import timedelta
    import torch.distributed as dist
    from fastforward_b200.engine import Engine, PackedModel
    from fastforward_b200 import _lib as L
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    eng = entry = None
    try:
        dims, src, req, layout = _case()
        pm = PackedModel(dims, src, device=dev, tp=(rank, world))
        T = layout.bucket
        ids, vis = req["ids"][:T].to(dev), req["visual"].to(dev)
        deep = [x.to(dev) for x in req["deep"]]
        res = {}
        for peer in (True, False):  # reductions through peer memory, then through NCCL
            eng = Engine(pm, tp_group=dist.group.WORLD, peer=peer)
            assert (eng.peer is not None) == peer, "peer mappings unavailable"
            z, _ = eng.forward(ids, vis, deep, req["pick"], req["k"], layout.image_start, layout.grid_h,
                               layout.grid_w, T=T)
            z = z.cpu().clone()
            entry = eng.capture(T, layout.image_start, layout.nv, layout.grid_h, layout.grid_w, req["k"], len(deep))
            zg, _ = eng.replay(entry, req["ids"][:layout.n_tokens].to(dev), vis, deep, req["pick"])
            zg = zg.cpu().clone()
            torch.cuda.synchronize()
            res["peer" if peer else "nccl"] = dict(z=z, zg=zg)
            res["splits"] = {k: p.splits for k, p in eng.plans[T].items()}
            res["error_word"] = L.device_error()
            dist.barrier()
            del entry
            entry = None
            eng.graphs.clear()
            eng.close_peers()
            eng = None
        if rank == 0:
            torch.save(res, out)
        dist.barrier()
    finally:
        if entry is not None:  # graphs holding NCCL work go before the process group
            del entry
        if eng is not None:
            eng.graphs.clear()
            eng.close_peers()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp2_engine_matches_oracle(tmp_path):
    import torch.multiprocessing as mp
    import oracle
    from fastforward_b200.mrope import position_ids
    out = str(tmp_path / "tp2.pt")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    res = torch.load(out)
    assert res["error_word"] == 0
    r = dict(res["peer"], splits=res["splits"])
    assert torch.equal(r["z"], r["zg"]), "graph replay (with the peer reductions) must equal the eager forward"
    assert torch.equal(res["nccl"]["z"], res["nccl"]["zg"]), "graph replay (with the NCCL all-reduces) == eager"
    assert torch.equal(r["z"].view(torch.int32), res["nccl"]["z"].view(torch.int32)), "peer and NCCL reductions"
    dims, src, req, layout = _case()
    T = layout.bucket
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)

    def score(block):
        old = oracle.set_attention_block(block)
        try:
            om = oracle.quantized_model(dims, src, "rowwise", splits=r["splits"], tp=2)
            return oracle.prefill_score(om, req["ids"][:T], req["visual"], req["deep"], pos, req["pick"], req["k"],
                                        image_start=layout.image_start)[0]
        finally:
            oracle.set_attention_block(old)
    zr = score(64)
    floor = (score(32) - zr).abs().max().item()
    err = (r["z"] - zr).abs().max().item()
    print(f"\n32B TP=2 |dz| = {err:.3g} (oracle's own blocking change {floor:.3g})")
    assert err <= 2e-2, (r["z"], zr, floor)
    assert oracle.response_argmax(r["z"]) == oracle.response_argmax(zr)
    assert torch.equal(r["z"].view(torch.int32), zr.view(torch.int32)), (r["z"], zr)

"""Batched multi-request prefill (`Engine.forward_batch`, `ffb_attention_segmented`).

The reference serialises requests; batching concatenates them into one sequence (each at a
64-row-aligned offset) so the weights stream once per batch.  Bars: segmented attention is
bit-identical to each request's own attention call (causal prefill and the tail's selected
rows); the batched forward computes, request by request, the CPU oracle's bytes for that
request run alone with the batch's K-split choices (bit-identical logits)."""
import pytest
import torch

import oracle
from fastforward_b200 import _lib as L
from fastforward_b200._lib import call, ptr
from fastforward_b200.config import MODELS, Layout
from fastforward_b200.engine import Engine, PackedModel
from fastforward_b200.mrope import position_ids
from fastforward_b200.synthetic import make_model_bf16, make_request
from tests._util import assert_bytes_equal

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
DEV = torch.device("cuda")
TOL = 2e-2


def _s():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("lens,HQ,HK", [((100, 64, 37), 16, 8), ((320, 200, 129, 1), 32, 8)])
def test_segmented_attention_is_per_request_attention(lens, HQ, HK):
    g = torch.Generator().manual_seed(5)
    rows = [-(-n // 64) * 64 for n in lens]
    offs = [sum(rows[:i]) for i in range(len(rows))]
    T = sum(rows)
    q = (torch.randn((HQ, T, 128), generator=g)).to(BF16).to(DEV)
    k = (torch.randn((HK, T, 128), generator=g)).to(BF16).to(DEV)
    v = (torch.randn((HK, T, 128), generator=g)).to(BF16).to(DEV)
    lo = torch.repeat_interleave(torch.tensor(offs, dtype=torch.int32), torch.tensor(rows)).to(DEV)
    out = torch.zeros((T, HQ * 128), dtype=BF16, device=DEV)
    call("ffb_attention_segmented", ptr(q), ptr(k), ptr(v), None, 0, ptr(lo), ptr(out), T, T, HQ, HK, 128 ** -0.5, _s())
    # the tail's selected rows: the last real row of each request
    picks = torch.tensor([o + n - 1 for o, n in zip(offs, lens)], dtype=torch.long, device=DEV)
    tail_lo = torch.tensor(offs, dtype=torch.int32, device=DEV)
    sel = torch.zeros((len(lens), HQ * 128), dtype=BF16, device=DEV)
    call("ffb_attention_segmented", ptr(q), ptr(k), ptr(v), ptr(picks), 1, ptr(tail_lo), ptr(sel), len(lens), T, HQ, HK,
         128 ** -0.5, _s())
    for i, (o, n, nr) in enumerate(zip(offs, lens, rows)):
        qi, ki, vi = (x[:, o:o + nr].contiguous() for x in (q, k, v))
        ref = torch.zeros((nr, HQ * 128), dtype=BF16, device=DEV)
        call("ffb_attention", ptr(qi), ptr(ki), ptr(vi), None, 0, ptr(ref), nr, nr, HQ, HK, 128 ** -0.5, _s())
        pos = torch.tensor([n - 1], dtype=torch.long, device=DEV)
        ref_sel = torch.zeros((1, HQ * 128), dtype=BF16, device=DEV)
        call("ffb_attention", ptr(qi), ptr(ki), ptr(vi), ptr(pos), 1, ptr(ref_sel), 1, nr, HQ, HK, 128 ** -0.5, _s())
        torch.cuda.synchronize()
        assert_bytes_equal(out[o:o + nr], ref, f"request {i} causal rows")
        assert_bytes_equal(sel[i:i + 1], ref_sel, f"request {i} selected row")
    assert L.device_error() == 0


def _requests(dims):
    shapes = [(8, 8, 40, 2, 0), (12, 12, 100, 8, 5), (16, 16, 33, 4, 0)]  # grid_h/2, grid_w/2, text, k, prefix
    reqs = []
    for i, (gh, gw, nt, k, pre) in enumerate(shapes):
        lay = Layout(pre, 2 * gh, 2 * gw, nt, k=k)
        r = make_request(dims, lay, seed=10 + i)
        n = lay.n_tokens
        reqs.append(dict(ids=r["ids"][:n], visual=r["visual"], deep=r["deep"], pick=n - 1, k=k,
                         image_start=lay.image_start, grid_h=lay.grid_h, grid_w=lay.grid_w))
    return reqs


@pytest.mark.parametrize("mode", ["rowwise", "static"])
def test_forward_batch_matches_oracle_per_request(mode):
    from dataclasses import replace
    dims = replace(MODELS["2B"], vocab=4096)
    src = make_model_bf16(dims, seed=0, device="cpu", layers=3)
    reqs = _requests(dims)
    profile = None
    if mode == "static":  # bounds from the oracle's bf16 calibration on the first request
        r0 = reqs[0]
        nr = -(-r0["ids"].shape[0] // 64) * 64
        ids = torch.zeros(nr, dtype=torch.long)
        ids[:r0["ids"].shape[0]] = r0["ids"]
        pos = position_ids(nr, r0["image_start"], r0["grid_h"], r0["grid_w"])
        om_bf = oracle.quantized_model(dims, src, "bf16")
        profile, _ = oracle.calibration_profile(om_bf, [dict(ids=ids, visual=r0["visual"], deepstack=r0["deep"],
                                                            position_ids=pos, pick=r0["pick"], k=r0["k"],
                                                            image_start=r0["image_start"])])
    eng = Engine(PackedModel(dims, src, mode=mode, device=DEV, profile=profile), autotune=False)
    dreqs = [dict(r, ids=r["ids"].to(DEV), visual=r["visual"].to(DEV), deep=[x.to(DEV) for x in r["deep"]])
             for r in reqs]
    outs = eng.forward_batch(dreqs)
    got = [(z.cpu().clone(), lp.cpu().clone()) for z, lp in outs]
    # same batch again: the buffers are reused and the answer is the same
    again = [(z.cpu().clone(), lp.cpu().clone()) for z, lp in eng.forward_batch(dreqs)]
    for (z1, _), (z2, _) in zip(got, again):
        assert torch.equal(z1, z2)
    rows = [-(-r["ids"].shape[0] // 64) * 64 for r in reqs]
    T, R = sum(rows), len(reqs)
    sp = {key: p.splits for key, p in eng.plans[(T, R)].items()}
    om = oracle.quantized_model(dims, src, mode, None, sp, profile=profile)
    old = oracle.set_attention_block(64)
    for r, nr, (z, lp) in zip(reqs, rows, got):
        ids = torch.zeros(nr, dtype=torch.long)
        ids[:r["ids"].shape[0]] = r["ids"]
        pos = position_ids(nr, r["image_start"], r["grid_h"], r["grid_w"])
        args = (om, ids, r["visual"], r["deep"], pos, r["pick"], r["k"])
        zr, _ = oracle.prefill_score(*args, mode=mode, image_start=r["image_start"])
        oracle.set_attention_block(32)
        zr32, _ = oracle.prefill_score(*args, mode=mode, image_start=r["image_start"])
        oracle.set_attention_block(64)
        floor = (zr - zr32).abs().max().item()
        err = (z - zr).abs().max().item()
        print(f"\nbatched request rows={nr} k={r['k']}: |dz| = {err:.3g} (floor {floor:.3g})")
        assert err <= TOL, (z, zr, err, floor)
        assert oracle.response_argmax(z) == oracle.response_argmax(zr), (z, zr)
        assert torch.equal(z.view(torch.int32), zr.view(torch.int32)), (z, zr)  # the oracle's bytes
        torch.testing.assert_close(lp, oracle.log_softmax(z), atol=1e-5, rtol=1e-5)
    oracle.set_attention_block(old)
    assert L.device_error() == 0


def test_accelerator_prefill_score_batch_matches_forward_batch():
    """The public batched entry (host inputs, one device->host read) returns the engine's
    batched answers, request by request."""
    import threading
    from dataclasses import replace
    from fastforward_b200.api import Accelerator
    dims = replace(MODELS["2B"], vocab=4096)
    src = make_model_bf16(dims, seed=0, device="cpu", layers=2)
    eng = Engine(PackedModel(dims, src, device=DEV), autotune=False)
    acc = Accelerator.__new__(Accelerator)
    acc.engine, acc.dims, acc.device, acc.lock = eng, dims, DEV, threading.RLock()
    reqs = _requests(dims)
    got = acc.prefill_score_batch(reqs)
    want = eng.forward_batch([dict(r, ids=r["ids"].to(DEV), visual=r["visual"].to(DEV),
                                   deep=[x.to(DEV) for x in r["deep"]]) for r in reqs])
    for (z, lp), (zw, lw), r in zip(got, want, reqs):
        assert len(z) == r["k"] and z == zw.cpu().tolist() and lp == lw.cpu().tolist()


def test_accelerator_prefill_score_stream_matches_single_calls():
    """The streamed entry (copies overlapped with the forwards) answers each request exactly
    as a `prefill_score` call does."""
    import threading
    from dataclasses import replace
    from fastforward_b200.api import Accelerator
    from fastforward_b200.config import BUCKETS
    dims = replace(MODELS["2B"], vocab=4096)
    src = make_model_bf16(dims, seed=0, device="cpu", layers=2)
    eng = Engine(PackedModel(dims, src, device=DEV), autotune=False)
    acc = Accelerator.__new__(Accelerator)
    acc.engine, acc.dims, acc.device, acc.lock, acc.buckets = eng, dims, DEV, threading.RLock(), BUCKETS
    reqs = _requests(dims) * 2  # six requests, three geometries, slots reused
    got = acc.prefill_score_stream([dict(r, ids=r["ids"].pin_memory(), visual=r["visual"].pin_memory(),
                                         deep=[x.pin_memory() for x in r["deep"]]) for r in reqs])
    for (z, lp), r in zip(got, reqs):
        zw, lw = acc.prefill_score(r["ids"], r["visual"], r["deep"], r["k"], r["image_start"], r["grid_h"],
                                   r["grid_w"], r["pick"])
        assert z == zw and lp == lw

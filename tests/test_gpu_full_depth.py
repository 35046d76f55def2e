"""Full-depth parity at the benchmarked configurations: every layer, the full 151,936-row
vocabulary, T = 320 (256 visual rows on a 16 x 16 merged grid + 64 text ids), free-running
(no teacher forcing).

Bar: the choice argmax identical to the oracle's on every seeded request and the
final-position option logits within 2e-2.  The engine is held to the stronger property
that it computes exactly the oracle's bytes: every kernel's arithmetic, the attention
softmax included, is restated operation for operation by the oracle (tensor-core
accumulation model, the polynomial exponential, the kernels' summation orders), so the
logits must be bit-identical.  This matters at depth: the oracle's own logits move by
0.4-0.7 when only its softmax key blocking changes (64 -> 32 keys), so on these random-
weight models agreement within 2e-2 is reachable only by computing the same bits.  The
reference's own gate is the same kind of check: native vs graph logits within
3e-3 + 1e-4 |x| and equal argmax on a full-depth request
(`_legacy/sub10_runtime.py:164-165`).
"""
import time

import pytest
import torch

import oracle
from fastforward_b200.config import MODELS, WORKLOADS
from fastforward_b200.engine import Engine, PackedModel
from fastforward_b200.mrope import position_ids
from fastforward_b200.synthetic import make_model_bf16, make_request

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 2e-2

# (workload, request seeds): the north-star 4B FP8 case in both scale schemes and C2.
CASES = [("4B-fp8-T320", (1, 2, 3)), ("4B-fp8static-T320", (4,)), ("2B-fp8-T320", (1, 2, 3))]


def _oracle_model(dims, src, mode, eng, T, profile):
    return oracle.quantized_model(dims, src, mode, splits={k: p.splits for k, p in eng.plans[T].items()},
                                  profile=profile)


@pytest.mark.parametrize("workload,seeds", CASES, ids=[c[0] for c in CASES])
def test_full_depth_bit_identical(workload, seeds):
    name, layout, mode = WORKLOADS[workload]
    dims = MODELS[name]
    src = make_model_bf16(dims, seed=0, device=DEV)
    profile = None
    if mode == "static":
        # calibrated as the reference does (largest |x| into every linear, power-of-two
        # bound), on a request that is not among the scored ones
        from fastforward_b200.engine import calibrate_profile
        cal = make_request(dims, layout, seed=100)
        T = layout.bucket
        profile, _ = calibrate_profile(dims, src, [dict(
            ids=cal["ids"][:T].to(DEV), visual=cal["visual"].to(DEV), deep=[x.to(DEV) for x in cal["deep"]],
            pick=cal["pick"], k=cal["k"], image_start=layout.image_start, grid_h=layout.grid_h, grid_w=layout.grid_w,
            T=T)], device=DEV)
    eng = Engine(PackedModel(dims, src, mode=mode, device=DEV, profile=profile))
    T = layout.bucket
    eng.buffers_for(T)
    om = _oracle_model(dims, src, mode, eng, T, profile)
    del src
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    report = []
    for seed in seeds:
        req = make_request(dims, layout, seed=seed)
        vis, deep = req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]]
        entry = eng.capture(T, layout.image_start, layout.nv, layout.grid_h, layout.grid_w, layout.k, len(deep))
        z, lp = eng.replay(entry, req["ids"][:layout.n_tokens].to(DEV), vis, deep, req["pick"])
        z, lp = z.cpu().clone(), lp.cpu().clone()
        t0 = time.time()
        zr, lpr = oracle.prefill_score(om, req["ids"][:T], req["visual"], req["deep"], pos, req["pick"], layout.k,
                                       mode=mode, image_start=layout.image_start)
        dt = time.time() - t0
        err = (z - zr).abs().max().item()
        top2 = zr.sort(descending=True).values
        margin = (top2[0] - top2[1]).item()
        report.append((seed, err, margin, dt))
        print(f"\n{workload} seed {seed}: engine {z.tolist()} oracle {zr.tolist()} max|dz| {err:.3g} "
              f"(oracle top-2 margin {margin:.3g}; oracle {dt:.1f} s)")
        assert oracle.response_argmax(z) == oracle.response_argmax(zr), (seed, z, zr)
        assert err <= TOL, (seed, z, zr)
        assert torch.equal(z.view(torch.int32), zr.view(torch.int32)), (seed, z, zr)
        torch.testing.assert_close(lp, lpr, atol=1e-5, rtol=1e-5)  # host-side log-softmax of equal logits
    print(f"\n{workload}: {len(report)} requests, argmax identical on all, max|dz| "
          f"{max(r[1] for r in report):.3g}")

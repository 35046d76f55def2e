"""Whole-path parity: the engine's prefill + scoring vs the CPU oracle on seeded requests.

Bar: choice argmax identical, final-position option logits
within 2e-2 max-abs.  Plus the reference runtime's own gates: graph replay equals the
eager path, and bucket-padding rows cannot change the result (`sub10_runtime.py:166-167`:
pad tokens overwritten with another id must give a bit-identical output).
"""
import pytest
import torch

import oracle
from fastforward_b200.config import MODELS, Layout
from fastforward_b200.engine import Engine, PackedModel
from tests._model import oracle_model, small_case

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 2e-2


def _run_engine(dims, src, req, layout, mode="rowwise", graph=False):
    pm = PackedModel(dims, src, mode=mode, device=DEV)
    eng = Engine(pm)
    T = layout.bucket
    ids = req["ids"][:T]
    args = (ids.to(DEV), req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]], req["pick"], req["k"],
            layout.image_start, layout.grid_h, layout.grid_w)
    z, lp = eng.forward(*args, T=T)
    z, lp = z.cpu().clone(), lp.cpu().clone()
    return eng, z, lp


def _oracle(dims, src, req, layout, mode="rowwise", inv=None):
    om = oracle_model(dims, src, mode, inv)
    T = layout.bucket
    from fastforward_b200.mrope import position_ids
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    return oracle.prefill_score(om, req["ids"][:T], req["visual"], req["deep"], pos, req["pick"], req["k"],
                                mode=mode, image_start=layout.image_start)


def _check_logits(z, zr):
    assert (z - zr).abs().max().item() <= TOL, (z, zr)
    assert oracle.response_argmax(z) == oracle.response_argmax(zr), (z, zr)


@pytest.mark.parametrize("name", ["2B", "4B", "8B"])
def test_tail_only_matches_oracle(name):
    """Depth-1 model: embedding, the pick-row tail and the readout, nothing compounding."""
    dims, src, req, layout = small_case(MODELS[name], 1, vocab=4096)
    _, z, lp = _run_engine(dims, src, req, layout)
    zr, _ = _oracle(dims, src, req, layout)
    _check_logits(z, zr)
    torch.testing.assert_close(lp, oracle.log_softmax(z), atol=1e-5, rtol=1e-5)


def _teacher_forced(name, n_layers, vocab=4096, layout=None):
    """Run the engine once, capturing the residual stream entering each layer; feed each
    captured input to the oracle's layer and compare with the engine's next input.  The
    errors of one layer then cannot compound through the rest (an FP8 model amplifies any
    last-bit difference: the oracle run with fp32 instead of fp64 accumulation moves its own
    logits by 0.03-0.1 at 2-6 layers on these random weights)."""
    dims, src, req, layout = small_case(MODELS[name], n_layers, vocab=vocab, layout=layout)
    pm = PackedModel(dims, src, device=DEV)
    eng = Engine(pm)
    T = layout.bucket
    hs, z, _ = eng.trace(req["ids"][:T].to(DEV), req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]],
                         req["pick"], req["k"], layout.image_start, layout.grid_h, layout.grid_w, T=T)
    hs = [h.cpu() for h in hs]
    om = oracle_model(dims, src, "rowwise")
    from fastforward_b200.mrope import position_ids
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    cos, sin = oracle.mrope_cos_sin(pos, dims.d, dims.theta)
    nv = layout.nv
    stats = []
    for j in range(len(hs) - 1):
        deep = req["deep"][j] if j < len(req["deep"]) else None
        want = oracle.decoder_layer(om["layers"][j], hs[j], cos, sin, om["dims"], "rowwise", deep,
                                    layout.image_start, nv).float()
        got = hs[j + 1].float()
        err = (got - want).abs()
        stats.append((j, err.max().item() / want.abs().max().item(), err.mean().item() / want.abs().mean().item()))
    zr, _ = oracle.tail(om["layers"][-1], hs[-1], cos, sin, om["dims"], "rowwise", req["pick"], om["final_norm"],
                        om["head"], req["k"])
    return stats, z.cpu(), zr


@pytest.mark.parametrize("name,n_layers", [("2B", 4), ("4B", 3)])
def test_layers_teacher_forced(name, n_layers):
    stats, z, zr = _teacher_forced(name, n_layers)
    print(f"\n{name} per-layer (max rel, mean rel):", stats, "tail", (z - zr).abs().max().item())
    for j, max_rel, mean_rel in stats:
        assert max_rel <= 0.02 and mean_rel <= 2e-3, (j, max_rel, mean_rel)
    _check_logits(z, zr)


def test_graph_replay_equals_eager_and_padding_isolation():
    dims = MODELS["2B"]
    layout = Layout(0, 32, 32, 60, k=4)           # 316 real tokens -> bucket 320 (4 pad rows)
    dims, src, req, layout = small_case(dims, 3, layout=layout, vocab=4096)
    pm = PackedModel(dims, src, device=DEV)
    eng = Engine(pm)
    T = layout.bucket
    n = layout.n_tokens
    vis, deep = req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]]
    z_e, _ = eng.forward(req["ids"][:T].to(DEV), vis, deep, req["pick"], 4, 0, 32, 32, T=T)
    z_e = z_e.cpu().clone()
    entry = eng.capture(T, 0, vis.shape[0], 32, 32, 4, len(deep))
    z_g, _ = eng.replay(entry, req["ids"][:n].to(DEV), vis, deep, req["pick"])
    assert torch.equal(z_g.cpu(), z_e), "graph replay must be bit-identical to the eager path"
    # pad rows carry id 0 in the graph path; overwrite them with 42 in the eager path
    ids42 = req["ids"][:T].clone()
    ids42[n:] = 42
    z_p, _ = eng.forward(ids42.to(DEV), vis, deep, req["pick"], 4, 0, 32, 32, T=T)
    assert torch.equal(z_p.cpu(), z_e), "padding rows must not influence the pick row"


@pytest.mark.slow
def test_full_depth_2b_teacher_forced():
    """All 28 layers of the 2B shape at T=320, each checked against the oracle on the
    engine's own input, and the tail's logits/argmax against the oracle's tail."""
    stats, z, zr = _teacher_forced("2B", None, vocab=8192)
    print("\n2B full depth per-layer (max rel, mean rel):", stats, "tail", (z - zr).abs().max().item())
    for j, max_rel, mean_rel in stats:
        assert max_rel <= 0.02 and mean_rel <= 2e-3, (j, max_rel, mean_rel)
    _check_logits(z, zr)

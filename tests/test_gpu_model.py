"""Whole-path parity: the engine's prefill + scoring vs the CPU oracle on seeded requests.

Bar: choice argmax identical, final-position option logits within 2e-2 max-abs; the
engine in fact computes the oracle's bytes (bit-identical logits).  Full depth at the
benchmarked shapes: tests/test_gpu_full_depth.py.  Plus the reference runtime's own gates: graph replay equals the
eager path, and bucket-padding rows cannot change the result (`sub10_runtime.py:166-167`:
pad tokens overwritten with another id must give a bit-identical output).
"""
import math

import pytest
import torch

import oracle
from fastforward_b200.config import MODELS, Layout
from fastforward_b200.engine import Engine, PackedModel
from tests._model import oracle_model, small_case

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 2e-2


def _splits(eng, T):
    """The engine's K-split choices, so the oracle accumulates exactly as the GPU does."""
    return {k: p.splits for k, p in eng.plans[T].items()}


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


def _oracle(dims, src, req, layout, mode="rowwise", inv=None, splits=None):
    om = oracle.quantized_model(dims, src, mode, inv, splits)
    T = layout.bucket
    from fastforward_b200.mrope import position_ids
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    return oracle.prefill_score(om, req["ids"][:T], req["visual"], req["deep"], pos, req["pick"], req["k"],
                                mode=mode, image_start=layout.image_start)


def _check_logits(z, zr, tol=TOL):
    """Option logits within `tol` of the oracle's and the same choice."""
    err = (z - zr).abs().max().item()
    assert err <= tol, (z, zr, err, tol)
    assert oracle.response_argmax(z) == oracle.response_argmax(zr), (z, zr)
    return err


@pytest.mark.parametrize("name", ["2B", "4B", "8B"])
def test_tail_only_matches_oracle(name):
    """Depth-1 model: embedding, the pick-row tail and the readout."""
    dims, src, req, layout = small_case(MODELS[name], 1, vocab=4096)
    eng, z, lp = _run_engine(dims, src, req, layout)
    zr, _ = _oracle(dims, src, req, layout, splits=_splits(eng, layout.bucket))
    err = _check_logits(z, zr)
    print(f"\n{name} tail-only |dz| = {err:.3g}")
    torch.testing.assert_close(lp, oracle.log_softmax(z), atol=1e-5, rtol=1e-5)


def _with_attention_block(n, fn, *args, **kw):
    old = oracle.set_attention_block(n)
    try:
        return fn(*args, **kw)
    finally:
        oracle.set_attention_block(old)


@pytest.mark.parametrize("name,n_layers", [("2B", 3), ("4B", 2)])
def test_prefill_free_running_matches_oracle(name, n_layers):
    """A few whole layers without teacher forcing.  The oracle accumulates its FP8 GEMMs as
    the tensor cores do (with the engine's K splits), its norms exactly and its attention
    with the kernel's own arithmetic, so the logits are bit-identical.  For scale, the
    oracle's own change when only its softmax blocking changes (32-key blocks instead of
    64, exact products) is printed beside it."""
    dims, src, req, layout = small_case(MODELS[name], n_layers, vocab=4096)
    eng, z, _ = _run_engine(dims, src, req, layout)
    sp = _splits(eng, layout.bucket)
    zr, _ = _oracle(dims, src, req, layout, splits=sp)
    zr32, _ = _with_attention_block(32, _oracle, dims, src, req, layout, splits=sp)
    floor = (zr - zr32).abs().max().item()
    err = _check_logits(z, zr)
    assert torch.equal(z.view(torch.int32), zr.view(torch.int32)), (z, zr)
    print(f"\n{name} {n_layers} layers free-running |dz| = {err:.3g} (oracle blocking change {floor:.3g})")


def _profile(dims, src, req, layout):
    """A calibration profile for a small case: the oracle's bf16 calibration (the
    reference's procedure) on the case's own request."""
    from fastforward_b200.mrope import position_ids
    T = layout.bucket
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    om = oracle.quantized_model(dims, src, "bf16")
    prof, _ = oracle.calibration_profile(om, [dict(ids=req["ids"][:T], visual=req["visual"], deepstack=req["deep"],
                                                   position_ids=pos, pick=req["pick"], k=req["k"],
                                                   image_start=layout.image_start)])
    return prof


@pytest.mark.parametrize("name,mode", [("2B", "rowwise"), ("4B", "rowwise"), ("2B", "static"), ("4B", "static")])
def test_layer_ops_teacher_forced(name, mode):
    """Every op of a full decoder layer at the model's real shapes (T=320), each checked
    against the oracle fed with the engine's own inputs to that op: quantised bytes and
    norms bit-exact, GEMM outputs within one bf16 rounding of the exact FP8 products.
    Mode "static" runs the reference's shipped scheme (per-tensor weights, static
    activation scales from a calibration profile)."""
    from fastforward_b200.engine import GemmPlan
    from fastforward_b200 import _lib as L
    from tests._util import assert_bf16_near, assert_bytes_equal
    dims, src, req, layout = small_case(MODELS[name], 2, vocab=4096)
    prof = _profile(dims, src, req, layout) if mode == "static" else None
    # unfused launches, so every intermediate buffer still holds layer 0's values when the
    # hook for layer 1 runs (the fused forward is bit-identical: tests/test_gpu_fused.py;
    # the attention with its own rowwise FP8 output: tests/test_gpu_kernels.py)
    eng = Engine(PackedModel(dims, src, mode=mode, device=DEV, profile=prof), autotune=False, fuse=False,
                 attn_q8=False)
    T = layout.bucket
    eng.buffers_for(T)
    for key, p in eng.plans[T].items():          # keep every GEMM output in its bf16 buffer
        if p.epilogue == L.EPI_F32_PARTIAL:
            eng.plans[T][key] = GemmPlan(p.m, p.n, p.k, p.bn, 1, L.EPI_BF16)
    b = eng.buffers[T]
    snap = {}

    def grab(j, h):  # runs at enqueue time; the clones are stream-ordered with the kernels
        if j == 1:
            for n in ("hA", "hB", "yq", "yk", "yv", "attn", "o8", "os", "post8", "posts", "act",
                      "act8", "acts", "lin_out"):
                snap[n] = getattr(b, n).clone()
        elif j == 0:  # layer 0's input and its quantised copy (x8 is rewritten for layer 1)
            snap["h0"] = h.clone()
            snap["x8"] = b.x8.clone()
            snap["xs"] = b.xs.clone()
    vis, deep = req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]]
    eng.enqueue(T, 0, layout.nv, 32, 32, 4, vis, deep, eng.stage(T, req["ids"][:T].to(DEV), vis, req["pick"]),
                on_layer=grab)
    torch.cuda.synchronize()
    S = {k: v.cpu() for k, v in snap.items()}
    om = oracle.quantized_model(dims, src, mode, profile=prof)
    lay, eps, H, HQ, HK, I = om["layers"][0], dims.eps, dims.hidden, dims.hq, dims.hk, dims.inter
    pos = oracle.mrope_position_ids(T, 0, 32, 32)
    cos, sin = oracle.mrope_cos_sin(pos, dims.d, dims.theta)

    def lin(a8, sa, w):  # the oracle's FP8 linear on the engine's own quantised input
        return oracle.qwen_path._fp8_linear(a8, sa if mode == "rowwise" else w["a_scale"], w["w8"], w["w_scale"], 1)

    def quant(x, role, name):  # the oracle's activation quant; returns (bytes, per-token scales)
        if mode == "rowwise":
            q, s = oracle.quantize_rows(x)
            assert torch.equal(S[name], s[:T]), name
            return q
        return oracle.quantize_static(x, lay[role]["inv"])

    q = quant(oracle.rms_one(S["h0"], lay["in_norm"], eps), "qkv", "xs")
    assert_bytes_equal(S["x8"], q[:T], "x8")
    qkv = lin(S["x8"], S["xs"], lay["qkv"]).to(torch.bfloat16)  # fused qkv GEMM + norm + RoPE
    rq, rk = oracle.qk_pair(qkv[:, :HQ * 128].reshape(T, HQ, 128), qkv[:, HQ * 128:(HQ + HK) * 128].reshape(T, HK, 128),
                            lay["q_norm"], lay["k_norm"], cos, sin)
    assert_bytes_equal(S["yq"], rq, "yq")
    assert_bytes_equal(S["yk"], rk, "yk")
    assert_bytes_equal(S["yv"], qkv[:, (HQ + HK) * 128:].reshape(T, HK, 128).transpose(0, 1), "yv")
    att = oracle.attention_tc(S["yq"], S["yk"], S["yv"], 128 ** -0.5).reshape(T, HQ * 128)
    assert_bytes_equal(S["attn"], att, "attention")
    q = quant(S["attn"], "o", "os")
    assert_bytes_equal(S["o8"], q[:T], "o8")
    o = lin(S["o8"], S["os"], lay["o"]).to(torch.bfloat16)
    h_mid = (S["h0"].float() + o.float()).to(torch.bfloat16)
    assert_bytes_equal(S["hB"], h_mid, "residual after attention")
    q = quant(oracle.rms_one(S["hB"], lay["post_norm"], eps), "gateup", "posts")
    assert_bytes_equal(S["post8"], q[:T], "post8")
    gu = lin(S["post8"], S["posts"], lay["gateup"]).to(torch.bfloat16)
    act = oracle.swiglu(gu[:, :I], gu[:, I:])
    assert_bytes_equal(S["act"], act, "swiglu")
    q = quant(S["act"], "down", "acts")
    assert_bytes_equal(S["act8"], q[:T], "act8")
    dn = lin(S["act8"], S["acts"], lay["down"]).to(torch.bfloat16)
    h1 = (S["hB"].float() + dn.float()).to(torch.bfloat16).float()
    h1[:layout.nv] = (h1[:layout.nv] + req["deep"][0].float()).to(torch.bfloat16).float()
    assert_bytes_equal(S["hA"], h1.to(torch.bfloat16), "residual after mlp + deepstack")


def _teacher_forced(name, n_layers, vocab=4096, layout=None, mode="rowwise"):
    """Run the engine once, capturing the residual stream entering each layer; feed each
    captured input to the oracle's layer and compare with the engine's next input (so a
    mismatch is pinned to its layer)."""
    dims, src, req, layout = small_case(MODELS[name], n_layers, vocab=vocab, layout=layout)
    prof = _profile(dims, src, req, layout) if mode == "static" else None
    pm = PackedModel(dims, src, mode=mode, device=DEV, profile=prof)
    eng = Engine(pm)
    T = layout.bucket
    hs, z, _ = eng.trace(req["ids"][:T].to(DEV), req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]],
                         req["pick"], req["k"], layout.image_start, layout.grid_h, layout.grid_w, T=T)
    hs = [h.cpu() for h in hs]
    om = oracle.quantized_model(dims, src, mode, splits=_splits(eng, T), profile=prof)
    from fastforward_b200.mrope import position_ids
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    cos, sin = oracle.mrope_cos_sin(pos, dims.d, dims.theta)
    nv = layout.nv
    mismatched = []
    for j in range(len(hs) - 1):
        deep = req["deep"][j] if j < len(req["deep"]) else None
        want = oracle.decoder_layer(om["layers"][j], hs[j], cos, sin, om["dims"], mode, deep, layout.image_start, nv)
        n_bad = int((hs[j + 1].view(torch.int16) != want.view(torch.int16)).sum())
        if n_bad:
            mismatched.append((j, n_bad))
    zr, _ = oracle.tail(om["layers"][-1], hs[-1], cos, sin, om["dims"], mode, req["pick"], om["final_norm"],
                        om["head"], req["k"])
    return mismatched, z.cpu(), zr


@pytest.mark.parametrize("name,n_layers,mode", [("2B", 4, "rowwise"), ("4B", 3, "rowwise"), ("4B", 3, "static")])
def test_layers_teacher_forced(name, n_layers, mode):
    """Whole layers on the engine's own inputs: every layer's output bit-identical to the
    oracle's, and the tail's logits too."""
    mismatched, z, zr = _teacher_forced(name, n_layers, mode=mode)
    assert not mismatched, f"layers with differing residual elements: {mismatched}"
    _check_logits(z, zr)
    assert torch.equal(z.view(torch.int32), zr.view(torch.int32)), (z, zr)


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


def test_calibration_matches_oracle():
    """`Engine.calibrate` (the rowwise forward observing every linear's input) against the
    oracle's calibration of the same forward: the maxima and the power-of-two bounds are
    equal; against the reference's procedure (the
    bf16 forward) the bounds are equal wherever the maximum is not within the FP8 weight
    rounding (5%) of a bound boundary."""
    from fastforward_b200.engine import calibrate_profile
    from fastforward_b200.mrope import position_ids
    from fastforward_b200.synthetic import make_request
    dims, src, req, layout = small_case(MODELS["2B"], 3, vocab=4096)
    reqs = [req, make_request(dims, layout, seed=7)]
    T = layout.bucket
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    dev_reqs = [dict(ids=r["ids"][:T].to(DEV), visual=r["visual"].to(DEV), deep=[x.to(DEV) for x in r["deep"]],
                     pick=r["pick"], k=r["k"], image_start=layout.image_start, grid_h=layout.grid_h,
                     grid_w=layout.grid_w, T=T) for r in reqs]
    eng = Engine(PackedModel(dims, src, "rowwise", DEV), autotune=False)  # as calibrate_profile builds it
    prof, seen = eng.calibrate(dev_reqs)
    assert (prof, seen) == calibrate_profile(dims, src, dev_reqs, device=DEV)
    cpu_reqs = [dict(ids=r["ids"][:T], visual=r["visual"], deepstack=r["deep"], position_ids=pos, pick=r["pick"],
                     k=r["k"], image_start=layout.image_start) for r in reqs]
    assert set(prof) == {f"{j}:{r}" for j in range(3) for r in ("qkv", "output", "gateup", "down")}
    # the oracle with the engine's K splits computes the engine's bytes
    p_row, s_row = oracle.calibration_profile(oracle.quantized_model(dims, src, "rowwise", splits=_splits(eng, T)),
                                              cpu_reqs, mode="rowwise")
    p_bf, s_bf = oracle.calibration_profile(oracle.quantized_model(dims, src, "bf16"), cpu_reqs, mode="bf16")
    print("\nkey: engine max / oracle rowwise max / oracle bf16 max -> engine bound, bf16 bound")
    for key in sorted(prof):
        print(f"  {key}: {seen[key]:.5g} / {s_row[key]:.5g} / {s_bf[key]:.5g} -> {prof[key]:g}, {p_bf[key]:g}")
        # the engine's forward computes the oracle's bytes, so the maxima are equal
        assert seen[key] == s_row[key], key
        x = 448.0 / (s_bf[key] * 1.5)  # distance of the bf16 maximum from a boundary
        near = abs(x / 2.0 ** round(math.log2(x)) - 1.0) < 0.05
        if not near:
            assert prof[key] == p_bf[key], key
            assert prof[key] == p_row[key], key


def test_accelerator_static_calibrated_bundle(tmp_path):
    """A static-FP8 bundle calibrated at construction (`calibrate`: request count), then a
    `predict` through the public surface; the calibrated profile written to a file and
    named by path + sha256 + variant gives a bit-identical answer."""
    import json
    from fastforward_b200.api import Accelerator, sha256
    img = tmp_path / "img.png"
    img.write_bytes(b"\x89PNG synthetic")
    syn = dict(model="2B", layers=2, seed=0, mode="static", calibrate=2, layout=dict(grid_h=16, grid_w=16, n_text=32))
    c = dict(schema_version=1, task="visual_choice", architecture="qwen3_vl_family", synthetic=syn)
    p = tmp_path / "bundle.json"
    p.write_text(json.dumps(c))
    acc = Accelerator(p)
    assert set(acc.profile) == {f"{j}:{r}" for j in range(2) for r in ("qkv", "output", "gateup", "down")}
    r1 = acc.predict(img, "What is shown?", ["cat", "dog", "bird", "fish"])
    assert all(math.isfinite(x) for x in r1["logits"])
    prof = tmp_path / "profile.json"
    prof.write_text(json.dumps({"profiles": {"v": acc.profile}}))
    del acc
    syn2 = dict(syn)
    del syn2["calibrate"]
    p.write_text(json.dumps(dict(c, synthetic=syn2, profile_path=str(prof), profile_sha256=sha256(prof),
                                 variant="v")))
    r2 = Accelerator(p).predict(img, "What is shown?", ["cat", "dog", "bird", "fish"])
    assert r2["logits"] == r1["logits"]


def test_engine_attention_rowwise_output_is_bit_identical():
    """Engine(attn_q8=True): the attention writes the o projection's rowwise FP8 input itself
    (`ffb_attention_rowwise`), one launch per layer fewer; the logits equal the default
    forward's (attention + `ffb_quantize_fp8`) bit for bit, eager and through the graph."""
    dims, src, req, layout = small_case(MODELS["4B"], 3, vocab=4096)
    pm = PackedModel(dims, src, device=DEV)
    T = layout.bucket
    out = []
    for flag in (False, True):
        eng = Engine(pm, attn_q8=flag)
        assert eng.attn_uses_q8(T) == flag
        assert eng.launches_per_forward(T) == Engine(pm).launches_per_forward(T) - (2 if flag else 0)
        ids, vis, deep = req["ids"][:T].to(DEV), req["visual"].to(DEV), [x.to(DEV) for x in req["deep"]]
        z, _ = eng.forward(ids, vis, deep, req["pick"], req["k"], layout.image_start, layout.grid_h, layout.grid_w,
                           T=T)
        entry = eng.capture(T, layout.image_start, layout.nv, layout.grid_h, layout.grid_w, req["k"], len(deep))
        zg, _ = eng.replay(entry, req["ids"][:layout.n_tokens].to(DEV), vis, deep, req["pick"])
        out.append((z.cpu().clone(), zg.cpu().clone()))
    assert torch.equal(out[0][0].view(torch.int32), out[1][0].view(torch.int32))
    assert torch.equal(out[0][1].view(torch.int32), out[1][1].view(torch.int32))

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
    the tensor cores do (with the engine's K splits) and its norms bit-exactly, so only
    attention's rounding (exp, summation order) separates the two, and an FP8 network
    amplifies it.  Its size is measured as the oracle's own change when its softmax runs
    over 32-key blocks instead of 64: the engine must stay within TOL or that floor, i.e. no
    farther from the oracle than an equally valid blocking of the oracle itself."""
    dims, src, req, layout = small_case(MODELS[name], n_layers, vocab=4096)
    eng, z, _ = _run_engine(dims, src, req, layout)
    sp = _splits(eng, layout.bucket)
    zr, _ = _oracle(dims, src, req, layout, splits=sp)
    zr32, _ = _with_attention_block(32, _oracle, dims, src, req, layout, splits=sp)
    floor = (zr - zr32).abs().max().item()
    err = _check_logits(z, zr, max(TOL, floor))
    print(f"\n{name} {n_layers} layers free-running |dz| = {err:.3g} (oracle noise floor {floor:.3g})")


@pytest.mark.parametrize("name", ["2B", "4B"])
def test_layer_ops_teacher_forced(name):
    """Every op of a full decoder layer at the model's real shapes (T=320), each checked
    against the oracle fed with the engine's own inputs to that op: quantised bytes and
    norms bit-exact, GEMM outputs within one bf16 rounding of the exact FP8 products."""
    from fastforward_b200.engine import GemmPlan
    from fastforward_b200 import _lib as L
    from tests._util import assert_bf16_near, assert_bytes_equal
    dims, src, req, layout = small_case(MODELS[name], 2, vocab=4096)
    eng = Engine(PackedModel(dims, src, device=DEV), autotune=False)
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
    om = oracle.quantized_model(dims, src, "rowwise")
    lay, eps, H, HQ, HK, I = om["layers"][0], dims.eps, dims.hidden, dims.hq, dims.hk, dims.inter
    pos = oracle.mrope_position_ids(T, 0, 32, 32)
    cos, sin = oracle.mrope_cos_sin(pos, dims.d, dims.theta)

    def lin(a8, sa, w):  # the oracle's FP8 linear on the engine's own quantised input
        return oracle.qwen_path._fp8_linear(a8, sa, w["w8"], w["w_scale"], 1)

    q, s = oracle.quantize_rows(oracle.rms_one(S["h0"], lay["in_norm"], eps))
    assert_bytes_equal(S["x8"], q[:T], "x8")
    assert torch.equal(S["xs"], s[:T])
    qkv = lin(S["x8"], S["xs"], lay["qkv"]).to(torch.bfloat16)  # fused qkv GEMM + norm + RoPE
    rq, rk = oracle.qk_pair(qkv[:, :HQ * 128].reshape(T, HQ, 128), qkv[:, HQ * 128:(HQ + HK) * 128].reshape(T, HK, 128),
                            lay["q_norm"], lay["k_norm"], cos, sin)
    assert_bytes_equal(S["yq"], rq, "yq")
    assert_bytes_equal(S["yk"], rk, "yk")
    assert_bytes_equal(S["yv"], qkv[:, (HQ + HK) * 128:].reshape(T, HK, 128).transpose(0, 1), "yv")
    att = oracle.attention_direct(S["yq"], S["yk"], S["yv"], 128 ** -0.5).reshape(T, HQ * 128)
    torch.testing.assert_close(S["attn"].float(), att.float(), atol=2e-2, rtol=2e-2)
    q, s = oracle.quantize_rows(S["attn"])
    assert_bytes_equal(S["o8"], q[:T], "o8")
    o = lin(S["o8"], S["os"], lay["o"]).to(torch.bfloat16)
    h_mid = (S["h0"].float() + o.float()).to(torch.bfloat16)
    assert_bytes_equal(S["hB"], h_mid, "residual after attention")
    q, s = oracle.quantize_rows(oracle.rms_one(S["hB"], lay["post_norm"], eps))
    assert_bytes_equal(S["post8"], q[:T], "post8")
    gu = lin(S["post8"], S["posts"], lay["gateup"]).to(torch.bfloat16)
    act = oracle.swiglu(gu[:, :I], gu[:, I:])
    assert_bytes_equal(S["act"], act, "swiglu")
    q, s = oracle.quantize_rows(S["act"])
    assert_bytes_equal(S["act8"], q[:T], "act8")
    dn = lin(S["act8"], S["acts"], lay["down"]).to(torch.bfloat16)
    h1 = (S["hB"].float() + dn.float()).to(torch.bfloat16).float()
    h1[:layout.nv] = (h1[:layout.nv] + req["deep"][0].float()).to(torch.bfloat16).float()
    assert_bytes_equal(S["hA"], h1.to(torch.bfloat16), "residual after mlp + deepstack")


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
    om = oracle.quantized_model(dims, src, "rowwise", splits=_splits(eng, T))
    from fastforward_b200.mrope import position_ids
    pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
    cos, sin = oracle.mrope_cos_sin(pos, dims.d, dims.theta)
    nv = layout.nv
    stats = []
    for j in range(len(hs) - 1):
        deep = req["deep"][j] if j < len(req["deep"]) else None
        args = (om["layers"][j], hs[j], cos, sin, om["dims"], "rowwise", deep, layout.image_start, nv)
        want = oracle.decoder_layer(*args).float()
        alt = _with_attention_block(32, oracle.decoder_layer, *args).float()  # attention noise floor
        got = hs[j + 1].float()
        scale_max, scale_mean = want.abs().max().item(), want.abs().mean().item()
        err, flo = (got - want).abs(), (alt - want).abs()
        stats.append((j, err.max().item() / scale_max, err.mean().item() / scale_mean,
                      flo.max().item() / scale_max, flo.mean().item() / scale_mean))
    zr, _ = oracle.tail(om["layers"][-1], hs[-1], cos, sin, om["dims"], "rowwise", req["pick"], om["final_norm"],
                        om["head"], req["k"])
    return stats, z.cpu(), zr


@pytest.mark.parametrize("name,n_layers", [("2B", 4), ("4B", 3)])
def test_layers_teacher_forced(name, n_layers):
    """Whole layers on the engine's own inputs: only attention's rounding differs, so each
    layer's deviation stays within 2% of the output's max (0.1% on average) or within the
    oracle's own change under a different softmax blocking, whichever is larger."""
    stats, z, zr = _teacher_forced(name, n_layers)
    print(f"\n{name} per-layer (max rel, mean rel, floor max, floor mean):", stats, "tail",
          (z - zr).abs().max().item())
    for j, max_rel, mean_rel, fmax, fmean in stats:
        assert max_rel <= max(0.02, fmax) and mean_rel <= max(1e-3, fmean), stats[j]
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
    print("\n2B full depth per-layer (max rel, mean rel, floor max, floor mean):", stats, "tail",
          (z - zr).abs().max().item())
    for j, max_rel, mean_rel, fmax, fmean in stats:
        assert max_rel <= max(0.02, fmax) and mean_rel <= max(1e-3, fmean), stats[j]
    _check_logits(z, zr)

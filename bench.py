"""Benchmark: Qwen3-VL-4B-shaped FP8 prefill (T=320) + choice scoring on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload 4B-fp8-T320] [--batch B (request streams)]

One step = one request: prefill of T=320 tokens (256 visual rows on a 16x16 merged grid +
64 text ids) through all 36 layers and the 4-choice scoring, replayed from one CUDA graph.
`value` = whole-job prefill tokens/s with inputs resident in HBM (device-timed with CUDA
events, max over ranks); `e2e` = the same metric through `Accelerator.prefill_score_stream`
over the K steps' requests in pinned host memory (every step's H2D of ids/visual/deepstack
rows and D2H of its logits inside the timed region, neighbouring requests' copies
overlapped with the forwards), with one `Accelerator.prefill_score` call per request
(nothing overlapped) reported beside it.  Weights (3.6 GB FP8) exceed the 126 MB L2, so no
flush is needed between steps.  N > 1 (torchrun): one independent replica per GPU, no
collective on the data path ("replicas only"; requests are independent).

`--impl reference` times the reference's arithmetic on the host CPU: the oracle's
restatement of the reference path (the reference itself is Triton/CUDA-only and has no
CPU path), every step one whole request (all layers + scoring).  The GPU arm's own
`cpu_baseline` is a bounded sample of that: a few timed decoder layers scaled to the model.
"""
import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "prefill tok/s (Qwen3-VL-4B FP8, T=320 prefill + 4-choice scoring); p50 latency in ms_per_step"
UNIT = "tok/s"


def metric_for(workload):
    """The headline metric for the default workload; the same wording for the others."""
    if workload == "4B-fp8-T320":
        return METRIC
    from fastforward_b200.config import WORKLOADS
    name, layout, mode = WORKLOADS[workload]
    quant = {"int4": "W4A16", "static": "FP8 static-scale"}.get(mode, "FP8")
    return (f"prefill tok/s (Qwen3-VL-{name} {quant}, T={layout.bucket} prefill + {layout.k}-choice scoring); "
            "p50 latency in ms_per_step")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="4B-fp8-T320")
    p.add_argument("--cpu-layers", type=int, default=2, help="decoder layers in the CPU sample")
    p.add_argument("--batch", type=int, default=1,
                   help="request streams: requests concatenated into one forward (Engine.forward_batch); "
                        "1 = one graph replay per request")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extra", action="store_true",
                   help="N > 1: skip the 8B stream (C4) and 32B tensor-parallel (C5) blocks of the headline line")
    p.add_argument("--extra-requests", type=int, default=128,
                   help="N > 1: requests of the 8B stream block (C4)")
    p.add_argument("--cpu-threads", type=int, default=0,
                   help="--impl reference: host threads (0 = all; the reference runtime sets 1, api.py:60)")
    p.add_argument("--cpu-layer", action="store_true",
                   help="--impl reference: time one decoder layer of the workload's model per step (C1: "
                        "--workload 2B-layer-T512) instead of whole requests")
    p.add_argument("--layers", type=int, default=None,
                   help="build only this many decoder layers (same shapes; for small profiler captures)")
    p.add_argument("--tp-peer", action="store_true",
                   help="N > 1: also time the 32B tensor-parallel model with its reductions through peer memory "
                        "(Engine(peer=True)) beside the NCCL default")
    p.add_argument("--vision-ncu", action="store_true",
                   help="run only the 4B vision tower and replay one forward inside a profiler range")
    p.add_argument("--ncu-range", action="store_true",
                   help="after set-up, replay one forward inside a cudaProfilerStart/Stop range and exit "
                        "(for `ncu --profile-from-start off`); prints no bench line")
    return p.parse_args()


def read_peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sustained=d.get("bf16_tflops_sustained"),
                    src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, src="fallback")


class Clocks:
    """nvidia-smi sampling (every 20 ms) of one GPU during the timed region.  The sampler is
    started and its first sample awaited before the region begins (nvidia-smi takes ~0.1 s
    to start, longer than a short timed region); the summary keeps the samples taken
    inside the region (timestamps), or the first one after it starts if it was too short
    for any."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def __enter__(self):
        import datetime
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            deadline = time.time() + 5.0
            while time.time() < deadline and not Path(self.path).read_text().strip():
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.t0 = datetime.datetime.now()
        return self

    def __exit__(self, *a):
        import datetime
        self.t1 = datetime.datetime.now()
        time.sleep(0.05)  # the sample that covers the region's end
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        import datetime
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) >= 10:
                    rows.append(f)
        except Exception:
            pass
        if not rows:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["unsampled"], samples=0)

        def ts(r):
            try:
                return datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                return None
        inside = [r for r in rows if ts(r) and self.t0 and self.t0 <= ts(r) <= self.t1 + datetime.timedelta(seconds=0.03)]
        if not inside:
            after = [r for r in rows if ts(r) and self.t0 and ts(r) >= self.t0]
            inside = after[:1] or rows[-1:]
        sm = [float(r[2]) for r in inside if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in inside:
            for n, v in zip(names, r[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=float(inside[0][3]),
                    reasons=sorted(reasons), samples=len(inside))


class CpuSample:
    """The oracle (the reference path's arithmetic restated on the CPU) on the workload's
    model: built once (n_layers decoder layers + the tail layer), then timed one decoder
    layer, the tail, or a whole request at a time.

    Its linears multiply the e4m3 values in fp32 (products exact, fp32 sums, then the
    reference's scales and bf16 rounding).  CPU `torch._scaled_mm` would be the same
    arithmetic but is no usable CPU implementation: it accepts only per-tensor scales and
    took 240 s for one 320 x 19456 x 2560 GEMM on this image (0.1 s as an fp32 matmul)."""

    def __init__(self, dims, layout, threads, n_layers=1, mode="rowwise"):
        import torch
        import oracle
        from fastforward_b200.synthetic import make_model_bf16, make_request
        from fastforward_b200.mrope import position_ids
        torch.set_num_threads(threads)
        # a CPU implementation times ordinary fp32 GEMMs of the e4m3 values, not the
        # oracle's bit-level tensor-core accumulation model
        oracle.set_accumulation("fp32")
        self.o = oracle
        self.dims, self.layout = dims, layout
        src = make_model_bf16(dims, seed=0, device="cpu", layers=n_layers + 1)
        self.mode = mode
        self.om = oracle.quantized_model(dims, src, mode)
        del src
        self.req = make_request(dims, layout, seed=1)
        T = layout.bucket
        self.pos = position_ids(T, layout.image_start, layout.grid_h, layout.grid_w)
        self.cos, self.sin = oracle.mrope_cos_sin(self.pos, dims.d, dims.theta)
        self.h = oracle.embed_rows(self.om["embed"], self.req["ids"][:T], self.req["visual"], layout.image_start)
        self.n_layers = n_layers

    def layer(self, j=0):
        t0 = time.perf_counter()
        self.o.decoder_layer(self.om["layers"][j], self.h, self.cos, self.sin, self.om["dims"], self.mode,
                             self.req["deep"][0], self.layout.image_start, self.layout.nv)
        return time.perf_counter() - t0

    def tail(self):
        t0 = time.perf_counter()
        om = self.om
        self.o.tail(om["layers"][self.n_layers], self.h, self.cos, self.sin, om["dims"], self.mode,
                    self.req["pick"], om["final_norm"], om["head"], self.req["k"])
        return time.perf_counter() - t0

    def request(self):
        """One whole request: embedding, every decoder layer, the pick-row tail and the
        option scoring (`oracle.prefill_score`).  Returns seconds."""
        T = self.layout.bucket
        t0 = time.perf_counter()
        self.o.prefill_score(self.om, self.req["ids"][:T], self.req["visual"], self.req["deep"], self.pos,
                             self.req["pick"], self.req["k"], mode=self.mode, image_start=self.layout.image_start)
        return time.perf_counter() - t0

    def full_request_seconds(self, t_layer, t_tail):
        return t_layer * (self.dims.layers - 1) + t_tail


def bench_config(workload, name, mode, T, world, weight_bytes):
    """The `config` object of a bench line (the same for both arms)."""
    tp_mode = name == "32B" and world > 1
    return dict(workload=workload, model=f"Qwen3-VL-{name}-shaped", global_batch=1 if tp_mode else world,
                seq_len=T, parallelism=f"tp{world}" if tp_mode else f"replicas{world}", quant=mode,
                l2=f"weights ({weight_bytes / 1e9:.1f} GB) exceed L2; no flush needed", tokens_per_step=T)


def run_reference(args):
    """The reference's arithmetic for this path on the host CPU, whole requests: every step
    is one full prefill + scoring of the workload's model (all layers), all host threads.
    The reference itself has no CPU path (`api.py:56-57` refuses one) and its kernels are
    Triton/CUDA, so its CPU implementation here is the oracle's restatement."""
    import torch
    from fastforward_b200.config import MODELS, WORKLOADS
    name, layout, mode = WORKLOADS[args.workload]
    dims = MODELS[name]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return
    threads = args.cpu_threads or os.cpu_count() or 1
    t_build = time.perf_counter()
    cs = CpuSample(dims, layout, threads, n_layers=1 if args.cpu_layer else dims.layers - 1, mode=mode)
    t_build = time.perf_counter() - t_build
    times = []
    for i in range(args.warmup + args.steps):
        t = cs.layer() if args.cpu_layer else cs.request()
        if i >= args.warmup:
            times.append(t)
    T = layout.bucket
    per_req = statistics.median(times)
    value = T / per_req
    wfac = 0.5 + 2 / 128 if mode == "int4" else 1.0
    weight_bytes = dims.params_per_layer() * dims.layers * wfac
    cpu_model = ""
    try:
        cpu_model = next(l.split(":", 1)[1].strip() for l in open("/proc/cpuinfo") if l.startswith("model name"))
    except (OSError, StopIteration):
        pass
    line = dict(metric=metric_for(args.workload), value=value, unit=UNIT, n_gpus=world, steps=args.steps,
                warmup=args.warmup, ms_per_step=per_req * 1e3, higher_is_better=True,
                scaling="strong" if (name == "32B" and world > 1) else "weak", vs_baseline=None,
                dtype="int4-bf16" if mode == "int4" else "fp8-e4m3",
                data="synthetic (seeded N(0,0.02) weights, N(0,1) visual/deepstack rows, uniform text ids)",
                impl="reference", config=bench_config(args.workload, name, mode, T, world, weight_bytes),
                latency_ms=dict(p50=per_req * 1e3, min=min(times) * 1e3, max=max(times) * 1e3),
                cpu_baseline=dict(value=value, unit=UNIT, cores=threads, kind="port",
                                  sample=(f"one decoder layer per step ({args.steps} timed, +{args.warmup} warm-up)"
                                          if args.cpu_layer else
                                          f"whole requests: {args.steps} timed (+{args.warmup} warm-up) full "
                                          f"{dims.layers}-layer prefills + scoring") + f" at T={T} on {threads} threads "
                                         f"({cpu_model}); fp32 GEMMs of the e4m3 values; model built in "
                                         f"{t_build:.0f} s (untimed)"),
                e2e=dict(value=value, unit=UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- GPU side

PROFILE_GATEUP = ROOT / "profiles" / "fp8_gemm_gateup_4B_T320.md"


def ncu_traffic(workload, role):
    """DRAM bytes (read + write) per launch of the dominant GEMM, from the committed ncu
    summary of that kernel on this workload (None when there is no such summary)."""
    import re
    if workload != "4B-fp8-T320" or role != "gateup" or not PROFILE_GATEUP.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*(\d+)", PROFILE_GATEUP.read_text())
    return int(m.group(1)) if m else None


def gemm_roofline(eng, T, peaks, reps=20):
    """Times each GEMM role of the forward standalone (same shapes and plans as inside the
    graph) with CUDA events; returns per-role stats and the dominant role."""
    import torch
    m = eng.m
    b = eng.buffers_for(T)
    pl = eng._plans(T)
    s = torch.cuda.current_stream()
    eng._s = s.cuda_stream
    int4 = m.mode == "int4"
    if int4:  # bf16 GEMM inputs
        roles = {"qkv": (b.xb, None, b.qkv), "o": (b.attn, None, b.lin_out), "gateup": (b.postb, None, b.act),
                 "down": (b.act, None, b.lin_out)}
    else:
        roles = {"qkv": (b.x8, b.xs, b.qkv), "o": (b.o8, b.os, b.lin_out), "gateup": (b.post8, b.posts, b.act),
                 "down": (b.act8, b.acts, b.lin_out)}
    out = {}
    cos, sin = next(iter(eng.tables.values()))
    for role, (a, sc, o) in roles.items():
        p = pl[("full", role)]

        rowwise = m.mode == "rowwise"

        def one(i):
            lay_i = m.layers[i % m.depth]
            if role == "qkv":  # qkv GEMM (+ the fused QK-norm + RoPE epilogue in FP8 mode)
                eng._qkv(p, b, lay_i, cos, sin, T, int4, rowwise)
            elif int4:
                eng._w4(p, a, lay_i.lin[role], o, b.ws)
            else:
                eng._gemm(p, a, sc if rowwise else lay_i.ascale[role], lay_i.lin[role], o, b.ws, rowwise)
        for i in range(3):
            one(i)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(s)
        for i in range(reps):
            one(i)
        ev[1].record(s)
        torch.cuda.synchronize()
        dt = ev[0].elapsed_time(ev[1]) / reps * 1e-3
        flops = 2.0 * p.m * p.n * p.k
        wbytes = p.n * p.k * (0.5 + 2 / 128 if int4 else 1)
        out[role] = dict(m=p.m, n=p.n, k=p.k, bn=p.bn, splits=p.splits, us=dt * 1e6, tflops=flops / dt / 1e12,
                         weight_gbs=wbytes / dt / 1e9)
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist
    from fastforward_b200.config import MODELS, WORKLOADS
    from fastforward_b200.engine import Engine, PackedModel
    from fastforward_b200.synthetic import make_model_bf16, make_request

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    name, layout, mode = WORKLOADS[args.workload]
    dims = MODELS[name]
    T = layout.bucket
    peaks = read_peaks()
    # the 32B model is tensor-parallel over the ranks (one request stream shared by all of
    # them); the smaller models run one independent replica per rank
    tp_mode = name == "32B" and world > 1

    with torch.no_grad():
        src = make_model_bf16(dims, seed=0, device=dev, layers=args.layers)
        profile = None
        if mode == "static":  # calibrate the static activation bounds on one request first
            from fastforward_b200.engine import calibrate_profile
            r = make_request(dims, layout, seed=999, device=dev)
            profile, _ = calibrate_profile(
                dims, src, [dict(ids=r["ids"][:T], visual=r["visual"], deep=r["deep"], pick=r["pick"], k=r["k"],
                                 image_start=layout.image_start, grid_h=layout.grid_h, grid_w=layout.grid_w, T=T)],
                device=dev, tp=(rank, world) if tp_mode else None, tp_group=dist.group.WORLD if tp_mode else None)
        pm = PackedModel(dims, src, mode=mode, device=dev, free_source=True, tp=(rank, world) if tp_mode else None,
                         profile=profile)
        del src
        torch.cuda.empty_cache()
        eng = Engine(pm, tp_group=dist.group.WORLD if tp_mode else None)
        # requests: a pool of distinct synthetic requests in pinned host memory (the same
        # requests on every rank of a tensor-parallel group)
        n_pool = 8
        reqs = []
        for i in range(n_pool):
            r = make_request(dims, layout, seed=(0 if tp_mode else 1000 * rank) + i)
            reqs.append(dict(ids=r["ids"][:layout.n_tokens].pin_memory(), visual=r["visual"].pin_memory(),
                             deep=[x.pin_memory() for x in r["deep"]], pick=r["pick"], k=r["k"]))
        entry = eng.capture(T, layout.image_start, layout.nv, layout.grid_h, layout.grid_w, layout.k, dims.deepstack)
        dev_reqs = [dict(ids=r["ids"].to(dev), visual=r["visual"].to(dev), deep=[x.to(dev) for x in r["deep"]],
                         pick=r["pick"]) for r in reqs]
        torch.cuda.synchronize()

        # ---- value: graph replays, inputs resident in HBM
        def stage_dev(r):
            b = entry["buffers"]
            b.ids[:r["ids"].shape[0]].copy_(r["ids"])
            entry["visual"][:layout.nv].copy_(r["visual"])
            for dst, src_ in zip(entry["deep"], r["deep"]):
                dst.copy_(src_)
            b.pick.fill_(r["pick"])

        for i in range(args.warmup):
            stage_dev(dev_reqs[i % n_pool])
            entry["graph"].replay()
        torch.cuda.synchronize()
        if args.ncu_range:
            torch.cuda.profiler.start()
            entry["graph"].replay()
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            if rank == 0:
                print(json.dumps(dict(ncu_range="one graph replay", workload=args.workload, layers=pm.depth,
                                      launches=eng.launches_per_forward(T))), flush=True)
            return
        s = torch.cuda.current_stream()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        # stage all inputs for the timed steps ahead: each step's request already in HBM
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with Clocks(local) as clk:
            t_all0 = torch.cuda.Event(enable_timing=True)
            t_all1 = torch.cuda.Event(enable_timing=True)
            t_all0.record(s)
            for i in range(args.steps):
                starts[i].record(s)
                entry["graph"].replay()
                ends[i].record(s)
            t_all1.record(s)
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        total_s = t_all0.elapsed_time(t_all1) * 1e-3
        lat = sorted(a.elapsed_time(b_) for a, b_ in zip(starts, ends))
        p50 = lat[len(lat) // 2]
        p99 = lat[min(len(lat) - 1, int(round(0.99 * (len(lat) - 1))))]
        if world > 1:
            t = torch.tensor([total_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total_s = t.item()
        streams = 1 if tp_mode else world  # independent request streams
        value = streams * args.steps * T / total_s

        # ---- e2e: through the public entry with host (pinned) buffers, H2D + D2H per step
        from fastforward_b200.api import Accelerator

        class _Bound(Accelerator):
            def __init__(self, engine, dims_, buckets):
                import threading
                self.engine = engine
                self.dims = dims_
                self.device = dev
                self.lock = threading.RLock()
                self.buckets = buckets
        from fastforward_b200.config import BUCKETS
        acc = _Bound(eng, dims, BUCKETS)
        stream_reqs = [dict(ids=reqs[i % n_pool]["ids"], visual=reqs[i % n_pool]["visual"],
                            deep=reqs[i % n_pool]["deep"], k=reqs[i % n_pool]["k"], image_start=layout.image_start,
                            grid_h=layout.grid_h, grid_w=layout.grid_w) for i in range(args.steps)]
        acc.prefill_score_stream(stream_reqs[:max(args.warmup, 2)])
        # one call per request (no overlap between requests): reported beside the streamed e2e
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(s)
        n_single = min(args.steps, 50)
        for r in stream_reqs[:n_single]:
            acc.prefill_score(r["ids"], r["visual"], r["deep"], r["k"], layout.image_start, layout.grid_h,
                              layout.grid_w)
        c1.record(s)
        torch.cuda.synchronize()
        single_value = streams * n_single * T / (c0.elapsed_time(c1) * 1e-3)
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        w0 = time.perf_counter()
        acc.prefill_score_stream(stream_reqs)  # every step: H2D of its inputs, forward, D2H of its answer
        e1.record(s)
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
        e2e_s = max(e0.elapsed_time(e1) * 1e-3, 0.0)
        if world > 1:
            t = torch.tensor([e2e_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = t.item()
        e2e_value = streams * args.steps * T / e2e_s
        r0 = reqs[0]
        h2d = (r0["ids"].numel() * 8 + r0["visual"].numel() * 2 + sum(x.numel() * 2 for x in r0["deep"]) + 8)
        d2h = 2 * layout.k * 4

        # ---- roofline of the dominant kernel (the GEMM), standalone event timing
        roles = gemm_roofline(eng, T, peaks)
        int4 = mode == "int4"
        tc_peak = peaks["bf16"] if int4 else 2.0 * peaks["bf16"]
        wfac = 0.5 + 2 / 128 if int4 else 1.0  # weight bytes per parameter
        dom = max(roles, key=lambda k: roles[k]["us"])
        dr = roles[dom]
        if int4:
            peak_note = f"bf16 dense = {peaks['src']} cuBLAS bf16 {peaks['bf16']} TFLOP/s"
        else:
            peak_note = f"FP8 dense = 2 x {peaks['src']} cuBLAS bf16 {peaks['bf16']} TFLOP/s"
        roofline = dict(bound="tensor", achieved=dr["tflops"], peak=tc_peak, unit="TFLOP/s",
                        frac=dr["tflops"] / tc_peak, traffic=ncu_traffic(args.workload, dom),
                        traffic_note="ncu dram__bytes_read.sum + dram__bytes_write.sum per launch; "
                                     "algorithmic weight bytes per launch = %d" % int(dr["n"] * dr["k"] * wfac),
                        kernel=f"{'w4a16' if int4 else 'fp8'}_gemm_kernel ({dom})",
                        peak_note=peak_note,
                        weight_stream_gbs=dr["weight_gbs"], hbm_peak_gbs=peaks["hbm"],
                        per_role={k: {kk: (round(vv, 3) if isinstance(vv, float) else vv) for kk, vv in v.items()}
                                  for k, v in roles.items()})
        gemm_us = sum(v["us"] for v in roles.values()) * (dims.layers - 1)
        # whole-forward algorithmic roofline: max(FLOPs / tensor peak, weight bytes / HBM)
        P = dims.params_per_layer() * dims.layers
        flops = 2.0 * T * P + 4.0 * (T * (T + 1) / 2) * dims.d * dims.hq * dims.layers
        weight_bytes = P * wfac
        # a tensor-parallel group shares one request: its roofline has `world` GPUs' peaks
        gpus_per_stream = world if tp_mode else 1
        t_roof = max(flops / (tc_peak * 1e12), weight_bytes / (peaks["hbm"] * 1e9)) / gpus_per_stream

        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            cs = CpuSample(dims, layout, threads, mode=mode)
            t_layers = [cs.layer() for _ in range(args.cpu_layers)]
            t_tail = cs.tail()
            full = cs.full_request_seconds(statistics.median(t_layers), t_tail)
            cpu = dict(value=T / full, unit=UNIT, cores=threads, kind="port",
                       sample=f"{args.cpu_layers} timed decoder layers (median {statistics.median(t_layers):.2f}s) "
                              f"+ tail ({t_tail:.2f}s) of the {name} model at T={T}, scaled to "
                              f"{dims.layers - 1} layers + tail; fp32 GEMMs of the quantised weights")

    clk_sum = clk.summary()
    launches = eng.launches_per_forward(T) * args.steps
    extra = {}
    if world == 1 and args.workload == "4B-fp8-T320" and not args.no_extra:
        # the image side of the request: the 4B vision tower on the headline's 512 x 512 canvas
        extra["vision_4b"] = vision_measure(args, dev, peaks)
    if world > 1 and args.workload == "4B-fp8-T320" and not args.no_extra:
        # the multi-GPU configurations besides the headline's replicas, in the same line:
        # the 8B request stream served by N replicas (C4) and the 32B model tensor-parallel
        # over the N ranks (C5)
        del entry
        eng.graphs.clear()
        del eng, pm
        torch.cuda.empty_cache()
        extra["stream_8b"] = _summarise_stream(stream_measure(args, "8B-fp8-stream", world, rank, local, dev,
                                                              n_req=args.extra_requests))
        extra["tp_32b"] = tp32b_measure(args, world, rank, local, dev)
    if rank == 0:
        line = dict(metric=metric_for(args.workload), value=value, unit=UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
                    ms_per_step=p50, higher_is_better=True, scaling="strong" if tp_mode else "weak",
                    vs_baseline=None,
                    dtype="int4-bf16" if int4 else "fp8-e4m3", data="synthetic (seeded N(0,0.02) weights, N(0,1) visual/deepstack rows, uniform text ids)",
                    config=bench_config(args.workload, name, mode, T, world, weight_bytes),
                    latency_ms=dict(p50=p50, p99=p99, mean=total_s / args.steps * 1e3),
                    requests_per_s=streams * args.steps / total_s,
                    roofline=roofline,
                    forward_roofline=dict(flops=flops, weight_bytes=weight_bytes, t_roofline_ms=t_roof * 1e3,
                                          frac=t_roof * 1e3 / p50,
                                          note="max(FLOPs/tensor peak, weights/HBM) / GPUs per request / p50"),
                    gemm_share_est=gemm_us * 1e-3 / p50,
                    e2e=dict(value=e2e_value, unit=UNIT, h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                             wall_s=wall, api="Accelerator.prefill_score_stream",
                             one_call_per_request=dict(value=single_value, unit=UNIT, api="Accelerator.prefill_score",
                                                       requests=n_single)),
                    gpu_launches=launches,
                    clocks=clk_sum, cpu_baseline=cpu, **extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if not extra:
            del entry
            eng.graphs.clear()
            eng.close_peers()
        dist.destroy_process_group()


def vision_flops(v, n_p):
    """Useful FLOPs of one vision-tower forward over n_p patches (head dim unpadded)."""
    c, i, m2 = v.hidden, v.inter, v.merge * v.merge
    per_block = 2 * n_p * (c * 3 * c + c * c + 2 * c * i) + 4 * n_p * n_p * c
    merger = 2 * (n_p // m2) * (c * m2 * c * m2 + c * m2 * v.out_hidden)
    return 2 * n_p * 3 * v.temporal * v.patch * v.patch * c + v.depth * per_block + (len(v.deepstack) + 1) * merger


def vision_measure(args, dev, peaks, name="4B", side=512):
    """The vision tower in front of the language path (C1-C4's image side): seeded
    synthetic weights of the family's published vision config, a side x side canvas per
    image (32 x 32 patches -> the 256 visual rows of the headline layout).  Each step packs
    one canvas already in HBM (ffb_pack_rgb) and replays the tower's CUDA graph; device
    time with CUDA events; the 600 MB of weights exceed L2, so every step streams them."""
    import torch
    from fastforward_b200.config import VISION_MODELS
    from fastforward_b200.ops import pack_rectangle
    from fastforward_b200.synthetic import make_vision_bf16
    from fastforward_b200.vision import VisionTower
    v = VISION_MODELS[name]
    vt = VisionTower(v, make_vision_bf16(v, seed=0, device=dev), device=dev)
    grid = side // v.patch
    n_p = grid * grid
    g = torch.Generator().manual_seed(7)
    canvases = [torch.randint(0, 256, (side, side, 3), generator=g, dtype=torch.uint8).to(dev) for _ in range(4)]
    graph = vt.capture(grid, grid)
    buf = vt.bufs[n_p]
    for i in range(max(args.warmup, 3)):
        pack_rectangle(canvases[i % 4], pixels=buf.pixels)
        graph.replay()
    torch.cuda.synchronize()
    if getattr(args, "vision_ncu", False):
        torch.cuda.profiler.start()
        pack_rectangle(canvases[0], pixels=buf.pixels)
        graph.replay()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        return dict(ncu_range="one vision forward", launches=1 + VisionTower.launches(v))
    steps = max(min(args.steps, 50), 5)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        ev[i][0].record()
        pack_rectangle(canvases[i % 4], pixels=buf.pixels)
        graph.replay()
        ev[i][1].record()
    torch.cuda.synchronize()
    ms = sorted(a.elapsed_time(b) for a, b in ev)
    p50 = ms[len(ms) // 2]
    flops = vision_flops(v, n_p)
    # end to end: a host canvas (pinned) to the merged rows in host memory
    host = [c.cpu().pin_memory() for c in canvases]
    out = torch.empty(buf.merged.shape, dtype=buf.merged.dtype).pin_memory()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        canvases[i % 4].copy_(host[i % 4], non_blocking=True)
        pack_rectangle(canvases[i % 4], pixels=buf.pixels)
        graph.replay()
        out.copy_(buf.merged, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / steps
    tflops = flops / (p50 * 1e-3) / 1e12
    return dict(model=f"{name} vision tower ({v.depth} blocks, hidden {v.hidden}, deepstack {list(v.deepstack)})",
                canvas=f"{side}x{side}", patches=n_p, merged_rows=n_p // 4, steps=steps, ms_per_image_p50=p50,
                images_per_s=1e3 / p50, tflops=tflops, frac_of_bf16_peak=tflops / peaks["bf16"],
                peak_note=f"{peaks['bf16']} TFLOP/s bf16 ({peaks['src']}, burst)", flops_per_image=flops,
                gpu_launches_per_image=1 + VisionTower.launches(v),
                e2e=dict(ms_per_image=e2e_ms, h2d_bytes=side * side * 3, d2h_bytes=out.numel() * 2,
                         api="VisionTower graph: pinned canvas -> pack_rgb -> tower -> merged rows to host"))


def _summarise_stream(line):
    """The C4 block of a multi-GPU headline line (rank 0; None elsewhere)."""
    if line is None:
        return None
    return dict(workload=line["config"]["workload"], requests=line["steps"], value=line["value"], unit=line["unit"],
                latency_ms=line["latency_ms"], prefill_tok_per_s=line["prefill_tok_per_s"],
                e2e=dict(value=line["e2e"]["value"], unit=line["e2e"]["unit"], api=line["e2e"]["api"]),
                graphs=line["config"]["graphs"], parallelism=line["config"]["parallelism"], clocks=line["clocks"])


def tp32b_measure(args, world, rank, local, dev):
    """C5: the 32B FP8 model at T = 1024 tensor-parallel over the `world` ranks (each rank
    one shard; the process group is the caller's).  Graph replays device-timed, max over
    ranks; the two all-reduces of every decoder layer (fp32 [T, H] partials of o_proj and
    down_proj) and the per-token scale MAX all-reduces are timed alone with CUDA events.
    Returns rank 0's block (None elsewhere)."""
    import torch
    import torch.distributed as dist
    from fastforward_b200.config import MODELS, WORKLOADS
    from fastforward_b200.engine import Engine, PackedModel
    from fastforward_b200.synthetic import make_model_bf16, make_request
    wl = "32B-fp8-T1024"
    name, layout, mode = WORKLOADS[wl]
    dims = MODELS[name]
    T = layout.bucket
    s = torch.cuda.current_stream()
    with torch.no_grad():
        src = make_model_bf16(dims, seed=0, device=dev)
        pm = PackedModel(dims, src, mode=mode, device=dev, free_source=True, tp=(rank, world))
        del src
        torch.cuda.empty_cache()
        req = make_request(dims, layout, seed=1, device=dev)
        ids = req["ids"][:layout.n_tokens]
        steps = max(5, min(args.steps, 20))

        def time_engine(peer, clocks):
            """(seconds for `steps` replays max over ranks, sorted latencies, logits, engine's
            reduction path) of one engine's graph."""
            eng = Engine(pm, tp_group=dist.group.WORLD, peer=peer)
            entry = eng.capture(T, layout.image_start, layout.nv, layout.grid_h, layout.grid_w, layout.k,
                                len(req["deep"]))
            for _ in range(3):
                eng.replay(entry, ids, req["visual"], req["deep"], req["pick"])
            torch.cuda.synchronize()
            dist.barrier()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            with (clocks if clocks is not None else contextlib.nullcontext()):
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0.record(s)
                for a, b in evs:
                    a.record(s)
                    entry["graph"].replay()
                    b.record(s)
                t1.record(s)
                torch.cuda.synchronize()
            tot = torch.tensor([t0.elapsed_time(t1) * 1e-3], device=dev)
            dist.all_reduce(tot, op=dist.ReduceOp.MAX)
            lat_ = sorted(a.elapsed_time(b) for a, b in evs)
            zz = entry["buffers"].logits[:layout.k].float().cpu().tolist()
            path = "peer" if eng.peer is not None else "nccl"
            del entry
            eng.graphs.clear()
            eng.close_peers()
            del eng
            torch.cuda.empty_cache()
            dist.barrier()
            return tot.item(), lat_, zz, path

        clk = Clocks(local)
        total, lat, z, path = time_engine(False, clk)  # the default: NCCL collectives
        if args.tp_peer:
            total_peer, lat_peer, z_peer, peer_path = time_engine(True, None)
        p50 = lat[len(lat) // 2]

        def coll_us(numel, op):  # one collective alone, device-timed, median of 20, max over ranks
            buf = torch.zeros(numel, device=dev)
            for _ in range(3):
                dist.all_reduce(buf, op=op)
            ts = []
            for _ in range(20):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(s)
                dist.all_reduce(buf, op=op)
                b.record(s)
                b.synchronize()
                ts.append(a.elapsed_time(b) * 1e3)
            t = torch.tensor([statistics.median(ts)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.item()
        ar_us = coll_us(T * dims.hidden, dist.ReduceOp.SUM)
        scale_us = coll_us(T, dist.ReduceOp.MAX)
        del pm
        torch.cuda.empty_cache()
        dist.barrier()
    if rank != 0:
        return None
    per_req = total / steps
    n_ar = 2 * (dims.layers - 1) + 2
    return dict(workload=wl, parallelism=f"tp{world}", reductions=path, ms_per_request=per_req * 1e3,
                latency_ms=dict(p50=p50, p99=lat[-1]), tok_per_s=T / per_req, requests_per_s=1.0 / per_req,
                peer_reductions=(dict(ms_per_request=total_peer / steps * 1e3, p50=lat_peer[len(lat_peer) // 2],
                                      path=peer_path, logits_equal=z == z_peer,
                                      note="Engine(peer=True): the full layers' reductions read from peer memory "
                                           "inside ffb_add_rmsnorm_peers / ffb_quantize_fp8_peers")
                                 if args.tp_peer else None),
                allreduce=dict(per_call_us=ar_us, bytes_per_call=T * dims.hidden * 4, calls_per_request=n_ar,
                               busbw_gbs=2 * (world - 1) / world * T * dims.hidden * 4 / (ar_us * 1e-6) / 1e9,
                               share_of_request=n_ar * ar_us * 1e-3 / (per_req * 1e3),
                               scale_max_us=scale_us, scale_calls_per_request=n_ar,
                               note="NCCL all-reduce of one fp32 [T, H] partial / of the [T] scales, timed alone"),
                logits=z, clocks=clk.summary())


def run_stream(args):
    """A stream of independent requests of varying geometry (bucket, image grid, choices),
    one replica per GPU, each rank serving the whole seeded stream.  Every geometry's graph
    is captured during warm-up.  value = requests/s with each request's inputs already in
    HBM (graph replay, device-timed per request, max over ranks); e2e = the same stream
    through `Accelerator.prefill_score` with pinned host inputs (H2D + replay + D2H of the
    logits per request)."""
    import torch
    import torch.distributed as dist
    from fastforward_b200.config import MODELS, STREAMS, BUCKETS, stream_layouts
    from fastforward_b200.engine import Engine, PackedModel
    from fastforward_b200.synthetic import make_model_bf16, make_request
    from fastforward_b200.api import Accelerator

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    line = stream_measure(args, args.workload, world, rank, local, dev)
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def stream_measure(args, workload, world, rank, local, dev, n_req=None):
    """The request-stream measurement of `run_stream` (the process group, if any, is the
    caller's).  Returns rank 0's bench line (None elsewhere); n_req overrides the stream's
    length."""
    import torch
    import torch.distributed as dist
    from fastforward_b200.config import MODELS, STREAMS, BUCKETS, stream_layouts
    from fastforward_b200.engine import Engine, PackedModel
    from fastforward_b200.synthetic import make_model_bf16, make_request
    from fastforward_b200.api import Accelerator
    name, mode, n_stream = STREAMS[workload]
    n_req = n_req or n_stream
    dims = MODELS[name]
    layouts = stream_layouts(n_req, seed=1)
    with torch.no_grad():
        src = make_model_bf16(dims, seed=0, device=dev, layers=args.layers)
        pm = PackedModel(dims, src, mode=mode, device=dev, free_source=True)
        del src
        torch.cuda.empty_cache()
        eng = Engine(pm)
        reqs = []
        for i, lay in enumerate(layouts):
            r = make_request(dims, lay, seed=100 + i)
            reqs.append(dict(lay=lay, ids=r["ids"][:lay.n_tokens].pin_memory(), visual=r["visual"].pin_memory(),
                             deep=[x.pin_memory() for x in r["deep"]], pick=r["pick"], k=r["k"]))
        if args.batch > 1:
            return run_stream_batched(args, eng, reqs, dims, name, mode, n_req, world, rank, local, dev)
        entries = {}
        for r in reqs:  # capture every geometry (and autotune every bucket) before timing
            lay = r["lay"]
            key = (lay.bucket, lay.image_start, lay.nv, lay.grid_h, lay.grid_w, lay.k)
            if key not in entries:
                entries[key] = eng.capture(lay.bucket, lay.image_start, lay.nv, lay.grid_h, lay.grid_w, lay.k,
                                           dims.deepstack)
        dev_reqs = [dict(ids=r["ids"].to(dev), visual=r["visual"].to(dev), deep=[x.to(dev) for x in r["deep"]],
                         pick=r["pick"]) for r in reqs]
        torch.cuda.synchronize()
        s = torch.cuda.current_stream()

        def replay_all(timed):
            ev = []
            for r, d in zip(reqs, dev_reqs):
                lay = r["lay"]
                e = entries[(lay.bucket, lay.image_start, lay.nv, lay.grid_h, lay.grid_w, lay.k)]
                b = e["buffers"]
                b.ids[lay.n_tokens:].zero_()
                b.ids[:lay.n_tokens].copy_(d["ids"])
                e["visual"][:lay.nv].copy_(d["visual"])
                for dst, src_ in zip(e["deep"], d["deep"]):
                    dst[:lay.nv].copy_(src_)
                b.pick.fill_(d["pick"])
                if timed:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(s)
                e["graph"].replay()
                if timed:
                    e1.record(s)
                    ev.append((e0, e1))
            return ev

        for _ in range(max(1, args.warmup)):
            replay_all(False)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        with Clocks(local) as clk:
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(s)
            ev = replay_all(True)
            t1.record(s)
            torch.cuda.synchronize()
        total_s = t0.elapsed_time(t1) * 1e-3
        lat = sorted(a.elapsed_time(b_) for a, b_ in ev)  # per-request graph time, ms
        if world > 1:
            t = torch.tensor([total_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total_s = t.item()
        value = world * n_req / total_s

        class _Bound(Accelerator):
            def __init__(self, engine, buckets):
                import threading
                self.engine = engine
                self.dims = dims
                self.device = dev
                self.lock = threading.RLock()
                self.buckets = buckets
        acc = _Bound(eng, BUCKETS)
        for r in reqs[:8]:
            acc.prefill_score(r["ids"], r["visual"], r["deep"], r["k"], 0, r["lay"].grid_h, r["lay"].grid_w)
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        host_lat = []
        for r in reqs:
            w0 = time.perf_counter()
            acc.prefill_score(r["ids"], r["visual"], r["deep"], r["k"], 0, r["lay"].grid_h, r["lay"].grid_w)
            host_lat.append((time.perf_counter() - w0) * 1e3)
        e1.record(s)
        torch.cuda.synchronize()
        e2e_s = e0.elapsed_time(e1) * 1e-3
        if world > 1:
            t = torch.tensor([e2e_s], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = t.item()
        h2d = sum(r["ids"].numel() * 8 + r["visual"].numel() * 2 + sum(x.numel() * 2 for x in r["deep"]) + 8
                  for r in reqs) / n_req
        d2h = sum(2 * r["k"] * 4 for r in reqs) / n_req
        tokens = sum(r["lay"].n_tokens for r in reqs)
    clk_sum = clk.summary()
    host_lat.sort()
    line = None
    if rank == 0:
        pct = lambda xs, q: xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))]
        line = dict(metric=f"requests/s (Qwen3-VL-{name} FP8, {n_req}-request stream: 64/144/256 visual tokens, "
                           "32-128 text, 2-8 choices); p50 latency in ms_per_step",
                    value=value, unit="req/s", n_gpus=world, steps=n_req, warmup=args.warmup,
                    ms_per_step=pct(lat, 0.5), higher_is_better=True, scaling="weak", vs_baseline=None,
                    dtype="fp8-e4m3", data="synthetic (seeded weights, request geometries and inputs)",
                    config=dict(workload=workload, model=f"Qwen3-VL-{name}-shaped", global_batch=world,
                                seq_len="96-384 (bucketed)", parallelism=f"replicas{world}", quant=mode,
                                graphs=len(entries), prefill_tokens_per_replica=tokens,
                                l2="weights (6.9 GB) exceed L2; no flush needed"),
                    latency_ms=dict(p50=pct(lat, 0.5), p99=pct(lat, 0.99), mean=sum(lat) / len(lat)),
                    prefill_tok_per_s=world * tokens / total_s,
                    e2e=dict(value=world * n_req / e2e_s, unit="req/s", h2d_bytes_per_step=h2d,
                             d2h_bytes_per_step=d2h, api="Accelerator.prefill_score",
                             host_latency_ms=dict(p50=pct(host_lat, 0.5), p99=pct(host_lat, 0.99))),
                    gpu_launches=sum(eng.launches_per_forward(r["lay"].bucket) for r in reqs), clocks=clk_sum,
                    cpu_baseline=None)
    entries.clear()
    eng.graphs.clear()
    del eng, pm, reqs, dev_reqs
    torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
    return line


def run_stream_batched(args, eng, reqs, dims, name, mode, n_req, world, rank, local, dev):
    """The request stream served in batches of `args.batch` consecutive requests, each batch
    one eager forward over the requests' concatenated tokens (`Engine.forward_batch`).
    value = requests/s with inputs in HBM (device-timed, max over ranks); latency = each
    batch's device time (every request of a batch completes with it); e2e = the stream
    through `Accelerator.prefill_score_batch` with pinned host inputs."""
    import torch
    import torch.distributed as dist
    from fastforward_b200.api import Accelerator
    from fastforward_b200.config import BUCKETS
    B = args.batch

    def as_req(r, d):
        lay = r["lay"]
        return dict(ids=d["ids"], visual=d["visual"], deep=d["deep"], pick=lay.n_tokens - 1, k=r["k"],
                    image_start=lay.image_start, grid_h=lay.grid_h, grid_w=lay.grid_w)
    dev_reqs = [as_req(r, dict(ids=r["ids"].to(dev), visual=r["visual"].to(dev), deep=[x.to(dev) for x in r["deep"]]))
                for r in reqs]
    batches = [dev_reqs[i:i + B] for i in range(0, n_req, B)]
    for bt in batches[:max(3, args.warmup)]:
        eng.forward_batch(bt)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s = torch.cuda.current_stream()
    ev = []
    with Clocks(local) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(s)
        for bt in batches:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            eng.forward_batch(bt)
            e1.record(s)
            ev.append((e0, e1))
        t1.record(s)
        torch.cuda.synchronize()
    total_s = t0.elapsed_time(t1) * 1e-3
    lat = sorted(a.elapsed_time(b_) for a, b_ in ev)
    if world > 1:
        t = torch.tensor([total_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_s = t.item()
    value = world * n_req / total_s

    class _Bound(Accelerator):
        def __init__(self, engine, buckets):
            import threading
            self.engine = engine
            self.dims = dims
            self.device = dev
            self.lock = threading.RLock()
            self.buckets = buckets
    acc = _Bound(eng, BUCKETS)
    host_reqs = [as_req(r, r) for r in reqs]
    hb = [host_reqs[i:i + B] for i in range(0, n_req, B)]
    acc.prefill_score_batch(hb[0])
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for bt in hb:
        acc.prefill_score_batch(bt)
    e1.record(s)
    torch.cuda.synchronize()
    e2e_s = e0.elapsed_time(e1) * 1e-3
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = t.item()
    h2d = sum(r["ids"].numel() * 8 + r["visual"].numel() * 2 + sum(x.numel() * 2 for x in r["deep"]) for r in reqs) / n_req
    d2h = sum(2 * r["k"] * 4 for r in reqs) / n_req
    tokens = sum(r["lay"].n_tokens for r in reqs)
    clk_sum = clk.summary()
    if rank == 0:
        pct = lambda xs, q: xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))]
        line = dict(metric=f"requests/s (Qwen3-VL-{name} FP8, {n_req}-request stream: 64/144/256 visual tokens, "
                           "32-128 text, 2-8 choices); p50 latency in ms_per_step",
                    value=value, unit="req/s", n_gpus=world, steps=n_req, warmup=args.warmup,
                    ms_per_step=pct(lat, 0.5), higher_is_better=True, scaling="weak", vs_baseline=None,
                    dtype="fp8-e4m3", data="synthetic (seeded weights, request geometries and inputs)",
                    config=dict(workload=args.workload, model=f"Qwen3-VL-{name}-shaped", global_batch=world * B,
                                seq_len="96-384 per request, requests concatenated at 64-row offsets",
                                parallelism=f"replicas{world}", quant=mode, requests_per_forward=B,
                                prefill_tokens_per_replica=tokens, l2="weights (6.9 GB) exceed L2; no flush needed"),
                    latency_ms=dict(p50=pct(lat, 0.5), p99=pct(lat, 0.99), mean=sum(lat) / len(lat),
                                    note="per batch: every request of a batch completes with it"),
                    prefill_tok_per_s=world * tokens / total_s,
                    e2e=dict(value=world * n_req / e2e_s, unit="req/s", h2d_bytes_per_step=h2d,
                             d2h_bytes_per_step=d2h, api="Accelerator.prefill_score_batch"),
                    gpu_launches=sum(eng.launches_per_batch(len(bt)) for bt in batches), clocks=clk_sum,
                    cpu_baseline=None)
        return line
    return None


# ---------------------------------------------------------------------------- input packing

PACK_WORKLOADS = {"pack-rgb-256": (256, 256), "pack-rgb-320": (320, 320), "pack-rect-192x320": (192, 320)}
PACK_UNIT = "canvases/s"


def _pack_common(args):
    H, W = PACK_WORKLOADS[args.workload]
    n = args.batch if args.batch > 1 else 256  # canvases per step
    patch_rows = (H // 16) * (W // 16)
    bytes_per_canvas = H * W * 3 + patch_rows * 1536 * 2  # u8 canvas read + bf16 rows written
    metric = (f"input packing canvases/s ({H}x{W} RGB u8 -> {patch_rows}x1536 bf16 patch rows, "
              f"{n} canvases per step)")
    return H, W, n, patch_rows, bytes_per_canvas, metric


def run_pack_reference(args):
    """The reference's packing arithmetic on the host (the oracle restatement: the reference
    packs on the GPU only), a bounded sample of canvases per step."""
    import numpy as np
    import oracle
    if int(os.environ.get("RANK", "0")) != 0:
        return
    H, W, n, _, _, metric = _pack_common(args)
    g = np.random.default_rng(0)
    canvases = g.integers(0, 256, (4, H, W, 3), dtype=np.uint8)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        oracle.pack_rgb(canvases[i % 4])
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    value = 1.0 / statistics.median(times)
    print(json.dumps(dict(metric=metric, value=value, unit=PACK_UNIT, n_gpus=args.gpus, steps=args.steps,
                          warmup=args.warmup, ms_per_step=statistics.median(times) * 1e3 * n,
                          higher_is_better=True, scaling="weak", vs_baseline=None, dtype="u8->bf16",
                          data="synthetic (uniform random bytes)", impl="reference",
                          config=dict(workload=args.workload, canvases_per_step=n, parallelism="cpu"),
                          cpu_baseline=dict(value=value, unit=PACK_UNIT, cores=1, kind="port",
                                            sample="one canvas per timed step (numpy restatement), rate per canvas"),
                          e2e=dict(value=value, unit=PACK_UNIT, h2d_bytes_per_step=0, d2h_bytes_per_step=0))),
          flush=True)


def run_pack(args):
    """Input packing (`ffb_pack_rgb_batch`): one step = a batch of canvases packed into patch
    rows.  value = canvases/s with the canvases in HBM (CUDA events, max over ranks; the
    step's footprint exceeds L2 because 4 rotating input/output sets are used); e2e = the same
    through the public staging path: `staging.Packet.stage` (host copy into the pinned packet
    + ONE host->device copy) + `ops.pack_rgb`, reading back the last patch row."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from fastforward_b200 import ops, staging
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    H, W, n, patch_rows, bpc, metric = _pack_common(args)
    peaks = read_peaks()
    g = np.random.default_rng(rank)
    host = [g.integers(0, 256, (n, H, W, 3), dtype=np.uint8) for _ in range(2)]
    sets = 4
    rgb = [torch.from_numpy(host[i % 2]).to(dev) for i in range(sets)]
    pix = [torch.empty((n * patch_rows, 1536), dtype=torch.bfloat16, device=dev) for _ in range(sets)]
    s = torch.cuda.current_stream()
    for i in range(args.warmup):
        ops.pack_rgb(rgb[i % sets], pixels=pix[i % sets])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(s)
        for i in range(args.steps):
            ops.pack_rgb(rgb[i % sets], pixels=pix[i % sets])
        e1.record(s)
        torch.cuda.synchronize()
        dev_s = e0.elapsed_time(e1) / 1e3
        # e2e through the staging packet: host canvases -> pinned packet -> one H2D -> pack
        pk = staging.Packet([(n, H, W, 3)], [torch.uint8], device=dev)
        out = torch.empty((2, 1536), dtype=torch.bfloat16, pin_memory=True)
        for i in range(args.warmup):
            pk.stage(host[i % 2])
            ops.pack_rgb(pk.device_views[0], pixels=pix[0])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(args.steps):
            pk.stage(host[i % 2])
            ops.pack_rgb(pk.device_views[0], pixels=pix[0])
            out[i % 2].copy_(pix[0][-1], non_blocking=True)
        torch.cuda.synchronize()
        e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dev_s, e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s, e2e_s = t.tolist()
    value = world * n * args.steps / dev_s
    achieved = n * bpc / (dev_s / args.steps) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        ts = []
        for i in range(6):
            t0 = time.perf_counter()
            oracle.pack_rgb(host[0][i % n])
            ts.append(time.perf_counter() - t0)
        cpu = dict(value=1.0 / statistics.median(ts[1:]), unit=PACK_UNIT, cores=1, kind="port",
                   sample="5 canvases through the numpy restatement, median per canvas")
    if rank == 0:
        print(json.dumps(dict(
            metric=metric, value=value, unit=PACK_UNIT, n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=dev_s / args.steps * 1e3, higher_is_better=True, scaling="weak", vs_baseline=None,
            dtype="u8->bf16", data="synthetic (uniform random bytes)",
            config=dict(workload=args.workload, canvases_per_step=n, parallelism=f"replicas{world}",
                        l2=f"4 rotating input/output sets of {n * bpc / 1e6:.0f} MB each: footprint above L2"),
            roofline=dict(bound="hbm", achieved=achieved, peak=peaks["hbm"], unit="GB/s", frac=achieved / peaks["hbm"],
                          traffic=None, kernel="pack_rgb_kernel",
                          traffic_note=f"algorithmic bytes per canvas {bpc} (u8 read + bf16 write)",
                          peak_note=f"{peaks['src']} HBM copy bandwidth"),
            e2e=dict(value=world * n * args.steps / e2e_s, unit=PACK_UNIT, h2d_bytes_per_step=n * H * W * 3,
                     d2h_bytes_per_step=1536 * 2, api="staging.Packet.stage + ops.pack_rgb",
                     note="includes the host copy of the canvases into the pinned packet"),
            gpu_launches=args.steps, clocks=clk.summary(), cpu_baseline=cpu)), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    from fastforward_b200.config import STREAMS
    if args.workload in PACK_WORKLOADS:
        return run_pack_reference(args) if args.impl == "reference" else run_pack(args)
    if args.vision_ncu:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps(vision_measure(args, torch.device("cuda", 0), read_peaks())), flush=True)
        return
    if args.impl == "reference":
        if args.workload in STREAMS:
            print(json.dumps(dict(impl="reference", unavailable="the CPU reference arm times the fixed-geometry "
                                  "workloads only; use --workload 4B-fp8-T320")), flush=True)
            return
        run_reference(args)
    elif args.workload in STREAMS:
        run_stream(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

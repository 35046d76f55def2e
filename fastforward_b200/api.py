"""Public surface, mirroring FastForward's `fastforward_accel.api` (api.py:1-99).

`Accelerator(bundle, *, backend="fast")`, `.predict(image, question, candidates, item_id,
*, backend=None)`, `.warmup(requests)`, `.activate_fast()`, `validate_request`,
`response` keep the reference's names, argument meaning, return dict and errors
(ValueError for schema/backend/choices/sha problems, FileNotFoundError for missing
files, RuntimeError for device problems and non-finite outputs; one RLock per instance
serialises calls).  Behind them the B200 engine runs the prefill + scoring path.

Before the path, the reference decodes and resizes the image, runs the vision tower and
tokenizes the prompt (`_family/depth_runtime.py:54-82`).  Here the vision tower runs on this
package's kernels (`fastforward_b200.vision`: a pre-sized uint8 canvas -> patch rows ->
tower graph -> visual and deepstack rows); decode / resize and the tokenizer are outside it
(a `tokenizer(question, candidates) -> (prefix ids, suffix ids)` callable is passed in, or a
whole `encoder(image, question, candidates) -> Request`).  Checkpoint bundles (the
reference's `configs/*.json`: `model` = a Hugging Face Qwen3-VL directory, the recovery
`checkpoint`, the calibration `profile_path`) load the weights from the safetensors files
(`fastforward_b200.checkpoint`); bundles with a `synthetic` block (seeded random weights, no
checkpoint files) get a deterministic synthetic encoder -- with `"vision": true` the seeded
vision tower on the image canvas and synthetic text ids -- so the whole surface runs
without model assets.  `prefill_score` is the internal entry that `predict` calls after the
encoder; benchmarks call it directly.
"""
import hashlib
import json
import math
import threading
from dataclasses import dataclass, field
from pathlib import Path

BACKENDS = ("fast",)


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(1024 * 1024), b""):
            h.update(block)
    return h.hexdigest()


def validate_request(image, question, candidates):
    """Same checks and errors as the reference (`api.py:17-25`)."""
    if not Path(image).is_file():
        raise FileNotFoundError(image)
    if not isinstance(question, str) or not question.strip():
        raise ValueError("A nonempty question is required")
    if not isinstance(candidates, (list, tuple)) or not 2 <= len(candidates) <= 8:
        raise ValueError("Provide two to eight choices")
    if any(not isinstance(x, str) or not x.strip() for x in candidates):
        raise ValueError("Choices must be nonempty strings")


def response(logits, candidates, item_id, logprobs=None):
    """Argmax (first maximum wins) + softmax probabilities, as the reference (`api.py:28-34`).
    `logprobs` (the GPU log-softmax) is added when given."""
    if len(logits) != len(candidates) or not all(math.isfinite(x) for x in logits):
        raise RuntimeError("Invalid model output")
    prediction = max(range(len(logits)), key=lambda i: logits[i])
    exps = [math.exp(x - max(logits)) for x in logits]
    out = dict(id=item_id, answer=dict(letter=chr(65 + prediction), text=candidates[prediction]),
               logits=logits, probabilities=[x / sum(exps) for x in exps])
    if logprobs is not None:
        out["logprobs"] = logprobs
    return out


@dataclass
class Request:
    """What the path consumes for one request (the encoder's output)."""
    ids: "object"                 # [n] int64 token ids (image positions hold any id)
    visual: "object"              # [nv, H] bf16 visual-merger rows
    deep: list = field(default_factory=list)   # deepstack rows, each [nv, H]
    image_start: int = 0
    grid_h: int = 32              # patch grid before the 2x2 merge
    grid_w: int = 32
    k: int = 4

    @property
    def pick(self):
        return int(self.ids.shape[0]) - 1


class SyntheticEncoder:
    """Deterministic stand-in for image decode + vision tower + tokenizer: the request's
    bytes seed the synthetic visual rows and text ids of the bundle's layout."""

    def __init__(self, dims, layout):
        self.dims = dims
        self.layout = layout

    def __call__(self, image, question, candidates):
        import torch
        from .synthetic import make_request
        h = hashlib.sha256(Path(image).read_bytes() + question.encode() + "\x00".join(candidates).encode())
        seed = int.from_bytes(h.digest()[:8], "little") & ((1 << 62) - 1)
        lay = self.layout
        r = make_request(self.dims, lay, seed=seed)
        n = lay.n_tokens
        return Request(ids=r["ids"][:n], visual=r["visual"], deep=r["deep"], image_start=lay.image_start,
                       grid_h=lay.grid_h, grid_w=lay.grid_w, k=len(candidates))


class Accelerator:
    """Load one supported model and run its prefill + choice scoring on one B200.

    The caller owns the CUDA device (`device`, default the current one).  Graph capture
    happens on the first request of each geometry.  Calls are serialised by an RLock;
    graph buffers are private to the instance.
    """

    def __init__(self, bundle, *, backend="fast", device=None, encoder=None, tokenizer=None):
        self.bundle = Path(bundle).resolve()
        c = json.loads(self.bundle.read_text())
        if c.get("schema_version") != 1 or c.get("task") != "visual_choice":
            raise ValueError("Unsupported adaptation bundle schema or task")
        if backend not in BACKENDS:
            raise ValueError("Unknown backend")
        synthetic = c.get("synthetic")
        if synthetic is None:
            self._check_assets(c)
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("A CUDA GPU is required; CPU fallback is disabled")
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if torch.cuda.get_device_capability(dev)[0] != 10:
            raise RuntimeError("This backend requires a B200 (sm_100a)")
        if c.get("architecture") != "qwen3_vl_family":
            raise ValueError("No adapter registered for this architecture")
        from .config import MODELS, Layout, BUCKETS
        from .engine import Engine, PackedModel
        from .synthetic import make_model_bf16
        self.config = c
        self.backend = backend
        self.lock = threading.RLock()
        self.device = dev
        self.buckets = tuple(c.get("buckets", BUCKETS))
        if synthetic is not None:
            self.dims = MODELS[synthetic["model"]]
            mode = synthetic.get("mode", "rowwise")
            lay = synthetic.get("layout", {})
            self.layout = Layout(int(lay.get("image_start", 0)), int(lay.get("grid_h", 32)),
                                 int(lay.get("grid_w", 32)), int(lay.get("n_text", 64)))
        else:
            mode = self._checkpoint_mode(c)
            self.layout = None
        profile = self._read_profile(c) if mode == "static" else None
        with torch.cuda.device(dev), torch.no_grad():
            if synthetic is not None:
                src = make_model_bf16(self.dims, seed=int(synthetic.get("seed", 0)), device=dev,
                                      layers=synthetic.get("layers"))
                if mode == "static" and profile is None and synthetic.get("calibrate"):
                    profile = self._calibrate(src, int(synthetic["calibrate"]),
                                              float(c.get("fp8_calibration_margin", 1.5)))
            else:
                from .checkpoint import load_language_model
                self.dims, src = load_language_model(c["model"], device=dev, option_ids=c.get("option_ids"),
                                                      expected_dimensions=c.get("expected_dimensions"))
                if mode == "static" and profile is None:
                    raise ValueError("execution_mode fp8 needs the bundle's calibration profile (profile_path)")
            self.profile = profile
            self.model = PackedModel(self.dims, src, mode=mode, device=dev, free_source=True, profile=profile)
            del src
            torch.cuda.empty_cache()
            self.engine = Engine(self.model)
        self.vision = None
        if encoder is None:
            encoder = self._vision_encoder(c, synthetic, tokenizer)
        if encoder is None and synthetic is not None:
            encoder = SyntheticEncoder(self.dims, self.layout)
        self.encoder = encoder
        self._staging = {}

    def _vision_encoder(self, c, synthetic, tokenizer):
        """The image side of `predict` on this package's vision kernels, or None.

        Synthetic bundles opt in with `"vision": true` (or an object with `seed`, `depth`:
        a tower of fewer blocks, deepstack taken at its first blocks): a seeded tower of the
        family's published vision config, text ids from the synthetic stand-in unless a
        `tokenizer` is given.  Checkpoint bundles use the checkpoint's own vision tower
        when a `tokenizer(question, candidates) -> (prefix ids, suffix ids)` is given (no
        tokenizer ships with this package)."""
        import torch
        from .vision import VisionEncoder, VisionTower
        if synthetic is not None:
            spec = synthetic.get("vision")
            if not spec:
                return None
            spec = spec if isinstance(spec, dict) else {}
            from dataclasses import replace
            from .config import VISION_MODELS
            from .synthetic import make_vision_bf16
            v = VISION_MODELS[synthetic["model"]]
            if spec.get("depth"):
                depth = int(spec["depth"])
                v = replace(v, depth=depth, deepstack=tuple(min(i, depth - 1) for i in range(len(v.deepstack))))
            with torch.cuda.device(self.device):
                params = make_vision_bf16(v, seed=int(spec.get("seed", 0)), device=self.device)
                self.vision = VisionTower(v, params, device=self.device)
            lay = self.layout
            return VisionEncoder(self.vision, self.dims.vocab, tokenizer, n_prefix=lay.image_start, n_suffix=lay.n_text)
        if tokenizer is None:
            return None
        from .checkpoint import load_vision_tower
        v, params = load_vision_tower(c["model"], device=self.device)
        self.vision = VisionTower(v, params, device=self.device)
        return VisionEncoder(self.vision, self.dims.vocab, tokenizer)

    # ------------------------------------------------------------------ checkpoint bundles
    @staticmethod
    def _check_assets(c):
        """The reference's checks of a checkpoint bundle (`api.py:56-66`,
        `_family/family_api.py:19-23`): the model directory and the recovery checkpoint
        exist, the checkpoint's SHA256 matches, and its repair adapter is zero (the serving
        path applies it as the identity, `_family/night_runtime.py:88-94`)."""
        for key in ("model", "checkpoint"):
            if not Path(c[key]).exists():
                raise FileNotFoundError(c[key])
        if sha256(c["checkpoint"]) != c["checkpoint_sha256"]:
            raise ValueError("Recovery checkpoint SHA256 mismatch")
        import torch
        state = torch.load(c["checkpoint"], map_location="cpu", weights_only=True)
        state = state.get("state_dict", state)
        for key in ("up", "bias"):
            if key not in state or torch.count_nonzero(state[key]) != 0:
                raise ValueError(f"The recovery adapter's {key!r} is not zero; only the identity adapter is served")

    @staticmethod
    def _checkpoint_mode(c):
        """Weight format of a checkpoint bundle: `execution_mode` "fp8" is the reference's
        static-scale FP8 (`RuntimeScaleLinear` with the profile's bounds,
        `_family/family_api.py:27-31`), "fp8_rowwise" the per-row scheme
        (`_legacy/fp8_private.py`), "int4" the W4A16 path."""
        em = c.get("execution_mode", "fp8")
        modes = {"fp8": "static", "fp8_rowwise": "rowwise", "int4": "int4"}
        if em not in modes:
            raise ValueError(f"Unsupported execution_mode {em!r}")
        return modes[em]

    # ------------------------------------------------------------------ static FP8 profile
    @staticmethod
    def _read_profile(c):
        """The bundle's calibration profile for mode "static", as the reference's
        `activate_fast` reads it (`_family/family_api.py:27-31`): `profile_path` (JSON with
        a "profiles" map of variants) checked against `profile_sha256`, then the bounds of
        `variant` ("{layer}:{role}" -> bound).  None when the bundle names no profile."""
        path = c.get("profile_path")
        if path is None:
            return None
        if not Path(path).is_file():
            raise FileNotFoundError(path)
        if sha256(path) != c.get("profile_sha256"):
            raise ValueError("Calibration profile SHA256 mismatch")
        profiles = json.loads(Path(path).read_text())["profiles"]
        variant = c.get("variant")
        if variant not in profiles:
            raise ValueError(f"Unknown calibration variant {variant!r}")
        return {key: float(v) for key, v in profiles[variant].items()}

    def _calibrate(self, src, count, margin):
        """Calibrates static bounds on `count` seeded synthetic requests of the bundle's
        layout (the reference's `fp8_calibrate` rows, `_legacy/limit_runtime.py:78-97`)."""
        from .engine import calibrate_profile
        from .synthetic import make_request
        lay = self.layout
        T = next(b for b in self.buckets if b >= lay.n_tokens)
        reqs = []
        for i in range(count):
            r = make_request(self.dims, lay, seed=1000 + i, device=self.device)
            reqs.append(dict(ids=r["ids"][:T], visual=r["visual"], deep=r["deep"], pick=lay.n_tokens - 1,
                             k=lay.k, image_start=lay.image_start, grid_h=lay.grid_h, grid_w=lay.grid_w, T=T))
        profile, _ = calibrate_profile(self.dims, src, reqs, margin, device=self.device)
        return profile

    # ------------------------------------------------------------------ path entry
    def prefill_score(self, ids, visual, deep, k, image_start=0, grid_h=32, grid_w=32, pick=None):
        """Prefill + choice scoring of one request; returns (logits [k], logprobs [k]) lists.

        ids [n] int64, visual [nv, H] bf16, deep list of [nv, H] bf16 -- host (pinned or
        pageable) or device tensors.  n is padded with id 0 to the first bucket >= n."""
        import torch
        n = int(ids.shape[0])
        if not 2 <= k <= 8:
            raise ValueError("Provide two to eight choices")
        bucket = next((b for b in self.buckets if b >= n), None)
        if bucket is None:
            raise ValueError(f"{n} tokens exceed the largest bucket {self.buckets[-1]} (no truncation)")
        nv = int(visual.shape[0]) if visual is not None else 0
        if nv != (grid_h // 2) * (grid_w // 2):
            raise ValueError("visual rows must match the merged image grid")
        pick = n - 1 if pick is None else int(pick)
        with self.lock, torch.no_grad(), torch.cuda.device(self.device):
            entry = self.engine.capture(bucket, image_start, nv, grid_h, grid_w, k, len(deep or []))
            z, lp = self.engine.replay(entry, ids.to(self.device, non_blocking=True),
                                       visual.to(self.device, non_blocking=True) if nv else None,
                                       [x.to(self.device, non_blocking=True) for x in (deep or [])], pick)
            out = torch.stack([z, lp]).cpu()  # one device->host read, synchronises the stream
        return out[0].tolist(), out[1].tolist()

    def prefill_score_stream(self, requests):
        """Scores a sequence of requests, one forward (graph replay) each -- the same answers
        as `prefill_score` on each, in order -- with the host<->device traffic overlapped:
        request i+1's inputs are copied from host memory on a copy stream while request i's
        forward runs, and request i's answer is copied back into pinned host memory without
        waiting for it.  requests: dicts of `prefill_score`'s arguments (ids, visual, deep,
        k, image_start, grid_h, grid_w, optional pick).  Returns [(logits [k], logprobs [k])]."""
        import torch
        plan = []
        for r in requests:
            ids, vis, deep = r["ids"], r.get("visual"), list(r.get("deep") or [])
            n, k = int(ids.shape[0]), int(r["k"])
            if not 2 <= k <= 8:
                raise ValueError("Provide two to eight choices")
            bucket = next((b for b in self.buckets if b >= n), None)
            if bucket is None:
                raise ValueError(f"{n} tokens exceed the largest bucket {self.buckets[-1]} (no truncation)")
            nv = int(vis.shape[0]) if vis is not None else 0
            gh, gw = int(r.get("grid_h", 32)), int(r.get("grid_w", 32))
            if nv != (gh // 2) * (gw // 2):
                raise ValueError("visual rows must match the merged image grid")
            pick = n - 1 if r.get("pick") is None else int(r["pick"])
            plan.append((r, n, nv, bucket, k, pick, int(r.get("image_start", 0)), gh, gw, deep))
        if not plan:
            return []
        dev = self.device
        with self.lock, torch.no_grad(), torch.cuda.device(dev):
            main = torch.cuda.current_stream(dev)
            copy = torch.cuda.Stream(dev)
            n_max = max(p[1] for p in plan)
            nv_max = max([p[2] for p in plan] + [1])
            n_deep = max(len(p[9]) for p in plan)
            H = self.dims.hidden
            slots = [dict(ids=torch.empty(n_max, dtype=torch.long, device=dev),
                          visual=torch.empty((nv_max, H), dtype=torch.bfloat16, device=dev),
                          deep=[torch.empty((nv_max, H), dtype=torch.bfloat16, device=dev) for _ in range(n_deep)])
                     for _ in range(2)]
            ready = [torch.cuda.Event() for _ in range(2)]
            free = [torch.cuda.Event() for _ in range(2)]
            out = torch.zeros((len(plan), 2, 8), dtype=torch.float32, pin_memory=True)
            # The copy stream starts after everything already queued on the caller's stream:
            # device inputs the caller produced there are complete, and the slot buffers
            # (just allocated on that stream) are no longer in use by earlier work.
            copy.wait_stream(main)
            for i, (r, n, nv, bucket, k, pick, start, gh, gw, deep) in enumerate(plan):
                entry = self.engine.capture(bucket, start, nv, gh, gw, k, len(deep))
                sl = slots[i % 2]
                with torch.cuda.stream(copy):  # this request's inputs, once its slot is free again
                    if i >= 2:
                        copy.wait_event(free[i % 2])
                    sl["ids"][:n].copy_(r["ids"], non_blocking=True)
                    if nv:
                        sl["visual"][:nv].copy_(r["visual"], non_blocking=True)
                    for dst, src in zip(sl["deep"], deep):
                        dst[:nv].copy_(src, non_blocking=True)
                    ready[i % 2].record(copy)
                main.wait_event(ready[i % 2])
                b = entry["buffers"]
                if n < bucket:
                    b.ids[n:].zero_()
                b.ids[:n].copy_(sl["ids"][:n])
                if nv:
                    entry["visual"][:nv].copy_(sl["visual"][:nv])
                for dst, src in zip(entry["deep"], sl["deep"][:len(deep)]):
                    dst[:nv].copy_(src[:nv])
                b.pick.fill_(pick)
                free[i % 2].record(main)
                entry["graph"].replay()
                out[i, 0, :k].copy_(b.logits[:k], non_blocking=True)
                out[i, 1, :k].copy_(b.logprobs[:k], non_blocking=True)
            main.synchronize()
        return [(out[i, 0, :p[4]].tolist(), out[i, 1, :p[4]].tolist()) for i, p in enumerate(plan)]

    def prefill_score_batch(self, requests):
        """Prefill + choice scoring of several requests in one forward pass over their
        concatenated tokens (`Engine.forward_batch`; the reference serialises requests).
        requests: list of dicts with ids [n] int64, visual [nv, H] bf16, deep (list of
        [nv, H]), k, image_start, grid_h, grid_w, optional pick (default n - 1) -- host
        (pinned or pageable) or device tensors.  Returns [(logits [k], logprobs [k])] lists,
        one pair per request, in order."""
        import torch
        reqs = []
        for r in requests:
            k = int(r["k"])
            if not 2 <= k <= 8:
                raise ValueError("Provide two to eight choices")
            vis = r.get("visual")
            nv = int(vis.shape[0]) if vis is not None else 0
            if nv != (int(r["grid_h"]) // 2) * (int(r["grid_w"]) // 2):
                raise ValueError("visual rows must match the merged image grid")
            reqs.append(r)
        with self.lock, torch.no_grad(), torch.cuda.device(self.device):
            dev = [dict(r, ids=r["ids"].to(self.device, non_blocking=True),
                        visual=r["visual"].to(self.device, non_blocking=True) if r.get("visual") is not None else None,
                        deep=[x.to(self.device, non_blocking=True) for x in (r.get("deep") or [])]) for r in reqs]
            outs = self.engine.forward_batch(dev)
            flat = torch.cat([torch.cat([z, lp]) for z, lp in outs]).cpu()  # one device->host read
        res, i = [], 0
        for r in reqs:
            k = int(r["k"])
            res.append((flat[i:i + k].tolist(), flat[i + k:i + 2 * k].tolist()))
            i += 2 * k
        return res

    def predict(self, image, question, candidates, item_id="request", *, backend=None):
        validate_request(image, question, candidates)
        mode = self.backend if backend is None else backend
        if mode not in BACKENDS:
            raise ValueError("Unknown backend")
        if self.encoder is None:
            raise RuntimeError("No encoder: no tokenizer ships with this package; construct the Accelerator with "
                               "tokenizer=callable(question, candidates) -> (prefix ids, suffix ids) to run the "
                               "checkpoint's vision tower, or encoder=callable(image, question, candidates) -> Request")
        with self.lock:
            r = self.encoder(str(image), question, list(candidates))
            z, lp = self.prefill_score(r.ids, r.visual, r.deep, len(candidates), r.image_start, r.grid_h,
                                       r.grid_w)
        return response(z, candidates, item_id, logprobs=lp)

    def warmup(self, requests):
        for r in requests:
            self.predict(r["image_path"], r["instruction"], r["candidates"], r.get("item_id", "warmup"))

    def activate_fast(self):
        """The packed FP8/int4 weights are built at construction; kept for API parity."""
        with self.lock:
            self.backend = "fast"

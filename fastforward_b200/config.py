"""Model shapes and request layouts of the Qwen3-VL language decoders this path serves.

The four families are the ones FastForward ships bundles for (`configs/{2B,4B,8B,32B}.json`,
`expected_dimensions` = (layers, hidden, vision blocks)); the remaining dimensions are the
published Qwen3-VL text-config values.  Buckets follow the reference bundles: 64..2048 in
steps of 16 (`configs/*.json` "buckets").
"""
from dataclasses import dataclass, field, asdict

BUCKETS = tuple(range(64, 2049, 16))
VOCAB = 151936
# Eight fixed token ids standing in for the tokens of " A" .. " H"
# (`scaled_qwen_runtime.py:70-72` reads them from the tokenizer, which is absent here).
OPTION_IDS = (362, 425, 356, 422, 468, 434, 479, 472)


@dataclass(frozen=True)
class Dims:
    name: str
    layers: int
    hidden: int
    hq: int
    hk: int
    inter: int
    d: int = 128
    vocab: int = VOCAB
    tied: bool = True
    eps: float = 1e-6
    theta: float = 5_000_000.0
    sections: tuple = (24, 20, 20)
    deepstack: int = 3

    @property
    def qkv_out(self):
        return (self.hq + 2 * self.hk) * self.d

    def as_dict(self):
        return asdict(self)

    def params_per_layer(self):
        h, i = self.hidden, self.inter
        return self.qkv_out * h + h * self.hq * self.d + 2 * i * h + h * i


MODELS = {
    "2B": Dims("2B", 28, 2048, 16, 8, 6144, tied=True),
    "4B": Dims("4B", 36, 2560, 32, 8, 9728, tied=True),
    "8B": Dims("8B", 36, 4096, 32, 8, 12288, tied=False),
    "32B": Dims("32B", 64, 5120, 64, 8, 25600, tied=False),
}


@dataclass(frozen=True)
class VisionDims:
    """Shape of a Qwen3-VL vision tower (patch embedding, blocks, deepstack and final
    mergers).  `out_hidden` is the language model's hidden size."""
    hidden: int
    heads: int
    inter: int
    out_hidden: int
    depth: int
    deepstack: tuple
    num_pos: int = 2304           # 48 x 48 learned position table, sampled bilinearly
    patch: int = 16
    temporal: int = 2
    merge: int = 2
    eps: float = 1e-6
    theta: float = 10000.0
    act: str = "gelu_pytorch_tanh"

    @property
    def head_dim(self):
        return self.hidden // self.heads


# The published Qwen3-VL vision configs; the depths agree with the bundles'
# `expected_dimensions` (24 for 2B/4B, 27 for 8B/32B).
VISION_MODELS = {
    "2B": VisionDims(1024, 16, 4096, 2048, 24, (5, 11, 17)),
    "4B": VisionDims(1024, 16, 4096, 2560, 24, (5, 11, 17)),
    "8B": VisionDims(1152, 16, 4304, 4096, 27, (8, 16, 24)),
    "32B": VisionDims(1152, 16, 4304, 5120, 27, (8, 16, 24)),
}


@dataclass
class Layout:
    """Token layout of one request: [prefix text][image grid][suffix text] + bucket padding.

    `grid_h`/`grid_w` are patch-grid sizes before the 2x2 merge (as `image_grid_thw`),
    so the image contributes (grid_h/2)*(grid_w/2) visual tokens.
    """
    image_start: int
    grid_h: int
    grid_w: int
    n_text: int
    k: int = 4
    extra: dict = field(default_factory=dict)

    @property
    def nv(self):
        return (self.grid_h // 2) * (self.grid_w // 2)

    @property
    def n_tokens(self):
        return self.image_start + self.nv + self.n_text

    @property
    def bucket(self):
        n = self.n_tokens
        return next(b for b in BUCKETS if b >= n)

    @property
    def pick(self):
        return self.n_tokens - 1


# The benchmark configurations (synthetic stand-ins for the reference's VQA suites).
WORKLOADS = {
    # 2B-shaped, 256 visual tokens on a 16x16 LLM grid + 64 text, 4 choices
    "2B-fp8-T320": ("2B", Layout(0, 32, 32, 64, k=4), "rowwise"),
    # C1: the reference's CPU case, one 2B decoder layer at T = 512 (256 visual rows on a
    # 16x16 merged grid + 256 text positions); timed on the host only (bench --cpu-layer)
    "2B-layer-T512": ("2B", Layout(0, 32, 32, 256, k=4), "rowwise"),
    # north-star: 4B-shaped FP8 prefill of 320 tokens + choice scoring
    "4B-fp8-T320": ("4B", Layout(0, 32, 32, 64, k=4), "rowwise"),
    # the same with the reference's shipped FP8 scheme (per-tensor weight scales, static
    # activation scales from a calibration profile)
    "4B-fp8static-T320": ("4B", Layout(0, 32, 32, 64, k=4), "static"),
    # 4B-shaped W4A16, 512 visual tokens on a 16x32 grid + 64 text, 8 choices
    "4B-w4a16-T576": ("4B", Layout(0, 32, 64, 64, k=8), "int4"),
    # 32B-shaped FP8, 960 visual tokens on a 30x32 grid + 64 text, 4 choices
    "32B-fp8-T1024": ("32B", Layout(0, 60, 64, 64, k=4), "rowwise"),
}

# Request streams (independent requests of varying geometry): model, FP8 mode, size.
STREAMS = {
    # 8B-shaped FP8: visual tokens uniform in {64, 144, 256} on square grids, text length
    # uniform in [32, 128], choices uniform in 2..8
    "8B-fp8-stream": ("8B", "rowwise", 256),
}


def stream_layouts(n, seed=1):
    """The geometries of a synthetic request stream (seeded): list of Layout."""
    import random
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        side = rng.choice((8, 12, 16))  # merged grid side: 64 / 144 / 256 visual tokens
        out.append(Layout(0, 2 * side, 2 * side, rng.randint(32, 128), k=rng.randint(2, 8)))
    return out

"""Builds matching oracle / engine models from one seeded bf16 source (test helper)."""
import torch

import oracle
from fastforward_b200.config import Layout
from fastforward_b200.synthetic import make_model_bf16, make_request


def oracle_model(dims, src, mode="rowwise", inv=None):
    return oracle.quantized_model(dims, src, mode, inv)


def small_case(dims, n_layers, layout=None, seed=0, req_seed=1, vocab=None):
    """(bf16 source model on CPU, request on CPU, layout) with a reduced vocabulary so the
    CPU oracle stays fast; the GPU path is shape-identical otherwise."""
    from dataclasses import replace
    d = replace(dims, vocab=vocab) if vocab else dims
    layout = layout or Layout(0, 32, 32, 64, k=4)
    src = make_model_bf16(d, seed=seed, device="cpu", layers=n_layers)
    req = make_request(d, layout, seed=req_seed)
    return d, src, req, layout

"""The general route's own tcgen05 row GEMM (rowgemm) against cuBLAS on the same
requests: the forward with every GEMM on cuBLAS (lnet_b200_set_gemm_backend(1))
and with the row GEMM (default) must agree -- fp32 requests to 1e-5 (split-bf16 x3
is fp32-level), bf16 requests to 1e-3 (bf16 x bf16 products are exact, TF32
rounds the fp32 operands) -- and each must stay within the parity gates against
the float64 oracle.  Shapes: BASELINE configs 2, 3 (with all metadata) and 5 at
reduced batch and length (config 5: n = k = 256 on the pipelined kernel), plus
ragged shapes (k, n not multiples of 16; output pitches not multiples of 4)."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from conftest import record_margin, rel_err

from lnet_b200 import _lib
from oracle import alphabet_oracle as A

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

pytestmark = pytest.mark.gpu

CASES = {
    "cfg2": dict(bench.CONFIGS["2"], B=4, T=300),
    "cfg3": dict(bench.CONFIGS["3"], B=3, T=257),
    "cfg5": dict(bench.CONFIGS["5"], B=2, T=700),
    "ragged": dict(workload="ragged", B=3, T=99, C=13, D=40, M=12, K=7, dtype="fp32",
                   images=False),
    # output pitches D = 42 and 2M = 26 are not multiples of 4 floats: the
    # non-pipelined row GEMM (plain stores) serves them
    "ragged_pitch": dict(workload="ragged_pitch", B=2, T=131, C=11, D=42, M=13, K=5,
                         dtype="fp32", images=False),
    "ragged_bf16": dict(workload="ragged_bf16", B=2, T=140, C=24, D=56, M=20, K=5,
                        dtype="bf16", images=False),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_rowgemm_matches_cublas_and_oracle(name, cuda_device):
    cfg = CASES[name]
    model = bench.build_model(cfg, cuda_device)
    x = bench.make_inputs(cfg, cuda_device)
    meta = bench.synthetic_metadata(cfg, cuda_device) if cfg.get("meta") else {}
    lib = _lib.load()
    _lib.set_route(_lib.ROUTE_GENERAL)
    try:
        with torch.no_grad():
            lib.lnet_b200_set_gemm_backend(1)
            ref_cublas = model(x, **meta).cpu().numpy()
            lib.lnet_b200_set_gemm_backend(0)
            got = model(x, **meta).cpu().numpy()
    finally:
        lib.lnet_b200_set_gemm_backend(0)
        _lib.set_route(_lib.ROUTE_AUTO)
    bf16 = cfg["dtype"] == "bf16"
    assert rel_err(got, ref_cublas) <= (1e-3 if bf16 else 1e-5)
    params = {k: v.numpy().astype(np.float64) for k, v in bench.make_params(cfg).items()}
    kw = {k: v.cpu().numpy() for k, v in meta.items()}
    ref = A.alphabet_forward(x.float().cpu().numpy(), params, dtype=np.float64, **kw)
    gate = 2e-2 if bf16 else 1e-4
    nw, _ = record_margin(f"rowgemm:{name}:logits", got, ref, gate)
    assert nw <= gate

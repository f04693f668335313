"""The CPU oracle against golden vectors of the reference's own kernels (CPU test).

tests/golden/*.npz hold fp16 inputs and outputs of the reference's forward kernels (VoltaMma,
VoltaWmma, VoltaLayerNorm, VoltaGdp, VoltaGdpWmma), compiled from its sources for sm_100a by
oracle/legacy_ref/ and run on a B200 by tests/golden/make_golden.py.  Every case must match the
float64 oracle within atol = rtol = 2e-3 (the reference rounds P to fp16 before P V and every
output to fp16; measured worst deviations are ~1e-3 absolute on outputs of magnitude 1-4).
"""

import json
import sys
from pathlib import Path

import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import compare  # noqa: E402

INDEX = json.loads((GOLDEN / "index.json").read_text())


def test_golden_cases_present():
    ops = {m["op"] for m in INDEX.values()}
    assert ops == {"attention", "layer_norm", "gdp"}
    for name in INDEX:
        assert (GOLDEN / (name + ".npz")).is_file(), name


@pytest.mark.parametrize("name", sorted(INDEX))
def test_oracle_matches_reference_kernel(name):
    dev = compare.deviation(GOLDEN / (name + ".npz"), INDEX[name])
    assert dev["n"] > 0
    assert dev["worst_tol_ratio"] <= 1.0, dev


def test_ragged_fully_masked_case_needs_reference_padding():
    """The reference pads its last key tile with -1e4 logits and zero V rows; for a batch row
    whose keys are all masked this changes the output, and only the oracle's ref_block_k mode
    reproduces it (the B200 kernels follow the mathematical definition instead)."""
    import numpy as np
    import torch
    import oracle
    with np.load(GOLDEN / "attn_mma_d32_ragged_k_fully_masked.npz") as z:
        d = {k: torch.from_numpy(z[k]) for k in z.files}
    plain, _ = oracle.attention_fwd(d["q"], d["k"], d["v"], d["bias"], d["kmask"],
                                    float(d["scale"]))
    got = d["out"].double()
    dead = (d["kmask"] == 0).all(dim=1)
    assert dead.any() and not dead.all()
    # rows of live batch rows agree without the padding model; fully masked rows do not
    assert torch.allclose(plain[~dead], got[~dead], atol=2e-3, rtol=2e-3)
    assert not torch.allclose(plain[dead], got[dead], atol=2e-3, rtol=2e-3)

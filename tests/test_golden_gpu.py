"""The sm_100a kernels against outputs of the reference's own kernels (GPU test).

Runs cfk_attn_fwd, cfk_ln_fwd and cfk_gdp_fwd in fp16 on the inputs stored in tests/golden/
and compares with the outputs that the reference's kernels (VoltaMma, VoltaWmma,
VoltaLayerNorm, VoltaGdp, VoltaGdpWmma, built from its sources by oracle/legacy_ref/) produced
on a B200.  Both sides round to fp16; the tolerance is atol = rtol = 4e-3.  One documented
difference is excluded: for a batch row whose keys are all masked and Sk not a multiple of the
reference's block_k, the reference also averages over its zero-padded key slots, while these
kernels follow the mathematical definition (softmax over the Sk real keys).
"""

import json
from pathlib import Path

import numpy as np
import pytest

from conftest import assert_close_bf16

GOLDEN = Path(__file__).resolve().parent / "golden"
INDEX = json.loads((GOLDEN / "index.json").read_text())
TOL = 4e-3


def _load(name, device):
    import torch
    with np.load(GOLDEN / (name + ".npz")) as z:
        return {k: (torch.from_numpy(z[k]).to(device) if z[k].ndim else z[k][()])
                for k in z.files}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(n for n, m in INDEX.items() if m["op"] == "attention"))
def test_attention_fwd_matches_reference(cuda_device, name):
    import torch
    from colabfold_legacy_kernels import torch_ops
    d = _load(name, cuda_device)
    out, _ = torch_ops.attention_fwd(d["q"], d["k"], d["v"], d["bias"], d["kmask"],
                                     float(d["scale"]))
    torch.cuda.synchronize()
    got, ref = out.cpu(), d["out"].cpu()
    sk = d["k"].shape[2]
    if sk % int(d["block_k"]):
        live = ~(d["kmask"] == 0).all(dim=1).cpu()  # see the module docstring
        got, ref = got[live], ref[live]
    assert_close_bf16(got, ref, name, rtol=TOL, atol=TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(n for n, m in INDEX.items() if m["op"] == "layer_norm"))
def test_layer_norm_fwd_matches_reference(cuda_device, name):
    import torch
    from colabfold_legacy_kernels import torch_ops
    d = _load(name, cuda_device)
    y = torch_ops.layer_norm_fwd(d["x"], d["gamma"], d["beta"], float(d["eps"]))
    torch.cuda.synchronize()
    assert_close_bf16(y.cpu(), d["out"].cpu(), name, rtol=TOL, atol=TOL)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(n for n, m in INDEX.items() if m["op"] == "gdp"))
def test_gdp_fwd_matches_reference(cuda_device, name):
    import torch
    from colabfold_legacy_kernels import torch_ops
    d = _load(name, cuda_device)
    out = torch_ops.gdp_fwd(d["x"], d["wp"], d["bp"], d["wg"], d["bg"], d["mask"])
    torch.cuda.synchronize()
    assert_close_bf16(out.cpu(), d["out"].cpu(), name, rtol=TOL, atol=TOL)

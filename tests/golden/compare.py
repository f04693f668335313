"""Oracle-versus-golden comparison shared by tests/test_golden.py and make_golden.py.

The golden outputs are fp16 results of the reference's own kernels (see make_golden.py); the
oracle runs in float64 on the same fp16 inputs.  `deviation` returns the largest absolute
error, the largest error in units of (atol + rtol * |oracle|) for the tolerance of the op, and
the number of elements compared.
"""

import numpy as np
import torch

# atol = rtol per op.  The reference computes in fp16 with f32 accumulation, rounds the softmax
# weights to fp16 before P V (cuda/volta_mma_attn.cu:221) and rounds every output to fp16.
TOL = {"attention": 2e-3, "layer_norm": 2e-3, "gdp": 2e-3}


def oracle_out(data, meta):
    import oracle
    t = {k: torch.from_numpy(np.asarray(v)) for k, v in data.items()}
    if meta["op"] == "attention":
        out, _ = oracle.attention_fwd(t["q"], t["k"], t["v"], t["bias"], t["kmask"],
                                      float(data["scale"]), ref_block_k=int(data["block_k"]))
        return out
    if meta["op"] == "layer_norm":
        y, _, _ = oracle.layer_norm_fwd(t["x"], t["gamma"], t["beta"], float(data["eps"]),
                                        two_pass=False)
        return y
    if meta["op"] == "gdp":
        return oracle.gdp_fwd(t["x"], t["wp"], t["bp"], t["wg"], t["bg"], t["mask"])
    raise ValueError(meta["op"])


def deviation(path, meta):
    with np.load(path) as z:
        data = {k: z[k] for k in z.files}
    expect = oracle_out(data, meta).to(torch.float64)
    got = torch.from_numpy(data["out"].astype(np.float64))
    err = (got - expect).abs()
    tol = TOL[meta["op"]]
    ratio = (err / (tol + tol * expect.abs())).max().item()
    return {"max_abs_err": err.max().item(), "max_abs_out": expect.abs().max().item(),
            "worst_tol_ratio": ratio, "n": int(err.numel())}

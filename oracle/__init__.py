"""CPU oracle for the three Evoformer kernels -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU (float64 by default), the arithmetic of the
reference kernels of sokrypton/colabfold-legacy-kernels:

* attention with pair bias and key mask  -- cuda/volta_mma_attn.cu:139-271
  (and its sm_70 twin cuda/volta_wmma_attn.cu:157-232),
* LayerNorm                              -- cuda/volta_ops.cu:40-58,
* gated dual projection                  -- cuda/volta_ops.cu:185-207
  (and cuda/volta_gdp_wmma.cu:76-96),
* the triangle-attention module that composes them (module.py; the reference's caller, not
  part of the reference),

plus the backward passes, which the reference does not have: they are the exact derivatives of
those forward definitions (checked against torch.autograd in tests/test_oracle.py).

Only tests/, __graft_entry__.smoke() and the CPU legs of bench.py may import this package, and
only as the checker or the timed CPU baseline.  The product path (the CUDA library behind
include/cfk.h and colabfold_legacy_kernels) never calls it and has no CPU fallback.

Parity pin: the reference ships no tests, golden vectors or fixtures for this path.  The
forward restatements are pinned against outputs of the reference's own kernels, compiled from
its sources for sm_100a by oracle/legacy_ref/ and run on a B200; the vectors live in
tests/golden/ (made by tests/golden/make_golden.py, checked by tests/test_golden.py).  The
backward has no reference counterpart and is pinned to torch.autograd of the pinned forward.
"""

from .attention import (MASKED_LOGIT, attention_bwd, attention_fwd, attention_logits,
                        attention_fwd_chunked)
from .layer_norm import layer_norm_bwd, layer_norm_fwd
from .gdp import gdp_bwd, gdp_fwd
from . import configs, module

__all__ = [
    "MASKED_LOGIT", "attention_fwd", "attention_bwd", "attention_logits", "attention_fwd_chunked",
    "layer_norm_fwd", "layer_norm_bwd", "gdp_fwd", "gdp_bwd", "configs", "module",
]

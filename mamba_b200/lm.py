"""A CausalLM-shaped model's forward through the fused paths.

The reference's ``CausalLM.forward`` (models/causal_lm.py:50-58) runs, per block,
``h = h + dropout(mamba(norm(h)))`` (Block.forward, :30-37) with a PyTorch RMSNorm, the
MambaSimple block (permute copies, separate conv / SiLU / gate kernels) and an in-place
residual add, then a final RMSNorm and the tied lm_head.  ``causal_lm_forward(model, ids)``
computes the same logits from the same parameters with:

* ``rms_norm(..., residual=..., prenorm=True)`` — the residual add of one block fused with the
  RMSNorm that starts the next (and with the final norm);
* ``mamba_simple_forward`` — the fused block (conv + SiLU kernel, batched GEMMs, gated scan).

It is differentiable end to end (training) and applies the blocks' dropout modules as the
reference does.  The model is duck-typed on the reference's module tree.
"""
from __future__ import annotations

from .inner import mamba_simple_forward
from .norm import rms_norm


def causal_lm_hidden(model, input_ids):
    """Final normalised hidden states (batch, L, d_model)."""
    h = model.embedding(input_ids)
    res = y = None
    for layer in model.layers:
        x, res = rms_norm(layer.norm, h if res is None else y, residual=res, prenorm=True)
        y = mamba_simple_forward(layer.mamba, x)
        drop = getattr(layer, "dropout", None)
        if drop is not None:
            y = drop(y)
    if y is None:
        return rms_norm(model.norm, h)
    return rms_norm(model.norm, y, residual=res)


def causal_lm_forward(model, input_ids):
    """Logits (batch, L, vocab) of a reference CausalLM (models/causal_lm.py:50-58)."""
    return model.lm_head(causal_lm_hidden(model, input_ids))

"""Decoding for MambaSimple models: a prompt prefill that leaves per-layer states, single-token
steps that continue from them, and ``generate`` for CausalLM-shaped models.

The reference has no decode path: ``CausalLM.generate`` is a stub (models/causal_lm.py:61-62)
and ``MambaSimple`` has no step, so continuing a sequence there means re-running the whole
forward over it for every new token.  Here a block keeps two states per sequence:

* conv state (batch, d_inner, K-1) fp32 — the last K-1 inputs of its causal convolution;
* SSM state  (batch, d_inner, d_state) fp32 — h of the selective scan,

and a new token costs the block's input and output projections plus one fused mixer kernel
(``ss_mamba_step``: the conv step, the x and delta projections, the SSM step and the SiLU(z)
gate).  The prefill runs the fused block path
(``mamba_inner_prefill``: conv kernel, batched GEMMs, scan with ``return_last_state``); each
block's residual add is fused with the next RMSNorm (``rms_norm(..., prenorm=True)``); and the
per-token model step of ``Decoder`` is captured once in a CUDA graph and replayed, so a decode
step is one graph launch rather than a dozen kernel launches per layer from Python.

Models are duck-typed on the reference's structure (models/causal_lm.py:20-58): ``embedding``,
``layers`` (each with ``norm``, ``mamba``), ``norm``, ``lm_head``; each ``mamba`` has
MambaSimple's parameter names (modules/mamba_simple.py:33-85).  Dropout is not applied
(inference).
"""
from __future__ import annotations

import torch

from . import _lib as L
from .inner import mamba_inner_prefill
from .norm import rms_norm_fn
from .selective_scan_interface import _cuda_device


class _BlockParams:
    """A MambaSimple block's parameters in the form the step kernels take, computed once."""

    def __init__(self, blk):
        self.blk = blk
        self.d = blk.D.shape[0]
        self.n = blk.log_A.shape[1]
        self.R = blk.delta_proj.weight.shape[1]
        self.A = (-torch.exp(blk.log_A.detach().float())).contiguous()
        self.D = blk.D.detach().float().contiguous()
        self.dt_bias = blk.delta_proj.bias.detach().float().contiguous()
        w = blk.short_conv.weight.detach()
        self.conv_w = w.reshape(w.shape[0], -1).float().contiguous()
        self.conv_b = None if blk.short_conv.bias is None else blk.short_conv.bias.detach().float().contiguous()
        self.K = self.conv_w.shape[1]


@torch.no_grad()
def mamba_simple_prefill(block, hidden_states, params: _BlockParams | None = None):
    """Block forward over a prompt (batch, L, d_model) from zero states.  Returns
    (output (batch, L, d_model), conv_state, ssm_state)."""
    p = params or _BlockParams(block)
    xz = block.input_proj(hidden_states)
    return mamba_inner_prefill(xz, p.conv_w, p.conv_b, block.ssm_param_proj.weight, block.delta_proj.weight,
                               block.delta_proj.bias, block.output_proj.weight, block.output_proj.bias, p.A, p.D,
                               True)


def mamba_mixer_step(xz, conv_state, ssm_state, p: _BlockParams, x_proj_weight, delta_proj_weight):
    """The mixer of one decode step (conv step, x projection, delta projection, SSM step, gate)
    in one kernel (``ss_mamba_step``): xz (batch, 2 d) -> y (batch, d); both states update in
    place."""
    _cuda_device(xz, conv_state, ssm_state, x_proj_weight, delta_proj_weight)
    b = xz.shape[0]
    io = xz.dtype
    if xz.stride(-1) != 1:
        xz = xz.contiguous()
    Wx = x_proj_weight if x_proj_weight.dtype == io else x_proj_weight.to(io)
    Wdt = delta_proj_weight if delta_proj_weight.dtype == io else delta_proj_weight.to(io)
    Wx, Wdt = Wx.contiguous(), Wdt.contiguous()
    for t, shape in ((conv_state, (b, p.d, p.K - 1)), (ssm_state, (b, p.d, p.n))):
        if t.dtype != torch.float32 or tuple(t.shape) != shape or not t.is_contiguous():
            raise ValueError(f"state must be a contiguous fp32 {shape} tensor")
    y = torch.empty((b, p.d), dtype=io, device=xz.device)
    args = L.MambaStepArgs(b, p.d, p.n, p.K, p.R, L.dtype_code(io), 1, xz.data_ptr(), xz.stride(0),
                           L.ptr(conv_state) if p.K > 1 else None, p.conv_w.data_ptr(), L.ptr(p.conv_b),
                           Wx.data_ptr(), Wdt.data_ptr(), p.dt_bias.data_ptr(), p.A.data_ptr(), p.D.data_ptr(),
                           ssm_state.data_ptr(), y.data_ptr(), y.stride(0))
    with torch.cuda.device(xz.device):
        L.check(L.lib().ss_mamba_step(args, L.stream_of(xz.device)), "ss_mamba_step")
    return y


@torch.no_grad()
def mamba_simple_step(block, hidden, conv_state, ssm_state, params: _BlockParams | None = None):
    """One token (batch, d_model) through a block; updates both states in place.  Three kernels:
    the input projection (GEMM), the fused mixer step, the output projection (GEMM)."""
    p = params or _BlockParams(block)
    xz = block.input_proj(hidden)                                    # (b, 2 d)
    y = mamba_mixer_step(xz, conv_state, ssm_state, p, block.ssm_param_proj.weight, block.delta_proj.weight)
    return block.output_proj(y)


class Decoder:
    """Incremental decoding of a CausalLM-shaped model for a fixed batch size.

    ``prefill(input_ids)`` runs the prompt and returns the last position's logits;
    ``step(token_ids)`` feeds one token per sequence and returns the next logits (fp32).
    With ``cuda_graph`` the step is captured on first use and replayed afterwards."""

    def __init__(self, model, batch: int, cuda_graph: bool = True):
        self.model = model
        self.batch = batch
        self.params = [_BlockParams(layer.mamba) for layer in model.layers]
        # fp32 norm weights, cast once (a per-call cast would be one more kernel per layer and step)
        self.norms = [(layer.norm.weight.detach().float().contiguous(), layer.norm.eps) for layer in model.layers]
        self.final_norm = (model.norm.weight.detach().float().contiguous(), model.norm.eps)
        dev = model.lm_head.weight.device
        self.conv_states = [torch.zeros(batch, p.d, p.K - 1, device=dev) for p in self.params]
        self.ssm_states = [torch.zeros(batch, p.d, p.n, device=dev) for p in self.params]
        self.cuda_graph = cuda_graph
        self.graph = None
        self.tok = torch.zeros(batch, dtype=torch.long, device=dev)
        self.logits = None

    @torch.no_grad()
    def prefill(self, input_ids):
        if input_ids.shape[0] != self.batch:
            raise ValueError(f"batch {input_ids.shape[0]} != decoder batch {self.batch}")
        m = self.model
        h = m.embedding(input_ids)
        res = y = None
        for i, layer in enumerate(m.layers):
            # the residual add of the previous block fused with this block's RMSNorm
            x, res = self._norm(i, h if res is None else y, res)
            y, cs, ss = mamba_simple_prefill(layer.mamba, x, self.params[i])
            self.conv_states[i].copy_(cs)
            self.ssm_states[i].copy_(ss)
        w, eps = self.final_norm
        return m.lm_head(rms_norm_fn(y[:, -1], w, res[:, -1], eps)).float()

    def _norm(self, i, x, res):
        w, eps = self.norms[i]
        return rms_norm_fn(x, w, res, eps, True, True)

    def _step_eager(self, tok):
        m = self.model
        h = m.embedding(tok)
        res = y = None
        for i, layer in enumerate(m.layers):
            x, res = self._norm(i, h if res is None else y, res)
            y = mamba_simple_step(layer.mamba, x, self.conv_states[i], self.ssm_states[i], self.params[i])
        w, eps = self.final_norm
        return m.lm_head(rms_norm_fn(y, w, res, eps)).float()

    @torch.no_grad()
    def step(self, token_ids):
        if not self.cuda_graph:
            return self._step_eager(token_ids)
        self.tok.copy_(token_ids)
        if self.graph is None:
            self._capture()
        self.graph.replay()
        return self.logits

    def _capture(self):
        # warm-up on a side stream (library handles, cuBLAS workspaces), states saved around it
        saved = [t.clone() for t in self.conv_states + self.ssm_states]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step_eager(self.tok)
        torch.cuda.current_stream().wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = self._step_eager(self.tok)
        for t, v in zip(self.conv_states + self.ssm_states, saved):
            t.copy_(v)


def _sample(logits, temperature, top_k, generator):
    if temperature == 0:
        return logits.argmax(-1)
    logits = logits / temperature
    if top_k is not None:
        kth = torch.topk(logits, top_k, dim=-1).values[:, -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    return torch.multinomial(torch.softmax(logits, -1), 1, generator=generator).squeeze(-1)


@torch.no_grad()
def generate(model, input_ids, max_new_tokens: int = 50, temperature: float = 1.0, top_k: int | None = None,
             cuda_graph: bool = True, generator: torch.Generator | None = None):
    """Continue every sequence of ``input_ids`` (batch, L) by ``max_new_tokens`` tokens —
    the signature of the reference's stub CausalLM.generate (models/causal_lm.py:61), with
    ``temperature = 0`` meaning greedy.  Returns (batch, L + max_new_tokens) token ids."""
    dec = Decoder(model, input_ids.shape[0], cuda_graph=cuda_graph)
    out = [input_ids]
    logits = dec.prefill(input_ids)
    for i in range(max_new_tokens):
        tok = _sample(logits, temperature, top_k, generator)
        out.append(tok[:, None])
        if i + 1 < max_new_tokens:
            logits = dec.step(tok)
    return torch.cat(out, 1)

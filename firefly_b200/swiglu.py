"""SwiGLU MLP block built from BitLinear — the Llama-7B-shaped training workload.

``y = down(silu(g) * u)`` with ``[g | u] = gate_up(x)``: the gate and up projections
``d -> f`` are the two halves of one BitLinear ``d -> 2f`` (one int8 weight
``[2f, d]`` with per-row scales, the usual fused gate/up layout), and down is a
BitLinear ``f -> d``; no bias.  The reference ships no model code; this block is the
harness for its SwiGLU-MLP configuration (d_model 4096, ffn 11008).

``SwiGLUMLPFn`` is the fused training op of the block.  It computes exactly what the
composition ``down(F.silu(g) * u)`` of two BitLinear layers and torch's elementwise
ops computes, with the elementwise work moved into the quantisers:

* forward: ``ff_swiglu_gemm_i8`` computes ``h = silu(g) * u`` and its absmax in the gate/up
  GEMM's epilogue and quantises h (f a multiple of 128; otherwise ``ff_swiglu_quant_i8``
  computes h from the GEMM output in the quantiser's absmax pass);
* backward: ``ff_swiglu_bwd_gemm_i8`` forms ``[dg | du]`` from the dh tile and the saved g
  and u in the epilogue of the GEMM ``dh = dY·W_down`` (dh is never written) and quantises
  it (otherwise ``ff_swiglu_bwd_quant_i8`` does that from dh); ``dX`` is one GEMM over
  ``K = 2f``.

The unfused composition (``fused=False``, or ffn not a multiple of 8) runs the same
BitLinear kernels with torch's elementwise ops in between.
"""
from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from . import _capi
from .bitLinear import BitLinear
from .fireflykernels import (
    _accumulate_weight_grad,
    _as_float_input,
    _quantize_activation,
    clear_activation_cache,
    _weight_grad_gemm,
    _weight_operand,
)


class SwiGLUMLPFn(torch.autograd.Function):
    """Fused forward/backward of ``down(silu(g) * u)``, ``[g | u] = gate_up(x)``."""

    @staticmethod
    def forward(ctx, x2d, gu_weight, gu_scale, gu_handle, d_weight, d_scale, d_bias, d_handle):
        _capi._require_cuda(x2d, gu_weight, gu_scale, d_weight, d_scale, d_bias)
        F2, K = gu_weight.shape
        O, Fh = d_weight.shape
        if F2 != 2 * Fh or x2d.dim() != 2 or x2d.shape[1] != K:
            raise ValueError(f"SwiGLU shapes: x {tuple(x2d.shape)}, gate_up {tuple(gu_weight.shape)}, "
                             f"down {tuple(d_weight.shape)}")
        x = _as_float_input(x2d)
        T = x.shape[0]
        gu_ws = gu_scale.to(torch.float32).contiguous()
        d_ws = d_scale.to(torch.float32).contiguous()
        b = None if d_bias is None else d_bias.detach().to(torch.float32).contiguous()
        need_grad = any(ctx.needs_input_grad)
        y = torch.empty((T, O), dtype=torch.bfloat16, device=x.device)
        saved = (None, None, None, None, None)
        if T > 0:
            q_x, s_x, q_xt, s_xc = _quantize_activation(x, with_cols=need_grad)
            w_gu = _weight_operand(gu_handle, gu_weight)
            if Fh % 128 == 0:  # h and its absmax come out of the gate/up GEMM's epilogue
                gu, q_h, s_h, q_ht, s_hc, _ = _capi.swiglu_gemm(q_x, w_gu, K, s_x, gu_ws, cols=need_grad)
            else:
                gu = _capi.gemm_i8(q_x, w_gu, K, scale_a=s_x, scale_b=gu_ws, out_kind=_capi.FF_OUT_BF16)
                q_h, s_h, q_ht, s_hc, _ = _capi.swiglu_quant(gu, cols=need_grad)
            _capi.gemm_i8(q_h, _weight_operand(d_handle, d_weight), Fh, scale_a=s_h, scale_b=d_ws,
                          bias=b, out_kind=_capi.FF_OUT_BF16, out=y)
            if need_grad:
                saved = (q_xt, s_xc, gu, q_ht, s_hc)
        ctx.save_for_backward(*saved, gu_weight, gu_ws, d_weight, d_ws)
        ctx.handles = (int(gu_handle), int(d_handle))
        ctx.has_bias = d_bias is not None
        ctx.T = T
        return y

    @staticmethod
    def backward(ctx, grad_out):
        clear_activation_cache()
        q_xt, s_xc, gu, q_ht, s_hc, gu_weight, gu_ws, d_weight, d_ws = ctx.saved_tensors
        gu_handle, d_handle = ctx.handles
        F2, K = gu_weight.shape
        O, Fh = d_weight.shape
        T = ctx.T
        dev = grad_out.device
        need_dx = ctx.needs_input_grad[0]
        if T == 0:
            for h, (o, k) in ((gu_handle, (F2, K)), (d_handle, (O, Fh))):
                _accumulate_weight_grad(h, torch.zeros((o, k), dtype=torch.bfloat16, device=dev))
            dx = torch.zeros((0, K), dtype=grad_out.dtype, device=dev) if need_dx else None
            db = torch.zeros((O,), dtype=grad_out.dtype, device=dev) if ctx.has_bias else None
            return dx, None, None, None, None, None, db, None
        dy = grad_out.to(torch.bfloat16).contiguous()
        # down projection: dH = dY·W_d, dW_d = dYᵀ·H, db = Σ dY
        q_g, s_g, q_dyt, s_dy, *db = _capi.quant_dual(dy, row_colmul=d_ws, colsum=ctx.has_bias)
        w_d = _weight_operand(d_handle, d_weight)
        if Fh % 128 == 0:  # dH, the SwiGLU backward and [dg | du]'s absmax in one GEMM epilogue
            q_d, s_d, q_dt, s_dc, _ = _capi.swiglu_bwd_gemm(q_g, w_d, O, s_g, gu, colmul=gu_ws, rows=need_dx)
        else:
            dh = _capi.gemm_i8(q_g, w_d, O, scale_a=s_g, out_kind=_capi.FF_OUT_BF16, b_kn_cols=Fh)
            q_d, s_d, q_dt, s_dc, _ = _capi.swiglu_bwd_quant(dh, gu, colmul=gu_ws, rows=need_dx)
        _weight_grad_gemm(d_handle, q_dyt, s_dy, q_ht, s_hc, O, Fh, T, dev)
        db = db[0].to(grad_out.dtype) if ctx.has_bias else None
        dx = None
        if need_dx:
            dx = _capi.gemm_i8(q_d, _weight_operand(gu_handle, gu_weight), F2, scale_a=s_d,
                               out_kind=_capi.FF_OUT_BF16, b_kn_cols=K).to(grad_out.dtype)
        _weight_grad_gemm(gu_handle, q_dt, s_dc, q_xt, s_xc, F2, K, T, dev)
        return dx, None, None, None, None, None, db, None


class SwiGLUMLP(nn.Module):
    def __init__(self, d_model: int, ffn: int, fused: bool = True):
        super().__init__()
        self.ffn = int(ffn)
        self.gate_up = BitLinear(d_model, 2 * ffn)
        self.down = BitLinear(ffn, d_model)
        self.fused = fused

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused and self.ffn % 8 == 0:
            if x.shape[-1] != self.gate_up.in_features:
                raise ValueError(f"expected input last dim {self.gate_up.in_features}, got {x.shape[-1]}")
            y = SwiGLUMLPFn.apply(x.reshape(-1, x.shape[-1]), self.gate_up.int_weight,
                                  self.gate_up.weight_scale, self.gate_up._registered_handle,
                                  self.down.int_weight, self.down.weight_scale, self.down.bias,
                                  self.down._registered_handle)
            return y.view(*x.shape[:-1], y.shape[-1])
        g, u = self.gate_up(x).chunk(2, dim=-1)
        return self.down(F.silu(g) * u)

    @torch.no_grad()
    def init_normal_(self, std: float = 0.02, generator: torch.Generator | None = None) -> None:
        """Weights ~ N(0, std) quantised per row (the benchmark initialisation)."""
        from .fireflykernels import quantize_fp_to_int8

        for lin in (self.gate_up, self.down):
            w = torch.empty(lin.out_features, lin.in_features, device=lin.int_weight.device)
            w.normal_(0.0, std, generator=generator)
            q, s = quantize_fp_to_int8(w)
            lin.int_weight.copy_(q)
            lin.weight_scale.copy_(s)

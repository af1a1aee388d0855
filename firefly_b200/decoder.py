"""Decoder-only transformer with every Linear a BitLinear — the data-parallel training workload.

The reference ships no model code; this is the harness for its 1.3B data-parallel
configuration (24 layers, d_model 2048, 16 heads, ffn 8192 with GELU, vocab 32000,
sequence 2048).  Per layer (pre-LayerNorm):

    x = x + proj(attention(qkv(ln1(x))))        qkv: BitLinear d -> 3d, proj: BitLinear d -> d
    x = x + down(gelu(up(ln2(x))))              up:  BitLinear d -> ffn, down: BitLinear ffn -> d

then ``logits = lm_head(ln_f(x))`` (BitLinear d -> vocab) and the mean token cross-entropy.
The residual stream is bf16; causal attention (torch's ``scaled_dot_product_attention``) and the
loss are torch ops around the BitLinear path; the GELU (tanh form) and its backward run in the
epilogues of the MLP's GEMMs (``GeluMLPFn``), and each LayerNorm quantises its output for the
BitLinear that reads it (``LayerNormQuantFn``).
Dense parameters — token and position embeddings, LayerNorm weights and biases — are
stepped by ``AdamW8bitDense`` (block-wise 8-bit for the embeddings, fp32 moments for the
norms), the BitLinear weights by the fused DQT 8-bit AdamW, as ``FireFlyOptim`` splits
them (fireflyoptim.py:83-211).

``train_step`` runs one optimizer step over a list of micro-batches: the BitLinear weight
gradients accumulate in the grad cache (fireflykernels.py:200-210), the dense gradients in
``.grad``, and the optimizer steps once.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Sequence

import torch
from torch import nn
from torch.nn import functional as F

from . import _capi
from .bitLinear import BitLinear, collect_bitlinear_modules
from .fireflykernels import (
    _ACT_CACHE,
    _accumulate_weight_grad,
    _act_key,
    _as_float_input,
    _quantize_activation,
    clear_activation_cache,
    _weight_grad_gemm,
    _weight_operand,
)


@dataclass(frozen=True)
class DecoderConfig:
    vocab: int = 32000
    d_model: int = 2048
    heads: int = 16
    ffn: int = 8192
    layers: int = 24
    max_seq: int = 2048

    @property
    def bit_params(self) -> int:
        d = self.d_model
        return self.layers * (3 * d * d + d * d + 2 * d * self.ffn) + d * self.vocab

    def int8_ops_per_token(self) -> float:
        """Int8 GEMM operations per token of one training step (forward, dX and dW GEMMs)."""
        return 6.0 * self.bit_params


DECODER_1P3B = DecoderConfig()


class LayerNormQuantFn(torch.autograd.Function):
    """LayerNorm of a bf16 input with fp32 weight and bias (``ff_layernorm_i8``) that also
    quantises its output for the BitLinear that reads it next: the dual codes go into the op
    layer's activation cache under the output's key, so that layer's forward finds them instead
    of running the quantiser.  Backward: ``ff_layernorm_bwd`` (dx, dgamma, dbeta)."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps, with_cols):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        y, mean, rstd, codes = _capi.layernorm_quant(x2, weight, bias, eps, rows=True, cols=with_cols)
        if not with_cols:
            codes = (codes[0], codes[1], None, None)
        _ACT_CACHE["entry"] = (_act_key(y, with_cols), y, codes)
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.shape, ctx.in_dtype = shape, x.dtype
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, mean, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape).to(torch.bfloat16).contiguous()
        want_dx = ctx.needs_input_grad[0]
        want_w = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        dx, dg, db = _capi.layernorm_bwd(dy2, x2, mean, rstd, weight, dx=want_dx, wgrad=want_w)
        if dx is not None:
            dx = dx.view(ctx.shape).to(ctx.in_dtype)
        return dx, dg, db, None, None


class LayerNormBF16(nn.Module):
    """LayerNorm with fp32 parameters over a bf16 input.  ``fused``: ``LayerNormQuantFn`` (the
    output's int8 codes for the next BitLinear come out of the same call); otherwise torch's
    LayerNorm with the parameters cast to the input's dtype per call."""

    def __init__(self, d: int, eps: float = 1e-5, fused: bool = False):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))
        self.bias = nn.Parameter(torch.zeros(d))
        self.eps = eps
        self.fused = fused

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        d = x.shape[-1]
        if self.fused and x.is_cuda and d % 8 == 0 and d <= 4096:
            with_cols = torch.is_grad_enabled() and (x.requires_grad or self.weight.requires_grad
                                                     or self.bias.requires_grad)
            return LayerNormQuantFn.apply(x, self.weight, self.bias, self.eps, with_cols)
        return F.layer_norm(x, (d,), self.weight.to(x.dtype), self.bias.to(x.dtype), self.eps)


class GeluMLPFn(torch.autograd.Function):
    """Fused forward/backward of ``down(gelu(up(x)))`` (tanh GELU), up and down BitLinear.

    It computes exactly what the composition of the two BitLinear layers and torch's
    ``F.gelu(·, approximate="tanh")`` computes, with the elementwise work moved into the GEMMs:
    the up GEMM's epilogue writes u and h = gelu(u) and takes h's absmax (``ff_gelu_gemm_i8``),
    and the epilogue of the backward GEMM dh = dY·W_down forms du = dh·gelu'(u) and takes its
    absmax (``ff_gelu_bwd_gemm_i8``; dh is never written).
    """

    @staticmethod
    def forward(ctx, x2d, up_weight, up_scale, up_handle, d_weight, d_scale, d_bias, d_handle):
        _capi._require_cuda(x2d, up_weight, up_scale, d_weight, d_scale, d_bias)
        Fu, K = up_weight.shape
        O, Fh = d_weight.shape
        if Fu != Fh or x2d.dim() != 2 or x2d.shape[1] != K:
            raise ValueError(f"GELU MLP shapes: x {tuple(x2d.shape)}, up {tuple(up_weight.shape)}, "
                             f"down {tuple(d_weight.shape)}")
        x = _as_float_input(x2d)
        T = x.shape[0]
        up_ws = up_scale.to(torch.float32).contiguous()
        d_ws = d_scale.to(torch.float32).contiguous()
        b = None if d_bias is None else d_bias.detach().to(torch.float32).contiguous()
        need_grad = any(ctx.needs_input_grad)
        y = torch.empty((T, O), dtype=torch.bfloat16, device=x.device)
        saved = (None, None, None, None, None)
        if T > 0:
            q_x, s_x, q_xt, s_xc = _quantize_activation(x, with_cols=need_grad)
            u, q_h, s_h, q_ht, s_hc, _ = _capi.gelu_gemm(q_x, _weight_operand(up_handle, up_weight), K, s_x, up_ws,
                                                         cols=need_grad)
            _capi.gemm_i8(q_h, _weight_operand(d_handle, d_weight), Fh, scale_a=s_h, scale_b=d_ws, bias=b,
                          out_kind=_capi.FF_OUT_BF16, out=y)
            if need_grad:
                saved = (q_xt, s_xc, u, q_ht, s_hc)
        ctx.save_for_backward(*saved, up_weight, up_ws, d_weight, d_ws)
        ctx.handles = (int(up_handle), int(d_handle))
        ctx.has_bias = d_bias is not None
        ctx.T = T
        return y

    @staticmethod
    def backward(ctx, grad_out):
        clear_activation_cache()
        q_xt, s_xc, u, q_ht, s_hc, up_weight, up_ws, d_weight, d_ws = ctx.saved_tensors
        up_handle, d_handle = ctx.handles
        Fu, K = up_weight.shape
        O, Fh = d_weight.shape
        T = ctx.T
        dev = grad_out.device
        need_dx = ctx.needs_input_grad[0]
        if T == 0:
            for h, (o, k) in ((up_handle, (Fu, K)), (d_handle, (O, Fh))):
                _accumulate_weight_grad(h, torch.zeros((o, k), dtype=torch.bfloat16, device=dev))
            dx = torch.zeros((0, K), dtype=grad_out.dtype, device=dev) if need_dx else None
            db = torch.zeros((O,), dtype=grad_out.dtype, device=dev) if ctx.has_bias else None
            return dx, None, None, None, None, None, db, None
        dy = grad_out.to(torch.bfloat16).contiguous()
        # down projection: dH = dY·W_d (GELU backward and du's absmax in its epilogue), dW_d = dYᵀ·H
        q_g, s_g, q_dyt, s_dy, *db = _capi.quant_dual(dy, row_colmul=d_ws, colsum=ctx.has_bias)
        q_d, s_d, q_dt, s_dc, _ = _capi.gelu_bwd_gemm(q_g, _weight_operand(d_handle, d_weight), O, s_g, u,
                                                      colmul=up_ws, rows=need_dx)
        _weight_grad_gemm(d_handle, q_dyt, s_dy, q_ht, s_hc, O, Fh, T, dev)
        db = db[0].to(grad_out.dtype) if ctx.has_bias else None
        dx = None
        if need_dx:
            dx = _capi.gemm_i8(q_d, _weight_operand(up_handle, up_weight), Fu, scale_a=s_d,
                               out_kind=_capi.FF_OUT_BF16, b_kn_cols=K).to(grad_out.dtype)
        _weight_grad_gemm(up_handle, q_dt, s_dc, q_xt, s_xc, Fu, K, T, dev)
        return dx, None, None, None, None, None, db, None


class DecoderLayer(nn.Module):
    def __init__(self, cfg: DecoderConfig, fused: bool = True, fused_norm: bool | None = None):
        super().__init__()
        d = cfg.d_model
        if d % cfg.heads:
            raise ValueError(f"d_model {d} is not a multiple of heads {cfg.heads}")
        fused_norm = fused if fused_norm is None else fused_norm
        self.heads = cfg.heads
        self.ln1 = LayerNormBF16(d, fused=fused_norm)
        self.qkv = BitLinear(d, 3 * d)
        self.proj = BitLinear(d, d)
        self.ln2 = LayerNormBF16(d, fused=fused_norm)
        self.up = BitLinear(d, cfg.ffn)
        self.down = BitLinear(cfg.ffn, d)
        self.fused = fused

    def mlp(self, x: torch.Tensor) -> torch.Tensor:
        """down(gelu(up(x))): the fused GELU MLP op, or the composition of the two BitLinear
        layers and torch's GELU (``fused=False``, an up bias, or ffn not a multiple of 32)."""
        if self.fused and self.up.bias is None and self.up.out_features % 32 == 0:
            y = GeluMLPFn.apply(x.reshape(-1, x.shape[-1]), self.up.int_weight, self.up.weight_scale,
                                self.up._registered_handle, self.down.int_weight, self.down.weight_scale,
                                self.down.bias, self.down._registered_handle)
            return y.view(*x.shape[:-1], y.shape[-1])
        return self.down(F.gelu(self.up(x), approximate="tanh"))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, d = x.shape
        hd = d // self.heads
        # q, k, v as [B, H, S, hd] views of the packed [B, S, 3, H, hd] output (no copies; the
        # backward of unbind writes their gradients into one packed buffer), and the attention
        # output comes back in [B, S, H, hd] memory order, so the reshape below is a view
        q, k, v = self.qkv(self.ln1(x)).view(B, S, 3, self.heads, hd).unbind(2)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        x = x + self.proj(a.transpose(1, 2).reshape(B, S, d))
        return x + self.mlp(self.ln2(x))


class BitDecoder(nn.Module):
    """``fused``: the GELU MLP op; ``fused_norm`` (default: ``fused``): the LayerNorms that
    quantise their outputs for the next BitLinear."""

    def __init__(self, cfg: DecoderConfig = DECODER_1P3B, fused: bool = True, fused_norm: bool | None = None):
        super().__init__()
        fused_norm = fused if fused_norm is None else fused_norm
        self.cfg = cfg
        self.tok = nn.Embedding(cfg.vocab, cfg.d_model)
        self.pos = nn.Parameter(torch.zeros(cfg.max_seq, cfg.d_model))
        self.layers = nn.ModuleList(DecoderLayer(cfg, fused=fused, fused_norm=fused_norm) for _ in range(cfg.layers))
        self.ln_f = LayerNormBF16(cfg.d_model, fused=fused_norm)
        self.lm_head = BitLinear(cfg.d_model, cfg.vocab)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """Logits (bf16 [B, S, vocab]) of token ids [B, S]."""
        S = ids.shape[1]
        if S > self.cfg.max_seq:
            raise ValueError(f"sequence {S} longer than max_seq {self.cfg.max_seq}")
        x = (self.tok(ids) + self.pos[:S]).to(torch.bfloat16)
        for layer in self.layers:
            x = layer(x)
        return self.lm_head(self.ln_f(x))

    def loss(self, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        logits = self(ids)
        return F.cross_entropy(logits.view(-1, logits.shape[-1]), targets.reshape(-1))

    def bit_modules(self) -> list[BitLinear]:
        return collect_bitlinear_modules(self)

    def dense_parameters(self) -> list[nn.Parameter]:
        return [p for p in self.parameters() if p.requires_grad]

    @torch.no_grad()
    def init_normal_(self, std: float = 0.02, generator: torch.Generator | None = None) -> None:
        """Every weight ~ N(0, std) (BitLinear weights quantised per row), LayerNorms at (1, 0)."""
        from .fireflykernels import quantize_fp_to_int8

        for lin in self.bit_modules():
            w = torch.empty(lin.out_features, lin.in_features, device=lin.int_weight.device)
            w.normal_(0.0, std, generator=generator)
            q, s = quantize_fp_to_int8(w)
            lin.int_weight.copy_(q)
            lin.weight_scale.copy_(s)
        self.tok.weight.normal_(0.0, std, generator=generator)
        self.pos.normal_(0.0, std, generator=generator)


def build_decoder(cfg: DecoderConfig, device: torch.device, seed: int = 0, fused: bool = True,
                  fused_norm: bool | None = None) -> BitDecoder:
    """The decoder on ``device`` with N(0, 0.02) weights drawn from a seeded generator."""
    with torch.device(device):
        model = BitDecoder(cfg, fused=fused, fused_norm=fused_norm)
    gen = torch.Generator(device=device).manual_seed(seed)
    model.init_normal_(0.02, generator=gen)
    return model


def train_step(model: BitDecoder, opt, micro_batches: Sequence[tuple[torch.Tensor, torch.Tensor]]) -> torch.Tensor:
    """One optimizer step over ``micro_batches`` of (ids, targets); returns the mean loss
    (a device scalar, no host sync).  With a data-parallel optimizer that has ``no_sync``
    (``ZeroFireFlyOptim``), every backward but the last only accumulates, and the last one
    starts the gradient reduction bucket by bucket."""
    total = None
    n = len(micro_batches)
    for k, (ids, targets) in enumerate(micro_batches):
        last = k == n - 1
        ctx = opt.no_sync() if (not last and hasattr(opt, "no_sync")) else contextlib.nullcontext()
        with ctx:
            loss = model.loss(ids, targets)
            (loss / n).backward()
        total = loss.detach() if total is None else total + loss.detach()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return total / n


def synthetic_batches(cfg: DecoderConfig, sequences: int, seq: int, micro: int, device: torch.device,
                      seed: int = 0) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Token ids uniform over the vocabulary, split into micro-batches of ``micro`` sequences;
    the targets are the ids shifted by one."""
    gen = torch.Generator(device=device).manual_seed(seed)
    ids = torch.randint(0, cfg.vocab, (sequences, seq + 1), device=device, generator=gen)
    out = []
    for i in range(0, sequences, micro):
        chunk = ids[i:i + micro]
        out.append((chunk[:, :-1].contiguous(), chunk[:, 1:].contiguous()))
    return out


def attention_flops_per_sequence(cfg: DecoderConfig, seq: int) -> float:
    """Causal attention matmul FLOPs of one training step per sequence (forward 2 matmuls,
    backward 5, each 2·S·S/2·d per layer)."""
    return cfg.layers * 7 * 2 * seq * (seq / 2) * cfg.d_model


__all__ = ["DecoderConfig", "DECODER_1P3B", "BitDecoder", "DecoderLayer", "GeluMLPFn", "LayerNormBF16",
           "LayerNormQuantFn", "build_decoder",
           "train_step", "synthetic_batches", "attention_flops_per_sequence"]

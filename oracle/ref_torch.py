"""The reference's live PyTorch path, restated op for op.  TEST INFRASTRUCTURE ONLY.

This module is a checker and the CPU baseline.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline / reference legs of ``bench.py``
may import it; the product path (``firefly_b200``) never does.

The reference (fumitoshi0524/FireFly) is pure Python over torch.  Its own files
cannot be shipped with this repository, so the ops of its live path are restated
here in the same order, with the same dtypes and the same torch kernels, which
makes the results on the CPU bit-identical to the reference's (pinned by
``tests/test_oracle_golden.py`` against fixtures produced by running the
reference itself, ``tests/golden/make_golden.py``):

* ``linear_forward``      ``_forward_bf16``  fireflykernels.py:164-176 (bf16 dequantised
                          weight, ``torch.matmul``, bias added in place)
* ``linear_backward``     ``_backward_impl`` fireflykernels.py:184-210 (dX, dW, db in bf16;
                          dW added to the per-handle grad cache)
* ``encode_signed`` …     mu-law blockwise codecs fireflyoptim.py:13-80
* ``dqt_step``            the bit-module branch of ``FireFlyOptim.step``
                          fireflyoptim.py:136-209 (including ``update_int8_weight_``,
                          fireflykernels.py:218-223)
* ``SwiGLUBlock``         the benchmark block built from two such layers (gate/up as one
                          ``d -> 2f`` layer, down ``f -> d``) with torch's ``silu`` in
                          between; the reference ships no model code, so this block is
                          what a user of the reference would write.

Every function is device-agnostic torch code; on the CPU it is the reference's
CPU implementation of the path.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

_MU = 255.0
_1_OVER_LN1P_MU = 1.0 / 5.545177444479562  # fireflyoptim.py:10


# --------------------------------------------------------------------------
# BitLinear forward / backward (fireflykernels.py:164-210)
# --------------------------------------------------------------------------
def _dequantised_weight(int_weight: torch.Tensor, weight_scale: torch.Tensor) -> torch.Tensor:
    # fireflykernels.py:166-168 and :187-189: bf16 codes times the bf16 row scale
    return int_weight.to(torch.bfloat16) * weight_scale.to(torch.bfloat16).unsqueeze(1)


def linear_forward(x2d, int_weight, weight_scale, bias=None):
    """Returns ``(y, x_bf16)``; ``x_bf16`` is what the reference saves for backward."""
    xb = x2d.to(torch.bfloat16)
    y = torch.matmul(xb, _dequantised_weight(int_weight, weight_scale).t())
    if bias is not None:
        y.add_(bias)
    return y, xb


def linear_backward(grad_out, x_bf16, int_weight, weight_scale, has_bias=False, grad_cache=None, handle=0):
    """Returns ``(grad_in, grad_bias)``; dW (bf16) is stored in or added to ``grad_cache[handle]``."""
    go = grad_out.to(torch.bfloat16)
    w = int_weight.to(torch.bfloat16) * weight_scale.to(torch.bfloat16).unsqueeze(1)
    grad_in = torch.matmul(go, w)
    grad_w = torch.matmul(go.t(), x_bf16)
    if grad_cache is not None:
        prev = grad_cache.get(handle)
        if prev is None:
            grad_cache[handle] = grad_w.to(dtype=torch.bfloat16)
        else:
            prev.add_(grad_w.to(dtype=torch.bfloat16))
    grad_bias = go.sum(dim=0).to(dtype=grad_out.dtype) if has_bias else None
    return grad_in.to(dtype=grad_out.dtype), grad_bias


class _LinearFn(torch.autograd.Function):
    """Autograd wrapper of the two functions above (the role of ``Int8LinearFn``)."""

    @staticmethod
    def forward(ctx, x2d, int_weight, weight_scale, bias, grad_cache, handle):
        y, xb = linear_forward(x2d, int_weight, weight_scale, bias)
        ctx.save_for_backward(xb, int_weight, weight_scale)
        ctx.grad_cache, ctx.handle, ctx.has_bias = grad_cache, handle, bias is not None
        return y

    @staticmethod
    def backward(ctx, grad_out):
        xb, iw, ws = ctx.saved_tensors
        gi, gb = linear_backward(grad_out, xb, iw, ws, ctx.has_bias, ctx.grad_cache, ctx.handle)
        return gi, None, None, gb, None, None


# --------------------------------------------------------------------------
# mu-law blockwise codecs (fireflyoptim.py:13-80)
# --------------------------------------------------------------------------
def _as_blocks(t: torch.Tensor, bs: int) -> torch.Tensor:
    flat = t.contiguous().view(-1)
    nb = (flat.numel() + bs - 1) // bs
    pad = nb * bs - flat.numel()
    if pad:
        flat = torch.cat([flat, torch.zeros(pad, device=flat.device, dtype=flat.dtype)])
    return flat.view(nb, bs)


def encode_signed(x: torch.Tensor, bs: int):
    blocks = _as_blocks(x.float(), bs)
    absmax = blocks.abs().amax(dim=1).clamp_min(1e-12)
    n = (blocks / absmax.unsqueeze(1)).clamp(-1.0, 1.0)
    comp = torch.sign(n) * torch.log1p(_MU * n.abs()) * _1_OVER_LN1P_MU
    codes = torch.round(comp * 127.0).clamp(-127, 127).to(torch.int16)
    return (codes.view(-1)[: x.numel()] + 128).to(torch.uint8).view_as(x), absmax


def encode_unsigned(x: torch.Tensor, bs: int):
    blocks = _as_blocks(x.float(), bs)
    absmax = blocks.amax(dim=1).clamp_min(1e-12)
    n = (blocks / absmax.unsqueeze(1)).clamp(0.0, 1.0)
    comp = torch.log1p(_MU * n) * _1_OVER_LN1P_MU
    codes = torch.round(comp * 255.0).clamp(0, 255)
    return codes.view(-1)[: x.numel()].to(torch.uint8).view_as(x), absmax


def decode_signed(q: torch.Tensor, absmax: torch.Tensor, bs: int, shape):
    y = ((_as_blocks(q, bs).float() - 128.0) / 127.0).clamp(-1.0, 1.0)
    n = torch.sign(y) * (torch.exp(y.abs() / _1_OVER_LN1P_MU) - 1.0) / _MU
    return (n * absmax.unsqueeze(1)).view(-1)[: q.numel()].view(shape)


def decode_unsigned(q: torch.Tensor, absmax: torch.Tensor, bs: int, shape):
    y = (_as_blocks(q, bs).float() / 255.0).clamp(0.0, 1.0)
    n = (torch.exp(y / _1_OVER_LN1P_MU) - 1.0) / _MU
    return (n * absmax.unsqueeze(1)).view(-1)[: q.numel()].view(shape)


def init_state(shape, device="cpu", bs: int = 256) -> dict:
    """The reference's first-step states: zeros encoded by its own codecs (fireflyoptim.py:142-161)."""
    z = torch.zeros(shape, dtype=torch.float32, device=device)
    m_q, m_a = encode_signed(z, bs)
    v_q, v_a = encode_unsigned(z, bs)
    r_q, r_a = encode_signed(z, bs)
    return {"step": 0, "m_q": m_q, "m_absmax": m_a, "v_q": v_q, "v_absmax": v_a, "r_q": r_q, "r_absmax": r_a}


# --------------------------------------------------------------------------
# FireFlyOptim bit-module update (fireflyoptim.py:136-209)
# --------------------------------------------------------------------------
@torch.no_grad()
def dqt_step(int_weight, weight_scale, grad, state, *, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.1,
             sr_bias=0.15, bs=256, u=None):
    """One update of one module, in place on ``int_weight`` and ``state``.

    ``u`` (fp32 uniforms shaped like the weight) replaces the reference's ``torch.rand_like``
    draw (fireflyoptim.py:192) when given."""
    g = grad.float().contiguous()
    m = decode_signed(state["m_q"], state["m_absmax"], bs, g.shape)
    v = decode_unsigned(state["v_q"], state["v_absmax"], bs, g.shape)
    r = decode_signed(state["r_q"], state["r_absmax"], bs, g.shape)
    state["step"] += 1
    t = state["step"]
    m.mul_(beta1).add_(g, alpha=1.0 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1.0 - beta2)
    m_hat = m / (1.0 - beta1 ** t)
    v_hat = v / (1.0 - beta2 ** t)
    ws = weight_scale.float().unsqueeze(1).clamp_min(eps)
    adam = m_hat / (v_hat.sqrt() + eps)
    r = r + (-lr * (adam + wd * int_weight.float() * ws)) / ws
    mag = r.abs()
    whole = torch.floor(mag)
    threshold = (mag - whole + torch.tanh(adam) * sr_bias * torch.sign(r)).clamp(0.0, 1.0)
    draw = torch.rand_like(threshold) if u is None else u
    dq = (torch.sign(r) * (whole + (draw < threshold).float())).to(torch.int32)
    if torch.any(dq != 0):
        # update_int8_weight_ (fireflykernels.py:218-223)
        int_weight.copy_((int_weight.to(torch.int16) + dq.to(torch.int16)).clamp_(-127, 127).to(torch.int8))
        r = r - dq.float()
    state["r_q"], state["r_absmax"] = encode_signed(r, bs)
    state["m_q"], state["m_absmax"] = encode_signed(m, bs)
    state["v_q"], state["v_absmax"] = encode_unsigned(v, bs)
    return int_weight


# --------------------------------------------------------------------------
# The benchmark block on the reference's layers
# --------------------------------------------------------------------------
class SwiGLUBlock:
    """SwiGLU MLP of reference-path BitLinear layers: ``down(silu(g) * u)`` with ``[g | u] = gate_up(x)``.

    Weights: ``q_gu [2f, d]`` (gate rows then up rows), ``q_d [d, f]`` int8 with fp32 row scales."""

    def __init__(self, q_gu, s_gu, q_d, s_d):
        self.q_gu, self.s_gu, self.q_d, self.s_d = q_gu, s_gu, q_d, s_d
        self.f = q_d.shape[1]
        self.grads: dict[int, torch.Tensor] = {}
        self.states = [init_state(q_gu.shape, q_gu.device), init_state(q_d.shape, q_d.device)]

    def forward(self, x):
        gu = _LinearFn.apply(x, self.q_gu, self.s_gu, None, self.grads, 1)
        h = F.silu(gu[:, : self.f]) * gu[:, self.f:]
        return _LinearFn.apply(h, self.q_d, self.s_d, None, self.grads, 2)

    def train_step(self, x, dy, *, lr=1e-3, wd=0.01, sr_bias=0.15):
        """Forward, backward with upstream gradient ``dy`` and one optimizer step of both layers."""
        y = self.forward(x)
        y.backward(dy)
        for h, (q, s) in ((1, (self.q_gu, self.s_gu)), (2, (self.q_d, self.s_d))):
            g = self.grads.pop(h)
            dqt_step(q, s, g, self.states[h - 1], lr=lr, wd=wd, sr_bias=sr_bias)
        return y

"""Op layer of the FireFly INT8 hot path on B200 — the drop-in for ``fireflykernels.py``.

Same public names and behaviour as the reference module (fumitoshi0524/FireFly
``fireflykernels.py``):

* handle registry and weight-gradient cache (fireflykernels.py:7-41):
  ``next_bit_handle``, ``register_bit_handle``, ``release_bit_handle``,
  ``consume_bit_grad``, ``_BIT_GRAD_CACHE``
* ``quantize_fp_to_int8`` (fireflykernels.py:96-104) — per-row absmax int8
* ``Int8LinearFn`` (fireflykernels.py:110-124) — the autograd op
* ``update_int8_weight_`` (fireflykernels.py:218-223)
* ``_invalidate_weight_cache`` (fireflykernels.py:88-90) — bumps the per-handle
  weight version that keys the cached weight layouts

The reference's live path dequantises W to bf16 and calls ``torch.matmul``
(fireflykernels.py:164-210); its int8 design (``_forward_bnb``,
fireflykernels.py:132-156) was unreachable.  Here every GEMM is an int8
tensor-core GEMM on sm_100a:

* forward  ``Y = X Wᵀ``: X quantised per token, ``y = acc·s_x[t]·s_w[o] (+b)`` → bf16
* backward ``dX = dY W``: ``g = dY ⊙ s_w`` quantised per token, ``dx = acc·s_g[t]`` → bf16
* backward ``dW = dYᵀ X``: dY and X quantised per column over tokens,
  ``dw = acc·s_dy[o]·s_x[k]``, added into the bf16 grad cache in the GEMM epilogue
* ``db = Σ_t dY`` (fp32 sum, bf16 result) when there is a bias.

All device work goes through ``firefly_b200._capi`` (libfirefly_b200.so); there
is no CPU path.
"""
from __future__ import annotations

from typing import Callable

import torch

from . import _capi

# ---------------------------------------------------------------------------
# Handle registry (fireflykernels.py:7-41)
# ---------------------------------------------------------------------------
_NEXT_HANDLE = 1
_REGISTERED_HANDLES: set[int] = set()
_BIT_GRAD_CACHE: dict[int, torch.Tensor] = {}
# Preallocated gradient destinations (views into a flat bf16 arena, used by the
# data-parallel path).  When a handle has a slot and the cache is empty, the dW
# GEMM writes straight into the slot instead of allocating.
_GRAD_SLOTS: dict[int, torch.Tensor] = {}
# Called with the handle once that handle's weight gradient of the current backward has been
# issued (the data-parallel optimizer starts reducing a bucket of gradients from them).
_GRAD_READY_HOOKS: dict[int, Callable[[int], None]] = {}


def set_grad_ready_hook(handle: int, fn) -> None:
    """Register ``fn(handle)`` to run after each weight-gradient GEMM of ``handle`` is issued
    (``None`` removes it)."""
    if fn is None:
        _GRAD_READY_HOOKS.pop(int(handle), None)
    else:
        _GRAD_READY_HOOKS[int(handle)] = fn


def _grad_ready(handle: int) -> None:
    fn = _GRAD_READY_HOOKS.get(handle)
    if fn is not None:
        fn(handle)


def next_bit_handle() -> int:
    global _NEXT_HANDLE
    while _NEXT_HANDLE in _REGISTERED_HANDLES:
        _NEXT_HANDLE += 1
    handle = _NEXT_HANDLE
    _REGISTERED_HANDLES.add(handle)
    _NEXT_HANDLE += 1
    return handle


def register_bit_handle(handle: int) -> int:
    global _NEXT_HANDLE
    handle = int(handle)
    if handle <= 0:
        raise ValueError(f"handle must be > 0, got {handle}")
    _REGISTERED_HANDLES.add(handle)
    _BIT_GRAD_CACHE.pop(handle, None)
    if handle >= _NEXT_HANDLE:
        _NEXT_HANDLE = handle + 1
    return handle


def release_bit_handle(handle: int) -> None:
    handle = int(handle)
    _REGISTERED_HANDLES.discard(handle)
    _BIT_GRAD_CACHE.pop(handle, None)
    _GRAD_SLOTS.pop(handle, None)
    _GRAD_READY_HOOKS.pop(handle, None)
    _W_CACHE.pop(handle, None)


def consume_bit_grad(handle: int) -> torch.Tensor | None:
    return _BIT_GRAD_CACHE.pop(int(handle), None)


def set_grad_slot(handle: int, slot: torch.Tensor | None) -> None:
    """Route the weight gradient of ``handle`` into ``slot`` (bf16, contiguous ``[O, K]``)."""
    if slot is None:
        _GRAD_SLOTS.pop(int(handle), None)
        return
    if slot.dtype != torch.bfloat16 or not slot.is_contiguous():
        raise ValueError("grad slot must be a contiguous bf16 tensor")
    _GRAD_SLOTS[int(handle)] = slot


# ---------------------------------------------------------------------------
# Weight-layout cache (the role of _BNB_WCACHE, fireflykernels.py:64-90)
# ---------------------------------------------------------------------------
# handle -> {"key_k": (version, ptr, torch_version, shape), "wk": codes padded to a 16-multiple row}
_W_CACHE: dict[int, dict] = {}
_W_VERSION: dict[int, int] = {}


def _invalidate_weight_cache(handle: int) -> None:
    """Call after int_weight is modified (FireFlyOptim does, fireflyoptim.py:198)."""
    _W_VERSION[handle] = _W_VERSION.get(handle, 0) + 1


def _weight_key(handle: int, w: torch.Tensor):
    return (_W_VERSION.get(handle, 0), w.data_ptr(), w._version, tuple(w.shape))


def _weight_operand(handle: int, w: torch.Tensor) -> torch.Tensor:
    """W as a GEMM operand ``[O, ldk]`` with ``ldk % 16 == 0`` (W itself when it already is).

    The forward reads it as the N x K operand, the dX GEMM as the K x N operand."""
    O, K = w.shape
    if K % 16 == 0 and w.is_contiguous():
        return w
    ent = _W_CACHE.setdefault(handle, {})
    key = _weight_key(handle, w)
    if ent.get("key_k") != key:
        ldk = _capi.round_up(K, 16)
        wk = torch.zeros((O, ldk), dtype=torch.int8, device=w.device)
        wk[:, :K].copy_(w)
        ent["wk"], ent["key_k"] = wk, key
    return ent["wk"]


# ---------------------------------------------------------------------------
# Weight quantisation (fireflykernels.py:96-104)
# ---------------------------------------------------------------------------
def quantize_fp_to_int8(weight: torch.Tensor, eps: float = 1e-8):
    """Per-row absmax int8 quantisation: ``(q [O,K] int8, scale [O] fp32)``.

    Runs the ``ff_quant_rows_i8`` kernel.  A CPU tensor is quantised on the
    current CUDA device and the results are returned on the CPU, like the input.
    """
    if weight.ndim != 2:
        raise ValueError(
            f"weight must be 2D [out_features, in_features], got {tuple(weight.shape)}"
        )
    src = weight
    if not weight.is_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("firefly_b200 needs a CUDA device (no CPU path)")
        src = weight.to(device=torch.device("cuda", torch.cuda.current_device()))
    if src.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        src = src.float()
    q, s = _capi.quant_rows(src, eps=float(eps))
    if not weight.is_cuda:
        q, s = q.cpu(), s.cpu()
    return q.contiguous(), s.contiguous()


# ---------------------------------------------------------------------------
# Int8LinearFn (fireflykernels.py:110-124)
# ---------------------------------------------------------------------------
def _as_float_input(x: torch.Tensor) -> torch.Tensor:
    if x.dtype in (torch.float32, torch.bfloat16, torch.float16):
        return x
    return x.float()


# The activation codes of the last quantised input.  Two BitLinear layers that read the
# same tensor (the gate and up projections of a SwiGLU block) quantise it once.  The entry
# holds a reference to the tensor, so its storage cannot be reused while cached, and is
# keyed by storage, offset, shape, strides, dtype and the in-place version counter (the
# same counter autograd relies on).  A write that does not bump that counter (through
# ``.data``, ctypes, or a collective writing into the storage) is not seen by the key, so
# the entry is also dropped at the start of every backward pass and by every optimizer
# step: codes are then reused only within one forward pass.  Code that writes such an
# input out of band between two forward passes with neither in between calls
# ``clear_activation_cache()``.
_ACT_CACHE: dict = {}


def _act_key(x: torch.Tensor, with_cols: bool):
    return (x.untyped_storage().data_ptr(), x.storage_offset(), tuple(x.shape), tuple(x.stride()),
            x.dtype, x._version, with_cols, x.device)


def _quantize_activation(x: torch.Tensor, with_cols: bool):
    key = _act_key(x, with_cols)
    hit = _ACT_CACHE.get("entry")
    if hit is not None and hit[0] == key:
        return hit[2]
    if with_cols:
        codes = _capi.quant_dual(x)
    else:
        K = x.shape[1]
        q, s = _capi.quant_rows(x, ldq=_capi.round_up(K, 16))
        codes = (q, s, None, None)
    _ACT_CACHE["entry"] = (key, x, codes)
    return codes


def clear_activation_cache() -> None:
    _ACT_CACHE.clear()


class Int8LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, int_weight, weight_scale, bias, handle):
        _capi._require_cuda(x2d, int_weight, weight_scale, bias)
        if int_weight.dtype != torch.int8 or int_weight.dim() != 2:
            raise ValueError("int_weight must be a 2-D int8 tensor")
        O, K = int_weight.shape
        if x2d.dim() != 2 or x2d.shape[1] != K:
            raise ValueError(f"expected input [N, {K}], got {tuple(x2d.shape)}")
        x = _as_float_input(x2d)
        T = x.shape[0]
        ws = weight_scale.to(torch.float32).contiguous()
        b = None if bias is None else bias.detach().to(torch.float32).contiguous()
        handle = int(handle)
        need_grad = any(ctx.needs_input_grad)
        y = torch.empty((T, O), dtype=torch.bfloat16, device=x.device)
        saved_xt = saved_sx = None
        if T > 0:
            q_x, s_x, q_xt, s_xc = _quantize_activation(x, with_cols=need_grad)
            if need_grad:
                saved_xt, saved_sx = q_xt, s_xc
            w_op = _weight_operand(handle, int_weight)
            _capi.gemm_i8(q_x, w_op, K, scale_a=s_x, scale_b=ws, bias=b,
                          out_kind=_capi.FF_OUT_BF16, out=y)
        ctx.save_for_backward(saved_xt, saved_sx, int_weight, ws)
        ctx.handle = handle
        ctx.has_bias = bias is not None
        ctx.input_dtype = x2d.dtype
        ctx.T = T
        return y

    @staticmethod
    def backward(ctx, grad_out):
        _ACT_CACHE.clear()
        q_xt, s_xc, int_weight, ws = ctx.saved_tensors
        O, K = int_weight.shape
        T = ctx.T
        dy = grad_out
        if dy.dtype != torch.bfloat16:
            dy = dy.to(torch.bfloat16)
        dy = dy.contiguous()
        need_dx = ctx.needs_input_grad[0]
        grad_in = None
        if T == 0:
            gw = torch.zeros((O, K), dtype=torch.bfloat16, device=dy.device)
            _accumulate_weight_grad(ctx.handle, gw)
            if need_dx:
                grad_in = torch.zeros((0, K), dtype=grad_out.dtype, device=dy.device)
            db = torch.zeros((O,), dtype=grad_out.dtype, device=dy.device) if ctx.has_bias else None
            return grad_in, None, None, db, None
        # db = Σ_rows dY (fireflykernels.py:200) comes out of the same read of dY
        q_g, s_g, q_dyt, s_dy, *db = _capi.quant_dual(dy, row_colmul=ws, rows=need_dx, cols=True,
                                                      colsum=ctx.has_bias)
        if need_dx:
            # dX = dY·W contracts over O: W [O, K] is read directly as the K x N operand
            w_op = _weight_operand(ctx.handle, int_weight)
            grad_in = _capi.gemm_i8(q_g, w_op, O, scale_a=s_g, out_kind=_capi.FF_OUT_BF16, b_kn_cols=K)
        # dW = dYᵀ X, accumulated in the epilogue (fireflykernels.py:193-198)
        _weight_grad_gemm(ctx.handle, q_dyt, s_dy, q_xt, s_xc, O, K, T, dy.device)
        grad_bias = db[0] if ctx.has_bias else None
        if grad_bias is not None and grad_bias.dtype != grad_out.dtype:
            grad_bias = grad_bias.to(grad_out.dtype)
        if grad_in is not None and grad_in.dtype != grad_out.dtype:
            grad_in = grad_in.to(grad_out.dtype)
        # int_weight and weight_scale are buffers: no gradient (fireflykernels.py:202-203)
        return grad_in, None, None, grad_bias, None


def _weight_grad_gemm(handle, q_dyt, s_dy, q_xt, s_xc, O, K, T, device):
    cached = _BIT_GRAD_CACHE.get(handle)
    if cached is None:
        slot = _GRAD_SLOTS.get(handle)
        if slot is not None and slot.shape == (O, K) and slot.device == device:
            dest = slot
        else:
            dest = torch.empty((O, K), dtype=torch.bfloat16, device=device)
        _capi.gemm_i8(q_dyt, q_xt, T, scale_a=s_dy, scale_b=s_xc,
                      out_kind=_capi.FF_OUT_BF16, out=dest)
        _BIT_GRAD_CACHE[handle] = dest
    elif (cached.dtype == torch.bfloat16 and cached.is_cuda and cached.device == device
          and cached.shape == (O, K) and cached.is_contiguous()):
        _capi.gemm_i8(q_dyt, q_xt, T, scale_a=s_dy, scale_b=s_xc,
                      out_kind=_capi.FF_OUT_BF16_ACCUM, out=cached)
    else:
        gw = _capi.gemm_i8(q_dyt, q_xt, T, scale_a=s_dy, scale_b=s_xc,
                           out_kind=_capi.FF_OUT_BF16)
        cached.add_(gw.to(device=cached.device, dtype=cached.dtype))
    _grad_ready(handle)


def _accumulate_weight_grad(handle: int, gw: torch.Tensor) -> None:
    cached = _BIT_GRAD_CACHE.get(handle)
    if cached is None:
        _BIT_GRAD_CACHE[handle] = gw
    else:
        cached.add_(gw.to(dtype=cached.dtype))
    _grad_ready(handle)


# ---------------------------------------------------------------------------
# INT8 weight update (fireflykernels.py:218-223)
# ---------------------------------------------------------------------------
@torch.no_grad()
def update_int8_weight_(int_weight: torch.Tensor, delta_q: torch.Tensor) -> None:
    """In-place int8 weight update:  W += delta_q, clamped to [-127, 127]."""
    _capi.update_int8_weight(int_weight, delta_q)

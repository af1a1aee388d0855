"""``BitLinear`` — the drop-in for the reference's ``bitLinear.py``.

Same constructor, buffers, forward contract and checkpoint behaviour as
fumitoshi0524/FireFly ``bitLinear.py:30-108``:

* buffers ``int_weight`` int8 ``[O, K]``, ``weight_scale`` fp32 ``[O]``,
  ``_bit_handle`` int64 scalar (all persistent), optional fp32 ``bias`` Parameter
* ``forward(x)`` takes ``[..., K]`` of any float dtype and returns bf16 ``[..., O]``
* the weight gradient goes to the per-handle grad cache and is taken by
  ``consume_weight_grad()`` (bitLinear.py:96-97)
* loading a state dict re-registers the stored handle (bitLinear.py:99-104)

Forward and backward run on the int8 tensor cores (``Int8LinearFn``).  The
forward uses the handle cached on the module instead of reading the
``_bit_handle`` buffer with ``.item()`` on every call (bitLinear.py:92), which
would synchronise the host with the GPU each time.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from .fireflykernels import (
    Int8LinearFn,
    consume_bit_grad,
    next_bit_handle,
    quantize_fp_to_int8,
    register_bit_handle,
    release_bit_handle,
)


def _init_int8_weight(out_features: int, in_features: int):
    """Kaiming-uniform init quantised per row to int8 (bitLinear.py:15-27).

    The fp32 weights are drawn on the CPU from torch's default generator exactly
    as the reference does; the per-row quantisation runs on the GPU kernel.
    """
    weight = torch.empty((out_features, in_features), dtype=torch.float32)
    nn.init.kaiming_uniform_(weight, a=math.sqrt(5))
    return quantize_fp_to_int8(weight, eps=1e-8)


class BitLinear(nn.Module):
    """INT8 linear layer: ``y = x · (int_weight · weight_scale)ᵀ (+ bias)`` on int8 tensor cores."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False) -> None:
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        int_init, scale_init = _init_int8_weight(self.out_features, self.in_features)
        self.register_buffer("int_weight", int_init, persistent=True)
        self.register_buffer("weight_scale", scale_init, persistent=True)
        self.register_buffer(
            "_bit_handle", torch.tensor(next_bit_handle(), dtype=torch.int64), persistent=True
        )
        self._registered_handle = int(self._bit_handle.item())
        self.register_load_state_dict_post_hook(self._post_load_state_dict)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)

    @torch.no_grad()
    def reset_int8_(self) -> None:
        int_init, scale_init = _init_int8_weight(self.out_features, self.in_features)
        self.int_weight.copy_(int_init.to(device=self.int_weight.device))
        self.weight_scale.copy_(scale_init.to(device=self.weight_scale.device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"expected input last dim {self.in_features}, got {x.shape[-1]}")
        if self.int_weight.device != x.device:
            raise RuntimeError(
                "BitLinear input and int_weight must be on same device. "
                "Move module with model.to(device) before forward."
            )
        x2d = x.reshape(-1, self.in_features)
        out2d = Int8LinearFn.apply(
            x2d, self.int_weight, self.weight_scale, self.bias, self._registered_handle
        )
        return out2d.view(*x.shape[:-1], self.out_features)

    def consume_weight_grad(self) -> torch.Tensor | None:
        return consume_bit_grad(self._registered_handle)

    def _post_load_state_dict(self, module, incompatible_keys) -> None:
        del module, incompatible_keys
        new_handle = register_bit_handle(int(self._bit_handle.item()))
        if new_handle != self._registered_handle:
            release_bit_handle(self._registered_handle)
            self._registered_handle = new_handle

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def collect_bitlinear_modules(module: nn.Module) -> list[BitLinear]:
    return [m for m in module.modules() if isinstance(m, BitLinear)]

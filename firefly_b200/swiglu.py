"""SwiGLU MLP block built from BitLinear — the Llama-7B-shaped training workload.

``y = down(silu(gate(x)) * up(x))`` with gate/up ``d -> f`` and down ``f -> d``,
all three BitLinear (no bias).  The reference ships no model code; this block is
the harness for its SwiGLU-MLP configuration (d_model 4096, ffn 11008).
"""
from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from .bitLinear import BitLinear


class SwiGLUMLP(nn.Module):
    def __init__(self, d_model: int, ffn: int):
        super().__init__()
        self.gate = BitLinear(d_model, ffn)
        self.up = BitLinear(d_model, ffn)
        self.down = BitLinear(ffn, d_model)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down(F.silu(self.gate(x)) * self.up(x))

    @torch.no_grad()
    def init_normal_(self, std: float = 0.02, generator: torch.Generator | None = None) -> None:
        """Weights ~ N(0, std) quantised per row (the benchmark initialisation)."""
        from .fireflykernels import quantize_fp_to_int8

        for lin in (self.gate, self.up, self.down):
            w = torch.empty(lin.out_features, lin.in_features, device=lin.int_weight.device)
            w.normal_(0.0, std, generator=generator)
            q, s = quantize_fp_to_int8(w)
            lin.int_weight.copy_(q)
            lin.weight_scale.copy_(s)

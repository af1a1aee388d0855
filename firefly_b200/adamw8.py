"""Block-wise 8-bit AdamW for dense (non-BitLinear) parameters.

The reference's ``FireFlyOptim`` derives from bitsandbytes' ``AdamW8bit``
(fireflyoptim.py:2, :83, :124): every parameter that is not a BitLinear weight is
stepped by bitsandbytes' 8-bit AdamW.  bitsandbytes is a third-party library that is
not part of this build, so this module implements the published algorithm (Dettmers et
al., "8-bit Optimizers via Block-wise Quantization", ICLR 2022) on the B200 kernel
``ff_adamw8_blockwise``:

* both Adam moments are stored as uint8 codes of a 256-entry "dynamic tree" map, scaled
  per block of 2048 elements by the block's absmax (fp32);
* the map (``dynamic_qmap``): a sign bit (signed map only), then a run of zero bits whose
  length e selects the decade 10^-e, an indicator bit, and the remaining bits as a linear
  fraction in (0.1, 1];
* parameters with fewer than ``min_8bit_size`` elements (biases, norm scales), and
  parameters not on a CUDA device, keep fp32 moments (plain AdamW on the same formula);
  the CUDA ones of a parameter group are stepped together by one multi-tensor kernel
  (``ff_adamw32_multi``) rather than a dozen small kernels each.

State per parameter: ``step`` and either ``m_q``/``m_absmax``/``v_q``/``v_absmax`` (8-bit)
or ``exp_avg``/``exp_avg_sq`` (fp32).  The maps and the rounding of the update are this
build's own; bitsandbytes' results are not reproduced bit for bit.
"""
from __future__ import annotations

import torch

from . import _capi

DENSE_BLOCK = 2048


def dynamic_qmap(signed: bool) -> torch.Tensor:
    """The 256 values of the dynamic tree map, fp32, ascending.

    Signed: for e = 0..6 the 2^(6-e) magnitudes 10^-e * (0.1 + 0.9 k / 2^(6-e)), k = 1..2^(6-e)
    (127 in all), both signs, and zero twice (codes 127 and 128).  Unsigned: for e = 0..7 the
    2^(7-e) values 10^-e * (0.1 + 0.9 k / 2^(7-e)) (255 in all) and zero (code 0).  Both
    maps contain 1.0, so a block's largest value is represented exactly.
    """
    frac_bits = 6 if signed else 7
    mags = []
    for e in range(frac_bits + 1):
        f = frac_bits - e
        for k in range(1, 2 ** f + 1):
            mags.append(10.0 ** (-e) * (0.1 + 0.9 * k / 2 ** f))
    vals = [0.0, 0.0] + mags + [-v for v in mags] if signed else [0.0] + mags
    out = torch.tensor(sorted(vals), dtype=torch.float64).to(torch.float32)
    assert out.numel() == 256
    return out


_QMAPS: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}


def _qmaps_on(device: torch.device):
    t = _QMAPS.get(device)
    if t is None:
        t = (dynamic_qmap(True).to(device), dynamic_qmap(False).to(device))
        _QMAPS[device] = t
    return t


class AdamW8bitDense(torch.optim.Optimizer):
    """AdamW with block-wise 8-bit moments for parameters of at least ``min_8bit_size`` elements."""

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2, min_8bit_size=4096):
        if lr < 0.0 or eps < 0.0 or not (0.0 <= betas[0] < 1.0 and 0.0 <= betas[1] < 1.0):
            raise ValueError(f"invalid AdamW hyperparameters lr={lr} betas={betas} eps={eps}")
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.min_8bit_size = int(min_8bit_size)

    def _eight_bit(self, p: torch.Tensor) -> bool:
        return p.is_cuda and p.numel() >= self.min_8bit_size and p.dtype in (torch.float32, torch.bfloat16)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
            fused: dict[torch.device, list] = {}  # small CUDA parameters: one multi-tensor launch per device
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("AdamW8bitDense does not support sparse gradients")
                state = self.state[p]
                if self._eight_bit(p):
                    self._step_8bit(p, state, lr, b1, b2, eps, wd)
                elif p.is_cuda and p.is_contiguous() and p.dtype in (torch.float32, torch.bfloat16):
                    self._init_32bit(p, state)
                    state["step"] += 1
                    g = p.grad
                    if g.dtype not in (torch.float32, torch.bfloat16):
                        g = g.float()
                    fused.setdefault(p.device, []).append(
                        (p, g.contiguous(), state["exp_avg"], state["exp_avg_sq"], int(state["step"])))
                else:
                    self._step_32bit(p, state, lr, b1, b2, eps, wd)
            for items in fused.values():
                _capi.adamw32_multi(items, lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd)
        return loss

    def _step_8bit(self, p, state, lr, b1, b2, eps, wd):
        if "m_q" not in state:
            nb = (p.numel() + DENSE_BLOCK - 1) // DENSE_BLOCK
            state["step"] = 0
            state["m_q"] = torch.full((p.numel(),), 128, dtype=torch.uint8, device=p.device)
            state["m_absmax"] = torch.zeros((nb,), dtype=torch.float32, device=p.device)
            state["v_q"] = torch.zeros((p.numel(),), dtype=torch.uint8, device=p.device)
            state["v_absmax"] = torch.zeros((nb,), dtype=torch.float32, device=p.device)
        state["step"] += 1
        g = p.grad
        if not g.is_contiguous():
            g = g.contiguous()
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        if not p.is_contiguous():
            raise ValueError("AdamW8bitDense needs contiguous parameters")
        qs, qu = _qmaps_on(p.device)
        _capi.adamw8_blockwise(p, g, state["m_q"], state["m_absmax"], state["v_q"], state["v_absmax"],
                               lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd, step=int(state["step"]),
                               qmap_s=qs, qmap_u=qu)

    @staticmethod
    def _init_32bit(p, state):
        if "exp_avg" not in state:
            state["step"] = 0
            state["exp_avg"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)
            state["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)

    @staticmethod
    def _step_32bit(p, state, lr, b1, b2, eps, wd):
        """fp32-moment AdamW in torch ops: parameters off the GPU, or of other dtypes or layouts
        (CUDA fp32/bf16 parameters take the fused ``ff_adamw32_multi`` with the same roundings)."""
        AdamW8bitDense._init_32bit(p, state)
        state["step"] += 1
        t = int(state["step"])
        g = p.grad.float()
        w = p.float()
        if wd != 0.0:
            w.mul_(1.0 - lr * wd)
        m, v = state["exp_avg"], state["exp_avg_sq"]
        m.mul_(b1).add_(g * (1.0 - b1))
        v.mul_(b2).add_(g * (1.0 - b2) * g)
        bc1, bc2 = 1.0 - b1 ** t, 1.0 - b2 ** t
        w.sub_((m / (v.sqrt() + eps * bc2 ** 0.5)) * (lr * bc2 ** 0.5 / bc1))
        p.copy_(w)

    def load_state_dict(self, state_dict):
        # torch casts floating state tensors to the parameter's dtype; the block absmax
        # arrays and the fp32 moments stay fp32
        saved = {}
        for pid, st in state_dict["state"].items():
            saved[pid] = {k: v.clone() for k, v in st.items()
                          if k in ("m_absmax", "v_absmax", "exp_avg", "exp_avg_sq")}
        super().load_state_dict(state_dict)
        params = [p for group in self.param_groups for p in group["params"]]
        for pid, p in enumerate(params):
            st = self.state.get(p)
            if st is None or pid not in saved:
                continue
            for k, v in saved[pid].items():
                st[k] = v.to(device=p.device, dtype=torch.float32)


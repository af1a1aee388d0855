"""``FireFlyOptim`` — the drop-in for the reference's ``fireflyoptim.py``.

Same constructor, hyperparameters, state layout and checkpoint format as
fumitoshi0524/FireFly ``fireflyoptim.py:83-258``:

* per BitLinear (keyed by handle): ``step`` and three 8-bit mu-law blockwise
  states — ``m_q`` (signed, uint8 with +128 offset), ``v_q`` (unsigned),
  ``r_q`` (the DQT residual, signed) — each ``[O, K]`` uint8 with fp32 block
  absmax ``[ceil(O*K/256)]`` (fireflyoptim.py:142-161)
* hyperparameters from ``param_groups[0]`` (fireflyoptim.py:129-134)
* ``state_dict()["bit_state"]`` holds those tensors on the CPU (fireflyoptim.py:213-233)

The per-module update (fireflyoptim.py:137-209: decode, Adam moments, DQT
residual, momentum-biased stochastic rounding, int8 weight update, re-encode)
is one fused kernel launch, ``ff_dqt_adamw8``, with no host synchronisation
(the reference's ``torch.any(delta_q != 0)`` at fireflyoptim.py:195 is not
needed: a zero delta leaves weight and residual unchanged).

Stochastic-rounding uniforms: the reference draws ``torch.rand_like``
(fireflyoptim.py:192).  Here the kernel draws counter-based Philox4x32-10
uniforms keyed by (seed, step, global element index), so results do not depend
on how the update is split across GPUs.  ``uniform_source`` may supply the
uniforms instead (used to replay the reference's draws).

Dense (non-BitLinear) parameters: the reference steps them with
bitsandbytes ``AdamW8bit`` (fireflyoptim.py:83, :124), a third-party optimizer;
here ``FireFlyOptim`` derives from ``AdamW8bitDense`` (``firefly_b200/adamw8.py``),
the same block-wise 8-bit algorithm on the ``ff_adamw8_blockwise`` kernel, with fp32
moments for parameters under 4096 elements.
"""
from __future__ import annotations

from typing import Callable

import torch

from . import _capi
from .adamw8 import AdamW8bitDense
from .bitLinear import BitLinear
from .fireflykernels import _invalidate_weight_cache, clear_activation_cache

_MU = 255.0
_1_OVER_LN1P_MU = 1.0 / 5.545177444479562  # 1 / ln(1 + 255), fireflyoptim.py:10
BLOCK = 256


def decode_tables() -> tuple[torch.Tensor, torch.Tensor]:
    """x_norm of every uint8 code for the signed and unsigned mu-law codecs.

    Evaluated with the reference's own formula on the CPU (fireflyoptim.py:47-48,
    :77-78), so ``table[code] * absmax`` reproduces its decode bit for bit.
    """
    codes = torch.arange(256, dtype=torch.float32)
    y = ((codes - 128.0) / 127.0).clamp(-1.0, 1.0)
    dec_s = torch.sign(y) * (torch.exp(y.abs() / _1_OVER_LN1P_MU) - 1.0) / _MU
    yu = (codes / 255.0).clamp(0.0, 1.0)
    dec_u = (torch.exp(yu / _1_OVER_LN1P_MU) - 1.0) / _MU
    return dec_s.contiguous(), dec_u.contiguous()


_TABLES: dict[torch.device, tuple[torch.Tensor, torch.Tensor]] = {}


def _tables_on(device: torch.device):
    t = _TABLES.get(device)
    if t is None:
        s, u = decode_tables()
        t = (s.to(device), u.to(device))
        _TABLES[device] = t
    return t


def init_bit_state(shape, device, block: int = BLOCK) -> dict:
    """Zero states exactly as ``_quantize_blockwise_*`` encodes zeros (fireflyoptim.py:142-161)."""
    numel = 1
    for d in shape:
        numel *= int(d)
    nb = (numel + block - 1) // block
    tiny = torch.full((nb,), 1e-12, dtype=torch.float32, device=device)
    return {
        "step": 0,
        "m_q": torch.full(tuple(shape), 128, dtype=torch.uint8, device=device),
        "m_absmax": tiny.clone(),
        "v_q": torch.zeros(tuple(shape), dtype=torch.uint8, device=device),
        "v_absmax": tiny.clone(),
        "r_q": torch.full(tuple(shape), 128, dtype=torch.uint8, device=device),
        "r_absmax": tiny,
    }


def bit_rng_offsets(modules) -> list[int]:
    """Global element index of each module's first weight element (256-aligned)."""
    out, off = [], 0
    for m in modules:
        out.append(off)
        off += _capi.round_up(m.int_weight.numel(), BLOCK)
    return out


class FireFlyOptim(AdamW8bitDense):
    """Dense params: block-wise 8-bit AdamW.  BitLinear weights: fused 8-bit AdamW + DQT stochastic rounding."""

    def __init__(
        self,
        params,
        lr=1e-3,
        betas=(0.9, 0.999),
        eps=1e-8,
        weight_decay=0.1,
        bit_modules=None,
        block_size=256,
        sr_bias_scale=0.15,
    ):
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        if int(block_size) != BLOCK:
            raise ValueError(f"block_size must be {BLOCK} on this build, got {block_size}")
        self.bit_modules = list(bit_modules) if bit_modules is not None else []
        self._bit_handles = (
            [int(m._bit_handle.item()) for m in self.bit_modules] if bit_modules is not None else []
        )
        self._bit_state: dict[int, dict[str, torch.Tensor | int]] = {}
        self.block_size = int(block_size)
        self.sr_bias_scale = float(sr_bias_scale)
        # Philox key of the stochastic rounding, drawn from torch's default generator
        self.rng_seed = int(torch.randint(0, 2**62, (1,), dtype=torch.int64).item())
        # optional: callable(module, handle, step) -> fp32 uniforms shaped like int_weight
        self.uniform_source: Callable | None = None

    def add_bit_modules(self, modules) -> None:
        for module in modules:
            if not isinstance(module, BitLinear):
                raise TypeError(f"expected BitLinear, got {type(module).__name__}")
            if module not in self.bit_modules:
                self.bit_modules.append(module)
                self._bit_handles.append(int(module._bit_handle.item()))

    def _hyper(self):
        group = self.param_groups[0]
        beta1, beta2 = group["betas"]
        return (float(group["lr"]), float(beta1), float(beta2), float(group["eps"]),
                float(group["weight_decay"]))

    def _state_for(self, handle: int, module: BitLinear) -> dict:
        dev = module.int_weight.device
        state = self._bit_state.setdefault(handle, {})
        if "step" not in state:
            state.update(init_bit_state(module.int_weight.shape, dev, self.block_size))
        else:
            for k in ("m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax"):
                t = state[k]
                if t.device != dev or not t.is_contiguous():
                    state[k] = t.to(dev).contiguous()
        return state

    @torch.no_grad()
    def step(self, closure=None):
        loss = super().step(closure)
        clear_activation_cache()  # the next step's inputs are quantised afresh
        if not self.bit_modules:
            return loss
        lr, beta1, beta2, eps, wd = self._hyper()
        offsets = bit_rng_offsets(self.bit_modules)
        for module, handle, off in zip(self.bit_modules, self._bit_handles, offsets):
            g = module.consume_weight_grad()
            if g is None:
                continue
            if g.dtype != torch.bfloat16 or not g.is_contiguous() or g.device != module.int_weight.device:
                g = g.to(device=module.int_weight.device, dtype=torch.bfloat16).contiguous()
            state = self._state_for(handle, module)
            state["step"] += 1
            t = int(state["step"])
            u = None
            if self.uniform_source is not None:
                u = self.uniform_source(module, handle, t)
                u = u.to(device=module.int_weight.device, dtype=torch.float32).contiguous()
            dec_s, dec_u = _tables_on(module.int_weight.device)
            _capi.dqt_adamw8(
                module.int_weight, module.weight_scale, module.in_features, g,
                state["m_q"], state["m_absmax"], state["v_q"], state["v_absmax"],
                state["r_q"], state["r_absmax"],
                lr=lr, beta1=beta1, beta2=beta2, eps=eps, wd=wd, step=t,
                sr_bias=self.sr_bias_scale, seed=self.rng_seed, rng_offset=off, u=u,
                dec_s=dec_s, dec_u=dec_u, block=self.block_size,
            )
            _invalidate_weight_cache(handle)
        return loss

    def state_dict(self):
        state = super().state_dict()
        state["bit_state"] = {
            int(handle): {
                key: value.detach().cpu() if torch.is_tensor(value) else value
                for key, value in per_handle.items()
            }
            for handle, per_handle in self._bit_state.items()
        }
        state["bit_rng_seed"] = self.rng_seed
        return state

    def load_state_dict(self, state_dict):
        state_dict = dict(state_dict)
        bit_state = state_dict.pop("bit_state", {})
        seed = state_dict.pop("bit_rng_seed", None)
        super().load_state_dict(state_dict)
        self._bit_state = {}
        for handle, per_handle in bit_state.items():
            self._bit_state[int(handle)] = {
                key: value.clone() if torch.is_tensor(value) else value
                for key, value in per_handle.items()
            }
        if seed is not None:
            self.rng_seed = int(seed)


class FireFlyOptimSR(FireFlyOptim):
    """FireFlyOptim with unbiased stochastic rounding (no momentum bias), fireflyoptim.py:236-258."""

    def __init__(
        self,
        params,
        lr=1e-3,
        betas=(0.9, 0.999),
        eps=1e-8,
        weight_decay=0.1,
        bit_modules=None,
        block_size=256,
    ):
        super().__init__(
            params,
            lr=lr,
            betas=betas,
            eps=eps,
            weight_decay=weight_decay,
            bit_modules=bit_modules,
            block_size=block_size,
            sr_bias_scale=0.0,
        )

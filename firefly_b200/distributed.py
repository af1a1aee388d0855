"""Data-parallel BitLinear training with a ZeRO-1 sharded 8-bit optimizer.

The reference has no distributed code.  This module adds the path the training
step shards along: every GPU runs the same model on its own tokens (each GEMM
stays on one GPU), then

1. the bf16 weight gradients, which the dW GEMM epilogue wrote straight into one
   flat arena (``BitArena.g``), are reduce-scattered (average) over the process
   group, so each rank holds the averaged gradient of 1/world of the arena;
2. each rank runs the fused DQT 8-bit AdamW kernel on its shard only — the
   m/v/r codes and their block absmax exist only for that shard (ZeRO-1);
3. the int8 weights (one flat arena, ``BitArena.q``, that every BitLinear's
   ``int_weight`` is a view of) are all-gathered back to every rank.

Per step and rank that moves (p-1)/p x (2 + 1) bytes per parameter over NVLink.

Arena layout: module i occupies elements ``[off_i, off_i + numel_i)`` with
``off_i`` a multiple of 256, in ``bit_modules`` order, so its 256-element
optimizer blocks are exactly the reference's per-module blocks
(fireflyoptim.py:13-19, :142-161), and the global element index that keys the
stochastic-rounding uniforms is the same on 1 GPU (``FireFlyOptim``) and on
any number of GPUs: the sharded update equals the single-GPU update.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from . import _capi
from .adamw8 import AdamW8bitDense
from .bitLinear import BitLinear
from .fireflykernels import _BIT_GRAD_CACHE, _invalidate_weight_cache, set_grad_slot
from .fireflyoptim import BLOCK, _tables_on, bit_rng_offsets


@dataclass(frozen=True)
class Segment:
    """Part of one module inside this rank's shard."""

    module: int  # index into the module list
    lo: int  # arena element range [lo, hi)
    hi: int
    elem_base: int  # element index of ``lo`` within the module's weight


class ShardPlan:
    """Which arena elements (and module pieces) each rank updates.  Pure host logic."""

    def __init__(self, numels: Sequence[int], world_size: int, rank: int, block: int = BLOCK):
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"bad rank {rank} of {world_size}")
        self.block = block
        self.numels = [int(n) for n in numels]
        self.offsets = []
        off = 0
        for n in self.numels:
            self.offsets.append(off)
            off += _capi.round_up(n, block)
        self.used = off
        self.total = _capi.round_up(max(off, 1), block * world_size)
        self.world_size, self.rank = world_size, rank
        self.shard = self.total // world_size
        self.lo, self.hi = rank * self.shard, (rank + 1) * self.shard
        self.segments: list[Segment] = []
        for i, (o, n) in enumerate(zip(self.offsets, self.numels)):
            a, b = max(o, self.lo), min(o + n, self.hi)
            if a < b:
                self.segments.append(Segment(i, a, b, a - o))

    def local_blocks(self, seg: Segment) -> tuple[int, int]:
        """Block range of ``seg`` within this rank's absmax arrays."""
        return (seg.lo - self.lo) // self.block, (seg.hi - self.lo + self.block - 1) // self.block


class BitArena:
    """Flat int8 weight and bf16 gradient buffers shared by a list of BitLinear modules.

    After construction every module's ``int_weight`` buffer is a view of ``q`` and
    its weight gradient is routed into the matching view of ``g``.
    """

    def __init__(self, modules: Sequence[BitLinear], world_size: int = 1, rank: int = 0,
                 device: torch.device | None = None):
        self.modules = list(modules)
        if not self.modules:
            raise ValueError("BitArena needs at least one BitLinear")
        device = device or self.modules[0].int_weight.device
        self.plan = ShardPlan([m.int_weight.numel() for m in self.modules], world_size, rank)
        assert self.plan.offsets == bit_rng_offsets(self.modules)
        self.q = torch.zeros(self.plan.total, dtype=torch.int8, device=device)
        self.g = torch.zeros(self.plan.total, dtype=torch.bfloat16, device=device)
        self.g_views = []
        for m, off in zip(self.modules, self.plan.offsets):
            n = m.int_weight.numel()
            view = self.q[off:off + n].view(m.int_weight.shape)
            view.copy_(m.int_weight)
            m.int_weight = view  # replaces the registered buffer
            gv = self.g[off:off + n].view(m.int_weight.shape)
            set_grad_slot(m._registered_handle, gv)
            self.g_views.append(gv)

    def collect_grads(self) -> list[bool]:
        """Hand the gradients of this step over from the grad cache to the arena.

        Returns, per module, whether it produced a gradient.  Modules without one
        get zeros in their slot (and are skipped by the update, like
        fireflyoptim.py:137-139); a gradient that is not the slot itself (e.g.
        set by hand) is copied in.
        """
        has = []
        for m, gv in zip(self.modules, self.g_views):
            g = _BIT_GRAD_CACHE.pop(m._registered_handle, None)
            if g is None:
                gv.zero_()
            elif g.data_ptr() != gv.data_ptr():
                gv.copy_(g.reshape(gv.shape))
            has.append(g is not None)
        return has


def _reduce_scatter_avg(out: torch.Tensor, inp: torch.Tensor, group) -> None:
    ws = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.AVG, group=group)
    else:  # gloo: no AVG
        dist.reduce_scatter_tensor(out, inp, op=dist.ReduceOp.SUM, group=group)
        out.div_(ws)


class ZeroFireFlyOptim:
    """FireFlyOptim's BitLinear update, data-parallel with ZeRO-1 sharded 8-bit states.

    Same hyperparameters and update as ``FireFlyOptim`` (fireflyoptim.py:86-211).
    Call ``step()`` after the backward pass of every rank.  Dense parameters
    (``params``) are all-reduced (average) and stepped by AdamW on every rank.

    ``update_fn`` (default: the ``ff_dqt_adamw8`` kernel) receives keyword
    arguments for one segment; it exists so the sharding and collectives can be
    exercised with another implementation of the update (e.g. on CPU ranks).
    """

    def __init__(self, bit_modules: Sequence[BitLinear], params=(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.1, block_size=256, sr_bias_scale=0.15, process_group=None,
                 update_fn: Callable | None = None, seed: int | None = None):
        if int(block_size) != BLOCK:
            raise ValueError(f"block_size must be {BLOCK} on this build")
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.modules = list(bit_modules)
        for m in self.modules:
            if not isinstance(m, BitLinear):
                raise TypeError(f"expected BitLinear, got {type(m).__name__}")
        self.lr, self.betas, self.eps, self.wd = float(lr), tuple(betas), float(eps), float(weight_decay)
        self.sr_bias_scale = float(sr_bias_scale)
        self.arena = BitArena(self.modules, self.world, self.rank)
        self.plan = self.arena.plan
        dev = self.arena.q.device
        n = self.plan.shard
        nb = n // BLOCK
        self.m_q = torch.full((n,), 128, dtype=torch.uint8, device=dev)
        self.v_q = torch.zeros((n,), dtype=torch.uint8, device=dev)
        self.r_q = torch.full((n,), 128, dtype=torch.uint8, device=dev)
        self.m_absmax = torch.full((nb,), 1e-12, dtype=torch.float32, device=dev)
        self.v_absmax = self.m_absmax.clone()
        self.r_absmax = self.m_absmax.clone()
        self.g_shard = torch.empty((n,), dtype=torch.bfloat16, device=dev) if self.world > 1 else None
        self.steps = [0] * len(self.modules)
        if seed is None:
            seed = int(torch.randint(0, 2**62, (1,), dtype=torch.int64).item())
        if self.world > 1:
            t = torch.tensor([seed], dtype=torch.int64, device=dev if dev.type == "cuda" else "cpu")
            dist.broadcast(t, src=0, group=self.group)
            seed = int(t.item())
        self.rng_seed = seed
        self.update_fn = update_fn or self._kernel_update
        self.dense = [p for p in params if p.requires_grad]
        self.dense_opt = (AdamW8bitDense(self.dense, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
                          if self.dense else None)
        # every rank starts from rank 0's weights
        if self.world > 1:
            dist.broadcast(self.arena.q, src=0, group=self.group)
            for p in self.dense:
                dist.broadcast(p.data, src=0, group=self.group)
        for m in self.modules:
            _invalidate_weight_cache(m._registered_handle)

    # -- the per-segment update ------------------------------------------------
    def _kernel_update(self, *, q, wscale, row_len, elem_base, g, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax,
                       step, rng_offset):
        dec_s, dec_u = _tables_on(q.device)
        _capi.dqt_adamw8(q, wscale, row_len, g, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax,
                         lr=self.lr, beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, wd=self.wd,
                         step=step, sr_bias=self.sr_bias_scale, seed=self.rng_seed, rng_offset=rng_offset,
                         elem_base=elem_base, dec_s=dec_s, dec_u=dec_u)

    @torch.no_grad()
    def step(self) -> None:
        plan = self.plan
        has_grad = self.arena.collect_grads()
        if self.world > 1:
            _reduce_scatter_avg(self.g_shard, self.arena.g, self.group)
            g_local = self.g_shard
        else:
            g_local = self.arena.g[plan.lo:plan.hi]
        for i, h in enumerate(has_grad):
            self.steps[i] += int(h)
        for seg in plan.segments:
            if not has_grad[seg.module]:
                continue
            m = self.modules[seg.module]
            a, b = seg.lo - plan.lo, seg.hi - plan.lo
            ba, bb = plan.local_blocks(seg)
            self.update_fn(
                q=self.arena.q[seg.lo:seg.hi], wscale=m.weight_scale, row_len=m.in_features,
                elem_base=seg.elem_base, g=g_local[a:b], m_q=self.m_q[a:b], m_absmax=self.m_absmax[ba:bb],
                v_q=self.v_q[a:b], v_absmax=self.v_absmax[ba:bb], r_q=self.r_q[a:b],
                r_absmax=self.r_absmax[ba:bb], step=self.steps[seg.module], rng_offset=seg.lo,
            )
        if self.world > 1:
            dist.all_gather_into_tensor(self.arena.q, self.arena.q[plan.lo:plan.hi], group=self.group)
            for p in self.dense:
                if p.grad is not None:
                    if dist.get_backend(self.group) == "nccl":
                        dist.all_reduce(p.grad, op=dist.ReduceOp.AVG, group=self.group)
                    else:
                        dist.all_reduce(p.grad, group=self.group)
                        p.grad.div_(self.world)
        if self.dense_opt is not None:
            self.dense_opt.step()
        for m in self.modules:
            _invalidate_weight_cache(m._registered_handle)

    def zero_grad(self, set_to_none: bool = True) -> None:
        if self.dense_opt is not None:
            self.dense_opt.zero_grad(set_to_none=set_to_none)

    def shard_state(self) -> dict:
        """This rank's 8-bit states (flat, shard-local)."""
        return {"m_q": self.m_q, "m_absmax": self.m_absmax, "v_q": self.v_q, "v_absmax": self.v_absmax,
                "r_q": self.r_q, "r_absmax": self.r_absmax, "steps": list(self.steps)}

    def gather_bit_state(self) -> dict | None:
        """The full ``bit_state`` in the reference's checkpoint layout (fireflyoptim.py:213-222).

        Collective: every rank must call it; rank 0 gets ``{handle: {step, m_q, ...}}``
        with CPU tensors shaped like each weight, the other ranks get None.
        """
        plan = self.plan
        full = {}
        for key, is_abs in (("m_q", False), ("v_q", False), ("r_q", False),
                            ("m_absmax", True), ("v_absmax", True), ("r_absmax", True)):
            local = getattr(self, key)
            if self.world > 1:
                out = torch.empty((local.numel() * self.world,), dtype=local.dtype, device=local.device)
                dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
            else:
                out = local
            full[key] = out
        if self.rank != 0:
            return None
        res = {}
        for i, m in enumerate(self.modules):
            off, n = plan.offsets[i], plan.numels[i]
            b0, b1 = off // BLOCK, (off + n + BLOCK - 1) // BLOCK
            res[m._registered_handle] = {
                "step": self.steps[i],
                "m_q": full["m_q"][off:off + n].view(m.int_weight.shape).cpu().clone(),
                "m_absmax": full["m_absmax"][b0:b1].cpu().clone(),
                "v_q": full["v_q"][off:off + n].view(m.int_weight.shape).cpu().clone(),
                "v_absmax": full["v_absmax"][b0:b1].cpu().clone(),
                "r_q": full["r_q"][off:off + n].view(m.int_weight.shape).cpu().clone(),
                "r_absmax": full["r_absmax"][b0:b1].cpu().clone(),
            }
        return res

    def load_bit_state(self, bit_state: dict) -> None:
        """Load a full ``bit_state`` in the reference's checkpoint layout
        (``{handle: {step, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax}}``, fireflyoptim.py:213-233),
        keeping only this rank's shard of it (the ZeRO-1 scatter).

        Every rank passes the same dict (e.g. each loads the checkpoint file); the world size
        may differ from the one that saved it.  Modules absent from the dict keep fresh states.
        """
        plan = self.plan
        for i, m in enumerate(self.modules):
            ent = bit_state.get(m._registered_handle, bit_state.get(str(m._registered_handle)))
            if ent is None:
                continue
            self.steps[i] = int(ent["step"])
            off, n = plan.offsets[i], plan.numels[i]
            a, b = max(off, plan.lo), min(off + n, plan.hi)
            if a >= b:
                continue
            for key in ("m_q", "v_q", "r_q"):
                src = ent[key].reshape(-1)[a - off:b - off]
                getattr(self, key)[a - plan.lo:b - plan.lo].copy_(src.to(getattr(self, key).device))
            ga, gb = a // BLOCK, (b + BLOCK - 1) // BLOCK  # global 256-element blocks
            for key in ("m_absmax", "v_absmax", "r_absmax"):
                src = ent[key].reshape(-1)[ga - off // BLOCK:gb - off // BLOCK]
                dst = getattr(self, key)
                dst[ga - plan.lo // BLOCK:gb - plan.lo // BLOCK].copy_(src.to(dst.device))

    def state_dict(self) -> dict:
        """Collective (every rank calls it): ``bit_state`` in the reference layout on rank 0
        (None on the other ranks), ``bit_rng_seed``, and the dense optimizer's state."""
        return {"bit_state": self.gather_bit_state(), "bit_rng_seed": self.rng_seed,
                "dense": self.dense_opt.state_dict() if self.dense_opt is not None else None}

    def load_state_dict(self, state: dict) -> None:
        """Inverse of ``state_dict``: every rank passes the full dict saved by rank 0."""
        self.load_bit_state(state["bit_state"])
        if state.get("bit_rng_seed") is not None:
            self.rng_seed = int(state["bit_rng_seed"])
        if self.dense_opt is not None and state.get("dense") is not None:
            self.dense_opt.load_state_dict(state["dense"])

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
The arena is split into buckets of whole modules: a bucket's reduce-scatter starts from
the backward pass once its last weight gradient is issued (overlapping the rest of the
backward), and its all-gather right after its update (overlapping the next bucket's).

Arena layout: buckets of consecutive modules in ``bit_modules`` order; inside a bucket
module i occupies ``[off_i, off_i + numel_i)`` with ``off_i`` a multiple of 256, so its
256-element optimizer blocks are exactly the reference's per-module blocks
(fireflyoptim.py:13-19, :142-161).  The global element index that keys the
stochastic-rounding uniforms (module starts rounded up to 256, no bucket padding) is the
same on 1 GPU (``FireFlyOptim``) and on any number of GPUs: the sharded update equals the
single-GPU update.
"""
from __future__ import annotations

import weakref
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from . import _capi
from .adamw8 import AdamW8bitDense
from .bitLinear import BitLinear
from .fireflykernels import (
    _BIT_GRAD_CACHE,
    _invalidate_weight_cache,
    clear_activation_cache,
    set_grad_ready_hook,
    set_grad_slot,
)
from .fireflyoptim import BLOCK, _tables_on, bit_rng_offsets


@dataclass(frozen=True)
class Segment:
    """Part of one module inside this rank's shard."""

    module: int  # index into the module list
    lo: int  # arena element range [lo, hi)
    hi: int
    elem_base: int  # element index of ``lo`` within the module's weight
    rng: int  # global element index of ``lo`` (keys the stochastic rounding; world-size independent)
    local: int  # index of ``lo`` in this rank's state arrays
    bucket: int


@dataclass(frozen=True)
class Bucket:
    """Consecutive modules whose gradients are reduced (and weights gathered) by one collective."""

    modules: tuple[int, ...]
    lo: int  # arena range [lo, lo + size)
    size: int  # a multiple of block * world_size; rank r owns [lo + r*size/world, lo + (r+1)*size/world)
    local: int  # start of this rank's slice in the state arrays


class ShardPlan:
    """Which arena elements (and module pieces) each rank updates.  Pure host logic.

    Modules are grouped, in order, into buckets of at least ``bucket_elems`` elements (0: one
    bucket).  Inside a bucket every module starts at a multiple of ``block``; a bucket is padded
    to a multiple of ``block * world_size`` and each rank owns the same 1/world slice of every
    bucket, so a bucket's gradients are one reduce-scatter and its weights one all-gather.
    The global element index of a weight element (``rng_offsets[i]`` + its index in module i,
    module starts rounded up to ``block``) does not depend on the world size or the buckets.
    """

    def __init__(self, numels: Sequence[int], world_size: int, rank: int, block: int = BLOCK,
                 bucket_elems: int = 0):
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"bad rank {rank} of {world_size}")
        self.block = block
        self.numels = [int(n) for n in numels]
        self.world_size, self.rank = world_size, rank
        self.rng_offsets = []
        off = 0
        for n in self.numels:
            self.rng_offsets.append(off)
            off += _capi.round_up(n, block)
        self.used = off
        groups, cur, cur_elems = [], [], 0
        for i, n in enumerate(self.numels):
            cur.append(i)
            cur_elems += _capi.round_up(n, block)
            if bucket_elems > 0 and cur_elems >= bucket_elems:
                groups.append(cur)
                cur, cur_elems = [], 0
        if cur or not groups:
            groups.append(cur)
        self.offsets = [0] * len(self.numels)
        self.buckets: list[Bucket] = []
        arena = local = 0
        for mods in groups:
            start = self.rng_offsets[mods[0]] if mods else 0
            inner = sum(_capi.round_up(self.numels[i], block) for i in mods)
            size = _capi.round_up(max(inner, 1), block * world_size)
            for i in mods:
                self.offsets[i] = arena + self.rng_offsets[i] - start
            self.buckets.append(Bucket(tuple(mods), arena, size, local))
            arena += size
            local += size // world_size
        self.total = arena
        self.shard = local  # state elements on each rank
        self.bucket_of = [0] * len(self.numels)
        self.segments: list[Segment] = []
        for bi, bk in enumerate(self.buckets):
            lo, hi = self.rank_slice(bi)
            for i in bk.modules:
                self.bucket_of[i] = bi
                o, n = self.offsets[i], self.numels[i]
                a, e = max(o, lo), min(o + n, hi)
                if a < e:
                    self.segments.append(Segment(i, a, e, a - o, self.rng_offsets[i] + a - o, bk.local + a - lo, bi))

    def rank_slice(self, bucket: int, rank: int | None = None) -> tuple[int, int]:
        """Arena range of ``rank``'s slice of a bucket (this rank by default)."""
        bk = self.buckets[bucket]
        r = self.rank if rank is None else rank
        s = bk.size // self.world_size
        return bk.lo + r * s, bk.lo + (r + 1) * s

    def local_blocks(self, seg: Segment) -> tuple[int, int]:
        """Block range of ``seg`` within this rank's absmax arrays."""
        return seg.local // self.block, (seg.local + seg.hi - seg.lo + self.block - 1) // self.block

    def to_arena(self, gathered: torch.Tensor, unit: int = 1) -> torch.Tensor:
        """Reorder the rank-major concatenation of every rank's state array (``world * shard / unit``
        entries, ``unit`` arena elements per entry) into arena order (``total / unit`` entries)."""
        if self.world_size == 1:
            return gathered
        out = torch.empty((self.total // unit,), dtype=gathered.dtype, device=gathered.device)
        per = self.shard // unit
        for bk in self.buckets:
            s = bk.size // self.world_size // unit
            for r in range(self.world_size):
                src = r * per + bk.local // unit
                dst = bk.lo // unit + r * s
                out[dst:dst + s] = gathered[src:src + s]
        return out


class BitArena:
    """Flat int8 weight and bf16 gradient buffers shared by a list of BitLinear modules.

    After construction every module's ``int_weight`` buffer is a view of ``q`` and
    its weight gradient is routed into the matching view of ``g``.
    """

    def __init__(self, modules: Sequence[BitLinear], world_size: int = 1, rank: int = 0,
                 device: torch.device | None = None, bucket_elems: int = 0,
                 alloc: Callable[[int], tuple[torch.Tensor, torch.Tensor]] | None = None):
        self.modules = list(modules)
        if not self.modules:
            raise ValueError("BitArena needs at least one BitLinear")
        device = device or self.modules[0].int_weight.device
        self.plan = ShardPlan([m.int_weight.numel() for m in self.modules], world_size, rank,
                              bucket_elems=bucket_elems)
        assert self.plan.rng_offsets == bit_rng_offsets(self.modules)
        if alloc is None:
            self.q = torch.zeros(self.plan.total, dtype=torch.int8, device=device)
            self.g = torch.zeros(self.plan.total, dtype=torch.bfloat16, device=device)
        else:  # caller-provided memory (int8 and bf16 arrays of plan.total elements), zeroed here
            self.q, self.g = alloc(self.plan.total)
            self.q.zero_()
            self.g.zero_()
        self.g_views = []
        for m, off in zip(self.modules, self.plan.offsets):
            n = m.int_weight.numel()
            view = self.q[off:off + n].view(m.int_weight.shape)
            view.copy_(m.int_weight)
            m.int_weight = view  # replaces the registered buffer
            gv = self.g[off:off + n].view(m.int_weight.shape)
            set_grad_slot(m._registered_handle, gv)
            self.g_views.append(gv)

    def take_grad(self, i: int) -> bool:
        """Make module i's slot hold its gradient of this step (copying one that was set by hand
        elsewhere); False when it has none."""
        m, gv = self.modules[i], self.g_views[i]
        g = _BIT_GRAD_CACHE.get(m._registered_handle)
        if g is None:
            return False
        if g.data_ptr() != gv.data_ptr():
            gv.copy_(g.reshape(gv.shape))
            _BIT_GRAD_CACHE[m._registered_handle] = gv
        return True

    def collect_grads(self) -> list[bool]:
        """Hand the gradients of this step over from the grad cache to the arena.

        Returns, per module, whether it produced a gradient.  Modules without one
        get zeros in their slot (and are skipped by the update, like
        fireflyoptim.py:137-139); a gradient that is not the slot itself (e.g.
        set by hand) is copied in.
        """
        has = []
        for i, (m, gv) in enumerate(zip(self.modules, self.g_views)):
            h = self.take_grad(i)
            _BIT_GRAD_CACHE.pop(m._registered_handle, None)
            if not h:
                gv.zero_()
            has.append(h)
        return has


# dense gradients with at least this many elements are all-reduced in place, not flattened
_DENSE_INPLACE_NUMEL = 1 << 20


class ZeroFireFlyOptim:
    """FireFlyOptim's BitLinear update, data-parallel with ZeRO-1 sharded 8-bit states.

    Same hyperparameters and update as ``FireFlyOptim`` (fireflyoptim.py:86-211).
    Call ``step()`` after the backward pass of every rank.  Dense parameters
    (``params``) are all-reduced (average) and stepped by ``AdamW8bitDense`` on every rank.

    The arena is split into buckets of whole modules (``bucket_mb`` of bf16 gradient each).
    With ``overlap`` (and more than one rank) a bucket's reduce-scatter is issued from the
    backward pass once the weight-gradient GEMMs of all its modules have been issued, so it
    runs under the rest of the backward; buckets are always reduced in the same order on
    every rank (last bucket first; a complete bucket waits for the ones after it), which keeps
    the ranks' collectives matched when the backward produces gradients in another order or
    a module has no gradient on some ranks.  ``step()`` updates the buckets in that order,
    each as soon as its reduction is done, and issues each bucket's weight all-gather right
    after its update.  With gradient accumulation, run every backward but the last of a step
    under ``no_sync()`` (each BitLinear must produce one weight gradient per synced backward).

    A module that produced a weight gradient on some ranks only (e.g. it was not used in the
    forward of the others) is updated on every rank with the average in which the other ranks
    count zero, and its step count advances everywhere: the ranks agree on which modules have
    gradients through a small host-side all-reduce (gloo; a side group when the main group is
    NCCL), which never waits for the GPU.

    ``update_fn`` (default: the ``ff_dqt_adamw8`` kernel) receives keyword
    arguments for one segment; it exists so the sharding and collectives can be
    exercised with another implementation of the update (e.g. on CPU ranks).
    """

    def __init__(self, bit_modules: Sequence[BitLinear], params=(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.1, block_size=256, sr_bias_scale=0.15, process_group=None,
                 update_fn: Callable | None = None, seed: int | None = None, bucket_mb: float = 256.0,
                 overlap: bool = True, peer: bool | None = None):
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
        bucket_elems = int(bucket_mb * 2**20) // 2 if bucket_mb and bucket_mb > 0 else 0
        self._nccl = self.world > 1 and dist.get_backend(self.group) == "nccl"
        # host-side agreement on which modules have gradients (no GPU synchronisation)
        self._host_group = None
        if self.world > 1:
            if dist.get_backend(self.group) == "gloo":
                self._host_group = self.group
            else:
                ranks = None if self.group is None else dist.get_process_group_ranks(self.group)
                self._host_group = dist.new_group(ranks=ranks, backend="gloo")
        # peer mode: the ranks of one node read each other's gradient arena and write each other's
        # weight arena from the update kernel (ff_dqt_adamw8_peers) instead of the collectives
        want_peer = (peer is None or peer) and self._nccl and 2 <= self.world <= _capi.DQT_MAX_SOURCES and \
            update_fn is None
        if peer and not want_peer:
            raise ValueError("peer=True needs an NCCL process group of 2 to 8 ranks and the kernel update")
        self._ipc = None
        alloc = None
        if want_peer:
            dev0 = self.modules[0].int_weight.device

            def alloc(total, dev0=dev0):  # raises RuntimeError when the allocation fails
                qb, gb = _capi.IpcBuffer(total, dev0), _capi.IpcBuffer(2 * total, dev0)
                self._ipc = [qb, gb]
                return qb.tensor(torch.int8), gb.tensor(torch.bfloat16)
        try:
            self.arena = BitArena(self.modules, self.world, self.rank, bucket_elems=bucket_elems, alloc=alloc)
        except (RuntimeError, ValueError):
            if alloc is None:
                raise
            self._ipc = None  # no shareable memory here: the collectives path
            self.arena = BitArena(self.modules, self.world, self.rank, bucket_elems=bucket_elems)
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
        self.peer = False
        self._peer_maps: list = []
        if want_peer:
            self.peer = self._connect_peers()
            if peer and not self.peer:
                raise RuntimeError("peer=True: the ranks could not map each other's arenas")
        # with peer mode: the averaged gradient of this rank's shard is also written to g_shard
        self.keep_reduced_grad = False
        self._sync = True
        # None, or a list to which step() appends (phase, start event, end event) triples timing on
        # the current stream each wait for a collective (its exposed part) and the whole step
        self.comm_events: list | None = None
        self._module_of = {m._registered_handle: i for i, m in enumerate(self.modules)}
        self._reset_pending()
        self.overlap = bool(overlap) and self.world > 1 and not self.peer  # peer mode reduces in the update
        if self.overlap:
            # the hooks hold the optimizer weakly: a discarded optimizer stops reducing
            ref = weakref.ref(self)

            def hook(handle, ref=ref):
                opt = ref()
                if opt is not None:
                    opt._on_grad_ready(handle)

            for m in self.modules:
                set_grad_ready_hook(m._registered_handle, hook)

    def close(self) -> None:
        """Remove this optimizer's gradient hooks from its modules (later backward passes no
        longer start reductions for it) and unmap the other ranks' arenas (every rank closes)."""
        if self.overlap:
            for m in self.modules:
                set_grad_ready_hook(m._registered_handle, None)
            self.overlap = False
        if self.peer:
            torch.cuda.synchronize(self.arena.q.device)  # no update kernel still reads or writes a peer
            for mp in self._peer_maps:
                mp.close()
            self._peer_maps = []
            self.peer = False

    # -- peer mode -----------------------------------------------------------------
    def _connect_peers(self) -> bool:
        """Map every other rank's weight and gradient arenas into this process (CUDA IPC), when all
        ranks run on this node and have shareable arenas; all ranks agree on the outcome."""
        import socket

        dev = self.arena.q.device
        mine = None
        if self._ipc:
            try:
                mine = (socket.gethostname(), self._ipc[0].handle(), self._ipc[1].handle())
            except (RuntimeError, ValueError):
                mine = None
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=self._host_group)
        ok = all(v is not None for v in every) and len({v[0] for v in every}) == 1
        q_ptrs, g_ptrs, maps = [], [], []
        if ok:
            try:
                for r, v in enumerate(every):
                    if r == self.rank:
                        q_ptrs.append(self.arena.q.data_ptr())
                        g_ptrs.append(self.arena.g.data_ptr())
                        continue
                    mq, mg = _capi.IpcMapping(v[1], dev), _capi.IpcMapping(v[2], dev)
                    maps += [mq, mg]
                    q_ptrs.append(mq.ptr)
                    g_ptrs.append(mg.ptr)
            except (RuntimeError, ValueError):
                ok = False
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self._host_group)
        if int(flag.item()) == 0:
            for mp in maps:
                mp.close()
            return False
        self._peer_maps, self._q_ptrs, self._g_ptrs = maps, q_ptrs, g_ptrs
        self._fence_t = torch.zeros(1, dtype=torch.int32, device=dev)
        return True

    def _peer_fence(self) -> None:
        """Order this rank's stream after every rank's work issued so far: a one-element NCCL
        all-reduce on the stream completes only once every rank's stream has reached it."""
        t = self._mark()
        dist.all_reduce(self._fence_t, group=self.group)
        self._timed("peer_fence_wait", t)

    def _update_bucket_peer(self, b: int, has_grad: list[bool]) -> None:
        """This rank's slice of bucket b from every rank's gradient, its new weights written to every
        rank's arena (ff_dqt_adamw8_peers): the reduce-scatter and all-gather inside the update."""
        plan = self.plan
        dec_s, dec_u = _tables_on(self.arena.q.device)
        for seg in self._segments_of[b]:
            if not has_grad[seg.module]:
                continue
            m = self.modules[seg.module]
            a, e = seg.local, seg.local + seg.hi - seg.lo
            ba, bb = plan.local_blocks(seg)
            _capi.dqt_adamw8_peers(
                self.arena.q[seg.lo:seg.hi], m.weight_scale, m.in_features,
                [ptr + 2 * seg.lo for ptr in self._g_ptrs], [ptr + seg.lo for ptr in self._q_ptrs],
                self.m_q[a:e], self.m_absmax[ba:bb], self.v_q[a:e], self.v_absmax[ba:bb], self.r_q[a:e],
                self.r_absmax[ba:bb], lr=self.lr, beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, wd=self.wd,
                step=self.steps[seg.module], sr_bias=self.sr_bias_scale, seed=self.rng_seed, rng_offset=seg.rng,
                elem_base=seg.elem_base, g_out=self.g_shard[a:e] if self.keep_reduced_grad else None,
                dec_s=dec_s, dec_u=dec_u)

    # -- overlapped reduction ----------------------------------------------------
    def _reset_pending(self) -> None:
        self._ready: set[int] = set()
        self._remaining = [len(b.modules) for b in self.plan.buckets]
        self._rs_work: dict[int, object] = {}
        self._rs_order: list[int] = []
        self._next_reduce = len(self.plan.buckets) - 1  # buckets are reduced from the last one down

    def _launch_ready_reductions(self) -> None:
        """Issue the reduce-scatters of complete buckets, in the fixed order (last bucket first)."""
        while self._next_reduce >= 0 and self._remaining[self._next_reduce] == 0:
            self._launch_reduce(self._next_reduce)
            self._next_reduce -= 1

    @contextmanager
    def no_sync(self):
        """Backward passes inside only accumulate gradients (no reduction is issued)."""
        prev, self._sync = self._sync, False
        try:
            yield
        finally:
            self._sync = prev

    def _on_grad_ready(self, handle: int) -> None:
        if not self._sync:
            return
        i = self._module_of[handle]
        if i in self._ready:
            raise RuntimeError(
                f"BitLinear handle {handle} produced a second weight gradient in one synced backward; run the "
                "accumulating backward passes under no_sync(), or construct ZeroFireFlyOptim with overlap=False")
        self.arena.take_grad(i)
        self._ready.add(i)
        self._remaining[self.plan.bucket_of[i]] -= 1
        self._launch_ready_reductions()

    def _launch_reduce(self, b: int) -> None:
        bk = self.plan.buckets[b]
        s = bk.size // self.world
        out, inp = self.g_shard[bk.local:bk.local + s], self.arena.g[bk.lo:bk.lo + bk.size]
        op = dist.ReduceOp.AVG if self._nccl else dist.ReduceOp.SUM  # gloo has no AVG
        self._rs_work[b] = dist.reduce_scatter_tensor(out, inp, op=op, group=self.group, async_op=True)
        self._rs_order.append(b)

    def _finish_reduce(self, b: int) -> None:
        self._rs_work.pop(b).wait()  # the current stream waits for the reduction
        if not self._nccl:
            bk = self.plan.buckets[b]
            s = bk.size // self.world
            self.g_shard[bk.local:bk.local + s].div_(self.world)

    def _launch_dense_reduce(self):
        """One all-reduce (average) per dtype over the flattened dense gradients."""
        groups: dict[torch.dtype, list[torch.Tensor]] = {}
        for p in self.dense:
            if p.grad is not None:
                groups.setdefault(p.grad.dtype, []).append(p)
        pending = []
        op = dist.ReduceOp.AVG if self._nccl else dist.ReduceOp.SUM
        for params in groups.values():
            # large gradients (embeddings) are reduced where they lie; the small ones in one flat buffer
            small = []
            for p in params:
                if p.grad.numel() >= _DENSE_INPLACE_NUMEL and p.grad.is_contiguous():
                    pending.append(([p], None, dist.all_reduce(p.grad, op=op, group=self.group, async_op=True)))
                else:
                    small.append(p)
            if small:
                flat = torch._utils._flatten_dense_tensors([p.grad for p in small])
                pending.append((small, flat, dist.all_reduce(flat, op=op, group=self.group, async_op=True)))
        return pending

    def _finish_dense_reduce(self, pending) -> None:
        for params, flat, work in pending:
            work.wait()
            if flat is None:
                if not self._nccl:
                    params[0].grad.div_(self.world)
                continue
            if not self._nccl:
                flat.div_(self.world)
            # each gradient becomes its slice of the reduced buffer (no copy back)
            for p, f in zip(params, torch._utils._unflatten_dense_tensors(flat, [p.grad for p in params])):
                p.grad = f

    # -- the per-segment update ------------------------------------------------
    def _kernel_update(self, *, q, wscale, row_len, elem_base, g, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax,
                       step, rng_offset):
        dec_s, dec_u = _tables_on(q.device)
        _capi.dqt_adamw8(q, wscale, row_len, g, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax,
                         lr=self.lr, beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, wd=self.wd,
                         step=step, sr_bias=self.sr_bias_scale, seed=self.rng_seed, rng_offset=rng_offset,
                         elem_base=elem_base, dec_s=dec_s, dec_u=dec_u)

    def _update_bucket(self, b: int, g_local: torch.Tensor, has_grad: list[bool]) -> None:
        plan = self.plan
        for seg in self._segments_of[b]:
            if not has_grad[seg.module]:
                continue
            m = self.modules[seg.module]
            a, e = seg.local, seg.local + seg.hi - seg.lo
            ba, bb = plan.local_blocks(seg)
            self.update_fn(
                q=self.arena.q[seg.lo:seg.hi], wscale=m.weight_scale, row_len=m.in_features,
                elem_base=seg.elem_base, g=g_local[a:e], m_q=self.m_q[a:e], m_absmax=self.m_absmax[ba:bb],
                v_q=self.v_q[a:e], v_absmax=self.v_absmax[ba:bb], r_q=self.r_q[a:e],
                r_absmax=self.r_absmax[ba:bb], step=self.steps[seg.module], rng_offset=seg.rng,
            )

    @property
    def _segments_of(self) -> list[list[Segment]]:
        segs = getattr(self, "_segs_cache", None)
        if segs is None:
            segs = [[] for _ in self.plan.buckets]
            for seg in self.plan.segments:
                segs[seg.bucket].append(seg)
            self._segs_cache = segs
        return segs

    def _mark(self):
        if self.comm_events is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _timed(self, phase: str, start) -> None:
        if start is not None:
            self.comm_events.append((phase, start, self._mark()))

    @torch.no_grad()
    def step(self) -> None:
        plan = self.plan
        t_step = self._mark()
        clear_activation_cache()  # the next step's inputs are quantised afresh
        has_grad = self.arena.collect_grads()
        if self.world > 1:
            if not self.peer:
                # buckets not reduced during the backward (no overlap, or a module without a
                # gradient, whose slot now holds zeros) are reduced now, in the same fixed order
                for b in range(self._next_reduce, -1, -1):
                    self._launch_reduce(b)
                self._next_reduce = -1
            # a module with a gradient on any rank is updated on every rank
            flags = torch.tensor(has_grad, dtype=torch.int32)
            dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self._host_group)
            has_grad = [bool(v) for v in flags.tolist()]
        for i, h in enumerate(has_grad):
            self.steps[i] += int(h)
        if self.peer:
            self._peer_fence()  # every rank's gradients are complete
            dense = self._launch_dense_reduce()  # on the collective stream, under the updates
            t = self._mark()
            for b in range(len(plan.buckets)):
                self._update_bucket_peer(b, has_grad)
            self._timed("peer_update", t)
            self._peer_fence()  # every rank's new weights are written and its gradients read
            t = self._mark()
            self._finish_dense_reduce(dense)
            self._timed("dense_all_reduce_wait", t)
        elif self.world > 1:
            dense = self._launch_dense_reduce()
            gathers = []
            for b in list(self._rs_order):
                t = self._mark()
                self._finish_reduce(b)
                self._timed("reduce_scatter_wait", t)
                self._update_bucket(b, self.g_shard, has_grad)
                bk = plan.buckets[b]
                lo, hi = plan.rank_slice(b)
                gathers.append(dist.all_gather_into_tensor(self.arena.q[bk.lo:bk.lo + bk.size], self.arena.q[lo:hi],
                                                           group=self.group, async_op=True))
            t = self._mark()
            self._finish_dense_reduce(dense)
            self._timed("dense_all_reduce_wait", t)
            t = self._mark()
            for w in gathers:
                w.wait()  # the next forward reads the gathered weights
            self._timed("all_gather_wait", t)
        else:
            for b in range(len(plan.buckets)):
                self._update_bucket(b, self.arena.g, has_grad)
        self._reset_pending()
        if self.dense_opt is not None:
            self.dense_opt.step()
        for m in self.modules:
            _invalidate_weight_cache(m._registered_handle)
        self._timed("optimizer_step", t_step)

    def zero_grad(self, set_to_none: bool = True) -> None:
        if self.dense_opt is not None:
            self.dense_opt.zero_grad(set_to_none=set_to_none)

    def shard_state(self) -> dict:
        """This rank's 8-bit states (flat, shard-local: the rank's slice of every bucket)."""
        return {"m_q": self.m_q, "m_absmax": self.m_absmax, "v_q": self.v_q, "v_absmax": self.v_absmax,
                "r_q": self.r_q, "r_absmax": self.r_absmax, "steps": list(self.steps)}

    def gather_bit_state(self) -> dict | None:
        """The full ``bit_state`` in the reference's checkpoint layout (fireflyoptim.py:213-222).

        Collective: every rank must call it; rank 0 gets ``{handle: {step, m_q, ...}}``
        with CPU tensors shaped like each weight, the other ranks get None.
        """
        plan = self.plan
        full = {}
        for key, unit in (("m_q", 1), ("v_q", 1), ("r_q", 1), ("m_absmax", BLOCK), ("v_absmax", BLOCK),
                          ("r_absmax", BLOCK)):
            local = getattr(self, key)
            if self.world > 1:
                out = torch.empty((local.numel() * self.world,), dtype=local.dtype, device=local.device)
                dist.all_gather_into_tensor(out, local.contiguous(), group=self.group)
            else:
                out = local
            full[key] = plan.to_arena(out, unit)
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
        def entry(m):
            return bit_state.get(m._registered_handle, bit_state.get(str(m._registered_handle)))

        for i, m in enumerate(self.modules):
            ent = entry(m)
            if ent is not None:
                self.steps[i] = int(ent["step"])
        for seg in self.plan.segments:
            ent = entry(self.modules[seg.module])
            if ent is None:
                continue
            n = seg.hi - seg.lo
            for key in ("m_q", "v_q", "r_q"):
                src = ent[key].reshape(-1)[seg.elem_base:seg.elem_base + n]
                getattr(self, key)[seg.local:seg.local + n].copy_(src.to(getattr(self, key).device))
            ba, bb = self.plan.local_blocks(seg)
            g0 = seg.elem_base // BLOCK
            for key in ("m_absmax", "v_absmax", "r_absmax"):
                src = ent[key].reshape(-1)[g0:g0 + bb - ba]
                dst = getattr(self, key)
                dst[ba:bb].copy_(src.to(dst.device))

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

"""Data parallel + ZeRO-1 host logic on CPU ranks (gloo, world size 2).

The GPU update kernel is replaced by the oracle (``update_fn``), so these tests check the
sharding plan, the flat arenas, the reduce-scatter / all-gather plumbing and the
checkpoint gather, not the kernels (those are covered by the GPU tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from firefly_b200.distributed import ShardPlan

WD, LR, SEED = 0.01, 1e-3, 1234
SHAPES = [(48, 80), (33, 70), (16, 256), (7, 40)]


@pytest.mark.parametrize("bucket_elems", [0, 1, 5000])
def test_shard_plan_covers_every_element_once(bucket_elems):
    numels = [o * k for o, k in SHAPES]
    rng_starts = np.cumsum([0] + [-(-n // 256) * 256 for n in numels[:-1]])
    for world in (1, 2, 3, 4, 8):
        seen = np.zeros(sum(numels), np.int64)
        flat_starts = np.cumsum([0] + numels[:-1])
        total = None
        for rank in range(world):
            plan = ShardPlan(numels, world, rank, bucket_elems=bucket_elems)
            total = plan.total
            assert plan.total % (256 * world) == 0 and plan.shard * world == plan.total
            assert all(o % 256 == 0 for o in plan.offsets)
            assert plan.rng_offsets == list(rng_starts)
            if bucket_elems == 1:
                assert len(plan.buckets) == len(numels)
            for bi, bk in enumerate(plan.buckets):
                assert bk.size % (256 * world) == 0
                assert all(plan.bucket_of[i] == bi for i in bk.modules)
            local_seen = np.zeros(plan.shard, np.int64)
            for seg in plan.segments:
                lo, hi = plan.rank_slice(seg.bucket)
                assert lo <= seg.lo < seg.hi <= hi
                assert seg.lo % 256 == 0 and seg.local % 256 == 0
                off = plan.offsets[seg.module]
                assert seg.elem_base == seg.lo - off and seg.hi <= off + numels[seg.module]
                assert seg.rng == rng_starts[seg.module] + seg.elem_base
                assert seg.local == plan.buckets[seg.bucket].local + seg.lo - lo
                local_seen[seg.local:seg.local + seg.hi - seg.lo] += 1
                start = flat_starts[seg.module] + seg.elem_base
                seen[start:start + seg.hi - seg.lo] += 1
                b0, b1 = plan.local_blocks(seg)
                assert 0 <= b0 < b1 <= plan.shard // 256
            assert local_seen.max(initial=0) <= 1
        assert (seen == 1).all(), world
        assert total >= sum(-(-n // 256) * 256 for n in numels)


def test_shard_plan_to_arena_inverts_the_rank_major_gather():
    numels = [o * k for o, k in SHAPES]
    for world in (2, 3):
        plans = [ShardPlan(numels, world, r, bucket_elems=5000) for r in range(world)]
        arena = torch.arange(plans[0].total)
        gathered = torch.cat([torch.cat([arena[slice(*p.rank_slice(b))] for b in range(len(p.buckets))])
                              for p in plans])
        assert torch.equal(plans[0].to_arena(gathered), arena)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_modules(monkeypatch_quant=True):
    import firefly_b200.bitLinear as bl
    from oracle import firefly_oracle as O

    def cpu_quant(w, eps=1e-8):
        q, s = O.quantize_rows(w.detach().float().numpy(), eps)
        return torch.from_numpy(q), torch.from_numpy(s)

    bl.quantize_fp_to_int8 = cpu_quant  # this test runs the host logic on CPU ranks
    torch.manual_seed(SEED)
    return [bl.BitLinear(k, o) for o, k in SHAPES]


def _oracle_update(steps_done, seed):
    from oracle import firefly_oracle as O

    def update(*, q, wscale, row_len, elem_base, g, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax, step,
               rng_offset):
        n = q.numel()
        st = {"step": step - 1, "m_q": m_q.numpy(), "m_absmax": m_absmax.numpy(), "v_q": v_q.numpy(),
              "v_absmax": v_absmax.numpy(), "r_q": r_q.numpy(), "r_absmax": r_absmax.numpy()}
        u = O.philox_uniforms(n, seed=seed, step=step, elem_offset=rng_offset)
        g32 = g.float().numpy()
        qn, stn = O.dqt_adamw8_segment(q.numpy(), wscale.numpy(), row_len, elem_base, g32, st, lr=LR, wd=WD, u=u)
        q.copy_(torch.from_numpy(qn))
        for k, t in (("m_q", m_q), ("v_q", v_q), ("r_q", r_q), ("m_absmax", m_absmax), ("v_absmax", v_absmax),
                     ("r_absmax", r_absmax)):
            t.copy_(torch.from_numpy(np.ascontiguousarray(stn[k]).reshape(t.shape)))
        steps_done.append(step)
    return update


def _grads(step):
    g = torch.Generator().manual_seed(500 + step)
    return [(torch.randn(o, k, generator=g) * 1e-2).to(torch.bfloat16) for o, k in SHAPES]


def _run(rank, world, port, out_dir, buckets=False):
    """Three steps; with ``buckets`` the arena is split into two buckets and the gradients are
    announced module by module, last module first, as a backward pass does (the overlapped
    reduce-scatters start from those announcements)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE, _grad_ready

    mods = _make_modules()
    calls = []
    opt = ZeroFireFlyOptim(mods, lr=LR, weight_decay=WD, seed=SEED, update_fn=_oracle_update(calls, SEED),
                           bucket_mb=0.01 if buckets else 64.0)
    if buckets:
        assert [b.modules for b in opt.plan.buckets] == [(0, 1), (2, 3)]
    for step in range(3):
        for m, g in reversed(list(zip(mods, _grads(step)))):
            if step == 1 and m is mods[3]:
                continue  # a module without gradient this step is skipped
            _BIT_GRAD_CACHE[m._registered_handle] = g.clone()
            if buckets:
                _grad_ready(m._registered_handle)
        if buckets and world > 1:
            # bucket (2, 3) is complete only when module 3 has a gradient
            # buckets are reduced last first: bucket (0, 1) waits for (2, 3), which is complete
            # only when module 3 has a gradient (at step 1 both are reduced from step())
            assert opt._rs_order == ([] if step == 1 else [1, 0])
        opt.step()
    bits = opt.gather_bit_state()
    if rank == 0:
        torch.save({"q": [m.int_weight.clone() for m in mods], "bits": bits, "steps": list(opt.steps)},
                   os.path.join(out_dir, f"world{world}{'_buckets' if buckets else ''}.pt"))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _dense_grads(rank, step):
    g = torch.Generator().manual_seed(900 + 10 * step + rank)
    return [torch.randn(1100, 1000, generator=g), torch.randn(300, generator=g), torch.randn(7, 3, generator=g)]


def _run_dense(rank, world, port, out_dir):
    """Two steps with dense parameters beside the BitLinears: one large enough to be all-reduced
    in place, two that share a flat buffer; each rank has its own dense gradients."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from firefly_b200.distributed import _DENSE_INPLACE_NUMEL, ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE

    mods = _make_modules()
    g = torch.Generator().manual_seed(77)
    dense = [torch.nn.Parameter(torch.randn(1100, 1000, generator=g)), torch.nn.Parameter(torch.randn(300, generator=g)),
             torch.nn.Parameter(torch.randn(7, 3, generator=g))]
    assert dense[0].numel() >= _DENSE_INPLACE_NUMEL > dense[1].numel()
    opt = ZeroFireFlyOptim(mods, params=dense, lr=LR, weight_decay=WD, seed=SEED, update_fn=_oracle_update([], SEED))
    for step in range(2):
        for m, gb in zip(mods, _grads(step)):
            _BIT_GRAD_CACHE[m._registered_handle] = gb.clone()
        for p, gd in zip(dense, _dense_grads(rank, step)):
            p.grad = gd
        opt.step()
    torch.save([p.detach().clone() for p in dense], os.path.join(out_dir, f"dense_rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_zero1_dense_parameters_step_on_the_averaged_gradient(tmp_path):
    """Dense parameters are stepped by the dense optimizer on the rank average of their
    gradients (large ones reduced in place, small ones through a flat buffer): both ranks hold
    the parameters of a local AdamW step on (g0 + g1) / 2."""
    from firefly_b200.adamw8 import AdamW8bitDense

    mp.start_processes(_run_dense, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    got = [torch.load(tmp_path / f"dense_rank{r}.pt", weights_only=False) for r in range(2)]
    g = torch.Generator().manual_seed(77)
    ref = [torch.randn(1100, 1000, generator=g), torch.randn(300, generator=g), torch.randn(7, 3, generator=g)]
    states = [{} for _ in ref]
    with torch.no_grad():
        for step in range(2):
            for i, (p, st) in enumerate(zip(ref, states)):
                p.grad = (_dense_grads(0, step)[i] + _dense_grads(1, step)[i]) / 2
                AdamW8bitDense._step_32bit(p, st, LR, 0.9, 0.999, 1e-8, WD)
    for r in range(2):
        for a, b in zip(got[r], ref):
            assert torch.equal(a, b)


@pytest.mark.timeout(300)
def test_zero1_two_ranks_equal_single_rank(tmp_path):
    """Identical gradients on both ranks: averaging is exact, so the sharded update must
    reproduce the single-rank update bit for bit (same Philox stream by global index)."""
    _run(0, 1, _free_port(), str(tmp_path))
    mp.start_processes(_run, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    one = torch.load(tmp_path / "world1.pt", weights_only=False)
    two = torch.load(tmp_path / "world2.pt", weights_only=False)
    assert one["steps"] == two["steps"] == [3, 3, 3, 2]  # the last module had no gradient once
    for a, b in zip(one["q"], two["q"]):
        assert torch.equal(a, b)
    assert set(one["bits"]) == set(two["bits"])
    for h in one["bits"]:
        for k, v in one["bits"][h].items():
            w = two["bits"][h][k]
            assert (torch.equal(v, w) if torch.is_tensor(v) else v == w), (h, k)
    # the gathered state has the reference checkpoint layout (fireflyoptim.py:213-222)
    h0 = sorted(one["bits"])[0]
    ent = one["bits"][h0]
    assert set(ent) == {"step", "m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax"}
    assert ent["m_q"].shape == SHAPES[0] and ent["m_q"].dtype == torch.uint8
    assert ent["m_absmax"].shape == (-(-SHAPES[0][0] * SHAPES[0][1] // 256),)


@pytest.mark.timeout(300)
def test_zero1_overlapped_buckets_equal_single_rank(tmp_path):
    """Two buckets whose reduce-scatters start from the backward's gradient announcements:
    same weights and gathered states as the single-rank run."""
    _run(0, 1, _free_port(), str(tmp_path))
    mp.start_processes(_run, args=(2, _free_port(), str(tmp_path), True), nprocs=2, start_method="spawn")
    one = torch.load(tmp_path / "world1.pt", weights_only=False)
    two = torch.load(tmp_path / "world2_buckets.pt", weights_only=False)
    assert one["steps"] == two["steps"]
    for a, b in zip(one["q"], two["q"]):
        assert torch.equal(a, b)
    for h1, h2 in zip(sorted(one["bits"]), sorted(two["bits"])):
        for k, v in one["bits"][h1].items():
            w = two["bits"][h2][k]
            assert (torch.equal(v, w) if torch.is_tensor(v) else v == w), k


@pytest.mark.timeout(300)
def test_zero1_matches_unsharded_oracle(tmp_path):
    """The sharded result equals the per-module oracle update of the reference algorithm."""
    from oracle import firefly_oracle as O
    from firefly_b200.fireflyoptim import bit_rng_offsets

    mp.start_processes(_run, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    two = torch.load(tmp_path / "world2.pt", weights_only=False)
    mods = _make_modules()
    offs = bit_rng_offsets(mods)
    for i, (m, off) in enumerate(zip(mods, offs)):
        q = m.int_weight.numpy()
        ws = m.weight_scale.numpy()
        st = O.init_state(q.shape)
        for step in range(3):
            if step == 1 and i == 3:
                continue
            g = _grads(step)[i].float().numpy()
            t = st["step"] + 1
            u = O.philox_uniforms(q.size, seed=SEED, step=t, elem_offset=off).reshape(q.shape)
            q, st = O.dqt_adamw8_step(q, ws, g, st, lr=LR, wd=WD, u=u)
        np.testing.assert_array_equal(two["q"][i].numpy(), q)
        h = m._registered_handle
        got = two["bits"][sorted(two["bits"])[i]]
        np.testing.assert_array_equal(got["m_q"].numpy(), st["m_q"])
        np.testing.assert_array_equal(got["r_absmax"].numpy(), st["r_absmax"])
        assert got["step"] == st["step"]


def _run_resume(rank, world, port, out_dir, save_world):
    """Steps 0-1 at world size ``save_world`` are taken from a checkpoint written by a run
    of that size; this run (``world`` ranks) loads it and takes step 2."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE

    mods = _make_modules()
    ckpt = torch.load(os.path.join(out_dir, f"mid_world{save_world}.pt"), weights_only=False)
    with torch.no_grad():
        for m, q in zip(mods, ckpt["q"]):
            m.int_weight.copy_(q)
    opt = ZeroFireFlyOptim(mods, lr=LR, weight_decay=WD, seed=0, update_fn=None)
    # the checkpoint's handles are the modules' handles of the saving run, in module order
    state = ckpt["opt"]
    handles = sorted(state["bit_state"])
    state = dict(state, bit_state={m._registered_handle: state["bit_state"][h] for m, h in zip(mods, handles)})
    opt.load_state_dict(state)
    calls = []
    opt.update_fn = _oracle_update(calls, opt.rng_seed)
    for m, g in zip(mods, _grads(2)):
        _BIT_GRAD_CACHE[m._registered_handle] = g.clone()
    opt.step()
    bits = opt.gather_bit_state()
    if rank == 0:
        torch.save({"q": [m.int_weight.clone() for m in mods], "bits": bits},
                   os.path.join(out_dir, f"resumed_{save_world}_to_{world}.pt"))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _run_save_mid(rank, world, port, out_dir):
    """Two steps, then the optimizer's state_dict (collective) saved by rank 0."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE

    mods = _make_modules()
    opt = ZeroFireFlyOptim(mods, lr=LR, weight_decay=WD, seed=SEED, update_fn=_oracle_update([], SEED))
    for step in range(2):
        for m, g in zip(mods, _grads(step)):
            if step == 1 and m is mods[3]:
                continue
            _BIT_GRAD_CACHE[m._registered_handle] = g.clone()
        opt.step()
    state = opt.state_dict()
    if rank == 0:
        torch.save({"q": [m.int_weight.clone() for m in mods], "opt": state},
                   os.path.join(out_dir, f"mid_world{world}.pt"))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_zero1_checkpoint_resume_across_world_sizes(tmp_path):
    """A ZeRO-1 checkpoint (gathered into the reference bit_state layout) resumes at another
    world size: save after two steps at world 1 and at world 2, resume each at the other size
    for the third step, and compare with the uninterrupted three-step run."""
    _run(0, 1, _free_port(), str(tmp_path))
    _run_save_mid(0, 1, _free_port(), str(tmp_path))
    mp.start_processes(_run_save_mid, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    mp.start_processes(_run_resume, args=(2, _free_port(), str(tmp_path), 1), nprocs=2, start_method="spawn")
    _run_resume(0, 1, _free_port(), str(tmp_path), 2)
    full = torch.load(tmp_path / "world1.pt", weights_only=False)
    for name in ("resumed_1_to_2.pt", "resumed_2_to_1.pt"):
        res = torch.load(tmp_path / name, weights_only=False)
        for a, b in zip(full["q"], res["q"]):
            assert torch.equal(a, b), name
        for hf, hr in zip(sorted(full["bits"]), sorted(res["bits"])):
            for k, v in full["bits"][hf].items():
                w = res["bits"][hr][k]
                assert (torch.equal(v, w) if torch.is_tensor(v) else v == w), (name, k)


def _run_hook_lifetime(rank, world, port, out_dir):
    """A discarded or closed optimizer's gradient hooks do nothing."""
    import gc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE, _grad_ready

    mods = _make_modules()
    opt = ZeroFireFlyOptim(mods, lr=LR, weight_decay=WD, seed=SEED, update_fn=_oracle_update([], SEED),
                           bucket_mb=0.01)
    assert opt.overlap
    opt.close()
    for m, g in zip(mods, _grads(0)):
        _BIT_GRAD_CACHE[m._registered_handle] = g.clone()
        _grad_ready(m._registered_handle)
    assert opt._rs_order == []  # closed: no reduction started
    opt2 = ZeroFireFlyOptim(mods, lr=LR, weight_decay=WD, seed=SEED, update_fn=_oracle_update([], SEED),
                            bucket_mb=0.01)
    del opt2
    gc.collect()
    for m in mods:
        _grad_ready(m._registered_handle)  # the discarded optimizer's hooks are no-ops
    _BIT_GRAD_CACHE.clear()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_zero1_hooks_do_not_outlive_the_optimizer(tmp_path):
    mp.start_processes(_run_hook_lifetime, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")


def _run_uneven(rank, world, port, out_dir):
    """Three steps in which module 3 has no gradient on rank 1 at step 1 (as if it were not used
    in that rank's forward) while rank 0 has one.  On one rank the same steps see the average
    of the two ranks' gradients: module 3's gradient halved at step 1."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE, _grad_ready

    mods = _make_modules()
    opt = ZeroFireFlyOptim(mods, lr=LR, weight_decay=WD, seed=SEED, update_fn=_oracle_update([], SEED),
                           bucket_mb=0.01)
    for step in range(3):
        for i, (m, g) in reversed(list(enumerate(zip(mods, _grads(step))))):
            if step == 1 and i == 3:
                if world > 1 and rank == 1:
                    continue
                if world == 1:
                    g = g / 2  # exact in bf16
            _BIT_GRAD_CACHE[m._registered_handle] = g.clone()
            _grad_ready(m._registered_handle)
        opt.step()
    bits = opt.gather_bit_state()
    if rank == 0:
        torch.save({"q": [m.int_weight.clone() for m in mods], "bits": bits, "steps": list(opt.steps)},
                   os.path.join(out_dir, f"uneven{world}.pt"))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_zero1_module_without_gradient_on_one_rank(tmp_path):
    """A module with a gradient on rank 0 only is still updated on every rank with the averaged
    gradient, and its step count advances on all of them: the result equals one rank fed the
    averaged gradients (the reductions stay matched although rank 1 issues them from step())."""
    _run_uneven(0, 1, _free_port(), str(tmp_path))
    mp.start_processes(_run_uneven, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    one = torch.load(tmp_path / "uneven1.pt", weights_only=False)
    two = torch.load(tmp_path / "uneven2.pt", weights_only=False)
    assert one["steps"] == two["steps"] == [3, 3, 3, 3]
    for a, b in zip(one["q"], two["q"]):
        assert torch.equal(a, b)
    for h1, h2 in zip(sorted(one["bits"]), sorted(two["bits"])):
        for k, v in one["bits"][h1].items():
            w = two["bits"][h2][k]
            assert (torch.equal(v, w) if torch.is_tensor(v) else v == w), k

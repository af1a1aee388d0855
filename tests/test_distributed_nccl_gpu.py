"""ZeRO-1 data parallelism on real GPUs over NCCL (skipped with fewer than two GPUs).

Two ranks run a small BitLinear model on the same tokens, so their averaged gradients equal each
rank's own; the sharded, bucketed update must then give bit for bit the weights and the gathered
8-bit states of the same three steps on one GPU: the stochastic-rounding uniforms are keyed by the
global element index, not by the rank.  Both paths: the collectives (the DQT kernel on each rank's
slice, reduce-scatters issued from the backward, per-bucket all-gathers) and peer mode (one kernel
per slice reads both ranks' gradient arenas and writes both ranks' weight arenas over NVLink).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
SHAPES = [(256, 192), (128, 256), (96, 128)]  # (out, in): a chain 192 -> 256 -> 128 -> 96


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _train(rank, world, port, out_path, peer=False):
    import datetime

    import torch.distributed as dist

    from firefly_b200.bitLinear import BitLinear
    from firefly_b200.distributed import ZeroFireFlyOptim

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    if world > 1:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
    torch.manual_seed(0)
    mods = [BitLinear(k, o).to(dev) for o, k in SHAPES]
    # two buckets, so that a reduce-scatter starts from the backward before the last one
    opt = ZeroFireFlyOptim(mods, lr=1e-3, weight_decay=0.01, seed=5, bucket_mb=0.05, overlap=True,
                           peer=bool(peer) if world > 1 else None)
    assert opt.peer == (bool(peer) and world > 1)
    g = torch.Generator(device=dev).manual_seed(123)  # the same tokens on every rank
    for step in range(3):
        # the BitLinear weights are buffers: the input carries the autograd graph
        x = torch.randn(64, SHAPES[0][1], device=dev, generator=g).requires_grad_(True)
        y = mods[2](mods[1](mods[0](x)))
        y.float().pow(2).mean().backward()
        opt.step()
    bits = opt.gather_bit_state()
    opt.close()
    if rank == 0:
        torch.save({"q": [m.int_weight.cpu() for m in mods], "bits": bits, "buckets": len(opt.plan.buckets)},
                   out_path)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("peer", [False, True], ids=["collectives", "peer"])
def test_zero1_two_gpus_equal_one_gpu(tmp_path, peer):
    one, two = tmp_path / "one.pt", tmp_path / "two.pt"
    ctx = mp.get_context("spawn")  # a fresh process for each run (no CUDA state inherited)
    p = ctx.Process(target=_train, args=(0, 1, 0, str(one)))
    p.start()
    p.join(300)
    assert p.exitcode == 0
    mp.start_processes(_train, args=(2, _free_port(), str(two), peer), nprocs=2, start_method="spawn")
    a, b = torch.load(one, weights_only=False), torch.load(two, weights_only=False)
    assert b["buckets"] > 1
    for qa, qb in zip(a["q"], b["q"]):
        assert torch.equal(qa, qb)
    for ha, hb in zip(sorted(a["bits"]), sorted(b["bits"])):
        for k, v in a["bits"][ha].items():
            w = b["bits"][hb][k]
            assert (torch.equal(v, w) if torch.is_tensor(v) else v == w), k

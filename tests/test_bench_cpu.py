"""The benchmark's reference-side code on the CPU: the torch-eager comparator that bench.py times on
the GPU computes exactly what the pinned restatement of the reference (``oracle.ref_torch``, itself
equal to the reference's recorded outputs) computes, and the CPU baseline runs."""
import torch

import bench
from oracle import ref_torch as R


def _weights(o, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(o, k, generator=g) * 0.02
    s = w.abs().amax(dim=1).clamp_min(1e-8) / 127.0
    return torch.round(w / s.unsqueeze(1)).clamp(-127, 127).to(torch.int8), s


def test_eager_comparator_equals_reference_restatement():
    d, f, T = 64, 96, 32
    q_gu, s_gu = _weights(2 * f, d, 1)
    q_d, s_d = _weights(d, f, 2)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(T, d, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, d, generator=g).to(torch.bfloat16)
    # the restatement
    blk = R.SwiGLUBlock(q_gu.clone(), s_gu, q_d.clone(), s_d)
    xr = x.clone().requires_grad_(True)
    torch.manual_seed(11)
    for _ in range(2):
        yr = blk.train_step(xr, dy)
    # the comparator's pieces, assembled as reference_algorithm_on_gpu assembles them
    Fn = bench._EagerBitLinearFn.make()
    layers = [(q_gu.clone(), s_gu), (q_d.clone(), s_d)]
    states = []
    for q, _ in layers:
        z = torch.zeros(q.shape)
        mq, ma = bench._eager_codec(torch, z, True)
        vq, va = bench._eager_codec(torch, z, False)
        states.append({"t": 0, "m_q": mq, "m_a": ma, "v_q": vq, "v_a": va, "r_q": mq.clone(), "r_a": ma.clone()})
    cache = {}
    xe = x.clone().requires_grad_(True)
    torch.manual_seed(11)
    for _ in range(2):
        gu = Fn.apply(xe, *layers[0], cache, 0)
        ye = Fn.apply(torch.nn.functional.silu(gu[:, :f]) * gu[:, f:], *layers[1], cache, 1)
        ye.backward(dy)
        with torch.no_grad():
            for i, (q, sc) in enumerate(layers):
                bench._eager_dqt_step(torch, q, sc, cache.pop(i), states[i])
    assert torch.equal(yr, ye)
    assert torch.equal(xr.grad, xe.grad)
    for (qe, _), qr in zip(layers, (blk.q_gu, blk.q_d)):
        assert torch.equal(qe, qr)
    for se, sr in zip(states, blk.states):
        for ke, kr in (("m_q", "m_q"), ("m_a", "m_absmax"), ("v_q", "v_q"), ("v_a", "v_absmax"), ("r_q", "r_q"),
                       ("r_a", "r_absmax")):
            assert torch.equal(se[ke], sr[kr]), ke
        assert se["t"] == sr["step"] == 2


def test_cpu_reference_sample_runs():
    m = bench.RefCpuSample(64, 128, 32, slices=4, threads=1)
    m.step(record=False)
    m.step()
    assert m.fs == 32 and m.full_step_seconds() > 0
    assert "1/4 width slice" in m.describe()

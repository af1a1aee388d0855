"""Block-wise 8-bit AdamW of dense parameters (the reference's bitsandbytes AdamW8bit path).

bitsandbytes is absent, so parity is against the oracle's restatement of the published
algorithm with this build's map and rounding (``oracle.dense_adamw8_step``), not against
bitsandbytes itself: parity unpinned for this path.
"""
import numpy as np
import pytest
import torch

from firefly_b200.adamw8 import AdamW8bitDense, dynamic_qmap
from oracle import firefly_oracle as O

DEV = torch.device("cuda")


def test_dynamic_maps():
    for signed in (True, False):
        q = O.dynamic_qmap(signed)
        assert q.shape == (256,) and q.dtype == np.float32
        assert np.all(np.diff(q) >= 0)
        assert q[-1] == 1.0
        np.testing.assert_array_equal(q, dynamic_qmap(signed).numpy())
    qs, qu = O.dynamic_qmap(True), O.dynamic_qmap(False)
    np.testing.assert_array_equal(qs, -qs[::-1])  # symmetric
    assert qs[127] == qs[128] == 0.0 and qu[0] == 0.0 and qu[1] == np.float32(1e-7)
    # nearest-code encoding of the map's own values returns a code of the same value
    for q in (qs, qu):
        np.testing.assert_array_equal(q[O._nearest_codes(q, q)], q)


def test_oracle_zero_gradient_keeps_zero_state():
    st = O.init_dense_state(3000)
    p = np.ones(3000, np.float32)
    p2, st2 = O.dense_adamw8_step(p, np.zeros(3000, np.float32), st, lr=1e-3, wd=0.0)
    np.testing.assert_array_equal(p2, p)
    assert (st2["m_q"] == 128).all() and (st2["v_q"] == 0).all() and not st2["m_absmax"].any()


def _run_kernel_steps(n, pdt, steps=3, wd=0.01, seed=0):
    gen = torch.Generator().manual_seed(seed)
    p0 = (torch.randn(n, generator=gen) * 0.1).to(pdt)
    grads = [(torch.randn(n, generator=gen) * 1e-2) for _ in range(steps)]
    p = torch.nn.Parameter(p0.clone().to(DEV))
    opt = AdamW8bitDense([p], lr=1e-3, weight_decay=wd)
    pn = p0.float().numpy()
    st = O.init_dense_state(n)
    for g in grads:
        p.grad = g.to(DEV).to(pdt)
        opt.step()
        pn, st = O.dense_adamw8_step(pn, p.grad.float().cpu().numpy(), st, lr=1e-3, wd=wd)
        if pdt == torch.bfloat16:
            pn = O.round_bf16(pn)
    return p, opt.state[p], pn, st


@pytest.mark.gpu
@pytest.mark.parametrize("n,pdt", [(10000, torch.float32), (2048 * 3, torch.float32), (4097, torch.bfloat16),
                                   (50000, torch.bfloat16)])
def test_kernel_matches_oracle(n, pdt):
    p, st, pn, sto = _run_kernel_steps(n, pdt)
    np.testing.assert_array_equal(p.detach().float().cpu().numpy(), pn)
    for k in ("m_q", "v_q", "m_absmax", "v_absmax"):
        np.testing.assert_array_equal(st[k].cpu().numpy(), sto[k], err_msg=k)
    assert st["step"] == sto["step"] == 3


@pytest.mark.gpu
def test_small_params_keep_fp32_moments_and_checkpoint_roundtrip():
    big = torch.nn.Parameter(torch.randn(8192, device=DEV, dtype=torch.bfloat16))
    small = torch.nn.Parameter(torch.randn(100, device=DEV))
    opt = AdamW8bitDense([big, small], lr=1e-2, weight_decay=0.1)
    for _ in range(2):
        big.grad = torch.randn_like(big)
        small.grad = torch.randn_like(small)
        opt.step()
    assert set(opt.state[big]) == {"step", "m_q", "m_absmax", "v_q", "v_absmax"}
    assert opt.state[big]["m_absmax"].dtype == torch.float32
    assert set(opt.state[small]) == {"step", "exp_avg", "exp_avg_sq"}
    sd = opt.state_dict()
    opt2 = AdamW8bitDense([big, small], lr=1e-2, weight_decay=0.1)
    opt2.load_state_dict(sd)
    for k in ("m_q", "m_absmax", "v_q", "v_absmax"):
        assert torch.equal(opt2.state[big][k], opt.state[big][k]), k
    assert opt2.state[big]["m_absmax"].dtype == torch.float32  # not cast to the bf16 parameter's dtype


@pytest.mark.gpu
@pytest.mark.parametrize("wd", [0.0, 0.1])
def test_small_params_fused_step_equals_the_torch_chain(wd):
    """The small parameters' multi-tensor kernel (70 parameters: two launches) gives, bit for bit,
    the fp32-moment AdamW of torch ops (AdamW8bitDense._step_32bit), with fp32 and bf16
    parameters (gradients of the same dtype) and per-parameter step counts (one parameter
    skips a step)."""
    gen = torch.Generator().manual_seed(5)
    sizes = [int(s) for s in torch.randint(1, 4096, (70,), generator=gen)] + [4095, 1]
    dts = [torch.float32, torch.bfloat16]
    ps = [torch.nn.Parameter((torch.randn(n, generator=gen) * 0.1).to(dts[i % 2]).to(DEV))
          for i, n in enumerate(sizes)]
    ref = [torch.nn.Parameter(p.detach().clone()) for p in ps]
    opt = AdamW8bitDense(ps, lr=3e-3, betas=(0.9, 0.99), eps=1e-6, weight_decay=wd)
    states = [{} for _ in ref]
    for step in range(3):
        for i, (p, r) in enumerate(zip(ps, ref)):
            if step == 1 and i == 3:
                p.grad = r.grad = None
                continue
            g = torch.randn(p.shape, generator=gen).to(p.dtype).to(DEV)
            p.grad, r.grad = g, g.clone()
        opt.step()
        with torch.no_grad():
            for r, st in zip(ref, states):
                if r.grad is not None:
                    AdamW8bitDense._step_32bit(r, st, 3e-3, 0.9, 0.99, 1e-6, wd)
    for i, (p, r, st) in enumerate(zip(ps, ref, states)):
        assert opt.state[p]["step"] == st["step"] == (2 if i == 3 else 3)
        assert torch.equal(p.detach(), r.detach()), i
        assert torch.equal(opt.state[p]["exp_avg"], st["exp_avg"]), i
        assert torch.equal(opt.state[p]["exp_avg_sq"], st["exp_avg_sq"]), i
    # checkpoint round trip keeps the fp32 moments of bf16 parameters in fp32
    opt2 = AdamW8bitDense(ps, lr=3e-3, betas=(0.9, 0.99), eps=1e-6, weight_decay=wd)
    opt2.load_state_dict(opt.state_dict())
    assert opt2.state[ps[1]]["exp_avg"].dtype == torch.float32
    assert torch.equal(opt2.state[ps[1]]["exp_avg_sq"], opt.state[ps[1]]["exp_avg_sq"])


def _encode_probe_grads(n, seed=0):
    """Gradients whose values hit every map entry, every midpoint between neighbours and the
    floats just either side of both, with 1.0 first in each block (so the block absmax of m is
    1 and m * (1/absmax) = g when beta1 = 0)."""
    qs = O.dynamic_qmap(True)
    mids = ((qs[:-1].astype(np.float64) + qs[1:]) / 2).astype(np.float32)
    pts = np.concatenate([qs, mids])
    pts = np.concatenate([pts, np.nextafter(pts, np.float32(2)), np.nextafter(pts, np.float32(-2))])
    pts = pts[np.abs(pts) <= 1].astype(np.float32)
    rng = np.random.default_rng(seed)
    rest = n - pts.size
    extra = (rng.choice([-1, 1], rest) * 10.0 ** rng.uniform(-9, 0, rest)).astype(np.float32)
    g = np.concatenate([pts, extra]).astype(np.float32)
    rng.shuffle(g)
    g[::2048] = 1.0
    return g


@pytest.mark.gpu
@pytest.mark.parametrize("betas", [(0.0, 0.0), (0.9, 0.999)])
def test_codes_at_map_points_and_midpoints(betas):
    n = 2048 * 8
    g = _encode_probe_grads(n)
    p = torch.nn.Parameter(torch.zeros(n, device=DEV))
    opt = AdamW8bitDense([p], lr=1e-3, betas=betas, weight_decay=0.0)
    p.grad = torch.from_numpy(g).to(DEV)
    opt.step()
    pn, sto = O.dense_adamw8_step(np.zeros(n, np.float32), g, O.init_dense_state(n), lr=1e-3, beta1=betas[0],
                                  beta2=betas[1], wd=0.0)
    st = opt.state[p]
    for k in ("m_q", "v_q", "m_absmax", "v_absmax"):
        np.testing.assert_array_equal(st[k].cpu().numpy(), sto[k], err_msg=k)
    np.testing.assert_array_equal(p.detach().cpu().numpy(), pn)
    if betas[0] == 0.0:  # m = g: its codes are the nearest entries of g itself
        np.testing.assert_array_equal(st["m_q"].cpu().numpy(), O._nearest_codes(g, O.dynamic_qmap(True)))


@pytest.mark.gpu
def test_maps_without_bucket_property_take_the_search_path():
    # a linear signed map has no zero entry and a dense unsigned one puts two entries in one
    # bucket: the kernel must fall back to the binary search and still match the oracle
    from firefly_b200 import _capi

    qs = np.linspace(-1, 1, 256).astype(np.float32)
    qu = np.concatenate([[0.0], np.sort(np.random.default_rng(1).uniform(0.999, 1.0, 254)), [1.0]]).astype(np.float32)
    n = 2048 * 3 + 100
    rng = np.random.default_rng(2)
    g = (rng.standard_normal(n) * 1e-2).astype(np.float32)
    p0 = (rng.standard_normal(n) * 0.1).astype(np.float32)
    st = O.init_dense_state(n)
    st["m_q"][:] = 100
    st["m_absmax"][:] = 1e-2
    st["v_q"][:] = 7
    st["v_absmax"][:] = 1e-5
    pn, sto = O.dense_adamw8_step(p0, g, st, lr=1e-3, wd=0.01, qmaps=(qs, qu))
    p = torch.from_numpy(p0).to(DEV)
    m_q, v_q = torch.from_numpy(st["m_q"]).to(DEV), torch.from_numpy(st["v_q"]).to(DEV)
    m_a, v_a = torch.from_numpy(st["m_absmax"]).to(DEV), torch.from_numpy(st["v_absmax"]).to(DEV)
    _capi.adamw8_blockwise(p, torch.from_numpy(g).to(DEV), m_q, m_a, v_q, v_a, lr=1e-3, beta1=0.9, beta2=0.999,
                           eps=1e-8, wd=0.01, step=1, qmap_s=torch.from_numpy(qs).to(DEV),
                           qmap_u=torch.from_numpy(qu).to(DEV))
    np.testing.assert_array_equal(p.cpu().numpy(), pn)
    np.testing.assert_array_equal(m_q.cpu().numpy(), sto["m_q"])
    np.testing.assert_array_equal(v_q.cpu().numpy(), sto["v_q"])
    np.testing.assert_array_equal(m_a.cpu().numpy(), sto["m_absmax"])

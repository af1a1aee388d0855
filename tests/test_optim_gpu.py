"""Fused DQT 8-bit AdamW kernel against the oracle (and the reference's recorded steps).

Bar: int8 weights and 8-bit codes differ by at most one LSB on at most 0.1% of elements
(``tests._util.check_optim_step``), with the same uniforms fed to both sides."""
import numpy as np
import pytest
import torch

import firefly_b200 as ff
from firefly_b200 import _capi
from firefly_b200.fireflyoptim import _tables_on, init_bit_state
from oracle import firefly_oracle as O
from tests._util import check_optim_step, from_bf16_bits, load_golden

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
KEYS = ("m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax")


def _run_kernel(q, ws, g_bits, st, *, lr, b1, b2, eps, wd, sr, u=None, seed=0, rng_offset=0, elem_base=0,
                row_len=None):
    qd = torch.from_numpy(np.ascontiguousarray(q)).to(DEV)
    sd = {k: torch.from_numpy(np.ascontiguousarray(st[k])).to(DEV) for k in KEYS}
    gd = from_bf16_bits(g_bits, DEV).contiguous()
    dec_s, dec_u = _tables_on(DEV)
    _capi.dqt_adamw8(
        qd, torch.from_numpy(np.ascontiguousarray(ws)).to(DEV), row_len or q.shape[-1], gd,
        sd["m_q"], sd["m_absmax"], sd["v_q"], sd["v_absmax"], sd["r_q"], sd["r_absmax"],
        lr=lr, beta1=b1, beta2=b2, eps=eps, wd=wd, step=int(st["step"]) + 1, sr_bias=sr, seed=seed,
        rng_offset=rng_offset, elem_base=elem_base,
        u=None if u is None else torch.from_numpy(np.ascontiguousarray(u, np.float32)).to(DEV),
        dec_s=dec_s, dec_u=dec_u,
    )
    return qd.cpu().numpy(), {k: v.cpu().numpy() for k, v in sd.items()}


@pytest.mark.parametrize("case", ["cfg1like", "ragged", "defaultwd", "unbiased", "bigstep"])
def test_kernel_replays_reference_steps(case):
    z = load_golden("optim_step.npz")
    O_, K, bs = (int(v) for v in z[case + "_meta"])
    lr, b1, b2, eps, wd, sr = (float(v) for v in z[case + "_hyper"])
    ws = z[case + "_ws"]
    q = z[case + "_q0"]
    st = O.init_state((O_, K), bs)
    rows = np.nonzero(ws > eps)[0]
    for s in range(3):
        u = z[f"{case}_s{s}_u"]
        qg, stg = _run_kernel(q, ws, z[f"{case}_s{s}_g"], st, lr=lr, b1=b1, b2=b2, eps=eps, wd=wd, sr=sr, u=u)
        want = {k: z[f"{case}_s{s}_{k}"] for k in KEYS}
        # against the reference's recorded step (well-conditioned rows, see test_oracle_golden)
        sub = lambda d: {k: (d[k][rows] if d[k].shape == (O_, K) else d[k]) for k in KEYS}
        check_optim_step(qg[rows], sub(stg), z[f"{case}_s{s}_q"][rows], sub(want), f"{case} s{s} vs ref")
        # against the oracle on every element
        qo, sto = O.dqt_adamw8_step(q, ws, O.bf16_bits_to_f32(z[f"{case}_s{s}_g"]), st, lr=lr, beta1=b1,
                                    beta2=b2, eps=eps, wd=wd, sr_bias=sr, bs=bs, u=u)
        check_optim_step(qg[rows], sub(stg), qo[rows], sub(sto), f"{case} s{s} vs oracle")
        q = z[f"{case}_s{s}_q"]
        st = {"step": s + 1, **want}


def _random_case(O_, K, seed, steps_done=5):
    rng = np.random.default_rng(seed)
    q, ws = O.quantize_rows(rng.standard_normal((O_, K)).astype(np.float32) * 0.02)
    # states from a few oracle steps so that codes are spread out
    st = O.init_state((O_, K))
    for t in range(steps_done):
        g = O.round_bf16(rng.standard_normal((O_, K)).astype(np.float32) * 1e-3)
        u = rng.random((O_, K), dtype=np.float32)
        q, st = O.dqt_adamw8_step(q, ws, g, st, lr=1e-3, wd=0.01, u=u)
    g_bits = O.f32_to_bf16_bits(rng.standard_normal((O_, K)).astype(np.float32) * 1e-3)
    return q, ws, g_bits, st, rng


@pytest.mark.parametrize("O_,K", [(1024, 1024), (33, 70), (3, 5), (257, 1000)])
def test_kernel_matches_oracle_supplied_uniforms(O_, K):
    q, ws, g_bits, st, rng = _random_case(O_, K, seed=O_ + K)
    u = rng.random((O_, K), dtype=np.float32)
    for sr in (0.15, 0.0):
        qg, stg = _run_kernel(q, ws, g_bits, st, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, sr=sr, u=u)
        qo, sto = O.dqt_adamw8_step(q, ws, O.bf16_bits_to_f32(g_bits), st, lr=1e-3, wd=0.01, sr_bias=sr, u=u)
        check_optim_step(qg, stg, qo, sto, f"{O_}x{K} sr={sr}")


def test_kernel_philox_uniforms_match_oracle():
    O_, K = 96, 512
    q, ws, g_bits, st, _ = _random_case(O_, K, seed=3)
    seed, off = 123456789012345, 4096
    qg, stg = _run_kernel(q, ws, g_bits, st, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, sr=0.15,
                          seed=seed, rng_offset=off)
    u = O.philox_uniforms(O_ * K, seed=seed, step=int(st["step"]) + 1, elem_offset=off).reshape(O_, K)
    qo, sto = O.dqt_adamw8_step(q, ws, O.bf16_bits_to_f32(g_bits), st, lr=1e-3, wd=0.01, sr_bias=0.15, u=u)
    check_optim_step(qg, stg, qo, sto, "philox")


def test_sharded_update_equals_whole_update():
    """ZeRO-1 split: updating block-aligned shards separately (elem_base/rng_offset set)
    gives exactly the whole-tensor result."""
    O_, K = 64, 384
    q, ws, g_bits, st, _ = _random_case(O_, K, seed=4)
    whole_q, whole_st = _run_kernel(q, ws, g_bits, st, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, sr=0.15,
                                    seed=9, rng_offset=1024)
    n = O_ * K
    cut = 256 * 37
    parts = []
    for lo, hi in ((0, cut), (cut, n)):
        sub_st = {"step": st["step"]}
        for k in ("m_q", "v_q", "r_q"):
            sub_st[k] = st[k].ravel()[lo:hi]
        for k in ("m_absmax", "v_absmax", "r_absmax"):
            sub_st[k] = st[k][lo // 256:(hi + 255) // 256]
        qg, stg = _run_kernel(q.ravel()[lo:hi], ws, g_bits.ravel()[lo:hi], sub_st, lr=1e-3, b1=0.9, b2=0.999,
                              eps=1e-8, wd=0.01, sr=0.15, seed=9, rng_offset=1024 + lo, elem_base=lo, row_len=K)
        parts.append((qg, stg))
    np.testing.assert_array_equal(np.concatenate([p[0] for p in parts]), whole_q.ravel())
    for k in ("m_q", "v_q", "r_q"):
        np.testing.assert_array_equal(np.concatenate([p[1][k] for p in parts]), whole_st[k].ravel())
    for k in ("m_absmax", "v_absmax", "r_absmax"):
        np.testing.assert_array_equal(np.concatenate([p[1][k] for p in parts]), whole_st[k])


def test_fireflyoptim_module_step_against_oracle():
    torch.manual_seed(0)
    layer = ff.BitLinear(300, 70).to(DEV)
    dense = torch.nn.Parameter(torch.zeros(4, device=DEV))
    opt = ff.FireFlyOptim([dense], lr=1e-3, weight_decay=0.01, bit_modules=[layer])
    rng = np.random.default_rng(0)
    q = layer.int_weight.cpu().numpy()
    ws = layer.weight_scale.cpu().numpy()
    st = O.init_state(q.shape)
    us = {}
    opt.uniform_source = lambda m, h, t: torch.from_numpy(us[t])
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE
    h = layer._registered_handle
    for t in range(1, 4):
        g_bits = O.f32_to_bf16_bits(rng.standard_normal(q.shape).astype(np.float32) * 1e-2)
        us[t] = rng.random(q.shape, dtype=np.float32)
        _BIT_GRAD_CACHE[h] = from_bf16_bits(g_bits, DEV)
        dense.grad = torch.ones_like(dense)
        opt.step()
        q_o, st = O.dqt_adamw8_step(q, ws, O.bf16_bits_to_f32(g_bits), st, lr=1e-3, wd=0.01, u=us[t])
        got = {k: v.cpu().numpy() for k, v in opt._bit_state[h].items() if torch.is_tensor(v)}
        check_optim_step(layer.int_weight.cpu().numpy(), got, q_o, st, f"module step {t}")
        # continue both from the kernel's state so differences do not compound
        q = layer.int_weight.cpu().numpy()
        st = {"step": t, **got}
        assert opt._bit_state[h]["step"] == t
    assert _BIT_GRAD_CACHE.get(h) is None  # consumed
    # dense params were stepped
    assert not torch.equal(dense, torch.zeros_like(dense))


def test_state_dict_roundtrip_and_format():
    layer = ff.BitLinear(64, 32).to(DEV)
    opt = ff.FireFlyOptim([torch.nn.Parameter(torch.zeros(1, device=DEV))], bit_modules=[layer])
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE
    _BIT_GRAD_CACHE[layer._registered_handle] = torch.randn(32, 64, device=DEV).to(torch.bfloat16)
    opt.step()
    sd = opt.state_dict()
    bs = sd["bit_state"][layer._registered_handle]
    assert set(bs) == {"step", "m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax"}
    assert bs["m_q"].dtype == torch.uint8 and bs["m_q"].shape == (32, 64) and bs["m_q"].device.type == "cpu"
    assert bs["m_absmax"].shape == (8,) and bs["m_absmax"].dtype == torch.float32
    opt2 = ff.FireFlyOptim([torch.nn.Parameter(torch.zeros(1, device=DEV))], bit_modules=[layer])
    opt2.load_state_dict(sd)
    for k, v in bs.items():
        if torch.is_tensor(v):
            assert torch.equal(opt2._bit_state[layer._registered_handle][k], v)
    assert opt2.rng_seed == opt.rng_seed
    # the loaded (CPU) state is moved to the module's device on the next step
    _BIT_GRAD_CACHE[layer._registered_handle] = torch.randn(32, 64, device=DEV).to(torch.bfloat16)
    opt2.step()
    assert opt2._bit_state[layer._registered_handle]["m_q"].is_cuda


def test_zero_state_matches_reference_encoding():
    st = init_bit_state((5, 100), DEV)
    o = O.init_state((5, 100))
    for k in KEYS:
        np.testing.assert_array_equal(st[k].cpu().numpy(), o[k])


@pytest.mark.parametrize("O_,K,nsrc,offset", [(64, 512, 2, 0), (33, 70, 3, 0), (40, 96, 2, 8), (8, 1024, 8, 0)])
def test_multi_source_update_equals_update_on_the_averaged_gradient(O_, K, nsrc, offset):
    """ff_dqt_adamw8_peers with every source and destination on this GPU (stand-ins for the other
    ranks' arenas): the same result as ff_dqt_adamw8 on the gradient averaged the way the kernel
    defines it (fp32 sums in source order, times 1/nsrc, rounded to bf16), the new weights in every
    destination, the averaged gradient in g_out.  offset 8 makes the arrays 8-byte but not 16-byte
    aligned (no bulk staging: the per-element path); 33 x 70 ends in a ragged block."""
    q, ws, _, st, rng = _random_case(O_, K, seed=O_ * K + nsrc)
    n = O_ * K
    grads = [torch.from_numpy(rng.standard_normal(n).astype(np.float32) * 1e-3).to(DEV).to(torch.bfloat16)
             for _ in range(nsrc)]
    acc = grads[0].float()
    for g in grads[1:]:
        acc = acc + g.float()
    g_avg = (acc * torch.tensor(1.0 / nsrc, dtype=torch.float32, device=DEV)).to(torch.bfloat16)
    dec_s, dec_u = _tables_on(DEV)
    wsd = torch.from_numpy(np.ascontiguousarray(ws)).to(DEV)
    kw = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01, step=int(st["step"]) + 1, sr_bias=0.15,
              seed=77, rng_offset=512, dec_s=dec_s, dec_u=dec_u)

    def arrays(extra):  # q and the states, each starting `extra` bytes into a larger buffer
        def put(a, dtype):
            t = torch.from_numpy(np.ascontiguousarray(a).ravel()).to(DEV)
            buf = torch.zeros(t.numel() * t.element_size() + 64, dtype=torch.uint8, device=DEV)
            v = buf[extra:extra + t.numel() * t.element_size()].view(dtype)
            v.copy_(t.view(dtype))
            return v
        out = {"q": put(q, torch.int8)}
        for k in KEYS:
            out[k] = put(st[k], torch.float32 if "absmax" in k else torch.uint8)
        return out

    ref = arrays(0)
    _capi.dqt_adamw8(ref["q"], wsd, K, g_avg, ref["m_q"], ref["m_absmax"], ref["v_q"], ref["v_absmax"], ref["r_q"],
                     ref["r_absmax"], **kw)
    got = arrays(offset)
    q2 = torch.zeros_like(got["q"])  # a second rank's copy of the weights
    gsrc = []
    for g in grads:
        buf = torch.zeros(n * 2 + 64, dtype=torch.uint8, device=DEV)
        v = buf[16:16 + 2 * n].view(torch.bfloat16)
        v.copy_(g)
        gsrc.append(v)
    g_out = torch.empty(n, dtype=torch.bfloat16, device=DEV)
    _capi.dqt_adamw8_peers(got["q"], wsd, K, [t.data_ptr() for t in gsrc], [got["q"].data_ptr(), q2.data_ptr()],
                           got["m_q"], got["m_absmax"], got["v_q"], got["v_absmax"], got["r_q"], got["r_absmax"],
                           g_out=g_out, **kw)
    torch.cuda.synchronize()
    assert _capi.device_status() == 0
    assert torch.equal(g_out, g_avg)
    assert torch.equal(got["q"], ref["q"])
    assert torch.equal(q2, ref["q"])
    for k in KEYS:
        assert torch.equal(got[k], ref[k]), k


def test_multi_source_argument_checks():
    q = torch.zeros(256, dtype=torch.int8, device=DEV)
    st = {k: torch.zeros(256 if k.endswith("_q") else 1, dtype=torch.uint8 if k.endswith("_q") else torch.float32,
                         device=DEV) for k in KEYS}
    dec_s, dec_u = _tables_on(DEV)
    g = torch.zeros(256, dtype=torch.bfloat16, device=DEV)
    kw = dict(lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01, step=1, sr_bias=0.15, seed=1, dec_s=dec_s,
              dec_u=dec_u)
    args = (torch.ones(1, device=DEV), 256)
    states = (st["m_q"], st["m_absmax"], st["v_q"], st["v_absmax"], st["r_q"], st["r_absmax"])
    with pytest.raises(ValueError):  # q must be among the destinations
        _capi.dqt_adamw8_peers(q, *args, [g.data_ptr()], [g.data_ptr()], *states, **kw)
    with pytest.raises(ValueError):  # at most 8 sources
        _capi.dqt_adamw8_peers(q, *args, [g.data_ptr()] * 9, [q.data_ptr()], *states, **kw)
    with pytest.raises(ValueError):  # sources 16-byte aligned (checked by the library)
        _capi.dqt_adamw8_peers(q, *args, [g.data_ptr() + 2], [q.data_ptr()], *states, **kw)

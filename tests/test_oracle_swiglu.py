"""The oracle's SwiGLU formulas against torch's CPU bf16 ops (no GPU).

The reference has no model code, so the SwiGLU block's elementwise math is pinned to
torch itself: ``F.silu(g) * u`` and its autograd gradients on bf16 CPU tensors.
torch's CPU exp is vectorised (within about an ulp of the correctly rounded value
the oracle uses), so a bf16 result may differ by one step on a small fraction of
elements; the GPU tests pin the CUDA kernels to torch's CUDA ops exactly.
"""
import numpy as np
import torch
from torch.nn import functional as F

from oracle import firefly_oracle as O
from tests._util import bf16_bits, bf16_ulp_diff


def test_oracle_swiglu_matches_torch_cpu():
    gen = torch.Generator().manual_seed(0)
    T, Fh = 256, 384
    gu = (torch.randn(T, 2 * Fh, generator=gen) * 4).to(torch.bfloat16).requires_grad_(True)
    dh = torch.randn(T, Fh, generator=gen).to(torch.bfloat16)
    g, u = gu.chunk(2, dim=1)
    h = F.silu(g) * u
    h.backward(dh)
    gf, uf, dhf = (O.bf16_bits_to_f32(bf16_bits(t)) for t in (g, u, dh))
    h_o = O.f32_to_bf16_bits(O.swiglu_forward(gf, uf))
    dg_o, du_o = (O.f32_to_bf16_bits(a) for a in O.swiglu_backward(dhf, gf, uf))
    for what, got, want in (("h", bf16_bits(h), h_o), ("dg", bf16_bits(gu.grad[:, :Fh]), dg_o),
                            ("du", bf16_bits(gu.grad[:, Fh:]), du_o)):
        d = bf16_ulp_diff(got, want)
        assert d.max() <= 1, what
        assert (d > 0).mean() <= 5e-3, f"{what}: {(d > 0).mean():.2e} of elements differ"


def test_oracle_swiglu_mlp_step_shapes_and_consistency():
    rng = np.random.default_rng(1)
    T, d, f = 8, 32, 16
    q_gu, s_gu = O.quantize_rows(rng.standard_normal((2 * f, d)).astype(np.float32) * 0.02)
    q_d, s_d = O.quantize_rows(rng.standard_normal((d, f)).astype(np.float32) * 0.02)
    x = rng.standard_normal((T, d)).astype(np.float32)
    dy = O.f32_to_bf16_bits(rng.standard_normal((T, d)).astype(np.float32))
    out = O.swiglu_mlp_step(x, dy, q_gu, s_gu, q_d, s_d)
    assert out["y"].shape == (T, d) and out["dx"].shape == (T, d)
    assert out["gw_gu"].shape == (2 * f, d) and out["gw_d"].shape == (d, f)
    # the down projection's input is h = swiglu(g, u) quantised per row
    gu = O.bf16_bits_to_f32(out["gu"])
    q_h, s_h = O.quantize_rows(O.swiglu_forward(gu[:, :f], gu[:, f:]))
    np.testing.assert_array_equal(q_h, out["q_h"])
    np.testing.assert_array_equal(s_h, out["s_h"])

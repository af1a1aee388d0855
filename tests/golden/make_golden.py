"""Generate the golden fixtures in this folder by running the FireFly reference.

The reference is the pure-PyTorch package fumitoshi0524/FireFly (files
``fireflykernels.py``, ``bitLinear.py``, ``fireflyoptim.py``).  This script
imports it from a local checkout whose folder is given as the first argument
(or by the ``FIREFLY_REFERENCE`` environment variable), runs its CPU path on
small seeded inputs and stores inputs and outputs as ``.npz`` files next to this
script.  Nothing else in the repository reads the reference; the parity tests
only read the fixtures.

``fireflyoptim.py:2`` imports ``bitsandbytes.optim.AdamW8bit`` at module import
time.  bitsandbytes is not installed here, so a stand-in module whose
``AdamW8bit`` is ``torch.optim.AdamW`` is registered first.  It only affects
dense (non-BitLinear) parameters; the fixtures pass a single dummy dense
parameter, and the BitLinear branch (``fireflyoptim.py:126-209``) is pure torch.

``torch.rand_like`` draws of the optimizer step (``fireflyoptim.py:192``) are
recorded so that a replay can feed the same uniforms.

Run:  python tests/golden/make_golden.py <reference checkout>
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference(path: str | None):
    path = path or os.environ.get("FIREFLY_REFERENCE")
    if not path:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set FIREFLY_REFERENCE)")
    ref_dir = Path(path).resolve()
    if not (ref_dir / "fireflyoptim.py").exists():
        raise SystemExit(f"reference checkout not found at {ref_dir}")
    bnb = types.ModuleType("bitsandbytes")
    bnb_optim = types.ModuleType("bitsandbytes.optim")

    class AdamW8bit(torch.optim.AdamW):  # stand-in for dense params only
        pass

    bnb_optim.AdamW8bit = AdamW8bit
    bnb.optim = bnb_optim
    sys.modules.setdefault("bitsandbytes", bnb)
    sys.modules.setdefault("bitsandbytes.optim", bnb_optim)
    sys.path.insert(0, str(ref_dir.parent))
    import importlib

    pkg = importlib.import_module(ref_dir.name)
    fk = importlib.import_module(ref_dir.name + ".fireflykernels")
    fo = importlib.import_module(ref_dir.name + ".fireflyoptim")
    bl = importlib.import_module(ref_dir.name + ".bitLinear")
    # the fireflykernels bitsandbytes import is guarded; it must have failed,
    # because the stand-in has no ``functional`` submodule
    assert fk._BNB_F is None
    return pkg, fk, fo, bl


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


def gen_quant(fk) -> None:
    """``quantize_fp_to_int8`` (fireflykernels.py:96-104) on edge-case inputs."""
    g = torch.Generator().manual_seed(1234)
    cases = {}
    # plain normal rows, odd sizes
    cases["normal"] = torch.randn(37, 301, generator=g)
    # rows with zeros, a single non-zero, huge and tiny magnitudes
    w = torch.randn(9, 64, generator=g)
    w[0] = 0.0
    w[1] = 0.0
    w[1, 5] = -3.0
    w[2] *= 1e30
    w[3] *= 1e-30
    w[4] *= 1e-9
    cases["edges"] = w
    # exact .5 ties after division: row absmax 127 -> scale 1.0
    t = torch.zeros(4, 32)
    t[:, 0] = 127.0
    t[0, 1:17] = torch.arange(16) + 0.5
    t[1, 1:17] = -(torch.arange(16) + 0.5)
    t[2, 1:] = torch.linspace(-126.5, 126.5, 31)
    t[3, 1:] = torch.linspace(-2.5, 2.5, 31)
    cases["ties"] = t
    # bf16 input (BitLinear activations are often bf16)
    cases["bf16"] = (torch.randn(16, 96, generator=g) * 4).to(torch.bfloat16)
    # one column only
    cases["onecol"] = torch.randn(7, 1, generator=g)
    out = {}
    for name, x in cases.items():
        q, s = fk.quantize_fp_to_int8(x)
        out[f"{name}_x"] = x.float().numpy()
        out[f"{name}_q"] = q.numpy()
        out[f"{name}_s"] = s.numpy()
        out[f"{name}_isbf16"] = np.array(x.dtype == torch.bfloat16)
    # the same quantiser with a non-default eps
    x = torch.randn(5, 40, generator=g) * 1e-6
    q, s = fk.quantize_fp_to_int8(x, eps=1e-5)
    out["eps_x"], out["eps_q"], out["eps_s"] = x.numpy(), q.numpy(), s.numpy()
    out["eps_isbf16"] = np.array(False)
    np.savez_compressed(HERE / "quant_rows.npz", **out)


def gen_mulaw(fo) -> None:
    """mu-law blockwise codecs (fireflyoptim.py:22-80)."""
    g = torch.Generator().manual_seed(99)
    out = {}
    for name, n, bs in (("a", 1000, 256), ("b", 512, 256), ("c", 300, 128), ("d", 7, 256)):
        x = torch.randn(n, generator=g) * 0.01
        if name == "a":
            x[256:512] = 0.0  # an all-zero block
            x[600] = 5.0  # an outlier
        qs, as_ = fo._quantize_blockwise_signed(x, bs)
        y = x * x
        qu, au = fo._quantize_blockwise_unsigned(y, bs)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_bs"] = np.array(bs)
        out[f"{name}_qs"] = qs.numpy()
        out[f"{name}_as"] = as_.numpy()
        out[f"{name}_qu"] = qu.numpy()
        out[f"{name}_au"] = au.numpy()
        out[f"{name}_ds"] = fo._dequantize_blockwise_signed(qs, as_, bs, x.shape).numpy()
        out[f"{name}_du"] = fo._dequantize_blockwise_unsigned(qu, au, bs, y.shape).numpy()
    # every code decoded with absmax 1 (the decode tables)
    codes = torch.arange(256, dtype=torch.uint8)
    one = torch.ones(1)
    out["table_signed"] = fo._dequantize_blockwise_signed(codes, one, 256, codes.shape).numpy()
    out["table_unsigned"] = fo._dequantize_blockwise_unsigned(codes, one, 256, codes.shape).numpy()
    np.savez_compressed(HERE / "mulaw.npz", **out)


class _RandRecorder:
    """Wraps ``torch.rand_like`` and keeps every draw."""

    def __init__(self):
        self.draws = []
        self._orig = torch.rand_like

    def __enter__(self):
        def rec(t, *a, **k):
            u = self._orig(t, *a, **k)
            self.draws.append(u.clone())
            return u

        torch.rand_like = rec
        return self

    def __exit__(self, *exc):
        torch.rand_like = self._orig


def gen_optim(pkg, fk, fo) -> None:
    """Three ``FireFlyOptim.step`` calls per case (fireflyoptim.py:122-211).

    Each step: a bf16 weight gradient is placed in the reference's grad cache
    (the same object ``Int8LinearFn.backward`` fills, fireflykernels.py:193-198),
    then ``step()`` runs.  Recorded per step: the gradient, the uniforms drawn,
    and the module's int8 weight plus all 8-bit states afterwards.
    """
    cases = [
        # name, O, K, lr, wd, sr_bias, seed, grad std
        ("cfg1like", 48, 80, 1e-3, 0.01, 0.15, 0, 1e-1),
        ("ragged", 33, 70, 1e-3, 0.01, 0.15, 1, 1e-1),
        ("defaultwd", 16, 256, 1e-3, 0.1, 0.15, 2, 1e-3),
        ("unbiased", 24, 100, 5e-3, 0.01, 0.0, 3, 1.0),
        ("bigstep", 8, 512, 5e-2, 0.01, 0.15, 4, 1.0),
    ]
    out = {}
    for name, O, K, lr, wd, sr, seed, gstd in cases:
        torch.manual_seed(seed)
        layer = pkg.BitLinear(K, O)
        w = torch.randn(O, K) * 0.02
        q, s = fk.quantize_fp_to_int8(w)
        layer.int_weight.copy_(q)
        layer.weight_scale.copy_(s)
        if name == "ragged":
            layer.weight_scale[3] = 0.0  # exercises clamp_min(eps) (fireflyoptim.py:180)
            layer.int_weight[5, :] = 127  # exercises the +-127 clamp
            layer.int_weight[6, :] = -127
        dense = torch.nn.Parameter(torch.zeros(1))
        opt = fo.FireFlyOptim(
            [dense], lr=lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=wd,
            bit_modules=[layer], block_size=256, sr_bias_scale=sr,
        )
        h = int(layer._bit_handle.item())
        out[f"{name}_meta"] = np.array([O, K, 256], dtype=np.int64)
        out[f"{name}_hyper"] = np.array([lr, 0.9, 0.999, 1e-8, wd, sr], dtype=np.float64)
        out[f"{name}_q0"] = layer.int_weight.numpy().copy()
        out[f"{name}_ws"] = layer.weight_scale.numpy().copy()
        gen = torch.Generator().manual_seed(100 + seed)
        for step in range(3):
            grad = (torch.randn(O, K, generator=gen) * gstd).to(torch.bfloat16)
            if step == 2 and name == "ragged":
                grad[0] = 0.0  # an all-zero gradient row
            fk._BIT_GRAD_CACHE[h] = grad.clone()
            with _RandRecorder() as rec:
                opt.step()
            assert len(rec.draws) == 1
            st = opt._bit_state[h]
            out[f"{name}_s{step}_g"] = _bf16_bits(grad)
            out[f"{name}_s{step}_u"] = rec.draws[0].numpy()
            out[f"{name}_s{step}_q"] = layer.int_weight.numpy().copy()
            for key in ("m_q", "m_absmax", "v_q", "v_absmax", "r_q", "r_absmax"):
                out[f"{name}_s{step}_{key}"] = st[key].numpy().copy()
            assert st["step"] == step + 1
    np.savez_compressed(HERE / "optim_step.npz", **out)


def gen_linear(pkg, fk) -> None:
    """The live bf16 forward/backward (fireflykernels.py:164-210) on small inputs.

    Not a parity target for the int8 path; used to report how far the int8
    path is from the reference's bf16 numerics, and to pin API behaviour
    (output dtype, grad dtype, grad-cache accumulation).
    """
    out = {}
    for name, T, K, O, bias, xdt in (
        ("fp32", 64, 96, 80, False, torch.float32),
        ("bias_bf16", 48, 64, 32, True, torch.bfloat16),
    ):
        torch.manual_seed(7)
        layer = pkg.BitLinear(K, O, bias=bias)
        w = torch.randn(O, K) * 0.02
        q, s = fk.quantize_fp_to_int8(w)
        layer.int_weight.copy_(q)
        layer.weight_scale.copy_(s)
        if bias:
            with torch.no_grad():
                layer.bias.copy_(torch.randn(O) * 0.1)
        x = torch.randn(T, K).to(xdt).requires_grad_(True)
        y = layer(x)
        dy = torch.randn_like(y)
        y.backward(dy)
        # second backward accumulates into the grad cache (fireflykernels.py:197-198)
        y2 = layer(x)
        y2.backward(dy)
        gw = layer.consume_weight_grad()
        out[f"{name}_x"] = x.detach().float().numpy()
        out[f"{name}_xisbf16"] = np.array(xdt == torch.bfloat16)
        out[f"{name}_q"] = q.numpy()
        out[f"{name}_s"] = s.numpy()
        out[f"{name}_bias"] = layer.bias.detach().numpy() if bias else np.zeros(0, np.float32)
        out[f"{name}_y"] = _bf16_bits(y)
        out[f"{name}_dy"] = _bf16_bits(dy)
        out[f"{name}_dx"] = x.grad.float().numpy()
        out[f"{name}_dxdtype"] = np.array(str(x.grad.dtype))
        out[f"{name}_gw2"] = _bf16_bits(gw)
        if bias:
            out[f"{name}_db2"] = layer.bias.grad.numpy()
    np.savez_compressed(HERE / "linear_bf16.npz", **out)


def gen_init(pkg) -> None:
    """``BitLinear(K, O)`` construction under ``torch.manual_seed`` (bitLinear.py:15-27, :40-66):
    the Kaiming-uniform draw from torch's default CPU generator, quantised per row."""
    out = {}
    cases = [("sq", 64, 64, 0), ("wide", 300, 70, 1), ("tall", 33, 257, 2), ("one", 1, 5, 3), ("cfg1rows", 1024, 48, 4)]
    for name, K, O, seed in cases:
        torch.manual_seed(seed)
        layer = pkg.BitLinear(K, O)
        out[f"{name}_meta"] = np.array([K, O, seed], dtype=np.int64)
        out[f"{name}_q"] = layer.int_weight.numpy().copy()
        out[f"{name}_s"] = layer.weight_scale.numpy().copy()
        # the next draw of the default generator: the construction consumed exactly the Kaiming draw
        out[f"{name}_next"] = torch.rand(4).numpy()
    np.savez_compressed(HERE / "bitlinear_init.npz", **out)


def main() -> None:
    torch.set_num_threads(1)
    pkg, fk, fo, _ = _import_reference(sys.argv[1] if len(sys.argv) > 1 else None)
    gen_init(pkg)
    gen_quant(fk)
    gen_mulaw(fo)
    gen_optim(pkg, fk, fo)
    gen_linear(pkg, fk)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()

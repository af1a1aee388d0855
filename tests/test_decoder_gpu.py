"""The BitLinear decoder harness (the data-parallel training workload) on the GPU.

* its forward equals the same network computed in fp32 with the dequantised weights, up to
  the int8 activation quantisation (relative Frobenius error of the logits);
* a few optimizer steps (FireFlyOptim and the ZeRO-1 optimizer at world size 1) fit a fixed
  batch: the loss falls;
* every BitLinear weight gets a gradient in the arena and every dense parameter a ``.grad``.
"""
import math

import pytest
import torch
from torch.nn import functional as F

from firefly_b200.decoder import DecoderConfig, build_decoder, synthetic_batches, train_step
from firefly_b200.distributed import ZeroFireFlyOptim
from firefly_b200.fireflyoptim import FireFlyOptim

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TINY = DecoderConfig(vocab=512, d_model=256, heads=4, ffn=1024, layers=2, max_seq=64)


def _fp32_logits(model, ids):
    """The decoder's forward in fp32 with W = int_weight * weight_scale (no activation quantisation)."""
    def lin(m, x):
        w = m.int_weight.float() * m.weight_scale.float()[:, None]
        return F.linear(x, w, None if m.bias is None else m.bias.float())

    def ln(m, x):
        return F.layer_norm(x, (x.shape[-1],), m.weight.float(), m.bias.float(), m.eps)

    B, S = ids.shape
    x = model.tok(ids).float() + model.pos[:S].float()
    for L in model.layers:
        d = x.shape[-1]
        hd = d // L.heads
        qkv = lin(L.qkv, ln(L.ln1, x)).view(B, S, 3, L.heads, hd).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(qkv[0], qkv[1], qkv[2], is_causal=True)  # fp32: math backend
        x = x + lin(L.proj, a.transpose(1, 2).reshape(B, S, d))
        x = x + lin(L.down, F.gelu(lin(L.up, ln(L.ln2, x)), approximate="tanh"))
    return lin(model.lm_head, ln(model.ln_f, x))


def test_forward_matches_fp32_dequantised_network():
    model = build_decoder(TINY, DEV, seed=1)
    ids, _ = synthetic_batches(TINY, 4, 64, 4, DEV, seed=2)[0]
    with torch.no_grad():
        got = model(ids).float()
        ref = _fp32_logits(model, ids)
    assert got.shape == (4, 64, TINY.vocab) and model(ids).dtype == torch.bfloat16
    rel = (got - ref).norm() / ref.norm()
    # per-token int8 activations and bf16 residuals through 2 layers + head
    assert rel < 0.05, float(rel)


@pytest.mark.parametrize("zero", [False, True])
def test_training_steps_fit_a_fixed_batch(zero):
    model = build_decoder(TINY, DEV, seed=3)
    batches = synthetic_batches(TINY, 4, 64, 2, DEV, seed=4)  # 2 micro-batches of 2 sequences
    bits = model.bit_modules()
    if zero:
        opt = ZeroFireFlyOptim(bits, params=model.dense_parameters(), lr=3e-3, weight_decay=0.0, seed=5)
    else:
        opt = FireFlyOptim(model.dense_parameters(), lr=3e-3, weight_decay=0.0, bit_modules=bits)
    losses = [float(train_step(model, opt, batches)) for _ in range(25)]
    assert all(math.isfinite(v) for v in losses)
    assert abs(losses[0] - math.log(TINY.vocab)) < 0.5, losses[0]
    assert losses[-1] < losses[0] - 1.0, losses


def test_every_parameter_gets_a_gradient():
    model = build_decoder(TINY, DEV, seed=6)
    bits = model.bit_modules()
    opt = ZeroFireFlyOptim(bits, params=model.dense_parameters(), lr=1e-3, seed=7)
    ids, tgt = synthetic_batches(TINY, 2, 32, 2, DEV, seed=8)[0]
    model.loss(ids, tgt).backward()
    has = opt.arena.collect_grads()
    assert all(has) and len(has) == 4 * TINY.layers + 1
    for gv in opt.arena.g_views:
        assert gv.abs().sum() > 0
    for name, p in model.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name

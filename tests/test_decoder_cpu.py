"""Host-side pieces of the 1.3B decoder harness (no GPU): its size, the int8 operation count the
benchmark divides by, and the synthetic micro-batches (targets are the ids shifted by one)."""
import torch

from firefly_b200.decoder import DECODER_1P3B, DecoderConfig, attention_flops_per_sequence, synthetic_batches


def test_1p3b_configuration_counts():
    cfg = DECODER_1P3B
    assert (cfg.layers, cfg.d_model, cfg.heads, cfg.ffn, cfg.vocab, cfg.max_seq) == (24, 2048, 16, 8192, 32000, 2048)
    per_layer = 3 * 2048 * 2048 + 2048 * 2048 + 2 * 2048 * 8192
    assert cfg.bit_params == 24 * per_layer + 2048 * 32000 == 1_273_495_552
    assert cfg.int8_ops_per_token() == 6 * cfg.bit_params
    # causal attention: 7 matmuls of 2*S*(S/2)*d per layer and sequence
    assert attention_flops_per_sequence(cfg, 2048) == 24 * 7 * 2 * 2048 * 1024 * 2048


def test_synthetic_micro_batches():
    cfg = DecoderConfig(vocab=100, d_model=32, heads=2, ffn=64, layers=1, max_seq=16)
    batches = synthetic_batches(cfg, 10, 16, 4, torch.device("cpu"), seed=3)
    assert [ids.shape for ids, _ in batches] == [(4, 16), (4, 16), (2, 16)]
    for ids, tgt in batches:
        assert ids.dtype == torch.int64 and int(ids.min()) >= 0 and int(ids.max()) < cfg.vocab
        assert torch.equal(ids[:, 1:], tgt[:, :-1])
    again = synthetic_batches(cfg, 10, 16, 4, torch.device("cpu"), seed=3)
    assert all(torch.equal(a[0], b[0]) for a, b in zip(batches, again))

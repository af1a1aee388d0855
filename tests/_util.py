"""Shared helpers of the parity tests (the oracle is the checker)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import firefly_oracle as O

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def load_golden(name: str):
    return np.load(GOLDEN / name)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).cpu().view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(h: np.ndarray, device="cpu") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(h, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def bf16_ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 representable steps (sign-magnitude aware)."""
    def key(h):
        h = h.astype(np.int32)
        return np.where(h & 0x8000, -(h & 0x7FFF), h & 0x7FFF)
    return np.abs(key(a_bits) - key(b_bits))


def assert_close_rel(got: np.ndarray, want: np.ndarray, rel: float, what: str, ulp_bits=None, ulp_want=None):
    """|got-want| <= rel*max(|want|, floor); elements failing that may pass by being within
    one bf16 step of the rounded oracle (when bf16 bit patterns are given)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.maximum(np.abs(want), 1e-30)
    bad = np.abs(got - want) > rel * scale
    if ulp_bits is not None:
        bad &= bf16_ulp_diff(ulp_bits, ulp_want) > 1
    n = int(bad.sum())
    assert n == 0, f"{what}: {n} of {bad.size} elements outside rel {rel}; first at {np.argwhere(bad)[:3].tolist()}"


def code_mismatch(got, want):
    d = np.abs(np.asarray(got, np.int32) - np.asarray(want, np.int32))
    return d


def check_optim_step(q_got, st_got, q_want, st_want, what, frac=1e-3):
    """Optimizer parity bar: int8 weights and 8-bit codes differ by <=1 LSB on <=0.1% of
    elements.  An element whose stochastic-rounding decision flipped (its weight differs)
    carries a residual differing by ~1.0; such elements are counted in the budget but
    allowed any residual-code difference."""
    n = q_want.size
    dq = code_mismatch(q_got, q_want).ravel()
    assert dq.max(initial=0) <= 1, f"{what}: int8 weight off by {dq.max()}"
    flips = dq > 0
    assert flips.sum() <= frac * n, f"{what}: {flips.sum()} weight mismatches of {n}"
    for k in ("m_q", "v_q"):
        d = code_mismatch(st_got[k], st_want[k]).ravel()
        assert d.max(initial=0) <= 1, f"{what}: {k} off by {d.max()}"
        assert (d > 0).sum() <= frac * n, f"{what}: {k} {int((d > 0).sum())} mismatches of {n}"
    d = code_mismatch(st_got["r_q"], st_want["r_q"]).ravel()
    bad = (d > 1) & ~flips
    assert not bad.any(), f"{what}: r_q off by >1 at {np.argwhere(bad)[:5].ravel().tolist()}"
    assert (d > 0).sum() <= frac * n + flips.sum(), f"{what}: r_q {int((d > 0).sum())} mismatches of {n}"
    for k in ("m_absmax", "v_absmax", "r_absmax"):
        a, b = np.asarray(st_got[k], np.float64), np.asarray(st_want[k], np.float64)
        rel = np.abs(a - b) / np.maximum(np.abs(b), 1e-30)
        # an absmax equals one element's |value|: allow a few ulps, or a flip in that block
        assert (rel > 1e-5).sum() <= max(1, frac * b.size) + flips.sum(), f"{what}: {k} rel err {rel.max()}"

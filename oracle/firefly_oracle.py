"""CPU oracle for the FireFly INT8 training hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker.  Only ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` may import it; the product path
(``firefly_b200``) never does, and fails loudly if its CUDA library is missing.

It restates the reference algorithm (fumitoshi0524/FireFly) in numpy:

* ``quantize_rows``           fireflykernels.py:96-104 (``quantize_fp_to_int8``)
* ``quantize_cols_t``         the same math applied per column, codes transposed
                              (the dW operands of the int8 backward)
* ``gemm_i8`` + ``dequant``   int32 accumulation and the scale epilogue, the
                              structure of ``_forward_bnb`` fireflykernels.py:132-156
* ``linear_forward`` / ``linear_backward``
                              BitLinear through int8 GEMMs: Y = X Wᵀ, dX = dY W,
                              dW = dYᵀ X (fireflykernels.py:164-210 define the ops)
* ``encode_signed`` …         mu-law 8-bit blockwise codecs fireflyoptim.py:8-80
* ``dqt_adamw8_step``         FireFlyOptim bit-module update fireflyoptim.py:136-209
* ``philox_uniforms``         the counter-based uniforms the GPU optimizer draws
* ``dynamic_qmap`` / ``dense_adamw8_step``
                              block-wise 8-bit AdamW of dense parameters (the published
                              algorithm of the bitsandbytes optimizer the reference uses,
                              fireflyoptim.py:83, :124; bitsandbytes itself is absent, so
                              this follows the B200 build's own map and rounding)
* ``swiglu_forward`` / ``swiglu_backward`` / ``swiglu_mlp_step``
                              the SwiGLU MLP block of BitLinear layers (the benchmark
                              workload; the reference has no model code): torch's
                              bf16 silu, mul and their autograd formulas

Rounding model.  Every reference op is evaluated in fp32 with correct rounding:
``+ - * /`` are IEEE fp32, ``sqrt/exp/log1p/tanh`` are computed in fp64 and
rounded once to fp32.  The two fused multiply-adds that torch's CPU kernels
perform (``add_(g, alpha=…)`` and ``addcmul_``, fireflyoptim.py:175-176) are
modelled as FMAs.  torch's own CPU transcendental and sqrt kernels are within
about one ulp of this, so the oracle reproduces the reference's int8 codes
exactly and its 8-bit optimizer codes to within one code on a tiny fraction of
elements; ``tests/test_oracle_golden.py`` pins both against fixtures produced
by running the reference (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
_MU = F32(255.0)
_INV_LN1P_MU = F32(1.0 / 5.545177444479562)  # fireflyoptim.py:10


# --------------------------------------------------------------------------
# bf16 helpers (bf16 is carried as uint16 bit patterns)
# --------------------------------------------------------------------------
def f32_to_bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 (what ``tensor.to(torch.bfloat16)`` does)."""
    f = np.ascontiguousarray(x, dtype=np.float32)
    b = f.view(np.uint32)
    t = b >> 16
    t &= 1
    t += 0x7FFF
    t += b  # no uint32 overflow for finite values; NaN patterns are replaced below
    t >>= 16
    r = t.astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(h) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def _f64fn(fn, x):
    return fn(np.asarray(x, dtype=np.float32).astype(np.float64)).astype(np.float32)


def _fma(a, b, c):
    """fp32 fused multiply-add, rounded once (fp64 holds a*b exactly)."""
    a64 = np.asarray(a, np.float32).astype(np.float64)
    b64 = np.asarray(b, np.float32).astype(np.float64)
    c64 = np.asarray(c, np.float32).astype(np.float64)
    return (a64 * b64 + c64).astype(np.float32)


# --------------------------------------------------------------------------
# a1: per-row absmax int8 quantiser
# --------------------------------------------------------------------------
def quantize_rows(w, eps: float = 1e-8, colmul=None):
    """fireflykernels.py:96-104: ``s = max(|w|_row, eps)/127``, ``q = clamp(rint(w/s), ±127)``.

    ``colmul`` (optional, fp32 per column) multiplies ``w`` elementwise first;
    the backward uses it to fold the per-output weight scale into dY.
    """
    w = np.asarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError(f"weight must be 2D [out_features, in_features], got {w.shape}")
    if colmul is not None:
        w = w * np.asarray(colmul, np.float32)[None, :]
    if w.shape[1] == 0:
        raise ValueError("cannot quantise rows of length 0")
    absmax = np.abs(w).max(axis=1, keepdims=True) if w.shape[0] else np.zeros((0, 1), F32)
    scale = np.maximum(absmax, F32(eps)) / F32(127.0)
    with np.errstate(invalid="ignore", divide="ignore"):
        q = np.clip(np.rint(w / scale), -127, 127)
    q = np.where(np.isnan(q), 0, q).astype(np.int8)
    return q, scale[:, 0].astype(np.float32)


def quantize_cols_t(x, eps: float = 1e-8):
    """Per-column version of ``quantize_rows``: returns codes transposed ``[C, R]`` and ``s[C]``."""
    q, s = quantize_rows(np.asarray(x, np.float32).T, eps)
    return q, s


# --------------------------------------------------------------------------
# int8 GEMM + epilogue
# --------------------------------------------------------------------------
def gemm_i8(a, b) -> np.ndarray:
    """Exact ``A[M,K] · B[N,K]ᵀ`` accumulation of int8 codes, returned as int64."""
    a = np.asarray(a, np.int8)
    b = np.asarray(b, np.int8)
    # K chunks of 1024: every partial sum is an integer below 2^24, exact in fp32 BLAS;
    # chunks are summed in fp64 (exact below 2^53)
    acc = np.zeros((a.shape[0], b.shape[0]), np.float64)
    for k0 in range(0, a.shape[1], 1024):
        acc += a[:, k0:k0 + 1024].astype(np.float32) @ b[:, k0:k0 + 1024].astype(np.float32).T
    return np.rint(acc).astype(np.int64)


def dequant(acc, scale_a=None, scale_b=None, bias=None) -> np.ndarray:
    """Epilogue: ``((f32(acc) * sa[m]) * sb[n]) + bias[n]`` in fp32, each op rounded."""
    v = np.asarray(acc).astype(np.float32)
    if scale_a is not None:
        v = v * np.asarray(scale_a, np.float32)[:, None]
    if scale_b is not None:
        v = v * np.asarray(scale_b, np.float32)[None, :]
    if bias is not None:
        v = v + np.asarray(bias, np.float32)[None, :]
    return v


# --------------------------------------------------------------------------
# SwiGLU activation between BitLinear layers (bf16 tensors, as torch computes them)
# --------------------------------------------------------------------------
def _sigmoid_parts(g):
    """``(1 + exp(-g), 1 / (1 + exp(-g)))`` in fp32, exp rounded once from fp64."""
    g = np.asarray(g, np.float32)
    den = (F32(1.0) + _f64fn(np.exp, -g)).astype(np.float32)
    return den, (F32(1.0) / den).astype(np.float32)


def swiglu_forward(g, u):
    """``h = bf16(bf16(silu(g)) * u)`` for bf16-valued fp32 arrays g, u (torch's F.silu(g) * u)."""
    g = np.asarray(g, np.float32)
    den, _ = _sigmoid_parts(g)
    silu = round_bf16(g / den)
    return round_bf16(silu * np.asarray(u, np.float32))


def swiglu_backward(dh, g, u):
    """``(dg, du)`` of ``h = silu(g) * u`` as torch's autograd forms them in bf16:
    ``du = bf16(dh * bf16(silu(g)))`` and ``dg = bf16(ds * s * (1 + g * (1 - s)))`` with
    ``ds = bf16(dh * u)``, ``s = 1 / (1 + exp(-g))`` (the last term one FMA)."""
    dh, g, u = (np.asarray(a, np.float32) for a in (dh, g, u))
    den, sg = _sigmoid_parts(g)
    ds = round_bf16(dh * u)
    dg = round_bf16((ds * sg).astype(np.float32) * _fma(g, (F32(1.0) - sg).astype(np.float32), F32(1.0)))
    du = round_bf16(dh * round_bf16(g / den))
    return dg, du


def swiglu_mlp_step(x, dy, q_gu, s_gu, q_d, s_d, eps: float = 1e-8):
    """Forward + backward of ``y = down(silu(g) * u)``, ``[g | u] = gate_up(x)``.

    ``q_gu [2f, d]`` holds the gate rows then the up rows.  Returns a dict with y, dx
    and both weight gradients (bf16 bit patterns) and the intermediate codes."""
    x = np.asarray(x, np.float32)
    f = q_d.shape[1]
    gu_bits, q_x, s_x, _ = linear_forward(x, q_gu, s_gu, eps=eps)
    gu = bf16_bits_to_f32(gu_bits)
    g, u = gu[:, :f], gu[:, f:]
    h = swiglu_forward(g, u)
    y_bits, q_h, s_h, _ = linear_forward(h, q_d, s_d, eps=eps)
    bd = linear_backward(h, dy, q_d, s_d, eps=eps)
    dh = bf16_bits_to_f32(bd["dx"])
    dg, du = swiglu_backward(dh, g, u)
    bgu = linear_backward(x, np.concatenate([dg, du], axis=1), q_gu, s_gu, eps=eps)
    return {"y": y_bits, "dx": bgu["dx"], "gw_gu": bgu["gw"], "gw_d": bd["gw"], "gu": gu_bits,
            "q_h": q_h, "s_h": s_h, "q_dgu": bgu["q_g"], "s_dgu": bgu["s_g"],
            "q_dgut": bgu["q_dyt"], "s_dguc": bgu["s_dy"]}


# --------------------------------------------------------------------------
# BitLinear through int8 GEMMs
# --------------------------------------------------------------------------
def linear_forward(x, q_w, s_w, bias=None, eps: float = 1e-8):
    """Y = X·W_effᵀ (+b) with per-token int8 activations.  Returns (y_bf16_bits, q_x, s_x, acc)."""
    q_x, s_x = quantize_rows(x, eps)
    acc = gemm_i8(q_x, q_w)
    y = dequant(acc, s_x, s_w, bias)
    return f32_to_bf16_bits(y), q_x, s_x, acc


def linear_backward(x, dy, q_w, s_w, has_bias=False, eps: float = 1e-8, grad_cache=None):
    """int8 backward of ``fireflykernels.py:184-210``.

    * dX: quantise ``g = dY ⊙ s_w`` per token, ``dX = s_g[t] · (q_g · q_w)`` (contracts over O).
    * dW: quantise dY and X per column over tokens, ``dW = s_dy[o]·s_x[k]·(q_dyᵀ · q_xᵀᵀ)``.
      Added to ``grad_cache`` like ``_BIT_GRAD_CACHE`` (bf16 add of the bf16-rounded term).
    * db: fp32 column sum of dY, rounded to bf16.
    Returns dict with bf16 bit patterns for dx, gw, db and the intermediate codes.
    """
    x = np.asarray(x, np.float32)
    dyf = bf16_bits_to_f32(dy) if np.asarray(dy).dtype == np.uint16 else np.asarray(dy, np.float32)
    q_g, s_g = quantize_rows(dyf, eps, colmul=s_w)
    acc_dx = gemm_i8(q_g, np.ascontiguousarray(np.asarray(q_w, np.int8).T))
    dx = dequant(acc_dx, s_g, None)
    q_dyt, s_dy = quantize_cols_t(dyf, eps)
    q_xt, s_xc = quantize_cols_t(x, eps)
    acc_dw = gemm_i8(q_dyt, q_xt)
    gw = f32_to_bf16_bits(dequant(acc_dw, s_dy, s_xc))
    if grad_cache is not None:
        gw = f32_to_bf16_bits(bf16_bits_to_f32(grad_cache) + bf16_bits_to_f32(gw))
    out = {
        "dx": f32_to_bf16_bits(dx), "gw": gw,
        "q_g": q_g, "s_g": s_g, "acc_dx": acc_dx,
        "q_dyt": q_dyt, "s_dy": s_dy, "q_xt": q_xt, "s_xc": s_xc, "acc_dw": acc_dw,
    }
    if has_bias:
        out["db"] = f32_to_bf16_bits(dyf.astype(np.float64).sum(axis=0).astype(np.float32))
    return out


# --------------------------------------------------------------------------
# mu-law 8-bit blockwise codecs (fireflyoptim.py:8-80)
# --------------------------------------------------------------------------
def _blocks(x, bs):
    flat = np.asarray(x, np.float32).ravel()
    n = flat.size
    nb = (n + bs - 1) // bs
    pad = np.zeros(nb * bs, np.float32)
    pad[:n] = flat
    return pad.reshape(nb, bs), n


def encode_signed(x, bs: int = 256):
    """fireflyoptim.py:22-36. Returns (uint8 codes shaped like x, fp32 absmax[nblocks])."""
    blocks, n = _blocks(x, bs)
    absmax = np.maximum(np.abs(blocks).max(axis=1), F32(1e-12))
    xn = np.clip(blocks / absmax[:, None], F32(-1.0), F32(1.0))
    comp = (np.sign(xn) * _f64fn(np.log1p, _MU * np.abs(xn))) * _INV_LN1P_MU
    q = np.clip(np.rint(comp * F32(127.0)), -127, 127).astype(np.int16)
    codes = (q.ravel()[:n] + 128).astype(np.uint8)
    return codes.reshape(np.shape(x)), absmax.astype(np.float32)


def encode_unsigned(x, bs: int = 256):
    """fireflyoptim.py:53-67 (absmax is the plain block max, not |x|)."""
    blocks, n = _blocks(x, bs)
    absmax = np.maximum(blocks.max(axis=1), F32(1e-12))
    xn = np.clip(blocks / absmax[:, None], F32(0.0), F32(1.0))
    comp = _f64fn(np.log1p, _MU * xn) * _INV_LN1P_MU
    q = np.clip(np.rint(comp * F32(255.0)), 0, 255)
    codes = q.ravel()[:n].astype(np.uint8)
    return codes.reshape(np.shape(x)), absmax.astype(np.float32)


def decode_table_signed() -> np.ndarray:
    """x_norm for each signed code, fireflyoptim.py:47-48 (absmax factor excluded)."""
    y = np.clip((np.arange(256, dtype=np.float32) - F32(128.0)) / F32(127.0), F32(-1), F32(1))
    return (np.sign(y) * (_f64fn(np.exp, np.abs(y) / _INV_LN1P_MU) - F32(1.0))) / _MU


def decode_table_unsigned() -> np.ndarray:
    """x_norm for each unsigned code, fireflyoptim.py:77-78."""
    y = np.clip(np.arange(256, dtype=np.float32) / F32(255.0), F32(0), F32(1))
    return (_f64fn(np.exp, y / _INV_LN1P_MU) - F32(1.0)) / _MU


def _decode(codes, absmax, bs, table):
    c = np.asarray(codes, np.uint8).ravel()
    n = c.size
    xn = table[c]
    blk = np.arange(n) // bs
    return (xn * np.asarray(absmax, np.float32)[blk]).reshape(np.shape(codes))


def decode_signed(codes, absmax, bs: int = 256):
    """fireflyoptim.py:39-50."""
    return _decode(codes, absmax, bs, decode_table_signed())


def decode_unsigned(codes, absmax, bs: int = 256):
    """fireflyoptim.py:70-80."""
    return _decode(codes, absmax, bs, decode_table_unsigned())


def init_state(shape, bs: int = 256) -> dict:
    """Zero-initialised 8-bit states, fireflyoptim.py:142-161."""
    z = np.zeros(shape, np.float32)
    m_q, m_a = encode_signed(z, bs)
    v_q, v_a = encode_unsigned(z, bs)
    r_q, r_a = encode_signed(z, bs)
    return {"step": 0, "m_q": m_q, "m_absmax": m_a, "v_q": v_q, "v_absmax": v_a,
            "r_q": r_q, "r_absmax": r_a}


# --------------------------------------------------------------------------
# DQT-SR 8-bit AdamW step (fireflyoptim.py:136-209)
# --------------------------------------------------------------------------
def dqt_adamw8_step(q, ws, g, state, *, lr, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.1,
                    sr_bias=0.15, bs=256, u=None):
    """One bit-module update.  ``g`` is the fp32 (bf16-valued) gradient ``[O, K]``.

    Returns ``(q_new, state_new)``; ``state`` is not modified.  ``u`` are the
    uniforms of ``torch.rand_like`` (fireflyoptim.py:192), shape ``[O, K]``.
    """
    q = np.asarray(q, np.int8)
    g = np.asarray(g, np.float32)
    shape = q.shape
    m = decode_signed(state["m_q"], state["m_absmax"], bs)
    v = decode_unsigned(state["v_q"], state["v_absmax"], bs)
    r = decode_signed(state["r_q"], state["r_absmax"], bs)
    t = int(state["step"]) + 1
    m = _fma(g, F32(1.0 - beta1), m * F32(beta1))
    v = _fma(F32(1.0 - beta2) * g, g, v * F32(beta2))
    m_hat = m / F32(1.0 - beta1 ** t)
    v_hat = v / F32(1.0 - beta2 ** t)
    ws = np.asarray(ws, np.float32)
    if ws.shape == shape:  # one scale per element (a flat piece of a weight)
        ws_c = np.maximum(ws, F32(eps))
    else:  # one scale per row
        ws_c = np.maximum(ws.reshape(-1, 1), F32(eps))
        if len(shape) == 1:
            ws_c = ws_c.reshape(-1)
    iw = q.astype(np.float32)
    adam = m_hat / (_f64fn(np.sqrt, v_hat) + F32(eps))
    dwe = F32(-lr) * (adam + (F32(wd) * iw) * ws_c)
    r = r + dwe / ws_c
    abs_r = np.abs(r)
    base = np.floor(abs_r)
    frac = abs_r - base
    sgn = np.sign(r).astype(np.float32)
    bias = (_f64fn(np.tanh, adam) * F32(sr_bias)) * sgn
    fb = np.clip(frac + bias, F32(0.0), F32(1.0))
    if u is None:
        raise ValueError("the oracle needs the uniforms")
    extra = (np.asarray(u, np.float32) < fb).astype(np.float32)
    dq = (sgn * (base + extra)).astype(np.int32)
    if np.any(dq != 0):
        q = np.clip(q.astype(np.int16) + dq.astype(np.int16), -127, 127).astype(np.int8)
        r = r - dq.astype(np.float32)
    r_q, r_a = encode_signed(r, bs)
    m_q, m_a = encode_signed(m, bs)
    v_q, v_a = encode_unsigned(v, bs)
    return q, {"step": t, "m_q": m_q, "m_absmax": m_a, "v_q": v_q, "v_absmax": v_a,
               "r_q": r_q, "r_absmax": r_a}


def dqt_adamw8_segment(q, ws_rows, row_len, elem_base, g, state, *, lr, beta1=0.9, beta2=0.999, eps=1e-8,
                       wd=0.1, sr_bias=0.15, u, bs=256):
    """``dqt_adamw8_step`` on a flat piece of one weight: elements ``[elem_base, elem_base+n)``
    of a weight whose rows are ``row_len`` long and whose per-row scales are ``ws_rows``.
    ``elem_base`` must be a multiple of ``bs`` (blocks are those of the whole weight)."""
    q = np.asarray(q, np.int8).ravel()
    n = q.size
    rows = (elem_base + np.arange(n)) // int(row_len)
    ws_elem = np.asarray(ws_rows, np.float32)[rows]
    st = {k: (np.asarray(v).ravel() if k.endswith("_q") else v) for k, v in state.items()}
    return dqt_adamw8_step(q, ws_elem, np.asarray(g, np.float32).ravel(), st, lr=lr, beta1=beta1, beta2=beta2,
                           eps=eps, wd=wd, sr_bias=sr_bias, bs=bs, u=np.asarray(u, np.float32).ravel())


# --------------------------------------------------------------------------
# Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11) counter-based uniforms
# --------------------------------------------------------------------------
_PHILOX_M0 = np.uint64(0xD2511F53)
_PHILOX_M1 = np.uint64(0xCD9E8D57)
_PHILOX_W0 = np.uint32(0x9E3779B9)
_PHILOX_W1 = np.uint32(0xBB67AE85)


def philox4x32_10(c0, c1, c2, c3, k0, k1):
    """Vectorised Philox4x32 with 10 rounds; all arguments uint32 arrays/scalars."""
    c0, c1, c2, c3 = (np.asarray(c, np.uint32).copy() for c in (c0, c1, c2, c3))
    k0, k1 = int(k0) & 0xFFFFFFFF, int(k1) & 0xFFFFFFFF
    for _ in range(10):
        p0 = _PHILOX_M0 * c0.astype(np.uint64)
        p1 = _PHILOX_M1 * c2.astype(np.uint64)
        hi0, lo0 = (p0 >> np.uint64(32)).astype(np.uint32), p0.astype(np.uint32)
        hi1, lo1 = (p1 >> np.uint64(32)).astype(np.uint32), p1.astype(np.uint32)
        c0, c1, c2, c3 = hi1 ^ c1 ^ np.uint32(k0), lo1, hi0 ^ c3 ^ np.uint32(k1), lo0
        k0 = (k0 + int(_PHILOX_W0)) & 0xFFFFFFFF
        k1 = (k1 + int(_PHILOX_W1)) & 0xFFFFFFFF
    return c0, c1, c2, c3


def philox_uniforms(numel: int, seed: int, step: int, elem_offset: int = 0) -> np.ndarray:
    """Uniforms in (0,1) for global elements ``[elem_offset, elem_offset+numel)``.

    Element ``e`` uses Philox call ``e // 8`` (counter ``(e//8 lo, e//8 hi, step lo, step hi)``,
    key ``(seed lo, seed hi)``) and 16-bit lane ``e % 8`` of its 128-bit output
    (word ``(e%8)//2``, low half first); ``u = (h + 0.5) / 65536``.
    """
    if numel == 0:
        return np.zeros(0, np.float32)
    e = np.arange(elem_offset, elem_offset + numel, dtype=np.uint64)
    call = np.unique(e // np.uint64(8))
    lo = (call & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    hi = (call >> np.uint64(32)).astype(np.uint32)
    s_lo = np.uint32(step & 0xFFFFFFFF)
    s_hi = np.uint32((step >> 32) & 0xFFFFFFFF)
    w = philox4x32_10(lo, hi, np.full_like(lo, s_lo), np.full_like(lo, s_hi),
                      np.uint32(seed & 0xFFFFFFFF), np.uint32((seed >> 32) & 0xFFFFFFFF))
    words = np.stack(w, axis=1)  # [ncalls, 4]
    halves = np.stack([words & 0xFFFF, words >> 16], axis=2).reshape(-1, 8)  # [ncalls, 8]
    idx = (e // np.uint64(8) - call[0]).astype(np.int64)
    h = halves[idx, (e % np.uint64(8)).astype(np.int64)].astype(np.float32)
    return (h + F32(0.5)) * F32(1.0 / 65536.0)


# --------------------------------------------------------------------------
# Block-wise 8-bit AdamW of dense parameters
# --------------------------------------------------------------------------
DENSE_BLOCK = 2048


def dynamic_qmap(signed: bool) -> np.ndarray:
    """The dynamic tree map: sign (signed only), a zero run selecting the decade 10^-e, an
    indicator bit, and the remaining bits as a linear fraction in (0.1, 1].  Signed: e = 0..6
    with 6-e fraction bits, both signs, zero twice; unsigned: e = 0..7 with 7-e fraction bits
    and zero.  256 fp32 values, ascending."""
    fb = 6 if signed else 7
    mags = [10.0 ** (-e) * (0.1 + 0.9 * k / 2 ** (fb - e)) for e in range(fb + 1) for k in range(1, 2 ** (fb - e) + 1)]
    vals = ([0.0, 0.0] + mags + [-m for m in mags]) if signed else ([0.0] + mags)
    return np.array(sorted(vals), dtype=np.float64).astype(np.float32)


def _nearest_codes(x, q):
    """Nearest map entry of each value (ties to the lower code); x within [q[0], q[-1]]."""
    x = np.asarray(x, np.float32)
    lo = np.clip(np.searchsorted(q, x, side="right") - 1, 0, 255)
    hi = np.minimum(lo + 1, 255)
    d_lo = (x - q[lo]).astype(np.float32)
    d_hi = (q[hi] - x).astype(np.float32)
    return np.where((hi > lo) & (d_hi < d_lo), hi, lo).astype(np.uint8)


def init_dense_state(n: int) -> dict:
    nb = -(-n // DENSE_BLOCK)
    return {"step": 0, "m_q": np.full(n, 128, np.uint8), "m_absmax": np.zeros(nb, np.float32),
            "v_q": np.zeros(n, np.uint8), "v_absmax": np.zeros(nb, np.float32)}


def dense_adamw8_step(p, g, state, *, lr, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01, qmaps=None):
    """One block-wise 8-bit AdamW step (fp32, every operation rounded once):
    m = b1*m + (1-b1)*g, v = b2*v + ((1-b2)*g)*g, p = p*(1-lr*wd) - a_t*(m/(sqrt(v)+e_t)) with
    a_t = lr*sqrt(bc2)/bc1, e_t = eps*sqrt(bc2) (Kingma & Ba, section 2), then per block of 2048
    the absmax of |m| and v and the nearest codes of value*(1/absmax).  ``qmaps`` = (signed,
    unsigned) 256-entry ascending maps, the dynamic tree maps by default.  Returns (p, state)."""
    p = np.asarray(p, np.float32).ravel().copy()
    g = np.asarray(g, np.float32).ravel()
    n = p.size
    if qmaps is None:
        qs, qu = dynamic_qmap(True), dynamic_qmap(False)
    else:
        qs, qu = (np.asarray(q, np.float32) for q in qmaps)
    t = state["step"] + 1
    blk = np.arange(n) // DENSE_BLOCK
    m0 = (qs[state["m_q"]] * state["m_absmax"][blk]).astype(np.float32)
    v0 = (qu[state["v_q"]] * state["v_absmax"][blk]).astype(np.float32)
    F = np.float32
    b1, b2 = F(beta1), F(beta2)
    if wd != 0.0:
        p = (p * F(1.0 - lr * wd)).astype(np.float32)
    m = (b1 * m0 + (F(1.0 - beta1) * g).astype(np.float32)).astype(np.float32)
    v = (b2 * v0 + ((F(1.0 - beta2) * g).astype(np.float32) * g).astype(np.float32)).astype(np.float32)
    bc1, bc2 = 1.0 - beta1 ** t, 1.0 - beta2 ** t
    step_size, eps_hat = F(lr * np.sqrt(bc2) / bc1), F(eps * np.sqrt(bc2))
    den = (np.sqrt(v) + eps_hat).astype(np.float32)
    p = (p - (step_size * (m / den).astype(np.float32)).astype(np.float32)).astype(np.float32)
    nb = -(-n // DENSE_BLOCK)
    pad = nb * DENSE_BLOCK - n
    am = np.abs(np.pad(m, (0, pad))).reshape(nb, DENSE_BLOCK).max(axis=1).astype(np.float32)
    av = np.abs(np.pad(v, (0, pad))).reshape(nb, DENSE_BLOCK).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        im = np.where(am > 0, F(1.0) / am, F(1.0)).astype(np.float32)
        iv = np.where(av > 0, F(1.0) / av, F(1.0)).astype(np.float32)
    st = {"step": t, "m_q": _nearest_codes((m * im[blk]).astype(np.float32), qs), "m_absmax": am,
          "v_q": _nearest_codes((v * iv[blk]).astype(np.float32), qu), "v_absmax": av}
    return p, st

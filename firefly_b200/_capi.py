"""ctypes binding of libfirefly_b200.so (declared in include/firefly_b200.h).

Every wrapper takes CUDA tensors, launches on the tensor's device and on
torch's current stream of that device, and raises on a non-zero status:
``ValueError`` for FF_ERR_INVALID_ARG / FF_ERR_UNSUPPORTED, ``RuntimeError``
for FF_ERR_CUDA.  There is no CPU path: if the library is missing or a tensor
is not on a CUDA device, the call raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libfirefly_b200.so"

FF_OK = 0
FF_ERR_INVALID_ARG = 1
FF_ERR_UNSUPPORTED = 2
FF_ERR_CUDA = 3
FF_DEVICE_TIMEOUT = 0x1
FF_DEVICE_BADARG = 0x2
FF_DTYPE_F32 = 0
FF_DTYPE_BF16 = 1
FF_DTYPE_F16 = 2
FF_OUT_S32 = 0
FF_OUT_F32 = 1
FF_OUT_BF16 = 2
FF_OUT_BF16_ACCUM = 3

# every symbol declared in include/firefly_b200.h, with its ctypes signature
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float
_D = ctypes.c_double
_U64 = ctypes.c_uint64
SIGNATURES = {
    "ff_version": (ctypes.c_char_p, []),
    "ff_last_error": (ctypes.c_char_p, []),
    "ff_num_sms": (_I, [_P]),
    "ff_device_status": (_I, [_P, _I]),
    "ff_quant_rows_i8": (_I, [_P, _I, _I64, _I64, _I64, _P, _F, _P, _I64, _P, _P]),
    "ff_quant_dual_i8": (_I, [_P, _I, _I64, _I64, _I64, _P, _F, _P, _I64, _P, _P, _I64, _P, _P, _P]),
    "ff_quant_dual_i8_noalloc": (_I, [_P, _I, _I64, _I64, _I64, _P, _F, _P, _I64, _P, _P, _I64, _P, _P]),
    "ff_swiglu_selftest": (_I, [_P, _P, _P]),
    "ff_gelu_eval": (_I, [_P, _I64, _I, _I, _P, _P, _P]),
    "ff_layernorm_i8": (_I, [_P, _I64, _I64, _I64, _P, _P, _F, _P, _I64, _P, _P, _F, _P, _I64, _P, _P, _I64, _P,
                             _P, _P]),
    "ff_layernorm_bwd_ws_elems": (_I64, [_I64, _I64]),
    "ff_layernorm_bwd": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P, _P, _P, _P]),
    "ff_gelu_gemm_i8": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _F, _I, _P,
                             _I64, _P, _P, _I64, _P, _P, _P]),
    "ff_gelu_bwd_gemm_i8": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _F, _I, _P,
                                 _I64, _P, _P, _I64, _P, _P, _P]),
    "ff_swiglu_bwd_gemm_i8": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _F, _P,
                                   _I64, _P, _P, _I64, _P, _P, _P]),
    "ff_swiglu_gemm_i8": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _P, _I64, _I64, _I64, _I64, _F, _P, _I64,
                               _P, _P, _I64, _P, _P, _P]),
    "ff_swiglu_quant_i8": (_I, [_P, _P, _I64, _I64, _I64, _F, _P, _I64, _P, _I64, _P, _P, _I64, _P, _P, _P]),
    "ff_swiglu_bwd_quant_i8": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _F, _P, _I64, _P, _I64, _P, _P,
                                    _I64, _P, _P, _P]),
    "ff_transpose_i8": (_I, [_P, _I64, _I64, _I64, _P, _I64, _P]),
    "ff_gemm_i8": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _I, _I64, _I64, _I64, _P]),
    "ff_gemm_i8_ws_bytes": (_I64, [_I64, _I64, _I64]),
    "ff_set_wait_limit_ns": (_I, [_U64]),
    "ff_gemm_i8_ws": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _I, _I64, _I64, _I64, _P, _I64, _P]),
    "ff_gemm_i8_kn": (_I, [_P, _I64, _P, _I64, _P, _P, _P, _P, _I64, _I, _I64, _I64, _I64, _P]),
    "ff_colsum_ws_elems": (_I64, [_I64, _I64]),
    "ff_colsum_bf16": (_I, [_P, _I64, _I64, _I64, _P, _P, _P]),
    "ff_quant_dual_db_ws_elems": (_I64, [_I64, _I64]),
    "ff_quant_dual_i8_db": (_I, [_P, _I64, _I64, _I64, _P, _F, _P, _I64, _P, _P, _I64, _P, _P, _P, _P, _P]),
    "ff_dqt_adamw8": (_I, [_P, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _I64, _I64,
                           _D, _D, _D, _D, _D, _D, _D, _D, _U64, _U64, _I64, _P, _P, _P, _P]),
    "ff_dqt_adamw8_peers": (_I, [_P, _P, _I64, _I64, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P, _P, _I64, _I64,
                                 _D, _D, _D, _D, _D, _D, _D, _D, _U64, _U64, _I64, _P, _P, _P]),
    "ff_ipc_alloc": (_I, [_I64, ctypes.POINTER(ctypes.c_void_p)]),
    "ff_ipc_free": (_I, [_P]),
    "ff_ipc_get_handle": (_I, [_P, ctypes.c_char_p]),
    "ff_ipc_open": (_I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "ff_ipc_close": (_I, [_P]),
    "ff_update_int8_weight": (_I, [_P, _P, _I64, _P]),
    "ff_adamw8_blockwise": (_I, [_P, _I, _P, _I, _P, _P, _P, _P, _I64, _D, _D, _D, _D, _D, _I64, _P, _P, _P]),
    "ff_adamw32_multi": (_I, [_P, ctypes.c_int32, _F, ctypes.c_int32, _F, _F, _F, _F, _P]),
}


class Adamw32Tensor(ctypes.Structure):
    """``FfAdamw32Tensor``: one dense parameter of ``ff_adamw32_multi``."""
    _fields_ = [("param", _P), ("grad", _P), ("exp_avg", _P), ("exp_avg_sq", _P), ("numel", ctypes.c_int64),
                ("param_dtype", ctypes.c_int32), ("grad_dtype", ctypes.c_int32), ("eps_term", _F),
                ("step_scale", _F)]

_lib = None

# Instrumentation for benchmarks: number of this library's kernels launched so far,
# and an optional list that collects (start_event, end_event, ops, algorithmic bytes) per GEMM launch.
LAUNCHES = 0
GEMM_EVENTS: list | None = None
# the same for the GEMMs with a SwiGLU epilogue (their windows include the quantiser pass that
# the call launches after the GEMM)
FUSED_GEMM_EVENTS: list | None = None
_KERNELS_PER_CALL = {"ff_quant_rows_i8": 1, "ff_quant_dual_i8": 2, "ff_quant_dual_i8_noalloc": 2,
                     "ff_swiglu_quant_i8": 2, "ff_swiglu_bwd_quant_i8": 2, "ff_swiglu_selftest": 1,
                     "ff_swiglu_gemm_i8": 2, "ff_swiglu_bwd_gemm_i8": 2,
                     "ff_gelu_eval": 1, "ff_gelu_gemm_i8": 2, "ff_gelu_bwd_gemm_i8": 2,
                     "ff_layernorm_i8": 2, "ff_layernorm_bwd": 3,
                     "ff_transpose_i8": 1, "ff_gemm_i8": 1, "ff_gemm_i8_kn": 1, "ff_gemm_i8_ws": 1,
                     "ff_colsum_bf16": 2, "ff_quant_dual_i8_db": 3, "ff_dqt_adamw8": 1, "ff_dqt_adamw8_peers": 1, "ff_update_int8_weight": 1,
                     "ff_adamw8_blockwise": 1,
                     "ff_adamw32_multi": 1}


def lib() -> ctypes.CDLL:
    """Load the CUDA library once; raise if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"firefly_b200 CUDA library not found at {LIB_PATH}; "
                "build it with `python -m firefly_b200._build`"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def version() -> str:
    return lib().ff_version().decode()


def _raise(rc: int, name: str) -> None:
    msg = lib().ff_last_error().decode()
    if rc in (FF_ERR_INVALID_ARG, FF_ERR_UNSUPPORTED):
        raise ValueError(f"{name}: {msg}")
    raise RuntimeError(f"{name} failed ({rc}): {msg}")


def _call(name: str, *args) -> None:
    global LAUNCHES
    rc = getattr(lib(), name)(*args)
    if rc != FF_OK:
        _raise(rc, name)
    LAUNCHES += _KERNELS_PER_CALL.get(name, 0)


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("firefly_b200 kernels run on CUDA tensors only "
                               f"(got a tensor on {t.device})")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise ValueError("no tensor given")
    return dev


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return FF_DTYPE_F32
    if dt == torch.bfloat16:
        return FF_DTYPE_BF16
    if dt == torch.float16:
        return FF_DTYPE_F16
    raise ValueError(f"unsupported input dtype {dt}")


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _rows_view(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    """2-D tensor with unit column stride and its leading dimension."""
    if x.dim() != 2:
        raise ValueError(f"expected a 2-D tensor, got shape {tuple(x.shape)}")
    if x.stride(1) != 1 or x.stride(0) < x.shape[1]:
        x = x.contiguous()
    return x, max(x.stride(0), x.shape[1])


# ---------------------------------------------------------------------------
# typed wrappers
# ---------------------------------------------------------------------------
def num_sms(device: torch.device | None = None) -> int:
    out = ctypes.c_int(0)
    with torch.cuda.device(device or torch.cuda.current_device()):
        _call("ff_num_sms", ctypes.byref(out))
    return out.value


def device_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Read (and by default clear) the device status word; synchronises the device.  A nonzero
    status also drops the split-K workspaces (an aborted GEMM may have left partial sums)."""
    out = ctypes.c_uint32(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        _call("ff_device_status", ctypes.byref(out), int(clear))
    if out.value:
        _SPLITK_WS.clear()
    return out.value


# Split-K workspaces of the skinny GEMMs, per (device, stream): zero-filled once, and left
# all zeros by every ff_gemm_i8_ws call, so calls on one stream can share one.
_SPLITK_WS: dict = {}


def _splitk_ws(dev: torch.device, nbytes: int) -> torch.Tensor:
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    ws = _SPLITK_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros((max(nbytes, 1 << 20) + 15) // 16 * 16, dtype=torch.uint8, device=dev)
        _SPLITK_WS[key] = ws
    return ws


def quant_rows(x: torch.Tensor, colmul: torch.Tensor | None = None, eps: float = 1e-8,
               ldq: int | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row int8 quantiser.  Returns ``(q [R, ldq] int8, s [R] fp32)``."""
    dev = _require_cuda(x, colmul)
    x, ldx = _rows_view(x)
    R, C = x.shape
    if C == 0:
        raise ValueError("cannot quantise rows of length 0")
    ldq = C if ldq is None else ldq
    q = torch.empty((R, ldq), dtype=torch.int8, device=dev)
    s = torch.empty((R,), dtype=torch.float32, device=dev)
    if colmul is not None:
        colmul = colmul.to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        _call("ff_quant_rows_i8", _ptr(x), _dtype_code(x.dtype), R, C, ldx, _ptr(colmul),
              float(eps), _ptr(q), ldq, _ptr(s), _stream(dev))
    return q, s


def quant_dual(x: torch.Tensor, row_colmul: torch.Tensor | None = None, eps: float = 1e-8,
               rows: bool = True, cols: bool = True, colsum: bool = False):
    """Row codes ``[R, ldq]`` (ldq = round_up(C,16)) and transposed column codes
    ``[C, ldqt]`` (ldqt = round_up(R,16)) with their scales.  Either part may be skipped
    (returned as ``None``).  ``colsum=True`` (bf16 ``x`` only) appends a fifth output, the
    bf16 column sums of ``x`` (``colsum_bf16(x)``'s values), taken in the same read of x."""
    dev = _require_cuda(x, row_colmul)
    if colsum and x.dtype != torch.bfloat16:
        raise ValueError(f"quant_dual(colsum=True) needs a bf16 input, got {x.dtype}")
    x, ldx = _rows_view(x)
    R, C = x.shape
    if C == 0:
        raise ValueError("cannot quantise rows of length 0")
    ldq, ldqt = round_up(C, 16), round_up(max(R, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((R, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((R,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((C, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((C,), dtype=torch.float32, device=dev)
    ws = torch.empty((R + C,), dtype=torch.float32, device=dev)
    if row_colmul is not None:
        row_colmul = row_colmul.to(torch.float32).contiguous()
    if colsum:
        db = torch.empty((C,), dtype=torch.bfloat16, device=dev)
        db_ws = torch.empty((int(lib().ff_quant_dual_db_ws_elems(R, C)),), dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _call("ff_quant_dual_i8_db", _ptr(x), R, C, ldx, _ptr(row_colmul), float(eps), _ptr(q_rows), ldq,
                  _ptr(s_rows), _ptr(q_cols), ldqt, _ptr(s_cols), _ptr(ws), _ptr(db), _ptr(db_ws), _stream(dev))
        return q_rows, s_rows, q_cols, s_cols, db
    with torch.cuda.device(dev):
        _call("ff_quant_dual_i8", _ptr(x), _dtype_code(x.dtype), R, C, ldx, _ptr(row_colmul),
              float(eps), _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols), ldqt, _ptr(s_cols),
              _ptr(ws), _stream(dev))
    return q_rows, s_rows, q_cols, s_cols


_SWIGLU_CHECKED: set[int] = set()


def swiglu_selftest(device: torch.device | None = None) -> tuple[int, int, int | None]:
    """``(mismatches, ieee_inputs, first_mismatch)`` of the exhaustive check of the SwiGLU
    kernels' branch-free arithmetic over all 65536 bf16 inputs on ``device`` (synchronises);
    ``first_mismatch`` is the smallest mismatching bf16 bit pattern or None."""
    mism, ieee, first = ctypes.c_uint32(0), ctypes.c_uint32(0), ctypes.c_uint32(0)
    with torch.cuda.device(device or torch.cuda.current_device()):
        _call("ff_swiglu_selftest", ctypes.byref(mism), ctypes.byref(ieee), ctypes.byref(first))
    return int(mism.value), int(ieee.value), (None if first.value == 0xFFFFFFFF else int(first.value))


def _require_swiglu_math(dev: torch.device) -> None:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx in _SWIGLU_CHECKED:
        return
    mism, _, first = swiglu_selftest(torch.device("cuda", idx))
    if mism:
        raise RuntimeError(f"SwiGLU kernels' arithmetic differs from IEEE fp32 on cuda:{idx} for {mism} "
                           f"bf16 inputs (first: 0x{first:04x}); the fused SwiGLU path cannot be used")
    _SWIGLU_CHECKED.add(idx)


def _swiglu_halves(gu: torch.Tensor):
    """The gate and up halves ``[T, f]`` of a bf16 ``[T, 2f]`` projection output."""
    if gu.dtype != torch.bfloat16 or gu.dim() != 2 or gu.shape[1] % 2:
        raise ValueError(f"expected a bf16 [T, 2f] gate/up output, got {gu.dtype} {tuple(gu.shape)}")
    gu, ld = _rows_view(gu)
    return gu, ld, gu.shape[1] // 2


def swiglu_quant(gu: torch.Tensor, eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """Dual codes of ``h = silu(g) * u`` (bf16 as torch forms it) for ``gu = [g | u]``.

    Returns ``quant_dual(h)``'s four outputs and h itself (bf16 ``[T, f]``)."""
    dev = _require_cuda(gu)
    _require_swiglu_math(dev)
    gu, ld, F = _swiglu_halves(gu)
    T = gu.shape[0]
    ldq, ldqt = round_up(F, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((F, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((F,), dtype=torch.float32, device=dev)
    ldh = round_up(F, 8)
    h = torch.empty((T, ldh), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((T + F,), dtype=torch.float32, device=dev)
    u = gu[:, F:]
    with torch.cuda.device(dev):
        _call("ff_swiglu_quant_i8", _ptr(gu), _ptr(u), ld, T, F, float(eps), _ptr(h), ldh, _ptr(q_rows), ldq,
              _ptr(s_rows), _ptr(q_cols), ldqt, _ptr(s_cols), _ptr(ws), _stream(dev))
    return q_rows, s_rows, q_cols, s_cols, h[:, :F]


def swiglu_gemm(a: torch.Tensor, b: torch.Tensor, k: int, scale_a: torch.Tensor, scale_b: torch.Tensor,
                bias: torch.Tensor | None = None, eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """Gate/up GEMM of a SwiGLU block with h = silu(g) * u in its epilogue.

    ``a``: int8 activation codes ``[T, lda]``, ``b``: int8 weight ``[2F, ldb]`` (gate rows, then
    up rows), contraction over the first ``k`` columns.  Returns ``(gu, q_rows, s_rows,
    q_cols_t, s_cols, h)``: gu = ``[g | u]`` bf16 ``[T, 2F]`` as ``gemm_i8`` gives it, and the
    outputs of ``swiglu_quant(gu)``."""
    dev = _require_cuda(a, b, scale_a, scale_b, bias)
    _require_swiglu_math(dev)
    a, lda = _rows_view(a)
    b, ldb = _rows_view(b)
    T, F2 = a.shape[0], b.shape[0]
    F = F2 // 2
    ldq, ldqt = round_up(F, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((F, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((F,), dtype=torch.float32, device=dev)
    gu = torch.empty((T, F2), dtype=torch.bfloat16, device=dev)
    h = torch.empty((T, F), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((T + F,), dtype=torch.float32, device=dev)
    f32 = [None if t is None else t.to(torch.float32).contiguous() for t in (scale_a, scale_b, bias)]
    with torch.cuda.device(dev):
        ev = None
        if FUSED_GEMM_EVENTS is not None and T > 0:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        _call("ff_swiglu_gemm_i8", _ptr(a), lda, _ptr(b), ldb, _ptr(f32[0]), _ptr(f32[1]), _ptr(f32[2]),
              _ptr(gu), F2, _ptr(h), F, T, F, int(k), float(eps), _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols),
              ldqt, _ptr(s_cols), _ptr(ws), _stream(dev))
        if ev is not None:
            ev[1].record()
            FUSED_GEMM_EVENTS.append((ev[0], ev[1], 2 * T * F2 * int(k)))
    return gu, q_rows, s_rows, q_cols, s_cols, h


def swiglu_bwd_gemm(a: torch.Tensor, w: torch.Tensor, k: int, scale_a: torch.Tensor, gu: torch.Tensor,
                    colmul: torch.Tensor | None = None, eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """``dh = a · w[:k]`` (w: int8 ``[k, F]`` row-major, the down projection's weight) with the
    SwiGLU backward in the epilogue.  Returns ``swiglu_bwd_quant(dh, gu, colmul)``'s outputs
    ``(q_rows, s_rows, q_cols_t, s_cols, dgu)`` without writing dh."""
    dev = _require_cuda(a, w, scale_a, gu, colmul)
    _require_swiglu_math(dev)
    gu, ldgu, F = _swiglu_halves(gu)
    a, lda = _rows_view(a)
    w, ldw = _rows_view(w)
    T = a.shape[0]
    ldq, ldqt = round_up(2 * F, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((2 * F, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((2 * F,), dtype=torch.float32, device=dev)
    dgu = torch.empty((T, 2 * F), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((T + 2 * F,), dtype=torch.float32, device=dev)
    sa = scale_a.to(torch.float32).contiguous()
    if colmul is not None:
        colmul = colmul.to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        ev = None
        if FUSED_GEMM_EVENTS is not None and T > 0:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        _call("ff_swiglu_bwd_gemm_i8", _ptr(a), lda, _ptr(w), ldw, _ptr(sa), _ptr(gu), ldgu, _ptr(colmul),
              _ptr(dgu), 2 * F, T, F, int(k), float(eps), _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols), ldqt,
              _ptr(s_cols), _ptr(ws), _stream(dev))
        if ev is not None:
            ev[1].record()
            FUSED_GEMM_EVENTS.append((ev[0], ev[1], 2 * T * F * int(k)))
    return q_rows, s_rows, q_cols, s_cols, dgu


# ---------------------------------------------------------------------------
# LayerNorm with the first pass of the dual quantiser of its output
# ---------------------------------------------------------------------------
def layernorm_quant(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                    q_eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """LayerNorm of the rows of a bf16 ``[T, C]`` matrix (fp32 gamma, beta) and, unless both
    ``rows`` and ``cols`` are False, ``quant_dual`` of the bf16 output in the same call.
    Returns ``(y, mean, rstd, (q_rows, s_rows, q_cols_t, s_cols))``."""
    dev = _require_cuda(x, gamma, beta)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError(f"layernorm_quant takes a bf16 [T, C] matrix, got {x.dtype} {tuple(x.shape)}")
    x, ldx = _rows_view(x)
    T, C = x.shape
    ldq, ldqt = round_up(C, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = ws = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((C, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((C,), dtype=torch.float32, device=dev)
    if rows or cols:
        ws = torch.empty((T + C,), dtype=torch.float32, device=dev)
    y = torch.empty((T, C), dtype=torch.bfloat16, device=dev)
    mean = torch.empty((T,), dtype=torch.float32, device=dev)
    rstd = torch.empty((T,), dtype=torch.float32, device=dev)
    g = gamma.detach().to(torch.float32).contiguous()
    b = beta.detach().to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        _call("ff_layernorm_i8", _ptr(x), ldx, T, C, _ptr(g), _ptr(b), float(eps), _ptr(y), C, _ptr(mean), _ptr(rstd),
              float(q_eps), _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols), ldqt, _ptr(s_cols), _ptr(ws), _stream(dev))
    return y, mean, rstd, (q_rows, s_rows, q_cols, s_cols)


def layernorm_bwd(dy: torch.Tensor, x: torch.Tensor, mean: torch.Tensor, rstd: torch.Tensor, gamma: torch.Tensor,
                  dx: bool = True, wgrad: bool = True):
    """``(dx, dgamma, dbeta)`` of ``layernorm_quant``'s LayerNorm from its output gradient dy and
    input x (bf16 ``[T, C]``), the forward's mean and rstd and fp32 gamma (dx bf16, the others
    fp32; None where not asked for).  Deterministic."""
    dev = _require_cuda(dy, x, mean, rstd, gamma)
    dy, lddy = _rows_view(dy.to(torch.bfloat16))
    x, ldx = _rows_view(x)
    T, C = x.shape
    g = gamma.detach().to(torch.float32).contiguous()
    out_dx = torch.empty((T, C), dtype=torch.bfloat16, device=dev) if dx else None
    dgamma = dbeta = ws = None
    if wgrad:
        ws = torch.empty((max(int(lib().ff_layernorm_bwd_ws_elems(T, C)), 4),), dtype=torch.float32, device=dev)
        dgamma = torch.empty((C,), dtype=torch.float32, device=dev)
        dbeta = torch.empty((C,), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _call("ff_layernorm_bwd", _ptr(dy), lddy, _ptr(x), ldx, T, C, _ptr(mean.contiguous()), _ptr(rstd.contiguous()),
              _ptr(g), _ptr(out_dx), C, _ptr(dgamma), _ptr(dbeta), _ptr(ws), _stream(dev))
    return out_dx, dgamma, dbeta


# ---------------------------------------------------------------------------
# GELU (tanh form) in the GEMM epilogues of a BitLinear GELU MLP block
# ---------------------------------------------------------------------------
_GELU_VARIANT: dict[int, int] = {}


def gelu_eval(x: torch.Tensor, fwd_variant: int = 0, bwd_variant: int = 0):
    """``(gelu(x), gelu'(x))`` in fp32, as the GELU epilogues compute them, for a bf16 tensor x
    (``ff_gelu_eval``); the variant bits choose where multiplies and adds are fused."""
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise ValueError(f"gelu_eval takes bf16 inputs, got {x.dtype}")
    x = x.contiguous().view(-1)
    h = torch.empty(x.shape, dtype=torch.float32, device=dev)
    d = torch.empty(x.shape, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _call("ff_gelu_eval", _ptr(x), x.numel(), int(fwd_variant), int(bwd_variant), _ptr(h), _ptr(d), _stream(dev))
    return h, d


def _same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equal, NaNs equal to any NaN."""
    nan = torch.isnan(a.float())
    if not torch.equal(nan, torch.isnan(b.float())):
        return False
    ib = torch.int16 if a.element_size() == 2 else torch.int32
    return bool(torch.equal(a.view(ib)[~nan], b.view(ib)[~nan]))


def gelu_variant(device: torch.device | None = None) -> int:
    """Variant bits under which the GELU epilogues equal torch's tanh-form GELU kernels on
    ``device``: ``gelu(x, approximate="tanh")`` for every bf16 x, and ``gelu_backward`` (fp32,
    unit gradient, i.e. gelu'(x) itself) for every bf16-valued x.  Found once per device
    (synchronises); raises if no variant matches."""
    from torch.nn import functional as F

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx in _GELU_VARIANT:
        return _GELU_VARIANT[idx]
    dev = torch.device("cuda", idx)
    x = torch.arange(-32768, 32768, dtype=torch.int32, device=dev).to(torch.int16).view(torch.bfloat16)
    ref_h = F.gelu(x, approximate="tanh")
    ref_d = torch.ops.aten.gelu_backward(torch.ones(x.shape, dtype=torch.float32, device=dev), x.float(),
                                         approximate="tanh")
    fwd = next((v for v in (0, 1) if _same_bits(gelu_eval(x, v, 0)[0].to(torch.bfloat16), ref_h)), None)
    bwd = next((v for v in range(0, 64, 2) if _same_bits(gelu_eval(x, 0, v)[1], ref_d)), None)
    if fwd is None or bwd is None:
        def misses(a, b):
            ok = (a.view(torch.int32) == b.view(torch.int32)) | (torch.isnan(a) & torch.isnan(b))
            return int((~ok).sum())
        best = min((misses(gelu_eval(x, 0, v)[1], ref_d), v) for v in range(0, 64, 2))
        raise RuntimeError(f"no GELU epilogue variant reproduces torch's GELU kernels on cuda:{idx} "
                           f"(forward {'ok' if fwd is not None else 'unmatched'}, backward "
                           f"{'ok' if bwd is not None else f'unmatched: closest variant {best[1]} differs on {best[0]} inputs'}"
                           "); the fused GELU path cannot be used")
    # the bf16 backward is one more rounding of dy * gelu'(x): check it on sampled gradients
    g = torch.Generator(device=dev).manual_seed(0)
    dy = (torch.randn(x.shape, device=dev, generator=g) * 4).to(torch.bfloat16)
    got = (dy.float() * gelu_eval(x, 0, bwd)[1]).to(torch.bfloat16)
    if not _same_bits(got, torch.ops.aten.gelu_backward(dy, x, approximate="tanh")):
        raise RuntimeError(f"the GELU epilogues' bf16 backward differs from torch's on cuda:{idx}")
    _GELU_VARIANT[idx] = fwd | bwd
    return fwd | bwd


def gelu_gemm(a: torch.Tensor, b: torch.Tensor, k: int, scale_a: torch.Tensor, scale_b: torch.Tensor,
              bias: torch.Tensor | None = None, eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """Up GEMM of a GELU MLP block with h = gelu(u) (tanh form) in its epilogue.

    ``a``: int8 activation codes ``[T, lda]``, ``b``: int8 weight ``[F, ldb]``, contraction over
    the first ``k`` columns.  Returns ``(u, q_rows, s_rows, q_cols_t, s_cols, h)``: u bf16
    ``[T, F]`` as ``gemm_i8`` gives it, h = bf16(gelu(u)) as torch forms it, and h's dual codes
    (``quant_dual(h)``)."""
    dev = _require_cuda(a, b, scale_a, scale_b, bias)
    variant = gelu_variant(dev)
    a, lda = _rows_view(a)
    b, ldb = _rows_view(b)
    T, F = a.shape[0], b.shape[0]
    ldq, ldqt = round_up(F, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((F, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((F,), dtype=torch.float32, device=dev)
    u = torch.empty((T, F), dtype=torch.bfloat16, device=dev)
    h = torch.empty((T, F), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((T + F,), dtype=torch.float32, device=dev)
    f32 = [None if t is None else t.to(torch.float32).contiguous() for t in (scale_a, scale_b, bias)]
    with torch.cuda.device(dev):
        ev = None
        if FUSED_GEMM_EVENTS is not None and T > 0:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        _call("ff_gelu_gemm_i8", _ptr(a), lda, _ptr(b), ldb, _ptr(f32[0]), _ptr(f32[1]), _ptr(f32[2]), _ptr(u), F,
              _ptr(h), F, T, F, int(k), float(eps), variant, _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols), ldqt,
              _ptr(s_cols), _ptr(ws), _stream(dev))
        if ev is not None:
            ev[1].record()
            FUSED_GEMM_EVENTS.append((ev[0], ev[1], 2 * T * F * int(k)))
    return u, q_rows, s_rows, q_cols, s_cols, h


def gelu_bwd_gemm(a: torch.Tensor, w: torch.Tensor, k: int, scale_a: torch.Tensor, u: torch.Tensor,
                  colmul: torch.Tensor | None = None, eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """``dh = a · w[:k]`` (w: int8 ``[k, F]`` row-major, the down projection's weight) with the
    GELU backward ``du = dh * gelu'(u)`` in the epilogue.  Returns ``(q_rows, s_rows, q_cols_t,
    s_cols, du)``: du bf16 ``[T, F]`` as torch's ``gelu_backward`` forms it from the bf16 dh, and
    ``quant_dual(du, row_colmul=colmul)``; dh is not written."""
    dev = _require_cuda(a, w, scale_a, u, colmul)
    variant = gelu_variant(dev)
    if u.dtype != torch.bfloat16 or u.dim() != 2:
        raise ValueError(f"expected a bf16 [T, F] up output, got {u.dtype} {tuple(u.shape)}")
    u, ldu = _rows_view(u)
    a, lda = _rows_view(a)
    w, ldw = _rows_view(w)
    T, F = a.shape[0], u.shape[1]
    ldq, ldqt = round_up(F, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((F, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((F,), dtype=torch.float32, device=dev)
    du = torch.empty((T, F), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((T + F,), dtype=torch.float32, device=dev)
    sa = scale_a.to(torch.float32).contiguous()
    if colmul is not None:
        colmul = colmul.to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        ev = None
        if FUSED_GEMM_EVENTS is not None and T > 0:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        _call("ff_gelu_bwd_gemm_i8", _ptr(a), lda, _ptr(w), ldw, _ptr(sa), _ptr(u), ldu, _ptr(colmul), _ptr(du), F,
              T, F, int(k), float(eps), variant, _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols), ldqt, _ptr(s_cols),
              _ptr(ws), _stream(dev))
        if ev is not None:
            ev[1].record()
            FUSED_GEMM_EVENTS.append((ev[0], ev[1], 2 * T * F * int(k)))
    return q_rows, s_rows, q_cols, s_cols, du


def swiglu_bwd_quant(dh: torch.Tensor, gu: torch.Tensor, colmul: torch.Tensor | None = None,
                     eps: float = 1e-8, rows: bool = True, cols: bool = True):
    """Dual codes of the ``[T, 2f]`` gradient ``[dg | du]`` of ``gu`` given ``dh = dL/dh``.

    Returns ``quant_dual([dg | du], row_colmul=colmul)``'s four outputs (row codes
    ``[T, round_up(2f, 16)]``, column codes ``[2f, round_up(T, 16)]``) and ``[dg | du]``
    itself (bf16 ``[T, 2f]``)."""
    dev = _require_cuda(dh, gu, colmul)
    _require_swiglu_math(dev)
    gu, ld, F = _swiglu_halves(gu)
    if dh.dtype != torch.bfloat16 or tuple(dh.shape) != (gu.shape[0], F):
        raise ValueError(f"dh must be bf16 [{gu.shape[0]}, {F}], got {dh.dtype} {tuple(dh.shape)}")
    dh, ldh = _rows_view(dh)
    T = gu.shape[0]
    ldq, ldqt = round_up(2 * F, 16), round_up(max(T, 1), 16)
    q_rows = s_rows = q_cols = s_cols = None
    if rows:
        q_rows = torch.empty((T, ldq), dtype=torch.int8, device=dev)
        s_rows = torch.empty((T,), dtype=torch.float32, device=dev)
    if cols:
        q_cols = torch.empty((2 * F, ldqt), dtype=torch.int8, device=dev)
        s_cols = torch.empty((2 * F,), dtype=torch.float32, device=dev)
    dgu = torch.empty((T, 2 * F), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((T + 2 * F,), dtype=torch.float32, device=dev)
    if colmul is not None:
        colmul = colmul.to(torch.float32).contiguous()
    u = gu[:, F:]
    with torch.cuda.device(dev):
        _call("ff_swiglu_bwd_quant_i8", _ptr(dh), ldh, _ptr(gu), _ptr(u), ld, T, F, _ptr(colmul),
              float(eps), _ptr(dgu), 2 * F, _ptr(q_rows), ldq, _ptr(s_rows), _ptr(q_cols), ldqt, _ptr(s_cols),
              _ptr(ws), _stream(dev))
    return q_rows, s_rows, q_cols, s_cols, dgu


def transpose_i8(src: torch.Tensor, ldd: int | None = None) -> torch.Tensor:
    """``[R, C]`` int8 -> ``[C, ldd]`` with ``ldd = round_up(R, 16)`` by default."""
    dev = _require_cuda(src)
    src, lds = _rows_view(src)
    R, C = src.shape
    ldd = round_up(max(R, 1), 16) if ldd is None else ldd
    dst = torch.empty((C, ldd), dtype=torch.int8, device=dev)
    with torch.cuda.device(dev):
        _call("ff_transpose_i8", _ptr(src), R, C, lds, _ptr(dst), ldd, _stream(dev))
    return dst


def gemm_i8(a: torch.Tensor, b: torch.Tensor, k: int, scale_a: torch.Tensor | None = None,
            scale_b: torch.Tensor | None = None, bias: torch.Tensor | None = None,
            out_kind: int = FF_OUT_BF16, out: torch.Tensor | None = None, b_kn_cols: int | None = None) -> torch.Tensor:
    """``D = epi(A[:, :k] · B[:, :k]ᵀ)``; A ``[M, lda]``, B ``[N, ldb]`` int8 (row stride 16k).

    With ``b_kn_cols = N`` the B operand is instead a K x N row-major matrix ``b[:k, :N]``
    (``ff_gemm_i8_kn``): ``D = epi(A[:, :k] · B[:k, :N])``.
    """
    dev = _require_cuda(a, b, scale_a, scale_b, bias, out)
    if a.dtype != torch.int8 or b.dtype != torch.int8:
        raise ValueError("gemm_i8 operands must be int8")
    if a.stride(1) != 1 or b.stride(1) != 1:
        raise ValueError("gemm_i8 operands need unit column stride")
    M = a.shape[0]
    lda = a.stride(0) if M > 1 else a.shape[1]
    if b_kn_cols is None:
        N = b.shape[0]
        ldb = b.stride(0) if N > 1 else b.shape[1]
        fn = "ff_gemm_i8"
    else:
        N = int(b_kn_cols)
        ldb = b.stride(0) if b.shape[0] > 1 else b.shape[1]
        fn = "ff_gemm_i8_kn"
    odt = {FF_OUT_S32: torch.int32, FF_OUT_F32: torch.float32,
           FF_OUT_BF16: torch.bfloat16, FF_OUT_BF16_ACCUM: torch.bfloat16}[out_kind]
    if out is None:
        if out_kind == FF_OUT_BF16_ACCUM:
            raise ValueError("FF_OUT_BF16_ACCUM needs an existing output")
        out = torch.empty((M, N), dtype=odt, device=dev)
    if out.dtype != odt or out.shape[0] != M or out.shape[1] != N or out.stride(1) != 1:
        raise ValueError("gemm_i8: output has the wrong dtype/shape/layout")
    ldd = out.stride(0) if M > 1 else N
    sa = None if scale_a is None else scale_a.to(torch.float32).contiguous()
    sb = None if scale_b is None else scale_b.to(torch.float32).contiguous()
    bb = None if bias is None else bias.to(torch.float32).contiguous()
    with torch.cuda.device(dev):
        ev = None
        if GEMM_EVENTS is not None and M > 0 and N > 0:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        need = int(lib().ff_gemm_i8_ws_bytes(M, N, int(k))) if fn == "ff_gemm_i8" and M > 0 and N > 0 else 0
        if need > 0:  # skinny A: stream-K over all SMs with a split-K workspace
            ws = _splitk_ws(dev, need)
            _call("ff_gemm_i8_ws", _ptr(a), lda, _ptr(b), ldb, _ptr(sa), _ptr(sb), _ptr(bb), _ptr(out),
                  ldd, int(out_kind), M, N, int(k), _ptr(ws), ws.numel(), _stream(dev))
        else:
            _call(fn, _ptr(a), lda, _ptr(b), ldb, _ptr(sa), _ptr(sb), _ptr(bb), _ptr(out),
                  ldd, int(out_kind), M, N, int(k), _stream(dev))
        if ev is not None:
            ev[1].record()
            byts = M * int(k) + N * int(k) + M * N * out.element_size() * (2 if out_kind == FF_OUT_BF16_ACCUM else 1)
            GEMM_EVENTS.append((ev[0], ev[1], 2 * M * N * int(k), byts))
    return out


def colsum_bf16(x: torch.Tensor) -> torch.Tensor:
    """Deterministic fp32 column sums of a bf16 matrix, rounded to bf16."""
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16:
        x = x.to(torch.bfloat16)
    x, ldx = _rows_view(x)
    R, C = x.shape
    out = torch.empty((C,), dtype=torch.bfloat16, device=dev)
    ws = torch.empty((int(lib().ff_colsum_ws_elems(R, C)),), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _call("ff_colsum_bf16", _ptr(x), R, C, ldx, _ptr(out), _ptr(ws), _stream(dev))
    return out


def dqt_adamw8(q: torch.Tensor, wscale: torch.Tensor, row_len: int, g: torch.Tensor,
               m_q: torch.Tensor, m_absmax: torch.Tensor, v_q: torch.Tensor,
               v_absmax: torch.Tensor, r_q: torch.Tensor, r_absmax: torch.Tensor, *,
               lr: float, beta1: float, beta2: float, eps: float, wd: float, step: int,
               sr_bias: float, seed: int, rng_offset: int = 0, elem_base: int = 0,
               u: torch.Tensor | None = None, dec_s: torch.Tensor, dec_u: torch.Tensor,
               block: int = 256) -> None:
    """In-place fused DQT 8-bit AdamW update of one int8 weight (all tensors contiguous)."""
    dev = _require_cuda(q, wscale, g, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax, u, dec_s, dec_u)
    numel = q.numel()
    for name, t, dt in (("q", q, torch.int8), ("g", g, torch.bfloat16), ("m_q", m_q, torch.uint8),
                        ("v_q", v_q, torch.uint8), ("r_q", r_q, torch.uint8)):
        if t.dtype != dt or t.numel() != numel or not t.is_contiguous():
            raise ValueError(f"dqt_adamw8: {name} must be a contiguous {dt} tensor of {numel} elements")
    for name, t in (("m_absmax", m_absmax), ("v_absmax", v_absmax), ("r_absmax", r_absmax)):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < (numel + block - 1) // block:
            raise ValueError(f"dqt_adamw8: {name} must be contiguous fp32 with one entry per block")
    if u is not None and (u.dtype != torch.float32 or u.numel() != numel or not u.is_contiguous()):
        raise ValueError("dqt_adamw8: u must be contiguous fp32 with one entry per element")
    ws = wscale.to(torch.float32).contiguous()
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    with torch.cuda.device(dev):
        _call("ff_dqt_adamw8", _ptr(q), _ptr(ws), int(row_len), int(elem_base), _ptr(g), _ptr(m_q),
              _ptr(m_absmax), _ptr(v_q), _ptr(v_absmax), _ptr(r_q), _ptr(r_absmax), numel, block,
              float(lr), float(beta1), float(beta2), float(eps), float(wd), bc1, bc2, float(sr_bias),
              int(seed) & (2**64 - 1), int(step), int(rng_offset), _ptr(u), _ptr(dec_s), _ptr(dec_u),
              _stream(dev))


DQT_MAX_SOURCES = 8
IPC_HANDLE_BYTES = 64


def dqt_adamw8_peers(q: torch.Tensor, wscale: torch.Tensor, row_len: int, g_ptrs: list[int], q_ptrs: list[int],
                     m_q: torch.Tensor, m_absmax: torch.Tensor, v_q: torch.Tensor, v_absmax: torch.Tensor,
                     r_q: torch.Tensor, r_absmax: torch.Tensor, *, lr: float, beta1: float, beta2: float,
                     eps: float, wd: float, step: int, sr_bias: float, seed: int, rng_offset: int = 0,
                     elem_base: int = 0, g_out: torch.Tensor | None = None, dec_s: torch.Tensor,
                     dec_u: torch.Tensor, block: int = 256) -> None:
    """``dqt_adamw8`` of one rank of a data-parallel job (``ff_dqt_adamw8_peers``): the gradient is
    the average of the bf16 arrays at the device addresses ``g_ptrs`` (every rank's gradient of
    these ``q.numel()`` elements, in rank order) and the new weights go to every address of
    ``q_ptrs`` (every rank's copy, ``q`` among them).  ``g_out`` (optional, bf16) receives the
    averaged gradient."""
    dev = _require_cuda(q, wscale, m_q, m_absmax, v_q, v_absmax, r_q, r_absmax, g_out, dec_s, dec_u)
    numel = q.numel()
    for name, t, dt in (("q", q, torch.int8), ("m_q", m_q, torch.uint8), ("v_q", v_q, torch.uint8),
                        ("r_q", r_q, torch.uint8)) + ((("g_out", g_out, torch.bfloat16),) if g_out is not None else ()):
        if t.dtype != dt or t.numel() != numel or not t.is_contiguous():
            raise ValueError(f"dqt_adamw8_peers: {name} must be a contiguous {dt} tensor of {numel} elements")
    for name, t in (("m_absmax", m_absmax), ("v_absmax", v_absmax), ("r_absmax", r_absmax)):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < (numel + block - 1) // block:
            raise ValueError(f"dqt_adamw8_peers: {name} must be contiguous fp32 with one entry per block")
    if not 1 <= len(g_ptrs) <= DQT_MAX_SOURCES or not 1 <= len(q_ptrs) <= DQT_MAX_SOURCES:
        raise ValueError(f"dqt_adamw8_peers: 1 to {DQT_MAX_SOURCES} gradient sources and weight destinations")
    if q.data_ptr() not in q_ptrs:
        raise ValueError("dqt_adamw8_peers: q must be one of the weight destinations")
    gs = (ctypes.c_void_p * len(g_ptrs))(*[int(x) for x in g_ptrs])
    qs = (ctypes.c_void_p * len(q_ptrs))(*[int(x) for x in q_ptrs])
    ws = wscale.to(torch.float32).contiguous()
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    with torch.cuda.device(dev):
        _call("ff_dqt_adamw8_peers", _ptr(q), _ptr(ws), int(row_len), int(elem_base), ctypes.cast(gs, _P),
              len(g_ptrs), ctypes.cast(qs, _P), len(q_ptrs), _ptr(g_out), _ptr(m_q), _ptr(m_absmax), _ptr(v_q),
              _ptr(v_absmax), _ptr(r_q), _ptr(r_absmax), numel, block, float(lr), float(beta1), float(beta2),
              float(eps), float(wd), bc1, bc2, float(sr_bias), int(seed) & (2**64 - 1), int(step),
              int(rng_offset), _ptr(dec_s), _ptr(dec_u), _stream(dev))


class IpcBuffer:
    """A device allocation of this process that other processes of the node can map (CUDA IPC).

    ``tensor(dtype)`` views it as a flat tensor; ``handle()`` gives the bytes another process
    passes to ``IpcMapping``.  The allocation is freed when the object and every tensor view of it
    are gone."""

    def __init__(self, nbytes: int, device: torch.device):
        self.nbytes, self.device = int(nbytes), device
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _call("ff_ipc_alloc", self.nbytes, ctypes.byref(ptr))
        self.ptr = int(ptr.value)
        self._lib = lib()

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            _call("ff_ipc_get_handle", self.ptr, buf)
        return buf.raw

    def tensor(self, dtype: torch.dtype) -> torch.Tensor:
        """The whole allocation as a flat tensor of ``dtype`` (it keeps this object alive)."""
        iface = {"shape": (self.nbytes,), "typestr": "|u1", "data": (self.ptr, False), "version": 3,
                 "strides": None}
        holder = type("_IpcView", (), {"__cuda_array_interface__": iface, "owner": self})()
        return torch.as_tensor(holder, device=self.device).view(dtype)

    def __del__(self):
        try:
            with torch.cuda.device(self.device):
                self._lib.ff_ipc_free(ctypes.c_void_p(self.ptr))
        except Exception:
            pass


class IpcMapping:
    """Another process's ``IpcBuffer`` mapped into this process (``ptr``: its device address here)."""

    def __init__(self, handle: bytes, device: torch.device):
        if len(handle) != IPC_HANDLE_BYTES:
            raise ValueError(f"IpcMapping: a handle has {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
        self.device = device
        ptr = ctypes.c_void_p()
        with torch.cuda.device(device):
            _call("ff_ipc_open", handle, ctypes.byref(ptr))
        self.ptr = int(ptr.value)
        self._lib = lib()

    def close(self) -> None:
        if self.ptr:
            with torch.cuda.device(self.device):
                _call("ff_ipc_close", self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            if self.ptr:
                with torch.cuda.device(self.device):
                    self._lib.ff_ipc_close(ctypes.c_void_p(self.ptr))
        except Exception:
            pass


def update_int8_weight(w: torch.Tensor, dq: torch.Tensor) -> None:
    dev = _require_cuda(w, dq)
    if w.dtype != torch.int8 or not w.is_contiguous():
        raise ValueError("update_int8_weight: int_weight must be contiguous int8")
    dq = dq.to(torch.int32).contiguous()
    if dq.numel() != w.numel():
        raise ValueError("update_int8_weight: shape mismatch")
    with torch.cuda.device(dev):
        _call("ff_update_int8_weight", _ptr(w), _ptr(dq), w.numel(), _stream(dev))


def adamw8_blockwise(p: torch.Tensor, g: torch.Tensor, m_q: torch.Tensor, m_absmax: torch.Tensor,
                     v_q: torch.Tensor, v_absmax: torch.Tensor, *, lr: float, beta1: float, beta2: float,
                     eps: float, wd: float, step: int, qmap_s: torch.Tensor, qmap_u: torch.Tensor) -> None:
    """In-place block-wise 8-bit AdamW step of a dense parameter (fp32 or bf16, contiguous)."""
    dev = _require_cuda(p, g, m_q, m_absmax, v_q, v_absmax, qmap_s, qmap_u)
    n = p.numel()
    for name, t, want in (("g", g, n), ("m_q", m_q, n), ("v_q", v_q, n)):
        if t.numel() != want or not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous with {want} elements")
    nb = (n + 2047) // 2048
    if m_absmax.numel() != nb or v_absmax.numel() != nb or m_absmax.dtype != torch.float32:
        raise ValueError(f"absmax arrays must be fp32 with {nb} elements")
    if m_q.dtype != torch.uint8 or v_q.dtype != torch.uint8:
        raise ValueError("state codes must be uint8")
    with torch.cuda.device(dev):
        _call("ff_adamw8_blockwise", _ptr(p), _dtype_code(p.dtype), _ptr(g), _dtype_code(g.dtype), _ptr(m_q),
              _ptr(m_absmax), _ptr(v_q), _ptr(v_absmax), n, float(lr), float(beta1), float(beta2), float(eps),
              float(wd), int(step), _ptr(qmap_s.contiguous()), _ptr(qmap_u.contiguous()), _stream(dev))


def adamw32_multi(items, *, lr: float, beta1: float, beta2: float, eps: float, wd: float) -> None:
    """In-place fp32-moment AdamW step of many small dense parameters in one launch (per 64).

    ``items``: ``(p, g, exp_avg, exp_avg_sq, step)`` per parameter, all on one CUDA device, contiguous,
    p and g fp32 or bf16, the moments fp32; ``step`` is the parameter's step count after this step.
    The scalars are rounded to fp32 exactly as torch rounds python-float operands."""
    items = list(items)
    if not items:
        return
    dev = _require_cuda(*[t for it in items for t in it[:4]])
    arr = (Adamw32Tensor * len(items))()
    for k, (p, g, m, v, step) in enumerate(items):
        n = p.numel()
        for name, t in (("param", p), ("grad", g), ("exp_avg", m), ("exp_avg_sq", v)):
            if t.numel() != n or not t.is_contiguous() or t.device != dev:
                raise ValueError(f"adamw32_multi: {name} of item {k} must be contiguous on {dev} with {n} elements")
        if m.dtype != torch.float32 or v.dtype != torch.float32:
            raise ValueError("adamw32_multi: the moments must be fp32")
        if p.dtype not in (torch.float32, torch.bfloat16) or g.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"adamw32_multi: fp32 or bf16 parameters and gradients, got {p.dtype}/{g.dtype}")
        bc1, bc2 = 1.0 - beta1 ** step, 1.0 - beta2 ** step
        arr[k] = Adamw32Tensor(_ptr(p), _ptr(g), _ptr(m), _ptr(v), n, _dtype_code(p.dtype), _dtype_code(g.dtype),
                               eps * bc2 ** 0.5, lr * bc2 ** 0.5 / bc1)
    with torch.cuda.device(dev):
        _call("ff_adamw32_multi", ctypes.cast(arr, _P), len(items), 1.0 - lr * wd, int(wd != 0.0), beta1,
              1.0 - beta1, beta2, 1.0 - beta2, _stream(dev))

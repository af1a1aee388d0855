#!/usr/bin/env python
"""Benchmark of FireFly's INT8 training hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one training step of a BitLinear SwiGLU MLP block at Llama-7B shapes
(d_model 4096, ffn 11008, 8192 tokens per GPU, bf16 activations, weights
N(0, 0.02) quantised per row; gate and up are the two halves of one 4096 -> 22016
BitLinear, down is 11008 -> 4096): forward, backward with an upstream gradient
~N(0,1), and the 8-bit DQT AdamW step (lr 1e-3, betas 0.9/0.999, eps 1e-8,
wd 0.01, block 256).  With N GPUs (torchrun, one rank per GPU, NCCL) every
rank runs its own 8192 tokens, gradients are reduce-scattered, the optimizer
runs ZeRO-1 sharded, and int8 weights are all-gathered (weak scaling).

Rank 0 prints one JSON line.  ``value`` is whole-job tokens/s with inputs
resident in HBM (the upstream gradient dY is a fixed resident tensor); ``e2e`` is
the same metric through the public API with each step's data batch x copied from
pinned host memory and the loss L = sum(y * R) read back, R a resident projection
(so dL/dy = R is formed on the device, as in training).
``roofline`` is the int8 GEMM (the dominant kernel) timed per launch with CUDA
events inside the timed region.  Extra keys carry the INT8 GEMM sweep (TOPS),
the 8-bit AdamW step over 6.7e9 parameters (HBM GB/s) and the dense-parameter
8-bit AdamW over 268 M fp32 parameters (HBM GB/s) (one GPU only), and, on every
rank count, ``decoder_1p3b_dp``: the data-parallel training step of the 1.3B
BitLinear decoder (24 layers, d_model 2048, ffn 8192 GELU, vocab 32000) on a
global batch of 64 x 2048 tokens split over the ranks (strong scaling).
``cpu_baseline`` is the CPU restatement of the same step timed on the host cores on
a sample.

``--impl reference`` times the CPU implementation of the path (the oracle
restatement of the reference's algorithm; the reference itself is pure Python
and is not importable on the GPU host) on the same metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "BitLinear fwd+bwd tokens/s/GPU; INT8 GEMM TOPS; 8-bit AdamW HBM GB/s"
NOMINAL_INT8_TOPS = 4500.0
ADAMW_BYTES_PER_PARAM = 2 + 2 + 6 + 3 * 4 * 2 / 256  # g, q r/w, m/v/r r/w, absmax r/w


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--d-model", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=11008)
    ap.add_argument("--adamw-params", type=float, default=6.7e9)
    ap.add_argument("--no-sub", action="store_true", help="skip the GEMM sweep and the AdamW sub-benchmarks")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decoder", action="store_true", help="skip the 1.3B decoder data-parallel step")
    ap.add_argument("--decoder-steps", type=int, default=3)
    ap.add_argument("--decoder-warmup", type=int, default=2)
    ap.add_argument("--zero-bucket-mb", type=float, default=256.0,
                    help="ZeRO-1 gradient bucket size (MB of bf16); 0 = one bucket")
    ap.add_argument("--zero-overlap", type=int, choices=[0, 1], default=1,
                    help="start each bucket's reduce-scatter from the backward pass")
    ap.add_argument("--kernel-case", choices=["gemm8192", "gemm_skinny16", "adamw", "quant", "swiglu", "swiglu_bwd",
                                              "swiglu_gemm", "gelu_gemm", "dense_adamw", "mlp", "decoder4"],
                    help="run one launch of one kernel (for ncu captures) and exit")
    return ap.parse_args()


def kernel_case(args):
    """One launch of one kernel on a case sized for an ncu capture (a few GB at most)."""
    import torch

    from firefly_b200 import _capi
    from firefly_b200.fireflyoptim import _tables_on

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if args.kernel_case.startswith("gemm"):
        M, N, K = (8192, 8192, 8192) if args.kernel_case == "gemm8192" else (16, 8192, 8192)
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        sa, sb = torch.rand(M, device=dev) * 1e-2, torch.rand(N, device=dev) * 1e-2
        _capi.gemm_i8(a, b, K, sa, sb, out_kind=_capi.FF_OUT_BF16)
    elif args.kernel_case == "adamw":
        n = 268435456
        q = torch.randint(-127, 128, (n,), dtype=torch.int8, device=dev, generator=g)
        grad = torch.empty(n, dtype=torch.bfloat16, device=dev).normal_(0, 1e-3, generator=g)
        c = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g) for _ in range(3)]
        am = [torch.empty(n // 256, device=dev).uniform_(1e-4, 1e-2, generator=g) for _ in range(3)]
        ws = torch.empty(n // 4096, device=dev).uniform_(1e-4, 1e-3, generator=g)
        dec_s, dec_u = _tables_on(dev)
        _capi.dqt_adamw8(q, ws, 4096, grad, c[0], am[0], c[1], am[1], c[2], am[2], lr=1e-3, beta1=0.9,
                         beta2=0.999, eps=1e-8, wd=0.01, step=3, sr_bias=0.15, seed=1, dec_s=dec_s, dec_u=dec_u)
    elif args.kernel_case == "quant":
        x = torch.randn(8192, 11008, device=dev, generator=g).to(torch.bfloat16)
        cm = torch.rand(11008, device=dev) * 1e-3
        _capi.quant_dual(x, row_colmul=cm)
    elif args.kernel_case in ("swiglu", "swiglu_bwd"):
        gu = (torch.randn(8192, 2 * 11008, device=dev, generator=g) * 2).to(torch.bfloat16)
        if args.kernel_case == "swiglu":
            _capi.swiglu_quant(gu)
        else:
            dh = torch.randn(8192, 11008, device=dev, generator=g).to(torch.bfloat16)
            _capi.swiglu_bwd_quant(dh, gu, colmul=torch.rand(2 * 11008, device=dev) * 1e-3)
    elif args.kernel_case == "dense_adamw":  # block-wise 8-bit AdamW of 67 M dense fp32 parameters
        from firefly_b200.adamw8 import _qmaps_on

        n = 1 << 26
        p = torch.empty(n, device=dev).normal_(0, 0.02, generator=g)
        grad = torch.empty(n, device=dev).normal_(0, 1e-3, generator=g)
        codes = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g) for _ in range(2)]
        am = [torch.empty(n // 2048, device=dev).uniform_(1e-8, 1e-2, generator=g) for _ in range(2)]
        qs, qu = _qmaps_on(dev)
        _capi.adamw8_blockwise(p, grad, codes[0], am[0], codes[1], am[1], lr=1e-3, beta1=0.9, beta2=0.999,
                               eps=1e-8, wd=0.01, step=3, qmap_s=qs, qmap_u=qu)
    elif args.kernel_case == "decoder4":
        # two training steps of a 4-layer slice of the 1.3B decoder (d 2048, ffn 8192, vocab 32000)
        # on one micro-batch of 8 x 2048 tokens; profile the second
        from dataclasses import replace

        from firefly_b200.decoder import DECODER_1P3B, build_decoder, synthetic_batches, train_step
        from firefly_b200.distributed import ZeroFireFlyOptim

        cfg = replace(DECODER_1P3B, layers=4)
        model = build_decoder(cfg, dev)
        opt = ZeroFireFlyOptim(model.bit_modules(), params=model.dense_parameters(), lr=1e-4, weight_decay=0.01,
                               seed=1)
        batches = synthetic_batches(cfg, 8, 2048, 8, dev)
        for _ in range(2):
            train_step(model, opt, batches)
    elif args.kernel_case == "gelu_gemm":  # the 1.3B decoder's up GEMM (16384 x 8192 x 2048) with GELU in its epilogue
        a = torch.randint(-127, 128, (16384, 2048), dtype=torch.int8, device=dev, generator=g)
        w = torch.randint(-127, 128, (8192, 2048), dtype=torch.int8, device=dev, generator=g)
        sa, sb = torch.rand(16384, device=dev) * 1e-2, torch.rand(8192, device=dev) * 1e-3
        _capi.gelu_gemm(a, w, 2048, sa, sb)
    elif args.kernel_case == "swiglu_gemm":  # gate/up GEMM with h = silu(g) * u in its epilogue
        a = torch.randint(-127, 128, (8192, 4096), dtype=torch.int8, device=dev, generator=g)
        w = torch.randint(-127, 128, (2 * 11008, 4096), dtype=torch.int8, device=dev, generator=g)
        sa, sb = torch.rand(8192, device=dev) * 1e-2, torch.rand(2 * 11008, device=dev) * 1e-3
        _capi.swiglu_gemm(a, w, 4096, sa, sb)
    elif args.kernel_case == "mlp":
        # two training steps of the benchmark block; profile the second (skip the first's launches)
        from firefly_b200.distributed import ZeroFireFlyOptim
        from firefly_b200.swiglu import SwiGLUMLP

        model = SwiGLUMLP(args.d_model, args.ffn).to(dev)
        model.init_normal_(0.02, generator=torch.Generator(device=dev).manual_seed(42))
        opt = ZeroFireFlyOptim([model.gate_up, model.down], lr=1e-3, weight_decay=0.01, seed=7)
        xs = [torch.randn(args.tokens, args.d_model, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
              for _ in range(2)]
        dy = torch.randn(args.tokens, args.d_model, device=dev, generator=g).to(torch.bfloat16)
        for x in xs:  # a new input each step, as in training
            y = model(x)
            y.backward(dy)
            x.grad = None
            opt.step()
    torch.cuda.synchronize()
    assert _capi.device_status() == 0
    print("ok", args.kernel_case)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.samples = []
        self.proc = None
        self.marks = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.monotonic(), [x.strip() for x in line.split(",")]))

    def mark(self):
        self.marks.append(time.monotonic())

    def stop(self):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        lo, hi = (self.marks[0], self.marks[-1]) if len(self.marks) >= 2 else (0, 1e18)
        inside = [s for t, s in self.samples if lo - 0.15 <= t <= hi + 0.15] or [s for _, s in self.samples]

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(s[0]) for s in inside if num(s[0])]
        mx = [num(s[1]) for s in inside if num(s[1])]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for s in inside:
            for n, v in zip(names, s[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        pw = [num(s[2]) for s in inside if num(s[2])]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(inside),
                "power_w_max": max(pw) if pw else None}


# ---------------------------------------------------------------------------
# CPU restatement of the step (oracle) on a bounded sample
# ---------------------------------------------------------------------------
class CpuStepModel:
    """The training step run by the numpy oracle on the host cores (its BLAS threads).

    ``fwd_bwd(t)`` times forward+backward of the MLP block on ``t`` tokens, ``opt()`` the
    optimizer on a parameter sample.  ``estimate`` fits fwd+bwd as ``a + b*T`` over the
    timed token counts (the dW epilogue and weight transposes are per-step costs, the GEMM
    main loops per-token ones) and scales the optimizer sample linearly to all parameters.
    """

    def __init__(self, d, f, tokens, param_sample=524288):
        import numpy as np

        from oracle import firefly_oracle as O

        self.np, self.O = np, O
        self.d, self.f, self.tokens = d, f, tokens
        self.params_total = 2 * d * f + f * d
        rng = self.rng = np.random.default_rng(0)
        self.qgu, self.sgu = O.quantize_rows(rng.standard_normal((2 * f, d)).astype(np.float32) * 0.02)
        self.qd, self.sd = O.quantize_rows(rng.standard_normal((d, f)).astype(np.float32) * 0.02)
        self.n = max(param_sample // 4096, 1) * 4096
        self.q, self.ws = O.quantize_rows(rng.standard_normal((self.n // 4096, 4096)).astype(np.float32) * 0.02)
        self.st = O.init_state(self.q.shape)
        self.gr = O.round_bf16(rng.standard_normal(self.q.shape).astype(np.float32) * 1e-3)
        self.uu = rng.random(self.q.shape, dtype=np.float32)
        self.fb_times: list[tuple[int, float]] = []
        self.opt_times: list[float] = []

    def fwd_bwd(self, t, record=True):
        np, O = self.np, self.O
        x = O.round_bf16(self.rng.standard_normal((t, self.d)).astype(np.float32))
        dy = O.f32_to_bf16_bits(self.rng.standard_normal((t, self.d)).astype(np.float32))
        t0 = time.perf_counter()
        O.swiglu_mlp_step(x, dy, self.qgu, self.sgu, self.qd, self.sd)
        dt = time.perf_counter() - t0
        if record:
            self.fb_times.append((t, dt))
        return dt

    def opt(self, record=True):
        t0 = time.perf_counter()
        self.O.dqt_adamw8_step(self.q, self.ws, self.gr, self.st, lr=1e-3, wd=0.01, u=self.uu)
        dt = time.perf_counter() - t0
        if record:
            self.opt_times.append(dt)
        return dt

    def estimate(self):
        np = self.np
        ts = np.array([t for t, _ in self.fb_times], np.float64)
        ys = np.array([y for _, y in self.fb_times], np.float64)
        if len(set(ts.tolist())) >= 2:
            slope, fixed = np.polyfit(ts, ys, 1)
            slope, fixed = max(slope, 0.0), max(fixed, 0.0)
        else:
            slope, fixed = float(ys.mean() / ts.mean()), 0.0
        t_opt = float(np.mean(self.opt_times))
        est = fixed + slope * self.tokens + t_opt * self.params_total / self.n
        sample = (f"fwd+bwd of the block timed on {sorted(set(int(t) for t in ts))} of {self.tokens} tokens "
                  f"({len(ts)} runs; fitted a+b*T: a={fixed:.2f}s, b={slope * 1e3:.2f}ms/token) + optimizer on "
                  f"{self.n} of {self.params_total} params ({t_opt:.3f}s, scaled x{self.params_total / self.n:.1f})")
        return est, sample


def cpu_mlp_step_estimate(d, f, tokens, token_samples=(256, 1024)):
    """Seconds per full step of the oracle and a description of the sample."""
    m = CpuStepModel(d, f, tokens)
    m.fwd_bwd(token_samples[0], record=False)  # first-touch page faults, BLAS thread start-up
    m.opt(record=False)
    for t in token_samples:
        m.fwd_bwd(t)
    m.opt()
    return m.estimate()


def _cpu_threads():
    try:
        from threadpoolctl import threadpool_info

        n = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
        return int(n)
    except Exception:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    """CPU implementation of the step on the host cores; under torchrun only rank 0 works."""
    if rank != 0:
        return
    d, f, T = args.d_model, args.ffn, args.tokens
    m = CpuStepModel(d, f, T)
    budget_s, t_start, done = 240.0, time.perf_counter(), 0
    for i in range(args.warmup + args.steps):
        timed = i >= args.warmup
        m.fwd_bwd(256 if i % 2 == 0 else 1024, record=timed)
        m.opt(record=timed)
        done += int(timed)
        if timed and done >= 2 and time.perf_counter() - t_start > budget_s:
            break
    if len(set(t for t, _ in m.fb_times)) < 2:  # one token count only: add the other
        m.fwd_bwd(1024 if m.fb_times and m.fb_times[0][0] == 256 else 256)
        m.opt()
    est, sample = m.estimate()
    if done < args.steps:
        sample += f"; stopped after {done} of {args.steps} timed steps at the {budget_s:.0f}s budget"
    value = T / est
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": est * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"swiglu_mlp_train_step T={T}/GPU d={d} f={f} (BitLinear fwd+bwd + 8-bit DQT AdamW)",
                   "tokens_per_gpu": T, "parallelism": "cpu (rank 0 only)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": _cpu_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU sub-benchmarks
# ---------------------------------------------------------------------------
def _time_cuda(fn, iters, warm=3, flush=None):
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
    return statistics.median(times)


def gemm_sweep(dev):
    import torch

    from firefly_b200 import _capi

    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    res = []
    shapes = [(n, n, n) for n in (1024, 2048, 4096, 8192)] + [(16, 8192, 8192), (128, 8192, 8192)]
    for M, N, K in shapes:
        g = torch.Generator(device=dev).manual_seed(M + N + K)
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        b = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        sa = torch.empty(M, device=dev).uniform_(1e-3, 1e-2)
        sb = torch.empty(N, device=dev).uniform_(1e-3, 1e-2)
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        t = _time_cuda(lambda: _capi.gemm_i8(a, b, K, sa, sb, out_kind=_capi.FF_OUT_BF16, out=out), 10,
                       flush=lambda: flush_buf.zero_())
        ops = 2 * M * N * K
        byts = M * K + N * K + 2 * M * N + 4 * (M + N)
        res.append({"M": M, "N": N, "K": K, "us": round(t * 1e6, 2), "tops": round(ops / t / 1e12, 1),
                    "hbm_gbs": round(byts / t / 1e9, 1)})
        # the cuBLASLt int8 comparator through torch._int_mm (int32 out), same operands
        try:
            bt = b.t()
            if M >= 17:
                tl = _time_cuda(lambda: torch._int_mm(a, bt), 10, flush=lambda: flush_buf.zero_())
                res[-1]["torch_int_mm_us"] = round(tl * 1e6, 2)
                res[-1]["torch_int_mm_tops"] = round(ops / tl / 1e12, 1)
        except Exception as e:  # noqa: BLE001
            res[-1]["torch_int_mm"] = f"unavailable: {type(e).__name__}"
        del a, b, out
    del flush_buf
    torch.cuda.empty_cache()
    return res


def adamw_bench(dev, params: float, peak_gbs: float):
    import torch

    from firefly_b200 import _capi
    from firefly_b200.fireflyoptim import _tables_on

    n = int(params) // 4096 * 4096
    free, _ = torch.cuda.mem_get_info(dev)
    need = n * (1 + 2 + 3) + 3 * 4 * n // 256 + 2 * n // 4096
    if need > free * 0.8:
        n = int(free * 0.8 / 6.05) // 4096 * 4096
    rows = n // 4096
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randint(-127, 128, (n,), dtype=torch.int8, device=dev, generator=g)
    grad = torch.empty(n, dtype=torch.bfloat16, device=dev).normal_(0, 1e-3, generator=g)
    codes = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g) for _ in range(3)]
    absm = [torch.empty(n // 256, device=dev).uniform_(1e-4, 1e-2, generator=g) for _ in range(3)]
    ws = torch.empty(rows, device=dev).uniform_(1e-4, 1e-3, generator=g)
    dec_s, dec_u = _tables_on(dev)
    step = [0]

    def run():
        step[0] += 1
        _capi.dqt_adamw8(q, ws, 4096, grad, codes[0], absm[0], codes[1], absm[1], codes[2], absm[2],
                         lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01, step=step[0] + 1, sr_bias=0.15,
                         seed=1, dec_s=dec_s, dec_u=dec_u)

    t = _time_cuda(run, 5, warm=2)
    gbs = n * ADAMW_BYTES_PER_PARAM / t / 1e9
    del q, grad, codes, absm, ws
    torch.cuda.empty_cache()
    return {"params": n, "ms": round(t * 1e3, 3), "hbm_gbs": round(gbs, 1),
            "bytes_per_param": ADAMW_BYTES_PER_PARAM, "frac_of_measured_hbm": round(gbs / peak_gbs, 3)}


def decoder_dp_bench(dev, world: int, rank: int, steps: int, warmup: int, seqs: int = 64, seq: int = 2048,
                     micro: int = 8, bucket_mb: float = 256.0, overlap: bool = True):
    """Data-parallel training step of the 1.3B BitLinear decoder (24 layers, d 2048, 16 heads,
    ffn 8192 GELU, vocab 32000) on a global batch of ``seqs`` sequences of ``seq`` tokens split
    over the ranks (strong scaling), micro-batches of ``micro`` sequences, ZeRO-1 8-bit optimizer.
    Every rank runs it; the time is the max over ranks of CUDA-event time."""
    import torch
    import torch.distributed as dist

    from firefly_b200.decoder import DECODER_1P3B, attention_flops_per_sequence, build_decoder, synthetic_batches
    from firefly_b200.decoder import train_step
    from firefly_b200.distributed import ZeroFireFlyOptim

    cfg = DECODER_1P3B
    if seqs % world:
        raise ValueError(f"global batch {seqs} is not divisible by {world} ranks")
    per_rank = seqs // world
    model = build_decoder(cfg, dev, seed=0)
    opt = ZeroFireFlyOptim(model.bit_modules(), params=model.dense_parameters(), lr=1e-4, betas=(0.9, 0.999),
                           eps=1e-8, weight_decay=0.01, seed=11, bucket_mb=bucket_mb, overlap=overlap)
    batches = synthetic_batches(cfg, per_rank, seq, min(micro, per_rank), dev, seed=1000 + rank)
    for _ in range(max(warmup, 1)):
        train_step(model, opt, batches)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        loss = train_step(model, opt, batches)
    e1.record()
    torch.cuda.synchronize()
    sec = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(sec, op=dist.ReduceOp.MAX)
    sec = float(sec.item())
    tokens = seqs * seq * steps
    out = {
        "workload": (f"decoder_1p3b_dp_train_step: {cfg.layers} layers, d {cfg.d_model}, {cfg.heads} heads, ffn "
                     f"{cfg.ffn} GELU, vocab {cfg.vocab}, all Linears BitLinear ({cfg.bit_params / 1e9:.3f}e9 int8 "
                     f"params); global batch {seqs} x {seq} tokens over {world} GPU(s), micro-batches of "
                     f"{min(micro, per_rank)}, ZeRO-1 8-bit DQT AdamW + 8-bit dense AdamW"),
        "tokens_per_s": tokens / sec, "unit": "tokens/s", "scaling": "strong", "n_gpus": world,
        "steps": steps, "warmup": max(warmup, 1), "ms_per_step": sec / steps * 1e3,
        "int8_gemm_tops_effective": cfg.int8_ops_per_token() * tokens / sec / 1e12,
        "attention_tflops_effective": attention_flops_per_sequence(cfg, seq) * seqs * steps / sec / 1e12,
        "final_loss": float(loss), "data": "synthetic token ids uniform over the vocabulary; weights N(0,0.02)",
    }
    del model, opt, batches
    torch.cuda.empty_cache()
    return out


# block-wise 8-bit AdamW of a dense fp32 parameter with an fp32 gradient: p r/w 8 + g 4 + m, v codes r/w 4
# + two block absmax r/w (16 / 2048)
DENSE_ADAMW_BYTES_PER_PARAM = 8 + 4 + 4 + 16 / 2048


def dense_adamw_bench(dev, params: int, peak_gbs: float):
    """The dense-parameter 8-bit AdamW kernel (ff_adamw8_blockwise) on ``params`` fp32 parameters."""
    import torch

    from firefly_b200 import _capi
    from firefly_b200.adamw8 import _qmaps_on

    n = int(params) // 2048 * 2048
    g = torch.Generator(device=dev).manual_seed(0)
    p = torch.empty(n, device=dev).normal_(0, 0.02, generator=g)
    grad = torch.empty(n, device=dev).normal_(0, 1e-3, generator=g)
    m_q = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g)
    v_q = torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g)
    m_a = torch.empty(n // 2048, device=dev).uniform_(1e-4, 1e-2, generator=g)
    v_a = torch.empty(n // 2048, device=dev).uniform_(1e-8, 1e-6, generator=g)
    qs, qu = _qmaps_on(dev)
    step = [0]

    def run():
        step[0] += 1
        _capi.adamw8_blockwise(p, grad, m_q, m_a, v_q, v_a, lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01,
                               step=step[0] + 1, qmap_s=qs, qmap_u=qu)

    t = _time_cuda(run, 5, warm=2)
    gbs = n * DENSE_ADAMW_BYTES_PER_PARAM / t / 1e9
    del p, grad, m_q, v_q, m_a, v_a
    torch.cuda.empty_cache()
    return {"params": n, "ms": round(t * 1e3, 3), "hbm_gbs": round(gbs, 1),
            "bytes_per_param": DENSE_ADAMW_BYTES_PER_PARAM, "frac_of_measured_hbm": round(gbs / peak_gbs, 3)}


def load_traffic():
    """DRAM bytes per launch of the dominant kernel, from the committed ncu capture."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            return {}
    return {}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def bind_to_gpu_cpus(dev):
    """Restrict this process to the CPU cores NVML reports as nearest to its GPU, so that the
    pinned host buffers of the end-to-end run sit on the GPU's NUMA node.  Returns the core
    count, or None when NVML cannot tell."""
    try:
        import pynvml
        import torch

        prop = torch.cuda.get_device_properties(dev)
        bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * w + b for w, mask in enumerate(words) for b in range(64) if (int(mask) >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:  # no NVML, or a device it does not list: keep the inherited affinity
        return None
    return None


# ---------------------------------------------------------------------------
# main arm
# ---------------------------------------------------------------------------
def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.kernel_case:
        kernel_case(args)
        return

    import datetime

    import torch
    import torch.distributed as dist

    from firefly_b200 import _capi
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.swiglu import SwiGLUMLP

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    bound_cpus = bind_to_gpu_cpus(dev) if world > 1 else None
    if world > 1:
        # keep stdout to the one JSON line (NCCL's version banner would precede it)
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "WARN"
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    d, f, T = args.d_model, args.ffn, args.tokens
    torch.manual_seed(1234 + rank)
    model = SwiGLUMLP(d, f).to(dev)
    model.init_normal_(0.02, generator=torch.Generator(device=dev).manual_seed(42))
    mods = [model.gate_up, model.down]
    opt = ZeroFireFlyOptim(mods, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, seed=7,
                           bucket_mb=args.zero_bucket_mb, overlap=bool(args.zero_overlap))
    gen = torch.Generator(device=dev).manual_seed(100 + rank)
    # the block input is an activation of the model: it needs a gradient (dX is part of the step)
    # two resident input batches used alternately, so that every step quantises a new input
    # (the op layer reuses the codes of an input tensor it has just quantised)
    xs = [torch.randn(T, d, device=dev, generator=gen).to(torch.bfloat16).requires_grad_(True) for _ in range(2)]
    x = xs[0]
    dy = torch.randn(T, d, device=dev, generator=gen).to(torch.bfloat16)

    def step(xi, dyi):
        y = model(xi)
        y.backward(dyi)
        xi.grad = None
        opt.step()
        return y

    def barrier():
        if world > 1:
            dist.barrier()

    nwarm = max(args.warmup, 3)
    for i in range(nwarm):
        step(xs[i % 2], dy)
    torch.cuda.synchronize()
    assert _capi.device_status() == 0

    gpu_id = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")[local] if os.environ.get(
        "CUDA_VISIBLE_DEVICES") else str(local)
    clocks = ClockSampler(gpu_id)
    time.sleep(0.3)
    # ---- timed region: inputs resident in HBM
    _capi.GEMM_EVENTS = []
    _capi.FUSED_GEMM_EVENTS = []
    launches0 = _capi.LAUNCHES
    barrier()
    torch.cuda.synchronize()
    clocks.mark()
    t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0e.record()
    for i in range(nwarm, nwarm + args.steps):
        step(xs[i % 2], dy)
    t1e.record()
    torch.cuda.synchronize()
    barrier()
    clocks.mark()
    launches = _capi.LAUNCHES - launches0
    gemm_events, _capi.GEMM_EVENTS = _capi.GEMM_EVENTS, None
    fused_events, _capi.FUSED_GEMM_EVENTS = _capi.FUSED_GEMM_EVENTS, None
    f_ms = [a.elapsed_time(b) for a, b, _ in fused_events]
    f_ops = [o for _, _, o in fused_events]
    sec = t0e.elapsed_time(t1e) / 1e3
    sec_t = torch.tensor([sec], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(sec_t, op=dist.ReduceOp.MAX)
    sec = float(sec_t.item())
    g_ms = [a.elapsed_time(b) for a, b, _, _ in gemm_events]
    g_ops = [o for _, _, o, _ in gemm_events]
    alg_bytes = sum(b for _, _, _, b in gemm_events)

    # ---- e2e: every step's data batch x copied from pinned host memory, the loss read back.
    # The loss is L = sum(y * R) for a fixed projection R resident on the device (the block's
    # "head"), so the upstream gradient dL/dy = R needs no copy; the step's scalar result is L.
    # The copy of step i+1's batch (side stream, two device buffers) overlaps step i.
    xh = x.detach().cpu().pin_memory()
    loss_proj = dy  # R (bf16 [T, d]): dL/dy of L = sum(y * R)
    bufs = [torch.empty_like(x).requires_grad_(True) for _ in range(2)]
    loss_h = torch.empty((2,), dtype=torch.float32).pin_memory()
    copy_stream = torch.cuda.Stream(device=dev)
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(i):
        xb = bufs[i % 2]
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[i % 2])  # the buffer's previous step is done with it
            with torch.no_grad():
                xb.copy_(xh, non_blocking=True)
            ready[i % 2].record(copy_stream)

    def e2e_run(n):
        copy_stream.wait_stream(torch.cuda.current_stream())  # copies start inside the timed region
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            torch.cuda.current_stream().wait_event(ready[i % 2])
            xb = bufs[i % 2]
            y = step(xb, loss_proj)
            free[i % 2].record()
            with torch.no_grad():
                loss = (y * loss_proj).sum(dtype=torch.float32)  # the step's loss
            loss_h[i % 2].copy_(loss, non_blocking=True)

    e2e_steps = max(3, args.steps)  # as many steps as the device-resident measurement
    e2e_run(max(args.warmup, 3))  # warm-up: first-touch allocations of this path
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    e2e_run(e2e_steps)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clocks.stop()
    e2e_sec = e0.elapsed_time(e1) / 1e3
    et = torch.tensor([e2e_sec], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_sec = float(et.item())
    status = _capi.device_status()

    peaks = load_peaks()
    sub = {}
    del model, opt
    torch.cuda.empty_cache()
    if not args.no_decoder:  # every rank: the data-parallel step
        sub["decoder_1p3b_dp"] = decoder_dp_bench(dev, world, rank, args.decoder_steps, args.decoder_warmup,
                                                  bucket_mb=args.zero_bucket_mb, overlap=bool(args.zero_overlap))
    if rank == 0 and world == 1 and not args.no_sub:
        sub["int8_gemm_sweep"] = gemm_sweep(dev)
        sub["adamw8"] = adamw_bench(dev, args.adamw_params, peaks["hbm_gbs"])
        sub["dense_adamw8"] = dense_adamw_bench(dev, 268435456, peaks["hbm_gbs"])
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        est, sample = cpu_mlp_step_estimate(d, f, T)
        cpu = {"value": T / est, "unit": "tokens/s", "cores": _cpu_threads(), "kind": "port", "sample": sample}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens_total = T * world * args.steps
    value = tokens_total / sec
    ms_per_step = sec / args.steps * 1e3
    int8_peak = 2.0 * peaks["bf16_tflops_sustained"]
    avg_ms = sum(g_ms) / max(len(g_ms), 1)
    avg_ops = sum(g_ops) / max(len(g_ops), 1)
    achieved = avg_ops / (avg_ms / 1e3) / 1e12 if g_ms else None
    gemm_share = sum(g_ms) / 1e3 / (sec if world == 1 else sec) if g_ms else None
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (x, dY ~ N(0,1) bf16; weights N(0,0.02) quantised per row)",
        "config": {
            "workload": f"swiglu_mlp_train_step T={T}/GPU d={d} f={f} (BitLinear fwd+bwd + 8-bit DQT AdamW)",
            "tokens_per_gpu": T, "global_batch_tokens": T * world,
            "parallelism": f"dp{world}" + ("+zero1" if world > 1 else ""),
            "zero1": {"bucket_mb": args.zero_bucket_mb, "overlap": bool(args.zero_overlap)},
            "l2": "inputs larger than L2 (step working set > 126 MB)",
        },
        "e2e": {"value": T * world * e2e_steps / e2e_sec, "unit": "tokens/s",
                "h2d_bytes_per_step": int(xh.numel() * xh.element_size()), "d2h_bytes_per_step": 4,
                "host_cpus_per_rank": bound_cpus},
        "gpu_launches": launches,
        "roofline": {
            "kernel": "ff_gemm_i8 (tcgen05 kind::i8)", "bound": "tensor",
            "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s", "frac": achieved / int8_peak if achieved else None,
            "traffic": load_traffic().get("ff_gemm_i8 swiglu_mlp_train_step", {}).get("bytes_per_launch"),
            "traffic_algorithmic": alg_bytes / max(len(g_ms), 1) if g_ms else None,
            "note": ("int8 ops (2*M*N*K) per launch / mean CUDA-event launch time in the timed region; "
                     "peak = 2 x measured sustained cuBLAS bf16 (MEASURED_PEAKS.json), the B200 int8 rate "
                     f"being twice bf16; frac of nominal 4.5 POPS = {achieved / NOMINAL_INT8_TOPS:.3f}"
                     if achieved else ""),
            "gemm_launches": len(g_ms), "gemm_time_share": gemm_share,
            # the gate/up GEMM and the dh GEMM run separately, with the SwiGLU activation (its
            # backward) in their epilogues; their CUDA-event windows also hold the quantiser pass
            # over h ([dg | du]) launched by the same call
            "swiglu_epilogue_gemms": ({
                "launches": len(f_ms), "ms_mean": sum(f_ms) / len(f_ms),
                "achieved_incl_quant_pass": sum(f_ops) / len(f_ops) / (sum(f_ms) / len(f_ms) / 1e3) / 1e12,
                "unit": "TFLOP/s", "time_share": sum(f_ms) / 1e3 / sec,
            } if f_ms else None),
        },
        "clocks": clocks.summary(),
        "device_status": status,
        "peaks": peaks,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    line.update(sub)
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

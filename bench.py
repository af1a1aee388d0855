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
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's algorithm (torch eager) on the GPU")
    ap.add_argument("--no-decoder", action="store_true", help="skip the 1.3B decoder data-parallel step")
    ap.add_argument("--decoder-steps", type=int, default=3)
    ap.add_argument("--decoder-warmup", type=int, default=2)
    ap.add_argument("--zero-bucket-mb", type=float, default=256.0,
                    help="ZeRO-1 gradient bucket size (MB of bf16); 0 = one bucket")
    ap.add_argument("--zero-peer", choices=["auto", "0", "1"], default="auto",
                    help="ZeRO-1 peer mode (the update kernel reads and writes the other ranks' arenas over "
                         "NVLink): auto = where the ranks can map each other's memory")
    ap.add_argument("--zero-overlap", type=int, choices=[0, 1], default=1,
                    help="start each bucket's reduce-scatter from the backward pass")
    ap.add_argument("--kernel-case", choices=["gemm8192", "gemm_skinny16", "gemm_skinny128", "gemm2048", "gemm4096",
                                              "gemm_narrow", "adamw",
                                              "quant", "quant_rows", "swiglu", "swiglu_bwd", "swiglu_gemm",
                                              "swiglu_bwd_gemm", "gelu_gemm", "gelu_bwd_gemm", "layernorm",
                                              "colsum", "quant_db", "adamw_peers", "small", "dense_adamw", "mlp",
                                              "decoder4"],
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
        # gemm_narrow: 128 x 64 tiles on one CTA each (the shape spreads best over the SMs that way)
        M, N, K = {"gemm8192": (8192, 8192, 8192), "gemm_skinny16": (16, 8192, 8192),
                   "gemm_skinny128": (128, 8192, 8192), "gemm2048": (2048, 2048, 2048),
                   "gemm4096": (4096, 4096, 4096), "gemm_narrow": (4096, 512, 4096)}[args.kernel_case]
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
    elif args.kernel_case == "quant_rows":  # the forward activation quantiser of a 4096-wide BitLinear input
        x = torch.randn(8192, 4096, device=dev, generator=g).to(torch.bfloat16)
        _capi.quant_rows(x)
    elif args.kernel_case == "layernorm":  # the decoder's LayerNorm (T=16384, C=2048) forward + backward
        x = torch.randn(16384, 2048, device=dev, generator=g).to(torch.bfloat16)
        gamma, beta = torch.rand(2048, device=dev) + 0.5, torch.randn(2048, device=dev) * 0.1
        y, mean, rstd, _ = _capi.layernorm_quant(x, gamma, beta)
        dy = torch.randn(16384, 2048, device=dev, generator=g).to(torch.bfloat16)
        _capi.layernorm_bwd(dy, x, mean, rstd, gamma)
    elif args.kernel_case == "quant_db":  # dY's backward codes with db from the same read (T=8192, O=4096)
        x = torch.randn(8192, 4096, device=dev, generator=g).to(torch.bfloat16)
        _capi.quant_dual(x, row_colmul=torch.rand(4096, device=dev) * 1e-3, colsum=True)
    elif args.kernel_case == "adamw_peers":
        # the multi-source update of peer mode, two sources (both local here) and two weight copies:
        # 134 M parameters (rows of 4096)
        n = 134217728
        q = torch.randint(-127, 128, (n,), dtype=torch.int8, device=dev, generator=g)
        q2 = q.clone()
        grads = [torch.empty(n, dtype=torch.bfloat16, device=dev).normal_(0, 1e-3, generator=g) for _ in range(2)]
        c = [torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g) for _ in range(3)]
        am = [torch.empty(n // 256, device=dev).uniform_(1e-4, 1e-2, generator=g) for _ in range(3)]
        ws = torch.empty(n // 4096, device=dev).uniform_(1e-4, 1e-3, generator=g)
        dec_s, dec_u = _tables_on(dev)
        _capi.dqt_adamw8_peers(q, ws, 4096, [t.data_ptr() for t in grads], [q.data_ptr(), q2.data_ptr()], c[0],
                               am[0], c[1], am[1], c[2], am[2], lr=1e-3, beta1=0.9, beta2=0.999, eps=1e-8,
                               wd=0.01, step=3, sr_bias=0.15, seed=1, dec_s=dec_s, dec_u=dec_u)
    elif args.kernel_case == "small":
        # the fp32-moment AdamW of the 1.3B decoder's 98 LayerNorm parameters (2048 each), the int8
        # transpose of a 8192 x 4096 weight, and the int8 weight update of 64 M parameters
        ps = [torch.randn(2048, device=dev, generator=g) for _ in range(98)]
        items = [(p_, torch.randn(2048, device=dev, generator=g), torch.zeros(2048, device=dev),
                  torch.zeros(2048, device=dev), 1) for p_ in ps]
        _capi.adamw32_multi(items, lr=1e-4, beta1=0.9, beta2=0.999, eps=1e-8, wd=0.01)
        w = torch.randint(-127, 128, (8192, 4096), dtype=torch.int8, device=dev, generator=g)
        _capi.transpose_i8(w)
        w2 = torch.randint(-127, 128, (1 << 26,), dtype=torch.int8, device=dev, generator=g)
        dq = torch.randint(-3, 4, (1 << 26,), dtype=torch.int32, device=dev, generator=g)
        _capi.update_int8_weight(w2, dq)
    elif args.kernel_case == "colsum":  # db of a BitLinear with a bias (T=8192, O=11008)
        x = torch.randn(8192, 11008, device=dev, generator=g).to(torch.bfloat16)
        _capi.colsum_bf16(x)
    elif args.kernel_case == "swiglu_bwd_gemm":  # dh = dY W_down with the SwiGLU backward in the epilogue
        a = torch.randint(-127, 128, (8192, 4096), dtype=torch.int8, device=dev, generator=g)
        w = torch.randint(-127, 128, (4096, 11008), dtype=torch.int8, device=dev, generator=g)
        gu = (torch.randn(8192, 2 * 11008, device=dev, generator=g) * 2).to(torch.bfloat16)
        _capi.swiglu_bwd_gemm(a, w, 4096, torch.rand(8192, device=dev) * 1e-2, gu,
                              colmul=torch.rand(2 * 11008, device=dev) * 1e-3)
    elif args.kernel_case == "gelu_bwd_gemm":  # the 1.3B decoder's dh GEMM (16384 x 8192 x 2048) with GELU'
        a = torch.randint(-127, 128, (16384, 2048), dtype=torch.int8, device=dev, generator=g)
        w = torch.randint(-127, 128, (2048, 8192), dtype=torch.int8, device=dev, generator=g)
        u = (torch.randn(16384, 8192, device=dev, generator=g) * 2).to(torch.bfloat16)
        _capi.gelu_bwd_gemm(a, w, 2048, torch.rand(16384, device=dev) * 1e-2, u,
                            colmul=torch.rand(8192, device=dev) * 1e-3)
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
# The reference's CPU implementation of the step (oracle restatement) on a bounded sample
# ---------------------------------------------------------------------------
REF_SLICES = 16  # the CPU sample: 1/16 of the block's width


class RefCpuSample:
    """The reference's live path (``oracle.ref_torch``: bf16 dequantisation + ``torch.matmul`` for
    BitLinear forward/backward, fireflykernels.py:164-210, and ``FireFlyOptim``'s bit-module update
    in torch ops, fireflyoptim.py:136-209) on the host cores, on a width slice of the block.

    The slice keeps all ``T`` tokens and ``d`` and takes ``f / slices`` of the ffn width: every GEMM,
    weight, gradient and optimizer state of the block is cut along ``f``, so one sliced step is
    ``1/slices`` of the full step's arithmetic and bytes (plus one [T, d] dX output per slice).  The
    full step's time is taken as ``slices`` sliced steps, each of which is actually run and timed.
    """

    def __init__(self, d, f, tokens, slices=REF_SLICES, threads=None):
        import torch

        from oracle import ref_torch as R

        self.torch, self.R = torch, R
        self.threads = threads or os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.d, self.f, self.tokens, self.slices = d, f, tokens, slices
        fs = max(f // slices, 1)
        self.fs = fs
        g = torch.Generator().manual_seed(0)

        def qweight(o, k):
            w = torch.randn(o, k, generator=g) * 0.02
            s = w.abs().amax(dim=1).clamp_min(1e-8) / 127.0
            return torch.round(w / s.unsqueeze(1)).clamp(-127, 127).to(torch.int8), s

        q_gu, s_gu = qweight(2 * fs, d)
        q_d, s_d = qweight(d, fs)
        self.block = R.SwiGLUBlock(q_gu, s_gu, q_d, s_d)
        self.x = torch.randn(tokens, d, generator=g).to(torch.bfloat16).requires_grad_(True)
        self.dy = torch.randn(tokens, d, generator=g).to(torch.bfloat16)
        self.times: list[float] = []

    def step(self, record=True) -> float:
        t0 = time.perf_counter()
        self.block.train_step(self.x, self.dy, lr=1e-3, wd=0.01)
        dt = time.perf_counter() - t0
        self.x.grad = None
        if record:
            self.times.append(dt)
        return dt

    def full_step_seconds(self) -> float:
        return statistics.mean(self.times) * self.f / self.fs

    def describe(self) -> str:
        return (f"reference path (oracle.ref_torch: bf16 dequant + torch.matmul fwd/bwd, FireFlyOptim bit-module "
                f"update in torch ops) on a 1/{self.f // self.fs} width slice of the block (f {self.fs} of {self.f}, "
                f"T={self.tokens}, d={self.d}); {len(self.times)} timed sliced steps of "
                f"{statistics.mean(self.times):.3f}s each (after a warm-up step), full step = "
                f"{self.f / self.fs:.2f} x sliced step; torch.set_num_threads({self.threads})")


def cpu_reference_baseline(d, f, tokens, steps=3):
    """The reference's CPU path on all host threads, and on one thread (a narrower slice)."""
    import torch

    prev = torch.get_num_threads()
    try:
        m = RefCpuSample(d, f, tokens)
        m.step(record=False)
        for _ in range(steps):
            m.step()
        full = m.full_step_seconds()
        one = RefCpuSample(d, f, tokens, slices=REF_SLICES * 8, threads=1)
        one.step(record=False)
        for _ in range(2):
            one.step()
        full1 = one.full_step_seconds()
    finally:
        torch.set_num_threads(prev)
    return {"value": tokens / full, "unit": "tokens/s", "cores": m.threads, "kind": "port",
            "sample": m.describe(),
            "one_thread": {"value": tokens / full1, "unit": "tokens/s", "cores": 1, "sample": one.describe()}}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    """The reference's CPU implementation of the step on all host cores; under torchrun only rank 0
    works (the other ranks exit without work).  Each step is one sliced step of ``RefCpuSample``;
    ``steps`` in the line is the number of sliced steps actually timed."""
    if rank != 0:
        return
    d, f, T = args.d_model, args.ffn, args.tokens
    m = RefCpuSample(d, f, T)
    budget_s, t_start, done = 240.0, time.perf_counter(), 0
    for i in range(args.warmup + args.steps):
        timed = i >= args.warmup
        m.step(record=timed)
        done += int(timed)
        if timed and done >= 2 and time.perf_counter() - t_start > budget_s:
            break
    est = m.full_step_seconds()
    sample = m.describe()
    if done < args.steps:
        sample += f"; stopped after {done} of {args.steps} timed steps at the {budget_s:.0f}s budget"
    value = T / est
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": done, "steps_requested": args.steps, "warmup": args.warmup, "ms_per_step": est * 1e3,
        "sliced_ms_per_step": statistics.mean(m.times) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"swiglu_mlp_train_step T={T}/GPU d={d} f={f} (BitLinear fwd+bwd + 8-bit DQT AdamW)",
                   "tokens_per_gpu": T, "parallelism": "cpu (rank 0 only)"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": m.threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU sub-benchmarks
# ---------------------------------------------------------------------------
def _time_cuda(fn, iters, warm=3, flush=None, spacer_us=300.0):
    """Median CUDA-event time of ``fn`` on the device.  Before each timed launch the stream gets
    the L2 flush (if any) and a spin of ``spacer_us`` microseconds, queued ahead of the start
    event, so that the host-side work of ``fn`` (argument checks, tensor-map encoding, ctypes)
    overlaps that spin instead of sitting between the two events."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    clock_khz = torch.cuda.get_device_properties(torch.cuda.current_device()).clock_rate
    spin = int(spacer_us * clock_khz / 1e3)
    times = []
    for _ in range(iters):
        if flush is not None:
            flush()
        if spin > 0:
            torch.cuda._sleep(spin)
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

    # L2 flush between timed launches: write a buffer twice the size of L2, then read another one,
    # so that L2 holds only clean lines of unrelated data (no write-back of the flush's own dirty
    # lines lands on the timed kernel)
    flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    clean_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def l2_flush():
        flush_buf.zero_()
        clean_buf.sum()

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
                       flush=l2_flush)
        ops = 2 * M * N * K
        byts = M * K + N * K + 2 * M * N + 4 * (M + N)
        res.append({"M": M, "N": N, "K": K, "us": round(t * 1e6, 2), "tops": round(ops / t / 1e12, 1),
                    "hbm_gbs": round(byts / t / 1e9, 1)})
        # the cuBLASLt int8 comparator (the substitute for the reference's bitsandbytes igemmlt path,
        # fireflykernels.py:132-156) through torch._int_mm (int32 out), same operands
        try:
            bt = b.t()
            if M >= 17:
                tl = _time_cuda(lambda: torch._int_mm(a, bt), 10, flush=l2_flush)
                res[-1]["comparator"] = "cuBLASLt int8 via torch._int_mm (substitute for bitsandbytes igemmlt)"
                res[-1]["torch_int_mm_us"] = round(tl * 1e6, 2)
                res[-1]["torch_int_mm_tops"] = round(ops / tl / 1e12, 1)
        except Exception as e:  # noqa: BLE001
            res[-1]["torch_int_mm"] = f"unavailable: {type(e).__name__}"
        del a, b, out
    del flush_buf, clean_buf
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


ZERO1_CHECK_SHAPES = [(256, 192), (128, 256), (96, 128)]  # (out, in): a chain 192 -> 256 -> 128 -> 96


def zero1_parity_check(dev, world: int, rank: int, steps: int = 3) -> dict:
    """Multi-GPU correctness beside the multi-GPU speed: three ZeRO-1 steps of a small BitLinear chain
    (two gradient buckets, reduce-scatters issued from the backward, the DQT kernel on each rank's
    shard, per-bucket all-gathers) against an unsharded ``FireFlyOptim`` replay on rank 0 fed the
    same averaged gradients (the reduce-scatter outputs, gathered).  Each rank trains on its own
    tokens.  ``ok`` means the int8 weights and the gathered 8-bit states (the reference's
    ``bit_state`` layout) are bit-identical.  Collective: every rank calls it."""
    import torch
    import torch.distributed as dist

    from firefly_b200.bitLinear import BitLinear
    from firefly_b200.distributed import ZeroFireFlyOptim
    from firefly_b200.fireflykernels import _BIT_GRAD_CACHE
    from firefly_b200.fireflyoptim import FireFlyOptim

    torch.manual_seed(0)
    mods = [BitLinear(k, o).to(dev) for o, k in ZERO1_CHECK_SHAPES]
    opt = ZeroFireFlyOptim(mods, lr=1e-3, weight_decay=0.01, seed=5, bucket_mb=0.05, overlap=True)
    opt.keep_reduced_grad = True  # peer mode: the averaged gradient of each shard, for the replay
    path = "peer" if opt.peer else "collectives"
    plan = opt.plan
    gen = torch.Generator(device=dev).manual_seed(123 + rank)
    averaged = []
    for _ in range(steps):
        x = torch.randn(64, ZERO1_CHECK_SHAPES[0][1], device=dev, generator=gen).requires_grad_(True)
        y = mods[2](mods[1](mods[0](x)))
        y.float().pow(2).mean().backward()
        opt.step()
        full = torch.empty(plan.shard * world, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(full, opt.g_shard)
        averaged.append(plan.to_arena(full))
    bits = opt.gather_bit_state()
    q_sharded = [m.int_weight.clone() for m in mods]
    opt.close()
    if rank != 0:
        return {"checked_on": "rank 0"}
    torch.manual_seed(0)
    ref = [BitLinear(k, o).to(dev) for o, k in ZERO1_CHECK_SHAPES]
    ropt = FireFlyOptim([torch.nn.Parameter(torch.zeros(1, device=dev))], lr=1e-3, weight_decay=0.01,
                        bit_modules=ref)
    ropt.rng_seed = opt.rng_seed
    for g in averaged:
        for m, off in zip(ref, plan.offsets):
            _BIT_GRAD_CACHE[m._registered_handle] = g[off:off + m.int_weight.numel()].view(m.int_weight.shape).clone()
        ropt.step()
    ok = all(torch.equal(a, b.int_weight) for a, b in zip(q_sharded, ref))
    for m_z, m_r in zip(mods, ref):
        want = ropt._bit_state[m_r._registered_handle]
        got = bits[m_z._registered_handle]
        for k, v in got.items():
            w = want[k]
            ok = ok and (torch.equal(v, w.cpu()) if torch.is_tensor(v) else v == w)
    return {"ok": bool(ok), "world": world, "steps": steps, "buckets": len(plan.buckets), "path": path,
            "what": ("ZeRO-1 (peer: one kernel per shard reads every rank's gradient and writes every rank's "
                     "weights over NVLink; collectives: overlapped bucketed NCCL reduce-scatters, sharded DQT "
                     "update, all-gathers) vs an unsharded FireFlyOptim replay on the same averaged gradients: "
                     "int8 weights and gathered bit_state bit-identical")}


def zero_peer(args):
    return None if args.zero_peer == "auto" else args.zero_peer == "1"


def decoder_dp_bench(dev, world: int, rank: int, steps: int, warmup: int, seqs: int = 64, seq: int = 2048,
                     micro: int = 8, bucket_mb: float = 256.0, overlap: bool = True, peer: bool | None = None):
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
                           eps=1e-8, weight_decay=0.01, seed=11, bucket_mb=bucket_mb, overlap=overlap, peer=peer)
    batches = synthetic_batches(cfg, per_rank, seq, min(micro, per_rank), dev, seed=1000 + rank)
    for _ in range(max(warmup, 1)):
        train_step(model, opt, batches)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    opt.comm_events = []  # device time of the optimizer step and of its communication phases
    host_step = 0.0
    e0.record()
    for _ in range(steps):
        h0 = time.perf_counter()
        loss = train_step(model, opt, batches)
        host_step += time.perf_counter() - h0
    e1.record()
    torch.cuda.synchronize()
    sec = torch.tensor([e0.elapsed_time(e1) / 1e3], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(sec, op=dist.ReduceOp.MAX)
    sec = float(sec.item())
    phases = ["optimizer_step", "peer_update", "peer_fence_wait", "dense_all_reduce_wait", "reduce_scatter_wait",
              "all_gather_wait"]
    per = {k: 0.0 for k in phases}
    for k, a, b in opt.comm_events:
        per[k] += a.elapsed_time(b) / steps
    opt.comm_events = None
    per["host_train_step"] = host_step / steps * 1e3
    pt = torch.tensor([per[k] for k in per], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
    per = {k: round(v, 3) for k, v in zip(per, pt.tolist())}
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
        "zero1_path": "peer" if getattr(opt, "peer", False) else ("collectives" if world > 1 else "local"),
        "phases_ms_per_step": per,
        "phases_method": ("CUDA events on the compute stream, mean per step, max over ranks: optimizer_step = "
                          "the whole step() on the device (the rest of ms_per_step is the micro-batches' forward "
                          "and backward), the other device phases are parts of it; host_train_step = host wall "
                          "time of one train_step call (launch side)"),
    }
    del model, opt, batches
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# The reference's algorithm on the same GPU (torch eager), and the bitsandbytes probe
# ---------------------------------------------------------------------------
def bitsandbytes_probe():
    """Whether the reference's dead cuBLASLt path (bitsandbytes ``igemmlt``, fireflykernels.py:132-156)
    could run here."""
    try:
        import bitsandbytes
        import bitsandbytes.functional as bnbf
    except Exception as e:  # noqa: BLE001
        return {"importable": False, "reason": f"{type(e).__name__}: {e}"}
    return {"importable": True, "version": getattr(bitsandbytes, "__version__", None),
            "igemmlt": hasattr(bnbf, "igemmlt")}


class _EagerBitLinearFn:
    """BitLinear as the reference computes it on the GPU (fireflykernels.py:164-210): the int8 weight
    dequantised to bf16 and ``torch.matmul`` for y, dX and dW; dW added into a per-layer cache."""

    @staticmethod
    def make():
        import torch

        class Fn(torch.autograd.Function):
            @staticmethod
            def forward(ctx, x, q, s, cache, key):
                xb = x.to(torch.bfloat16)
                y = torch.matmul(xb, (q.to(torch.bfloat16) * s.to(torch.bfloat16).unsqueeze(1)).t())
                ctx.save_for_backward(xb, q, s)
                ctx.cache, ctx.key = cache, key
                return y

            @staticmethod
            def backward(ctx, go):
                xb, q, s = ctx.saved_tensors
                go = go.to(torch.bfloat16)
                w = q.to(torch.bfloat16) * s.to(torch.bfloat16).unsqueeze(1)
                gi = torch.matmul(go, w)
                gw = torch.matmul(go.t(), xb)
                prev = ctx.cache.get(ctx.key)
                if prev is None:
                    ctx.cache[ctx.key] = gw
                else:
                    prev.add_(gw)
                return gi, None, None, None, None

        return Fn


def _eager_codec(torch, x, signed, bs=256):
    """The reference's mu-law blockwise encode (fireflyoptim.py:22-67) in torch ops."""
    flat = x.float().contiguous().view(-1)
    nb = (flat.numel() + bs - 1) // bs
    if nb * bs > flat.numel():
        flat = torch.cat([flat, flat.new_zeros(nb * bs - flat.numel())])
    blocks = flat.view(nb, bs)
    if signed:
        absmax = blocks.abs().amax(dim=1).clamp_min(1e-12)
        n = (blocks / absmax.unsqueeze(1)).clamp(-1.0, 1.0)
        c = torch.round(torch.sign(n) * torch.log1p(255.0 * n.abs()) * (1.0 / 5.545177444479562) * 127.0)
        q = (c.clamp(-127, 127).to(torch.int16).view(-1)[: x.numel()] + 128).to(torch.uint8)
    else:
        absmax = blocks.amax(dim=1).clamp_min(1e-12)
        n = (blocks / absmax.unsqueeze(1)).clamp(0.0, 1.0)
        c = torch.round(torch.log1p(255.0 * n) * (1.0 / 5.545177444479562) * 255.0)
        q = c.clamp(0, 255).view(-1)[: x.numel()].to(torch.uint8)
    return q.view_as(x), absmax


def _eager_decode(torch, q, absmax, signed, bs=256):
    """The reference's mu-law blockwise decode (fireflyoptim.py:39-80) in torch ops (``q.numel()`` a
    multiple of the block, as the benchmark's weights are)."""
    blocks = q.contiguous().view(-1, bs).float()
    if signed:
        y = ((blocks - 128.0) / 127.0).clamp(-1.0, 1.0)
        n = torch.sign(y) * (torch.exp(y.abs() / (1.0 / 5.545177444479562)) - 1.0) / 255.0
    else:
        y = (blocks / 255.0).clamp(0.0, 1.0)
        n = (torch.exp(y / (1.0 / 5.545177444479562)) - 1.0) / 255.0
    return (n * absmax.unsqueeze(1)).view_as(q)


def _eager_dqt_step(torch, q, s, g, st, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.01, sr=0.15):
    """``FireFlyOptim.step``'s bit-module update (fireflyoptim.py:163-209) in torch ops, with the
    reference's ``torch.any`` host synchronisation and ``torch.rand_like`` draw."""
    g = g.float()
    m = _eager_decode(torch, st["m_q"], st["m_a"], True)
    v = _eager_decode(torch, st["v_q"], st["v_a"], False)
    r = _eager_decode(torch, st["r_q"], st["r_a"], True)
    st["t"] += 1
    m.mul_(b1).add_(g, alpha=1.0 - b1)
    v.mul_(b2).addcmul_(g, g, value=1.0 - b2)
    adam = (m / (1.0 - b1 ** st["t"])) / ((v / (1.0 - b2 ** st["t"])).sqrt() + eps)
    ws = s.float().unsqueeze(1).clamp_min(eps)
    r = r + (-lr * (adam + wd * q.float() * ws)) / ws
    mag = r.abs()
    whole = torch.floor(mag)
    thr = (mag - whole + torch.tanh(adam) * sr * torch.sign(r)).clamp(0.0, 1.0)
    dq = (torch.sign(r) * (whole + (torch.rand_like(thr) < thr).float())).to(torch.int32)
    if torch.any(dq != 0):
        q.copy_((q.to(torch.int16) + dq.to(torch.int16)).clamp_(-127, 127).to(torch.int8))
        r = r - dq.float()
    st["r_q"], st["r_a"] = _eager_codec(torch, r, True)
    st["m_q"], st["m_a"] = _eager_codec(torch, m, True)
    st["v_q"], st["v_a"] = _eager_codec(torch, v, False)


def reference_algorithm_on_gpu(dev, d, f, T, steps=5, warmup=2):
    """The benchmark step computed the reference's way on the same B200: torch eager ops (bf16
    dequantisation + cuBLAS bf16 matmuls for the BitLinear layers, torch's silu, and the ~40-op
    torch update of ``FireFlyOptim`` per layer), none of this repository's kernels.  CUDA-event
    time over ``steps`` steps after ``warmup``."""
    import torch
    import torch.nn.functional as F

    Fn = _EagerBitLinearFn.make()
    g = torch.Generator(device=dev).manual_seed(0)

    def qweight(o, k):
        w = torch.randn(o, k, device=dev, generator=g) * 0.02
        sc = w.abs().amax(dim=1).clamp_min(1e-8) / 127.0
        return torch.round(w / sc.unsqueeze(1)).clamp(-127, 127).to(torch.int8), sc

    layers = [qweight(2 * f, d), qweight(d, f)]
    states = []
    for q, _ in layers:
        z = torch.zeros(q.shape, device=dev)
        mq, ma = _eager_codec(torch, z, True)
        vq, va = _eager_codec(torch, z, False)
        states.append({"t": 0, "m_q": mq, "m_a": ma, "v_q": vq, "v_a": va, "r_q": mq.clone(), "r_a": ma.clone()})
    xs = [torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True) for _ in range(2)]
    dy = torch.randn(T, d, device=dev, generator=g).to(torch.bfloat16)
    cache: dict = {}

    def step(x):
        gu = Fn.apply(x, *layers[0], cache, 0)
        y = Fn.apply(F.silu(gu[:, :f]) * gu[:, f:], *layers[1], cache, 1)
        y.backward(dy)
        x.grad = None
        with torch.no_grad():
            for i, (q, sc) in enumerate(layers):
                _eager_dqt_step(torch, q, sc, cache.pop(i), states[i])

    for i in range(warmup):
        step(xs[i % 2])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        step(xs[i % 2])
    e1.record()
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / steps
    del layers, states, xs, dy, cache
    torch.cuda.empty_cache()
    return {"tokens_per_s": T / sec, "ms_per_step": sec * 1e3, "steps": steps, "warmup": warmup,
            "what": ("the reference's live algorithm on this GPU in torch eager ops: BitLinear as bf16 "
                     "dequantisation + torch.matmul (fireflykernels.py:164-210), torch silu, FireFlyOptim's "
                     "bit-module update as torch ops with torch.rand_like (fireflyoptim.py:136-209); "
                     "CUDA-event time")}


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
                           bucket_mb=args.zero_bucket_mb, overlap=bool(args.zero_overlap), peer=zero_peer(args))
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
    opt.comm_events = [] if world > 1 else None
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
    comm = None
    if world > 1:  # the compute stream's waits for the collectives (their exposed part), per step
        phases = ["reduce_scatter_wait", "dense_all_reduce_wait", "all_gather_wait", "peer_fence_wait",
                  "peer_update", "optimizer_step"]
        per = {k: 0.0 for k in phases}
        for k, a, b in opt.comm_events:
            per[k] += a.elapsed_time(b) / args.steps
        opt.comm_events = None
        pt = torch.tensor([per[k] for k in phases], dtype=torch.float64, device=dev)
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        per = dict(zip(phases, pt.tolist()))
        comm = {"zero1_path": "peer" if opt.peer else "collectives",
                "exposed_ms_per_step": (per["reduce_scatter_wait"] + per["dense_all_reduce_wait"] + per["all_gather_wait"]
                                        + per["peer_fence_wait"]),
                "by_phase_ms_per_step": per,
                "method": "CUDA events on the compute stream around each wait for a collective in the optimizer "
                          "step (time the stream stood still for communication), mean per step, max over ranks; "
                          "peer_update = the fused update kernels of peer mode (their NVLink reads and writes "
                          "overlap the update arithmetic); optimizer_step = the whole step() on the device"}

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
                                                  bucket_mb=args.zero_bucket_mb, overlap=bool(args.zero_overlap),
                                                  peer=zero_peer(args))
    if world > 1:
        sub["zero1_parity"] = zero1_parity_check(dev, world, rank)
    if rank == 0 and world == 1 and not args.no_sub:
        sub["int8_gemm_sweep"] = gemm_sweep(dev)
        sub["adamw8"] = adamw_bench(dev, args.adamw_params, peaks["hbm_gbs"])
        sub["dense_adamw8"] = dense_adamw_bench(dev, 268435456, peaks["hbm_gbs"])
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        ref = reference_algorithm_on_gpu(dev, d, f, T)
        ref["bitsandbytes"] = bitsandbytes_probe()
        sub["reference_on_b200"] = ref
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_baseline(d, f, T)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens_total = T * world * args.steps
    value = tokens_total / sec
    ms_per_step = sec / args.steps * 1e3
    int8_peak = NOMINAL_INT8_TOPS
    avg_ms = sum(g_ms) / max(len(g_ms), 1)
    avg_ops = sum(g_ops) / max(len(g_ops), 1)
    achieved = avg_ops / (avg_ms / 1e3) / 1e12 if g_ms else None
    gemm_share = sum(g_ms) / 1e3 / sec if g_ms else None  # this rank's GEMM time / the step time
    mm = [r for r in sub.get("int8_gemm_sweep", []) if r["M"] == 8192 and "torch_int_mm_tops" in r]
    int8_burst = mm[0]["torch_int_mm_tops"] if mm else None
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
            "zero1": {"bucket_mb": args.zero_bucket_mb, "overlap": bool(args.zero_overlap), "peer": args.zero_peer},
            "l2": "inputs larger than L2 (step working set > 126 MB)",
        },
        "e2e": {"value": T * world * e2e_steps / e2e_sec, "unit": "tokens/s",
                "h2d_bytes_per_step": int(xh.numel() * xh.element_size()), "d2h_bytes_per_step": 4,
                "host_cpus_per_rank": bound_cpus},
        "gpu_launches": launches,
        "comm": comm,
        "roofline": {
            "kernel": "ff_gemm_i8 (tcgen05 kind::i8)", "bound": "tensor",
            "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s", "frac": achieved / int8_peak if achieved else None,
            "traffic": load_traffic().get("ff_gemm_i8 swiglu_mlp_train_step", {}).get("bytes_per_launch"),
            "traffic_algorithmic": alg_bytes / max(len(g_ms), 1) if g_ms else None,
            "peak_kind": "nominal dense int8 (4.5 POPS)",
            "frac_of_2x_measured_bf16_burst": (achieved / (2.0 * peaks["bf16_tflops"]) if achieved else None),
            "int8_burst_measured_cublaslt": int8_burst,
            "frac_of_int8_burst_measured": (achieved / int8_burst if achieved and int8_burst else None),
            "note": ("int8 ops (2*M*N*K) per launch / mean CUDA-event launch time in the timed region; peak = "
                     "the nominal dense int8 rate; beside it 2 x the measured cuBLAS bf16 burst "
                     f"({2.0 * peaks['bf16_tflops']:.0f}, MEASURED_PEAKS.json) and the cuBLASLt int8 rate "
                     "measured here (torch._int_mm at 8192^3, int32 output, in int8_gemm_sweep)"
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
    ref = sub.get("reference_on_b200")
    if ref:
        ref["ours_over_reference"] = value / ref["tokens_per_s"]
        ref["ours_e2e_over_reference"] = line["e2e"]["value"] / ref["tokens_per_s"]
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""nanoGPT fwd+VJP (value_and_grad) tokens/s on B200.

Workload (weak scaling, one process per GPU): every rank runs the
nanoGPT-char value_and_grad step -- 6 layers, 6 heads, d_model 384, block 256,
vocab 65, batch 64, pre-LN, GELU MLP 4x, causal attention, cross-entropy --
on its own batch of 64 x 256 token ids, bf16 parameters (fp32 accumulation),
through the executor's C ABI (`<module>.value_and_grad`). With N > 1 ranks the
loss and gradients are averaged over NVLink by NCCL inside the step.

Inputs are synthetic and seeded: parameters N(0, 0.02) (layer-norm gains 1),
token ids uniform in [0, 65), mirroring init-gpt-params and random-randint.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sheaf_b200|reference]

`--config gpt2` runs GPT-2-small instead (12L/12H/768, T=1024, V=50304,
batch 8 per GPU); `--dtype f32` the fp32 step; `--strong` splits the
reference's global batch of 64 over the GPUs instead of giving every GPU its
own (strong scaling). The line's `roofline` is the step's fc GEMM with its
GELU epilogue timed alone; `kernels` lists the step's main kernels likewise.

Prints one JSON line on rank 0. `--sample` instead times autoregressive
sampling (generate-token + slide-window, 256 new tokens from a one-token
prompt, batch 1 and 32, bf16, temperature 1.0 over the whole vocabulary) on
one GPU and prints one line per batch size.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "nanoGPT fwd+VJP tokens/sec"
UNIT = "tokens/s"
# nanoGPT-char (the headline workload) and GPT-2-small (the data-parallel
# workload: 12L/12H/768, T=1024, V=50304, global batch 64 = 8 per GPU at 8 GPUs)
CONFIGS = {
    "nanogpt": dict(n_layer=6, n_head=6, n_embd=384, block_size=256, vocab_size=65, batch=64, seq=256),
    "gpt2": dict(n_layer=12, n_head=12, n_embd=768, block_size=1024, vocab_size=50304, batch=8, seq=1024),
}
CFG = CONFIGS["nanogpt"]
WORKLOAD = {
    "nanogpt": "nanoGPT-char value_and_grad 6L/6H/384 T=256 V=65",
    "gpt2": "GPT-2-small value_and_grad 12L/12H/768 T=1024 V=50304",
}
# global batch of the strong-scaling line (the reference's own batch)
STRONG_GLOBAL = {"nanogpt": 64, "gpt2": 64}
BF16 = 0x22000010
F32 = 0x21000020
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the nanoGPT
# fc GEMM with its GELU epilogue (13.8 MB read: A and B once; 41.5 MB of the
# 100.7 MB of gelu(u) and gelu'(u) written reach DRAM during the launch)
FC_GELU_DRAM_BYTES = {"nanogpt": 55.3e6}
# FP32 CUDA-core peak, nominal: 148 SMs x 128 lanes x 2 flops x 1.965 GHz
FP32_NOMINAL_TFLOPS = 74.4


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def model_flops_per_token(c=CFG) -> float:
    """6*N_mm + 12*L*T*D (matmul params incl. LM head; full T x T attention)."""
    L, D, V, T = c["n_layer"], c["n_embd"], c["vocab_size"], c["seq"]
    n_mm = L * 12 * D * D + V * D
    return 6.0 * n_mm + 12.0 * L * T * D


def leaf_shapes(c=CFG):
    L, D, V, P = c["n_layer"], c["n_embd"], c["vocab_size"], c["block_size"]
    s = [(V, D)]
    for _ in range(L):
        s += [(3 * D, D), (D, D), (D,), (D,), (4 * D, D), (D, 4 * D)]
    return s + [(D,), (P, D), (V, D)]


def synthetic_inputs(seed: int, c=CFG):
    rng = np.random.default_rng(seed)
    leaves = []
    for shp in leaf_shapes(c):
        leaves.append(np.ones(shp, np.float32) if len(shp) == 1 else
                      (rng.standard_normal(shp, dtype=np.float32) * np.float32(0.02)))
    x = rng.integers(0, c["vocab_size"], (c["batch"], c["seq"])).astype(np.float32)
    y = rng.integers(0, c["vocab_size"], (c["batch"], c["seq"])).astype(np.float32)
    return leaves, x, y


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []
        self.start = 0  # samples taken before the timed region

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a moment to start (longer with one per rank):
            # wait for its first sample so that the timed region, tens of ms
            # long, is sampled
            t0 = time.perf_counter()
            while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 5.0:
                time.sleep(0.005)
            self.start = len(self.lines)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # the samples taken during the region, else the last one before it
        lines = self.lines[self.start:] or self.lines[-1:]
        for ln in lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def allmax(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# --------------------------------------------------------------------------
# CPU baseline: the oracle (numpy restatement of the reference math)
# --------------------------------------------------------------------------

def _oracle_cfg(c):
    from oracle import models

    return models.GPTConfig(n_layer=c["n_layer"], n_head=c["n_head"], n_embd=c["n_embd"],
                            block_size=c["block_size"], vocab_size=c["vocab_size"], batch=c["batch"], seq=c["seq"])


def _cpu_batch(name: str, c) -> int:
    """Sequences per CPU step: the whole batch for nanoGPT-char (a few seconds
    on the host cores), one sequence of GPT-2-small's eight."""
    return c["batch"] if name == "nanogpt" else 1


def _cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample(name: str, c, dtype: str, target_s: float = 15.0):
    """Times the oracle's fwd+VJP (numpy, BLAS on every host core) on a
    bounded sample of the workload. Returns (tokens/s, cores, sample)."""
    from oracle import models

    batch = _cpu_batch(name, c)
    cc = dict(c, batch=batch)
    cfg = _oracle_cfg(cc)
    leaves, x, y = synthetic_inputs(0, cc)
    npdt = np.float32
    models.gpt_value_and_grad(leaves, x[:1, :64], y[:1, :64], _oracle_cfg(dict(c, batch=1, seq=64)), dtype=npdt)
    t0 = time.perf_counter()
    n = 0
    while True:
        models.gpt_value_and_grad(leaves, x, y, cfg, dtype=npdt)
        n += 1
        el = time.perf_counter() - t0
        if el >= target_s or n >= 20:
            break
    tok = n * batch * c["seq"] / el
    cores = _cpu_threads()
    return tok, cores, (f"{n} x fp32 numpy oracle fwd+VJP steps of batch {batch} (of {c['batch']}) x {c['seq']} "
                        f"tokens, same model; BLAS on {cores} threads of {cpu_model()}")


REF_BUDGET_S = 200.0  # host seconds the reference arm's timed steps may take


def run_reference(args, world, rank):
    """Reference arm: the reference's own math on the host cores (the oracle
    port; the reference's IREE llvm-cpu path cannot be built here). Rank 0
    alone runs it."""
    if rank != 0:
        return
    from oracle import models

    name, c = args.config, CONFIGS[args.config]
    batch = _cpu_batch(name, c)
    cc = dict(c, batch=batch)
    cfg = _oracle_cfg(cc)
    leaves, x, y = synthetic_inputs(0, cc)
    t0 = time.perf_counter()
    for _ in range(max(1, min(args.warmup, 1))):
        models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float32)
    per_seq = (time.perf_counter() - t0) / batch
    # Each step is the whole batch unless K such steps would take longer than
    # REF_BUDGET_S: then the largest halving of it whose K steps fit.
    while batch > 1 and batch % 2 == 0 and args.steps * per_seq * batch > REF_BUDGET_S:
        batch //= 2
    if batch != cc["batch"]:
        cc = dict(c, batch=batch)
        cfg = _oracle_cfg(cc)
        x, y = x[:batch], y[:batch]
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float32)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    v = args.steps * batch * c["seq"] / tot
    cores = _cpu_threads()
    sample = (f"each step: fp32 numpy oracle fwd+VJP of batch {batch} (of {c['batch']}) x {c['seq']} tokens, "
              f"{WORKLOAD[name]}; BLAS on {cores} threads of {cpu_model()}")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD[name], "global_batch": batch, "seq_len": c["seq"],
                       "parallelism": "host cores", "cpu": cpu_model(), "threads": cores},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# B200 arm
# --------------------------------------------------------------------------

def _rotated_ms(launch, copies: int, reps: int, st) -> float:
    """Average ms per launch of launch(i) for i over `copies` operand sets,
    launched back to back between two CUDA events on stream `st` (so no launch
    finds its operands left in L2 by the previous one); mean of `reps` rounds
    after 3 warm-up launches."""
    import torch

    for i in range(3):
        launch(i)
    out = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(copies):
            launch(i)
        e1.record(st)
        st.synchronize()
        out.append(e0.elapsed_time(e1) / copies)
    return sum(out) / len(out)


def measure_step_kernels(session, c, elem, reps: int = 5):
    """Times the step's own kernels alone, at the step's shapes and with the
    epilogues the plan uses, with CUDA events on the session stream: the fc
    GEMM with its GELU epilogue (both outputs), the fc weight-gradient GEMM
    (dU^T h2 over every token, split-K with its reduction), the attention
    forward and VJP, the layer-norm forward and VJP, the cross-entropy. Each
    is launched back to back over enough operand sets to exceed L2.
    Returns one dict per kernel (ms, algorithmic work, achieved, bound)."""
    import torch

    import sheaf_b200 as sb

    L = sb.lib()
    bf = elem == BF16
    dt = torch.bfloat16 if bf else torch.float32
    es = 2 if bf else 4
    N, D, H, T, B, V = c["batch"] * c["seq"], c["n_embd"], c["n_head"], c["seq"], c["batch"], c["vocab_size"]
    Hd = D // H
    ldl = (V + 7) // 8 * 8
    dev = torch.device(f"cuda:{session.device}")
    st = torch.cuda.ExternalStream(session.stream, device=dev)
    sp = session.stream
    res = []

    def nsets(bytes_per_set):
        return max(2, min(16, int(1.2e9 // max(bytes_per_set, 1))))

    def add(name, kernel, ms, work, unit, bound):
        res.append({"kernel": name, "template": kernel, "ms": ms, "work": work, "bound": bound,
                    "achieved": work / (ms / 1e3) / (1e12 if unit == "TFLOP/s" else 1e9), "unit": unit})

    with torch.cuda.stream(st):
        r = lambda *shape: torch.randn(*shape, device=dev).to(dt)  # noqa: E731
        # fc GEMM + GELU epilogue: u = h2 W_fc^T; gelu(u), gelu'(u) stored
        k = nsets(N * D * es + 4 * D * D * es + 2 * N * 4 * D * es)
        sets = [(r(N, D), r(4 * D, D), torch.empty(N, 4 * D, device=dev, dtype=dt),
                 torch.empty(N, 4 * D, device=dev, dtype=dt)) for _ in range(k)]

        fws = L.sb_op_matmul_workspace_size(elem, 0, 1, N, 4 * D, D)
        fwsb = torch.empty(max(fws // 4, 1), device=dev)

        def fc(i):
            a, w, g, gd = sets[i % k]
            if bf:
                assert L.sb_op_matmul_gelu(elem, a.data_ptr(), D, w.data_ptr(), D, N, 4 * D, D, g.data_ptr(),
                                           gd.data_ptr(), 4 * D, sp) == 0
            else:  # the fp32 plan's fc GEMM: bf16x6 on the tensor cores (its GELU is a separate f32 pass)
                assert L.sb_op_matmul(elem, a.data_ptr(), D, 0, w.data_ptr(), D, 1, N, 4 * D, D, g.data_ptr(),
                                      4 * D, elem, fwsb.data_ptr(), fws, sp) == 0
        add("fc GEMM + GELU epilogue" if bf else "fc GEMM (bf16x6 split on the tensor cores)",
            "gemm_tc_kernel<256,0,0,5,1>" if bf else "split6_kernel + gemm_tc_kernel (K' = 6K, split-K)",
            _rotated_ms(fc, k, reps, st), 2.0 * N * D * 4 * D, "TFLOP/s", "tensor")
        del sets, fwsb
        # fc weight gradient: dW_fc [4D, D] = dU^T [4D, N] h2 [N, D]
        wsb = L.sb_op_matmul_workspace_size(elem, 1, 0, 4 * D, D, N)
        ws = torch.empty(max(wsb // 4, 1), device=dev)
        k = nsets(N * 4 * D * es + N * D * es)
        sets = [(r(N, 4 * D), r(N, D), torch.empty(4 * D, D, device=dev, dtype=dt)) for _ in range(k)]

        def dw(i):
            du, h2, o = sets[i % k]
            assert L.sb_op_matmul(elem, du.data_ptr(), 4 * D, 1, h2.data_ptr(), D, 0, 4 * D, D, N, o.data_ptr(), D,
                                  elem, ws.data_ptr(), wsb, sp) == 0
        add("fc weight-gradient GEMM (+ split-K reduction)", "gemm_tc_kernel<384,1,1,4,1> + splitk_reduce_kernel"
            if bf else "split6_kernel + gemm_tc_kernel (K' = 6K, split-K)", _rotated_ms(dw, k, reps, st),
            2.0 * N * D * 4 * D, "TFLOP/s", "tensor")
        del sets, ws
        # attention forward and VJP (causal: half the dense T x T work)
        wsb = L.sb_op_attention_bwd_workspace_size(elem, B, T, H, Hd)
        ws = torch.empty(wsb // 4 + 1, device=dev)
        k = nsets(N * 3 * D * es * 2 + N * D * es * 3)
        sets = [(r(N, 3 * D), torch.empty(N, D, device=dev, dtype=dt), r(N, D),
                 torch.empty(N, 3 * D, device=dev, dtype=dt), torch.empty(B * H * T, device=dev)) for _ in range(k)]

        def afwd(i):
            q, o, do, dq, lse = sets[i % k]
            assert L.sb_op_attention_fwd(elem, q.data_ptr(), o.data_ptr(), lse.data_ptr(), B, T, H, Hd, sp) == 0

        def abwd(i):
            q, o, do, dq, lse = sets[i % k]
            assert L.sb_op_attention_bwd(elem, q.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                                         dq.data_ptr(), ws.data_ptr(), wsb, B, T, H, Hd, sp) == 0
        causal = 2.0 * B * H * T * T * Hd  # QK^T + PV over the lower triangle
        for i in range(k):
            afwd(i)  # real O and lse for the VJP
        add("attention forward", "attn_fwd_tc" if bf else "attn_fwd_simt", _rotated_ms(afwd, k, reps, st), causal,
            "TFLOP/s", "tensor" if bf else "fp32 FFMA")
        add("attention VJP", "attn_bwd_tc + dq_convert_kernel" if bf else "attn_bwd_simt",
            _rotated_ms(abwd, k, reps, st), 2.5 * causal, "TFLOP/s", "tensor" if bf else "fp32 FFMA")
        del sets, ws
        # layer norm forward / VJP over [N, D] (residual stream f32)
        wsb = L.sb_op_layernorm_bwd_workspace_size(N, D)
        ws = torch.empty(wsb // 4 + 1, device=dev)
        k = nsets(N * D * (4 + es + 4 + 4 + 4))
        g = r(D)
        sets = [(torch.randn(N, D, device=dev), torch.empty(N, D, device=dev, dtype=dt), torch.empty(N, device=dev),
                 torch.empty(N, device=dev), torch.randn(N, D, device=dev), torch.zeros(N, D, device=dev),
                 torch.empty(D, device=dev, dtype=dt)) for _ in range(k)]

        def lnf(i):
            x, y, mu, rs, dy, dres, dg = sets[i % k]
            assert L.sb_op_layernorm_fwd(elem, x.data_ptr(), g.data_ptr(), y.data_ptr(), mu.data_ptr(),
                                         rs.data_ptr(), N, D, sp) == 0

        def lnb(i):
            x, y, mu, rs, dy, dres, dg = sets[i % k]
            assert L.sb_op_layernorm_bwd(elem, dy.data_ptr(), x.data_ptr(), mu.data_ptr(), rs.data_ptr(),
                                         g.data_ptr(), dres.data_ptr(), dg.data_ptr(), ws.data_ptr(), wsb, N, D,
                                         sp) == 0
        add("layer-norm forward", "ln_fwd_kernel", _rotated_ms(lnf, k, reps, st), N * D * (4 + es) + 8 * N, "GB/s",
            "hbm")
        add("layer-norm VJP (+ dgamma column sums)", "ln_bwd_kernel + column_sum_kernel",
            _rotated_ms(lnb, k, reps, st), N * D * 16 + 8 * N, "GB/s", "hbm")
        del sets, ws
        # cross-entropy forward + VJP over [N, V] logits (rows padded to ldl)
        wsb = L.sb_op_cross_entropy_workspace_size(N)
        ws = torch.empty(wsb // 4 + 1, device=dev)
        k = nsets(2 * N * ldl * es)
        tg = torch.randint(0, V, (N,), device=dev).float()
        loss = torch.zeros(1, device=dev)
        sets = [(r(N, ldl), torch.empty(N, ldl, device=dev, dtype=dt)) for _ in range(k)]

        def ce(i):
            lg, dl = sets[i % k]
            assert L.sb_op_cross_entropy(elem, lg.data_ptr(), ldl, N, V, tg.data_ptr(), dl.data_ptr(), ldl,
                                         ws.data_ptr(), wsb, loss.data_ptr(), sp) == 0
        add("cross-entropy fwd+VJP", "ce_fwd_bwd_kernel", _rotated_ms(ce, k, reps, st), 2 * N * V * es + 4 * N,
            "GB/s", "hbm")
        del sets, ws
    torch.cuda.synchronize(dev)
    return res


# --------------------------------------------------------------------------
# Primitive op sweep (bf16 and fp32): dot_general M=N=K in {512, 2048, 8192},
# the step's fc GEMM [16384, 384] x [384, 1536]^T (and, bf16, with its GELU
# epilogue), attention [16, 12, 1024, 64] and the step's [64, 6, 256, 64] fwd + VJP,
# layer-norm over [8192, 4096] and the step's [16384, 384], gelu over
# [8192, 4096]; N(0,1) values, seed 0. One JSON line per op.
# --------------------------------------------------------------------------

def _time_op(fn, reps: int, flush=None) -> float:
    """Average ms per call of fn() over `reps`, CUDA events on the current
    stream, L2 flushed before every timed call."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / reps


def sweep_ops(only: str | None = None, reps: int = 10):
    import torch

    import sheaf_b200 as sb

    L = sb.lib()
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    hbm, tc_burst, _, src = peaks()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    st = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731
    lines = []

    def emit(d):
        d.update({"data": "synthetic N(0,1) seed 0", "peak_source": src})
        print(json.dumps(d), flush=True)
        lines.append(d)

    def want(name):
        return only is None or only == name

    for kind, elem, dt in [("bf16", BF16, torch.bfloat16), ("f32", F32, torch.float32)]:
        for n in (512, 2048, 8192):
            name = f"gemm_{kind}_{n}"
            if not want(name):
                continue
            a = torch.randn(n, n, device=dev).to(dt)
            b = torch.randn(n, n, device=dev).to(dt)
            c = torch.empty(n, n, device=dev, dtype=dt)
            wsb = L.sb_op_matmul_workspace_size(elem, 0, 0, n, n, n)
            ws = torch.empty(max(wsb // 4, 1), device=dev)
            fn = lambda: L.sb_op_matmul(elem, a.data_ptr(), n, 0, b.data_ptr(), n, 0, n, n, n, c.data_ptr(), n,  # noqa
                                        elem, ws.data_ptr(), wsb, st())
            ms = _time_op(fn, reps, flush)
            tf = 2.0 * n ** 3 / (ms / 1e3) / 1e12
            emit({"op": name, "ms": ms, "achieved": tf, "unit": "TFLOP/s", "bound": "tensor" if kind == "bf16" else
                  "tensor, bf16x6 (fp32 FFMA below 6.7e7 multiply-adds)", "frac_of_bf16_peak": tf / tc_burst})
        name = f"gemm_{kind}_step_fc"  # the step's fc GEMM: [16384, 384] x [384, 1536]^T
        if want(name):
            M, N, K = CFG["batch"] * CFG["seq"], 4 * CFG["n_embd"], CFG["n_embd"]
            a = torch.randn(M, K, device=dev).to(dt)
            w = torch.randn(N, K, device=dev).to(dt)
            c = torch.empty(M, N, device=dev, dtype=dt)
            wsb = L.sb_op_matmul_workspace_size(elem, 0, 1, M, N, K)
            ws = torch.empty(max(wsb // 4, 1), device=dev)
            fn = lambda: L.sb_op_matmul(elem, a.data_ptr(), K, 0, w.data_ptr(), K, 1, M, N, K, c.data_ptr(), N,  # noqa
                                        elem, ws.data_ptr(), wsb, st())
            ms = _time_op(fn, reps, flush)
            tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
            emit({"op": name, "ms": ms, "achieved": tf, "unit": "TFLOP/s", "bound": "tensor" if kind == "bf16" else
                  "tensor, bf16x6", "frac_of_bf16_peak": tf / tc_burst})
        name = f"gemm_{kind}_step_fc_gelu"  # the same GEMM as the step runs it: gelu(u) and gelu'(u) stored
        if kind == "bf16" and want(name):
            M, N, K = CFG["batch"] * CFG["seq"], 4 * CFG["n_embd"], CFG["n_embd"]
            a = torch.randn(M, K, device=dev).to(dt)
            w = torch.randn(N, K, device=dev).to(dt)
            g = torch.empty(M, N, device=dev, dtype=dt)
            gd = torch.empty(M, N, device=dev, dtype=dt)
            fn = lambda: L.sb_op_matmul_gelu(elem, a.data_ptr(), K, w.data_ptr(), K, M, N, K, g.data_ptr(),  # noqa
                                             gd.data_ptr(), N, st())
            ms = _time_op(fn, reps, flush)
            tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
            emit({"op": name, "ms": ms, "achieved": tf, "unit": "TFLOP/s", "bound": "tensor + output bytes",
                  "frac_of_bf16_peak": tf / tc_burst, "out_bytes": 2 * M * N * g.element_size()})
        name = f"gemm_{kind}_step_dw_fc"  # the step's fc weight gradient: dU^T [1536, 16384] x h2 [16384, 384]
        if want(name):
            M, N, K = 4 * CFG["n_embd"], CFG["n_embd"], CFG["batch"] * CFG["seq"]
            du = torch.randn(K, M, device=dev).to(dt)
            h2 = torch.randn(K, N, device=dev).to(dt)
            c = torch.empty(M, N, device=dev, dtype=dt)
            wsb = L.sb_op_matmul_workspace_size(elem, 1, 0, M, N, K)
            ws = torch.empty(max(wsb // 4, 1), device=dev)
            fn = lambda: L.sb_op_matmul(elem, du.data_ptr(), M, 1, h2.data_ptr(), N, 0, M, N, K, c.data_ptr(), N,  # noqa
                                        elem, ws.data_ptr(), wsb, st())
            ms = _time_op(fn, reps, flush)
            tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
            emit({"op": name, "ms": ms, "achieved": tf, "unit": "TFLOP/s", "bound": "tensor" if kind == "bf16" else
                  "tensor, bf16x6", "frac_of_bf16_peak": tf / tc_burst})
        # GPT-2-small's GEMMs (8192 tokens, d 768): forward qkv / fc / fc2 / head,
        # a dX (B MN-major) and a weight gradient (both MN-major), plain stores
        for nm, M, N, K, ta, tb in (("qkv", 8192, 2304, 768, 0, 1), ("fc", 8192, 3072, 768, 0, 1),
                                    ("fc2", 8192, 768, 3072, 0, 1), ("head", 8192, 50304, 768, 0, 1),
                                    ("dx_fc", 8192, 768, 3072, 0, 0), ("dw_fc", 3072, 768, 8192, 1, 0)):
            name = f"gemm_{kind}_gpt2_{nm}"
            if kind != "bf16" or not want(name):
                continue
            a = torch.randn(*((K, M) if ta else (M, K)), device=dev).to(dt)
            b = torch.randn(*((N, K) if tb else (K, N)), device=dev).to(dt)
            c = torch.empty(M, N, device=dev, dtype=dt)
            wsb = L.sb_op_matmul_workspace_size(elem, ta, tb, M, N, K)
            ws = torch.empty(max(wsb // 4, 1), device=dev)
            fn = lambda: L.sb_op_matmul(elem, a.data_ptr(), a.shape[1], ta, b.data_ptr(), b.shape[1], tb, M, N, K,  # noqa
                                        c.data_ptr(), N, elem, ws.data_ptr(), wsb, st())
            ms = _time_op(fn, reps, flush)
            tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
            emit({"op": name, "ms": ms, "achieved": tf, "unit": "TFLOP/s", "bound": "tensor",
                  "frac_of_bf16_peak": tf / tc_burst})
        es_ = 2 if kind == "bf16" else 4
        for R, V in ((CFG["batch"] * CFG["seq"], CFG["vocab_size"]), (8192, 50304)):
            name = f"cross_entropy_{kind}_{R}x{V}"
            if not want(name):
                continue
            ldv = (V + 7) // 8 * 8
            lg = torch.randn(R, ldv, device=dev).to(dt)
            dl = torch.empty(R, ldv, device=dev, dtype=dt)
            tg = torch.randint(0, V, (R,), device=dev).float()
            loss = torch.zeros(1, device=dev)
            wsb = L.sb_op_cross_entropy_workspace_size(R)
            ws = torch.empty(wsb // 4 + 1, device=dev)
            ms = _time_op(lambda: L.sb_op_cross_entropy(elem, lg.data_ptr(), ldv, R, V, tg.data_ptr(), dl.data_ptr(),  # noqa
                                                        ldv, ws.data_ptr(), wsb, loss.data_ptr(), st()), reps, flush)
            b = 2 * R * V * es_ + 4 * R
            emit({"op": name, "ms": ms, "achieved": b / (ms / 1e3) / 1e9, "unit": "GB/s", "bound": "hbm", "peak": hbm,
                  "frac": b / (ms / 1e3) / 1e9 / hbm})
        for Bt, T, P, V, D in ((CFG["batch"], CFG["seq"], CFG["block_size"], CFG["vocab_size"], CFG["n_embd"]),
                               (8, 1024, 1024, 50304, 768)):
            name = f"embedding_{kind}_{Bt * T}x{V}x{D}"
            if not want(name):
                continue
            ids = torch.randint(0, V, (Bt * T,), device=dev).float()
            wte = torch.randn(V, D, device=dev).to(dt)
            wpe = torch.randn(P, D, device=dev).to(dt)
            x = torch.empty(Bt * T, D, device=dev)
            dx = torch.randn(Bt * T, D, device=dev)
            dwte = torch.empty(V, D, device=dev, dtype=dt)
            dwpe = torch.empty(P, D, device=dev, dtype=dt)
            wsb = L.sb_op_embedding_bwd_workspace_size(V, D)
            ws = torch.empty(wsb // 4 + 1, device=dev)
            mf = _time_op(lambda: L.sb_op_embedding_fwd(elem, ids.data_ptr(), wte.data_ptr(), wpe.data_ptr(),  # noqa
                                                        x.data_ptr(), Bt * T, T, V, D, st()), reps, flush)
            mb = _time_op(lambda: L.sb_op_embedding_bwd(elem, ids.data_ptr(), dx.data_ptr(), Bt, T, P, V, D,  # noqa
                                                        dwte.data_ptr(), dwpe.data_ptr(), ws.data_ptr(), wsb, st()),
                          reps, flush)
            # gather: ids + rows read (wte, wpe) + f32 rows written; VJP: f32 rows read + both tables written
            bf_ = Bt * T * (4 + 2 * D * es_ + 4 * D)
            bb_ = Bt * T * (4 + 4 * D) + (V + P) * D * es_
            emit({"op": name, "fwd_ms": mf, "vjp_ms": mb, "achieved_fwd": bf_ / (mf / 1e3) / 1e9,
                  "achieved_vjp": bb_ / (mb / 1e3) / 1e9, "unit": "GB/s", "bound": "hbm", "peak": hbm,
                  "frac_fwd": bf_ / (mf / 1e3) / 1e9 / hbm, "frac_vjp": bb_ / (mb / 1e3) / 1e9 / hbm})
        for B, T, H, Hd in ((16, 1024, 12, 64), (CFG["batch"], CFG["seq"], CFG["n_head"], CFG["n_embd"] // CFG["n_head"])):
            name = f"attention_{kind}_{B}x{H}x{T}x{Hd}"
            if not want(name):
                continue
            D = H * Hd
            qkv = torch.randn(B * T, 3 * D, device=dev).to(dt)
            o = torch.empty(B * T, D, device=dev, dtype=dt)
            do = torch.randn(B * T, D, device=dev).to(dt)
            dqkv = torch.empty(B * T, 3 * D, device=dev, dtype=dt)
            lse = torch.empty(B * H * T, device=dev)
            wsb = L.sb_op_attention_bwd_workspace_size(elem, B, T, H, Hd)
            ws = torch.empty(wsb // 4 + 1, device=dev)
            f_fwd = lambda: L.sb_op_attention_fwd(elem, qkv.data_ptr(), o.data_ptr(), lse.data_ptr(), B, T, H, Hd,  # noqa
                                                  st())
            f_bwd = lambda: L.sb_op_attention_bwd(elem, qkv.data_ptr(), o.data_ptr(), do.data_ptr(),  # noqa
                                                  lse.data_ptr(), dqkv.data_ptr(), ws.data_ptr(), wsb, B, T, H, Hd,
                                                  st())
            mf, mb = _time_op(f_fwd, reps, flush), _time_op(f_bwd, reps, flush)
            dense = 4.0 * B * H * T * T * Hd
            emit({"op": name, "fwd_ms": mf, "vjp_ms": mb, "dense_fwd_gflop": dense / 1e9,
                  "achieved_fwd": dense / 2 / (mf / 1e3) / 1e12, "achieved_vjp": 2.5 * dense / 2 / (mb / 1e3) / 1e12,
                  "unit": "TFLOP/s (causal: half the dense count)", "bound": "tensor",
                  "frac_fwd": dense / 2 / (mf / 1e3) / 1e12 / tc_burst})
        es = 2 if kind == "bf16" else 4
        for R, C in ((8192, 4096), (CFG["batch"] * CFG["seq"], CFG["n_embd"])):
            name = f"layernorm_{kind}_{R}x{C}"
            if not want(name):
                continue
            x = torch.randn(R, C, device=dev)
            g = torch.randn(C, device=dev).to(dt)
            y = torch.empty(R, C, device=dev, dtype=dt)
            mean, rstd = torch.empty(R, device=dev), torch.empty(R, device=dev)
            dy, dres = torch.randn(R, C, device=dev), torch.zeros(R, C, device=dev)
            dg = torch.empty(C, device=dev, dtype=dt)
            wsb = L.sb_op_layernorm_bwd_workspace_size(R, C)
            ws = torch.empty(wsb // 4 + 1, device=dev)
            f_fwd = lambda: L.sb_op_layernorm_fwd(elem, x.data_ptr(), g.data_ptr(), y.data_ptr(), mean.data_ptr(),  # noqa
                                                  rstd.data_ptr(), R, C, st())
            f_bwd = lambda: L.sb_op_layernorm_bwd(elem, dy.data_ptr(), x.data_ptr(), mean.data_ptr(),  # noqa
                                                  rstd.data_ptr(), g.data_ptr(), dres.data_ptr(), dg.data_ptr(),
                                                  ws.data_ptr(), wsb, R, C, st())
            mf, mb = _time_op(f_fwd, reps, flush), _time_op(f_bwd, reps, flush)
            bf = R * C * (4 + es)          # x (f32) in, y out
            bb = R * C * (4 + 4 + 4 + 4)   # dy, x in; dres in/out
            emit({"op": name, "fwd_ms": mf, "vjp_ms": mb, "achieved_fwd": bf / (mf / 1e3) / 1e9,
                  "achieved_vjp": bb / (mb / 1e3) / 1e9, "unit": "GB/s", "bound": "hbm", "peak": hbm,
                  "frac_fwd": bf / (mf / 1e3) / 1e9 / hbm, "frac_vjp": bb / (mb / 1e3) / 1e9 / hbm})
        R, C = 8192, 4096
        name = f"gelu_{kind}_8192x4096"
        if want(name):
            n = R * C
            x = torch.randn(n, device=dev).to(dt)
            gg = torch.randn(n, device=dev).to(dt)
            y = torch.empty(n, device=dev, dtype=dt)
            mf = _time_op(lambda: L.sb_op_gelu_fwd(elem, x.data_ptr(), y.data_ptr(), n, st()), reps, flush)
            mb = _time_op(lambda: L.sb_op_gelu_bwd(elem, x.data_ptr(), gg.data_ptr(), y.data_ptr(), n, st()), reps,
                          flush)
            emit({"op": name, "fwd_ms": mf, "vjp_ms": mb, "achieved_fwd": 2 * n * es / (mf / 1e3) / 1e9,
                  "achieved_vjp": 3 * n * es / (mb / 1e3) / 1e9, "unit": "GB/s", "bound": "hbm", "peak": hbm,
                  "frac_fwd": 2 * n * es / (mf / 1e3) / 1e9 / hbm, "frac_vjp": 3 * n * es / (mb / 1e3) / 1e9 / hbm})
    return lines


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="sheaf_b200", choices=["sheaf_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="primitive op sweep (one JSON line per op)")
    ap.add_argument("--op", default=None, help="run only this op of the sweep (e.g. gemm_bf16_8192)")
    ap.add_argument("--sample", action="store_true", help="autoregressive sampling tokens/s (1 GPU)")
    ap.add_argument("--config", default="nanogpt", choices=sorted(CONFIGS),
                    help="nanogpt: nanoGPT-char, batch 64 per GPU; gpt2: GPT-2-small, batch 8 per GPU")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f32"])
    ap.add_argument("--strong", action="store_true",
                    help="strong scaling: the reference's global batch (64) split over the GPUs")
    args = ap.parse_args()
    if args.sweep or args.op:
        sweep_ops(args.op, reps=args.steps if args.op else 10)
        return
    if args.sample:
        bench_sample(args)
        return
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    bench_b200(args, world, rank, local)


def bench_sample(args, n_new: int = 256):
    """Generated tokens/s of the sampling module: each call decodes n_new
    tokens for every sequence, each token one full-window forward (batch x
    256 positions) plus the on-device top-k / softmax / choice."""
    import torch

    from sheaf_b200.runtime import Session

    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    c = {k: v for k, v in CFG.items() if k not in ("batch", "seq")}
    leaves, _, _ = synthetic_inputs(1234)
    steps = max(1, min(args.steps, 10))
    for batch in (1, 32):
        s = Session(0)
        s.create_gpt_sampler("gen", **c, batch=batch, n_new=n_new, top_k=c["vocab_size"], temperature=1.0,
                             elem=BF16)
        rng = np.random.default_rng(7)
        ids = np.zeros((batch, c["block_size"]), np.float32)
        ids[:, -1] = rng.integers(0, c["vocab_size"], batch)  # encode-prompt of a one-token prompt
        # (random-key b) for sequence b: words (b, 0) as four 16-bit limbs
        keys = np.zeros((batch, 4), np.float32)
        keys[:, 0] = np.arange(batch) & 0xFFFF
        keys[:, 1] = np.arange(batch) >> 16
        inputs = [s.upload(l, BF16) for l in leaves] + [s.upload(ids, F32), s.upload(keys, F32)]
        st = torch.cuda.ExternalStream(s.stream, device=dev)
        for _ in range(max(args.warmup, 3)):
            outs = s.call("gen.generate", inputs)
        del outs
        s.synchronize()
        k0 = s.stats()["kernel_launches"]
        events = []
        with ClockSampler(0) as clk:
            with torch.cuda.stream(st):
                for _ in range(steps):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                    outs = s.call("gen.generate", inputs)
                    e1.record(st)
                    events.append((e0, e1))
                    del outs
                s.synchronize()
                torch.cuda.synchronize(dev)
        launches = s.stats()["kernel_launches"] - k0
        ms = sum(a.elapsed_time(b) for a, b in events)
        # e2e: prompt window and keys from host, generated tokens back to host
        pin = torch.from_numpy(ids).pin_memory().numpy()
        s.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            inputs[-2].write(pin)
            outs = s.call("gen.generate", inputs)
            _ = outs[0].to_host()
            del outs
        e2e_s = time.perf_counter() - t0
        gen = batch * n_new * steps
        line = {
            "metric": "nanoGPT sampling tokens/sec", "value": gen / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / steps, "higher_is_better": True,
            "scaling": "none", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"nanoGPT-char generate 6L/6H/384 window 256 V=65, batch {batch}, "
                                   f"{n_new} new tokens from a 1-token prompt, temperature 1.0, top_k = vocab",
                       "ms_per_token": ms / steps / n_new, "l2": "not flushed (weights stay L2-resident across "
                                                              "tokens, as in real decoding)"},
            "clocks": clk.summary(), "gpu_launches": int(launches),
            "e2e": {"value": gen / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(ids.nbytes),
                    "d2h_bytes_per_step": batch * n_new * 4},
        }
        print(json.dumps(line), flush=True)
        del inputs
        s.close()


def bench_b200(args, world, rank, local):
    import torch

    from sheaf_b200.runtime import Session

    name = args.config
    strong = args.strong
    base = CONFIGS[name]
    if strong:
        gb = STRONG_GLOBAL[name]
        if gb % world:
            raise SystemExit(f"global batch {gb} does not split over {world} GPUs")
        c = dict(base, batch=gb // world)
    else:
        c = dict(base)
    elem = BF16 if args.dtype == "bf16" else F32
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    s = Session(local)
    if world > 1:
        import torch.distributed as dist

        obj = [Session.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        s.join_group(obj[0], rank, world)
    s.create_gpt_vag("gpt", **c, elem=elem)
    leaves, x, y = synthetic_inputs(1234 + rank, c)
    inputs = [s.upload(l, elem) for l in leaves]
    xb, yb = s.upload(x, F32), s.upload(y, F32)
    inputs += [xb, yb]
    st = torch.cuda.ExternalStream(s.stream, device=dev)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)  # 256 MB > 126 MB L2

    outs = None
    for _ in range(max(args.warmup, 3)):
        outs = s.call("gpt.value_and_grad", inputs)
    loss0 = float(outs[0].to_host())
    del outs
    s.synchronize()

    # ---- device-timed steps: inputs resident, L2 flushed before every step
    barrier(world)
    torch.cuda.synchronize(dev)
    k0 = s.stats()["kernel_launches"]
    events = []
    with ClockSampler(local) as clk:
        with torch.cuda.stream(st):
            for _ in range(args.steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                outs = s.call("gpt.value_and_grad", inputs)
                e1.record(st)
                events.append((e0, e1))
                del outs
            s.synchronize()
            torch.cuda.synchronize(dev)
    launches = s.stats()["kernel_launches"] - k0
    local_ms = sum(a.elapsed_time(b) for a, b in events)
    total_ms = allmax(local_ms, world)
    barrier(world)
    tokens = world * c["batch"] * c["seq"] * args.steps
    value = tokens / (total_ms / 1e3)
    ms_per_step = total_ms / args.steps

    # ---- e2e: host ids -> device (pinned), call, loss -> host, every step
    pin_x = torch.from_numpy(x).pin_memory()
    pin_y = torch.from_numpy(y).pin_memory()
    hx, hy = pin_x.numpy(), pin_y.numpy()
    barrier(world)
    s.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        xb.write(hx)
        yb.write(hy)
        outs = s.call("gpt.value_and_grad", inputs)
        _ = outs[0].to_host()
        del outs
    e2e_s = allmax(time.perf_counter() - t0, world)
    e2e_value = tokens / e2e_s

    # ---- the step's own kernels, each timed alone (rank 0's GPU)
    hbm, tc_burst, tc_sust, src = peaks()
    bf = elem == BF16
    kernels = measure_step_kernels(s, c, elem) if rank == 0 else []
    # fp32: GEMMs run as bf16x6 (six bf16 products per f32 product) on the
    # tensor cores, so their ceiling is a sixth of the bf16 peak; attention
    # runs on the CUDA cores (FP32 nominal)
    for kr in kernels:
        if kr["unit"] == "GB/s":
            kr["peak"], kr["frac"] = hbm, kr["achieved"] / hbm
        else:
            kr["peak"] = tc_burst if bf else (tc_burst / 6 if kr["bound"] == "tensor" else FP32_NOMINAL_TFLOPS)
            kr["frac"] = kr["achieved"] / kr["peak"]
    head = kernels[0] if kernels else None
    step_tf = model_flops_per_token(c) * c["batch"] * c["seq"] / (ms_per_step / 1e3) / 1e12
    step_peak = tc_sust if bf else tc_sust / 6
    parallel = f"dp{world}" + (" strong" if strong else "")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": args.dtype, "data": "synthetic",
        "config": {"workload": f"{WORKLOAD[name]}, batch {c['batch']} per GPU", "global_batch": c["batch"] * world,
                   "seq_len": c["seq"], "parallelism": parallel,
                   "l2": "256 MB buffer written before every timed step (outside the events)",
                   "step_tflops": step_tf, "step_frac_of_peak": step_tf / step_peak,
                   "step_peak": ("measured bf16_tflops_sustained" if bf else
                                 "measured bf16_tflops_sustained / 6 (fp32 GEMMs as bf16x6 on the tensor cores)") +
                                f" {step_peak}",
                   "model_flop_per_token": model_flops_per_token(c), "loss_at_warmup": loss0},
        "clocks": clk.summary(),
        "gpu_launches": int(launches),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(x.nbytes + y.nbytes),
                "d2h_bytes_per_step": 2 if bf else 4},
    }
    if head is not None:
        line["roofline"] = {
            "bound": head["bound"], "kernel": f"{head['template']}: {head['kernel']} "
                                              f"[{c['batch'] * c['seq']} x {c['n_embd']}] x [{c['n_embd']} x "
                                              f"{4 * c['n_embd']}], as the step runs it",
            "achieved": head["achieved"], "peak": head["peak"], "unit": head["unit"], "frac": head["frac"],
            "traffic": FC_GELU_DRAM_BYTES.get(name) if bf else None,
            "traffic_unit": "bytes per launch (ncu dram read + write)",
            "peak_source": (f"{src} bf16_tflops (burst, kernel timed alone)" if bf else
                            f"{src} bf16_tflops / 6 (bf16x6 split of an f32 product)"),
            "timing": "back-to-back launches between CUDA events on the session stream, each on its own operands "
                      "(over 1 GB in all, above L2); mean of 5 rounds",
            "launch_ms": head["ms"]}
        line["kernels"] = [{k: v for k, v in kr.items() if k != "work"} for kr in kernels]
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_sample(name, c, args.dtype)
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    s.synchronize()
    barrier(world)
    del inputs, xb, yb
    s.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

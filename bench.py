#!/usr/bin/env python
"""Headline benchmark: train tokens/s of the BASELINE GPT step on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: d_model 512, 8 heads, 4 pre-LN layers,
GELU 4x FFN, seq 512, vocab 50257, untied head, bf16 compute / f32 master,
AdamW (lr 1e-3, warmup 200), batch 32 PER RANK (weak scaling; global batch
32*N), synthetic Zipf(1.1) tokens.  One step = forward + backward + gradient
all-reduce + AdamW.  For N > 1 run under torchrun (one rank per GPU, NCCL).

Reported (one JSON line from rank 0):
  value          tokens/s of the whole job, device-timed with CUDA events over
                 exactly K steps (barrier + synchronize on both sides, max over
                 ranks), token batches already resident in HBM.  On one GPU
                 the steps are replays of one captured CUDA graph of the whole
                 step (Trainer.capture_step / step_graphed); with N > 1 ranks
                 they are eager launches.  The eager figure is also reported.
  e2e            same metric through the public API (Trainer.train_step_async:
                 host token arrays in pinned memory -> H2D copy -> step (graph
                 replay at one rank, eager with N > 1) -> D2H copy of the loss,
                 every step; the host reads each loss one step late)
  roofline       the dominant launch family of the step: the 16 weight-gradient
                 GEMMs of the four blocks (gemm_pair_kernel<1,1>, dW += X^T dY
                 at K = 16384), timed live with CUDA events on the launching
                 stream over the eager timed region, algorithmic 2*M*N*K per
                 launch, vs the sustained bf16 peak of MEASURED_PEAKS.json;
                 `roofline_lm_head` the same for the LM-head forward GEMM
  gemm_sweep     configs[1]: fwd / dX / dW of each (K, N) model shape at
                 M = 16384 through the step's calls, L2 flushed between
                 launches, TFLOP/s and fraction of the burst peak
  lce            configs[2]: the fused LM-head CE composite (fwd + bwd,
                 2.530 TFLOP algorithmic), and the materialised-logit path
  ce_row         the CE row kernel (`ce_fwd` + `ce_bwd` in one pass, in place)
                 at (16384, 50257), f32 and bf16: GB/s and fraction of HBM
  flash_attention  op-level causal attention fwd+bwd TFLOP/s at configs[0]
  decode         inference: graph-replayed KV-cache decode steps, tokens/s at
                 batch 1 and 32 (not part of the headline metric)
  tail_ms        per step: device time from the end of the last backward
                 kernel to the end of the step (gradient exchange + optimizer
                 not hidden behind the backward)
  strong         (N > 1) the same step at GLOBAL batch 32 (32/N per rank)
  cpu_baseline   the CPU oracle step (oracle/model.py) on the host cores, at
                 the bench's own configuration (bs32 x 512)
--impl reference times that CPU implementation alone at bs32 x 512 (rank 0;
others exit 0).  nlearn's own JAX CPU path would be preferred, but JAX is not
importable in this image (the line records the import error).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train tokens/s d512·4L·seq512 bs32 @1/2/4/8 B200; flash fwd+bwd TFLOPS"
UNIT = "tokens/s"
BATCH, SEQ = 32, 512
FLOP_PER_TOKEN = 236.2e6           # 6*(matmul params) + causal attention, per token
HEAD_GEMM_FLOP = 2 * 16384 * 512 * 50257  # one LM-head forward GEMM at bs32/seq512


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), d["hbm_gbs"], "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                c = [x.strip() for x in line.split(",")]
                if len(c) < 9:
                    continue
                try:
                    sm.append(float(c[1]))
                    smax = float(c[2])
                except ValueError:
                    continue
                for n, v in zip(names, c[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_step_rate(threads: int | None = None, batch: int = BATCH, steps: int = 2):
    """CPU oracle (oracle/model.py, float32 PyTorch on the host cores): one full
    training step (fwd + bwd + AdamW) on `batch` sequences of SEQ tokens; a
    bounded sample of the bs32 workload, reported in tokens/s."""
    import torch
    from oracle.model import OracleGPT, OracleAdamW
    from nlearn_b200.model import GPTConfig, param_specs
    if threads:
        torch.set_num_threads(threads)
    cfg = GPTConfig()
    g = torch.Generator().manual_seed(0)
    params = {}
    for name, shape, init in param_specs(cfg):
        if init[0] == "normal":
            params[name] = torch.randn(*shape, generator=g) * init[1]
        elif init[0] == "ones":
            params[name] = torch.ones(*shape)
        else:
            params[name] = torch.zeros(*shape)
    m = OracleGPT(params)
    opt = OracleAdamW(m.p)
    tok = torch.randint(0, cfg.vocab, (batch, SEQ + 1), generator=g)
    x, y = tok[:, :-1], tok[:, 1:]
    m.loss(x, y).backward()
    opt.step(1e-3)  # warm-up step
    t0 = time.perf_counter()
    for _ in range(steps):
        m.loss(x, y).backward()
        opt.step(1e-3)
    dt = (time.perf_counter() - t0) / steps
    return batch * SEQ / dt, torch.get_num_threads(), f"{steps} steps of batch {batch}x{SEQ} after 1 warm-up step"


def _jax_status() -> str:
    try:
        import jax  # noqa: F401
        return "importable"
    except Exception as e:  # the image has no JAX: nlearn's own CPU path cannot run
        return f"not importable ({type(e).__name__}: {e})"


def run_reference(args, rank):
    if rank != 0:
        return
    ncores = len(os.sched_getaffinity(0))
    steps = max(1, min(args.steps, 2))
    v, cores, sample = cpu_step_rate(threads=ncores, batch=BATCH, steps=steps)
    cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample, "same_config": True}
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
                      "steps": steps, "warmup": 1, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                      "config": {"workload": "BASELINE GPT training step (CPU float32 restatement of nlearn's "
                                             "step, oracle/model.py)", "per_rank_batch": BATCH, "seq_len": SEQ,
                                 "same_config": True},
                      "jax": _jax_status(),
                      "cpu_baseline": cpu,
                      "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


# ----------------------------------------------------------------------------- op-level benchmarks
class FlushTimer:
    """Device time of one launch sequence with L2 flushed before each call:
    `iters` x (flush, fn) and `iters` x (flush) are each captured in a CUDA
    graph and replayed; the difference, divided by `iters`, is the call's time
    (CUDA events on the replaying stream).  The flush writes 256 MB, twice the
    126 MB L2."""

    def __init__(self, dev, iters: int = 10):
        import torch
        self.torch, self.dev, self.iters = torch, dev, iters
        self.buf = torch.empty(64 << 20, device=dev, dtype=torch.float32)

    def _graph(self, body):
        torch = self.torch
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            body()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(self.iters):
                body()
        return g

    def _time(self, g, reps=3):
        torch = self.torch
        g.replay()
        best = float("inf")
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        return best

    def ms(self, fn, flush: bool = True) -> float:
        flush_fn = (lambda: self.buf.fill_(1.0)) if flush else (lambda: None)

        def both():
            flush_fn()
            fn()
        g_both = self._graph(both)
        t_both = self._time(g_both)
        t_flush = self._time(self._graph(flush_fn)) if flush else 0.0
        return max(t_both - t_flush, 1e-6) / self.iters


def gemm_sweep(dev):
    """M = 16384, each (K, N) model shape, fwd (bf16 store), dX =
    dY W^T (bf16, W read in place) and dW += X^T dY (f32 accumulate), the calls
    the training step makes.  x ~ N(0,1), W ~ N(0,0.02), dY ~ N(0,1)."""
    import torch
    from nlearn_b200 import _lib
    from nlearn_b200.kernels.gemm import gemm_ex
    M = 16384
    burst = peaks()[0]
    ft = FlushTimer(dev)
    shapes = {}
    total_flop, total_ms = 0.0, 0.0
    for K, N, name in ((512, 1536, "qkv"), (512, 512, "proj"), (512, 2048, "ffn_up"), (2048, 512, "ffn_down"),
                       (512, 50257, "lm_head")):
        g = torch.Generator(device=dev).manual_seed(K + N)
        Np = (N + 63) // 64 * 64
        x = torch.randn(M, K, generator=g, device=dev).bfloat16()
        W = (torch.randn(K, Np, generator=g, device=dev) * 0.02).bfloat16()[:, :N]
        dY = torch.randn(M, Np, generator=g, device=dev).bfloat16()[:, :N]
        y = torch.empty(M, Np, device=dev, dtype=torch.bfloat16)[:, :N]
        dx = torch.empty(M, K, device=dev, dtype=torch.bfloat16)
        dw = torch.zeros(K, Np, device=dev)[:, :N]
        flop = 2.0 * M * N * K
        rec = {}
        for part, fn in (("fwd", lambda: gemm_ex(x, W, out=y)),
                         ("dX", lambda: gemm_ex(dY, W, b_trans=True, out=dx)),
                         ("dW", lambda: gemm_ex(x, dY, a_trans=True, out=dw, epilogue=_lib.EPI_ACCUM))):
            ms = ft.ms(fn)
            tf = flop / (ms * 1e-3) / 1e12
            rec[part] = {"ms": ms, "tflops": tf, "frac": tf / burst}
            total_flop += flop
            total_ms += ms
        shapes[f"{name} K={K} N={N}"] = rec
        del x, W, dY, y, dx, dw
    torch.cuda.empty_cache()
    tf = total_flop / (total_ms * 1e-3) / 1e12
    return {"M": M, "timing": "CUDA-graph replay, L2 flushed before each launch", "peak": burst,
            "peak_source": "measured bf16_tflops (burst: launches timed alone)", "shapes": shapes,
            "sweep_tflop": total_flop / 1e12, "sweep_ms": total_ms, "sweep_tflops": tf, "sweep_frac": tf / burst}


def lce_bench(dev):
    """hidden (16384, 512) bf16 ~ N(0,1), untied head W (512, 50257)
    ~ N(0, 0.02), int32 targets uniform -> mean CE loss and dX, dW.  Fused:
    nl_lce_fwd + nl_lce_bwd (no logits in memory).  Materialised: logits GEMM
    (bf16 [M, V]) + nl_ce_fwd_bwd in place + dX and dW GEMMs.  Algorithmic work
    6 * M * D * V = 2.530 TFLOP either way (the fused backward recomputes the
    logits: 3.373 TFLOP executed)."""
    import torch
    from nlearn_b200 import _lib
    from nlearn_b200.kernels.cross_entropy import ce_fwd_bwd, lce_bwd_raw, lce_fwd_raw
    from nlearn_b200.kernels.gemm import gemm_ex
    M, D, V = 16384, 512, 50257
    Vp = (V + 63) // 64 * 64
    g = torch.Generator(device=dev).manual_seed(2)
    X = torch.randn(M, D, generator=g, device=dev).bfloat16()
    W = (torch.randn(D, Vp, generator=g, device=dev) * 0.02).bfloat16()[:, :V]
    t = torch.randint(0, V, (M,), generator=g, device=dev, dtype=torch.int32)
    dX = torch.zeros(M, D, device=dev)
    dW = torch.zeros(D, Vp, device=dev)[:, :V]
    logits = torch.empty(M, Vp, device=dev, dtype=torch.bfloat16)[:, :V]
    dXb = torch.empty(M, D, device=dev, dtype=torch.bfloat16)

    def fused():
        loss, lse = lce_fwd_raw(X, W, t)
        lce_bwd_raw(X, W, t, lse, dX=dX, dW=dW, dw_accumulate=True)

    def materialised():
        gemm_ex(X, W, out=logits)
        ce_fwd_bwd(logits, t, out=logits)
        gemm_ex(X, logits, a_trans=True, out=dW, epilogue=_lib.EPI_ACCUM)
        gemm_ex(logits, W, b_trans=True, out=dXb)

    ft = FlushTimer(dev, iters=5)
    sustained = peaks()[1]
    burst = peaks()[0]
    alg = 6.0 * M * D * V
    out = {"config": "M 16384, D 512, V 50257 (configs[2])", "algorithmic_tflop": alg / 1e12,
           "peak": burst, "peak_source": "measured bf16_tflops (burst: composite timed alone)"}
    for name, fn in (("fused", fused), ("materialised", materialised)):
        ms = ft.ms(fn)
        tf = alg / (ms * 1e-3) / 1e12
        out[name] = {"ms": ms, "tflops": tf, "frac": tf / burst, "frac_of_sustained": tf / sustained}
    del X, W, dX, dW, logits, dXb
    torch.cuda.empty_cache()
    return out


def ce_row_bench(dev):
    """The materialised-logit CE row kernel (`ce_fwd` + `ce_bwd` in one pass,
    dlogits written over the logits) at (16384, 50257), f32 (the reference's
    dtype) and bf16.  Algorithmic bytes: read the logits once, write dlogits
    once, plus targets, loss and lse (12 B per row).  The logits (1.6-3.3 GB)
    exceed L2, so no flush is needed."""
    import torch
    from nlearn_b200.kernels.cross_entropy import ce_fwd_bwd
    M, V = 16384, 50257
    hbm = peaks()[2]
    ft = FlushTimer(dev, iters=10)
    out = {"config": "M 16384, V 50257, in place", "peak_gbs": hbm, "peak_source": "measured hbm_gbs"}
    for dt, nb in ((torch.float32, 4), (torch.bfloat16, 2)):
        x = torch.randn(M, V, device=dev).to(dt)
        t = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        ms = ft.ms(lambda: ce_fwd_bwd(x, t, out=x), flush=False)
        byts = M * V * 2 * nb + 12 * M
        gbs = byts / (ms * 1e-3) / 1e9
        out["f32" if nb == 4 else "bf16"] = {"ms": ms, "bytes": byts, "gbs": gbs, "frac": gbs / hbm}
        del x
    torch.cuda.empty_cache()
    return out


def flash_op_tflops(dev, iters=20):
    """Causal attention fwd+bwd TFLOP/s (bf16, d=64): configs[0] (BH 32, S 512)
    and, for context, the full-model shapes (BH 256 x S 512 inside the bs32
    step, BH 64 x S 4096 long context).  Two timings per shape, both CUDA
    events: `eager` (back-to-back calls through the Python binding, host
    dispatch included) and `graph` (the same fwd+bwd captured once in a CUDA
    graph and replayed, i.e. device time of the four kernels).  The headline
    `tflops` is the graph figure.  FLOPs: fwd 4*BH*S^2*d/2, bwd 2.5x fwd."""
    import torch
    from nlearn_b200 import attention as A
    out = {}
    for name, n, s in (("configs[0] BH=32 S=512", 32, 512), ("BH=256 S=512", 256, 512), ("BH=64 S=4096", 64, 4096)):
        torch.manual_seed(0)
        Q, K, V, dO = (torch.randn(n, s, 64, device=dev).bfloat16() for _ in range(4))

        def step():
            O, L = A._flash_fwd_raw(Q, K, V)
            A._flash_bwd_raw(Q, K, V, O, L, dO)

        def timed(fn):
            for _ in range(3):
                fn()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / iters

        flop = 3.5 * 4 * n * s * s * 64 / 2
        ms_eager = timed(step)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()  # warm-up on the capture stream
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        ms_graph = timed(g.replay)
        del g
        out[name] = {"ms_fwd_bwd": ms_graph, "tflops": flop / (ms_graph * 1e-3) / 1e12,
                     "eager_ms_fwd_bwd": ms_eager, "eager_tflops": flop / (ms_eager * 1e-3) / 1e12}
    c0 = out["configs[0] BH=32 S=512"]
    return {"config": "BH=32 S=512 d=64 causal bf16 (configs[0])", "timing": "CUDA-graph replay of fwd+bwd",
            "ms_fwd_bwd": c0["ms_fwd_bwd"], "tflops": c0["tflops"], "shapes": out}


def decode_rate(dev, P, cfg, batch: int, prompt_len: int = 64, steps: int = 128):
    """Inference: tokens/s of graph-replayed KV-cache decode steps after a
    prompt prefill (nlearn_b200.generate.Decoder), CUDA-event timed.  At batch
    1 a step reads every bf16 weight once, so `weight_gbs` is that traffic
    divided by the step time (HBM-bound kernel family)."""
    import numpy as np
    import torch
    from nlearn_b200.generate import Decoder
    dec = Decoder(P, cfg, batch=batch)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab, (batch, prompt_len)).astype(np.int32)
    dec.prefill(torch.from_numpy(prompt).to(dev), 0, 1.0)
    dec.step(0, 1.0)
    dec.capture(0, 1.0)
    for _ in range(3):
        dec._graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        dec._graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    wbytes = sum(int(np.prod(shape)) for name, shape, _ in P.specs if len(shape) == 2 and name not in ("wte", "wpe")) * 2
    del dec
    torch.cuda.empty_cache()
    return {"batch": batch, "prompt": prompt_len, "ms_per_token_step": ms, "tokens_per_s": batch / (ms * 1e-3),
            "weight_gbs": wbytes / (ms * 1e-3) / 1e9}


def long_context(dev, rank, world, steps=5, warmup=3, graphs=True):
    """the same model at seq 4096, GLOBAL batch 8 split over the
    ranks (strong scaling; one sequence per rank at 8 GPUs).  Device-timed
    tokens/s of the whole job, max over ranks."""
    import torch
    import torch.distributed as dist
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig
    per_rank = max(1, 8 // world)
    tr = Trainer(GPTConfig(max_seq=4096), TrainConfig(batch=per_rank, seq=4096, steps=1000, peak_lr=1e-3,
                                                      warmup=200), dev, rank, world)
    bat = [tr.device_batch(*tr.loader.next()) for _ in range(warmup + steps)]
    for i in range(warmup):
        tr.step_on_device(*bat[i])
    step = tr.step_on_device
    if world == 1 and graphs:
        tr.capture_step()
        tr.step_graphed(*bat[0])
        step = tr.step_graphed
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, warmup + steps):
        step(*bat[i])
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t) / steps
    tokens = per_rank * world * 4096
    del tr, bat
    torch.cuda.empty_cache()
    return {"config": "seq 4096, global batch 8 (configs[4]), strong scaling", "per_rank_batch": per_rank,
            "ms_per_step": ms, "value": tokens / (ms * 1e-3), "unit": UNIT,
            "timing": "CUDA-graph replay" if (world == 1 and graphs) else "eager launches",
            "mfu": tokens / (ms * 1e-3) * 280.2e6 / (world * peaks()[1] * 1e12)}


def _strong_scaling(dev, rank, world, steps, warmup):
    """The bs32 x 512 step at GLOBAL batch 32 (32 / N sequences per rank),
    eager, device-timed, max over ranks: the strong-scaling companion of the
    weak-scaling headline (efficiency basis: T(N) / T(1) of this figure)."""
    import torch
    import torch.distributed as dist
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig
    per_rank = max(1, BATCH // world)
    tr = Trainer(GPTConfig(), TrainConfig(batch=per_rank, seq=SEQ, steps=1000, peak_lr=1e-3, warmup=200), dev, rank,
                 world)
    bat = [tr.device_batch(*tr.loader.next()) for _ in range(warmup + steps)]
    for i in range(warmup):
        tr.step_on_device(*bat[i])
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, warmup + steps):
        tr.step_on_device(*bat[i])
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t) / steps
    del tr, bat
    torch.cuda.empty_cache()
    return {"config": "global batch 32 x 512 split over the ranks", "per_rank_batch": per_rank, "ms_per_step": ms,
            "value": per_rank * world * SEQ / (ms * 1e-3), "unit": UNIT, "timing": "eager launches"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sharded-optimizer", action="store_true",
                    help="N > 1: reduce-scatter, AdamW on this rank's shard, all-gather the weights")
    ap.add_argument("--dense-exchange", action="store_true",
                    help="all-reduce the whole token-table gradient instead of the touched rows (N > 1)")
    ap.add_argument("--no-long", action="store_true", help="skip the seq-4096 long-context measurement")
    ap.add_argument("--no-graph", action="store_true", help="time eager launches instead of CUDA-graph replay")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the op-level benchmarks (GEMM sweep, LM-head CE, CE row, attention, decode)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    import torch.distributed as dist
    from nlearn_b200 import _lib
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig, init_distributed

    rank, world, local = init_distributed()
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    cfg = GPTConfig()
    tr = Trainer(cfg, TrainConfig(batch=BATCH, seq=SEQ, steps=1000, peak_lr=1e-3, warmup=200,
                                  compact_embedding_exchange=not args.dense_exchange,
                                  sharded_optimizer=args.sharded_optimizer), dev, rank, world)

    # device-resident batches for the timed region
    nb = args.warmup + args.steps
    host = [tr.loader.next() for _ in range(nb)]
    dbat = [tr.device_batch(x, y) for x, y in host]

    # live per-launch timing (CUDA events on the launching stream) of the step's
    # dominant launch family, the weight-gradient GEMMs (dW += X^T dY), and of
    # the LM-head forward GEMM
    import nlearn_b200.model as M
    from nlearn_b200.kernels import cross_entropy as CE
    head_ev, dw_ev = [], []
    orig_fwd, orig_gemm = CE.lce_fwd_raw, M.gemm_ex

    def timed_lce_fwd(*a, **k):
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        r = orig_fwd(*a, **k)
        e0.record()
        head_ev.append((s0, e0))
        return r

    def timed_gemm(A, B, **k):
        if not (k.get("a_trans") and k.get("epilogue") == _lib.EPI_ACCUM):
            return orig_gemm(A, B, **k)
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        r = orig_gemm(A, B, **k)
        e0.record()
        Mo, No, Ko = A.shape[1], B.shape[1], A.shape[0]
        dw_ev.append((s0, e0, 2.0 * Mo * No * Ko))
        return r

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()  # sampled over warm-up, timed, end-to-end and long-context runs (all under load)
    for i in range(args.warmup):
        tr.step_on_device(*dbat[i])
    barrier()
    l0 = _lib.lib.nl_launch_count()
    tr.tail_events = []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.warmup, nb):
        loss = tr.step_on_device(*dbat[i])
    e1.record()
    barrier()
    launches = _lib.lib.nl_launch_count() - l0
    ms = e0.elapsed_time(e1)
    tail_ms = statistics.mean(a.elapsed_time(b) for a, b in tr.tail_events)
    tr.tail_events = None
    t = torch.tensor([ms, tail_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_eager, tail_ms = float(t[0]), float(t[1])
    tokens = BATCH * SEQ * world * args.steps
    value_eager = tokens / (ms_eager * 1e-3)

    # the kernel timings: a separate eager pass with events around the launches
    # (events between launches cost a little overlap, so the headline steps above
    # run without them)
    CE.lce_fwd_raw = M.lce_fwd_raw = timed_lce_fwd
    M.gemm_ex = timed_gemm
    for i in range(args.warmup, min(nb, args.warmup + 5)):
        tr.step_on_device(*dbat[i])
    barrier()
    CE.lce_fwd_raw = M.lce_fwd_raw = orig_fwd
    M.gemm_ex = orig_gemm
    head_avg_ms = statistics.mean(a.elapsed_time(b) for a, b in head_ev)
    dw_ms = sum(a.elapsed_time(b) for a, b, _ in dw_ev)
    dw_flop = sum(f for _, _, f in dw_ev)
    dw_per_step = len(dw_ev) // max(1, min(nb, args.warmup + 5) - args.warmup)

    # the same steps replayed from one captured CUDA graph (single rank)
    graphed = world == 1 and not args.no_graph
    ms_max, value = ms_eager, value_eager
    if graphed:
        per_step = tr.capture_step()
        for i in range(2):
            tr.step_graphed(*dbat[i])
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        for i in range(args.warmup, nb):
            loss = tr.step_graphed(*dbat[i])
        g1.record()
        barrier()
        ms_max = g0.elapsed_time(g1)
        value = tokens / (ms_max * 1e-3)
        launches = per_step * args.steps

    # end to end through the public API: host arrays in, host loss out
    pinned = [(torch.from_numpy(x).pin_memory(), torch.from_numpy(y).pin_memory()) for x, y in host[:args.steps]]
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record()
    if not graphed:
        tr._graph = None
    lv = None
    for x, y in pinned:
        # H2D of the batch, the step, D2H of its loss into pinned memory; the
        # host reads the previous step's loss (so it never waits on the step
        # it has just queued)
        prev = tr.train_step_async(x, y)
        lv = prev if prev is not None else lv
    f1.record()
    lv = tr.flush_loss()                       # the last step's loss, read inside the timed region
    barrier()
    t2 = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_value = tokens / (float(t2) * 1e-3)
    del tr, dbat
    torch.cuda.empty_cache()

    strong = _strong_scaling(dev, rank, world, args.steps, args.warmup) if world > 1 else None
    extras = rank == 0 and not args.no_extras
    sweep = gemm_sweep(dev) if extras else None
    lce = lce_bench(dev) if extras else None
    ce_row = ce_row_bench(dev) if extras else None
    flash = flash_op_tflops(dev) if extras else None
    longc = long_context(dev, rank, world, graphs=not args.no_graph) if not args.no_long else None
    decode = None
    if extras:
        from nlearn_b200.model import FlatParams
        P = FlatParams(cfg, dev, seed=0)
        decode = [decode_rate(dev, P, cfg, b) for b in (1, 32)]
        del P
    clk = clocks.stop()
    burst, sustained, hbm, src = peaks()
    achieved_dw = dw_flop / (dw_ms * 1e-3) / 1e12
    achieved_head = HEAD_GEMM_FLOP / (head_avg_ms * 1e-3) / 1e12
    # DRAM bytes per launch of the same kernels, from the committed ncu summaries
    import re

    def traffic_from(fname, key):
        tf = os.path.join(ROOT, "profiles", fname)
        if not os.path.exists(tf):
            return None
        with open(tf) as f:
            mt = re.search(key + r"\s*=\s*(\d+)", f.read())
        return int(mt.group(1)) if mt else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_step_rate(threads=len(os.sched_getaffinity(0)), batch=BATCH, steps=1)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample, "same_config": True}
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE GPT training step: d512/8h/4L pre-LN GELU-4x, seq 512, vocab 50257 "
                                   "untied, bf16 compute + f32 master, AdamW",
                       "global_batch": BATCH * world, "per_rank_batch": BATCH, "seq_len": SEQ,
                       "parallelism": f"dp{world}", "tokens": "Zipf(1.1) synthetic",
                       "l2": "no flush: per-step working set (activations ~1.5 GB, weights+grads+moments 1.1 GB) "
                             "exceeds the 126 MB L2; op-level benchmarks flush L2 before each launch"},
            "mfu": value * FLOP_PER_TOKEN / (world * sustained * 1e12),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": 2 * BATCH * SEQ * 4,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": launches,
            "timing": {"mode": "CUDA-graph replay of the whole step" if graphed else "eager launches",
                       "eager_value": value_eager, "eager_ms_per_step": ms_eager / args.steps,
                       "roofline_from": "a separate eager pass with CUDA events around the timed launches"},
            "tail_ms": tail_ms,
            "roofline": {"bound": "tensor",
                         "kernel": f"weight-gradient GEMMs (gemm_pair_kernel<1,1>, dW += X^T dY, K 16384; "
                                   f"{dw_per_step} launches per step)",
                         "achieved": achieved_dw, "peak": sustained, "unit": "TFLOP/s",
                         "frac": achieved_dw / sustained, "peak_source": f"{src} bf16_tflops_sustained",
                         "traffic": traffic_from("gemm_wgrad_M512_N2048_K16384.md", "wgrad_bytes_per_launch"),
                         "traffic_launch": "w1 gradient, M 512 N 2048 K 16384",
                         "avg_launch_ms": dw_ms / max(1, len(dw_ev)),
                         "algorithmic_gflop_per_step": dw_flop / 1e9 / max(1, len(dw_ev)) * dw_per_step},
            "roofline_lm_head": {"bound": "tensor", "kernel": "LM-head forward GEMM (nl_lce_fwd, M16384 N50257 K512)",
                                 "achieved": achieved_head, "peak": sustained, "unit": "TFLOP/s",
                                 "frac": achieved_head / sustained, "peak_source": f"{src} bf16_tflops_sustained",
                                 "traffic": traffic_from("gemm_lce_head_fwd_M16384.md",
                                                         "lce_head_gemm_bytes_per_launch"),
                                 "avg_launch_ms": head_avg_ms},
            "strong": strong,
            "gemm_sweep": sweep,
            "lce": lce,
            "ce_row": ce_row,
            "flash_attention": flash,
            "decode": decode,
            "long_context": longc,
            "clocks": clk,
            "cpu_baseline": cpu,
            "final_loss": lv,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

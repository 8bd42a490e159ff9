"""Data-parallel training of the BASELINE GPT on B200s: one process per GPU,
``torch.distributed`` (NCCL over NVLink / NVSwitch) for the gradient exchange.

Mirrors nlearn/train.py's step (make_train_step 328-341: loss -> grads ->
optax update, one device boundary per step) with:
  * synthetic Zipf(1.1) token batches standing in for fineweb-edu
    (the container has no dataset; BASELINE configs name this stand-in);
  * a bucketed gradient all-reduce that starts each bucket on a side stream
    the moment the backward has produced its last gradient, overlapping the
    rest of the backward (one flat f32 gradient buffer, no copies);
  * fused AdamW and the warmup-cosine schedule of nlearn/train.py:487-508;
  * atomic checkpoint / resume of {params, opt_state, step, data position}
    (nlearn/train.py:76-99: tmp file + os.replace).
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from .model import GPT, AdamW, FlatParams, GPTConfig, lr_schedule


# ----------------------------------------------------------------------------- data
def zipf_tokens(rng: np.random.Generator, shape, vocab: int, a: float = 1.1) -> np.ndarray:
    """Zipf(a) token ids in [0, vocab): draws >= vocab are redrawn."""
    out = rng.zipf(a, size=shape) - 1
    bad = out >= vocab
    while bad.any():
        out[bad] = rng.zipf(a, size=int(bad.sum())) - 1
        bad = out >= vocab
    return out.astype(np.int32)


class ZipfLoader:
    """Per-rank stream of (inputs, targets) [B, S] int32 batches, each a
    window of S+1 tokens.  Deterministic in (seed, rank, step)."""

    def __init__(self, batch: int, seq: int, vocab: int, seed: int = 0, rank: int = 0):
        self.batch, self.seq, self.vocab, self.seed, self.rank = batch, seq, vocab, seed, rank
        self.step = 0

    def host_batch(self, step: int | None = None):
        s = self.step if step is None else step
        rng = np.random.default_rng([self.seed, self.rank, s])
        w = zipf_tokens(rng, (self.batch, self.seq + 1), self.vocab)
        return w[:, :-1].copy(), w[:, 1:].copy()

    def next(self):
        b = self.host_batch()
        self.step += 1
        return b


# ----------------------------------------------------------------------------- DP
class BucketReducer:
    """Gradient exchange and optimizer, bucket by bucket, overlapped with the
    backward.

    The flat gradient buffer is cut into contiguous buckets in gradient-
    production order.  When the backward reports every parameter of a bucket
    final (and its weights read for the last time), the bucket is all-reduced
    (mean) on a side stream and, if an optimizer is attached, AdamW updates it
    right after on the same stream, while the backward goes on.  With one rank
    there is no exchange; the per-bucket AdamW still overlaps the backward.

    The token table (``wte``) is its own bucket and is handled by rows
    (``begin_rows``): its gradient is zero on every row that no input token of
    the global batch touched, so those rows get their zero-gradient AdamW
    update at the start of the step, and after the backward only the touched
    rows are updated.  The touched set comes from the token ids (all-reduced
    across ranks), known before the forward.  With ``compact_exchange`` only
    the touched rows are gathered, all-reduced and scattered back (fewer bytes
    over NVLink at a host wait for their count); otherwise the whole table
    gradient is all-reduced.  Results equal the dense exchange and the dense
    AdamW."""

    def __init__(self, params: FlatParams, bucket_bytes: int = 64 << 20, group=None, optimizer=None,
                 sparse_rows: bool | None = None, compact_exchange: bool = False, sharded: bool = False):
        self.P = params
        self.optimizer = optimizer  # if set, each bucket's AdamW runs right after its all-reduce
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.use_avg = dist.is_initialized() and dist.get_backend(group) == "nccl"
        cuda = params.device.type == "cuda"
        self.sparse = (cuda and optimizer is not None) if sparse_rows is None else bool(sparse_rows)
        # all-reduce only the touched rows (needs their count on the host, read
        # after the backward: a host wait on the step's start, which stalls a
        # host that is not far ahead of the device); otherwise the whole table
        # gradient is all-reduced (zero on untouched rows) and only the AdamW
        # is split by rows
        self.compact = self.sparse and compact_exchange and self.world > 1
        # ZeRO-1 style: reduce-scatter each bucket, AdamW on this rank's shard,
        # all-gather the updated master weights (the same NVLink bytes as the
        # all-reduce, 1/world of the optimizer work); bucket ranges are padded
        # to the parameters' 2 KB alignment so they split evenly
        from .model import PARAM_ALIGN
        self.sharded = (sharded and self.world > 1 and optimizer is not None and cuda
                        and (PARAM_ALIGN // 64) % self.world == 0)
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        cap = max(1, bucket_bytes // 4)
        self.buckets = []  # (start, end, {names})
        cur_names, start = set(), None
        end = 0
        for name, shape, _ in params.specs:
            off, shp = params.offsets[name]
            n = int(np.prod(shp))
            if self.sparse and name == "wte" and cur_names:   # the token table is a bucket of its own
                self.buckets.append((start, end, cur_names))
                cur_names, start = set(), None
            if start is None:
                start = off
            cur_names.add(name)
            end = off + n
            if end - start >= cap or (self.sparse and name == "wte"):
                self.buckets.append((start, end, cur_names))
                cur_names, start = set(), None
        if cur_names:
            self.buckets.append((start, end, cur_names))
        if self.sharded:   # extend each bucket over the padding up to the next parameter
            self.buckets = [(st, min(-(-en // PARAM_ALIGN) * PARAM_ALIGN, params.numel), ns)
                            for st, en, ns in self.buckets]
        self.owner = {n: i for i, (_, _, ns) in enumerate(self.buckets) for n in ns}
        self.stream = torch.cuda.Stream(device=params.device) if cuda else None
        self._pending = None
        self._launched = []
        self._rows_ready = False
        if self.sparse:
            V, D = params.offsets["wte"][1]
            self.V, self.D = V, D
            dev = params.device
            self.mark = torch.zeros(V, device=dev, dtype=torch.int32)
            self.idx_on = torch.empty(V, device=dev, dtype=torch.int32)
            self.idx_off = torch.empty(V, device=dev, dtype=torch.int32)
            self.counts = torch.zeros(2 + (V + 1023) // 1024, device=dev, dtype=torch.int32)
            self.counts_host = torch.zeros(2, dtype=torch.int32).pin_memory()
            self.counts_event = torch.cuda.Event()
            self.rows_buf = torch.empty(V, D, device=dev, dtype=torch.float32) if self.compact else None

    def active(self) -> bool:
        """Whether buckets are processed during the backward (exchange with
        more than one rank, or the overlapped optimizer)."""
        return self.world > 1 or self.optimizer is not None

    def begin(self):
        self._pending = [set(ns) for (_, _, ns) in self.buckets]
        self._launched = []

    def begin_rows(self, tok: torch.Tensor):
        """Start of a step (after the optimizer's schedule is staged): find the
        token rows this step touches across all ranks and update the others."""
        if not self.sparse:
            return
        from ._lib import check, lib, ptr
        cur = torch.cuda.current_stream()
        ev = torch.cuda.Event()
        ev.record(cur)
        self.stream.wait_event(ev)
        with torch.cuda.stream(self.stream):
            h = torch.cuda.current_stream().cuda_stream
            check(lib.nl_rows_mark(ptr(tok), tok.numel(), ptr(self.mark), self.V, h), "nl_rows_mark")
            if self.world > 1:
                dist.all_reduce(self.mark, op=dist.ReduceOp.MAX, group=self.group)
            check(lib.nl_rows_compact(ptr(self.mark), self.V, ptr(self.idx_on), ptr(self.idx_off), ptr(self.counts),
                                      h), "nl_rows_compact")
            if self.compact:  # the exchange's element count is needed on the host after the backward
                self.counts_host.copy_(self.counts[:2], non_blocking=True)
                self.counts_event.record()
            self._adamw_rows(self.idx_off, self.counts[1:], None)
        self._rows_ready = True

    def _adamw_rows(self, idx, count, g):
        from ._lib import check, lib, ptr
        P, o = self.P, self.optimizer
        off = P.offsets["wte"][0]
        h = torch.cuda.current_stream().cuda_stream
        check(lib.nl_adamw_rows(ptr(P.master[off:]), None if g is None else ptr(g), ptr(P.exp_avg[off:]),
                                ptr(P.exp_avg_sq[off:]), ptr(P.shadow[off:]), ptr(idx), ptr(count), self.D, self.V,
                                ptr(o.hyper), o.b1, o.b2, o.eps, o.wd, int(o.zero_grad), h), "nl_adamw_rows")

    def ready(self, name: str):
        if not self.active():
            return
        i = self.owner[name]
        self._pending[i].discard(name)
        if not self._pending[i]:
            self._launch(i)

    def _launch(self, i: int):
        start, end, names = self.buckets[i]
        if self.stream is not None:
            ev = torch.cuda.Event()
            ev.record()
            self.stream.wait_event(ev)
            with torch.cuda.stream(self.stream):
                self._process(start, end, names)
        else:
            self._process(start, end, names)
        self._launched.append(i)

    def _process(self, start: int, end: int, names):
        if self.sparse and names == {"wte"} and self._rows_ready:
            self._process_rows()
            return
        if self.sharded:
            self._process_sharded(start, end)
            return
        buf = self.P.grad[start:end]
        if self.world > 1:
            self._allreduce(buf)
        if self.optimizer is not None:
            self.optimizer.step_range(start, end)

    def _shard(self, start: int, end: int):
        c = (end - start) // self.world
        return start + self.rank * c, c

    def _process_sharded(self, start: int, end: int):
        from ._lib import check, lib, ptr
        P = self.P
        s0, c = self._shard(start, end)
        op = dist.ReduceOp.AVG if self.use_avg else dist.ReduceOp.SUM
        dist.reduce_scatter_tensor(P.grad[s0:s0 + c], P.grad[start:end], op=op, group=self.group)
        if not self.use_avg:
            P.grad[s0:s0 + c].div_(self.world)
        self.optimizer.step_range(s0, s0 + c)
        dist.all_gather_into_tensor(P.master[start:end], P.master[s0:s0 + c], group=self.group)
        check(lib.nl_cast_bf16(ptr(P.master[start:]), ptr(P.shadow[start:]), end - start,
                               torch.cuda.current_stream().cuda_stream), "nl_cast_bf16")

    def gather_sharded(self, bufs):
        """Sharded mode: make every rank's copy of ``bufs`` (flat buffers such
        as the reduced gradient or the AdamW moments, each valid only on the
        rank's own shard of each bucket) whole again.  Collective: every rank
        calls it."""
        if not self.sharded:
            return
        torch.cuda.current_stream().wait_stream(self.stream)
        for start, end, names in self.buckets:
            if self.sparse and names == {"wte"}:
                continue
            s0, c = self._shard(start, end)
            for b in bufs:
                dist.all_gather_into_tensor(b[start:end], b[s0:s0 + c].clone(), group=self.group)

    def _process_rows(self):
        """The token table after the backward: touched rows only."""
        from ._lib import check, lib, ptr
        g = self.P.g("wte")
        on = self.counts[:1]
        if self.world > 1 and not self.compact:
            self._allreduce(g.view(-1))
        elif self.world > 1:
            h = torch.cuda.current_stream().cuda_stream
            self.counts_event.synchronize()      # recorded at the step's start: long complete
            U = int(self.counts_host[0])
            check(lib.nl_rows_gather(ptr(g), ptr(self.idx_on), ptr(on), self.D, ptr(self.rows_buf), self.V, h),
                  "nl_rows_gather")
            if U > 0:
                self._allreduce(self.rows_buf[:U])
            check(lib.nl_rows_scatter(ptr(self.rows_buf), ptr(self.idx_on), ptr(on), self.D, ptr(g), self.V, h),
                  "nl_rows_scatter")
        if self.optimizer is not None:
            self._adamw_rows(self.idx_on, on, g)
        self._rows_ready = False

    def _allreduce(self, buf):
        if self.use_avg:
            dist.all_reduce(buf, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group)
            buf.div_(self.world)

    def finish(self):
        if not self.active():
            return
        for i in range(len(self.buckets)):
            if i not in self._launched:
                self._launch(i)
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)


# ----------------------------------------------------------------------------- trainer
@dataclass
class TrainConfig:
    batch: int = 32            # per rank
    seq: int = 512
    steps: int = 1000          # schedule length (decay_steps)
    peak_lr: float = 1e-3
    warmup: int = 200          # the BASELINE warmup; capped at steps // 5 as train.py:488
    weight_decay: float = 0.1
    seed: int = 0
    # layer-sized buckets (a block's parameters are 12.6 MB in f32): each
    # block's exchange starts as soon as that block's backward is done, so only
    # the first block and the token table are left for the step's tail (with
    # 64 MB buckets the four blocks shared one bucket, launched at the end)
    bucket_mb: int = 16
    fused_lmhead: bool | None = None   # None: NLEARN_FUSED_LMHEAD (model.fused_lmhead_default)
    # False: AdamW clears each gradient after reading it and the step skips its
    # zeroing pass; measured 0.4 ms/step slower on B200 (the clearing writes
    # land on the side stream while the backward runs), so off by default
    keep_grads: bool = True
    sparse_embedding_rows: bool = True  # token-table AdamW by rows: untouched rows at the step's start
    # and all-reduce only the touched rows (the host waits, after the backward,
    # for their count, known since the step's start); measured at 2 ranks:
    # tail 0.37 -> 0.22 ms, 6.27 -> 6.19 ms/step
    compact_embedding_exchange: bool = True
    # N > 1: reduce-scatter + AdamW on this rank's shard + all-gather; measured
    # at 2 ranks no faster than the all-reduce (6.34 vs 6.27 ms/step), so off
    sharded_optimizer: bool = False


class Trainer:
    def __init__(self, cfg: GPTConfig, tcfg: TrainConfig, device, rank: int = 0, world: int = 1, group=None):
        self.cfg, self.tcfg = cfg, tcfg
        self.device = torch.device(device)
        self.rank, self.world = rank, world
        self.P = FlatParams(cfg, self.device, seed=tcfg.seed)   # same init on every rank
        self.model = GPT(cfg, self.P, fused_lmhead=tcfg.fused_lmhead)
        self.opt = AdamW(self.P, weight_decay=tcfg.weight_decay)
        # keep_grads=False: the optimizer clears the gradients it consumed and
        # the step needs no zeroing pass over the 256 MB gradient buffer
        self.opt.zero_grad = not tcfg.keep_grads
        # the optimizer runs per bucket, overlapped with the remaining backward,
        # right after that bucket's all-reduce (with one rank: as soon as the
        # bucket's gradients are final); the token table by rows
        overlap = self.device.type == "cuda" or world > 1
        self.reducer = BucketReducer(self.P, tcfg.bucket_mb << 20, group, optimizer=self.opt if overlap else None,
                                     sparse_rows=tcfg.sparse_embedding_rows and self.device.type == "cuda",
                                     compact_exchange=tcfg.compact_embedding_exchange,
                                     sharded=tcfg.sharded_optimizer)
        self.loader = ZipfLoader(tcfg.batch, tcfg.seq, cfg.vocab, tcfg.seed, rank)
        self.step_idx = 0
        self.warmup = min(tcfg.warmup, tcfg.steps // 5)
        self.tail_events = None   # set to a list to record (end of backward, end of step) events per step

    def lr(self, step: int) -> float:
        return lr_schedule(step, self.tcfg.peak_lr, self.warmup, self.tcfg.steps)

    def device_batch(self, inputs, targets):
        tok = torch.as_tensor(inputs, device=self.device)
        tgt = torch.as_tensor(targets, device=self.device)
        return tok, tgt

    def _step_body(self, tok: torch.Tensor, tgt: torch.Tensor) -> torch.Tensor:
        if not self.opt.zero_grad:
            self.P.grad.zero_()
        # the schedule (optax warmup_cosine_decay, nlearn/train.py:487-505) is
        # evaluated on the device: no per-step host copy for the host to race
        self.opt.advance_on_device(self.tcfg.peak_lr, self.warmup, self.tcfg.steps, self.tcfg.peak_lr / 10)
        self.reducer.begin_rows(tok)
        loss, saved = self.model.forward(tok, tgt)
        self.reducer.begin()
        self.model.backward(saved, on_grad_ready=self.reducer.ready)
        tail = None
        if self.tail_events is not None:  # device time of the exchange/optimizer tail after the backward
            tail = torch.cuda.Event(enable_timing=True)
            tail.record()
        self.reducer.finish()
        if self.reducer.optimizer is None:
            self.opt.step()
        if tail is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            self.tail_events.append((tail, end))
        return loss

    def step_on_device(self, tok: torch.Tensor, tgt: torch.Tensor) -> torch.Tensor:
        """One optimizer step on device-resident tokens; returns the loss tensor
        (not synchronised)."""
        loss = self._step_body(tok, tgt)
        self.step_idx += 1
        return loss

    # ------------------------------------------------------------- CUDA graph
    def capture_step(self) -> int:
        """Capture one whole training step (zero grads, schedule, forward,
        backward, AdamW) into a CUDA graph over static token buffers; replay
        with ``step_graphed``.  One rank only (the multi-rank step, with its
        NCCL buckets on a side stream, stays eager).  Run a few eager steps
        first so that every kernel and workspace is initialised.  Returns the
        number of library kernels in the graph."""
        if self.world != 1:
            raise RuntimeError("capture_step: single-rank only")
        B, S = self.tcfg.batch, self.tcfg.seq
        self._gtok = torch.zeros(B, S, device=self.device, dtype=torch.int32)
        self._gtgt = torch.zeros(B, S, device=self.device, dtype=torch.int32)
        self.opt.sync_device_step()
        t0 = self.opt.t
        from . import _lib
        n0 = _lib.lib.nl_launch_count()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._gloss = self._step_body(self._gtok, self._gtgt)
        self.opt.t = t0  # capture runs nothing; the counter advances per replay
        self.opt.t_dev_value = t0
        self.graph_launches = _lib.lib.nl_launch_count() - n0
        self._graph = g
        return self.graph_launches

    def step_graphed(self, tok: torch.Tensor, tgt: torch.Tensor) -> torch.Tensor:
        """Replay the captured step on this batch (device tensors, or pinned
        host tensors copied in asynchronously); returns the static loss tensor,
        valid until the next replay."""
        if self.opt.t_dev_value != self.opt.t:  # a resume or set_lr since the last step
            self.opt.sync_device_step()
        self._gtok.copy_(tok, non_blocking=True)
        self._gtgt.copy_(tgt, non_blocking=True)
        self._graph.replay()
        self.opt.t += 1
        self.opt.t_dev_value = self.opt.t
        self.step_idx += 1
        return self._gloss

    def train_step(self, inputs: np.ndarray, targets: np.ndarray) -> float:
        """Host batch in, host loss out (the reference's loop body)."""
        tok, tgt = self.device_batch(inputs, targets)
        return float(self.step_on_device(tok, tgt))

    def train_step_async(self, inputs: torch.Tensor, targets: torch.Tensor):
        """Host batch in (pinned CPU int32 tensors), host loss out one step
        late: the step is launched (the replayed CUDA graph at one rank when
        captured, else eager), its loss is copied into a pinned host slot, and
        the PREVIOUS step's loss is returned (None on the first call), so the
        host never waits for the step it has just queued.  ``flush_loss()``
        returns the last one."""
        if getattr(self, "_graph", None) is not None:
            loss = self.step_graphed(inputs, targets)
        else:
            loss = self.step_on_device(inputs.to(self.device, non_blocking=True),
                                       targets.to(self.device, non_blocking=True))
        if not hasattr(self, "_loss_slots"):
            self._loss_slots = [torch.zeros(1, dtype=torch.float32).pin_memory() for _ in range(2)]
            self._loss_events = [torch.cuda.Event(), torch.cuda.Event()]
            self._loss_k = 0
            self._loss_pending = None
        k = self._loss_k
        self._loss_slots[k].copy_(loss.reshape(1), non_blocking=True)
        self._loss_events[k].record()
        prev, self._loss_pending, self._loss_k = self._loss_pending, k, k ^ 1
        if prev is None:
            return None
        self._loss_events[prev].synchronize()
        return float(self._loss_slots[prev][0])

    def flush_loss(self):
        """The loss of the last train_step_async call (waits for that step)."""
        k = getattr(self, "_loss_pending", None)
        if k is None:
            return None
        self._loss_events[k].synchronize()
        self._loss_pending = None
        return float(self._loss_slots[k][0])

    # ------------------------------------------------------------- checkpoint
    def gather_state(self, grads: bool = False):
        """With the sharded optimizer each rank holds its own shard of the AdamW
        moments (and of the reduced gradient): all-gather them so that every
        rank has the whole state.  Collective (every rank calls it); a no-op
        otherwise.  save / save_reference call it."""
        bufs = [self.P.exp_avg, self.P.exp_avg_sq] + ([self.P.grad] if grads else [])
        self.reducer.gather_sharded(bufs)

    def save(self, path: str):
        self.gather_state()
        if self.rank != 0:
            return
        state = {"params": self.P.state_dict(), "step": self.step_idx, "opt_t": self.opt.t,
                 "loader_step": self.loader.step, "config": self.cfg.__dict__, "train": self.tcfg.__dict__}
        tmp = path + ".tmp"
        torch.save({k: (v if not isinstance(v, dict) else {kk: (vv.cpu() if torch.is_tensor(vv) else vv)
                                                           for kk, vv in v.items()}) for k, v in state.items()},
                   tmp)
        os.replace(tmp, path)

    def _named(self, buf: torch.Tensor) -> dict:
        return {name: self.P.view(buf, name).detach().cpu().numpy() for name, _, _ in self.P.specs}

    def _load_named(self, buf: torch.Tensor, named: dict):
        for name, shape, _ in self.P.specs:
            self.P.view(buf, name).copy_(torch.from_numpy(np.asarray(named[name], np.float32).reshape(shape)))

    def save_reference(self, path: str):
        """Resume state in the reference's pickle format ({params, opt_state,
        step}, nested numpy trees; nlearn/train.py:74-87)."""
        from .checkpoint import save_resume_state
        self.gather_state()
        if self.rank != 0:
            return
        save_resume_state(self._named(self.P.master), self._named(self.P.exp_avg), self._named(self.P.exp_avg_sq),
                          self.opt.t, self.step_idx, self.cfg, path)

    def load_reference(self, path: str) -> bool:
        """Resume from a reference-format pickle; False when the file is absent
        (nlearn/train.py:90-96).  The data stream continues at the step count."""
        from .checkpoint import load_resume_state
        st = load_resume_state(path, self.cfg)
        if st is None:
            return False
        params, mu, nu, count, step = st
        self._load_named(self.P.master, params)
        self._load_named(self.P.exp_avg, mu)
        self._load_named(self.P.exp_avg_sq, nu)
        self.P.refresh_shadow()
        self.opt.t = count
        self.step_idx = step
        self.loader.step = step
        return True

    def load(self, path: str):
        state = torch.load(path, map_location="cpu", weights_only=False)
        self.P.load_state_dict({k: v.to(self.device) for k, v in state["params"].items()})
        self.step_idx = state["step"]
        self.opt.t = state["opt_t"]
        self.loader.step = state["loader_step"]


def init_distributed():
    """(rank, world, local_rank) from torchrun's environment; NCCL when CUDA."""
    if "RANK" not in os.environ or int(os.environ.get("WORLD_SIZE", "1")) == 1:
        return 0, 1, 0
    backend = "nccl" if torch.cuda.is_available() else "gloo"
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        torch.cuda.set_device(local)
    dist.init_process_group(backend=backend, timeout=__import__("datetime").timedelta(seconds=120))
    return dist.get_rank(), dist.get_world_size(), local


def main(argv=None):  # pragma: no cover - CLI
    import argparse
    ap = argparse.ArgumentParser(description="nlearn-b200 data-parallel training (synthetic Zipf tokens)")
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--checkpoint", default=None)
    ap.add_argument("--resume", action="store_true")
    a = ap.parse_args(argv)
    rank, world, local = init_distributed()
    cfg = GPTConfig(max_seq=max(512, a.seq))
    tr = Trainer(cfg, TrainConfig(batch=a.batch, seq=a.seq, steps=a.steps, peak_lr=a.lr, seed=a.seed),
                 f"cuda:{local}", rank, world)
    if a.resume and a.checkpoint and os.path.exists(a.checkpoint):
        tr.load(a.checkpoint)
    while tr.step_idx < a.steps:
        t0 = time.time()
        loss = tr.train_step(*tr.loader.next())
        if rank == 0:
            print(f"step {tr.step_idx} loss {loss:.4f} {time.time() - t0:.3f}s", flush=True)
    if a.checkpoint:
        tr.save(a.checkpoint)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":  # pragma: no cover
    main()

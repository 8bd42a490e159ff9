"""The BASELINE GPT training step on the B200 kernels: forward, hand-written
backward, AdamW — all device work through ``libnl_ops.so``.

Model (the configuration the headline metric is quoted on): d_model 512,
8 heads of 64, 4 pre-LN blocks (LayerNorm with gain and bias, eps 1e-5),
GELU (tanh) FFN of 2048 with biases, learned position table, untied LM head,
vocab 50257, bf16 compute with f32 master weights.  It is the older nlearn
model the metric names (nlearn/model.py is now a RMSNorm/RoPE/SwiGLU variant);
initialisation follows nlearn/model.py (N(0, 0.02); output projections of the
residual branches scaled by (2 L)^-1/2, model.py:31, 130, 262).

Per block (M = batch*seq rows, activations bf16):
    h1  = LN1(x)                                   nl_layernorm_fwd
    qkv = h1 @ Wqkv                                nl_gemm_ex (bf16 out)       [M, 3D]
    o   = attention(q, k, v) read in place         nl_flash_attention_fwd_strided
    x2  = x + o @ Wo                               nl_gemm_ex (residual epilogue)
    h2  = LN2(x2)
    u   = gelu(h2 @ W1 + b1)  (pre-act saved)      nl_gemm_ex (bias+GELU epilogue)
    x3  = x2 + u @ W2 + b2                         nl_gemm_ex (bias+residual epilogue)
then LN_f and the loss, on one of the reference's two paths
(nlearn/train.py:270-285, chosen by NLEARN_FUSED_LMHEAD):
    fused (NLEARN_FUSED_LMHEAD=1, and the default here when the variable is
    unset): the LM-head CE without logits, nl_lce_fwd / nl_lce_bwd;
    materialised (NLEARN_FUSED_LMHEAD=0; the reference's default): logits =
    linear(h_f, W_head) as bf16 [M, V] (nl_gemm_ex), then the `ce_fwd` /
    `ce_bwd` pair as one fused pass writing dlogits over the logits in place
    (nl_ce_fwd_bwd), then dX = dlogits W^T and dW += h_f^T dlogits.
The backward
mirrors it; every weight gradient GEMM accumulates (f32) straight into its
slot of one flat gradient buffer, which the data-parallel reducer all-reduces
in buckets and AdamW consumes in place.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_handle
from .kernels.gemm import gemm_ex
from .kernels.cross_entropy import ce_fwd_bwd, lce_bwd_bf16_dx, lce_fwd_raw


def fused_lmhead_default() -> bool:
    """NLEARN_FUSED_LMHEAD as nlearn/train.py:28 reads it ("1" selects the
    fused LM-head CE), except that unset also means fused here: on B200 the
    fused path is the default and "0" selects the materialised one."""
    return os.environ.get("NLEARN_FUSED_LMHEAD", "1") != "0"


@dataclass(frozen=True)
class GPTConfig:
    vocab: int = 50257
    d_model: int = 512
    n_heads: int = 8
    n_layers: int = 4
    d_ff: int = 2048
    max_seq: int = 512
    ln_eps: float = 1e-5

    @property
    def vocab_padded(self) -> int:
        """LM-head row pitch: a multiple of 64 columns (16-byte TMA rows)."""
        return (self.vocab + 63) // 64 * 64


def param_specs(cfg: GPTConfig):
    """(name, shape, init) in gradient-production order of the backward:
    LM head first, embeddings last, so that contiguous buckets of the flat
    gradient buffer complete in order."""
    D, F, V = cfg.d_model, cfg.d_ff, cfg.vocab_padded
    rs = (2 * cfg.n_layers) ** -0.5
    specs = [("head.w", (D, V), ("normal", 0.02)), ("lnf.g", (D,), ("ones",)), ("lnf.b", (D,), ("zeros",))]
    for layer in reversed(range(cfg.n_layers)):
        p = f"blocks.{layer}."
        specs += [(p + "w2", (F, D), ("normal", 0.02 * rs)), (p + "b2", (D,), ("zeros",)),
                  (p + "w1", (D, F), ("normal", 0.02)), (p + "b1", (F,), ("zeros",)),
                  (p + "ln2.g", (D,), ("ones",)), (p + "ln2.b", (D,), ("zeros",)),
                  (p + "wo", (D, D), ("normal", 0.02 * rs)),
                  (p + "wqkv", (D, 3 * D), ("normal", 0.02)),
                  (p + "ln1.g", (D,), ("ones",)), (p + "ln1.b", (D,), ("zeros",))]
    specs += [("wpe", (cfg.max_seq, D), ("normal", 0.02)), ("wte", (cfg.vocab, D), ("normal", 0.02))]
    return specs


def _align(n: int, a: int = 64) -> int:
    return (n + a - 1) // a * a


# Every parameter starts on a 512-element (2 KB) boundary: then any run of
# whole parameters, padded to the next boundary, splits into 2, 4 or 8 equal
# 256-byte aligned shards (the sharded optimizer's reduce-scatter / all-gather).
PARAM_ALIGN = 512


class FlatParams:
    """All parameters in one f32 master buffer (+ bf16 compute copy, f32 grads,
    AdamW moments), each parameter a view at a 2 KB aligned offset."""

    def __init__(self, cfg: GPTConfig, device, seed: int = 0):
        self.cfg = cfg
        self.specs = param_specs(cfg)
        self.offsets = {}
        off = 0
        for name, shape, _ in self.specs:
            self.offsets[name] = (off, shape)
            off = _align(off + math.prod(shape), PARAM_ALIGN)
        self.numel = off
        self.device = torch.device(device)
        self.master = torch.zeros(self.numel, device=self.device, dtype=torch.float32)
        self.grad = torch.zeros_like(self.master)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.shadow = torch.zeros(self.numel, device=self.device, dtype=torch.bfloat16)
        gen = torch.Generator(device="cpu").manual_seed(seed)
        for name, shape, init in self.specs:
            v = self.view(self.master, name)
            if init[0] == "normal":
                t = torch.randn(*shape, generator=gen) * init[1]
                if name == "head.w":
                    t[:, cfg.vocab:] = 0.0  # vocabulary padding columns stay zero
                v.copy_(t)
            elif init[0] == "ones":
                v.fill_(1.0)
        self.refresh_shadow()

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        off, shape = self.offsets[name]
        return buf[off:off + math.prod(shape)].view(*shape)

    def p(self, name):  # bf16 compute copy
        return self.view(self.shadow, name)

    def f(self, name):  # f32 master
        return self.view(self.master, name)

    def g(self, name):  # f32 gradient
        return self.view(self.grad, name)

    def refresh_shadow(self):
        check(lib.nl_cast_bf16(ptr(self.master), ptr(self.shadow), self.numel, stream_handle()), "nl_cast_bf16")

    def state_dict(self):
        return {"master": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq}

    def load_state_dict(self, sd):
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.refresh_shadow()


def _ln_fwd(x, g, b, eps, M, D):
    y = torch.empty_like(x)
    mean = torch.empty(M, device=x.device, dtype=torch.float32)
    rstd = torch.empty_like(mean)
    check(lib.nl_layernorm_fwd(ptr(x), ptr(g), ptr(b), ptr(y), ptr(mean), ptr(rstd), M, D, eps, stream_handle()),
          "nl_layernorm_fwd")
    return y, mean, rstd


def _ln_bwd(dy, x, mean, rstd, g, dres, dres_bf, dg, db, M, D, accumulate, dsum=None):
    """LayerNorm backward into the residual gradient; ``dsum`` (optional)
    accumulates the column sums of the new residual gradient, i.e. the bias
    gradient of the FFN output projection that consumes it next."""
    check(lib.nl_layernorm_bwd(ptr(dy), ptr(x), ptr(mean), ptr(rstd), ptr(g), ptr(dres), ptr(dres_bf), ptr(dg),
                               ptr(db), ptr(dsum), M, D, int(accumulate), stream_handle()), "nl_layernorm_bwd")


class GPT:
    """Forward + backward of the BASELINE GPT on one device's micro-batch."""

    def __init__(self, cfg: GPTConfig, params: FlatParams, fused_lmhead: bool | None = None):
        self.cfg = cfg
        self.P = params
        self.fused_lmhead = fused_lmhead_default() if fused_lmhead is None else bool(fused_lmhead)

    # ------------------------------------------------------------------ forward
    def forward(self, tok: torch.Tensor, targets: torch.Tensor):
        """tok, targets: int32 [B, S] on the device.  Returns (mean loss tensor,
        saved activations)."""
        cfg, P = self.cfg, self.P
        B, S = tok.shape
        M, D, H, F = B * S, cfg.d_model, cfg.n_heads, cfg.d_ff
        dev = tok.device
        x = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
        check(lib.nl_embed_fwd(ptr(tok), ptr(P.p("wte")), ptr(P.p("wpe")), ptr(x), M, S, D, stream_handle()),
              "nl_embed_fwd")
        saved = {"tok": tok, "targets": targets, "B": B, "S": S, "layers": []}
        qs = (3 * D, 64, S * 3 * D)          # Q/K/V strides inside qkv [B, S, 3, H, 64]
        os_ = (D, 64, S * D)                 # O strides [B, S, H, 64]
        for layer in range(cfg.n_layers):
            pre = f"blocks.{layer}."
            h1, m1, r1 = _ln_fwd(x, P.f(pre + "ln1.g"), P.f(pre + "ln1.b"), cfg.ln_eps, M, D)
            qkv = gemm_ex(h1, P.p(pre + "wqkv"), out_dtype=torch.bfloat16)
            o = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
            L = torch.empty(B * H, S, device=dev, dtype=torch.float32)
            check(lib.nl_flash_attention_fwd_strided(ptr(qkv), ptr(qkv[:, D:]), ptr(qkv[:, 2 * D:]), *qs, ptr(o),
                                                     *os_, ptr(L), B, H, S, 64, stream_handle()), "attn fwd")
            x2 = gemm_ex(o, P.p(pre + "wo"), out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID, resid=x)
            h2, m2, r2 = _ln_fwd(x2, P.f(pre + "ln2.g"), P.f(pre + "ln2.b"), cfg.ln_eps, M, D)
            a = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
            u = gemm_ex(h2, P.p(pre + "w1"), out_dtype=torch.bfloat16, epilogue=_lib.EPI_BIAS_GELU,
                        bias=P.f(pre + "b1"), aux=a)
            x3 = gemm_ex(u, P.p(pre + "w2"), out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID,
                         bias=P.f(pre + "b2"), resid=x2)
            saved["layers"].append(dict(x=x, h1=h1, m1=m1, r1=r1, qkv=qkv, o=o, L=L, x2=x2, h2=h2, m2=m2, r2=r2,
                                        a=a, u=u))
            x = x3
        hf, mf, rf = _ln_fwd(x, P.f("lnf.g"), P.f("lnf.b"), cfg.ln_eps, M, D)
        t = targets.reshape(-1)
        V = cfg.vocab
        saved.update(xf=x, hf=hf, mf=mf, rf=rf)
        if self.fused_lmhead:
            loss_rows, lse = lce_fwd_raw(hf, P.p("head.w")[:, :V], t)
            saved["lse"] = lse
        else:
            # logits bf16 [M, V] at the head's padded row pitch, then loss, lse and
            # dlogits = (softmax - onehot) / M from one read, written in place
            logits = torch.empty(M, cfg.vocab_padded, device=dev, dtype=torch.bfloat16)[:, :V]
            gemm_ex(hf, P.p("head.w")[:, :V], out=logits)
            loss_rows, lse, _ = ce_fwd_bwd(logits, t, out=logits)
            saved.update(lse=lse, dlogits=logits)
        return loss_rows.mean(), saved

    # ------------------------------------------------------------------ backward
    def backward(self, saved, on_grad_ready=None):
        """Accumulates d(mean loss) into P.grad.  ``on_grad_ready(name)`` is
        called once a parameter's gradient is final AND the backward has made
        its last read of that parameter, so the callee may reduce the gradient
        and update the weight in place (bucket trigger)."""
        cfg, P = self.cfg, self.P
        B, S = saved["B"], saved["S"]
        M, D, H, F, V = B * S, cfg.d_model, cfg.n_heads, cfg.d_ff, cfg.vocab
        dev = saved["hf"].device
        notify = on_grad_ready or (lambda name: None)
        t = saved["targets"].reshape(-1)
        if self.fused_lmhead:
            # LM head + CE: dhf written in bf16 by the dX GEMM, d head.w accumulated in place
            dhf_bf = lce_bwd_bf16_dx(saved["hf"], P.p("head.w")[:, :V], t, saved["lse"], dW=P.g("head.w")[:, :V])
            notify("head.w")
        else:
            dl = saved["dlogits"]                      # bf16 [M, V], already / M
            gemm_ex(saved["hf"], dl, a_trans=True, out=P.g("head.w")[:, :V], epilogue=_lib.EPI_ACCUM)
            dhf_bf = gemm_ex(dl, P.p("head.w")[:, :V], b_trans=True, out_dtype=torch.bfloat16)
            notify("head.w")
        dres = torch.empty(M, D, device=dev, dtype=torch.float32)
        dres_bf = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
        last = f"blocks.{cfg.n_layers - 1}."
        _ln_bwd(dhf_bf, saved["xf"], saved["mf"], saved["rf"], P.f("lnf.g"), dres, dres_bf, P.g("lnf.g"),
                P.g("lnf.b"), M, D, accumulate=False, dsum=P.g(last + "b2"))
        notify("lnf.g"); notify("lnf.b")
        qs = (3 * D, 64, S * 3 * D)
        os_ = (D, 64, S * D)
        for layer in reversed(range(cfg.n_layers)):
            pre = f"blocks.{layer}."
            sv = saved["layers"][layer]
            # x3 = x2 + u @ W2 + b2
            # (b2's gradient, the column sums of dres, came with the LayerNorm backward that made dres)
            gemm_ex(sv["u"], dres_bf, a_trans=True, out=P.g(pre + "w2"), epilogue=_lib.EPI_ACCUM)
            da = gemm_ex(dres_bf, P.p(pre + "w2"), b_trans=True, out_dtype=torch.bfloat16,
                         epilogue=_lib.EPI_DGELU, aux=sv["a"])           # d(pre-activation)
            notify(pre + "w2"); notify(pre + "b2")   # (after the last read of W2)
            gemm_ex(sv["h2"], da, a_trans=True, out=P.g(pre + "w1"), epilogue=_lib.EPI_ACCUM)
            check(lib.nl_colsum_bf16(ptr(da), ptr(P.g(pre + "b1")), M, F, stream_handle()), "colsum")
            dh2 = gemm_ex(da, P.p(pre + "w1"), b_trans=True, out_dtype=torch.bfloat16)
            notify(pre + "w1"); notify(pre + "b1")
            _ln_bwd(dh2, sv["x2"], sv["m2"], sv["r2"], P.f(pre + "ln2.g"), dres, dres_bf, P.g(pre + "ln2.g"),
                    P.g(pre + "ln2.b"), M, D, accumulate=True)
            notify(pre + "ln2.g"); notify(pre + "ln2.b")
            # x2 = x + o @ Wo
            gemm_ex(sv["o"], dres_bf, a_trans=True, out=P.g(pre + "wo"), epilogue=_lib.EPI_ACCUM)
            do = gemm_ex(dres_bf, P.p(pre + "wo"), b_trans=True, out_dtype=torch.bfloat16)
            notify(pre + "wo")
            dqkv = torch.empty(M, 3 * D, device=dev, dtype=torch.bfloat16)
            Dws = torch.empty(B * H, S, device=dev, dtype=torch.float32)
            acc = torch.empty(B * H, S, 64, device=dev, dtype=torch.float32)
            qkv = sv["qkv"]
            check(lib.nl_flash_attention_bwd_strided(ptr(qkv), ptr(qkv[:, D:]), ptr(qkv[:, 2 * D:]), *qs,
                                                     ptr(sv["o"]), ptr(do), *os_, ptr(sv["L"]), ptr(Dws),
                                                     ptr(dqkv), ptr(dqkv[:, D:]), ptr(dqkv[:, 2 * D:]), ptr(acc),
                                                     B, H, S, 64, stream_handle()), "attn bwd")
            gemm_ex(sv["h1"], dqkv, a_trans=True, out=P.g(pre + "wqkv"), epilogue=_lib.EPI_ACCUM)
            dh1 = gemm_ex(dqkv, P.p(pre + "wqkv"), b_trans=True, out_dtype=torch.bfloat16)
            notify(pre + "wqkv")
            _ln_bwd(dh1, sv["x"], sv["m1"], sv["r1"], P.f(pre + "ln1.g"), dres, dres_bf, P.g(pre + "ln1.g"),
                    P.g(pre + "ln1.b"), M, D, accumulate=True,
                    dsum=P.g(f"blocks.{layer - 1}.b2") if layer > 0 else None)
            notify(pre + "ln1.g"); notify(pre + "ln1.b")
        check(lib.nl_embed_bwd(ptr(saved["tok"]), ptr(dres), ptr(P.g("wte")), ptr(P.g("wpe")), M, S, D,
                               stream_handle()), "nl_embed_bwd")
        notify("wpe"); notify("wte")


def lr_schedule(step: int, peak_lr: float, warmup: int, decay_steps: int) -> float:
    """optax.warmup_cosine_decay_schedule(0, peak, warmup, decay_steps, peak/10)
    as nlearn/train.py:487-505 builds it; ``step`` counts from 0."""
    end = peak_lr / 10
    if warmup > 0 and step < warmup:
        return peak_lr * step / warmup
    if decay_steps <= warmup:
        return end
    frac = min(max(step - warmup, 0), decay_steps - warmup) / (decay_steps - warmup)
    return end + (peak_lr - end) * 0.5 * (1 + math.cos(math.pi * frac))


class AdamW:
    """Fused AdamW over the flat parameter buffer (nl_adamw_step)."""

    def __init__(self, params: FlatParams, b1=0.9, b2=0.999, eps=1e-8, weight_decay=0.1):
        self.P = params
        self.b1, self.b2, self.eps, self.wd = b1, b2, eps, weight_decay
        self.t = 0
        self.hyper = torch.zeros(3, device=params.device, dtype=torch.float32)
        self._hyper_host = torch.zeros(3, dtype=torch.float32).pin_memory() if params.device.type == "cuda" \
            else torch.zeros(3)
        self.t_dev = torch.zeros(1, device=params.device, dtype=torch.int32)  # device step counter
        self.t_dev_value = 0   # what t_dev holds (host view); None when unknown
        self.zero_grad = False  # clear each gradient element once AdamW has read it

    def set_lr(self, lr: float):
        """Stage an explicit learning rate (and this step's bias corrections)
        into device memory.  Synchronous with respect to the host buffer: the
        copy is complete when this returns, so a host that runs ahead of the
        device cannot overwrite a value still waiting to be copied (the
        training step itself uses advance_on_device, with no host copy)."""
        self.t += 1
        h = self._hyper_host
        h[0] = lr
        h[1] = 1 - self.b1 ** self.t
        h[2] = 1 - self.b2 ** self.t
        self.hyper.copy_(h, non_blocking=True)
        torch.cuda.current_stream().synchronize() if self.hyper.is_cuda else None
        self.t_dev_value = None  # the device counter no longer follows t

    def advance_on_device(self, peak_lr: float, warmup: int, decay_steps: int, end_lr: float):
        """One step of the schedule on the device: a one-thread kernel advances
        the device step counter and writes the warmup-cosine lr and the bias
        corrections into ``hyper`` (no host-to-device copy, so eager steps can
        run ahead of the device and a captured CUDA graph replays it)."""
        if self.t_dev_value != self.t:
            self.sync_device_step()
        self.t += 1
        check(lib.nl_adamw_schedule(ptr(self.hyper), ptr(self.t_dev), peak_lr, warmup, decay_steps, end_lr, self.b1,
                                    self.b2, stream_handle()), "nl_adamw_schedule")
        self.t_dev_value = self.t

    def sync_device_step(self):
        """Set the device step counter to ``t`` (after a resume, or set_lr)."""
        self.t_dev.fill_(self.t)
        self.t_dev_value = self.t

    def step(self):
        self.step_range(0, self.P.numel)

    def step_range(self, start: int, end: int):
        """AdamW on elements [start, end) of the flat buffers (start, end
        multiples of 4), on the current stream.  With ``zero_grad`` set the
        kernel clears the gradients it has read."""
        P = self.P
        n = end - start
        check(lib.nl_adamw_step(ptr(P.master[start:]), ptr(P.grad[start:]), ptr(P.exp_avg[start:]),
                                ptr(P.exp_avg_sq[start:]), ptr(P.shadow[start:]), n, ptr(self.hyper), self.b1,
                                self.b2, self.eps, self.wd, int(self.zero_grad), stream_handle()), "nl_adamw_step")

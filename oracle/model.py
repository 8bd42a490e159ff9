"""CPU oracle of the BASELINE GPT training step — TEST INFRASTRUCTURE ONLY.

A float32 PyTorch-on-CPU restatement (autograd for the backward) of the model
and optimizer the headline metric trains:
  * model: nlearn's d512 / 8 heads / 4 pre-LN blocks / GELU(tanh) 4x FFN /
    learned positions / untied head (the metric's configuration; block
    structure nlearn/model.py:315-324, attention nlearn/attention.py:138-156,
    LayerNorm + GELU as iree_metal/kernels/test/bf16_metal_test.py:6-12);
  * loss: mean softmax CE of the next token (nlearn/train.py:270-285);
  * optimizer: optax.adamw(b1 .9, b2 .999, eps 1e-8, wd .1 on every leaf)
    with warmup_cosine_decay_schedule (nlearn/train.py:487-508), written out
    from optax's published update rule.
Parity of the optimizer is unpinned by any reference test (optax is a
third-party dependency absent here); the formulas are restated.

Pinned: tests/golden/ln_gelu.npz (the reference's ln_gelu) pins
``layer_norm`` + ``gelu_tanh`` + residual; the flash fixtures' ``O_std``
(the reference's ``_attention_standard``) pin ``causal_attention``; and
tests/golden/model_small.npz pins ``OracleGPT.hidden`` / ``logits`` / ``loss``
on a small model run through the reference's own ``block_forward``,
``linear``, ``attention`` and one-hot ``cross_entropy``.  The gradients are
autograd of that pinned forward.

Parameters are keyed by the same names as nlearn_b200.model.param_specs so
tests can load the exact initial weights of the GPU run.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use this module.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def layer_norm(x, g, b, eps=1e-5):
    """LayerNorm with gain and bias over the last dim, biased variance
    (iree_metal/kernels/test/bf16_metal_test.py:8-10)."""
    return F.layer_norm(x, (x.shape[-1],), g, b, eps)


def gelu_tanh(h):
    """tanh-approximated GELU (bf16_metal_test.py:11)."""
    return F.gelu(h, approximate="tanh")


def causal_attention(Q, K, V):
    """softmax(Q K^T / sqrt(d) + causal mask) V over [..., s, d]
    (nlearn/attention.py:138-156 `_attention_standard`)."""
    S = Q.shape[-2]
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    sc = (Q @ K.transpose(-1, -2)) / math.sqrt(Q.shape[-1])
    return torch.softmax(sc.masked_fill(mask, float("-inf")), -1) @ V


class OracleGPT:
    def __init__(self, params: dict, n_layers=4, n_heads=8, vocab=50257, eps=1e-5):
        # params: name -> f32 CPU tensor (head.w may be column-padded)
        self.p = {k: torch.as_tensor(v).detach().clone().float().requires_grad_(True) for k, v in params.items()}
        self.L, self.H, self.V, self.eps = n_layers, n_heads, vocab, eps

    def loss(self, tok: torch.Tensor, tgt: torch.Tensor) -> torch.Tensor:
        logits = self.logits(tok)
        return F.cross_entropy(logits.reshape(-1, self.V), tgt.reshape(-1).long())

    def hidden(self, tok: torch.Tensor) -> torch.Tensor:
        """[B, S] tokens -> final-LayerNorm hidden states [B, S, D]: the
        pre-LN block wiring of nlearn/model.py:315-324 (x += attn(LN1 x);
        x += ffn(LN2 x)) at the BASELINE architecture."""
        p, H = self.p, self.H
        B, S = tok.shape
        D = p["wte"].shape[1]
        x = p["wte"][tok.long()] + p["wpe"][:S][None]
        for layer in range(self.L):
            q = f"blocks.{layer}."
            h = layer_norm(x, p[q + "ln1.g"], p[q + "ln1.b"], self.eps)
            qkv = (h @ p[q + "wqkv"]).view(B, S, 3, H, D // H)
            Q, K, V = (qkv[:, :, i].transpose(1, 2) for i in range(3))
            o = causal_attention(Q, K, V).transpose(1, 2).reshape(B, S, D)
            x = x + o @ p[q + "wo"]
            h = layer_norm(x, p[q + "ln2.g"], p[q + "ln2.b"], self.eps)
            u = gelu_tanh(h @ p[q + "w1"] + p[q + "b1"])
            x = x + u @ p[q + "w2"] + p[q + "b2"]
        return layer_norm(x, p["lnf.g"], p["lnf.b"], self.eps)

    def logits(self, tok: torch.Tensor) -> torch.Tensor:
        """[B, S] tokens -> [B, S, V] f32 logits (the model forward of
        nlearn/model.py:361-398 at the BASELINE architecture)."""
        return self.hidden(tok) @ self.p["head.w"][:, :self.V]

    def grads(self):
        return {k: (v.grad if v.grad is not None else torch.zeros_like(v)) for k, v in self.p.items()}


def lr_at(step, peak, warmup, decay_steps):
    """optax.warmup_cosine_decay_schedule(0, peak, warmup, decay_steps, peak/10)."""
    end = peak / 10
    if warmup > 0 and step < warmup:
        return peak * step / warmup
    if decay_steps <= warmup:
        return end
    frac = min(max(step - warmup, 0), decay_steps - warmup) / (decay_steps - warmup)
    return end + (peak - end) * 0.5 * (1 + math.cos(math.pi * frac))


class OracleAdamW:
    """optax.adamw update: m, v EMAs; bias-corrected; decoupled decay."""

    def __init__(self, params: dict, b1=0.9, b2=0.999, eps=1e-8, wd=0.1):
        self.params = params
        self.b1, self.b2, self.eps, self.wd = b1, b2, eps, wd
        self.m = {k: torch.zeros_like(v) for k, v in params.items()}
        self.v = {k: torch.zeros_like(v) for k, v in params.items()}
        self.t = 0

    @torch.no_grad()
    def step(self, lr):
        self.t += 1
        bc1, bc2 = 1 - self.b1 ** self.t, 1 - self.b2 ** self.t
        for k, p in self.params.items():
            g = p.grad if p.grad is not None else torch.zeros_like(p)
            self.m[k].mul_(self.b1).add_(g, alpha=1 - self.b1)
            self.v[k].mul_(self.b2).addcmul_(g, g, value=1 - self.b2)
            upd = (self.m[k] / bc1) / ((self.v[k] / bc2).sqrt() + self.eps) + self.wd * p
            p.sub_(lr * upd)
            p.grad = None

"""Text generation on B200: prompt prefill + KV-cache decode steps.

Mirrors the reference's ``generate(params, prompt_ids, n_tokens, key,
temperature)`` (nlearn/model.py:449-465): same prompt trimming (keep the last
``max_seq - n_tokens`` prompt tokens), same output (prompt followed by the new
tokens), sampling from softmax(logits / temperature) (temperature 0 = greedy).
The reference re-runs the whole model over the full token buffer for every
new token (model.py:417-447); here the prompt is run once through the
training kernels (flash forward, fused-epilogue GEMMs), every layer's q|k|v
rows are kept as the KV cache, and each further token is one decode step:

    embed(tok, pos) -> per layer: LN + qkv GEMM (M = batch), decode attention
    (appends k|v at pos), proj GEMM + residual, LN + FFN up + bias + GELU,
    FFN down + bias + residual -> final LN + LM-head GEMM (f32 logits)
    -> sampler -> pos += 1

(each "LN + GEMM" is one kernel at batch <= 8: the small-M GEMM applies the
LayerNorm while staging its A operand).

The position lives in device memory, so one decode step is captured into a
CUDA graph once and replayed per token.  The random stream (seed, position,
row) is this library's own counter-based one (the reference's JAX PRNG key is
replaced by an integer seed).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from ._lib import check, lib, ptr, stream_handle
from .kernels.gemm import gemm_ex
from .model import FlatParams, GPTConfig


class Decoder:
    """Static buffers, KV caches and the captured decode step for one batch
    size; ``generate`` may be called repeatedly."""

    def __init__(self, params: FlatParams, cfg: GPTConfig, batch: int = 1, max_len: int | None = None):
        self.P, self.cfg, self.B = params, cfg, batch
        self.S = max_len or cfg.max_seq
        if self.S > cfg.max_seq:
            raise ValueError(f"max_len {self.S} exceeds the positional table ({cfg.max_seq})")
        B, D, F, Vp = batch, cfg.d_model, cfg.d_ff, cfg.vocab_padded
        dev = params.device
        bf = dict(device=dev, dtype=torch.bfloat16)
        self.cache = [torch.zeros(B, self.S, 3 * D, **bf) for _ in range(cfg.n_layers)]
        self.tok = torch.zeros(B, device=dev, dtype=torch.int32)
        self.pos = torch.zeros(1, device=dev, dtype=torch.int32)
        self.out = torch.zeros(B, self.S + 1, device=dev, dtype=torch.int32)
        self.x, self.x2, self.x3, self.h, self.o = (torch.empty(B, D, **bf) for _ in range(5))
        self.qkv = torch.empty(B, 3 * D, **bf)
        self.a, self.u = torch.empty(B, F, **bf), torch.empty(B, F, **bf)
        self.mean = torch.empty(B, device=dev, dtype=torch.float32)
        self.rstd = torch.empty_like(self.mean)
        self.logits = torch.empty(B, Vp, device=dev, dtype=torch.float32)
        nbytes = lib.nl_decode_workspace_bytes(B, cfg.n_heads, self.S)
        self.ws = torch.zeros(nbytes, device=dev, dtype=torch.uint8)
        self._graph = None
        self._graph_key = None
        self._fuse_ln = True  # LayerNorm folded into the small-M GEMM (batch <= 8)

    # ------------------------------------------------------------------ pieces
    def _ln(self, x, y, g, b, M):
        check(lib.nl_layernorm_fwd(ptr(x), ptr(g), ptr(b), ptr(y), ptr(self.mean if M == self.B else
                                                                          torch.empty(M, device=x.device)),
                                   ptr(self.rstd if M == self.B else torch.empty(M, device=x.device)), M,
                                   self.cfg.d_model, self.cfg.ln_eps, stream_handle()), "nl_layernorm_fwd")

    def _head_and_sample(self, hf_rows, seed: int, temperature: float):
        V = self.cfg.vocab
        gemm_ex(hf_rows, self.P.p("head.w")[:, :V], out=self.logits[:, :V])
        self._sample(seed, temperature)

    def _sample(self, seed: int, temperature: float):
        V = self.cfg.vocab
        check(lib.nl_sample_tokens(ptr(self.logits), self.logits.stride(0), V, float(temperature), int(seed),
                                   ptr(self.pos), ptr(self.tok), ptr(self.out), self.out.stride(0), self.B,
                                   stream_handle()), "nl_sample_tokens")
        check(lib.nl_decode_advance(ptr(self.pos), stream_handle()), "nl_decode_advance")

    def prefill(self, prompt: torch.Tensor, seed: int, temperature: float):
        """Run the [B, P] prompt, fill the caches for positions 0..P-1, sample
        the token for position P; afterwards pos = P."""
        cfg, P = self.cfg, self.P
        B, Pl = prompt.shape
        D, H, F = cfg.d_model, cfg.n_heads, cfg.d_ff
        M = B * Pl
        dev = prompt.device
        tok = prompt.to(torch.int32).contiguous()
        self.out[:, :Pl] = tok
        x = torch.empty(M, D, device=dev, dtype=torch.bfloat16)
        check(lib.nl_embed_fwd(ptr(tok), ptr(P.p("wte")), ptr(P.p("wpe")), ptr(x), M, Pl, D, stream_handle()),
              "nl_embed_fwd")
        h = torch.empty_like(x)
        o = torch.empty_like(x)
        L = torch.empty(B * H, Pl, device=dev, dtype=torch.float32)
        qs = (3 * D, 64, Pl * 3 * D)
        os_ = (D, 64, Pl * D)
        for layer in range(cfg.n_layers):
            pre = f"blocks.{layer}."
            self._ln(x, h, P.f(pre + "ln1.g"), P.f(pre + "ln1.b"), M)
            qkv = gemm_ex(h, P.p(pre + "wqkv"), out_dtype=torch.bfloat16)
            self.cache[layer][:, :Pl].copy_(qkv.view(B, Pl, 3 * D))
            check(lib.nl_flash_attention_fwd_strided(ptr(qkv), ptr(qkv[:, D:]), ptr(qkv[:, 2 * D:]), *qs, ptr(o),
                                                     *os_, ptr(L), B, H, Pl, 64, stream_handle()), "attn fwd")
            x2 = gemm_ex(o, P.p(pre + "wo"), out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID, resid=x)
            self._ln(x2, h, P.f(pre + "ln2.g"), P.f(pre + "ln2.b"), M)
            a = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
            u = gemm_ex(h, P.p(pre + "w1"), out_dtype=torch.bfloat16, epilogue=_lib.EPI_BIAS_GELU,
                        bias=P.f(pre + "b1"), aux=a)
            x = gemm_ex(u, P.p(pre + "w2"), out_dtype=torch.bfloat16, epilogue=_lib.EPI_RESID,
                        bias=P.f(pre + "b2"), resid=x2)
        self._ln(x, h, P.f("lnf.g"), P.f("lnf.b"), M)
        self.pos.fill_(Pl - 1)
        self._head_and_sample(h.view(B, Pl, D)[:, -1], seed, temperature)

    def _ln_linear(self, x, g, b, W, out, epilogue=_lib.EPI_STORE, bias=None, aux=None):
        """out = LayerNorm(x) . W (+ epilogue): one fused small-M kernel when the
        shape allows (batch <= 8), else LayerNorm then the GEMM."""
        if self._fuse_ln:
            dt = _lib.F32 if out.dtype == torch.float32 else _lib.BF16
            st = lib.nl_linear_ln_small(ptr(x), x.stride(0), ptr(g), ptr(b), self.cfg.ln_eps, ptr(W), W.stride(0),
                                        ptr(out), out.stride(0), dt, out.shape[0], out.shape[1], W.shape[0],
                                        epilogue, ptr(bias), ptr(aux), None, stream_handle())
            if st == 0:
                return
            if st != -1:  # anything but NL_ERR_SHAPE ("not a shape the fused kernel takes") is an error
                check(st, "nl_linear_ln_small")
            self._fuse_ln = False
        self._ln(x, self.h, g, b, self.B)
        gemm_ex(self.h, W, out=out, epilogue=epilogue, bias=bias, aux=aux)

    def step(self, seed: int, temperature: float):
        """One decode step: the token in ``tok`` at position ``pos``."""
        cfg, P = self.cfg, self.P
        D, H, V = cfg.d_model, cfg.n_heads, cfg.vocab
        check(lib.nl_decode_embed(ptr(self.tok), ptr(self.pos), ptr(P.p("wte")), ptr(P.p("wpe")), ptr(self.x),
                                  self.B, D, stream_handle()), "nl_decode_embed")
        x = self.x
        for layer in range(cfg.n_layers):
            pre = f"blocks.{layer}."
            self._ln_linear(x, P.f(pre + "ln1.g"), P.f(pre + "ln1.b"), P.p(pre + "wqkv"), self.qkv)
            check(lib.nl_decode_attention(ptr(self.qkv), ptr(self.cache[layer]), ptr(self.o), ptr(self.pos),
                                          ptr(self.ws), self.ws.numel(), self.B, H, self.S, 64, stream_handle()),
                  "nl_decode_attention")
            gemm_ex(self.o, P.p(pre + "wo"), out=self.x2, epilogue=_lib.EPI_RESID, resid=x)
            self._ln_linear(self.x2, P.f(pre + "ln2.g"), P.f(pre + "ln2.b"), P.p(pre + "w1"), self.u,
                            epilogue=_lib.EPI_BIAS_GELU, bias=P.f(pre + "b1"), aux=self.a)
            gemm_ex(self.u, P.p(pre + "w2"), out=self.x3, epilogue=_lib.EPI_RESID, bias=P.f(pre + "b2"),
                    resid=self.x2)
            x = self.x3
        self._ln_linear(x, P.f("lnf.g"), P.f("lnf.b"), P.p("head.w")[:, :V], self.logits[:, :V])
        self._sample(seed, temperature)

    def capture(self, seed: int, temperature: float):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step(seed, temperature)
        self._graph, self._graph_key = g, (int(seed), float(temperature))

    # ------------------------------------------------------------------ API
    def generate(self, prompt_ids, n_tokens: int, seed: int = 0, temperature: float = 1.0,
                 use_graph: bool = True) -> np.ndarray:
        """[P] or [B, P] prompt ids -> [B, P' + n_tokens] (P' after trimming)."""
        p = np.asarray(prompt_ids, np.int32)
        if p.ndim == 1:
            p = p[None]
        if p.shape[0] != self.B:
            raise ValueError(f"decoder built for batch {self.B}, prompt batch {p.shape[0]}")
        if n_tokens <= 0:
            return p.copy()
        if n_tokens >= self.S:
            raise ValueError(f"n_tokens {n_tokens} must be below max_len {self.S}")
        if p.shape[1] + n_tokens > self.S:  # keep the most recent prompt tokens (model.py:462-463)
            p = p[:, -(self.S - n_tokens):]
        Pl = p.shape[1]
        self.prefill(torch.from_numpy(p).to(self.P.device), seed, temperature)
        for i in range(1, n_tokens):
            if use_graph and i >= 2:
                if self._graph is None or self._graph_key != (int(seed), float(temperature)):
                    self.capture(seed, temperature)
                self._graph.replay()
            else:
                self.step(seed, temperature)
        return self.out[:, :Pl + n_tokens].cpu().numpy()


def generate(trainer_or_params, prompt_ids, n_tokens: int, seed: int = 0, temperature: float = 1.0,
             cfg: GPTConfig | None = None) -> np.ndarray:
    """Reference-shaped entry point: a Trainer (or FlatParams + cfg), a 1-D or
    [B, P] prompt -> tokens (1-D for a 1-D prompt)."""
    P = getattr(trainer_or_params, "P", trainer_or_params)
    cfg = cfg or getattr(trainer_or_params, "cfg", None) or P.cfg
    p = np.asarray(prompt_ids, np.int32)
    dec = Decoder(P, cfg, batch=1 if p.ndim == 1 else p.shape[0])
    out = dec.generate(p, n_tokens, seed, temperature)
    return out[0] if p.ndim == 1 else out

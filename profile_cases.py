"""Single-kernel microbenchmarks of the hot-path operators at chosen shapes.

    python profile_cases.py CASE [--M .. --N .. --K ..] [--iters N]

CASE is one of: head_fwd, head_bwd (fused LM-head CE), gemm (plain GEMM;
--layout nn|nt|tn|tt gives the transposition of A and B as in gemm_ex),
attn_fwd, attn_bwd, ce (materialised-logit CE fwd+bwd, in place), colsum (bias
gradient: column sums of a bf16 [M, N]).  Prints one
JSON line with the CUDA-event time per call and the achieved TFLOP/s or GB/s.
Small shapes make it the command to run under Nsight Compute for one kernel.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def _time(fn, iters):
    for _ in range(3):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--M", type=int, default=16384)
    ap.add_argument("--N", type=int, default=50257)
    ap.add_argument("--K", type=int, default=512)
    ap.add_argument("--heads", type=int, default=256)
    ap.add_argument("--seq", type=int, default=512)
    ap.add_argument("--layout", default="nn")
    ap.add_argument("--chunk", type=int, default=0)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--pad", type=int, default=0, help="extra elements of row pitch for the GEMM operands")
    ap.add_argument("--accum", action="store_true", help="GEMM into an f32 accumulator (weight-gradient form)")
    ap.add_argument("--epi", default="store", choices=["store", "bias", "bias_gelu", "resid", "dgelu"],
                    help="fused epilogue of the bf16-output GEMM")
    a = ap.parse_args(argv)
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    out = {"case": a.case}
    if a.case in ("head_fwd", "head_bwd"):
        from nlearn_b200.kernels.cross_entropy import lce_bwd_raw, lce_fwd_raw
        M, D, V = a.M, a.K, a.N
        Vp = (V + 63) // 64 * 64
        X = torch.randn(M, D, device=dev).bfloat16()
        W = torch.zeros(D, Vp, device=dev, dtype=torch.bfloat16)
        W[:, :V] = (torch.randn(D, V, device=dev) * 0.02).bfloat16()
        Wv = W[:, :V]
        t = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        loss, lse = lce_fwd_raw(X, Wv, t)
        if a.case == "head_fwd":
            ms = _time(lambda: lce_fwd_raw(X, Wv, t), a.iters)
            flop = 2 * M * D * V
        else:
            dX = torch.zeros(M, D, device=dev)
            dW = torch.zeros(D, Vp, device=dev)[:, :V]
            ms = _time(lambda: lce_bwd_raw(X, Wv, t, lse, dX=dX, dW=dW, dw_accumulate=True,
                                           chunk=a.chunk or None), a.iters)
            flop = 4 * M * D * V  # algorithmic: dX + dW (recompute not counted)
        out.update(M=M, D=D, V=V, ms=ms, tflops=flop / ms / 1e9)
    elif a.case == "gemm":
        from nlearn_b200.kernels.gemm import gemm_ex
        M, N, K = a.M, a.N, a.K
        at, bt = a.layout[0] == "t", a.layout[1] == "t"
        def mk(r, c):  # rows x cols with row pitch c + pad
            return torch.randn(r, c + a.pad, device=dev).bfloat16()[:, :c]
        A = mk(*((K, M) if at else (M, K)))
        B = mk(*((N, K) if bt else (K, N)))
        if a.accum:
            from nlearn_b200.kernels.gemm import EPI_ACCUM
            C = torch.zeros(M, N, device=dev, dtype=torch.float32)
            ms = _time(lambda: gemm_ex(A, B, a_trans=at, b_trans=bt, out=C, epilogue=EPI_ACCUM), a.iters)
        else:
            from nlearn_b200 import _lib as L
            C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            epi = {"store": L.EPI_STORE, "bias": L.EPI_BIAS, "bias_gelu": L.EPI_BIAS_GELU, "resid": L.EPI_RESID,
                   "dgelu": L.EPI_DGELU}[a.epi]
            bias = torch.randn(N, device=dev) if a.epi in ("bias", "bias_gelu", "resid") else None
            aux = torch.randn(M, N, device=dev).bfloat16() if a.epi in ("bias_gelu", "dgelu") else None
            resid = torch.randn(M, N, device=dev).bfloat16() if a.epi == "resid" else None
            ms = _time(lambda: gemm_ex(A, B, a_trans=at, b_trans=bt, out=C, epilogue=epi, bias=bias, aux=aux,
                                       resid=resid), a.iters)
        out.update(M=M, N=N, K=K, layout=a.layout, pad=a.pad, accum=a.accum, epi=a.epi, ms=ms,
                   tflops=2 * M * N * K / ms / 1e9)
    elif a.case in ("attn_fwd", "attn_bwd"):
        from nlearn_b200 import attention as A
        n, s = a.heads, a.seq
        Q, K, V, dO = (torch.randn(n, s, 64, device=dev).bfloat16() for _ in range(4))
        O, L = A._flash_fwd_raw(Q, K, V)
        fwd = 4 * n * s * s * 64 / 2
        if a.case == "attn_fwd":
            ms = _time(lambda: A._flash_fwd_raw(Q, K, V), a.iters)
            flop = fwd
        else:
            ms = _time(lambda: A._flash_bwd_raw(Q, K, V, O, L, dO), a.iters)
            flop = 2.5 * fwd
        out.update(heads=n, seq=s, ms=ms, tflops=flop / ms / 1e9)
    elif a.case == "colsum":
        from nlearn_b200 import _lib
        M, N = a.M, a.N
        x = torch.randn(M, N, device=dev).bfloat16()
        o = torch.zeros(N, device=dev)
        ms = _time(lambda: _lib.check(_lib.lib.nl_colsum_bf16(_lib.ptr(x), _lib.ptr(o), M, N, _lib.stream_handle()),
                                      "colsum"), a.iters)
        out.update(M=M, N=N, ms=ms, gbs=M * N * 2 / ms / 1e6)
    elif a.case == "ce":
        from nlearn_b200.kernels.cross_entropy import ce_fwd_bwd
        M, V = a.M, a.N
        x = torch.randn(M, V, device=dev)
        t = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        ms = _time(lambda: ce_fwd_bwd(x, t, out=x), a.iters)
        out.update(M=M, V=V, ms=ms, gbs=(M * V * 8 + 12 * M) / ms / 1e6)
    else:
        raise SystemExit(f"unknown case {a.case}")
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

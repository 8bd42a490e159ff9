"""Inference path on the GPU: KV-cache decode attention, the sampler and whole
generation against the oracle (oracle/decode.py, oracle/model.py).

* decode attention: one new query row per (batch, head) over positions 0..pos
  of the cache vs an fp32 torch reference; the new k|v row lands in the cache;
* sampler: the exact token of the NumPy restatement (same random bits), and
  argmax for temperature 0;
* generation: every step's logits (prefill, then decode steps) vs the
  oracle's full recompute on the same token sequence (the reference's
  generation loop, nlearn/model.py:417-447), within max|err|/max|ref| 2e-2;
  each sampled token is the oracle's sample up to that logit tolerance;
  the graph-replayed steps give the tokens of eager steps.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from oracle import decode as OD  # noqa: E402
from oracle.model import OracleGPT  # noqa: E402
from nlearn_b200 import _lib  # noqa: E402
from nlearn_b200.generate import Decoder, generate  # noqa: E402
from nlearn_b200.model import FlatParams, GPTConfig  # noqa: E402

lib = _lib.lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("t", [0, 1, 127, 255, 256, 300, 511])
def test_decode_attention(cuda, t):
    B, H, S, D = 2, 8, 512, 512
    g = torch.Generator(device="cpu").manual_seed(t)
    cache = torch.randn(B, S, 3 * D, generator=g).bfloat16().to(cuda)
    new = torch.randn(B, 3 * D, generator=g).bfloat16().to(cuda)
    before = cache.clone()
    o = torch.empty(B, D, device=cuda, dtype=torch.bfloat16)
    pos = torch.tensor([t], device=cuda, dtype=torch.int32)
    nb = lib.nl_decode_workspace_bytes(B, H, S)
    ws = torch.zeros(nb, device=cuda, dtype=torch.uint8)
    for _ in range(2):  # twice: the merge counters must reset themselves
        assert lib.nl_decode_attention(new.data_ptr(), cache.data_ptr(), o.data_ptr(), pos.data_ptr(),
                                       ws.data_ptr(), nb, B, H, S, 64, _stream()) == 0
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    # reference: keys / values 0..t-1 from the cache, t from the new row
    kv = before.float().clone()
    kv[:, t] = new.float()
    q = new.float()[:, :D].view(B, H, 64)
    k = kv[:, :t + 1, D:2 * D].view(B, t + 1, H, 64)
    v = kv[:, :t + 1, 2 * D:].view(B, t + 1, H, 64)
    sc = torch.einsum("bhd,bjhd->bhj", q, k) / 8.0
    ref = torch.einsum("bhj,bjhd->bhd", torch.softmax(sc, -1), v).reshape(B, D)
    err = ((o.float() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-2, err
    assert torch.equal(cache[:, t, D:], new[:, D:])          # k|v appended
    assert torch.equal(cache[:, :t], before[:, :t])          # nothing else touched
    assert torch.equal(cache[:, t + 1:], before[:, t + 1:])


@pytest.mark.parametrize("temperature", [0.0, 0.7, 1.0])
def test_sampler_matches_restatement(cuda, temperature):
    B, V = 3, 50257
    rng = np.random.default_rng(5)
    lg = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    Vp = 50304
    logits = torch.zeros(B, Vp, device=cuda)
    logits[:, :V] = torch.from_numpy(lg).to(cuda)
    for pos_v, seed in [(0, 0), (17, 12345), (400, 2 ** 40 + 7)]:
        pos = torch.tensor([pos_v], device=cuda, dtype=torch.int32)
        tok = torch.zeros(B, device=cuda, dtype=torch.int32)
        out = torch.zeros(B, 512, device=cuda, dtype=torch.int32)
        assert lib.nl_sample_tokens(logits.data_ptr(), Vp, V, temperature, seed, pos.data_ptr(), tok.data_ptr(),
                                    out.data_ptr(), 512, B, _stream()) == 0
        torch.cuda.synchronize()
        want = OD.sample(lg, seed, pos_v, temperature)
        np.testing.assert_array_equal(tok.cpu().numpy(), want)
        np.testing.assert_array_equal(out[:, pos_v + 1].cpu().numpy(), want)


def _oracle(P, cfg):
    params = {}
    for name, shape, _ in P.specs:
        w = P.f(name).detach().float().cpu()
        params[name] = w.bfloat16().float() if len(shape) == 2 else w  # the GPU's bf16 matrices
    return OracleGPT(params, n_layers=cfg.n_layers, n_heads=cfg.n_heads, vocab=cfg.vocab, eps=cfg.ln_eps)


def test_generation_matches_full_recompute(cuda):
    cfg = GPTConfig()
    P = FlatParams(cfg, cuda, seed=0)
    B, Pl, n, seed, T = 2, 37, 6, 3, 1.0
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, (B, Pl)).astype(np.int32)
    dec = Decoder(P, cfg, batch=B)
    # eager steps, logits read after each
    dec.prefill(torch.from_numpy(prompt).to(cuda), seed, T)
    step_logits = [dec.logits[:, :cfg.vocab].cpu().numpy()]
    for _ in range(n - 1):
        dec.step(seed, T)
        step_logits.append(dec.logits[:, :cfg.vocab].cpu().numpy())
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    toks = dec.out[:, :Pl + n].cpu().numpy()
    np.testing.assert_array_equal(toks[:, :Pl], prompt)
    model = _oracle(P, cfg)
    with torch.no_grad():
        full = model.logits(torch.from_numpy(toks[:, :Pl + n - 1])).numpy()
    for i in range(n):
        pos = Pl - 1 + i
        ref = full[:, pos]
        got = step_logits[i]
        err = np.abs(got - ref).max() / np.abs(ref).max()
        assert err < 2e-2, (i, err)
        # the sampled token is the oracle's choice up to that logit tolerance
        tol = 2 * np.abs(got - ref).max() / T + 1e-3
        for b in range(B):
            u = OD.uniforms(seed, pos, b, cfg.vocab).astype(np.float64)
            pert = ref[b].astype(np.float64) / T - np.log(-np.log(u))
            assert pert[toks[b, pos + 1]] >= pert.max() - tol, (i, b)
    # graph replay gives the eager tokens
    dec2 = Decoder(P, cfg, batch=B)
    g_out = dec2.generate(prompt, n, seed, T, use_graph=True)
    e_out = Decoder(P, cfg, batch=B).generate(prompt, n, seed, T, use_graph=False)
    np.testing.assert_array_equal(g_out, e_out)
    np.testing.assert_array_equal(g_out, toks)


def test_generate_entry_point_greedy_and_trim(cuda):
    cfg = GPTConfig()
    P = FlatParams(cfg, cuda, seed=1)
    prompt = np.arange(600, dtype=np.int32) % cfg.vocab  # longer than max_seq: trimmed as the reference does
    out = generate(P, prompt, 8, seed=0, temperature=0.0, cfg=cfg)
    assert out.shape == (cfg.max_seq,)
    np.testing.assert_array_equal(out[:cfg.max_seq - 8], prompt[-(cfg.max_seq - 8):])
    again = generate(P, prompt, 8, seed=99, temperature=0.0, cfg=cfg)  # greedy ignores the seed
    np.testing.assert_array_equal(out, again)
    assert _lib.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(1, 1536, 512), (3, 2048, 512), (8, 50257, 512), (2, 200, 72)])
def test_linear_ln_small(cuda, M, N, K):
    """LayerNorm folded into the small-M GEMM's A staging vs LayerNorm (rounded
    to bf16, as the LN kernel writes it) followed by the product."""
    g = torch.Generator(device="cpu").manual_seed(M * N + K)
    x = (torch.randn(M, K, generator=g) * 3 + 1).bfloat16().to(cuda)
    gamma = (torch.rand(K, generator=g) + 0.5).to(cuda)
    beta = torch.randn(K, generator=g).to(cuda)
    Np = (N + 63) // 64 * 64
    W = (torch.randn(K, Np, generator=g) * 0.05).bfloat16().to(cuda)[:, :N]
    h = torch.nn.functional.layer_norm(x.float(), (K,), gamma, beta, 1e-5).bfloat16().float()
    ref = h @ W.float()
    bias = torch.randn(N, device=cuda)

    def run(out, epi, b=None, aux=None, expect=0):
        dt = _lib.F32 if out.dtype == torch.float32 else _lib.BF16
        st = lib.nl_linear_ln_small(x.data_ptr(), x.stride(0), gamma.data_ptr(), beta.data_ptr(), 1e-5,
                                    W.data_ptr(), W.stride(0), out.data_ptr(), out.stride(0), dt, M, N, K, epi,
                                    None if b is None else b.data_ptr(), None if aux is None else aux.data_ptr(),
                                    None, _stream())
        assert st == expect
        torch.cuda.synchronize()

    C = torch.empty(M, N, device=cuda)
    run(C, _lib.EPI_STORE)
    assert ((C - ref).abs().max() / ref.abs().max()).item() < 1e-3
    U = torch.empty(M, N, device=cuda, dtype=torch.bfloat16)
    A = torch.empty_like(U)
    run(U, _lib.EPI_BIAS_GELU, bias, A)
    pre = ref + bias
    assert ((A.float() - pre).abs().max() / pre.abs().max()).item() < 1e-2
    gl = torch.nn.functional.gelu(pre, approximate="tanh")
    assert ((U.float() - gl).abs().max() / gl.abs().max()).item() < 1e-2
    assert _lib.device_error() == 0


def test_linear_ln_small_declines_large_batch(cuda):
    x = torch.zeros(9, 512, device=cuda, dtype=torch.bfloat16)
    W = torch.zeros(512, 512, device=cuda, dtype=torch.bfloat16)
    g = torch.ones(512, device=cuda)
    C = torch.empty(9, 512, device=cuda)
    st = lib.nl_linear_ln_small(x.data_ptr(), 512, g.data_ptr(), g.data_ptr(), 1e-5, W.data_ptr(), 512,
                                C.data_ptr(), 512, _lib.F32, 9, 512, 512, _lib.EPI_STORE, None, None, None,
                                _stream())
    assert st == -1  # NL_ERR_SHAPE: the caller runs LayerNorm + GEMM instead


def test_position_guards(cuda):
    """A device position outside the cache (or past the output row) is
    reported through the device error word; the cache, the attention output
    and the output row are left untouched (the sampled token is written)."""
    B, H, S, D = 1, 8, 256, 512
    cache = torch.randn(B, S, 3 * D, device=cuda).bfloat16()
    before = cache.clone()
    new = torch.randn(B, 3 * D, device=cuda).bfloat16()
    o = torch.full((B, D), 0.5, device=cuda, dtype=torch.bfloat16)
    nb = lib.nl_decode_workspace_bytes(B, H, S)
    ws = torch.zeros(nb, device=cuda, dtype=torch.uint8)
    assert _lib.device_error() == 0
    for bad in (S, -1):
        pos = torch.tensor([bad], device=cuda, dtype=torch.int32)
        assert lib.nl_decode_attention(new.data_ptr(), cache.data_ptr(), o.data_ptr(), pos.data_ptr(),
                                       ws.data_ptr(), nb, B, H, S, 64, _stream()) == 0
        torch.cuda.synchronize()
        assert _lib.device_error() == 3
        assert torch.equal(cache, before)
        assert (o == 0.5).all()       # not recomputed: stale contents stay
    logits = torch.randn(B, 64, device=cuda)
    tok = torch.zeros(B, device=cuda, dtype=torch.int32)
    out = torch.full((B, 8), -5, device=cuda, dtype=torch.int32)
    pos = torch.tensor([7], device=cuda, dtype=torch.int32)  # would write out[:, 8] of an 8-wide row
    assert lib.nl_sample_tokens(logits.data_ptr(), 64, 64, 0.0, 0, pos.data_ptr(), tok.data_ptr(), out.data_ptr(),
                                8, B, _stream()) == 0
    torch.cuda.synchronize()
    assert _lib.device_error() == 3
    assert (out == -5).all() and tok.item() == int(logits.argmax())
    assert _lib.device_error() == 0  # reading cleared it

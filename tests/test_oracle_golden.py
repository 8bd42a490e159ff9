"""Pin the CPU oracle (oracle/ops.py) to the reference's own outputs.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py from
the reference itself (its pure-JAX fallbacks run on a NumPy jax stand-in, and
the NumPy references inside its kernel tests).  Tolerances are the reference
tests' own: atol 1e-4 for the f32 flash KATs (validate_flash*.py), exact-ish
for CE / LCE (f32 round-off only)."""
from pathlib import Path

import numpy as np
import pytest

from oracle import ops

G = Path(__file__).resolve().parent / "golden"


def load(name):
    return dict(np.load(G / f"{name}.npz"))


@pytest.mark.parametrize("name", ["flash_fwd_small", "flash_fwd_tiled"])
def test_attention_fwd_matches_reference(name):
    g = load(name)
    O, L = ops.attention_fwd(g["Q"], g["K"], g["V"])
    np.testing.assert_allclose(O, g["O"], atol=1e-4)
    np.testing.assert_allclose(O, g["O_std"], atol=1e-4)  # reference _attention_standard
    if "L" in g:
        np.testing.assert_allclose(L, g["L"], atol=1e-4)


@pytest.mark.parametrize("name", ["flash_bwd_small", "flash_bwd_128"])
def test_attention_bwd_matches_reference(name):
    g = load(name)
    dQ, dK, dV, D = ops.attention_bwd(g["Q"], g["K"], g["V"], g["dO"])
    O, _ = ops.attention_fwd(g["Q"], g["K"], g["V"])
    np.testing.assert_allclose(O, g["O"], atol=1e-4)
    np.testing.assert_allclose(dQ, g["dQ"], atol=1e-4)
    np.testing.assert_allclose(dK, g["dK"], atol=1e-4)
    np.testing.assert_allclose(dV, g["dV"], atol=1e-4)
    np.testing.assert_allclose(D, (g["dO"] * g["O"]).sum(-1), atol=1e-4)


def test_ce_matches_reference():
    g = load("ce_512x1024")
    loss, lse = ops.ce_fwd(g["logits"], g["targets"])
    assert abs(float(loss.mean()) - float(g["loss"])) < 1e-5
    assert abs(float(loss.mean()) - float(g["loss_fallback"])) < 1e-5
    assert abs(ops.cross_entropy(g["logits"], g["targets"]) - float(g["loss"])) < 1e-5
    d = ops.ce_bwd(g["logits"], g["targets"], lse)
    # softmax - onehot rows sum to zero; mean over rows folded in as 1/M
    np.testing.assert_allclose(d.sum(1), 0.0, atol=1e-6)
    M = d.shape[0]
    assert np.all(d[np.arange(M), g["targets"]] < 0)


@pytest.mark.parametrize("name", ["lce_256_64_2050", "lce_512_256_12000"])
def test_lce_matches_reference(name):
    g = load(name)
    M, D, V = int(g["M"]), int(g["D"]), int(g["V"])
    rng = np.random.default_rng(0)  # check_lce.py:33-37 input recipe
    X = (rng.standard_normal((M, D)) * 0.1).astype(np.float32)
    W = (rng.standard_normal((D, V)) * 0.05).astype(np.float32)
    tgt = rng.integers(0, V, (M,)).astype(np.int32)
    np.testing.assert_array_equal(X[:4, :4], g["X_head"])
    np.testing.assert_array_equal(tgt, g["targets"])
    loss, lse, dX, dW = ops.linear_cross_entropy(X, W, tgt)
    assert abs(loss - float(g["loss"])) < 1e-5
    assert abs(loss - float(g["loss_chunked"])) < 1e-5   # reference's chunked path agrees
    np.testing.assert_allclose(lse, g["lse"], atol=1e-5)
    np.testing.assert_allclose(dX, g["dX"], atol=1e-7, rtol=1e-4)
    np.testing.assert_allclose(dX, g["dX_chunked"], atol=1e-7, rtol=1e-4)
    np.testing.assert_allclose(dW[:, :256], g["dW_cols"], atol=1e-7, rtol=1e-4)
    np.testing.assert_allclose(dW[:, :256], g["dW_chunked_cols"], atol=1e-7, rtol=1e-4)
    np.testing.assert_allclose(dW.sum(0), g["dW_colsum"], atol=1e-6)


@pytest.mark.parametrize("name", ["gemm_small", "gemm_medium", "gemm_large"])
def test_gemm_matches_reference(name):
    g = load(name)
    C = ops.gemm(g["A"], g["B"])
    np.testing.assert_allclose(C, g["C"], rtol=1e-5, atol=1e-5 * np.abs(g["C"]).max())


def test_bf16_round_matches_ml_dtypes():
    x = np.random.default_rng(3).standard_normal(10000).astype(np.float32) * 100
    import ml_dtypes
    np.testing.assert_array_equal(ops.bf16_round(x), x.astype(ml_dtypes.bfloat16).astype(np.float32))


# ------------------------------------------------------------------ step oracle
def test_ln_gelu_matches_reference():
    """oracle.model's LayerNorm + tanh-GELU + residual against the reference's
    ln_gelu (iree_metal/kernels/test/bf16_metal_test.py:6-12)."""
    import torch
    from oracle.model import gelu_tanh, layer_norm
    g = load("ln_gelu")
    x = torch.from_numpy(g["x"])
    y = x + gelu_tanh(layer_norm(x, torch.from_numpy(g["g"]), torch.from_numpy(g["b"])))
    np.testing.assert_allclose(y.numpy(), g["y"], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize("name", ["flash_fwd_small", "flash_fwd_tiled"])
def test_model_attention_matches_reference(name):
    """The attention inside oracle.model against _attention_standard."""
    import torch
    from oracle.model import causal_attention
    g = load(name)
    O = causal_attention(*(torch.from_numpy(g[k]) for k in ("Q", "K", "V")))
    np.testing.assert_allclose(O.numpy(), g["O_std"], atol=1e-5)


def test_model_forward_matches_reference_block_wiring():
    """OracleGPT (hidden states, logits, loss) against a small BASELINE model
    run through the reference's block_forward / linear / attention /
    cross_entropy (tests/golden/make_golden.py, section 6)."""
    import importlib.util
    import torch
    from oracle.model import OracleGPT
    spec = importlib.util.spec_from_file_location("make_golden", G / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    g = load("model_small")
    named, tok, tgt = mg.small_model_params()
    cfg = mg.SMALL
    orc = OracleGPT({k: torch.from_numpy(v) for k, v in named.items()}, n_layers=cfg["n_layers"],
                    n_heads=cfg["n_heads"], vocab=cfg["vocab"])
    with torch.no_grad():
        h = orc.hidden(torch.from_numpy(tok))
        lg = orc.logits(torch.from_numpy(tok))
        loss = orc.loss(torch.from_numpy(tok), torch.from_numpy(tgt))
    np.testing.assert_allclose(h.numpy(), g["hidden"], atol=1e-4, rtol=1e-4)
    np.testing.assert_allclose(lg[..., :64].numpy(), g["logits_head"], atol=1e-5)
    np.testing.assert_allclose(torch.logsumexp(lg, -1).numpy(), g["lse"], atol=1e-5)
    assert abs(float(loss) - float(g["loss"])) < 1e-5

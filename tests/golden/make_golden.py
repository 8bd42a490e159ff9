"""Generate the golden fixtures in this folder FROM THE REFERENCE ITSELF.

Run in a container that has the nlearn reference checked out (it is read, never
modified, and never needed at test time):

    python tests/golden/make_golden.py /path/to/nlearn

Two sources, both the reference's own code:

1. The reference's pure-JAX CPU fallbacks — ``_attention_standard``
   (nlearn/attention.py:138-156), the one-hot ``cross_entropy`` fallback
   (nlearn/kernels/cross_entropy.py:79-81) and the chunked fused linear CE
   ``_lce_loss_lse`` / ``_lce_bwd_rule`` (nlearn/kernels/cross_entropy.py:
   106-167) — imported from the reference files and executed with a small
   NumPy stand-in for ``jax`` / ``jax.numpy`` (JAX is not installed here).
   Those functions only use array primitives that NumPy implements with the
   same semantics (matmul, where, exp, max, pad, one_hot, logsumexp, softmax).
2. The NumPy reference implementations inside the reference's kernel tests
   (iree_metal/kernels/test/validate_flash*.py, check_lce.py ``ref_np``,
   check_gemm_bf16.py), executed on those tests' own seeded inputs after
   dropping the lines that drive the Metal runtime.

Outputs: ``*.npz`` fixtures (float32) next to this script.
"""
from __future__ import annotations

import ast
import importlib.util
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


# ----------------------------------------------------------------------- jax stand-in
def _install_numpy_jax():
    jnp = types.ModuleType("jax.numpy")
    jnp.__getattr__ = lambda name: getattr(np, name)  # type: ignore[attr-defined]

    def softmax(x, axis=-1):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m)
        return e / e.sum(axis=axis, keepdims=True)

    def one_hot(x, n, dtype=np.float32):
        return (np.asarray(x)[..., None] == np.arange(n)).astype(dtype)

    def logsumexp(x, axis=None):
        m = np.max(x, axis=axis, keepdims=True)
        return (np.squeeze(m, axis=axis) + np.log(np.exp(x - m).sum(axis=axis))).astype(np.asarray(x).dtype)

    class custom_vjp:  # noqa: N801 — mirrors jax.custom_vjp's call surface
        def __init__(self, fun):
            self.fun = fun

        def __call__(self, *a):
            return self.fun(*a)

        def defvjp(self, f, b):
            self.fwd, self.bwd = f, b

    class _Dev:
        platform = "cpu"

    jax = types.ModuleType("jax")
    jax.numpy = jnp
    jax.nn = types.SimpleNamespace(softmax=softmax, one_hot=one_hot)
    jax.scipy = types.SimpleNamespace(special=types.SimpleNamespace(logsumexp=logsumexp))
    jax.custom_vjp = custom_vjp
    jax.devices = lambda: [_Dev()]
    jax.dtypes = types.SimpleNamespace(float0=np.bool_)
    jax.ffi = types.SimpleNamespace(ffi_call=None)
    jax.lax = types.SimpleNamespace(rsqrt=lambda v: (1.0 / np.sqrt(v)).astype(np.asarray(v).dtype))
    jax.jit = lambda f=None, **kw: f if f is not None else (lambda g: g)
    jax.checkpoint = lambda f, **kw: f
    jax.tree_util = types.SimpleNamespace(tree_map=lambda fn, t: t)
    jax.random = types.SimpleNamespace()
    import ml_dtypes
    jnp.bfloat16 = ml_dtypes.bfloat16
    jnp.float16 = np.float16
    jnp.float32 = np.float32
    jax.ShapeDtypeStruct = None
    sys.modules["jax"] = jax
    sys.modules["jax.numpy"] = jnp
    sys.modules["jax.random"] = jax.random


def _load(ref: Path, rel: str, name: str):
    spec = importlib.util.spec_from_file_location(name, ref / rel)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _run_test_script(path: Path, drop_from: str | None = None) -> dict:
    """Execute a reference test script's top-level statements, minus those
    that touch the Metal runtime (names rt / ctx / vmfb / m / *_k) and minus
    everything from the first statement whose text contains `drop_from`."""
    src = path.read_text()
    tree = ast.parse(src)
    keep = []
    bad = {"rt", "ctx", "vmfb", "m", "iree"}
    for node in tree.body:
        text = ast.get_source_segment(src, node) or ""
        if drop_from and drop_from in text:
            break
        names = {n.id for n in ast.walk(node) if isinstance(n, ast.Name)}
        if isinstance(node, (ast.Import, ast.ImportFrom)):
            if any(a.name.startswith(("iree", "nlearn")) for a in node.names) or \
               (isinstance(node, ast.ImportFrom) and (node.module or "").startswith(("iree", "nlearn"))):
                continue
        if not isinstance(node, ast.FunctionDef) and (names & bad or any(n.endswith("_k") for n in names)):
            continue
        keep.append(node)
    g: dict = {"__name__": "golden", "__file__": str(path)}
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(path), "exec"), g)
    return g


# Small BASELINE-architecture model for the step fixture (parameters regenerate
# from the seed; tests/test_oracle_golden.py rebuilds them with this function).
SMALL = dict(vocab=1000, d_model=128, n_heads=2, n_layers=2, d_ff=512, seq=64, batch=2, seed=11)


def small_model_params(cfg=SMALL) -> dict:
    """Flat-name f32 parameters (nlearn_b200.model.param_specs names) of the
    small model, from numpy's PCG64 stream (stable across numpy versions)."""
    rng = np.random.default_rng(cfg["seed"])
    D, F, V, S = cfg["d_model"], cfg["d_ff"], cfg["vocab"], cfg["seq"]
    p = {"wte": rng.standard_normal((V, D)) * 0.02, "wpe": rng.standard_normal((S, D)) * 0.02,
         "head.w": rng.standard_normal((D, V)) * 0.02,
         "lnf.g": 1 + 0.1 * rng.standard_normal(D), "lnf.b": 0.1 * rng.standard_normal(D)}
    for i in range(cfg["n_layers"]):
        q = f"blocks.{i}."
        p.update({q + "ln1.g": 1 + 0.1 * rng.standard_normal(D), q + "ln1.b": 0.1 * rng.standard_normal(D),
                  q + "wqkv": rng.standard_normal((D, 3 * D)) * 0.05, q + "wo": rng.standard_normal((D, D)) * 0.05,
                  q + "ln2.g": 1 + 0.1 * rng.standard_normal(D), q + "ln2.b": 0.1 * rng.standard_normal(D),
                  q + "w1": rng.standard_normal((D, F)) * 0.05, q + "b1": 0.1 * rng.standard_normal(F),
                  q + "w2": rng.standard_normal((F, D)) * 0.05, q + "b2": 0.1 * rng.standard_normal(D)})
    tok = rng.integers(0, V, (cfg["batch"], S + 1))
    return {k: np.asarray(v, np.float32) for k, v in p.items()}, tok[:, :-1].astype(np.int32), \
        tok[:, 1:].astype(np.int32)


def small_model_fixture(ref: Path, attn, ce) -> dict:
    gemm_mod = _load(ref, "nlearn/kernels/gemm.py", "nlearn.kernels.gemm")
    pkg = types.ModuleType("nlearn")
    kpkg = types.ModuleType("nlearn.kernels")
    pkg.attention, pkg.kernels, kpkg.gemm = attn, kpkg, gemm_mod
    sys.modules.update({"nlearn": pkg, "nlearn.attention": attn, "nlearn.kernels": kpkg,
                        "nlearn.kernels.gemm": gemm_mod})
    model = _load(ref, "nlearn/model.py", "nlearn.model")
    cfg = SMALL
    H, D = cfg["n_heads"], cfg["d_model"]
    linear = model.linear                       # reference linear (jnp.matmul off IREE-Metal)
    assert not gemm_mod.USE_IREE_GEMM and not attn.USE_IREE_FLASH and not attn.HAS_CUDNN

    def layer_norm(p, x):                       # the LayerNorm of ln_gelu (bf16_metal_test.py:8-10)
        mu = x.mean(-1, keepdims=True)
        var = ((x - mu) ** 2).mean(-1, keepdims=True)
        return (x - mu) * (1.0 / np.sqrt(var + 1e-5)) * p["gamma"] + p["beta"]

    def gelu(h):                                # the GELU of ln_gelu (bf16_metal_test.py:11)
        return 0.5 * h * (1 + np.tanh(0.7978845608 * (h + 0.044715 * h ** 3)))

    def attention_forward(p, x):                # model.py:159-198 without QK-norm / RoPE
        bs, s, _ = x.shape

        def proj(W):
            return linear(x, W).reshape(bs, s, H, D // H).transpose(0, 2, 1, 3).reshape(bs * H, s, D // H)
        o = model.attention(proj(p["W_q"]), proj(p["W_k"]), proj(p["W_v"]))
        o = o.reshape(bs, H, s, D // H).transpose(0, 2, 1, 3).reshape(bs, s, D)
        return linear(o, p["W_o"])

    def ffn_forward(p, x):                      # GELU FFN with biases (the BASELINE FFN)
        return linear(gelu(linear(x, p["W_up"]) + p["b_up"]), p["W_down"]) + p["b_down"]

    model.layer_norm, model.attention_forward, model.ffn_forward = layer_norm, attention_forward, ffn_forward
    named, tok, tgt = small_model_params(cfg)
    blocks = []
    for i in range(cfg["n_layers"]):
        q = f"blocks.{i}."
        w = named[q + "wqkv"]
        blocks.append({"ln1": {"gamma": named[q + "ln1.g"], "beta": named[q + "ln1.b"]},
                       "attn": {"W_q": w[:, :D], "W_k": w[:, D:2 * D], "W_v": w[:, 2 * D:], "W_o": named[q + "wo"]},
                       "ln2": {"gamma": named[q + "ln2.g"], "beta": named[q + "ln2.b"]},
                       "ffn": {"W_up": named[q + "w1"], "b_up": named[q + "b1"], "W_down": named[q + "w2"],
                               "b_down": named[q + "b2"]}})
    x = named["wte"][tok] + named["wpe"][None, :tok.shape[1]]
    for bp in blocks:
        x = model.block_forward(bp, x)          # reference wiring, model.py:315-324
    h = layer_norm({"gamma": named["lnf.g"], "beta": named["lnf.b"]}, x)
    logits = linear(h, named["head.w"])
    loss = ce.cross_entropy(logits, tgt)        # reference one-hot CE fallback
    lse = np.log(np.exp(logits - logits.max(-1, keepdims=True)).sum(-1)) + logits.max(-1)
    return dict(hidden=np.asarray(h, np.float32), logits_head=np.asarray(logits[..., :64], np.float32),
                lse=np.asarray(lse, np.float32), loss=np.float32(loss))


def main(ref: Path) -> None:
    _install_numpy_jax()
    attn = _load(ref, "nlearn/attention.py", "ref_attention")
    ce = _load(ref, "nlearn/kernels/cross_entropy.py", "ref_cross_entropy")
    tdir = ref / "iree_metal/kernels/test"
    out = {}

    # 1. flash forward KATs: validate_flash.py (2,16,8) and validate_flash_tiled.py (2,128,64)
    g = _run_test_script(tdir / "validate_flash.py", drop_from="vmfb =")
    out["flash_fwd_small"] = dict(Q=g["Q"], K=g["K"], V=g["V"], O=g["ref"](g["Q"], g["K"], g["V"]),
                                  O_std=attn._attention_standard(g["Q"], g["K"], g["V"]))
    g = _run_test_script(tdir / "validate_flash_tiled.py", drop_from="vmfb =")
    O, L = g["ref"](g["Q"], g["K"], g["V"])
    out["flash_fwd_tiled"] = dict(Q=g["Q"], K=g["K"], V=g["V"], O=O, L=L,
                                  O_std=attn._attention_standard(g["Q"], g["K"], g["V"]))

    # 2. flash backward KATs: validate_flash_bwd.py (2,16,8) and validate_flash_bwd128.py (2,128,64)
    for key, fname in (("flash_bwd_small", "validate_flash_bwd.py"), ("flash_bwd_128", "validate_flash_bwd128.py")):
        g = _run_test_script(tdir / fname, drop_from="ok = all(")
        out[key] = dict(Q=g["Q"], K=g["K"], V=g["V"], dO=g["dO"], O=g["Or"], dQ=g["dQr"], dK=g["dKr"],
                        dV=g["dVr"])

    # 3. CE: check_ce.py reference (one-hot CE through the reference's own
    #    fallback) on its (512, 1024) case, seed 0.
    rng = np.random.default_rng(0)
    M, V = 512, 1024
    logits = rng.standard_normal((M, V)).astype(np.float32)
    tgt = rng.integers(0, V, (M,)).astype(np.int32)
    g = _run_test_script(tdir / "check_ce.py", drop_from="for (M, V)")
    out["ce_512x1024"] = dict(logits=logits, targets=tgt, loss=np.float32(g["ref_ce"](logits, tgt)),
                              loss_fallback=np.float32(ce.cross_entropy(logits, tgt)))

    # 4. fused linear CE: check_lce.py cases, inputs exactly as check_lce.py:33-37
    for (M, D, V) in [(256, 64, 2050), (512, 256, 12000)]:
        rng = np.random.default_rng(0)
        X = (rng.standard_normal((M, D)) * 0.1).astype(np.float32)
        W = (rng.standard_normal((D, V)) * 0.05).astype(np.float32)
        tgt = rng.integers(0, V, (M,)).astype(np.int32)
        g = _run_test_script(tdir / "check_lce.py", drop_from="for spec in")
        loss_np, dX_np, dW_np = g["ref_np"](X, W, tgt)
        loss_c, lse_c = ce._lce_loss_lse(X, W, tgt)            # reference's chunked forward
        dX_c, dW_c, _ = ce._lce_bwd_rule((X, W, tgt, lse_c), np.float32(1.0))
        rec = dict(M=M, D=D, V=V, X_head=X[:4, :4], targets=tgt, loss=np.float32(loss_np),
                   loss_chunked=np.float32(loss_c), lse=np.asarray(lse_c, np.float32), dX=dX_np.astype(np.float32),
                   dX_chunked=np.asarray(dX_c, np.float32), dW_cols=dW_np[:, :256].astype(np.float32),
                   dW_chunked_cols=np.asarray(dW_c, np.float32)[:, :256],
                   dW_colsum=dW_np.sum(0).astype(np.float32))
        out[f"lce_{M}_{D}_{V}"] = rec

    # 5. GEMM: check_gemm_bf16.py cases (bf16-rounded operands, f32 accumulate)
    import ml_dtypes
    for (M, K, N, scale, label) in [(64, 128, 64, 0.1, "small"), (256, 512, 256, 1.0, "medium"),
                                    (64, 128, 64, 300.0, "large")]:
        rng = np.random.default_rng(0)
        A = (rng.standard_normal((M, K)) * scale).astype(np.float32)
        B = (rng.standard_normal((K, N)) * scale).astype(np.float32)
        Ab = A.astype(ml_dtypes.bfloat16).astype(np.float32)
        Bb = B.astype(ml_dtypes.bfloat16).astype(np.float32)
        out[f"gemm_{label}"] = dict(A=A, B=B, C=(Ab @ Bb).astype(np.float32))

    # 6. training-step pieces: ln_gelu and a small BASELINE model through the
    #    reference's block_forward / linear / attention / cross_entropy
    g = _run_test_script(tdir / "bf16_metal_test.py", drop_from="for dt in")
    rng = np.random.default_rng(6)
    x = (rng.standard_normal((2, 32, 512)) * 1.5 + 0.3).astype(np.float32)
    gam = (1.0 + 0.1 * rng.standard_normal(512)).astype(np.float32)
    bet = (0.1 * rng.standard_normal(512)).astype(np.float32)
    out["ln_gelu"] = dict(x=x, g=gam, b=bet, y=np.asarray(g["ln_gelu"](x, gam, bet), np.float32))
    out["model_small"] = small_model_fixture(ref, attn, ce)

    for key, rec in out.items():
        np.savez_compressed(HERE / f"{key}.npz", **{k: np.asarray(v) for k, v in rec.items()})
        print(f"wrote {key}.npz")


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "../nlearn"))

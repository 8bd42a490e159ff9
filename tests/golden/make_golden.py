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
    jax.ShapeDtypeStruct = None
    sys.modules["jax"] = jax
    sys.modules["jax.numpy"] = jnp


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

    for key, rec in out.items():
        np.savez_compressed(HERE / f"{key}.npz", **{k: np.asarray(v) for k, v in rec.items()})
        print(f"wrote {key}.npz")


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "../nlearn"))

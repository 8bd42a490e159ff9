"""Reference-format checkpoints (nlearn/train.py:45-96) on CPU: the pickles
hold nested numpy trees in the reference's layout, unpickle with numpy alone,
and round-trip every parameter and both AdamW moments exactly."""
import pickle
import pickletools

import numpy as np

from nlearn_b200 import checkpoint as C
from nlearn_b200.model import GPTConfig, param_specs

CFG = GPTConfig(vocab=1000, d_model=256, n_heads=4, n_layers=2, d_ff=1024, max_seq=64)


def _named(seed):
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape, _ in param_specs(CFG):
        a = rng.standard_normal(shape).astype(np.float32)
        if name == "head.w":
            a[:, CFG.vocab:] = 0.0  # padding columns are zero in the trainer
        out[name] = a
    return out


def _globals(path):
    mods = set()
    with open(path, "rb") as f:
        for op, arg, _ in pickletools.genops(f):
            if op.name in ("GLOBAL", "STACK_GLOBAL") and isinstance(arg, str):
                mods.add(arg.split()[0])
            if op.name == "SHORT_BINUNICODE" and isinstance(arg, str) and "." in arg and " " not in arg:
                mods.add(arg)
    return mods


def test_resume_state_round_trip(tmp_path):
    p, mu, nu = _named(0), _named(1), _named(2)
    path = str(tmp_path / "sub" / "resume.pkl")
    C.save_resume_state(p, mu, nu, count=7, step=7, cfg=CFG, path=path)
    with open(path, "rb") as f:
        raw = pickle.load(f)
    assert set(raw) == {"params", "opt_state", "step"} and raw["step"] == 7
    t = raw["params"]
    assert set(t) == {"embeddings", "blocks", "ln_final", "lm_head"}
    assert len(t["blocks"]) == CFG.n_layers
    assert t["embeddings"]["token_embed"].shape == (CFG.vocab, CFG.d_model)
    assert t["blocks"][0]["attn"]["W_q"].shape == (CFG.d_model, CFG.d_model)
    assert t["lm_head"].shape == (CFG.d_model, CFG.vocab)
    assert set(raw["opt_state"]) == {"count", "mu", "nu"}
    assert not any(m.startswith(("torch", "nlearn")) for m in _globals(path))
    got = C.load_resume_state(path, CFG)
    assert got is not None
    gp, gmu, gnu, count, step = got
    assert count == 7 and step == 7
    for src, dst in ((p, gp), (mu, gmu), (nu, gnu)):
        assert set(src) == set(dst)
        for k in src:
            np.testing.assert_array_equal(src[k], dst[k])


def test_params_only_checkpoint_and_missing_resume(tmp_path):
    p = _named(3)
    path = str(tmp_path / "step_000010.pkl")
    C.save_checkpoint(p, CFG, path)
    back = C.load_checkpoint(path, CFG)
    for k in p:
        np.testing.assert_array_equal(p[k], back[k])
    assert C.load_resume_state(str(tmp_path / "absent.pkl"), CFG) is None

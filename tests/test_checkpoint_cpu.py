"""Reference-format checkpoints (nlearn/train.py:45-96) on CPU: the pickles
hold nested numpy trees in the reference's layout, the resume file's
opt_state is optax.adamw's own state structure, and every parameter and both
AdamW moments round-trip exactly."""
import pickle
import sys
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
        raw = C._ResumeUnpickler(f).load()   # optax classes -> local stand-ins (no optax here)
    assert set(raw) == {"params", "opt_state", "step"} and raw["step"] == 7
    t = raw["params"]
    assert set(t) == {"embeddings", "blocks", "ln_final", "lm_head"}
    assert len(t["blocks"]) == CFG.n_layers
    assert t["embeddings"]["token_embed"].shape == (CFG.vocab, CFG.d_model)
    assert t["blocks"][0]["attn"]["W_q"].shape == (CFG.d_model, CFG.d_model)
    assert t["lm_head"].shape == (CFG.d_model, CFG.vocab)
    assert len(raw["opt_state"]) == 3 and int(raw["opt_state"][0].count) == 7
    assert not any(m.startswith(("torch", "nlearn")) for m in _globals(path))
    assert "optax" not in sys.modules  # writing registered no lasting optax stand-in
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


def _optax_stub_modules():
    """A stand-in ``optax`` package holding optax's state classes under their
    real module paths (optax 0.2.x: optax/_src/transform.py, optax/_src/base.py),
    as an unpickling reference process would have them."""
    import sys
    import types
    from typing import NamedTuple

    class ScaleByAdamState(NamedTuple):
        count: object
        mu: object
        nu: object

    class EmptyState(NamedTuple):
        pass

    class ScaleByScheduleState(NamedTuple):
        count: object

    class MultiStepsState(NamedTuple):
        mini_step: object
        gradient_step: object
        inner_opt_state: object
        acc_grads: object
        skip_state: object = ()

    mods = {m: types.ModuleType(m) for m in ("optax", "optax._src", "optax._src.transform", "optax._src.base",
                                             "optax._src.wrappers")}
    for cls, m in ((ScaleByAdamState, "optax._src.transform"), (ScaleByScheduleState, "optax._src.transform"),
                   (EmptyState, "optax._src.base"), (MultiStepsState, "optax._src.wrappers")):
        cls.__module__ = m
        cls.__qualname__ = cls.__name__
        setattr(mods[m], cls.__name__, cls)
    mods["optax"].MultiStepsState = MultiStepsState
    return mods, ScaleByAdamState, EmptyState, ScaleByScheduleState


def test_resume_opt_state_is_optax_adamw_structure(tmp_path, monkeypatch):
    """opt_state unpickles (under an optax stand-in) as optax.adamw's chain
    state, and one AdamW update (optax's formulas, restated in numpy) runs
    over its trees leaf by leaf against the params tree."""
    import sys
    p, mu, nu = _named(0), _named(1), {k: np.abs(v) for k, v in _named(2).items()}
    path = str(tmp_path / "resume.pkl")
    C.save_resume_state(p, mu, nu, count=5, step=5, cfg=CFG, path=path)
    assert {"optax._src.transform", "optax._src.base"} <= _globals(path)
    mods, Adam, Empty, Sched = _optax_stub_modules()
    for k, v in mods.items():
        monkeypatch.setitem(sys.modules, k, v)
    with open(path, "rb") as f:
        raw = pickle.load(f)
    st = raw["opt_state"]
    assert isinstance(st, tuple) and len(st) == 3
    assert type(st[0]) is Adam and type(st[1]) is Empty and type(st[2]) is Sched
    assert st[0].count.dtype == np.int32 and int(st[0].count) == 5 and int(st[2].count) == 5

    # optax.adamw update over the trees (scale_by_adam -> add_decayed_weights -> -lr)
    def leaves(t, path=()):
        if isinstance(t, dict):
            for k in sorted(t):
                yield from leaves(t[k], path + (k,))
        elif isinstance(t, list):
            for i, x in enumerate(t):
                yield from leaves(x, path + (i,))
        else:
            yield path, t
    P, MU, NU = (dict(leaves(x)) for x in (raw["params"], st[0].mu, st[0].nu))
    assert set(P) == set(MU) == set(NU)
    g = {k: np.ones_like(v) for k, v in P.items()}
    c = int(st[0].count) + 1
    for k in P:
        assert P[k].shape == MU[k].shape == NU[k].shape
        m = 0.9 * MU[k] + 0.1 * g[k]
        v = 0.999 * NU[k] + 0.001 * g[k] ** 2
        upd = (m / (1 - 0.9 ** c)) / (np.sqrt(v / (1 - 0.999 ** c)) + 1e-8) + 0.1 * P[k]
        assert np.isfinite(P[k] - 1e-3 * upd).all()


def test_resume_reads_wrapped_optax_states_and_rejects_others(tmp_path, monkeypatch):
    """chain(clip_by_global_norm, adamw) and MultiSteps wrappers (the
    reference's GRAD_CLIP / GRAD_ACCUM options) resume; a parameter tree of
    another architecture is refused with a ValueError, not a KeyError."""
    import sys
    mods, Adam, Empty, Sched = _optax_stub_modules()
    for k, v in mods.items():
        monkeypatch.setitem(sys.modules, k, v)
    p, mu, nu = _named(4), _named(5), _named(6)
    tree = C.to_tree(p, CFG)
    adam = (Adam(np.int32(3), C.to_tree(mu, CFG), C.to_tree(nu, CFG)), Empty(), Sched(np.int32(3)))
    Multi = mods["optax"].MultiStepsState
    for opt_state in ((Empty(), adam), Multi(np.int32(0), np.int32(3), adam, C.to_tree(p, CFG))):
        path = str(tmp_path / "wrapped.pkl")
        with open(path, "wb") as f:
            pickle.dump({"params": tree, "opt_state": opt_state, "step": 3}, f)
        for k in list(mods):
            monkeypatch.delitem(sys.modules, k)   # the reader has no optax
        got = C.load_resume_state(path, CFG)
        for k, v in mods.items():
            monkeypatch.setitem(sys.modules, k, v)
        assert got[3] == 3 and got[4] == 3
        np.testing.assert_array_equal(got[1]["wte"], mu["wte"])
    bad = str(tmp_path / "bad.pkl")
    with open(bad, "wb") as f:
        pickle.dump({"params": {"embeddings": {"token_embed": np.zeros((4, 4))}, "blocks": []},
                     "opt_state": adam, "step": 1}, f)
    import pytest
    with pytest.raises(ValueError):
        C.load_resume_state(bad, CFG)
    with open(bad, "wb") as f:
        pickle.dump({"params": tree, "opt_state": (Empty(),), "step": 1}, f)
    with pytest.raises(ValueError):
        C.load_resume_state(bad, CFG)

"""Checkpoints in the reference's on-disk format.

nlearn writes two pickles (nlearn/train.py:45-96):

* ``save_checkpoint`` / ``load_checkpoint``: the parameter tree alone, a nested
  dict of numpy arrays (written in place there; atomically here);
* ``save_resume_state`` / ``load_resume_state``: ``{"params", "opt_state",
  "step"}``, written to a temporary file and renamed into place so that a
  crash mid-write leaves the previous file intact.

This module writes and reads the same containers for the B200 trainer, so a
run can be resumed from, or its weights handed to, code that unpickles the
reference's files.  The parameter tree uses the reference's nesting and names
(``embeddings/token_embed``, ``blocks[i]/ln1``, ``attn/W_q`` ... ,
``ln_final``) for the tensors both architectures share; the BASELINE model's
own tensors carry names in the same style (``embeddings/pos_embed``, LayerNorm
``beta``, ``ffn/W_up, b_up, W_down, b_down``, an untied ``lm_head``).

The optimizer state is pickled as optax's own ``adamw`` state, the object
``optimizer.init(params)`` returns in the reference (nlearn/train.py:505-508,
``optax.adamw(schedule, weight_decay)``, optax 0.2.8 per
requirements-jaxmetal.txt:70): the chain tuple
``(ScaleByAdamState(count, mu, nu), EmptyState(), ScaleByScheduleState(count))``
with ``count`` an int32 scalar and ``mu``/``nu`` parameter-shaped trees, the
classes referenced under their optax module paths
(``optax._src.transform`` / ``optax._src.base``).  So the reference's
``load_resume_state`` + ``optimizer.update`` (train.py:90-96, 544-553)
continue from a B200 ``resume.pkl``.  Writing needs no optax (the classes are
stood in for while pickling); reading maps those classes to local stand-ins
when optax is not importable.  The reference's other optimizer shapes are
read too: ``chain(clip_by_global_norm, adamw)`` (GRAD_CLIP > 0) and
``MultiSteps`` (its ``inner_opt_state``); anything else, or a parameter tree of
another architecture (the reference's current RMSNorm / tied-embedding model),
is rejected with a ``ValueError`` that says what was found.

The conversion works on ``{flat name: numpy array}`` maps (the names of
``model.param_specs``); ``Trainer`` glue moves tensors to and from the device.
"""
from __future__ import annotations

import os
import pickle
import sys
import types
from typing import NamedTuple

import numpy as np

from .model import GPTConfig


def to_tree(named: dict, cfg: GPTConfig) -> dict:
    """{flat name: array} -> the reference-style nested parameter tree."""
    D = cfg.d_model
    blocks = []
    for i in range(cfg.n_layers):
        p = f"blocks.{i}."
        wqkv = np.asarray(named[p + "wqkv"])
        blocks.append({
            "ln1": {"gamma": named[p + "ln1.g"], "beta": named[p + "ln1.b"]},
            "attn": {"W_q": wqkv[:, :D].copy(), "W_k": wqkv[:, D:2 * D].copy(), "W_v": wqkv[:, 2 * D:].copy(),
                     "W_o": named[p + "wo"]},
            "ln2": {"gamma": named[p + "ln2.g"], "beta": named[p + "ln2.b"]},
            "ffn": {"W_up": named[p + "w1"], "b_up": named[p + "b1"], "W_down": named[p + "w2"],
                    "b_down": named[p + "b2"]},
        })
    return {
        "embeddings": {"token_embed": named["wte"], "pos_embed": named["wpe"]},
        "blocks": blocks,
        "ln_final": {"gamma": named["lnf.g"], "beta": named["lnf.b"]},
        "lm_head": np.asarray(named["head.w"])[:, :cfg.vocab].copy(),
    }


def from_tree(tree: dict, cfg: GPTConfig) -> dict:
    """Inverse of ``to_tree``; the LM head comes back at the padded width."""
    D, V, Vp = cfg.d_model, cfg.vocab, cfg.vocab_padded
    named = {"wte": tree["embeddings"]["token_embed"], "wpe": tree["embeddings"]["pos_embed"],
             "lnf.g": tree["ln_final"]["gamma"], "lnf.b": tree["ln_final"]["beta"]}
    head = np.zeros((D, Vp), np.float32)
    head[:, :V] = tree["lm_head"]
    named["head.w"] = head
    if len(tree["blocks"]) != cfg.n_layers:
        raise ValueError(f"checkpoint has {len(tree['blocks'])} blocks, config {cfg.n_layers}")
    for i, b in enumerate(tree["blocks"]):
        p = f"blocks.{i}."
        a = b["attn"]
        named.update({
            p + "ln1.g": b["ln1"]["gamma"], p + "ln1.b": b["ln1"]["beta"],
            p + "wqkv": np.concatenate([a["W_q"], a["W_k"], a["W_v"]], axis=1), p + "wo": a["W_o"],
            p + "ln2.g": b["ln2"]["gamma"], p + "ln2.b": b["ln2"]["beta"],
            p + "w1": b["ffn"]["W_up"], p + "b1": b["ffn"]["b_up"],
            p + "w2": b["ffn"]["W_down"], p + "b2": b["ffn"]["b_down"],
        })
    return {k: np.asarray(v, np.float32) for k, v in named.items()}


def _atomic_pickle(obj, path: str) -> None:
    """tmp file + rename (nlearn/train.py:84-87)."""
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        pickle.dump(obj, f)
    os.replace(tmp, path)


def save_checkpoint(named: dict, cfg: GPTConfig, path: str) -> None:
    """Parameters only (nlearn/train.py:45-58)."""
    _atomic_pickle(to_tree(named, cfg), path)


def load_checkpoint(path: str, cfg: GPTConfig) -> dict:
    """-> {flat name: array} (nlearn/train.py:60-66)."""
    with open(path, "rb") as f:
        return from_tree(pickle.load(f), cfg)


# ---------------------------------------------------------------- optax state
# Stand-ins with optax's field names and module paths.  ``ScaleByAdamState``
# and ``ScaleByScheduleState`` live in optax/_src/transform.py, ``EmptyState``
# in optax/_src/base.py (optax 0.2.x); all three are NamedTuples, so a pickle
# records the class path plus the field tuple and unpickles into real optax.
_OPTAX_TRANSFORM = "optax._src.transform"
_OPTAX_BASE = "optax._src.base"


class ScaleByAdamState(NamedTuple):
    count: np.ndarray
    mu: dict
    nu: dict


class EmptyState(NamedTuple):
    pass


class ScaleByScheduleState(NamedTuple):
    count: np.ndarray


_STANDINS = {(_OPTAX_TRANSFORM, "ScaleByAdamState"): ScaleByAdamState,
             (_OPTAX_BASE, "EmptyState"): EmptyState,
             (_OPTAX_TRANSFORM, "ScaleByScheduleState"): ScaleByScheduleState}


def _optax_classes():
    """The real optax classes when optax imports, else None."""
    try:
        from optax._src import base, transform  # noqa: F401
    except Exception:
        return None
    return {k: getattr(sys.modules[k[0]], k[1]) for k in _STANDINS}


def adamw_state(mu_tree, nu_tree, count: int):
    """optax.adamw(...).init-shaped state after ``count`` updates."""
    real = _optax_classes()
    c = np.asarray(count, np.int32)
    if real is not None:
        A, E, S = (real[k] for k in _STANDINS)
    else:
        A, E, S = ScaleByAdamState, EmptyState, ScaleByScheduleState
    return (A(count=c, mu=mu_tree, nu=nu_tree), E(), S(count=np.asarray(count, np.int32)))


def _dump_with_optax_paths(obj, f) -> None:
    """Temporarily register modules named like optax's that hold the
    stand-ins, so the standard pickler writes ``optax._src.transform
    ScaleByAdamState`` (etc.) as each class's global reference."""
    if _optax_classes() is not None:  # real optax: its own classes pickle themselves
        pickle.dump(obj, f)
        return
    saved = {m: sys.modules.get(m) for m in ("optax", "optax._src", _OPTAX_TRANSFORM, _OPTAX_BASE)}
    mods = {m: types.ModuleType(m) for m in saved}
    mods["optax"]._src = mods["optax._src"]
    mods["optax._src"].transform = mods[_OPTAX_TRANSFORM]
    mods["optax._src"].base = mods[_OPTAX_BASE]
    orig = {}
    for (mod, name), cls in _STANDINS.items():
        setattr(mods[mod], name, cls)
        orig[cls] = (cls.__module__, cls.__qualname__)
        cls.__module__, cls.__qualname__ = mod, name
    try:
        sys.modules.update(mods)
        pickle.dump(obj, f)
    finally:
        for cls, (m, q) in orig.items():
            cls.__module__, cls.__qualname__ = m, q
        for m, old in saved.items():
            if old is None:
                sys.modules.pop(m, None)
            else:
                sys.modules[m] = old


class _ResumeUnpickler(pickle.Unpickler):
    """Maps optax's state classes to the stand-ins when optax is absent."""

    def find_class(self, module, name):
        if module.startswith("optax") and _optax_classes() is None:
            cls = _STANDINS.get((module, name))
            if cls is not None:
                return cls
            # other optax states (clip, MultiSteps): a generic field container
            return _generic_state(module, name)
        return super().find_class(module, name)


_GENERIC: dict = {}


def _generic_state(module: str, name: str):
    key = (module, name)
    if key not in _GENERIC:
        def _new(cls, *args):
            return tuple.__new__(cls, args)
        _GENERIC[key] = type(name, (tuple,), {"__new__": _new, "__module__": module})
    return _GENERIC[key]


def _adam_state_of(opt_state):
    """Find the ScaleByAdamState inside the reference's optimizer state:
    adamw's chain tuple, chain(clip, adamw)'s nested tuple, or MultiSteps'
    inner_opt_state.  -> (count, mu_tree, nu_tree); ValueError otherwise."""
    if isinstance(opt_state, dict) and set(opt_state) == {"count", "mu", "nu"}:  # older files of this module
        return opt_state["count"], opt_state["mu"], opt_state["nu"]
    stack = [opt_state]
    while stack:
        o = stack.pop()
        if type(o).__name__ == "ScaleByAdamState":
            if hasattr(o, "mu"):
                return o.count, o.mu, o.nu
            return o[0], o[1], o[2]
        if type(o).__name__ == "MultiStepsState":
            inner = getattr(o, "inner_opt_state", None)
            stack.append(inner if inner is not None else o[2])
            continue
        if isinstance(o, tuple):
            stack.extend(reversed(o))
    raise ValueError(f"resume file's opt_state ({type(opt_state).__name__}) holds no optax ScaleByAdamState: "
                     "only optax.adamw (optionally under clip_by_global_norm or MultiSteps) can be resumed")


def save_resume_state(named: dict, mu: dict, nu: dict, count: int, step: int, cfg: GPTConfig, path: str) -> None:
    """{"params", "opt_state", "step"} (nlearn/train.py:74-87), opt_state in
    optax.adamw's own structure."""
    state = {"params": to_tree(named, cfg),
             "opt_state": adamw_state(to_tree(mu, cfg), to_tree(nu, cfg), count),
             "step": int(step)}
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        _dump_with_optax_paths(state, f)
    os.replace(tmp, path)


def _tree_of(tree, cfg: GPTConfig, what: str) -> dict:
    try:
        return from_tree(tree, cfg)
    except (KeyError, TypeError, IndexError) as e:
        keys = sorted(tree) if isinstance(tree, dict) else type(tree).__name__
        raise ValueError(f"{what} is not a tree of this model (LayerNorm, learned positions, untied head): "
                         f"missing {e!s} (top level: {keys})") from None


def load_resume_state(path: str, cfg: GPTConfig):
    """-> (params, mu, nu, count, step) as flat-name maps, or None when the
    file does not exist (nlearn/train.py:90-96)."""
    if not os.path.exists(path):
        return None
    with open(path, "rb") as f:
        st = _ResumeUnpickler(f).load()
    count, mu, nu = _adam_state_of(st["opt_state"])
    return (_tree_of(st["params"], cfg, "params"), _tree_of(mu, cfg, "opt_state mu"),
            _tree_of(nu, cfg, "opt_state nu"), int(np.asarray(count)), int(st["step"]))

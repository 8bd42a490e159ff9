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
``beta``, ``ffn/W_up, b_up, W_down, b_down``, an untied ``lm_head``).  The
optimizer state is optax's ``ScaleByAdamState`` written as a plain dict
(``count``, ``mu``, ``nu``; ``mu`` and ``nu`` are parameter-shaped trees), so
that unpickling needs numpy only.

The conversion works on ``{flat name: numpy array}`` maps (the names of
``model.param_specs``); ``Trainer`` glue moves tensors to and from the device.
"""
from __future__ import annotations

import os
import pickle

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


def save_resume_state(named: dict, mu: dict, nu: dict, count: int, step: int, cfg: GPTConfig, path: str) -> None:
    """{"params", "opt_state", "step"} (nlearn/train.py:74-87)."""
    state = {"params": to_tree(named, cfg),
             "opt_state": {"count": np.int32(count), "mu": to_tree(mu, cfg), "nu": to_tree(nu, cfg)},
             "step": int(step)}
    _atomic_pickle(state, path)


def load_resume_state(path: str, cfg: GPTConfig):
    """-> (params, mu, nu, count, step) as flat-name maps, or None when the
    file does not exist (nlearn/train.py:90-96)."""
    if not os.path.exists(path):
        return None
    with open(path, "rb") as f:
        st = pickle.load(f)
    o = st["opt_state"]
    return (from_tree(st["params"], cfg), from_tree(o["mu"], cfg), from_tree(o["nu"], cfg), int(o["count"]),
            int(st["step"]))

"""CPU oracle of the inference path — TEST INFRASTRUCTURE ONLY.

* ``sample``: the B200 sampler's rule restated in NumPy, bit-exact in its
  random bits: token = argmax_j(logit_j / T + G_j) with Gumbel noise
  G_j = -log(-log(u_j)), u_j = ((r >> 40) + 0.5) / 2^24 and r the SplitMix64
  finaliser (Steele, Lea & Flood, OOPSLA 2014) of key + j, key = mix(seed ^
  mix((pos << 32) ^ row)).  Gumbel-max draws from categorical(softmax(logits
  / T)), the distribution of the reference's jax.random.categorical
  (nlearn/model.py:439-441); the random stream itself is this library's.
* ``generate_full``: the reference's generation loop (nlearn/model.py:417-465):
  the whole model runs on the full buffer for every new token, the logits of
  the last filled position are sampled.  Uses ``OracleGPT.logits``.

Only tests/ use this module.
"""
from __future__ import annotations

import numpy as np

_M64 = (1 << 64) - 1


def _mix(z: np.ndarray) -> np.ndarray:
    z = (z + np.uint64(0x9E3779B97F4A7C15)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & np.uint64(_M64)
    return z ^ (z >> np.uint64(31))


def uniforms(seed: int, pos: int, row: int, V: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        inner = _mix(np.array([(pos << 32) ^ row], np.uint64))[0]
        key = _mix(np.array([np.uint64(seed) ^ inner], np.uint64))[0]
        r = _mix(key + np.arange(V, dtype=np.uint64))
    return ((r >> np.uint64(40)).astype(np.float32) + np.float32(0.5)) * np.float32(1.0 / 16777216.0)


def sample(logits: np.ndarray, seed: int, pos: int, temperature: float) -> np.ndarray:
    """[B, V] f32 logits -> [B] int32 tokens."""
    logits = np.asarray(logits, np.float32)
    B, V = logits.shape
    if temperature <= 0:
        return logits.argmax(1).astype(np.int32)
    out = np.empty(B, np.int32)
    for b in range(B):
        u = uniforms(seed, pos, b, V)
        g = -np.log(-np.log(u.astype(np.float64)))
        out[b] = int(np.argmax(logits[b].astype(np.float64) / temperature + g))
    return out


def generate_full(model, prompt: np.ndarray, n_tokens: int, seed: int, temperature: float):
    """[B, P] prompt -> ([B, P + n] tokens, [n, B, V] logits used per token)."""
    import torch
    buf = np.asarray(prompt, np.int32)
    used = []
    for _ in range(n_tokens):
        with torch.no_grad():
            lg = model.logits(torch.from_numpy(buf))[:, -1].numpy()
        used.append(lg)
        t = sample(lg, seed, buf.shape[1] - 1, temperature)
        buf = np.concatenate([buf, t[:, None]], 1)
    return buf, np.stack(used)

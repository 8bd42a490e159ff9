"""CPU-only tests of the host side: the C-ABI export table, the schedule and
optimizer restatements, the data stream, and the data-parallel bucket
reducer over a 2-rank gloo group (no GPU anywhere)."""
import math
import os
import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "nl_ops.h").read_text()
    return sorted(set(re.findall(r"NL_API\s+[\w\s\*]+?\b(nl_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from nlearn_b200 import _lib
    if not _lib.LIB_PATH.exists():
        from nlearn_b200.build import build
        build()
    syms = header_symbols()
    assert len(syms) >= 20
    dll = _lib.lib._load()
    for s in syms:
        assert hasattr(dll, s), s
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert b"sm_100a" in _lib.lib.nl_version()


def test_lr_schedule_matches_optax_restatement():
    from nlearn_b200.model import lr_schedule
    from oracle.model import lr_at
    for s in [0, 1, 5, 9, 10, 11, 25, 49, 50, 70]:
        assert lr_schedule(s, 1e-3, 10, 50) == pytest.approx(lr_at(s, 1e-3, 10, 50))
    assert lr_schedule(0, 1e-3, 10, 50) == 0.0
    assert lr_schedule(10, 1e-3, 10, 50) == pytest.approx(1e-3)
    assert lr_schedule(50, 1e-3, 10, 50) == pytest.approx(1e-4)
    assert lr_schedule(30, 1e-3, 10, 50) == pytest.approx(1e-4 + 0.9e-3 * 0.5)


def test_oracle_adamw_hand_computed():
    from oracle.model import OracleAdamW
    p = torch.tensor([1.0, -2.0], requires_grad=True)
    opt = OracleAdamW({"p": p}, wd=0.1)
    p.grad = torch.tensor([0.5, 0.25])
    opt.step(0.01)
    # step 1: m_hat = g, v_hat = g^2 -> update = sign(g)*(|g|/(|g|+eps)) + wd*p
    exp = torch.tensor([1.0 - 0.01 * (0.5 / (0.5 + 1e-8) + 0.1), -2.0 - 0.01 * (0.25 / (0.25 + 1e-8) - 0.2)])
    assert torch.allclose(p.detach(), exp, atol=1e-7)


def test_zipf_stream():
    from nlearn_b200.train import ZipfLoader, zipf_tokens
    rng = np.random.default_rng(0)
    t = zipf_tokens(rng, (4, 1000), 50257)
    assert t.min() >= 0 and t.max() < 50257 and t.dtype == np.int32
    assert (t == 0).mean() > 0.05  # Zipf head
    a = ZipfLoader(2, 16, 100, seed=1, rank=0)
    b = ZipfLoader(2, 16, 100, seed=1, rank=0)
    x1, y1 = a.next()
    x2, y2 = b.next()
    assert np.array_equal(x1, x2) and np.array_equal(x1[:, 1:], y1[:, :-1])
    c = ZipfLoader(2, 16, 100, seed=1, rank=1)
    assert not np.array_equal(c.next()[0], x1)


class _FakeParams:
    """The parts of FlatParams the reducer uses, on the CPU."""

    def __init__(self, sizes):
        self.specs = [(f"p{i}", (n,), None) for i, n in enumerate(sizes)]
        self.offsets, off = {}, 0
        for name, shape, _ in self.specs:
            self.offsets[name] = (off, shape)
            off += shape[0]
        self.grad = torch.zeros(off)
        self.device = torch.device("cpu")


def _reducer_worker(rank, world, port, out):
    import torch.distributed as dist
    from nlearn_b200.train import BucketReducer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    P = _FakeParams([10, 300, 7, 1000, 5])
    P.grad.copy_(torch.arange(P.grad.numel(), dtype=torch.float32) * (rank + 1))
    r = BucketReducer(P, bucket_bytes=400 * 4)
    assert len(r.buckets) >= 2
    r.begin()
    for name, _, _ in reversed(P.specs[2:]):
        r.ready(name)
    r.finish()  # launches the rest
    out[rank] = P.grad.clone()
    dist.destroy_process_group()


def test_bucket_reducer_two_ranks_gloo():
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    port = 29500 + os.getpid() % 1000
    mp.spawn(_reducer_worker, args=(2, port, out), nprocs=2, join=True)
    n = out[0].numel()
    exp = torch.arange(n, dtype=torch.float32) * 1.5   # mean of x1 and x2
    assert torch.allclose(out[0], exp) and torch.allclose(out[1], exp)


def test_lce_chunk_balancing():
    """The LM-head backward's vocabulary chunks: multiples of 256 columns that
    cover V in equal parts (no thin tail), at most the target width + 255."""
    from nlearn_b200.kernels.cross_entropy import _balanced_chunk
    for V in (50257, 2050, 12000, 100, 1):
        for target in (64, 4096, 16384, 65536):
            c = _balanced_chunk(V, target)
            assert c % 256 == 0 and c >= 256
            n = -(-V // c)
            tail = V - (n - 1) * c
            assert n == 1 or tail > c // 2 or c == 256  # no thin tail chunk
    assert _balanced_chunk(50257, 16384) == 16896 and _balanced_chunk(50257, 65536) == 50432


def test_sampler_restatement_properties():
    """oracle.decode.sample: deterministic in (seed, pos, row), greedy at
    temperature 0, and Gumbel-max frequencies follow softmax(logits / T)."""
    from oracle import decode as OD
    lg = np.log(np.array([[0.5, 0.3, 0.15, 0.05]], np.float32))
    assert OD.sample(lg, 1, 2, 0.0)[0] == 0
    a = [OD.sample(lg, s, 7, 1.0)[0] for s in range(4000)]
    b = [OD.sample(lg, s, 7, 1.0)[0] for s in range(4000)]
    assert a == b
    freq = np.bincount(a, minlength=4) / len(a)
    assert np.abs(freq - np.array([0.5, 0.3, 0.15, 0.05])).max() < 0.03, freq
    u = OD.uniforms(3, 5, 0, 1000)
    assert u.min() > 0 and u.max() < 1 and abs(float(u.mean()) - 0.5) < 0.05


def test_operators_refuse_cpu_tensors():
    """The operator surface has no CPU path: CPU tensors raise before any
    library call (no silent fallback to torch.matmul)."""
    from nlearn_b200.kernels.gemm import linear, matmul, gemm_ex
    from nlearn_b200.kernels.cross_entropy import cross_entropy, linear_cross_entropy
    from nlearn_b200.attention import attention
    x = torch.randn(4, 8, 16)
    W = torch.randn(16, 8)
    for fn, args in ((linear, (x, W)), (matmul, (x[0], W)), (gemm_ex, (x[0].bfloat16(), W.bfloat16())),
                     (cross_entropy, (torch.randn(4, 10), torch.zeros(4, dtype=torch.long))),
                     (linear_cross_entropy, (x[0], W, torch.zeros(8, dtype=torch.long))),
                     (attention, (torch.randn(2, 8, 64),) * 3)):
        with pytest.raises(ValueError):
            fn(*args)

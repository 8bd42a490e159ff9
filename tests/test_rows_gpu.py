"""Token-table rows (nl_rows_*, nl_adamw_rows): the touched-row set, the
gather / scatter used around the data-parallel exchange, and AdamW by rows,
which must equal the dense AdamW bit for bit (touched rows with their
gradient, the other rows with a zero gradient)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200._lib import check, lib, ptr, stream_handle  # noqa: E402
from nlearn_b200 import _lib  # noqa: E402


def _rows(tok, V, dev):
    mark = torch.zeros(V, device=dev, dtype=torch.int32)
    on = torch.full((V,), -1, device=dev, dtype=torch.int32)
    off = torch.full((V,), -1, device=dev, dtype=torch.int32)
    cnt = torch.zeros(2 + (V + 1023) // 1024, device=dev, dtype=torch.int32)
    check(lib.nl_rows_mark(ptr(tok), tok.numel(), ptr(mark), V, stream_handle()), "mark")
    check(lib.nl_rows_compact(ptr(mark), V, ptr(on), ptr(off), ptr(cnt), stream_handle()), "compact")
    torch.cuda.synchronize()
    return mark, on, off, cnt


@pytest.mark.parametrize("V", [50257, 1000, 1023, 7])
def test_mark_and_compact(cuda, V):
    rng = np.random.default_rng(V)
    tok_np = rng.integers(0, V, (4, 97)).astype(np.int32)
    tok = torch.from_numpy(tok_np).to(cuda)
    mark, on, off, cnt = _rows(tok, V, cuda)
    want = np.unique(tok_np)
    U = len(want)
    assert cnt[:2].tolist() == [U, V - U]
    assert np.array_equal(on[:U].cpu().numpy(), want)
    rest = np.setdiff1d(np.arange(V), want)
    assert np.array_equal(off[:V - U].cpu().numpy(), rest)
    assert int(mark.abs().sum()) == 0          # cleared for the next step


def test_gather_scatter_and_adamw_rows_equal_dense(cuda):
    V, D = 50257, 512
    rng = np.random.default_rng(3)
    tok = torch.from_numpy(rng.zipf(1.1, 16384).clip(1, V) - 1).to(cuda).int()
    _, on, off, cnt = _rows(tok, V, cuda)
    U = int(cnt[0])
    touched = on[:U].long()
    g = torch.zeros(V, D, device=cuda)
    g[touched] = torch.randn(U, D, device=cuda)
    buf = torch.empty(V, D, device=cuda)
    check(lib.nl_rows_gather(ptr(g), ptr(on), ptr(cnt[:1]), D, ptr(buf), V, stream_handle()), "gather")
    torch.cuda.synchronize()
    assert torch.equal(buf[:U], g[touched])
    g2 = torch.zeros_like(g)
    check(lib.nl_rows_scatter(ptr(buf), ptr(on), ptr(cnt[:1]), D, ptr(g2), V, stream_handle()), "scatter")
    torch.cuda.synchronize()
    assert torch.equal(g2, g)

    p = torch.randn(V, D, device=cuda)
    m = torch.randn(V, D, device=cuda) * 0.01
    v = torch.rand(V, D, device=cuda) * 0.01
    hyper = torch.tensor([1e-3, 1 - 0.9 ** 3, 1 - 0.999 ** 3], device=cuda)
    dense = [t.clone() for t in (p, m, v)]
    sh_dense = torch.empty(V, D, device=cuda, dtype=torch.bfloat16)
    check(lib.nl_adamw_step(ptr(dense[0]), ptr(g), ptr(dense[1]), ptr(dense[2]), ptr(sh_dense), V * D, ptr(hyper),
                            0.9, 0.999, 1e-8, 0.1, 0, stream_handle()), "dense")
    sh_rows = torch.empty_like(sh_dense)
    check(lib.nl_adamw_rows(ptr(p), None, ptr(m), ptr(v), ptr(sh_rows), ptr(off), ptr(cnt[1:]), D, V, ptr(hyper),
                            0.9, 0.999, 1e-8, 0.1, 0, stream_handle()), "rows off")
    check(lib.nl_adamw_rows(ptr(p), ptr(g), ptr(m), ptr(v), ptr(sh_rows), ptr(on), ptr(cnt[:1]), D, V, ptr(hyper),
                            0.9, 0.999, 1e-8, 0.1, 0, stream_handle()), "rows on")
    torch.cuda.synchronize()
    assert torch.equal(p, dense[0]) and torch.equal(m, dense[1]) and torch.equal(v, dense[2])
    assert torch.equal(sh_rows, sh_dense)
    assert _lib.device_error() == 0


def test_trainer_sparse_rows_match_dense(cuda):
    """The trainer with the token table handled by rows (overlapped AdamW on
    a side stream) against the plain dense optimizer after the step: the same
    loss sequence and weights within f32 round-off of the backward."""
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig
    res = []
    init = None
    for sparse in (True, False):
        tr = Trainer(GPTConfig(), TrainConfig(batch=4, seq=256, steps=20, warmup=2, sparse_embedding_rows=sparse),
                     cuda)
        if not sparse:
            tr.reducer.optimizer = None            # plain path: one dense AdamW after the backward
        init = tr.P.master.clone()
        losses = [tr.train_step(*tr.loader.next()) for _ in range(3)]
        torch.cuda.synchronize()
        res.append((losses, tr.P.master.clone()))
    assert np.allclose(res[0][0], res[1][0], rtol=0, atol=1e-4), (res[0][0], res[1][0])
    # Adam moves near-zero-gradient elements by ~lr in a direction set by
    # round-off, so the update vectors are compared normwise
    ua, ub = res[0][1] - init, res[1][1] - init
    rel = ((ua - ub).norm() / ub.norm()).item()
    assert rel < 1e-2, rel

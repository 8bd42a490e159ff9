"""The whole training step captured in one CUDA graph (Trainer.capture_step)
replays to the same losses and weights as eager steps, including the
device-side learning-rate schedule and AdamW bias corrections
(nl_adamw_schedule) across the warmup and into the cosine decay."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200 import _lib  # noqa: E402
from nlearn_b200.model import GPTConfig, lr_schedule  # noqa: E402
from nlearn_b200.train import Trainer, TrainConfig  # noqa: E402


def test_schedule_kernel_matches_host(cuda):
    hyper = torch.zeros(3, device=cuda)
    step = torch.zeros(1, device=cuda, dtype=torch.int32)
    peak, warm, decay = 1e-3, 10, 40
    for t in range(1, 60):
        assert _lib.lib.nl_adamw_schedule(hyper.data_ptr(), step.data_ptr(), peak, warm, decay, peak / 10,
                                          0.9, 0.999, torch.cuda.current_stream().cuda_stream) == 0
        h = hyper.cpu().numpy()
        assert int(step.item()) == t
        assert abs(h[0] - lr_schedule(t - 1, peak, warm, decay)) < 1e-9 + 1e-6 * peak
        assert abs(h[1] - (1 - 0.9 ** t)) < 1e-6 and abs(h[2] - (1 - 0.999 ** t)) < 1e-6


def test_graph_replay_matches_eager(cuda):
    cfg = GPTConfig()
    tc = TrainConfig(batch=2, seq=128, steps=12, warmup=10)
    a = Trainer(cfg, tc, cuda)
    b = Trainer(cfg, tc, cuda)
    batches = [a.loader.next() for _ in range(8)]
    dev = [a.device_batch(*x) for x in batches]
    for i in range(2):  # eager warm-up on both (initialises every kernel)
        a.step_on_device(*dev[i])
        b.step_on_device(*dev[i])
    w0 = a.P.master.clone()
    n = b.capture_step()
    assert n > 20
    la = [float(a.step_on_device(*dev[i])) for i in range(2, 8)]
    lb = [float(b.step_graphed(*dev[i])) for i in range(2, 8)]
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert np.allclose(la, lb, rtol=0, atol=1e-3), (la, lb)  # the CE-loss bar; atomics differ run to run
    assert b.opt.t == a.opt.t and b.step_idx == a.step_idx
    # float atomics (split-K, dQ, LayerNorm / bias reductions) make two runs
    # differ in the last bits, which Adam amplifies on near-zero gradients:
    # compare the update vectors normwise, as the data-parallel test does
    ua, ub = a.P.master - w0, b.P.master - w0
    rel = ((ua - ub).norm() / ua.norm()).item()
    assert rel < 5e-2, rel
    # host (pinned) batches through the same graph, and an eager step in between
    x, y = (torch.from_numpy(t).pin_memory() for t in a.loader.next())
    l1 = float(a.step_on_device(x.to(cuda), y.to(cuda)))
    l2 = float(b.step_graphed(x, y))
    assert abs(l1 - l2) < 1e-3
    l1 = float(a.step_on_device(*dev[0]))
    l2 = float(b.step_on_device(*dev[0]))
    assert abs(l1 - l2) < 1e-3
    l1 = float(a.step_on_device(*dev[1]))
    l2 = float(b.step_graphed(*dev[1]))
    assert abs(l1 - l2) < 1e-3


def test_train_step_async_returns_each_loss_one_step_late(cuda):
    """train_step_async (pinned host batches in, the previous step's loss out)
    gives the same loss sequence as the synchronous train_step."""
    import numpy as np
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig
    cfg = GPTConfig()
    tc = TrainConfig(batch=2, seq=128, steps=20, warmup=2)
    a, b = Trainer(cfg, tc, cuda), Trainer(cfg, tc, cuda)
    batches = [a.loader.next() for _ in range(4)]
    sync = [a.train_step(x, y) for x, y in batches]
    got = []
    for x, y in batches:
        r = b.train_step_async(torch.from_numpy(x).pin_memory(), torch.from_numpy(y).pin_memory())
        if r is not None:
            got.append(r)
    got.append(b.flush_loss())
    assert np.allclose(got, sync, rtol=0, atol=2e-3), (got, sync)

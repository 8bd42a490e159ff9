"""Training-step parity: the B200 step (nlearn_b200.model / train) against the
CPU float32 oracle (oracle/model.py) on identical weights and tokens.

Bars (north star): per-step loss within 1% of the oracle over 50 steps;
first-step loss within 1e-2 absolute, gradients within 5e-2 normwise (bf16
activations vs f32)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from nlearn_b200.model import GPTConfig, param_specs  # noqa: E402
from nlearn_b200.train import Trainer, TrainConfig  # noqa: E402
from nlearn_b200 import _lib  # noqa: E402
from oracle.model import OracleGPT, OracleAdamW, lr_at  # noqa: E402


def host_params(tr):
    return {name: tr.P.f(name).detach().cpu().clone() for name, _, _ in param_specs(tr.cfg)}


def nrel(a, b):
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-12)).item()


def test_first_step_loss_and_grads(cuda):
    cfg = GPTConfig()
    tr = Trainer(cfg, TrainConfig(batch=2, seq=512, steps=50), cuda)
    x, y = tr.loader.next()
    tok, tgt = tr.device_batch(x, y)
    tr.P.grad.zero_()
    loss, saved = tr.model.forward(tok, tgt)
    tr.model.backward(saved)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    orc = OracleGPT(host_params(tr))
    lo = orc.loss(torch.from_numpy(x), torch.from_numpy(y))
    lo.backward()
    assert abs(loss.item() - lo.item()) < 1e-2, (loss.item(), lo.item())
    og = orc.grads()
    for name in ["head.w", "lnf.g", "blocks.3.w2", "blocks.3.b1", "blocks.2.wqkv", "blocks.0.ln1.g", "wpe", "wte"]:
        g = tr.P.g(name).cpu()
        r = og[name]
        if name == "head.w":
            g, r = g[:, :cfg.vocab], r[:, :cfg.vocab]
        assert nrel(g, r) < 5e-2, (name, nrel(g, r))


def test_loss_tracks_oracle_50_steps(cuda):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cfg = GPTConfig()
    steps = 50
    tc = TrainConfig(batch=2, seq=256, steps=steps, peak_lr=1e-3, warmup=10)
    tr = Trainer(cfg, tc, cuda)
    orc = OracleGPT(host_params(tr))
    opt = OracleAdamW(orc.p)
    worst = 0.0
    for s in range(steps):
        x, y = tr.loader.next()
        lg = tr.train_step(x, y)
        lo = orc.loss(torch.from_numpy(x), torch.from_numpy(y))
        lo.backward()
        opt.step(lr_at(s, tc.peak_lr, tr.warmup, steps))
        worst = max(worst, abs(lg - lo.item()) / abs(lo.item()))
        assert worst < 1e-2, (s, lg, lo.item())
    assert _lib.device_error() == 0


def test_checkpoint_resume_reproduces(cuda, tmp_path):
    cfg = GPTConfig()
    tc = TrainConfig(batch=2, seq=128, steps=20, warmup=2)
    a = Trainer(cfg, tc, cuda)
    for _ in range(3):
        a.train_step(*a.loader.next())
    ck = str(tmp_path / "ck.pt")
    a.save(ck)
    la = [a.train_step(*a.loader.next()) for _ in range(3)]
    b = Trainer(cfg, tc, cuda)
    b.load(ck)
    lb = [b.train_step(*b.loader.next()) for _ in range(3)]
    assert np.allclose(la, lb, rtol=0, atol=2e-3), (la, lb)


def test_reference_format_resume_reproduces(cuda, tmp_path):
    """Resume through the reference's pickle ({params, opt_state, step},
    nlearn/train.py:74-96) continues the run as the uninterrupted trainer does."""
    cfg = GPTConfig()
    tc = TrainConfig(batch=2, seq=128, steps=20, warmup=2)
    a = Trainer(cfg, tc, cuda)
    for _ in range(3):
        a.train_step(*a.loader.next())
    ck = str(tmp_path / "resume.pkl")
    a.save_reference(ck)
    la = [a.train_step(*a.loader.next()) for _ in range(3)]
    b = Trainer(cfg, tc, cuda)
    assert not b.load_reference(str(tmp_path / "absent.pkl"))
    assert b.load_reference(ck)
    assert b.step_idx == 3 and b.opt.t == a.opt.t - 3
    lb = [b.train_step(*b.loader.next()) for _ in range(3)]
    assert np.allclose(la, lb, rtol=0, atol=2e-3), (la, lb)

"""Training-step parity: the B200 step (nlearn_b200.model / train) against the
CPU float32 oracle (oracle/model.py) on identical weights and tokens.

Bars (north star): per-step loss within 1% of the oracle over 50 steps;
first-step loss within 1e-2 absolute, gradients within 5e-2 normwise (bf16
activations vs f32).  The first step is checked at the BASELINE batch
(bs32 x 512, configs[3]) on both loss paths (fused LM-head CE and the
materialised logits + `ce_fwd`/`ce_bwd` path, NLEARN_FUSED_LMHEAD); the
50-step run uses 4 x 512 so the CPU oracle finishes in about a minute.
The oracle's forward is pinned to the reference's own code
(tests/test_oracle_golden.py)."""
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


GRAD_NAMES = ["head.w", "lnf.g", "lnf.b", "blocks.3.w2", "blocks.3.b2", "blocks.3.w1", "blocks.3.b1",
              "blocks.3.ln2.g", "blocks.2.wo", "blocks.2.wqkv", "blocks.0.ln1.g", "blocks.0.ln1.b", "wpe", "wte"]


@pytest.mark.parametrize("fused", [True, False], ids=["fused_lmhead", "materialised_ce"])
def test_first_step_loss_and_grads_bs32(cuda, fused):
    cfg = GPTConfig()
    torch.set_num_threads(max(1, len(__import__("os").sched_getaffinity(0))))
    tr = Trainer(cfg, TrainConfig(batch=32, seq=512, steps=50, fused_lmhead=fused), cuda)
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
    for name in GRAD_NAMES:
        g = tr.P.g(name).cpu()
        r = og[name]
        if name == "head.w":
            g, r = g[:, :cfg.vocab], r[:, :cfg.vocab]
        assert nrel(g, r) < 5e-2, (name, nrel(g, r))


def test_fused_and_materialised_paths_agree(cuda):
    """The two loss paths of nlearn/train.py:279-285 on the same weights and
    batch: same loss, same gradients within bf16 round-off."""
    cfg = GPTConfig()
    out = []
    for fused in (True, False):
        tr = Trainer(cfg, TrainConfig(batch=4, seq=512, steps=50, fused_lmhead=fused), cuda)
        tok, tgt = tr.device_batch(*tr.loader.next())
        tr.P.grad.zero_()
        loss, saved = tr.model.forward(tok, tgt)
        tr.model.backward(saved)
        torch.cuda.synchronize()
        out.append((loss.item(), tr.P.grad.clone()))
    assert abs(out[0][0] - out[1][0]) < 1e-3
    assert nrel(out[1][1], out[0][1]) < 2e-2


def test_loss_tracks_oracle_50_steps(cuda):
    torch.set_num_threads(max(1, len(__import__("os").sched_getaffinity(0))))
    cfg = GPTConfig()
    steps = 50
    tc = TrainConfig(batch=4, seq=512, steps=steps, peak_lr=1e-3, warmup=10)
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

"""Data-parallel step on 2 GPUs (NCCL) matches the 1-GPU step on the union of
the two ranks' batches.

After one step each rank's gradient buffer holds the all-reduced mean
gradient, which must equal the 1-GPU full-batch gradient: elementwise within
1e-2 relative on every element whose magnitude clears 1e-2 of its tensor's
largest, 1e-3 of the tensor's largest anywhere, and 1e-3 normwise.  Both sides
run the same kernels; only the f32 summation order of the weight-gradient
reductions and of the all-reduce differs.  The replicas' weights must stay
bit-identical, and after the step's AdamW the update vector must match the
1-GPU one within 1e-2 normwise (Adam moves near-zero-gradient elements by
about lr in a direction set by round-off, so that check is normwise).
Skipped when fewer than 2 GPUs are visible."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 1


def _rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig
    tr = Trainer(GPTConfig(), TrainConfig(batch=2, seq=128, steps=10, warmup=2, bucket_mb=16), f"cuda:{rank}",
                 rank, world)
    losses = [tr.train_step(*tr.loader.next()) for _ in range(STEPS)]
    torch.cuda.synchronize()
    out[rank] = (tr.P.master.cpu().numpy(), losses, tr.P.grad.cpu().numpy())
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp2_matches_single_gpu_full_batch():
    import torch.multiprocessing as mp
    from nlearn_b200.model import GPTConfig
    from nlearn_b200.train import Trainer, TrainConfig, ZipfLoader
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_rank, args=(2, 29600 + os.getpid() % 300, out), nprocs=2, join=True)
    m0, l0, g0 = out[0]
    m1, _, g1 = out[1]
    assert np.array_equal(m0, m1)  # replicas stay identical
    assert np.array_equal(g0, g1)  # both hold the same reduced gradient
    ref = Trainer(GPTConfig(), TrainConfig(batch=4, seq=128, steps=10, warmup=2), "cuda:0")
    m_init = ref.P.master.cpu().numpy()
    a, b = ZipfLoader(2, 128, 50257, 0, 0), ZipfLoader(2, 128, 50257, 0, 1)
    for _ in range(STEPS):
        (xa, ya), (xb, yb) = a.next(), b.next()
        ref.train_step(np.concatenate([xa, xb]), np.concatenate([ya, yb]))
    torch.cuda.synchronize()
    mr = ref.P.master.cpu().numpy()
    gr = ref.P.grad.cpu().numpy()
    for name, shape, _ in ref.P.specs:
        off, shp = ref.P.offsets[name]
        n = int(np.prod(shp))
        gd, gf = g0[off:off + n].astype(np.float64), gr[off:off + n].astype(np.float64)
        top = np.abs(gf).max()
        if top == 0:
            assert np.abs(gd).max() == 0, name
            continue
        big = np.abs(gf) > 1e-2 * top
        assert (np.abs(gd - gf)[big] <= 1e-2 * np.abs(gf)[big]).all(), name
        assert np.abs(gd - gf).max() <= 1e-3 * top, (name, np.abs(gd - gf).max() / top)
        assert np.linalg.norm(gd - gf) <= 1e-3 * np.linalg.norm(gf), name
    ud, ur = (m0 - m_init).astype(np.float64), (mr - m_init).astype(np.float64)
    rel = np.linalg.norm(ud - ur) / np.linalg.norm(ur)
    assert rel < 1e-2, rel

"""``Trainer.step_from_host(wait=False)`` queues a step and the copy of its
loss; reading each loss while the next step runs gives the losses of the
waiting form."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _losses(wait: bool, cuda_graph: bool):
    from underhfs_b200.data import SyntheticTokens
    from underhfs_b200.distributed import DistributedPolicy
    from underhfs_b200.train import Trainer, TrainConfig, build_model

    torch.cuda.set_device(0)
    cfg = TrainConfig(model="125m", batch=2, seq_len=256, lr=3e-4, cuda_graph=cuda_graph)
    model = build_model(cfg, device="cuda:0")
    tr = Trainer(model, cfg, policy=DistributedPolicy(world_size=1, rank=0))
    src = SyntheticTokens(model.vocab_size, cfg.batch, cfg.seq_len, seed=3, rank=0)
    hosts = [torch.empty((2, cfg.batch, cfg.seq_len), dtype=torch.int64, pin_memory=True) for _ in range(4)]
    for h in hosts:
        src.next_host(h)
    if wait:
        out = [tr.step_from_host(h) for h in hosts]
    else:
        out, pending = [], None
        for h in hosts:
            queued = tr.step_from_host(h, wait=False)
            if pending is not None:
                out.append(pending.result())
            pending = queued
        out.append(pending.result())
    tr.release()
    return out


@pytest.mark.parametrize("cuda_graph", [False, True])
def test_async_loss_readback_matches(cuda_graph):
    a = _losses(True, cuda_graph)
    b = _losses(False, cuda_graph)
    assert len(a) == len(b) == 4
    for x, y in zip(a, b):
        # weight gradients accumulate with fp32 atomics: runs differ in the last bits
        assert abs(x - y) <= 1e-4 * abs(x), (a, b)

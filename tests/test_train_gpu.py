"""Training workload on one B200: bf16 autocast, meta-device init on the GPU, AdamW steps."""
from dataclasses import replace

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_train_step_bf16_one_gpu(cuda):
    from comm_opt_b200.models.llama import TINY
    from comm_opt_b200.models.train import TrainConfig, Trainer, synthetic_batch

    cfg = replace(TINY, layers=2, vocab=4096)
    tr = Trainer(cfg, TrainConfig(tp=1), cuda)
    assert all(p.device.type == "cuda" for p in tr.model.parameters())
    losses = []
    for st in range(4):
        t = synthetic_batch(cfg, 2, 256, 0, 0, pin=True).to(cuda, non_blocking=True)  # the same batch each step
        losses.append(float(tr.step(t[:, :-1], t[:, 1:])))
    assert all(torch.isfinite(torch.tensor(losses)))
    assert abs(losses[0] - torch.log(torch.tensor(4096.0)).item()) < 1.0  # random init: near ln(vocab)
    assert losses[-1] < losses[0]  # the same batch four times: AdamW fits it

"""Tiny end-to-end decode of the flagship model family (used by __graft_entry__.smoke)."""
from __future__ import annotations

import torch

from ..parallel.communicator import TPCommunicator
from .llama import LlamaWeights, TPDecodeRunner, tiny_config


def tiny_decode_step(device, steps: int = 2) -> torch.Tensor:
    cfg = tiny_config(layers=2)
    comm = TPCommunicator(None, device=device, dtype=torch.bfloat16, max_rows=8, max_hidden=cfg.hidden)
    w = LlamaWeights(cfg, 0, 1, device, seed=0)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=2, max_seq=64, device=device, gemm="cob")
    prompts = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(0))
    first = runner.prefill(prompts)
    runner.start(2, first, prompts.shape[1])
    runner.capture(2)
    host_in = torch.empty(2, dtype=torch.int32).pin_memory()
    host_out = torch.empty(2, dtype=torch.int32).pin_memory()
    host_in.copy_(first.cpu())
    for _ in range(steps):
        runner.decode(2, host_in, host_out)
        host_in.copy_(host_out)
    assert int(host_out.min()) >= 0 and int(host_out.max()) < cfg.vocab
    runner.release_graphs()
    return host_out

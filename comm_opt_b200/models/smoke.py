"""Tiny end-to-end decode of the flagship model family (used by __graft_entry__.smoke), checked
against the unsharded fp32 forward."""
from __future__ import annotations

import torch

from ..parallel.communicator import TPCommunicator
from .llama import LlamaWeights, TPDecodeRunner, reference_logits, tiny_config


def near_argmax(logits: torch.Tensor, ids: torch.Tensor, rel: float = 2 ** -5) -> torch.Tensor:
    """Per row: the chosen id's fp32 logit is within `rel` x (logit range) of the row maximum, i.e. it
    is the argmax up to bf16 rounding of near-ties."""
    chosen = logits.gather(1, ids.long().view(-1, 1).to(logits.device)).squeeze(1)
    top = logits.max(-1).values
    spread = (top - logits.min(-1).values).clamp_min(1e-6)
    return (top - chosen) <= rel * spread


def tiny_decode_step(device, steps: int = 2) -> torch.Tensor:
    cfg = tiny_config(layers=2)
    comm = TPCommunicator(None, device=device, dtype=torch.bfloat16, max_rows=8, max_hidden=cfg.hidden)
    full = LlamaWeights.full_random(cfg, device=device, seed=0)
    w = LlamaWeights(cfg, 0, 1, device, full=full)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=2, max_seq=64, device=device, gemm="cob")
    prompts = torch.randint(0, cfg.vocab, (2, 16), generator=torch.Generator().manual_seed(0))
    first = runner.prefill(prompts)
    runner.start(2, first, prompts.shape[1])
    runner.capture(2)
    host_in = torch.empty(2, dtype=torch.int32).pin_memory()
    host_out = torch.empty(2, dtype=torch.int32).pin_memory()
    host_in.copy_(first.cpu())
    toks = torch.cat([prompts, first.cpu().long()[:, None]], 1)
    for step in range(steps):
        runner.decode(2, host_in, host_out)
        ids = host_out.clone()
        assert int(ids.min()) >= 0 and int(ids.max()) < cfg.vocab
        ok = near_argmax(reference_logits(cfg, full, toks, device), ids)
        assert bool(ok.all()), f"decode step {step}: ids {ids.tolist()} are not the fp32 argmax"
        toks = torch.cat([toks, ids.long()[:, None]], 1)
        host_in.copy_(ids)
    runner.release_graphs()
    return host_out

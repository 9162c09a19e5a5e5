"""Llama-3 training step, tensor parallel (Megatron style with sequence parallel) x FSDP on a 2-D mesh.

The workload of the reference's end-to-end training measurement (exp/M5_e2e_comm_share/titan_recipes.py:31-75:
Llama-3 1B / 8B architecture, random init, TP in {8, 4, 2} x fully-sharded data parallel = 8 / TP, a fixed
global batch of 8 sequences x 2048 tokens, AdamW at 3e-4, bf16 compute with fp32 gradient reduction),
written directly on torch.distributed (DTensor tensor parallelism, `fully_shard`) because torchtitan is
not part of this stack. Its communication is what the reference measured: the sequence-parallel
all-gathers / reduce-scatters around every attention and MLP block (bf16), FSDP's parameter all-gathers
and fp32 gradient reduce-scatters, the fp32 all-reduce of the gradient norm and the int64 all-reduce of
the step's token count. The decode kernels of this package are not on this path: training uses torch's
GEMMs and scaled-dot-product attention, and the interesting output is the split of each step into
compute, exposed communication and overlap (harness/train_share.py).

Layout per rank: dp = world / tp data-parallel groups of tp ranks; mesh dims ("dp", "tp").
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..ops.reference import rope_tables
from .llama import LlamaConfig


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, heads, D]; cos / sin [S, D/2]. Rotate-half convention (the decode kernels use the same)."""
    half = x.shape[-1] // 2
    c = cos[None, :, None, :].to(x.dtype)
    s = sin[None, :, None, :].to(x.dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        H, D = cfg.hidden, cfg.head_dim
        self.head_dim = D
        self.group = cfg.heads // cfg.kv_heads
        self.wq = nn.Linear(H, cfg.heads * D, bias=False)
        self.wk = nn.Linear(H, cfg.kv_heads * D, bias=False)
        self.wv = nn.Linear(H, cfg.kv_heads * D, bias=False)
        self.wo = nn.Linear(cfg.heads * D, H, bias=False)

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        B, S, _ = x.shape
        D = self.head_dim
        # head counts come from the (possibly column-sharded) projection widths
        q = apply_rope(self.wq(x).view(B, S, -1, D), cos, sin)
        k = apply_rope(self.wk(x).view(B, S, -1, D), cos, sin)
        v = self.wv(x).view(B, S, -1, D)
        k = k.repeat_interleave(self.group, dim=2)
        v = v.repeat_interleave(self.group, dim=2)
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        return self.wo(o.transpose(1, 2).reshape(B, S, -1))


class FeedForward(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.w1 = nn.Linear(cfg.hidden, cfg.inter, bias=False)  # gate
        self.w3 = nn.Linear(cfg.hidden, cfg.inter, bias=False)  # up
        self.w2 = nn.Linear(cfg.inter, cfg.hidden, bias=False)  # down

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class Block(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.attention_norm = nn.RMSNorm(cfg.hidden, eps=cfg.eps)
        self.attention = Attention(cfg)
        self.ffn_norm = nn.RMSNorm(cfg.hidden, eps=cfg.eps)
        self.feed_forward = FeedForward(cfg)

    def forward(self, x, cos, sin):
        h = x + self.attention(self.attention_norm(x), cos, sin)
        return h + self.feed_forward(self.ffn_norm(h))


class TrainLlama(nn.Module):
    """Dense Llama-3 decoder for training (untied embedding and output head, as the 1B / 8B recipes)."""

    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.tok_embeddings = nn.Embedding(cfg.vocab, cfg.hidden)
        self.layers = nn.ModuleList(Block(cfg) for _ in range(cfg.layers))
        self.norm = nn.RMSNorm(cfg.hidden, eps=cfg.eps)
        self.output = nn.Linear(cfg.hidden, cfg.vocab, bias=False)
        self._rope: tuple | None = None

    def rope(self, S: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        if self._rope is None or self._rope[0].shape[0] < S or self._rope[0].device != device:
            self._rope = rope_tables(S, self.cfg.head_dim, self.cfg.rope_theta, device=device)
        return self._rope[0][:S], self._rope[1][:S]

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        cos, sin = self.rope(tokens.shape[1], tokens.device)
        h = self.tok_embeddings(tokens)
        for layer in self.layers:
            h = layer(h, cos, sin)
        return self.output(self.norm(h))

    def init_weights(self, seed: int, std: float = 0.02):
        """Random init of whatever this rank holds (full tensors, or the local shards of DTensors): normal(0,
        std) for matrices with the output projections scaled by 1/sqrt(2 * layers), ones for norm weights.
        Draws on the tensors' own device from a generator seeded with `seed`."""
        out_std = std / math.sqrt(2 * self.cfg.layers)
        gens: dict = {}
        with torch.no_grad():
            for name, p in self.named_parameters():
                t = p.to_local() if hasattr(p, "to_local") else p
                if "norm" in name:
                    t.fill_(1.0)
                    continue
                g = gens.setdefault(t.device, torch.Generator(device=t.device).manual_seed(seed))
                s = out_std if name.endswith(("wo.weight", "w2.weight")) else std
                t.normal_(0.0, s, generator=g)


def tp_plan(model: TrainLlama, loss_parallel: bool) -> dict:
    """Module -> placement plan of the sequence-parallel Megatron layout: the residual stream is sharded
    along the sequence between blocks; attention / MLP inputs are all-gathered, their row-parallel
    outputs reduce-scattered back to sequence shards."""
    from torch.distributed.tensor import Replicate, Shard
    from torch.distributed.tensor.parallel import (ColwiseParallel, PrepareModuleInput, RowwiseParallel,
                                                   SequenceParallel)

    plan = {
        "tok_embeddings": RowwiseParallel(input_layouts=Replicate(), output_layouts=Shard(1)),
        "norm": SequenceParallel(),
        "output": ColwiseParallel(input_layouts=Shard(1), output_layouts=Shard(-1) if loss_parallel else Replicate(),
                                  use_local_output=not loss_parallel),
    }
    for i in range(len(model.layers)):
        p = f"layers.{i}."
        plan.update({
            p + "attention_norm": SequenceParallel(),
            p + "attention": PrepareModuleInput(input_layouts=(Shard(1), None, None),
                                                desired_input_layouts=(Replicate(), None, None)),
            p + "attention.wq": ColwiseParallel(),
            p + "attention.wk": ColwiseParallel(),
            p + "attention.wv": ColwiseParallel(),
            p + "attention.wo": RowwiseParallel(output_layouts=Shard(1)),
            p + "ffn_norm": SequenceParallel(),
            p + "feed_forward": PrepareModuleInput(input_layouts=(Shard(1),), desired_input_layouts=(Replicate(),)),
            p + "feed_forward.w1": ColwiseParallel(),
            p + "feed_forward.w3": ColwiseParallel(),
            p + "feed_forward.w2": RowwiseParallel(output_layouts=Shard(1)),
        })
    return plan


@dataclass
class TrainConfig:
    tp: int = 1
    lr: float = 3e-4
    max_norm: float = 1.0
    bf16: bool = True  # bf16 compute, fp32 master weights and fp32 gradient reduction
    loss_parallel: bool = True  # cross-entropy on vocab-sharded logits (no logits all-gather)
    remat: bool = False  # activation checkpointing per block
    init: str = "meta"  # "meta": allocate shards only and init them per rank; "full": seeded full model, then shard
    seed: int = 0
    count_tokens: bool = True  # int64 all-reduce of the step's tokens (the per-step token accounting)


class Trainer:
    """One optimizer step per `step(tokens, labels)`: forward, loss, backward, gradient-norm clip, AdamW."""

    def __init__(self, cfg: LlamaConfig, tc: TrainConfig, device: torch.device):
        """Builds the (dp, tp) mesh over the default process group (or runs unsharded without one)."""
        import torch.distributed as dist

        self.cfg, self.tc, self.device = cfg, tc, torch.device(device)
        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        assert world % tc.tp == 0, f"world {world} not divisible by tp {tc.tp}"
        self.world, self.rank, self.tp, self.dp = world, rank, tc.tp, world // tc.tp
        cfg.shard(tc.tp)  # raises when heads / kv heads / intermediate / vocab do not split tp ways
        self.mesh = None
        if world > 1:
            from torch.distributed.device_mesh import init_device_mesh

            self.mesh = init_device_mesh(self.device.type, (self.dp, self.tp), mesh_dim_names=("dp", "tp"))
        self.dp_rank = self.mesh.get_local_rank("dp") if self.mesh is not None else 0
        lp = tc.loss_parallel and self.tp > 1
        self.loss_parallel = lp
        if tc.init == "full":
            torch.manual_seed(tc.seed)
            model = TrainLlama(cfg)
            model.init_weights(tc.seed)
            model.to(self.device)
        else:
            with torch.device("meta"):
                model = TrainLlama(cfg)
        if self.tp > 1:
            from torch.distributed.tensor.parallel import parallelize_module

            parallelize_module(model, self.mesh["tp"], tp_plan(model, lp))
        if tc.remat:
            from torch.utils.checkpoint import checkpoint

            for blk in model.layers:
                fwd = blk.forward
                blk.forward = (lambda f: lambda *a: checkpoint(f, *a, use_reentrant=False))(fwd)
        self.mp = self.device.type == "cuda" and tc.bf16
        if self.dp > 1:
            from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

            mpp = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32) if self.mp else \
                MixedPrecisionPolicy()
            for i, blk in enumerate(model.layers):
                # the last block's parameters are gathered again right away by the backward: keep them
                fully_shard(blk, mesh=self.mesh["dp"], mp_policy=mpp,
                            reshard_after_forward=i < len(model.layers) - 1)
            fully_shard(model, mesh=self.mesh["dp"], mp_policy=mpp)
        if tc.init != "full":
            model.to_empty(device=self.device)
            # per-rank seed: shards differ across ranks, as independent draws of one random model would
            model.init_weights(tc.seed * 1000 + rank)
        self.model = model
        self.opt = torch.optim.AdamW(model.parameters(), lr=tc.lr, betas=(0.9, 0.95), weight_decay=0.1,
                                     foreach=True)
        self._tokens = torch.zeros((), dtype=torch.int64, device=self.device)

    def clip_(self) -> torch.Tensor:
        params = [p for p in self.model.parameters() if p.grad is not None]
        norm = torch.nn.utils.get_total_norm([p.grad for p in params], 2.0, foreach=True)
        if hasattr(norm, "full_tensor"):
            norm = norm.full_tensor()  # sums the squared norms over the mesh (fp32 all-reduce)
        torch.nn.utils.clip_grads_with_norm_(params, self.tc.max_norm, norm, foreach=True)
        return norm

    def step(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """tokens / labels [B_local, S] of this data-parallel rank (the same on every rank of its TP group).
        Returns the (rank-local) loss as a device tensor; nothing here synchronizes with the host."""
        import torch.distributed as dist

        if self.tc.count_tokens:
            n = torch.full((), labels.numel(), dtype=torch.int64, device=self.device)
            if self.world > 1:
                dist.all_reduce(n)  # every data-parallel group's tokens, once per TP rank of the group
                n = n // self.tp
            self._tokens += n  # stays on the device: no host sync inside the step
        # without FSDP's mixed-precision policy (dp == 1) bf16 compute comes from autocast
        ctx = torch.autocast("cuda", dtype=torch.bfloat16) if (self.mp and self.dp == 1) else contextlib.nullcontext()
        with ctx:
            logits = self.model(tokens)
        if self.loss_parallel:
            from torch.distributed.tensor.parallel import loss_parallel

            with loss_parallel():
                loss = F.cross_entropy(logits.flatten(0, 1).float(), labels.flatten())
                loss.backward()
        else:
            loss = F.cross_entropy(logits.flatten(0, 1).float(), labels.flatten())
            loss.backward()
        self.clip_()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach()

    @property
    def tokens_seen(self) -> int:
        """Tokens trained on so far over all data-parallel ranks (reads the device counter)."""
        return int(self._tokens)

    def local_shapes(self) -> dict:
        return {n: tuple((p.to_local() if hasattr(p, "to_local") else p).shape) for n, p in self.model.named_parameters()}


def synthetic_batch(cfg: LlamaConfig, batch: int, seq: int, step: int, dp_rank: int, pin: bool = False):
    """Random token ids [batch, seq + 1] (host tensor; pinned when asked) for one data-parallel rank and step:
    inputs are [:, :-1], labels [:, 1:]. Seeded by (step, dp_rank), so every TP rank of a group agrees."""
    g = torch.Generator().manual_seed(1_000_003 * step + dp_rank)
    t = torch.randint(0, cfg.vocab, (batch, seq + 1), generator=g)
    return t.pin_memory() if pin else t

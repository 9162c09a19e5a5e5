"""Llama-shaped tensor-parallel decoder for decode-time measurement (TP = 1/2/4/8).

The reference measured the share of communication in TP=8 decode through vLLM
(exp/M5_e2e_comm_share/infer.py:37-88) and never replaced vLLM's kernels; this runner is the
framework layer that puts the fused collective where it belongs: both row-parallel outputs of
every layer (o_proj and down_proj, the two all-reduce points of exp/M5_e2e_comm_share/README.md:111)
go through ``TPCommunicator.fused_allreduce_add_rmsnorm``, which also performs the residual add
and the following RMSNorm. Everything in the decode step is one of this package's kernels:
embedding, RMSNorm, the projection GEMMs, RoPE + paged-KV append, paged GQA decode attention,
SiLU*mul, the fused collective, and a distributed greedy argmax; one step is captured in a CUDA
graph per batch size.

Sharding (Megatron style): QKV and gate/up are column-parallel, o_proj and down_proj are
row-parallel, the LM head is vocab-parallel, the embedding table is replicated (2.1 GB at vocab
128256 x 8192 bf16 - cheap on a 180 GB part and saves a collective per step).
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass, replace

import torch
import torch.nn.functional as F

from ..ops import kernels as K
from ..ops.reference import rope_tables
from ..parallel.communicator import TPCommunicator
from .gemm import GateUpLinear, Linear, PackedWeight, dense, pack_weight


@dataclass(frozen=True)
class LlamaConfig:
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int
    vocab: int
    eps: float = 1e-5
    rope_theta: float = 500000.0
    qkv_bias: bool = False  # Qwen2-style attention: the QKV projection has a bias

    def shard(self, tp: int) -> dict:
        """Per-rank head counts and sizes. With more ranks than KV heads (tp a multiple of kv_heads) each
        rank keeps one KV head, replicated on tp / kv_heads ranks (as vLLM shards such models)."""
        kv_ok = self.kv_heads % tp == 0 or tp % self.kv_heads == 0
        assert self.heads % tp == 0 and kv_ok and self.inter % tp == 0 and self.vocab % tp == 0, \
            f"{self.name} does not shard {tp} ways"
        return dict(nq=self.heads // tp, nkv=max(1, self.kv_heads // tp), inter=self.inter // tp,
                    vocab=self.vocab // tp)

    def kv_head0(self, rank: int, tp: int) -> int:
        """First KV head held by `rank`: the one its query heads attend to (grouped-query attention)."""
        return rank * (self.heads // tp) // (self.heads // self.kv_heads)

    @property
    def params(self) -> int:
        H, D = self.hidden, self.head_dim
        per_layer = H * (self.heads + 2 * self.kv_heads) * D + self.heads * D * H + 3 * H * self.inter + 2 * H
        if self.qkv_bias:
            per_layer += (self.heads + 2 * self.kv_heads) * D
        return self.layers * per_layer + 2 * self.vocab * H + H


LLAMA3_8B = LlamaConfig("llama3-8b", 4096, 32, 32, 8, 128, 14336, 128256)
LLAMA3_70B = LlamaConfig("llama3-70b", 8192, 80, 64, 8, 128, 28672, 128256)
LLAMA3_1B = LlamaConfig("llama3-1b", 2048, 16, 32, 8, 64, 8192, 128256)
# TinyLlama-1.1B shapes, the smaller model of the reference's end-to-end inference study
# (exp/M5_e2e_comm_share/run_infer.py:15-16): head_dim 64, 4 KV heads (replicated at TP = 8), vocab 32000.
TINYLLAMA = LlamaConfig("tinyllama-1.1b", 2048, 22, 32, 4, 64, 5632, 32000, eps=1e-5, rope_theta=10000.0)
# Qwen2.5-32B-Instruct shapes, the larger model of the reference's end-to-end inference study
# (exp/M5_e2e_comm_share/run_infer.py:15-19): hidden 5120 is the hidden size of the reference's fused-op
# measurements; 40 query / 8 KV heads, SwiGLU 27648, vocab 152064, QKV bias, RoPE theta 1e6.
QWEN25_32B = LlamaConfig("qwen2.5-32b", 5120, 64, 40, 8, 128, 27648, 152064, eps=1e-6, rope_theta=1e6, qkv_bias=True)
TINY = LlamaConfig("tiny", 1024, 2, 16, 8, 128, 2048, 4096)
TINY_BIAS = replace(TINY, name="tiny-qkv-bias", heads=20, kv_heads=4, qkv_bias=True)  # 5 query heads per KV head
TINY_HD64 = replace(TINY, name="tiny-hd64", heads=16, kv_heads=2, head_dim=64)  # KV heads replicated at TP >= 4
PRESETS = {"llama3-1b": LLAMA3_1B, "1b": LLAMA3_1B, "llama3-8b": LLAMA3_8B, "8b": LLAMA3_8B, "llama3-70b": LLAMA3_70B,
           "70b": LLAMA3_70B, "qwen2.5-32b": QWEN25_32B, "qwen32b": QWEN25_32B, "tinyllama-1.1b": TINYLLAMA,
           "tinyllama": TINYLLAMA, "tiny": TINY, "tiny-qkv-bias": TINY_BIAS, "tiny-hd64": TINY_HD64}


class LayerWeights:
    def __init__(self, wqkv, wo, wgu, wdown, ln1, ln2, bqkv=None):
        self.wqkv, self.wo, self.wgu, self.wdown, self.ln1, self.ln2 = wqkv, wo, wgu, wdown, ln1, ln2
        self.bqkv = bqkv  # [(nq + 2 nkv) * head_dim] of this rank, or None


class LlamaWeights:
    """This rank's shards. Weight matrices are [out_features, in_features] (K-major)."""

    def __init__(self, cfg: LlamaConfig, tp_rank: int, tp: int, device, dtype=torch.bfloat16, seed: int = 0,
                 std: float = 0.02, full: dict | None = None):
        self.cfg, self.tp_rank, self.tp, self.dtype = cfg, tp_rank, tp, dtype
        s = cfg.shard(tp)
        H, D = cfg.hidden, cfg.head_dim
        gen = torch.Generator(device=device)

        def rnd(shape, key):
            gen.manual_seed(seed * 1_000_003 + key * 8 + tp_rank)
            return torch.empty(shape, dtype=dtype, device=device).normal_(0.0, std, generator=gen)

        def norm_w(key):
            gen.manual_seed(seed * 1_000_003 + key)
            return (1.0 + 0.1 * torch.randn(H, device=device, generator=gen)).to(dtype)

        if full is not None:  # slices of one full model (tests: TP result == TP1 result)
            self.embed = full["embed"].to(device)
            self.final_norm = full["final_norm"].to(device)
            self.lm_head = full["lm_head"].chunk(tp, 0)[tp_rank].contiguous().to(device)
            self.layers = []
            kv0, nkv = cfg.kv_head0(tp_rank, tp), s["nkv"]

            def qkv_rows(t):  # this rank's q, k and v heads of a [(heads + 2 kv_heads) * D, ...] tensor
                q, k, v = t.split([cfg.heads * D, cfg.kv_heads * D, cfg.kv_heads * D], 0)
                return torch.cat([q.chunk(tp, 0)[tp_rank], k[kv0 * D:(kv0 + nkv) * D], v[kv0 * D:(kv0 + nkv) * D]], 0)

            for L in full["layers"]:
                wqkv = qkv_rows(L["wqkv"])
                g, u = L["wgu"].chunk(2, 0)
                wgu = torch.cat([g.chunk(tp, 0)[tp_rank], u.chunk(tp, 0)[tp_rank]], 0)
                bqkv = qkv_rows(L["bqkv"]).contiguous().to(device) if L.get("bqkv") is not None else None
                self.layers.append(LayerWeights(
                    wqkv.contiguous().to(device), L["wo"].chunk(tp, 1)[tp_rank].contiguous().to(device),
                    wgu.contiguous().to(device), L["wdown"].chunk(tp, 1)[tp_rank].contiguous().to(device),
                    L["ln1"].to(device), L["ln2"].to(device), bqkv))
            return
        gen.manual_seed(seed * 1_000_003 + 1)  # replicated tensors: same seed on every rank
        self.embed = torch.empty(cfg.vocab, H, dtype=dtype, device=device).normal_(0.0, 1.0, generator=gen)
        self.final_norm = norm_w(2)
        self.lm_head = rnd((s["vocab"], H), 3)
        self.layers = []
        replicated = tp > cfg.kv_heads

        def qkv_weight(k0):
            if not replicated:
                return rnd(((s["nq"] + 2 * s["nkv"]) * D, H), k0)
            # ranks that share a KV head get the same k and v rows (seeded by the head, not the rank)
            gen.manual_seed(seed * 1_000_003 + (k0 + 7) * 8 + cfg.kv_head0(tp_rank, tp))
            kv = torch.empty((2 * D, H), dtype=dtype, device=device).normal_(0.0, std, generator=gen)
            return torch.cat([rnd((s["nq"] * D, H), k0), kv], 0)

        for i in range(cfg.layers):
            k0 = 16 + 8 * i
            self.layers.append(LayerWeights(
                qkv_weight(k0), rnd((H, s["nq"] * D), k0 + 1),
                rnd((2 * s["inter"], H), k0 + 2), rnd((H, s["inter"]), k0 + 3), norm_w(k0 + 4), norm_w(k0 + 5),
                rnd(((s["nq"] + 2 * s["nkv"]) * D,), k0 + 6) if cfg.qkv_bias else None))

    @staticmethod
    def full_random(cfg: LlamaConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0, std: float = 0.02) -> dict:
        """Unsharded weights (small configs only), to be sliced by every rank."""
        g = torch.Generator(device=device).manual_seed(seed)
        H, D = cfg.hidden, cfg.head_dim

        def rnd(*shape, scale=std):
            return (scale * torch.randn(*shape, generator=g, device=device)).to(dtype)

        def nw():
            return (1.0 + 0.1 * torch.randn(H, generator=g, device=device)).to(dtype)

        layers = [dict(wqkv=rnd((cfg.heads + 2 * cfg.kv_heads) * D, H), wo=rnd(H, cfg.heads * D),
                       wgu=rnd(2 * cfg.inter, H), wdown=rnd(H, cfg.inter), ln1=nw(), ln2=nw())
                  for _ in range(cfg.layers)]
        if cfg.qkv_bias:  # only present with a bias, so every tensor of a layer dict is a real tensor
            for L in layers:
                L["bqkv"] = rnd((cfg.heads + 2 * cfg.kv_heads) * D, scale=0.5)
        return dict(embed=rnd(cfg.vocab, H, scale=1.0), final_norm=nw(), lm_head=rnd(cfg.vocab, H), layers=layers)


class BlockAllocator:
    """Free list of 16-token KV pages shared by all layers (same page id in every layer)."""

    def __init__(self, num_blocks: int):
        self.free = list(range(num_blocks - 1, -1, -1))

    def alloc(self, n: int) -> list[int]:
        if n > len(self.free):
            raise RuntimeError(f"KV cache exhausted: need {n} pages, {len(self.free)} free")
        return [self.free.pop() for _ in range(n)]

    def release(self, pages: list[int]):
        self.free.extend(reversed(pages))


class PagedKVCache:
    BLOCK = 16

    def __init__(self, cfg: LlamaConfig, tp: int, max_batch: int, max_seq: int, device, dtype=torch.bfloat16,
                 extra_blocks: int = 0):
        s = cfg.shard(tp)
        self.max_blocks_per_seq = (max_seq + self.BLOCK - 1) // self.BLOCK
        self.num_blocks = max_batch * self.max_blocks_per_seq + extra_blocks
        shape = (self.num_blocks, s["nkv"], self.BLOCK, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(cfg.layers)]
        self.v = [torch.zeros(shape, dtype=dtype, device=device) for _ in range(cfg.layers)]
        self.alloc = BlockAllocator(self.num_blocks)
        self.block_tables = torch.zeros(max_batch, self.max_blocks_per_seq, dtype=torch.int32, device=device)
        self.pages: list[list[int]] = [[] for _ in range(max_batch)]

    def reserve(self, batch: int, seq: int):
        """Give sequences 0..batch-1 pages for `seq` tokens (shuffled pages: the indirection is real)."""
        nb = (seq + self.BLOCK - 1) // self.BLOCK
        assert nb <= self.max_blocks_per_seq
        for b in range(batch):
            if len(self.pages[b]) < nb:
                self.pages[b] += self.alloc.alloc(nb - len(self.pages[b]))
        rows = torch.tensor([p + [0] * (self.max_blocks_per_seq - len(p)) for p in self.pages[:batch]],
                            dtype=torch.int32)
        self.block_tables[:batch].copy_(rows)

    @property
    def bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.k + self.v)


class TPDecodeRunner:
    """Greedy TP decoding: torch prefill, then graph-captured decode steps built from our kernels."""

    def __init__(self, cfg: LlamaConfig, weights: LlamaWeights, comm: TPCommunicator, max_batch: int, max_seq: int,
                 device, gemm: str = "cob", nccl_group=None, pdl: bool = True, fuse_boundary: bool = False,
                 fuse_epilogues: bool = False, collective: str = "ours", tune_boundaries: bool = True,
                 car_group=None, l2_prefetch: int = 0, pack_weights: bool = True, fuse_append: bool = True):
        self.cfg, self.w, self.comm, self.device = cfg, weights, comm, torch.device(device)
        self.tp, self.rank = comm.world, comm.rank
        self.s = cfg.shard(self.tp)
        self.max_batch, self.max_seq = max_batch, max_seq
        self.dtype = weights.dtype
        self.nccl_group = nccl_group
        self.cache = PagedKVCache(cfg, self.tp, max_batch, max_seq, self.device, self.dtype)
        self.cos, self.sin = rope_tables(max_seq, cfg.head_dim, cfg.rope_theta, self.device)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.gemm = gemm
        # RoPE + KV append of the new token inside the attention kernel (one kernel less per layer)
        self.fuse_append = bool(fuse_append)
        # packed weights (this package's GEMMs only): every projection matrix is converted in place, once,
        # into the bulk-load block layout (models.gemm.PackedWeight); the prefill unpacks one matrix at a time.
        # The gate/up rows are interleaved by 64 on the way (every output tile pairs 64 gate features with
        # their up features), so SiLU * up runs in the GEMM's cluster reduction or in a consumer GEMM's
        # epilogue from the same copy of the weights
        self.packed = bool(pack_weights and gemm == "cob")
        il = 64 if self.s["inter"] % 64 == 0 else 0
        if self.packed:
            for L in weights.layers:
                L.wqkv, L.wo, L.wdown = (pack_weight(dense(t)) for t in (L.wqkv, L.wo, L.wdown))
                L.wgu = pack_weight(dense(L.wgu), interleave=il)
            weights.lm_head = pack_weight(dense(weights.lm_head))
        self.lin = {}
        for i, L in enumerate(weights.layers):
            self.lin[(i, "qkv")] = Linear(L.wqkv, gemm)
            self.lin[(i, "o")] = Linear(L.wo, gemm)
            self.lin[(i, "gu")] = GateUpLinear(L.wgu, gemm)  # gate_up GEMM + SiLU * up (one kernel or two)
            self.lin[(i, "down")] = Linear(L.wdown, gemm)
        self.lin["head"] = Linear(weights.lm_head, gemm)
        self.graphs: dict[int, tuple] = {}
        self.kernels_per_step: dict[int, int] = {}
        self.pdl = pdl  # programmatic dependent launch between the kernels of a captured step
        # weight tiles each GEMM prefetches into L2 beyond its ring while it waits for its activations
        self.l2_prefetch = int(l2_prefetch)
        # layer-boundary fusion: o_proj / down_proj push their partial sums straight into the
        # all-reduce landing buffers, and the all-reduce + residual + RMSNorm runs inside the next
        # GEMM (gate_up, the next layer's qkv, the LM head); needs TP > 1, bf16 and this package's GEMMs
        # "ours": the fused all-reduce + residual + RMSNorm kernel; "nccl": the baseline decode step, NCCL
        # all-reduce (captured in the graph) followed by this package's add + RMSNorm kernel; "vllm": the
        # reference's baseline stack, vLLM's custom all-reduce (NCCL where vLLM declines a size, as vLLM
        # does) followed by vLLM's fused_add_rms_norm; it needs a gloo group (`car_group`) for vLLM's
        # buffer exchange
        assert collective in ("ours", "nccl", "vllm")
        self.collective = collective
        self._car = self._vllm_ops = None
        if collective == "vllm" and self.tp > 1:
            import vllm._custom_ops  # noqa: F401  registers torch.ops._C
            from vllm.distributed.device_communicators.custom_all_reduce import CustomAllreduce

            assert car_group is not None, "collective='vllm' needs a gloo process group (car_group)"
            self._vllm_ops = torch.ops._C
            self._car = CustomAllreduce(car_group, self.device, max_size=max(8 << 20, 2 * max_batch * cfg.hidden * 2))
            if self._car.disabled:
                raise RuntimeError("vLLM custom all-reduce is disabled on this system")
        self.fuse_boundary = bool(fuse_boundary and self.tp > 1 and self.dtype == torch.bfloat16 and gemm == "cob"
                                  and collective == "ours")
        self.fuse_error = ""
        # with fuse_boundary: SiLU * up and RoPE + KV append inside the consumer GEMMs' epilogues
        self.fuse_epilogues = bool(fuse_epilogues)
        self._fuse_epi: dict[int, tuple[bool, bool]] = {}
        self._wgu_il: list | None = None
        # per batch size: (attention-output boundary fused, MLP-output boundary fused); with
        # tune_boundaries the capture times each combination and keeps the fastest (max over ranks)
        self.fuse_kinds: dict[int, tuple[bool, bool]] = {}
        # per batch size: (SiLU epilogue in the gate_up consumer, RoPE + KV append in the QKV consumer)
        # used where available; chosen together with the boundary kinds when tuning
        self.epi_use: dict[int, tuple[bool, bool]] = {}
        self.tune_boundaries = bool(tune_boundaries)
        self.boundary_times: dict[int, dict[str, float]] = {}
        if self.fuse_boundary:
            comm.prepare_fused_gemm(cfg.hidden)

    # ------------------------------------------------------------------ prefill (plain torch)
    def _ar(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            import torch.distributed as dist

            dist.all_reduce(x, group=self.nccl_group)
        return x

    @torch.no_grad()
    def prefill(self, prompts: torch.Tensor, chunk_tokens: int = 4096) -> torch.Tensor:
        """prompts [B, P] int -> first generated token ids [B] (int32, on device)."""
        cfg, s, D = self.cfg, self.s, self.cfg.head_dim
        B, P = prompts.shape
        self.cache.reserve(B, self.max_seq)
        bt = self.cache.block_tables[:B].long()
        pos = torch.arange(P, device=self.device)
        x = self.w.embed[prompts.to(self.device).long()]  # [B, P, H]
        c, sn = self.cos[pos][None, :, None, :], self.sin[pos][None, :, None, :]

        def rope(t):  # [B, P, heads, D]
            t1, t2 = t[..., :D // 2].float(), t[..., D // 2:].float()
            return torch.cat([t1 * c - t2 * sn, t2 * c + t1 * sn], -1).to(self.dtype)

        res = x
        for i, L in enumerate(self.w.layers):
            h = F.rms_norm(res.float(), (cfg.hidden,), L.ln1.float(), cfg.eps).to(self.dtype)
            qkv = h @ dense(L.wqkv).t()
            if L.bqkv is not None:
                qkv = qkv + L.bqkv
            q, k, v = qkv.split([s["nq"] * D, s["nkv"] * D, s["nkv"] * D], -1)
            q = rope(q.view(B, P, s["nq"], D))
            k = rope(k.view(B, P, s["nkv"], D))
            v = v.view(B, P, s["nkv"], D)
            nb = (P + 15) // 16
            pad = nb * 16 - P
            kp = F.pad(k, (0, 0, 0, 0, 0, pad)).view(B, nb, 16, s["nkv"], D).permute(0, 1, 3, 2, 4)
            vp = F.pad(v, (0, 0, 0, 0, 0, pad)).view(B, nb, 16, s["nkv"], D).permute(0, 1, 3, 2, 4)
            self.cache.k[i][bt[:, :nb]] = kp
            self.cache.v[i][bt[:, :nb]] = vp
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True, enable_gqa=True, scale=self.scale)
            o = self._ar(a.transpose(1, 2).reshape(B, P, -1) @ dense(L.wo).t())
            res = res + o
            h = F.rms_norm(res.float(), (cfg.hidden,), L.ln2.float(), cfg.eps).to(self.dtype)
            g, u = (h @ dense(L.wgu).t()).chunk(2, -1)
            d = self._ar((F.silu(g.float()) * u.float()).to(self.dtype) @ dense(L.wdown).t())
            res = res + d
        h = F.rms_norm(res[:, -1].float(), (cfg.hidden,), self.w.final_norm.float(), cfg.eps).to(self.dtype)
        logits = (h @ dense(self.w.lm_head).t()).float()
        val, idx = logits.max(-1)
        idx = idx + self.rank * self.s["vocab"]
        if self.tp > 1:
            import torch.distributed as dist

            vals = [torch.empty_like(val) for _ in range(self.tp)]
            idxs = [torch.empty_like(idx) for _ in range(self.tp)]
            dist.all_gather(vals, val, group=self.nccl_group)
            dist.all_gather(idxs, idx, group=self.nccl_group)
            v = torch.stack(vals)
            best = v.argmax(0)
            idx = torch.stack(idxs).gather(0, best[None])[0]
        self.prompt_len = P
        return idx.to(torch.int32)

    # ------------------------------------------------------------------ decode step (our kernels)
    def _buffers(self, B: int) -> dict:
        cfg, s, D, dev, dt = self.cfg, self.s, self.cfg.head_dim, self.device, self.dtype
        e = lambda *shape: torch.empty(*shape, dtype=dt, device=dev)  # noqa: E731
        return dict(
            ids=torch.zeros(B, dtype=torch.int32, device=dev),
            pos=torch.zeros(B, dtype=torch.int32, device=dev),
            lens=torch.zeros(B, dtype=torch.int32, device=dev),
            res=e(B, cfg.hidden), h=e(B, cfg.hidden), part=e(B, cfg.hidden),
            qkv=e(B, (s["nq"] + 2 * s["nkv"]) * D), q=e(B, s["nq"], D), attn=e(B, s["nq"], D),
            gu=e(B, 2 * s["inter"]), act=e(B, s["inter"]), logits=e(B, s["vocab"]),
            keys=torch.zeros(B, dtype=torch.int64, device=dev),
            gathered=torch.zeros(self.tp, B, dtype=torch.int64, device=dev),
            attn_op=K.DecodeAttention(B, s["nq"], s["nkv"], D, self.cache.max_blocks_per_seq, dev,
                                      torch.cuda.get_device_properties(dev).multi_processor_count),
        )

    def _step(self, B: int, buf: dict) -> int:
        """Issue one decode step on the current stream; returns the number of kernels launched."""
        cfg, s, w, comm = self.cfg, self.s, self.w, self.comm
        bt = self.cache.block_tables[:B]
        n = 0
        K.embedding(buf["ids"], w.embed, out=buf["res"])  # residual stream starts as the embedding
        K.rmsnorm(buf["res"], w.layers[0].ln1, cfg.eps, out=buf["h"])
        n += 2
        ours = 1 if self.gemm == "cob" else 0
        ar_ours = 0 if self._car is not None else 1  # the vLLM stack's two kernels per boundary are not ours
        if self.fuse_boundary:
            return n + self._step_fused(B, buf, bt)
        h = buf["h"]
        for i, L in enumerate(w.layers):
            self.lin[(i, "qkv")](h, out=buf["qkv"])
            n += self._attention(i, L, B, buf, bt)
            self.lin[(i, "o")](buf["attn"].view(B, -1), out=buf["part"])
            h = self._allreduce_add_rmsnorm(buf, L.ln2)
            n += self._gate_up(i, h, B, buf)
            self.lin[(i, "down")](buf["act"], out=buf["part"])
            nxt = w.layers[i + 1].ln1 if i + 1 < len(w.layers) else w.final_norm
            h = self._allreduce_add_rmsnorm(buf, nxt)
            n += 2 * ar_ours + 3 * ours
        self.lin["head"](h, out=buf["logits"])
        K.argmax_local(buf["logits"], self.rank * s["vocab"], keys=buf["keys"])
        n += 1 + ours
        if self.tp > 1:
            comm.all_gather_u32(buf["keys"].view(torch.int32), out=buf["gathered"].view(torch.int32).view(self.tp, 2 * B))
            n += 1
        K.argmax_combine(buf["gathered"] if self.tp > 1 else buf["keys"].view(1, B), self.tp, ids=buf["ids"],
                         positions=buf["pos"], seq_lens=buf["lens"], local_keys=buf["keys"])
        return n + 1

    def _gate_up(self, i: int, h: torch.Tensor, B: int, buf: dict) -> int:
        """buf["act"] = silu(gate) * up of layer i's gate/up projection of h; returns this package's kernel
        count (the GEMM with the SwiGLU epilogue, or the GEMM and the SiLU * up kernel)."""
        lin = self.lin[(i, "gu")]
        lin(h, out=buf["act"])
        return 1 if lin.kernels(B) == 1 else 1 + (1 if self.gemm == "cob" else 0)

    def _allreduce_add_rmsnorm(self, buf: dict, gamma: torch.Tensor) -> torch.Tensor:
        """h = RMSNorm(residual + sum_ranks(part)) * gamma, residual updated (one or two kernels). Returns
        the tensor that holds h: buf["h"], or on the vLLM path the all-reduce's own output."""
        if self.tp > 1 and self.collective in ("nccl", "vllm"):
            import torch.distributed as dist

            out = self._car.custom_all_reduce(buf["part"]) if self._car is not None else None
            if out is None:  # NCCL (the "nccl" step, or a size vLLM's custom all-reduce declines)
                dist.all_reduce(buf["part"], group=self.nccl_group)
                out = buf["part"]
            if self._car is not None:
                self._vllm_ops.fused_add_rms_norm(out, buf["res"], gamma, self.cfg.eps)
                return out
            K.add_rmsnorm(out, buf["res"], gamma, self.cfg.eps, out=buf["h"])
            return buf["h"]
        self.comm.fused_allreduce_add_rmsnorm(buf["part"], buf["res"], gamma, self.cfg.eps, out=buf["h"])
        return buf["h"]

    def _fused_epilogues(self, B: int, buf: dict) -> tuple[bool, bool]:
        """(swiglu in the gate_up GEMM, RoPE + KV append in the QKV GEMM) for batch B: used when the
        consumer GEMM has a launch geometry for them (2..8 K-splits per output tile)."""
        if not self.fuse_epilogues:
            return False, False
        if B not in self._fuse_epi:
            cfg, s, L, comm = self.cfg, self.s, self.w.layers[0], self.comm
            comm.ar_norm_gemm(buf["res"], L.ln2, L.wgu, dry_run=True, epilogue="swiglu")
            sw = comm.last_fused_gemm[1][2] > 0 and s["inter"] % 64 == 0
            comm.ar_norm_gemm(buf["res"], L.ln1, L.wqkv, dry_run=True, epilogue="rope_kv")
            # the QKV epilogue has no bias term: a QKV bias keeps RoPE + append in its own kernel
            rp = comm.last_fused_gemm[1][2] > 0 and cfg.head_dim == 128 and not cfg.qkv_bias
            if sw and self._wgu_il is None:
                if self._gu_interleave() == 64:  # the packed gate/up weights are already in that order
                    self._wgu_il = [Lw.wgu for Lw in self.w.layers]
                else:  # tile-interleaved gate/up copies (allocated outside capture)
                    il = [comm.interleave_gate_up(dense(Lw.wgu)) for Lw in self.w.layers]
                    self._wgu_il = [pack_weight(t) for t in il] if self.packed else il
            self._fuse_epi[B] = (sw, rp)
        return self._fuse_epi[B]

    def _gu_interleave(self) -> int:
        """Row interleave of the gate/up weights as stored (0: [gate; up])."""
        wgu = self.w.layers[0].wgu
        return wgu.il if isinstance(wgu, PackedWeight) else 0

    def _attention(self, i: int, L, B: int, buf: dict, bt: torch.Tensor) -> int:
        """RoPE + paged-KV append of the new token and the attention of layer i from buf["qkv"]; one kernel
        with `fuse_append` (the attention kernel rotates and appends), else two. Returns the kernel count."""
        s = self.s
        if self.fuse_append:
            buf["attn_op"](buf["q"], self.cache.k[i], self.cache.v[i], bt, buf["lens"], buf["attn"], self.scale,
                           append=dict(qkv=buf["qkv"], positions=buf["pos"], cos=self.cos, sin=self.sin, bias=L.bqkv))
            return 1
        K.rope_append_kv(buf["qkv"], buf["pos"], self.cos, self.sin, bt, buf["q"], self.cache.k[i],
                         self.cache.v[i], s["nq"], s["nkv"], bias=L.bqkv)
        buf["attn_op"](buf["q"], self.cache.k[i], self.cache.v[i], bt, buf["lens"], buf["attn"], self.scale)
        return 2

    def fused_epilogues_used(self, B: int) -> tuple[bool, bool]:
        """(SiLU in gate_up, RoPE + KV append in QKV) as the captured step for batch B runs them."""
        if not self.fuse_boundary or B not in self._fuse_epi:
            return False, False
        fa, fm = self.fuse_kinds.get(B, (True, True))
        ua, um = self.epi_use.get(B, (True, True))
        sw, rp = self._fuse_epi[B]
        return bool(sw and fa and ua), bool(rp and fm and um)

    def _step_fused(self, B: int, buf: dict, bt: torch.Tensor) -> int:
        """Decode step with fused layer boundaries (after the embedding and first norm). Each of the two
        boundary kinds of a layer - attention output (o_proj -> all-reduce + residual + RMSNorm ->
        gate_up) and MLP output (down_proj -> ... -> next layer's QKV, or the LM head) - is either fused
        (push GEMM + consumer GEMM, 2 kernels) or separate (GEMM, fused all-reduce kernel, GEMM), as
        `fuse_kinds[B]` says (both fused by default). Where the consumer GEMM supports it, SiLU * up runs
        in the gate_up epilogue and RoPE + the paged-KV append in the QKV epilogue."""
        cfg, s, w, comm = self.cfg, self.s, self.w, self.comm
        fa, fm = self.fuse_kinds.get(B, (True, True))
        ua, um = self.epi_use.get(B, (True, True))
        sw, rp = self._fused_epilogues(B, buf)
        sw, rp = sw and fa and ua, rp and fm and um
        n = 0
        self.lin[(0, "qkv")](buf["h"], out=buf["qkv"])
        n += 1
        for i, L in enumerate(w.layers):
            if i == 0 or not rp:
                n += self._attention(i, L, B, buf, bt)
            else:  # the previous consumer GEMM's epilogue rotated q and appended k / v
                buf["attn_op"](buf["q"], self.cache.k[i], self.cache.v[i], bt, buf["lens"], buf["attn"], self.scale)
                n += 1
            # attention-output boundary
            if fa:
                comm.gemm_push(buf["attn"].view(B, -1), L.wo)
                if sw:
                    comm.ar_norm_gemm(buf["res"], L.ln2, self._wgu_il[i], cfg.eps, out=buf["act"], epilogue="swiglu")
                else:  # outputs in the stored gate/up order
                    comm.ar_norm_gemm(buf["res"], L.ln2, L.wgu, cfg.eps, out=buf["gu"])
                    K.silu_mul(buf["gu"], out=buf["act"], interleave=self._gu_interleave())
                    n += 1
                n += 2
            else:
                self.lin[(i, "o")](buf["attn"].view(B, -1), out=buf["part"])
                h = self._allreduce_add_rmsnorm(buf, L.ln2)
                n += 2 + self._gate_up(i, h, B, buf)
            # MLP-output boundary
            last = i + 1 == len(w.layers)
            nxt = None if last else w.layers[i + 1]
            gamma = w.final_norm if last else nxt.ln1
            if fm:
                comm.gemm_push(buf["act"], L.wdown)
                if last:
                    comm.ar_norm_gemm(buf["res"], gamma, w.lm_head, cfg.eps, out=buf["logits"])
                elif rp:
                    comm.ar_norm_gemm(buf["res"], gamma, nxt.wqkv, cfg.eps, out=buf["q"], epilogue="rope_kv",
                                      rope=dict(positions=buf["pos"], cos=self.cos, sin=self.sin, block_tables=bt,
                                                k_cache=self.cache.k[i + 1], v_cache=self.cache.v[i + 1],
                                                nq=s["nq"], nkv=s["nkv"]))
                else:
                    comm.ar_norm_gemm(buf["res"], gamma, nxt.wqkv, cfg.eps, out=buf["qkv"])
                n += 2
            else:
                self.lin[(i, "down")](buf["act"], out=buf["part"])
                h = self._allreduce_add_rmsnorm(buf, gamma)
                if last:
                    self.lin["head"](h, out=buf["logits"])
                else:
                    self.lin[(i + 1, "qkv")](h, out=buf["qkv"])
                n += 3
        K.argmax_local(buf["logits"], self.rank * s["vocab"], keys=buf["keys"])
        comm.all_gather_u32(buf["keys"].view(torch.int32), out=buf["gathered"].view(torch.int32).view(self.tp, 2 * B))
        K.argmax_combine(buf["gathered"], self.tp, ids=buf["ids"], positions=buf["pos"], seq_lens=buf["lens"],
                         local_keys=buf["keys"])
        return n + 3

    def _tune_fusion(self, B: int, buf: dict, saved: dict, warm: int = 2, reps: int = 5) -> tuple[bool, bool]:
        """Time one captured decode step per choice of fused / separate boundaries (attention output,
        MLP output) and, where a fused boundary's consumer GEMM supports its epilogue (SiLU * up in
        gate_up, RoPE + KV append in the next QKV) and `fuse_epilogues` is set, with and without it.
        The per-choice times are reduced with MAX over the ranks before the choice, so every rank takes
        the same one; the decode state is restored after each. Sets `epi_use[B]`, returns the kinds."""
        import torch.distributed as dist

        sw_ok, rp_ok = self._fused_epilogues(B, buf)
        combos = []
        for fa in (True, False):
            for fm in (True, False):
                for ua in ((True, False) if fa and sw_ok else (False,)):
                    for um in ((True, False) if fm and rp_ok else (False,)):
                        combos.append((fa, fm, ua, um))
        times = torch.zeros(len(combos), dtype=torch.float64, device=self.device)
        for j, (fa, fm, ua, um) in enumerate(combos):
            self.fuse_kinds[B], self.epi_use[B] = (fa, fm), (ua, um)
            s = torch.cuda.Stream(self.device)  # one eager step first, as before any capture
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self._step(B, buf)
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            for k, v in saved.items():
                buf[k].copy_(v)
            g = torch.cuda.CUDAGraph()
            old = K.set_pdl(self.pdl)
            try:
                with torch.cuda.graph(g):
                    self._step(B, buf)
            finally:
                K.set_pdl(old)
            for _ in range(warm):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            torch.cuda.synchronize(self.device)
            times[j] = e0.elapsed_time(e1) / reps
            del g
            for k, v in saved.items():
                buf[k].copy_(v)
        dist.all_reduce(times, op=dist.ReduceOp.MAX, group=self.nccl_group)
        t = times.tolist()

        def label(c):  # S: separate, F: fused, E: fused with the consumer's epilogue
            fa, fm, ua, um = c
            return ("E" if ua else "F" if fa else "S") + ("E" if um else "F" if fm else "S")

        self.boundary_times[B] = {label(c): round(x, 4) for c, x in zip(combos, t)}
        best = combos[min(range(len(combos)), key=lambda k: (t[k], k))]
        self.epi_use[B] = best[2:]
        if not best[2] and self._wgu_il is not None and all(not u[0] for u in self.epi_use.values()):
            self._wgu_il = None  # the interleaved gate/up copies are not used by the chosen step
            self._fuse_epi = {b: (False, v[1]) for b, v in self._fuse_epi.items()}
        return best[:2]

    def start(self, B: int, first_ids: torch.Tensor, prompt_len: int):
        """Set up decoding of B sequences whose prompts (length prompt_len) are in the cache."""
        if B not in self.graphs:
            self.graphs[B] = (None, self._buffers(B))
        buf = self.graphs[B][1]
        buf["ids"].copy_(first_ids.to(torch.int32))
        buf["pos"].fill_(prompt_len)
        buf["lens"].fill_(prompt_len + 1)
        return buf

    def tune(self, B: int):
        """Pick the fastest measured GEMM schedule of every projection shape for batch B (cached per shape)."""
        for lin in self.lin.values():
            lin.tune(B)

    def capture(self, B: int, tune: bool = True):
        """Capture one decode step for batch B in a CUDA graph (buffers are static)."""
        old = K.set_l2_prefetch(self.l2_prefetch) if self.gemm == "cob" else None
        try:
            return self._capture(B, tune)
        finally:
            if old is not None:
                K.set_l2_prefetch(old)

    def _capture(self, B: int, tune: bool):
        if tune and self.gemm == "cob":
            self.tune(B)
        buf = self.graphs[B][1]
        saved = {k: v.clone() for k, v in buf.items() if k in ("ids", "pos", "lens")}
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        try:
            with torch.cuda.stream(s):
                self._step(B, buf)  # warm-up outside the graph (also compiles lazy modules)
        except RuntimeError as e:
            if not self.fuse_boundary:
                raise
            # a fused layer boundary rejected this geometry (the launcher's residency / capacity
            # checks, identical on every rank): re-initialise the collective state and run unfused
            torch.cuda.synchronize(self.device)
            self.comm.reset()
            self.fuse_boundary = False
            self.fuse_error = str(e)
            for k, v in saved.items():
                buf[k].copy_(v)
            with torch.cuda.stream(s):
                self._step(B, buf)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        for k, v in saved.items():
            buf[k].copy_(v)
        if self.fuse_boundary and self.tune_boundaries and self.nccl_group is not None and B not in self.fuse_kinds:
            try:
                self.fuse_kinds[B] = self._tune_fusion(B, buf, saved)
            except RuntimeError as e:
                # a host-side rejection is the same on every rank (same shapes), so every rank lands
                # here at the same point: re-initialise the collective state and keep both kinds fused.
                # (A timed-out device wait is reported by the caller's comm.check(), not here.)
                torch.cuda.synchronize(self.device)
                self.comm.reset()
                self.fuse_kinds[B] = (True, True)
                self.fuse_error = f"boundary tuning: {e}"
                for k, v in saved.items():
                    buf[k].copy_(v)
        g = torch.cuda.CUDAGraph()
        old = K.set_pdl(self.pdl)
        try:
            # vLLM registers the buffers its all-reduce used in the graph when its capture context ends
            with (self._car.capture() if self._car is not None else contextlib.nullcontext()):
                with torch.cuda.graph(g):
                    self.kernels_per_step[B] = self._step(B, buf)
        finally:
            K.set_pdl(old)
        self.graphs[B] = (g, buf)
        # the warm-up step advanced the device state once; restore the decode position
        for k, v in saved.items():
            buf[k].copy_(v)
        torch.cuda.synchronize(self.device)
        return g

    def step(self, B: int, use_graph: bool = True) -> torch.Tensor:
        g, buf = self.graphs[B]
        if use_graph and g is not None:
            g.replay()
        else:
            self._step(B, buf)
        return buf["ids"]

    def decode(self, B: int, host_ids: torch.Tensor, host_out: torch.Tensor, monitor=None,
               sync_timeout_s: float = 60.0) -> torch.Tensor:
        """One end-to-end greedy step through the public API: copy this step's input token ids from
        pinned host memory, run the captured step, read the next ids back into pinned host memory.
        With a `parallel.health.RankMonitor`, every rank first meets the others at the step boundary on
        the host (RankFailure if a peer failed, left or is late), so no kernel is launched that waits for
        a rank that is gone; without one, nothing is added to the step."""
        if monitor is not None:
            monitor.sync(sync_timeout_s)
        g, buf = self.graphs[B]
        buf["ids"].copy_(host_ids, non_blocking=True)
        if g is not None:
            g.replay()
        else:
            self._step(B, buf)
        host_out.copy_(buf["ids"], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return host_out

    def release_graphs(self):
        """Drop captured graphs (required before destroying the process group) and, on the vLLM path,
        vLLM's all-reduce buffers (collective: every rank calls it)."""
        self.graphs = {B: (None, buf) for B, (g, buf) in self.graphs.items()}
        if self._car is not None:
            self._car.close()
            self._car = None


def reference_logits(cfg: LlamaConfig, full: dict, tokens: torch.Tensor, device) -> torch.Tensor:
    """Unsharded fp32 forward of `tokens` [B, T] (no KV cache: full recompute); logits [B, vocab] of
    the last position."""
    W = {k: v for k, v in full.items() if k != "layers"}
    D = cfg.head_dim
    toks = tokens.to(device).long()
    B, P = toks.shape
    cos, sin = rope_tables(P, D, cfg.rope_theta, device)
    c, sn = cos[:P][None, :, None, :], sin[:P][None, :, None, :]

    def rope(t):
        t1, t2 = t[..., :D // 2], t[..., D // 2:]
        return torch.cat([t1 * c - t2 * sn, t2 * c + t1 * sn], -1)

    x = W["embed"].to(device).float()[toks]
    for L in full["layers"]:
        L = {k: v.to(device).float() for k, v in L.items()}
        h = F.rms_norm(x, (cfg.hidden,), L["ln1"], cfg.eps)
        qkv = h @ L["wqkv"].t() + (L["bqkv"] if "bqkv" in L else 0.0)
        q, k, v = qkv.split([cfg.heads * D, cfg.kv_heads * D, cfg.kv_heads * D], -1)
        q, k = rope(q.view(B, P, cfg.heads, D)), rope(k.view(B, P, cfg.kv_heads, D))
        v = v.view(B, P, cfg.kv_heads, D)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                           enable_gqa=True, scale=1.0 / math.sqrt(D))
        x = x + a.transpose(1, 2).reshape(B, P, -1) @ L["wo"].t()
        h = F.rms_norm(x, (cfg.hidden,), L["ln2"], cfg.eps)
        g, u = (h @ L["wgu"].t()).chunk(2, -1)
        x = x + (F.silu(g) * u) @ L["wdown"].t()
    h = F.rms_norm(x[:, -1], (cfg.hidden,), W["final_norm"].to(device).float(), cfg.eps)
    return h @ W["lm_head"].to(device).float().t()


def reference_greedy(cfg: LlamaConfig, full: dict, prompts: torch.Tensor, steps: int, device) -> torch.Tensor:
    """Unsharded fp32 greedy decoding (no KV cache: full recompute), tokens [B, steps+1]."""
    toks = prompts.to(device).long()
    out = []
    for _ in range(steps + 1):
        nxt = reference_logits(cfg, full, toks, device).argmax(-1)
        out.append(nxt)
        toks = torch.cat([toks, nxt[:, None]], 1)
    return torch.stack(out, 1)


def tiny_config(**kw) -> LlamaConfig:
    return replace(TINY, **kw)

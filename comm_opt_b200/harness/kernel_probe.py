"""Single-kernel drivers on one GPU: a fixed, small workload per hot kernel, timed with CUDA events
(warm-up, then `--iters` launches, p50; `--graph K` times graphs of K back-to-back launches, which
removes the host launch interval), and the command a profiler capture of that kernel runs.

    python -m comm_opt_b200.harness.kernel_probe fused_ar --variant lamport_1s --world 2 --rows 8
    python -m comm_opt_b200.harness.kernel_probe attention --batch 8 --ctx 2048
    python -m comm_opt_b200.harness.kernel_probe decode_ops --batch 8
    python -m comm_opt_b200.harness.kernel_probe allgather --world 8 --rows 16
    ncu --set full --clock-control none -k regex:k_oneshot -s 3 -c 1 -o oneshot \
        python -m comm_opt_b200.harness.kernel_probe fused_ar --variant lamport_1s --world 2 --rows 8 --iters 4

Shapes default to one Llama-70B TP=8 rank: hidden 8192, 8 query heads / 1 KV head of 128, SwiGLU
shard 3584. Fused-op ranks are emulated in one launch (see TPCommunicator(emulate_world=...)).
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops import kernels as K
from ..ops.reference import rope_tables
from ..parallel import TPCommunicator


GRAPH_OPS = 0  # > 0: time graphs of this many back-to-back launches (device time per launch)


def timed(fn, iters: int) -> dict:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    per, g = 1, None
    if GRAPH_OPS > 0:
        per, g = GRAPH_OPS, torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(per):
                fn()
        g.replay()
        torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(iters + 1)]
    ev[0].record()
    for i in range(iters):
        g.replay() if g is not None else fn()
        ev[i + 1].record()
    torch.cuda.synchronize()
    us = sorted(ev[i].elapsed_time(ev[i + 1]) * 1000.0 / per for i in range(iters))
    return dict(p50_us=round(us[len(us) // 2], 3), min_us=round(us[0], 3), iters=iters, per_graph=per)


def fused_ar(a, dev) -> dict:
    comm = TPCommunicator(emulate_world=a.world, device=dev, dtype=torch.bfloat16, max_rows=a.rows, max_hidden=a.hidden)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(a.world, a.rows, a.hidden, generator=g, device=dev).bfloat16()
    res = torch.randn(a.world, a.rows, a.hidden, generator=g, device=dev).bfloat16()
    gamma = torch.ones(a.hidden, device=dev).bfloat16()
    out = torch.empty_like(x)
    r = timed(lambda: comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, out=out, variant=a.variant), a.iters)
    comm.check()
    return dict(r, variant=a.variant, world=a.world, rows=a.rows, hidden=a.hidden, choice=comm.last_choice.__dict__,
                bytes_per_rank=a.rows * a.hidden * 2)


def allgather(a, dev) -> dict:
    """The argmax all-gather (`k_allgather_u32`): `--rows` 32-bit words per rank, ranks emulated in one launch."""
    comm = TPCommunicator(emulate_world=a.world, device=dev, dtype=torch.bfloat16, max_rows=a.rows, max_hidden=a.hidden)
    inp = torch.arange(a.world * a.rows, dtype=torch.int32, device=dev).view(a.world, a.rows)
    out = torch.empty(a.world, a.world, a.rows, dtype=torch.int32, device=dev)
    r = timed(lambda: comm.all_gather_u32(inp, out=out), a.iters)
    comm.check()
    assert torch.equal(out, inp.unsqueeze(0).expand(a.world, -1, -1)), "all-gather mismatch"
    return dict(r, world=a.world, words=a.rows)


def attention(a, dev) -> dict:
    B, nq, nkv, D, blk = a.batch, a.heads, a.kv_heads, a.head_dim, 16
    pages = (a.ctx + blk - 1) // blk
    nblocks = B * pages + 16
    g = torch.Generator(device=dev).manual_seed(0)
    kc = torch.randn(nblocks, nkv, blk, D, generator=g, device=dev).bfloat16()
    vc = torch.randn(nblocks, nkv, blk, D, generator=g, device=dev).bfloat16()
    perm = torch.randperm(nblocks, generator=torch.Generator().manual_seed(1))[:B * pages]
    bt = perm.view(B, pages).to(torch.int32).to(dev)
    lens = torch.full((B,), a.ctx, dtype=torch.int32, device=dev)
    q = torch.randn(B, nq, D, generator=g, device=dev).bfloat16()
    out = torch.empty_like(q)
    op = K.DecodeAttention(B, nq, nkv, D, pages, dev, torch.cuda.get_device_properties(dev).multi_processor_count)
    if a.splits:  # explicit split count (cluster merge up to 16)
        from .._ext import native

        op.pps = -(-pages // a.splits)
        op.splits = -(-pages // op.pps)
        op.cluster = op.splits <= 16 and not a.no_cluster
        op.scratch = torch.zeros(native().attn_scratch_bytes(B, nkv, op.splits, nq // nkv, D), dtype=torch.uint8,
                                 device=dev)
    if a.append:  # the decode step's form: q and the new token's k / v from the QKV output, rotated here
        qkv = torch.randn(B, (nq + 2 * nkv) * D, generator=g, device=dev).bfloat16()
        pos = (lens - 1).contiguous()
        cos, sin = rope_tables(a.ctx + 16, D, 5e5, dev)
        app = dict(qkv=qkv, positions=pos, cos=cos, sin=sin)
        r = timed(lambda: op(q, kc, vc, bt, lens, out, D ** -0.5, append=app), a.iters)
    else:
        r = timed(lambda: op(q, kc, vc, bt, lens, out, D ** -0.5), a.iters)
    kv_bytes = 2 * B * nkv * a.ctx * D * 2
    return dict(r, batch=B, ctx=a.ctx, heads=nq, kv_heads=nkv, head_dim=D, splits=op.splits,
                pages_per_split=op.pps, cluster=op.cluster, kv_bytes=kv_bytes)


def decode_ops(a, dev) -> dict:
    B, H, nq, nkv, D, inter = a.batch, a.hidden, a.heads, a.kv_heads, 128, a.inter
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(B, H, generator=g, device=dev).bfloat16()
    gamma = torch.ones(H, device=dev).bfloat16()
    h = torch.empty_like(x)
    qkv = torch.randn(B, (nq + 2 * nkv) * D, generator=g, device=dev).bfloat16()
    pages = 8
    kc = torch.zeros(B * pages, nkv, 16, D, device=dev).bfloat16()
    vc = torch.zeros_like(kc)
    bt = torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages)
    pos = torch.full((B,), 100, dtype=torch.int32, device=dev)
    cos, sin = rope_tables(256, D, 5e5, dev)
    q = torch.empty(B, nq, D, device=dev).bfloat16()
    gu = torch.randn(B, 2 * inter, generator=g, device=dev).bfloat16()
    act = torch.empty(B, inter, device=dev).bfloat16()
    res = torch.randn(B, H, generator=g, device=dev).bfloat16()
    table = torch.randn(a.vocab, H, generator=g, device=dev).bfloat16()
    ids = torch.randint(0, a.vocab, (B,), generator=torch.Generator().manual_seed(2)).to(torch.int32).to(dev)
    logits = torch.randn(B, a.vocab, generator=g, device=dev).bfloat16()
    keys = torch.zeros(B, dtype=torch.int64, device=dev)
    out = {}
    out["rmsnorm"] = timed(lambda: K.rmsnorm(x, gamma, 1e-5, out=h), a.iters)
    out["add_rmsnorm"] = timed(lambda: K.add_rmsnorm(x, res, gamma, 1e-5, out=h), a.iters)
    out["rope_append"] = timed(lambda: K.rope_append_kv(qkv, pos, cos, sin, bt, q, kc, vc, nq, nkv), a.iters)
    out["silu_mul"] = timed(lambda: K.silu_mul(gu, out=act), a.iters)
    out["embedding"] = timed(lambda: K.embedding(ids, table, out=h), a.iters)
    out["argmax"] = timed(lambda: K.argmax_combine(K.argmax_local(logits, 0, keys=keys).view(1, B), 1,
                                                   local_keys=keys), a.iters)
    return dict(batch=B, hidden=H, inter=inter, **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["fused_ar", "allgather", "attention", "decode_ops"])
    ap.add_argument("--variant", default="lamport_1s")
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--rows", type=int, default=8)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--kv-heads", type=int, default=1)
    ap.add_argument("--inter", type=int, default=3584)
    ap.add_argument("--head-dim", type=int, default=128, choices=[64, 128])
    ap.add_argument("--vocab", type=int, default=16032, help="decode_ops: embedding rows and argmax width")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--splits", type=int, default=0, help="attention: override the split plan")
    ap.add_argument("--graph", type=int, default=0, help="time CUDA graphs of this many launches")
    ap.add_argument("--no-cluster", action="store_true", help="attention with --splits: merge through global memory")
    ap.add_argument("--attn-stages", type=int, default=0, help="attention KV ring depth (6: deep ring; 0: default)")
    ap.add_argument("--append", action="store_true", help="attention with the fused RoPE + KV append")
    a = ap.parse_args()
    global GRAPH_OPS
    GRAPH_OPS = a.graph
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.attn_stages:
        K.set_attn_stages(a.attn_stages)
    r = {"fused_ar": fused_ar, "allgather": allgather, "attention": attention,
         "decode_ops": decode_ops}[a.kernel](a, dev)
    print(json.dumps(dict(kernel=a.kernel, **r)))


if __name__ == "__main__":
    main()

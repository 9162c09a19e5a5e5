"""Launch geometry of every kernel of one decode step, from the host planners (no GPU).

    python -m comm_opt_b200.harness.launch_geometry [--model 70b] [--batch 8] [--ctx 2048] [--tp 1,2,4,8]

For each kernel of the step at each tensor-parallel degree: grid (CTAs), threads per CTA, dynamic shared
memory, and what one SM can hold - the launch's CTAs over the 148 SMs ("waves"), and whether a CTA of
the kernel fits on an SM beside a CTA of the kernel before it (the condition for a programmatic
dependent launch to start its prologue while the previous kernel runs). The GEMM plans are the
planners' defaults before the capture-time tuning picks among candidates; the fused all-reduce
geometry is the measured variant table's entry or the launcher's rule.
"""
from __future__ import annotations

import argparse
import math

SMS, SMEM_SM, REGS_SM = 148, 228 * 1024, 65536
# registers per thread from the bf16 ptxas table (csrc; python -m comm_opt_b200.harness.ptxas_report)
REGS = {"gemm": 139, "gemm_push": 108, "ar_norm_gemm": 164, "attention": 141, "attention64": 92, "oneshot1": 74,
        "twoshot": 122, "rmsnorm": 80, "rope": 32, "silu": 30, "argmax": 32}


def attn_smem(D: int) -> int:
    return 1024 + 4 * 3 * 2 * 16 * D * 2 + 16 * D * 2 + 4 * 3 * 8 + 512 * 4 + 64


def gemm_smem(bn: int, small: bool) -> int:
    stage = 128 * 64 * 2 + bn * 64 * 2
    stages = min(12, (100 if small else 200) * 1024 // stage)
    return max(stages * stage, bn * 132 * 4) + 1024 + 1024 + bn * 8 + 2048 * 4


def rows_for(model: str, batch: int, ctx: int, tp: int) -> list[dict]:
    from .._ext import native
    from ..models.llama import PRESETS
    from ..ops.kernels import attention_split_plan
    from ..parallel.variant_table import VariantTable

    C = native()
    cfg = PRESETS[model]
    s, D, H = cfg.shard(tp), cfg.head_dim, cfg.hidden
    out = []

    def add(kernel, ctas, threads, smem, regs):
        per_sm = min(SMEM_SM // (smem + 1024) if smem else 32, REGS_SM // (threads * regs), 2048 // threads, 32)
        out.append(dict(kernel=kernel, ctas=ctas, threads=threads, smem_kb=round(smem / 1024, 1), regs=regs,
                        ctas_per_sm=per_sm, waves=round(ctas / (SMS * max(per_sm, 1)), 2), smem=smem))

    shapes = {"qkv": ((s["nq"] + 2 * s["nkv"]) * D, H), "o": (H, s["nq"] * D), "gate_up": (2 * s["inter"], H),
              "down": (H, s["inter"])}
    if tp == 1:
        for name in ("qkv", "o", "gate_up", "down"):
            bn, tiles, ctas, ws = C.gemm_plan(batch, *shapes[name], SMS, 0)
            add(f"gemm {name} (stream-K)", ctas, 192, gemm_smem(bn, False), REGS["gemm"])
    else:
        for name, consumer in (("o", False), ("gate_up", True), ("down", False), ("qkv", True)):
            bn, tiles, splits, kps, xctas, ctas, smem = C.fused_gemm_plan(batch, *shapes[name], 0, SMS, consumer, 0)
            kind = "ar_norm_gemm" if consumer else "gemm_push"
            add(f"{kind} {name} ({tiles} tiles x {splits} splits)", ctas, 192, smem, REGS[kind])
        t = VariantTable.load()
        import torch

        ch = t.lookup(tp, torch.bfloat16, 2, H, batch, True)
        L = C.plan_layout(tp, 512, 8192, 2, 4096)
        rc, v, b, th, cl = C.fused_ar_config(L, tp, batch, H, 2, ch.variant, ch.blocks, ch.threads, ch.cluster, 0,
                                             SMS, True)
        add(f"fused all-reduce (separate boundary; variant {v}, cluster {cl})", b, th, 0,
            REGS["oneshot1"] if v in (1, 3, 5, 7) else REGS["twoshot"])
    pages = (ctx + 15) // 16
    splits, pps, cluster = attention_split_plan(batch, s["nkv"], pages, SMS)
    add(f"attention ({splits} splits, {'cluster' if cluster else 'global'} merge)", batch * s["nkv"] * splits, 128,
        attn_smem(D), REGS["attention" if D == 128 else "attention64"])
    add("rope + KV append", batch * (s["nq"] + 2 * s["nkv"]), 64, 0, REGS["rope"])
    return out


def pair_fits(a: dict, b: dict) -> bool:
    """One CTA of `b` fits on an SM that holds one CTA of `a` (shared memory and registers)."""
    return (a["smem"] + 1024 + b["smem"] + 1024 <= SMEM_SM and
            a["threads"] * a["regs"] + b["threads"] * b["regs"] <= REGS_SM)


def markdown(model: str, batch: int, ctx: int, tps: list[int]) -> str:
    lines = []
    for tp in tps:
        rows = rows_for(model, batch, ctx, tp)
        lines.append(f"\n### {model}, TP={tp}, batch {batch}, context {ctx}\n")
        lines.append("| kernel | CTAs | threads | smem KB | regs | CTAs/SM | waves |")
        lines.append("|---|---|---|---|---|---|---|")
        for r in rows:
            lines.append(f"| {r['kernel']} | {r['ctas']} | {r['threads']} | {r['smem_kb']} | {r['regs']} | "
                         f"{r['ctas_per_sm']} | {r['waves']} |")
        att = next(r for r in rows if r["kernel"].startswith("attention"))
        nxt = next((r for r in rows if r["kernel"].startswith(("gemm_push o", "gemm o"))), None)
        if nxt:
            lines.append(f"\nattention -> {nxt['kernel'].split(' (')[0]}: a CTA of each fits on one SM: "
                         f"{'yes' if pair_fits(att, nxt) else 'no'}; attention leaves "
                         f"{max(0, SMS - math.ceil(att['ctas'] / max(att['ctas_per_sm'], 1)))} SMs without a CTA "
                         f"when spread one per SM.")
    return "\n".join(lines) + "\n"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="70b")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--tp", default="1,2,4,8")
    a = ap.parse_args()
    print(markdown(a.model, a.batch, a.ctx, [int(t) for t in a.tp.split(",")]))


if __name__ == "__main__":
    main()

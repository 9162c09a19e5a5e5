"""Layer-boundary fusion bench at Llama-70B TP shapes: row-parallel down_proj GEMM [B, 3584] x [8192, 3584]^T
-> all-reduce + residual + RMSNorm -> column-parallel QKV GEMM [B, 8192] x [1280, 8192]^T, per rank.

Implementations (each one call = the whole boundary, captured K times in a CUDA graph):
  fused        gemm_push + ar_norm_gemm: two kernels, the collective inside the GEMMs
  ours_split   this package's GEMM -> fused all-reduce + add + RMSNorm kernel -> GEMM (three kernels)
  nccl_cublas  cuBLAS GEMM -> NCCL all-reduce -> vLLM fused_add_rms_norm -> cuBLAS GEMM (separate
               launches; torch add + RMSNorm when vLLM is missing)
  vllm_cublas  cuBLAS GEMM -> vLLM custom all-reduce -> fused_add_rms_norm -> cuBLAS GEMM
Timing as in the fused-op sweep: graph of K calls, R replays, per replay the MAX over ranks, p50 / p99.
Roofline per call: the slower of the weight bytes at the measured HBM copy bandwidth and the bytes
each rank must push over NVLink ((W - 1) x B x 8192 x 2) at the measured peer bandwidth (the newest
committed results/platform record, utils.peaks.link_gbs);
reported as roofline_us / p50_us. Correctness of every implementation against an fp32 oracle
(max|out - ref| / max|ref| <= 2^-5).

    timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \
        --master-addr 127.0.0.1 --master-port 29551 -m comm_opt_b200.harness.boundary_bench
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..models.gemm import Linear, pack_weight
from ..ops.reference import TOL, rel_err
from ..parallel import TPCommunicator
from ..utils.results import RunDir, gpu_state
from ..utils.stats import summary

ROOT = Path(__file__).resolve().parents[2]
from ..utils.peaks import NoRecord, hbm_gbs, link_gbs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", default="1,8,32,128")
    ap.add_argument("--k1", type=int, default=3584, help="down_proj inner size per rank (28672 / TP=8)")
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--n2", type=int, default=1280, help="QKV outputs per rank ((64 + 16) x 128 / TP=8)")
    ap.add_argument("--impls", default="fused,ours_split,nccl_cublas,vllm_cublas")
    ap.add_argument("--graph-ops", type=int, default=10)
    ap.add_argument("--replays", type=int, default=30)
    ap.add_argument("--eps", type=float, default=1e-5)
    ap.add_argument("--out-dir", default=None)
    ap.add_argument("--packed", type=int, choices=[0, 1], default=1,
                    help="our GEMMs (fused and ours_split) read packed weights (models.gemm.pack_weight)")
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    cpu = dist.new_group(backend="gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    H, K1, N2 = a.hidden, a.k1, a.n2
    batches = [int(b) for b in a.batch.split(",")]
    Bmax = max(batches)
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=torch.bfloat16, max_rows=Bmax, max_hidden=H)
    comm.prepare_fused_gemm(H)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    w1 = (0.02 * torch.randn(H, K1, generator=g, device=dev)).bfloat16()
    w2 = (0.02 * torch.randn(N2, H, generator=g, device=dev)).bfloat16()
    gs = torch.Generator(device=dev).manual_seed(7)  # replicated
    gamma = (1 + 0.1 * torch.randn(H, generator=gs, device=dev)).bfloat16()
    # our kernels read packed weights (as the decode runner's); cuBLAS keeps the row-major ones
    pw1, pw2 = (pack_weight(w1), pack_weight(w2)) if a.packed else (w1, w2)
    lin1, lin2 = Linear(pw1, "cob"), Linear(pw2, "cob")
    try:
        import vllm._custom_ops  # noqa: F401

        vops = torch.ops._C
    except Exception:
        vops = None
    car = None
    if "vllm_cublas" in a.impls:
        try:
            from vllm.distributed.device_communicators.custom_all_reduce import CustomAllreduce

            car = CustomAllreduce(cpu, dev, max_size=Bmax * H * 2 * 2)
            car = None if car.disabled else car
        except Exception:
            car = None
    run = RunDir("boundary_bench", Path(a.out_dir) if a.out_dir else None) if rank == 0 else None
    if run:
        run.snapshot()
    roof_hbm = (H * K1 + N2 * H) * 2 / (hbm_gbs() * 1e3)  # us
    try:
        peer_gbs = link_gbs()
    except NoRecord as e:  # the roofline then counts the weight bytes only
        peer_gbs = None
        if rank == 0:
            print(f"note: {e}", flush=True)
    rows, n_job = [], 0
    for B in batches:
        x = torch.randn(B, K1, generator=g, device=dev).bfloat16()
        res0 = torch.randn(B, H, generator=gs, device=dev).bfloat16()
        # fp32 oracle (needs every rank's x and w1)
        xs = [torch.empty_like(x) for _ in range(world)]
        ws = [torch.empty_like(w1) for _ in range(world)]
        dist.all_gather(xs, x)
        dist.all_gather(ws, w1)
        h_ref = res0.float() + sum(xs[r].float() @ ws[r].float().t() for r in range(world))
        n_ref = h_ref * torch.rsqrt(h_ref.pow(2).mean(-1, keepdim=True) + a.eps) * gamma.float()
        out_ref = n_ref @ w2.float().t()
        del xs, ws
        for impl in a.impls.split(","):
            t0, state = time.time(), gpu_state() if rank == 0 else ""
            res = res0.clone()
            out = torch.empty(B, N2, dtype=torch.bfloat16, device=dev)
            part = torch.empty(B, H, dtype=torch.bfloat16, device=dev)
            hn = torch.empty(B, H, dtype=torch.bfloat16, device=dev)
            ctx = None
            if impl == "fused":
                def fn():
                    comm.gemm_push(x, pw1)
                    comm.ar_norm_gemm(res, gamma, pw2, a.eps, out=out)
            elif impl == "ours_split":
                lin1.tune(B)
                lin2.tune(B)

                def fn():
                    lin1(x, out=part)
                    comm.fused_allreduce_add_rmsnorm(part, res, gamma, a.eps, out=hn)
                    lin2(hn, out=out)
            elif impl == "nccl_cublas":
                def fn():
                    torch.matmul(x, w1.t(), out=part)
                    dist.all_reduce(part)
                    if vops is not None:
                        vops.fused_add_rms_norm(part, res, gamma, a.eps)  # part <- norm(part + res), res <- sum
                        torch.matmul(part, w2.t(), out=out)
                    else:
                        res.add_(part)
                        torch.matmul(torch.nn.functional.rms_norm(res.float(), (H,), gamma.float(), a.eps).bfloat16(),
                                     w2.t(), out=out)
            elif impl == "vllm_cublas":
                if car is None or vops is None:
                    fn = None
                else:
                    ctx = car.capture

                    def fn():
                        torch.matmul(x, w1.t(), out=part)
                        s = car.custom_all_reduce(part)
                        vops.fused_add_rms_norm(s, res, gamma, a.eps)
                        torch.matmul(s, w2.t(), out=out)
            else:
                fn = None
            err, rel, times = "", float("nan"), []
            ok_all = [None] * world
            dist.all_gather_object(ok_all, fn is not None, group=cpu)
            if all(ok_all):
                try:
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu)
                    fn()
                    torch.cuda.synchronize()
                    rel = max(rel_err(out, out_ref), rel_err(res, h_ref))
                    for _ in range(3):
                        fn()
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu)
                    graph = torch.cuda.CUDAGraph()
                    import contextlib

                    with (ctx() if ctx else contextlib.nullcontext()):
                        with torch.cuda.graph(graph):
                            for _ in range(a.graph_ops):
                                fn()
                    for _ in range(3):
                        graph.replay()
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu)
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.replays + 1)]
                    ev[0].record()
                    for i in range(a.replays):
                        graph.replay()
                        ev[i + 1].record()
                    torch.cuda.synchronize()
                    times = [ev[i].elapsed_time(ev[i + 1]) * 1000.0 / a.graph_ops for i in range(a.replays)]
                    del graph
                    comm.check()
                except Exception as e:  # recorded; every rank takes the gather below
                    err = f"{type(e).__name__}: {str(e)[:200]}"
            gathered = [None] * world
            dist.all_gather_object(gathered, (times, rel, err), group=cpu)
            if rank == 0:
                okt = all(len(t[0]) == a.replays for t in gathered)
                per = [max(t[0][i] for t in gathered) for i in range(a.replays)] if okt else []
                st = summary(per) if per else {}
                worst = max((t[1] for t in gathered if t[1] == t[1]), default=float("nan"))
                errs = next((t[2] for t in gathered if t[2]), "" if all(ok_all) else "unavailable")
                roof_link = (world - 1) * B * H * 2 / (peer_gbs * 1e3) if peer_gbs else 0.0
                roof = max(roof_hbm, roof_link)
                row = dict(impl=impl, world=world, batch=B, p50_us=st.get("p50"), p99_us=st.get("p99"),
                           max_rel_err=worst, correct=bool(worst == worst and worst <= TOL), error=errs,
                           roofline_us=roof, frac_of_roofline=(roof / st["p50"]) if st else None,
                           plan=comm.last_fused_gemm if impl == "fused" else None)
                rows.append(row)
                print(f"{impl:12s} w{world} B{B:4d} p50 {row['p50_us'] or float('nan'):8.2f} us  roofline "
                      f"{roof:6.2f} us ({(row['frac_of_roofline'] or 0) * 100:5.1f}%)  err {worst:.1e} {errs}",
                      flush=True)
                run.schedule(n_job, f"{impl}_B{B}", t0, time.time() - t0, 1 if errs else 0, state)
                n_job += 1
    if rank == 0:
        run.write_json("boundary.json", dict(args=vars(a), world=world, hbm_gbs=hbm_gbs(), peer_gbs=peer_gbs,
                                             comm=comm.describe(), rows=rows,
                                             baseline_norm="vllm fused_add_rms_norm" if vops is not None
                                             else "torch add + rms_norm (vLLM missing)"))
        print(json.dumps(dict(results=str(run.path))), flush=True)
    if car is not None:
        car.close()
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

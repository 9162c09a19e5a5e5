"""Experiment runner: independent launches in a randomised, recorded order (the reference's
exp/lib/ncclrun.py:18-106 - Job, GPU sets, "no other GPU processes" guard, env snapshot, schedule.tsv,
DRY_RUN), driving this repository's torchrun entry points instead of nccl-tests binaries.

    from comm_opt_b200.harness.runner import Job, run_all
    jobs = [Job("collectives", 8, rep=r, args=("--colls", "all_reduce")) for r in range(3)]
    run_all(jobs, "collective_baseline", seed=0)        # DRY_RUN=1 only prints the commands
"""
from __future__ import annotations

import os
import random
import shlex
import subprocess
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

from ..utils.results import ROOT, RunDir, gpu_state

ENTRY = {
    "collectives": "comm_opt_b200.harness.collectives",
    "fused_sweep": "comm_opt_b200.harness.fused_sweep",
    "selftest": "comm_opt_b200.harness.mp_selftest",
    "bakeoff": "comm_opt_b200.harness.allreduce_bakeoff",
    "phases": "comm_opt_b200.harness.phase_profile",
    "boundary": "comm_opt_b200.harness.boundary_bench",
    "comm_share": "comm_opt_b200.harness.comm_share",
    "train_share": "comm_opt_b200.harness.train_share",
    "bench": "bench.py",  # a script at the repository root, not a module
}

GPUSETS = {  # set A: first GPUs; set B: other physical GPUs / rank order (the reference's second set)
    1: {"A": "0", "B": "7"},
    2: {"A": "0,1", "B": "6,7"},
    4: {"A": "0,1,2,3", "B": "4,5,6,7"},
    8: {"A": "0,1,2,3,4,5,6,7", "B": "0,2,4,6,1,3,5,7"},
}


@dataclass
class Job:
    entry: str
    ngpus: int
    gpuset: str = "A"
    rep: int = 0
    variant: str = "default"
    env: dict = field(default_factory=dict)
    args: tuple = ()
    timeout_s: int = 1500

    @property
    def tag(self) -> str:
        return f"{self.entry}_g{self.ngpus}{self.gpuset}_{self.variant}_r{self.rep}"


def gpu_processes() -> str:
    """Compute processes on the GPUs that are not ours (the reference's rule: do not measure next to others)."""
    try:
        out = subprocess.run(["nvidia-smi", "--query-compute-apps=pid,process_name,used_memory",
                              "--format=csv,noheader"], capture_output=True, text=True, timeout=30).stdout
    except (OSError, subprocess.TimeoutExpired):
        return ""
    return "\n".join(l for l in out.splitlines() if l.strip())


def command(job: Job, out: Path, port: int) -> tuple[list[str], dict]:
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=GPUSETS[job.ngpus][job.gpuset], **job.env)
    target = [ENTRY[job.entry]] if ENTRY[job.entry].endswith(".py") else ["-m", ENTRY[job.entry]]
    cmd = ["timeout", "-k", "60", str(job.timeout_s), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={job.ngpus}", "--master-addr=127.0.0.1", f"--master-port={port}", *target, *job.args]
    if job.entry == "collectives":
        cmd += ["--out", str(out / f"{job.tag}.json")]
        # NCCL's set-up (version, channels, NVLS, rings) per job, init-time only (no per-call logging)
        for k, v in (("NCCL_DEBUG", "INFO"), ("NCCL_DEBUG_SUBSYS", "INIT,ENV,GRAPH"),
                     ("NCCL_DEBUG_FILE", str(out / f"{job.tag}.nccl.%h.%p.log"))):
            env.setdefault(k, v)  # a job's own setting (or the caller's environment) wins
    elif job.entry == "fused_sweep":
        cmd += ["--out-dir", str(out / "runs"), "--ts", job.tag]
    elif job.entry in ("bakeoff", "phases", "boundary"):
        cmd += ["--out-dir", str(out / "runs")]
    elif job.entry in ("comm_share", "train_share"):
        cmd += ["--out-dir", str(out / "runs" / job.tag)]  # one trace set per job
    elif job.entry == "bench":
        cmd += ["--gpus", str(job.ngpus), "--out", str(out / f"{job.tag}.json")]
    return cmd, env


def run_all(jobs: list[Job], name: str, seed: int, base: Path | None = None) -> Path | None:
    dry = bool(os.environ.get("DRY_RUN"))
    jobs = list(jobs)
    random.Random(seed).shuffle(jobs)
    if dry:
        for i, j in enumerate(jobs):
            cmd, _ = command(j, Path("results") / name / "DRY", 29700 + i)
            print(shlex.join(cmd))
        print(f"{len(jobs)} jobs, seed {seed}", file=sys.stderr)
        return None
    if procs := gpu_processes():
        sys.exit(f"GPUs have running processes; not measuring:\n{procs}")
    run = RunDir(name, base)
    run.snapshot()
    (run.path / "seed.txt").write_text(f"{seed}\n")
    for i, j in enumerate(jobs):
        if run.done(f"{j.tag}.log"):
            continue  # resume: this job already ran in this directory
        if procs := gpu_processes():
            sys.exit(f"stopped before job {i}: other GPU processes appeared:\n{procs}")
        state, t0 = gpu_state(), time.time()
        cmd, env = command(j, run.path, 29700 + i % 100)
        with open(run.path / f"{j.tag}.log", "w") as log:
            rc = subprocess.run(cmd, stdout=log, stderr=subprocess.STDOUT, env=env, cwd=ROOT).returncode
        run.schedule(i, j.tag, t0, time.time() - t0, rc, state, env=j.env, variant=j.variant, ngpus=j.ngpus,
                     gpuset=j.gpuset, rep=j.rep)
        print(f"[{i + 1}/{len(jobs)}] {j.tag} rc={rc} {time.time() - t0:.1f}s", file=sys.stderr, flush=True)
    return run.path


def collective_baseline_jobs(gpus=(2, 4, 8), reps: int = 1) -> list[Job]:
    """The M0 baseline: six collectives x sizes x GPU counts, graph mode as nccl-tests -G 20."""
    return [Job("collectives", g, rep=r, args=("--begin", "8", "--end", "256M", "--graph", "20")) for g in gpus
            for r in range(reps)]


def nccl_variant_jobs(ngpus: int = 8) -> list[Job]:
    """The M7 "where slow" idea on NCCL knobs available here: algorithm / protocol / NVLS on and off."""
    variants = {"default": {}, "nvls_off": {"NCCL_NVLS_ENABLE": "0"}, "ll": {"NCCL_PROTO": "LL"},
                "ll128": {"NCCL_PROTO": "LL128"}, "ring": {"NCCL_ALGO": "Ring"}, "tree": {"NCCL_ALGO": "Tree"}}
    return [Job("collectives", ngpus, variant=k, env=v, args=("--colls", "all_reduce", "--begin", "1K", "--end", "8M",
                                                               "--graph", "20")) for k, v in variants.items()]


def repeat_jobs(reps: int = 5) -> list[Job]:
    """The reference's M4 study (exp/M4_repeat/run.py:14-26): the collective baseline's notable points
    repeated in independent launches on two GPU sets, so that a phenomenon counts only when the [min, max]
    intervals of both sets agree. (collective, GPU counts, size range)."""
    plan = [("sendrecv", (2, 4, 8), "4M", "256M"), ("alltoall", (2, 8), "64M", "4G"),
            ("all_gather", (2, 8), "1M", "4G"), ("reduce_scatter", (2, 8), "1M", "4G"),
            ("all_reduce", (2, 8), "1M", "4G"), ("broadcast", (2, 8), "1M", "2G")]
    return [Job("collectives", g, gpuset=gs, rep=r, variant=c,
                args=("--colls", c, "--begin", lo, "--end", hi))
            for c, gs_counts, lo, hi in plan for g in gs_counts for gs in ("A", "B") for r in range(reps)]


def p2p_channel_jobs(reps: int = 5) -> list[Job]:
    """The reference's M2 study (exp/M2_p2p_channels/run.py:14-30) on NCCL's P2P knobs: point-to-point and
    all-to-all from 1 MB to 1 GB at 8 GPUs with more P2P channels and smaller NVLink chunks, and the same
    chunk sizes at 2 GPUs (does a smaller chunk hurt the 2-GPU case)."""
    variants = {"default": {}, "minp2p64": {"NCCL_MIN_P2P_NCHANNELS": "64"},
                "chunk128k": {"NCCL_P2P_NVL_CHUNKSIZE": "131072"}, "chunk64k": {"NCCL_P2P_NVL_CHUNKSIZE": "65536"},
                "minp2p64_chunk128k": {"NCCL_MIN_P2P_NCHANNELS": "64", "NCCL_P2P_NVL_CHUNKSIZE": "131072"}}
    jobs = [Job("collectives", 8, rep=r, variant=f"{c}_{v}", env=e, args=("--colls", c, "--begin", "1M", "--end", "1G"))
            for v, e in variants.items() for c in ("sendrecv", "alltoall") for r in range(reps)]
    jobs += [Job("collectives", 2, rep=r, variant=f"sendrecv_{v}", env=variants[v],
                 args=("--colls", "sendrecv", "--begin", "1M", "--end", "1G"))
             for v in ("default", "chunk128k", "chunk64k") for r in range(reps)]
    return jobs


def headline_jobs(gpus=(2, 4, 8), batches=(1, 8, 32, 128)) -> list[Job]:
    """Every headline measurement of the project as independent jobs: the fused-op sweep against all
    baselines (hidden 8192 bf16, and the reference's fp16 hidden 5120), the layer-boundary bench, and the TP decode (fused / separate boundaries / NCCL baseline
    step) at each GPU count, the 70B decode batch sweep at 8 GPUs, and the 8B decode (prompt 1024, batch
    1 / 8 / 64) against the NCCL step at each GPU count."""
    sweep_impls = ("ours:auto,ours:lamport_1s,ours:lamport_2s,ours:pull_1s,ours:pull_2s,ours:nvls_1s,"
                   "ours:nvls_2s,nccl_norm,vllm_car,trt_oneshot,trt_twoshot")  # lamport_1sx: the validate plan
    jobs = []
    for g in gpus:
        jobs.append(Job("fused_sweep", g, args=("--impls", sweep_impls + (",ref_m16nf" if g == 8 else ""),
                                                "--replays", "20")))
        # the reference's own quoting configuration: fp16, hidden 5120, 10 KB - 1.25 MB
        jobs.append(Job("fused_sweep", g, variant="h5120_fp16",
                        args=("--impls", sweep_impls + (",ref_m16nf" if g == 8 else ""), "--hidden", "5120",
                              "--dtype", "float16", "--tokens", "1,2,4,8,16,32,64,128", "--replays", "20")))
        jobs.append(Job("boundary", g))
        for variant, extra in (("fused", ()), ("separate", ("--fuse-boundary", "0")),
                               ("nccl", ("--collective", "nccl")), ("vllm", ("--collective", "vllm"))):
            jobs.append(Job("bench", g, variant=variant, args=("--steps", "64", "--warmup", "4", *extra)))
    for B in batches:
        if B != 8:
            jobs.append(Job("bench", max(gpus), variant=f"b{B}", args=("--steps", "32", "--warmup", "3",
                                                                       "--batch", str(B))))
    # Llama-3-8B shapes at every GPU count: prompt 1024, batch 1 / 8 / 64, ours and the NCCL step
    for g in gpus:
        for B in (1, 8, 64):
            for variant, extra in (("8b", ()), ("8b_nccl", ("--collective", "nccl"))):
                jobs.append(Job("bench", g, variant=f"{variant}_b{B}",
                                args=("--model", "8b", "--prompt", "1024", "--batch", str(B), "--steps", "64",
                                      "--warmup", "4", *extra)))
    return jobs


def validate_jobs(gpus=(2, 4, 8)) -> list[Job]:
    """First runs of what was written without a GPU at hand (the kernels' own one-GPU tests run with
    `COB_EXPERIMENTAL=1 pytest -m gpu`): the multi-GPU self-test parts that cover them, the one-shot with
    and without the cluster row-sum exchange against the two-shot forms and FlashInfer's one-shot, and
    the decode bench with the L2 weight prefetch and the boundary choice switched on and off."""
    exp = {"COB_EXPERIMENTAL": "1"}
    jobs = [Job("selftest", 2, variant="experimental", env=exp,
                args=("--parts", "functional,stress,decode_mixed,decode_qkv_bias,decode_hd64,decode_vllm")),
            Job("selftest", 4, variant="kv_replicated", env=exp, args=("--parts", "decode_hd64,decode_mixed"))]
    impls = "ours:lamport_1s,ours:lamport_1sx,ours:lamport_2s,ours:pull_2s,ours:nvls_2s,trt_oneshot,trt_twoshot"
    for g in gpus:
        jobs.append(Job("fused_sweep", g, variant="experimental", env=exp, args=("--impls", impls, "--replays", "20")))
        # the attention-output boundary at Llama-70B shapes (o_proj -> all-reduce + RMSNorm -> gate_up), the
        # kind the whole-step measurement points at; the MLP-output boundary is the bench's default shape
        jobs.append(Job("boundary", g, variant="attn_out", args=("--k1", str(8192 // g), "--n2",
                                                                  str(2 * 28672 // g))))
    top = max(gpus)
    for variant, extra in (("default", ()), ("no_tuning", ("--tune-boundaries", "0")),
                           ("l2pf8", ("--l2-prefetch", "8")), ("l2pf16", ("--l2-prefetch", "16"))):
        jobs.append(Job("bench", top, variant=variant, args=("--steps", "64", "--warmup", "4", *extra)))
    jobs.append(Job("bench", 1, variant="l2pf8", args=("--steps", "32", "--warmup", "3", "--l2-prefetch", "8")))
    return jobs


def e2e_share_jobs(ngpus: int = 8, reps: int = 3) -> list[Job]:
    """The reference's M5 matrix (exp/M5_e2e_comm_share/run_train.py:14-16 and run_infer.py): training of
    Llama-3 1B / 8B at TP 8 / 4 / 2 x FSDP ngpus / TP, 8 x 2048 tokens per step, `reps` launches each; and
    the communication share of TP decode (70B, batch 1 / 8 / 128, fused and separate layer boundaries;
    Qwen2.5-32B and TinyLlama-1.1B shapes, prompt 128, batch 1 / 8 / 32 / 128)."""
    jobs = [Job("train_share", ngpus, variant=f"{m}_tp{tp}", rep=r, timeout_s=1800,
                args=("--model", m, "--tp", str(tp), "--seq", "2048", "--global-seqs", "8", "--steps", "10",
                      "--profile", "5"))
            for m in ("1b", "8b") for tp in (8, 4, 2) if tp <= ngpus for r in range(reps)]
    for B in (1, 8, 128):
        for fb in (1, 0):
            jobs.append(Job("comm_share", ngpus, variant=f"70b_b{B}_fb{fb}",
                            args=("--model", "70b", "--batch", str(B), "--fuse-boundary", str(fb))))
    # the reference's own decode matrix on its models' shapes (exp/M5_e2e_comm_share/run_infer.py:14-19:
    # Qwen2.5-32B and TinyLlama-1.1B, decode:<batch>:128 for batch 1 / 8 / 32 / 128)
    for B in (1, 8, 32, 128):
        for model, tag in (("qwen2.5-32b", "qwen32b"), ("tinyllama-1.1b", "tinyllama")):
            jobs.append(Job("comm_share", ngpus, variant=f"{tag}_b{B}",
                            args=("--model", model, "--batch", str(B), "--prompt", "128")))
    return jobs


def fused_hidden_jobs(ngpus: int = 8, impls: str = "ours:auto,vllm_car,trt_oneshot") -> list[Job]:
    """The reference's M10 question (exp/M10_why_fused_slow/run.py:24-42): the same message bytes at
    narrower rows (hidden 8192 / 4096 / 2048 / 1024 with 1x / 2x / 4x / 8x the tokens), and its register-limit
    check: hidden 6400 / 6656, where the TRT-LLM fused kernel stopped launching on A100."""
    base = (1, 2, 4, 8, 16, 32, 64)
    jobs = [Job("fused_sweep", ngpus, variant=f"h{8192 // k}",
                args=("--hidden", str(8192 // k), "--tokens", ",".join(str(t * k) for t in base), "--impls", impls,
                      "--replays", "20"))
            for k in (1, 2, 4, 8)]
    jobs += [Job("fused_sweep", ngpus, variant=f"h{h}", args=("--hidden", str(h), "--tokens", ",".join(map(str, base)),
                                                              "--impls", impls, "--replays", "20"))
             for h in (6400, 6656)]
    return jobs


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("plan", choices=["collective_baseline", "nccl_variants", "fused_hidden", "headline", "e2e_share",
                                     "repeat", "p2p_channels", "validate"])
    ap.add_argument("--gpus", default="2,4,8")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args()
    gp = tuple(int(g) for g in a.gpus.split(","))
    jobs = {"collective_baseline": lambda: collective_baseline_jobs(gp), "nccl_variants": lambda: nccl_variant_jobs(max(gp)),
            "fused_hidden": lambda: fused_hidden_jobs(max(gp)), "headline": lambda: headline_jobs(gp),
            "e2e_share": lambda: e2e_share_jobs(max(gp)), "repeat": repeat_jobs,
            "p2p_channels": p2p_channel_jobs, "validate": lambda: validate_jobs(gp)}[a.plan]()
    print(run_all(jobs, a.plan, a.seed))

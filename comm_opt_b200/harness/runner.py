"""Experiment runner: each measurement is an independent torchrun launch, described by a `Launch`
record, executed in a seeded pseudo-random order and written to ``results/<plan>/<timestamp>/``
(env.txt, schedule.tsv, one output per launch).

Design (the reference drives nccl-tests binaries from exp/lib/ncclrun.py:18-106; this runner drives the
package's own torchrun entry points):

* order: launches are sorted by a keyed hash of (seed, name), so the order is reproducible from the
  seed alone, independent of plan-list order, and different seeds interleave differently;
* placement: ``low`` puts rank r on device r; ``mirror`` puts rank r on device (count - 1 - r), i.e.
  the highest-numbered devices in reverse order - a second physical placement for the repeat study
  (a result that holds under only one placement is about those GPUs, not the method);
* quiet-GPU guard: before every launch NVML is asked for compute processes on the devices the
  launch will use; a process that is not a child of this runner stops the plan (numbers measured
  beside someone else's job are not kept, and their job is not disturbed);
* ledger: every finished launch appends one line to schedule.tsv; a re-run of the plan into the same
  directory (``--resume <dir>``) skips launches whose output file already exists.

    from comm_opt_b200.harness.runner import Launch, execute
    plan = [Launch("collectives", 8, repeat=r, argv=("--colls", "all_reduce")) for r in range(3)]
    execute(plan, "collective_baseline", seed=0)        # DRY_RUN=1 prints the commands only
"""
from __future__ import annotations

import hashlib
import os
import shlex
import subprocess
import sys
import time
from dataclasses import dataclass, field
from pathlib import Path

from ..utils.results import ROOT, RunDir, gpu_state

# torchrun targets: a module path, or a script at the repository root (ends in .py)
TARGETS = {
    "collectives": "comm_opt_b200.harness.collectives",
    "fused_sweep": "comm_opt_b200.harness.fused_sweep",
    "selftest": "comm_opt_b200.harness.mp_selftest",
    "bakeoff": "comm_opt_b200.harness.allreduce_bakeoff",
    "phases": "comm_opt_b200.harness.phase_profile",
    "boundary": "comm_opt_b200.harness.boundary_bench",
    "comm_share": "comm_opt_b200.harness.comm_share",
    "train_share": "comm_opt_b200.harness.train_share",
    "probes": "comm_opt_b200.harness.probes",
    "bench": "bench.py",
}
PLACEMENTS = ("low", "mirror")
BASE_PORT = 29700


def placement_devices(world: int, placement: str = "low", count: int = 8) -> list[int]:
    """Physical devices of ranks 0..world-1 on a node with `count` GPUs."""
    if world > count:
        raise ValueError(f"{world} ranks on a {count}-GPU node")
    if placement == "low":
        return list(range(world))
    if placement == "mirror":
        return [count - 1 - r for r in range(world)]
    raise ValueError(f"unknown placement {placement!r}")


@dataclass(frozen=True)
class Launch:
    target: str                      # key of TARGETS
    world: int                       # ranks (one GPU each)
    placement: str = "low"           # see placement_devices
    repeat: int = 0                  # index of an independent repetition
    label: str = "default"           # what distinguishes launches of the same target and world
    env: dict = field(default_factory=dict, hash=False)
    argv: tuple = ()
    limit_s: int = 1500              # hard limit of the whole torchrun process tree

    @property
    def name(self) -> str:
        return f"{self.target}.w{self.world}.{self.placement}.{self.label}.{self.repeat}"

    def order_key(self, seed: int) -> str:
        return hashlib.sha256(f"{seed}:{self.name}".encode()).hexdigest()


def ordered(plan: list[Launch], seed: int) -> list[Launch]:
    names = [l.name for l in plan]
    dup = {n for n in names if names.count(n) > 1}
    if dup:
        raise ValueError(f"launch names must be unique: {sorted(dup)}")
    return sorted(plan, key=lambda l: l.order_key(seed))


def foreign_gpu_pids(devices: list[int]) -> list[tuple[int, int, int]]:
    """(device, pid, MiB) of compute processes on `devices` that are not this process or its children.
    Empty when NVML cannot be read (no driver here: nothing to protect)."""
    try:
        import pynvml
    except ImportError:
        return []
    try:
        pynvml.nvmlInit()
    except pynvml.NVMLError:
        return []
    mine = {os.getpid()}
    try:
        import psutil

        mine |= {c.pid for c in psutil.Process().children(recursive=True)}
    except Exception:
        pass
    found = []
    try:
        for d in devices:
            h = pynvml.nvmlDeviceGetHandleByIndex(d)
            for p in pynvml.nvmlDeviceGetComputeRunningProcesses(h):
                if p.pid not in mine:
                    found.append((d, p.pid, (p.usedGpuMemory or 0) >> 20))
    except pynvml.NVMLError:
        pass
    finally:
        pynvml.nvmlShutdown()
    return found


def _output_args(launch: Launch, out: Path) -> list[str]:
    """Where each target writes its result inside the run directory."""
    if launch.target == "collectives":
        return ["--out", str(out / f"{launch.name}.json")]
    if launch.target == "fused_sweep":
        return ["--out-dir", str(out / "runs"), "--ts", launch.name]
    if launch.target in ("bakeoff", "phases", "boundary"):
        return ["--out-dir", str(out / "runs")]
    if launch.target == "probes":
        return ["--out", str(out / f"{launch.name}.json")]
    if launch.target in ("comm_share", "train_share"):
        return ["--out-dir", str(out / "runs" / launch.name)]
    if launch.target == "bench":
        return ["--gpus", str(launch.world), "--out", str(out / f"{launch.name}.json")]
    return []


def compose(launch: Launch, out: Path, port: int) -> tuple[list[str], dict]:
    """Command line and environment of one launch (rendezvous on 127.0.0.1)."""
    devices = placement_devices(launch.world, launch.placement)
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = ",".join(map(str, devices))
    if launch.target == "collectives":
        # NCCL's set-up (version, channels, NVLS, rings) once per communicator, no per-call lines
        env.update(NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="INIT,ENV,GRAPH",
                   NCCL_DEBUG_FILE=str(out / f"{launch.name}.nccl.%h.%p.log"))
        env.update({k: v for k, v in os.environ.items() if k in ("NCCL_DEBUG", "NCCL_DEBUG_SUBSYS")})
    env.update(launch.env)  # the launch's own settings win
    tgt = TARGETS[launch.target]
    entry = [str(ROOT / tgt)] if tgt.endswith(".py") else ["-m", tgt]
    cmd = ["timeout", "-k", "60", str(launch.limit_s), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={launch.world}", "--master-addr=127.0.0.1",
           f"--master-port={port}", *entry, *launch.argv, *_output_args(launch, out)]
    return cmd, env


def execute(plan: list[Launch], name: str, seed: int, base: Path | None = None,
            resume: Path | None = None) -> Path | None:
    """Run `plan` in seeded order; returns the run directory (None for a dry run)."""
    todo = ordered(plan, seed)
    if os.environ.get("DRY_RUN"):
        for i, l in enumerate(todo):
            print(shlex.join(compose(l, Path("results") / name / "DRY", BASE_PORT + i % 100)[0]))
        print(f"dry run of plan {name!r}: {len(todo)} launches (order seed {seed})", file=sys.stderr)
        return None
    run = RunDir(name, base) if resume is None else RunDir.at(Path(resume))
    if resume is None:
        run.snapshot()
        (run.path / "seed.txt").write_text(f"{seed}\n")
    for i, l in enumerate(todo):
        if run.done(f"{l.name}.log"):
            continue
        busy = foreign_gpu_pids(placement_devices(l.world, l.placement))
        if busy:
            listing = ", ".join(f"GPU {d}: pid {p} ({m} MiB)" for d, p, m in busy)
            sys.exit(f"plan {name!r} halted at launch {i} ({l.name}): other compute processes found ({listing}); "
                     f"finished launches are in {run.path}")
        before, t0 = gpu_state(), time.time()
        cmd, env = compose(l, run.path, BASE_PORT + i % 100)
        with open(run.path / f"{l.name}.log", "w") as log:
            rc = subprocess.run(cmd, stdout=log, stderr=subprocess.STDOUT, env=env, cwd=ROOT).returncode
        took = time.time() - t0
        run.schedule(i, l.name, t0, took, rc, before, variant=l.label, ngpus=l.world, placement=l.placement,
                     gpuset="A" if l.placement == "low" else "B", rep=l.repeat)
        status = "ok" if rc == 0 else f"exit {rc}"
        print(f"{name} {i + 1}/{len(todo)} {l.name}: {status} after {took:.0f} s", file=sys.stderr, flush=True)
    return run.path


# ------------------------------------------------------------------------------------------- plans
def collective_baseline_plan(worlds=(2, 4, 8), repeats: int = 1) -> list[Launch]:
    """Six collectives, 8 B - 256 MB, 20 ops per CUDA graph (nccl-tests' -G 20), at each world size
    (the reference's M0 baseline, exp/M0_baseline)."""
    return [Launch("collectives", w, repeat=r, argv=("--begin", "8", "--end", "256M", "--graph", "20"))
            for w in worlds for r in range(repeats)]


def nccl_variant_plan(world: int = 8) -> list[Launch]:
    """All-reduce 1 KB - 8 MB under NCCL's algorithm / protocol / NVLS switches (the M7 question: where
    is NCCL slow, and which of its own choices would have been faster)."""
    knobs = {"default": {}, "nvls_off": {"NCCL_NVLS_ENABLE": "0"}, "ll": {"NCCL_PROTO": "LL"},
             "ll128": {"NCCL_PROTO": "LL128"}, "ring": {"NCCL_ALGO": "Ring"}, "tree": {"NCCL_ALGO": "Tree"}}
    return [Launch("collectives", world, label=k, env=v,
                   argv=("--colls", "all_reduce", "--begin", "1K", "--end", "8M", "--graph", "20"))
            for k, v in knobs.items()]


def repeat_plan(repeats: int = 5) -> list[Launch]:
    """Notable points of the collective baseline repeated in independent launches under both placements
    (the reference's M4 study, exp/M4_repeat/run.py:14-26): a phenomenon counts only when the
    [min, max] intervals agree across placements. (collective, world sizes, size range)."""
    points = [("sendrecv", (2, 4, 8), "4M", "256M"), ("alltoall", (2, 8), "64M", "4G"),
              ("all_gather", (2, 8), "1M", "4G"), ("reduce_scatter", (2, 8), "1M", "4G"),
              ("all_reduce", (2, 8), "1M", "4G"), ("broadcast", (2, 8), "1M", "2G")]
    return [Launch("collectives", w, placement=pl, repeat=r, label=c, argv=("--colls", c, "--begin", lo, "--end", hi))
            for c, worlds, lo, hi in points for w in worlds for pl in PLACEMENTS for r in range(repeats)]


def p2p_channel_plan(repeats: int = 5) -> list[Launch]:
    """NCCL's P2P knobs (the reference's M2 study, exp/M2_p2p_channels/run.py:14-30): point-to-point and
    all-to-all, 1 MB - 1 GB, at 8 GPUs with more P2P channels and smaller NVLink chunks, and the chunk
    sizes alone at 2 GPUs (does a smaller chunk hurt the 2-GPU case)."""
    knobs = {"default": {}, "minp2p64": {"NCCL_MIN_P2P_NCHANNELS": "64"},
             "chunk128k": {"NCCL_P2P_NVL_CHUNKSIZE": "131072"}, "chunk64k": {"NCCL_P2P_NVL_CHUNKSIZE": "65536"},
             "minp2p64_chunk128k": {"NCCL_MIN_P2P_NCHANNELS": "64", "NCCL_P2P_NVL_CHUNKSIZE": "131072"}}
    plan = [Launch("collectives", 8, repeat=r, label=f"{c}_{k}", env=v, argv=("--colls", c, "--begin", "1M", "--end", "1G"))
            for k, v in knobs.items() for c in ("sendrecv", "alltoall") for r in range(repeats)]
    plan += [Launch("collectives", 2, repeat=r, label=f"sendrecv_{k}", env=knobs[k],
                    argv=("--colls", "sendrecv", "--begin", "1M", "--end", "1G"))
             for k in ("default", "chunk128k", "chunk64k") for r in range(repeats)]
    return plan


SWEEP_IMPLS = ("ours:auto,ours:lamport_1s,ours:lamport_2s,ours:pull_1s,ours:pull_2s,ours:nvls_1s,"
               "ours:nvls_2s,nccl_norm,vllm_car,trt_oneshot,trt_twoshot")


def headline_plan(worlds=(2, 4, 8), batches=(1, 8, 32, 128)) -> list[Launch]:
    """Every headline measurement as independent launches: the fused-op sweep against all baselines
    (hidden 8192 bf16, and the reference's own fp16 hidden 5120 quoting shape), the layer-boundary bench,
    the 70B TP decode in four forms (fused and separate boundaries, the NCCL and the vLLM baseline stacks)
    at each world size, the 70B batch sweep at the largest world in the same four forms, and the 8B decode
    (prompt 1024, batch 1 / 8 / 64) against the NCCL step at each world size."""
    plan: list[Launch] = []
    forms = (("fused", ()), ("separate", ("--fuse-boundary", "0")), ("nccl", ("--collective", "nccl")),
             ("vllm", ("--collective", "vllm")))
    for w in worlds:
        ref = ",ref_m16nf" if w == 8 else ""
        plan.append(Launch("fused_sweep", w, argv=("--impls", SWEEP_IMPLS + ref, "--replays", "20")))
        plan.append(Launch("fused_sweep", w, label="h5120_fp16",
                           argv=("--impls", SWEEP_IMPLS + ref, "--hidden", "5120", "--dtype", "float16",
                                 "--tokens", "1,2,4,8,16,32,64,128", "--replays", "20")))
        plan.append(Launch("boundary", w))
        for label, extra in forms:
            plan.append(Launch("bench", w, label=label, argv=("--steps", "64", "--warmup", "4", *extra)))
    top = max(worlds)
    for B in batches:
        if B == 8:
            continue
        for label, extra in forms:
            plan.append(Launch("bench", top, label=f"b{B}_{label}",
                               argv=("--steps", "32", "--warmup", "3", "--batch", str(B), *extra)))
    for w in worlds:
        for B in (1, 8, 64):
            for label, extra in (("8b", ()), ("8b_nccl", ("--collective", "nccl"))):
                plan.append(Launch("bench", w, label=f"{label}_b{B}",
                                   argv=("--model", "8b", "--prompt", "1024", "--batch", str(B), "--steps", "64",
                                         "--warmup", "4", *extra)))
    return plan


def validate_plan(worlds=(2, 4, 8)) -> list[Launch]:
    """First multi-GPU runs of code written without a GPU (its one-GPU tests run with
    `COB_EXPERIMENTAL=1 pytest -m gpu`): the self-test parts that cover it, the one-shot with and without
    the cluster row-sum exchange against the two-shot forms and FlashInfer's one-shot, the attention-output
    boundary, and the decode bench with the L2 weight prefetch and the boundary choice on and off."""
    exp = {"COB_EXPERIMENTAL": "1"}
    plan = [Launch("selftest", 2, label="experimental", env=exp,
                   argv=("--parts", "functional,stress,decode_mixed,decode_qkv_bias,decode_hd64,decode_vllm")),
            Launch("selftest", 4, label="kv_replicated", env=exp, argv=("--parts", "decode_hd64,decode_mixed"))]
    impls = "ours:lamport_1s,ours:lamport_1sx,ours:lamport_2s,ours:pull_2s,ours:nvls_2s,trt_oneshot,trt_twoshot"
    for w in worlds:
        plan.append(Launch("fused_sweep", w, label="experimental", env=exp, argv=("--impls", impls, "--replays", "20")))
        # attention-output boundary at Llama-70B shapes: o_proj -> all-reduce + RMSNorm -> gate_up
        plan.append(Launch("boundary", w, label="attn_out", argv=("--k1", str(8192 // w), "--n2", str(2 * 28672 // w))))
    top = max(worlds)
    for label, extra in (("default", ()), ("no_tuning", ("--tune-boundaries", "0")),
                         ("l2pf8", ("--l2-prefetch", "8")), ("l2pf16", ("--l2-prefetch", "16"))):
        plan.append(Launch("bench", top, label=label, argv=("--steps", "64", "--warmup", "4", *extra)))
    plan.append(Launch("bench", 1, label="l2pf8", argv=("--steps", "32", "--warmup", "3", "--l2-prefetch", "8")))
    return plan


def e2e_share_plan(world: int = 8, repeats: int = 3) -> list[Launch]:
    """Communication share end to end (the reference's M5 matrix, exp/M5_e2e_comm_share/run_train.py:14-16
    and run_infer.py): training of Llama-3 1B / 8B at TP 8 / 4 / 2 x FSDP world / TP, 8 x 2048 tokens per
    step; TP decode of the 70B (batch 1 / 8 / 128, fused and separate boundaries); and the reference's
    own decode matrix on its models' shapes (Qwen2.5-32B, TinyLlama-1.1B; prompt 128, batch 1-128)."""
    plan = [Launch("train_share", world, label=f"{m}_tp{tp}", repeat=r, limit_s=1800,
                   argv=("--model", m, "--tp", str(tp), "--seq", "2048", "--global-seqs", "8", "--steps", "10",
                         "--profile", "5"))
            for m in ("1b", "8b") for tp in (8, 4, 2) if tp <= world for r in range(repeats)]
    for B in (1, 8, 128):
        for fb in (1, 0):
            plan.append(Launch("comm_share", world, label=f"70b_b{B}_fb{fb}",
                               argv=("--model", "70b", "--batch", str(B), "--fuse-boundary", str(fb))))
    for B in (1, 8, 32, 128):
        for model, tag in (("qwen2.5-32b", "qwen32b"), ("tinyllama-1.1b", "tinyllama")):
            plan.append(Launch("comm_share", world, label=f"{tag}_b{B}",
                               argv=("--model", model, "--batch", str(B), "--prompt", "128")))
    return plan


def fused_hidden_plan(world: int = 8, impls: str = "ours:auto,vllm_car,trt_oneshot") -> list[Launch]:
    """The M10 question (exp/M10_why_fused_slow/run.py:24-42): the same message bytes at narrower rows
    (hidden 8192 / 4096 / 2048 / 1024 with 1x / 2x / 4x / 8x the tokens), and hidden 6400 / 6656, where the
    TRT-LLM fused kernel stopped launching on A100 (register limit)."""
    base = (1, 2, 4, 8, 16, 32, 64)
    plan = [Launch("fused_sweep", world, label=f"h{8192 // k}",
                   argv=("--hidden", str(8192 // k), "--tokens", ",".join(str(t * k) for t in base), "--impls", impls,
                         "--replays", "20"))
            for k in (1, 2, 4, 8)]
    plan += [Launch("fused_sweep", world, label=f"h{h}",
                    argv=("--hidden", str(h), "--tokens", ",".join(map(str, base)), "--impls", impls, "--replays", "20"))
             for h in (6400, 6656)]
    return plan


def calibrate_validate_plan(worlds=(2, 8), repeats: int = 3, hiddens=(8192, 5120, 4096),
                            dtypes=("bfloat16", "float16")) -> list[Launch]:
    """Sweeps of every variant plus ours:auto per (world, hidden, dtype), `repeats` independent launches
    each. Calibrate: `analyze_sweep --calibrate` over one run of this plan writes the variant table.
    Validate: run the plan again (fresh launches reading the new table) and `analyze_sweep --validate`
    over its sweeps applies the >= 3 % / disjoint-interval rule to ours:auto against every variant."""
    impls = "ours:auto,ours:lamport_1s,ours:lamport_1sx,ours:lamport_2s,ours:pull_1s,ours:pull_2s,ours:nvls_1s,ours:nvls_2s"
    plan = []
    for w in worlds:
        for h in hiddens:
            for dt in dtypes:
                for r in range(repeats):
                    plan.append(Launch("fused_sweep", w, repeat=r, label=f"h{h}_{dt}", env={"COB_EXPERIMENTAL": "1"},
                                       argv=("--impls", impls, "--hidden", str(h), "--dtype", dt,
                                             "--tokens", "1,2,4,8,16,32,64,128,256,512", "--replays", "20")))
    return plan


def primitives_plan(worlds=(2, 4, 8)) -> list[Launch]:
    """Which NVLink primitive wins where (the reference's M11 / M12-M13 / M8 probes, re-asked on B200):
    the reduce-scatter by remote vector atomics, push vs pull all-gather / reduce-scatter in steady state
    (with the NVSwitch multicast forms), and the 128-byte line premise, at each world size."""
    plan = []
    for w in worlds:
        plan.append(Launch("probes", w, label="rs_atomic", argv=("--sizes", "81920,327680,1310720")))
        plan.append(Launch("probes", w, label="prim", argv=("--prim", "--sizes", "81920,327680,1310720")))
        plan.append(Launch("probes", w, label="line", argv=("--line", "--lines", str(1 << 18))))
    return plan


PLANS = {
    "collective_baseline": lambda w: collective_baseline_plan(w),
    "nccl_variants": lambda w: nccl_variant_plan(max(w)),
    "fused_hidden": lambda w: fused_hidden_plan(max(w)),
    "headline": lambda w: headline_plan(w),
    "e2e_share": lambda w: e2e_share_plan(max(w)),
    "repeat": lambda w: repeat_plan(),
    "p2p_channels": lambda w: p2p_channel_plan(),
    "validate": lambda w: validate_plan(w),
    "primitives": lambda w: primitives_plan(w),
    "calibrate_validate": lambda w: calibrate_validate_plan(w),
}


def main(argv=None):
    import argparse

    ap = argparse.ArgumentParser(description="run a measurement plan as independent torchrun launches")
    ap.add_argument("plan", choices=sorted(PLANS))
    ap.add_argument("--gpus", default="2,4,8", help="world sizes of the plan")
    ap.add_argument("--seed", type=int, default=0, help="order seed")
    ap.add_argument("--resume", default=None, help="finish a previous run of the same plan in this directory")
    a = ap.parse_args(argv)
    worlds = tuple(int(g) for g in a.gpus.split(","))
    print(execute(PLANS[a.plan](worlds), a.plan, a.seed, resume=Path(a.resume) if a.resume else None))


if __name__ == "__main__":
    main()

"""Harness pieces on CPU: collective sweep over gloo, runner dry run, loaders and statistics."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT, free_port


def test_collectives_gloo_two_ranks(tmp_path):
    out = tmp_path / "c.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={free_port()}", "-m", "comm_opt_b200.harness.collectives",
           "--device", "cpu", "--begin", "64", "--end", "4K", "--iters", "3", "--warmup", "1", "--out", str(out)]
    p = subprocess.run(["timeout", "-k", "10", "240"] + cmd, cwd=ROOT, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    doc = json.loads(out.read_text())
    colls = {r["coll"] for r in doc["results"]}
    assert colls == {"all_reduce", "all_gather", "reduce_scatter", "alltoall", "broadcast", "sendrecv"}
    assert all(r["nwrong"] == 0 for r in doc["results"])
    ar = [r for r in doc["results"] if r["coll"] == "all_reduce"]
    assert all(abs(r["busbw"] - r["algbw"] * 2 * (2 - 1) / 2) < 1e-9 for r in ar)


def test_runner_dry_run_prints_commands():
    env = dict(os.environ, DRY_RUN="1")
    code = ("from comm_opt_b200.harness.runner import *; execute(collective_baseline_plan((2, 8)), 'x', 3);"
            "execute(nccl_variant_plan(8), 'y', 4); execute(fused_hidden_plan(8), 'z', 5)")
    p = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stderr
    lines = [l for l in p.stdout.splitlines() if "torch.distributed.run" in l]
    assert len(lines) == 2 + 6 + 6 and all("127.0.0.1" in l and "timeout" in l for l in lines)
    assert sum("--hidden 1024" in l and "--tokens 8,16,32" in l for l in lines) == 1
    assert "dry run of plan 'x': 2 launches" in p.stderr


def test_runner_order_is_seeded_and_independent_of_list_order():
    from comm_opt_b200.harness.runner import Launch, ordered

    plan = [Launch("bench", 8, label=f"v{i}") for i in range(12)]
    a, b = ordered(plan, 1), ordered(list(reversed(plan)), 1)
    assert [l.name for l in a] == [l.name for l in b]
    assert [l.name for l in ordered(plan, 2)] != [l.name for l in a]
    with pytest.raises(ValueError):
        ordered(plan + [Launch("bench", 8, label="v0")], 0)


def test_runner_placements():
    from comm_opt_b200.harness.runner import Launch, compose, placement_devices

    assert placement_devices(2) == [0, 1] and placement_devices(2, "mirror") == [7, 6]
    assert placement_devices(8, "mirror") == list(range(7, -1, -1))
    with pytest.raises(ValueError):
        placement_devices(9)
    _, env = compose(Launch("bench", 4, placement="mirror"), ROOT / "results" / "x", 29999)
    assert env["CUDA_VISIBLE_DEVICES"] == "7,6,5,4"


def test_runner_resume_skips_finished_launches(tmp_path, monkeypatch):
    """A launch whose log exists in the run directory is not run again; the others are, in seeded order,
    each recorded in schedule.tsv with its placement."""
    import comm_opt_b200.harness.runner as R

    ran = []

    def fake_run(cmd, stdout, stderr, env, cwd):
        ran.append(env["CUDA_VISIBLE_DEVICES"])
        return subprocess.CompletedProcess(cmd, 0)

    monkeypatch.setattr(R.subprocess, "run", fake_run)
    monkeypatch.setattr(R, "foreign_gpu_pids", lambda devices: [])
    monkeypatch.setattr(R, "gpu_state", lambda: "")
    (tmp_path / "r").mkdir()
    plan = [R.Launch("bench", 2, label="a"), R.Launch("bench", 2, placement="mirror", label="b")]
    (tmp_path / "r" / f"{plan[0].name}.log").write_text("done before")
    out = R.execute(plan, "p", 0, resume=tmp_path / "r")
    assert out == tmp_path / "r" and ran == ["7,6"]
    sched = (tmp_path / "r" / "schedule.tsv").read_text().splitlines()
    assert len(sched) == 2 and '"placement": "mirror"' in sched[1]


def test_runner_halts_beside_foreign_processes(tmp_path, monkeypatch):
    import comm_opt_b200.harness.runner as R

    monkeypatch.setattr(R, "foreign_gpu_pids", lambda devices: [(devices[0], 4242, 1000)])
    monkeypatch.setattr(R, "gpu_state", lambda: "")
    monkeypatch.setattr(R.subprocess, "run", lambda *a, **k: pytest.fail("must not launch"))
    (tmp_path / "r").mkdir()
    with pytest.raises(SystemExit, match="pid 4242"):
        R.execute([R.Launch("bench", 2)], "p", 0, resume=tmp_path / "r")


def test_runner_headline_plan():
    from comm_opt_b200.harness.runner import compose, headline_plan

    plan = headline_plan((2, 4, 8))
    # per world: 2 sweeps, boundary, 4 decode forms (fused, separate, NCCL stack, vLLM stack),
    # 8B x 3 batches x 2 collectives; 3 extra 70B batches at 8 in the same 4 forms
    assert len(plan) == 3 * (7 + 6) + 3 * 4
    cmds = [" ".join(compose(l, ROOT / "results" / "x", 29000 + i)[0]) for i, l in enumerate(plan)]
    assert sum("bench.py" in c and "--collective nccl" in c for c in cmds) == 3 + 3 + 9
    assert sum("bench.py" in c and "--collective vllm" in c for c in cmds) == 3 + 3
    assert sum("--model 8b --prompt 1024" in c for c in cmds) == 18
    assert all(("bench.py" in c) != (" -m comm_opt_b200" in c.split("torch.distributed.run")[1]) for c in cmds)
    assert sum("ref_m16nf" in c for c in cmds) == 2  # both sweeps at 8 GPUs
    assert sum("--hidden 5120 --dtype float16" in c for c in cmds) == 3


def test_collective_loader_and_bound(tmp_path):
    from comm_opt_b200.harness.collective_analysis import achievable_us, fit_bound, load_run, summarize
    from comm_opt_b200.utils.stats import disjoint

    for rep in range(3):
        doc = dict(results=[dict(coll="all_reduce", world=8, size=s, p50_us=5.0 + s / 1e5 + rep, busbw=s / 1e4 + rep,
                                 time_us=1.0) for s in (1024, 1 << 20)])
        (tmp_path / f"j{rep}.json").write_text(json.dumps(doc))
    rows = load_run(tmp_path)
    assert len(rows) == 6
    s = summarize(rows, ("coll", "world", "size"), "p50_us")
    m = s[("all_reduce", 8, 1024)]
    assert m["n"] == 3 and m["lo"] <= m["med"] <= m["hi"]
    assert not disjoint(s[("all_reduce", 8, 1024)], s[("all_reduce", 8, 1024)])
    l0, bw = fit_bound(rows)
    assert achievable_us(1 << 20, 8, l0, bw) > l0


def test_trace_decomposition(tmp_path):
    """Synthetic two-rank trace: comm kernel partly overlapped by compute; rank 1 waits longer."""
    from comm_opt_b200.harness.traces import decompose

    def trace(comm_dur):
        ev = [dict(cat="gpu_user_annotation", name="decode_step", ts=0, dur=100),
              dict(cat="kernel", name="k_gemm_streamk<16>", ts=0, dur=40),
              dict(cat="kernel", name="void k_oneshot<bf16, 8, 1>", ts=30, dur=comm_dur),
              dict(cat="kernel", name="k_decode_attn", ts=30 + comm_dur, dur=20)]
        return dict(traceEvents=ev)

    for r, d in enumerate((20, 30)):
        (tmp_path / f"trace_rank{r}.json").write_text(json.dumps(trace(d)))
    rows = decompose(sorted(tmp_path.glob("trace_rank*.json")), "decode_step")
    r0 = next(r for r in rows if r["rank"] == 0)
    assert abs(r0["overlap_us"] - 10) < 1e-6 and abs(r0["exposed_comm_us"] - 10) < 1e-6
    assert abs(r0["compute_only_us"] - (40 - 10 + 20)) < 1e-6
    assert abs(r0["idle_us"] - (100 - 70)) < 1e-6
    r1 = next(r for r in rows if r["rank"] == 1)
    assert r1["exposed_wait_us"] > 0 and abs(r1["exposed_transfer_us"] + r1["exposed_wait_us"] - r1["exposed_comm_us"]) < 1e-9


def test_phase_decomposition_from_stamps():
    """Synthetic stamps of 2 graph replays x 3 calls, 2 blocks: phases, inter-call gap within a replay."""
    import torch

    from comm_opt_b200.harness.phase_profile import decompose

    cap, blocks, ops = 16, 2, 3
    st = torch.zeros(cap, 160, 5, dtype=torch.int64)
    t = 1_000_000
    epochs = list(range(5, 11))
    for e in epochs:
        for b in range(blocks):
            st[e % cap, b] = torch.tensor([t + 100 * b, t + 500, 0, t + 3000, t + 4000 + 100 * b])
        t += 4100 + 900  # 0.9 us gap to the next call
    ph, starts = decompose(st, epochs, blocks, ops)
    assert abs(ph["sent"] - 0.5) < 1e-9 and abs(ph["received"] - 3.0) < 1e-9 and abs(ph["done"] - 4.1) < 1e-9
    assert ph["reduced"] is None  # phase not stamped by this variant
    assert abs(ph["gap"] - 0.9) < 1e-9 and len(starts) == 6


def test_bakeoff_shapes_and_runner_entries():
    from comm_opt_b200.harness.allreduce_bakeoff import shape_of
    from comm_opt_b200.harness.runner import TARGETS, Launch, compose

    assert shape_of(1024, 2) == (1, 512) and shape_of(8 << 20, 2) == (512, 8192) and shape_of(48 << 10, 2) == (3, 8192)
    for e in ("bakeoff", "phases", "collectives", "fused_sweep", "selftest", "probes"):
        assert e in TARGETS
    cmd, env = compose(Launch("bakeoff", 8), ROOT / "results" / "x", 29999)
    assert "--out-dir" in cmd and env["CUDA_VISIBLE_DEVICES"] == "0,1,2,3,4,5,6,7"


def test_report_tables(tmp_path):
    from comm_opt_b200.harness.report import render

    d = tmp_path / "b"
    d.mkdir()
    rows = [dict(impl=i, batch=B, p50_us=v, correct=True, error="", roofline_us=12.2, frac_of_roofline=12.2 / v)
            for B in (1, 8) for i, v in (("fused", 27.0), ("ours_split", 34.0))]
    (d / "boundary.json").write_text(json.dumps(dict(world=8, rows=rows)))
    t = render(d)
    assert "| 1 | 27.00 | 34.00 | 12.20 | 0.452 |" in t
    f = tmp_path / "bench.json"
    f.write_text(json.dumps(dict(metric="m", n_gpus=8, value=7.7, e2e=dict(value=7.74), kernels_per_step=566,
                                 config=dict(parallelism="tp8"))) + "\n" +
                 json.dumps(dict(impl="reference", unavailable="not installable")) + "\n")
    t = render(f)
    assert "| m | 8 | 7.700 | 7.740 | 566 | parallelism=tp8 |" in t and "unavailable: not installable" in t


def test_e2e_share_plan():
    """The M5 matrix: 1B / 8B x TP 8 / 4 / 2 x 3 launches of training, plus the decode comm-share jobs; each
    job writes its traces into its own directory."""
    from comm_opt_b200.harness.runner import Launch, compose, e2e_share_plan

    plan = e2e_share_plan(8)
    train = [l for l in plan if l.target == "train_share"]
    assert len(train) == 18 and {l.label for l in train} == {f"{m}_tp{t}" for m in ("1b", "8b") for t in (8, 4, 2)}
    share = [l for l in plan if l.target == "comm_share"]
    assert len(share) == 6 + 8 and {l.label for l in share if l.label.startswith("qwen32b")} == {
        f"qwen32b_b{b}" for b in (1, 8, 32, 128)}
    cmd, _ = compose(Launch("train_share", 8, label="8b_tp4"), ROOT / "results" / "x", 29999)
    assert cmd[-1].endswith("runs/train_share.w8.low.8b_tp4.0") and "comm_opt_b200.harness.train_share" in cmd
    assert len(e2e_share_plan(4, repeats=1)) == 4 + 6 + 8  # TP 8 needs 8 GPUs


def test_nccl_log_summary_and_gpuset_comparison(tmp_path):
    """NCCL's set-up read from an INIT / ENV / GRAPH log, attached to every row of the job; sets A and B
    compared per point over repeated launches."""
    from comm_opt_b200.harness.collective_analysis import compare_gpusets, load_run, nccl_log_summary

    log = ("h:1:1 [0] NCCL INFO NCCL version 2.28.9+cuda12.9\n"
           "h:1:1 [0] NCCL INFO NCCL_P2P_NVL_CHUNKSIZE set by environment to 131072\n"
           "h:1:1 [0] NCCL INFO comm 0x1 rank 0 nRanks 8 nNodes 1 localRanks 8 localRank 0 MNNVL 0\n"
           + "".join(f"h:1:1 [0] NCCL INFO Channel {c:02d}/24 :    0   1   2   3   4   5   6   7\n" for c in range(24))
           + "h:1:1 [0] NCCL INFO NVLS multicast support is available on dev 0 (NVLS_NCHANNELS 16)\n"
           "h:1:1 [0] NCCL INFO 24 coll channels, 24 collnet channels, 16 nvls channels, 32 p2p channels, "
           "32 p2p channels per peer\n")
    s = nccl_log_summary(log)
    assert s == dict(nccl_version="2.28.9+cuda12.9", nranks=8, coll_channels=24, nvls_channels=16, p2p_channels=32,
                     p2p_channels_per_peer=32, rings=24, nvls=True, env={"NCCL_P2P_NVL_CHUNKSIZE": "131072"})
    assert nccl_log_summary("nothing here") == {}
    from comm_opt_b200.utils.results import RunDir

    run = RunDir("repeat", tmp_path, "t")
    for i, (gs, rep) in enumerate((g, r) for g in "AB" for r in range(3)):
        tag = f"collectives_g8{gs}_all_reduce_r{rep}"
        bw = (100.0 if gs == "A" else 104.0) + rep
        (run.path / f"{tag}.json").write_text(json.dumps(dict(results=[
            dict(coll="all_reduce", world=8, size=1 << 20, busbw=bw, p50_us=10.0)])))
        run.schedule(i, tag, 0.0, 1.0, 0, "", variant="all_reduce", gpuset=gs, rep=rep)
        if i == 0:
            (run.path / f"{tag}.nccl.h.1.log").write_text(log)
    rows = load_run(run.path)
    assert len(rows) == 6 and rows[0]["nccl"]["coll_channels"] == 24 and rows[1]["nccl"] == {}
    (c,) = compare_gpusets(rows)
    assert c["a"]["med"] == 101.0 and c["b"]["med"] == 105.0 and c["disjoint"] and abs(c["rel_diff"] - 4 / 101) < 1e-12


def test_repeat_and_p2p_channel_plans():
    from comm_opt_b200.harness.runner import Launch, compose, p2p_channel_plan, repeat_plan

    rp = repeat_plan(5)
    assert len(rp) == (3 + 2 * 5) * 2 * 5 and {l.placement for l in rp} == {"low", "mirror"}
    pp = p2p_channel_plan(5)
    assert len(pp) == 5 * 2 * 5 + 3 * 5
    assert any(l.env.get("NCCL_MIN_P2P_NCHANNELS") == "64" for l in pp)
    cmd, env = compose(Launch("collectives", 8, env={"NCCL_DEBUG": "WARN"}), ROOT / "results" / "x", 29999)
    assert env["NCCL_DEBUG"] == "WARN" and env["NCCL_DEBUG_SUBSYS"] == "INIT,ENV,GRAPH"
    assert env["NCCL_DEBUG_FILE"].endswith("collectives.w8.low.default.0.nccl.%h.%p.log")


def test_figures_from_runs(tmp_path):
    """SVG + CSV figures of a fused sweep, a layer-boundary run and a training share summary land in
    figures/<exp>/<ts>/ and are well-formed XML."""
    import xml.dom.minidom

    from comm_opt_b200.harness.figures import render

    def run(exp, name, doc):
        d = tmp_path / "results" / exp / "20260101_000000"
        d.mkdir(parents=True)
        (d / name).write_text(json.dumps(doc))
        return d

    sweep = dict(world=8, rows=[dict(impl=i, world=8, dtype="bfloat16", hidden=8192, tokens=t, bytes=t * 16384,
                                     p50_us=v * t ** 0.5, correct=True) for i, v in (("ours", 8.0), ("nccl", 29.0))
                                for t in (1, 4, 16, 64)])
    bnd = dict(world=8, rows=[dict(impl=i, batch=B, p50_us=v, correct=True, error="", roofline_us=12.2)
                              for B in (1, 8) for i, v in (("fused", 27.0), ("split", 34.0))])
    share = dict(model="llama3-8b", world=8, tp=4, dp=2, step_ms=700.0, tokens_per_s=23000.0,
                 breakdown=dict(compute_pct=68.0, hidden_cost_pct=3.0, transfer_pct=14.0, other_pct=15.0))
    for exp, name, doc, files in (("fused_sweep", "sweep.json", sweep,
                                   ("per_op.csv", "latency.svg", "roofline.csv", "roofline.svg")),
                                  ("boundary_bench", "boundary.json", bnd, ("boundary.csv", "boundary.svg")),
                                  ("train_share", "summary.json", share, ("share.csv", "share.svg"))):
        out = render(run(exp, name, doc), base=tmp_path, link_gbs=770.0)
        assert [p.name for p in out] == list(files)
        assert out[0].parent == tmp_path / "figures" / exp / "20260101_000000"
        xml.dom.minidom.parse(str(out[1]))
        assert len(out[0].read_text().splitlines()) >= 2


def test_nvlink_counters_against_fake_nvml():
    """NVLink byte deltas from NVML's per-link throughput counters (KiB), read-only, on a fake NVML:
    absent links skipped, a link whose read fails reported, only enabled links summed."""
    import types

    from comm_opt_b200.utils.nvlink import NvlinkCounters

    class FakeNVML:
        NVML_NVLINK_MAX_LINKS = 4
        NVML_FEATURE_ENABLED = 1
        NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX = 138
        NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX = 139

        class NVMLError(Exception):
            pass

        def __init__(self):
            self.kib = {0: [100, 50], 1: [200, 70], 2: [0, 0]}  # link -> [tx, rx]
            self.calls = []

        def nvmlInit(self):
            pass

        def nvmlDeviceGetHandleByIndex(self, i):
            return ("gpu", i)

        def nvmlDeviceGetNvLinkState(self, h, link):
            if link == 3:
                raise self.NVMLError("not present")
            return 1 if link in (0, 1, 2) else 0

        def nvmlDeviceGetFieldValues(self, h, req):
            self.calls.append(list(req))
            out = []
            for f, link in req:
                ok = 0 if link != 2 else 3  # link 2's counter cannot be read
                val = self.kib[link][0 if f == 138 else 1]
                out.append(types.SimpleNamespace(nvmlReturn=ok, value=types.SimpleNamespace(ullVal=val)))
            return out

    nv = FakeNVML()
    ctr = NvlinkCounters(0, nvml=nv)
    assert ctr.links == [0, 1, 2] and ctr.available
    assert ctr.read() == dict(tx_kib=300, rx_kib=120, failed_links=[2])
    with ctr.measure(settle_s=0) as m:
        nv.kib[0][0] += 7 * 16  # 7 peers x 16 KiB sent on link 0
        nv.kib[1][1] += 3
    assert m["tx_bytes"] == 112 * 1024 and m["rx_bytes"] == 3 * 1024 and m["links"] == 3 and m["failed_links"] == [2]
    assert all(f in (138, 139) for f, _ in nv.calls[0])  # only counter reads were issued


def test_expected_nvlink_bytes_and_link_table():
    from comm_opt_b200.harness.analyze_sweep import expected_tx_bytes, link_table

    S = 16384
    assert expected_tx_bytes("ours:lamport_1s", S, 8) == 7 * S
    assert expected_tx_bytes("ours:lamport_2s", S, 8) == 2 * 7 / 8 * S
    assert expected_tx_bytes("trt_oneshot", S, 4) == 3 * S and expected_tx_bytes("nccl_norm", S, 8) is None
    rows = [dict(impl="ours:auto", world=8, tokens=1, bytes=S, correct=True, nvlink_tx_bytes_per_op=7.1 * S,
                 variant=dict(variant=1)),
            dict(impl="nccl_norm", world=8, tokens=1, bytes=S, correct=True, nvlink_tx_bytes_per_op=2.0 * S)]
    t = link_table(rows)
    assert "| ours:auto | 8 | 1 | 16 | 113.6 | 112.0 | 1.01 |" in t and "| nccl_norm | 8 | 1 | 16 | 32.0 | - | - |" in t


def test_ptxas_report_parse():
    """Resource lines of `-Xptxas -v` -> one row per kernel; names shortened for the table."""
    from comm_opt_b200.harness.ptxas_report import markdown, parse, short

    log = """ptxas info    : Compiling entry function '_Z1kv' for 'sm_100a'
ptxas info    : Function properties for _Z1kv
    40 bytes stack frame, 40 bytes spill stores, 44 bytes spill loads
ptxas info    : Used 128 registers, used 1 barriers, 136 bytes smem
ptxas info    : Compiling entry function '_Z1jv' for 'sm_100a'
ptxas info    : Function properties for _Z1jv
    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 74 registers
"""
    rows = parse(log)
    assert [(r["name"], r["regs"], r["spill_st"], r["spill_ld"], r["smem"]) for r in rows] == [
        ("_Z1kv", 128, 40, 44, 136), ("_Z1jv", 74, 0, 0, 0)]
    assert short("void cob::(anonymous namespace)::k_oneshot<__nv_bfloat16, 8, 1, 1, false>(cob::ARParams)") == \
        "k_oneshot<bfloat16, 8, 1, 1, false>"
    for r in rows:
        r.update(source="x.cu", kernel=r["name"])
    assert markdown(rows).count("\n") == 4


def test_bench_reference_arm_line():
    """`bench.py --impl reference` prints one JSON line naming why the reference arm cannot run."""
    import json
    import subprocess
    import sys

    from conftest import ROOT

    p = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], cwd=ROOT, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    line = json.loads(p.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and len(line["unavailable"]) > 20


def test_bench_clock_summary():
    """Clock record of the timed region: median SM clock, max clock, the throttle reasons seen."""
    import bench

    rows = [["0", "1965", "1965", "650.1", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
            ["0", "1320", "1965", "997.0", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
            ["0", "1410", "1965", "990.0", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
            ["[N/A]"]]
    s = bench.ClockSampler.summarize(rows)
    assert s["sm_mhz"] == 1410.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 997.0
    assert bench.ClockSampler.summarize([])["sm_mhz"] is None


def test_validate_plan():
    """The first-GPU-run plan: self-test parts with the experimental variants, A/B sweeps at every GPU
    count, the decode bench with the new switches on and off."""
    from comm_opt_b200.harness.runner import compose, validate_plan

    plan = validate_plan((2, 4, 8))
    assert sum(l.target == "selftest" for l in plan) == 2 and all(l.env.get("COB_EXPERIMENTAL") == "1"
                                                                  for l in plan if l.target in ("selftest", "fused_sweep"))
    assert sorted(l.world for l in plan if l.target == "fused_sweep") == [2, 4, 8]
    attn = [l for l in plan if l.target == "boundary"]
    assert [(l.world, l.argv) for l in attn if l.world == 8] == [(8, ("--k1", "1024", "--n2", "7168"))]
    cmds = [" ".join(compose(l, ROOT / "results" / "x", 29000 + i)[0]) for i, l in enumerate(plan)]
    assert sum("--l2-prefetch" in c for c in cmds) == 3 and sum("--tune-boundaries 0" in c for c in cmds) == 1
    assert any("decode_vllm" in c for c in cmds) and any("ours:lamport_1sx" in c for c in cmds)


def test_launch_geometry_table():
    """Host-planner geometry of the decode step: every kernel row present at TP 1 and 8, attention at
    TP = 8 leaves SMs free and a push-GEMM CTA fits beside it."""
    import pytest

    from comm_opt_b200._ext import available

    if not available():
        pytest.skip("native extension not built")
    from comm_opt_b200.harness.launch_geometry import markdown, pair_fits, rows_for

    r8 = rows_for("70b", 8, 2048, 8)
    names = [r["kernel"].split(" ")[0] for r in r8]
    assert names[:4] == ["gemm_push", "ar_norm_gemm", "gemm_push", "ar_norm_gemm"] and "attention" in names
    att = next(r for r in r8 if r["kernel"].startswith("attention"))
    assert att["ctas"] == 64 and pair_fits(att, r8[0])
    assert all(r["ctas"] <= 296 for r in r8 if r["kernel"].startswith("ar_norm_gemm"))  # per-block epoch words
    assert "stream-K" in markdown("8b", 8, 1024, [1])


def test_bench_result_line_contract():
    """The JSON line the driver parses: every required key, with the types it expects, and the whole-job
    value, the end-to-end figure with its host transfers, and our launches in the timed region."""
    import json
    from types import SimpleNamespace

    import bench
    from comm_opt_b200.models.llama import PRESETS

    args = SimpleNamespace(batch=8, prompt=2048, steps=64, warmup=4, model="70b", layers=None, gemm="cob",
                           collective="ours", l2_prefetch=0)
    runner = SimpleNamespace(fuse_boundary=True, fuse_epilogues=False, fuse_error="", fuse_kinds={8: (False, True)},
                             boundary_times={8: {"FF": 7.8, "SF": 7.5}}, kernels_per_step={8: 566},
                             fused_epilogues_used=lambda B: (False, True),
                             lin={(0, "gu"): SimpleNamespace(kernels=lambda B: 1)})
    clocks = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": []}
    line = bench.result_line(args, PRESETS["70b"], 8, 7.5, 7.55, 64, 5.0, clocks, runner)
    json.dumps(line)
    for k, t in (("metric", str), ("value", float), ("unit", str), ("n_gpus", int), ("steps", int), ("warmup", int),
                 ("ms_per_step", float), ("higher_is_better", bool), ("scaling", str), ("dtype", str), ("data", str),
                 ("config", dict), ("e2e", dict), ("gpu_launches", int), ("clocks", dict)):
        assert isinstance(line[k], t), k
    assert "vs_baseline" in line and line["higher_is_better"] is False and line["scaling"] in ("weak", "strong")
    assert {"model", "global_batch", "seq_len", "parallelism"} <= set(line["config"])
    assert line["config"]["parallelism"] == "tp8" and line["gpu_launches"] == 566 * 64
    assert line["config"]["gate_up_swiglu_epilogue"] is True
    assert {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"} <= set(line["e2e"])
    assert line["config"]["fused_boundaries"]["attention_out"] is False and "141 GB" in line["config"]["l2"]
    assert line["config"]["fused_boundaries"]["epilogues"] == {"swiglu": False, "rope_kv": True}


def test_measured_link_rate_from_newest_record(tmp_path):
    """The NVLink denominator comes from the newest platform record; no record, no number."""
    from comm_opt_b200.utils.peaks import NoRecord, hbm_gbs, link_gbs

    with pytest.raises(NoRecord):
        link_gbs(tmp_path)
    for ts, v in (("20261201_000000", 700.0), ("20261202_000000", 771.5)):
        (tmp_path / ts).mkdir()
        (tmp_path / ts / "link.json").write_text(json.dumps(dict(gpus=8, peer_copy_gbs_median=v)))
    assert link_gbs(tmp_path) == 771.5
    (tmp_path / "20261203_000000").mkdir()
    (tmp_path / "20261203_000000" / "link.json").write_text(json.dumps(dict(gpus=1, hbm_copy_gbs=[6500.0])))
    with pytest.raises(NoRecord):
        link_gbs(tmp_path)  # a one-GPU record has no peer copy
    (tmp_path / "peaks.json").write_text(json.dumps(dict(hbm_gbs=6542.4)))
    assert hbm_gbs(tmp_path / "peaks.json") == 6542.4

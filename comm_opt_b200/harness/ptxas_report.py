"""Per-kernel resources of the native extension as the compiler assigns them (no GPU needed).

    python -m comm_opt_b200.harness.ptxas_report [--sources fused_ar.cu,attention.cu] [--filter regex]
                                                  [--out table.md]

Compiles every CUDA source of the extension for sm_100a with the build's own flags plus
``-Xptxas -v`` into a temporary directory and tabulates, per kernel instantiation: registers per
thread, stack frame, spill stores / loads and static shared memory (dynamic shared memory is set at
launch and not shown). Spills and register counts are what to check before spending GPU time: a
kernel capped by ``__launch_bounds__`` at 128 registers that spills keeps part of its state in local
memory.
"""
from __future__ import annotations

import argparse
import importlib.util
import re
import shutil
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "csrc"


def build_flags():
    spec = importlib.util.spec_from_file_location("cob_build_flags", CSRC / "build_flags.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def include_dirs() -> list[str]:
    from torch.utils.cpp_extension import include_paths

    return [str(CSRC)] + include_paths("cuda")


def compile_verbose(src: str, outdir: Path) -> str:
    """nvcc -c with -Xptxas -v; returns the compiler's resource lines (stderr)."""
    f = build_flags()
    cmd = ["nvcc", *f.NVCC, "-Xptxas", "-v", *[f"-I{d}" for d in include_dirs()], "-c", str(CSRC / src), "-o",
           str(outdir / (Path(src).stem + ".o"))]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{p.stderr[-4000:]}")
    return p.stdout + p.stderr


_ENTRY = re.compile(r"Compiling entry function '(\S+)'")
_FRAME = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")
_USED = re.compile(r"Used (\d+) registers")
_SMEM = re.compile(r"(\d+) bytes smem")


def parse(text: str) -> list[dict]:
    """Resource rows of one ptxas log: name (mangled), regs, stack, spill_st, spill_ld, smem."""
    rows, cur, frame = [], None, (0, 0, 0)
    for line in text.splitlines():
        m = _ENTRY.search(line)
        if m:
            cur, frame = m.group(1), (0, 0, 0)
            continue
        m = _FRAME.search(line)
        if m and cur:
            frame = tuple(int(x) for x in m.groups())
            continue
        m = _USED.search(line)
        if m and cur:
            s = _SMEM.search(line)
            rows.append(dict(name=cur, regs=int(m.group(1)), stack=frame[0], spill_st=frame[1], spill_ld=frame[2],
                             smem=int(s.group(1)) if s else 0))
            cur = None
    return rows


def demangle(names: list[str]) -> list[str]:
    if not shutil.which("c++filt"):
        return names
    p = subprocess.run(["c++filt"], input="\n".join(names), capture_output=True, text=True)
    out = p.stdout.splitlines()
    return out if len(out) == len(names) else names


def short(name: str) -> str:
    """Kernel name with its template arguments, without namespaces and the parameter list."""
    name = name.replace("(anonymous namespace)::", "").replace("cob::", "").replace("__nv_", "")
    depth, cut = 0, len(name)
    for i, ch in enumerate(name):  # drop the parameter list: the first '(' outside template brackets
        if ch == "<":
            depth += 1
        elif ch == ">":
            depth -= 1
        elif ch == "(" and depth == 0 and i > 0:
            cut = i
            break
    return name[:cut].replace("void ", "").strip()


def report(sources: list[str], pattern: str | None = None) -> list[dict]:
    with tempfile.TemporaryDirectory() as td, ThreadPoolExecutor(max_workers=len(sources)) as ex:
        logs = list(ex.map(lambda s: (s, compile_verbose(s, Path(td))), sources))
    rows = []
    for src, text in logs:
        rs = parse(text)
        for r, d in zip(rs, demangle([r["name"] for r in rs])):
            r.update(source=src, kernel=short(d))
            if pattern is None or re.search(pattern, r["kernel"]):
                rows.append(r)
    return rows


def markdown(rows: list[dict]) -> str:
    out = ["| source | kernel | regs | stack B | spill st/ld B | static smem B |", "|---|---|---|---|---|---|"]
    for r in sorted(rows, key=lambda r: (r["source"], r["kernel"])):
        out.append(f"| {r['source']} | `{r['kernel']}` | {r['regs']} | {r['stack']} | {r['spill_st']}/{r['spill_ld']} "
                   f"| {r['smem']} |")
    return "\n".join(out) + "\n"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--sources", default=",".join(build_flags().CUDA_SOURCES))
    ap.add_argument("--filter", default=None, help="regex on the demangled kernel name")
    ap.add_argument("--out", default=None)
    a = ap.parse_args(argv)
    rows = report([s for s in a.sources.split(",") if s], a.filter)
    text = markdown(rows)
    spills = [r for r in rows if r["spill_st"] or r["spill_ld"]]
    text += f"\n{len(rows)} kernels, {len(spills)} with spills.\n"
    if a.out:
        Path(a.out).write_text(text)
    sys.stdout.write(text)


if __name__ == "__main__":
    main()

"""Re-run the measurements behind the published tables with one command.

    python -m quantized_flash_communication_b200.benchmarks.reproduce --gpus 8 \
        [--only flagship,variants,breakdown,allreduce,norm,decode,tables,quant,kernels] [--out results.jsonl] [--dry-run]

Every item is a list of commands: the benchmark modules of this package (one process
per GPU under ``torch.distributed.run`` with the rendezvous on 127.0.0.1 when an item
needs several GPUs) and ``bench.py`` for the flagship.  Items that need more GPUs than
``--gpus`` are skipped.  Each command runs in its own process group under a time limit
(``--timeout`` seconds; the whole group is killed when it runs out), and every JSON line
it prints is appended to ``--out`` tagged with the item, the command and its exit code.
While the commands run, ``nvidia-smi`` samples the clocks and throttle reasons of the
visible GPUs into ``<out>.clocks.csv`` (a failure to start it is reported, not fatal).

Items (BASELINE.json configurations in brackets):
  flagship   bench.py, ours and the reference arm, at 1, 2, 4, 8 GPUs   [3]
  variants   prefill step under each all-reduce variant at 2, 4, 8      [3]
  breakdown  per-operator device time of the flagship step at 1, 2, 4, 8 [3]
  allreduce  all-reduce sweep vs NCCL bf16 at 2, 4, 8, and the reference's
             flash_all_reduce at group 128                               [2]
  norm       all-reduce + residual + RMSNorm: 1, 2, 4 warps per row      [3]
  decode     Llama-3-8B decode at TP 1, 2, 4, 8 (ours and reference), Llama-3-70B
             TP 8 INT4 prefill + decode                                  [4, 5]
  tables     the reference's Tables 1-4 and its QA generation (main) at 1, 2, 4, 8
  quant      standalone quantizers vs the reference's                    [kernels]
  kernels    one kernel_probe line per hand-written kernel               [kernels]
"""
from __future__ import annotations

import argparse
import json
import os
import shlex
import signal
import socket
import subprocess
import sys
import time
from typing import Dict, List, Tuple

PKG = "quantized_flash_communication_b200.benchmarks"
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

SMI_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(n: int, target: List[str]) -> List[str]:
    """Command line for ``target`` (["-m", module, ...] or ["bench.py", ...]) on n GPUs."""
    if n <= 1:
        return [sys.executable] + target
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
            "--master-addr", "127.0.0.1", f"--master-port={_free_port()}"] + target


def items(gpus: int) -> Dict[str, List[Tuple[int, List[str]]]]:
    """item -> [(GPUs needed, target argv)]"""
    ns = [n for n in (1, 2, 4, 8) if n <= gpus]
    multi = [n for n in ns if n > 1]
    out: Dict[str, List[Tuple[int, List[str]]]] = {}
    out["flagship"] = []
    for n in ns:
        out["flagship"].append((n, ["bench.py", "--gpus", str(n), "--steps", "10", "--warmup", "3"]))
        out["flagship"].append((n, ["bench.py", "--impl", "reference", "--gpus", str(n), "--steps", "5",
                                    "--warmup", "3"]))
    out["variants"] = [(n, ["-m", f"{PKG}.bench_prefill_variants", "--steps", "10", "--warmup", "3"]) for n in multi]
    out["breakdown"] = [(n, ["bench.py", "--gpus", str(n), "--breakdown", "--steps", "3", "--warmup", "3"]) for n in ns]
    sweep = ["--tokens", "1,16,128,1024,4096,16384", "--hidden", "4096,8192", "--iters", "10"]
    out["allreduce"] = []
    for n in multi:
        out["allreduce"].append((n, ["-m", f"{PKG}.bench_allreduce"] + sweep + ["--bits", "8,4", "--gs", "32,64,128",
                                                                              "--stages", "1,2"]))
        out["allreduce"].append((n, ["-m", f"{PKG}.bench_allreduce"] + sweep + ["--bits", "8,4", "--gs", "128",
                                                                              "--reference"]))
    out["norm"] = [(n, ["-m", f"{PKG}.bench_allreduce", "--tokens", "1024,8192", "--hidden", "4096", "--bits", "8",
                        "--gs", "128", "--norm", "--norm-wpr", "1,2,4", "--iters", "10"]) for n in multi]
    out["decode"] = []
    for n in ns:
        out["decode"].append((n, ["-m", f"{PKG}.bench_decode", "--model", "llama3-8b", "--batch", "64", "--ctx", "4096",
                                  "--new", "128", "--bits", "8"]))
        out["decode"].append((n, ["-m", f"{PKG}.bench_decode", "--model", "llama3-8b", "--batch", "64", "--ctx", "4096",
                                  "--new", "128", "--impl", "reference"]))
    if gpus >= 8:
        for extra in ([], ["--gemv"]):
            out["decode"].append((8, ["-m", f"{PKG}.bench_decode", "--model", "llama3-70b", "--batch", "4", "--ctx",
                                      "2048", "--new", "128", "--bits", "4"] + extra))
    out["tables"] = [(n, ["-m", "quantized_flash_communication_b200.main", "--max-new-tokens", "32"]) for n in ns]
    out["quant"] = [(1, ["-m", f"{PKG}.bench_quant", "--reference"])]
    probes = [["gemm"], ["attention", "8", "1024", "32", "32"], ["attention", "4", "2048", "64", "8"],
              ["attention", "2", "4096", "32", "8"], ["attention", "8", "1024", "32", "32", "--attn-packed"],
              ["attention", "4", "2048", "64", "8", "--attn-packed"], ["allreduce", "2", "16384", "4096", "8"],
              ["allreduce", "8", "8192", "4096", "8"], ["allreduce", "8", "8192", "4096", "8", "--stages", "2"],
              ["allreduce_norm", "8", "8192", "4096", "8"], ["allreduce_norm", "8", "8192", "4096", "8", "--norm-wpr", "4"],
              ["gemm_small", "4", "8192", "8192"], ["gemm_small", "4", "8192", "8192", "--gemv"], ["quantize"], ["decode"], ["rmsnorm"], ["rope_decode"],
              ["silu_mul"], ["pack"], ["unpack"], ["oneshot"], ["gemm_qs8"], ["gemm_small"], ["qkv_rope"]]
    out["kernels"] = [(1, ["-m", f"{PKG}.kernel_probe"] + p + ["--iters", "10"]) for p in probes]
    return out


def _run(cmd: List[str], timeout: float, env: Dict[str, str]) -> Tuple[int, str]:
    """Run in a new process group; on timeout kill the whole group.  Returns (rc, stdout)."""
    p = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                         start_new_session=True)
    try:
        out, _ = p.communicate(timeout=timeout)
        return p.returncode, out
    except subprocess.TimeoutExpired:
        os.killpg(p.pid, signal.SIGKILL)
        out, _ = p.communicate()
        return 124, out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--only", default="flagship,variants,breakdown,allreduce,norm,decode,tables,quant,kernels")
    ap.add_argument("--out", default="reproduce_results.jsonl")
    ap.add_argument("--timeout", type=float, default=300.0, help="seconds per command")
    ap.add_argument("--dry-run", action="store_true", help="print the commands only")
    ap.add_argument("--ns", default="", help="run only the commands for these GPU counts, e.g. 8 or 2,4")
    args = ap.parse_args(argv)
    table = items(args.gpus)
    if args.ns:
        keep = {int(v) for v in args.ns.split(",") if v}
        table = {k: [(n, t) for n, t in v if n in keep] for k, v in table.items()}
    wanted = [w for w in args.only.split(",") if w]
    unknown = [w for w in wanted if w not in table]
    if unknown:
        ap.error(f"unknown items {unknown}; choose from {sorted(table)}")
    env = dict(os.environ)
    env.setdefault("QFC_COMM_TIMEOUT_MS", "3000")  # bounded waits end a stuck rank quickly
    smi = smi_log = None
    if not args.dry_run:
        try:
            smi_log = open(args.out + ".clocks.csv", "w")
            smi = subprocess.Popen(["nvidia-smi", f"--query-gpu={SMI_QUERY}", "--format=csv", "-lms", "500"],
                                   stdout=smi_log, stderr=subprocess.STDOUT, start_new_session=True)
        except OSError as e:
            print(f"clock sampler not started: {e}", file=sys.stderr)
    failures = 0
    try:
        for item in wanted:
            for n, target in table[item]:
                cmd = _launch(n, target)
                line = " ".join(shlex.quote(c) for c in cmd)
                if args.dry_run:
                    print(f"[{item}] {line}")
                    continue
                t0 = time.time()
                rc, out = _run(cmd, args.timeout, env)
                failures += rc != 0
                with open(args.out, "a") as f:
                    for ln in out.splitlines():
                        if ln.startswith("{"):
                            try:
                                rec = json.loads(ln)
                            except ValueError:
                                continue
                            f.write(json.dumps({"item": item, "n_gpus": n, "cmd": line, "rc": rc, **rec}) + "\n")
                    if rc != 0:
                        f.write(json.dumps({"item": item, "n_gpus": n, "cmd": line, "rc": rc,
                                            "tail": out.splitlines()[-5:]}) + "\n")
                print(f"[{item}] rc={rc} {time.time() - t0:.0f}s  {line}", flush=True)
    finally:
        if smi is not None:
            os.killpg(smi.pid, signal.SIGTERM)
            smi.wait(timeout=10)
        if smi_log is not None:
            smi_log.close()
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())

"""Deployment CLI: the counterpart of ``python3 -m c35.deploy`` (c35/deploy.py:40-204)
and of ``load_and_infer`` (c35/executor.py:997-1265), with batch sharding over
the GPUs of one node.

    python -m hackathon_b200.deploy (--model NAME | --onnx MODEL) --input DIR --output DIR
                                    [--batch-size N] [--precision fp32|bf16] [--gpus G]

Input contract (same as the reference): ``DIR/manifest.json`` lists
``{"tensors": [{"name", "file", "dtype", "shape"}]}`` with ``.npy`` files beside
it; every input shares the leading batch dimension.  Output: ``logits.npy`` and
``manifest.json`` (c35/executor.py:1180-1201), non-finite logits rejected
(executor.py:1177), exit code 1 on any error (deploy.py:122-126).

With ``--gpus G > 1`` the parent starts one worker process per GPU
(``CUDA_VISIBLE_DEVICES=r``); worker r runs the contiguous rows
``[r*N/G, (r+1)*N/G)`` through its own executor and arena and writes its logits
shard; the parent checks every worker's exit status under a deadline and
concatenates the shards in order.  No collective is involved: samples are
independent.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from typing import Dict, List, Optional, Tuple

import numpy as np


def positive_int(value: str) -> int:
    """c35/deploy.py:22-37: --batch-size must be a positive integer."""
    try:
        v = int(value)
    except ValueError:
        raise argparse.ArgumentTypeError(f"batch-size must be an integer, got '{value}'")
    if v <= 0:
        raise argparse.ArgumentTypeError(f"batch-size must be positive, got {v}")
    return v


def read_inputs(input_dir: str) -> Dict[str, np.ndarray]:
    """Manifest + .npy inputs with the reference's checks (c35/executor.py:1036-1121)."""
    mpath = os.path.join(input_dir, "manifest.json")
    if not os.path.isfile(mpath):
        raise FileNotFoundError(f"Input manifest not found: {mpath}")
    manifest = json.load(open(mpath))
    arrays: Dict[str, np.ndarray] = {}
    for e in manifest.get("tensors", []):
        name = e["name"]
        if name in arrays:
            raise ValueError(f"Duplicate input tensor in manifest: '{name}'")
        path = os.path.join(input_dir, e["file"])
        if not os.path.isfile(path):
            raise FileNotFoundError(f"Input file not found: {path}")
        a = np.load(path, allow_pickle=False)
        if e.get("dtype") is not None and np.dtype(e["dtype"]) != a.dtype:
            raise ValueError(f"Input '{name}' dtype mismatch: manifest={e['dtype']}, npy={a.dtype}")
        if e.get("shape") is not None and list(a.shape) != list(e["shape"]):
            raise ValueError(f"Input '{name}' shape mismatch: manifest={e['shape']}, npy={list(a.shape)}")
        arrays[name] = a
    if not arrays:
        raise ValueError("No input tensors found in manifest")
    if len({a.shape[0] for a in arrays.values()}) != 1:
        raise ValueError("All graph inputs must have the same batch dimension")
    return arrays


def write_outputs(output_dir: str, logits: np.ndarray, name: str = "logits") -> None:
    if not np.isfinite(logits).all():
        raise ValueError("Output contains non-finite values (NaN or Inf)")
    os.makedirs(output_dir, exist_ok=True)
    np.save(os.path.join(output_dir, "logits.npy"), logits.astype(np.float32))
    manifest = {"tensors": [{"name": name, "file": "logits.npy", "dtype": "float32", "shape": list(logits.shape)}]}
    with open(os.path.join(output_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=2)


def load_graph(model: Optional[str], onnx_path: Optional[str]):
    from .workloads import BUILDERS
    if model:
        if model not in BUILDERS:
            raise ValueError(f"unknown model {model!r}; choose from {sorted(BUILDERS)}")
        return BUILDERS[model]()
    from .onnx_import import import_onnx
    return import_onnx(onnx_path)


def validate_inputs(graph, feeds: Dict[str, np.ndarray]) -> None:
    for vi in graph.inputs:
        if vi.name not in feeds:
            raise ValueError(f"missing graph input '{vi.name}'")
        a = feeds[vi.name]
        if np.dtype(vi.dtype) != a.dtype:
            raise ValueError(f"Input '{vi.name}' dtype {a.dtype} != graph dtype {vi.dtype}")
        want = [d for d in vi.shape]
        if len(want) != a.ndim or any(not isinstance(d, str) and int(d) != s for d, s in zip(want, a.shape)):
            raise ValueError(f"Input '{vi.name}' shape {list(a.shape)} does not match graph {want}")


def infer(graph, feeds: Dict[str, np.ndarray], batch_size: Optional[int], precision: str) -> np.ndarray:
    """Batch loop of load_and_infer (c35/executor.py:1137-1164), one plan per batch size."""
    from .lowering import lower
    from .program import Executor
    n = next(iter(feeds.values())).shape[0]
    bs = min(batch_size or n, n)
    executors: Dict[int, Executor] = {}
    outs: List[np.ndarray] = []
    for start in range(0, n, bs):
        b = min(bs, n - start)
        if b not in executors:
            executors[b] = Executor(lower(graph, b, precision))
        ex = executors[b]
        res = ex.run({k: v[start:start + b] for k, v in feeds.items()})
        outs.append(res[ex.prog.outputs[0]])
    for ex in executors.values():
        ex.native.close()
    return np.concatenate(outs, axis=0)


def shard_bounds(n: int, world: int, rank: int) -> Tuple[int, int]:
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def run_sharded(argv: List[str], n: int, gpus: int, workdir: str, timeout_s: float,
                worker_cmd: Optional[List[str]] = None) -> np.ndarray:
    """Spawn one worker per GPU, enforce the deadline and exit codes, gather shards."""
    procs = []
    for r in range(gpus):
        env = dict(os.environ, CUDA_VISIBLE_DEVICES=str(r), C3B_RANK=str(r), C3B_WORLD=str(gpus))
        cmd = (worker_cmd or [sys.executable, "-m", "hackathon_b200.deploy"]) + argv + \
            ["--_worker", workdir, "--gpus", "1"]
        procs.append(subprocess.Popen(cmd, env=env))
    deadline = time.time() + timeout_s
    failed = []
    for r, p in enumerate(procs):
        try:
            rc = p.wait(timeout=max(1.0, deadline - time.time()))
        except subprocess.TimeoutExpired:
            p.kill()
            p.wait()
            rc = "timeout"
        if rc != 0:
            failed.append((r, rc))
    if failed:
        for p in procs:
            if p.poll() is None:
                p.kill()
        raise RuntimeError(f"worker(s) failed: {failed}")
    shards = []
    for r in range(gpus):
        path = os.path.join(workdir, f"logits_rank{r}.npy")
        if not os.path.isfile(path):
            raise RuntimeError(f"worker {r} wrote no shard")
        shards.append(np.load(path))
    out = np.concatenate(shards, axis=0)
    if out.shape[0] != n:
        raise ValueError(f"Output sample count mismatch: got {out.shape[0]}, expected {n}")
    return out


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="C3.5 deployment on B200 (native backend)")
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--model", help="built-in seeded workload (mlp, resnet18, tx_small, tx_large)")
    src.add_argument("--onnx", help="path to an ONNX model (needs the onnx package)")
    ap.add_argument("--input", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--batch-size", type=positive_int, default=None)
    ap.add_argument("--precision", choices=["fp32", "bf16"], default="fp32")
    ap.add_argument("--gpus", type=positive_int, default=1)
    ap.add_argument("--timeout", type=float, default=1800.0)
    ap.add_argument("--_worker", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args(argv)
    raw = list(argv if argv is not None else sys.argv[1:])
    try:
        t0 = time.perf_counter()
        feeds = read_inputs(args.input)
        graph = load_graph(args.model, args.onnx)
        validate_inputs(graph, feeds)
        n = next(iter(feeds.values())).shape[0]
        if args._worker:
            rank, world = int(os.environ.get("C3B_RANK", 0)), int(os.environ.get("C3B_WORLD", 1))
            s, e = shard_bounds(n, world, rank)
            out = infer(graph, {k: v[s:e] for k, v in feeds.items()}, args.batch_size, args.precision)
            np.save(os.path.join(args._worker, f"logits_rank{rank}.npy"), out)
            return 0
        if args.gpus > 1:
            keep = []
            skip = False
            for tok in raw:
                if skip:
                    skip = False
                    continue
                if tok == "--gpus":
                    skip = True
                    continue
                if tok.startswith("--gpus="):
                    continue
                keep.append(tok)
            with tempfile.TemporaryDirectory() as wd:
                logits = run_sharded(keep, n, args.gpus, wd, args.timeout)
        else:
            logits = infer(graph, feeds, args.batch_size, args.precision)
        write_outputs(args.output, logits, graph.outputs[0].name)
        info = {"samples": int(n), "gpus": args.gpus, "precision": args.precision,
                "seconds": round(time.perf_counter() - t0, 4), "output_shape": list(logits.shape)}
        print("C3B_EVIDENCE_JSON=" + json.dumps(info))
        return 0
    except Exception as e:  # fail closed with exit 1, as c35/deploy.py:122-126
        print(f"error: {type(e).__name__}: {e}", file=sys.stderr)
        return 1


if __name__ == "__main__":
    sys.exit(main())

"""Deploy CLI host logic and the multi-process shard launcher, without a GPU.

Failure detection follows the reference's fail-closed contract (c35/deploy.py:
122-126, c35/standard_runner.py:441-446): a worker that exits non-zero or
never finishes makes the launcher report an error instead of writing output.
"""

import json
import os
import sys

import numpy as np
import pytest

from hackathon_b200 import deploy as D

FAKE_WORKER = r"""
import os, sys, time, numpy as np
args = sys.argv[1:]
wd = args[args.index('--_worker') + 1]
rank, world = int(os.environ['C3B_RANK']), int(os.environ['C3B_WORLD'])
mode = os.environ.get('FAKE_MODE', 'ok')
if mode == 'fail' and rank == 1:
    sys.exit(3)
if mode == 'hang' and rank == 0:
    time.sleep(60)
n = int(os.environ['FAKE_N'])
base, extra = divmod(n, world)
s = rank * base + min(rank, extra)
e = s + base + (1 if rank < extra else 0)
np.save(os.path.join(wd, f'logits_rank{rank}.npy'), np.arange(s, e, dtype=np.float32)[:, None] * np.ones((1, 3), np.float32))
"""


def _fake_cmd(tmp_path):
    p = tmp_path / "fake_worker.py"
    p.write_text(FAKE_WORKER)
    return [sys.executable, str(p)]


def test_shard_bounds_cover_all_rows():
    for n in (1, 7, 4096, 4097):
        for w in (1, 2, 3, 8):
            spans = [D.shard_bounds(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c


def test_launcher_gathers_shards_in_order(tmp_path, monkeypatch):
    monkeypatch.setenv("FAKE_N", "11")
    out = D.run_sharded([], 11, 3, str(tmp_path), 30, worker_cmd=_fake_cmd(tmp_path))
    assert np.array_equal(out[:, 0], np.arange(11, dtype=np.float32))


def test_launcher_detects_failed_worker(tmp_path, monkeypatch):
    monkeypatch.setenv("FAKE_N", "8")
    monkeypatch.setenv("FAKE_MODE", "fail")
    with pytest.raises(RuntimeError, match=r"worker\(s\) failed: \[\(1, 3\)\]"):
        D.run_sharded([], 8, 2, str(tmp_path), 30, worker_cmd=_fake_cmd(tmp_path))


def test_launcher_deadline_kills_hung_worker(tmp_path, monkeypatch):
    monkeypatch.setenv("FAKE_N", "8")
    monkeypatch.setenv("FAKE_MODE", "hang")
    with pytest.raises(RuntimeError, match="timeout"):
        D.run_sharded([], 8, 2, str(tmp_path), 2.0, worker_cmd=_fake_cmd(tmp_path))


def test_batch_size_validation():
    import argparse
    assert D.positive_int("3") == 3
    for bad in ("0", "-2", "x"):
        with pytest.raises(argparse.ArgumentTypeError):
            D.positive_int(bad)


def _write_input_dir(d, arrays, manifest_extra=None):
    os.makedirs(d, exist_ok=True)
    ents = []
    for k, v in arrays.items():
        np.save(os.path.join(d, f"{k}.npy"), v)
        ents.append({"name": k, "file": f"{k}.npy", "dtype": str(v.dtype), "shape": list(v.shape)})
    if manifest_extra:
        ents[0].update(manifest_extra)
    json.dump({"tensors": ents}, open(os.path.join(d, "manifest.json"), "w"))


def test_input_manifest_checks(tmp_path):
    d = str(tmp_path / "in")
    x = np.zeros((4, 784), np.float32)
    _write_input_dir(d, {"input": x})
    assert D.read_inputs(d)["input"].shape == (4, 784)
    _write_input_dir(d, {"input": x}, {"dtype": "float64"})
    with pytest.raises(ValueError, match="dtype mismatch"):
        D.read_inputs(d)
    with pytest.raises(FileNotFoundError):
        D.read_inputs(str(tmp_path / "missing"))
    g = D.load_graph("mlp", None)
    with pytest.raises(ValueError, match="does not match graph"):
        D.validate_inputs(g, {"input": np.zeros((4, 3), np.float32)})


def test_cli_fails_closed_with_exit_1(tmp_path):
    rc = D.main(["--model", "mlp", "--input", str(tmp_path / "none"), "--output", str(tmp_path / "o")])
    assert rc == 1


def test_output_contract(tmp_path):
    D.write_outputs(str(tmp_path), np.ones((3, 10), np.float32))
    m = json.load(open(tmp_path / "manifest.json"))
    assert m["tensors"][0] == {"name": "logits", "file": "logits.npy", "dtype": "float32", "shape": [3, 10]}
    with pytest.raises(ValueError, match="non-finite"):
        D.write_outputs(str(tmp_path), np.array([[np.nan]], np.float32))

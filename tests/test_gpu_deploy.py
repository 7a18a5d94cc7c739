"""The deploy CLI end to end on the GPU (c35/deploy.py contract): manifest in,
logits.npy + manifest.json out, ragged batch loops (the reference's CLI tests
use batch sizes 1, 7, 97, c35/test_c35.py:84-219), one plan per distinct batch
size, and the multi-GPU launcher path with one worker."""

import json
import os

import numpy as np
import pytest

from oracle.evaluate import run_graph

pytestmark = pytest.mark.gpu


def _input_dir(path, feeds):
    os.makedirs(path, exist_ok=True)
    ents = []
    for k, v in feeds.items():
        np.save(os.path.join(path, f"{k}.npy"), v)
        ents.append({"name": k, "file": f"{k}.npy", "dtype": str(v.dtype), "shape": list(v.shape)})
    json.dump({"tensors": ents}, open(os.path.join(path, "manifest.json"), "w"))


@pytest.mark.parametrize("batch_size", [None, 1, 7, 97])
def test_cli_mlp_fp32_batches(tmp_path, batch_size):
    from hackathon_b200 import deploy
    from hackathon_b200.workloads import build_mlp, make_inputs
    g = build_mlp()
    feeds = make_inputs(g, 100)
    _input_dir(str(tmp_path / "in"), feeds)
    argv = ["--model", "mlp", "--input", str(tmp_path / "in"), "--output", str(tmp_path / "out")]
    if batch_size:
        argv += ["--batch-size", str(batch_size)]
    assert deploy.main(argv) == 0
    out = np.load(tmp_path / "out" / "logits.npy")
    ref = run_graph(g, feeds)["logits"]
    assert out.shape == (100, 10)
    assert np.abs(out - ref).max() / np.abs(ref).max() < 1e-4
    m = json.load(open(tmp_path / "out" / "manifest.json"))
    assert m["tensors"][0]["shape"] == [100, 10]


def test_cli_resnet_bf16_ragged_and_sharded(tmp_path):
    from hackathon_b200 import deploy
    from hackathon_b200.workloads import build_resnet18, make_inputs
    g = build_resnet18()
    feeds = make_inputs(g, 37)
    _input_dir(str(tmp_path / "in"), feeds)
    base = ["--model", "resnet18", "--input", str(tmp_path / "in"), "--precision", "bf16"]
    assert deploy.main(base + ["--output", str(tmp_path / "o1"), "--batch-size", "16"]) == 0
    out = np.load(tmp_path / "o1" / "logits.npy")
    ref = run_graph(g, feeds)["logits"]
    assert np.abs(out - ref).max() / np.abs(ref).max() < 2e-2
    # launcher path (one worker process on this GPU) gives the same bits
    wd = tmp_path / "wd"
    wd.mkdir()
    sharded = deploy.run_sharded(base + ["--output", str(tmp_path / "o2"), "--batch-size", "16"], 37, 1,
                                 str(wd), 600)
    assert np.array_equal(sharded, out)


def test_cli_rejects_bad_input_shape(tmp_path):
    from hackathon_b200 import deploy
    _input_dir(str(tmp_path / "in"), {"input": np.zeros((4, 3, 16, 16), np.float32)})
    rc = deploy.main(["--model", "resnet18", "--input", str(tmp_path / "in"), "--output", str(tmp_path / "o")])
    assert rc == 1
    assert not os.path.exists(tmp_path / "o" / "logits.npy")

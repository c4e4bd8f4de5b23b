"""The C++20 host side: the EHAPPruner / CORINGPruner / TBWriter / safetensors
API (tensorbit-core_b200/include/tensorbit/core) and the tb-prune CLI.

CPU: the API driver's GPU-free checks (the reference's own unit tests, .tb and
safetensors IO).  GPU: the driver's device checks, and tb-prune runs whose
output files must be byte-identical to the reference CLI's (golden digests made
by tests/golden/make_golden.py from the reference binary).
"""
import hashlib
import json
import os
import subprocess

import pytest

import inputs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tensorbit-core_b200", "bin")
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


@pytest.fixture(scope="module")
def binaries(tblib):
    for name in ("tb-prune", "tb-api-test"):
        if not os.path.exists(os.path.join(BIN, name)):
            import build
            build.build()
    return BIN


def sha_file(path):
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


def test_api_driver_cpu_checks(binaries):
    r = subprocess.run([os.path.join(binaries, "tb-api-test")], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


@pytest.mark.gpu
def test_api_driver_gpu_checks(binaries, cuda):
    r = subprocess.run([os.path.join(binaries, "tb-api-test"), "--gpu"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed (with GPU checks)" in r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("key", sorted(inputs.MOCK_RUNS))
def test_tb_prune_mock_runs_byte_identical(binaries, cuda, tmp_path, key):
    out = str(tmp_path / (key + ".tb"))
    r = subprocess.run([os.path.join(binaries, "tb-prune"), *inputs.MOCK_RUNS[key], "--output", out],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert sha_file(out) == GOLD["tb_prune_mock_runs"][key]


@pytest.mark.gpu
def test_tb_prune_real_mode_byte_identical(binaries, cuda, tmp_path):
    model = str(tmp_path / "model.safetensors")
    inputs.small_model(model)
    outdir = tmp_path / "out"
    r = subprocess.run([os.path.join(binaries, "tb-prune"), "--model", model, "--output", str(outdir)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    gold = GOLD["tb_prune_real_small_model"]
    assert sorted(os.listdir(outdir)) == sorted(gold)
    for name, digest in gold.items():
        assert sha_file(str(outdir / name)) == digest, name

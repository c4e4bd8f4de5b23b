"""GPU: tb-prune real mode as a pipeline (a reader thread prefetching the next
tensors into pinned buffers, one worker thread per GPU, outputs written in
tensor order) on a multi-tensor checkpoint with F32, BF16 and F16 tensors, a
tensor CORING must skip and a non-float tensor: every output file, model.tbm
included, byte-identical to the reference CLI's (compiled from the reference's
sources under oracle/_ref), with one GPU and, where there are two, with
--gpus 2."""
import os
import subprocess

import pytest

import inputs

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tensorbit-core_b200", "bin", "tb-prune")
REF = os.path.join(ROOT, "oracle", "_ref", "tb-prune")


def run(exe, model, out, *extra):
    r = subprocess.run([exe, "--model", model, "--output", out, *extra], capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    return {name: open(os.path.join(out, name), "rb").read() for name in sorted(os.listdir(out))}


def test_real_mode_pipeline_matches_reference_cli(cuda, tblib, tmp_path):
    if not os.path.exists(REF):
        pytest.skip("the reference CLI was not compiled here (needs the reference sources at build time)")
    model = str(tmp_path / "model.safetensors")
    inputs.layered_model(model)
    want = run(REF, model, str(tmp_path / "ref"))
    assert "model.tbm" in want and len(want) == 3 * 3 + 2  # 3 layers x 3 matrices + lm_head + model.tbm
    got = run(BIN, model, str(tmp_path / "one"))
    assert sorted(got) == sorted(want)
    for name in want:
        assert got[name] == want[name], name
    if cuda.cuda.device_count() >= 2:
        got2 = run(BIN, model, str(tmp_path / "two"), "--gpus", "2")
        assert got2 == want


def test_gpus_flag_beyond_visible_devices_fails(cuda, tblib, tmp_path):
    model = str(tmp_path / "m.safetensors")
    inputs.small_model(model)
    r = subprocess.run([BIN, "--model", model, "--output", str(tmp_path / "o"), "--gpus",
                        str(cuda.cuda.device_count() + 1)], capture_output=True, text=True, timeout=300)
    assert r.returncode != 0

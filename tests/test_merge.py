"""tb-merge, the native .tbm merge (the reference's scripts/merge_tbm.py).

The runs of tests/inputs.MERGE_RUNS over the shard tree of
tests/inputs.merge_tree() must give the exit code, stdout and container bytes
that the reference script gave on the same tree (tests/golden/merge.json,
made by tests/golden/make_merge_golden.py).  No GPU is involved.
"""
import hashlib
import json
import os
import subprocess

import pytest

import inputs

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TB_MERGE = os.path.join(ROOT, "tensorbit-core_b200", "bin", "tb-merge")
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "merge.json")))


@pytest.fixture(scope="module")
def tb_merge():
    if not os.path.exists(TB_MERGE):
        import build
        build.build()
    return TB_MERGE


def run(exe, args, cwd):
    return subprocess.run([exe, *args], cwd=cwd, capture_output=True, text=True)


@pytest.mark.parametrize("key", sorted(inputs.MERGE_RUNS))
def test_merge_matches_reference_script(tb_merge, tmp_path, key):
    args, cwd = inputs.MERGE_RUNS[key]
    inputs.merge_tree(str(tmp_path))
    run_dir = tmp_path / cwd
    r = run(tb_merge, args, run_dir)
    gold = GOLD[key]
    assert r.returncode == gold["returncode"], r.stderr
    assert r.stdout == gold["stdout"]
    path = run_dir / args[args.index("--output") + 1]
    if "sha256" not in gold:
        assert not path.exists()
        return
    data = path.read_bytes()
    n = int.from_bytes(data[-4:], "little")
    assert json.loads(data[-4 - n:-4].decode("utf-8")) == gold["index"]
    assert len(data) == gold["size"]
    assert hashlib.sha256(data).hexdigest() == gold["sha256"]


def test_merge_container_holds_the_files(tb_merge, tmp_path):
    """Every tensor's bytes sit at its index offset while files match their
    headers; the index is compact ASCII JSON followed by its u32 length."""
    s1, s2 = inputs.merge_tree(str(tmp_path))
    for name in ("lm_head.weight.tb", "short_payload.tb"):  # sizes that disagree with their headers
        for d in (s1, s2):
            p = os.path.join(d, name)
            if os.path.exists(p):
                os.remove(p)
    out = tmp_path / "m.tbm"
    r = run(tb_merge, ["--input", s1, s2, "--output", str(out)], tmp_path)
    assert r.returncode == 0, r.stderr
    data = out.read_bytes()
    n = int.from_bytes(data[-4:], "little")
    raw = data[-4 - n:-4]
    assert raw.isascii() and b", " not in raw and b": " not in raw
    index = json.loads(raw)
    assert index["config"]["num_layers"] == len(index["tensors"])
    files = {}
    for d in (s1, s2):
        for f in sorted(os.listdir(d)):
            if f.endswith(".tb"):
                files.setdefault(f[:-3].replace(".tbm", "").replace(".tb", ""), os.path.join(d, f))
    for t in index["tensors"]:
        blob = open(files[t["name"]], "rb").read()
        assert data[t["offset"]:t["offset"] + len(blob)] == blob
        assert len(blob) == 4096 + 4 * t["num_weights"] + t["num_mask_bytes"]


def test_merge_rejects_control_characters_before_writing(tb_merge, tmp_path):
    inputs.merge_tree(str(tmp_path))
    inputs._tb_file(str(tmp_path / "shard1" / "bad\x01name.tb"), 2, 4, 8, 2, 0, 1)
    r = run(tb_merge, ["--input", "shard1", "--output", "o.tbm"], tmp_path)
    assert r.returncode == 1
    assert "unprintable char 0x01" in r.stderr
    assert not (tmp_path / "o.tbm").exists()


@pytest.mark.parametrize("args", [[], ["--input", "shard1"], ["--output", "o.tbm"], ["--input", "--output", "o.tbm"],
                                  ["--input", "shard1", "--output"], ["--input", "shard1", "--output", "o", "--bogus"]])
def test_merge_command_line_errors(tb_merge, tmp_path, args):
    inputs.merge_tree(str(tmp_path))
    r = run(tb_merge, args, tmp_path)
    assert r.returncode == 2
    assert r.stderr.startswith("usage: tb-merge")
    assert not (tmp_path / "o.tbm").exists() and not (tmp_path / "o").exists()


def test_merge_abbreviated_and_inline_options(tb_merge, tmp_path):
    args, cwd = inputs.MERGE_RUNS["shards"]
    inputs.merge_tree(str(tmp_path))
    r = run(tb_merge, ["--in", "./shard1/", "shard2", "missing_dir", "--output=out/full/model.tbm", "--arch=llama"],
            tmp_path)
    assert r.returncode == 0
    assert r.stdout == GOLD["shards"]["stdout"]
    assert hashlib.sha256((tmp_path / "out/full/model.tbm").read_bytes()).hexdigest() == GOLD["shards"]["sha256"]

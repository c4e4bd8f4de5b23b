"""Regenerates the golden fixtures in this directory from the REFERENCE itself.

    make -C oracle ref && python tests/golden/make_golden.py

Runs the reference's own CPU code (oracle/_ref, compiled from the reference
sources) on the seeded inputs of tests/inputs.py and records its outputs:

* golden.json - sha256 digests of every output array of the small-tensor
  pass (weights 128x128 FP32, 8 gradient samples, OBD, 2:4) for each mask
  strategy, of the tb-prune mock run's .tb file, of the BF16/F16 decode of all
  65536 bit patterns, plus the documented pins (docs/TODO.md:101,
  docs/DOCUMENTATION.md:57-70), and of the files the reference tb-prune CLI
  writes for the mock variants of tests/inputs.MOCK_RUNS and for the mixed-dtype
  checkpoint of tests/inputs.small_model (one .tb per tensor + model.tbm).
  The BlockOBS run uses the reference built with the test-only Eigen stand-in.
* ties.npz - the reference's top-N masks for every 2:4-family weak-order
  pattern ({0..3}^4 for n = 1, 2, 3) and for 4096 random tie-heavy 8-element
  groups (n = 1, 2, 4, 6), the cases where std::nth_element's tie order decides.

The reference tree is needed only to run this script; the fixtures it writes
are committed and read by the CPU test suite on any machine.
"""
import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

from oracle import REF_CLI, Oracle  # noqa: E402
import inputs  # noqa: E402


def sha(a) -> str:
    if isinstance(a, (bytes, bytearray)):
        return hashlib.sha256(a).hexdigest()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    R = Oracle("ref")
    out = {"generator": "tests/golden/make_golden.py (reference CPU code via oracle/_ref)"}

    # The 128x128 tensor with 8 samples: score+mask+pack without the EHAP pre-prune.
    w, g = inputs.tensor_128x128_s8()
    small = {"inputs": {"w": sha(w), "g": sha(g)}}
    for strategy in ("topn", "optimal", "iterative"):
        rc, wp, mask, F, s, _, cp = R.pipeline(w, g, mode="obd", strategy=strategy, redist="proportional")
        assert rc == 0
        small[strategy] = {"w_out": sha(wp), "mask": sha(mask), "fisher": sha(F), "scores": sha(s),
                          "tb": sha(R.tb_bytes(wp, mask, 2, 4)), "coring_pruned": cp,
                          "mask_head": mask[:16].tolist()}
    for mode in ("obs", "normalized"):
        rc, wp, mask, F, s, _, cp = R.pipeline(w, g, mode=mode, strategy="optimal", redist="proportional")
        assert rc == 0
        small["optimal_" + mode] = {"w_out": sha(wp), "mask": sha(mask), "scores": sha(s)}
    # tb-prune mode: EHAP one-shot global pre-prune, then CORING top-N.
    rc, wp, mask, F, s, ep, cp = R.pipeline(w, g, mode="obd", ehap_strategy="oneshot", strategy="topn")
    assert rc == 0
    small["tbprune_oneshot_topn"] = {"w_out": sha(wp), "mask": sha(mask), "scores": sha(s),
                                    "ehap_pruned": ep, "coring_pruned": cp}
    out["tensor_128x128_s8"] = small

    # tb-prune --mock-size 16384 --sparsity 2:4 (docs/DOCUMENTATION.md:57-70).
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "mock.tb")
        subprocess.run([REF_CLI, "--mock-size", "16384", "--sparsity", "2:4", "--output", path],
                       check=True, capture_output=True)
        data = open(path, "rb").read()
        out["tb_prune_mock_16384"] = {"size": len(data), "sha256": sha(data),
                                      "header_sha256": sha(data[:4096]),
                                      "mask_sha256": sha(data[4096 + 16384 * 4:])}
    mw, mg = R.mock_tensor(16384)
    out["mock_tensor_16384"] = {"w": sha(mw), "g": sha(mg)}

    # Documented pin: importance [5,1,4,2] -> mask 0b0101 (docs/TODO.md:101).
    out["todo_pin"] = {s: int(R.nm_mask(np.array([5, 1, 4, 2], np.float32), 2, 4, s)[1][0])
                       for s in ("topn", "optimal", "iterative")}

    # Half-precision decode of every bit pattern (src/main.cpp:213-245).
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out["decode_sha256"] = {"bf16": sha(R.decode_half(bits, True)), "f16": sha(R.decode_half(bits, False))}

    # Error behaviour of generate_nm_mask (coring.hpp:94-100,321-330).
    cases = [(0, 0, 2, 4), (8, 4, 2, 4), (6, 6, 2, 4), (8, 8, 4, 4), (8, 8, 0, 4), (8, 8, 2, 0)]
    out["mask_status"] = [[*c, R.nm_mask_status(*c)] for c in cases]

    # tb-prune runs of the reference CLI: mock variants and a real-mode checkpoint.
    runs = {}
    with tempfile.TemporaryDirectory() as d:
        for key, args in inputs.MOCK_RUNS.items():
            path = os.path.join(d, key + ".tb")
            subprocess.run([REF_CLI, *args, "--output", path], check=True, capture_output=True)
            runs[key] = sha(open(path, "rb").read())
        model = os.path.join(d, "model.safetensors")
        inputs.small_model(model)
        outdir = os.path.join(d, "out")
        subprocess.run([REF_CLI, "--model", model, "--output", outdir], check=True, capture_output=True)
        real = {name: sha(open(os.path.join(outdir, name), "rb").read()) for name in sorted(os.listdir(outdir))}
    out["tb_prune_mock_runs"] = runs
    out["tb_prune_real_small_model"] = real

    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)

    # Tie patterns.
    pats4 = np.array(np.meshgrid(*[np.arange(4)] * 4, indexing="ij")).reshape(4, -1).T[:, ::-1].astype(np.float32)
    masks4 = {}
    for n in (1, 2, 3):
        rc, mk = R.nm_mask(pats4.reshape(-1).copy(), n, 4, "topn")
        assert rc == 0
        masks4[n] = mk
    rng = np.random.default_rng(7)
    pats8 = rng.integers(0, 4, (4096, 8)).astype(np.float32)
    masks8 = {}
    for n in (1, 2, 4, 6):
        rc, mk = R.nm_mask(pats8.reshape(-1).copy(), n, 8, "topn")
        assert rc == 0
        masks8[n] = mk
    np.savez(os.path.join(HERE, "ties.npz"), pats4=pats4, pats8=pats8,
             **{f"m4_n{n}": v for n, v in masks4.items()}, **{f"m8_n{n}": v for n, v in masks8.items()})
    print("wrote golden.json and ties.npz")


if __name__ == "__main__":
    main()

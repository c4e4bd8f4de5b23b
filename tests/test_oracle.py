"""CPU: the port oracle is pinned to the reference's outputs.

Two pins: the committed golden fixtures (made by tests/golden/make_golden.py
from the reference's own compiled CPU code), checked everywhere; and, where the
reference tree was present at build time, a live differential run against the
reference (oracle/_ref) on many random and tie-heavy cases.
"""
import hashlib
import json
import os

import numpy as np
import pytest

import inputs

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))
TIES = np.load(os.path.join(os.path.dirname(__file__), "golden", "ties.npz"))


def sha(a):
    if isinstance(a, (bytes, bytearray)):
        return hashlib.sha256(a).hexdigest()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and a.tobytes() == b.tobytes()


# --- golden fixtures --------------------------------------------------------

def test_inputs_are_the_fixture_inputs():
    w, g = inputs.tensor_128x128_s8()
    assert sha(w) == GOLD["tensor_128x128_s8"]["inputs"]["w"]
    assert sha(g) == GOLD["tensor_128x128_s8"]["inputs"]["g"]


@pytest.mark.parametrize("strategy", ["topn", "optimal", "iterative"])
def test_128x128_pass_matches_golden(port, strategy):
    w, g = inputs.tensor_128x128_s8()
    rc, wp, mask, F, s, _, cp = port.pipeline(w, g, mode="obd", strategy=strategy, redist="proportional")
    gold = GOLD["tensor_128x128_s8"][strategy]
    assert rc == 0
    assert sha(F) == gold["fisher"]
    assert sha(s) == gold["scores"]
    assert sha(mask) == gold["mask"]
    assert sha(wp) == gold["w_out"]
    assert cp == gold["coring_pruned"]
    assert sha(port.tb_bytes(wp, mask, 2, 4)) == gold["tb"]


@pytest.mark.parametrize("mode", ["obs", "normalized"])
def test_128x128_modes_match_golden(port, mode):
    w, g = inputs.tensor_128x128_s8()
    rc, wp, mask, F, s, _, _ = port.pipeline(w, g, mode=mode, strategy="optimal", redist="proportional")
    gold = GOLD["tensor_128x128_s8"]["optimal_" + mode]
    assert rc == 0 and sha(s) == gold["scores"] and sha(mask) == gold["mask"] and sha(wp) == gold["w_out"]


def test_tbprune_oneshot_matches_golden(port):
    w, g = inputs.tensor_128x128_s8()
    rc, wp, mask, F, s, ep, cp = port.pipeline(w, g, mode="obd", ehap_strategy="oneshot", strategy="topn")
    gold = GOLD["tensor_128x128_s8"]["tbprune_oneshot_topn"]
    assert rc == 0 and ep == gold["ehap_pruned"] and cp == gold["coring_pruned"]
    assert sha(s) == gold["scores"] and sha(mask) == gold["mask"] and sha(wp) == gold["w_out"]


def test_tb_prune_mock_file_matches_golden(port):
    """The port reproduces tb-prune --mock-size 16384 --sparsity 2:4 byte for byte
    (src/main.cpp:366-418; 73,728 bytes per docs/DOCUMENTATION.md:57-70)."""
    w, g = port.mock_tensor(16384)
    assert sha(w) == GOLD["mock_tensor_16384"]["w"] and sha(g) == GOLD["mock_tensor_16384"]["g"]
    rc, wp, mask, F, s, ep, cp = port.pipeline(w, g[None, :], alpha=0.01, mode="obd",
                                               ehap_strategy="oneshot", strategy="topn",
                                               redist="proportional")
    assert rc == 0 and ep == 8192 and cp == 8192
    data = port.tb_bytes(wp, mask, 2, 4)
    gold = GOLD["tb_prune_mock_16384"]
    assert len(data) == gold["size"] == 73728
    assert sha(data[:4096]) == gold["header_sha256"]
    assert sha(data[4096 + 16384 * 4:]) == gold["mask_sha256"]
    assert sha(data) == gold["sha256"]


def test_documented_mask_pin(port):
    """docs/TODO.md:101: importance [5,1,4,2] -> mask 0b0101."""
    for strategy in ("topn", "optimal", "iterative"):
        rc, mk = port.nm_mask(np.array([5, 1, 4, 2], np.float32), 2, 4, strategy)
        assert rc == 0 and int(mk[0]) == GOLD["todo_pin"][strategy] == 0b0101


def test_decode_matches_golden(port):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    assert sha(port.decode_half(bits, True)) == GOLD["decode_sha256"]["bf16"]
    assert sha(port.decode_half(bits, False)) == GOLD["decode_sha256"]["f16"]


def test_mask_error_codes_match_golden(port):
    for ns, nm, n, m, code in GOLD["mask_status"]:
        assert port.nm_mask_status(ns, nm, n, m) == code


@pytest.mark.parametrize("n", [1, 2, 3])
def test_topn_ties_2_4_family(port, n):
    pats = TIES["pats4"]
    rc, mk = port.nm_mask(pats.reshape(-1).copy(), n, 4, "topn")
    assert rc == 0 and same(mk, TIES[f"m4_n{n}"])


@pytest.mark.parametrize("n", [1, 2, 4, 6])
def test_topn_ties_m8(port, n):
    pats = TIES["pats8"]
    rc, mk = port.nm_mask(pats.reshape(-1).copy(), n, 8, "topn")
    assert rc == 0 and same(mk, TIES[f"m8_n{n}"])


def test_ties_differ_from_lowest_index(port):
    """The reference's top-N does not break ties by lowest index: the golden
    table must contain patterns where it keeps a higher index."""
    pats = TIES["pats4"]
    mk = TIES["m4_n2"]
    lowest = []
    for p in pats:
        order = sorted(range(4), key=lambda i: (-p[i], i))
        lowest.append((1 << order[0]) | (1 << order[1]))
    assert (np.array(lowest) != mk).sum() == 88


# --- live differential run against the reference -----------------------------

CASES_NM = [(2, 4), (1, 4), (3, 4), (2, 8), (4, 8), (1, 8), (6, 8), (1, 2), (2, 3), (3, 7), (2, 5), (3, 6)]


@pytest.mark.parametrize("n,m", CASES_NM)
@pytest.mark.parametrize("strategy", ["topn", "optimal", "iterative"])
@pytest.mark.parametrize("permute", [False, True])
def test_port_vs_reference_masks(port, ref, n, m, strategy, permute):
    rng = np.random.default_rng(n * 100 + m)
    for kind in range(3):
        N = m * 1500
        if kind == 0:
            s = rng.random(N).astype(np.float32)
        elif kind == 1:
            s = rng.integers(0, 4, N).astype(np.float32)
        else:
            s = rng.integers(-3, 4, N).astype(np.float32)
        a = port.nm_mask(s, n, m, strategy, 3, permute)
        b = ref.nm_mask(s, n, m, strategy, 3, permute)
        assert a[0] == b[0] and same(a[1], b[1])


@pytest.mark.parametrize("mode", ["obd", "obs", "normalized"])
@pytest.mark.parametrize("use_fisher", [True, False])
@pytest.mark.parametrize("normalize", [False, True])
def test_port_vs_reference_importance(port, ref, mode, use_fisher, normalize):
    g = inputs.normal((5, 3000), 1e-3, 3)
    w = inputs.normal(3000, 0.02, 4)
    a = port.importance(g, w, mode=mode, use_fisher=use_fisher, normalize=normalize)
    b = ref.importance(g, w, mode=mode, use_fisher=use_fisher, normalize=normalize)
    assert a[0] == b[0] and same(a[1], b[1])


@pytest.mark.parametrize("redist", ["none", "proportional", "uniform"])
def test_port_vs_reference_redistribution(port, ref, redist):
    rng = np.random.default_rng(11)
    s = rng.random(4000).astype(np.float32)
    w = rng.standard_normal(4000).astype(np.float32)
    mk = rng.integers(0, 16, 1000).astype(np.uint8)
    for do_apply in (0, 1):
        a = port.apply_redistribute(w, mk, s, 2, 4, redist, do_apply)
        b = ref.apply_redistribute(w, mk, s, 2, 4, redist, do_apply)
        assert a[0] == b[0] and same(a[1], b[1]) and a[2] == b[2]


@pytest.mark.parametrize("sp", [0.5, 0.3, 0.9, 1e-4, 0.99999, 1.0, 0.0])
def test_port_vs_reference_select(port, ref, sp):
    s = np.random.default_rng(5).integers(0, 50, 3001).astype(np.float32)
    a = port.select_mask(s, sp)
    b = ref.select_mask(s, sp)
    assert a[0] == b[0] and same(a[1], b[1]) and a[2] == b[2]


@pytest.mark.parametrize("ehap", [None, "oneshot", "iterative"])
@pytest.mark.parametrize("strategy", ["topn", "optimal", "iterative"])
@pytest.mark.parametrize("mode", ["obd", "obs", "normalized"])
def test_port_vs_reference_pipeline(port, ref, ehap, strategy, mode):
    w = inputs.normal(4096, 0.02, 21)
    g = inputs.normal((3, 4096), 1e-3, 22)
    a = port.pipeline(w, g, mode=mode, ehap_strategy=ehap, strategy=strategy)
    b = ref.pipeline(w, g, mode=mode, ehap_strategy=ehap, strategy=strategy)
    assert a[0] == b[0] and a[5:] == b[5:]
    for x, y in zip(a[1:5], b[1:5]):
        assert same(x, y)


def test_port_vs_reference_tie_heavy_pipeline(port, ref):
    w, g = inputs.tie_heavy(8192, 3, 9)
    for ehap in (None, "oneshot"):
        for strategy in ("topn", "iterative", "optimal"):
            a = port.pipeline(w, g, ehap_strategy=ehap, strategy=strategy)
            b = ref.pipeline(w, g, ehap_strategy=ehap, strategy=strategy)
            assert a[0] == b[0] and a[5:] == b[5:]
            for x, y in zip(a[1:5], b[1:5]):
                assert same(x, y)


@pytest.mark.parametrize("N,block,K,S,use_fisher,sp", [
    (1024, 128, 4, 1, True, 0.5), (1000, 128, 4, 2, True, 0.5), (4096, 128, 0, 1, True, 0.5),
    (2048, 64, 2, 3, True, 0.3), (777, 100, 4, 1, True, 0.5), (4096, 128, 4, 1, False, 0.5),
    (5000, 224, 3, 1, True, 0.7), (3000, 32, 1, 1, True, 0.9)])
def test_port_vs_reference_block_obs(port, ref, N, block, K, S, use_fisher, sp):
    w = inputs.normal(N, 0.5, N)
    g = inputs.normal((S, N), 0.05, N + 1)
    hist = (np.stack([g[0] * (np.float32(0.9) + np.float32(0.02) * np.float32(k)) for k in range(K)])
            .astype(np.float32) if K else None)
    a = port.block_obs(w, g, hist, block=block, sparsity=sp, use_fisher=use_fisher, hist_size=max(K, 1))
    b = ref.block_obs(w, g, hist, block=block, sparsity=sp, use_fisher=use_fisher, hist_size=max(K, 1))
    assert a[0] == b[0] == 0 and a[2] == b[2] and same(a[1], b[1])


def test_sparsegpt_torch_rows_equal_the_numpy_restatement():
    """The float64 sweep written with torch (used on the device for the full
    4096 x 14336 layer) equals the numpy restatement on a small layer."""
    import torch
    import sparsegpt_ref as sref
    X = inputs.activations(192, 256, 5)
    W = inputs.normal(48 * 256, 0.02, 6).reshape(48, 256)
    Wn, mn, U, gn = sref.sparsegpt(W, X, 0.01, 2, 4, 128)
    Wt, mt, gt = sref.sparsegpt_rows_torch(torch, torch.from_numpy(W.astype(np.float64)),
                                           torch.from_numpy(U), 2, 4, 128)
    assert np.array_equal(mt.numpy(), mn)
    np.testing.assert_allclose(Wt.numpy(), Wn, rtol=0, atol=1e-12)
    np.testing.assert_allclose(gt.numpy(), gn, rtol=1e-9, atol=1e-12)

"""GPU: tb_prune_one_shot_nm, tb-prune's per-tensor sequence in three device
passes (Fisher + scores, global radix select, threshold + CORING + pack),
against the oracle's restatement of the same sequence (EHAPPruner one-shot
then CORINGPruner::prune and generate_nm_mask, src/main.cpp:372-409).

Bar: bit-exact pruned weights, masks, Fisher state and final scores, the same
EHAP pruned count; and the tb-prune mock file byte-identical to the
reference's golden digest.
"""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))
STRATS = ["topn", "optimal", "iterative"]


def one_shot(torch, tb, w, g, *, n=2, m=4, strategy="topn", mode="obd", use_fisher=True, sparsity=0.5,
             damping=0.01):
    N = w.size
    S = g.shape[0] if g is not None else 0
    wd = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    gd = torch.from_numpy(np.ascontiguousarray(g)).cuda() if S else None
    wo = torch.full((N,), float("nan"), device="cuda")
    mk = torch.full((N // m,), 0xAA, dtype=torch.uint8, device="cuda")
    F = torch.full((N,), float("nan"), device="cuda")
    s = torch.full((N,), float("nan"), device="cuda")
    a = tb.prune_args(weights=wd.data_ptr(), w_dtype=tb.F32, grads=gd.data_ptr() if S else None, g_dtype=tb.F32,
                      S=S, N=N, damping=damping, mode=mode, use_fisher=use_fisher, n=n, m=m, strategy=strategy,
                      redist="proportional", w_out=wo.data_ptr(), mask_out=mk.data_ptr(), fisher_out=F.data_ptr(),
                      scores_out=s.data_ptr())
    thr, ep, cp = C.c_float(), C.c_uint64(), C.c_uint64()
    rc = tb.lib().tb_prune_one_shot_nm(C.byref(a), sparsity, C.byref(thr), C.byref(ep), C.byref(cp), None)
    torch.cuda.synchronize()
    return rc, wo.cpu().numpy(), mk.cpu().numpy(), F.cpu().numpy(), s.cpu().numpy(), ep.value, cp.value


def check(torch, tb, port, w, g, **kw):
    rc, wo, mk, F, s, ep, cp = one_shot(torch, tb, w, g, **kw)
    assert rc == 0, tb.lib().tb_last_error()
    o = port.pipeline(w, g if g is not None else np.zeros((0, w.size), np.float32), ehap_strategy="oneshot", n=kw.get("n", 2), m=kw.get("m", 4),
                      strategy=kw.get("strategy", "topn"), mode=kw.get("mode", "obd"),
                      use_fisher=kw.get("use_fisher", True), sparsity=kw.get("sparsity", 0.5),
                      redist="proportional")
    orc, owp, omk, oF, os_, oep, ocp = o
    assert orc == 0
    assert wo.tobytes() == owp.tobytes(), "pruned weights differ"
    assert mk.tobytes() == omk.tobytes(), "masks differ"
    assert s.tobytes() == os_.tobytes(), "final scores differ"
    if kw.get("use_fisher", True):
        assert F.tobytes() == oF.tobytes(), "Fisher state differs"
    assert ep == oep and cp == ocp
    return ep


@pytest.mark.parametrize("strategy", STRATS)
@pytest.mark.parametrize("n,m", [(2, 4), (1, 4), (2, 8), (4, 8)])
def test_one_shot_nm_matches_oracle(cuda, tblib, port, strategy, n, m):
    w = inputs.normal(65536, 0.02, 60 + m)
    g = inputs.normal((3, 65536), 1e-3, 61)
    check(cuda, tblib, port, w, g, n=n, m=m, strategy=strategy)


@pytest.mark.parametrize("mode", ["obd", "obs", "normalized"])
@pytest.mark.parametrize("sparsity", [0.5, 0.3, 0.9])
def test_one_shot_nm_modes_and_sparsities(cuda, tblib, port, mode, sparsity):
    w = inputs.normal(200_000, 0.02, 70)
    g = inputs.normal((2, 200_000), 1e-3, 71)
    check(cuda, tblib, port, w, g, mode=mode, sparsity=sparsity)


def test_one_shot_nm_magnitude_method(cuda, tblib, port):
    # tb-prune --method Magnitude: no Fisher state, scores w*w
    w = inputs.normal(100_000, 0.02, 72)
    check(cuda, tblib, port, w, None, use_fisher=False)


@pytest.mark.parametrize("strategy", STRATS)
def test_one_shot_nm_ties_and_ragged_tail(cuda, tblib, port, strategy):
    # tie-heavy scores (many equal to the threshold: all kept) and N not a
    # multiple of 16, so the scalar kernel handles the tail
    w, g = inputs.tie_heavy(40_004, 2, 73)
    check(cuda, tblib, port, w, g, strategy=strategy)


def test_one_shot_nm_mock_file_byte_identical(cuda, tblib, port):
    """tb-prune --mock-size 16384 --sparsity 2:4 through the fused sequence
    gives the reference's .tb file byte for byte (73,728 bytes)."""
    w, g = port.mock_tensor(16384)
    rc, wo, mk, F, s, ep, cp = one_shot(cuda, tblib, w, g[None, :])
    assert rc == 0 and ep == 8192 and cp == 8192
    data = port.tb_bytes(wo, mk, 2, 4)
    assert len(data) == 73728
    assert hashlib.sha256(data).hexdigest() == GOLD["tb_prune_mock_16384"]["sha256"]


def test_one_shot_nm_checks_sparsity_before_nm(cuda, tblib):
    w = np.zeros(64, np.float32)
    for sp in (0.0, 1.0, -0.5):
        rc = one_shot(cuda, tblib, w, None, use_fisher=False, sparsity=sp, n=4, m=4)[0]
        assert rc == tblib.TB_ERR_CONFIG
    assert one_shot(cuda, tblib, w, None, use_fisher=False, n=4, m=4)[0] == tblib.TB_ERR_CONFIG  # N:M 4:4
    assert one_shot(cuda, tblib, np.zeros(66, np.float32), None, use_fisher=False)[0] == tblib.TB_ERR_SHAPE


@pytest.mark.parametrize("N,sparsity", [(200_000, 0.5), (200_000, 0.9), (3 << 20, 0.1)])
def test_one_shot_nm_async_equals_sync(cuda, tblib, N, sparsity):
    """The async entry writes the same tensors as the synchronous one and its
    stream-ordered threshold / EHAP count (one to device memory, one to pinned
    host memory) equal the synchronous host values."""
    torch, tb = cuda, tblib
    w = inputs.normal(N, 0.02, 90)
    g = inputs.normal((2, N), 1e-3, 91)
    wd = torch.from_numpy(w).cuda()
    gd = torch.from_numpy(g).cuda()
    outs = []
    for variant in ("sync", "async"):
        wo = torch.full((N,), float("nan"), device="cuda")
        mk = torch.full((N // 4,), 0xAA, dtype=torch.uint8, device="cuda")
        F = torch.full((N,), float("nan"), device="cuda")
        s = torch.full((N,), float("nan"), device="cuda")
        a = tb.prune_args(weights=wd.data_ptr(), w_dtype=tb.F32, grads=gd.data_ptr(), g_dtype=tb.F32, S=2, N=N,
                          mode="obd", strategy="topn", redist="proportional", w_out=wo.data_ptr(),
                          mask_out=mk.data_ptr(), fisher_out=F.data_ptr(), scores_out=s.data_ptr())
        cp = C.c_uint64()
        if variant == "sync":
            thr, ep = C.c_float(), C.c_uint64()
            rc = tb.lib().tb_prune_one_shot_nm(C.byref(a), sparsity, C.byref(thr), C.byref(ep), C.byref(cp), None)
            counts = (thr.value, ep.value)
        else:
            dthr = torch.full((1,), float("nan"), device="cuda")
            hcnt = torch.full((1,), -1, dtype=torch.int64).pin_memory()  # pinned host destination
            rc = tb.lib().tb_prune_one_shot_nm_async(C.byref(a), sparsity, dthr.data_ptr(), hcnt.data_ptr(),
                                                     C.byref(cp), None)
            torch.cuda.synchronize()
            counts = (float(dthr.item()), int(hcnt.item()))
        assert rc == 0, tb.lib().tb_last_error()
        torch.cuda.synchronize()
        outs.append((wo.cpu().numpy().tobytes(), mk.cpu().numpy().tobytes(), F.cpu().numpy().tobytes(),
                     s.cpu().numpy().tobytes(), counts, cp.value))
    assert outs[0] == outs[1]
    assert outs[0][4][1] > 0

"""GPU parity of the EHAP stages (global threshold select, 1-byte mask apply,
Fisher normalisation, compensation) and of the whole tb-prune per-tensor
sequence composed from the C-ABI stage entries.

Bar: bit-exact against the oracle; the tb-prune mock run must reproduce the
reference's 73,728-byte .tb file byte for byte.
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


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def select(torch, tb, s, sp):
    sd = dev(torch, s)
    mask = torch.full((max(s.size, 1),), 7, dtype=torch.uint8, device="cuda")
    thr, pruned = C.c_float(-1), C.c_uint64(0)
    rc = tb.lib().tb_threshold_select(sd.data_ptr(), s.size, sp, mask.data_ptr(), C.byref(thr), C.byref(pruned), None)
    return rc, mask.cpu().numpy()[: s.size], thr.value, pruned.value


SCORES = {
    "uniform": lambda n, r: r.random(n).astype(np.float32),
    "ties": lambda n, r: r.integers(0, 50, n).astype(np.float32),
    "zeros": lambda n, r: np.where(r.random(n) < 0.6, 0.0, r.random(n)).astype(np.float32),
    "signed": lambda n, r: np.where(r.random(n) < 0.5, -0.0, 1.0).astype(np.float32) * r.integers(-3, 4, n),
    "tiny": lambda n, r: (r.random(n) * 1e-38).astype(np.float32),
}


@pytest.mark.parametrize("kind", list(SCORES))
@pytest.mark.parametrize("N", [1, 2, 3, 1000, 65536, 1 << 20, 3000017])
@pytest.mark.parametrize("sp", [0.5, 0.3, 0.9, 1e-4, 0.99999])
def test_threshold_select_matches_oracle(cuda, tblib, port, kind, N, sp):
    rng = np.random.default_rng(N)
    s = np.ascontiguousarray(SCORES[kind](N, rng), np.float32)
    rc, mask, thr, pruned = select(cuda, tblib, s, sp)
    rco, masko, prunedo = port.select_mask(s, sp)
    assert rc == 0 and rco == 0
    assert mask.tobytes() == masko.tobytes()
    assert pruned == prunedo
    keep = max(1, int(np.float32(sp) * np.float32(N)))
    if keep < N:
        assert thr == np.partition(s, N - keep)[N - keep]


def test_threshold_select_errors(cuda, tblib):
    s = np.ones(16, np.float32)
    for sp in (0.0, 1.0, -0.5, 2.0):
        assert select(cuda, tblib, s, sp)[0] == tblib.TB_ERR_CONFIG
    assert select(cuda, tblib, np.zeros(0, np.float32), 0.5)[0] == tblib.TB_ERR_ZERO_SIZE


def test_threshold_select_misaligned_scores(cuda, tblib, port):
    s = np.random.default_rng(3).random(100003).astype(np.float32)
    big = dev(cuda, np.concatenate([np.zeros(1, np.float32), s]))
    mask = cuda.empty(s.size, dtype=cuda.uint8, device="cuda")
    thr, pruned = C.c_float(), C.c_uint64()
    tblib.check(tblib.lib().tb_threshold_select(big.data_ptr() + 4, s.size, 0.5, mask.data_ptr(),
                                                C.byref(thr), C.byref(pruned), None))
    rco, masko, prunedo = port.select_mask(s, 0.5)
    assert mask.cpu().numpy().tobytes() == masko.tobytes() and pruned.value == prunedo


def test_ehap_apply_and_compensate(cuda, tblib, port):
    rng = np.random.default_rng(5)
    for N in (1, 7, 8, 1003, 65536 + 5):
        w = rng.standard_normal(N).astype(np.float32)
        s = rng.random(N).astype(np.float32)
        m = rng.integers(0, 2, N).astype(np.uint8)
        wd, md, sd = dev(cuda, w), dev(cuda, m), dev(cuda, s)
        cnt = C.c_uint64()
        tblib.check(tblib.lib().tb_ehap_apply_mask(wd.data_ptr(), md.data_ptr(), N, C.byref(cnt), None))
        wa = np.where(m == 0, np.float32(0), w).astype(np.float32)
        assert wd.cpu().numpy().tobytes() == wa.tobytes() and cnt.value == int((m == 0).sum())
        for mode in (0, 1, 2):
            wc = dev(cuda, wa)
            tblib.check(tblib.lib().tb_compensate(wc.data_ptr(), md.data_ptr(), sd.data_ptr(), N, mode, None))
            cuda.cuda.synchronize()
            assert wc.cpu().numpy().tobytes() == port.compensate(wa, m, s, mode).tobytes(), (N, mode)


def test_fisher_normalize_matches_oracle(cuda, tblib, port):
    L = tblib.lib()
    N = 200003
    g = inputs.normal((3, N), 1e-3, 7)
    w = inputs.normal(N, 0.02, 8)
    gd = dev(cuda, g)
    F = cuda.empty(N, dtype=cuda.float32, device="cuda")
    for k in range(3):
        tblib.check(L.tb_fisher_ema_step(F.data_ptr(), gd[k].data_ptr(), 0, N, 0.01, 0.99, int(k == 0), None))
    tblib.check(L.tb_fisher_normalize(F.data_ptr(), N, None))
    for mode in (0, 1, 2):
        s = cuda.empty(N, dtype=cuda.float32, device="cuda")
        wd = dev(cuda, w)
        tblib.check(L.tb_importance(wd.data_ptr(), 0, F.data_ptr(), s.data_ptr(), N, 0.01, mode, None))
        cuda.cuda.synchronize()
        rc, so = port.importance(g, w, mode=["obd", "obs", "normalized"][mode], normalize=True)
        assert s.cpu().numpy().tobytes() == so.tobytes()


def tb_prune_sequence(torch, tb, w, g, *, n=2, m=4, strategy=0, redist=1, sparsity=0.5, alpha=0.01,
                      beta=0.99, damping=0.01, mode=0):
    """tb-prune's per-tensor sequence (src/main.cpp:372-409) composed from the
    C-ABI stage entries, all on the device."""
    L = tb.lib()
    N = w.size
    S = g.shape[0]
    wd, gd = dev(torch, w), dev(torch, g)
    F = torch.empty(N, dtype=torch.float32, device="cuda")
    s = torch.empty(N, dtype=torch.float32, device="cuda")
    m1 = torch.empty(N, dtype=torch.uint8, device="cuda")
    for k in range(S):  # accumulate_fisher
        tb.check(L.tb_fisher_ema_step(F.data_ptr(), gd[k].data_ptr(), 0, N, alpha, beta, int(k == 0), None))
    # EHAPPruner::prune_one_shot: importance -> global threshold -> apply
    tb.check(L.tb_importance(wd.data_ptr(), 0, F.data_ptr(), s.data_ptr(), N, damping, mode, None))
    thr, ep = C.c_float(), C.c_uint64()
    tb.check(L.tb_threshold_select(s.data_ptr(), N, sparsity, m1.data_ptr(), C.byref(thr), C.byref(ep), None))
    ep2 = C.c_uint64()
    tb.check(L.tb_ehap_apply_mask(wd.data_ptr(), m1.data_ptr(), N, C.byref(ep2), None))
    # compute_importance on the pruned weights, then CORINGPruner::prune
    tb.check(L.tb_importance(wd.data_ptr(), 0, F.data_ptr(), s.data_ptr(), N, damping, mode, None))
    mk = torch.empty(N // m, dtype=torch.uint8, device="cuda")
    tb.check(L.tb_nm_mask(s.data_ptr(), mk.data_ptr(), N, n, m, strategy, 3, 0, None))
    tb.check(L.tb_apply_mask(wd.data_ptr(), mk.data_ptr(), N, m, None))
    tb.check(L.tb_redistribute(wd.data_ptr(), mk.data_ptr(), s.data_ptr(), N, m, redist, None))
    mk2 = torch.empty(N // m, dtype=torch.uint8, device="cuda")  # generate_nm_mask again for the .tb
    tb.check(L.tb_nm_mask(s.data_ptr(), mk2.data_ptr(), N, n, m, strategy, 3, 0, None))
    torch.cuda.synchronize()
    return wd.cpu().numpy(), mk2.cpu().numpy(), s.cpu().numpy(), F.cpu().numpy(), ep.value, ep2.value


def test_tb_prune_mock_file_byte_identical(cuda, tblib, port):
    """tb-prune --mock-size 16384 --sparsity 2:4 on the device reproduces the
    reference's .tb file byte for byte (73,728 bytes)."""
    w, g = port.mock_tensor(16384)
    wp, mask, s, F, ep, ep2 = tb_prune_sequence(cuda, tblib, w, g[None, :])
    assert ep == ep2 == 8192
    data = port.tb_bytes(wp, mask, 2, 4)
    gold = GOLD["tb_prune_mock_16384"]
    assert len(data) == 73728
    assert hashlib.sha256(data).hexdigest() == gold["sha256"]


@pytest.mark.parametrize("strategy", [0, 1, 2])
@pytest.mark.parametrize("n,m", [(2, 4), (1, 4), (2, 8), (4, 8)])
def test_tb_prune_sequence_matches_oracle(cuda, tblib, port, strategy, n, m):
    w = inputs.normal(65536, 0.02, 40 + m)
    g = inputs.normal((3, 65536), 1e-3, 41)
    wp, mask, s, F, ep, _ = tb_prune_sequence(cuda, tblib, w, g, n=n, m=m, strategy=strategy)
    rc, wo, mo, Fo, so, epo, cpo = port.pipeline(w, g, ehap_strategy="oneshot", n=n, m=m,
                                                 strategy=["topn", "optimal", "iterative"][strategy],
                                                 redist="proportional")
    assert rc == 0 and ep == epo
    assert wp.tobytes() == wo.tobytes() and mask.tobytes() == mo.tobytes() and s.tobytes() == so.tobytes()

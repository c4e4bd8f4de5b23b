"""GPU parity: the sm_100a kernels, called through the C ABI, against the oracle.

Bar: bit-exact.  Scores, Fisher state and pruned weights are compared as raw
FP32 bits, masks byte for byte (ties included), .tb images byte for byte.  The
oracle is the CPU restatement (oracle/tb_oracle.cpp), itself pinned to the
reference's outputs by tests/test_oracle.py; the 128x128 tensor's outputs are also
checked directly against the reference's golden digests.
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
TIES = np.load(os.path.join(os.path.dirname(__file__), "golden", "ties.npz"))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits_equal(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and a.tobytes() == b.tobytes()


def dev(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


def encode(torch, x_f32, dt):
    """Device tensor of dtype `dt` holding x, and the FP32 values the oracle must see."""
    if dt == "f32":
        return dev(torch, x_f32), x_f32, 0
    if dt == "bf16":
        b = inputs.to_bf16_bits(x_f32)
        return dev(torch, b.view(np.int16)), inputs.bf16_bits_to_f32(b), 2
    h = np.ascontiguousarray(x_f32, np.float32).astype(np.float16).view(np.uint16)
    from oracle import Oracle
    return dev(torch, h.view(np.int16)), Oracle("port").decode_half(h, False).reshape(h.shape), 1


def run_fused(torch, tb, w, g, *, wdt="f32", gdt="f32", n=2, m=4, strategy="optimal", mode="obd",
              redist="proportional", rounds=3, permute=False, use_fisher=True, alpha=0.01, beta=0.99,
              damping=0.01, fisher_in=None, steps_in=0, g_pad=0, w_offset=0, want_ties=True):
    N = w.size
    wt, w32, wcode = encode(torch, w, wdt)
    S = g.shape[0] if g is not None else 0
    if S:
        gp = np.zeros((S, N + g_pad), np.float32)
        gp[:, :N] = g
        gt, g32, gcode = encode(torch, gp, gdt)
        g32 = np.ascontiguousarray(g32.reshape(S, N + g_pad)[:, :N])
    else:
        gt, g32, gcode = None, np.zeros((0, N), np.float32), 0
    if w_offset:
        # Shift weights off 16-byte alignment to exercise the scalar kernel.
        big = torch.zeros(wt.numel() + w_offset, dtype=wt.dtype, device="cuda")
        big[w_offset:] = wt
        wt = big[w_offset:]
    w_out = torch.empty(N, dtype=torch.float32, device="cuda")
    mask = torch.empty(N // m, dtype=torch.uint8, device="cuda")
    F = torch.full((N,), -1.0, dtype=torch.float32, device="cuda")
    s = torch.empty(N, dtype=torch.float32, device="cuda")
    ties = torch.zeros(1, dtype=torch.int64, device="cuda")
    fin = dev(torch, fisher_in) if fisher_in is not None else None
    a = tb.prune_args(weights=wt.data_ptr(), w_dtype=wcode, grads=gt.data_ptr() if S else None,
                      g_dtype=gcode, S=S, N=N, g_stride=(N + g_pad) if S else 0,
                      fisher_in=fin.data_ptr() if fin is not None else None, fisher_steps_in=steps_in,
                      alpha=alpha, beta=beta, damping=damping, mode=mode, use_fisher=use_fisher,
                      n=n, m=m, strategy=strategy, rounds=rounds, redist=redist, permute=permute,
                      w_out=w_out.data_ptr(), mask_out=mask.data_ptr(), fisher_out=F.data_ptr(),
                      scores_out=s.data_ptr(), near_ties=ties.data_ptr() if want_ties else None)
    rc = tb.score_mask_pack(a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    tb.check(rc)
    return dict(w_out=w_out.cpu().numpy(), mask=mask.cpu().numpy(), F=F.cpu().numpy(),
                s=s.cpu().numpy(), ties=int(ties.item()), w32=w32, g32=g32)


def oracle_pass(port, w32, g32, **kw):
    rc, wp, mask, F, s, _, cp = port.pipeline(w32, g32, **kw)
    assert rc == 0
    return wp, mask, F, s


# --- the 128x128 tensor against the reference's golden digests ---------------

@pytest.mark.parametrize("strategy", ["topn", "optimal", "iterative"])
def test_128x128_matches_reference_golden(cuda, tblib, port, strategy):
    w, g = inputs.tensor_128x128_s8()
    r = run_fused(cuda, tblib, w, g, strategy=strategy)
    gold = GOLD["tensor_128x128_s8"][strategy]
    assert sha(r["F"]) == gold["fisher"]
    assert sha(r["s"]) == gold["scores"]
    assert sha(r["mask"]) == gold["mask"]
    assert sha(r["w_out"]) == gold["w_out"]
    assert hashlib.sha256(port.tb_bytes(r["w_out"], r["mask"], 2, 4)).hexdigest() == gold["tb"]


@pytest.mark.parametrize("mode", ["obs", "normalized"])
def test_128x128_modes_match_reference_golden(cuda, tblib, mode):
    w, g = inputs.tensor_128x128_s8()
    r = run_fused(cuda, tblib, w, g, strategy="optimal", mode=mode)
    gold = GOLD["tensor_128x128_s8"]["optimal_" + mode]
    assert sha(r["s"]) == gold["scores"] and sha(r["mask"]) == gold["mask"] and sha(r["w_out"]) == gold["w_out"]


# --- fused pass against the oracle ---------------------------------------------

def check_against_oracle(port, r, *, n=2, m=4, strategy="optimal", mode="obd", redist="proportional",
                         rounds=3, permute=False, use_fisher=True, alpha=0.01, beta=0.99, damping=0.01,
                         check_fisher=True):
    wp, mask, F, s = oracle_pass(port, r["w32"], r["g32"], n=n, m=m, strategy=strategy, mode=mode,
                                 redist=redist, rounds=rounds, permute=permute, use_fisher=use_fisher,
                                 alpha=alpha, beta=beta, damping=damping)
    assert bits_equal(r["s"], s), "scores differ"
    if check_fisher and use_fisher and r["g32"].shape[0]:
        assert bits_equal(r["F"], F), "Fisher state differs"
    assert bits_equal(r["mask"], mask), f"masks differ in {(r['mask'] != mask).sum()} groups"
    assert bits_equal(r["w_out"], wp), "pruned weights differ"
    assert r["ties"] == port.near_ties(s, n, m)


@pytest.mark.parametrize("wdt,gdt", [("f32", "f32"), ("bf16", "bf16"), ("f16", "f32"), ("bf16", "f32"),
                                     ("f32", "bf16"), ("f16", "f16")])
@pytest.mark.parametrize("strategy", ["topn", "optimal", "iterative"])
def test_dtypes_and_strategies(cuda, tblib, port, wdt, gdt, strategy):
    w = inputs.normal(4096 * 8, 0.02, 31)
    g = inputs.normal((7, 4096 * 8), 1e-3, 32)
    r = run_fused(cuda, tblib, w, g, wdt=wdt, gdt=gdt, strategy=strategy)
    check_against_oracle(port, r, strategy=strategy)


@pytest.mark.parametrize("mode", ["obd", "obs", "normalized"])
@pytest.mark.parametrize("redist", ["none", "proportional", "uniform"])
def test_modes_and_redistribution(cuda, tblib, port, mode, redist):
    w = inputs.normal(16384, 0.02, 41)
    g = inputs.normal((5, 16384), 1e-3, 42)
    r = run_fused(cuda, tblib, w, g, mode=mode, redist=redist, strategy="topn")
    check_against_oracle(port, r, mode=mode, redist=redist, strategy="topn")


@pytest.mark.parametrize("n,m", [(1, 2), (1, 4), (2, 4), (3, 4), (1, 8), (2, 8), (4, 8), (7, 8),
                                 (2, 3), (2, 5), (3, 6), (3, 7)])
@pytest.mark.parametrize("strategy", ["topn", "optimal", "iterative"])
def test_nm_patterns(cuda, tblib, port, n, m, strategy):
    N = m * 16 * 67
    w = inputs.normal(N, 0.02, 50 + m)
    g = inputs.normal((3, N), 1e-3, 60 + n)
    r = run_fused(cuda, tblib, w, g, n=n, m=m, strategy=strategy, rounds=4)
    check_against_oracle(port, r, n=n, m=m, strategy=strategy, rounds=4)


@pytest.mark.parametrize("n,m", [(2, 4), (1, 4), (2, 8), (4, 8)])
def test_70b_sweep_settings(cuda, tblib, port, n, m):
    """The 70B sweep's settings on a 256 x 8192 slice of a hidden-8192
    projection: BF16 weights, 32 BF16 gradient samples, OBS scores, iterative
    swap-refine with 4 passes, each of the sweep's patterns; bit-exact."""
    N = 256 * 8192
    w = inputs.normal(N, 0.02, 90 + m)
    g = inputs.normal((32, N), 1e-3, 91 + n)
    r = run_fused(cuda, tblib, w, g, wdt="bf16", gdt="bf16", n=n, m=m, strategy="iterative", mode="obs", rounds=4)
    check_against_oracle(port, r, n=n, m=m, strategy="iterative", mode="obs", rounds=4)


@pytest.mark.parametrize("n,m", [(2, 4), (1, 4), (2, 8), (4, 8)])
@pytest.mark.parametrize("strategy", ["topn", "iterative", "optimal"])
@pytest.mark.parametrize("permute", [False, True])
def test_tie_heavy_inputs(cuda, tblib, port, n, m, strategy, permute):
    """Many groups tie at the N-th score (zeros, repeated magnitudes): the top-N
    choice must follow the reference's std::nth_element, not lowest index."""
    w, g = inputs.tie_heavy(8192 * m // 4, 3, 70 + m)
    r = run_fused(cuda, tblib, w, g, n=n, m=m, strategy=strategy, permute=permute)
    check_against_oracle(port, r, n=n, m=m, strategy=strategy, permute=permute)
    assert r["ties"] > 0


def test_permutation_with_signed_scores(cuda, tblib, port):
    """Permuted groups are sorted by |s|; with scores of mixed sign the stable
    order decides.  Scores come from the weights alone when the Fisher is off
    (s = w*w >= 0), so signed scores are fed through the standalone mask entry."""
    rng = np.random.default_rng(3)
    s = rng.integers(-3, 4, 8 * 4000).astype(np.float32)
    for (n, m) in [(2, 4), (4, 8), (2, 8)]:
        for strategy in ("topn", "optimal", "iterative"):
            st = dev(cuda, s)
            out = cuda.empty(s.size // m, dtype=cuda.uint8, device="cuda")
            tblib.check(tblib.lib().tb_nm_mask(st.data_ptr(), out.data_ptr(), s.size, n, m,
                                               tblib.STRATEGY[strategy], 3, 1, None))
            cuda.cuda.synchronize()
            rc, mk = port.nm_mask(s, n, m, strategy, 3, True)
            assert rc == 0 and bits_equal(out.cpu().numpy(), mk)


def test_no_fisher_and_no_samples(cuda, tblib, port):
    w = inputs.normal(8192, 0.02, 80)
    g = inputs.normal((4, 8192), 1e-3, 81)
    r = run_fused(cuda, tblib, w, g, use_fisher=False)
    check_against_oracle(port, r, use_fisher=False)
    assert (r["F"] == -1.0).all()  # no Fisher state is written when the Fisher is off
    r = run_fused(cuda, tblib, w, None)
    check_against_oracle(port, r)


def test_fisher_continuation_equals_single_pass(cuda, tblib):
    """Splitting the samples over two calls (fisher_in / fisher_steps_in) gives the
    same bits as one call: the EMA recurrence is continued, not restarted."""
    w = inputs.normal(16384, 0.02, 90)
    g = inputs.normal((9, 16384), 1e-3, 91)
    full = run_fused(cuda, tblib, w, g)
    part = run_fused(cuda, tblib, w, g[:4])
    rest = run_fused(cuda, tblib, w, g[4:], fisher_in=part["F"], steps_in=4)
    assert bits_equal(rest["F"], full["F"]) and bits_equal(rest["mask"], full["mask"])
    assert bits_equal(rest["w_out"], full["w_out"]) and bits_equal(rest["s"], full["s"])


@pytest.mark.parametrize("g_pad,w_offset", [(8, 0), (3, 0), (0, 1), (0, 2)])
def test_strides_and_misalignment(cuda, tblib, port, g_pad, w_offset):
    """Row-strided gradients and weights off 16-byte alignment take the scalar
    path; results must not change."""
    w = inputs.normal(4096, 0.02, 100)
    g = inputs.normal((5, 4096), 1e-3, 101)
    r = run_fused(cuda, tblib, w, g, g_pad=g_pad, w_offset=w_offset)
    check_against_oracle(port, r)


@pytest.mark.parametrize("N", [4, 8, 12, 16, 20, 4100, 65540])
def test_ragged_sizes(cuda, tblib, port, N):
    w = inputs.normal(N, 0.02, N)
    g = inputs.normal((3, N), 1e-3, N + 1)
    r = run_fused(cuda, tblib, w, g, strategy="topn")
    check_against_oracle(port, r, strategy="topn")


def test_error_codes(cuda, tblib):
    t = cuda.zeros(64, dtype=cuda.float32, device="cuda")
    mk = cuda.zeros(64, dtype=cuda.uint8, device="cuda")
    base = dict(weights=t.data_ptr(), w_dtype=0, grads=t.data_ptr(), g_dtype=0, S=1, N=64,
                w_out=t.data_ptr(), mask_out=mk.data_ptr())
    assert tblib.score_mask_pack(tblib.prune_args(**{**base, "N": 0})) == tblib.TB_ERR_ZERO_SIZE
    assert tblib.score_mask_pack(tblib.prune_args(**{**base, "N": 62})) == tblib.TB_ERR_SHAPE
    assert tblib.score_mask_pack(tblib.prune_args(**{**base, "n": 4, "m": 4})) == tblib.TB_ERR_CONFIG
    assert tblib.score_mask_pack(tblib.prune_args(**{**base, "n": 0})) == tblib.TB_ERR_CONFIG
    assert tblib.score_mask_pack(tblib.prune_args(**{**base, "m": 16})) == tblib.TB_ERR_UNSUPPORTED
    assert tblib.score_mask_pack(tblib.prune_args(**{**base, "grads": None})) == tblib.TB_ERR_ARG


# --- stage entry points and legacy launchers ------------------------------------

@pytest.mark.parametrize("n", [1, 2, 3])
def test_mask_entry_all_2_4_tie_patterns(cuda, tblib, n):
    pats = TIES["pats4"].reshape(-1).copy()
    st = dev(cuda, pats)
    out = cuda.empty(pats.size // 4, dtype=cuda.uint8, device="cuda")
    tblib.check(tblib.lib().tb_nm_mask(st.data_ptr(), out.data_ptr(), pats.size, n, 4, 0, 3, 0, None))
    cuda.cuda.synchronize()
    assert bits_equal(out.cpu().numpy(), TIES[f"m4_n{n}"])


@pytest.mark.parametrize("n", [1, 2, 4, 6])
def test_mask_entry_m8_tie_patterns(cuda, tblib, n):
    pats = TIES["pats8"].reshape(-1).copy()
    st = dev(cuda, pats)
    out = cuda.empty(pats.size // 8, dtype=cuda.uint8, device="cuda")
    tblib.check(tblib.lib().tb_nm_mask(st.data_ptr(), out.data_ptr(), pats.size, n, 8, 2, 3, 0, None))
    cuda.cuda.synchronize()
    assert bits_equal(out.cpu().numpy(), TIES[f"m8_n{n}"])


def test_legacy_launchers(cuda, tblib, port):
    """The seven kernels.hpp launchers, composed the way EHAPPruner /
    CORINGPruner call them, reproduce the host path bit for bit."""
    L = tblib.lib()
    N = 40000
    g = inputs.normal((4, N), 1e-3, 120)
    w = inputs.normal(N, 0.02, 121)
    gd = dev(cuda, g)
    F = cuda.zeros(N, dtype=cuda.float32, device="cuda")
    for k in range(4):
        if k:
            tblib.check(L.tb_fisher_beta_decay(F.data_ptr(), 0.99, N, None))
        alpha = 0.01 if k == 0 else np.float32(0.01) * (np.float32(1) - np.float32(0.99))
        tblib.check(L.tb_fisher_accumulate(F.data_ptr(), gd[k].data_ptr(), N, float(alpha), None))
    cuda.cuda.synchronize()
    rc, Fo = port.fisher(g)
    assert rc == 0 and bits_equal(F.cpu().numpy(), Fo)
    wd = dev(cuda, w)
    s = cuda.empty(N, dtype=cuda.float32, device="cuda")
    tblib.check(L.tb_ehap_importance(wd.data_ptr(), F.data_ptr(), s.data_ptr(), N, 0.01, None))
    cuda.cuda.synchronize()
    rc, so = port.importance(g, w, mode="obd")
    assert bits_equal(s.cpu().numpy(), so)
    mk = cuda.empty(N // 4, dtype=cuda.uint8, device="cuda")
    tblib.check(L.tb_nm_mask_2_4(s.data_ptr(), mk.data_ptr(), N, None))
    cuda.cuda.synchronize()
    rc, mo = port.nm_mask(so, 2, 4, "topn")
    assert bits_equal(mk.cpu().numpy(), mo)
    mk8 = cuda.empty(N // 8, dtype=cuda.uint8, device="cuda")
    tblib.check(L.tb_nm_mask_generic(s.data_ptr(), mk8.data_ptr(), N, 2, 8, None))
    cuda.cuda.synchronize()
    assert bits_equal(mk8.cpu().numpy(), port.nm_mask(so, 2, 8, "topn")[1])
    tblib.check(L.tb_apply_mask(wd.data_ptr(), mk.data_ptr(), N, 4, None))
    cuda.cuda.synchronize()
    rc, wo, _ = port.apply_redistribute(w, mo, so, 2, 4, "none", 1)
    assert bits_equal(wd.cpu().numpy(), wo)
    # fisher_diagonal: sum of squares in sample order
    Fd = cuda.empty(N, dtype=cuda.float32, device="cuda")
    tblib.check(L.tb_fisher_diagonal(gd.data_ptr(), Fd.data_ptr(), 4, N, None))
    cuda.cuda.synchronize()
    acc = np.zeros(N, np.float32)
    for k in range(4):
        acc = (acc + g[k] * g[k]).astype(np.float32)
    assert bits_equal(Fd.cpu().numpy(), acc)


@pytest.mark.parametrize("gdt", ["f32", "bf16", "f16"])
def test_ema_step_and_importance_entries(cuda, tblib, port, gdt):
    L = tblib.lib()
    N = 30000
    g = inputs.normal((3, N), 1e-3, 130)
    w = inputs.normal(N, 0.02, 131)
    gt, g32, gcode = encode(cuda, g, gdt)
    F = cuda.empty(N, dtype=cuda.float32, device="cuda")
    for k in range(3):
        tblib.check(L.tb_fisher_ema_step(F.data_ptr(), gt[k].data_ptr(), gcode, N, 0.01, 0.99, int(k == 0), None))
    for mode in (0, 1, 2):
        s = cuda.empty(N, dtype=cuda.float32, device="cuda")
        wd = dev(cuda, w)
        tblib.check(L.tb_importance(wd.data_ptr(), 0, F.data_ptr(), s.data_ptr(), N, 0.01, mode, None))
        cuda.cuda.synchronize()
        rc, so = port.importance(g32, w, mode=["obd", "obs", "normalized"][mode])
        assert bits_equal(s.cpu().numpy(), so)
    rc, Fo = port.fisher(g32)
    assert bits_equal(F.cpu().numpy(), Fo)


@pytest.mark.parametrize("redist", ["proportional", "uniform"])
@pytest.mark.parametrize("m", [4, 8])
def test_redistribute_entry_moves_weight(cuda, tblib, port, redist, m):
    """Standalone redistribution on weights that were NOT zeroed first, so
    magnitude actually moves (inside prune() it never does)."""
    rng = np.random.default_rng(140 + m)
    N = 8000
    w = rng.standard_normal(N).astype(np.float32)
    s = rng.random(N).astype(np.float32)
    mk = rng.integers(0, 1 << m, N // m).astype(np.uint8)
    wd, sd, md = dev(cuda, w), dev(cuda, s), dev(cuda, mk)
    tblib.check(tblib.lib().tb_redistribute(wd.data_ptr(), md.data_ptr(), sd.data_ptr(), N, m,
                                            tblib.REDIST[redist], None))
    cuda.cuda.synchronize()
    rc, wo, _ = port.apply_redistribute(w, mk, s, 2, m, redist, 0)
    assert rc == 0 and bits_equal(wd.cpu().numpy(), wo)
    assert not bits_equal(wo, w)


# --- host-buffer path ----------------------------------------------------------

@pytest.mark.parametrize("gdt", ["f32", "bf16"])
def test_host_path_equals_device_path(cuda, tblib, port, gdt):
    N = 3 * 65536 + 64
    w = inputs.normal(N, 0.02, 150)
    g = inputs.normal((6, N), 1e-3, 151)
    r = run_fused(cuda, tblib, w, g, gdt=gdt, strategy="topn")
    gh = g if gdt == "f32" else inputs.to_bf16_bits(g)
    gh = np.ascontiguousarray(gh)
    w_out = np.empty(N, np.float32)
    mask = np.empty(N // 4, np.uint8)
    F = np.empty(N, np.float32)
    s = np.empty(N, np.float32)
    ties = np.zeros(1, np.uint64)
    a = tblib.prune_args(weights=w.ctypes.data, w_dtype=0, grads=gh.ctypes.data,
                         g_dtype=0 if gdt == "f32" else 2, S=6, N=N, w_out=w_out.ctypes.data,
                         mask_out=mask.ctypes.data, fisher_out=F.ctypes.data, scores_out=s.ctypes.data,
                         near_ties=ties.ctypes.data, strategy="topn")
    tblib.check(tblib.score_mask_pack_host(a))
    assert bits_equal(w_out, r["w_out"]) and bits_equal(mask, r["mask"])
    assert bits_equal(F, r["F"]) and bits_equal(s, r["s"]) and int(ties[0]) == r["ties"]


# --- layer-sized pass: oracle on a full q_proj, properties on the largest ------

def test_q_proj_shape_against_oracle(cuda, tblib, port):
    """4096x4096 BF16 weights, 16 BF16 gradient samples with 5% outlier columns,
    Normalized scoring, optimal 2:4: every output bit-exact vs the oracle."""
    w, g = inputs.outlier_columns(4096, 4096, 16, 160)
    r = run_fused(cuda, tblib, w, g, wdt="bf16", gdt="bf16", mode="normalized", strategy="optimal")
    check_against_oracle(port, r, mode="normalized", strategy="optimal")


def test_gate_proj_full_size_properties(cuda, tblib, port):
    """14336x4096 BF16 weights with 128 BF16 samples (the per-matrix size of a
    7B-class decoder layer's gate_proj): generated on the device, checked by properties
    that do not depend on size, and on 4096 random groups against the oracle."""
    torch = cuda
    rows, cols, S = 14336, 4096, 128
    N = rows * cols
    gen = torch.Generator(device="cuda").manual_seed(5)
    w = (torch.randn(N, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    g = (torch.randn(S, rows, cols, device="cuda", generator=gen) * 1e-3)
    hot = torch.randperm(cols, device="cuda", generator=gen)[: cols // 20]
    g[:, :, hot] *= 10
    g = g.to(torch.bfloat16).reshape(S, N)
    w_out = torch.empty(N, dtype=torch.float32, device="cuda")
    mask = torch.empty(N // 4, dtype=torch.uint8, device="cuda")
    s = torch.empty(N, dtype=torch.float32, device="cuda")
    a = tblib.prune_args(weights=w.data_ptr(), w_dtype=2, grads=g.data_ptr(), g_dtype=2, S=S, N=N,
                         mode="normalized", strategy="optimal", w_out=w_out.data_ptr(),
                         mask_out=mask.data_ptr(), scores_out=s.data_ptr())
    tblib.check(tblib.score_mask_pack(a, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    # exactly two kept per group
    pop = torch.zeros_like(mask, dtype=torch.int32)
    for b in range(4):
        pop += ((mask >> b) & 1).int()
    assert bool((pop == 2).all())
    # kept weights are the widened inputs, pruned ones are +0
    bits = torch.stack([(mask >> b) & 1 for b in range(4)], 1).reshape(-1).bool()
    wf = w.float()
    assert bool((w_out[bits] == wf[bits]).all())
    assert bool((w_out[~bits].view(torch.int32) == 0).all())
    # 4096 random groups recomputed by the oracle from their own columns
    idx = torch.randint(0, N // 4, (4096,), device="cuda", generator=gen)
    cols_idx = (idx[:, None] * 4 + torch.arange(4, device="cuda")).reshape(-1)
    wg = wf[cols_idx].cpu().numpy()
    gg = g[:, cols_idx].float().cpu().numpy()
    wp, mk, F, so = oracle_pass(port, wg, gg, mode="normalized", strategy="optimal")
    assert bits_equal(s[cols_idx].cpu().numpy(), so)
    assert bits_equal(mask[idx].cpu().numpy(), mk)
    assert bits_equal(w_out[cols_idx].cpu().numpy(), wp)

"""GPU: the fused pass with 16-bit gradients on tensors of many thousand
vector chunks (whole 16-element chunks plus a ragged tail for the scalar
kernel), against the oracle bit for bit - every N:M pattern, both 16-bit
gradient types, a prior Fisher state, optional outputs and the near-tie
counter - and the sample split's producer, tb_fisher_partial_scatter,
against tb_fisher_weighted_sum."""
import ctypes as C

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


def case(N, S, seed, gdt):
    w = inputs.normal(N, 0.02, seed)
    g32 = inputs.normal((S, N), 1e-3, seed + 1)
    if gdt == "bf16":
        bits = inputs.to_bf16_bits(g32)
        return w, bits.view(np.int16), inputs.bf16_bits_to_f32(bits), 2
    h = g32.astype(np.float16)
    from oracle import Oracle
    return w, h.view(np.int16), Oracle("port").decode_half(h.view(np.uint16), False).reshape(S, N), 1


def run(torch, tb, w, gbits, gcode, n, m, strategy, *, fin=None, steps_in=0, outs=True):
    N = w.size
    S = gbits.shape[0]
    wd = torch.from_numpy(w).cuda()
    gd = torch.from_numpy(np.ascontiguousarray(gbits)).cuda()
    wo = torch.full((N,), float("nan"), device="cuda")
    mk = torch.full((N // m,), 0x5A, dtype=torch.uint8, device="cuda")
    F = torch.full((N,), float("nan"), device="cuda")
    s = torch.full((N,), float("nan"), device="cuda")
    ties = torch.zeros(1, dtype=torch.int64, device="cuda")
    fd = torch.from_numpy(fin).cuda() if fin is not None else None
    a = tb.prune_args(weights=wd.data_ptr(), w_dtype=tb.F32, grads=gd.data_ptr(), g_dtype=gcode, S=S, N=N,
                      fisher_in=fd.data_ptr() if fd is not None else None, fisher_steps_in=steps_in, n=n, m=m,
                      strategy=strategy, mode="obd", redist="proportional", w_out=wo.data_ptr(),
                      mask_out=mk.data_ptr(), fisher_out=F.data_ptr() if outs else None,
                      scores_out=s.data_ptr() if outs else None, near_ties=ties.data_ptr())
    tb.check(tb.score_mask_pack(a, None))
    torch.cuda.synchronize()
    return wo.cpu().numpy(), mk.cpu().numpy(), F.cpu().numpy(), s.cpu().numpy(), int(ties.item())


@pytest.mark.parametrize("gdt", ["bf16", "f16"])
@pytest.mark.parametrize("n,m,strategy", [(2, 4, "optimal"), (2, 4, "topn"), (1, 4, "iterative"),
                                          (2, 8, "iterative"), (4, 8, "topn"), (1, 2, "optimal")])
def test_grads16_match_oracle(cuda, tblib, port, gdt, n, m, strategy):
    N = 600 * 4096 + 96  # more chunks than one wave of the grid, and a ragged tail
    w, gbits, g32, gcode = case(N, 19, 80 + m, gdt)
    wo, mk, F, s, ties = run(cuda, tblib, w, gbits, gcode, n, m, strategy)
    rc, wp, mp, Fp, sp, _, _ = port.pipeline(w, g32, n=n, m=m, strategy=strategy, redist="proportional")
    assert rc == 0
    assert wo.tobytes() == wp.tobytes() and mk.tobytes() == mp.tobytes()
    assert F.tobytes() == Fp.tobytes() and s.tobytes() == sp.tobytes()
    assert ties == port.near_ties(sp, n, m)


def test_grads16_continue_a_prior_fisher_state(cuda, tblib, port):
    N, S = 8 * 4096, 6
    w, gbits, g32, gcode = case(N, S, 91, "bf16")
    rc, F0 = port.fisher(inputs.normal((3, N), 1e-3, 92))
    wo, mk, F, s, _ = run(cuda, tblib, w, gbits, gcode, 2, 4, "optimal", fin=F0, steps_in=3)
    Fr = F0.copy()
    beta, contrib = np.float32(0.99), np.float32(np.float32(0.01) * (np.float32(1) - np.float32(0.99)))
    for k in range(S):
        Fr = (beta * Fr + (contrib * g32[k]) * g32[k]).astype(np.float32)
    assert F.tobytes() == Fr.tobytes()


@pytest.mark.parametrize("gdt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("P", [1, 2, 3, 8])
def test_partial_scatter_equals_weighted_sum(cuda, tblib, gdt, P):
    """tb_fisher_partial_scatter with P owners emulated by buffers on this one
    device: every owner's slot holds exactly tb_fisher_weighted_sum's values
    for its range (vector kernel, plus the scalar kernel for the tail)."""
    import tbdist as td
    torch = cuda
    N, S = 300 * 4096 + 48, 17
    if gdt == "f32":
        gd = torch.from_numpy(inputs.normal((S, N), 1e-3, 97)).cuda()
        code = tblib.F32
    else:
        _, gbits, _, code = case(N, S, 97, gdt)
        gd = torch.from_numpy(np.ascontiguousarray(gbits)).cuda()
    c = td.ema_weights(S, 0.01, 0.99)
    ref = torch.empty(N, device="cuda")
    tblib.check(tblib.lib().tb_fisher_weighted_sum(ref.data_ptr(), gd.data_ptr(), code, S, N, N, c.ctypes.data, 0,
                                                   None))
    ranges = [td.group_shard(N, 4, P, r) for r in range(P)]
    slot = td.push_slot(N, 4, P)
    owners = [torch.full((slot,), float("nan"), device="cuda") for _ in range(P)]
    starts = (C.c_uint64 * (P + 1))(*([a for a, _ in ranges] + [N]))
    dest = (C.c_void_p * P)(*[o.data_ptr() for o in owners])
    tblib.check(tblib.lib().tb_fisher_partial_scatter(gd.data_ptr(), code, S, N, N, c.ctypes.data, P, starts,
                                                      C.cast(dest, C.POINTER(C.c_void_p)), (P - 1) // 2, None))
    torch.cuda.synchronize()
    for (e0, e1), o in zip(ranges, owners):
        assert torch.equal(o[:e1 - e0].view(torch.int32), ref[e0:e1].view(torch.int32))


@pytest.mark.parametrize("P", [1, 3, 8])
@pytest.mark.parametrize("n,m,strategy", [(2, 4, "optimal"), (2, 8, "iterative"), (1, 4, "topn")])
def test_peer_pass_sums_partials_in_rank_order(cuda, tblib, P, n, m, strategy):
    """tb_score_mask_pack_peer with P partials in this device's memory (as a
    rank sees its own and the received slots): the Fisher state is exactly
    ((p0 + p1) + ...) + p_{P-1} in FP32, and every output equals
    tb_score_mask_pack given that sum as its Fisher state."""
    torch = cuda
    N = 40 * 4096 + 8 * m  # vector chunks and a tail for the scalar kernel
    parts = [torch.from_numpy(np.abs(inputs.normal(N, 1e-6, 120 + k))).cuda() for k in range(P)]
    w = torch.from_numpy(inputs.to_bf16_bits(inputs.normal(N, 0.02, 130)).view(np.int16)).cuda()
    F = parts[0].clone()
    for p in parts[1:]:
        F = F + p
    outs = []
    for peer in (True, False):
        wo = torch.full((N,), float("nan"), device="cuda")
        mk = torch.full((N // m,), 0x33, dtype=torch.uint8, device="cuda")
        fo = torch.full((N,), float("nan"), device="cuda")
        so = torch.full((N,), float("nan"), device="cuda")
        a = tblib.prune_args(weights=w.data_ptr(), w_dtype=tblib.BF16, grads=None, g_dtype=tblib.BF16, S=0, N=N,
                             fisher_in=None if peer else F.data_ptr(), fisher_steps_in=64, n=n, m=m,
                             strategy=strategy, mode="obs", redist="proportional", w_out=wo.data_ptr(),
                             mask_out=mk.data_ptr(), fisher_out=fo.data_ptr(), scores_out=so.data_ptr())
        if peer:
            ptrs = (C.c_void_p * P)(*[p.data_ptr() for p in parts])
            tblib.check(tblib.lib().tb_score_mask_pack_peer(C.byref(a), C.cast(ptrs, C.POINTER(C.c_void_p)), P,
                                                             None))
        else:
            tblib.check(tblib.score_mask_pack(a, None))
        torch.cuda.synchronize()
        outs.append((wo, mk, fo, so))
    (wp, mp, fp, sp), (ws, ms, fs, ss) = outs
    assert torch.equal(fp.view(torch.int32), F.view(torch.int32))
    assert torch.equal(fp.view(torch.int32), fs.view(torch.int32))
    assert torch.equal(sp.view(torch.int32), ss.view(torch.int32))
    assert torch.equal(wp.view(torch.int32), ws.view(torch.int32)) and torch.equal(mp, ms)


def test_peer_pass_argument_checks(cuda, tblib):
    torch = cuda
    N = 4096
    w = torch.zeros(N, device="cuda")
    p0 = torch.zeros(N, device="cuda")
    wo = torch.zeros(N, device="cuda")
    mk = torch.zeros(N // 4, dtype=torch.uint8, device="cuda")
    L = tblib.lib()

    def call(P, **kw):
        base = dict(weights=w.data_ptr(), w_dtype=tblib.F32, grads=None, g_dtype=tblib.F32, S=0, N=N,
                    fisher_steps_in=8, w_out=wo.data_ptr(), mask_out=mk.data_ptr())
        base.update(kw)
        a = tblib.prune_args(**base)
        ptrs = (C.c_void_p * max(P, 1))(*([p0.data_ptr()] * max(P, 1)))
        return L.tb_score_mask_pack_peer(C.byref(a), C.cast(ptrs, C.POINTER(C.c_void_p)), P, None)

    assert call(1) == tblib.TB_OK
    assert call(0) == tblib.TB_ERR_ARG and call(9) == tblib.TB_ERR_ARG           # 1..8 partials
    assert call(2, fisher_in=p0.data_ptr()) == tblib.TB_ERR_ARG                  # the partials are the state
    assert call(2, fisher_steps_in=0) == tblib.TB_ERR_ARG                        # must count the samples
    assert call(2, S=1, grads=p0.data_ptr()) == tblib.TB_ERR_ARG                 # no samples read here
    # the producer side: ranges must cover [0, N), inner starts on multiples of 8, S <= 128
    starts = (C.c_uint64 * 3)(0, 100, N)
    dest = (C.c_void_p * 2)(p0.data_ptr(), p0.data_ptr())
    cw = np.ones(4, np.float32)
    g = torch.zeros(4, N, dtype=torch.bfloat16, device="cuda")
    rc = L.tb_fisher_partial_scatter(g.data_ptr(), tblib.BF16, 4, N, N, cw.ctypes.data, 2, starts,
                                     C.cast(dest, C.POINTER(C.c_void_p)), 0, None)
    assert rc == tblib.TB_ERR_ARG
    starts[1] = 96
    rc = L.tb_fisher_partial_scatter(g.data_ptr(), tblib.BF16, 4, N, N, cw.ctypes.data, 2, starts,
                                     C.cast(dest, C.POINTER(C.c_void_p)), 2, None)
    assert rc == tblib.TB_ERR_ARG                                                 # start_owner outside 0..1
    big = np.ones(129, np.float32)
    rc = L.tb_fisher_partial_scatter(g.data_ptr(), tblib.BF16, 129, N, N, big.ctypes.data, 2, starts,
                                     C.cast(dest, C.POINTER(C.c_void_p)), 0, None)
    assert rc == tblib.TB_ERR_CAPACITY
    torch.cuda.synchronize()

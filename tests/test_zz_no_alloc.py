"""GPU: the host-buffer pass for callers that cannot allocate device memory.

tb_score_mask_pack_host_noalloc serves processes whose GPU memory is already
reserved by another allocator (a framework's caching pool, or a server with a
fixed memory budget), where a cudaMalloc from this library would fail or
fragment that pool.  It stages through a static 16 MiB device array instead.
These tests call it through the C ABI and require exactly the output of the
allocating entry point, tb_score_mask_pack_host, on two calls in a row (the
array keeps the previous call's contents, so the second call shows that
nothing stale leaks through).  The file name makes pytest collect it last.
"""
import ctypes as C
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

import inputs

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tensorbit-core_b200")

pytestmark = pytest.mark.gpu


def host_case(S, N, seed):
    w = inputs.normal(N, 0.02, seed)
    g = inputs.to_bf16_bits(inputs.normal((S, N), 1e-3, seed + 1))
    return w, np.ascontiguousarray(g)


def run(tb, entry, w, g, S, strategy, seed_out):
    N = w.size
    w_out = np.full(N, seed_out, np.float32)
    mask = np.full(N // 4, 0xAA, np.uint8)
    F = np.full(N, seed_out, np.float32)
    s = np.full(N, seed_out, np.float32)
    ties = np.zeros(1, np.uint64)
    a = tb.prune_args(weights=w.ctypes.data, w_dtype=tb.F32, grads=g.ctypes.data, g_dtype=tb.BF16,
                      S=S, N=N, strategy=strategy, mode="obd", redist="proportional",
                      w_out=w_out.ctypes.data, mask_out=mask.ctypes.data, fisher_out=F.ctypes.data,
                      scores_out=s.ctypes.data, near_ties=ties.ctypes.data)
    tb.check(getattr(tb.lib(), entry)(C.byref(a)))
    return w_out, mask, F, s, int(ties[0])


@pytest.mark.parametrize("strategy", ["optimal", "topn"])
def test_no_alloc_matches_allocating_entry_twice(cuda, tblib, strategy):
    # 600,000 elements with 24 samples span several chunks of the 16 MiB array
    # and leave a ragged tail.
    S, N = 24, 600_004
    w, g = host_case(S, N, 11)
    ref = run(tblib, "tb_score_mask_pack_host", w, g, S, strategy, -1.0)
    for call in range(2):
        got = run(tblib, "tb_score_mask_pack_host_noalloc", w, g, S, strategy, float(call) + 7.0)
        for a, b in zip(got[:4], ref[:4]):
            assert a.tobytes() == b.tobytes(), f"call {call}: output differs from tb_score_mask_pack_host"
        assert got[4] == ref[4]


def test_no_alloc_rejects_requests_beyond_its_array(cuda, tblib):
    # 200,000 FP32 samples: one 64-element chunk needs ~51 MB, over 16 MiB.
    S, N = 200_000, 64
    w = np.zeros(N, np.float32)
    g = np.zeros(1, np.float32)  # never read: the size check comes first
    out = np.zeros(N, np.float32)
    mask = np.zeros(N // 4, np.uint8)
    a = tblib.prune_args(weights=w.ctypes.data, w_dtype=tblib.F32, grads=g.ctypes.data, g_dtype=tblib.F32,
                         S=S, N=N, strategy="optimal", w_out=out.ctypes.data, mask_out=mask.ctypes.data)
    rc = tblib.lib().tb_score_mask_pack_host_noalloc(C.byref(a))
    assert rc == tblib.TB_ERR_CAPACITY
    assert b"static staging array holds 16777216 bytes" in tblib.lib().tb_last_error()


def test_no_alloc_call_leaves_device_free_memory_unchanged(cuda, tblib):
    # The one property this entry point exists for: once the device is set up
    # (tie table built where allocation is allowed, the array's address
    # resolved by a first call), a call takes no device memory at all.
    S, N = 24, 600_004
    w, g = host_case(S, N, 13)
    tblib.check(tblib.lib().tb_prepare_nm(2, 4))
    first = run(tblib, "tb_score_mask_pack_host_noalloc", w, g, S, "topn", 3.0)
    cuda.cuda.synchronize()
    free0, _ = cuda.cuda.mem_get_info()
    again = run(tblib, "tb_score_mask_pack_host_noalloc", w, g, S, "topn", 5.0)
    free1, _ = cuda.cuda.mem_get_info()
    assert free1 == free0, f"device free memory changed across a no-alloc call: {free0} -> {free1}"
    for a, b in zip(again[:4], first[:4]):
        assert a.tobytes() == b.tobytes()


def test_no_alloc_top_n_without_tie_table_is_unsupported(cuda, tblib):
    # In a fresh process no tie table exists; building one would allocate, so
    # a top-N call must refuse with TB_ERR_UNSUPPORTED (and allocate nothing).
    code = textwrap.dedent(f"""
        import ctypes as C, sys
        import numpy as np
        sys.path.insert(0, {PKG!r})
        import tbabi as tb
        N = 4096
        w = np.zeros(N, np.float32); out = np.zeros(N, np.float32); mask = np.zeros(N // 8, np.uint8)
        a = tb.prune_args(weights=w.ctypes.data, w_dtype=tb.F32, grads=None, g_dtype=tb.F32, S=0, N=N,
                          n=3, m=8, strategy="topn", use_fisher=False,
                          w_out=out.ctypes.data, mask_out=mask.ctypes.data)
        rc = tb.lib().tb_score_mask_pack_host_noalloc(C.byref(a))
        print(rc, tb.lib().tb_last_error().decode())
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    rc, msg = r.stdout.strip().split(" ", 1)
    assert int(rc) == tblib.TB_ERR_UNSUPPORTED, r.stdout
    assert "tie table for 3:8" in msg

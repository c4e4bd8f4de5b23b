"""GPU: tb_score_mask_pack_host called from several host threads at once.

The host-buffer entry keeps one set of staging buffers, streams and a tie
counter per device and grows the buffers on demand.  Two threads calling it on
the same device must each get exactly the outputs of a serial call (the
per-device call lock keeps one call from reusing or freeing the other's
buffers), including when the second call needs larger buffers than the first.
"""
import threading

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


def case(S, N, seed):
    w = inputs.normal(N, 0.02, seed)
    g = np.ascontiguousarray(inputs.to_bf16_bits(inputs.normal((S, N), 1e-3, seed + 1)))
    return S, N, w, g


def call(tb, c, strategy):
    S, N, w, g = c
    w_out = np.full(N, np.nan, np.float32)
    mask = np.full(N // 4, 0x55, np.uint8)
    F = np.full(N, np.nan, np.float32)
    ties = np.zeros(1, np.uint64)
    a = tb.prune_args(weights=w.ctypes.data, w_dtype=tb.F32, grads=g.ctypes.data, g_dtype=tb.BF16, S=S, N=N,
                      strategy=strategy, mode="obd", redist="proportional", w_out=w_out.ctypes.data,
                      mask_out=mask.ctypes.data, fisher_out=F.ctypes.data, near_ties=ties.ctypes.data)
    rc = tb.score_mask_pack_host(a)
    return rc, w_out, mask, F, int(ties[0])


def test_two_threads_match_serial_calls(cuda, tblib):
    # Different sample counts give different staging sizes, so whichever call
    # comes second on the device may have to grow the shared slots.
    cases = [case(8, 1_500_016, 31), case(48, 2_200_004, 33)]
    strategies = ["topn", "optimal"]
    tblib.check(tblib.lib().tb_prepare_nm(2, 4))
    serial = []
    for c, st in zip(cases, strategies):
        rc, *out = call(tblib, c, st)
        tblib.check(rc)
        serial.append(out)
    results = [[None] * 4 for _ in cases]
    start = threading.Barrier(len(cases))

    def worker(i):
        start.wait()
        for k in range(4):
            results[i][k] = call(tblib, cases[i], strategies[i])

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(cases))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    for i, runs in enumerate(results):
        for k, (rc, *out) in enumerate(runs):
            assert rc == 0, f"thread {i} call {k}: status {rc}"
            for a, b in zip(out[:3], serial[i][:3]):
                assert a.tobytes() == b.tobytes(), f"thread {i} call {k}: output differs from the serial call"
            assert out[3] == serial[i][3]

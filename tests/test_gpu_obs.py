"""GPU parity of the reference-semantics block OBS (tb_block_obs) against the
oracle, which is itself bit-identical to the reference's prune_block_obs built
with the stand-in Eigen (tests/test_oracle.py).  Bar: bit-exact weights and
the same pruned count."""
import ctypes as C

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu


def run_gpu(torch, tb, w, F, hist, block, sparsity, damping=0.01, off_alpha=0.01):
    wd = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    Fd = torch.from_numpy(np.ascontiguousarray(F)).cuda() if F is not None else None
    hd = [torch.from_numpy(np.ascontiguousarray(h)).cuda() for h in (hist if hist is not None else [])]
    ptrs = (C.c_void_p * max(1, len(hd)))(*[h.data_ptr() for h in hd]) if hd else None
    pruned = C.c_uint64()
    tb.check(tb.lib().tb_block_obs(wd.data_ptr(), Fd.data_ptr() if Fd is not None else None, ptrs, len(hd),
                                   w.size, block, sparsity, damping, off_alpha, C.byref(pruned), None))
    torch.cuda.synchronize()
    return wd.cpu().numpy(), pruned.value


CASES = [  # N, block, K, S, use_fisher, sparsity
    (1024, 128, 4, 1, True, 0.5),
    (1000, 128, 4, 2, True, 0.5),
    (4096, 128, 0, 1, True, 0.5),
    (2048, 64, 2, 3, True, 0.3),
    (777, 100, 4, 1, True, 0.5),
    (4096, 128, 4, 1, False, 0.5),
    (16384, 128, 4, 1, True, 0.5),
    (5000, 224, 3, 1, True, 0.7),
    (3000, 32, 1, 1, True, 0.9),
    (65536, 128, 4, 1, True, 0.5),
    (8000, 224, 16, 1, True, 0.5),    # largest block and history: ~218 KB of shared memory
    (4097, 128, 4, 1, True, 0.5),     # last block of one weight (target 0)
    (20000, 128, 4, 1, True, 0.98),   # 2 % pruned: many blocks with target 0 or 1
    (300, 2, 1, 1, True, 0.5),        # blocks of two weights
    (131072, 128, 4, 1, True, 0.5),   # 1024 blocks over many target groups
]


@pytest.mark.parametrize("N,block,K,S,use_fisher,sp", CASES)
def test_block_obs_matches_oracle(cuda, tblib, port, N, block, K, S, use_fisher, sp):
    w = inputs.normal(N, 0.5, N)
    g = inputs.normal((S, N), 0.05, N + 1)
    hist = (np.stack([g[0] * (np.float32(0.9) + np.float32(0.02) * np.float32(k)) for k in range(K)])
            .astype(np.float32) if K else None)
    rc, wo, po = port.block_obs(w, g, hist, block=block, sparsity=sp, use_fisher=use_fisher, hist_size=max(K, 1))
    assert rc == 0
    F = port.fisher(g)[1] if use_fisher else None
    wg, pg = run_gpu(cuda, tblib, w, F, hist, block, sp)
    assert pg == po
    assert wg.tobytes() == wo.tobytes(), f"{int((wg != wo).sum())} weights differ"


def test_block_obs_mock_tensor_like_tb_prune(cuda, tblib, port):
    """tb-prune --strategy BlockOBS on the mock tensor: Fisher from one sample,
    four scaled snapshots of it (src/main.cpp:375-385)."""
    w, g = port.mock_tensor(16384)
    hist = np.stack([g * (np.float32(0.9) + np.float32(0.02) * np.float32(k)) for k in range(4)]).astype(np.float32)
    rc, wo, po = port.block_obs(w, g[None, :], hist)
    F = port.fisher(g[None, :])[1]
    wg, pg = run_gpu(cuda, tblib, w, F, hist, 128, 0.5)
    assert rc == 0 and pg == po and wg.tobytes() == wo.tobytes()


def test_block_obs_errors(cuda, tblib):
    w = cuda.zeros(256, device="cuda")
    pr = C.c_uint64()
    L = tblib.lib()
    assert L.tb_block_obs(w.data_ptr(), None, None, 0, 0, 128, 0.5, 0.01, 0.01, C.byref(pr), None) == tblib.TB_ERR_ZERO_SIZE
    assert L.tb_block_obs(w.data_ptr(), None, None, 0, 256, 0, 0.5, 0.01, 0.01, C.byref(pr), None) == tblib.TB_ERR_CONFIG
    assert L.tb_block_obs(w.data_ptr(), None, None, 0, 256, 256, 0.5, 0.01, 0.01, C.byref(pr), None) == tblib.TB_ERR_UNSUPPORTED
    assert L.tb_block_obs(w.data_ptr(), None, None, 17, 256, 128, 0.5, 0.01, 0.01, C.byref(pr), None) == tblib.TB_ERR_UNSUPPORTED

"""CPU: the multi-rank host logic of tensorbit-core_b200/tbdist.py with two gloo
ranks (no GPU).  The kernels themselves are exercised by test_gpu_dist.py;
here the per-rank results are produced by the oracle, so what is checked is
the sharding plan, the regrouped EMA weights with the all-reduce, and the .tb
assembled from slices written by different processes."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

import inputs
import tbdist

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.mark.parametrize("N,m", [(4096, 4), (4100, 4), (64, 4), (16384 + 8, 8), (96, 2), (7 * 48, 3)])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_group_shards_cover_and_align(N, m, world):
    ranges = [tbdist.group_shard(N, m, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == N
    unit = m * 16 // np.gcd(m, 16)
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for r, (e0, e1) in enumerate(ranges):
        assert e0 <= e1 and e0 % unit == 0 and (e1 - e0) % m == 0
        if r < world - 1:
            assert e1 % unit == 0


LAYER_7B = [4096 * 4096, 1024 * 4096, 1024 * 4096, 4096 * 4096, 14336 * 4096, 14336 * 4096, 4096 * 14336]
LAYER_70B = [8192 * 8192, 1024 * 8192, 1024 * 8192, 8192 * 8192, 28672 * 8192, 28672 * 8192, 8192 * 28672]


@pytest.mark.parametrize("sizes,m", [(LAYER_7B * 32, 4), (LAYER_70B * 80, 8), (LAYER_70B * 80, 4),
                                     ([64, 4096, 8, 100_000, 12, 16, 48], 4), ([24, 24, 8], 8), ([4], 4),
                                     (LAYER_7B, 4)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 5, 7, 8])
def test_model_shards_cover_align_and_balance(sizes, m, world):
    unit = m * 16 // np.gcd(m, 16)
    seen = {t: [] for t in range(len(sizes))}
    per_rank = []
    for r in range(world):
        pieces = tbdist.model_shard(sizes, m, world, r)
        per_rank.append(sum(e1 - e0 for _, e0, e1 in pieces))
        prev = None
        for t, e0, e1 in pieces:
            assert 0 <= e0 < e1 <= sizes[t] and e0 % m == 0 and e1 % m == 0
            assert e0 % unit == 0 and (e1 == sizes[t] or e1 % unit == 0)
            assert prev is None or (t, e0) > prev  # model order
            prev = (t, e1)
            seen[t].append((e0, e1))
    for t, ranges in seen.items():  # every tensor exactly covered once
        ranges.sort()
        assert ranges and ranges[0][0] == 0 and ranges[-1][1] == sizes[t]
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    total = sum(sizes)
    # each cut moves down by less than one alignment unit from its even share
    assert all(abs(p - total / world) < unit + 1 for p in per_rank), per_rank


@pytest.mark.parametrize("weights", [[22.0, 22.1, 32.5, 32.4], [1.0, 3.0], [5.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0, 2.0]])
def test_weighted_model_shards_cover_and_follow_weights(weights):
    sizes = LAYER_7B * 3 + [4096 * 16 + 64]
    world, m = len(weights), 4
    unit = 16
    total = sum(sizes)
    covered = {t: [] for t in range(len(sizes))}
    for r in range(world):
        pieces = tbdist.model_shard(sizes, m, world, r, weights=weights)
        for t, e0, e1 in pieces:
            assert e0 % unit == 0 and (e1 == sizes[t] or e1 % unit == 0)
            covered[t].append((e0, e1))
        share = total * weights[r] / sum(weights)
        assert abs(sum(e1 - e0 for _, e0, e1 in pieces) - share) < 2 * unit + 2
    for t, ranges in covered.items():
        ranges.sort()
        assert ranges[0][0] == 0 and ranges[-1][1] == sizes[t]
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    # equal weights give the unweighted cut
    for r in range(world):
        assert tbdist.model_shard(sizes, m, world, r, weights=[2.0] * world) == tbdist.model_shard(sizes, m, world, r)
    with pytest.raises(ValueError):
        tbdist.model_shard(sizes, m, world, 0, weights=[1.0] * (world + 1))


def test_model_shards_keep_whole_tensors_when_layers_divide():
    # 32 equal layers over 1/2/4/8 ranks: every cut lands on a layer boundary
    for world in (1, 2, 4, 8):
        for r in range(world):
            pieces = tbdist.model_shard(LAYER_7B * 32, 4, world, r)
            assert len(pieces) == 224 // world
            assert all(e0 == 0 and e1 == (LAYER_7B * 32)[t] for t, e0, e1 in pieces)


def test_ema_weights_equal_the_recurrence(port):
    g = inputs.normal((64, 5000), 1e-3, 3)
    rc, F = port.fisher(g, alpha=0.01, beta=0.99)
    c = tbdist.ema_weights(64, 0.01, 0.99).astype(np.float64)
    Fw = (c[:, None] * g.astype(np.float64) ** 2).sum(0)
    assert rc == 0
    np.testing.assert_allclose(Fw, F, rtol=1e-5, atol=0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port_no, tmpdir, results):
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tensorbit-core_b200"), HERE]
    import torch
    import torch.distributed as dist
    import inputs as inp
    import tbdist as td
    from oracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O = Oracle("port")
    # --- sample split: partial sums over this rank's samples, all-reduced ---
    S, N = 32, 6000
    g = inp.normal((S, N), 1e-3, 11)
    s0, s1 = td.sample_shard(S, world, rank)
    c = td.ema_weights(S, 0.01, 0.99)
    part = np.zeros(N, np.float32)
    for t in range(s0, s1):
        part = (part + (c[t] * g[t]) * g[t]).astype(np.float32)
    F = torch.from_numpy(part)
    dist.all_reduce(F)
    results[f"F{rank}"] = F.numpy().copy()
    # --- group sharding: each rank writes its slice of one .tb ---
    w, gg = inp.tensor_128x128_s8()
    path = os.path.join(tmpdir, "sharded.tb")
    N2, m = w.size, 4
    e0, e1 = td.group_shard(N2, m, world, rank)
    if rank == 0:
        td.create_tb(path, N2, 2, m)
    dist.barrier()
    rc, wp, mk, *_ = O.pipeline(w[e0:e1], gg[:, e0:e1], strategy="optimal", redist="proportional")
    assert rc == 0
    td.write_tb_slice(path, N2, m, e0, wp, mk)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks(port, tmp_path):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), results), nprocs=2, join=True,
                       start_method="spawn")
    # all-reduced partial sums == the serial EMA within FP32 rounding, same on both ranks
    g = inputs.normal((32, 6000), 1e-3, 11)
    rc, F = port.fisher(g)
    assert np.array_equal(results["F0"], results["F1"])
    np.testing.assert_allclose(results["F0"], F, rtol=1e-5, atol=0)
    # the .tb assembled from two ranks' slices == the single-process file
    w, gg = inputs.tensor_128x128_s8()
    rc, wp, mk, *_ = port.pipeline(w, gg, strategy="optimal", redist="proportional")
    assert open(tmp_path / "sharded.tb", "rb").read() == port.tb_bytes(wp, mk, 2, 4)


@pytest.mark.parametrize("r,n", [(4096, 2048), (256, 64), (640, 1344)])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_obs_row_and_token_shards(r, n, world):
    rows = [tbdist.obs_row_shard(r, world, k) for k in range(world)]
    toks = [tbdist.token_shard(n, world, k) for k in range(world)]
    for ranges, unit, total in ((rows, 128, r), (toks, 64, n)):
        assert ranges[0][0] == 0 and ranges[-1][1] == total
        for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
            assert a1 == b0
        assert all(a % unit == 0 and b % unit == 0 and a <= b for a, b in ranges)


def _obs_worker(rank, world, port_no, tmpdir):
    sys.path[:0] = [os.path.join(ROOT, "tensorbit-core_b200"), HERE]
    import torch
    import torch.distributed as dist
    import tbdist as td

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n, d = 320, 96
    X = np.random.default_rng(11).standard_normal((n, d))
    t0, t1 = td.token_shard(n, world, rank)
    # the partial each rank forms (scale 1/n_total), summed by the all-reduce
    H = torch.from_numpy(X[t0:t1].T @ X[t0:t1] / n)
    dist.all_reduce(H)
    np.save(os.path.join(tmpdir, f"H{rank}.npy"), H.numpy())
    dist.destroy_process_group()


def test_obs_token_split_sum_is_the_full_hessian(tmp_path):
    """Two gloo ranks: partials over the token shards with the global 1/n scale
    all-reduce to X^T X / n of all tokens, identically on both ranks."""
    mp.start_processes(_obs_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    X = np.random.default_rng(11).standard_normal((320, 96))
    H0, H1 = np.load(tmp_path / "H0.npy"), np.load(tmp_path / "H1.npy")
    assert np.array_equal(H0, H1)
    np.testing.assert_allclose(H0, X.T @ X / 320, rtol=1e-12, atol=1e-12)

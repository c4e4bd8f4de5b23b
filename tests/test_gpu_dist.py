"""GPU, two or more devices: group sharding and sample splitting of one
tensor's pass (tensorbit-core_b200/tbdist.py), checked against the single-GPU
pass.  Group sharding must give the identical .tb file; sample splitting, with
the exchange as an NCCL all-reduce or fused into the pass over peer memory,
must give a Fisher within 1e-5 relative and masks equal outside near-tie
groups; the peer variant's Fisher must be exactly the rank-order sum of the
ranks' partials."""
import os
import socket
import sys

import numpy as np
import pytest

import inputs

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port_no, tmpdir):
    sys.path[:0] = [os.path.join(ROOT, "tensorbit-core_b200"), HERE]
    import datetime

    import torch
    import torch.distributed as dist
    import inputs as inp
    import tbabi as tb
    import tbdist as td

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    # group sharding through the host-buffer entry, one shared .tb
    w = inp.normal(1 << 20, 0.02, 5)
    g = inp.to_bf16_bits(inp.normal((8, 1 << 20), 1e-3, 6))
    td.prune_group_sharded(dist, w, tb.F32, g, tb.BF16, os.path.join(tmpdir, "group.tb"), strategy="optimal")
    # sample splitting on the device: rank r holds samples [s0, s1) of all elements
    S, N = 16, 1 << 20
    wd = torch.from_numpy(inp.to_bf16_bits(inp.normal(N, 0.02, 7)).view(np.int16)).cuda()
    gall = inp.to_bf16_bits(inp.normal((S, N), 1e-3, 8))
    s0, s1 = td.sample_shard(S, world, rank)
    gd = torch.from_numpy(np.ascontiguousarray(gall[s0:s1]).view(np.int16)).cuda()
    out_w = torch.zeros(N, dtype=torch.float32, device="cuda")
    out_m = torch.zeros(N // 4, dtype=torch.uint8, device="cuda")
    r = td.prune_sample_split(dist, torch, wd, tb.BF16, gd, tb.BF16, S, s0, out_w, out_m, strategy="optimal",
                              redist="proportional", mode="obd")
    torch.cuda.synchronize()
    e0, e1 = r["e0"], r["e1"]
    np.save(os.path.join(tmpdir, f"ss_w{rank}.npy"), out_w[e0:e1].cpu().numpy())
    np.save(os.path.join(tmpdir, f"ss_m{rank}.npy"), out_m[e0 // 4:e1 // 4].cpu().numpy())
    np.save(os.path.join(tmpdir, f"ss_F{rank}.npy"), r["fisher"].cpu().numpy())
    np.save(os.path.join(tmpdir, f"ss_t{rank}.npy"), np.array([int(r["near_ties"].item()), e0, e1]))
    # the same split with the exchange fused into the pass (peer reads of the partials)
    bufs = td.PeerBuffers(dist, 4 * N, 2)
    pw = torch.zeros(N, dtype=torch.float32, device="cuda")
    pm = torch.zeros(N // 4, dtype=torch.uint8, device="cuda")
    pF = torch.zeros(N, dtype=torch.float32, device="cuda")
    for k in (0, 1, 0):  # reuse of buffer 0 after buffer 1 exercises the alternation
        td.prune_sample_split_peer(dist, torch, bufs, k, wd, tb.BF16, gd, tb.BF16, S, s0, pw, pm,
                                   strategy="optimal", redist="proportional", mode="obd", fisher_out=pF)
    torch.cuda.synchronize()
    part = torch.empty(N, dtype=torch.float32, device="cuda")
    tb.check(tb.lib().tb_memcpy_d2d(part.data_ptr(), bufs.local[0], 4 * N, None))
    torch.cuda.synchronize()
    np.save(os.path.join(tmpdir, f"pp_part{rank}.npy"), part.cpu().numpy())
    np.save(os.path.join(tmpdir, f"pp_w{rank}.npy"), pw[e0:e1].cpu().numpy())
    np.save(os.path.join(tmpdir, f"pp_m{rank}.npy"), pm[e0 // 4:e1 // 4].cpu().numpy())
    np.save(os.path.join(tmpdir, f"pp_F{rank}.npy"), pF[e0:e1].cpu().numpy())
    bufs.close()
    # and with the exchange as NVLink writes from the partial kernel (push)
    bufs = td.PeerBuffers(dist, 4 * world * td.push_slot(N, 4, world), 2)
    qw = torch.zeros(N, dtype=torch.float32, device="cuda")
    qm = torch.zeros(N // 4, dtype=torch.uint8, device="cuda")
    qF = torch.zeros(N, dtype=torch.float32, device="cuda")
    for k in (0, 1, 0):
        td.prune_sample_split_push(dist, torch, bufs, k, wd, tb.BF16, gd, tb.BF16, S, s0, qw, qm,
                                   strategy="optimal", redist="proportional", mode="obd", fisher_out=qF)
    torch.cuda.synchronize()
    np.save(os.path.join(tmpdir, f"pu_w{rank}.npy"), qw[e0:e1].cpu().numpy())
    np.save(os.path.join(tmpdir, f"pu_m{rank}.npy"), qm[e0 // 4:e1 // 4].cpu().numpy())
    np.save(os.path.join(tmpdir, f"pu_F{rank}.npy"), qF[e0:e1].cpu().numpy())
    # and with the owners' ranges moved by the copy engines
    scratch = torch.empty(N, dtype=torch.float32, device="cuda")
    cw, cm, cF = torch.zeros_like(qw), torch.zeros_like(qm), torch.zeros_like(qF)
    for k in (0, 1, 0):
        td.prune_sample_split_copy(dist, torch, bufs, k, scratch, wd, tb.BF16, gd, tb.BF16, S, s0, cw, cm,
                                   strategy="optimal", redist="proportional", mode="obd", fisher_out=cF)
    torch.cuda.synchronize()
    np.save(os.path.join(tmpdir, f"cp_w{rank}.npy"), cw[e0:e1].cpu().numpy())
    np.save(os.path.join(tmpdir, f"cp_m{rank}.npy"), cm[e0 // 4:e1 // 4].cpu().numpy())
    np.save(os.path.join(tmpdir, f"cp_F{rank}.npy"), cF[e0:e1].cpu().numpy())
    # the copy exchange pipelined over a sequence of tensors: the same bits as
    # the one-tensor copy pass for each, over two runs of seven tensors (so the
    # three exchange buffers rotate across the runs' boundary)
    sizes = (N, (1 << 18) + 4 * 37, 3 << 16)
    wts = [wd] + [torch.from_numpy(inp.to_bf16_bits(inp.normal(n_, 0.02, 30 + i)).view(np.int16)).cuda()
                  for i, n_ in enumerate(sizes[1:])]
    gts = [gd] + [torch.from_numpy(np.ascontiguousarray(
        inp.to_bf16_bits(inp.normal((S, n_), 1e-3, 40 + i))[s0:s1]).view(np.int16)).cuda()
        for i, n_ in enumerate(sizes[1:])]
    want = []
    for i, n_ in enumerate(sizes):
        a0, a1 = td.group_shard(n_, 4, world, rank)
        ow = torch.zeros(n_, dtype=torch.float32, device="cuda")
        om = torch.zeros(n_ // 4, dtype=torch.uint8, device="cuda")
        td.prune_sample_split_copy(dist, torch, bufs, i & 1, scratch, wts[i], tb.BF16, gts[i], tb.BF16, S, s0,
                                   ow, om, strategy="optimal", redist="proportional", mode="obd")
        torch.cuda.synchronize()
        want.append((ow[a0:a1].cpu().numpy(), om[a0 // 4:a1 // 4].cpu().numpy()))
    assert want[0][0].tobytes() == cw[e0:e1].cpu().numpy().tobytes()
    pipe = td.CopyExchangePipeline(dist, torch, N, 4)
    order = (0, 1, 2, 0, 1, 2, 1)
    runs = []
    for _ in range(2):
        jobs = []
        for i in order:
            a0, a1 = td.group_shard(sizes[i], 4, world, rank)
            jobs.append((wts[i], tb.BF16, gts[i], tb.BF16,
                         torch.full((max(1, a1 - a0),), -1.0, dtype=torch.float32, device="cuda"),
                         torch.full((max(1, (a1 - a0) // 4),), 7, dtype=torch.uint8, device="cuda")))
        pipe.run(jobs, S, s0, strategy="optimal", redist="proportional", mode="obd")
        runs.append(jobs)
    torch.cuda.synchronize()
    for jobs in runs:
        for i, job in zip(order, jobs):
            got_w, got_m = job[4].cpu().numpy(), job[5].cpu().numpy()
            assert got_w[:want[i][0].size].tobytes() == want[i][0].tobytes(), f"pipeline weights of tensor {i}"
            assert got_m[:want[i][1].size].tobytes() == want[i][1].tobytes(), f"pipeline mask of tensor {i}"
    pipe.close()
    bufs.close()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


def test_two_rank_group_shard_and_sample_split(cuda, tblib, port, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    if cuda.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    # group sharding: identical file to one process
    w = inputs.normal(1 << 20, 0.02, 5)
    gbits = inputs.to_bf16_bits(inputs.normal((8, 1 << 20), 1e-3, 6))
    rc, wp, mk, *_ = port.pipeline(w, inputs.bf16_bits_to_f32(gbits), strategy="optimal", redist="proportional")
    assert rc == 0
    assert open(tmp_path / "group.tb", "rb").read() == port.tb_bytes(wp, mk, 2, 4)
    # sample splitting: Fisher within 1e-5 relative; masks equal outside near-ties
    S, N = 16, 1 << 20
    w32 = inputs.bf16_bits_to_f32(inputs.to_bf16_bits(inputs.normal(N, 0.02, 7)))
    g32 = inputs.bf16_bits_to_f32(inputs.to_bf16_bits(inputs.normal((S, N), 1e-3, 8)))
    rc, wo, mo, Fo, so, *_ = port.pipeline(w32, g32, strategy="optimal", redist="proportional")
    F0 = np.load(tmp_path / "ss_F0.npy")
    assert np.array_equal(F0, np.load(tmp_path / "ss_F1.npy"))
    np.testing.assert_allclose(F0, Fo, rtol=1e-5, atol=0)
    masks = np.concatenate([np.load(tmp_path / f"ss_m{r}.npy") for r in range(world)])
    wgot = np.concatenate([np.load(tmp_path / f"ss_w{r}.npy") for r in range(world)])
    differ = masks != mo
    srt = -np.sort(-so.reshape(-1, 4), axis=1)
    a, b = srt[:, 1], srt[:, 2]
    near = np.abs(a - b) <= np.float32(1e-6) * np.maximum(np.abs(a), np.finfo(np.float32).tiny)
    assert not (differ & ~near).any(), "a mask differs outside the near-tie groups"
    same = np.repeat(~differ, 4)
    assert np.array_equal(wgot[same], wo[same])
    # peer variant: F is exactly part_0 + part_1 (FP32, rank order) on each rank's range,
    # within 1e-5 of the serial recurrence; masks equal the all-reduce variant's outside near ties
    parts = [np.load(tmp_path / f"pp_part{r}.npy") for r in range(world)]
    Fsum = (parts[0] + parts[1]).astype(np.float32)
    Fp = np.concatenate([np.load(tmp_path / f"pp_F{r}.npy") for r in range(world)])
    assert Fp.tobytes() == Fsum.tobytes()
    np.testing.assert_allclose(Fp, Fo, rtol=1e-5, atol=0)
    mp_ = np.concatenate([np.load(tmp_path / f"pp_m{r}.npy") for r in range(world)])
    assert not ((mp_ != mo) & ~near).any(), "a peer-variant mask differs outside the near-tie groups"
    wpp = np.concatenate([np.load(tmp_path / f"pp_w{r}.npy") for r in range(world)])
    samep = np.repeat(mp_ == mo, 4)
    assert np.array_equal(wpp[samep], wo[samep])
    # push variant: the same partials (same arithmetic), so the same bits as the peer-read variant
    for variant in ("pu", "cp"):  # push (SM stores) and copy (copy engines)
        for key, ref_ in (("F", Fp), ("m", mp_), ("w", wpp)):
            got = np.concatenate([np.load(tmp_path / f"{variant}_{key}{r}.npy") for r in range(world)])
            assert got.tobytes() == ref_.tobytes(), f"{variant} variant {key} differs from the peer-read variant"


def _obs_worker(rank, world, port_no, tmpdir):
    sys.path[:0] = [os.path.join(ROOT, "tensorbit-core_b200"), HERE]
    import datetime

    import torch
    import torch.distributed as dist
    import inputs as inp
    import tbdist as td

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    r, d, n = OBS_SHAPE
    X = inp.activations(n, d, 17)
    W = inp.normal(r * d, 0.02, 18).reshape(r, d)
    t0, t1 = td.token_shard(n, world, rank)
    xt = torch.from_numpy(np.ascontiguousarray(X[t0:t1].T)).cuda().to(torch.bfloat16).contiguous()
    H = torch.empty(d, d, device="cuda")
    td.obs_hessian_token_split(dist, torch, xt, d, n, H)
    r0, r1 = td.obs_row_shard(r, world, rank)
    Wl = torch.from_numpy(np.ascontiguousarray(W[r0:r1])).cuda()
    ml = torch.zeros((r1 - r0) * d // 4, dtype=torch.uint8, device="cuda")
    td.prune_obs_row_split(dist, torch, Wl, H, ml)
    torch.cuda.synchronize()
    np.save(os.path.join(tmpdir, f"obs_H{rank}.npy"), H.cpu().numpy())
    np.save(os.path.join(tmpdir, f"obs_W{rank}.npy"), Wl.cpu().numpy())
    np.save(os.path.join(tmpdir, f"obs_m{rank}.npy"), ml.cpu().numpy().reshape(r1 - r0, d // 4))
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


OBS_SHAPE = (256, 512, 1024)


def test_two_rank_obs_token_and_row_split(cuda, tblib, tmp_path):
    import sparsegpt_ref as ref
    import torch.multiprocessing as mp
    world = 2
    if cuda.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_obs_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r, d, n = OBS_SHAPE
    X = inputs.activations(n, d, 17)
    W = inputs.normal(r * d, 0.02, 18).reshape(r, d)
    H0 = np.load(tmp_path / "obs_H0.npy")
    assert np.array_equal(H0, np.load(tmp_path / "obs_H1.npy"))
    Hd = X.astype(np.float64).T @ X.astype(np.float64) / n
    low = np.tril(np.ones((d // 128, d // 128), bool)).repeat(128, 0).repeat(128, 1)
    assert np.abs(H0 - Hd)[low].max() <= 1e-5 * np.abs(Hd).max()
    Wg = np.concatenate([np.load(tmp_path / f"obs_W{k}.npy") for k in range(world)])
    mg = np.concatenate([np.load(tmp_path / f"obs_m{k}.npy") for k in range(world)])
    Wr, mr, U, gap = ref.sparsegpt(W, X, 0.01, 2, 4, 128)
    differ = mg != mr
    assert differ.mean() <= 1e-3
    first = np.argmax(differ, axis=1)
    rows = np.nonzero(differ.any(1))[0]
    assert (gap[rows, first[rows]] < 1e-2).all()
    lg, lr = ref.layer_loss(W, Wg, X), ref.layer_loss(W, Wr, X)
    assert abs(lg - lr) <= 0.01 * lr, (lg, lr)

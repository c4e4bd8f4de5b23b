"""Multi-GPU pruning: one process per GPU, torch.distributed for the plumbing.

Two ways to spread one tensor's pass over P ranks (the reference has none; its
docs prune shards in separate processes, docs/CLOUD.md:155-170):

* **group sharding** (`prune_group_sharded`): rank r owns a contiguous range of
  N:M groups (row blocks of the matrix).  Groups are independent, so each rank
  runs the fused pass on its range with no communication and writes its slice
  of the shared `.tb` file in place: weights at 4096 + 4*e0, mask bytes at
  masks_offset + e0/M.  Results are bit-identical to a single-GPU pass.
* **sample splitting** (`prune_sample_split`, `prune_sample_split_peer`): rank r holds a subset of the S
  calibration gradients for all elements.  The EMA recurrence
  F_S = beta F_{S-1} + alpha (1-beta) g^2 (ehap.hpp:190-197) is regrouped as
  F = sum_t c_t g_t^2; each rank sums its own samples (tb_fisher_weighted_sum),
  one NCCL all-reduce adds the partials over NVLink, and every rank then scores,
  masks and packs its group range from the summed Fisher.  The peer variants
  replace the all-reduce by a reduce-scatter over peer memory, half the NVLink
  bytes of an all-reduce and no reduction kernel: `prune_sample_split_peer`
  reads the other ranks' partials of its range inside the pass;
  `prune_sample_split_push` has each rank's partial kernel store every
  owner's range straight into that owner's memory, and
  `prune_sample_split_copy` moves the owners' ranges of a locally written
  partial with device-to-device copies (the copy engines), so the pass reads
  all partials locally; `CopyExchangePipeline` runs the copies of one tensor
  on a second stream beside the next tensor's partial.  F matches the
  serial recurrence to FP32 rounding (the association differs), so masks can
  differ only in near-tie groups, which the pass counts.

Column-block exact OBS of one layer (`obs_hessian_token_split`,
`prune_obs_row_split`): the calibration tokens are split across ranks, each
rank forms X_r^T X_r / n on tensor cores and one NCCL all-reduce of the d x d
FP32 Hessian sums them; every rank then factors the same H (replicated, not
scaled) and sweeps only its own rows of W, which are independent.

Ranks read RANK / WORLD_SIZE / LOCAL_RANK from the environment like torchrun.
"""
from __future__ import annotations

import bisect
import ctypes as C
import math
import os

import numpy as np

import tbabi as tb

TB_HEADER = 4096


def group_shard(N: int, m: int, world: int, rank: int) -> tuple[int, int]:
    """Element range [e0, e1) of `rank`: contiguous, balanced by whole units of
    lcm(M, 16) elements (so every rank but the last keeps the 16-element vector
    path aligned); the last rank also takes the ragged tail."""
    if N % m:
        raise ValueError(f"numel {N} not divisible by M={m}")
    unit = m * 16 // math.gcd(m, 16)
    units = N // unit
    e0 = units * rank // world * unit
    e1 = units * (rank + 1) // world * unit if rank < world - 1 else N
    return e0, e1


def model_shard(sizes: list[int], m: int, world: int, rank: int,
                weights: list[float] | None = None) -> list[tuple[int, int, int]]:
    """This rank's share of a whole model's pass.  The tensors (element counts
    `sizes`, each a multiple of M) are laid end to end as one range of N:M
    groups and cut into `world` contiguous parts of equal size, each cut moved
    down to a multiple of lcm(M, 16) elements inside the tensor it falls in (so
    every piece but a tensor's last keeps the 16-element vector path aligned).
    Returns [(tensor index, e0, e1)]: element ranges inside the tensors, in
    model order.  Ranks differ by at most one alignment unit per cut, however
    unequal the tensors are; whole tensors stay whole unless a cut falls inside
    one.  With `weights` (one positive number per rank, the same list on every
    rank) part r is sized in proportion to weights[r] instead, e.g. to each
    rank's measured host-link bandwidth when the inputs stream from host
    memory."""
    if weights is not None:
        if len(weights) != world or any(not (x > 0) for x in weights):
            raise ValueError("weights: one positive value per rank")
        acc = [0.0]
        for x in weights:
            acc.append(acc[-1] + float(x))
    for t, n in enumerate(sizes):
        if n % m:
            raise ValueError(f"tensor {t}: numel {n} not divisible by M={m}")
    unit = m * 16 // math.gcd(m, 16)
    starts = [0]
    for n in sizes:
        starts.append(starts[-1] + n)
    total = starts[-1]

    def cut(k):  # (tensor index, element offset in it) of cut k
        if k <= 0:
            return 0, 0
        if k >= world:
            return len(sizes), 0
        pos = total * k // world if weights is None else min(total, int(total * (acc[k] / acc[-1])))
        t = bisect.bisect_right(starts, pos) - 1
        return t, (pos - starts[t]) // unit * unit

    (t0, l0), (t1, l1) = cut(rank), cut(rank + 1)
    pieces = []
    t, lo = t0, l0
    while t < len(sizes) and (t, lo) < (t1, l1):
        hi = l1 if t == t1 else sizes[t]
        if hi > lo:
            pieces.append((t, lo, hi))
        t, lo = t + 1, 0
    return pieces


def sample_shard(S: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous sample range [s0, s1) of `rank`."""
    return S * rank // world, S * (rank + 1) // world


def ema_weights(S: int, alpha: float, beta: float) -> np.ndarray:
    """c_t such that sum_t c_t g_t^2 equals S steps of accumulate_fisher:
    c_0 = alpha beta^(S-1), c_t = alpha (1-beta) beta^(S-1-t) for t >= 1, with
    alpha (1-beta) formed in FP32 as the reference does (ehap.hpp:164-165,195)."""
    a, b = np.float32(alpha), np.float32(beta)
    contrib = np.float32(a * (np.float32(1.0) - b))
    c = np.empty(S, np.float32)
    for t in range(S):
        powb = float(b) ** (S - 1 - t)
        c[t] = np.float32((float(a) if t == 0 else float(contrib)) * powb)
    return c


def tb_header(n: int, m: int, num_weights: int) -> bytes:
    """The 4096-byte .tb header TBWriter writes for FP32 weights
    (serialization.hpp:30-54,115-134)."""
    h = bytearray(TB_HEADER)
    num_mask = num_weights // m
    fields = [(0, "<I", 0x31304254), (4, "<I", 1), (8, "<I", n), (12, "<I", m), (16, "<Q", num_weights),
              (24, "<Q", num_mask), (32, "<Q", TB_HEADER), (40, "<Q", TB_HEADER + 4 * num_weights)]
    import struct
    for off, fmt, v in fields:
        struct.pack_into(fmt, h, off, v)
    h[48] = 0
    return bytes(h)


def create_tb(path: str, N: int, n: int, m: int) -> None:
    """Rank 0: writes the header and sizes the file so ranks can fill their slices."""
    with open(path, "wb") as f:
        f.write(tb_header(n, m, N))
        f.truncate(TB_HEADER + 4 * N + N // m)


def write_tb_slice(path: str, N: int, m: int, e0: int, w_out: np.ndarray, mask: np.ndarray) -> None:
    """Writes one rank's weights and mask bytes at their offsets in the .tb."""
    fd = os.open(path, os.O_WRONLY)
    try:
        os.pwrite(fd, np.ascontiguousarray(w_out, np.float32).tobytes(), TB_HEADER + 4 * e0)
        os.pwrite(fd, np.ascontiguousarray(mask, np.uint8).tobytes(), TB_HEADER + 4 * N + e0 // m)
    finally:
        os.close(fd)


def _check(rc: int) -> None:
    tb.check(rc)


def prune_group_sharded(dist, w: np.ndarray, w_dtype: int, g: np.ndarray, g_dtype: int, out_path: str, *,
                        n=2, m=4, **cfg) -> dict:
    """Group-sharded pass of one tensor held in host memory on every rank
    (w [N], g [S, N]); each rank prunes its range through the host-buffer entry
    and writes its slice of `out_path`.  Returns this rank's counters."""
    rank, world = dist.get_rank(), dist.get_world_size()
    N = w.size
    S = g.shape[0] if g is not None and g.size else 0
    e0, e1 = group_shard(N, m, world, rank)
    if rank == 0:
        create_tb(out_path, N, n, m)
    dist.barrier()
    L = e1 - e0
    w_out = np.empty(L, np.float32)
    mask = np.empty(L // m, np.uint8)
    ties = np.zeros(1, np.uint64)
    wsz = 4 if w_dtype == tb.F32 else 2
    gsz = 4 if g_dtype == tb.F32 else 2
    if L:
        a = tb.prune_args(weights=w.ctypes.data + e0 * wsz, w_dtype=w_dtype,
                          grads=(g.ctypes.data + e0 * gsz) if S else None, g_dtype=g_dtype, S=S, N=L,
                          g_stride=N if S else 0, n=n, m=m, w_out=w_out.ctypes.data, mask_out=mask.ctypes.data,
                          near_ties=ties.ctypes.data, **cfg)
        _check(tb.score_mask_pack_host(a))
        write_tb_slice(out_path, N, m, e0, w_out, mask)
    dist.barrier()
    return {"e0": e0, "e1": e1, "near_ties": int(ties[0])}


def prune_sample_split(dist, torch, w_dev, w_dtype: int, g_local_dev, g_dtype: int, S_total: int, s0: int,
                       out_w, out_mask, *, n=2, m=4, alpha=0.01, beta=0.99, fisher_out=None, **cfg) -> dict:
    """Sample-split pass of one tensor on the device: g_local_dev holds this
    rank's samples [s0, s0 + S_local) of all N elements.  Partial Fisher, NCCL
    all-reduce (sum), then the fused pass over this rank's group range from the
    summed Fisher.  out_w / out_mask are full-size device tensors; this rank
    fills [e0, e1).  Returns the range and near-tie count."""
    rank, world = dist.get_rank(), dist.get_world_size()
    N = w_dev.numel()
    S_local = g_local_dev.shape[0] if g_local_dev is not None else 0
    stream = torch.cuda.current_stream().cuda_stream
    F = fisher_out if fisher_out is not None else torch.empty(N, dtype=torch.float32, device=w_dev.device)
    c = ema_weights(S_total, alpha, beta)[s0:s0 + S_local].copy()
    _check(tb.lib().tb_fisher_weighted_sum(F.data_ptr(), g_local_dev.data_ptr() if S_local else None, g_dtype,
                                           S_local, N, N, c.ctypes.data if S_local else None, 0, stream))
    dist.all_reduce(F)
    e0, e1 = group_shard(N, m, world, rank)
    ties = torch.zeros(1, dtype=torch.int64, device=w_dev.device)
    if e1 > e0:
        wsz = w_dev.element_size()
        a = tb.prune_args(weights=w_dev.data_ptr() + e0 * wsz, w_dtype=w_dtype, grads=None, g_dtype=g_dtype, S=0,
                          N=e1 - e0, fisher_in=F.data_ptr() + 4 * e0, fisher_steps_in=S_total, alpha=alpha, beta=beta,
                          n=n, m=m, w_out=out_w.data_ptr() + 4 * e0, mask_out=out_mask.data_ptr() + e0 // m,
                          near_ties=ties.data_ptr(), **cfg)
        _check(tb.score_mask_pack(a, stream))
    return {"e0": e0, "e1": e1, "near_ties": ties, "fisher": F}


class PeerBuffers:
    """`count` device buffers of `nbytes` on every rank, each mapped into every
    other rank's address space (tb_ipc_handle / tb_ipc_open over the process
    group), for the sample-split pass that reads the ranks' partial Fisher sums
    straight from peer memory.  ptrs[k][r] is rank r's buffer k as this rank's
    kernels address it; local[k] is this rank's own."""

    def __init__(self, dist, nbytes: int, count: int = 2):
        self.dist = dist
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        L = tb.lib()
        self.local = []
        for _ in range(count):
            p = C.c_void_p()
            _check(L.tb_malloc(C.byref(p), nbytes))
            self.local.append(p.value)
        handles = []
        for p in self.local:
            h = C.create_string_buffer(64)
            _check(L.tb_ipc_handle(p, h))
            handles.append(h.raw)
        every = [None] * self.world
        dist.all_gather_object(every, handles)
        self.opened = []
        self.ptrs = []
        for k in range(count):
            row = []
            for r in range(self.world):
                if r == self.rank:
                    row.append(self.local[k])
                else:
                    q = C.c_void_p()
                    _check(L.tb_ipc_open(every[r][k], C.byref(q)))
                    self.opened.append(q.value)
                    row.append(q.value)
            self.ptrs.append(row)

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's; every rank must
        have finished reading (a barrier comes first)."""
        self.dist.barrier()
        L = tb.lib()
        for q in self.opened:
            _check(L.tb_ipc_close(q))
        self.dist.barrier()
        for p in self.local:
            _check(L.tb_free(p))
        self.opened, self.local, self.ptrs = [], [], []


def prune_sample_split_peer(dist, torch, bufs: PeerBuffers, k: int, w_dev, w_dtype: int, g_local_dev, g_dtype: int,
                            S_total: int, s0: int, out_w, out_mask, *, n=2, m=4, alpha=0.01, beta=0.99,
                            flag=None, fisher_out=None, near_ties=None, **cfg) -> dict:
    """Sample-split pass of one tensor with the exchange fused into the pass:
    this rank writes its partial Fisher (its samples [s0, s0 + S_local) of all
    N elements) into its exchange buffer k, a one-element all-reduce orders
    every rank's partial before any read (stream-ordered, no host wait), and
    tb_score_mask_pack_peer sums the P partials of this rank's group range from
    peer memory in rank order and prunes it.  Callers alternate k between
    consecutive tensors: the next write into buffer k comes after the next
    tensor's all-reduce, which every rank enters only after its read of buffer
    k finished.  out_w / out_mask are full-size device tensors; this rank fills
    [e0, e1)."""
    rank, world = dist.get_rank(), dist.get_world_size()
    N = w_dev.numel()
    S_local = g_local_dev.shape[0] if g_local_dev is not None else 0
    stream = torch.cuda.current_stream().cuda_stream
    L = tb.lib()
    c = ema_weights(S_total, alpha, beta)[s0:s0 + S_local].copy()
    _check(L.tb_fisher_weighted_sum(bufs.local[k], g_local_dev.data_ptr() if S_local else None, g_dtype, S_local,
                                    N, N, c.ctypes.data if S_local else None, 0, stream))
    if flag is None:
        flag = torch.zeros(1, dtype=torch.float32, device=w_dev.device)
    dist.all_reduce(flag)
    e0, e1 = group_shard(N, m, world, rank)
    if e1 > e0:
        parts = (C.c_void_p * world)(*[bufs.ptrs[k][r] + 4 * e0 for r in range(world)])
        wsz = w_dev.element_size()
        a = tb.prune_args(weights=w_dev.data_ptr() + e0 * wsz, w_dtype=w_dtype, grads=None, g_dtype=g_dtype, S=0,
                          N=e1 - e0, fisher_steps_in=S_total, alpha=alpha, beta=beta, n=n, m=m,
                          w_out=out_w.data_ptr() + 4 * e0, mask_out=out_mask.data_ptr() + e0 // m,
                          fisher_out=(fisher_out.data_ptr() + 4 * e0) if fisher_out is not None else None,
                          near_ties=near_ties.data_ptr() if near_ties is not None else None, **cfg)
        _check(L.tb_score_mask_pack_peer(C.byref(a), C.cast(parts, C.POINTER(C.c_void_p)), world, stream))
    return {"e0": e0, "e1": e1}


def push_slot(N: int, m: int, world: int) -> int:
    """Floats per writer slot in an owner's exchange buffer: the largest group
    range rounded up to 16 elements (every slot stays 64-byte aligned)."""
    longest = max(e1 - e0 for e0, e1 in (group_shard(N, m, world, r) for r in range(world)))
    return (longest + 15) // 16 * 16


def prune_sample_split_push(dist, torch, bufs: PeerBuffers, k: int, w_dev, w_dtype: int, g_local_dev, g_dtype: int,
                            S_total: int, s0: int, out_w, out_mask, *, n=2, m=4, alpha=0.01, beta=0.99,
                            flag=None, fisher_out=None, near_ties=None, **cfg) -> dict:
    """Sample-split pass of one tensor with the exchange done as writes: this
    rank's partial Fisher over its samples is computed once for all N
    elements and each owner's range is stored straight into that owner's
    exchange buffer k, in this rank's slot (tb_fisher_partial_scatter; remote
    stores over NVLink); after a one-element all-reduce (stream-ordered
    barrier) every rank sums the P slots of its own range from local memory
    inside the fused pass (tb_score_mask_pack_peer).  Buffers alternate per
    tensor as in prune_sample_split_peer; each holds P slots of push_slot()
    floats."""
    rank, world = dist.get_rank(), dist.get_world_size()
    N = w_dev.numel()
    S_local = g_local_dev.shape[0] if g_local_dev is not None else 0
    stream = torch.cuda.current_stream().cuda_stream
    L = tb.lib()
    slot = push_slot(N, m, world)
    ranges = [group_shard(N, m, world, r) for r in range(world)]
    starts = (C.c_uint64 * (world + 1))(*([e0 for e0, _ in ranges] + [N]))
    dest = (C.c_void_p * world)(*[bufs.ptrs[k][r] + 4 * rank * slot for r in range(world)])
    c = ema_weights(S_total, alpha, beta)[s0:s0 + S_local].copy()
    _check(L.tb_fisher_partial_scatter(g_local_dev.data_ptr() if S_local else None, g_dtype, S_local, N, N,
                                       c.ctypes.data if S_local else None, world, starts,
                                       C.cast(dest, C.POINTER(C.c_void_p)), (rank + 1) % world, stream))
    if flag is None:
        flag = torch.zeros(1, dtype=torch.float32, device=w_dev.device)
    dist.all_reduce(flag)
    e0, e1 = ranges[rank]
    if e1 > e0:
        parts = (C.c_void_p * world)(*[bufs.local[k] + 4 * q * slot for q in range(world)])
        wsz = w_dev.element_size()
        a = tb.prune_args(weights=w_dev.data_ptr() + e0 * wsz, w_dtype=w_dtype, grads=None, g_dtype=g_dtype, S=0,
                          N=e1 - e0, fisher_steps_in=S_total, alpha=alpha, beta=beta, n=n, m=m,
                          w_out=out_w.data_ptr() + 4 * e0, mask_out=out_mask.data_ptr() + e0 // m,
                          fisher_out=(fisher_out.data_ptr() + 4 * e0) if fisher_out is not None else None,
                          near_ties=near_ties.data_ptr() if near_ties is not None else None, **cfg)
        _check(L.tb_score_mask_pack_peer(C.byref(a), C.cast(parts, C.POINTER(C.c_void_p)), world, stream))
    return {"e0": e0, "e1": e1}


def prune_sample_split_copy(dist, torch, bufs: PeerBuffers, k: int, scratch, w_dev, w_dtype: int, g_local_dev,
                            g_dtype: int, S_total: int, s0: int, out_w, out_mask, *, n=2, m=4, alpha=0.01,
                            beta=0.99, flag=None, fisher_out=None, near_ties=None, **cfg) -> dict:
    """Sample-split pass of one tensor with the exchange on the copy engines:
    this rank's partial Fisher over its samples is written to its own
    `scratch` (a device tensor of at least N floats; tb_fisher_partial_scatter
    with every range local), each other owner's range then goes to that
    owner's exchange buffer k by one device-to-device copy over NVLink (DMA,
    no SM time), a one-element all-reduce orders the ranks, and the owner's
    fused pass sums its own partial and the P - 1 received slots from local
    memory (tb_score_mask_pack_peer).  Same bits as the other sample-split
    passes (same partials, summed in rank order).  Buffers alternate per
    tensor; `scratch` is rewritten by the next tensor only after this rank's
    copies and its own pass, which precede it on the stream."""
    rank, world = dist.get_rank(), dist.get_world_size()
    N = w_dev.numel()
    S_local = g_local_dev.shape[0] if g_local_dev is not None else 0
    stream = torch.cuda.current_stream().cuda_stream
    L = tb.lib()
    slot = push_slot(N, m, world)
    ranges = [group_shard(N, m, world, r) for r in range(world)]
    starts = (C.c_uint64 * (world + 1))(*([e0 for e0, _ in ranges] + [N]))
    base = scratch.data_ptr()
    local = (C.c_void_p * world)(*[base + 4 * e0 for e0, _ in ranges])
    c = ema_weights(S_total, alpha, beta)[s0:s0 + S_local].copy()
    _check(L.tb_fisher_partial_scatter(g_local_dev.data_ptr() if S_local else None, g_dtype, S_local, N, N,
                                       c.ctypes.data if S_local else None, world, starts,
                                       C.cast(local, C.POINTER(C.c_void_p)), rank, stream))
    for j in range(1, world):  # rank + 1 first: each peer receives from one sender at a time
        r = (rank + j) % world
        e0, e1 = ranges[r]
        if e1 > e0:
            _check(L.tb_memcpy_d2d(bufs.ptrs[k][r] + 4 * rank * slot, base + 4 * e0, 4 * (e1 - e0), stream))
    if flag is None:
        flag = torch.zeros(1, dtype=torch.float32, device=w_dev.device)
    dist.all_reduce(flag)
    e0, e1 = ranges[rank]
    if e1 > e0:
        parts = (C.c_void_p * world)(*[(base + 4 * e0) if q == rank else (bufs.local[k] + 4 * q * slot)
                                       for q in range(world)])
        wsz = w_dev.element_size()
        a = tb.prune_args(weights=w_dev.data_ptr() + e0 * wsz, w_dtype=w_dtype, grads=None, g_dtype=g_dtype, S=0,
                          N=e1 - e0, fisher_steps_in=S_total, alpha=alpha, beta=beta, n=n, m=m,
                          w_out=out_w.data_ptr() + 4 * e0, mask_out=out_mask.data_ptr() + e0 // m,
                          fisher_out=(fisher_out.data_ptr() + 4 * e0) if fisher_out is not None else None,
                          near_ties=near_ties.data_ptr() if near_ties is not None else None, **cfg)
        _check(L.tb_score_mask_pack_peer(C.byref(a), C.cast(parts, C.POINTER(C.c_void_p)), world, stream))
    return {"e0": e0, "e1": e1}


class CopyExchangePipeline:
    """The copy-engine sample split over a sequence of tensors, with the
    exchange of tensor t overlapped with the partial of tensor t + 1.

    Tensors are numbered u = 0, 1, 2, ... over every run() of the pipeline.
    Per tensor u: the partial (over this rank's samples) goes to scratch
    buffer u % 2 on the compute stream; a copy stream waits for it, copies
    each other owner's range into that owner's exchange buffer u % 3 (rank + 1
    first) and runs the one-element all-reduce that orders the ranks; the
    compute stream meanwhile computes the partial of tensor u + 1, then waits
    for the exchange of u and runs the fused pass that sums the P slots of
    its range.  Why the buffers suffice: on the compute stream the partial of
    u + 2 is queued after the pass of u (also across runs, which is why the
    numbering continues); a scratch buffer is rewritten by the partial of
    u + 2, after this rank's pass of u, which waited for the copies of u; an
    exchange buffer is rewritten by a peer's copies of u + 3, which follow
    that peer's all-reduce of u + 2, which no rank enters before its partial
    of u + 2, which follows its pass of u.  Same bits as
    prune_sample_split_copy."""

    def __init__(self, dist, torch, n_max: int, m: int):
        self.dist, self.torch, self.m = dist, torch, m
        self.rank, self.world = dist.get_rank(), dist.get_world_size()
        dev = torch.device("cuda", torch.cuda.current_device())
        self.bufs = PeerBuffers(dist, 4 * max(n_max, self.world * push_slot(n_max, m, self.world)), 3)
        self.scratch = [torch.empty(n_max, dtype=torch.float32, device=dev) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(device=dev)
        self.flag = torch.zeros(1, dtype=torch.float32, device=dev)
        self.ev_part = [torch.cuda.Event() for _ in range(2)]
        self.ev_done = [torch.cuda.Event() for _ in range(2)]
        self.count = 0  # tensors queued so far: buffers keep rotating from one run to the next

    def close(self):
        self.torch.cuda.synchronize()
        self.bufs.close()

    def run(self, jobs, S_total: int, s0: int, *, n=2, alpha=0.01, beta=0.99, near_ties=None, **cfg):
        """jobs: [(w_dev, w_dtype, g_local_dev, g_dtype, out_w, out_mask)], each a
        tensor's N weights, this rank's samples [s0, s0 + S_local) of all N
        elements ([S_local, N], contiguous), and the outputs of this rank's
        group range [e0, e1) = group_shard(N, m, world, rank): out_w holds
        e1 - e0 FP32 weights, out_mask (e1 - e0) / m mask bytes (views
        out_w_full[e0:e1] and out_mask_full[e0 // m : e1 // m] of full-size
        outputs do).  Work is queued on the current stream and the pipeline's
        copy stream; the call returns without a host wait."""
        torch, L, m, world, rank = self.torch, tb.lib(), self.m, self.world, self.rank
        compute = torch.cuda.current_stream()
        cp = self.copy_stream
        ev_part, ev_done, u0 = self.ev_part, self.ev_done, self.count
        plans = []
        for (w, wdt, g, gdt, ow, om) in jobs:
            N = w.numel()
            if N > self.scratch[0].numel():
                raise ValueError(f"tensor of {N} elements exceeds the pipeline's n_max {self.scratch[0].numel()}")
            ranges = [group_shard(N, m, world, r) for r in range(world)]
            plans.append((N, ranges, push_slot(N, m, world)))

        def partial(t):
            (w, wdt, g, gdt, ow, om), (N, ranges, slot) = jobs[t], plans[t]
            S_local = g.shape[0] if g is not None else 0
            c = ema_weights(S_total, alpha, beta)[s0:s0 + S_local].copy()
            base = self.scratch[(u0 + t) % 2].data_ptr()
            starts = (C.c_uint64 * (world + 1))(*([e0 for e0, _ in ranges] + [N]))
            local = (C.c_void_p * world)(*[base + 4 * e0 for e0, _ in ranges])
            _check(L.tb_fisher_partial_scatter(g.data_ptr() if S_local else None, gdt, S_local, N, N,
                                               c.ctypes.data if S_local else None, world, starts,
                                               C.cast(local, C.POINTER(C.c_void_p)), rank, compute.cuda_stream))
            ev_part[(u0 + t) % 2].record(compute)

        def exchange(t):
            (N, ranges, slot), k = plans[t], (u0 + t) % 3
            base = self.scratch[(u0 + t) % 2].data_ptr()
            cp.wait_event(ev_part[(u0 + t) % 2])
            for j in range(1, world):
                r = (rank + j) % world
                e0, e1 = ranges[r]
                if e1 > e0:
                    _check(L.tb_memcpy_d2d(self.bufs.ptrs[k][r] + 4 * rank * slot, base + 4 * e0, 4 * (e1 - e0),
                                           cp.cuda_stream))
            with torch.cuda.stream(cp):
                self.dist.all_reduce(self.flag)
            ev_done[(u0 + t) % 2].record(cp)

        def consume(t):
            (w, wdt, g, gdt, ow, om), (N, ranges, slot) = jobs[t], plans[t]
            k = (u0 + t) % 3
            compute.wait_event(ev_done[(u0 + t) % 2])
            e0, e1 = ranges[rank]
            if e1 <= e0:
                return
            base = self.scratch[(u0 + t) % 2].data_ptr()
            parts = (C.c_void_p * world)(*[(base + 4 * e0) if q == rank else (self.bufs.local[k] + 4 * q * slot)
                                           for q in range(world)])
            a = tb.prune_args(weights=w.data_ptr() + e0 * w.element_size(), w_dtype=wdt, grads=None, g_dtype=gdt,
                              S=0, N=e1 - e0, fisher_steps_in=S_total, alpha=alpha, beta=beta, n=n, m=m,
                              w_out=ow.data_ptr(), mask_out=om.data_ptr(),
                              near_ties=near_ties.data_ptr() if near_ties is not None else None, **cfg)
            _check(L.tb_score_mask_pack_peer(C.byref(a), C.cast(parts, C.POINTER(C.c_void_p)), world,
                                             compute.cuda_stream))

        if not jobs:
            return
        partial(0)
        for t in range(len(jobs)):
            exchange(t)
            if t + 1 < len(jobs):
                partial(t + 1)
            consume(t)
        self.count += len(jobs)


# ---- column-block exact OBS --------------------------------------------------
OBS_ROW_UNIT = 128   # rows of W per unit (tb_obs_sparsegpt takes multiples of 128)
OBS_TOKEN_UNIT = 64  # tokens per unit (tb_obs_hessian_scaled takes multiples of 64)


def obs_row_shard(r: int, world: int, rank: int) -> tuple[int, int]:
    """Row range [r0, r1) of W for `rank`: whole 128-row units, balanced."""
    if r % OBS_ROW_UNIT:
        raise ValueError(f"rows {r} not a multiple of {OBS_ROW_UNIT}")
    units = r // OBS_ROW_UNIT
    return units * rank // world * OBS_ROW_UNIT, units * (rank + 1) // world * OBS_ROW_UNIT


def token_shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Token range [t0, t1) of `rank`: whole 64-token units, balanced."""
    if n % OBS_TOKEN_UNIT:
        raise ValueError(f"tokens {n} not a multiple of {OBS_TOKEN_UNIT}")
    units = n // OBS_TOKEN_UNIT
    return units * rank // world * OBS_TOKEN_UNIT, units * (rank + 1) // world * OBS_TOKEN_UNIT


def obs_hessian_token_split(dist, torch, xt_local_dev, d: int, n_total: int, H, events=None) -> None:
    """H = X^T X / n_total over all ranks' tokens.  xt_local_dev is this rank's
    tokens as X^T (BF16 [d][n_local], n_local a multiple of 64, may be None
    for no tokens); H is a d x d FP32 device tensor, overwritten.  The partial
    is formed with scale 1/n_total, so the all-reduced sum needs no rescaling;
    tiles above the diagonal stay zero on every rank and sum to zero.
    `events` (two CUDA events, optional) are recorded on the current stream
    just before and after the all-reduce, for timing it."""
    stream = torch.cuda.current_stream().cuda_stream
    H.zero_()
    n_local = xt_local_dev.shape[1] if xt_local_dev is not None else 0
    if n_local:
        _check(tb.lib().tb_obs_hessian_scaled(xt_local_dev.data_ptr(), d, n_local, 1.0 / n_total, H.data_ptr(),
                                              stream))
    if events:
        events[0].record()
    dist.all_reduce(H)
    if events:
        events[1].record()


def prune_obs_row_split(dist, torch, W_local, H, mask_local, *, damp_frac=0.01, n_keep=2, m=4) -> None:
    """Prunes this rank's rows of W (FP32 device [rows][d], in place) against
    the all-reduced H; mask_local gets rows * d / 4 bytes.  The Cholesky factor
    of H^-1 is computed on every rank (it is the same on all of them)."""
    rows, d = W_local.shape
    if rows == 0:
        return
    stream = torch.cuda.current_stream().cuda_stream
    _check(tb.lib().tb_obs_sparsegpt(W_local.data_ptr(), rows, d, H.data_ptr(), damp_frac, n_keep, m,
                                     mask_local.data_ptr(), None, stream))

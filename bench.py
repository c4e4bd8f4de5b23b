"""Throughput of the fused score -> 2:4 mask -> pack pass on B200.

Workload (default): a 7B-class decoder - 32 layers of
q/k/v/o (4096x4096, 1024x4096 x2, 4096x4096), gate/up (14336x4096) and down
(4096x14336) BF16 matrices, 6,979,321,856 prunable parameters - each matrix
with 64 BF16 gradient samples ~ N(0, 1e-3^2), weights ~ N(0, 0.02^2); Fisher EMA
(alpha 0.01, beta 0.99), OBD scoring (lambda 0.01), optimal C(4,2) 2:4 mask,
proportional redistribution, FP32 weights + packed mask bytes written.

One step = the whole 32-layer pass (224 fused launches).  Gradients for all 32
layers do not fit in HBM (~0.9 TB), so two resident random-init layer sets (A,
B; 29 GB each) alternate layer by layer; every launch streams 0.5-7.6 GB, far
above the 126 MB L2, so no L2 flush is needed between launches.  Each rank runs
the same per-rank job (weak scaling): the path has no cross-rank data
dependency, only the timing barrier and max-over-ranks reduction.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tensorbit-core_b200"))

LAYER = [("q_proj", 4096, 4096), ("k_proj", 1024, 4096), ("v_proj", 1024, 4096),
         ("o_proj", 4096, 4096), ("gate_proj", 14336, 4096), ("up_proj", 14336, 4096),
         ("down_proj", 4096, 14336)]
LAYERS = 32
S = 64
PARAMS_PER_LAYER = sum(r * c for _, r, c in LAYER)          # 218,103,808
PARAMS_PER_STEP = PARAMS_PER_LAYER * LAYERS                   # 6,979,321,856
BYTES_PER_PARAM = 2 + 2 * S + 4 + 0.25                        # W bf16 + 64 grads bf16 + W' f32 + mask
METRIC = "2:4 score+mask+pack Gparams/s at 1/2/4/8 B200; % HBM roofline; OBS TFLOP/s"
WORKLOAD = "7B-class decoder (32 layers, hidden 4096, inter 14336, 32q/8kv heads x128), 64 BF16 grads/tensor, OBD, optimal 2:4 + proportional redistribution"


def parse():
    global LAYER, LAYERS, PARAMS_PER_LAYER, PARAMS_PER_STEP
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-obs", action="store_true", help="skip the column-block exact OBS measurement")
    ap.add_argument("--no-block-obs", action="store_true", help="skip the reference-semantics block OBS timing")
    ap.add_argument("--no-ties", action="store_true", help="skip the untimed near-tie counting pass")
    ap.add_argument("--obs-only", action="store_true", help="only the column-block exact OBS measurement")
    ap.add_argument("--block-obs-only", action="store_true", help="only the reference-semantics block OBS timing")
    ap.add_argument("--block-obs-size", type=int, default=4096 * 4096,
                    help="weights of the block OBS tensor (default one 4096 x 4096 q_proj)")
    ap.add_argument("--obs-steps", type=int, default=3)
    ap.add_argument("--obs-shape", type=int, nargs=3, metavar=("R", "D", "N"),
                    help="rows, columns and tokens of the exact-OBS pass (default: the 4096 x 14336, 2048-token down_proj)")
    ap.add_argument("--gemm-probe", type=int, nargs=3, metavar=("M", "N", "K"),
                    help="time the tcgen05 NT GEMM (3xTF32 and BF16) at one shape and exit")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decoder layers per step (profiling a smaller case only; default 32)")
    ap.add_argument("--matrices", default="",
                    help="comma list restricting the per-layer matrices (profiling only), e.g. q_proj")
    a = ap.parse_args()
    if a.matrices:
        keep = set(a.matrices.split(","))
        LAYER = [x for x in LAYER if x[0] in keep]
    LAYERS = a.layers
    PARAMS_PER_LAYER = sum(r * c for _, r, c in LAYER)
    PARAMS_PER_STEP = PARAMS_PER_LAYER * LAYERS
    return a


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    """nvidia-smi samples (200 ms) of this rank's GPU while the timed region runs."""
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, uuid: str, index: str):
        self.uuid, self.index = uuid.lower(), str(index)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            return None
        rows = [[x.strip() for x in line.split(",")] for line in out.strip().splitlines()]
        rows = [r for r in rows if len(r) >= 9]
        mine = [r for r in rows if self.uuid and r[1].lower().endswith(self.uuid)]
        if not mine:
            mine = [r for r in rows if r[0] == self.index]
        sm, mx, power, reasons = [], [], [], set()
        for r in mine:
            try:
                sm.append(float(r[2]))
                mx.append(float(r[3]))
                power.append(float(r[4]))
            except ValueError:
                continue
            for nm, v in zip(self.NAMES, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "power_w_max": max(power),
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# roofline denominators and ncu traffic
# ---------------------------------------------------------------------------
def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic_per_param():
    """dram bytes read+written per parameter of the fused BF16 2:4 kernel from the
    committed ncu summary (profiles/), or None when no capture is committed."""
    p = os.path.join(ROOT, "profiles", "fused_vec_bf16_2of4_traffic.txt")
    if not os.path.exists(p):
        return None
    m = re.search(r"dram_bytes_per_param\s*=\s*([0-9.]+)", open(p).read())
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def make_layer_set(torch, gen, dev):
    tensors = []
    for name, r, c in LAYER:
        n = r * c
        w = (torch.randn(n, device=dev, generator=gen, dtype=torch.bfloat16) * 0.02)
        g = (torch.randn(S, n, device=dev, generator=gen, dtype=torch.bfloat16) * 1e-3)
        w_out = torch.empty(n, device=dev, dtype=torch.float32)
        mask = torch.empty(n // 4, device=dev, dtype=torch.uint8)
        tensors.append((name, n, w, g, w_out, mask))
    return tensors


def prune_args_for(tb, n, w_ptr, g_ptr, w_out_ptr, mask_ptr, g_stride=0):
    return tb.prune_args(weights=w_ptr, w_dtype=tb.BF16, grads=g_ptr, g_dtype=tb.BF16, S=S, N=n,
                         g_stride=g_stride, alpha=0.01, beta=0.99, damping=0.01, mode="obd",
                         use_fisher=True, n=2, m=4, strategy="optimal", redist="proportional",
                         w_out=w_out_ptr, mask_out=mask_ptr)


def run_ours(args):
    import torch
    import torch.distributed as dist
    import tbabi as tb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    tb.lib()
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    if args.gemm_probe:
        if rank == 0:
            print(json.dumps({"gemm_probe": gemm_probe(torch, tb, dev, *args.gemm_probe)}), flush=True)
        return
    if args.block_obs_only:
        if rank == 0:
            print(json.dumps({"block_obs": run_block_obs(torch, tb, dev, n=args.block_obs_size,
                                                         cpu=not args.no_cpu)}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.obs_only:
        obs = run_obs(torch, tb, dev, args.obs_steps, args.obs_shape, dist if world > 1 else None)
        if rank == 0:
            print(json.dumps({"metric": METRIC, "obs": obs, "n_gpus": world}), flush=True)
        if world > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()
        return

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = [make_layer_set(torch, gen, dev), make_layer_set(torch, gen, dev)]
    plan = []
    for layer in range(LAYERS):
        for (name, n, w, g, w_out, mask) in sets[layer % 2]:
            plan.append((n, prune_args_for(tb, n, w.data_ptr(), g.data_ptr(), w_out.data_ptr(), mask.data_ptr())))
    torch.cuda.synchronize()

    def step(events=None):
        for i, (n, a) in enumerate(plan):
            if events is not None:
                events[i][0].record(stream)
            rc = tb.lib().tb_score_mask_pack(C.byref(a), sptr)
            if rc:
                tb.check(rc)
            if events is not None:
                events[i][1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    events = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in plan]
              for _ in range(args.steps)]
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    phys = vis.split(",")[local] if vis and len(vis.split(",")) > local else str(local)
    clocks = Clocks(str(getattr(torch.cuda.get_device_properties(dev), "uuid", "")), phys)
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for k in range(args.steps):
        step(events[k])
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize()
    clk = clocks.stop()
    elapsed_ms = t0.elapsed_time(t1)
    kernel_ms = sum(a.elapsed_time(b) for ev in events for a, b in ev)
    launches = args.steps * len(plan)
    t = torch.tensor([elapsed_ms, kernel_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, kernel_ms = t.tolist()

    params_total = PARAMS_PER_STEP * args.steps * world
    value = params_total / (elapsed_ms / 1e3) / 1e9
    peak, peak_kind = hbm_peak()
    per_launch_bytes = PARAMS_PER_STEP * BYTES_PER_PARAM / len(plan)
    achieved = per_launch_bytes / (kernel_ms / launches / 1e3) / 1e9
    traffic_pp = ncu_traffic_per_param()

    # ---- near-tie groups of the pass (one extra, untimed pass with the counter) --
    ties = None
    if not args.no_ties:
        cnt = torch.zeros(1, dtype=torch.int64, device=dev)
        for _, a in plan:
            a.near_ties = cnt.data_ptr()
            rc = tb.lib().tb_score_mask_pack(C.byref(a), sptr)
            a.near_ties = None
            if rc:
                raise tb.TbError(rc, tb.lib().tb_last_error().decode())
        torch.cuda.synchronize()
        groups = PARAMS_PER_STEP // 4
        ties = {"groups": groups, "near_tie_groups": int(cnt.item()),
                "rule": "|s(N) - s(N+1)| <= 1e-6 max(|s(N)|, FLT_MIN) among a group's sorted scores; the masks of "
                        "these groups are bit-exact too (the reference's selection and tie order are reproduced, "
                        "for top-N through its nth_element tie tables)"}

    # ---- end to end through the host-buffer entry point --------------------
    e2e = None
    del sets
    torch.cuda.empty_cache()
    if not args.no_e2e:
        e2e = run_e2e(torch, tb, dev, gen, args, world, rank, local)

    # ---- column-block exact OBS on tensor cores ------------------------------
    obs = None
    if not args.no_obs:
        obs = run_obs(torch, tb, dev, args.obs_steps, args.obs_shape, dist if world > 1 else None)

    # ---- reference-semantics block OBS (wall time; rank 0, single GPU) ------
    block_obs = None
    if rank == 0 and world == 1 and not args.no_block_obs:
        block_obs = run_block_obs(torch, tb, dev, cpu=not args.no_cpu)

    # ---- CPU baseline (rank 0, single GPU only) ----------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(torch, dev, threads=os.cpu_count() or 1, seconds=4.0)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 3),
            "unit": "Gparams/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded torch Philox; random-init weights and gradients of the 7B shapes)",
            "config": {"workload": WORKLOAD, "params_per_rank_step": PARAMS_PER_STEP, "grad_samples": S,
                       "weights": "bf16", "grads": "bf16", "outputs": "fp32 weights + u8 mask",
                       "layer_sets_resident": 2,
                       "l2": "no flush: every launch streams 0.5-7.6 GB >> 126 MB L2",
                       "parallelism": f"weak: {world} rank(s), each its own 32-layer pass, no data-path collective"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_param": BYTES_PER_PARAM,
                         "traffic": (round(traffic_pp * PARAMS_PER_STEP / len(plan)) if traffic_pp else None),
                         "traffic_per_param": traffic_pp,
                         "kernel": "fused_vec_kernel<BF16,BF16,M=4>",
                         "kernel_ms_total": round(kernel_ms, 3)},
            "gpu_launches": launches,
            "near_ties": ties,
            "clocks": clk,
            "e2e": e2e,
            "obs": obs,
            "block_obs": block_obs,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_e2e(torch, tb, dev, gen, args, world, rank, local):
    """Same metric through tb_score_mask_pack_host with pinned host buffers: every
    step copies that step's inputs host->device and the results back inside the
    timed region.  One step = one decoder layer (7 matrices, 218,103,808 params);
    the 7B pass is 32 identical layers."""
    import torch.distributed as dist
    nmax = max(r * c for _, r, c in LAYER)
    hw = torch.empty(nmax, dtype=torch.bfloat16, pin_memory=True)
    hg = torch.empty(S, nmax, dtype=torch.bfloat16, pin_memory=True)
    hwo = torch.empty(nmax, dtype=torch.float32, pin_memory=True)
    hm = torch.empty(nmax // 4, dtype=torch.uint8, pin_memory=True)
    hw.copy_((torch.randn(nmax, device=dev, generator=gen) * 0.02).to(torch.bfloat16))
    for s0 in range(0, S, 8):
        hg[s0:s0 + 8].copy_((torch.randn(8, nmax, device=dev, generator=gen) * 1e-3).to(torch.bfloat16))
    torch.cuda.synchronize()
    calls = []
    h2d = d2h = 0
    for name, r, c in LAYER:
        n = r * c
        # All matrices read the leading n columns of the shared pinned buffers.
        calls.append(prune_args_for(tb, n, hw.data_ptr(), hg.data_ptr(), hwo.data_ptr(), hm.data_ptr(), g_stride=nmax))
        h2d += n * 2 + S * n * 2
        d2h += n * 4 + n // 4

    def layer():
        for a in calls:
            tb.check(tb.lib().tb_score_mask_pack_host(C.byref(a)))

    layer()  # warm-up: staging buffers, streams
    if world > 1:
        dist.barrier(device_ids=[local])
    t0 = time.perf_counter()
    for _ in range(args.e2e_steps):
        layer()
    el = time.perf_counter() - t0
    t = torch.tensor([el], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    el = t.item()
    value = PARAMS_PER_LAYER * args.e2e_steps * world / el / 1e9
    return {"value": round(value, 4), "unit": "Gparams/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": args.e2e_steps, "step": "one decoder layer (7 matrices) via tb_score_mask_pack_host, pinned host memory",
            "s_per_step": round(el / args.e2e_steps, 4)}


# ---------------------------------------------------------------------------
# column-block exact OBS on tensor cores
# ---------------------------------------------------------------------------
OBS_D, OBS_R, OBS_N, OBS_B = 14336, 4096, 2048, 128


def obs_flops(d, r, n):
    """Algorithmic FLOPs of one exact-OBS pass, independent of how the kernels
    split the work: X^T X on the lower triangle (d(d+1)/2 dot products of
    length n, 2 flops per term), Cholesky d^3/3, triangular inverse d^3/3, and
    the column sweep r d^2 (column q's error updates the d-q later columns of
    its row: sum over q of 2 r (d - q))."""
    return d * (d + 1) * n + 2 * d ** 3 // 3 + r * d * d


def gemm_probe(torch, tb, dev, M, N, K, reps=5):
    """TFLOP/s of the tcgen05 NT GEMM at one shape (each product counted once)."""
    L = tb.lib()
    sptr = torch.cuda.current_stream().cuda_stream
    A = torch.randn(M, K, device=dev)
    B = torch.randn(N, K, device=dev)
    C = torch.empty(M, N, device=dev)
    ah, al, bh, bl = (torch.empty_like(A), torch.empty_like(A), torch.empty_like(B), torch.empty_like(B))
    tb.check(L.tb_split_tf32(A.data_ptr(), ah.data_ptr(), al.data_ptr(), A.numel(), sptr))
    tb.check(L.tb_split_tf32(B.data_ptr(), bh.data_ptr(), bl.data_ptr(), B.numel(), sptr))
    Ab, Bb = A.bfloat16(), B.bfloat16()
    out = {"shape": [M, N, K]}
    for kind in ("tf32x3", "bf16"):
        def once():
            if kind == "tf32x3":
                return L.tb_gemm_nt_tf32x3(ah.data_ptr(), al.data_ptr(), K, bh.data_ptr(), bl.data_ptr(), K, M, N, K,
                                           1.0, 0.0, None, N, C.data_ptr(), N, 0, sptr)
            return L.tb_gemm_nt_bf16(Ab.data_ptr(), K, Bb.data_ptr(), K, M, N, K, 1.0, 0.0, None, N, C.data_ptr(), N,
                                     0, sptr)
        tb.check(once())
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            tb.check(once())
        e1.record()
        torch.cuda.synchronize()
        tb.check(L.tb_gemm_status(sptr))
        ms = e0.elapsed_time(e1) / reps
        out[kind] = {"ms": round(ms, 3), "tflops": round(2 * M * N * K / ms / 1e9, 1)}
    return out


def sparsegpt_flops(d, r, n):
    """FLOPs of the standard column-block OBS formulation (full X^T X, Cholesky
    of H, explicit inverse, Cholesky of H^-1, lazy updates, in-block), the
    count a route that forms H^-1 explicitly performs."""
    return 2 * n * d * d + d ** 3 // 3 + 2 * d ** 3 // 3 + d ** 3 // 3 + r * d * d + r * d * 128


def run_obs(torch, tb, dev, steps, shape=None, dist=None):
    """Column-block exact OBS of one down_proj on tensor cores.  With several ranks the tokens are
    split for X^T X (one NCCL all-reduce of H) and the rows of W for the sweep;
    the factorisation of H is replicated on every rank.  Time per pass is the
    maximum over ranks."""
    import tbdist as td
    OBS_R, OBS_D, OBS_N = shape or (globals()["OBS_R"], globals()["OBS_D"], globals()["OBS_N"])
    world = dist.get_world_size() if dist is not None else 1
    rank = dist.get_rank() if dist is not None else 0
    gen = torch.Generator(device=dev).manual_seed(4)
    X = torch.randn(OBS_N, OBS_D, device=dev, generator=gen)
    hot = torch.randperm(OBS_D, device=dev, generator=gen)[: OBS_D // 100]
    X[:, hot] *= 20
    t0, t1 = td.token_shard(OBS_N, world, rank)
    xt = X[t0:t1].t().contiguous().to(torch.bfloat16)
    del X
    r0, r1 = td.obs_row_shard(OBS_R, world, rank)
    W0 = (torch.randn(OBS_R, OBS_D, device=dev, generator=gen) * 0.02).to(torch.bfloat16).float()[r0:r1].contiguous()
    W = torch.empty_like(W0)
    H = torch.zeros(OBS_D, OBS_D, device=dev)
    mask = torch.empty(max(1, (r1 - r0) * OBS_D // 4), dtype=torch.uint8, device=dev)
    L = tb.lib()
    sptr = torch.cuda.current_stream().cuda_stream
    ms = []
    for k in range(steps + 1):  # the first pass warms up (workspace, module load)
        W.copy_(W0)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if world > 1:
            td.obs_hessian_token_split(dist, torch, xt, OBS_D, OBS_N, H)
            td.prune_obs_row_split(dist, torch, W, H, mask)
        else:
            tb.check(L.tb_obs_hessian(xt.data_ptr(), OBS_D, OBS_N, H.data_ptr(), sptr))
            tb.check(L.tb_obs_sparsegpt(W.data_ptr(), OBS_R, OBS_D, H.data_ptr(), 0.01, 2, 4, mask.data_ptr(),
                                        None, sptr))
        e1.record()
        torch.cuda.synchronize()
        if k:
            ms.append(e0.elapsed_time(e1))
    pop = sum(((mask >> b) & 1).int() for b in range(4))
    assert r1 == r0 or bool((pop == 2).all()), "OBS mask is not 2:4"
    t = torch.tensor([sum(ms) / len(ms)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t = float(t.item())
    f = obs_flops(OBS_D, OBS_R, OBS_N)
    fs = sparsegpt_flops(OBS_D, OBS_R, OBS_N)
    bf16_peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"] \
        if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")) else 1590.0
    tflops = f / (t / 1e3) / 1e12
    return {"workload": f"column-block exact OBS: {OBS_R}x{OBS_D} down_proj (BF16 -> FP32), X {OBS_N}x{OBS_D} BF16 N(0,1) with 1% columns x20, "
                        "damp 0.01 mean(diag), 128-column blocks, 2:4",
            "ms_per_pass": round(t, 2), "passes": steps, "flops_per_pass": f, "tflops": round(tflops, 1),
            "unit": "TFLOP/s", "flop_count": "algorithmic for this route: d(d+1)n + 2d^3/3 + r d^2 (bench.obs_flops)",
            "sparsegpt_flops_per_pass": fs,
            "tflops_sparsegpt_equivalent": round(fs / (t / 1e3) / 1e12, 1),
            "parallelism": (f"{world} ranks: tokens split for X^T X + NCCL all-reduce of H, factorisation replicated, "
                            f"rows split for the sweep" if world > 1 else "1 GPU"),
            "tensor_peak_bf16_tflops": bf16_peak,
            "frac_of_bf16_peak": round(tflops / bf16_peak, 4),
            "frac_of_3xtf32_ceiling": round(tflops / (bf16_peak / 2 / 3), 4)}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own CPU code (oracle/_ref) or the port
# ---------------------------------------------------------------------------
def run_block_obs(torch, tb, dev, passes=3, n=4096 * 4096, cpu=True):
    """tb-prune --strategy BlockOBS on one 4096 x 4096 q_proj (n weights; the reference's
    prune_block_obs semantics: 128-element blocks, Fisher from one gradient
    sample, four scaled snapshots of it, sparsity 0.5): wall time per tensor,
    and the reference's own CPU code (one thread, as it runs) on a bounded
    sample of the same tensor's blocks, per block."""
    import numpy as np
    block, K = 128, 4
    gen = torch.Generator(device=dev).manual_seed(77)
    w0 = torch.randn(n, device=dev, generator=gen) * 0.02
    g = torch.randn(n, device=dev, generator=gen) * 1e-3
    F = (g * g) * 0.01
    hist = [g * (0.9 + 0.02 * k) for k in range(K)]
    ptrs = (C.c_void_p * K)(*[h.data_ptr() for h in hist])
    w = torch.empty_like(w0)
    L = tb.lib()
    ms = []
    pruned = C.c_uint64()
    for k in range(passes + 1):  # the first pass warms up
        w.copy_(w0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        tb.check(L.tb_block_obs(w.data_ptr(), F.data_ptr(), ptrs, K, n, block, 0.5, 0.01, 0.01, C.byref(pruned),
                                torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        if k:
            ms.append((time.perf_counter() - t0) * 1e3)
    t = statistics.median(ms)
    shape = "one 4096x4096 q_proj" if n == 4096 * 4096 else f"{n} weights"
    out = {"workload": f"tb-prune BlockOBS on {shape} (FP32 weights), 128-element blocks, Fisher from "
                       "one gradient sample, 4 scaled snapshots, sparsity 0.5, damping 0.01",
           "ms_per_tensor": round(t, 2), "passes": passes, "blocks": n // block,
           "blocks_per_s": round(n / block / (t / 1e3)), "gparams_per_s": round(n / (t / 1e3) / 1e9, 4),
           "pruned": pruned.value}
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, ref_available
    if cpu and ref_available() and n >= 256 * block:
        m = 256 * block  # the tensor's first 256 blocks
        wc = w0[:m].cpu().numpy()
        gc = g[:m].cpu().numpy()[None, :]
        hc = np.stack([h[:m].cpu().numpy() for h in hist])
        o = Oracle("ref")
        t0 = time.perf_counter()
        rc, _, _ = o.block_obs(wc, gc, hc, block=block, sparsity=0.5)
        el = time.perf_counter() - t0
        assert rc == 0, rc
        out["cpu_reference"] = {"blocks_per_s": round(256 / el, 1), "cores": 1, "kind": "reference",
                                "sample": f"the first 256 blocks (32,768 params) of the same tensor, one thread, "
                                          f"{el:.2f} s",
                                "ms_per_tensor_extrapolated": round(el / 256 * (n // block) * 1e3)}
    return out


def cpu_sample(torch, dev):
    import numpy as np
    n = 4096 * 4096
    gen = torch.Generator(device=dev).manual_seed(99)
    w = (torch.randn(n, device=dev, generator=gen) * 0.02).to(torch.bfloat16).float().cpu().numpy()
    g = (torch.randn(S, n, device=dev, generator=gen) * 1e-3).to(torch.bfloat16).float().cpu().numpy()
    return np.ascontiguousarray(w), np.ascontiguousarray(g), n


def cpu_baseline(torch, dev, threads, seconds):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, ref_available
    kind = "reference" if ref_available() else "port"
    w, g, n = cpu_sample(torch, dev)
    if kind == "reference":
        o = Oracle("ref")
        run = lambda: o.parallel_pass(w.copy(), g, mode="obd", n=2, m=4, strategy="optimal",
                                      redist="proportional", threads=threads)
    else:
        o = Oracle("port")
        run = lambda: (o.pipeline(w, g, mode="obd", strategy="optimal", redist="proportional")[0], None)
        threads = 1
    done = 0
    t0 = time.perf_counter()
    while True:
        rc, _ = run()
        assert rc == 0, rc
        done += 1
        if time.perf_counter() - t0 >= seconds:
            break
    el = time.perf_counter() - t0
    return {"value": round(n * done / el / 1e9, 5), "unit": "Gparams/s", "cores": threads, "kind": kind,
            "sample": f"one 4096x4096 matrix (16,777,216 params) with 64 FP32-widened BF16 gradient samples, "
                      f"OBD + optimal 2:4 + proportional, {threads} contiguous shards on {threads} threads, "
                      f"{done} pass(es) in {el:.1f} s"}


def run_reference(args):
    """Reference arm: the reference's CPU implementation of this path on the
    host cores (rank 0 only), same metric and unit."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle, ref_available
    kind = "reference" if ref_available() else "port"
    threads = os.cpu_count() or 1
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cuda":
        w, g, n = cpu_sample(torch, dev)
    else:
        import numpy as np
        n = 4096 * 4096
        rng = np.random.default_rng(99)
        w = (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02))
        g = (rng.standard_normal((S, n), dtype=np.float32) * np.float32(1e-3))
    o = Oracle("ref" if kind == "reference" else "port")

    def one():
        if kind == "reference":
            rc, _ = o.parallel_pass(w.copy(), g, mode="obd", n=2, m=4, strategy="optimal",
                                    redist="proportional", threads=threads)
        else:
            rc = o.pipeline(w, g, mode="obd", strategy="optimal", redist="proportional")[0]
        assert rc == 0

    for _ in range(args.warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one()
    el = time.perf_counter() - t0
    value = n * args.steps / el / 1e9
    cores = threads if kind == "reference" else 1
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "Gparams/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample_per_step": "one 4096x4096 matrix, 64 FP32-widened BF16 gradient samples"},
        "cpu_baseline": {"value": round(value, 5), "unit": "Gparams/s", "cores": cores, "kind": kind,
                         "sample": f"per step one 4096x4096 matrix (16,777,216 params) x 64 samples, {cores} shard(s) on {cores} thread(s)"},
        "e2e": {"value": round(value, 5), "unit": "Gparams/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

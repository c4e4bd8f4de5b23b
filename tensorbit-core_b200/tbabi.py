"""ctypes binding of the C ABI in include/tb_kernels.h.

This is the same boundary a foreign host would bind through cgo or JNI: plain
pointers, sizes and int status codes.  Device
pointers are passed as integers (e.g. ``tensor.data_ptr()``), streams as
``torch.cuda.current_stream().cuda_stream``.

Loading fails loudly if the library has not been built: there is no CPU
fallback behind this module.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
# TB_LIB may name another build of the same library (e.g. one compiled with
# different tuning constants); the in-tree build is the default.
LIB_PATH = os.environ.get("TB_LIB") or os.path.join(PKG, "lib", "libtb_b200.so")
HEADER = os.path.join(ROOT, "include", "tb_kernels.h")

TB_OK, TB_ERR_SHAPE, TB_ERR_ZERO_SIZE, TB_ERR_CONFIG, TB_ERR_CUDA = 0, -1, -2, -3, -4
TB_ERR_TIMEOUT, TB_ERR_UNSUPPORTED, TB_ERR_ARG, TB_ERR_NO_DEVICE, TB_ERR_CAPACITY = -5, -6, -7, -8, -9
F32, F16, BF16 = 0, 1, 2
IMP = {"obd": 0, "obs": 1, "normalized": 2}
STRATEGY = {"topn": 0, "optimal": 1, "iterative": 2}
REDIST = {"none": 0, "proportional": 1, "uniform": 2}


class TbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"tb status {code}: {msg}")
        self.code = code


class PruneArgs(C.Structure):
    _fields_ = [
        ("struct_size", C.c_uint32),
        ("weights", C.c_void_p),
        ("w_dtype", C.c_int32),
        ("g_dtype", C.c_int32),
        ("grads", C.c_void_p),
        ("S", C.c_uint64),
        ("N", C.c_uint64),
        ("g_stride", C.c_uint64),
        ("fisher_in", C.c_void_p),
        ("fisher_steps_in", C.c_uint64),
        ("alpha", C.c_float),
        ("beta", C.c_float),
        ("damping", C.c_float),
        ("importance_mode", C.c_int32),
        ("use_fisher", C.c_int32),
        ("nm_n", C.c_int32),
        ("nm_m", C.c_int32),
        ("mask_strategy", C.c_int32),
        ("iterative_rounds", C.c_int32),
        ("redist_mode", C.c_int32),
        ("permute", C.c_int32),
        ("w_out", C.c_void_p),
        ("mask_out", C.c_void_p),
        ("fisher_out", C.c_void_p),
        ("scores_out", C.c_void_p),
        ("near_ties", C.c_void_p),
    ]


def header_symbols() -> list[str]:
    """Names of every function declared in include/tb_kernels.h."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return re.findall(r"\b(tb_[a-z0-9_]+)\s*\(", txt)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is not built; run `python tensorbit-core_b200/build.py` (needs nvcc)")
        L = C.CDLL(LIB_PATH)
        vp, sz, i32, f32 = C.c_void_p, C.c_size_t, C.c_int, C.c_float
        sig = {
            "tb_abi_version": ([], i32),
            "tb_last_error": ([], C.c_char_p),
            "tb_device_count": ([C.POINTER(C.c_int)], i32),
            "tb_set_device": ([i32], i32),
            "tb_malloc": ([C.POINTER(vp), sz], i32),
            "tb_free": ([vp], i32),
            "tb_host_alloc": ([C.POINTER(vp), sz], i32),
            "tb_host_free": ([vp], i32),
            "tb_memcpy_h2d": ([vp, vp, sz, vp], i32),
            "tb_memcpy_d2h": ([vp, vp, sz, vp], i32),
            "tb_memcpy_d2d": ([vp, vp, sz, vp], i32),
            "tb_memset": ([vp, i32, sz, vp], i32),
            "tb_stream_sync": ([vp], i32),
            "tb_prepare_nm": ([i32, i32], i32),
            "tb_ipc_handle": ([vp, vp], i32),
            "tb_ipc_open": ([vp, C.POINTER(vp)], i32),
            "tb_ipc_close": ([vp], i32),
            "tb_enable_peer_access": ([i32], i32),
            "tb_fisher_diagonal": ([vp, vp, sz, sz, vp], i32),
            "tb_fisher_accumulate": ([vp, vp, sz, f32, vp], i32),
            "tb_fisher_beta_decay": ([vp, f32, sz, vp], i32),
            "tb_ehap_importance": ([vp, vp, vp, sz, f32, vp], i32),
            "tb_nm_mask_2_4": ([vp, vp, sz, vp], i32),
            "tb_nm_mask_generic": ([vp, vp, sz, i32, i32, vp], i32),
            "tb_apply_mask": ([vp, vp, sz, i32, vp], i32),
            "tb_decode_to_f32": ([vp, i32, vp, sz, vp], i32),
            "tb_fisher_weighted_sum": ([vp, vp, i32, sz, sz, sz, vp, i32, vp], i32),
            "tb_fisher_ema_step": ([vp, vp, i32, sz, f32, f32, i32, vp], i32),
            "tb_importance": ([vp, i32, vp, vp, sz, f32, i32, vp], i32),
            "tb_nm_mask": ([vp, vp, sz, i32, i32, i32, i32, i32, vp], i32),
            "tb_redistribute": ([vp, vp, vp, sz, i32, i32, vp], i32),
            "tb_threshold_select": ([vp, sz, f32, vp, C.POINTER(C.c_float), C.POINTER(C.c_uint64), vp], i32),
            "tb_ehap_apply_mask": ([vp, vp, sz, C.POINTER(C.c_uint64), vp], i32),
            "tb_fisher_normalize": ([vp, sz, vp], i32),
            "tb_compensate": ([vp, vp, vp, sz, i32, vp], i32),
            "tb_block_obs": ([vp, vp, C.POINTER(vp), i32, sz, sz, f32, f32, f32, C.POINTER(C.c_uint64), vp], i32),
            "tb_block_obs_phase_times": ([C.POINTER(C.c_float), i32], i32),
            "tb_split_tf32": ([vp, vp, vp, sz, vp], i32),
            "tb_gemm_nt_tf32x3": ([vp, vp, C.c_longlong, vp, vp, C.c_longlong, i32, i32, i32, f32, f32, vp,
                                   C.c_longlong, vp, C.c_longlong, i32, vp], i32),
            "tb_gemm_nt_bf16": ([vp, C.c_longlong, vp, C.c_longlong, i32, i32, i32, f32, f32, vp, C.c_longlong,
                                 vp, C.c_longlong, i32, vp], i32),
            "tb_gemm_status": ([vp], i32),
            "tb_obs_hessian": ([vp, i32, i32, vp, vp], i32),
            "tb_obs_hessian_scaled": ([vp, i32, i32, f32, vp, vp], i32),
            "tb_obs_sparsegpt": ([vp, i32, i32, vp, f32, i32, i32, vp, vp, vp], i32),
            "tb_obs_sparsegpt_phase_times": ([C.POINTER(C.c_float), i32], i32),
            "tb_score_mask_pack": ([C.POINTER(PruneArgs), vp], i32),
            "tb_fisher_partial_scatter": ([vp, i32, sz, sz, sz, vp, i32, C.POINTER(C.c_uint64), C.POINTER(vp), i32,
                                           vp], i32),
            "tb_prune_one_shot_nm": ([C.POINTER(PruneArgs), f32, C.POINTER(C.c_float), C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_uint64), vp], i32),
            "tb_prune_one_shot_nm_async": ([C.POINTER(PruneArgs), f32, vp, vp, C.POINTER(C.c_uint64), vp], i32),
            "tb_score_mask_pack_peer": ([C.POINTER(PruneArgs), C.POINTER(vp), i32, vp], i32),
            "tb_score_mask_pack_host": ([C.POINTER(PruneArgs)], i32),
            "tb_score_mask_pack_host_noalloc": ([C.POINTER(PruneArgs)], i32),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc: int) -> int:
    if rc != TB_OK:
        raise TbError(rc, lib().tb_last_error().decode())
    return rc


def call(name: str, *args) -> int:
    """Calls an entry point and returns its raw status."""
    return getattr(lib(), name)(*args)


def prune_args(*, weights, w_dtype, grads, g_dtype, S, N, w_out, mask_out, g_stride=0,
               fisher_in=None, fisher_steps_in=0, alpha=0.01, beta=0.99, damping=0.01,
               mode="obd", use_fisher=True, n=2, m=4, strategy="optimal", rounds=3,
               redist="proportional", permute=False, fisher_out=None, scores_out=None,
               near_ties=None) -> PruneArgs:
    a = PruneArgs()
    a.struct_size = C.sizeof(PruneArgs)
    a.weights, a.w_dtype, a.grads, a.g_dtype = weights, w_dtype, grads, g_dtype
    a.S, a.N, a.g_stride = S, N, g_stride
    a.fisher_in, a.fisher_steps_in = fisher_in, fisher_steps_in
    a.alpha, a.beta, a.damping = alpha, beta, damping
    a.importance_mode = IMP[mode] if isinstance(mode, str) else mode
    a.use_fisher = int(use_fisher)
    a.nm_n, a.nm_m = n, m
    a.mask_strategy = STRATEGY[strategy] if isinstance(strategy, str) else strategy
    a.iterative_rounds = rounds
    a.redist_mode = REDIST[redist] if isinstance(redist, str) else redist
    a.permute = int(permute)
    a.w_out, a.mask_out, a.fisher_out, a.scores_out, a.near_ties = (
        w_out, mask_out, fisher_out, scores_out, near_ties)
    return a


def score_mask_pack(args: PruneArgs, stream=None) -> int:
    return lib().tb_score_mask_pack(C.byref(args), stream)


def score_mask_pack_host(args: PruneArgs) -> int:
    return lib().tb_score_mask_pack_host(C.byref(args))

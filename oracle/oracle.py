"""numpy front end for the two CPU oracles of the pruning path.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` to check or time against; the shipped
library never imports it.

* ``Oracle("port")`` - the CPU restatement in ``oracle/tb_oracle.cpp``
  (built by ``make -C oracle port``; needs only g++, so it can be rebuilt on any
  box of this image).
* ``Oracle("ref")``  - the reference's own CPU code compiled from its sources
  (``make -C oracle ref``; needs the reference tree, so it exists only where the
  reference was present at build time).

Both expose the same methods with the same status codes, so a test can run a
case through both and compare byte for byte.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "libtb_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtb_ref.so")
REF_CLI = os.path.join(HERE, "_ref", "tb-prune")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_sz = C.c_size_t
_szp = C.POINTER(C.c_size_t)

IMP = {"obd": 0, "obs": 1, "normalized": 2}
STRATEGY = {"topn": 0, "optimal": 1, "iterative": 2}
REDIST = {"none": 0, "proportional": 1, "uniform": 2}
EHAP_STRATEGY = {None: -1, "oneshot": 0, "iterative": 1, "blockobs": 2}


def build_port() -> str:
    if not os.path.exists(PORT_SO):
        subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    return PORT_SO


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def _null_f32():
    return None


class Oracle:
    def __init__(self, kind: str = "port"):
        self.kind = kind
        path = build_port() if kind == "port" else REF_SO
        if not os.path.exists(path):
            raise FileNotFoundError(f"oracle library missing: {path}")
        self.lib = C.CDLL(path)
        p = "port_" if kind == "port" else "ref_"
        self._p = p
        L = self.lib
        fp = C.POINTER(C.c_float)
        self._fisher = getattr(L, p + "fisher")
        self._fisher.argtypes = [_f32p, _sz, _sz, C.c_float, C.c_float, C.c_int, _f32p]
        self._imp = getattr(L, p + "importance")
        self._imp.argtypes = [_f32p, _sz, _f32p, _sz, C.c_float, C.c_float, C.c_float, C.c_int,
                              C.c_int, C.c_int, _f32p]
        self._mask = getattr(L, p + "nm_mask")
        self._mask.argtypes = [_f32p, _sz, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _u8p]
        self._mask_status = getattr(L, p + "nm_mask_status")
        self._mask_status.argtypes = [_sz, _sz, C.c_int, C.c_int]
        self._cprune = getattr(L, p + "coring_prune")
        self._cprune.argtypes = [_f32p, _f32p, _sz, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                 C.c_int, C.c_int, _u8p, _szp]
        self._apply = getattr(L, p + "apply_redistribute")
        self._apply.argtypes = [_f32p, _u8p, _f32p, _sz, C.c_int, C.c_int, C.c_int, C.c_int, _szp]
        self._select = getattr(L, p + "select_mask")
        self._select.argtypes = [_f32p, _sz, C.c_float, _u8p, _szp]
        self._pipe = getattr(L, p + "pipeline")
        self._pipe.argtypes = [_f32p, C.c_void_p, _sz, _sz, C.c_float, C.c_float, C.c_float, C.c_int,
                               C.c_int, C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p, _sz,
                               C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                               C.c_void_p, _u8p, _szp, _szp]
        self._comp = getattr(L, p + "compensate")
        self._comp.argtypes = [_f32p, _u8p, _f32p, _sz, C.c_int]
        self._bobs = getattr(L, p + "block_obs")
        self._bobs.argtypes = [_f32p, C.c_void_p, _sz, C.c_void_p, _sz, _sz, _sz, C.c_float, C.c_float,
                               C.c_float, C.c_float, C.c_int, _sz, _szp]
        self._mock = getattr(L, p + "mock_tensor")
        self._mock.argtypes = [_sz, _f32p, _f32p]
        if kind == "port":
            self._hdr = L.port_tb_header
            self._hdr.argtypes = [_u8p, C.c_uint32, C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint32]
            self._dec = L.port_decode_half
            self._dec.argtypes = [_u16p, _sz, C.c_int, _f32p]
            self._ties = L.port_near_ties
            self._ties.argtypes = [_f32p, _sz, C.c_int, C.c_int]
            self._ties.restype = _sz
            self._topn1 = L.port_topn_group
            self._topn1.argtypes = [_f32p, C.c_int, C.c_int, _u8p]
        else:
            self._wtb = L.ref_write_tb
            self._wtb.argtypes = [C.c_char_p, _f32p, _sz, _u8p, _sz, C.c_uint32, C.c_uint32]
            self._dec = L.ref_decode_half
            self._dec.argtypes = [_u16p, _sz, C.c_int, C.c_char_p, _f32p]
            self._par = L.ref_parallel_pass
            self._par.argtypes = [_f32p, _f32p, _sz, _sz, C.c_float, C.c_float, C.c_float, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _u8p, C.c_int]

    # -- stage 1 ------------------------------------------------------------
    def fisher(self, grads, alpha=0.01, beta=0.99, use_fisher=True):
        g = np.ascontiguousarray(grads, np.float32)
        S, N = g.shape
        F = np.zeros(N, np.float32)
        rc = self._fisher(g.reshape(-1) if S else np.zeros(1, np.float32), S, N, alpha, beta,
                          int(use_fisher), F)
        return rc, F

    def importance(self, grads, w, alpha=0.01, beta=0.99, damping=0.01, mode="obd",
                   use_fisher=True, normalize=False):
        g = np.ascontiguousarray(grads, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        S = g.shape[0]
        N = w.size
        s = np.zeros(max(N, 1), np.float32)
        rc = self._imp(g.reshape(-1) if g.size else np.zeros(1, np.float32), S,
                       w if N else np.zeros(1, np.float32), N, alpha, beta, damping, IMP[mode],
                       int(use_fisher), int(normalize), s)
        return rc, s[:N]

    # -- stage 2 ------------------------------------------------------------
    def nm_mask(self, s, n=2, m=4, strategy="topn", rounds=3, permute=False, hw_layout=False):
        s = np.ascontiguousarray(s, np.float32)
        out = np.zeros(max(s.size, 1), np.uint8)
        rc = self._mask(s if s.size else np.zeros(1, np.float32), s.size, n, m, STRATEGY[strategy],
                        rounds, int(permute), int(hw_layout), out)
        return rc, out[: s.size // m] if rc == 0 else out[:0]

    def nm_mask_status(self, n_scores, n_mask, n=2, m=4):
        return self._mask_status(n_scores, n_mask, n, m)

    def coring_prune(self, s, w, n=2, m=4, strategy="topn", rounds=3, redist="none",
                     permute=False, hw_layout=False):
        s = np.ascontiguousarray(s, np.float32)
        w = np.array(w, np.float32, copy=True)
        mask = np.zeros(max(s.size // m, 1), np.uint8)
        pr = C.c_size_t(0)
        rc = self._cprune(s, w, s.size, n, m, STRATEGY[strategy], rounds, REDIST[redist],
                          int(permute), int(hw_layout), mask, C.byref(pr))
        return rc, w, mask[: s.size // m], pr.value

    def apply_redistribute(self, w, mask, s, n=2, m=4, redist="proportional", do_apply=True):
        w = np.array(w, np.float32, copy=True)
        mask = np.ascontiguousarray(mask, np.uint8)
        s = np.ascontiguousarray(s, np.float32)
        pr = C.c_size_t(0)
        rc = self._apply(w, mask, s, w.size, n, m, REDIST[redist], int(do_apply), C.byref(pr))
        return rc, w, pr.value

    def select_mask(self, s, sparsity=0.5):
        s = np.ascontiguousarray(s, np.float32)
        out = np.zeros(max(s.size, 1), np.uint8)
        pr = C.c_size_t(0)
        rc = self._select(s if s.size else np.zeros(1, np.float32), s.size, sparsity, out,
                          C.byref(pr))
        return rc, out[: s.size], pr.value

    def pipeline(self, w, grads, alpha=0.01, beta=0.99, damping=0.01, mode="obd",
                 use_fisher=True, normalize=False, ehap_strategy=None, sparsity=0.5,
                 prune_rounds=5, hist=None, n=2, m=4, strategy="topn", rounds=3,
                 redist="proportional", permute=False):
        """tb-prune's per-tensor sequence; returns (rc, w', mask, F, s, ehap_pruned, coring_pruned)."""
        w = np.array(w, np.float32, copy=True).reshape(-1)
        g = np.ascontiguousarray(grads, np.float32)
        S = g.shape[0] if g.ndim == 2 else 0
        N = w.size
        F = np.zeros(N, np.float32)
        s = np.zeros(N, np.float32)
        mask = np.zeros(max(N // m, 1), np.uint8)
        hp = None
        K = 0
        if hist is not None:
            hist = np.ascontiguousarray(hist, np.float32)
            K = hist.shape[0]
            hp = hist.ctypes.data
        ep, cp = C.c_size_t(0), C.c_size_t(0)
        rc = self._pipe(w, g.ctypes.data if S else None, S, N, alpha, beta, damping, IMP[mode],
                        int(use_fisher), int(normalize), EHAP_STRATEGY[ehap_strategy], sparsity,
                        prune_rounds, hp, K, n, m, STRATEGY[strategy], rounds, REDIST[redist],
                        int(permute), F.ctypes.data, s.ctypes.data, mask, C.byref(ep), C.byref(cp))
        return rc, w, mask[: N // m], F, s, ep.value, cp.value

    # -- formats ------------------------------------------------------------
    def tb_bytes(self, w, mask, n, m):
        """The complete .tb image TBWriter::write produces for FP32 weights."""
        w = np.ascontiguousarray(w, np.float32)
        mask = np.ascontiguousarray(mask, np.uint8)
        if self.kind == "port":
            hdr = np.zeros(4096, np.uint8)
            self._hdr(hdr, n, m, w.size, mask.size, 4)
            return hdr.tobytes() + w.tobytes() + mask.tobytes()
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "x.tb")
            rc = self._wtb(path.encode(), w, w.size, mask if mask.size else np.zeros(1, np.uint8),
                           mask.size, n, m)
            assert rc == 0, rc
            with open(path, "rb") as f:
                return f.read()

    def decode_half(self, bits, is_bf16):
        bits = np.ascontiguousarray(bits, np.uint16)
        out = np.zeros(bits.size, np.float32)
        if self.kind == "port":
            self._dec(bits, bits.size, int(is_bf16), out)
        else:
            with tempfile.TemporaryDirectory() as d:
                rc = self._dec(bits, bits.size, int(is_bf16),
                               os.path.join(d, "x.safetensors").encode(), out)
                assert rc == 0, rc
        return out

    def compensate(self, w, mask, s, mode):
        """EHAPPruner::compensate_weights on a 1-byte-per-element mask; returns new weights."""
        w = np.array(w, np.float32, copy=True)
        rc = self._comp(w, np.ascontiguousarray(mask, np.uint8), np.ascontiguousarray(s, np.float32),
                        w.size, mode)
        if self.kind == "ref":
            assert rc == 0, rc
        return w

    def block_obs(self, w, grads, hist=None, block=128, sparsity=0.5, damping=0.01, off_alpha=0.01,
                  fisher_alpha=0.01, use_fisher=True, hist_size=4):
        """accumulate_fisher x S, store_gradient x K, prune_block_obs; returns (rc, w', pruned)."""
        w = np.array(w, np.float32, copy=True).reshape(-1)
        g = np.ascontiguousarray(grads, np.float32)
        S = g.shape[0] if g.ndim == 2 else 0
        K = 0
        hp = None
        if hist is not None:
            hist = np.ascontiguousarray(hist, np.float32)
            K, hp = hist.shape[0], hist.ctypes.data
        pr = C.c_size_t(0)
        rc = self._bobs(w, g.ctypes.data if S else None, S, hp, K, w.size, block, sparsity, damping,
                        off_alpha, fisher_alpha, int(use_fisher), hist_size, C.byref(pr))
        return rc, w, pr.value

    def mock_tensor(self, N):
        w = np.zeros(N, np.float32)
        g = np.zeros(N, np.float32)
        self._mock(N, w, g)
        return w, g

    def near_ties(self, s, n, m):
        s = np.ascontiguousarray(s, np.float32)
        return int(self._ties(s, s.size, n, m))

    def topn_group(self, vals, n, m):
        v = np.ascontiguousarray(vals, np.float32)
        out = np.zeros(1, np.uint8)
        self._topn1(v, n, m, out)
        return int(out[0])

    def parallel_pass(self, w, grads, alpha=0.01, beta=0.99, damping=0.01, mode="obd", n=2, m=4,
                      strategy="optimal", rounds=3, redist="proportional", threads=1):
        """Reference score+mask+pack over `threads` disjoint shards (CPU baseline)."""
        S, N = grads.shape
        mask = np.zeros(N // m, np.uint8)
        rc = self._par(w, grads.reshape(-1), S, N, alpha, beta, damping, IMP[mode], n, m,
                       STRATEGY[strategy], rounds, REDIST[redist], mask, threads)
        return rc, mask

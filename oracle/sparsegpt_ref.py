"""Float64 restatement of column-block exact OBS on an activation Hessian.

TEST INFRASTRUCTURE ONLY (imported by tests/ to check tb_obs_sparsegpt).

PARITY UNPINNED: the reference has no implementation of this algorithm
(docs/EHAP.md:248-250; its kBlockOBS, ehap.hpp:502-704, is a different
algorithm).  This follows the published column-block formulation (Frantar &
Alistarh 2023, "SparseGPT") with the reference's OBS saliency w^2/[H^-1]_qq
(ehap.hpp:683) and update (ehap.hpp:687-691) taken along the upper Cholesky
factor U of H^-1, in float64:

  H = X^T X / n;  H += frac * mean(diag H) * I;  U = chol_upper(H^-1)
  for each block of B columns: for each group of M columns, prune the M-N
  smallest w^2 / U_qq^2 (lowest index first on ties); for each column q,
  err = (w_q - kept_q) / U_qq, w_j -= err U_qj for j >= q in the block; then
  W[:, later] -= E U[block, later].
"""
import numpy as np


def chol_upper_of_inverse(H):
    return np.linalg.cholesky(np.linalg.inv(H)).T


def sparsegpt(W, X, damp_frac=0.01, n_keep=2, m=4, block=128):
    """Returns (pruned weights, mask bytes [r, d/m] with bit k = keep column
    g*m+k, U, per-group saliency gap of the last decision)."""
    X = np.asarray(X, np.float64)
    n = X.shape[0]
    H = X.T @ X / n
    H[np.diag_indices_from(H)] += damp_frac * np.mean(np.diag(H))
    U = chol_upper_of_inverse(H)
    W = np.array(W, np.float64, copy=True)
    r, d = W.shape
    mask = np.zeros((r, d // m), np.uint8)
    gap = np.zeros((r, d // m), np.float64)
    rows = np.arange(r)[:, None]
    prune_cnt = m - n_keep
    for i1 in range(0, d, block):
        i2 = min(i1 + block, d)
        W1 = W[:, i1:i2].copy()
        Q1 = np.zeros_like(W1)
        E1 = np.zeros_like(W1)
        U1 = U[i1:i2, i1:i2]
        keep = None
        for i in range(i2 - i1):
            if i % m == 0:
                sal = W1[:, i:i + m] ** 2 / np.diag(U1)[i:i + m] ** 2
                order = np.argsort(sal, axis=1, kind="stable")
                keep = np.ones((r, m), bool)
                keep[rows, order[:, :prune_cnt]] = False
                g = (i1 + i) // m
                mask[:, g] = (keep * (1 << np.arange(m))).sum(1).astype(np.uint8)
                s = np.sort(sal, axis=1)
                gap[:, g] = (s[:, prune_cnt] - s[:, prune_cnt - 1]) / np.maximum(s[:, prune_cnt], 1e-300)
            w = W1[:, i]
            q = np.where(keep[:, i % m], w, 0.0)
            Q1[:, i] = q
            err = (w - q) / U1[i, i]
            W1[:, i:] -= np.outer(err, U1[i, i:])
            E1[:, i] = err
        W[:, i1:i2] = Q1
        W[:, i2:] -= E1 @ U[i1:i2, i2:]
    return W, mask, U, gap


def layer_loss(W0, W1, X):
    """||(W0 - W1) X^T||_F^2 / ||W0 X^T||_F^2 in float64."""
    X = np.asarray(X, np.float64)
    D = (np.asarray(W0, np.float64) - np.asarray(W1, np.float64)) @ X.T
    B = np.asarray(W0, np.float64) @ X.T
    return float((D ** 2).sum() / (B ** 2).sum())


def sparsegpt_rows_torch(torch, W, U, n_keep=2, m=4, block=128):
    """The same float64 sweep for a few rows with torch tensors (any device):
    W [r, d] float64 rows of the layer, U [d, d] float64 upper Cholesky factor
    of the damped H^-1.  Rows are independent given U, so checking a subset of
    a large layer's rows needs only U.  Returns (pruned rows, mask bytes
    [r, d/m], per-group saliency gap)."""
    W = W.clone()
    r, d = W.shape
    dev = W.device
    mask = torch.zeros(r, d // m, dtype=torch.uint8, device=dev)
    gap = torch.zeros(r, d // m, dtype=torch.float64, device=dev)
    bitw = 1 << torch.arange(m, device=dev)
    prune_cnt = m - n_keep
    for i1 in range(0, d, block):
        i2 = min(i1 + block, d)
        W1 = W[:, i1:i2].clone()
        Q1 = torch.zeros_like(W1)
        E1 = torch.zeros_like(W1)
        U1 = U[i1:i2, i1:i2]
        du = torch.diagonal(U1)
        keep = None
        for i in range(i2 - i1):
            if i % m == 0:
                sal = W1[:, i:i + m] ** 2 / du[i:i + m] ** 2
                order = torch.argsort(sal, dim=1, stable=True)
                keep = torch.ones(r, m, dtype=torch.bool, device=dev)
                keep.scatter_(1, order[:, :prune_cnt], False)
                g = (i1 + i) // m
                mask[:, g] = (keep.long() * bitw).sum(1).to(torch.uint8)
                s = torch.sort(sal, dim=1).values
                gap[:, g] = (s[:, prune_cnt] - s[:, prune_cnt - 1]) / torch.clamp(s[:, prune_cnt], min=1e-300)
            w = W1[:, i]
            q = torch.where(keep[:, i % m], w, torch.zeros_like(w))
            Q1[:, i] = q
            err = (w - q) / U1[i, i]
            W1[:, i:] -= torch.outer(err, U1[i, i:])
            E1[:, i] = err
        W[:, i1:i2] = Q1
        W[:, i2:] -= E1 @ U[i1:i2, i2:]
    return W, mask, gap

"""CPU restatement of the chunked (WY / UT) evaluation of the gated-DeltaNet
recurrence that the GPU scan runs (clef-rs_b200/csrc/delta_scan.cu).

TEST INFRASTRUCTURE ONLY: imported by tests/ as a checker of the chunk algebra;
nothing on the product path imports it.

The reference states the per-token recurrence (delta_recurrence_prefill,
crates/core/src/models/qwen.rs:826-882)

    S <- S e^{g_t};  d_t = (v_t - S^T k_t) beta_t;  S <- S + k_t d_t^T;  o_t = S^T q_t

and evaluates it a chunk at a time in its chunkwise candidate
(crates/core/src/chunk.rs:16-149, chunk.metal:10-164). Per chunk of C tokens
with chunk-relative cumulative log-decays G_i = sum_{s <= i} g_s:

    A_ij = beta_i e^{G_i - G_j} k_i . k_j   (j < i),      T = (I + A)^{-1}
    P_ij = e^{G_i - G_j} q_i . k_j          (j <= i)
    R    = V - diag(e^G) K S                 residual of the chunk's old state
    D    = T diag(beta) R                    the chunk's delta rows
    O    = diag(e^G) Q S + P D
    S   <- e^{G_last} S + K^T diag(e^{G_last - G}) D

and a state captured after row c of a chunk is
    S_c  = e^{G_c} S + K^T diag(e^{G_c - G_j} [j <= c]) D.
Every decay factor is the exponential of a non-positive difference, so a
decay of -1000 per token stays exact. Evaluated in float64 here; the kernels
use split-BF16 tensor-core products with F32 accumulation.
"""
from __future__ import annotations

import numpy as np


def _l2(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float64)
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + 1e-6)


def chunked_scan(q, k, v, g, beta, state=None, capture=0, chunk=64):
    """q, k [T, Hk, dk] (normalised inside, q scaled by 1/sqrt(dk), as the
    reference recurrence does), v [T, Hv, dv], g, beta [T, Hv]; state
    [Hv, dk, dv] or None. Returns (o [T, Hv, dv], final state, captured state
    after token `capture` or None), all float64."""
    t, hk, kd = q.shape
    hv, vd = v.shape[1], v.shape[2]
    rep = hv // hk
    qn = _l2(q) / np.sqrt(kd)
    kn = _l2(k)
    S = np.zeros((hv, kd, vd)) if state is None else np.array(state, np.float64)
    out = np.zeros((t, hv, vd))
    cap = None
    for t0 in range(0, t, chunk):
        n = min(chunk, t - t0)
        for h in range(hv):
            K = kn[t0:t0 + n, h // rep]
            Q = qn[t0:t0 + n, h // rep]
            V = v[t0:t0 + n, h].astype(np.float64)
            b = beta[t0:t0 + n, h].astype(np.float64)
            G = np.cumsum(g[t0:t0 + n, h].astype(np.float64))
            dec = np.exp(np.minimum(G[:, None] - G[None, :], 0.0))  # e^{G_i - G_j}, used for j <= i
            low = np.tril(np.ones((n, n)), -1)
            A = b[:, None] * dec * (K @ K.T) * low
            T = np.linalg.inv(np.eye(n) + A)
            P = dec * (Q @ K.T) * np.tril(np.ones((n, n)))
            eg = np.exp(G)
            R = V - eg[:, None] * (K @ S[h])
            D = (T * b[None, :]) @ R
            out[t0:t0 + n, h] = eg[:, None] * (Q @ S[h]) + P @ D
            if capture and t0 < capture <= t0 + n:
                c = capture - 1 - t0
                w = np.where(np.arange(n) <= c, np.exp(np.minimum(G[c] - G, 0.0)), 0.0)
                if cap is None:
                    cap = np.zeros((hv, kd, vd))
                cap[h] = np.exp(G[c]) * S[h] + K.T @ (w[:, None] * D)
            S[h] = np.exp(G[-1]) * S[h] + K.T @ (np.exp(G[-1] - G)[:, None] * D)
    return out, S, cap

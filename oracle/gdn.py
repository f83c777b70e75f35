"""TEST INFRASTRUCTURE -- numpy f64 restatement of the reference's GatedDeltaNet rows:
gdn_kkt_solve (reference src/adjoint/host/gdn_kkt.cpp) and gdn_chunk_scan
(reference src/adjoint/host/gdn_scan.cpp), twins and host adjoints, per (sequence, head, chunk), with
the reference's own stage structure vectorised per chunk. Pinned against the reference's compiled rows
in tests/test_oracle_pin_gdn.py. Only tests and the bench's CPU baseline use it.

Shapes follow the reference: q, k [T, Hg, K]; v [T, H, V]; g, beta [T, H] (g the within-chunk
cumulative log decay); A [T, H, chunk]; h0 / ht [n_seq, H, V, K]; cu [n_seq + 1].
"""
from __future__ import annotations

import numpy as np


def _decay(gc, k=0):
    """e^{g_i - g_j} on the lower triangle (j <= i + k), zero above it, without forming the overflowing
    upper entries."""
    L = len(gc)
    low = np.tri(L, k=k, dtype=bool)
    return np.where(low, np.exp(np.where(low, gc[:, None] - gc[None, :], 0.0)), 0.0)


def _chunks(cu, chunk):
    for s in range(len(cu) - 1):
        bos, slen = int(cu[s]), int(cu[s + 1]) - int(cu[s])
        yield s, bos, slen, [(c0, min(chunk, slen - c0)) for c0 in range(0, slen, chunk)]


def kkt_fwd(k, beta, g, cu, chunk=64):
    """A = (I + M)^-1 per chunk, M[i,l] = beta_i (k_i . k_l) e^{g_i - g_l} for l < i
    (reference src/adjoint/host/gdn_kkt.cpp:221-270)."""
    T, Hg, K = k.shape
    H = beta.shape[1]
    grp = H // Hg
    A = np.zeros((T, H, chunk))
    for s, bos, slen, cs in _chunks(cu, chunk):
        for h in range(H):
            for c0, L in cs:
                rows = slice(bos + c0, bos + c0 + L)
                kc, bc, gc = k[rows, h // grp], beta[rows, h], g[rows, h]
                M = bc[:, None] * (kc @ kc.T) * _decay(gc, -1)
                Ainv = np.linalg.solve(np.eye(L) + M, np.eye(L))
                A[rows, h, :L] = np.tril(Ainv)
    return A


def kkt_bwd(k, beta, g, cu, A, dA, chunk=64):
    """dk, dbeta, dg of kkt_fwd for the cotangent dA (reference src/adjoint/host/gdn_kkt.cpp:272-352):
    Et = -(A^T Ac A^T) on the strict lower block, then the three chain terms."""
    T, Hg, K = k.shape
    H = beta.shape[1]
    grp = H // Hg
    dk, dbeta, dg = np.zeros_like(k), np.zeros_like(beta), np.zeros_like(g)
    for s, bos, slen, cs in _chunks(cu, chunk):
        for h in range(H):
            hk = h // grp
            for c0, L in cs:
                rows = slice(bos + c0, bos + c0 + L)
                kc, bc, gc = k[rows, hk], beta[rows, h], g[rows, h]
                Al = np.tril(A[rows, h, :L])
                Ac = np.tril(dA[rows, h, :L])
                Y = np.tril(Ac @ Al.T)
                Et = np.tril(-(Al.T @ Y), -1)
                # e^{g_i - g_l} on the strict lower block only (the reference forms it only there; above the
                # diagonal it can overflow)
                phi = _decay(gc, -1)
                C = (kc @ kc.T) * phi
                Mm = bc[:, None] * C
                dbeta[rows, h] += (Et * C).sum(1)
                G = Et * Mm
                dg[rows, h] += G.sum(1) - G.sum(0)
                E = Et * bc[:, None] * phi
                dk[rows, hk] += E @ kc + E.T @ kc
    return dk, dbeta, dg


def _state_in(h0, s, h):
    return np.zeros((0, 0)) if h0 is None else h0[s, h].T.copy()  # [V,K] -> S[d][e]


def scan_fwd(q, k, v, A, g, beta, cu, h0=None, scale=None, chunk=64):
    """o and the final state (reference src/adjoint/host/gdn_scan.cpp:219-284 chunk_forward, 418-485 twin)."""
    T, Hg, K = q.shape
    H, V = v.shape[1], v.shape[2]
    grp = H // Hg
    scale = 1.0 / np.sqrt(K) if scale is None else scale
    o = np.zeros((T, H, V))
    n_seq = len(cu) - 1
    ht = np.zeros((n_seq, H, V, K))
    for s, bos, slen, cs in _chunks(cu, chunk):
        for h in range(H):
            S = np.zeros((K, V)) if h0 is None else h0[s, h].T.copy()
            for c0, L in cs:
                rows = slice(bos + c0, bos + c0 + L)
                qc, kc, vc = q[rows, h // grp], k[rows, h // grp], v[rows, h]
                Ac, gc, bc = np.tril(A[rows, h, :L]), g[rows, h], beta[rows, h]
                ge = np.exp(gc)
                W = bc[:, None] * (vc - ge[:, None] * (kc @ S))
                Vp = Ac @ W
                P = (qc @ kc.T) * _decay(gc)
                o[rows, h] = scale * (ge[:, None] * (qc @ S) + P @ Vp)
                gl = gc[L - 1]
                S = np.exp(gl) * S + (kc * np.exp(gl - gc)[:, None]).T @ Vp
            ht[s, h] = S.T
    return o, ht


def scan_bwd(q, k, v, A, g, beta, cu, do, dht=None, h0=None, scale=None, chunk=64):
    """dq, dk, dv, dA, dg, dbeta of scan_fwd (reference src/adjoint/host/gdn_scan.cpp:286-416 chunk_backward
    stages 1-4, 487-580 adjoint): replay the states forward, then walk the chunks backward carrying the
    state cotangent; the first chunk's cotangent is h0's (returned as dh0)."""
    T, Hg, K = q.shape
    H, V = v.shape[1], v.shape[2]
    grp = H // Hg
    scale = 1.0 / np.sqrt(K) if scale is None else scale
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    dA, dg, db = np.zeros_like(A), np.zeros_like(g), np.zeros_like(beta)
    n_seq = len(cu) - 1
    dh0 = np.zeros((n_seq, H, V, K))
    for s, bos, slen, cs in _chunks(cu, chunk):
        for h in range(H):
            hk = h // grp
            S = np.zeros((K, V)) if h0 is None else h0[s, h].T.copy()
            states = []
            for c0, L in cs:
                states.append(S)
                rows = slice(bos + c0, bos + c0 + L)
                kc, vc = k[rows, hk], v[rows, h]
                Ac, gc, bc = np.tril(A[rows, h, :L]), g[rows, h], beta[rows, h]
                W = bc[:, None] * (vc - np.exp(gc)[:, None] * (kc @ S))
                Vp = Ac @ W
                gl = gc[L - 1]
                S = np.exp(gl) * S + (kc * np.exp(gl - gc)[:, None]).T @ Vp
            St1 = np.zeros((K, V)) if dht is None else dht[s, h].T.copy()
            for ci in range(len(cs) - 1, -1, -1):
                c0, L = cs[ci]
                S0 = states[ci]
                rows = slice(bos + c0, bos + c0 + L)
                qc, kc, vc = q[rows, hk], k[rows, hk], v[rows, h]
                Ac, gc, bc = np.tril(A[rows, h, :L]), g[rows, h], beta[rows, h]
                oc = do[rows, h]
                eg = np.exp(gc)
                W = bc[:, None] * (vc - eg[:, None] * (kc @ S0))
                Vp = Ac @ W
                gl = gc[L - 1]
                el = np.exp(gl)
                dqc, dkc = np.zeros((L, K)), np.zeros((L, K))
                dVp = np.zeros((L, V))
                dgc = np.zeros(L)
                dS0 = el * St1
                # stage 1: the state update
                dgc[L - 1] += (St1 * (el * S0)).sum()
                G = np.exp(gl - gc)
                Wk = (Vp @ St1.T) * G[:, None]
                dkc += Wk
                gw = (Wk * kc).sum(1)
                dgc -= gw
                dgc[L - 1] += gw.sum()
                dVp += G[:, None] * (kc @ St1)
                # stage 2: the output's state read and the intra-chunk path
                E = scale * eg
                S0oc = oc @ S0.T
                dqc += E[:, None] * S0oc
                dgc += E * (qc * S0oc).sum(1)
                dS0 += (qc * E[:, None]).T @ oc
                Phi = scale * _decay(gc)
                QK, VO = qc @ kc.T, oc @ Vp.T
                dqc += (Phi * VO) @ kc
                dkc += (Phi * VO).T @ qc
                dVp += (Phi * QK).T @ oc
                Gp = Phi * QK * VO
                dgc += Gp.sum(1) - Gp.sum(0)
                # stage 3: V' = A W
                dAc = np.tril(dVp @ W.T)
                dW = Ac.T @ dVp
                # stage 4: W = beta (v - e^g k S0)
                SK = kc @ S0
                db[rows, h] += (dW * (vc - eg[:, None] * SK)).sum(1)
                dv[rows, h] += bc[:, None] * dW
                be = bc * eg
                dgc -= be * (dW * SK).sum(1)
                dkc -= be[:, None] * (dW @ S0.T)
                dS0 -= (kc * be[:, None]).T @ dW
                dq[rows, hk] += dqc
                dk[rows, hk] += dkc
                dA[rows, h, :L] += dAc
                dg[rows, h] += dgc
                St1 = dS0
            dh0[s, h] = St1.T
    return dq, dk, dv, dA, dg, db, dh0


def layer_fwd_bwd(q, k, v, g, beta, cu, do, h0=None, dht=None, scale=None, chunk=64):
    """The composed pair: A = kkt(k, beta, g); o, ht = scan(...); total input cotangents with the kkt
    adjoint of the scan's dA added (what the B200 fused backward returns)."""
    A = kkt_fwd(k, beta, g, cu, chunk)
    o, ht = scan_fwd(q, k, v, A, g, beta, cu, h0, scale, chunk)
    dq, dk, dv, dA, dg, db, dh0 = scan_bwd(q, k, v, A, g, beta, cu, do, dht, h0, scale, chunk)
    dk2, db2, dg2 = kkt_bwd(k, beta, g, cu, A, dA, chunk)
    return dict(A=A, o=o, ht=ht, dq=dq, dk=dk + dk2, dv=dv, dg=dg + dg2, dbeta=db + db2, dh0=dh0, dA=dA)


def synth_inputs(T_list, H, Hg, K=128, V=128, seed=0, do_std=1e-2):
    """Config-2-like inputs over ragged sequences: q, k L2-normalised from N(0,1), v ~ N(0,1),
    beta = sigmoid(N(0,1)), the per-token log decay -softplus(N(0,1)) accumulated within chunks of 64,
    upstream grad ~ N(0, do_std)."""
    rs = np.random.RandomState(seed)
    T = int(sum(T_list))
    cu = np.concatenate([[0], np.cumsum(T_list)]).astype(np.int32)
    q = rs.normal(size=(T, Hg, K))
    k = rs.normal(size=(T, Hg, K))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rs.normal(size=(T, H, V))
    beta = 1.0 / (1.0 + np.exp(-rs.normal(size=(T, H))))
    inc = -np.log1p(np.exp(rs.normal(size=(T, H))))
    g = np.zeros((T, H))
    for s in range(len(T_list)):
        bos, slen = int(cu[s]), int(T_list[s])
        for c0 in range(0, slen, 64):
            r = slice(bos + c0, bos + min(slen, c0 + 64))
            g[r] = np.cumsum(inc[r], axis=0)
    do = rs.normal(size=(T, H, V)) * do_std
    return dict(q=q, k=k, v=v, g=g, beta=beta, cu=cu, do=do)

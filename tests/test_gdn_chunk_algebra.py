"""The chunk (WY) form the tensor-core GDN prefill kernels implement
(``csrc/gdn_chunk.cu``), checked in float64 against the token recurrence
S_t = g_t S_{t-1} + k_t d_t^T, d_t = beta_t (v_t - g_t S_{t-1}^T k_t), o_t = S_t^T q_t
over several chunks (a partial last chunk included) and a non-zero initial state."""
import numpy as np
import pytest


def token_recurrence(q, k, v, beta, lg, S0):
    S = S0.copy()
    out = []
    for t in range(len(q)):
        S = np.exp(lg[t]) * S
        d = beta[t] * (v[t] - S.T @ k[t])
        S = S + np.outer(k[t], d)
        out.append(S.T @ q[t])
    return np.array(out), S


def chunk_form(q, k, v, beta, lg, S0, C=64):
    S = S0.copy()
    out = []
    for c0 in range(0, len(q), C):
        n = min(C, len(q) - c0)
        D = q.shape[1]
        K = np.zeros((C, D)); Q = np.zeros((C, D)); V = np.zeros((C, v.shape[1]))
        K[:n], Q[:n], V[:n] = k[c0:c0 + n], q[c0:c0 + n], v[c0:c0 + n]
        B = np.zeros(C); L = np.zeros(C)
        B[:n], L[:n] = beta[c0:c0 + n], lg[c0:c0 + n]
        G = np.cumsum(L)                      # rows past n: log g = 0, beta = 0
        dec = np.exp(G[:, None] - G[None, :])
        tril = np.tril(np.ones((C, C)), -1)
        A = B[:, None] * dec * (K @ K.T) * tril
        P = dec * (Q @ K.T) * np.tril(np.ones((C, C)))
        T = np.linalg.inv(np.eye(C) + A)
        W = T @ (np.diag(B * np.exp(G)) @ K)
        U = T @ (np.diag(B) @ V)
        d = U - W @ S
        O = np.diag(np.exp(G)) @ Q @ S + P @ d
        S = np.exp(G[-1]) * S + K.T @ (np.exp(G[-1] - G)[:, None] * d)
        out.append(O[:n])
    return np.concatenate(out), S


@pytest.mark.parametrize("T", [1, 37, 64, 200])
def test_wy_chunk_form_matches_token_recurrence(T):
    rng = np.random.default_rng(T)
    D = 32
    k = rng.standard_normal((T, D)); k /= np.linalg.norm(k, axis=1, keepdims=True)
    q = rng.standard_normal((T, D)); q /= np.linalg.norm(q, axis=1, keepdims=True) * np.sqrt(D)
    v = rng.standard_normal((T, D))
    beta = 1 / (1 + np.exp(-rng.standard_normal(T)))
    lg = -np.log1p(np.exp(rng.standard_normal(T))) * rng.uniform(0.05, 2.0, T)  # log g < 0, some strong decays
    S0 = rng.standard_normal((D, D)) * 0.1
    o_ref, s_ref = token_recurrence(q, k, v, beta, lg, S0)
    o, s = chunk_form(q, k, v, beta, lg, S0)
    assert np.abs(o - o_ref).max() < 1e-9
    assert np.abs(s - s_ref).max() < 1e-9

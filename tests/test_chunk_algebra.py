"""The chunked forms of the gated delta rule, restated in numpy and held to the oracle's token-sequential recurrence
(crates/evie-core/src/model.rs:362-387, recur_body model.rs:501-541) on the CPU.

Per chunk of C <= 64 tokens entering with state S, with G_t = g_0 + ... + g_t, Gam_t = exp(G_t), E_t =
exp(G_C - G_t), N[t][s] = beta_t (k_t . k_s) exp(G_t - G_s) for s < t and P[t][s] = (q_t . k_s) exp(G_t - G_s)
for s <= t, T = (I + N)^-1 diag(beta):

  one pass (the form gdn_chunk_prefill_kernel computes):
      U = T (V - diag(Gam) K S),  O = diag(Gam) Q S + P U,  S' = Gam_C S + K^T diag(E) U
  three passes (per-chunk work that does not depend on S moved to a parallel pre-pass):
      W = T diag(Gam) K,  U0 = T V                      (pre-pass, any order over chunks)
      R = U0 - W S,  S' = Gam_C S + K^T diag(E) R       (the only sequential part; columns of S independent)
      O = diag(Gam) Q S + P R                           (given each chunk's entering S)

Each form runs twice: in float64, which pins the algebra, and with the tensor-core operand format of the device
kernels. In that format every f32 operand is split into bf16 planes hi + lo. A product with an exact bf16 operand
(q, k, v) takes two partial products; a product of two split operands takes three, with lo . lo dropped. Partial
products are accumulated in f32, and the three-pass form stores W and U0 as split planes between its passes."""
import numpy as np
import pytest

import oracle
from tests._inputs import bf16_bits, gdn_prefill_inputs


def _bf16(x):
    """f32 -> the nearest bf16 value (ties to even), as f32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def _split(x):
    x = np.asarray(x, np.float32)
    hi = _bf16(x)
    return hi, _bf16(x - hi)


def _mm(a, b, fmt):
    """a @ b, f32 result. fmt: 'f64' exact; 'es' a exact bf16 x b split; 'se' a split x b exact; 'ss' both split."""
    if fmt == "f64":
        return (np.asarray(a, np.float64) @ np.asarray(b, np.float64)).astype(np.float32)
    f = lambda m: np.asarray(m, np.float64)
    if fmt == "es":
        bh, bl = _split(b)
        return (f(a) @ f(bh)).astype(np.float32) + (f(a) @ f(bl)).astype(np.float32)
    if fmt == "se":
        ah, al = _split(a)
        return (f(ah) @ f(b)).astype(np.float32) + (f(al) @ f(b)).astype(np.float32)
    ah, al = _split(a)
    bh, bl = _split(b)
    return ((f(ah) @ f(bh)).astype(np.float32) + (f(ah) @ f(bl)).astype(np.float32)
            + (f(al) @ f(bh)).astype(np.float32))


def _chunk_consts(K, Q, g, beta):
    n = len(g)
    G = np.cumsum(g.astype(np.float64))
    diff = G[:, None] - G[None, :]
    t, s = np.meshgrid(np.arange(n), np.arange(n), indexing="ij")
    D = np.where(s <= t, np.exp(np.minimum(diff, 0.0)), 0.0)
    KK = K.astype(np.float64) @ K.astype(np.float64).T
    QK = Q.astype(np.float64) @ K.astype(np.float64).T
    N = np.where(s < t, beta.astype(np.float64)[:, None] * KK * D, 0.0)
    P = (QK * D).astype(np.float32)
    T = np.linalg.solve(np.eye(n) + N, np.diag(beta.astype(np.float64))).astype(np.float32)
    Gam = np.exp(G).astype(np.float32)
    E = np.exp(G[-1] - G).astype(np.float32)
    return T, P, Gam, E


def _one_pass(S, q, k, v, g, beta, split):
    S = S.astype(np.float32).copy()
    o = np.zeros((q.shape[0], v.shape[1]), np.float32)
    e, ss = ("es", "ss") if split else ("f64", "f64")
    for c0 in range(0, q.shape[0], 64):
        c = slice(c0, min(q.shape[0], c0 + 64))
        K, Q, V = k[c], q[c], v[c]
        T, P, Gam, E = _chunk_consts(K, Q, g[c], beta[c])
        KS, QS = _mm(K, S, e), _mm(Q, S, e)
        U = _mm(T, V - Gam[:, None] * KS, ss)
        o[c] = Gam[:, None] * QS + _mm(P, U, ss)
        S = Gam[-1] * S + _mm(K.T, E[:, None] * U, e)
    return S, o


def _three_pass(S, q, k, v, g, beta, split):
    e, ss, se = ("es", "ss", "se") if split else ("f64", "f64", "f64")
    chunks = []
    for c0 in range(0, q.shape[0], 64):  # pre-pass: independent of S
        c = slice(c0, min(q.shape[0], c0 + 64))
        T, P, Gam, E = _chunk_consts(k[c], q[c], g[c], beta[c])
        W = _mm(T * Gam[None, :], k[c], se)
        U0 = _mm(T, v[c], se)
        if split:  # stored between the passes as bf16 planes hi + lo
            W, U0 = (sum(_split(W)), sum(_split(U0)))
        chunks.append((c, P, Gam, E, W, U0))
    S = S.astype(np.float32).copy()
    o = np.zeros((q.shape[0], v.shape[1]), np.float32)
    for c, P, Gam, E, W, U0 in chunks:  # the chain, and the outputs from each chunk's entering state
        R = U0 - _mm(W, S, ss)
        o[c] = Gam[:, None] * _mm(q[c], S, e) + _mm(P, R, ss)
        S = Gam[-1] * S + _mm(k[c].T, E[:, None] * R, e)
    return S, o


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _cases():
    # (T, H, entering state): a ragged last chunk, several chunks, a single partial chunk
    return [(200, 2, True), (130, 1, False), (63, 1, True)]


@pytest.mark.parametrize("T,H,s0", _cases())
@pytest.mark.parametrize("form", ["one_pass", "three_pass"])
def test_chunked_forms_match_token_recurrence(T, H, s0, form):
    x = gdn_prefill_inputs(1, T, H, 7, s0=s0)
    S_ref = x["S"].numpy().copy()
    o_ref = oracle.gdn_prefill(S_ref, bf16_bits(x["q"]), bf16_bits(x["k"]), bf16_bits(x["v"]), x["g"].numpy(),
                               x["beta"].numpy())
    q, k, v = (x[n].float().numpy()[0] for n in ("q", "k", "v"))
    g, beta = x["g"].numpy()[0], x["beta"].numpy()[0]
    run = {"one_pass": _one_pass, "three_pass": _three_pass}[form]
    for h in range(H):
        S0 = x["S"].numpy()[0, h]
        for split, tol in ((False, 1e-6), (True, 2e-5)):  # measured: <= 8e-8 / 2.4e-7 and <= 6.2e-6 / 5.1e-6
            S, o = run(S0, q[:, h], k[:, h], v[:, h], g[:, h], beta[:, h], split)
            assert _rel(S, S_ref[0, h]) < tol, (form, split, _rel(S, S_ref[0, h]))
            assert _rel(o, o_ref[0, :, h]) < tol, (form, split, _rel(o, o_ref[0, :, h]))


def test_blocked_triangular_solve_forms_agree():
    """T = (I + N)^-1 diag(beta) in 32-row blocks. The diagonal blocks T11, T22 come from forward substitution.
    The off-diagonal block either comes from (I + N22) T21 = -N21 T11 by substitution, as the kernel solves it, or
    is the product -T22 (M21 T11). Here M21 is N21 without its beta_t factors (the rows of (I + N22)^-1 = T22
    diag(1/beta_2)), so that form needs no division by beta. Both equal the corresponding block of the direct
    inverse."""
    x = gdn_prefill_inputs(1, 64, 1, 11)
    K = x["k"].float().numpy()[0, :, 0].astype(np.float64)
    g, beta = x["g"].numpy()[0, :, 0].astype(np.float64), x["beta"].numpy()[0, :, 0].astype(np.float64)
    G = np.cumsum(g)
    t, s = np.meshgrid(np.arange(64), np.arange(64), indexing="ij")
    M = np.where(s < t, (K @ K.T) * np.exp(np.minimum(G[:, None] - G[None, :], 0.0)), 0.0)  # without beta
    N = beta[:, None] * M
    T = np.linalg.solve(np.eye(64) + N, np.diag(beta))
    h = slice(0, 32), slice(32, 64)
    T11 = np.linalg.solve(np.eye(32) + N[h[0], h[0]], np.diag(beta[h[0]]))
    T22 = np.linalg.solve(np.eye(32) + N[h[1], h[1]], np.diag(beta[h[1]]))
    T21_sub = np.linalg.solve(np.eye(32) + N[h[1], h[1]], -N[h[1], h[0]] @ T11)
    T21_prod = -T22 @ (M[h[1], h[0]] @ T11)
    ref = T[h[1], h[0]]
    assert np.allclose(T11, T[h[0], h[0]], rtol=0, atol=1e-12) and np.allclose(T22, T[h[1], h[1]], rtol=0, atol=1e-12)
    assert _rel(T21_sub, ref) < 1e-12 and _rel(T21_prod, ref) < 1e-12

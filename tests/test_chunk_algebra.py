"""CPU check (float64 torch) of the chunked WY algebra the tensor-core DeltaNet /
GatedDeltaNet kernels implement (edifice_b200/csrc/delta_prep.cuh,
delta_chunked.cu, delta_chunked_bwd.cu, delta_chunked_post.cu), against
autograd of the token recurrence S_t = alpha_t S_{t-1} + beta_t (v_t - alpha_t
S_{t-1} k_t) k_t^T, o_t = S_t q_t (lib/edifice/cuda/fused_scan.ex:2256-2284; alpha = 1
is the delta rule, :2212-2236).

Every quantity is formed the way the kernels form it: per chunk of C tokens the
in-chunk log-decay cumsum g, gamma = exp(g), Gamma_ts = exp(g_t - g_s) (s <= t);
the forward products (T, W = T diag(beta gamma) K, U0, U~, O, S_C); the state
pass (dU~, dS_0 with the gamma_C scale between its two products); the post
kernel's gradients with the row scales kept apart (dQa~, dK~, T_b^T dW) and the
log-decay gradient dg gathered from the same six places, then dalpha_s =
sum_{t >= s} dg_t / alpha_s.  A mistake in the derivation shows here at
float64 precision, independent of the GPU.
"""
import pytest
import torch

DT = torch.float64


def _token_forward(q, k, v, beta, alpha):
    L, d = q.shape
    S = torch.zeros(d, d, dtype=DT)
    out = []
    for t in range(L):
        Sd = alpha[t] * S
        S = Sd + torch.outer(beta[t] * (v[t] - Sd @ k[t]), k[t])
        out.append(S @ q[t])
    return torch.stack(out)


def _chunk_forward(q, k, v, beta, alpha, C):
    L, d = q.shape
    S = torch.zeros(d, d, dtype=DT)
    O = torch.zeros(L, d, dtype=DT)
    saved = []
    for t0 in range(0, L, C):
        n = min(C, L - t0)
        pad = lambda x: torch.cat([x[t0:t0 + n], x.new_zeros((C - n,) + x.shape[1:])])
        Q, K, V, b = pad(q), pad(k), pad(v), pad(beta)
        la = torch.cat([torch.log(alpha[t0:t0 + n]), alpha.new_zeros(C - n)])  # pad: alpha = 1
        g = torch.cumsum(la, 0)
        gam, kap = torch.exp(g), torch.exp(g[-1] - g)
        Gam = torch.tril(torch.exp(g[:, None] - g[None, :]))
        G = K @ K.T
        A = torch.tril(b[:, None] * (G * Gam), -1)
        T = torch.linalg.inv(torch.eye(C, dtype=DT) + A)
        Tb = T * b[None, :]
        W = Tb @ (gam[:, None] * K)
        M = torch.tril(Q @ K.T) * Gam
        S0 = S.clone()
        Ut = Tb @ V - W @ S0.T
        O[t0:t0 + n] = ((gam[:, None] * Q) @ S0.T + M @ Ut)[:n]
        S = torch.exp(g[-1]) * S0 + Ut.T @ (kap[:, None] * K)
        saved.append(dict(Q=Q, K=K, V=V, b=b, g=g, gam=gam, kap=kap, Gam=Gam, G=G, T=T, Tb=Tb,
                          W=W, M=M, S0=S0, Ut=Ut, n=n, t0=t0))
    return O, saved


def _chunk_backward(saved, dO_all, alpha):
    L, d = dO_all.shape
    dq, dk, dv = (torch.zeros(L, d, dtype=DT) for _ in range(3))
    db, da = torch.zeros(L, dtype=DT), torch.zeros(L, dtype=DT)
    dS = torch.zeros(d, d, dtype=DT)
    for c in reversed(saved):
        n, t0 = c["n"], c["t0"]
        C = c["Q"].shape[0]
        dO = torch.zeros(C, d, dtype=DT)
        dO[:n] = dO_all[t0:t0 + n]
        gam, kap, Gam, S0, Ut, K, Q = c["gam"], c["kap"], c["Gam"], c["S0"], c["Ut"], c["K"], c["Q"]
        gC = torch.exp(c["g"][-1])
        dSC = dS
        # state pass: dU~ = M^T dO + K~ dS_C^T, dS_0 = gamma_C dS_C + dO^T Q~ - dU~^T W
        dU = c["M"].T @ dO + (kap[:, None] * K) @ dSC.T
        dS = gC * dSC + dO.T @ (gam[:, None] * Q) - dU.T @ c["W"]
        # post kernel
        dQa, dW, dK1 = dO @ S0, -dU @ S0, Ut @ dSC
        dMraw = torch.tril(dO @ Ut.T)
        dTb = dW @ (gam[:, None] * K).T + dU @ c["V"].T
        Xp = c["T"].T @ dTb
        dA = torch.tril(-(Xp @ c["Tb"].T), -1)
        GG = torch.tril(c["G"] * Gam, -1)
        dbeta = (dA * GG).sum(1) + torch.diagonal(Xp)
        E0 = (c["b"][:, None] * dA) * Gam
        E = E0 + E0.T
        dMt = dMraw * Gam
        dKW = c["Tb"].T @ dW
        dQ = gam[:, None] * dQa + dMt @ K
        dK = dMt.T @ Q + E @ K + kap[:, None] * dK1 + gam[:, None] * dKW
        dV = c["Tb"].T @ dU
        dg = torch.zeros(C, dtype=DT)
        dg[-1] += gC * (dSC * S0).sum()
        MM = dMraw * c["M"]
        AA = dA * (c["b"][:, None] * GG)
        dg += MM.sum(1) - MM.sum(0) + AA.sum(1) - AA.sum(0)
        k1 = kap[:, None] * dK1
        dg += ((gam[:, None] * dQa) * Q).sum(1) + (K * (gam[:, None] * dKW - k1)).sum(1)
        dg[-1] += (K * k1).sum()
        dlog = torch.flip(torch.cumsum(torch.flip(dg, [0]), 0), [0])
        dq[t0:t0 + n], dk[t0:t0 + n], dv[t0:t0 + n] = dQ[:n], dK[:n], dV[:n]
        db[t0:t0 + n] = dbeta[:n]
        da[t0:t0 + n] = dlog[:n] / alpha[t0:t0 + n]
    return dq, dk, dv, db, da


@pytest.mark.parametrize("L,d,C,alpha_lo", [(20, 6, 8, 0.3), (37, 5, 8, 0.01), (8, 4, 8, 0.5),
                                            (3, 4, 8, 0.2), (70, 8, 16, 1.0)])
def test_chunked_gated_algebra_matches_token_autograd(L, d, C, alpha_lo):
    g = torch.Generator().manual_seed(L * 31 + d)
    q = torch.randn(L, d, dtype=DT, generator=g)
    k = torch.randn(L, d, dtype=DT, generator=g)
    k = k / k.norm(dim=1, keepdim=True)
    v = torch.randn(L, d, dtype=DT, generator=g)
    beta = torch.sigmoid(torch.randn(L, dtype=DT, generator=g))
    alpha = alpha_lo + (1 - alpha_lo) * torch.rand(L, dtype=DT, generator=g)
    dO = torch.randn(L, d, dtype=DT, generator=g)
    leaves = [x.clone().requires_grad_(True) for x in (q, k, v, beta, alpha)]
    o_ref = _token_forward(*leaves)
    o_ref.backward(dO)
    o, saved = _chunk_forward(q, k, v, beta, alpha, C)
    assert (o - o_ref.detach()).abs().max() <= 1e-12
    for got, leaf in zip(_chunk_backward(saved, dO, alpha), leaves):
        ref = leaf.grad
        assert (got - ref).abs().max() <= 1e-11 * max(1.0, ref.abs().max().item())

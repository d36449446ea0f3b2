"""CPU check of the Gated DeltaNet restatement in the oracle (oracle/ref_compose.c,
kref_gdn_apply) against an independent float64 numpy formulation of the published gated
delta rule in matrix form (Yang, Kautz, Hatamizadeh, "Gated Delta Networks", ICLR 2025):

    S_t = exp(g_t) S_{t-1} (I - beta_t k_t k_t^T) + beta_t v_t k_t^T,   o_t = S_t q_t

with the Qwen3-Next / Qwen3.5 layer around it (causal depthwise conv + SiLU, per-head L2
norms, q scaled by 1/sqrt(dk), beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias),
RMSNorm(o) * w * silu(z)). The reference has no source for this mixer, so this pins the
restatement's algebra; the plugin's kernel is checked against the restatement on the GPU."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import rel_l2


def gdn_numpy(nk, nv, dh, K, eps, conv, a_log, dt_bias, norm_w, qkv, z, b, a):
    T, Cn = qkv.shape
    X = qkv.astype(np.float64)
    pad = np.vstack([np.zeros((K - 1, Cn)), X])
    cv = np.stack([(pad[t:t + K] * conv.T.astype(np.float64)).sum(0) for t in range(T)])
    act = cv / (1.0 + np.exp(-cv))
    q = act[:, :nk * dh].reshape(T, nk, dh)
    k = act[:, nk * dh:2 * nk * dh].reshape(T, nk, dh)
    v = act[:, 2 * nk * dh:].reshape(T, nv, dh)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6) / np.sqrt(dh)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    beta = 1.0 / (1.0 + np.exp(-b.astype(np.float64)))
    g = -np.exp(a_log.astype(np.float64)) * np.log1p(np.exp(a.astype(np.float64) + dt_bias))
    ratio = nv // nk
    S = np.zeros((nv, dh, dh))
    out = np.zeros((T, nv, dh))
    eye = np.eye(dh)
    for t in range(T):
        for h in range(nv):
            kt, qt = k[t, h // ratio], q[t, h // ratio]
            S[h] = np.exp(g[t, h]) * S[h] @ (eye - beta[t, h] * np.outer(kt, kt)) \
                + beta[t, h] * np.outer(v[t, h], kt)
            o = S[h] @ qt
            zz = z[t, h * dh:(h + 1) * dh].astype(np.float64)
            out[t, h] = o / np.sqrt((o * o).mean() + eps) * norm_w * zz / (1.0 + np.exp(-zz))
    return out.reshape(T, nv * dh)


@pytest.mark.parametrize("nk,nv,dh,K,T", [(2, 4, 64, 4, 12), (1, 1, 128, 3, 6), (2, 2, 32, 2, 9)])
def test_gdn_restatement_matches_matrix_form(ref, nk, nv, dh, K, T):
    rng = np.random.default_rng(nk * 100 + nv * 10 + K)
    Cn, VD = (2 * nk + nv) * dh, nv * dh
    f = lambda *s, sc=1.0: (rng.normal(0, sc, s)).astype(np.float32)  # noqa: E731
    conv, qkv, z = f(Cn, K, sc=0.3), f(T, Cn), f(T, VD)
    b, a = f(T, nv), f(T, nv)
    a_log = np.log(rng.uniform(1, 16, nv)).astype(np.float32)
    dt_bias = rng.uniform(-4, -2, nv).astype(np.float32)
    norm_w = (1 + 0.1 * rng.normal(0, 1, dh)).astype(np.float32)
    out = np.zeros((T, VD), np.float32)
    L = ref.L
    L.kref_gdn_apply.restype = C.c_int
    L.kref_gdn_apply.argtypes = [C.c_int] * 5 + [C.c_float] + [C.c_void_p] * 9
    rc = L.kref_gdn_apply(nk, nv, dh, K, T, 1e-6, *[x.ctypes.data for x in
                                                    (conv, a_log, dt_bias, norm_w, qkv, z, b, a, out)])
    assert rc == 0
    want = gdn_numpy(nk, nv, dh, K, 1e-6, conv, a_log, dt_bias, norm_w, qkv, z, b, a)
    assert rel_l2(out, want) <= 1e-5
    # the recurrence matters: step t > 0 differs from a state-free evaluation
    assert np.abs(out[-1]).sum() > 0

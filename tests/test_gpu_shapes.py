"""Layer shapes of other members of the model families, beyond the benchmark configs.

MoE: a Qwen3-30B-A3B-like layer (hidden 2048, 128 experts, expert FFN 768, top-8) through the
fused batch-1 kernel, the ragged batch (DP4A and tensor-core groups) and the expert-parallel
stages (4 virtual ranks on one GPU). Dense: small Qwen3-family decoders (head_dim 128, GQA
2:1 and 4:1) with greedy tokens byte-identical to the reference's CPU decode."""
import numpy as np
import pytest
import torch

from katali_lab_b200 import MOE_Q8_1, DenseModel
from katali_lab_b200.ep import EpMoeLayer, local_experts
from katali_lab_b200.synth import DenseConfig, make_dense_model
from oracle.oracle import RefDense, rel_l2
from tests.test_gpu_moe import DevLayer, dev, empty, host

pytestmark = pytest.mark.gpu

E, H, F, K = 128, 2048, 768, 8


@pytest.fixture(scope="module")
def a3b(plugin):
    return DevLayer(plugin, E, H, F, K, seed=81)


def inputs(seed, T, hot=0):
    rng = np.random.default_rng(seed)
    X = rng.normal(0, 1, (T, H)).astype(np.float32)
    L = rng.normal(0, 1, (T, E)).astype(np.float32)
    if hot:
        L[:, :hot] += 8.0
    return X, L


def test_a3b_fused_layer(a3b, port):
    for s in range(4):
        X, L = inputs(810 + s, 1)
        y = a3b.run(X[0], L[0], MOE_Q8_1)
        want, _, _, _ = port.moe_layer(a3b.host, X[0], L[0], mode=0)
        assert rel_l2(y, want) <= 1e-5
        assert np.mean(y == want) >= 0.999


@pytest.mark.parametrize("T,hot,tol", [(9, 0, 1e-5), (40, 8, 5e-4)])
def test_a3b_batch(a3b, port, T, hot, tol):
    X, L = inputs(820 + T, T, hot)
    Y = empty(T * H).view(T, H)
    a3b.layer.forward_batch(dev(X), dev(L), Y)
    Y = host(Y)
    for t in sorted({0, T // 2, T - 1}):
        want, _, _, _ = port.moe_layer(a3b.host, X[t], L[t], mode=0)
        assert rel_l2(Y[t], want) <= tol, t


def test_a3b_expert_parallel_stages(plugin, a3b):
    plugin.set_stream(torch.cuda.current_stream())
    G, Ts = 4, [3, 1, 0, 2]
    tmax = max(Ts)
    eps = [EpMoeLayer(plugin, E, H, F, K, [a3b.ptrs[e] for e in local_experts(E, G, r)], G, r, tmax)
           for r in range(G)]
    ins = [inputs(830 + r, max(T, 1)) for r, T in enumerate(Ts)]
    xs = [dev(x) for x, _ in ins]
    ls = [dev(l) for _, l in ins]

    def exchange(outs):
        ch = [torch.chunk(o, G) for o in outs]
        return [torch.cat([ch[d][r] for d in range(G)]).contiguous() for r in range(G)]

    sends = [eps[r].dispatch(Ts[r], xs[r], ls[r]).clone() for r in range(G)]
    recvs = exchange(sends)
    rets = [eps[r].experts(recvs[r]).clone() for r in range(G)]
    backs = exchange(rets)
    for r in range(G):
        if not Ts[r]:
            continue
        y = empty(Ts[r] * H).view(Ts[r], H)
        eps[r].combine(Ts[r], backs[r], y)
        want = empty(Ts[r] * H).view(Ts[r], H)
        a3b.layer.forward_batch(xs[r][:Ts[r]], ls[r][:Ts[r]], want)
        assert rel_l2(host(y).ravel(), host(want).ravel()) <= 1e-5
    for e in eps:
        e.close()
    plugin.set_stream(None)


@pytest.mark.parametrize("cfg", [
    DenseConfig(n_layers=3, hidden=1024, ffn=3072, n_heads=16, n_kv_heads=8, head_dim=128,
                vocab=8192, kv_cap=128),   # 0.6B-like heads (GQA 2:1)
    DenseConfig(n_layers=2, hidden=2048, ffn=6144, n_heads=16, n_kv_heads=4, head_dim=128,
                vocab=4096, kv_cap=128),   # 1.7B/4B-like heads (GQA 4:1)
])
def test_dense_family_greedy(plugin, ref, port, cfg):
    model = make_dense_model(plugin, cfg, seed=cfg.hidden + cfg.n_heads)
    dm = DenseModel(plugin, model)
    rd = RefDense(ref, model)
    prompt, n_gen = [2, 11, 400], 12
    got = dm.generate(prompt, n_gen).tolist()
    tok, want = None, []
    for s in range(len(prompt) + n_gen - 1):
        lg = rd.step(prompt[s] if s < len(prompt) else tok, s)
        tok = port.argmax(lg)
        if s >= len(prompt) - 1:
            want.append(tok)
    assert got == want
    rd.close()
    dm.close()

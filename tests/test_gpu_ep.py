"""GPU parity of the expert-parallel stages (katali_cuda_moe_ep_*) on one GPU.

G ranks are emulated in one process: G layer objects, each holding only its block
of experts, exchange their slot buffers by device copies. Bars: dispatch slots
equal the oracle's restatement (headers, owned ids, weights bit-identical, q8_1 rows
byte-identical); the experts stage's per-slot partial sums within rel_L2 <= 1e-5 of
the oracle's on the same received bytes; every token's output within rel_L2 <= 1e-5
of katali_cuda_moe_batch on the full layer with >= 99.9 % of elements bit-equal, also with
every token on the same experts (tensor-core groups in the experts stage)."""
import numpy as np
import pytest
import torch

from katali_lab_b200.ep import EpMoeLayer, local_experts
from oracle.oracle import rel_l2
from tests.test_gpu_moe import DevLayer, dev, empty, host

pytestmark = pytest.mark.gpu

E, H, F, K = 64, 2048, 512, 8


@pytest.fixture(scope="module")
def full(plugin):
    return DevLayer(plugin, E, H, F, K, seed=51)


def exchange(outs, G):
    chunks = [torch.chunk(o, G) for o in outs]
    return [torch.cat([chunks[d][r] for d in range(G)]).contiguous() for r in range(G)]


def ep_layers(plugin, full, G, tmax):
    return [EpMoeLayer(plugin, E, H, F, K, [full.ptrs[e] for e in local_experts(E, G, r)], G, r,
                       tmax) for r in range(G)]


def inputs(seed, T):
    rng = np.random.default_rng(seed)
    return rng.normal(0, 1, (T, H)).astype(np.float32), rng.normal(0, 1, (T, E)).astype(np.float32)


@pytest.mark.parametrize("G,Ts", [(2, [5, 3]), (4, [1, 7, 0, 4]), (8, [1] * 8)])
def test_ep_virtual_ranks_vs_batch(plugin, full, G, Ts):
    # the exchange below runs on torch's current stream: order the stages on it too
    plugin.set_stream(torch.cuda.current_stream())
    tmax = max(Ts)
    eps = ep_layers(plugin, full, G, tmax)
    ins = [inputs(60 + r, T) for r, T in enumerate(Ts)]
    xs = [dev(x) if T else empty(H).view(1, H) for (x, _), T in zip(ins, Ts)]
    ls = [dev(l) if T else empty(E).view(1, E) for (_, l), T in zip(ins, Ts)]
    sends = [eps[r].dispatch(Ts[r], xs[r], ls[r]).clone() for r in range(G)]
    recvs = exchange(sends, G)
    rets = [eps[r].experts(recvs[r]).clone() for r in range(G)]
    backs = exchange(rets, G)
    for r in range(G):
        if Ts[r] == 0:
            continue
        y = empty(Ts[r] * H).view(Ts[r], H)
        eps[r].combine(Ts[r], backs[r], y)
        want = empty(Ts[r] * H).view(Ts[r], H)
        full.layer.forward_batch(xs[r], ls[r], want)
        y, want = host(y), host(want)
        for t in range(Ts[r]):
            assert rel_l2(y[t], want[t]) <= 1e-5, (r, t)
            assert np.mean(y[t] == want[t]) >= 0.999, (r, t)
    for e in eps:
        e.close()
    plugin.set_stream(None)


def test_ep_virtual_ranks_tensor_core_groups(plugin, full):
    """Every token on the same 8 experts (4 on each of 2 virtual ranks): each rank's experts
    stage sees groups of 48 received slots, so gate/up and down run on the tensor cores.
    A token's arithmetic there does not depend on its place in the group, so each rank's
    outputs equal katali_cuda_moe_batch of all ranks' tokens on the full layer (the same
    groups) at the expert-parallel bars."""
    plugin.set_stream(torch.cuda.current_stream())
    G, T = 2, 24
    eps = ep_layers(plugin, full, G, T)
    hot = [3, 9, 20, 30, 35, 41, 50, 60]
    ins = []
    for r in range(G):
        X, L = inputs(90 + r, T)
        L[:, hot] += 8.0
        ins.append((X, L))
    sends = [eps[r].dispatch(T, dev(ins[r][0]), dev(ins[r][1])).clone() for r in range(G)]
    recvs = exchange(sends, G)
    rets = [eps[r].experts(recvs[r]).clone() for r in range(G)]
    backs = exchange(rets, G)
    want = empty(G * T * H).view(G * T, H)
    full.layer.forward_batch(dev(np.concatenate([x for x, _ in ins])),
                             dev(np.concatenate([l for _, l in ins])), want)
    want = host(want)
    for r in range(G):
        y = empty(T * H).view(T, H)
        eps[r].combine(T, backs[r], y)
        y = host(y)
        for t in range(T):
            assert rel_l2(y[t], want[r * T + t]) <= 1e-5, (r, t)
            assert np.mean(y[t] == want[r * T + t]) >= 0.999, (r, t)
    for e in eps:
        e.close()
    plugin.set_stream(None)


def test_ep_dispatch_matches_oracle(plugin, port, full):
    G, T, tmax = 4, 6, 8
    (ep,) = ep_layers(plugin, full, G, tmax)[:1]
    X, L = inputs(70, T)
    send = host(ep.dispatch(T, dev(X), dev(L)))
    want, src = port.ep_dispatch(full.host, G, tmax, X, L)
    sb = port.ep_slot_bytes(H, K)
    assert ep.slot_bytes == sb
    got, want = send.reshape(G, tmax, sb), want.reshape(G, tmax, sb)
    hdr = 16 + 8 * K
    for d in range(G):
        for t in range(tmax):
            n = int(want[d, t, :4].view(np.int32)[0])
            assert np.array_equal(got[d, t, :16], want[d, t, :16]), (d, t)
            if t < T:
                assert np.array_equal(got[d, t, 16:hdr], want[d, t, 16:hdr]), (d, t)
            if n:
                assert np.array_equal(got[d, t, 80:], want[d, t, 80:]), (d, t)
    ep.close()


def test_ep_experts_match_oracle(plugin, port, full):
    """The experts stage of rank 1 of 2 on slots the oracle packed."""
    G, tmax = 2, 5
    eps = ep_layers(plugin, full, G, tmax)
    sends = []
    for r, T in enumerate([5, 3]):
        X, L = inputs(80 + r, T)
        s, _ = port.ep_dispatch(full.host, G, tmax, X, L)
        sends.append(torch.from_numpy(s))
    recv1 = exchange(sends, G)[1]
    got = host(eps[1].experts(recv1.cuda()))
    want = port.ep_experts(full.host, G, 1, tmax, recv1.numpy())
    sb = port.ep_slot_bytes(H, K)
    slots = recv1.numpy().reshape(G * tmax, sb)
    n_checked = 0
    for s in range(G * tmax):
        if slots[s, :4].view(np.int32)[0] > 0:
            a, b = got[s * H:(s + 1) * H], want[s * H:(s + 1) * H]
            assert rel_l2(a, b) <= 1e-5, s
            n_checked += 1
    assert n_checked > 0
    for e in eps:
        e.close()


@pytest.mark.parametrize("G,Ts", [(8, [1] * 8), (2, [5, 3])])
def test_ep_experts_fused_matches_pipeline(plugin, full, monkeypatch, G, Ts):
    """Up to 16 received slots run the experts stage in the fused MoE kernel (pairs of
    the slots in rounds of K, one token's x per pair); the same sums as the ragged-batch
    pipeline within rel_L2 <= 1e-5 per slot and >= 99.9 % bit-equal. (2, [5, 3]) gives
    each rank ~30 pairs: four rounds, with slots whose pairs span two rounds."""
    plugin.set_stream(torch.cuda.current_stream())  # the exchange runs on torch's stream
    tmax = max(Ts)
    eps = ep_layers(plugin, full, G, tmax)
    sends = []
    for r, T in enumerate(Ts):
        X, L = inputs(95 + r, T)
        sends.append(eps[r].dispatch(T, dev(X), dev(L)).clone())
    recvs = exchange(sends, G)
    sb = eps[0].slot_bytes
    for r in sorted({0, G // 2, G - 1}):
        monkeypatch.delenv("KATALI_CUDA_NO_EP_FUSED", raising=False)
        fused = host(eps[r].experts(recvs[r])).copy()
        monkeypatch.setenv("KATALI_CUDA_NO_EP_FUSED", "1")
        staged = host(eps[r].experts(recvs[r])).copy()
        slots = host(recvs[r]).reshape(G * tmax, sb)
        n_checked = 0
        for s_ in range(G * tmax):
            ids = slots[s_, 16:16 + 4 * K].view(np.int32)
            if slots[s_, :4].view(np.int32)[0] > 0 and (ids >= 0).any():
                a, b = fused[s_ * H:(s_ + 1) * H], staged[s_ * H:(s_ + 1) * H]
                assert rel_l2(a, b) <= 1e-5, (r, s_)
                assert np.mean(a == b) >= 0.999, (r, s_)
                n_checked += 1
        assert n_checked > 0
    for e in eps:
        e.close()
    plugin.set_stream(None)


def test_ep_arg_checks(plugin, full):
    from katali_lab_b200 import KataliError
    ep = ep_layers(plugin, full, 2, 4)[0]
    x, lg = dev(inputs(90, 2)[0]), dev(inputs(90, 2)[1])
    with pytest.raises(KataliError) as e:
        ep.dispatch(5, x, lg)  # n_tokens > max_tokens
    assert e.value.code == 3
    # a layer of 64 experts does not split over 3 ranks
    from katali_lab_b200.ep import EpMoeLayer
    with pytest.raises(ValueError):
        EpMoeLayer(plugin, E, H, F, K, [], 3, 0, 4)
    ep.close()

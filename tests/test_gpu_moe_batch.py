"""GPU parity of the ragged-batch MoE layer (katali_cuda_moe_batch), through the C ABI.

Bars, per token of a batch: routing identical to the batch-1 kernel, output within
rel_L2 <= 1e-5 of the q8_1 restatement (port.moe_layer, mode 0) and at least 99.9 %
of elements bit-equal to it; the same bars against the batch-1 kernel's output for
the same token. Groups of >= 16 tokens run gate/up on the tensor cores (tcgen05
int8 MMA) with fp32 block terms; their bar is TC_TOL below. Groups of >= 8 tokens run
the Q6_K down projection there, at the strict bars; the strict bars are also checked
with every group on the DP4A kernels (KATALI_CUDA_NO_TC=1). Their Q6_K down projection
also runs there, with exact integer block sums and double accumulation in the
restatement's order, so a layer whose gate/up stay on the DP4A kernels (Q6_K gate and
up) keeps the strict bars with its down projection on the tensor cores. Edge cases: one token,
every token on the same experts, groups of 16 / 33 / 100 tokens, batch sizes that
grow and shrink between calls, no-norm routing, 1024 experts with top-16, and the
argument checks."""
import numpy as np
import pytest

from katali_lab_b200 import MOE_F32, MOE_Q8_1, Q6_K, KataliError
from oracle.oracle import MoeWeights, rel_l2
from tests.test_gpu_moe import DevLayer, dev, empty, host

pytestmark = pytest.mark.gpu


def batch_inputs(seed, T, H, E, bias=None):
    rng = np.random.default_rng(seed)
    X = rng.normal(0, 1, (T, H)).astype(np.float32)
    L = rng.normal(0, 1, (T, E)).astype(np.float32)
    if bias is not None:
        L[:, bias] += 8.0
    return X, L


def run_batch(layer, X, L):
    T, H = X.shape
    Y = empty(T * H).view(T, H)
    layer.layer.forward_batch(dev(X), dev(L), Y)
    return host(Y)


def check_tokens(layer, port, X, L, Y, against_batch1=True):
    for t in range(X.shape[0]):
        want, _, _, _ = port.moe_layer(layer.host, X[t], L[t], mode=0)
        assert rel_l2(Y[t], want) <= 1e-5, t
        assert np.mean(Y[t] == want) >= 0.999, t
        if against_batch1:
            y1 = layer.run(X[t], L[t], MOE_Q8_1)
            assert rel_l2(Y[t], y1) <= 1e-5, t
            assert np.mean(Y[t] == y1) >= 0.999, t


@pytest.fixture(scope="module")
def c3_layer(plugin):
    return DevLayer(plugin, 64, 2048, 512, 8, seed=31)


@pytest.mark.parametrize("T", [1, 5, 17, 64])
def test_batch_vs_restatement(c3_layer, port, monkeypatch, T):
    """As run (at T = 64 groups of 8 to 15 tokens take the tensor-core down projection),
    then with every group on the DP4A kernels; the strict bars both times."""
    X, L = batch_inputs(300 + T, T, 2048, 64)
    Y = run_batch(c3_layer, X, L)
    check_tokens(c3_layer, port, X, L, Y, against_batch1=T <= 17)
    monkeypatch.setenv("KATALI_CUDA_NO_TC", "1")
    Y = run_batch(c3_layer, X, L)
    check_tokens(c3_layer, port, X, L, Y, against_batch1=T <= 17)


def test_batch_single_token_equals_batch1(c3_layer):
    for s in range(4):
        X, L = batch_inputs(400 + s, 1, 2048, 64)
        Y = run_batch(c3_layer, X, L)
        y1 = c3_layer.run(X[0], L[0], MOE_Q8_1)
        assert rel_l2(Y[0], y1) <= 1e-5
        assert np.mean(Y[0] == y1) >= 0.999


TC_TOL = 5e-4  # tensor-core gate/up: fp32 block terms, then q8_1 of h can flip a rounding


def check_tokens_tc(layer, port, X, L, Y):
    """Tokens whose experts ran on the tensor-core path: each block term is rounded to
    fp32 (the DP4A path keeps exact double terms), and the q8_1 quantisation of h can
    then flip the odd rounding, so the bar against the q8_1 restatement is TC_TOL, two
    orders of magnitude below the q8_1 vs fp32 activation difference (~1e-2)."""
    for t in range(X.shape[0]):
        want, _, _, _ = port.moe_layer(layer.host, X[t], L[t], mode=0)
        assert rel_l2(Y[t], want) <= TC_TOL, t


def test_batch_skewed_routing(c3_layer, port, monkeypatch):
    """Every token on the same 8 experts: 48 tokens per expert, the tensor-core path
    (tcgen05 int8 MMA) for gate/up; and the same batch with it switched off."""
    X, L = batch_inputs(500, 48, 2048, 64, bias=[3, 9, 10, 17, 33, 40, 41, 63])
    Y = run_batch(c3_layer, X, L)
    check_tokens_tc(c3_layer, port, X, L, Y)
    monkeypatch.setenv("KATALI_CUDA_NO_TC", "1")
    Y2 = run_batch(c3_layer, X, L)
    check_tokens(c3_layer, port, X[:12], L[:12], Y2[:12], against_batch1=False)
    check_tokens(c3_layer, port, X[40:], L[40:], Y2[40:], against_batch1=False)
    assert rel_l2(Y.ravel(), Y2.ravel()) <= TC_TOL


@pytest.mark.parametrize("T,hot", [(16, 8), (33, 8), (100, 8), (64, 3)])
def test_batch_tensor_core_groups(c3_layer, port, T, hot):
    """Groups of exactly 16, of 33 (a partial second token tile), of 100 tokens, and a
    mix where some experts have >= 16 tokens and others fewer."""
    X, L = batch_inputs(600 + T + hot, T, 2048, 64, bias=list(range(hot)))
    Y = run_batch(c3_layer, X, L)
    idx = sorted({0, T // 3, T // 2, T - 1})
    check_tokens_tc(c3_layer, port, X[idx], L[idx], Y[idx])


@pytest.fixture(scope="module")
def q6_layer(plugin, port):
    """Q6_K gate, up and down (16 experts, H 2048, F 512, top-4; Q6_K gate/up rows are
    16-byte multiples from H 2048): gate/up stay on the DP4A kernels, the down projection
    of groups of >= 16 tokens runs on the tensor cores."""
    E, H, F, K = 16, 2048, 512, 4
    rng = np.random.default_rng(41)

    def store(rows, cols):
        return np.stack([port.quantize(Q6_K, rng.normal(0, 0.02, rows * cols).astype(np.float32))
                         for _ in range(E)])

    mw = MoeWeights(store(F, H), store(F, H), store(H, F), H, F, K, True,
                    gate_type=Q6_K, up_type=Q6_K, down_type=Q6_K)
    return DevLayer(plugin, E, H, F, K, seed=0, from_host=mw)


@pytest.mark.parametrize("T", [20, 64])
def test_batch_tensor_core_down_strict(q6_layer, port, monkeypatch, T):
    """Every token on the same 4 experts: groups of T tokens (one partial token tile at
    T = 20, two full tiles at 64) whose down projection runs on the tensor cores; the
    strict bars against the restatement, and bit-equality with the all-DP4A run."""
    X, L = batch_inputs(950 + T, T, 2048, 16, bias=[2, 5, 11, 13])
    Y = run_batch(q6_layer, X, L)
    check_tokens(q6_layer, port, X, L, Y, against_batch1=False)
    monkeypatch.setenv("KATALI_CUDA_NO_TC", "1")
    Y2 = run_batch(q6_layer, X, L)
    assert np.mean(Y == Y2) >= 0.999


def test_batch_ragged_sequence(c3_layer, port, monkeypatch):
    """Scratch grows and shrinks: T = 3, 40, 7, 64, 2 on one layer object, as run and with
    every group on the DP4A kernels; the strict bars both times."""
    for no_tc in ("0", "1"):
        monkeypatch.setenv("KATALI_CUDA_NO_TC", no_tc)
        for i, T in enumerate([3, 40, 7, 64, 2]):
            X, L = batch_inputs(600 + i, T, 2048, 64)
            Y = run_batch(c3_layer, X, L)
            idx = sorted({0, T // 2, T - 1})
            check_tokens(c3_layer, port, X[idx], L[idx], Y[idx], against_batch1=False)


def test_batch_deterministic(c3_layer):
    X, L = batch_inputs(700, 33, 2048, 64)
    a = run_batch(c3_layer, X, L)
    b = run_batch(c3_layer, X, L)
    assert np.array_equal(a, b)


def test_batch_no_norm_small_shapes(plugin, port):
    lay = DevLayer(plugin, 256, 512, 256, 8, seed=32, norm=False)
    X, L = batch_inputs(800, 23, 512, 256)
    Y = run_batch(lay, X, L)
    check_tokens(lay, port, X, L, Y)


def test_batch_1024_experts_top16(plugin, port):
    lay = DevLayer(plugin, 1024, 256, 256, 16, seed=33)
    X, L = batch_inputs(900, 9, 256, 1024)
    Y = run_batch(lay, X, L)
    check_tokens(lay, port, X, L, Y)


def test_batch_arg_checks(c3_layer):
    X, L = batch_inputs(1000, 2, 2048, 64)
    x, lg = dev(X), dev(L)
    y = empty(2 * 2048)
    lay = c3_layer.layer
    lay.forward_batch(x, lg, y, n_tokens=0)  # empty batch: nothing to do
    with pytest.raises(KataliError) as e:
        lay.forward_batch(x, lg, y, mode=MOE_F32)
    assert e.value.code == 4  # KATALI_ERR_UNSUPPORTED_TYPE
    with pytest.raises(KataliError) as e:
        lay.forward_batch(x, lg, y, n_tokens=4097)
    assert e.value.code == 3  # KATALI_ERR_BAD_ARG

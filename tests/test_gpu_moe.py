"""GPU parity of the fused MoE layer (katali_cuda_moe_layer), through the C ABI.

Bars: routing ids identical and weights bit-identical to the restatement;
q8_1-mode layer output within rel_L2 <= 1e-5 of the restatement (the design
makes it bit-exact except for astronomically rare double-rounding ties);
fp32-mode layer output within rel_L2 <= 1e-5 of the layer composed from the
reference's own CPU kernels; deterministic across calls."""
import numpy as np
import pytest

from katali_lab_b200 import MOE_F32, MOE_Q8_1, MoeLayer
from katali_lab_b200.synth import make_expert_store
from oracle.oracle import MoeWeights, make_moe_weights, rel_l2
from tests.golden.make_golden import MOE_CASE, moe_inputs

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def empty(n, dtype="float32"):
    import torch
    return torch.empty(n, dtype=getattr(torch, dtype), device="cuda")


class DevLayer:
    """A layer resident on the device plus its host copy for the oracles."""

    def __init__(self, plugin, E, H, F, K, seed, norm=True, from_host: MoeWeights | None = None):
        if from_host is None:
            st = make_expert_store(plugin, E, H, F, seed)
            self.bufs = (st.gate, st.up, st.down)
            self.host = MoeWeights(host(st.gate), host(st.up), host(st.down), H, F, K, norm)
        else:
            self.bufs = (dev(from_host.gate), dev(from_host.up), dev(from_host.down))
            self.host = from_host
        g, u, d = self.bufs
        ptrs = [(g.data_ptr() + e * g.shape[1], u.data_ptr() + e * u.shape[1],
                 d.data_ptr() + e * d.shape[1]) for e in range(E)]
        self.ptrs = ptrs
        self.layer = MoeLayer(plugin, E, H, F, K, ptrs, norm_topk=norm, gate_type=self.host.gate_type,
                              up_type=self.host.up_type, down_type=self.host.down_type)
        self.H, self.E, self.K = H, E, K

    def run(self, x, logits, mode=MOE_Q8_1):
        y = empty(self.H)
        self.layer.forward(dev(x), dev(logits), y, mode)
        return host(y)


@pytest.fixture(scope="module")
def c2_small(plugin):
    return DevLayer(plugin, 32, 2048, 512, 8, seed=21)


def rand_inputs(seed, H, E):
    rng = np.random.default_rng(seed)
    return rng.normal(0, 1, H).astype(np.float32), rng.normal(0, 1, E).astype(np.float32)


@pytest.mark.parametrize("norm", [True, False])
def test_routing_matches_restatement(plugin, port, norm):
    L = DevLayer(plugin, 256, 512, 256, 8, seed=5, norm=norm)
    ids, w = empty(8, "int32"), empty(8)
    rng = np.random.default_rng(6)
    for _ in range(25):
        logits = rng.normal(0, 1, 256).astype(np.float32)
        L.layer.route(dev(logits), ids, w)
        eids, ew = port.route(logits, 8, norm=norm)
        assert host(ids).tolist() == eids.tolist()
        assert np.array_equal(host(w), ew)


def test_routing_edge_cases(plugin, port):
    L = DevLayer(plugin, 64, 512, 256, 5, seed=7)
    ids, w = empty(5, "int32"), empty(5)
    cases = [np.zeros(64, np.float32), np.full(64, -1.0, np.float32)]
    lg = np.full(64, -1.0, np.float32)
    lg[[5, 9, 40]] = 2.0
    lg[3] = np.nan
    lg[7], lg[8] = -0.0, 0.0
    cases.append(lg)
    cases.append(np.arange(64, dtype=np.float32)[::-1].copy())
    for c in cases:
        L.layer.route(dev(c), ids, w)
        eids, ew = port.route(c, 5)
        assert host(ids).tolist() == eids.tolist()
        assert np.array_equal(host(w), ew)


def test_routing_1024_experts_top16(plugin, port):
    L = DevLayer(plugin, 1024, 256, 256, 16, seed=8)
    ids, w = empty(16, "int32"), empty(16)
    logits = np.random.default_rng(9).normal(0, 1, 1024).astype(np.float32)
    L.layer.route(dev(logits), ids, w)
    eids, ew = port.route(logits, 16)
    assert host(ids).tolist() == eids.tolist() and np.array_equal(host(w), ew)


def test_moe_q8_vs_restatement(c2_small, port):
    for s in range(6):
        x, logits = rand_inputs(100 + s, 2048, 32)
        y = c2_small.run(x, logits, MOE_Q8_1)
        want, _, _, _ = port.moe_layer(c2_small.host, x, logits, mode=0)
        assert rel_l2(y, want) <= 1e-5
        assert np.mean(y == want) >= 0.999


def test_moe_f32_vs_reference_kernels(c2_small, ref):
    for s in range(3):
        x, logits = rand_inputs(200 + s, 2048, 32)
        y = c2_small.run(x, logits, MOE_F32)
        want, _, _ = ref.moe_layer(c2_small.host, x, logits)
        assert rel_l2(y, want) <= 1e-5


def test_moe_f32_vs_golden(plugin, port, golden):
    layer, x, logits = moe_inputs(port)
    c = MOE_CASE
    L = DevLayer(plugin, c["n_experts"], c["hidden"], c["ffn"], c["top_k"], 0, from_host=layer)
    y = L.run(x, logits, MOE_F32)
    assert rel_l2(y, golden["moe_small/y"]) <= 1e-5
    yq = L.run(x, logits, MOE_Q8_1)
    want, _, _, _ = port.moe_layer(layer, x, logits, mode=0)
    assert rel_l2(yq, want) <= 1e-5


def test_moe_routed_equals_routing(c2_small, port):
    x, logits = rand_inputs(300, 2048, 32)
    ids, w = port.route(logits, 8)
    y1 = c2_small.run(x, logits)
    y2 = empty(2048)
    c2_small.layer.forward_routed(dev(x), dev(ids), dev(w), y2)
    assert np.array_equal(y1, host(y2))


def test_moe_deterministic_and_rearmed(c2_small):
    inputs = [rand_inputs(400 + s, 2048, 32) for s in range(4)]
    first = [c2_small.run(x, lg) for x, lg in inputs]
    for rep in range(5):
        for (x, lg), y0 in zip(inputs, first):
            assert np.array_equal(c2_small.run(x, lg), y0)


def test_moe_full_c2_shape(plugin, port):
    L = DevLayer(plugin, 256, 2048, 512, 8, seed=31)
    x, logits = rand_inputs(500, 2048, 256)
    y = L.run(x, logits)
    want, _, _, _ = port.moe_layer(L.host, x, logits, mode=0)
    assert rel_l2(y, want) <= 1e-5


def test_moe_top1_no_norm(plugin, port):
    L = DevLayer(plugin, 16, 1024, 512, 1, seed=41, norm=False)
    x, logits = rand_inputs(600, 1024, 16)
    y = L.run(x, logits)
    want, _, _, _ = port.moe_layer(L.host, x, logits, mode=0)
    assert rel_l2(y, want) <= 1e-5


def test_moe_set_expert_swaps_weights(plugin, port):
    L = DevLayer(plugin, 16, 512, 256, 2, seed=51)
    x, logits = rand_inputs(700, 512, 16)
    ids, _ = port.route(logits, 2)
    e0 = int(ids[0])
    other = make_moe_weights(port, 1, 512, 256, seed=52, top_k=2)
    g, u, d = dev(other.gate), dev(other.up), dev(other.down)
    L.layer.set_expert(e0, g.data_ptr(), u.data_ptr(), d.data_ptr())
    swapped = MoeWeights(L.host.gate.copy(), L.host.up.copy(), L.host.down.copy(), 512, 256, 2)
    swapped.gate[e0], swapped.up[e0], swapped.down[e0] = other.gate[0], other.up[0], other.down[0]
    y = L.run(x, logits)
    want, _, _, _ = port.moe_layer(swapped, x, logits, mode=0)
    assert rel_l2(y, want) <= 1e-5

"""CPU tests of the oracle: the C restatement against the reference's own kernels
(live, compiled from its checkout) and against the committed golden fixtures."""
import hashlib

import numpy as np
import pytest

from oracle.oracle import Q4_K, Q6_K, Q8_1, rel_l2, row_bytes
from tests.golden.make_golden import MATVEC_CASES, MOE_CASE, matvec_inputs, moe_inputs, \
    random_blocks


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# -- reference self-tests and golden vectors --------------------------------
def test_reference_selftests_recorded_pass(golden):
    assert golden["selftests"].tolist() == [0, 0]


def test_reference_selftests_live(ref):
    assert ref.L.katali_dtype_selftest() == 0
    assert ref.L.katali_dtype_simd_selftest() == 0


@pytest.mark.parametrize("name,qt", [("q4k_blocks", Q4_K), ("q6k_blocks", Q6_K)])
def test_dequant_bit_exact_vs_golden(port, golden, name, qt):
    got = port.dequant(qt, golden[f"{name}/bytes"], 16 * 256)
    assert np.array_equal(got.view(np.uint32), golden[f"{name}/dequant"].view(np.uint32))


@pytest.mark.parametrize("qt", [Q4_K, Q6_K])
@pytest.mark.parametrize("seed", range(5))
def test_dequant_bit_exact_vs_reference_live(port, ref, qt, seed):
    blob = random_blocks(qt, 64, 1000 + seed)
    a = port.dequant(qt, blob, 64 * 256)
    b = ref.dequant(qt, blob, 64 * 256)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("name", list(MATVEC_CASES))
def test_matvec_f32_vs_golden(port, golden, name):
    qt, rows, cols, seed = MATVEC_CASES[name]
    w, x = matvec_inputs(port, qt, rows, cols, seed)
    assert sha(w) == str(golden[f"{name}/w_sha"]), "input regeneration changed"
    y = port.matvec_f32(qt, w, rows, cols, x)
    assert rel_l2(y, golden[f"{name}/y"]) <= 1e-5
    assert rel_l2(y, golden[f"{name}/y_vec_dot_ref"]) <= 1e-6


# -- formats ------------------------------------------------------------------
def test_f16_rne_matches_ieee(port):
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.normal(0, s, 4000) for s in (1e-6, 1e-3, 1, 1e3, 3e4)]
                          + [np.array([0.0, -0.0, 65504, 65519.99, 65520, 6e-8, 2.98e-8, 1e-9,
                                       np.inf, -np.inf])]).astype(np.float32)
    got = np.array([port.f32_to_f16(float(v)) for v in vals], np.uint16)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_expf_accuracy(port):
    xs = np.linspace(-87, 88, 20001).astype(np.float32)
    e = np.array([port.expf(float(v)) for v in xs], np.float64)
    assert np.max(np.abs(e / np.exp(xs.astype(np.float64)) - 1)) < 3e-7
    assert port.expf(0.0) == 1.0
    assert port.expf(-1000.0) > 0 and np.isfinite(port.expf(1000.0))


@pytest.mark.parametrize("qt,tol", [(Q4_K, 0.1), (Q6_K, 0.025)])
def test_encoder_roundtrip_and_reference_decode(port, ref, qt, tol):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.02, (32, 512)).astype(np.float32)
    blob = port.quantize(qt, x)
    assert blob.shape == (32, row_bytes(qt, 512))
    dec = ref.dequant(qt, blob, x.size)
    assert rel_l2(dec, x.reshape(-1)) < tol
    assert np.array_equal(dec, port.dequant(qt, blob, x.size))


@pytest.mark.parametrize("qt", [Q4_K, Q6_K])
def test_encoder_edge_blocks(port, qt):
    zeros = np.zeros((1, 256), np.float32)
    assert np.all(port.dequant(qt, port.quantize(qt, zeros), 256) == 0)
    const = np.full((1, 256), 0.5, np.float32)
    assert rel_l2(port.dequant(qt, port.quantize(qt, const), 256), const.reshape(-1)) < 0.05
    big = np.random.default_rng(1).normal(0, 100, (2, 256)).astype(np.float32)
    assert rel_l2(port.dequant(qt, port.quantize(qt, big), 512), big.reshape(-1)) < 0.1


def test_q8_1_quantiser(port):
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.normal(0, 1, 256), np.zeros(32), np.full(32, -3.0)]).astype(np.float32)
    blob = port.quantize(Q8_1, x).reshape(-1, 36)
    q = blob[:, 4:].view(np.int8).astype(np.int32)
    assert q.min() >= -127 and q.max() <= 127
    d = blob[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    xb = x.reshape(-1, 32)
    amax = np.abs(xb).max(1)
    assert np.all(np.abs(q).max(1)[amax > 0] == 127)
    assert np.all(q[amax == 0] == 0)
    err = np.abs(q * d[:, None] - xb)
    assert np.all(err <= (amax / 127 * 0.5 + amax * 1e-3)[:, None] + 1e-12)


def _unpack_q4k(row, cols):
    """numpy decode of Q4_K nibbles, independent of the C code."""
    nb = cols // 256
    blk = row.reshape(nb, 144)
    qs = blk[:, 16:].reshape(nb, 4, 32)
    lo, hi = qs & 15, qs >> 4
    return np.stack([lo, hi], axis=2).reshape(nb * 8, 32).astype(np.int32)


def test_q4k_isums_independent(port):
    rng = np.random.default_rng(3)
    cols = 1024
    w = port.quantize(Q4_K, rng.normal(0, 0.02, (1, cols)).astype(np.float32)).reshape(-1)
    xq = port.quantize(Q8_1, rng.normal(0, 1, cols).astype(np.float32))
    isum, xsum = port.row_isums(Q4_K, w, xq, cols)
    qx = xq.reshape(-1, 36)[:, 4:].view(np.int8).astype(np.int32)
    q4 = _unpack_q4k(w, cols)
    assert np.array_equal(isum, (q4 * qx).sum(1))
    assert np.array_equal(xsum, qx.sum(1))


def test_q6k_isums_independent(port):
    rng = np.random.default_rng(4)
    cols = 512
    xw = rng.normal(0, 0.02, (1, cols)).astype(np.float32)
    w = port.quantize(Q6_K, xw).reshape(-1)
    xq = port.quantize(Q8_1, rng.normal(0, 1, cols).astype(np.float32))
    isum, _ = port.row_isums(Q6_K, w, xq, cols)
    # decode q-32 through d*sc*(q-32) = dequant: q-32 = dequant / (d*sc)
    deq = port.dequant(Q6_K, w, cols).reshape(-1, 16)
    blk = w.reshape(-1, 210)
    d = blk[:, 208:210].copy().view(np.float16).astype(np.float32).reshape(-1, 1)
    sc = blk[:, 192:208].view(np.int8).astype(np.float32).reshape(-1, 16)
    scale = (d * sc).reshape(-1, 1)
    q = np.where(scale != 0, np.rint(deq / np.where(scale == 0, 1, scale)), 0).astype(np.int32)
    qx = xq.reshape(-1, 36)[:, 4:].view(np.int8).astype(np.int32).reshape(-1, 16)
    nz = scale.reshape(-1) != 0
    assert np.array_equal(isum[nz], (q * qx).sum(1)[nz])


@pytest.mark.parametrize("qt,cols", [(Q4_K, 2048), (Q6_K, 512), (Q6_K, 4096)])
def test_dot_q8_equals_f32_dot_of_dequantised_activations(port, ref, qt, cols):
    rng = np.random.default_rng(6)
    rows = 16
    w = port.quantize(qt, rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    xq = port.quantize(Q8_1, rng.normal(0, 1, cols).astype(np.float32))
    y = port.matvec_q8(qt, w, rows, cols, xq)
    y_ref = ref.matvec(qt, w, rows, cols, port.dequant(Q8_1, xq, cols), n_threads=1)
    assert rel_l2(y, y_ref) < 1e-6


# -- routing ------------------------------------------------------------------
def test_route_topk_matches_numpy(port):
    rng = np.random.default_rng(7)
    for _ in range(20):
        logits = rng.normal(0, 1, 256).astype(np.float32)
        ids, w = port.route(logits, 8, norm=True)
        assert ids.tolist() == np.argsort(-logits, kind="stable")[:8].tolist()
        e = np.exp(logits[ids].astype(np.float64) - logits[ids[0]])
        assert np.allclose(w, e / e.sum(), rtol=1e-6)
        ids2, w2 = port.route(logits, 8, norm=False)
        p = np.exp(logits.astype(np.float64) - logits.max())
        assert np.array_equal(ids, ids2) and np.allclose(w2, p[ids] / p.sum(), rtol=1e-6)


def test_route_ties_and_nan(port):
    ids, w = port.route(np.zeros(256, np.float32), 8)
    assert ids.tolist() == list(range(8)) and np.allclose(w, 1 / 8)
    lg = np.full(64, -1.0, np.float32)
    lg[[5, 9, 40]] = 2.0
    lg[3] = np.nan
    lg[7] = -0.0
    lg[8] = 0.0
    ids, _ = port.route(lg, 5)
    assert ids.tolist() == [5, 9, 40, 7, 8]
    ids, w = port.route(np.array([1.0], np.float32), 1)
    assert ids.tolist() == [0] and w[0] == 1.0


# -- MoE layer ----------------------------------------------------------------
def test_moe_f32_vs_golden(port, golden):
    layer, x, logits = moe_inputs(port)
    wsha = sha(np.concatenate([layer.gate.reshape(-1), layer.up.reshape(-1), layer.down.reshape(-1)]))
    assert wsha == str(golden["moe_small/w_sha"])
    y, ids, w, _ = port.moe_layer(layer, x, logits, mode=1)
    assert ids.tolist() == golden["moe_small/ids"].tolist()
    assert np.allclose(w, golden["moe_small/w"], rtol=1e-6)
    assert rel_l2(y, golden["moe_small/y"]) <= 1e-5


def test_moe_q8_vs_reference_composition(port, ref):
    layer, x, logits = moe_inputs(port)
    yq, ids, _, _ = port.moe_layer(layer, x, logits, mode=0)
    yr, idr, _ = ref.moe_layer(layer, x, logits, n_threads=2)
    assert ids.tolist() == idr.tolist()
    assert rel_l2(yq, yr) < 3e-2  # q8_1 activation rounding of x and h


def test_moe_routed_equals_routing(port):
    layer, x, logits = moe_inputs(port)
    y, ids, w, h = port.moe_layer(layer, x, logits, mode=0)
    y2, _, _, h2 = port.moe_layer(layer, x, None, mode=0, ids=ids, w=w)
    assert np.array_equal(y, y2) and np.array_equal(h, h2)


def test_argmax_first_strict_max(port):
    assert port.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert port.argmax(np.array([-5, -5], np.float32)) == 0

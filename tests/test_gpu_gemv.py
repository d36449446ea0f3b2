"""GPU parity of the dense GEMV family, the q8_1 quantiser and the block encoders,
all called through the plugin's C ABI.

Bars: fp32-activation GEMV within rel_L2 <= 1e-5 of the reference's own CPU
kernels (katali_ggml_matvec); integer in-block sums bit-exact against the C
restatement; q8_1-activation rows equal to the restatement (same exact per-block
terms, double accumulation) within 1e-6; encoder bytes identical."""
import numpy as np
import pytest

from katali_lab_b200 import Q4_K, Q6_K, Q8_1, KataliError
from katali_lab_b200.synth import make_dense
from oracle.oracle import rel_l2, row_bytes
from tests.golden.make_golden import MATVEC_CASES, matvec_inputs

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def empty(n, dtype="float32"):
    import torch
    return torch.empty(n, dtype=getattr(torch, dtype), device="cuda")


@pytest.mark.parametrize("qt", [Q4_K, Q6_K, Q8_1])
def test_device_encoder_bytes_equal_oracle(plugin, port, qt):
    rng = np.random.default_rng(0)
    rows, cols = 64, 512
    x = np.concatenate([rng.normal(0, 0.02, (rows - 5, cols)), np.zeros((1, cols)),
                        np.full((1, cols), 0.25), rng.normal(0, 50, (2, cols)),
                        rng.normal(0, 1e-6, (1, cols))]).astype(np.float32)
    want = port.quantize(qt, x).reshape(-1)
    out = empty(want.size, "uint8")
    plugin.quantize_rows(qt, dev(x), rows, cols, out)
    assert np.array_equal(host(out), want)


def test_quantize_q8_1_entry_point(plugin, port):
    x = np.random.default_rng(1).normal(0, 3, 4096).astype(np.float32)
    out = empty(4096 // 32 * 36, "uint8")
    plugin.quantize_q8_1(dev(x), 4096, out)
    assert np.array_equal(host(out), port.quantize(Q8_1, x))


@pytest.mark.parametrize("qt,cols", [(Q4_K, 2048), (Q4_K, 4096), (Q4_K, 256), (Q6_K, 512),
                                     (Q6_K, 4096), (Q6_K, 768)])
def test_row_isums_bit_exact(plugin, port, qt, cols):
    rng = np.random.default_rng(2)
    rows = 37
    w = port.quantize(qt, rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    xq = port.quantize(Q8_1, rng.normal(0, 1, cols).astype(np.float32))
    ng = cols // (32 if qt == Q4_K else 16)
    isum, xsum = empty(rows * ng, "int32"), empty(rows * ng, "int32")
    plugin.row_isums(qt, dev(w), rows, cols, dev(xq), isum, xsum)
    gi, gx = host(isum).reshape(rows, ng), host(xsum).reshape(rows, ng)
    for r in range(rows):
        ei, ex = port.row_isums(qt, w[r], xq, cols)
        assert np.array_equal(gi[r], ei)
        assert np.array_equal(gx[r], ex)


@pytest.mark.parametrize("name", list(MATVEC_CASES))
def test_matvec_f32_vs_reference_golden(plugin, port, golden, name):
    qt, rows, cols, seed = MATVEC_CASES[name]
    w, x = matvec_inputs(port, qt, rows, cols, seed)
    y = empty(rows)
    plugin.matvec(qt, dev(w), rows, cols, dev(x), y)
    assert rel_l2(host(y), golden[f"{name}/y"]) <= 1e-5


def test_matvec_c1_shape_vs_reference(plugin, ref):
    import torch
    rows, cols = 6144, 2048
    w = make_dense(plugin, Q4_K, rows, cols, seed=0)
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(cols, generator=g, device="cuda")
    y = empty(rows)
    plugin.matvec(Q4_K, w, rows, cols, x, y)
    y_ref = ref.matvec(Q4_K, host(w), rows, cols, host(x))
    assert rel_l2(host(y), y_ref) <= 1e-5


@pytest.mark.parametrize("qt,rows,cols", [(Q4_K, 6144, 2048), (Q4_K, 1, 2048), (Q4_K, 13, 4096),
                                          (Q6_K, 2048, 512), (Q6_K, 5, 512), (Q6_K, 1001, 768),
                                          (Q6_K, 300, 4096), (Q4_K, 64, 12288)])
def test_matvec_q8_vs_oracle(plugin, port, qt, rows, cols):
    rng = np.random.default_rng(rows + cols)
    w = port.quantize(qt, rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    xq = port.quantize(Q8_1, rng.normal(0, 1, cols).astype(np.float32))
    y = empty(rows)
    plugin.matvec_q8_1(qt, dev(w), rows, cols, dev(xq), y)
    want = port.matvec_q8(qt, w, rows, cols, xq)
    got = host(y)
    assert rel_l2(got, want) <= 1e-6
    assert np.mean(got == want) >= 0.999


@pytest.mark.parametrize("qt,rows,cols", [(Q4_K, 777, 2048), (Q6_K, 130, 4096), (Q6_K, 3, 512)])
def test_matvec_f32_vs_reference_ragged(plugin, ref, port, qt, rows, cols):
    rng = np.random.default_rng(rows)
    w = port.quantize(qt, rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    x = rng.normal(0, 1, cols).astype(np.float32)
    y = empty(rows)
    plugin.matvec(qt, dev(w), rows, cols, dev(x), y)
    assert rel_l2(host(y), ref.matvec(qt, w, rows, cols, x)) <= 1e-5


def test_matvec_dp4a_switch(plugin, port, monkeypatch):
    rng = np.random.default_rng(9)
    rows, cols = 256, 2048
    w = port.quantize(Q4_K, rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    x = rng.normal(0, 1, cols).astype(np.float32)
    monkeypatch.setenv("KATALI_CUDA_DP4A", "1")
    y = empty(rows)
    plugin.matvec(Q4_K, dev(w), rows, cols, dev(x), y)
    want = port.matvec_q8(Q4_K, w, rows, cols, port.quantize(Q8_1, x))
    assert rel_l2(host(y), want) <= 1e-6


def test_matvec_multi_bit_identical_to_single(plugin, port):
    rng = np.random.default_rng(4)
    cols = 2048
    specs = [(Q4_K, 100), (Q6_K, 37), (Q4_K, 8), (Q6_K, 512)]
    ws = [dev(port.quantize(qt, rng.normal(0, 0.02, (r, cols)).astype(np.float32))) for qt, r in specs]
    x = dev(rng.normal(0, 1, cols).astype(np.float32))
    ys = [empty(r) for _, r in specs]
    plugin.matvec_multi([qt for qt, _ in specs], ws, [r for _, r in specs], cols, x, ys)
    for (qt, r), w, y in zip(specs, ws, ys):
        y1 = empty(r)
        plugin.matvec(qt, w, r, cols, x, y1)
        assert np.array_equal(host(y), host(y1))


def test_lm_head_sized_q6k(plugin, ref):
    import torch
    rows, cols = 32768, 4096
    w = make_dense(plugin, Q6_K, rows, cols, seed=3)
    x = torch.randn(cols, generator=torch.Generator(device="cuda").manual_seed(4), device="cuda")
    y = empty(rows)
    plugin.matvec(Q6_K, w, rows, cols, x, y)
    assert rel_l2(host(y), ref.matvec(Q6_K, host(w), rows, cols, host(x))) <= 1e-5


def test_argument_errors(plugin):
    import torch
    w = torch.zeros(144 * 8 + 16, dtype=torch.uint8, device="cuda")
    x, y = empty(2048), empty(8)
    with pytest.raises(KataliError) as e:
        plugin.matvec(Q4_K, w.data_ptr() + 4, 1, 2048, x, y)  # misaligned weights
    assert e.value.code == 3
    with pytest.raises(KataliError) as e:
        plugin.matvec(2, w, 1, 2048, x, y)
    assert e.value.code == 4
    with pytest.raises(KataliError) as e:
        plugin.matvec(Q4_K, w, 1, 100, x, y)
    assert e.value.code == 5

"""GPU tests of the expert residency tier (katali_cuda_expert_*).

Experts live in host memory (numpy, the stand-in for an mmap'd GGUF file) and are
uploaded into device slots on the cache's side stream. Bars: a layer whose
selected experts are bound through the cache gives bit-identical output to the
same layer fully resident (same kernel, same bytes); slot contents equal the host
bytes; a call that selects an unbound or evicted expert returns
KATALI_ERR_NOT_RESIDENT (9) and later calls still work; slots are reused least
recently used first."""
import numpy as np
import pytest

from katali_lab_b200 import MOE_Q8_1, ExpertCache, KataliError, MoeLayer
from tests.test_gpu_moe import DevLayer, dev, empty, host

pytestmark = pytest.mark.gpu

E, H, F, K = 32, 2048, 512, 8


@pytest.fixture(scope="module")
def full(plugin):
    return DevLayer(plugin, E, H, F, K, seed=71)


def slot_bytes(full):
    w = full.host
    a16 = lambda n: (n + 15) // 16 * 16
    return a16(w.gate.shape[1]) + a16(w.up.shape[1]) + a16(w.down.shape[1])


def make_cache(plugin, full, n_slots):
    c = ExpertCache(plugin, slot_bytes(full), n_slots)
    for e in range(E):
        c.register(e, full.host.gate[e], full.host.up[e], full.host.down[e])
    return c


def empty_layer(plugin):
    return MoeLayer(plugin, E, H, F, K, [(0, 0, 0)] * E)


def inputs(seed):
    rng = np.random.default_rng(seed)
    return rng.normal(0, 1, H).astype(np.float32), rng.normal(0, 1, E).astype(np.float32)


def run(layer, x, lg):
    y = empty(H)
    layer.forward(dev(x), dev(lg), y, MOE_Q8_1)
    return host(y)


def test_bound_experts_match_resident_layer(plugin, port, full):
    cache = make_cache(plugin, full, n_slots=12)
    layer = empty_layer(plugin)
    for s in range(4):
        x, lg = inputs(900 + s)
        ids, _ = port.route(lg, K)
        for e in ids:
            cache.bind(int(e), layer, int(e))
        assert np.array_equal(run(layer, x, lg), full.run(x, lg, MOE_Q8_1))
    cache.sync()
    e = int(ids[0])
    g, u, d = cache.lookup(e)
    buf = np.empty(full.host.down.shape[1], np.uint8)
    plugin.check(plugin.L.katali_cuda_download(buf.ctypes.data, d, buf.nbytes))
    assert np.array_equal(buf, full.host.down[e])
    layer.close()
    cache.close()


def test_not_resident_is_reported(plugin, port, full):
    cache = make_cache(plugin, full, n_slots=8)
    layer = empty_layer(plugin)
    x, lg = inputs(910)
    with pytest.raises(KataliError) as err:
        run(layer, x, lg)
    assert err.value.code == 9
    ids, _ = port.route(lg, K)
    for e in ids[:-1]:
        cache.bind(int(e), layer, int(e))
    with pytest.raises(KataliError) as err:  # one selected expert still missing
        run(layer, x, lg)
    assert err.value.code == 9
    cache.bind(int(ids[-1]), layer, int(ids[-1]))
    assert np.array_equal(run(layer, x, lg), full.run(x, lg, MOE_Q8_1))
    layer.close()
    cache.close()


def test_lru_reuse_and_eviction_unbinds(plugin, port, full):
    cache = make_cache(plugin, full, n_slots=3)
    for k in (0, 1, 2):
        cache.prefetch(k)
    cache.prefetch(3)  # evicts 0, the least recently used
    assert cache.lookup(0) is None and cache.lookup(3) is not None
    cache.prefetch(1)  # 1 is used again
    cache.prefetch(4)  # evicts 2
    assert cache.lookup(2) is None and cache.lookup(1) is not None
    # a bound expert whose slot is refilled becomes not resident
    x, lg = inputs(920)
    ids, _ = port.route(lg, K)
    layer = empty_layer(plugin)
    big = make_cache(plugin, full, n_slots=K)
    for e in ids:
        big.bind(int(e), layer, int(e))
    assert np.array_equal(run(layer, x, lg), full.run(x, lg, MOE_Q8_1))
    big.evict(int(ids[3]))
    with pytest.raises(KataliError) as err:
        run(layer, x, lg)
    assert err.value.code == 9
    big.bind(int(ids[3]), layer, int(ids[3]))
    assert np.array_equal(run(layer, x, lg), full.run(x, lg, MOE_Q8_1))
    layer.close()
    big.close()
    cache.close()


def test_batch_path_through_cache(plugin, port, full):
    cache = make_cache(plugin, full, n_slots=E)
    layer = empty_layer(plugin)
    rng = np.random.default_rng(930)
    T = 9
    X = rng.normal(0, 1, (T, H)).astype(np.float32)
    L = rng.normal(0, 1, (T, E)).astype(np.float32)
    sel = sorted({int(e) for t in range(T) for e in port.route(L[t], K)[0]})
    for e in sel:
        cache.bind(e, layer, e)
    y = empty(T * H).view(T, H)
    want = empty(T * H).view(T, H)
    layer.forward_batch(dev(X), dev(L), y)
    full.layer.forward_batch(dev(X), dev(L), want)
    assert np.array_equal(host(y), host(want))
    layer.close()
    cache.close()


def test_destroying_cache_leaves_layer_not_resident(plugin, port, full):
    cache = make_cache(plugin, full, n_slots=K)
    layer = empty_layer(plugin)
    x, lg = inputs(940)
    for e in port.route(lg, K)[0]:
        cache.bind(int(e), layer, int(e))
    cache.close()
    with pytest.raises(KataliError) as err:
        run(layer, x, lg)
    assert err.value.code == 9
    layer.close()

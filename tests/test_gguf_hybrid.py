"""CPU tests of the hybrid MoE decoder's GGUF loader (katali_cuda_hybrid_create_from_gguf):
a complete qwen35moe file parses all the way to the device step (KATALI_ERR_NO_DEVICE here),
a missing tensor names itself (KATALI_ERR_BAD_ARG), and what the decoder does not run is
refused before any device work: shared experts, another architecture, a wrong expert shape."""
import ctypes as C

import pytest

from katali_lab_b200 import Gguf, Plugin
from katali_lab_b200.synth import HybridConfig
from tests.gguf_files import build, hybrid_model_file, sample_file

TINY = HybridConfig(n_layers=2, hidden=256, vocab=512, kv_cap=32, n_heads=2, n_kv_heads=1,
                    head_dim=128, rope_dim=64, ssm_k_heads=1, ssm_v_heads=2, ssm_head_dim=128,
                    ssm_conv=4, n_experts=4, ffn=256, top_k=2, attn_every=2)

OK, BAD_ARG, UNSUPPORTED_TYPE, UNSUPPORTED_SHAPE, NO_DEVICE = 0, 3, 4, 5, 1


@pytest.fixture(scope="module")
def lib():
    from katali_lab_b200.build import build as build_plugin
    build_plugin()
    return Plugin()


@pytest.fixture(scope="module")
def tiny(port):
    return hybrid_model_file(port, TINY, seed=3)


def _open(lib, tmp_path, data, name="m.gguf"):
    path = tmp_path / name
    path.write_bytes(data)
    return Gguf(lib, str(path))


def _create(lib, g):
    h = C.c_void_p()
    rc = lib.L.katali_cuda_hybrid_create_from_gguf(g.h, 32, 0, None, C.byref(h))
    return rc, lib.status()


def _rebuild(data, drop=(), add=(), arch=None, reshape=None):
    """The file again with tensors dropped / added / reshaped, or another architecture."""
    g_kv, g_t = _parse(data)
    kvs = [(k, t, (arch if (k == "general.architecture" and arch) else v)) for k, t, v in g_kv]
    ts = [t for t in g_t if t[0] not in drop]
    if reshape:
        ts = [(n, ty, reshape[n] if n in reshape else d, b) for n, ty, d, b in ts]
    return build(kvs, ts + list(add))[0]


def _parse(data):
    """(kvs, tensors) of a file written by tests.gguf_files.build (scalars, strings, string
    arrays; version 3, alignment 32)."""
    import struct
    from tests import gguf_files as gf
    at = 24
    n_t, n_kv = struct.unpack_from("<QQ", data, 8)

    def s():
        nonlocal at
        n, = struct.unpack_from("<Q", data, at)
        v = data[at + 8:at + 8 + n].decode()
        at += 8 + n
        return v

    def val(t):
        nonlocal at
        if t == gf.STR:
            return s()
        if t == gf.ARR:
            et, n = struct.unpack_from("<IQ", data, at)
            at += 12
            return (et, [val(et) for _ in range(n)])
        fmt = {gf.U32: "<I", gf.F32: "<f", gf.U8: "<B", gf.BOOL: "<B"}[t]
        v, = struct.unpack_from(fmt, data, at)
        at += struct.calcsize(fmt)
        return v

    kvs = []
    for _ in range(n_kv):
        k = s()
        t, = struct.unpack_from("<I", data, at)
        at += 4
        kvs.append((k, t, val(t)))
    infos = []
    for _ in range(n_t):
        name = s()
        nd, = struct.unpack_from("<I", data, at)
        dims = struct.unpack_from(f"<{nd}Q", data, at + 4)
        ty, rel = struct.unpack_from("<IQ", data, at + 4 + 8 * nd)
        at += 4 + 8 * nd + 12
        infos.append((name, ty, dims, rel))
    base = (at + 31) // 32 * 32
    rels = sorted(r for _, _, _, r in infos) + [len(data) - base]
    ts = []
    for name, ty, dims, rel in infos:
        nxt = min(r for r in rels if r > rel) if any(r > rel for r in rels) else len(data) - base
        ts.append((name, ty, dims, data[base + rel: base + nxt]))
    return kvs, ts


def test_complete_file_reaches_the_device(lib, tiny, tmp_path):
    data, _ = tiny
    g = _open(lib, tmp_path, data)
    rc, why = _create(lib, g)
    g.close()
    assert rc == NO_DEVICE, why  # every tensor and key found; no GPU in this container


def test_missing_tensor_is_named(lib, tiny, tmp_path):
    data, _ = tiny
    g = _open(lib, tmp_path, _rebuild(data, drop=("blk.1.ffn_down_exps.weight",)))
    rc, why = _create(lib, g)
    g.close()
    assert rc == BAD_ARG and "blk.1.ffn_down_exps.weight" in why


def test_refusals(lib, tiny, tmp_path):
    data, _ = tiny
    shexp = ("blk.0.ffn_gate_shexp.weight", 0, (4,), b"\0" * 16)
    for blob, want, word in ((_rebuild(data, add=(shexp,)), UNSUPPORTED_SHAPE, "shared"),
                             (_rebuild(data, arch="qwen3"), UNSUPPORTED_SHAPE, "qwen35moe"),
                             (_rebuild(data, reshape={"blk.0.ffn_up_exps.weight": (256, 256, 3)}),
                              UNSUPPORTED_TYPE, "ffn_up_exps"),
                             (sample_file()[0], UNSUPPORTED_SHAPE, "qwen35moe")):
        g = _open(lib, tmp_path, blob)
        rc, why = _create(lib, g)
        g.close()
        assert rc == want and word in why, (rc, why)

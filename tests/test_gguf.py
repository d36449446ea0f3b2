"""CPU tests of the plugin's GGUF reader (katali_cuda_gguf_*, no GPU needed) against the
reference's own reader (V/src/gguf_reader.c compiled into the oracle) on the same files:
the tensor directory (names, types, dims, absolute data offsets, byte sizes), metadata of
every value type, custom alignment, GGUF v2, an unknown tensor type (parsed, not sized),
and the malformed files both must reject (the reference's parser tests, test_core.c:
184-283: bad magic, bad version, truncation, out-of-range tensor offset, nested array)."""
import ctypes as C

import pytest

from katali_lab_b200 import Gguf, KataliError, Plugin
from tests.gguf_files import malformed, sample_file


@pytest.fixture(scope="module")
def lib():
    from katali_lab_b200.build import build
    build()
    return Plugin()


class RefReader:
    def __init__(self, ref, path):
        L = ref.L
        L.kref_gguf_open.restype = C.c_void_p
        L.kref_gguf_open.argtypes = [C.c_char_p, C.c_char_p, C.c_int]
        L.kref_gguf_close.argtypes = [C.c_void_p]
        L.kref_gguf_counts.argtypes = [C.c_void_p, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                       C.POINTER(C.c_uint32)]
        L.kref_gguf_tensor.argtypes = [C.c_void_p, C.c_uint64, C.POINTER(C.c_char_p),
                                       C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                       C.POINTER(C.c_uint64), C.POINTER(C.c_uint64),
                                       C.POINTER(C.c_uint64)]
        L.kref_gguf_get_int.restype = C.c_int64
        L.kref_gguf_get_int.argtypes = [C.c_void_p, C.c_char_p, C.c_int64]
        L.kref_gguf_get_float.restype = C.c_double
        L.kref_gguf_get_float.argtypes = [C.c_void_p, C.c_char_p, C.c_double]
        L.kref_gguf_get_str.restype = C.c_void_p
        L.kref_gguf_get_str.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_size_t)]
        L.kref_gguf_array_len.restype = C.c_int64
        L.kref_gguf_array_len.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32)]
        L.kref_gguf_array_int.restype = C.c_int64
        L.kref_gguf_array_int.argtypes = [C.c_void_p, C.c_char_p, C.c_uint64]
        self.L = L
        err = C.create_string_buffer(256)
        self.h = L.kref_gguf_open(str(path).encode(), err, 256)
        self.err = err.value.decode()

    def counts(self):
        nt, nkv, v = C.c_uint64(), C.c_uint64(), C.c_uint32()
        self.L.kref_gguf_counts(self.h, C.byref(nt), C.byref(nkv), C.byref(v))
        return nt.value, nkv.value, v.value

    def tensor(self, i):
        name, t, nd = C.c_char_p(), C.c_uint32(), C.c_uint32()
        dims, off, nb = (C.c_uint64 * 4)(), C.c_uint64(), C.c_uint64()
        assert self.L.kref_gguf_tensor(self.h, i, C.byref(name), C.byref(t), C.byref(nd), dims,
                                       C.byref(off), C.byref(nb)) == 0
        return {"name": name.value.decode(), "type": t.value, "n_dims": nd.value,
                "dims": tuple(dims[:nd.value]), "offset": off.value, "nbytes": nb.value}

    def close(self):
        if self.h:
            self.L.kref_gguf_close(self.h)
            self.h = None


@pytest.mark.parametrize("alignment,version", [(None, 3), (64, 3), (None, 2)])
def test_directory_matches_reference(lib, ref, tmp_path, alignment, version):
    data, offsets = sample_file(alignment=alignment, version=version)
    path = tmp_path / "m.gguf"
    path.write_bytes(data)
    g, r = Gguf(lib, str(path)), RefReader(ref, path)
    assert r.h, r.err
    assert (g.n_tensors, g.n_kv, g.version) == r.counts()
    for i in range(g.n_tensors):
        mine, theirs = g.tensor(i), r.tensor(i)
        assert {k: mine[k] for k in ("name", "type", "n_dims", "dims")} == \
               {k: theirs[k] for k in ("name", "type", "n_dims", "dims")}
        if theirs["nbytes"]:  # a type both readers size: same bytes at the same place
            assert mine["nbytes"] == theirs["nbytes"]
            assert mine["offset"] == theirs["offset"] == offsets[mine["name"]]
            assert data[mine["offset"]:mine["offset"] + mine["nbytes"]] == \
                data[theirs["offset"]:theirs["offset"] + theirs["nbytes"]]
    assert g.find("q6k.weight") == [t["name"] for t in g.tensors()].index("q6k.weight")
    assert g.find("missing") is None
    # the unknown type parses and is not uploadable (both readers: no byte size)
    odd = g.tensor(g.find("odd.weight"))
    assert odd["nbytes"] == 0 and r.tensor(g.find("odd.weight"))["nbytes"] == 0
    g.close()
    r.close()


def test_metadata_matches_reference(lib, ref, tmp_path):
    data, _ = sample_file()
    path = tmp_path / "m.gguf"
    path.write_bytes(data)
    g, r = Gguf(lib, str(path)), RefReader(ref, path)
    L = r.L
    for key in ("qwen3.block_count", "general.flag", "t.u8", "t.i8", "t.u16", "t.i16", "t.i32",
                "t.u64", "t.i64"):
        assert g.get_int(key) == L.kref_gguf_get_int(r.h, key.encode(), -999), key
    for key in ("qwen3.rope.freq_base", "t.f64"):
        assert g.get_float(key) == L.kref_gguf_get_float(r.h, key.encode(), -1.0), key
    n = C.c_size_t()
    s = L.kref_gguf_get_str(r.h, b"general.architecture", C.byref(n))
    assert g.get_str("general.architecture") == C.string_at(s, n.value).decode() == "qwen3"
    et = C.c_uint32()
    assert g.array("tokenizer.ggml.tokens") == (8, L.kref_gguf_array_len(r.h, b"tokenizer.ggml.tokens", C.byref(et)))
    assert et.value == 8
    assert g.array("test.nums") == (5, 3)
    for i in range(3):
        assert g.array_int("test.nums", i) == L.kref_gguf_array_int(r.h, b"test.nums", i)
        assert g.array_int("test.u8s", i) == L.kref_gguf_array_int(r.h, b"test.u8s", i)
    # missing keys and type mismatches are errors, not defaults
    assert g.get_int("nope") is None and g.get_str("qwen3.block_count") is None
    assert g.get_int("general.architecture") is None and g.array_int("test.nums", 3) is None
    g.close()
    r.close()


@pytest.mark.parametrize("case", [c for c, _ in malformed()])
def test_malformed_rejected_by_both(lib, ref, tmp_path, case):
    data = dict(malformed())[case]
    path = tmp_path / "bad.gguf"
    path.write_bytes(data)
    with pytest.raises(KataliError) as e:
        Gguf(lib, str(path))
    assert e.value.code == 3
    r = RefReader(ref, path)
    assert not r.h, case


def test_missing_file(lib, tmp_path):
    with pytest.raises(KataliError):
        Gguf(lib, str(tmp_path / "absent.gguf"))


def _dense_file(tmp_path, drop=None, arch="qwen3"):
    from oracle.oracle import Port
    from katali_lab_b200.synth import DenseConfig
    from tests.gguf_files import STR, build, dense_model_file
    import struct
    cfg = DenseConfig(n_layers=2, hidden=256, ffn=512, n_heads=2, n_kv_heads=1, head_dim=128,
                      vocab=256, kv_cap=32)
    data, _ = dense_model_file(Port(), cfg, seed=1)
    g_path = tmp_path / "d.gguf"
    g_path.write_bytes(data)
    if drop is None and arch == "qwen3":
        return g_path
    # rebuild with one tensor renamed away or another architecture string
    L = Plugin()
    g = Gguf(L, str(g_path))
    tensors = []
    for t in g.tensors():
        name = t["name"] if t["name"] != drop else "unused.weight"
        tensors.append((name, t["type"], t["dims"], data[t["offset"]:t["offset"] + t["nbytes"]]))
    kvs = [("general.architecture", STR, arch)]
    for key in ("block_count", "embedding_length", "feed_forward_length", "attention.head_count",
                "attention.head_count_kv", "attention.key_length", "context_length"):
        kvs.append((f"{arch}.{key}", 4, g.get_int(f"qwen3.{key}")))
    g.close()
    out, _ = build(kvs, tensors)
    p = tmp_path / "bad.gguf"
    p.write_bytes(out)
    return p


@pytest.mark.parametrize("drop,arch,code", [("blk.1.ffn_up.weight", "qwen3", 3),
                                            (None, "llama", 5)])
def test_dense_from_gguf_rejects_before_any_gpu_work(lib, tmp_path, drop, arch, code):
    """A missing tensor or another architecture is reported from the file alone."""
    import ctypes as C2
    path = _dense_file(tmp_path, drop=drop, arch=arch)
    g = Gguf(lib, str(path))
    h = C2.c_void_p()
    rc = lib.L.katali_cuda_dense_create_from_gguf(g.h, 16, 0, C2.byref(h))
    assert rc == code
    if drop:
        assert drop in lib.status()
    g.close()

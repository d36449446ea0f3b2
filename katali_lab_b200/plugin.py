"""ctypes binding of libkatali_cuda.so for tests and the benchmark.

Every call goes through the plugin's C ABI (include/katali_cuda.h) exactly as
the reference engine's C code calls katali_cuda.dll. Device buffers are torch
CUDA tensors (torch is only used for device memory and streams here); the
binding passes their raw pointers. A missing library raises: there is no CPU
fallback in this package.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import os
import re

from . import build as _build

Q8_1, Q4_K, Q6_K = 9, 12, 14
MOE_Q8_1, MOE_F32 = 0, 1
MOE_NORM_TOPK = 1

HEADER = os.path.join(_build.INCLUDE, "katali_cuda.h")

_vp, _u32, _u64, _i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int


class KataliError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"katali_cuda error {code}: {msg}")
        self.code = code


class KataliDenseLayerW(C.Structure):
    _fields_ = [("attn_norm", _vp), ("ffn_norm", _vp), ("q_norm", _vp), ("k_norm", _vp),
                ("wq", _vp), ("wk", _vp), ("wv", _vp), ("wo", _vp), ("gate", _vp), ("up", _vp),
                ("down", _vp), ("wq_type", _u32), ("wk_type", _u32), ("wv_type", _u32),
                ("wo_type", _u32), ("gate_type", _u32), ("up_type", _u32), ("down_type", _u32)]


class KataliDenseDesc(C.Structure):
    _fields_ = [("n_layers", _u32), ("hidden", _u32), ("ffn", _u32), ("n_heads", _u32),
                ("n_kv_heads", _u32), ("head_dim", _u32), ("vocab", _u32), ("kv_cap", _u32),
                ("rope_dim", _u32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("embed", _vp), ("embed_type", _u32), ("out_norm", _vp), ("lm_head", _vp),
                ("lm_head_type", _u32), ("layers", C.POINTER(KataliDenseLayerW)),
                ("flags", _u32)]


class KataliHybridLayerW(C.Structure):
    _fields_ = [("kind", _u32), ("attn_norm", _vp), ("ffn_norm", _vp), ("router", _vp), ("moe", _vp),
                ("ssm_qkv", _vp), ("ssm_z", _vp), ("ssm_b", _vp), ("ssm_a", _vp), ("ssm_out", _vp),
                ("ssm_qkv_type", _u32), ("ssm_z_type", _u32), ("ssm_b_type", _u32),
                ("ssm_a_type", _u32), ("ssm_out_type", _u32), ("ssm_conv", _vp), ("ssm_a_log", _vp),
                ("ssm_dt_bias", _vp), ("ssm_norm", _vp), ("wq", _vp), ("wk", _vp), ("wv", _vp),
                ("wo", _vp), ("wq_type", _u32), ("wk_type", _u32), ("wv_type", _u32),
                ("wo_type", _u32), ("q_norm", _vp), ("k_norm", _vp), ("ssm_decay", _vp)]


class KataliHybridDesc(C.Structure):
    _fields_ = [("n_layers", _u32), ("hidden", _u32), ("vocab", _u32), ("kv_cap", _u32),
                ("n_heads", _u32), ("n_kv_heads", _u32), ("head_dim", _u32), ("rope_dim", _u32),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("ssm_k_heads", _u32),
                ("ssm_v_heads", _u32), ("ssm_head_dim", _u32), ("ssm_conv", _u32), ("embed", _vp),
                ("embed_type", _u32), ("out_norm", _vp), ("lm_head", _vp), ("lm_head_type", _u32),
                ("layers", C.POINTER(KataliHybridLayerW)), ("flags", _u32)]


class KataliGgufTensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", _u32), ("n_dims", _u32), ("dims", _u64 * 4),
                ("offset", _u64), ("nbytes", _u64)]


class KataliMoeDesc(C.Structure):
    _fields_ = [("n_experts", _u32), ("hidden", _u32), ("ffn", _u32), ("top_k", _u32),
                ("gate_type", _u32), ("up_type", _u32), ("down_type", _u32), ("flags", _u32),
                ("experts", C.POINTER(_vp))]


def header_symbols(path: str = HEADER) -> list[str]:
    """Every function the public header declares."""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(katali_cuda_\w+)\s*\(", src)))


def _ptr(t) -> int:
    """Device pointer of a torch tensor (or an int address)."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


class Plugin:
    def __init__(self, path: str | None = None):
        path = path or _build.PLUGIN
        if not os.path.exists(path):
            raise FileNotFoundError(
                f"{path} is missing; build it with `python -m katali_lab_b200.build`")
        self.path = path
        L = C.CDLL(path)
        self.L = L
        self.stream = None  # what set_stream last received (None: the plugin's own stream)
        sig = {
            "katali_cuda_probe": ([], _i32),
            "katali_cuda_status": ([], C.c_char_p),
            "katali_cuda_strerror": ([_i32], C.c_char_p),
            "katali_cuda_malloc": ([C.POINTER(_vp), C.c_size_t], _i32),
            "katali_cuda_free": ([_vp], _i32),
            "katali_cuda_upload": ([_vp, _vp, C.c_size_t], _i32),
            "katali_cuda_download": ([_vp, _vp, C.c_size_t], _i32),
            "katali_cuda_supports_type": ([_u32], _i32),
            "katali_cuda_matvec": ([_u32, _vp, _u64, _u64, _vp, _vp], _i32),
            "katali_cuda_set_stream": ([_vp], _i32),
            "katali_cuda_set_async": ([_i32], _i32),
            "katali_cuda_sync": ([], _i32),
            "katali_cuda_matvec_multi": ([_i32, C.POINTER(_u32), C.POINTER(_vp), C.POINTER(_u64),
                                          _u64, _vp, C.POINTER(_vp)], _i32),
            "katali_cuda_quantize_q8_1": ([_vp, _u64, _vp], _i32),
            "katali_cuda_matvec_q8_1": ([_u32, _vp, _u64, _u64, _vp, _vp], _i32),
            "katali_cuda_quantize_rows": ([_u32, _vp, _u64, _u64, _vp], _i32),
            "katali_cuda_moe_create": ([C.POINTER(KataliMoeDesc), C.POINTER(_vp)], _i32),
            "katali_cuda_moe_set_expert": ([_vp, _u32, _vp, _vp, _vp], _i32),
            "katali_cuda_moe_destroy": ([_vp], _i32),
            "katali_cuda_moe_layer": ([_vp, _vp, _vp, _vp, _u32], _i32),
            "katali_cuda_moe_layer_routed": ([_vp, _vp, _vp, _vp, _vp, _u32], _i32),
            "katali_cuda_moe_batch": ([_vp, _u32, _vp, _vp, _vp, _u32], _i32),
            "katali_cuda_moe_ep_slot_bytes": ([_vp, C.POINTER(_u64), C.POINTER(_u64)], _i32),
            "katali_cuda_moe_ep_dispatch": ([_vp, _u32, _u32, _u32, _vp, _vp, _vp], _i32),
            "katali_cuda_moe_ep_experts": ([_vp, _u32, _u32, _u32, _vp, _vp], _i32),
            "katali_cuda_moe_ep_combine": ([_vp, _u32, _u32, _u32, _vp, _vp], _i32),
            "katali_cuda_expert_cache_create": ([_u64, _u32, C.POINTER(_vp)], _i32),
            "katali_cuda_expert_cache_destroy": ([_vp], _i32),
            "katali_cuda_expert_register": ([_vp, _u64, _vp, _u64, _vp, _u64, _vp, _u64], _i32),
            "katali_cuda_expert_prefetch_async": ([_vp, _u64], _i32),
            "katali_cuda_expert_bind": ([_vp, _u64, _vp, _u32], _i32),
            "katali_cuda_expert_evict": ([_vp, _u64], _i32),
            "katali_cuda_expert_lookup": ([_vp, _u64, C.POINTER(_i32), C.POINTER(_vp), C.POINTER(_vp),
                                           C.POINTER(_vp)], _i32),
            "katali_cuda_expert_sync": ([_vp], _i32),
            "katali_cuda_dense_create": ([C.POINTER(KataliDenseDesc), C.POINTER(_vp)], _i32),
            "katali_cuda_dense_destroy": ([_vp], _i32),
            "katali_cuda_dense_reset": ([_vp], _i32),
            "katali_cuda_dense_generate": ([_vp, _vp, _u32, _u32, _vp], _i32),
            "katali_cuda_dense_logits": ([_vp, C.POINTER(_vp), C.POINTER(_i32)], _i32),
            "katali_cuda_hybrid_create": ([C.POINTER(KataliHybridDesc), C.POINTER(_vp)], _i32),
            "katali_cuda_hybrid_destroy": ([_vp], _i32),
            "katali_cuda_hybrid_reset": ([_vp], _i32),
            "katali_cuda_hybrid_generate": ([_vp, _vp, _u32, _u32, _vp], _i32),
            "katali_cuda_hybrid_logits": ([_vp, C.POINTER(_vp), C.POINTER(_i32)], _i32),
            "katali_cuda_hybrid_set_ep": ([_vp, _vp], _i32),
            "katali_cuda_gguf_open": ([C.c_char_p, C.POINTER(_vp)], _i32),
            "katali_cuda_gguf_close": ([_vp], _i32),
            "katali_cuda_gguf_counts": ([_vp, C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u32)], _i32),
            "katali_cuda_gguf_tensor": ([_vp, _u64, C.POINTER(KataliGgufTensorInfo)], _i32),
            "katali_cuda_gguf_find": ([_vp, C.c_char_p, C.POINTER(_u64)], _i32),
            "katali_cuda_gguf_get_int": ([_vp, C.c_char_p, C.POINTER(C.c_int64)], _i32),
            "katali_cuda_gguf_get_float": ([_vp, C.c_char_p, C.POINTER(C.c_double)], _i32),
            "katali_cuda_gguf_get_str": ([_vp, C.c_char_p, C.POINTER(_vp), C.POINTER(_u64)], _i32),
            "katali_cuda_gguf_array": ([_vp, C.c_char_p, C.POINTER(_u32), C.POINTER(_u64)], _i32),
            "katali_cuda_gguf_array_int": ([_vp, C.c_char_p, _u64, C.POINTER(C.c_int64)], _i32),
            "katali_cuda_gguf_upload": ([_vp, _u64, _vp], _i32),
            "katali_cuda_dense_create_from_gguf": ([_vp, _u32, _u32, C.POINTER(_vp)], _i32),
            "katali_cuda_hybrid_create_from_gguf": ([_vp, _u32, _u32, _vp, C.POINTER(_vp)], _i32),
            "katali_cuda_ep_unique_id": ([_vp], _i32),
            "katali_cuda_ep_create": ([_u32, _u32, _vp, C.POINTER(_vp)], _i32),
            "katali_cuda_ep_destroy": ([_vp], _i32),
            "katali_cuda_ep_use_peer_memory": ([_vp, _i32], _i32),
            "katali_cuda_moe_ep_layer": ([_vp, _vp, _u32, _u32, _vp, _vp, _vp], _i32),
            "katali_cuda_debug_row_isums": ([_u32, _vp, _u64, _u64, _vp, _vp, _vp], _i32),
            "katali_cuda_debug_route": ([_vp, _vp, _vp, _vp], _i32),
            "katali_cuda_debug_moe_trace": ([_vp, _vp, C.POINTER(_i32)], _i32),
            "katali_cuda_moe_layer_static": ([C.POINTER(KataliMoeDesc), _vp, _vp, _vp, _u32, _vp],
                                             _i32),
        }
        for name, (args, res) in sig.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res

    # -- basics ----------------------------------------------------------
    def probe(self) -> bool:
        return bool(self.L.katali_cuda_probe())

    def status(self) -> str:
        return self.L.katali_cuda_status().decode()

    def check(self, rc: int) -> None:
        if rc != 0:
            raise KataliError(rc, f"{self.L.katali_cuda_strerror(rc).decode()} ({self.status()})")

    def set_stream(self, stream) -> None:
        """stream: a torch.cuda.Stream, a raw cudaStream_t int, or None (plugin stream)."""
        raw = getattr(stream, "cuda_stream", stream)
        if stream is not None and not isinstance(stream, int) and raw == 0:
            raw = 1  # torch's default stream is the legacy NULL stream: cudaStreamLegacy
        self.check(self.L.katali_cuda_set_stream(raw or None))
        self.stream = stream

    @contextlib.contextmanager
    def torch_stream(self):
        """Within the block, plugin calls run on torch's current CUDA stream, so they are
        ordered with torch's own work on it (the plugin's own stream is non-blocking)."""
        import torch
        prev = self.stream
        self.set_stream(torch.cuda.current_stream())
        try:
            yield self
        finally:
            self.set_stream(prev)

    def set_async(self, on: bool) -> None:
        self.check(self.L.katali_cuda_set_async(int(on)))

    def sync(self) -> None:
        self.check(self.L.katali_cuda_sync())

    # -- dense -----------------------------------------------------------
    def matvec(self, qtype, w, rows, cols, x, y) -> None:
        self.check(self.L.katali_cuda_matvec(qtype, _ptr(w), rows, cols, _ptr(x), _ptr(y)))

    def matvec_multi(self, qtypes, ws, rows, cols, x, ys) -> None:
        n = len(qtypes)
        self.check(self.L.katali_cuda_matvec_multi(
            n, (_u32 * n)(*qtypes), (_vp * n)(*[_ptr(w) for w in ws]), (_u64 * n)(*rows), cols,
            _ptr(x), (_vp * n)(*[_ptr(y) for y in ys])))

    def quantize_q8_1(self, x, n, xq) -> None:
        self.check(self.L.katali_cuda_quantize_q8_1(_ptr(x), n, _ptr(xq)))

    def matvec_q8_1(self, qtype, w, rows, cols, xq, y) -> None:
        self.check(self.L.katali_cuda_matvec_q8_1(qtype, _ptr(w), rows, cols, _ptr(xq), _ptr(y)))

    def quantize_rows(self, qtype, src, rows, cols, dst) -> None:
        self.check(self.L.katali_cuda_quantize_rows(qtype, _ptr(src), rows, cols, _ptr(dst)))

    def row_isums(self, qtype, w, rows, cols, xq, isum, xsum) -> None:
        self.check(self.L.katali_cuda_debug_row_isums(qtype, _ptr(w), rows, cols, _ptr(xq),
                                                       _ptr(isum), _ptr(xsum)))


class MoeLayer:
    """One MoE layer's expert table inside the plugin (katali_cuda_moe_*)."""

    def __init__(self, plugin: Plugin, n_experts, hidden, ffn, top_k, experts, norm_topk=True,
                 gate_type=Q4_K, up_type=Q4_K, down_type=Q6_K):
        """experts: list of (gate_ptr, up_ptr, down_ptr) device addresses, one per expert."""
        self.p = plugin
        flat = (_vp * (3 * n_experts))(*[int(a) for tri in experts for a in tri])
        self._flat = flat
        desc = KataliMoeDesc(n_experts, hidden, ffn, top_k, gate_type, up_type, down_type,
                             MOE_NORM_TOPK if norm_topk else 0, C.cast(flat, C.POINTER(_vp)))
        h = _vp()
        plugin.check(plugin.L.katali_cuda_moe_create(C.byref(desc), C.byref(h)))
        self.h = h
        self.top_k = top_k

    def forward(self, x, logits, y, mode=MOE_Q8_1) -> None:
        self.p.check(self.p.L.katali_cuda_moe_layer(self.h, _ptr(x), _ptr(logits), _ptr(y), mode))

    def forward_routed(self, x, ids, w, y, mode=MOE_Q8_1) -> None:
        self.p.check(self.p.L.katali_cuda_moe_layer_routed(self.h, _ptr(x), _ptr(ids), _ptr(w),
                                                           _ptr(y), mode))

    def forward_batch(self, x, logits, y, n_tokens=None, mode=MOE_Q8_1) -> None:
        """Ragged batch: x [T, H], logits [T, n_experts], y [T, H] device buffers."""
        T = int(x.shape[0]) if n_tokens is None else int(n_tokens)
        self.p.check(self.p.L.katali_cuda_moe_batch(self.h, T, _ptr(x), _ptr(logits), _ptr(y),
                                                    mode))

    def route(self, logits, ids, w) -> None:
        self.p.check(self.p.L.katali_cuda_debug_route(self.h, _ptr(logits), _ptr(ids), _ptr(w)))

    def set_trace(self, buf) -> int:
        """Record per-CTA phase timestamps into `buf` (uint64 CUDA tensor, >= grid*32
        entries, zeroed) on later calls; None switches it off. Returns the grid size."""
        g = _i32()
        self.p.check(self.p.L.katali_cuda_debug_moe_trace(self.h, _ptr(buf), C.byref(g)))
        return g.value

    def set_expert(self, e, gate, up, down) -> None:
        self.p.check(self.p.L.katali_cuda_moe_set_expert(self.h, e, int(gate), int(up), int(down)))

    def close(self) -> None:
        if self.h:
            self.p.L.katali_cuda_moe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ExpertCache:
    """The plugin's expert residency tier (katali_cuda_expert_*): device slots fed from
    host memory by asynchronous uploads on a side stream."""

    def __init__(self, plugin: Plugin, slot_bytes: int, n_slots: int):
        self.p = plugin
        h = _vp()
        plugin.check(plugin.L.katali_cuda_expert_cache_create(slot_bytes, n_slots, C.byref(h)))
        self.h = h
        self._keep = {}  # host arrays must outlive their registration

    def register(self, key: int, gate, up, down) -> None:
        """gate/up/down: contiguous host numpy uint8 arrays (borrowed, kept alive here)."""
        self._keep[key] = (gate, up, down)
        self.p.check(self.p.L.katali_cuda_expert_register(
            self.h, key, gate.ctypes.data, gate.nbytes, up.ctypes.data, up.nbytes,
            down.ctypes.data, down.nbytes))

    def prefetch(self, key: int) -> None:
        self.p.check(self.p.L.katali_cuda_expert_prefetch_async(self.h, key))

    def bind(self, key: int, layer: "MoeLayer", e: int) -> None:
        self.p.check(self.p.L.katali_cuda_expert_bind(self.h, key, layer.h, e))

    def evict(self, key: int) -> None:
        self.p.check(self.p.L.katali_cuda_expert_evict(self.h, key))

    def lookup(self, key: int):
        """None when not resident, else the (gate, up, down) device addresses."""
        r = _i32()
        g, u, d = _vp(), _vp(), _vp()
        self.p.check(self.p.L.katali_cuda_expert_lookup(self.h, key, C.byref(r), C.byref(g),
                                                        C.byref(u), C.byref(d)))
        return (g.value, u.value, d.value) if r.value else None

    def sync(self) -> None:
        self.p.check(self.p.L.katali_cuda_expert_sync(self.h))

    def close(self) -> None:
        if self.h:
            self.p.L.katali_cuda_expert_cache_destroy(self.h)
            self.h = None


class DenseModel:
    """A dense Qwen3-style decoder resident on the device (katali_cuda_dense_*)."""

    def __init__(self, plugin: Plugin, model, q8: bool = False):
        """model: katali_lab_b200.synth.DenseWeights (device tensors) or any object with the
        same attributes. q8: q8_1 activations (DP4A) instead of fp32."""
        self.p = plugin
        cfg = model.cfg
        ly = (KataliDenseLayerW * cfg.n_layers)()
        for l, w in enumerate(model.layers):
            ly[l] = KataliDenseLayerW(
                _ptr(w["attn_norm"]), _ptr(w["ffn_norm"]), _ptr(w.get("q_norm")),
                _ptr(w.get("k_norm")), _ptr(w["wq"]), _ptr(w["wk"]), _ptr(w["wv"]), _ptr(w["wo"]),
                _ptr(w["gate"]), _ptr(w["up"]), _ptr(w["down"]), *[model.types[k] for k in
                ("wq", "wk", "wv", "wo", "gate", "up", "down")])
        self._layers = ly
        desc = KataliDenseDesc(cfg.n_layers, cfg.hidden, cfg.ffn, cfg.n_heads, cfg.n_kv_heads,
                               cfg.head_dim, cfg.vocab, cfg.kv_cap, cfg.rope_dim, cfg.rms_eps,
                               cfg.rope_theta, _ptr(model.embed), model.types["embed"],
                               _ptr(model.out_norm), _ptr(model.lm_head), model.types["lm_head"],
                               C.cast(ly, C.POINTER(KataliDenseLayerW)), 1 if q8 else 0)
        h = _vp()
        plugin.check(plugin.L.katali_cuda_dense_create(C.byref(desc), C.byref(h)))
        self.h = h
        self.vocab = cfg.vocab

    @classmethod
    def from_gguf(cls, plugin: Plugin, gguf, kv_cap: int, q8: bool = False) -> "DenseModel":
        """The decoder of a qwen3-architecture GGUF file (katali_cuda_dense_create_from_gguf);
        gguf: an open katali_lab_b200.Gguf."""
        self = cls.__new__(cls)
        self.p = plugin
        h = _vp()
        plugin.check(plugin.L.katali_cuda_dense_create_from_gguf(gguf.h, kv_cap, 1 if q8 else 0,
                                                                 C.byref(h)))
        self.h = h
        nt = gguf.find("token_embd.weight")
        self.vocab = gguf.tensor(nt)["dims"][1]
        return self

    def reset(self) -> None:
        self.p.check(self.p.L.katali_cuda_dense_reset(self.h))

    def generate(self, prompt, n_gen: int):
        import numpy as np
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, dtype=np.int32)
        self.p.check(self.p.L.katali_cuda_dense_generate(self.h, pr.ctypes.data, pr.size, n_gen,
                                                         out.ctypes.data))
        return out

    def logits(self):
        """(device address of the last step's logits, next position)."""
        ptr, pos = _vp(), _i32()
        self.p.check(self.p.L.katali_cuda_dense_logits(self.h, C.byref(ptr), C.byref(pos)))
        return ptr.value, pos.value

    def close(self) -> None:
        if self.h:
            self.p.L.katali_cuda_dense_destroy(self.h)
            self.h = None


class HybridModel:
    """A hybrid MoE decoder (Gated DeltaNet + gated attention, MoE every layer) resident on
    the device (katali_cuda_hybrid_*)."""

    def __init__(self, plugin: Plugin, model, q8: bool = False):
        """model: katali_lab_b200.synth.HybridWeights (device tensors). q8: q8_1 activations
        (DP4A) in the projections and the MoE block instead of fp32."""
        self.p = plugin
        cfg = model.cfg
        T = model.types
        self.moes = []
        ly = (KataliHybridLayerW * cfg.n_layers)()
        for l, w in enumerate(model.layers):
            st = w["experts"]
            # experts [base, base + n) of the layer are resident here (all of them on one GPU;
            # this rank's block under expert parallelism); the other table entries stay NULL
            base = w.get("expert_base", 0)
            table = [(0, 0, 0)] * cfg.n_experts
            for i, ptrs in enumerate(st.pointers()):
                table[base + i] = ptrs
            moe = MoeLayer(plugin, cfg.n_experts, cfg.hidden, cfg.ffn, cfg.top_k, table,
                           norm_topk=True, gate_type=T["gate"], up_type=T["up"], down_type=T["down"])
            self.moes.append(moe)
            e = KataliHybridLayerW()
            e.kind = w["kind"]
            e.attn_norm, e.ffn_norm, e.router = _ptr(w["attn_norm"]), _ptr(w["ffn_norm"]), _ptr(w["router"])
            e.moe = moe.h.value
            if w["kind"] == 0:
                for k in ("ssm_qkv", "ssm_z", "ssm_b", "ssm_a", "ssm_out"):
                    setattr(e, k, _ptr(w[k]))
                    setattr(e, k + "_type", T[k])
                for k in ("ssm_conv", "ssm_a_log", "ssm_dt_bias", "ssm_norm", "ssm_decay"):
                    if w.get(k) is not None:
                        setattr(e, k, _ptr(w[k]))
            else:
                for k in ("wq", "wk", "wv", "wo"):
                    setattr(e, k, _ptr(w[k]))
                    setattr(e, k + "_type", T[k])
                e.q_norm, e.k_norm = _ptr(w.get("q_norm")), _ptr(w.get("k_norm"))
            ly[l] = e
        self._layers = ly
        desc = KataliHybridDesc(cfg.n_layers, cfg.hidden, cfg.vocab, cfg.kv_cap, cfg.n_heads,
                                cfg.n_kv_heads, cfg.head_dim, cfg.rope_dim, cfg.rms_eps,
                                cfg.rope_theta, cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim,
                                cfg.ssm_conv, _ptr(model.embed), T["embed"], _ptr(model.out_norm),
                                _ptr(model.lm_head), T["lm_head"],
                                C.cast(ly, C.POINTER(KataliHybridLayerW)), 1 if q8 else 0)
        h = _vp()
        rc = plugin.L.katali_cuda_hybrid_create(C.byref(desc), C.byref(h))
        if rc != 0:
            for m in self.moes:
                m.close()
            plugin.check(rc)
        self.h = h
        self.vocab = cfg.vocab

    @classmethod
    def from_gguf(cls, plugin: Plugin, gguf, kv_cap: int, q8: bool = False,
                  cache=None) -> "HybridModel":
        """The decoder of a qwen35moe-architecture GGUF file
        (katali_cuda_hybrid_create_from_gguf); gguf: an open katali_lab_b200.Gguf; cache: an
        ExpertCache feeding the experts from the file's mapping on demand (None: all resident).
        The decoder owns its MoE objects; the file and the cache must outlive it."""
        self = cls.__new__(cls)
        self.p = plugin
        self.moes = []
        h = _vp()
        plugin.check(plugin.L.katali_cuda_hybrid_create_from_gguf(
            gguf.h, kv_cap, 1 if q8 else 0, cache.h if cache is not None else None, C.byref(h)))
        self.h = h
        self.vocab = gguf.tensor(gguf.find("token_embd.weight"))["dims"][1]
        return self

    def reset(self) -> None:
        self.p.check(self.p.L.katali_cuda_hybrid_reset(self.h))

    def set_ep(self, comm) -> None:
        """Expert-parallel MoE blocks over `comm` (katali_lab_b200.ep.EpComm in peer-memory
        mode; collective). None: back to the local MoE launches."""
        self.p.check(self.p.L.katali_cuda_hybrid_set_ep(self.h, comm.h if comm is not None else None))

    def generate(self, prompt, n_gen: int):
        import numpy as np
        pr = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, dtype=np.int32)
        self.p.check(self.p.L.katali_cuda_hybrid_generate(self.h, pr.ctypes.data, pr.size, n_gen,
                                                          out.ctypes.data))
        return out

    def logits(self):
        """(device address of the last step's logits, next position)."""
        ptr, pos = _vp(), _i32()
        self.p.check(self.p.L.katali_cuda_hybrid_logits(self.h, C.byref(ptr), C.byref(pos)))
        return ptr.value, pos.value

    def close(self) -> None:
        if self.h:
            self.p.L.katali_cuda_hybrid_destroy(self.h)
            self.h = None
        for m in self.moes:
            m.close()
        self.moes = []


class Gguf:
    """A GGUF model file parsed by the plugin (katali_cuda_gguf_*); tensors upload to the
    device in their native block layout."""

    def __init__(self, plugin: Plugin, path: str):
        self.p = plugin
        h = _vp()
        plugin.check(plugin.L.katali_cuda_gguf_open(os.fsencode(path), C.byref(h)))
        self.h = h
        nt, nkv, ver = _u64(), _u64(), _u32()
        plugin.check(plugin.L.katali_cuda_gguf_counts(h, C.byref(nt), C.byref(nkv), C.byref(ver)))
        self.n_tensors, self.n_kv, self.version = nt.value, nkv.value, ver.value

    def tensor(self, i: int) -> dict:
        info = KataliGgufTensorInfo()
        self.p.check(self.p.L.katali_cuda_gguf_tensor(self.h, i, C.byref(info)))
        return {"name": info.name.decode(), "type": info.type, "n_dims": info.n_dims,
                "dims": tuple(info.dims[:info.n_dims]), "offset": info.offset, "nbytes": info.nbytes}

    def tensors(self) -> list:
        return [self.tensor(i) for i in range(self.n_tensors)]

    def find(self, name: str) -> int | None:
        i = _u64()
        rc = self.p.L.katali_cuda_gguf_find(self.h, name.encode(), C.byref(i))
        return i.value if rc == 0 else None

    def get_int(self, key: str):
        v = C.c_int64()
        return v.value if self.p.L.katali_cuda_gguf_get_int(self.h, key.encode(), C.byref(v)) == 0 else None

    def get_float(self, key: str):
        v = C.c_double()
        return v.value if self.p.L.katali_cuda_gguf_get_float(self.h, key.encode(), C.byref(v)) == 0 else None

    def get_str(self, key: str):
        ptr, n = _vp(), _u64()
        if self.p.L.katali_cuda_gguf_get_str(self.h, key.encode(), C.byref(ptr), C.byref(n)) != 0:
            return None
        return C.string_at(ptr.value, n.value).decode()

    def array(self, key: str):
        et, n = _u32(), _u64()
        if self.p.L.katali_cuda_gguf_array(self.h, key.encode(), C.byref(et), C.byref(n)) != 0:
            return None
        return et.value, n.value

    def array_int(self, key: str, i: int):
        v = C.c_int64()
        return v.value if self.p.L.katali_cuda_gguf_array_int(self.h, key.encode(), i, C.byref(v)) == 0 else None

    def upload(self, i: int, dev) -> None:
        self.p.check(self.p.L.katali_cuda_gguf_upload(self.h, i, _ptr(dev)))

    def close(self) -> None:
        if self.h:
            self.p.L.katali_cuda_gguf_close(self.h)
            self.h = None

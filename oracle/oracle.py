"""ctypes bindings for the CPU checkers (test infrastructure only).

Two libraries, both built by ``oracle/Makefile``:

* ``_port/libkq_oracle.so`` -- ``kq_oracle.c``, the C restatement of the block
  formats, encoders, q8_1 quantiser, integer block dots, routing and the fused
  MoE layer (see the header of ``kq_oracle.h`` for the reference file:line each
  piece follows).
* ``_ref/libkatali_ref.so`` -- the reference's own CPU kernels compiled from its
  checkout, plus ``ref_compose.c`` (the CPU MoE layer assembled from them).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module. The plugin never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_LIB = os.path.join(HERE, "_port", "libkq_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libkatali_ref.so")
DROPIN = os.path.join(HERE, "_ref", "katali_dropin")  # the reference's dense backend + our loader

Q8_1, Q4_K, Q6_K = 9, 12, 14
BLOCK = {Q8_1: (32, 36), Q4_K: (256, 144), Q6_K: (256, 210)}

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def reference_root() -> str | None:
    """The reference checkout (the katali-lab tree): $KATALI_REF_ROOT, else a directory
    named ``reference`` beside this repository; None where neither exists (a GPU box,
    which uses the prebuilt libraries)."""
    cand = os.environ.get("KATALI_REF_ROOT") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isdir(cand) else None


def build(force: bool = False) -> None:
    """Build the checkers with make (the reference part only where its checkout exists)."""
    root = reference_root()
    if force or not os.path.exists(PORT_LIB) or (
            root and not (os.path.exists(REF_LIB) and os.path.exists(DROPIN))):
        env = dict(os.environ)
        if root:
            env["KATALI_REF_ROOT"] = root
        subprocess.run(["make", "-s", "-C", HERE], check=True, env=env)


def row_bytes(qtype: int, cols: int) -> int:
    bs, bb = BLOCK[qtype]
    if cols % bs:
        raise ValueError(f"cols={cols} is not a multiple of {bs}")
    return cols // bs * bb


class Port:
    """The C restatement (kq_oracle.c)."""

    def __init__(self, path: str = PORT_LIB):
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        self.L = L
        L.kqo_f32_to_f16.argtypes = [C.c_float]
        L.kqo_f32_to_f16.restype = C.c_uint16
        L.kqo_f16_to_f32.argtypes = [C.c_uint16]
        L.kqo_f16_to_f32.restype = C.c_float
        L.kqo_expf.argtypes = [C.c_float]
        L.kqo_expf.restype = C.c_float
        L.kqo_silu.argtypes = [C.c_float]
        L.kqo_silu.restype = C.c_float
        L.kqo_dequant.argtypes = [C.c_uint32, _u8p, C.c_uint64, _f32p]
        L.kqo_quantize.argtypes = [C.c_uint32, _f32p, C.c_uint64, _u8p]
        L.kqo_row_isums.argtypes = [C.c_uint32, _u8p, _u8p, C.c_uint64, _i32p, C.c_void_p]
        L.kqo_dot_q8.argtypes = [C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint64]
        L.kqo_dot_q8.restype = C.c_float
        L.kqo_matvec_q8.argtypes = [C.c_uint32, _u8p, C.c_uint64, C.c_uint64, _u8p, _f32p]
        L.kqo_matvec_f32.argtypes = [C.c_uint32, _u8p, C.c_uint64, C.c_uint64, _f32p, _f32p]
        L.kqo_route_topk.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, _i32p, _f32p]
        L.kqo_moe_layer.argtypes = [C.c_void_p, _f32p, _f32p, _f32p, C.c_int,
                                    _i32p, _f32p, C.c_void_p]
        L.kqo_moe_layer_routed.argtypes = [C.c_void_p, _f32p, _i32p, _f32p, _f32p,
                                           C.c_int, C.c_void_p]
        L.kqo_argmax.argtypes = [_f32p, C.c_int]
        L.kqo_ep_slot_bytes.argtypes = [C.c_int, C.c_int]
        L.kqo_ep_slot_bytes.restype = C.c_uint32
        L.kqo_ep_dispatch.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.c_void_p]
        L.kqo_ep_experts.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                     C.c_void_p]
        L.kqo_ep_combine.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                     C.c_void_p, C.c_void_p]

    # -- scalars ---------------------------------------------------------
    def f32_to_f16(self, v: float) -> int:
        return self.L.kqo_f32_to_f16(v)

    def expf(self, v: float) -> float:
        return self.L.kqo_expf(v)

    # -- arrays ----------------------------------------------------------
    def quantize(self, qtype: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = 1 if x.ndim == 1 else x.shape[0]
        cols = x.shape[-1]
        out = np.zeros(rows * row_bytes(qtype, cols), dtype=np.uint8)
        if self.L.kqo_quantize(qtype, x.reshape(-1), x.size, out) != 0:
            raise ValueError("quantize failed")
        return out.reshape(rows, -1) if x.ndim > 1 else out

    def dequant(self, qtype: int, blob: np.ndarray, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.float32)
        if self.L.kqo_dequant(qtype, np.ascontiguousarray(blob).reshape(-1), n, out) != 0:
            raise ValueError("dequant failed")
        return out

    def row_isums(self, qtype: int, row: np.ndarray, xq: np.ndarray, cols: int):
        ng = cols // (32 if qtype == Q4_K else 16)
        isum = np.zeros(ng, dtype=np.int32)
        xsum = np.zeros(ng, dtype=np.int32)
        rc = self.L.kqo_row_isums(qtype, np.ascontiguousarray(row).reshape(-1),
                                  np.ascontiguousarray(xq).reshape(-1), cols, isum,
                                  xsum.ctypes.data)
        if rc != 0:
            raise ValueError("row_isums failed")
        return isum, xsum

    def matvec_q8(self, qtype: int, w: np.ndarray, rows: int, cols: int, xq: np.ndarray):
        y = np.zeros(rows, dtype=np.float32)
        rc = self.L.kqo_matvec_q8(qtype, np.ascontiguousarray(w).reshape(-1), rows, cols,
                                  np.ascontiguousarray(xq).reshape(-1), y)
        if rc != 0:
            raise ValueError("matvec_q8 failed")
        return y

    def matvec_f32(self, qtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray):
        y = np.zeros(rows, dtype=np.float32)
        rc = self.L.kqo_matvec_f32(qtype, np.ascontiguousarray(w).reshape(-1), rows, cols,
                                   np.ascontiguousarray(x, dtype=np.float32), y)
        if rc != 0:
            raise ValueError("matvec_f32 failed")
        return y

    def route(self, logits: np.ndarray, k: int, norm: bool = True):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        ids = np.zeros(k, dtype=np.int32)
        w = np.zeros(k, dtype=np.float32)
        if self.L.kqo_route_topk(logits, logits.size, k, int(norm), ids, w) != 0:
            raise ValueError("route failed")
        return ids, w

    def argmax(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return self.L.kqo_argmax(x, x.size)

    def moe_layer(self, layer: "MoeWeights", x: np.ndarray, logits: np.ndarray | None = None,
                  mode: int = 0, ids=None, w=None):
        """mode 0 = q8_1 activations, 1 = fp32 activations. Returns (y, ids, w, h)."""
        desc, _keep = layer.oracle_desc()
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(layer.hidden, dtype=np.float32)
        h = np.zeros(layer.top_k * layer.ffn, dtype=np.float32)
        if ids is None:
            ids = np.zeros(layer.top_k, dtype=np.int32)
            w = np.zeros(layer.top_k, dtype=np.float32)
            rc = self.L.kqo_moe_layer(C.byref(desc), x,
                                      np.ascontiguousarray(logits, dtype=np.float32),
                                      y, mode, ids, w, h.ctypes.data)
        else:
            ids = np.ascontiguousarray(ids, dtype=np.int32)
            w = np.ascontiguousarray(w, dtype=np.float32)
            rc = self.L.kqo_moe_layer_routed(C.byref(desc), x, ids, w, y, mode, h.ctypes.data)
        if rc != 0:
            raise ValueError("moe_layer failed")
        return y, ids, w, h.reshape(layer.top_k, layer.ffn)


    # -- expert-parallel slot protocol (kqo_ep_*) ------------------------
    def ep_slot_bytes(self, hidden: int, top_k: int) -> int:
        return int(self.L.kqo_ep_slot_bytes(hidden, top_k))

    def ep_dispatch(self, layer: "MoeWeights", n_ranks, max_tokens, x, logits, send=None):
        """Returns (send buffer uint8 [n_ranks*max_tokens*slot], src_ids int32 [T, K])."""
        desc, _keep = layer.oracle_desc()
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, layer.hidden)
        logits = np.ascontiguousarray(logits, dtype=np.float32).reshape(x.shape[0],
                                                                         layer.n_experts)
        sb = self.ep_slot_bytes(layer.hidden, layer.top_k)
        if send is None:
            send = np.zeros(n_ranks * max_tokens * sb, dtype=np.uint8)
        src = np.zeros((max(x.shape[0], 1), layer.top_k), dtype=np.int32)
        rc = self.L.kqo_ep_dispatch(C.byref(desc), n_ranks, max_tokens, x.shape[0],
                                    x.ctypes.data, logits.ctypes.data, send.ctypes.data,
                                    src.ctypes.data)
        if rc != 0:
            raise ValueError("ep_dispatch failed")
        return send, src[:x.shape[0]]

    def ep_experts(self, layer: "MoeWeights", n_ranks, rank, max_tokens, recv, ret=None):
        desc, _keep = layer.oracle_desc()
        recv = np.ascontiguousarray(recv, dtype=np.uint8)
        if ret is None:
            ret = np.zeros(n_ranks * max_tokens * layer.hidden, dtype=np.float64)
        rc = self.L.kqo_ep_experts(C.byref(desc), n_ranks, rank, max_tokens, recv.ctypes.data,
                                   ret.ctypes.data)
        if rc != 0:
            raise ValueError("ep_experts failed")
        return ret

    def ep_combine(self, layer: "MoeWeights", n_ranks, max_tokens, src_ids, back):
        desc, _keep = layer.oracle_desc()
        src_ids = np.ascontiguousarray(src_ids, dtype=np.int32)
        back = np.ascontiguousarray(back, dtype=np.float64)
        y = np.zeros((src_ids.shape[0], layer.hidden), dtype=np.float32)
        rc = self.L.kqo_ep_combine(C.byref(desc), n_ranks, max_tokens, src_ids.shape[0],
                                   src_ids.ctypes.data, back.ctypes.data, y.ctypes.data)
        if rc != 0:
            raise ValueError("ep_combine failed")
        return y


class _KqoMoe(C.Structure):
    _fields_ = [("n_experts", C.c_int), ("hidden", C.c_int), ("ffn", C.c_int),
                ("top_k", C.c_int), ("norm_topk", C.c_int),
                ("gate_type", C.c_uint32), ("up_type", C.c_uint32), ("down_type", C.c_uint32),
                ("gate", C.POINTER(C.c_void_p)), ("up", C.POINTER(C.c_void_p)),
                ("down", C.POINTER(C.c_void_p))]


class MoeWeights:
    """One MoE layer's expert matrices in native GGUF block layout (host numpy).

    gate/up: [n_experts, ffn * row_bytes(hidden)], down: [n_experts, hidden * row_bytes(ffn)].
    """

    def __init__(self, gate, up, down, hidden, ffn, top_k=8, norm_topk=True,
                 gate_type=Q4_K, up_type=Q4_K, down_type=Q6_K):
        self.gate, self.up, self.down = (np.ascontiguousarray(a) for a in (gate, up, down))
        self.n_experts = self.gate.shape[0]
        self.hidden, self.ffn, self.top_k, self.norm_topk = hidden, ffn, top_k, norm_topk
        self.gate_type, self.up_type, self.down_type = gate_type, up_type, down_type

    def _ptrs(self, arr):
        p = (C.c_void_p * self.n_experts)()
        base = arr.ctypes.data
        for e in range(self.n_experts):
            p[e] = base + e * arr.shape[1]
        return p

    def oracle_desc(self):
        g, u, d = self._ptrs(self.gate), self._ptrs(self.up), self._ptrs(self.down)
        desc = _KqoMoe(self.n_experts, self.hidden, self.ffn, self.top_k, int(self.norm_topk),
                       self.gate_type, self.up_type, self.down_type,
                       C.cast(g, C.POINTER(C.c_void_p)), C.cast(u, C.POINTER(C.c_void_p)),
                       C.cast(d, C.POINTER(C.c_void_p)))
        return desc, (g, u, d)

    @property
    def expert_bytes(self) -> int:
        return self.gate.shape[1] + self.up.shape[1] + self.down.shape[1]


class Ref:
    """The reference's own CPU kernels (compiled from its checkout) + ref_compose.c."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (run make -C oracle)")
        L = C.CDLL(path)
        self.L = L
        L.katali_ggml_dequant_ref.argtypes = [C.c_uint32, _u8p, C.c_uint64, _f32p]
        L.katali_ggml_vec_dot_ref.argtypes = [C.c_uint32, C.c_void_p, _f32p, C.c_uint64]
        L.katali_ggml_vec_dot_ref.restype = C.c_float
        L.katali_ggml_vec_dot.argtypes = [C.c_uint32, C.c_void_p, _f32p, C.c_uint64]
        L.katali_ggml_vec_dot.restype = C.c_float
        L.kref_matvec.argtypes = [C.c_uint32, C.c_void_p, C.c_uint64, C.c_uint64, _f32p, _f32p,
                                  C.c_int]
        L.katali_dtype_selftest.restype = C.c_int
        L.katali_dtype_simd_selftest.restype = C.c_int
        L.katali_gguf_softmax.argtypes = [_f32p, C.c_size_t]
        L.katali_gguf_get_threads.restype = C.c_int
        L.kref_moe_scratch_new.argtypes = [C.c_int] * 4
        L.kref_moe_scratch_new.restype = C.c_void_p
        L.kref_moe_scratch_free.argtypes = [C.c_void_p]
        L.kref_moe_layer.argtypes = [C.c_int] * 5 + [C.c_uint32] * 3 + [
            C.POINTER(C.c_void_p)] * 3 + [_f32p, _f32p, _f32p, C.c_int, C.c_void_p,
                                          C.c_void_p, C.c_void_p]

    def dequant(self, qtype, blob, n):
        out = np.zeros(n, dtype=np.float32)
        if self.L.katali_ggml_dequant_ref(qtype, np.ascontiguousarray(blob).reshape(-1), n,
                                          out) != 0:
            raise ValueError("dequant failed")
        return out

    def matvec(self, qtype, w, rows, cols, x, n_threads=0):
        w = np.ascontiguousarray(w)
        y = np.zeros(rows, dtype=np.float32)
        self.L.kref_matvec(qtype, w.ctypes.data, rows, cols,
                           np.ascontiguousarray(x, dtype=np.float32), y, n_threads)
        return y

    def threads(self) -> int:
        return self.L.katali_gguf_get_threads()

    def moe_scratch(self, layer: MoeWeights):
        return self.L.kref_moe_scratch_new(layer.n_experts, layer.hidden, layer.ffn, layer.top_k)

    def moe_layer(self, layer: MoeWeights, x, logits, n_threads=0, scratch=None):
        """fp32-activation MoE layer from the reference's kernels. Returns (y, ids, w)."""
        own = scratch is None
        if own:
            scratch = self.moe_scratch(layer)
        g, u, d = layer._ptrs(layer.gate), layer._ptrs(layer.up), layer._ptrs(layer.down)
        y = np.zeros(layer.hidden, dtype=np.float32)
        ids = np.zeros(layer.top_k, dtype=np.int32)
        w = np.zeros(layer.top_k, dtype=np.float32)
        rc = self.L.kref_moe_layer(layer.n_experts, layer.hidden, layer.ffn, layer.top_k,
                                   int(layer.norm_topk), layer.gate_type, layer.up_type,
                                   layer.down_type, C.cast(g, C.POINTER(C.c_void_p)),
                                   C.cast(u, C.POINTER(C.c_void_p)),
                                   C.cast(d, C.POINTER(C.c_void_p)),
                                   np.ascontiguousarray(x, dtype=np.float32),
                                   np.ascontiguousarray(logits, dtype=np.float32), y,
                                   n_threads, scratch, ids.ctypes.data, w.ctypes.data)
        if own:
            self.L.kref_moe_scratch_free(scratch)
        if rc != 0:
            raise ValueError("kref_moe_layer failed")
        return y, ids, w


def make_moe_weights(port: Port, n_experts: int, hidden: int, ffn: int, seed: int,
                     top_k: int = 8, std: float = 0.02, norm_topk: bool = True) -> MoeWeights:
    """Seeded synthetic expert matrices: N(0, std) fp32 -> our Q4_K / Q6_K encoders."""
    rng = np.random.default_rng(seed)
    rb_g = row_bytes(Q4_K, hidden)
    rb_d = row_bytes(Q6_K, ffn)
    gate = np.zeros((n_experts, ffn * rb_g), np.uint8)
    up = np.zeros((n_experts, ffn * rb_g), np.uint8)
    down = np.zeros((n_experts, hidden * rb_d), np.uint8)
    for e in range(n_experts):
        gate[e] = port.quantize(Q4_K, rng.normal(0, std, (ffn, hidden)).astype(np.float32)).reshape(-1)
        up[e] = port.quantize(Q4_K, rng.normal(0, std, (ffn, hidden)).astype(np.float32)).reshape(-1)
        down[e] = port.quantize(Q6_K, rng.normal(0, std, (hidden, ffn)).astype(np.float32)).reshape(-1)
    return MoeWeights(gate, up, down, hidden, ffn, top_k, norm_topk)


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


class RefDense:
    """The dense decode step composed from the reference's kernels (kref_dense_*), on HOST
    copies of a katali_lab_b200.synth.DenseWeights model."""

    def __init__(self, ref: "Ref", model, n_threads: int = 0):
        import torch  # noqa: F401  (host copies come from torch tensors)
        cfg = model.cfg
        self.ref, self.cfg = ref, cfg
        h = lambda t: np.ascontiguousarray(t.cpu().numpy())  # noqa: E731
        self._keep = []
        keep = self._keep.append
        NL = cfg.n_layers
        an = (C.c_void_p * NL)(); fn = (C.c_void_p * NL)(); qn = (C.c_void_p * NL)(); kn = (C.c_void_p * NL)()
        ws = (C.c_void_p * (7 * NL))(); ts = (C.c_uint32 * (7 * NL))()
        names = ("wq", "wk", "wv", "wo", "gate", "up", "down")
        for l, w in enumerate(model.layers):
            for arr, key in ((an, "attn_norm"), (fn, "ffn_norm"), (qn, "q_norm"), (kn, "k_norm")):
                a = h(w[key]); keep(a); arr[l] = a.ctypes.data
            for i, k in enumerate(names):
                a = h(w[k]); keep(a); ws[7 * l + i] = a.ctypes.data; ts[7 * l + i] = model.types[k]
        emb, lm, on = h(model.embed), h(model.lm_head), h(model.out_norm)
        for a in (emb, lm, on, an, fn, qn, kn, ws, ts):
            keep(a)
        L = ref.L
        L.kref_dense_new.restype = C.c_void_p
        L.kref_dense_new.argtypes = [C.c_int] * 9 + [C.c_float, C.c_float, C.c_void_p, C.c_uint32,
                                                     C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p,
                                                     C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                     C.c_void_p, C.c_int]
        L.kref_dense_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.kref_dense_free.argtypes = [C.c_void_p]
        self.h = L.kref_dense_new(NL, cfg.hidden, cfg.ffn, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                                  cfg.vocab, cfg.kv_cap, cfg.rope_dim, cfg.rms_eps, cfg.rope_theta,
                                  emb.ctypes.data, model.types["embed"], lm.ctypes.data,
                                  model.types["lm_head"], on.ctypes.data, an, fn, qn, kn, ws, ts,
                                  n_threads or os.cpu_count() or 1)
        self.logits = np.zeros(cfg.vocab, dtype=np.float32)

    def step(self, token: int, pos: int) -> np.ndarray:
        if self.ref.L.kref_dense_step(self.h, int(token), int(pos), self.logits.ctypes.data) != 0:
            raise ValueError("kref_dense_step failed")
        return self.logits

    def close(self):
        if self.h:
            self.ref.L.kref_dense_free(self.h)
            self.h = None


class _KrefHybridLayer(C.Structure):
    _fields_ = [("kind", C.c_int32), ("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p),
                ("router", C.c_void_p), ("w_qkv", C.c_void_p), ("w_z", C.c_void_p),
                ("w_b", C.c_void_p), ("w_a", C.c_void_p), ("w_out", C.c_void_p),
                ("t_qkv", C.c_uint32), ("t_z", C.c_uint32), ("t_b", C.c_uint32), ("t_a", C.c_uint32),
                ("t_out", C.c_uint32), ("conv", C.c_void_p), ("a_log", C.c_void_p),
                ("dt_bias", C.c_void_p), ("ssm_norm", C.c_void_p), ("wq", C.c_void_p),
                ("wk", C.c_void_p), ("wv", C.c_void_p), ("wo", C.c_void_p), ("tq", C.c_uint32),
                ("tk", C.c_uint32), ("tv", C.c_uint32), ("to", C.c_uint32), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p), ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p)]


class RefHybrid:
    """The hybrid MoE decode step (kref_hybrid_*: the reference's kernels plus the Gated
    DeltaNet restatement) on HOST copies of a katali_lab_b200.synth.HybridWeights model."""

    def __init__(self, ref: "Ref", model, n_threads: int = 0):
        cfg = model.cfg
        self.ref, self.cfg = ref, cfg
        h = lambda t: np.ascontiguousarray(t.cpu().numpy())  # noqa: E731
        self._keep = []
        keep = self._keep.append
        T = model.types
        NL = cfg.n_layers
        ly = (_KrefHybridLayer * NL)()
        for l, w in enumerate(model.layers):
            e = _KrefHybridLayer()
            e.kind = w["kind"]

            def hp(key):
                a = h(w[key])
                keep(a)
                return a.ctypes.data
            e.attn_norm, e.ffn_norm, e.router = hp("attn_norm"), hp("ffn_norm"), hp("router")
            if w["kind"] == 0:
                e.w_qkv, e.w_z, e.w_b, e.w_a, e.w_out = (hp(k) for k in ("ssm_qkv", "ssm_z", "ssm_b",
                                                                         "ssm_a", "ssm_out"))
                e.t_qkv, e.t_z, e.t_b, e.t_a, e.t_out = (T[k] for k in ("ssm_qkv", "ssm_z", "ssm_b",
                                                                        "ssm_a", "ssm_out"))
                e.conv, e.a_log, e.dt_bias, e.ssm_norm = (hp(k) for k in ("ssm_conv", "ssm_a_log",
                                                                          "ssm_dt_bias", "ssm_norm"))
            else:
                e.wq, e.wk, e.wv, e.wo = (hp(k) for k in ("wq", "wk", "wv", "wo"))
                e.tq, e.tk, e.tv, e.to = (T[k] for k in ("wq", "wk", "wv", "wo"))
                e.q_norm, e.k_norm = hp("q_norm"), hp("k_norm")
            st = w["experts"]
            for name, dev in (("gate", st.gate), ("up", st.up), ("down", st.down)):
                a = h(dev)
                keep(a)
                ptrs = (C.c_void_p * cfg.n_experts)(*[a.ctypes.data + i * a.shape[1]
                                                      for i in range(cfg.n_experts)])
                keep(ptrs)
                setattr(e, name, C.cast(ptrs, C.c_void_p).value)
            ly[l] = e
        keep(ly)
        emb, lm, on = h(model.embed), h(model.lm_head), h(model.out_norm)
        for a in (emb, lm, on):
            keep(a)
        dims = (C.c_int32 * 16)(NL, cfg.hidden, cfg.vocab, cfg.kv_cap, cfg.n_heads, cfg.n_kv_heads,
                                cfg.head_dim, cfg.rope_dim, cfg.ssm_k_heads, cfg.ssm_v_heads,
                                cfg.ssm_head_dim, cfg.ssm_conv, cfg.n_experts, cfg.ffn, cfg.top_k, 1)
        keep(dims)
        L = ref.L
        L.kref_hybrid_new.restype = C.c_void_p
        L.kref_hybrid_new.argtypes = [C.c_void_p, C.c_float, C.c_float, C.c_void_p, C.c_uint32,
                                      C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint32,
                                      C.c_uint32, C.c_void_p, C.c_int]
        L.kref_hybrid_step.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.kref_hybrid_step.restype = C.c_int
        L.kref_hybrid_free.argtypes = [C.c_void_p]
        L.kref_hybrid_reset.argtypes = [C.c_void_p]
        L.kref_hybrid_route_gaps.argtypes = [C.c_void_p, C.c_void_p]
        self.h = L.kref_hybrid_new(dims, cfg.rms_eps, cfg.rope_theta, emb.ctypes.data, T["embed"],
                                   lm.ctypes.data, T["lm_head"], on.ctypes.data, T["gate"], T["up"],
                                   T["down"], C.cast(ly, C.c_void_p), n_threads or os.cpu_count() or 1)
        if not self.h:
            raise MemoryError("kref_hybrid_new failed")
        self.logits = np.zeros(cfg.vocab, dtype=np.float32)

    def reset(self):
        self.ref.L.kref_hybrid_reset(self.h)

    def step(self, token: int, pos: int) -> np.ndarray:
        if self.ref.L.kref_hybrid_step(self.h, int(token), int(pos), self.logits.ctypes.data) != 0:
            raise ValueError("kref_hybrid_step failed")
        return self.logits

    def route_gaps(self) -> np.ndarray:
        """Per layer, for the last step: the relative margin between the top_k-th and the
        (top_k + 1)-th router logit (where a ~1e-7 difference in the logits can change
        which experts are selected)."""
        out = np.empty(self.cfg.n_layers, np.float32)
        self.ref.L.kref_hybrid_route_gaps(C.c_void_p(self.h), out.ctypes.data)
        return out

    def close(self):
        if self.h:
            self.ref.L.kref_hybrid_free(self.h)
            self.h = None

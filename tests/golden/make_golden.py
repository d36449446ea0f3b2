"""Generate tests/golden/golden.npz from the reference's own CPU kernels.

Run in the build container, where the reference checkout exists and
oracle/Makefile has compiled it into oracle/_ref/libkatali_ref.so:

    python tests/golden/make_golden.py

Inputs are regenerated at test time from the seeds below (numpy default_rng +
the C encoder in oracle/kq_oracle.c); the fixture stores the sha256 of every
encoded weight blob, so a test fails loudly if regeneration ever differs, and
the reference's outputs for those inputs:

* q4k_matvec / q6k_matvec: katali_ggml_matvec (AVX2 row loop, Q4_K sums hoist)
  and katali_ggml_vec_dot_ref per row (V/src/gguf_dtype.c:544-559, 784-856).
* q4k_blocks / q6k_blocks: random block bytes with finite fp16 scales, the same
  construction as the reference's own selftest (V/src/gguf_dtype.c:1161-1176),
  decoded by katali_ggml_dequant_ref.
* moe_small: the CPU MoE layer composed from the reference kernels
  (oracle/ref_compose.c) for a small layer.
* selftests: return codes of katali_dtype_selftest / katali_dtype_simd_selftest.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Q4_K, Q6_K, Port, Ref, make_moe_weights  # noqa: E402

OUT = os.path.join(HERE, "golden.npz")

MATVEC_CASES = {  # name: (type, rows, cols, seed)
    "q4k_matvec": (Q4_K, 96, 2048, 11),
    "q6k_matvec": (Q6_K, 96, 512, 12),
    "q4k_matvec_wide": (Q4_K, 8, 4096, 14),
    "q6k_matvec_wide": (Q6_K, 8, 4096, 15),
}
MOE_CASE = dict(n_experts=8, hidden=512, ffn=256, top_k=2, seed=13)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def matvec_inputs(port: Port, qtype: int, rows: int, cols: int, seed: int):
    rng = np.random.default_rng(seed)
    w = port.quantize(qtype, rng.normal(0, 0.02, (rows, cols)).astype(np.float32))
    x = rng.normal(0, 1, cols).astype(np.float32)
    return w, x


def random_blocks(qtype: int, nblocks: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    bb = 144 if qtype == Q4_K else 210
    blob = rng.integers(0, 256, (nblocks, bb), dtype=np.uint8)
    half = np.array([0.05], np.float16).view(np.uint8)
    if qtype == Q4_K:
        blob[:, 0:2] = half
        blob[:, 2:4] = half
    else:
        blob[:, 208:210] = half
    return blob.reshape(-1)


def moe_inputs(port: Port):
    c = MOE_CASE
    layer = make_moe_weights(port, c["n_experts"], c["hidden"], c["ffn"], seed=c["seed"],
                             top_k=c["top_k"])
    rng = np.random.default_rng(c["seed"] + 1000)
    x = rng.normal(0, 1, c["hidden"]).astype(np.float32)
    logits = rng.normal(0, 1, c["n_experts"]).astype(np.float32)
    return layer, x, logits


def main() -> None:
    port, ref = Port(), Ref()
    out = {}
    for name, (qt, rows, cols, seed) in MATVEC_CASES.items():
        w, x = matvec_inputs(port, qt, rows, cols, seed)
        rb = w.shape[1]
        out[f"{name}/w_sha"] = np.array(sha(w))
        out[f"{name}/y"] = ref.matvec(qt, w, rows, cols, x, n_threads=1)
        out[f"{name}/y_vec_dot_ref"] = np.array(
            [ref.L.katali_ggml_vec_dot_ref(qt, w.ctypes.data + r * rb, x, cols) for r in range(rows)],
            np.float32)
    for name, qt, seed in (("q4k_blocks", Q4_K, 21), ("q6k_blocks", Q6_K, 22)):
        blob = random_blocks(qt, 16, seed)
        out[f"{name}/bytes"] = blob
        out[f"{name}/dequant"] = ref.dequant(qt, blob, 16 * 256)
    layer, x, logits = moe_inputs(port)
    y, ids, w = ref.moe_layer(layer, x, logits, n_threads=1)
    out["moe_small/w_sha"] = np.array(sha(np.concatenate([layer.gate.reshape(-1), layer.up.reshape(-1),
                                                          layer.down.reshape(-1)])))
    out["moe_small/y"] = y
    out["moe_small/ids"] = ids
    out["moe_small/w"] = w
    out["selftests"] = np.array([ref.L.katali_dtype_selftest(), ref.L.katali_dtype_simd_selftest()],
                                np.int32)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()

"""Helpers for the drop-in tests: the reference's own dense backend (oracle/_ref/katali_dropin,
built from the reference checkout by oracle/Makefile) run on a synthetic qwen3 GGUF file."""
from __future__ import annotations

import json
import os
import subprocess
import types

import numpy as np

from katali_lab_b200.synth import DenseConfig
from oracle.oracle import DROPIN, Q4_K, Q6_K, row_bytes
from tests.gguf_files import dense_model_file

CFG = DenseConfig(n_layers=2, hidden=1024, ffn=3072, n_heads=8, n_kv_heads=2, head_dim=128,
                  vocab=4096, kv_cap=256)
PROMPT = "hi!"      # byte tokens 104, 105, 33 (the file's first 256 tokens are the byte tokens)
N_TOKENS = 16


def write_model(port, path, seed=21):
    data, offsets = dense_model_file(port, CFG, seed=seed, byte_vocab=True)
    with open(path, "wb") as f:
        f.write(data)
    return data, offsets


def run_reference(model_path, out_prefix, cuda: bool, plugin_path: str | None = None):
    """The reference's greedy generate; returns (json record, logits [n, vocab], ids [n])."""
    env = {"PATH": os.environ.get("PATH", "/usr/bin"), "KATALI_CUDA": "1" if cuda else "0",
           "KATALI_GGUF_NO_BATCH_PREFILL": "1"}  # the prompt runs through gguf_forward_token
    if plugin_path:
        env["KATALI_CUDA_DLL"] = plugin_path
    for k in ("CUDA_VISIBLE_DEVICES", "LD_LIBRARY_PATH"):
        if k in os.environ:
            env[k] = os.environ[k]
    r = subprocess.run([DROPIN, str(model_path), str(N_TOKENS), PROMPT, str(out_prefix)],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    rec = json.loads(r.stdout.strip().splitlines()[-1])
    lg = np.fromfile(f"{out_prefix}.logits", np.float32).reshape(-1, rec["vocab"])
    ids = np.fromfile(f"{out_prefix}.ids", np.int32)
    return rec, lg, ids


def host_model(data, offsets):
    """The file's tensors as host torch tensors in the layout oracle.RefDense reads."""
    import torch
    H, F, NH, NKV, HD, V = CFG.hidden, CFG.ffn, CFG.n_heads, CFG.n_kv_heads, CFG.head_dim, CFG.vocab

    def mat(name, qt, rows, cols):
        n = rows * row_bytes(qt, cols)
        return torch.from_numpy(np.frombuffer(data, np.uint8, n, offsets[name]).copy())

    def f32(name, n):
        return torch.from_numpy(np.frombuffer(data, np.float32, n, offsets[name]).copy())

    types_ = {"wq": Q4_K, "wk": Q4_K, "wv": Q6_K, "wo": Q4_K, "gate": Q4_K, "up": Q4_K, "down": Q6_K,
              "embed": Q4_K, "lm_head": Q6_K}
    shapes = {"wq": (NH * HD, H), "wk": (NKV * HD, H), "wv": (NKV * HD, H), "wo": (H, NH * HD),
              "gate": (F, H), "up": (F, H), "down": (H, F)}
    names = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "gate": "ffn_gate",
             "up": "ffn_up", "down": "ffn_down"}
    layers = []
    for l in range(CFG.n_layers):
        p = f"blk.{l}."
        w = {k: mat(p + v + ".weight", types_[k], *shapes[k]) for k, v in names.items()}
        w.update(attn_norm=f32(p + "attn_norm.weight", H), ffn_norm=f32(p + "ffn_norm.weight", H),
                 q_norm=f32(p + "attn_q_norm.weight", HD), k_norm=f32(p + "attn_k_norm.weight", HD))
        layers.append(w)
    return types.SimpleNamespace(cfg=CFG, embed=mat("token_embd.weight", Q4_K, V, H),
                                 lm_head=mat("output.weight", Q6_K, V, H),
                                 out_norm=f32("output_norm.weight", H), layers=layers, types=types_)


def prompt_ids():
    return list(PROMPT.encode())

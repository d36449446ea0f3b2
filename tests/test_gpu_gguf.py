"""A dense model read from a GGUF file by the plugin's reader and uploaded to the device in
its native block layout (katali_cuda_gguf_upload): every tensor's device bytes equal the
file's, and the on-device decoder built from the uploaded tensors produces the greedy tokens
of the reference's CPU decode step (logits within rel_L2 <= 1e-5 at every step)."""
import types

import numpy as np
import pytest

from katali_lab_b200 import DenseModel, Gguf
from katali_lab_b200.synth import DenseConfig
from oracle.oracle import RefDense, rel_l2
from tests.gguf_files import dense_model_file

pytestmark = pytest.mark.gpu

CFG = DenseConfig(n_layers=2, hidden=1024, ffn=3072, n_heads=8, n_kv_heads=2, head_dim=128,
                  vocab=4096, kv_cap=128)


def test_gguf_upload_and_decode(plugin, ref, port, tmp_path):
    import torch
    data, offsets = dense_model_file(port, CFG, seed=9)
    path = tmp_path / "dense.gguf"
    path.write_bytes(data)
    g = Gguf(plugin, str(path))
    # the configuration comes from the file's metadata
    cfg = DenseConfig(n_layers=g.get_int("qwen3.block_count"), hidden=g.get_int("qwen3.embedding_length"),
                      ffn=g.get_int("qwen3.feed_forward_length"),
                      n_heads=g.get_int("qwen3.attention.head_count"),
                      n_kv_heads=g.get_int("qwen3.attention.head_count_kv"),
                      head_dim=g.get_int("qwen3.attention.key_length"), vocab=g.array("tokenizer.ggml.tokens")[1],
                      kv_cap=g.get_int("qwen3.context_length"),
                      rope_theta=g.get_float("qwen3.rope.freq_base"),
                      rms_eps=g.get_float("qwen3.attention.layer_norm_rms_epsilon"))
    assert (cfg.n_layers, cfg.hidden, cfg.ffn, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.vocab,
            cfg.kv_cap, cfg.rope_theta) == (CFG.n_layers, CFG.hidden, CFG.ffn, CFG.n_heads,
                                            CFG.n_kv_heads, CFG.head_dim, CFG.vocab, CFG.kv_cap,
                                            CFG.rope_theta)
    assert abs(cfg.rms_eps - CFG.rms_eps) < 1e-12  # stored as f32
    dev, types_ = {}, {}
    for i, t in enumerate(g.tensors()):
        buf = torch.empty(t["nbytes"], dtype=torch.uint8, device="cuda")
        g.upload(i, buf)
        assert t["offset"] == offsets[t["name"]]
        back = buf.cpu().numpy().tobytes()
        assert back == data[t["offset"]:t["offset"] + t["nbytes"]], t["name"]
        dev[t["name"]] = buf.view(torch.float32) if t["type"] == 0 else buf
        types_[t["name"]] = t["type"]
    g.close()
    names = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "gate": "ffn_gate",
             "up": "ffn_up", "down": "ffn_down", "attn_norm": "attn_norm", "ffn_norm": "ffn_norm",
             "q_norm": "attn_q_norm", "k_norm": "attn_k_norm"}
    layers = [{k: dev[f"blk.{l}.{v}.weight"] for k, v in names.items()} for l in range(cfg.n_layers)]
    model = types.SimpleNamespace(
        cfg=cfg, embed=dev["token_embd.weight"], lm_head=dev["output.weight"],
        out_norm=dev["output_norm.weight"], layers=layers,
        types={**{k: types_[f"blk.0.{v}.weight"] for k, v in names.items() if "norm" not in k},
               "embed": types_["token_embd.weight"], "lm_head": types_["output.weight"]})
    dm = DenseModel(plugin, model)
    rd = RefDense(ref, model)
    tok_g = tok_c = 7
    for s in range(12):
        tok_g = int(dm.generate([tok_g], 1)[0])
        lc = rd.step(tok_c, s)
        tok_c = port.argmax(lc)
        ptr, _ = dm.logits()
        lg = np.empty(cfg.vocab, np.float32)
        plugin.check(plugin.L.katali_cuda_download(lg.ctypes.data, ptr, lg.nbytes))
        assert rel_l2(lg, lc) <= 1e-5, s
        assert tok_g == tok_c, s
    rd.close()
    dm.close()


def test_dense_decoder_straight_from_gguf(plugin, ref, port, tmp_path):
    """katali_cuda_dense_create_from_gguf builds the decoder from the file alone (metadata,
    tensor names, uploads); its greedy tokens and logits equal the reference CPU decode of the
    same file's tensors."""
    import torch
    data, _ = dense_model_file(port, CFG, seed=13)
    path = tmp_path / "dense.gguf"
    path.write_bytes(data)
    g = Gguf(plugin, str(path))
    dm = DenseModel.from_gguf(plugin, g, kv_cap=CFG.kv_cap)
    # the reference decode on host copies of the same tensors
    host = {t["name"]: torch.from_numpy(np.frombuffer(data, np.uint8, t["nbytes"], t["offset"]).copy())
            for t in g.tensors()}
    types_ = {t["name"]: t["type"] for t in g.tensors()}
    g.close()
    f32 = lambda n: host[n].view(torch.float32)  # noqa: E731
    names = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "gate": "ffn_gate",
             "up": "ffn_up", "down": "ffn_down"}
    layers = [{**{k: host[f"blk.{l}.{v}.weight"] for k, v in names.items()},
               "attn_norm": f32(f"blk.{l}.attn_norm.weight"), "ffn_norm": f32(f"blk.{l}.ffn_norm.weight"),
               "q_norm": f32(f"blk.{l}.attn_q_norm.weight"), "k_norm": f32(f"blk.{l}.attn_k_norm.weight")}
              for l in range(CFG.n_layers)]
    model = types.SimpleNamespace(
        cfg=CFG, embed=host["token_embd.weight"], lm_head=host["output.weight"],
        out_norm=f32("output_norm.weight"), layers=layers,
        types={**{k: types_[f"blk.0.{v}.weight"] for k, v in names.items()},
               "embed": types_["token_embd.weight"], "lm_head": types_["output.weight"]})
    rd = RefDense(ref, model)
    tok_g = tok_c = 11
    for s in range(10):
        tok_g = int(dm.generate([tok_g], 1)[0])
        lc = rd.step(tok_c, s)
        tok_c = port.argmax(lc)
        ptr, _ = dm.logits()
        lg = np.empty(CFG.vocab, np.float32)
        plugin.check(plugin.L.katali_cuda_download(lg.ctypes.data, ptr, lg.nbytes))
        assert rel_l2(lg, lc) <= 1e-5, s
        assert tok_g == tok_c, s
    rd.close()
    dm.close()

"""The hybrid MoE decoder read from a qwen35moe GGUF file (katali_cuda_hybrid_create_from_gguf):
1. every tensor uploaded by the loader: logits bit-identical, step by step, to the decoder
   built through katali_cuda_hybrid_create from the same file tensors uploaded one by one
   (the loader's wiring: names, shapes, expert slicing, the file's decay rates A);
2. experts fed by the residency tier from the file's read-only mapping (a cache of 24 slots
   for 64 experts, uploaded on demand after each layer's router): the same greedy tokens,
   logits within rel_L2 <= 1e-5 of the all-resident decoder (the router runs as its own
   kernel there), with at most the cache's 24 experts on the device at any time."""
import types

import numpy as np
import pytest

from katali_lab_b200 import ExpertCache, Gguf, HybridModel
from katali_lab_b200.synth import ExpertStore, HybridConfig
from oracle.oracle import rel_l2
from tests.gguf_files import hybrid_model_file

pytestmark = pytest.mark.gpu

SMALL = HybridConfig(n_layers=4, hidden=1024, vocab=4096, kv_cap=64, n_heads=4, n_kv_heads=2,
                     head_dim=256, rope_dim=64, ssm_k_heads=2, ssm_v_heads=4, ssm_head_dim=128,
                     ssm_conv=4, n_experts=16, ffn=512, top_k=4)
STEPS = 10


def _logits(plugin, m):
    ptr, _ = m.logits()
    out = np.empty(m.vocab, dtype=np.float32)
    plugin.check(plugin.L.katali_cuda_download(out.ctypes.data, ptr, out.nbytes))
    return out


def _decode(plugin, m, prompt):
    toks, lgs = [], []
    nxt = m.generate(prompt, 1)[0]
    for _ in range(STEPS):
        toks.append(int(nxt))
        lgs.append(_logits(plugin, m))
        nxt = m.generate([nxt], 1)[0]
    return toks, lgs


def _by_hand(plugin, g, cfg):
    """HybridModel through the descriptor API from the file's tensors uploaded one by one."""
    import torch
    dev, ty = {}, {}
    for i, t in enumerate(g.tensors()):
        buf = torch.empty(t["nbytes"], dtype=torch.uint8, device="cuda")
        g.upload(i, buf)
        dev[t["name"]] = buf.view(torch.float32) if t["type"] == 0 else buf
        ty[t["name"]] = t["type"]
    E, layers = cfg.n_experts, []
    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        w = {"kind": 0 if p + "attn_qkv.weight" in dev else 1, "attn_norm": dev[p + "attn_norm.weight"],
             "ffn_norm": dev[p + "post_attention_norm.weight"], "router": dev[p + "ffn_gate_inp.weight"],
             "experts": ExpertStore(dev[p + "ffn_gate_exps.weight"].view(E, -1),
                                    dev[p + "ffn_up_exps.weight"].view(E, -1),
                                    dev[p + "ffn_down_exps.weight"].view(E, -1), cfg.hidden, cfg.ffn),
             "expert_base": 0}
        if w["kind"] == 0:
            names = {"ssm_qkv": "attn_qkv.weight", "ssm_z": "attn_gate.weight", "ssm_b": "ssm_beta.weight",
                     "ssm_a": "ssm_alpha.weight", "ssm_out": "ssm_out.weight", "ssm_conv": "ssm_conv1d.weight",
                     "ssm_decay": "ssm_a", "ssm_dt_bias": "ssm_dt.bias", "ssm_norm": "ssm_norm.weight"}
        else:
            names = {"wq": "attn_q.weight", "wk": "attn_k.weight", "wv": "attn_v.weight",
                     "wo": "attn_output.weight", "q_norm": "attn_q_norm.weight", "k_norm": "attn_k_norm.weight"}
        w.update({k: dev[p + v] for k, v in names.items()})
        layers.append(w)
    gdn = next(l for l in range(cfg.n_layers) if cfg.kind(l) == 0)
    att = next(l for l in range(cfg.n_layers) if cfg.kind(l) == 1)
    types_ = {k: ty[f"blk.{gdn}.{v}"] for k, v in (("ssm_qkv", "attn_qkv.weight"), ("ssm_z", "attn_gate.weight"),
                                                   ("ssm_b", "ssm_beta.weight"), ("ssm_a", "ssm_alpha.weight"),
                                                   ("ssm_out", "ssm_out.weight"))}
    types_.update({k: ty[f"blk.{att}.{v}"] for k, v in (("wq", "attn_q.weight"), ("wk", "attn_k.weight"),
                                                        ("wv", "attn_v.weight"), ("wo", "attn_output.weight"))})
    types_.update(embed=ty["token_embd.weight"], lm_head=ty["output.weight"], gate=ty["blk.0.ffn_gate_exps.weight"],
                  up=ty["blk.0.ffn_up_exps.weight"], down=ty["blk.0.ffn_down_exps.weight"])
    model = types.SimpleNamespace(cfg=cfg, embed=dev["token_embd.weight"], lm_head=dev["output.weight"],
                                  out_norm=dev["output_norm.weight"], layers=layers, types=types_)
    return HybridModel(plugin, model, q8=True), dev


def test_hybrid_from_gguf(plugin, port, tmp_path):
    data, _ = hybrid_model_file(port, SMALL, seed=5)
    path = tmp_path / "hybrid.gguf"
    path.write_bytes(data)
    g = Gguf(plugin, str(path))
    prompt = [5, 17, 99]
    hand, keep = _by_hand(plugin, g, SMALL)
    t_hand, l_hand = _decode(plugin, hand, prompt)
    hand.close()
    a = HybridModel.from_gguf(plugin, g, SMALL.kv_cap, q8=True)
    t_a, l_a = _decode(plugin, a, prompt)
    assert t_a == t_hand
    for x, y in zip(l_a, l_hand):
        assert np.array_equal(x, y)
    # residency tier: 24 slots of one expert each for the 64 experts of the 4 layers
    slot = 512 * 576 * 2 + 1024 * 420
    cache = ExpertCache(plugin, (slot + 4095) // 4096 * 4096, 24)
    c = HybridModel.from_gguf(plugin, g, SMALL.kv_cap, q8=True, cache=cache)
    t_c, l_c = _decode(plugin, c, prompt)
    assert t_c == t_a
    for x, y in zip(l_c, l_a):
        assert rel_l2(x, y) <= 1e-5
    resident = sum(cache.lookup(k) is not None for k in range(SMALL.n_layers * SMALL.n_experts))
    assert 0 < resident <= 24
    c.close()
    a.close()
    cache.close()
    g.close()

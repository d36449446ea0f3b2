"""Seeded synthetic inputs for the benchmark and the GPU tests.

No model files exist in this setting, so layers are synthesised as the
benchmark configurations describe them: fp32 weights ~ N(0, std) from torch's
seeded CUDA generator, encoded on the device into native GGUF blocks by the
plugin's own encoder (katali_cuda_quantize_rows), which is byte-identical to
the CPU encoder of the test oracle.

Expert store layout in HBM, per layer: three contiguous uint8 tensors
  gate [E, F * row_bytes(Q4_K, H)], up [E, F * row_bytes(Q4_K, H)],
  down [E, H * row_bytes(Q6_K, F)]
so expert e of a layer is three 16-byte-aligned slices (one per matrix).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .plugin import Q4_K, Q6_K, Plugin


def row_bytes(qtype: int, cols: int) -> int:
    return cols // 256 * (144 if qtype == Q4_K else 210)


def quantize_matrix(plugin: Plugin, qtype: int, w32: torch.Tensor) -> torch.Tensor:
    """Encode a [rows, cols] fp32 CUDA tensor into a [rows, row_bytes] uint8 tensor."""
    rows, cols = w32.shape
    out = torch.empty((rows, row_bytes(qtype, cols)), dtype=torch.uint8, device=w32.device)
    with plugin.torch_stream():  # ordered after the torch work that produced w32
        plugin.quantize_rows(qtype, w32.contiguous(), rows, cols, out)
    return out


@dataclass
class ExpertStore:
    gate: torch.Tensor  # [E, F*rbg]
    up: torch.Tensor    # [E, F*rbu]
    down: torch.Tensor  # [E, H*rbd]
    hidden: int
    ffn: int

    @property
    def n_experts(self) -> int:
        return self.gate.shape[0]

    @property
    def expert_bytes(self) -> int:
        return self.gate.shape[1] + self.up.shape[1] + self.down.shape[1]

    def pointers(self):
        E = self.n_experts
        g, u, d = self.gate.data_ptr(), self.up.data_ptr(), self.down.data_ptr()
        sg, su, sd = self.gate.shape[1], self.up.shape[1], self.down.shape[1]
        return [(g + e * sg, u + e * su, d + e * sd) for e in range(E)]


def make_expert_store(plugin: Plugin, n_experts: int, hidden: int, ffn: int, seed: int,
                      std: float = 0.02, device: str = "cuda", chunk: int = 64) -> ExpertStore:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    rbg, rbd = row_bytes(Q4_K, hidden), row_bytes(Q6_K, ffn)
    gate = torch.empty((n_experts, ffn * rbg), dtype=torch.uint8, device=device)
    up = torch.empty_like(gate)
    down = torch.empty((n_experts, hidden * rbd), dtype=torch.uint8, device=device)
    for which, dst, qt, rows, cols in (("gate", gate, Q4_K, ffn, hidden), ("up", up, Q4_K, ffn, hidden),
                                       ("down", down, Q6_K, hidden, ffn)):
        for e0 in range(0, n_experts, chunk):
            n = min(chunk, n_experts - e0)
            w = torch.randn((n * rows, cols), generator=gen, device=device, dtype=torch.float32)
            w.mul_(std)
            with plugin.torch_stream():  # ordered after randn on torch's stream
                plugin.quantize_rows(qt, w, n * rows, cols, dst[e0:e0 + n])
            del w
    return ExpertStore(gate, up, down, hidden, ffn)


def make_dense(plugin: Plugin, qtype: int, rows: int, cols: int, seed: int, std: float = 0.02,
               device: str = "cuda") -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    w = torch.randn((rows, cols), generator=gen, device=device, dtype=torch.float32).mul_(std)
    return quantize_matrix(plugin, qtype, w)


# ---------------------------------------------------------------------------
# Dense decoder (Qwen3 layout) with synthetic weights
# ---------------------------------------------------------------------------
@dataclass
class DenseConfig:
    n_layers: int
    hidden: int
    ffn: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    kv_cap: int
    rope_dim: int = 0
    rms_eps: float = 1e-6
    rope_theta: float = 1e6


# Qwen3-8B shape (36 layers, hidden 4096, FFN 12288, 32 q / 8 kv heads of 128, vocab 151936).
QWEN3_8B = DenseConfig(36, 4096, 12288, 32, 8, 128, 151936, 4096)

# "Q4_K_M"-style types: Q4_K everywhere except Q6_K for attn_v, ffn_down and the output.
DENSE_TYPES = {"wq": Q4_K, "wk": Q4_K, "wv": Q6_K, "wo": Q4_K, "gate": Q4_K, "up": Q4_K,
               "down": Q6_K, "embed": Q4_K, "lm_head": Q6_K}


@dataclass
class DenseWeights:
    cfg: DenseConfig
    embed: torch.Tensor
    lm_head: torch.Tensor
    out_norm: torch.Tensor
    layers: list
    types: dict

    @property
    def weight_bytes_per_token(self) -> int:
        """Quantised bytes one decode step reads (every matrix once, one embedding row)."""
        n = self.lm_head.numel() + self.embed.shape[1]
        for w in self.layers:
            n += sum(w[k].numel() for k in ("wq", "wk", "wv", "wo", "gate", "up", "down"))
        return n


def make_dense_model(plugin: Plugin, cfg: DenseConfig, seed: int, std: float = 0.02) -> DenseWeights:
    """Weights ~ N(0, std) encoded on the device; norm weights 1 + 0.1 N(0, 1) (fp32)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    H, F, NH, NKV, HD = cfg.hidden, cfg.ffn, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    T = DENSE_TYPES

    def mat(kind, rows, cols):
        w = torch.randn((rows, cols), generator=gen, device="cuda", dtype=torch.float32).mul_(std)
        return quantize_matrix(plugin, T[kind], w)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=gen, device="cuda", dtype=torch.float32)).contiguous()

    layers = []
    for _ in range(cfg.n_layers):
        layers.append({
            "attn_norm": norm(H), "ffn_norm": norm(H), "q_norm": norm(HD), "k_norm": norm(HD),
            "wq": mat("wq", NH * HD, H), "wk": mat("wk", NKV * HD, H), "wv": mat("wv", NKV * HD, H),
            "wo": mat("wo", H, NH * HD), "gate": mat("gate", F, H), "up": mat("up", F, H),
            "down": mat("down", H, F)})
    embed = mat("embed", cfg.vocab, H)
    lm_head = mat("lm_head", cfg.vocab, H)
    out_norm = norm(H)
    torch.cuda.synchronize()
    return DenseWeights(cfg, embed, lm_head, out_norm, layers, dict(T))


# ---------------------------------------------------------------------------
# Hybrid MoE decoder (Gated DeltaNet + gated attention, MoE every layer)
# ---------------------------------------------------------------------------
@dataclass
class HybridConfig:
    n_layers: int
    hidden: int
    vocab: int
    kv_cap: int
    n_heads: int          # gated attention: query heads
    n_kv_heads: int
    head_dim: int
    rope_dim: int         # RoPE on the first rope_dim dimensions of a head
    ssm_k_heads: int      # GDN: q/k heads
    ssm_v_heads: int      # GDN: value heads (a multiple of ssm_k_heads)
    ssm_head_dim: int     # dk = dv
    ssm_conv: int         # causal conv kernel
    n_experts: int
    ffn: int              # expert FFN
    top_k: int
    attn_every: int = 4   # layer l is full attention when (l + 1) % attn_every == 0
    rms_eps: float = 1e-6
    rope_theta: float = 1e7

    def kind(self, l: int) -> int:
        return 1 if (l + 1) % self.attn_every == 0 else 0


# 35B-A3B class (config 5): 40 layers = 30 GDN + 10 gated attention, hidden 2048, MoE every
# layer as config 2 (256 experts, FFN 512, top-8, renormalised top-k weights). Mixer
# dimensions follow the Qwen3.5 / Qwen3-Next family: GDN 16 q/k heads and 32 value heads of
# 128, conv kernel 4; attention 16 q / 2 kv heads of 256 with RoPE on 64 dims (theta 1e7);
# vocab 248320.
HYBRID_35B = HybridConfig(n_layers=40, hidden=2048, vocab=248320, kv_cap=4096, n_heads=16,
                          n_kv_heads=2, head_dim=256, rope_dim=64, ssm_k_heads=16,
                          ssm_v_heads=32, ssm_head_dim=128, ssm_conv=4, n_experts=256, ffn=512,
                          top_k=8)

HYBRID_TYPES = {"ssm_qkv": Q4_K, "ssm_z": Q4_K, "ssm_b": Q4_K, "ssm_a": Q4_K, "ssm_out": Q4_K,
                "wq": Q4_K, "wk": Q4_K, "wv": Q6_K, "wo": Q4_K, "embed": Q4_K, "lm_head": Q6_K,
                "gate": Q4_K, "up": Q4_K, "down": Q6_K}


@dataclass
class HybridWeights:
    cfg: HybridConfig
    embed: torch.Tensor
    lm_head: torch.Tensor
    out_norm: torch.Tensor
    layers: list          # dicts of device tensors; "experts" holds the layer's ExpertStore
    types: dict

    @property
    def weight_bytes_per_token(self) -> int:
        """Weight bytes one decode step reads: every mixer matrix and router once, the
        top_k selected experts of every layer, the LM head and one embedding row."""
        c = self.cfg
        n = self.lm_head.numel() + self.embed.shape[1]
        for w in self.layers:
            keys = ("ssm_qkv", "ssm_z", "ssm_b", "ssm_a", "ssm_out", "ssm_conv") if w["kind"] == 0 \
                else ("wq", "wk", "wv", "wo")
            n += sum(w[k].numel() * w[k].element_size() for k in keys)
            n += w["router"].numel() * 4 + c.top_k * w["experts"].expert_bytes  # top_k experts read
        return n

    @property
    def state_bytes_per_token(self) -> int:
        """Recurrent-state bytes one decode step reads and writes (GDN states)."""
        c = self.cfg
        n_gdn = sum(1 for w in self.layers if w["kind"] == 0)
        return 2 * n_gdn * c.ssm_v_heads * c.ssm_head_dim * c.ssm_head_dim * 4


def make_hybrid_model(plugin: Plugin, cfg: HybridConfig, seed: int, std: float = 0.02,
                      ep: tuple | None = None) -> HybridWeights:
    """GGUF matrices ~ N(0, std) encoded on the device; fp32 router rows ~ N(0, std); norm
    weights 1 + 0.1 N(0, 1); conv taps N(0, 0.3); A_log = log U(1, 16); dt_bias U(-4, -2).
    ep = (n_ranks, rank): only this rank's block of n_experts / n_ranks experts per layer is
    generated (seeded by layer and block, so the ranks together hold one consistent model;
    the mixer, router and LM-head weights depend on `seed` only)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    H, T = cfg.hidden, HYBRID_TYPES
    C = (2 * cfg.ssm_k_heads + cfg.ssm_v_heads) * cfg.ssm_head_dim
    VD = cfg.ssm_v_heads * cfg.ssm_head_dim
    QD, KD = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim

    def randn(*shape, s=1.0):
        return torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).mul_(s)

    def mat(kind, rows, cols):
        return quantize_matrix(plugin, T[kind], randn(rows, cols, s=std))

    def norm(n):
        return (1.0 + 0.1 * randn(n)).contiguous()

    def uniform(n, lo, hi):
        return (lo + (hi - lo) * torch.rand(n, generator=gen, device="cuda")).contiguous()

    layers = []
    for l in range(cfg.n_layers):
        w = {"kind": cfg.kind(l), "attn_norm": norm(H), "ffn_norm": norm(H),
             "router": randn(cfg.n_experts, H, s=std).contiguous()}
        if w["kind"] == 0:
            w.update({"ssm_qkv": mat("ssm_qkv", C, H), "ssm_z": mat("ssm_z", VD, H),
                      "ssm_b": mat("ssm_b", cfg.ssm_v_heads, H), "ssm_a": mat("ssm_a", cfg.ssm_v_heads, H),
                      "ssm_out": mat("ssm_out", H, VD),
                      "ssm_conv": randn(C, cfg.ssm_conv, s=0.3).contiguous(),
                      "ssm_a_log": torch.log(uniform(cfg.ssm_v_heads, 1.0, 16.0)).contiguous(),
                      "ssm_dt_bias": uniform(cfg.ssm_v_heads, -4.0, -2.0),
                      "ssm_norm": norm(cfg.ssm_head_dim)})
        else:
            w.update({"wq": mat("wq", 2 * QD, H), "wk": mat("wk", KD, H), "wv": mat("wv", KD, H),
                      "wo": mat("wo", H, QD), "q_norm": norm(cfg.head_dim),
                      "k_norm": norm(cfg.head_dim)})
        if ep is None:
            w["experts"] = make_expert_store(plugin, cfg.n_experts, H, cfg.ffn, seed=seed * 1000 + l, std=std)
            w["expert_base"] = 0
        else:
            G, r = ep
            per = cfg.n_experts // G
            w["experts"] = make_expert_store(plugin, per, H, cfg.ffn, seed=(seed * 1000 + l) * 64 + r, std=std)
            w["expert_base"] = r * per
        layers.append(w)
    embed = mat("embed", cfg.vocab, H)
    lm_head = mat("lm_head", cfg.vocab, H)
    out_norm = norm(H)
    torch.cuda.synchronize()
    return HybridWeights(cfg, embed, lm_head, out_norm, layers, dict(T))


def hybrid_ep_view(model: HybridWeights, n_ranks: int, rank: int) -> HybridWeights:
    """The same model with only rank's block of every layer's experts (views of the full
    stores): what one rank of an expert-parallel decoder holds."""
    per = model.cfg.n_experts // n_ranks
    layers = []
    for w in model.layers:
        st = w["experts"]
        sl = slice(rank * per, (rank + 1) * per)
        v = dict(w)
        v["experts"] = ExpertStore(st.gate[sl], st.up[sl], st.down[sl], st.hidden, st.ffn)
        v["expert_base"] = rank * per
        layers.append(v)
    return HybridWeights(model.cfg, model.embed, model.lm_head, model.out_norm, layers, model.types)

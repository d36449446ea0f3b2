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

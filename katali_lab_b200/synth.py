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

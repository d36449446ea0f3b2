"""Closed-form byte counts of the benchmark configurations (no GPU).

The roofline numerators in bench.py and the synthetic model shapes in
katali_lab_b200.synth must agree with the per-unit figures of the configurations:
C1 7,077,888 B of Q4_K per GEMV call, C2 2,039,808 B per expert and 16,318,464 B per
top-8 call, C4 122,585,088 B per layer and 4,923,568,128 B per token, C5 30 GDN + 10
attention layers with 652,738,560 B of experts per token.
"""
import bench
from katali_lab_b200.plugin import Q4_K, Q6_K
from katali_lab_b200.synth import DENSE_TYPES, HYBRID_35B, QWEN3_8B, row_bytes


def test_block_sizes():
    assert row_bytes(Q4_K, 256) == 144 and row_bytes(Q6_K, 256) == 210
    assert row_bytes(Q4_K, 2048) == 8 * 144 and row_bytes(Q6_K, 512) == 2 * 210


def test_c1_c2_numerators():
    assert bench.C1_BYTES == 6144 * row_bytes(Q4_K, 2048) == 7_077_888
    expert = 2 * 512 * row_bytes(Q4_K, 2048) + 2048 * row_bytes(Q6_K, 512)
    assert bench.EXPERT_BYTES == expert == 2_039_808
    assert bench.CALL_BYTES == 8 * expert == 16_318_464


def test_c4_bytes_per_token():
    c, T = QWEN3_8B, DENSE_TYPES
    H, F, q, kv = c.hidden, c.ffn, c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
    layer = (q * row_bytes(T["wq"], H) + kv * row_bytes(T["wk"], H) + kv * row_bytes(T["wv"], H)
             + H * row_bytes(T["wo"], q) + F * row_bytes(T["gate"], H) + F * row_bytes(T["up"], H)
             + H * row_bytes(T["down"], F))
    assert layer == 122_585_088
    lm_head = c.vocab * row_bytes(T["lm_head"], H)
    assert lm_head == 510_504_960
    assert c.n_layers * layer + lm_head == 4_923_568_128


def test_c5_layer_mix_and_expert_bytes():
    c = HYBRID_35B
    kinds = [c.kind(l) for l in range(c.n_layers)]
    assert kinds.count(0) == 30 and kinds.count(1) == 10
    assert c.ssm_v_heads % c.ssm_k_heads == 0
    assert c.n_layers * c.top_k * bench.EXPERT_BYTES == 652_738_560


def test_hybrid_ep_view_partitions_every_layers_experts():
    """Each rank's view holds the contiguous block [r E/G, (r+1) E/G) of every layer's
    experts, as views of the full store, and the blocks of all ranks tile the store."""
    import torch
    from dataclasses import replace
    from katali_lab_b200.synth import ExpertStore, HybridWeights, hybrid_ep_view
    cfg = replace(HYBRID_35B, n_layers=2, n_experts=16)
    layers = []
    for l in range(cfg.n_layers):
        st = ExpertStore(torch.arange(16 * 4, dtype=torch.uint8).view(16, 4) + l,
                         torch.zeros(16, 4, dtype=torch.uint8), torch.zeros(16, 2, dtype=torch.uint8),
                         cfg.hidden, cfg.ffn)
        layers.append({"kind": cfg.kind(l), "experts": st})
    full = HybridWeights(cfg, None, None, None, layers, {})
    for G in (1, 2, 4, 8):
        seen = [[] for _ in range(cfg.n_layers)]
        for r in range(G):
            v = hybrid_ep_view(full, G, r)
            for l, w in enumerate(v.layers):
                st = w["experts"]
                assert st.n_experts == 16 // G and w["expert_base"] == r * (16 // G)
                assert st.gate.data_ptr() == layers[l]["experts"].gate[r * (16 // G)].data_ptr()
                assert st.expert_bytes == layers[l]["experts"].expert_bytes
                seen[l].extend(st.gate[:, 0].tolist())
        for l in range(cfg.n_layers):
            assert seen[l] == layers[l]["experts"].gate[:, 0].tolist()

"""katali_cuda_moe_layer_static: the MoE layer for callers that cannot allocate.

Hosts whose device memory is owned by another allocator, or that may not allocate
once a layer runs, call this entry point instead of katali_cuda_moe_layer; it keeps
its scratch in a fixed device array inside the library. This checks, through the C
ABI, that calls in a row give bit-for-bit the output of the allocating entry point
(the same kernel, deterministic), that the q8_1 output matches the C restatement of
the layer, and that a layer larger than the fixed array is refused. Collected last
(zz) so a failure here cannot stop the rest of the GPU suite.
"""
import ctypes as C

import numpy as np
import pytest

from katali_lab_b200 import MOE_NORM_TOPK, MOE_Q8_1, MOE_F32, Q4_K, Q6_K, MoeLayer
from katali_lab_b200.plugin import KataliMoeDesc
from katali_lab_b200.synth import make_expert_store
from oracle.oracle import MoeWeights, rel_l2

pytestmark = pytest.mark.gpu


def _desc(store, top_k, flat):
    return KataliMoeDesc(store.n_experts, store.hidden, store.ffn, top_k, Q4_K, Q4_K, Q6_K,
                         MOE_NORM_TOPK, C.cast(flat, C.POINTER(C.c_void_p)))


def test_static_entry_matches_allocating_entry(plugin, port):
    import torch
    E, H, F, K = 64, 2048, 512, 8
    store = make_expert_store(plugin, E, H, F, seed=61)
    ptrs = store.pointers()
    layer = MoeLayer(plugin, E, H, F, K, ptrs)
    flat = (C.c_void_p * (3 * E))(*[a for tri in ptrs for a in tri])
    desc = _desc(store, K, flat)
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(62)
    for call, mode in enumerate((MOE_Q8_1, MOE_Q8_1, MOE_F32, MOE_F32)):
        x = torch.randn(H, generator=g, device="cuda")
        logits = torch.randn(E, generator=g, device="cuda")
        y_ref = torch.empty(H, device="cuda")
        y = torch.full((H,), float("nan"), device="cuda")
        layer.forward(x, logits, y_ref, mode)
        rc = plugin.L.katali_cuda_moe_layer_static(C.byref(desc), x.data_ptr(), logits.data_ptr(),
                                                   y.data_ptr(), mode, stream)
        assert rc == 0, plugin.status()
        a, b = y.cpu().numpy(), y_ref.cpu().numpy()
        assert np.all(np.isfinite(a)), f"call {call}"
        assert np.array_equal(a, b), f"call {call}: rel_L2 {rel_l2(a, b)}"
        if call == 1:  # the second q8_1 call against the restatement (bar of test_gpu_moe)
            host = MoeWeights(store.gate.cpu().numpy(), store.up.cpu().numpy(),
                              store.down.cpu().numpy(), H, F, K)
            want, _, _, _ = port.moe_layer(host, x.cpu().numpy(), logits.cpu().numpy(), mode=0)
            assert rel_l2(a, want) <= 1e-5, f"restatement rel_L2 {rel_l2(a, want)}"
    layer.close()


def test_static_entry_rejects_layers_beyond_its_array(plugin):
    import torch
    store = make_expert_store(plugin, 8, 256, 4096, seed=63)  # top_k * ffn = 8 * 4096 = 32768 > 16384
    flat = (C.c_void_p * 24)(*[a for tri in store.pointers() for a in tri])
    desc = _desc(store, 8, flat)
    x = torch.zeros(256, device="cuda")
    lg = torch.zeros(8, device="cuda")
    y = torch.zeros(256, device="cuda")
    rc = plugin.L.katali_cuda_moe_layer_static(C.byref(desc), x.data_ptr(), lg.data_ptr(),
                                               y.data_ptr(), MOE_Q8_1, None)
    assert rc == 5  # KATALI_ERR_UNSUPPORTED_SHAPE
    assert "exceed the static scratch" in plugin.status()

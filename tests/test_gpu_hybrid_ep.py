"""The hybrid MoE decoder with expert-parallel MoE blocks across GPUs: two (or four)
processes, one GPU each, each decoding its own sequence while holding 1/G of every layer's
experts; each layer's MoE block runs as the single-launch expert-parallel layer over NVLink
peer memory (katali_cuda_hybrid_set_ep). Bar: at every step, each rank's logits within
rel_L2 <= 1e-5 of the same decoder with all experts on its own GPU (q8_1 activations; only
the association of the per-rank double partial sums differs) and the same greedy tokens.
Skipped with fewer than two GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest

from katali_lab_b200.synth import HybridConfig

pytestmark = pytest.mark.gpu

CFG = HybridConfig(n_layers=4, hidden=2048, vocab=4096, kv_cap=64, n_heads=4, n_kv_heads=2,
                   head_dim=256, rope_dim=64, ssm_k_heads=2, ssm_v_heads=4, ssm_head_dim=128,
                   ssm_conv=4, n_experts=16, ffn=512, top_k=8)
STEPS = 10


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _logits(hm, vocab):
    ptr, _ = hm.logits()
    out = np.empty(vocab, np.float32)
    hm.p.check(hm.p.L.katali_cuda_download(out.ctypes.data, ptr, out.nbytes))
    return out


def _rank(rank, world, port_no, out_dir):
    import torch
    import torch.distributed as dist

    from katali_lab_b200 import HybridModel, Plugin
    from katali_lab_b200.ep import EpComm
    from katali_lab_b200.synth import hybrid_ep_view, make_hybrid_model

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    comm = hm_ep = hm_full = None
    try:
        plugin = Plugin()
        full = make_hybrid_model(plugin, CFG, seed=77)  # the same model on every rank
        hm_full = HybridModel(plugin, full, q8=True)
        hm_ep = HybridModel(plugin, hybrid_ep_view(full, world, rank), q8=True)
        comm = EpComm.from_process_group(plugin)
        comm.use_peer_memory(True)
        hm_ep.set_ep(comm)
        tok_e = tok_f = 3 + 11 * rank  # every rank its own sequence
        toks_e, toks_f, errs = [], [], []
        for _ in range(STEPS):
            tok_e = int(hm_ep.generate([tok_e], 1)[0])
            tok_f = int(hm_full.generate([tok_f], 1)[0])
            le, lf = _logits(hm_ep, CFG.vocab), _logits(hm_full, CFG.vocab)
            errs.append(float(np.sqrt(((le.astype(np.float64) - lf) ** 2).sum() / (lf.astype(np.float64) ** 2).sum())))
            toks_e.append(tok_e)
            toks_f.append(tok_f)
        # a second sequence after reset (the recurrent and conv states cleared on every rank)
        hm_ep.reset()
        hm_full.reset()
        again_e = hm_ep.generate([5 + rank], 6).tolist()
        again_f = hm_full.generate([5 + rank], 6).tolist()
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), toks_e=np.array(toks_e),
                 toks_f=np.array(toks_f), errs=np.array(errs), again_e=np.array(again_e),
                 again_f=np.array(again_f))
    finally:
        for h in (hm_ep, hm_full):
            if h is not None:
                h.close()
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_hybrid_ep_multi_gpu(tmp_path):
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 4 if n >= 4 else 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    for r in range(world):
        d = np.load(tmp_path / f"r{r}.npz")
        assert d["errs"].max() <= 1e-5, (r, d["errs"])
        assert d["toks_e"].tolist() == d["toks_f"].tolist(), r
        assert d["again_e"].tolist() == d["again_f"].tolist(), r

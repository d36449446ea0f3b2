"""Expert parallelism across GPUs: two (or four) processes, one GPU each.

Each rank holds half of the experts and brings its own tokens; the layer runs with
torch.distributed's all_to_all_single as the exchange, with the plugin's own NCCL
communicator (katali_cuda_moe_ep_layer), and twice with the exchange over NVLink peer
memory inside the kernels (katali_cuda_ep_use_peer_memory; both window parities). Bar: every token's output
within rel_L2 <= 1e-5 of katali_cuda_moe_batch on the full layer on the same GPU and
>= 99.9 % of elements bit-equal. Skipped with fewer than two GPUs; four ranks on a box with four GPUs or more."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

E, H, F, K = 64, 2048, 512, 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port_no, out_dir):
    import torch
    import torch.distributed as dist

    from katali_lab_b200 import Plugin
    from katali_lab_b200.ep import EpComm, EpMoeLayer, local_experts, torch_exchange
    from tests.test_gpu_moe import DevLayer, dev, empty, host

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    comm = None
    try:
        plugin = Plugin()
        full = DevLayer(plugin, E, H, F, K, seed=61)
        # world 2: 12 slots; world 4: 16 slots (both within the single-launch peer-memory layer)
        T, tmax = ([5, 3][rank], 6) if world == 2 else ([4, 3, 2, 4][rank], 4)
        rng = np.random.default_rng(300 + rank)
        X = rng.normal(0, 1, (T, H)).astype(np.float32)
        L = rng.normal(0, 1, (T, E)).astype(np.float32)
        ep = EpMoeLayer(plugin, E, H, F, K, [full.ptrs[e] for e in local_experts(E, world, rank)],
                        world, rank, tmax)
        x, lg = dev(X), dev(L)
        y1 = empty(T * H).view(T, H)
        ep.forward(x, lg, y1, exchange=torch_exchange())
        comm = EpComm.from_process_group(plugin)
        y2 = empty(T * H).view(T, H)
        ep.forward(x, lg, y2, comm=comm)
        comm.use_peer_memory(True)  # the same layer over NVLink peer memory, both parities
        y3 = empty(T * H).view(T, H)
        ep.forward(x, lg, y3, comm=comm)
        y4 = empty(T * H).view(T, H)
        ep.forward(x, lg, y4, comm=comm)
        want = empty(T * H).view(T, H)
        full.layer.forward_batch(x, lg, want)
        torch.cuda.synchronize()
        store_sum = [int(b.sum(dtype=torch.int64)) for b in full.bufs]
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), y1=host(y1), y2=host(y2), y3=host(y3),
                 y4=host(y4), want=host(want), store_sum=np.array(store_sum))
        ep.close()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_ep_multi_gpu(tmp_path):
    """Two ranks, or four when the box has four GPUs or more."""
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 4 if n >= 4 else 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    from oracle.oracle import rel_l2
    sums = [np.load(tmp_path / f"r{r}.npz")["store_sum"] for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(sums[0], sums[r]), "the ranks built different expert stores"
    for r in range(world):
        d = np.load(tmp_path / f"r{r}.npz")
        for key in ("y1", "y2", "y3", "y4"):
            for t in range(d["want"].shape[0]):
                assert rel_l2(d[key][t], d["want"][t]) <= 1e-5, (r, key, t)
                assert np.mean(d[key][t] == d["want"][t]) >= 0.999, (r, key, t)

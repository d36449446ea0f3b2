"""Expert-parallel host logic on the CPU: the slot protocol restated in the oracle,
driven by katali_lab_b200.ep.ep_step, over virtual ranks in one process and over two
gloo ranks. Bar: every token's output within rel_L2 <= 1e-5 of the single-process
q8_1 restatement (port.moe_layer) and >= 99.9 % of elements bit-equal."""
import os
import socket

import numpy as np
import pytest
import torch

from katali_lab_b200.ep import ep_step, experts_per_rank, local_experts, owner
from oracle.oracle import Port, make_moe_weights, rel_l2
from tests.ep_oracle_stages import OracleStages, local_exchange

E, H, F, K = 16, 256, 256, 4


def tokens(seed, T, E_=E):
    rng = np.random.default_rng(seed)
    return (rng.normal(0, 1, (T, H)).astype(np.float32),
            rng.normal(0, 1, (T, E_)).astype(np.float32))


def check_against_oracle(port, layer, X, L, Y):
    for t in range(X.shape[0]):
        want, _, _, _ = port.moe_layer(layer, X[t], L[t], mode=0)
        assert rel_l2(Y[t], want) <= 1e-5, t
        assert np.mean(Y[t] == want) >= 0.999, t


def test_partition_helpers():
    assert experts_per_rank(256, 8) == 32
    assert owner(255, 256, 8) == 7 and owner(31, 256, 8) == 0 and owner(32, 256, 8) == 1
    assert list(local_experts(16, 4, 2)) == [8, 9, 10, 11]
    with pytest.raises(ValueError):
        experts_per_rank(10, 4)


def test_slot_bytes(port):
    assert port.ep_slot_bytes(2048, 8) == 80 + 2304  # header 16 + 8*8, q8_1 row 64 x 36 B
    assert port.ep_slot_bytes(256, 5) == 64 + 288    # 16 + 40 -> 64


@pytest.mark.parametrize("G,Ts", [(2, [3, 1]), (4, [2, 0, 5, 1])])
def test_virtual_ranks(port, G, Ts):
    layer = make_moe_weights(port, E, H, F, seed=41, top_k=K)
    tmax = max(max(Ts), 1)
    stages = [OracleStages(port, layer, G, r, tmax) for r in range(G)]
    ins = [tokens(100 + r, T) for r, T in enumerate(Ts)]
    sends = [stages[r].dispatch(Ts[r], *ins[r]) for r in range(G)]
    recvs = local_exchange(sends, G)
    rets = [stages[r].experts(recvs[r]) for r in range(G)]
    backs = local_exchange(rets, G)
    for r in range(G):
        y = np.zeros((Ts[r], H), np.float32)
        stages[r].combine(Ts[r], backs[r], y)
        check_against_oracle(port, layer, ins[r][0], ins[r][1], y)


def test_dispatch_slots(port):
    """Headers carry owned ids only; the row is present exactly when a pair is owned."""
    layer = make_moe_weights(port, E, H, F, seed=42, top_k=K)
    X, L = tokens(7, 3)
    L[1, :] = -5.0
    L[1, [0, 1, 2, 3]] = 5.0  # token 1 entirely on rank 0 of 2
    send, src = port.ep_dispatch(layer, 2, 4, X, L)
    sb = port.ep_slot_bytes(H, K)
    slots = send.reshape(2, 4, sb)
    hdr = slots[:, :, :16].copy().view(np.int32).reshape(2, 4, 4)
    ids = slots[:, :, 16:16 + 4 * K].copy().view(np.int32).reshape(2, 4, K)
    assert hdr[0, 1, 0] == 4 and hdr[1, 1, 0] == 0
    assert (hdr[:, 3, 0] == 0).all()  # t >= n_tokens: empty
    for t in range(3):
        for d in range(2):
            own = [e for e in src[t] if e // (E // 2) == d]
            assert hdr[d, t, 0] == len(own)
            assert [e for e in ids[d, t] if e >= 0] == own


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port_no, out_dir):
    import torch.distributed as dist

    from katali_lab_b200.ep import torch_exchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_no))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        port = Port()
        layer = make_moe_weights(port, E, H, F, seed=43, top_k=K)
        T = [5, 2][rank]
        X, L = tokens(200 + rank, T)
        st = OracleStages(port, layer, world, rank, max_tokens=6)
        y = np.zeros((T, H), np.float32)
        ep_step(st, torch_exchange(), T, X, L, y)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), X=X, L=L, y=y)
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks(port, tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_gloo_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    layer = make_moe_weights(port, E, H, F, seed=43, top_k=K)
    for r in range(2):
        d = np.load(tmp_path / f"r{r}.npz")
        check_against_oracle(port, layer, d["X"], d["L"], d["y"])

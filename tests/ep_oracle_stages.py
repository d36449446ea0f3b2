"""The expert-parallel stages restated on the CPU (oracle kqo_ep_*), shaped like
katali_lab_b200.ep.EpMoeLayer so that katali_lab_b200.ep.ep_step drives either.
Test infrastructure: buffers are CPU torch tensors, so torch.distributed gloo can
exchange them."""
import numpy as np
import torch

from oracle.oracle import MoeWeights, Port


class OracleStages:
    def __init__(self, port: Port, layer: MoeWeights, n_ranks: int, rank: int, max_tokens: int):
        self.port, self.layer = port, layer
        self.n_ranks, self.rank, self.max_tokens = n_ranks, rank, max_tokens
        self.src_ids = None

    def dispatch(self, n_tokens, x, logits):
        send, self.src_ids = self.port.ep_dispatch(self.layer, self.n_ranks, self.max_tokens,
                                                   np.asarray(x)[:n_tokens],
                                                   np.asarray(logits)[:n_tokens])
        return torch.from_numpy(send)

    def experts(self, recv):
        ret = self.port.ep_experts(self.layer, self.n_ranks, self.rank, self.max_tokens,
                                   recv.numpy())
        return torch.from_numpy(ret)

    def combine(self, n_tokens, back, y):
        y[:n_tokens] = self.port.ep_combine(self.layer, self.n_ranks, self.max_tokens,
                                            self.src_ids[:n_tokens], back.numpy())
        return y


def local_exchange(sends_by_rank, n_ranks):
    """All-to-all among virtual ranks in one process: in_r[d] = out_d[r]."""
    chunks = [torch.chunk(s, n_ranks) for s in sends_by_rank]
    return [torch.cat([chunks[d][r] for d in range(n_ranks)]) for r in range(n_ranks)]

"""Expert-parallel MoE layer on the host side: one process per GPU.

Experts of a layer are split over the ranks in contiguous blocks of
n_experts / n_ranks (rank r owns [r*per, (r+1)*per)). Every rank brings its own
tokens. One layer call is three plugin stages around two all-to-all exchanges of
fixed-size slots (katali_cuda_moe_ep_dispatch / _experts / _combine):

    dispatch  route + q8_1 + one slot per (destination rank, token) -> send
    exchange  recv[d] = what rank d sent here
    experts   every received slot's pairs on this rank's experts  -> ret
    exchange  back[d] = what rank d returned for this rank's tokens
    combine   y[t] = sum over ranks (rank order) of back[d][t]

`ep_step` is that sequence for any stage implementation and any exchange (NCCL
through torch.distributed, the plugin's own NCCL communicator, or gloo on the
CPU with the test oracle's restatement of the stages). The slot capacity is
fixed (max_tokens per rank), so no counts are exchanged and a call can be
captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes as C

from .plugin import MoeLayer, Plugin, _ptr

_vp = C.c_void_p


def experts_per_rank(n_experts: int, n_ranks: int) -> int:
    if n_ranks <= 0 or n_experts % n_ranks:
        raise ValueError(f"{n_experts} experts do not split over {n_ranks} ranks")
    return n_experts // n_ranks


def owner(expert: int, n_experts: int, n_ranks: int) -> int:
    return expert // experts_per_rank(n_experts, n_ranks)


def local_experts(n_experts: int, n_ranks: int, rank: int) -> range:
    per = experts_per_rank(n_experts, n_ranks)
    return range(rank * per, (rank + 1) * per)


def ep_step(stages, exchange, n_tokens, x, logits, y):
    """One expert-parallel layer call. stages: dispatch(n_tokens, x, logits) -> send,
    experts(recv) -> ret, combine(n_tokens, back, y); exchange(out, kind) -> in, where
    kind is "slots" or "partials" and `in[d]` is what rank d sent to this rank."""
    send = stages.dispatch(n_tokens, x, logits)
    recv = exchange(send, "slots")
    ret = stages.experts(recv)
    back = exchange(ret, "partials")
    return stages.combine(n_tokens, back, y)


def torch_exchange(group=None):
    """An exchange over torch.distributed all_to_all_single (NCCL for CUDA tensors,
    gloo for CPU tensors); the output buffer is allocated per call."""
    import torch
    import torch.distributed as dist

    def ex(out, kind):
        inp = torch.empty_like(out)
        dist.all_to_all_single(inp, out, group=group)
        return inp
    return ex


class EpComm:
    """The plugin's own NCCL communicator (katali_cuda_ep_create)."""

    def __init__(self, plugin: Plugin, n_ranks: int, rank: int, unique_id: bytes):
        if len(unique_id) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        self.p = plugin
        buf = C.create_string_buffer(unique_id, 128)
        h = _vp()
        plugin.check(plugin.L.katali_cuda_ep_create(n_ranks, rank, buf, C.byref(h)))
        self.h = h
        self.n_ranks, self.rank = n_ranks, rank

    @staticmethod
    def unique_id(plugin: Plugin) -> bytes:
        buf = C.create_string_buffer(128)
        plugin.check(plugin.L.katali_cuda_ep_unique_id(buf))
        return buf.raw

    @classmethod
    def from_process_group(cls, plugin: Plugin, group=None) -> "EpComm":
        """Rank 0 makes the id; torch.distributed broadcasts it (any backend)."""
        import torch.distributed as dist
        rank, n = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id(plugin) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(plugin, n, rank, obj[0])

    def use_peer_memory(self, on: bool = True) -> None:
        """Exchange over NVLink peer memory inside the kernels instead of NCCL (the windows
        are mapped by the next layer call, collectively)."""
        self.p.check(self.p.L.katali_cuda_ep_use_peer_memory(self.h, int(on)))

    def close(self) -> None:
        if self.h:
            self.p.L.katali_cuda_ep_destroy(self.h)
            self.h = None


class EpMoeLayer:
    """This rank's share of one expert-parallel MoE layer (device buffers in torch)."""

    def __init__(self, plugin: Plugin, n_experts, hidden, ffn, top_k, local_ptrs, n_ranks,
                 rank, max_tokens, norm_topk=True, **types):
        """local_ptrs: (gate, up, down) device addresses of experts local_experts(...)."""
        import torch
        rng = local_experts(n_experts, n_ranks, rank)
        if len(local_ptrs) != len(rng):
            raise ValueError(f"rank {rank} holds {len(rng)} experts, got {len(local_ptrs)}")
        table = [(0, 0, 0)] * n_experts
        for e, ptrs in zip(rng, local_ptrs):
            table[e] = tuple(int(a) for a in ptrs)
        self.p = plugin
        self.layer = MoeLayer(plugin, n_experts, hidden, ffn, top_k, table, norm_topk, **types)
        self.n_ranks, self.rank, self.max_tokens, self.hidden = n_ranks, rank, max_tokens, hidden
        sb, rb = C.c_uint64(), C.c_uint64()
        plugin.check(plugin.L.katali_cuda_moe_ep_slot_bytes(self.layer.h, C.byref(sb), C.byref(rb)))
        self.slot_bytes, self.ret_slot_bytes = sb.value, rb.value
        n = n_ranks * max_tokens
        self.send = torch.empty(n * self.slot_bytes, dtype=torch.uint8, device="cuda")
        self.ret = torch.empty(n * hidden, dtype=torch.float64, device="cuda")

    # -- the three stages --------------------------------------------------
    def dispatch(self, n_tokens, x, logits):
        self.p.check(self.p.L.katali_cuda_moe_ep_dispatch(
            self.layer.h, self.n_ranks, self.max_tokens, n_tokens, _ptr(x), _ptr(logits),
            _ptr(self.send)))
        return self.send

    def experts(self, recv):
        self.p.check(self.p.L.katali_cuda_moe_ep_experts(
            self.layer.h, self.n_ranks, self.rank, self.max_tokens, _ptr(recv), _ptr(self.ret)))
        return self.ret

    def combine(self, n_tokens, back, y):
        self.p.check(self.p.L.katali_cuda_moe_ep_combine(
            self.layer.h, self.n_ranks, self.max_tokens, n_tokens, _ptr(back), _ptr(y)))
        return y

    # -- one call ------------------------------------------------------------
    def forward(self, x, logits, y, n_tokens=None, exchange=None, comm: EpComm | None = None):
        """exchange: an `ep_step` exchange (e.g. torch_exchange()); comm: the plugin's
        NCCL communicator (katali_cuda_moe_ep_layer). Exactly one of the two."""
        T = int(x.shape[0]) if n_tokens is None else int(n_tokens)
        if comm is not None:
            with self.p.torch_stream():
                self.p.check(self.p.L.katali_cuda_moe_ep_layer(
                    self.layer.h, comm.h, self.max_tokens, T, _ptr(x), _ptr(logits), _ptr(y)))
            return y
        if exchange is None:
            raise ValueError("give an exchange or a communicator")
        # torch's collectives complete on torch's current stream: run the stages there
        # so each one sees the exchange before it.
        with self.p.torch_stream():
            return ep_step(self, exchange, T, x, logits, y)

    def close(self) -> None:
        self.layer.close()

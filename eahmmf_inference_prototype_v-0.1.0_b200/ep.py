"""Expert-parallel MoE layer: the experts of one layer sharded across ranks, tokens
dispatched to the ranks that own their routed experts and the expert outputs combined back, over
torch.distributed all-to-all (NCCL over NVLink on GPUs; gloo on CPU for the host-logic tests).

Per call, on every rank (one process per GPU, each holding its own tokens):

  1. routing of the local tokens (eahmmf_cuda_route_topk: the reference's top-k, qwen3moe.cpp:1011-1023);
  2. count exchange, then dispatch: each routed (token, k) slot sends its fp32 activation row and the
     owner-local expert id to rank e // (E / P), slots ordered by destination rank;
  3. the received rows go through the rank's experts (the MoE block with k = 1 and one-hot logits: the
     assigned expert's gate/up/SiLU/down with weight exactly 1 added to a zero row, i.e. y itself);
  4. the outputs return by the inverse all-to-all;
  5. the weighted combine in ascending expert order into the residual (eahmmf_cuda_moe_combine), the
     reference's summation order (qwen3moe.cpp:1025-1069).

Every slot's output depends only on its own row, so the result equals the single-GPU layer's up to the
kernel path (GEMV or grouped) that each rank picks for its batch size.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def shard(ex, rank: int, world: int):
    """The experts [rank E/P, (rank + 1) E/P) of an ExpertSet."""
    import synth
    E = ex.n_expert
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    n = E // world
    sl = slice(rank * n, (rank + 1) * n)
    return synth.ExpertSet(D=ex.D, FF=ex.FF, n_expert=n, types=ex.types, gate=ex.gate[sl], up=ex.up[sl],
                           down=ex.down[sl])


class _CudaExperts:
    """Applies each received row's assigned local expert with the device MoE block (k = 1)."""

    def __init__(self, local, device):
        import eahmmf_b200 as eb
        self.eb = eb
        self.layer = eb.MoeLayer.from_expert_set(local, n_used=1)
        self.E = local.n_expert
        self.device = device
        self.ws = None
        self.ws_T = 0

    def __call__(self, rows: torch.Tensor, eid: torch.Tensor) -> torch.Tensor:
        R = rows.shape[0]
        y = torch.zeros_like(rows)
        if R == 0:
            return y
        if R > self.ws_T:
            self.ws = torch.empty(self.layer.workspace_bytes(R), dtype=torch.uint8, device=self.device)
            self.ws_T = R
        onehot = torch.full((R, self.E), float("-inf"), dtype=torch.float32, device=self.device)
        onehot[torch.arange(R, device=self.device), eid.long()] = 0.0
        rc = self.layer(R, rows.contiguous(), onehot, y, self.ws)
        if rc:
            raise RuntimeError(f"eahmmf_cuda_moe_layer returned {rc}")
        return y


class _CpuExperts:
    """The same through the CPU oracle (host-logic tests on gloo)."""

    def __init__(self, local):
        import oracle
        self.orc = oracle.Oracle()
        self.local = local

    def __call__(self, rows: torch.Tensor, eid: torch.Tensor) -> torch.Tensor:
        R = rows.shape[0]
        if R == 0:
            return torch.zeros_like(rows)
        lx = self.local
        onehot = np.full((R, lx.n_expert), -np.inf, np.float32)
        onehot[np.arange(R), eid.numpy()] = 0.0
        y, _, _ = self.orc.moe_layer(np.zeros((R, lx.D), np.float32), rows.numpy(), onehot, list(lx.gate),
                                     list(lx.up), list(lx.down), lx.types, lx.row_bytes, 1)
        return torch.from_numpy(y)


class EpMoeLayer:
    """One MoE layer whose experts are split over the ranks of `group` (rank r owns experts
    [r E/P, (r+1) E/P)). Call with this rank's tokens: (xn [T x D], logits [T x E], x [T x D] updated
    in place); returns the routing (ids, weights) of the local tokens."""

    def __init__(self, ex, n_used: int, group=None, device: torch.device | None = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.E = ex.n_expert
        self.K = n_used
        self.D = ex.D
        self.E_loc = self.E // self.world
        self.device = device if device is not None else torch.device("cpu")
        local = shard(ex, self.rank, self.world)
        self.cuda = self.device.type == "cuda"
        self.experts = _CudaExperts(local, self.device) if self.cuda else _CpuExperts(local)

    def _route(self, logits: torch.Tensor):
        if self.cuda:
            import eahmmf_b200 as eb
            return eb.route_topk(logits.contiguous(), self.K)
        import oracle
        ids, w = oracle.Oracle().route(logits.numpy(), self.K)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def __call__(self, xn: torch.Tensor, logits: torch.Tensor, x: torch.Tensor):
        T, D, K, dev = xn.shape[0], self.D, self.K, self.device
        ids, w = self._route(logits) if T else (torch.zeros((0, K), dtype=torch.int32, device=dev),
                                                torch.zeros((0, K), dtype=torch.float32, device=dev))
        S = T * K
        flat = ids.reshape(-1).long()
        dest = flat // self.E_loc
        order = torch.argsort(dest * max(S, 1) + torch.arange(S, device=dev))  # by destination, then slot
        send_counts = torch.bincount(dest, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts, None, None)  # one count per rank
        send_splits, recv_splits = send_counts.tolist(), recv_counts.tolist()
        R = int(sum(recv_splits))
        send_x = xn.index_select(0, order // K).contiguous()
        send_e = (flat[order] - dest[order] * self.E_loc).to(torch.int32)
        recv_x = torch.empty((R, D), dtype=xn.dtype, device=dev)
        recv_e = torch.empty((R,), dtype=torch.int32, device=dev)
        self._a2a(recv_x, send_x, recv_splits, send_splits)
        self._a2a(recv_e, send_e, recv_splits, send_splits)
        y_recv = self.experts(recv_x, recv_e)
        y_back = torch.empty((S, D), dtype=y_recv.dtype, device=dev)
        self._a2a(y_back, y_recv.contiguous(), send_splits, recv_splits)
        y = torch.empty_like(y_back)
        y[order] = y_back  # slot s = t * K + k
        if T:
            # each token's slots in ascending expert order, the reference's combine order
            token_slots = (torch.arange(T, device=dev)[:, None] * K + torch.argsort(ids.long(), dim=1)).to(torch.int32)
            slot_w = w.reshape(-1).contiguous()
            if self.cuda:
                import eahmmf_b200 as eb
                rc = eb.moe_combine(token_slots.contiguous(), slot_w, y, x)
                if rc:
                    raise RuntimeError(f"eahmmf_cuda_moe_combine returned {rc}")
            else:
                _combine_cpu(token_slots.numpy(), slot_w.numpy(), y.numpy(), x.numpy())
        return ids, w


def _combine_cpu(token_slots, slot_w, y, x):
    T, K = token_slots.shape
    for t in range(T):
        acc = np.zeros(x.shape[1], np.float32)
        for k in range(K):
            s = token_slots[t, k]
            acc = (acc + np.float32(slot_w[s]) * y[s]).astype(np.float32)
        x[t] += acc

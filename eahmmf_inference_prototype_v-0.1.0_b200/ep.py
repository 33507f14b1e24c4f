"""Expert-parallel MoE layer: the experts of one layer sharded across ranks, tokens
dispatched to the ranks that own their routed experts and the expert outputs combined back, over
torch.distributed all-to-all (NCCL over NVLink on GPUs; gloo on CPU for the host-logic tests).

Per call, on every rank (one process per GPU, each holding its own tokens), with no host synchronisation:

  1. routing of the local tokens (the reference's top-k, qwen3moe.cpp:1011-1023);
  2. pack: each routed (token, k) slot's expert-input row and owner-local expert id go to block
     e // (E / P) of a dispatch buffer of P blocks of `cap` rows (cap = t_max * k, so no block can
     overflow); each block's first row carries its count;
  3. dispatch: one all-to-all of whole blocks (equal splits: no split size needs to reach the host);
  4. unpack: the received valid rows compacted to the front, their assigned experts beside them;
  5. the rank's experts applied to those rows directly (no second routing: assigned expert, weight 1);
  6. return: the outputs scattered back to their received positions, one all-to-all back;
  7. the weighted combine in ascending expert order into the residual, the reference's summation order
     (qwen3moe.cpp:1025-1069), reading the returned rows in place.

Every slot's output depends only on its own row, so the result equals the single-GPU layer's up to the
kernel path (GEMV or grouped) that each rank picks for the rows it receives.

The stages run on a backend object: `CudaEpBackend` (libeahmmf_b200's kernels, the product) by default.
Callers can pass any object with the same methods (the CPU tests pass one built on their checker).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

EP_HDR = 4  # header floats before each row of a dispatch buffer (EAHMMF_EP_HDR)
STAGE_NAMES = ("route_pack", "dispatch_a2a", "experts", "return_a2a", "combine")


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


class CudaEpBackend:
    """The exchange and expert stages on the GPU (libeahmmf_b200.so): routing (eahmmf_cuda_route_topk),
    pack / unpack / return (eahmmf_cuda_ep_*), the rank's experts on assigned rows
    (eahmmf_cuda_moe_experts) and the expert-ordered combine (eahmmf_cuda_moe_combine)."""

    def __init__(self, local, n_used: int, device, graph: bool = True):
        import eahmmf_b200 as eb
        self.eb = eb
        self.layer = eb.MoeLayer.from_expert_set(local, n_used=1)
        self.K = n_used
        self.device = device
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.ws = None
        # the receiver's stage (unpack, the rank's experts, return) works on the layer's fixed buffers:
        # after its first eager run it is captured once into a CUDA graph and replayed (one launch for
        # its ~20 kernels; no collective inside)
        self.use_graph = graph
        self.graph, self.graph_key = None, None

    def _st(self):
        return torch.cuda.current_stream(self.device)

    def alloc(self, shape, dtype):
        return torch.empty(shape, dtype=dtype, device=self.device)

    def route(self, logits):
        return self.eb.route_topk(logits.contiguous(), self.K, stream=self._st(), d_status=self.status)

    def pack(self, ids, w, xn, E_loc, world, cap, send, token_pos, pos_w):
        rc = self.eb.ep_pack(ids, w, xn.contiguous(), self.K, E_loc, world, cap, send, token_pos, pos_w,
                             stream=self._st(), d_status=self.status)
        if rc:
            raise RuntimeError(f"eahmmf_cuda_ep_pack returned {rc}")

    def unpack(self, recv, D, world, cap, rows, eid, src, y):
        rc = self.eb.ep_unpack(recv, D, world, cap, rows, eid, src, y, stream=self._st())
        if rc:
            raise RuntimeError(f"eahmmf_cuda_ep_unpack returned {rc}")

    def apply(self, rows, eid, y):
        R = rows.shape[0]
        need = self.layer.experts_workspace_bytes(R)
        if self.ws is None or self.ws.numel() < need:
            self.ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        rc = self.layer.apply_experts(R, rows, eid, y, self.ws, stream=self._st(), d_status=self.status)
        if rc:
            raise RuntimeError(f"eahmmf_cuda_moe_experts returned {rc}")

    def ret(self, y, src, D, world, cap, out):
        rc = self.eb.ep_return(y, src, D, world, cap, out, stream=self._st())
        if rc:
            raise RuntimeError(f"eahmmf_cuda_ep_return returned {rc}")

    def post(self, recv, D, world, cap, rows, eid, src, y, out):
        """unpack, apply and ret in one go: replayed from a CUDA graph after the first call."""
        key = (recv.data_ptr(), D, world, cap, rows.data_ptr(), eid.data_ptr(), src.data_ptr(), y.data_ptr(),
               out.data_ptr())
        if self.graph is not None and self.graph_key == key:
            self.graph.replay()
            return

        def run():
            self.unpack(recv, D, world, cap, rows, eid, src, y)
            self.apply(rows, eid, y)
            self.ret(y, src, D, world, cap, out)

        run()  # this call's results, and the workspace
        if self.use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                run()
            self.graph, self.graph_key = g, key

    def combine(self, token_pos, pos_w, back, x):
        rc = self.eb.moe_combine(token_pos, pos_w, back, x, stream=self._st())
        if rc:
            raise RuntimeError(f"eahmmf_cuda_moe_combine returned {rc}")

    def check(self) -> int:
        """Kernel status bits raised so far (0 = none); reads the device status word (synchronises)."""
        return int(self.status.item())


class EpMoeLayer:
    """One MoE layer whose experts are split over the ranks of `group` (rank r owns experts
    [r E/P, (r+1) E/P)). `local` holds this rank's experts (an ExpertSet of E/P experts); `t_max` bounds
    the tokens any rank passes per call (the dispatch blocks hold t_max * k rows). Call with this rank's
    tokens: (xn [T x D], logits [T x E], x [T x D] updated in place); returns the routing (ids, weights)
    of the local tokens. `stages` (optional, 6 CUDA events) times the stages of STAGE_NAMES."""

    def __init__(self, local, n_expert: int, n_used: int, t_max: int, group=None, device=None, backend=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if n_expert % self.world or local.n_expert != n_expert // self.world:
            raise ValueError(f"{local.n_expert} local experts do not match {n_expert} over {self.world} ranks")
        self.E, self.K, self.D, self.E_loc = n_expert, n_used, local.D, local.n_expert
        self.device = device if device is not None else torch.device("cpu")
        self.be = backend if backend is not None else CudaEpBackend(local, n_used, self.device)
        self.t_max = t_max
        self.cap = t_max * n_used
        W, cap, D = self.world, self.cap, self.D
        a = self.be.alloc
        self.send = a((W * cap * (D + EP_HDR),), torch.float32)
        self.recv = a((W * cap * (D + EP_HDR),), torch.float32) if W > 1 else self.send
        self.rows = a((W * cap, D), torch.float32)
        self.eid = a((W * cap,), torch.int32)
        self.src = a((W * cap,), torch.int32)
        self.y = a((W * cap, D), torch.float32)
        self.ret = a((W * cap, D), torch.float32)
        self.back = a((W * cap, D), torch.float32) if W > 1 else self.ret
        self.token_pos = a((t_max, n_used), torch.int32)
        self.pos_w = a((W * cap,), torch.float32)

    @classmethod
    def from_full(cls, ex, n_used: int, t_max: int, group=None, device=None, backend=None):
        """From the whole layer's ExpertSet (each rank keeps its shard)."""
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        return cls(shard(ex, rank, world), ex.n_expert, n_used, t_max, group=group, device=device, backend=backend)

    def _a2a(self, out, inp):
        dist.all_to_all_single(out, inp, group=self.group)  # equal splits: one block per rank

    def __call__(self, xn: torch.Tensor, logits: torch.Tensor, x: torch.Tensor, stages=None):
        T, D, K, W, cap = xn.shape[0], self.D, self.K, self.world, self.cap
        if T > self.t_max:
            raise ValueError(f"{T} tokens exceed t_max = {self.t_max}")

        def mark(i):
            if stages:
                stages[i].record()

        mark(0)
        if T:
            ids, w = self.be.route(logits)
        else:
            ids = self.be.alloc((0, K), torch.int32)
            w = self.be.alloc((0, K), torch.float32)
        token_pos = self.token_pos[:T]
        self.be.pack(ids, w, xn, self.E_loc, W, cap, self.send, token_pos, self.pos_w)
        mark(1)
        if W > 1:
            self._a2a(self.recv, self.send)
        mark(2)
        if hasattr(self.be, "post"):
            self.be.post(self.recv, D, W, cap, self.rows, self.eid, self.src, self.y, self.ret)
        else:
            self.be.unpack(self.recv, D, W, cap, self.rows, self.eid, self.src, self.y)
            self.be.apply(self.rows, self.eid, self.y)
            self.be.ret(self.y, self.src, D, W, cap, self.ret)
        mark(3)
        if W > 1:
            self._a2a(self.back, self.ret)
        mark(4)
        if T:
            self.be.combine(token_pos, self.pos_w, self.back, x)
        mark(5)
        return ids, w


def stage_events(n: int = 6):
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def stage_ms(ev) -> dict:
    """Per-stage milliseconds of one profiled call (waits for its last event)."""
    ev[-1].synchronize()
    return {name: float(ev[i].elapsed_time(ev[i + 1])) for i, name in enumerate(STAGE_NAMES)}

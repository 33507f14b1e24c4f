"""Expert-parallel layer (ep.py) host logic on CPU: two gloo ranks, each owning half the experts and
its own tokens, against the single-process oracle layer over all tokens.

The layer runs its stages on a CPU backend defined here (the checker's routing and expert application,
numpy restatements of the pack / unpack / return / combine kernels' buffer semantics), so what is
checked is the layer's own flow: buffer shapes, the equal-split all-to-alls of whole dispatch blocks,
the count headers, the compaction and the return positions, and the expert-ordered combine. Routed ids
exact, layer output within 1e-5 relative L2 (the combine here rounds each product; the oracle's may
fuse it).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import synth

HDR = 4


def _i2f(v: int) -> np.float32:
    return np.array([v], np.int32).view(np.float32)[0]


def _f2i(v) -> int:
    return int(np.array([v], np.float32).view(np.int32)[0])


class CpuEpBackend:
    """ep.py's backend interface on the CPU, for the host-logic tests only."""

    def __init__(self, local, n_used):
        import oracle
        self.orc = oracle.Oracle()
        self.local = local
        self.K = n_used

    def alloc(self, shape, dtype):
        return torch.zeros(shape, dtype=dtype)

    def route(self, logits):
        ids, w = self.orc.route(logits.numpy(), self.K)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def pack(self, ids, w, xn, E_loc, world, cap, send, token_pos, pos_w):
        T, K, D = xn.shape[0], self.K, xn.shape[1]
        buf = send.numpy().reshape(world * cap, D + HDR)
        ids_np, w_np, xn_np = ids.numpy().reshape(-1), w.numpy().reshape(-1), xn.numpy()
        fill = [0] * world
        for s in range(T * K):  # slots in ascending order, each to the next row of its owner's block
            t, e = s // K, int(ids_np[s])
            d = e // E_loc
            pos = d * cap + fill[d]
            fill[d] += 1
            buf[pos, 0] = _i2f(e - d * E_loc)
            buf[pos, HDR:] = xn_np[t]
            rank = int(np.sum(ids_np[t * K:(t + 1) * K] < e))
            token_pos.numpy()[t, rank] = pos
            pos_w.numpy()[pos] = w_np[s]
        for d in range(world):
            buf[d * cap, 1] = _i2f(fill[d])

    def unpack(self, recv, D, world, cap, rows, eid, src, y):
        buf = recv.numpy().reshape(world * cap, D + HDR)
        cnt = [_f2i(buf[q * cap, 1]) for q in range(world)]
        R = sum(cnt)
        eid_np, src_np, rows_np = eid.numpy(), src.numpy(), rows.numpy()
        # valid rows by ascending local expert, within an expert in (source, row) order
        valid = sorted(((_f2i(buf[q * cap + i, 0]), q * cap + i) for q in range(world) for i in range(cnt[q])))
        for j, (e, b) in enumerate(valid):
            rows_np[j] = buf[b, HDR:]
            eid_np[j] = e
            src_np[j] = b
        rows_np[R:] = 0
        eid_np[R:] = -1
        src_np[R:] = -1
        y.zero_()

    def apply(self, rows, eid, y):
        valid = eid.numpy() >= 0
        R = int(valid.sum())
        if R == 0:
            return
        lx = self.local
        onehot = np.full((R, lx.n_expert), -np.inf, np.float32)
        onehot[np.arange(R), eid.numpy()[valid]] = 0.0
        out, _, _ = self.orc.moe_layer(np.zeros((R, lx.D), np.float32), rows.numpy()[valid], onehot, list(lx.gate),
                                       list(lx.up), list(lx.down), lx.types, lx.row_bytes, 1)
        y.numpy()[valid] += out

    def ret(self, y, src, D, world, cap, out):
        for j, b in enumerate(src.numpy()):
            if b >= 0:
                out.numpy()[b] = y.numpy()[j]

    def combine(self, token_pos, pos_w, back, x):
        T, K = token_pos.shape
        for t in range(T):
            acc = np.zeros(x.shape[1], np.float32)
            for k in range(K):
                p = int(token_pos[t, k])
                acc = (acc + np.float32(pos_w[p]) * back.numpy()[p]).astype(np.float32)
            x.numpy()[t] += acc


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, T_per, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import ep
        ex = synth.expert_set(D=256, FF=256, n_expert=8, types=(12, 12, 14), seed=11, d_sigma=0.002)
        local = ep.shard(ex, rank, world)
        layer = ep.EpMoeLayer(local, ex.n_expert, n_used=2, t_max=max(T_per), backend=CpuEpBackend(local, 2))
        T = T_per[rank]
        x = synth.activations(T, 256, seed=50 + rank) if T else np.zeros((0, 256), np.float32)
        xn = synth.activations(T, 256, seed=60 + rank) if T else np.zeros((0, 256), np.float32)
        lg = synth.router_logits(T, 8, seed=70 + rank) if T else np.zeros((0, 8), np.float32)
        xt = torch.from_numpy(x.copy())
        ids, w = layer(torch.from_numpy(xn), torch.from_numpy(lg), xt)
        np.savez(out_path + f".{rank}.npz", x=x, xn=xn, lg=lg, y=xt.numpy(), ids=ids.numpy(), w=w.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_per", [(5, 7), (0, 9), (33, 1)])
def test_ep_layer_two_ranks_matches_single_process(tmp_path, orc, T_per):
    out = str(tmp_path / "ep")
    mp.start_processes(_rank_main, args=(2, _port(), T_per, out), nprocs=2, join=True, start_method="spawn")
    ex = synth.expert_set(D=256, FF=256, n_expert=8, types=(12, 12, 14), seed=11, d_sigma=0.002)
    for r in range(2):
        d = np.load(out + f".{r}.npz")
        if T_per[r] == 0:
            assert d["y"].shape[0] == 0
            continue
        yo, io, wo = orc.moe_layer(d["x"], d["xn"], d["lg"], list(ex.gate), list(ex.up), list(ex.down), ex.types,
                                   ex.row_bytes, 2)
        np.testing.assert_array_equal(d["ids"], io)
        np.testing.assert_allclose(d["w"], wo, rtol=1e-6, atol=0)
        num = np.linalg.norm((d["y"] - d["x"]) - (yo - d["x"]))
        assert num / np.linalg.norm(yo - d["x"]) < 1e-5


def test_ep_package_has_no_cpu_path():
    """The product's EP layer imports no checker and has no CPU expert path of its own."""
    import ep
    src = open(ep.__file__).read()
    assert "oracle" not in src
    assert "numpy" not in src

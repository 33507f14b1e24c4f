"""Expert-parallel layer (ep.py) host logic on CPU: two gloo ranks, each owning half the experts and
its own tokens, against the single-process oracle layer over all tokens.

Checks the dispatch bookkeeping (slot order by destination, owner-local expert ids), both all-to-alls
and the expert-ordered combine: routed ids exact, layer output within 1e-5 relative L2 (the CPU combine
here rounds each product, the oracle's may fuse it).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import synth


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
        layer = ep.EpMoeLayer(ex, n_used=2)
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

"""Expert-parallel layer (ep.py) on GPUs: one NCCL rank per visible GPU (at most 2; one rank still runs
the whole pack / exchange / assigned-expert / return / combine path), against the CPU oracle over each
rank's tokens.

Routed ids exact; layer output rel-L2 < 1e-5 where every rank's received rows take the 64-token GEMV path,
< 5e-4 where it takes the grouped f16 tensor-core path (>= 256 received rows, >= 16 per local expert).
"""
import os
import socket

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, T_per, out_path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import ep
        ex = synth.expert_set(D=512, FF=256, n_expert=16, types=(12, 12, 14), seed=21, d_sigma=0.004)
        layer = ep.EpMoeLayer.from_full(ex, n_used=4, t_max=max(T_per), device=dev)
        T = T_per[rank]
        x = synth.activations(T, 512, seed=80 + rank)
        xn = synth.activations(T, 512, seed=90 + rank)
        lg = synth.router_logits(T, 16, seed=100 + rank)
        xt = torch.from_numpy(x.copy()).to(dev)
        ids, w = layer(torch.from_numpy(xn).to(dev), torch.from_numpy(lg).to(dev), xt)
        torch.cuda.synchronize()
        assert layer.be.check() == 0
        # a second call replays the receiver stage's CUDA graph: the same bits
        xt2 = torch.from_numpy(x.copy()).to(dev)
        layer(torch.from_numpy(xn).to(dev), torch.from_numpy(lg).to(dev), xt2)
        torch.cuda.synchronize()
        assert layer.be.check() == 0
        assert layer.be.graph is not None
        assert torch.equal(xt, xt2)
        np.savez(out_path + f".{rank}.npz", x=x, xn=xn, lg=lg, y=xt.cpu().numpy(), ids=ids.cpu().numpy(),
                 w=w.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T_per,tol", [((6, 11), 1e-5), ((300, 70), 5e-4)])
def test_ep_layer_nccl_matches_oracle(tmp_path, orc, T_per, tol):
    import torch
    import torch.multiprocessing as mp
    assert torch.cuda.is_available()
    world = min(2, torch.cuda.device_count())
    T_per = T_per[:world]
    out = str(tmp_path / "ep")
    mp.start_processes(_rank_main, args=(world, _port(), T_per, out), nprocs=world, join=True, start_method="spawn")
    ex = synth.expert_set(D=512, FF=256, n_expert=16, types=(12, 12, 14), seed=21, d_sigma=0.004)
    for r in range(world):
        d = np.load(out + f".{r}.npz")
        yo, io, wo = orc.moe_layer(d["x"], d["xn"], d["lg"], list(ex.gate), list(ex.up), list(ex.down), ex.types,
                                   ex.row_bytes, 4)
        np.testing.assert_array_equal(d["ids"], io)
        np.testing.assert_allclose(d["w"], wo, rtol=1e-6, atol=0)
        err = np.linalg.norm((d["y"] - d["x"]) - (yo - d["x"])) / np.linalg.norm(yo - d["x"])
        assert err < tol, (r, err)


@pytest.mark.parametrize("world,cap,D", [(2, 24, 64), (8, 32, 32), (4, 1100, 16)])
def test_ep_unpack_orders_rows_by_expert(world, cap, D):
    """eahmmf_cuda_ep_unpack: the valid received rows, compacted by ascending local expert and, within an
    expert, in (source, row) order (up to 4096 positions; beyond that in (source, row) order alone), the
    expert ids and source positions beside them, -1 and zero rows after them; the return puts each
    compact row back at its source position."""
    import torch
    import eahmmf_b200 as eb
    rng = np.random.default_rng(world * 1000 + cap)
    E_loc, HDR, R = 7, 4, world * cap
    recv = np.zeros((R, D + HDR), np.float32)
    valid, ids = [], {}
    for q in range(world):
        n = int(rng.integers(0, cap + 1))
        recv[q * cap, 1] = np.array([n], np.int32).view(np.float32)[0]
        for i in range(n):
            b = q * cap + i
            e = int(rng.integers(0, E_loc))
            recv[b, 0] = np.array([e], np.int32).view(np.float32)[0]
            recv[b, HDR:] = rng.normal(size=D).astype(np.float32)
            valid.append(b)
            ids[b] = e
    want = sorted(valid, key=lambda b: (ids[b], b)) if R <= 4096 else valid
    dev = torch.device("cuda", 0)
    d_recv = torch.from_numpy(recv.reshape(-1)).to(dev)
    rows = torch.full((R, D), 7.0, device=dev)
    eid = torch.zeros(R, dtype=torch.int32, device=dev)
    src = torch.zeros(R, dtype=torch.int32, device=dev)
    y = torch.full((R, D), 3.0, device=dev)
    assert eb.ep_unpack(d_recv, D, world, cap, rows, eid, src, y) == 0
    ret = torch.zeros((R, D), device=dev)
    assert eb.ep_return(rows, src, D, world, cap, ret) == 0
    torch.cuda.synchronize()
    n = len(want)
    np.testing.assert_array_equal(src.cpu().numpy()[:n], np.array(want, np.int32))
    np.testing.assert_array_equal(eid.cpu().numpy()[:n], np.array([ids[b] for b in want], np.int32))
    np.testing.assert_array_equal(rows.cpu().numpy()[:n], recv[want, HDR:])
    assert (src.cpu().numpy()[n:] == -1).all() and (eid.cpu().numpy()[n:] == -1).all()
    assert not rows.cpu().numpy()[n:].any() and not y.cpu().numpy().any()
    np.testing.assert_array_equal(ret.cpu().numpy()[valid], recv[valid, HDR:])

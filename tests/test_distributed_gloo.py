"""Multi-rank host logic of rdna4_conv3d.distributed on CPU (gloo, world size 2).

The GPU paths of these functions run the same collectives over NCCL; here the
data movement and the math around it (halo exchange and its adjoint, the
depth-sharded conv's forward/backward, the gradient all-reducer) are checked
against single-process references. Ranks are spawned processes talking over
127.0.0.1.
"""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=__import__("datetime").timedelta(seconds=60))


def _slab(full, rank):
    d = full.shape[2] // WORLD
    return full[:, :, rank * d:(rank + 1) * d].contiguous()


def _worker_halo(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401  (registers the package modules)
    from rdna4_conv3d.distributed import halo_exchange, halo_reduce
    _init(rank, port)
    try:
        g = torch.Generator().manual_seed(0)
        full = torch.randn(2, 3, 8, 5, 4, generator=g, dtype=torch.float64)
        x = _slab(full, rank)
        xp = halo_exchange(x, 1)
        # the halo planes hold the neighbours' edge planes, zeros at the volume ends
        d = x.shape[2]
        lo_ref = full[:, :, rank * d - 1:rank * d] if rank > 0 else torch.zeros_like(x[:, :, :1])
        hi_ref = full[:, :, (rank + 1) * d:(rank + 1) * d + 1] if rank < WORLD - 1 else torch.zeros_like(x[:, :, :1])
        ok = torch.equal(xp[:, :, 1:1 + d], x) and torch.equal(xp[:, :, :1], lo_ref) and torch.equal(xp[:, :, -1:], hi_ref)
        # adjoint: <halo_exchange(x), gp> summed over ranks == <x, halo_reduce(gp)> summed over ranks
        gp = torch.randn(xp.shape, generator=torch.Generator().manual_seed(10 + rank), dtype=torch.float64)
        lhs = torch.tensor([(xp * gp).sum().item()], dtype=torch.float64)
        rhs = torch.tensor([(x * halo_reduce(gp, 1)).sum().item()], dtype=torch.float64)
        dist.all_reduce(lhs)
        dist.all_reduce(rhs)
        torch.save({"ok": ok, "lhs": lhs.item(), "rhs": rhs.item()}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _worker_depth_conv(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    from rdna4_conv3d.distributed import depth_sharded_conv3d
    _init(rank, port)
    try:
        g = torch.Generator().manual_seed(1)
        full = torch.randn(1, 4, 8, 6, 5, generator=g, dtype=torch.float64)
        w = torch.randn(3, 4, 3, 3, 3, generator=g, dtype=torch.float64)
        b = torch.randn(3, generator=g, dtype=torch.float64)
        gy_full = torch.randn(1, 3, 8, 6, 5, generator=g, dtype=torch.float64)
        x = _slab(full, rank).requires_grad_(True)
        wl = w.clone().requires_grad_(True)
        bl = b.clone().requires_grad_(True)
        y = depth_sharded_conv3d(x, wl, bl)
        y.backward(_slab(gy_full, rank))
        torch.save({"y": y.detach(), "gx": x.grad, "gw": wl.grad, "gb": bl.grad}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _worker_reducer(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    from rdna4_conv3d.distributed import GradAllReducer
    _init(rank, port)
    try:
        a = torch.full((4, 3), float(rank + 1))
        b = torch.arange(5, dtype=torch.float32) * (rank + 1)
        red = GradAllReducer(average=True)
        pend = red.reduce_async([a, None, b])
        pend.wait()
        red_sum = GradAllReducer(average=False)
        c = torch.ones(2) * (rank + 1)
        red_sum.reduce_async([c]).wait()
        torch.save({"a": a, "b": b, "c": c}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _run(worker):
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(worker, args=(_free_port(), td), nprocs=WORLD, join=True)
        return [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(WORLD)]


def test_halo_exchange_contents_and_adjoint():
    res = _run(_worker_halo)
    for r in res:
        assert r["ok"]
        assert abs(r["lhs"] - r["rhs"]) <= 1e-9 * max(1.0, abs(r["lhs"]))


def test_depth_sharded_conv_matches_full_volume():
    res = _run(_worker_depth_conv)
    g = torch.Generator().manual_seed(1)
    full = torch.randn(1, 4, 8, 6, 5, generator=g, dtype=torch.float64).requires_grad_(True)
    w = torch.randn(3, 4, 3, 3, 3, generator=g, dtype=torch.float64).requires_grad_(True)
    b = torch.randn(3, generator=g, dtype=torch.float64).requires_grad_(True)
    gy_full = torch.randn(1, 3, 8, 6, 5, generator=g, dtype=torch.float64)
    y = F.conv3d(full, w, b, 1, 1)
    y.backward(gy_full)
    y_sh = torch.cat([r["y"] for r in res], dim=2)
    gx_sh = torch.cat([r["gx"] for r in res], dim=2)
    torch.testing.assert_close(y_sh, y.detach(), rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(gx_sh, full.grad, rtol=1e-10, atol=1e-10)
    for r in res:  # dW / db are all-reduced: every rank holds the full-volume gradient
        torch.testing.assert_close(r["gw"], w.grad, rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(r["gb"], b.grad, rtol=1e-10, atol=1e-10)


def test_grad_allreducer_average_and_sum():
    res = _run(_worker_reducer)
    for r in res:
        torch.testing.assert_close(r["a"], torch.full((4, 3), 1.5))
        torch.testing.assert_close(r["b"], torch.arange(5, dtype=torch.float32) * 1.5)
        torch.testing.assert_close(r["c"], torch.ones(2) * 3.0)

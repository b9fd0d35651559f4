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


def _worker_gradsync(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    from rdna4_conv3d.distributed import GradSync
    _init(rank, port)
    try:
        torch.manual_seed(0)
        net = torch.nn.Sequential(torch.nn.Linear(4, 3), torch.nn.Tanh(), torch.nn.Linear(3, 2)).double()
        sync = GradSync(net, bucket_bytes=40)       # small buckets: several flushes per backward
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(5, 4, generator=g, dtype=torch.float64)
        for _ in range(2):                          # the hooks re-arm for every backward pass
            net.zero_grad(set_to_none=True)
            net(x).pow(2).sum().backward()
        torch.save({"grads": [p.grad.clone() for p in net.parameters()], "flushed": sync.buckets_flushed},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gradsync_averages_bucketed_grads():
    res = _run(_worker_gradsync)
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(4, 3), torch.nn.Tanh(), torch.nn.Linear(3, 2)).double()
    per_rank = []
    for rank in range(WORLD):
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(5, 4, generator=g, dtype=torch.float64)
        net.zero_grad(set_to_none=True)
        net(x).pow(2).sum().backward()
        per_rank.append([p.grad.clone() for p in net.parameters()])
    want = [(a + b) / 2 for a, b in zip(*per_rank)]
    for r in res:
        assert r["flushed"] >= 4
        for got, ref in zip(r["grads"], want):
            torch.testing.assert_close(got, ref, rtol=1e-12, atol=1e-12)


def _small_unet():
    from rdna4_conv3d.unet3d import UNet3D
    torch.manual_seed(3)
    return UNet3D(in_channels=1, n_classes=2, base=4, levels=3).double()


def _worker_depth_unet(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    from rdna4_conv3d.distributed import GradSync, depth_shard_model
    _init(rank, port)
    try:
        net = _small_unet()
        partial = depth_shard_model(net)
        GradSync(partial, average=False)
        g = torch.Generator().manual_seed(9)
        x = torch.randn(1, 1, 16, 8, 8, generator=g, dtype=torch.float64)
        gy = torch.randn(1, 2, 16, 8, 8, generator=g, dtype=torch.float64)
        y = net(_slab(x, rank))
        (y * _slab(gy, rank)).sum().backward()
        torch.save({"y": y.detach(), "grads": {n: p.grad.clone() for n, p in net.named_parameters()},
                    "bufs": {n: b.clone() for n, b in net.named_buffers()}}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_depth_sharded_unet_matches_full_volume():
    """A whole UNet (k3 convs with halos, whole-volume BatchNorm statistics,
    pooling, k2s2 transpose convs, skip concatenation, k1 head) over two D
    slabs against the same UNet on the full volume, fp64."""
    res = _run(_worker_depth_unet)
    net = _small_unet()
    g = torch.Generator().manual_seed(9)
    x = torch.randn(1, 1, 16, 8, 8, generator=g, dtype=torch.float64)
    gy = torch.randn(1, 2, 16, 8, 8, generator=g, dtype=torch.float64)
    y = net(x)
    (y * gy).sum().backward()
    torch.testing.assert_close(torch.cat([r["y"] for r in res], dim=2), y.detach(), rtol=1e-9, atol=1e-9)
    for r in res:
        for n, p in net.named_parameters():
            torch.testing.assert_close(r["grads"][n], p.grad, rtol=1e-8, atol=1e-9, msg=n)
        for n, b in net.named_buffers():
            if b.dtype.is_floating_point:
                torch.testing.assert_close(r["bufs"][n], b, rtol=1e-9, atol=1e-9, msg=n)

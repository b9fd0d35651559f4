"""Multi-GPU paths over NCCL on two B200s (skipped with fewer than two GPUs).

* The depth-sharded k3 conv on the kernel path (interior planes from the
  local slab, edge planes after the NCCL halo exchange, dW's halo terms,
  dW/db all-reduced) against the reference's CPU path on the full volume
  (stock PyTorch fp32 on the same bf16-rounded inputs), with the north-star
  tolerances.
* GradSync (bucketed data-parallel gradients overlapped with backward)
  against the average of the ranks' own gradients.
* A depth-sharded UNet3D under AMP against the same UNet on the full volume
  on one GPU: loss within the north-star 1e-3.

Ranks are spawned processes (one per GPU) on 127.0.0.1 with a short
process-group timeout, so a rank that fails ends the others' collectives
with an error instead of a wait.
"""
import datetime
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
FWD_TOL = 2e-2
DW_TOL = 3e-2


def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))


def _run(worker, *args):
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(worker, args=(_free_port(), td) + args, nprocs=WORLD, join=True)
        return [torch.load(os.path.join(td, f"r{r}.pt")) for r in range(WORLD)]


def _slab(t, rank):
    d = t.shape[2] // WORLD
    return t[:, :, rank * d:(rank + 1) * d]


def _conv_case(cin, cout, d, h, w):
    g = torch.Generator().manual_seed(cin + cout)
    x = torch.randn(1, cin, d, h, w, generator=g).to(torch.bfloat16)
    wt = (torch.randn(cout, cin, 3, 3, 3, generator=g) / (cin * 27) ** 0.5).to(torch.bfloat16)
    b = torch.randn(cout, generator=g).to(torch.bfloat16)
    go = torch.randn(1, cout, d, h, w, generator=g).to(torch.bfloat16)
    return x, wt, b, go


CONV_CASES = [(24, 24, 16, 32, 32), (1, 24, 8, 16, 16), (48, 48, 4, 8, 8)]


def _worker_depth_conv(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    from rdna4_conv3d import _native
    from rdna4_conv3d.distributed import depth_sharded_conv3d
    _init(rank, port)
    try:
        out = {}
        cl = torch.channels_last_3d
        for case in CONV_CASES:
            x, wt, b, go = _conv_case(*case)
            xs = _slab(x, rank).cuda().contiguous(memory_format=cl).requires_grad_(True)
            wl = wt.cuda().requires_grad_(True)
            bl = b.cuda().requires_grad_(True)
            y = depth_sharded_conv3d(xs, wl, bl)
            y.backward(_slab(go, rank).cuda().contiguous(memory_format=cl))
            torch.cuda.synchronize()
            out[case] = {"y": y.detach().cpu(), "gx": xs.grad.cpu(), "gw": wl.grad.float().cpu(),
                         "gb": bl.grad.float().cpu()}
        out["err"] = _native.device_error()
        torch.save(out, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_depth_sharded_conv_on_kernels_matches_full_volume(cuda_ready):
    _need_two_gpus()
    import oracle as O
    res = _run(_worker_depth_conv)
    for case in CONV_CASES:
        x, wt, b, go = _conv_case(*case)
        y = torch.cat([r[case]["y"] for r in res], dim=2)
        gx = torch.cat([r[case]["gx"] for r in res], dim=2)
        assert O.max_rel(y, O.torch_conv_fwd(x, wt, b, 1)) <= FWD_TOL, case
        assert O.max_rel(gx, O.torch_conv_dx(x.shape, wt, go, 1)) <= FWD_TOL, case
        dwr = O.torch_conv_dw(x, go, wt.shape, 1)
        for r in res:      # dW / db are all-reduced: every rank holds the whole volume's
            # the weight is bf16 here, so dW comes back rounded to bf16
            assert O.norm_rel(r[case]["gw"], dwr) <= DW_TOL, case
            assert O.norm_rel(r[case]["gb"], go.float().sum(dim=(0, 2, 3, 4))) <= DW_TOL, case
    assert all(r["err"] == 0 for r in res)


def _worker_gradsync(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    from rdna4_conv3d import Conv3dWmma
    from rdna4_conv3d.distributed import GradSync
    _init(rank, port)
    try:
        def make():
            torch.manual_seed(0)
            return torch.nn.Sequential(Conv3dWmma(8, 16, 3, padding=1), torch.nn.ReLU(),
                                       Conv3dWmma(16, 8, 1)).cuda()
        g = torch.Generator().manual_seed(50 + rank)
        x = torch.randn(2, 8, 6, 8, 8, generator=g).to(torch.bfloat16).cuda()
        x = x.contiguous(memory_format=torch.channels_last_3d)
        local = make()
        local(x).float().pow(2).sum().backward()
        mine = torch.cat([p.grad.reshape(-1) for p in local.parameters()])
        both = [torch.empty_like(mine) for _ in range(WORLD)]
        dist.all_gather(both, mine)
        want = (both[0] + both[1]) / 2
        synced = make()
        GradSync(synced, bucket_bytes=4096)
        synced(x).float().pow(2).sum().backward()
        got = torch.cat([p.grad.reshape(-1) for p in synced.parameters()])
        torch.cuda.synchronize()
        torch.save({"err": (got - want).abs().max().item(), "scale": want.abs().max().item()},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_gradsync_on_nccl(cuda_ready):
    _need_two_gpus()
    for r in _run(_worker_gradsync):
        assert r["err"] <= 1e-6 * r["scale"], r


def _unet_inputs():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 1, 32, 32, 32, generator=g)
    tgt = torch.randint(0, 4, (1, 32, 32, 32), generator=g)
    return x, tgt


def _worker_depth_unet(rank, port, outdir):
    import rdna4_conv3d  # noqa: F401
    import torch.nn.functional as F
    from rdna4_conv3d.distributed import GradSync, depth_shard_model
    from rdna4_conv3d.unet3d import unet3d
    _init(rank, port)
    try:
        torch.manual_seed(0)
        net = unet3d(8, levels=3, wmma=True, device="cuda")
        GradSync(depth_shard_model(net), average=False)
        x, tgt = _unet_inputs()
        xs = _slab(x, rank).cuda().contiguous(memory_format=torch.channels_last_3d)
        ts = tgt[:, rank * 16:(rank + 1) * 16].cuda()
        opt = torch.optim.Adam(net.parameters(), lr=1e-3)
        losses = []
        for _ in range(5):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                # the volume's mean loss: each slab's mean over its half
                loss = F.cross_entropy(net(xs), ts) / WORLD
            loss.backward()
            opt.step()
            tot = loss.detach().clone()
            dist.all_reduce(tot)
            losses.append(float(tot))
        torch.save({"losses": losses}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_depth_sharded_unet_loss_matches_one_gpu(cuda_ready):
    _need_two_gpus()
    import torch.nn.functional as F
    from rdna4_conv3d.unet3d import unet3d
    res = _run(_worker_depth_unet)
    torch.manual_seed(0)
    net = unet3d(8, levels=3, wmma=True, device="cuda")
    x, tgt = _unet_inputs()
    x = x.cuda().contiguous(memory_format=torch.channels_last_3d)
    tgt = tgt.cuda()
    opt = torch.optim.Adam(net.parameters(), lr=1e-3)
    ref = []
    for _ in range(5):
        opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = F.cross_entropy(net(x), tgt)
        loss.backward()
        opt.step()
        ref.append(float(loss.detach()))
    for r in res:
        diffs = [abs(a - b) for a, b in zip(r["losses"], ref)]
        assert max(diffs) <= 1e-3, (diffs, ref)

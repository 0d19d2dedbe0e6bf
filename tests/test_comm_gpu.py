"""GPU: the fused tensor-parallel all-reduce + residual add + RMSNorm + rotation (exl3_ar_add_norm_rot).

On one GPU the kernel runs as rank 0 of a 2-rank group whose "peer" buffer is a second local buffer
and whose peer flag is preset, so nothing waits on another launch; with 2+ GPUs, two processes run
the real NVLink path. Expected values: the ranks' partials summed in rank order in fp32 and rounded
to the model dtype, then exactly add_norm_rot (h bit-exact, xn/xh within the add_norm_rot bounds)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _expected(x, parts, w, eps, suh):
    from omlx_exl3_b200 import kernels
    s = parts[0].float()
    for p in parts[1:]:
        s = s + p.float()
    d = s.to(x.dtype)
    return kernels.add_norm_rot(x, d, w, eps, suh)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k,nm", [(1, 5120, 2), (3, 5120, 3), (8, 2560, 1)])
def test_ar_add_norm_rot_emulated_two_ranks(cuda, dtype, rows, k, nm):
    from omlx_exl3_b200.comm import PeerGroup
    g = torch.Generator(device=cuda)
    g.manual_seed(rows * 31 + k + nm)
    A = PeerGroup(1, 0, cuda, 8, 8192)
    B = PeerGroup(1, 0, cuda, 8, 8192)
    try:
        A.desc.world = 2
        A.desc.base[1] = B.own
        A.flags()[1] = 0x7FFFFFFF                       # "rank 1 is always ready"
        w = (1 + 0.1 * torch.randn(k, device=cuda, generator=g)).to(dtype)
        suh = (0.5 * torch.randn((nm, k), device=cuda, generator=g)).half()
        for call, slot in enumerate((0, 1, 0)):
            x = (3 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d0 = (2 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d1 = (2 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            A.slot_view(slot, rows, k, dtype).copy_(d0)
            B.slot_view(slot, rows, k, dtype).copy_(d1)
            h, xn, xh = A.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            eh, exn, exh = _expected(x, [d0, d1], w, 1e-6, suh)
            torch.cuda.synchronize()
            assert torch.equal(h, eh)
            assert float((xn.float() - exn.float()).abs().max()) <= 2 * float(exn.float().abs().max()) * 2 ** -7
            ref = O.rot(xn.float().cpu().numpy(), suh.cpu().numpy())
            assert O.max_rel(xh.float().cpu().numpy(), ref) < 1e-3
            assert int(A.flags()[8]) == call + 1            # epoch advanced once per call
            assert int(A.flags()[0]) == call + 1            # own arrival flag
        assert A.status() == 0
    finally:
        A.close()
        B.close()


def _two_rank_worker(rank, world, port, out_q):
    import torch.distributed as dist
    from omlx_exl3_b200.comm import PeerGroup
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        pg = PeerGroup(world, rank, dev, 8, 8192)
        k, rows, nm = 5120, 2, 2
        dtype = torch.bfloat16
        ok = True
        for call in range(4):
            slot = call & 1
            parts = []
            for r in range(world):
                g = torch.Generator(device=dev)
                g.manual_seed(1000 * call + r)
                parts.append((2 * torch.randn((rows, k), device=dev, generator=g)).to(dtype))
            g = torch.Generator(device=dev)
            g.manual_seed(77 + call)
            x = (3 * torch.randn((rows, k), device=dev, generator=g)).to(dtype)
            w = (1 + 0.1 * torch.randn(k, device=dev, generator=g)).to(dtype)
            suh = (0.5 * torch.randn((nm, k), device=dev, generator=g)).half()
            pg.slot_view(slot, rows, k, dtype).copy_(parts[rank])
            h, xn, xh = pg.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            eh, exn, exh = _expected(x, parts, w, 1e-6, suh)
            torch.cuda.synchronize(dev)
            ok = ok and torch.equal(h, eh) and bool((xn.float() - exn.float()).abs().max() <= 0.05)
        ok = ok and pg.status() == 0
        dist.barrier(device_ids=[rank])
        pg.close()
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ar_add_norm_rot_two_processes():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}

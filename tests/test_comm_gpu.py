"""GPU: the fused tensor-parallel all-reduce + residual add + RMSNorm + rotation (exl3_ar_add_norm_rot)
and its producers (exl3_peer_put, exl3_gemv_peer).

On one GPU two single-rank buffers are wired into an emulated 2-rank group (rank 0 and rank 1 views
of the same two buffers); both ranks' partials are pushed before either all-reduce launches, so no
kernel ever waits on another launch. With 2+ GPUs, two processes run the real NVLink path.
Expected values: the ranks' partials summed in rank order in fp32 and rounded to the model dtype,
then exactly add_norm_rot (h bit-exact, xn/xh within the add_norm_rot bounds)."""
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


def _emulated_pair(cuda, max_rows=8, max_k=8192):
    """Rank 0 and rank 1 views of a 2-rank group over two local buffers."""
    from omlx_exl3_b200.comm import PeerGroup
    A = PeerGroup(1, 0, cuda, max_rows, max_k, capacity_world=2)
    B = PeerGroup(1, 0, cuda, max_rows, max_k, capacity_world=2)
    for pg, rank in ((A, 0), (B, 1)):
        pg.desc.world, pg.desc.rank = 2, rank
        pg.desc.base[0], pg.desc.base[1] = A.own, B.own
        pg.world, pg.rank = 2, rank
    return A, B


def _check(h, xn, xh, eh, exn, suh):
    assert torch.equal(h, eh)
    assert float((xn.float() - exn.float()).abs().max()) <= 2 * float(exn.float().abs().max()) * 2 ** -7
    ref = O.rot(xn.float().cpu().numpy(), suh.cpu().numpy())
    assert O.max_rel(xh.float().cpu().numpy(), ref) < 1e-3


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k,nm", [(1, 5120, 2), (3, 5120, 3), (8, 2560, 1), (2, 1152, 1)])
def test_ar_add_norm_rot_emulated_two_ranks(cuda, dtype, rows, k, nm):
    g = torch.Generator(device=cuda)
    g.manual_seed(rows * 31 + k + nm)
    A, B = _emulated_pair(cuda)
    try:
        w = (1 + 0.1 * torch.randn(k, device=cuda, generator=g)).to(dtype)
        suh = (0.5 * torch.randn((nm, k), device=cuda, generator=g)).half()
        for call, slot in enumerate((0, 1, 0, 1)):
            x = (3 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d0 = (2 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d1 = (2 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            A.put(slot, d0)
            B.put(slot, d1)
            h, xn, xh = A.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            h1, xn1, xh1 = B.ar_add_norm_rot(slot, x, w, 1e-6, suh, want_xn=False)
            eh, exn, exh = _expected(x, [d0, d1], w, 1e-6, suh)
            torch.cuda.synchronize()
            _check(h, xn, xh, eh, exn, suh)
            assert xn1 is None and torch.equal(h1, h) and torch.equal(xh1, xh)   # every rank: the same bits
            assert int(A.flags()[8]) == call + 1 and int(B.flags()[8]) == call + 1   # epoch once per call
        assert A.status() == 0 and B.status() == 0
    finally:
        A.close()
        B.close()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows", [1, 3])
def test_gemv_peer_feeds_ar(cuda, dtype, rows):
    """exl3_gemv_peer as rank 0's producer: the all-reduce sees exactly the plain GEMV's output."""
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    k_in, k, K = 1024, 2560, 5
    g = torch.Generator(device=cuda)
    g.manual_seed(rows + 7)
    tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (k_in * k * K // 32,), dtype=torch.int32, device=cuda, generator=g)
    svh = (torch.randint(0, 2, (k,), device=cuda, generator=g).half() * 2 - 1) * 0.03
    plan = TrellisGemvPlan(k_in, [k], K, 0, svh, rows, dtype)
    A, B = _emulated_pair(cuda)
    try:
        w = (1 + 0.1 * torch.randn(k, device=cuda, generator=g)).to(dtype)
        suh = (0.5 * torch.randn((2, k), device=cuda, generator=g)).half()
        for call, slot in enumerate((0, 1, 0)):
            xh_in = torch.randn((1, rows, k_in), device=cuda, generator=g).half()
            x = (3 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d1 = (2 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d0 = plan(xh_in, [tr])
            plan.peer(xh_in, [tr], A, slot)
            B.put(slot, d1)
            h, xn, xh = A.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            h1, _, _ = B.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            eh, exn, _ = _expected(x, [d0, d1], w, 1e-6, suh)
            torch.cuda.synchronize()
            _check(h, xn, xh, eh, exn, suh)
            assert torch.equal(h1, h)
        assert A.status() == 0 and int(plan.counters.abs().sum().item()) == 0
    finally:
        A.close()
        B.close()


@pytest.mark.parametrize("rows", [1, 4])
def test_gemv_swiglu_peer_feeds_ar(cuda, rows):
    """exl3_gemv_swiglu_peer (the tensor-parallel down_proj: SwiGLU + rotation + GEMV + push in one
    launch) as rank 0's producer: the all-reduce sees exactly swiglu_rot + the plain GEMV's output."""
    from omlx_exl3_b200 import kernels
    from omlx_exl3_b200.kernels import TrellisGemvPlan
    k_in, k, K, dtype = 2176, 2560, 6, torch.bfloat16
    g = torch.Generator(device=cuda)
    g.manual_seed(rows + 11)
    tr = torch.randint(-2 ** 31, 2 ** 31 - 1, (k_in * k * K // 32,), dtype=torch.int32, device=cuda, generator=g)
    svh = (torch.randint(0, 2, (k,), device=cuda, generator=g).half() * 2 - 1) * 0.03
    dsuh = (torch.randint(0, 2, (k_in,), device=cuda, generator=g) * 2 - 1).half()
    plan = TrellisGemvPlan(k_in, [k], K, 0, svh, rows, dtype)
    A, B = _emulated_pair(cuda)
    try:
        w = (1 + 0.1 * torch.randn(k, device=cuda, generator=g)).to(dtype)
        suh = (0.5 * torch.randn((1, k), device=cuda, generator=g)).half()
        for call, slot in enumerate((0, 1)):
            gu = (2 * torch.randn((rows, 2 * k_in), device=cuda, generator=g)).half()
            x = (3 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d1 = (2 * torch.randn((rows, k), device=cuda, generator=g)).to(dtype)
            d0 = plan(kernels.swiglu_rot(gu, dsuh), [tr])
            plan.swiglu_call(gu, dsuh, [tr], peers=A, slot=slot)
            B.put(slot, d1)
            h, xn, xh = A.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            B.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            eh, exn, _ = _expected(x, [d0, d1], w, 1e-6, suh)
            torch.cuda.synchronize()
            _check(h, xn, xh, eh, exn, suh)
        assert A.status() == 0 and int(plan.counters.abs().sum().item()) == 0
    finally:
        A.close()
        B.close()


def test_ar_wait_times_out_with_status(cuda):
    """A source rank that never pushes: the bounded wait gives up after ~2 s, sets status bit 4 and
    returns; the context stays usable."""
    A, B = _emulated_pair(cuda)
    try:
        k, rows = 1024, 1
        x = torch.randn((rows, k), device=cuda).half()
        w = torch.ones(k, device=cuda).half()
        suh = torch.ones((1, k), device=cuda).half()
        A.put(0, torch.zeros((rows, k), device=cuda).half())         # rank 1 never pushes
        A.ar_add_norm_rot(0, x, w, 1e-6, suh)
        torch.cuda.synchronize()
        assert A.status() == 4
        assert float(torch.ones(4, device=cuda).sum()) == 4.0
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
            pg.put(slot, parts[rank])
            h, xn, xh = pg.ar_add_norm_rot(slot, x, w, 1e-6, suh)
            eh, exn, exh = _expected(x, parts, w, 1e-6, suh)
            torch.cuda.synchronize(dev)
            ok = ok and torch.equal(h, eh) and bool((xn.float() - exn.float()).abs().max() <= 0.05)
        # the row-parallel GEMV as the producer (exl3_gemv_peer)
        from omlx_exl3_b200.kernels import TrellisGemvPlan
        k_in, K = 1024, 5
        plans, trs, xhs = [], [], []
        for r in range(world):
            g = torch.Generator(device=dev)
            g.manual_seed(500 + r)
            trs.append(torch.randint(-2 ** 31, 2 ** 31 - 1, (k_in * k * K // 32,), dtype=torch.int32, device=dev,
                                     generator=g))
            svh = (torch.randint(0, 2, (k,), device=dev, generator=g).half() * 2 - 1) * 0.03
            plans.append(TrellisGemvPlan(k_in, [k], K, 0, svh, rows, dtype))
            xhs.append(torch.randn((1, rows, k_in), device=dev, generator=g).half())
        for call in range(4, 7):
            slot = call & 1
            parts = [plans[r](xhs[r], [trs[r]]) for r in range(world)]
            plans[rank].peer(xhs[rank], [trs[rank]], pg, slot)
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

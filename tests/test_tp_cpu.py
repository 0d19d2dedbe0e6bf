"""CPU: tensor-parallel sharding of EXL3 linears (column- and row-parallel) with world_size-2 gloo
ranks. Each rank evaluates its shard with the fp32 oracle; the all-reduce (row-parallel) and the
all-gather (column-parallel) must reproduce the unsharded layer. Also the shard ranges and the seeded
per-tensor bitrates of the 27B-class model."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from omlx_exl3_b200.loader import shard_exl3_part
        from omlx_exl3_b200.model import TP
        from oracle import oracle as O

        tp = TP(rank, world)
        rng = np.random.default_rng(0)
        k, n, K = 512, 768, 5
        t = O.random_trellis(k, n, K, 21)
        suh = np.where(rng.random(k) < 0.5, -1, 1).astype(np.float16)
        svh = (rng.standard_normal(n) * 0.05).astype(np.float16)
        x = rng.standard_normal((3, k)).astype(np.float32)
        full = O.linear_forward(t, k, n, K, 0, x, suh, svh)

        # row-parallel: this rank's k rows, partial output, summed across ranks
        tr = np.ascontiguousarray(shard_exl3_part("trellis", t, "row", k, n, tp))
        su = shard_exl3_part("suh", suh, "row", k, n, tp)
        r0 = rank * (k // world)
        part = O.linear_forward(tr, tr.shape[0] * 16, n, K, 0, x[:, r0:r0 + tr.shape[0] * 16], su, svh)
        yt = torch.from_numpy(part.astype(np.float64))
        dist.all_reduce(yt)
        err_row = float(np.abs(yt.numpy() - full).max() / np.abs(full).max())

        # column-parallel: this rank's output columns, gathered
        tc = np.ascontiguousarray(shard_exl3_part("trellis", t, "col", k, n, tp))
        sv = shard_exl3_part("svh", svh, "col", k, n, tp)
        cols = O.linear_forward(tc, k, tc.shape[1] * 16, K, 0, x, suh, sv)
        parts = [torch.zeros(3, n // world, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(cols.astype(np.float64)))
        err_col = float(np.abs(torch.cat(parts, 1).numpy() - full).max() / np.abs(full).max())
        q.put((rank, err_row, err_col))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, repr(e), None))


def test_tp2_row_and_column_parallel_match_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, er, ec in res:
        assert isinstance(er, float), er
        assert er < 1e-5 and ec < 1e-6, (rank, er, ec)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shards_cover_blocks(size):
    from omlx_exl3_b200.model import TP, column_shard, row_shard
    for n in (5120, 1024, 17408, 151936):
        got = [column_shard(n, TP(r, size)) for r in range(size)]
        assert got[0][0] == 0 and got[-1][1] == n
        for (a0, a1), (b0, b1) in zip(got, got[1:]):
            assert a1 == b0 and a0 % 128 == 0 and a1 > a0
        sizes = [b - a for a, b in got]
        assert max(sizes) - min(sizes) <= 128
        assert [row_shard(n, TP(r, size)) for r in range(size)] == got


def test_bits_draw_averages_six():
    from omlx_exl3_b200.loader import draw_bits
    from omlx_exl3_b200.model import ModelConfig
    cfg = ModelConfig()
    layers = draw_bits(64, seed=0, cfg=cfg)
    assert len(layers) == 64
    h, hd, ni = cfg.hidden_size, cfg.head_dim, cfg.intermediate_size
    sizes = {"q_proj": h * 40 * hd, "k_proj": h * 8 * hd, "v_proj": h * 8 * hd, "o_proj": 40 * hd * h,
             "gate_proj": h * ni, "up_proj": h * ni, "down_proj": ni * h}
    tot = sum(sizes.values()) * 64
    mean = sum(sizes[k] * b[k] for b in layers for k in sizes) / tot
    assert abs(mean - 6.0) <= 0.01
    assert all(5 <= b[k] <= 8 for b in layers for k in b)
    assert draw_bits(64, seed=0, cfg=cfg) == layers       # seeded


def test_inventory_reads_safetensors_headers(tmp_path):
    from safetensors.numpy import save_file
    from omlx_exl3_b200.loader import inventory, is_exl3_config
    t = np.zeros((4, 8, 64), np.int16)
    save_file({"model.layers.0.mlp.down_proj.trellis": t, "model.layers.0.mlp.down_proj.suh": np.ones(64, np.float16),
               "model.layers.0.mlp.down_proj.svh": np.ones(128, np.float16),
               "model.layers.0.mlp.down_proj.mcg": np.zeros(1, np.int32),
               "model.embed_tokens.weight": np.zeros((4, 4), np.float16)}, str(tmp_path / "model.safetensors"))
    inv = inventory(tmp_path)
    assert list(inv) == ["model.layers.0.mlp.down_proj"]
    parts = inv["model.layers.0.mlp.down_proj"]
    assert parts["trellis"][0] == (4, 8, 64) and parts["trellis"][1] == torch.int16
    assert set(parts) == {"trellis", "suh", "svh", "mcg"}
    assert is_exl3_config({"quantization_config": {"quant_method": "EXL3"}})
    assert not is_exl3_config({})


def test_linear_prepare_on_cpu_tensors():
    """Module construction, codebook / bitrate detection and the half-integer rejection need no GPU."""
    from omlx_exl3_b200 import EXL3Linear
    lin = EXL3Linear(256, 128, {"trellis": ((16, 8, 64), torch.int16), "suh": ((256,), torch.float16),
                                "svh": ((128,), torch.float16), "mul1": ((1,), torch.int32)})
    assert lin.bits == 4 and lin.codebook == 2 and lin.rot_suh.shape == (1, 256)
    half = EXL3Linear(256, 128, {"trellis": ((16, 8, 40), torch.int16), "suh": ((256,), torch.float16),
                                 "svh": ((128,), torch.float16)})
    with pytest.raises(NotImplementedError):
        half.runtime()

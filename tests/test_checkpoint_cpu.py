"""CPU: the checkpoint load path (loader.load) on a synthetic EXL3 checkpoint directory.

The directory is written from a seeded random-init model (tests/ckpt_util.py): config.json with an exl3
quantization_config, two safetensors shards with an index, some linears with the legacy packed su/sv
sign vectors, codebook markers (mcg, mul1) on others, a bias on one row-parallel and one column-parallel
linear. load() must rebuild exactly those tensors (TP1), and with tensor parallelism over two gloo ranks
each rank must read exactly its slice: whole 128-column blocks of column-parallel linears, whole 128-row
blocks of row-parallel ones, the row-parallel bias on rank 0 only. The slices' oracle outputs, summed
(row-parallel) or concatenated (column-parallel) over the ranks, must reproduce the unsharded linear.
Reference: daig/omlx-exl3 src/omlx/exl3/loader.py:58-72 (inventory), :183-223 (load),
src/omlx/exl3/linear.py:36-40 (packed signs), :63-65 (codebook markers)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

LEGACY = ("model.layers.0.self_attn.o_proj", "model.layers.1.self_attn.q_proj", "model.layers.1.self_attn.k_proj")
MARKERS = {"model.layers.0.mlp.down_proj": "mcg", "model.layers.1.self_attn.k_proj": "mul1"}


def _source_model(seed=11):
    from omlx_exl3_b200.loader import synthetic_model
    from omlx_exl3_b200.model import ModelConfig
    cfg = ModelConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                      intermediate_size=2048, num_hidden_layers=2, vocab_size=2048, max_position_embeddings=512)
    bits = [{"q_proj": 5, "k_proj": 6, "v_proj": 6, "o_proj": 4, "gate_proj": 6, "up_proj": 6, "down_proj": 5},
            {"q_proj": 6, "k_proj": 6, "v_proj": 6, "o_proj": 5, "gate_proj": 4, "up_proj": 4, "down_proj": 6}]
    return synthetic_model(cfg, bits, 8, device="cpu", seed=seed, fuse=False)


def _biases(model):
    g = torch.Generator().manual_seed(5)
    return {"model.layers.1.self_attn.o_proj": torch.randn(1024, generator=g).half(),
            "model.layers.0.mlp.up_proj": torch.randn(2048, generator=g).half()}


def _write(tmp_path):
    from tests.ckpt_util import write_checkpoint
    model = _source_model()
    written = write_checkpoint(model, tmp_path, n_shards=2, legacy=LEGACY, markers=MARKERS, biases=_biases(model))
    return model, written


def test_load_tp1_round_trip(tmp_path):
    from omlx_exl3_b200.linear import EXL3Linear, unpack_signs
    from omlx_exl3_b200.loader import inventory, load
    src, written = _write(tmp_path)
    inv = inventory(tmp_path)
    assert set(inv) == {n for n, m in src.named_modules() if isinstance(m, EXL3Linear)}
    assert set(inv["model.layers.1.self_attn.k_proj"]) == {"trellis", "su", "sv", "mul1"}
    assert inv["model.layers.0.mlp.down_proj"]["mcg"] == ((1,), torch.int32)
    model = load(tmp_path, device="cpu")
    for name, lin in model.named_modules():
        if not isinstance(lin, EXL3Linear):
            continue
        ref = src.get_submodule(name)
        assert torch.equal(lin.trellis, ref.trellis), name
        assert torch.equal(lin.rot_suh.reshape(-1), ref.suh), name
        assert lin.codebook == {"mcg": 1, "mul1": 2}.get(MARKERS.get(name), 0), name
        if name in LEGACY:
            # packed signs carry only the sign of svh (the source model's svh is scaled)
            assert "su" in lin and "suh" not in lin and "sv" in lin
            assert torch.equal(unpack_signs(lin.su), ref.suh)
            assert torch.equal(lin.output_signs, torch.sign(ref.svh)), name
        else:
            assert torch.equal(lin.output_signs, ref.svh), name
        if name.endswith("layers.1.self_attn.o_proj") or name.endswith("layers.0.mlp.up_proj"):
            assert "bias" in lin and torch.equal(lin.bias, written[f"{name}.bias"])
    for name, p in model.named_parameters():
        assert torch.equal(p, dict(src.named_parameters())[name]), name
    # siblings grouped by (bitrate, codebook): layer 1's k_proj carries mul1, so q/v are not one group with it
    at1 = model.model.layers[1].self_attn
    assert at1.k_proj._group is None and at1.q_proj._group is at1.v_proj._group is not None
    assert model.model.layers[0].self_attn.q_proj._group is None          # q at 5 bpw, k/v at 6
    assert model.model.layers[0].self_attn.k_proj._group is model.model.layers[0].self_attn.v_proj._group


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from omlx_exl3_b200.linear import EXL3Linear
        from omlx_exl3_b200.loader import load, shard_exl3_part
        from omlx_exl3_b200.model import TP
        from oracle import oracle as O
        src = load(path, device="cpu")               # the same checkpoint unsharded: the reference
        written = {}
        from safetensors.torch import load_file
        for f in sorted(os.listdir(path)):
            if f.endswith(".safetensors"):
                written.update(load_file(os.path.join(path, f)))
        model = load(path, tp_rank=rank, tp_size=world, device="cpu")
        tp = TP(rank, world)
        mism = []
        for name, lin in model.named_modules():
            if not isinstance(lin, EXL3Linear):
                continue
            full = src.get_submodule(name)
            kind = "row" if name.endswith(("o_proj", "down_proj")) else "col"
            k, n = full.in_features, full.out_features
            for part in ("trellis", "suh", "svh", "su", "sv", "bias"):
                if f"{name}.{part}" not in written:
                    continue
                want = shard_exl3_part(part, written[f"{name}.{part}"], kind, k, n, tp)
                if part == "bias" and kind == "row" and rank:
                    want = torch.zeros_like(want)
                if not torch.equal(lin._buffers[part], want.to(lin._buffers[part].dtype)):
                    mism.append(f"{name}.{part}")
        # oracle outputs of the slices, combined over the ranks, against the unsharded linear
        rng = np.random.default_rng(3)
        errs = {}
        for name, kind in (("model.layers.1.self_attn.o_proj", "row"), ("model.layers.0.mlp.up_proj", "col"),
                           ("model.layers.0.mlp.down_proj", "row")):
            full, part = src.get_submodule(name), model.get_submodule(name)
            x = rng.standard_normal((2, full.in_features)).astype(np.float32)

            def fwd(m, xx):
                b = m.bias.float().numpy() if "bias" in m else None
                return O.linear_forward(m.trellis.numpy(), m.in_features, m.out_features, m.bits, m.codebook, xx,
                                        m.rot_suh.reshape(-1).float().numpy(), m.output_signs.float().numpy(), b)
            ref = fwd(full, x)
            if kind == "row":
                r0 = rank * (full.in_features // world)
                y = torch.from_numpy(fwd(part, x[:, r0:r0 + part.in_features]).astype(np.float64))
                dist.all_reduce(y)
                got = y.numpy()
            else:
                ys = [torch.zeros((2, part.out_features), dtype=torch.float64) for _ in range(world)]
                dist.all_gather(ys, torch.from_numpy(fwd(part, x).astype(np.float64)))
                got = torch.cat(ys, 1).numpy()
            errs[name] = float(np.abs(got - ref).max() / np.abs(ref).max())
        q.put((rank, mism, errs))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        import traceback
        q.put((rank, traceback.format_exc(), None))


def test_load_tp2_shards_gloo(tmp_path):
    _write(tmp_path)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, mism, errs in res:
        assert errs is not None, mism
        assert mism == [], (rank, mism)
        assert all(e < 1e-5 for e in errs.values()), (rank, errs)

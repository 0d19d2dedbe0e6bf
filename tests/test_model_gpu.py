"""GPU: the EXL3 decoder path (EXL3Linear / sibling groups / fused norms and MLP / decode graph) against
the fp32 oracle forward, by logit KL (north star: KL <= 1e-4), plus the unfused and prefill paths."""
import numpy as np
import pytest
import torch

from oracle import model_oracle, oracle as O

pytestmark = pytest.mark.gpu


def _small_model(dev, fuse=True, bits=None, head_bits=8, layers=2, seed=3):
    from omlx_exl3_b200.loader import synthetic_model
    from omlx_exl3_b200.model import ModelConfig
    cfg = ModelConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                      intermediate_size=2048, num_hidden_layers=layers, vocab_size=2048,
                      max_position_embeddings=1024)
    b = bits or {"q_proj": 6, "k_proj": 6, "v_proj": 6, "o_proj": 5, "gate_proj": 6, "up_proj": 6, "down_proj": 4}
    return synthetic_model(cfg, [dict(b) for _ in range(layers)], head_bits, device=dev, seed=seed, fuse=fuse)


def _kl(ref_logits, logits):
    return O.kl_div(ref_logits, logits)


MIXED_BITS = {"q_proj": 5, "k_proj": 6, "v_proj": 6, "o_proj": 5, "gate_proj": 6, "up_proj": 4, "down_proj": 6}


@pytest.mark.parametrize("path", ["step", "step_mixed", "modules_fused", "modules_plain"])
@pytest.mark.parametrize("rows", [1, 3])
def test_decode_logits_kl(cuda, path, rows):
    """step: the fused decode step (Qwen3EXL3._forward_decode); step_mixed: the same with q/k/v and
    gate/up at different bitrates (one mixed-bitrate launch each); modules_*: the per-module path with
    and without the norm/MLP fusions."""
    torch.manual_seed(0)
    model = _small_model(cuda, fuse=path != "modules_plain", bits=MIXED_BITS if path == "step_mixed" else None)
    model.fused_decode = path.startswith("step")
    cache = model.make_cache(512)
    cache.fill_random(200, seed=1)
    toks = torch.tensor([5, 77, 1999][:rows], device=cuda)
    pos = torch.arange(200, 200 + rows, device=cuda)
    ck = [c.float().cpu().numpy() for c in cache.k]
    cv = [c.float().cpu().numpy() for c in cache.v]
    with torch.no_grad():
        logits = model(toks, cache, pos).float().cpu().numpy()
    ref = model_oracle.forward(model, toks.cpu().numpy(), ck, cv, 200)
    kl = _kl(ref, logits[:, : ref.shape[1]])
    assert kl.mean() < 1e-4, kl
    assert (logits.argmax(-1) == ref.argmax(-1)).all()


def test_prefill_rows_match_oracle(cuda):
    """rows > 8 goes through the prefill path (decode_wt + fp16 GEMM + output rotation)."""
    model = _small_model(cuda, fuse=True, layers=1)
    cache = model.make_cache(512)
    cache.fill_random(64, seed=2)
    rows = 16
    toks = torch.arange(rows, device=cuda) * 37 % 2048
    pos = torch.arange(64, 64 + rows, device=cuda)
    ck = [c.float().cpu().numpy() for c in cache.k]
    cv = [c.float().cpu().numpy() for c in cache.v]
    with torch.no_grad():
        logits = model(toks, cache, pos).float().cpu().numpy()
    ref = model_oracle.forward(model, toks.cpu().numpy(), ck, cv, 64)
    assert _kl(ref, logits).mean() < 1e-4


def test_decode_runner_graph_matches_eager(cuda):
    from omlx_exl3_b200.decode import DecodeRunner
    model = _small_model(cuda, fuse=True)
    cache = model.make_cache(512)
    cache.fill_random(300, seed=4)
    r_graph = DecodeRunner(model, cache, rows=1, use_graph=True)
    a = r_graph.step(torch.tensor([11], device=cuda)).clone()
    la = r_graph.logits.clone()
    b = r_graph.step(torch.tensor([11], device=cuda)).clone()
    assert torch.equal(a, b)
    with torch.no_grad():
        eager = model(torch.tensor([11], device=cuda), cache, torch.tensor([300], device=cuda))
    assert torch.equal(la, eager)
    assert int(a.item()) == int(eager.float().argmax(-1).item())


def test_fused_step_matches_module_path(cuda):
    """The fused decode step and the module path compute the same roundings: logits agree closely."""
    model = _small_model(cuda, fuse=True)
    cache = model.make_cache(512)
    cache.fill_random(100, seed=6)
    toks = torch.tensor([3, 9], device=cuda)
    pos = torch.tensor([100, 101], device=cuda)
    with torch.no_grad():
        model.fused_decode = True
        a = model(toks, cache, pos).float()
        model.fused_decode = False
        b = model(toks, cache, pos).float()
    assert torch.allclose(a, b, rtol=2e-2, atol=2e-2)
    assert torch.equal(a.argmax(-1), b.argmax(-1))


def test_decode_plan_uses_mixed_bitrate_groups(cuda):
    """q/k/v and gate/up of different bitrates are each one mixed-bitrate launch in the decode step."""
    from omlx_exl3_b200.model import _MixedGroup
    model = _small_model(cuda, bits=MIXED_BITS)
    assert model._decode_ready()
    lp = model.__dict__["_decode_plans"][0]
    assert isinstance(lp.qkv_group, _MixedGroup) and lp.qkv_group.Ks == [5, 6, 6]
    assert len(lp.gate_up.units) == 1 and isinstance(lp.gate_up.units[0], _MixedGroup)
    assert lp.gate_up.units[0].Ks == [6, 4] and lp.gu_at == [(0, 0, 2048), (0, 2048, 2048)]


def test_sibling_group_and_fusion_installed(cuda):
    model = _small_model(cuda, fuse=True)
    layer = model.model.layers[0]
    g = layer.self_attn.q_proj._group
    assert g is not None and g is layer.self_attn.k_proj._group and len(g.members) == 3
    assert layer.mlp.gate_proj._group is layer.mlp.up_proj._group
    # the fusion replaces the norm's forward on the instance only: its class and state stay as they were
    from omlx_exl3_b200.fusion import NormSite
    from omlx_exl3_b200.model import RMSNorm
    assert type(layer.input_layernorm) is RMSNorm and "forward" in layer.input_layernorm.__dict__
    sites = model.__dict__["_exl3_fusion_sites"]
    assert any(isinstance(s, NormSite) and s.module is layer.input_layernorm for s in sites)
    # mixed bitrates: q alone, k/v grouped
    m2 = _small_model(cuda, bits={"q_proj": 5, "k_proj": 6, "v_proj": 6, "o_proj": 5, "gate_proj": 6,
                                  "up_proj": 6, "down_proj": 6})
    at = m2.model.layers[0].self_attn
    assert at.q_proj._group is None and at.k_proj._group is at.v_proj._group is not None


def test_exl3linear_matches_oracle_rows(cuda):
    from omlx_exl3_b200 import EXL3Linear
    rng = np.random.default_rng(8)
    k, n, K = 1024, 768, 5
    t = O.random_trellis(k, n, K, 12)
    suh = np.where(rng.random(k) < 0.5, -1, 1).astype(np.float16)
    svh = (rng.standard_normal(n) * 0.02).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float16)
    lin = EXL3Linear(k, n, {"trellis": (t.shape, torch.int16), "suh": ((k,), torch.float16),
                            "svh": ((n,), torch.float16), "bias": ((n,), torch.float16)}, device=cuda)
    lin.load_state_dict({"trellis": torch.from_numpy(t), "suh": torch.from_numpy(suh), "svh": torch.from_numpy(svh),
                         "bias": torch.from_numpy(bias)})
    for rows in (1, 2, 8, 9, 33):
        x = rng.standard_normal((rows, k)).astype(np.float32)
        for dt in (torch.float16, torch.bfloat16):
            y = lin(torch.from_numpy(x).to(cuda, dt)).float().cpu().numpy()
            ref = O.linear_forward(t, k, n, K, 0, torch.from_numpy(x).to(dt).float().numpy(), suh, svh, bias)
            assert O.max_rel(y, ref) < 1e-2, (rows, dt)


def test_legacy_packed_signs(cuda):
    from omlx_exl3_b200 import EXL3Linear
    rng = np.random.default_rng(9)
    k, n, K = 512, 256, 4
    t = O.random_trellis(k, n, K, 13)
    su = rng.integers(0, 2 ** 16, k // 16, dtype=np.uint32).astype(np.uint16).view(np.int16)
    sv = rng.integers(0, 2 ** 16, n // 16, dtype=np.uint32).astype(np.uint16).view(np.int16)
    lin = EXL3Linear(k, n, {"trellis": (t.shape, torch.int16), "su": ((k // 16,), torch.int16),
                            "sv": ((n // 16,), torch.int16), "mcg": ((1,), torch.int32)}, device=cuda)
    lin.load_state_dict({"trellis": torch.from_numpy(t), "su": torch.from_numpy(su), "sv": torch.from_numpy(sv),
                         "mcg": torch.zeros(1, dtype=torch.int32)})
    x = rng.standard_normal((2, k)).astype(np.float32)
    y = lin(torch.from_numpy(x).to(cuda, torch.float16)).float().cpu().numpy()
    ref = O.linear_forward(t, k, n, K, 1, x.astype(np.float16).astype(np.float32), O.unpack_signs(su),
                           O.unpack_signs(sv))
    assert lin.codebook == 1
    assert O.max_rel(y, ref) < 1e-2


def test_exl3linear_bound_launch(cuda):
    """The eager module call binds its launch once per (rows, dtype): its output equals the unbound
    rot_call's bit for bit, call after call, for 1-D / 2-D / 3-D and non-contiguous inputs; after the
    buffers are replaced and reset_runtime() is called the new weights are used; bad inputs raise."""
    from omlx_exl3_b200 import EXL3Linear
    rng = np.random.default_rng(21)
    k, n, K = 1024, 512, 6
    t1, t2 = O.random_trellis(k, n, K, 31), O.random_trellis(k, n, K, 32)
    suh = torch.from_numpy(np.where(rng.random(k) < 0.5, -1, 1).astype(np.float16))
    svh = torch.from_numpy((rng.standard_normal(n) * 0.02).astype(np.float16))
    lin = EXL3Linear(k, n, {"trellis": (t1.shape, torch.int16), "suh": ((k,), torch.float16),
                            "svh": ((n,), torch.float16)}, device=cuda)
    lin.load_state_dict({"trellis": torch.from_numpy(t1), "suh": suh, "svh": svh})
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    for rows in (1, 3):
        rt = lin.runtime()
        plan = lin.plan(rows, torch.float16)
        for _ in range(3):
            x = torch.randn((rows, k), device=cuda, generator=g).half()
            ref = plan.rot_call(x, rt.suh, [rt.words]).clone()
            assert torch.equal(lin(x), ref)
            assert torch.equal(lin(x.reshape(1, rows, k)).reshape(rows, n), ref)
            xt = torch.randn((k, rows), device=cuda, generator=g).half().t()       # non-contiguous
            assert torch.equal(lin(xt), plan.rot_call(xt.contiguous(), rt.suh, [rt.words]))
    x1 = torch.randn(k, device=cuda, generator=g).half()
    assert lin(x1).shape == (n,)
    before = lin(x1).clone()
    lin.trellis.copy_(torch.from_numpy(t2).to(cuda))
    lin.reset_runtime()
    after = lin(x1)
    ref = lin.plan(1, torch.float16).rot_call(x1.reshape(1, k), lin.runtime().suh, [lin.runtime().words])
    assert torch.equal(after.reshape(1, n), ref) and not torch.equal(after, before)
    with pytest.raises(ValueError):
        lin(torch.zeros((1, k), dtype=torch.float16))                              # host tensor
    with pytest.raises(TypeError):
        lin(torch.zeros((1, k), dtype=torch.int32, device=cuda))

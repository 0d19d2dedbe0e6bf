"""GPU: a synthetic EXL3 checkpoint directory loaded with loader.load() onto the GPU gives the oracle's
logits (KL <= 1e-4, same greedy token) through the decode step: with biases present the per-module path
(the fused step needs bias-free projections), without them the fused, graph-capturable step. The
checkpoint mixes suh/svh and packed su/sv sign vectors and the 3inst / mcg / mul1 codebooks (see
test_checkpoint_cpu.py)."""
import numpy as np
import pytest
import torch

from oracle import model_oracle, oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("with_bias", [True, False])
@pytest.mark.parametrize("rows", [1, 4])
def test_loaded_checkpoint_logits_match_oracle(cuda, tmp_path, with_bias, rows):
    from omlx_exl3_b200.loader import load
    from tests.ckpt_util import write_checkpoint
    from tests.test_checkpoint_cpu import LEGACY, MARKERS, _biases, _source_model
    src = _source_model()
    write_checkpoint(src, tmp_path, n_shards=2, legacy=LEGACY, markers=MARKERS,
                     biases=_biases(src) if with_bias else None)
    model = load(tmp_path, device=cuda)
    assert model._decode_ready() == (not with_bias)
    cache = model.make_cache(256)
    cache.fill_random(100, seed=4)
    toks = torch.tensor([3, 1500, 77, 9][:rows], device=cuda)
    pos = torch.arange(100, 100 + rows, device=cuda)
    ck = [c.float().cpu().numpy() for c in cache.k]
    cv = [c.float().cpu().numpy() for c in cache.v]
    with torch.no_grad():
        logits = model(toks, cache, pos).float().cpu().numpy()
    ref = model_oracle.forward(model, toks.cpu().numpy(), ck, cv, 100)
    kl = O.kl_div(ref, logits[:, : ref.shape[1]])
    assert kl.max() < 1e-4, kl
    assert (logits[:, : ref.shape[1]].argmax(-1) == ref.argmax(-1)).all()

"""A layer read from an expert-cache directory (the reference relayout
format) and made resident in HBM computes exactly what the same layer built
in memory does."""
import numpy as np
import pytest

from tinygiant_b200 import expert_cache as EC
from tinygiant_b200 import synth
from tinygiant_b200.layer import ResidentLayer

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["qwen", "gptoss"])
def test_cache_layer_equals_in_memory_layer(gpu, tmp_path, kind):
    if kind == "qwen":
        L = synth.qwen_layer(seed=1, n_experts=16)
    else:
        L = synth.gptoss_layer(seed=3, n_experts=8, D=512, I=512)
    EC.write_cache(tmp_path, [L])
    G = EC.layer_from_cache(tmp_path, 0, L.router_w, act="gptoss" if kind == "gptoss" else "silu")
    a_l, b_l = ResidentLayer(L, max_tokens=4, lib=gpu), ResidentLayer(G, max_tokens=4, lib=gpu)
    try:
        x = np.random.default_rng(11).standard_normal((3, L.embed_dim)).astype(np.float32)
        a = a_l.forward(x, normalize=True)
        b = b_l.forward(x, normalize=True)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert np.array_equal(a_l.last_routing(3)[0], b_l.last_routing(3)[0])
    finally:
        a_l.close()
        b_l.close()

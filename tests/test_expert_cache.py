"""Expert-cache directories (the reference relayout tool's layer files and
index.json) read into MoeLayers: byte-identical matrices, shapes, formats and
routing parameters; malformed directories are rejected; and, where the
reference package is importable here, its own ExpertCache reads the files
this module writes to the same bytes."""
import json
import os
import sys

import numpy as np
import pytest

from tinygiant_b200 import expert_cache as EC
from tinygiant_b200 import quants as Q
from tinygiant_b200 import synth


def _small_qwen(seed, layer):
    return synth.qwen_layer(seed=seed, layer=layer, n_experts=4, D=512, I=256, top_k=2)


def _small_gptoss(seed, layer):
    return synth.gptoss_layer(seed=seed, layer=layer, n_experts=4, D=256, I=256, top_k=2)


@pytest.mark.parametrize("make", [_small_qwen, _small_gptoss])
def test_round_trip(tmp_path, make):
    layers = [make(5, 0), make(5, 1)]
    EC.write_cache(tmp_path, layers)
    idx = EC.read_index(tmp_path)
    assert idx["n_layers"] == 2 and idx["n_experts"] == 4 and idx["dtype"] == "quant"
    act = "gptoss" if layers[0].gate_fmt == Q.FMT_MXFP4 else "silu"
    got = EC.stack_from_cache(tmp_path, [L.router_w for L in layers], act=act)
    for L, G in zip(layers, got):
        assert (G.embed_dim, G.inter_dim, G.gate_fmt, G.top_k, G.act) == (L.embed_dim, L.inter_dim, L.gate_fmt,
                                                                           L.top_k, L.act)
        assert G.down_fmts == L.down_fmts
        for a, b in zip(L.gates + L.ups + L.downs, G.gates + G.ups + G.downs):
            assert np.array_equal(a, b)
        np.testing.assert_array_equal(G.router_w, L.router_w)


def test_rejects_malformed(tmp_path):
    L = _small_qwen(6, 0)
    EC.write_cache(tmp_path, [L])
    with pytest.raises(ValueError):
        EC.layer_from_cache(tmp_path, 0, np.zeros((3, 512), np.float32))   # router shape
    with pytest.raises(ValueError):
        EC.layer_from_cache(tmp_path, 7, L.router_w)                       # no such layer
    idx = EC.read_index(tmp_path)
    bad = json.loads(json.dumps(idx))
    bad["layers"]["0"]["tensor_formats"]["up"] = "q6_k"                     # gate and up differ
    with pytest.raises(ValueError):
        EC.layer_from_cache(tmp_path, 0, L.router_w, index=bad)
    bad = json.loads(json.dumps(idx))
    bad["layers"]["0"]["expert_offsets"]["1"]["sizes"]["down"] -= 16        # size / shape mismatch
    with pytest.raises(ValueError):
        EC.layer_from_cache(tmp_path, 0, L.router_w, index=bad)
    with open(tmp_path / "layer_000.q4.bin", "r+b") as f:                  # truncated file
        f.truncate(os.path.getsize(tmp_path / "layer_000.q4.bin") - 100)
    with pytest.raises(ValueError):
        EC.layer_from_cache(tmp_path, 0, L.router_w)


def test_reference_reader_sees_the_same_bytes(tmp_path):
    # the reference checkout, where the oracle build finds it (REF in oracle/Makefile)
    ref = os.environ.get("REF", os.path.join(os.sep, "root", "reference"))
    if not os.path.isdir(os.path.join(ref, "tinygiant")):
        pytest.skip("reference package not present")
    sys.path.insert(0, ref)
    try:
        from tinygiant.cache import ExpertCache
    except Exception as e:   # its optional dependencies
        pytest.skip(f"reference cache not importable: {e}")
    finally:
        sys.path.remove(ref)
    layers = [_small_qwen(7, 0), _small_qwen(7, 1)]
    EC.write_cache(tmp_path, layers)
    cache = ExpertCache(tmp_path, EC.read_index(tmp_path))
    mine = EC.stack_from_cache(tmp_path, [L.router_w for L in layers])
    for l, G in enumerate(mine):
        for e in range(G.n_experts):
            v = cache.get(l, e)
            for k, m in zip(EC.KEYS, (G.gates[e], G.ups[e], G.downs[e])):
                assert np.array_equal(np.asarray(v[k]), m)
    cache.close()

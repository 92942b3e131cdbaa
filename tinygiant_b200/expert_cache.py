"""Expert-cache directories straight into HBM.

The reference's relayout tool writes a model's routed experts as one file
per layer, `layer_NNN.q4.bin`: for every expert, in id order, one contiguous
record of its raw GGUF blocks, gate then up then down, each matrix row-major
[out_dim rows][blocks].  `index.json` beside the files holds the model's
counts (`n_layers`, `n_experts`, `n_experts_used`, `embed_dim`), the
matrices' shapes (`q4_sizes`: out_dim / in_dim per matrix) and, per layer,
the file name, each expert's byte offset and matrix sizes, and the
matrices' formats (`tensor_formats`: "q4_k", "q6_k", "mxfp4", ...)
(tinygiant/relayout.py:147-162, 285-341).  The reference engine maps those
records (tinygiant/cache.py:29-54) and reads them through an SSD / page-cache
tier on every token.

Here the same directory becomes `MoeLayer`s whose matrices are zero-copy
views of the mapped files; `ResidentLayer` (or `tg_layer_create`) uploads
each expert once and keeps every layer resident in HBM, which replaces the
cache tiers.  The routers live in the GGUF, not in the cache, so the caller
passes them.  `write_cache` writes the same format (tests, and converting
layers built in memory).
"""
import json
import mmap
import os
from pathlib import Path

import numpy as np

from . import quants as Q
from .synth import MoeLayer

KEYS = ("gate", "up", "down")
FMT_NAMES = {"q4_k": Q.FMT_Q4K, "float16": Q.FMT_F16, "q6_k": Q.FMT_Q6K, "mxfp4": Q.FMT_MXFP4,
             "q8_0": Q.FMT_Q80}
ACT_CODES = {"silu": 0, "gptoss": 1}
MAGIC = "NWSMOE01"   # the reference index's magic string


def read_index(cache_dir):
    with open(Path(cache_dir) / "index.json") as f:
        return json.load(f)


def _matrix_bytes(fmt, rows, cols):
    return rows * (cols * 2 if fmt == Q.FMT_F16 else Q.row_bytes(fmt, cols))


def layer_from_cache(cache_dir, layer_idx, router_w, router_b=None, act="silu", top_k=None, index=None,
                     inter_dim=None):
    """MoeLayer `layer_idx` of an expert-cache directory.

    router_w: fp32 [n_experts, embed_dim] (and router_b [n_experts] or None)
    from the model; act: "silu" or "gptoss"; top_k defaults to the index's
    n_experts_used; inter_dim defaults to the index's gate out_dim.  The
    matrices are read-only views of the mapped layer file, which stays
    mapped while the layer object lives.  Raises ValueError on a directory
    that does not describe a quantized expert layout this path runs."""
    cache_dir = Path(cache_dir)
    index = index if index is not None else read_index(cache_dir)
    if index.get("dtype") != "quant":
        raise ValueError(f"{cache_dir}: dtype {index.get('dtype')!r}: only quantized expert caches are supported")
    info = index["layers"].get(str(layer_idx), index["layers"].get(layer_idx))
    if info is None:
        raise ValueError(f"{cache_dir}: no layer {layer_idx} in index.json")
    E, D = int(index["n_experts"]), int(index["embed_dim"])
    shapes = index.get("q4_sizes", {})
    I = int(inter_dim if inter_dim is not None else shapes["gate"]["out_dim"])
    formats = info.get("tensor_formats", {})
    fmts = {}
    for k in KEYS:
        name = formats.get(k, "q4_k")
        if name not in FMT_NAMES:
            raise ValueError(f"{cache_dir}: layer {layer_idx}: unknown {k} format {name!r}")
        fmts[k] = FMT_NAMES[name]
    if fmts["up"] != fmts["gate"]:
        raise ValueError(f"{cache_dir}: layer {layer_idx}: gate and up formats differ "
                         f"({formats.get('gate')}, {formats.get('up')}); the MoE call takes one gate/up format")
    want = {"gate": _matrix_bytes(fmts["gate"], I, D), "up": _matrix_bytes(fmts["up"], I, D),
            "down": _matrix_bytes(fmts["down"], D, I)}
    for k, (rows, cols) in (("gate", (I, D)), ("up", (I, D)), ("down", (D, I))):
        s = shapes.get(k)
        if s is not None and (int(s["out_dim"]), int(s["in_dim"])) != (rows, cols):
            raise ValueError(f"{cache_dir}: {k} shape {s} does not match embed_dim {D}, inter_dim {I}")

    path = cache_dir / info["file"]
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    offs = info["expert_offsets"]
    if len(offs) != E:
        raise ValueError(f"{path}: {len(offs)} experts, index says {E}")
    L = MoeLayer(D, I, fmts["gate"], ACT_CODES[act] if isinstance(act, str) else int(act),
                 int(top_k if top_k is not None else index["n_experts_used"]))
    for e in range(E):
        rec = offs[str(e)]
        pos = int(rec["offset"])
        views = []
        for k in KEYS:
            n = int(rec["sizes"][k])
            if n != want[k]:
                raise ValueError(f"{path}: expert {e} {k}: {n} bytes, the shapes and format need {want[k]}")
            if pos + n > len(mm):
                raise ValueError(f"{path}: expert {e} {k} runs past the end of the file")
            views.append(np.frombuffer(mm, dtype=np.uint8, count=n, offset=pos))
            pos += n
        L.gates.append(views[0])
        L.ups.append(views[1])
        L.downs.append(views[2])
        L.down_fmts.append(fmts["down"])
    L.router_w = np.ascontiguousarray(router_w, dtype=np.float32)
    if L.router_w.shape != (E, D):
        raise ValueError(f"router_w has shape {L.router_w.shape}, want {(E, D)}")
    L.router_b = None if router_b is None else np.ascontiguousarray(router_b, dtype=np.float32)
    L._mapping = mm   # the views point into it
    return L


def stack_from_cache(cache_dir, routers, router_biases=None, act="silu", top_k=None, layers=None):
    """One MoeLayer per layer index (all of the index's layers by default),
    with routers[i] / router_biases[i] for the i-th of them."""
    index = read_index(cache_dir)
    ids = sorted(int(k) for k in index["layers"]) if layers is None else list(layers)
    biases = router_biases if router_biases is not None else [None] * len(ids)
    return [layer_from_cache(cache_dir, l, routers[i], biases[i], act, top_k, index) for i, l in enumerate(ids)]


def write_cache(cache_dir, layers, n_experts_used=None, layer_ids=None, model="synthetic"):
    """Writes MoeLayers in the expert-cache format (layer files and
    index.json).  Every layer must have the same shapes and formats."""
    cache_dir = Path(cache_dir)
    cache_dir.mkdir(parents=True, exist_ok=True)
    ids = list(range(len(layers))) if layer_ids is None else list(layer_ids)
    names = {v: k for k, v in FMT_NAMES.items()}
    L0 = layers[0]
    D, I = L0.embed_dim, L0.inter_dim
    index = {"magic": MAGIC, "version": 2, "model": model, "model_path": "", "n_layers": len(layers),
             "n_experts": L0.n_experts, "n_experts_used": int(n_experts_used or L0.top_k), "embed_dim": D,
             "dtype": "quant", "expert_shapes": {}, "layers": {}, "activation_profile": None,
             "tensor_formats": {},
             "q4_sizes": {"gate": {"out_dim": I, "in_dim": D}, "up": {"out_dim": I, "in_dim": D},
                          "down": {"out_dim": D, "in_dim": I}}}
    for lid, L in zip(ids, layers):
        if (L.embed_dim, L.inter_dim, L.n_experts) != (D, I, L0.n_experts):
            raise ValueError("all layers must share embed_dim, inter_dim and n_experts")
        if len(set(L.down_fmts)) != 1:
            raise ValueError("one down format per layer")
        fname = f"layer_{lid:03d}.q4.bin"
        offsets, off = {}, 0
        with open(cache_dir / fname, "wb") as f:
            for e in range(L.n_experts):
                sizes = {}
                for k, m in zip(KEYS, (L.gates[e], L.ups[e], L.downs[e])):
                    b = np.ascontiguousarray(m, dtype=np.uint8).tobytes()
                    f.write(b)
                    sizes[k] = len(b)
                offsets[str(e)] = {"offset": off, "sizes": sizes}
                off += sum(sizes.values())
        index["layers"][str(lid)] = {"file": fname, "total_bytes": off, "expert_offsets": offsets,
                                     "tensor_formats": {"gate": names[L.gate_fmt], "up": names[L.gate_fmt],
                                                        "down": names[L.down_fmts[0]]}}
    tmp = cache_dir / "index.json.tmp"
    with open(tmp, "w") as f:
        json.dump(index, f, indent=2)
    os.replace(tmp, cache_dir / "index.json")
    return index

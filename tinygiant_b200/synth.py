"""Seeded synthetic inputs for the benchmark configurations.

There are no model files; every configuration is drawn from fixed seeds:
  C1  one Qwen3-30B-A3B-shaped expert, all Q4_K (gate/up 768x2048, down
      2048x768), W ~ N(0, 0.02), seed 0, x ~ N(0, 1).
  C2  one Qwen3 MoE layer: 128 experts, Q4_K gate/up, Q6_K down, fp32 router
      W_r ~ N(0, 0.02) [128 x 2048], top-8 softmax over the selected, seed 1.
  C3  C2 shapes with T in {1, 8, 64, 512} and a per-expert router bias that
      makes expert load Zipf(s=1.1)-skewed, seed 2.
  C4  gpt-oss-120b-shaped MXFP4 layers: D = I = 2880, 128 experts, top-4,
      e8m0 exponents uniform in [-8, -4], uniform e2m1 codes, seed 3.
  C5  48 stacked C2-shaped layers, residual x ~ N(0, 1) from seed 4.
Weights of expert e in layer l come from numpy's PCG64 seeded with
[seed, l, e], so any subset can be regenerated independently and in
parallel.

`route()` restates the reference router (tinygiant/router.py:29-42) and the
engine's union / row-weight construction (tinygiant/engine.py:297-318).
"""
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field

import numpy as np

from . import quants as Q

STD = 0.02


@dataclass
class MoeLayer:
    embed_dim: int
    inter_dim: int
    gate_fmt: int
    act: int
    top_k: int
    gates: list = field(default_factory=list)     # uint8 arrays, one per expert
    ups: list = field(default_factory=list)
    downs: list = field(default_factory=list)
    down_fmts: list = field(default_factory=list)
    router_w: np.ndarray = None                   # fp32 [E, D]
    router_b: np.ndarray = None                   # fp32 [E] or None

    @property
    def n_experts(self):
        return len(self.gates)

    def expert_bytes(self, e):
        return self.gates[e].nbytes + self.ups[e].nbytes + self.downs[e].nbytes


def _threads():
    import os
    return max(1, min(16, os.cpu_count() or 1))


def qwen_expert(seed, layer, e, D=2048, I=768, down_fmt=Q.FMT_Q6K):
    rng = np.random.default_rng([seed, layer, e])
    g = rng.standard_normal((I, D), dtype=np.float32) * STD
    u = rng.standard_normal((I, D), dtype=np.float32) * STD
    d = rng.standard_normal((D, I), dtype=np.float32) * STD
    pack_d = Q.pack_q6k if down_fmt == Q.FMT_Q6K else Q.pack_q4k
    return Q.pack_q4k(g), Q.pack_q4k(u), pack_d(d)


def gptoss_expert(seed, layer, e, D=2880, I=2880):
    rng = np.random.default_rng([seed, layer, e])
    return Q.mxfp4_random(I, D, rng), Q.mxfp4_random(I, D, rng), Q.mxfp4_random(D, I, rng)


def c1_expert(seed=0, D=2048, I=768):
    """One contiguous [gate | up | down] all-Q4_K expert (tg_expert_forward)."""
    g, u, d = qwen_expert(seed, 0, 0, D, I, down_fmt=Q.FMT_Q4K)
    return np.concatenate([g, u, d])


def qwen_layer(seed=1, layer=0, n_experts=128, D=2048, I=768, top_k=8, router_bias=None):
    L = MoeLayer(D, I, Q.FMT_Q4K, 0, top_k)
    with ThreadPoolExecutor(_threads()) as ex:
        parts = list(ex.map(lambda e: qwen_expert(seed, layer, e, D, I), range(n_experts)))
    for g, u, d in parts:
        L.gates.append(g)
        L.ups.append(u)
        L.downs.append(d)
        L.down_fmts.append(Q.FMT_Q6K)
    rng = np.random.default_rng([seed, layer, 1 << 20])
    L.router_w = rng.standard_normal((n_experts, D), dtype=np.float32) * STD
    L.router_b = router_bias
    return L


def gptoss_layer(seed=3, layer=0, n_experts=128, D=2880, I=2880, top_k=4):
    L = MoeLayer(D, I, Q.FMT_MXFP4, 1, top_k)
    with ThreadPoolExecutor(_threads()) as ex:
        parts = list(ex.map(lambda e: gptoss_expert(seed, layer, e, D, I), range(n_experts)))
    for g, u, d in parts:
        L.gates.append(g)
        L.ups.append(u)
        L.downs.append(d)
        L.down_fmts.append(Q.FMT_MXFP4)
    rng = np.random.default_rng([seed, layer, 1 << 20])
    L.router_w = rng.standard_normal((n_experts, D), dtype=np.float32) * STD
    return L


def zipf_bias(seed=2, n_experts=128, s=1.1):
    """Router bias b_e = -s*ln(rank_e) over a random ranking of the experts, so
    the chance of an expert being selected falls off as a Zipf(s) law of
    its rank."""
    rng = np.random.default_rng([seed, 1 << 21])
    rank = rng.permutation(n_experts) + 1
    return (-s * np.log(rank)).astype(np.float32)


def rms_norm(x, w=None, eps=1e-6):
    """The engine's ffn RMSNorm (engine.py:281-282): X / sqrt(mean(X^2) + eps) * w."""
    x = np.asarray(x, dtype=np.float32)
    rr = np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + np.float32(eps))
    y = x / rr
    return (y * w if w is not None else y).astype(np.float32)


def route(layer, N):
    """Reference routing for rows N [T, D].

    Per row: logits = W_r @ n (+ b); top-k by argpartition, ordered by
    descending logit; weights = softmax over the selected logits (float32)
    (router.py:29-42).  The union of selected experts, ascending by id, with a
    dense [n, T] row-weight matrix (engine.py:297-318).
    Returns (experts[n], row_w[n, T], idx[T, k], wts[T, k]).
    """
    N = np.atleast_2d(np.asarray(N, dtype=np.float32))
    T = N.shape[0]
    k = layer.top_k
    idxs, wts = [], []
    union = {}
    for r in range(T):
        logits = layer.router_w @ N[r]
        if layer.router_b is not None:
            logits = logits + layer.router_b
        idx = np.argpartition(logits, -k)[-k:]
        idx = idx[np.argsort(logits[idx])[::-1]]
        l = logits[idx]
        e = np.exp(l - l.max())
        w = (e / e.sum()).astype(np.float32)
        idxs.append(idx)
        wts.append(w)
        for ei, wt in zip(idx, w):
            union.setdefault(int(ei), {})[r] = float(wt)
    experts = sorted(union)
    row_w = np.zeros((len(experts), T), np.float32)
    for i, e in enumerate(experts):
        for r, wt in union[e].items():
            row_w[i, r] = wt
    return np.array(experts, dtype=np.int64), row_w, np.array(idxs), np.array(wts, dtype=np.float32)

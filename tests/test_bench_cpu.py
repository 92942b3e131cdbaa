"""bench.py's reference arm and workload plumbing on the host (no GPU): the
reference arm prints one JSON line in the contract's shape for a stack
workload, and the stack / layer selection follows --config and --layers."""
import json
import os
import subprocess
import sys
import types

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _args(**kw):
    a = types.SimpleNamespace(config="c2", layers=None, tokens=None)
    a.__dict__.update(kw)
    return a


def test_stack_selection():
    assert not bench.is_stack(_args(config="c2"))
    assert bench.is_stack(_args(config="c5")) and bench.n_layers(_args(config="c5")) == 48
    assert bench.is_stack(_args(config="c4")) and bench.n_layers(_args(config="c4")) == 36
    assert not bench.is_stack(_args(config="c4", layers=1))
    assert bench.n_layers(_args(config="c5", layers=3)) == 3


def test_stack_bytes_counts_distinct_experts():
    from tinygiant_b200 import synth
    L = synth.qwen_layer(seed=1, n_experts=8)
    one = bench.stack_bytes(L, 2, 1)
    assert one == 2 * (L.top_k * L.expert_bytes(0) + L.router_w.nbytes + 2 * L.embed_dim * 4)
    assert bench.stack_bytes(L, 2, 4, uniq=5.0) == 2 * (5.0 * L.expert_bytes(0) + L.router_w.nbytes + 8 * L.embed_dim * 4)


def test_reference_arm_prints_contract_line():
    env = dict(os.environ, RANK="0")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "c5",
                          "--layers", "2", "--steps", "1", "--warmup", "1"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["value"] > 0
    assert d["config"]["layers"] == 2
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["cores"] >= 1


def _run_reference_arm(*args):
    """The reference arm in a child process; returns (its JSON line, the
    shared objects the process had mapped when it finished)."""
    code = ("import sys; sys.argv = ['bench.py'] + sys.argv[1:]; import bench; bench.main(); "
            "maps = open('/proc/self/maps').read(); "
            "print('MAPS ' + ' '.join(sorted({l.split()[-1] for l in maps.splitlines() if '.so' in l})))")
    env = dict(os.environ, RANK="0")
    out = subprocess.run([sys.executable, "-c", code, "--impl", "reference", *args], capture_output=True, text=True,
                         timeout=600, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    maps = [l for l in out.stdout.splitlines() if l.startswith("MAPS ")]
    assert len(lines) == 1 and len(maps) == 1
    return json.loads(lines[0]), maps[0].split()[1:]


def test_reference_arm_matches_our_config_and_loads_no_product_code():
    """C2 on the reference arm: the same `config` our arm reports (same layer
    copies), and only the reference's own C library from this repository is
    mapped (never tinygiant_b200/libtinygiant.so)."""
    from tinygiant_b200 import synth
    d, maps = _run_reference_arm("--config", "c2", "--copies", "2", "--steps", "2", "--warmup", "1")
    L = synth.qwen_layer(seed=1)
    assert d["config"] == bench.workload_desc("c2", 1, 2, L)
    assert d["scaling"] == "strong" and d["e2e"]["d2h_bytes_per_step"] == 0
    assert not any("libtinygiant.so" in m and "oracle" not in m for m in maps), maps
    assert any("oracle" in m for m in maps)


def test_reference_arm_c1():
    d, _ = _run_reference_arm("--config", "c1", "--copies", "3", "--steps", "3", "--warmup", "1")
    assert d["config"] == bench.workload_desc("c1", 1, 3, None)
    assert d["value"] > 0 and d["unit"] == "tok/s"


def test_parallel_defaults_to_expert_sharding_on_several_gpus(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    monkeypatch.setenv("WORLD_SIZE", "4")
    a = bench.parse()
    assert a.parallel == "ep" and bench.scaling_of(a, "c2") == "strong"
    monkeypatch.setenv("WORLD_SIZE", "1")
    assert bench.parse().parallel == "dp"
    monkeypatch.setattr(sys, "argv", ["bench.py", "--parallel", "dp"])
    monkeypatch.setenv("WORLD_SIZE", "4")
    a = bench.parse()
    assert a.parallel == "dp" and bench.scaling_of(a, "c2") == "weak"

"""bench.py's reference arm runs on the host alone: its CPU ports build
numpy inputs, load neither torch nor this runtime, and report the same
config object as the GPU arm's line."""
import argparse
import importlib.util
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_ports_need_no_gpu_runtime():
    code = (
        "import sys, argparse; sys.argv=['bench.py']\n"
        "import importlib.util, os\n"
        f"spec=importlib.util.spec_from_file_location('b', {os.path.join(ROOT, 'bench.py')!r})\n"
        "b=importlib.util.module_from_spec(spec); spec.loader.exec_module(b)\n"
        "a=argparse.Namespace(groups=0, chunk_pages=0)\n"
        "for n in ('sampling', 'decode_ring'):\n"
        "    r=b.WORKLOADS[n].cpu_port(a, 2, 0.2)\n"
        "    assert r['value'] > 0 and r['kind'] == 'port', r\n"
        "assert 'torch' not in sys.modules, 'the reference arm imported torch'\n"
        "assert 'gb300_rl_runtime_b200' not in sys.modules, 'the reference arm loaded the runtime'\n"
        "print('ok')\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert "ok" in out.stdout


def test_both_arms_share_the_config_object():
    b = _bench()
    a = argparse.Namespace(groups=0, chunk_pages=0)
    for name, cls in b.WORKLOADS.items():
        for world in (1, 2, 8):
            c1 = cls.line_config(a, world)
            c2 = cls.line_config(a, world)
            assert c1 == c2 and c1["workload"] == cls.name
            assert ("dp" in c1["parallelism"]) == (cls.scaling == "strong" and world > 1)
    assert b.WORKLOADS["rollout"].scaling == "strong"
    assert b.WORKLOADS["rollout_c4"].line_config(a, 1)["rollouts"] == 1024

"""bench.py's reference arm runs the CPU restatement only: it must not load
the CUDA library (the arm measures the reference's CPU path, not this
build), and its `config` must equal the CUDA arm's for the same workload."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROBE = r"""
import argparse, json, sys
sys.path.insert(0, ROOT)
import bench
args = argparse.Namespace(config="c2", warmup=1, steps=1, t_stop=None, binning="contributing")
cfg = dict(bench.CONFIGS["c2"], n=3000, W=64, H=48, views=2)
res = bench.reference_train(args, cfg, 1)
maps = open("/proc/self/maps").read()
print(json.dumps({"res": res, "cuda_lib": "libgsplat_cuda" in maps, "oracle_lib": "libgs_oracle" in maps,
                  "config": bench.workload_config(args, cfg, 1)}))
"""


def test_reference_arm_loads_only_the_oracle():
    out = subprocess.run([sys.executable, "-c", PROBE.replace("ROOT", repr(ROOT))], capture_output=True,
                         text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["oracle_lib"] and not d["cuda_lib"]
    res = d["res"]
    assert res["impl"] == "reference" and res["value"] > 0
    assert res["config"] == d["config"]
    assert res["e2e"]["h2d_bytes_per_step"] == 0 and res["cpu_baseline"]["kind"] == "port"


def test_oracle_default_config_equals_the_library_default(oracle):
    import ctypes as C
    from helpers import _abi
    a = oracle.default_config()
    b = _abi.default_config()
    assert bytes(a) == bytes(b)
    assert C.sizeof(a) == C.sizeof(_abi.RasterConfig)

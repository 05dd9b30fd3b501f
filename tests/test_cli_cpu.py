"""Every command-line entry point imports and parses its arguments (``--help``) without a GPU."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENTRY_POINTS = [
    ["train.py"], ["generate.py"], ["bench.py"], ["bench_inference.py"], ["bench_kernels.py"],
    ["-m", "pan2_b200.checkpoint.convert"], ["-m", "pan2_b200.inference.prompt_rewriter"],
    ["-m", "pan2_b200.data.make_sample_data"], ["-m", "pan2_b200.checkpoint.io"],
]


@pytest.mark.parametrize("cmd", ENTRY_POINTS, ids=[" ".join(c) for c in ENTRY_POINTS])
def test_entry_point_help(cmd):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable] + cmd + ["--help"], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "usage" in r.stdout.lower()


def test_graft_entry_imports_built_extension():
    if not any(f.startswith("_C.") and f.endswith(".so") for f in os.listdir(os.path.join(ROOT, "pan2_b200"))):
        pytest.skip("extension not built")
    r = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.import_package(); print('ok')"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-2000:]

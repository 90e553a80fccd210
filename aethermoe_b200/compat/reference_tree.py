"""Runs an AetherMoE checkout's own Python tests and benchmarks against this
library, unmodified.

The reference's tests and benchmarks find the kernels by putting paths
relative to their own file on ``sys.path``: ``src/kernels`` (and
``validation``, ``prototype``), see ``tests/python/test_gating_numerical.py:20-28``
and ``benchmarks/bench_gating.py:24`` -- and they import ``mlx.core``.
``make_tree(ref_root, dest)`` lays out a tree in which those paths resolve to
this build:

* ``tests/python``, ``benchmarks``, ``validation`` and ``prototype`` are
  copied from the checkout as they are (nothing is edited);
* ``src/kernels/{fused_gating_metal,reference_gating,quantized_gemm}.py`` are
  one-statement modules that make the import name refer to this package's
  shim module (``aethermoe_b200.kernels.*``), so the reference's
  ``from fused_gating_metal import fused_gating`` gets the CUDA path;

and ``environment()`` gives the ``PYTHONPATH`` under which ``mlx.core``
resolves to the NumPy stand-in ``aethermoe_b200/compat/mlx``.

    python -m aethermoe_b200.compat.reference_tree <AetherMoE root> <dest> [--run]

``--run`` then runs ``pytest tests/python`` and the two kernel benchmarks in
that tree (each as a subprocess) and exits non-zero if any fails.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PACKAGE_ROOT = os.path.dirname(os.path.dirname(HERE))  # the directory holding aethermoe_b200/

COPIED = ("tests/python", "benchmarks", "validation", "prototype")
SHIMS = ("fused_gating_metal", "reference_gating", "quantized_gemm")
BENCHMARKS = (
    ("benchmarks/bench_gating.py", ["--n-tokens", "256", "--d-model", "1024",
                                    "--num-experts", "16", "--k", "4"]),
    ("benchmarks/bench_quantized_gemm.py", []),
)

_ALIAS = '''"""Import name of the reference module; resolves to aethermoe_b200.kernels.{name}."""
import importlib
import sys

sys.modules[__name__] = importlib.import_module("aethermoe_b200.kernels.{name}")
'''


def make_tree(ref_root, dest):
    """Builds the drop-in tree under ``dest`` from the checkout at ``ref_root``."""
    ref_root = os.path.abspath(ref_root)
    if not os.path.isdir(os.path.join(ref_root, "tests", "python")):
        raise FileNotFoundError(f"{ref_root} has no tests/python: not an AetherMoE checkout")
    os.makedirs(dest, exist_ok=True)
    for rel in COPIED:
        src = os.path.join(ref_root, rel)
        if os.path.isdir(src):
            shutil.copytree(src, os.path.join(dest, rel), dirs_exist_ok=True,
                            ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    kdir = os.path.join(dest, "src", "kernels")
    os.makedirs(kdir, exist_ok=True)
    for name in SHIMS:
        with open(os.path.join(kdir, name + ".py"), "w") as f:
            f.write(_ALIAS.format(name=name))
    return dest


def environment(base=None):
    """Environment for processes run in the tree: this package and the
    ``mlx`` stand-in first on ``PYTHONPATH``."""
    env = dict(os.environ if base is None else base)
    paths = [PACKAGE_ROOT, HERE]
    if env.get("PYTHONPATH"):
        paths.append(env["PYTHONPATH"])
    env["PYTHONPATH"] = os.pathsep.join(paths)
    return env


def run(dest, timeout=900):
    """Runs the reference's pytest suite and kernel benchmarks in the tree;
    returns ``[(what, returncode, output)]``."""
    env = environment()
    results = []
    cmd = [sys.executable, "-m", "pytest", "tests/python", "-q", "-p", "no:cacheprovider",
           "-rs"]
    r = subprocess.run(cmd, cwd=dest, env=env, stdout=subprocess.PIPE,
                       stderr=subprocess.STDOUT, text=True, timeout=timeout)
    results.append(("pytest tests/python", r.returncode, r.stdout))
    for script, extra in BENCHMARKS:
        if not os.path.exists(os.path.join(dest, script)):
            continue
        r = subprocess.run([sys.executable, script] + extra, cwd=dest, env=env,
                           stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                           timeout=timeout)
        results.append((script, r.returncode, r.stdout))
    return results


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) < 2:
        print(__doc__)
        return 2
    dest = make_tree(argv[0], argv[1])
    if "--run" not in argv:
        print(dest)
        return 0
    rc = 0
    for what, code, out in run(dest):
        print(f"==== {what}: exit {code}\n{out}")
        rc = rc or code
    return rc


if __name__ == "__main__":
    sys.exit(main())

"""The reference's own Python tests and kernel benchmarks, unmodified, against
this library (``aethermoe_b200.compat.reference_tree``).

The GPU test needs an AetherMoE checkout: ``AEM_REFERENCE_ROOT=<root>``.  Its
test files are copied into a temporary tree at run time (they are not part of
this repository); without the variable the test is skipped with that reason.
The CPU test checks the tree's import plumbing on a stand-in checkout.
"""
import os
import subprocess
import sys
import textwrap

import pytest

from aethermoe_b200.compat import reference_tree


def test_tree_resolves_reference_imports_to_the_shim(tmp_path):
    """A stand-in checkout whose test imports the kernels the way the
    reference's tests do (``sys.path`` relative to the test file) gets this
    package's shim modules and the ``mlx.core`` stand-in."""
    ref = tmp_path / "ref"
    (ref / "tests" / "python").mkdir(parents=True)
    (ref / "tests" / "python" / "test_probe.py").write_text(textwrap.dedent('''
        import os, sys
        sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "..", "src", "kernels"))
        import mlx.core as mx
        from fused_gating_metal import fused_gating, MAX_EXPERTS
        from quantized_gemm import quantize_weights, fused_quantized_matmul
        import reference_gating

        def test_probe():
            assert fused_gating.__module__ == "aethermoe_b200.kernels.fused_gating_metal"
            assert reference_gating.__name__ == "aethermoe_b200.kernels.reference_gating"
            assert mx.__name__ == "mlx.core" and hasattr(mx, "array")
            assert MAX_EXPERTS == 256
    '''))
    dest = reference_tree.make_tree(str(ref), str(tmp_path / "tree"))
    r = subprocess.run([sys.executable, "-m", "pytest", "tests/python", "-q", "-p",
                        "no:cacheprovider"], cwd=dest, env=reference_tree.environment(),
                       stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=300)
    assert r.returncode == 0, r.stdout
    assert "1 passed" in r.stdout


@pytest.mark.gpu
def test_reference_suite_passes_through_the_shim(cuda, tmp_path):
    """``tests/python/*.py`` (pytest) and ``benchmarks/bench_gating.py`` /
    ``bench_quantized_gemm.py`` of the checkout at AEM_REFERENCE_ROOT, run
    unmodified: every test passes (none skipped for a missing ``mlx``) and
    both benchmarks exit 0 (their own regression checks included)."""
    root = os.environ.get("AEM_REFERENCE_ROOT")
    if not root or not os.path.isdir(os.path.join(root, "tests", "python")):
        pytest.skip("AEM_REFERENCE_ROOT does not name an AetherMoE checkout")
    dest = reference_tree.make_tree(root, str(tmp_path / "tree"))
    results = reference_tree.run(dest)
    report = "\n".join(f"==== {w}: exit {c}\n{o}" for w, c, o in results)
    print(report)
    assert all(c == 0 for _, c, _ in results), report
    suite = results[0][2]
    assert " passed" in suite and "failed" not in suite and "skipped" not in suite, suite

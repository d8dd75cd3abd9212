"""Runs the HELM reference's own allocator and cache-manager unit tests against
helm_b200.runtime (the drop-in check of the Python boundary).

    python tests/golden/run_reference_tests.py [--ref <helm checkout>]

The reference's tests import `helm.runtime.kv_allocator` and
`helm.runtime.kv_cache`; a throw-away package named `helm` in a temporary
directory re-exports helm_b200.runtime's modules under those names, the two
test files are copied next to it, and pytest runs them there (nothing is
written into the reference checkout or this repository).  Tests that need a
GPU skip on a machine without one; their restatements run on the GPU in
tests/test_reference_cases_gpu.py.  The reference's attention tests are not
run: they compute attention for queries on the CPU, which helm_b200 leaves to
HELM's own code.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
FILES = ("test_kv_allocator.py", "test_kv_cache.py")
SHIM = '''from helm_b200.runtime import {mod} as _m
globals().update({{k: getattr(_m, k) for k in dir(_m) if not k.startswith("__")}})
'''


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HELM_REFERENCE"),
                    help="HELM checkout whose tests to run (default: $HELM_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the HELM checkout with --ref or HELM_REFERENCE")
    src = os.path.join(args.ref, "tests", "unit", "runtime")
    with tempfile.TemporaryDirectory() as tmp:
        pkg = os.path.join(tmp, "helm", "runtime")
        os.makedirs(pkg)
        open(os.path.join(tmp, "helm", "__init__.py"), "w").close()
        open(os.path.join(pkg, "__init__.py"), "w").close()
        for mod in ("kv_allocator", "kv_cache"):
            with open(os.path.join(pkg, mod + ".py"), "w") as f:
                f.write(SHIM.format(mod=mod))
        for name in FILES:
            shutil.copy(os.path.join(src, name), tmp)
        env = dict(os.environ, PYTHONPATH=os.pathsep.join([tmp, REPO]),
                   PYTHONDONTWRITEBYTECODE="1")
        res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-rs", "-p",
                              "no:cacheprovider", *FILES], cwd=tmp, env=env,
                             capture_output=True, text=True)
    print("\n".join(res.stdout.strip().splitlines()[-20:]))
    return res.returncode


if __name__ == "__main__":
    sys.exit(main())

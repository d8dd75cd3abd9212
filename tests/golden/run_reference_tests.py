"""Runs the HELM reference's own allocator and cache-manager unit tests against
helm_b200.runtime (the drop-in check of the Python boundary).

    python tests/golden/run_reference_tests.py [--ref <helm checkout>]

The reference's tests import `helm.runtime.kv_allocator` and
`helm.runtime.kv_cache`; a throw-away package named `helm` in a temporary
directory re-exports helm_b200.runtime's modules under those names, the two
test files are copied next to it, and pytest runs them there (nothing is
written into the reference checkout).  The outcome is stored in
tests/golden/reference_unit_tests.txt.  Tests that need a GPU skip on a
machine without one.  The reference's attention tests are not run: they
compute attention for queries on the CPU, which helm_b200 leaves to HELM's own
code.
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
    ap.add_argument("--ref", default=os.environ.get("HELM_REFERENCE", "/root/reference"))
    args = ap.parse_args()
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
    report = res.stdout.strip().splitlines()
    out = os.path.join(HERE, "reference_unit_tests.txt")
    with open(out, "w") as f:
        f.write("HELM's tests/unit/runtime/{" + ",".join(FILES) + "} run against "
                "helm_b200.runtime (tests/golden/run_reference_tests.py)\n\n")
        f.write("\n".join(report[-20:]) + "\n")
    print("\n".join(report[-5:]))
    return res.returncode


if __name__ == "__main__":
    sys.exit(main())

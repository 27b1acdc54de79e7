"""The build entry point compiles (a no-op when up to date) and imports both
extensions in a fresh interpreter, as a build check on a machine without a GPU does."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_build_entry_point_imports_extensions():
    r = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.build(); print('BUILD_OK')"],
                       cwd=ROOT, capture_output=True, text=True, timeout=1800)
    assert r.returncode == 0 and "BUILD_OK" in r.stdout, (r.stdout + r.stderr)[-3000:]

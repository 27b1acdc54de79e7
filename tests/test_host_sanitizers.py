"""The C++ host core under AddressSanitizer + UndefinedBehaviorSanitizer (CPU).

Builds csrc/host/*.cpp with -fsanitize=address,undefined into a temporary
`_host` module, then runs the tokenizer and data-pipeline tests in a child
process with that module in place of the regular build (the sanitizer runtime
is preloaded; leak checking is off because the interpreter itself does not
free everything at exit). Any sanitizer report fails the child, and so this test.
"""
import glob
import os
import subprocess
import sys
import sysconfig

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PLUGIN = r'''
import importlib.util, os, sys
import rs_nanogpt_b200
spec = importlib.util.spec_from_file_location("rs_nanogpt_b200._host", os.environ["NANOGPT_SANITIZED_HOST"])
mod = importlib.util.module_from_spec(spec)
spec.loader.exec_module(mod)
sys.modules["rs_nanogpt_b200._host"] = mod
rs_nanogpt_b200._host = mod
'''


def _runtime(name):
    out = subprocess.run(["g++", f"-print-file-name={name}"], capture_output=True, text=True).stdout.strip()
    return out if os.path.isabs(out) and os.path.exists(out) else None


@pytest.mark.slow
def test_host_core_under_asan_ubsan(tmp_path):
    asan, ubsan = _runtime("libasan.so"), _runtime("libubsan.so")
    if asan is None or ubsan is None:
        pytest.skip("no sanitizer runtimes in this toolchain")
    import pybind11
    so = tmp_path / "_host_sanitized.so"
    srcs = sorted(glob.glob(os.path.join(ROOT, "csrc", "host", "*.cpp")))
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined",
           "-fno-sanitize-recover=undefined", "-shared", "-fPIC", "-pthread", "-fvisibility=hidden",
           "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"], *srcs, "-o", str(so)]
    subprocess.run(cmd, check=True, cwd=ROOT)
    (tmp_path / "sanitized_host_plugin.py").write_text(PLUGIN)
    env = dict(os.environ)
    env.update({
        "LD_PRELOAD": f"{asan}:{ubsan}",
        "ASAN_OPTIONS": "detect_leaks=0:verify_asan_link_order=0:abort_on_error=1",
        "UBSAN_OPTIONS": "print_stacktrace=1:halt_on_error=1",
        "NANOGPT_SANITIZED_HOST": str(so),
        "PYTHONPATH": str(tmp_path) + os.pathsep + ROOT,
    })
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                        "-p", "sanitized_host_plugin", "-m", "not gpu and not slow",
                        "tests/test_tokenizer.py", "tests/test_data.py"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    assert "AddressSanitizer" not in tail and "runtime error" not in tail, tail

"""The host-side native runtime (.dlvk container, batch gather thread pool,
IDX files, SafeTensors / GGUF) built and run under AddressSanitizer +
UndefinedBehaviorSanitizer and under ThreadSanitizer (no GPU needed)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "dlvk_b200", "csrc")
SRCS = [os.path.join(CSRC, "tests", "runtime_selftest.cpp")] + [
    os.path.join(CSRC, "runtime", f) for f in ("dlvk_io.cpp", "data_loader.cpp", "export_formats.cpp")]


def _build_and_run(tmp_path, flags):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    exe = str(tmp_path / "selftest")
    b = subprocess.run(["g++", "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", *flags, "-I",
                        os.path.join(CSRC, "include"), *SRCS, "-o", exe, "-lpthread"],
                       capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "sanitize" in b.stderr:
        pytest.skip("sanitizer runtime not available: " + b.stderr[-300:])
    assert b.returncode == 0, b.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=1", UBSAN_OPTIONS="halt_on_error=1",
               TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and "ok" in r.stdout, (r.stdout + r.stderr)[-3000:]


def test_runtime_asan_ubsan(tmp_path):
    _build_and_run(tmp_path, ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"])


def test_runtime_tsan(tmp_path):
    _build_and_run(tmp_path, ["-fsanitize=thread"])

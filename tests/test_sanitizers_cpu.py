"""Host C++ runtime (block manager, IPC framing, GGUF index) under AddressSanitizer and
UndefinedBehaviorSanitizer: the sources are rebuilt instrumented and driven from a
child Python process with the sanitizer runtimes preloaded."""
import os
import pathlib
import shutil
import subprocess
import sys
import sysconfig

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_runtime_under_asan_ubsan(tmp_path):
    import pybind11
    libs = [subprocess.check_output(["gcc", f"-print-file-name={n}"], text=True).strip()
            for n in ("libasan.so", "libubsan.so")]
    if not all(os.path.isabs(l) and os.path.exists(l) for l in libs):
        pytest.skip("sanitizer runtimes not installed")
    out = tmp_path / ("_rt" + sysconfig.get_config_var("EXT_SUFFIX"))
    srcs = [str(ROOT / "csrc/runtime" / f) for f in ("block_manager.cpp", "ipc.cpp", "gguf.cpp", "module.cpp")]
    subprocess.check_call(["g++", "-O1", "-g", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
                           "-fno-sanitize-recover=undefined", "-std=c++17", "-shared", "-fPIC",
                           f"-I{ROOT / 'csrc'}", f"-I{sysconfig.get_paths()['include']}",
                           f"-I{pybind11.get_include()}", *srcs, "-o", str(out)])
    env = dict(os.environ, LD_PRELOAD=" ".join(libs), ASAN_OPTIONS="detect_leaks=0:abort_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
    r = subprocess.run([sys.executable, str(ROOT / "tests/sanitize/drive_runtime.py"), str(tmp_path)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    assert "AddressSanitizer" not in r.stderr and "runtime error" not in r.stderr
    assert "ok" in r.stdout

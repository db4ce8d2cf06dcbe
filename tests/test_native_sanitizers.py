"""Host runtime under sanitizers: the shard directory, the AMF disk store and the n-gram index are built
from source with AddressSanitizer + UndefinedBehaviorSanitizer and with ThreadSanitizer,
and a multi-threaded stress program (csrc/native/tests/native_stress.cpp) runs against
each build. A data race, leak, overflow or undefined behaviour aborts the program."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = [os.path.join(ROOT, "csrc", "native", f) for f in ("tests/native_stress.cpp", "amf_store.cpp", "shard_dir.cpp", "ngram.cpp")]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
@pytest.mark.parametrize("san", ["address,undefined", "thread"])
def test_native_store_under_sanitizer(san, tmp_path):
    exe = tmp_path / "native_stress"
    build = subprocess.run(["g++", "-std=c++17", "-O1", "-g", f"-fsanitize={san}", "-fno-omit-frame-pointer",
                            "-DAXR_NO_PYBIND", "-I", os.path.join(ROOT, "csrc", "native"), *SRC, "-o", str(exe), "-lpthread", "-lrt"],
                           capture_output=True, text=True, timeout=600)
    assert build.returncode == 0, build.stderr[-3000:]
    data = tmp_path / "amf"
    data.mkdir()
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=1", UBSAN_OPTIONS="halt_on_error=1",
               TSAN_OPTIONS="halt_on_error=1")
    r = subprocess.run([str(exe), str(data)], capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "native_stress ok" in r.stdout

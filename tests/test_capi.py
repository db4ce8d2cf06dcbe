"""C ABI (libkorith_b200.so, csrc/capi/korith.h): the korith_* and korith_engine_* entry
points, called through ctypes in this process and from a plain C program in a child
process (which starts its own embedded Python runtime)."""
import ctypes
import os
import subprocess
import sys
import tempfile

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "axropus_deploy_b200", "libkorith_b200.so")
PROMPT = b"hello korith, tell me about paged kv caches"


class Params(ctypes.Structure):
    _fields_ = [("n_ctx", ctypes.c_int32), ("n_batch", ctypes.c_int32), ("n_gpu", ctypes.c_int32),
                ("model_path", ctypes.c_char_p)]


class Metrics(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("prefill_ms", "decode_ms", "total_ms", "restore_ms", "verify_ms",
                                               "draft_ms")] + \
               [(n, ctypes.c_int32) for n in ("tokens_out", "accepted_tokens", "rejected_tokens")]


def _lib():
    if not os.path.exists(LIB):
        pytest.skip("libkorith_b200.so not built")
    lib = ctypes.CDLL(LIB)
    lib.korith_init.restype = ctypes.c_bool
    lib.korith_init.argtypes = [ctypes.c_char_p, ctypes.c_int]
    lib.korith_tokenize.argtypes = [ctypes.c_char_p]
    lib.korith_last_error.restype = ctypes.c_char_p
    for f in ("korith_engine_init_model", "korith_engine_prefill", "korith_engine_decode_step",
              "korith_engine_get_logits", "korith_engine_export_snapshot", "korith_engine_import_snapshot",
              "korith_engine_verify_tokens", "korith_engine_cuda_probe", "korith_engine_apply_kv_replay"):
        getattr(lib, f).restype = ctypes.c_bool
    return lib


def _reference_tokens(n):
    """Greedy continuation of the byte-tokenised prompt by the engine (same preset/seed)."""
    from axropus_deploy_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    m = LlamaModel(get_config("tiny128"), "cpu", torch.float32, seed=0)
    eng = LLMEngine(m, EngineConfig(num_blocks=64, max_batch=2, max_model_len=256))
    return eng.generate([list(PROMPT)], SamplingParams(max_tokens=n))[0]


@pytest.fixture(autouse=True)
def _cpu(monkeypatch):
    monkeypatch.setenv("AXR_DEVICE", "cpu")


def test_korith_init_tokenize_step():
    lib = _lib()
    assert lib.korith_init(b"tiny128", 256), lib.korith_last_error()
    assert lib.korith_tokenize(PROMPT) == len(PROMPT)
    got = [lib.korith_step() for _ in range(6)]
    lib.korith_shutdown()
    # the first generated token comes from the prompt's logits; korith_step returns it
    assert got == _reference_tokens(6)
    assert lib.korith_step() == -1  # shut down: no session


def test_engine_abi_roundtrip():
    lib = _lib()
    p = Params(256, 64, 0, b"tiny128")
    assert lib.korith_engine_init_model(ctypes.byref(p)), lib.korith_last_error()
    toks = (ctypes.c_int32 * len(PROMPT))(*PROMPT)
    assert lib.korith_engine_prefill(toks, len(PROMPT))
    logits = (ctypes.c_float * 32000)()
    assert lib.korith_engine_get_logits(logits, 32000)
    first = max(range(32000), key=lambda i: logits[i])
    out = ctypes.c_int32()
    assert lib.korith_engine_decode_step(ctypes.byref(out)) and out.value == first
    # verification: propose the next greedy tokens (computed by a second session), all accepted
    ref = _reference_tokens(5)
    prop = (ctypes.c_int32 * 4)(*ref[1:5])
    acc = ctypes.c_int32(-1)
    assert lib.korith_engine_verify_tokens(prop, 4, ctypes.byref(acc)) and acc.value == 4
    bad = (ctypes.c_int32 * 2)(7, 7)
    assert lib.korith_engine_verify_tokens(bad, 2, ctypes.byref(acc)) and acc.value < 2
    m = Metrics()
    lib.korith_engine_get_metrics(ctypes.byref(m))
    assert m.tokens_out == 1 and m.accepted_tokens >= 4 and m.prefill_ms > 0
    # snapshot: 48 tokens = 3 full pages, exported, re-imported into a fresh session
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "snap.kv").encode()
        assert lib.korith_engine_export_snapshot(path)
        lib.korith_engine_shutdown()
        assert lib.korith_engine_init_model(ctypes.byref(p))
        assert lib.korith_engine_import_snapshot(path), lib.korith_last_error()
        l2 = (ctypes.c_float * 32000)()
        assert lib.korith_engine_get_logits(l2, 32000)
        # reference: the same 48 tokens prefilled directly
        from axropus_deploy_b200 import capi

        s = capi.CSession("tiny128", 256, "cpu")
        full = list(PROMPT) + [first] + ref[1:5]
        s.prefill(full[:48])
        want = s.get_logits()
        assert max(abs(l2[i] - float(want[i])) for i in range(0, 32000, 97)) < 1e-3
    lib.korith_engine_shutdown()
    assert not lib.korith_engine_cuda_probe() or torch.cuda.is_available()


C_PROGRAM = r"""
#include <dlfcn.h>
#include <stdbool.h>
#include <stdio.h>
int main(int argc, char** argv) {
  void* h = dlopen(argv[1], RTLD_NOW | RTLD_GLOBAL);
  if (!h) { fprintf(stderr, "dlopen: %s\n", dlerror()); return 2; }
  bool (*init)(const char*, int) = dlsym(h, "korith_init");
  int (*tok)(const char*) = dlsym(h, "korith_tokenize");
  int (*step)(void) = dlsym(h, "korith_step");
  void (*shut)(void) = dlsym(h, "korith_shutdown");
  const char* (*err)(void) = dlsym(h, "korith_last_error");
  if (!init("tiny128", 256)) { fprintf(stderr, "init: %s\n", err()); return 3; }
  int n = tok(argv[2]);
  printf("prompt %d\n", n);
  for (int i = 0; i < 6; ++i) printf("%d\n", step());
  shut();
  return 0;
}
"""


def test_standalone_c_program():
    _lib()
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "main.c"), os.path.join(d, "main")
        with open(src, "w") as f:
            f.write(C_PROGRAM)
        subprocess.check_call(["gcc", "-O1", src, "-o", exe, "-ldl"])
        env = dict(os.environ, AXR_DEVICE="cpu")
        r = subprocess.run([exe, LIB, PROMPT.decode()], capture_output=True, text=True, env=env, timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        lines = r.stdout.split()
        assert lines[:2] == ["prompt", str(len(PROMPT))]
        assert [int(x) for x in lines[2:]] == _reference_tokens(6)

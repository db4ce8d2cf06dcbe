"""Device-side failure detection without a GPU fault: a bounded wait is made to run out.

The tensor-parallel all-gather -> GEMM kernel (csrc/kernels/gemm_tp.cu, AG mode) is
launched on one GPU as rank 0 of a group of two whose peer never announces its shard:
the peer's "ready" flag lives in a buffer nothing writes. The kernel's communication
warps wait for it with the bound AXR_PEER_WAIT_MS (50 ms here), record the wait's error
code, drain and return; the host reads the code, and the serving engine refuses to use
the step (LLMEngine.step raises). Runs in a child process so the wait bound (read once
per process) is the short one. Nothing spins without a bound, nothing faults, and the
context stays usable (the child runs an engine step afterwards)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys, time, torch
sys.path.insert(0, sys.argv[1])
from axropus_deploy_b200.ops._ext import cuda_ext
from axropus_deploy_b200.ops.gemm import error_flag
dev = torch.device("cuda", 0)
C = cuda_ext()
rows, K, N, W = 128, 256, 256, 2
staging = torch.zeros(W * rows, K, dtype=torch.bfloat16, device=dev)
staging[:rows].normal_()
w = torch.randn(N, K, device=dev).to(torch.bfloat16)
out = torch.empty(W * rows, N, dtype=torch.bfloat16, device=dev)
flags = torch.zeros(W * rows // 128 * 8, dtype=torch.int32, device=dev)
ready = torch.zeros(W, dtype=torch.int32, device=dev)
silent_peer_ready = torch.zeros(W, dtype=torch.int32, device=dev)   # the peer's flags: never raised for us
silent_peer_rows = torch.zeros(rows, K, dtype=torch.bfloat16, device=dev)
peer_a = torch.tensor([staging.data_ptr(), silent_peer_rows.data_ptr()], dtype=torch.int64, device=dev)
peer_ready = torch.tensor([ready.data_ptr(), silent_peer_ready.data_ptr()], dtype=torch.int64, device=dev)
err = error_flag(dev)
err.zero_()
t0 = time.perf_counter()
C.gemm_tp(staging[:rows], w, out, 1, 0, W, rows, 1, peer_a, staging, flags, ready, peer_ready,
          None, None, None, None, err)
torch.cuda.synchronize()
dt = time.perf_counter() - t0
code = int(err[0].item())
# whichever bounded wait runs out first records its code: the peer-flag waits (5, 7) or the
# waits of the roles that depend on them (stage 2, accumulator 3)
assert code in (2, 3, 5, 7), f"expected a wait code, got {code}"
assert dt < 10.0, f"the kernel took {dt:.1f} s to give up"

from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams
from axropus_deploy_b200.models.config import get_config
from axropus_deploy_b200.models.llama import LlamaModel
model = LlamaModel(get_config("tiny128"), dev, seed=0)
eng = LLMEngine(model, EngineConfig(num_blocks=64, max_model_len=512, max_batch=2))
eng.add_request(list(range(40)), SamplingParams(max_tokens=2))
try:
    eng.step()
except RuntimeError as e:
    assert "gave up waiting" in str(e), e
else:
    raise AssertionError("the engine used a step after a kernel gave up waiting")
err.zero_()                       # cleared: the context is still usable
while eng.has_unfinished():
    eng.step()
print("FAILURE_DETECTED", code, round(dt, 3))
"""


def test_bounded_peer_wait_runs_out_and_engine_refuses_step():
    env = dict(os.environ, AXR_PEER_WAIT_MS="50")
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "FAILURE_DETECTED" in r.stdout

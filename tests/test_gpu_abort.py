"""The tensor-core GEMM's bounded waits giving up, for real: with the poll limit set to
zero (ekernel_set_wait_limit), the first pipeline wait that is not already met raises the
CTA's abort flag; every role leaves its loop, the producer drains its copies, the MMA
issuer drains its MMAs, tensor memory is freed and the call returns ECPU_ERR_KERNEL with
the pipeline message in synchronous mode.  The next call, with the kernel's own limit,
gives the oracle's result: the context is intact and the stream-K arrival counters that
the aborted launch left behind were cleared.  Both schedules (split and stream-K) run.
No fault, trap or endless wait is involved: every wait is bounded and the timeout is the
kernel's own error path.  Runs in a child process (synchronous mode is read at load)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

_SCRIPT = r"""
import sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from oracle import kernels as ok
from pilm_b200 import bindings as abi, ckernel as ck
from tests._gpu import assert_bf16_close, bf16_from_bits, bits_of
abi.init()
lib = abi.lib()
rng = np.random.default_rng(3)
for (M, N, K) in [(96, 2048, 2048), (96, 19000, 512)]:  # split schedule, then stream-K (149 tiles)
    x = ok.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    qw, s = ok.quantize_i4_grouped(w, 128)
    ref = ok.linear_w4a16g_bf16(x, qw, s, 128)
    xd, qd, sd = bf16_from_bits(x), torch.from_numpy(qw).cuda(), torch.from_numpy(s).cuda()
    lib.ekernel_set_wait_limit(0)
    try:
        ck.linear_w4a16g128_bf16(xd, qd, sd)
        raise SystemExit(f"{N}x{K}: the pipeline did not give up")
    except RuntimeError as e:
        assert "rc=-4" in str(e) and "timed out" in str(e), e
    lib.ekernel_set_wait_limit(-1)
    for _ in range(2):
        y = ck.linear_w4a16g128_bf16(xd, qd, sd)
        torch.cuda.synchronize()
        assert_bf16_close(bits_of(y), ref, ulp_frac=0.99)
print("ABORT_PATH_OK")
"""


@pytest.mark.gpu
def test_gemm_wait_timeout_reports_error_and_next_call_is_exact():
    env = dict(os.environ, PILM_CUDA_SYNC="1", PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", _SCRIPT, str(ROOT)], capture_output=True, text=True, timeout=600,
                       env=env)
    assert r.returncode == 0 and "ABORT_PATH_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]

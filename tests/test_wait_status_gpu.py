"""The bounded wait of the shared-memory-staged softmax kernel reports its
give-up as a device status and returns, instead of hanging.

The wait (on a bulk copy of a row into shared memory) cannot run out with
valid arguments, so the test lowers its poll budget to 0 through
XN_STAGE_WAIT_POLLS (read once per process) in a child process: every stage
wait then gives up at once, on valid inputs. The kernel must still let its
copies in flight land (that drain keeps the full budget), write NaN to the
rows it had not finished, set XN_DEVERR_WAIT in the caller's error word and
return with the CUDA context usable. No GPU fault is involved: every copy
completes normally. In this process (default budget) the same call returns
correct values and a zero error word."""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_close, from_device, randn, rng, to_device, to_storage

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]

CHILD = r"""
import json, sys
sys.path[:0] = [sys.argv[1] + "/random-things_b200"]
import torch
import xn_fused as xn
dev = torch.device("cuda:0")
g = torch.Generator(device=dev).manual_seed(0)
x = torch.randn((64, 4096), device=dev, generator=g).to(torch.bfloat16)  # 512 vectors: the staged kernel
y = torch.zeros_like(x)
err = torch.zeros(1, dtype=torch.int32, device=dev)
xn.softmax_status_(y, x, err)
torch.cuda.synchronize()
res = {"err": int(err.item()), "all_nan": bool(torch.isnan(y.float()).all().item())}
# The context is still usable: a second call and an unrelated torch op both run.
err2 = torch.zeros(1, dtype=torch.int32, device=dev)
xn.softmax_status_(y, x, err2, scale=0.5)
res["err2"] = int(err2.item())
res["torch_ok"] = torch.ones(1000, device=dev).sum().item() == 1000.0
torch.cuda.synchronize()
print(json.dumps(res))
"""


def test_stage_wait_gives_up_with_status():
    env = dict(os.environ, XN_STAGE_WAIT_POLLS="0")
    out = subprocess.run([sys.executable, "-c", CHILD, str(REPO)], env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res["err"] == 2 and res["err2"] == 2, res  # XN_DEVERR_WAIT
    assert res["all_nan"], res
    assert res["torch_ok"], res


def test_stage_wait_status_zero_on_success(oracle, xn, cuda):
    r = rng(3)
    x = to_storage(randn(r, (64, 4096), 2.0), "bf16")
    X = to_device(x, "bf16", cuda)
    Y = torch.empty_like(X)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    xn.softmax_status_(Y, X, err)
    assert int(err.item()) == 0
    assert_close(from_device(Y, "bf16"), oracle.softmax(x, "bf16"), "bf16", "softmax_status bf16 64x4096")

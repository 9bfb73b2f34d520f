"""Failure detection on the GPU without a fault: every wait in the library's kernels is
bounded (1 s of GPU time).  The self-test kernel waits on a barrier that nothing completes,
gives up, and records ERR_TIMEOUT; the host reads it through b200lab_device_status, the flag
is cleared, and the context keeps working (the reference's CUDA_CHECK -> exit(1),
src/attn_sm75.cu:40-48, has no such path)."""
import time

import numpy as np
import pytest
import torch

import b200lab
import oracle
import workloads
from helpers import assert_close, to_np

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    assert b200lab.device_status() == b200lab.OK
    t0 = time.monotonic()
    b200lab.watchdog_selftest()
    assert b200lab.device_status() == b200lab.ERR_TIMEOUT
    waited = time.monotonic() - t0
    assert 0.5 < waited < 30.0, waited
    assert b200lab.device_status() == b200lab.OK  # read and cleared
    # the context is intact: a normal launch after the timeout is still correct
    Q, K, V = workloads.attn_inputs(1, 2, 2, 130, 128, torch.bfloat16, seed=3, device="cpu")
    dev = torch.device("cuda:0")
    O = b200lab.attn_fwd(Q.to(dev), K.to(dev), V.to(dev), causal=True)
    assert b200lab.device_status() == b200lab.OK
    assert_close(to_np(O), oracle.attn_fwd(to_np(Q), to_np(K), to_np(V), 1 / np.sqrt(128), True), "after timeout")

"""Failure detection on the GPU without a fault: the bounded-wait give-up path.

ALPACA_ATTN_FLAG_DEBUG_FORCE_TIMEOUT makes the tensor-core prefill kernel wait on an mbarrier that nothing
arrives at, with a ~2 ms limit. The kernel must record ALPACA_CUDA_ERR_DEVICE_TIMEOUT in the device error word,
drain its own copies, free TMEM and return, leaving the context usable: the next normal call is correct.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests._util import max_abs_check

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_forced_wait_timeout_reports_and_recovers(cuda_lib):
    from alpaca_b200 import (FLAG_DEBUG_FORCE_TIMEOUT, AlpacaCUDAError, Kernel, Status, attention_device,
                             device_status)
    T, H, kvh, d = 256, 9, 3, 64
    q = oracle.f16_round(oracle.splitmix_normal(1, (T, H, d)))
    k = oracle.f16_round(oracle.splitmix_normal(2, (T, kvh, d)))
    v = oracle.f16_round(oracle.splitmix_normal(3, (T, kvh, d)))
    dev = torch.device("cuda")
    qd, kd, vd = (torch.from_numpy(x).to(dev).half() for x in (q, k, v))
    out = torch.zeros((T, H, d), dtype=torch.float32, device=dev)
    device_status()  # clean slate

    attention_device(qd, kd, vd, out, kind=Kernel.PREFILL_TC, flags=FLAG_DEBUG_FORCE_TIMEOUT)
    with pytest.raises(AlpacaCUDAError) as e:
        device_status()
    assert e.value.status == Status.DEVICE_TIMEOUT
    device_status()  # the word was cleared by the previous read

    attention_device(qd, kd, vd, out, kind=Kernel.PREFILL_TC)
    device_status()
    max_abs_check(out.cpu().numpy(), oracle.attention(q, k, v, 0), 2e-3, "prefill after a forced timeout")


def test_timeout_reported_only_to_its_stream(cuda_lib):
    """Device errors belong to the stream of the call that raised them: with a forced bounded-wait timeout on one
    stream and a normal prefill on another (issued in between, both in flight together), only the first stream's
    status reports DEVICE_TIMEOUT; the second reports OK and its output matches the oracle."""
    from alpaca_b200 import (FLAG_DEBUG_FORCE_TIMEOUT, AlpacaCUDAError, Kernel, Status, attention_device,
                             device_status)
    T, H, kvh, d = 512, 9, 3, 64
    q = oracle.f16_round(oracle.splitmix_normal(11, (T, H, d)))
    k = oracle.f16_round(oracle.splitmix_normal(12, (T, kvh, d)))
    v = oracle.f16_round(oracle.splitmix_normal(13, (T, kvh, d)))
    dev = torch.device("cuda")
    qd, kd, vd = (torch.from_numpy(x).to(dev).half() for x in (q, k, v))
    out_bad = torch.zeros((T, H, d), dtype=torch.float32, device=dev)
    out_ok = torch.zeros((T, H, d), dtype=torch.float32, device=dev)
    s_bad, s_ok = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_bad.wait_stream(torch.cuda.current_stream())
    s_ok.wait_stream(torch.cuda.current_stream())
    device_status(s_bad)
    device_status(s_ok)
    attention_device(qd, kd, vd, out_bad, kind=Kernel.PREFILL_TC, flags=FLAG_DEBUG_FORCE_TIMEOUT, stream=s_bad)
    attention_device(qd, kd, vd, out_ok, kind=Kernel.PREFILL_TC, stream=s_ok)
    device_status(s_ok)  # synchronises s_ok only; the timeout on s_bad is not reported here
    with pytest.raises(AlpacaCUDAError) as e:
        device_status(s_bad)
    assert e.value.status == Status.DEVICE_TIMEOUT
    device_status(s_bad)  # cleared
    torch.cuda.synchronize()
    max_abs_check(out_ok.cpu().numpy(), oracle.attention(q, k, v, 0), 2e-3, "prefill on the other stream")

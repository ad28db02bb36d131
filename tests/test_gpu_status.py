"""Device-side wait budgets of the tensor-core decode, tested without a fault.

The tensor-core decode is a pipeline of warps that wait on one another
(query tables and page copies arriving in shared memory, stages released by
the consumers).  Every wait is bounded.  Here the budget is set to a few
nanoseconds, so the first wait that is not already satisfied gives up: the
kernel must stop, let the copies it issued land, report the timeout in the
caller's status word and in the device counters, and leave the context
usable, so that the next decode with the default budget matches the oracle.
"""

import numpy as np
import pytest
import torch

from gpu_cases import make_case, run_gpu, run_oracle, tag_map_for
from intent_attention import _native as N
from intent_attention import paged_decode

pytestmark = pytest.mark.gpu


def _decode(case, **kw):
    return paged_decode(case["q"], case["pool"], case["table"], case["counts"], case["tags"],
                        tag_map_for(case["formats"]), 0, out_dtype=torch.float32, kernel="tensor", **kw)


def test_tiny_wait_budget_reports_timeout_and_context_stays_usable():
    N.device_status(reset=True)
    case = make_case(901, B=8, Hq=32, Ht=8, D=128, W=256, NP=3000, counts="full", pad_frac=0.0)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _decode(case, status=status, wait_budget_ns=1)
    torch.cuda.synchronize()
    assert int(status.item()) & N.STATUS_DECODE_TIMEOUT
    counts = N.device_status(reset=True)
    assert counts["decode"] > 0
    assert N.device_status(reset=False) == {"decode": 0, "mla": 0, "prefill": 0}   # the reset cleared them

    # the default budget: no timeout, and the result matches the oracle
    status.zero_()
    out = _decode(case, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert N.device_status(reset=True) == {"decode": 0, "mla": 0, "prefill": 0}
    np.testing.assert_allclose(out.cpu().numpy(), run_oracle(case), atol=2e-3, rtol=1e-2)


def test_status_word_stays_clear_on_normal_decodes():
    case = make_case(903, B=2, Hq=8, Ht=2, D=128, W=64, NP=200)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for splits in (0, 1, 3):
        _decode(case, status=status, num_splits=splits)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    N.raise_on_timeouts()


def test_status_must_be_a_cuda_int_tensor():
    case = make_case(905, B=1, Hq=4, Ht=1, D=128, W=16, NP=40)
    with pytest.raises(ValueError, match="status"):
        _decode(case, status=torch.zeros(1, dtype=torch.float32, device="cuda"))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        _decode(case, status=torch.zeros(1, dtype=torch.int32))

"""The bounded device-side waits: a wait that runs out is reported, not hung on.

Every kernel of libq38 that waits (on an mbarrier phase) gives up after a limit, records
Q38_DEV_TIMEOUT in the context's status word and returns; q38_ctx_check_device reports
it as Q38_ERR_DEVICE_TIMEOUT.  q38_ctx_test_wait_timeout runs that same wait helper on a
phase that nothing completes, with a short host-set limit, so the path is exercised
without a fault: the context must stay usable afterwards.
"""
import numpy as np
import pytest
import torch

import oracle as O
from test_qmm_gpu import check_close, dev_bf16, dev_u32, host_bf16, make_weight

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_context_stays_usable(q38):
    q38.check_device()  # nothing pending
    q38.test_wait_timeout(2_000_000)  # about a millisecond at B200 clocks
    with pytest.raises(q38.Q38Error) as e:
        q38.check_device()
    assert e.value.status == 5
    q38.check_device()  # the word was cleared
    # the context still runs products correctly
    c, s, b = make_weight(1700, 256, 1024, 4)
    x = O.normal_bf16(1701, (2, 1024))
    y = q38.quantized_matmul(dev_bf16(x), dev_u32(c), dev_bf16(s), dev_bf16(b), True, 64, 4)
    torch.cuda.synchronize()
    check_close(host_bf16(y), O.qmm(x, c, s, b, 64, 4, f32=True))
    q38.check_device()


def test_wait_limit_is_validated(q38):
    with pytest.raises(q38.Q38ArgumentError):
        q38.test_wait_timeout(-1)

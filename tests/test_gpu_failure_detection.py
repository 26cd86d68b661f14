"""Failure detection on the GPU without a fault: a kernel whose bounded wait runs out returns and
reports a status code, and the device stays usable.

gtb_selftest_wait_timeout launches a one-warp kernel that waits on an mbarrier nothing ever
arrives at, through the same bounded wait (sm100::mbar_wait) every kernel of the library uses,
with a short limit. The wait gives up, the kernel records status 90 and returns; gtb_device_status
reports the code once and clears it, and the next attention call runs normally."""

from __future__ import annotations

import pytest

from tests._util import assert_close, seeded, to_dev
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_an_expired_wait_is_reported_and_the_device_stays_usable():
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    assert _C.device_status() == 0
    stream = torch.cuda.current_stream().cuda_stream
    _C.check_rc(_C.lib.gtb_selftest_wait_timeout(200_000, stream), "selftest")  # ~0.1 ms of waiting
    assert _C.device_status() == 90          # the kernel returned and left its code
    assert _C.device_status() == 0           # read once, then cleared
    # the next normal call runs and is right
    O.manual_seed(3)
    q, k, v = seeded((1, 2, 130, 64), "bf16", 0.5), seeded((1, 2, 130, 64), "bf16", 0.5), seeded((1, 2, 130, 64), "bf16", 0.5)
    out, _ = Fn.sdpa_forward(to_dev(q, "bf16"), to_dev(k, "bf16"), to_dev(v, "bf16"), None, 0.125, True)
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    assert_close(out, O.sdpa_fwd(q, k, v, scale=0.125, is_causal=True), 2e-2, 1e-2, "forward after the timeout")


def test_selftest_rejects_limits_outside_the_bounded_range():
    from gguf_train_b200 import _C

    assert _C.lib.gtb_selftest_wait_timeout(10, None) != 0
    assert b"limit_cycles" in _C.lib.gtb_last_error()
    assert _C.lib.gtb_selftest_wait_timeout(1 << 40, None) != 0

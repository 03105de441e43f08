"""Device failure detection without a GPU fault: a test hook makes the producer
skip the Q loads, so the MMA warp's bounded wait expires; the kernel records a
watchdog status, every CTA drains its copies and returns, and the context
stays usable for the next call."""
import pytest
import torch

from oracle import attention_oracle as orc
from tests import abi_ctypes as abi

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d", [128, 64])  # d=64: dual-tile items (named barriers in the merge)
def test_wait_timeout_reports_status_and_context_survives(sm100, d):
    lib = abi.load()
    cfg = orc.AttnConfig("t", 1, 2, 2, 512, d, False)
    q, k, v = (t.cuda() for t in orc.make_inputs(cfg, seed=3))
    o = torch.empty_like(q)
    lib.fa_device_status(1)             # clear any earlier record
    assert lib.fa_device_status(0) == 0
    lib.fa_set_watchdog_ns(20_000_000)  # 20 ms per wait
    lib.fa_set_debug_flags(1)           # FA_DEBUG_SKIP_Q_LOAD
    try:
        assert abi.fa_fwd(q, k, v, o, None, causal=False) == 0
        torch.cuda.synchronize()        # the kernel returns: no hang, no fault
    finally:
        lib.fa_set_debug_flags(0)
        lib.fa_set_watchdog_ns(1_000_000_000)
    status = lib.fa_device_status(1)
    assert status >= 100, status        # FA_ERR_TIMEOUT_BASE + wait site
    assert lib.fa_device_status(0) == 0  # reset worked
    # the same context computes correctly afterwards
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device="cuda")
    assert abi.fa_fwd(q, k, v, o, lse, causal=False) == 0
    torch.cuda.synchronize()
    ref, ref_l = orc.attention_fp32(q.cpu(), k.cpu(), v.cpu(), causal=False)
    assert orc.check(o.cpu(), ref)["ok"]
    assert lib.fa_device_status(0) == 0

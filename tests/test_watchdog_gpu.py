"""Device watchdog: a bounded mbarrier wait that nothing completes gives up
after its limit, records its site code and returns; the context stays usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_watchdog_probe_records_and_recovers(felix):
    assert felix.watchdog_status(clear=True) == 0
    felix.watchdog_probe(2000)  # 2 ms limit
    code = felix.watchdog_status(clear=True)
    assert code == 6  # kWdProbe
    assert felix.watchdog_status(clear=True) == 0
    # the context is still healthy: run a GEMM
    A = torch.randn(64, 64, device="cuda")
    C = torch.empty(64, 64, device="cuda")
    felix.sgemm(A, A, C)
    torch.cuda.synchronize()
    torch.testing.assert_close(C, A @ A, rtol=1e-4, atol=1e-4)

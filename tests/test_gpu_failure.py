"""The device-side failure path, exercised without a fault.

Every tcgen05 kernel bounds its mbarrier waits with a time limit; when one
expires the kernel writes an error code to the device status word, stops and
returns, and the host sees C3B_E_DEVICE from c3b_plan_sync (the
PlannedGraphExecutor.run_planned failure contract: an exception instead of a
hang, c35/executor.py:305-310).  Here the limit is shortened to 1 ms and a probe
kernel waits on a barrier that nothing arms, so the wait runs out on purpose;
the context must stay usable afterwards.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _plan_with_probe(L, code):
    from hackathon_b200.kernels import Launch
    from hackathon_b200.runtime import NativePlan
    p = NativePlan(256, n_streams=1)
    p.kernel(0, Launch(L.K_WAIT_PROBE, [], [], L.WaitProbeParams(code)), "wait_probe")
    p.finalize(use_graph=False)
    return p


def test_expired_wait_reports_device_status_and_context_survives():
    import torch
    from hackathon_b200 import _lib as L
    assert L.device_status() == 0
    L.set_wait_limit_ns(1_000_000)  # 1 ms
    try:
        plan = _plan_with_probe(L, 41)
        with pytest.raises(RuntimeError, match="device status 41"):
            plan.run()  # c3b_plan_launch + c3b_plan_sync -> C3B_E_DEVICE
        # c3b_plan_sync read and cleared the word
        assert L.device_status() == 0
        # a direct launch: the status word carries the probe's code
        L.launch(L.K_WAIT_PROBE, [], [], L.WaitProbeParams(7))
        assert L.device_status() == 7
        plan.close()
    finally:
        L.set_wait_limit_ns(2_000_000_000)
    # the context is intact: a tcgen05 GEMM right after gives exact results
    rng = np.random.default_rng(3)
    a = rng.integers(-4, 5, (256, 128)).astype(np.float32)
    b = rng.integers(-4, 5, (64, 128)).astype(np.float32)
    ta = torch.from_numpy(a).cuda().to(torch.bfloat16)
    tb = torch.from_numpy(b).cuda().to(torch.bfloat16)
    out = torch.empty((256, 64), dtype=torch.float32, device="cuda")
    g = L.GemmTcParams()
    g.M, g.N, g.K, g.bias_mode, g.act, g.has_residual, g.block_n = 256, 64, 128, L.BIAS_NONE, 0, 0, 0
    L.launch(L.K_GEMM_TC, [L.make_tensor(ta.data_ptr(), L.BF16, (256, 128)),
                           L.make_tensor(tb.data_ptr(), L.BF16, (64, 128))],
             [L.make_tensor(out.data_ptr(), L.F32, (256, 64))], g, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), a @ b.T)  # small integers: exact in fp32
    assert L.device_status() == 0


def test_wait_limit_rejects_out_of_range_values():
    from hackathon_b200 import _lib as L
    with pytest.raises(RuntimeError, match="wait limit"):
        L.set_wait_limit_ns(10)

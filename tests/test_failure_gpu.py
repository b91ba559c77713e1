"""Device-side failure detection, exercised without a GPU fault: a bounded
wait that nothing completes gives up after its limit, the kernel records it
in the device status word and returns, and the context stays usable."""
import time

import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(cuda):
    L = mb.lib()
    L.mamba_device_status(1)  # start clean
    t0 = time.perf_counter()
    assert L.mamba_selftest_bounded_wait(20000, None) == 0, mb.last_error()  # 20 ms limit
    took = time.perf_counter() - t0
    assert 0.015 < took < 5.0
    status = L.mamba_device_status(0)
    assert status & 8
    L.mamba_device_status(1)
    assert L.mamba_device_status(0) == 0
    # the context is intact: a scan afterwards is correct and clean
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 64, 128)).astype(np.float32)
    dr = rng.normal(-4.6, 0.5, (2, 64, 128)).astype(np.float32)
    B = rng.standard_normal((2, 64, 16)).astype(np.float32)
    C = rng.standard_normal((2, 64, 16)).astype(np.float32)
    A = np.tile(-np.arange(1, 17, dtype=np.float32), (128, 1))
    Dk = np.ones(128, np.float32)
    y_ref, _ = oracle.scan(x, dr, B, C, A, Dk)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    y = mb.selective_scan(t(x), t(dr), t(A), t(B), t(C), D=t(Dk))
    torch.cuda.synchronize()
    assert oracle.normwise_rel_err(y.cpu().numpy(), y_ref) < 1e-5
    assert L.mamba_device_status(0) == 0


def test_selftest_rejects_bad_limits(cuda):
    L = mb.lib()
    assert L.mamba_selftest_bounded_wait(0, None) == -1
    assert L.mamba_selftest_bounded_wait(2000000, None) == -1
    assert "limit" in mb.last_error()


def test_debug_mode_names_the_failing_operation(cuda, monkeypatch):
    """MAMBA_DEBUG=1 synchronises and checks the stream after every
    operation.  With a clean device the debug-mode forward equals the normal
    one; with a status flag left set (by the bounded-wait self-test, no
    fault) the first checked operation reports it, and the call fails naming
    rmsnorm of layer 0; once the flag is cleared the model works again."""
    rng = np.random.default_rng(3)
    cfg = mb.MambaConfig(64, 16, 4, 2, 2, mb.F16)
    layers = [mb.random_layer_weights(cfg, rng) for _ in range(2)]
    blob = mb.make_weight_blob(cfg, layers)
    h = rng.standard_normal((2, 40, 64)).astype(np.float32)
    plain = mb.Model(64, 16, 4, 2, 2, mb.F16)
    plain.load_weights(blob)
    ref = plain.forward(h)
    monkeypatch.setenv("MAMBA_DEBUG", "1")
    m = mb.Model(64, 16, 4, 2, 2, mb.F16)
    m.load_weights(blob)
    L = mb.lib()
    L.mamba_device_status(1)
    assert np.array_equal(m.forward(h), ref)
    st = m.create_state(2)
    st.step(h[:, 0])  # the decode step runs checked too (no graph in debug mode)
    assert L.mamba_selftest_bounded_wait(20000, None) == 0
    with pytest.raises(mb.MambaError, match="MAMBA_DEBUG: operation rmsnorm of layer 0"):
        m.forward(h)
    L.mamba_device_status(1)
    assert np.array_equal(m.forward(h), ref)

"""GPU parity of the model-level C API (mamba_forward / mamba_step) against the
CPU block reference (oracle.block_ref) on identical seeded weights and
inputs.  Tolerance: normwise 2e-3 for FP16 activations, 1e-4 for FP32."""
import ctypes

import numpy as np
import pytest
import torch

import mamba_b200 as mb
import oracle
from oracle import block_ref

pytestmark = pytest.mark.gpu


def build_model(rng, d_model, n_layer, dtype, d_state=16, d_conv=4, expand=2):
    m = mb.Model(d_model, d_state, d_conv, expand, n_layer, dtype)
    layers = [mb.random_layer_weights(m.cfg, rng) for _ in range(n_layer)]
    m.load_weights(mb.make_weight_blob(m.cfg, layers))
    return m, layers


def test_block_forward_workload(cuda):
    """One Mamba block at d_model=768, expand=2, d_state=16, dt_rank=48,
    batch=8, L=2048, FP16 activations, FP32 state and residual."""
    rng = np.random.default_rng(100)
    m, layers = build_model(rng, 768, 1, mb.F16)
    h = rng.standard_normal((8, 2048, 768)).astype(np.float32)
    out = m.forward(h)
    ref = block_ref.model_forward(h, layers, m.cfg, block_ref.F16)
    assert oracle.normwise_rel_err(out - h, ref - h) < 2e-3
    assert oracle.normwise_rel_err(out, ref) < 2e-3


@pytest.mark.parametrize("dtype,tol", [(mb.F16, 2e-3), (mb.F32, 1e-4)])
def test_multilayer_forward(cuda, dtype, tol):
    rng = np.random.default_rng(101)
    m, layers = build_model(rng, 96, 3, dtype, d_state=16, d_conv=4)
    h = rng.standard_normal((3, 77, 96)).astype(np.float32)
    out = m.forward(h)
    ref = block_ref.model_forward(h, layers, m.cfg, dtype)
    assert oracle.normwise_rel_err(out - h, ref - h) < tol


def test_odd_config_forward(cuda):
    """d_model not a multiple of 16 (dt_rank = ceil(d_model/16)), d_state 5,
    d_conv 3, expand 3."""
    rng = np.random.default_rng(102)
    m, layers = build_model(rng, 40, 2, mb.F16, d_state=5, d_conv=3, expand=3)
    h = rng.standard_normal((2, 45, 40)).astype(np.float32)
    out = m.forward(h)
    ref = block_ref.model_forward(h, layers, m.cfg, block_ref.F16)
    assert oracle.normwise_rel_err(out - h, ref - h) < 2e-3


def test_long_sequence_chunked_forward(cuda):
    """batch 1, L 4096: the scan splits time into chunks inside the model."""
    rng = np.random.default_rng(103)
    m, layers = build_model(rng, 64, 1, mb.F16)
    h = rng.standard_normal((1, 4096, 64)).astype(np.float32)
    out = m.forward(h)
    ref = block_ref.model_forward(h, layers, m.cfg, block_ref.F16)
    assert oracle.normwise_rel_err(out - h, ref - h) < 2e-3


@pytest.mark.parametrize("dtype,tol", [(mb.F16, 2e-3), (mb.F32, 1e-4)])
def test_step_matches_reference_and_forward(cuda, dtype, tol):
    """mamba_step over T tokens (state batch 4) equals the CPU decode
    reference, and equals mamba_forward on the same tokens."""
    rng = np.random.default_rng(104)
    m, layers = build_model(rng, 64, 2, dtype)
    bsz, T = 4, 24
    h = rng.standard_normal((bsz, T, 64)).astype(np.float32)
    st = m.create_state(bsz)
    ref_state = block_ref.new_state(m.cfg, bsz)
    outs = []
    for t in range(T):
        o = st.step(h[:, t])
        r = block_ref.model_step(h[:, t], layers, ref_state, m.cfg, dtype)
        assert oracle.normwise_rel_err(o - h[:, t], r - h[:, t]) < tol, t
        outs.append(o)
    fwd = m.forward(h)
    assert oracle.normwise_rel_err(np.stack(outs, 1) - h, fwd - h) < tol
    # reset gives back the first-token output
    st.reset()
    o0 = st.step(h[:, 0])
    assert np.allclose(o0, outs[0], rtol=1e-6, atol=1e-6)


def test_device_forward_equals_host_forward(cuda):
    rng = np.random.default_rng(105)
    m, _ = build_model(rng, 128, 2, mb.F16)
    h = rng.standard_normal((2, 300, 128)).astype(np.float32)
    out_host = m.forward(h)
    dh = torch.from_numpy(h).cuda()
    dout = torch.empty_like(dh)
    m.forward_device(dh.data_ptr(), dout.data_ptr(), 2, 300)
    m2 = torch.cuda.current_stream()
    torch.cuda.synchronize()
    assert np.array_equal(dout.cpu().numpy(), out_host)
    # in place
    m.forward_device(dh.data_ptr(), dh.data_ptr(), 2, 300)
    torch.cuda.synchronize()
    assert np.array_equal(dh.cpu().numpy(), out_host)
    del m2


def test_random_init_is_deterministic(cuda):
    a = mb.Model(64, 16, 4, 2, 2, mb.F16)
    b = mb.Model(64, 16, 4, 2, 2, mb.F16)
    a.init_random(7)
    b.init_random(7)
    h = np.random.default_rng(0).standard_normal((2, 50, 64)).astype(np.float32)
    ya, yb = a.forward(h), b.forward(h)
    assert np.array_equal(ya, yb)
    assert not np.array_equal(ya, h)


def test_load_weights_rejects_bad_blobs(cuda):
    rng = np.random.default_rng(106)
    m = mb.Model(32, 16, 4, 2, 1, mb.F16)
    blob = mb.make_weight_blob(m.cfg, [mb.random_layer_weights(m.cfg, rng)])
    L = mb.lib()
    bad_magic = b"XXXXXXXX" + blob[8:]
    assert L.mamba_load_weights(m.handle, bad_magic, len(bad_magic)) == -1
    assert "magic" in mb.last_error()
    assert L.mamba_load_weights(m.handle, blob[:-4], len(blob) - 4) == -1
    assert "size" in mb.last_error()
    other = mb.MambaConfig(32, 16, 4, 2, 2, mb.F16)
    wrong = mb.make_weight_blob(other, [mb.random_layer_weights(other, rng) for _ in range(2)])
    assert L.mamba_load_weights(m.handle, wrong, len(wrong)) == -1
    assert L.mamba_load_weights(m.handle, blob, 10) == -1
    assert L.mamba_load_weights(m.handle, blob, len(blob)) == 0


def test_zero_weight_model_is_identity(cuda):
    """Freshly created (zero) weights: every block adds zero to the residual."""
    m = mb.Model(64, 16, 4, 2, 2, mb.F16)
    h = np.random.default_rng(0).standard_normal((1, 20, 64)).astype(np.float32)
    assert np.array_equal(m.forward(h), h)


def test_state_handle_outlives_model(cuda):
    """As in the reference, destroying the model does not free its states."""
    m = mb.Model(32, 16, 4, 2, 1, mb.F16)
    st = m.create_state(2)
    c, s = st.buffers(0)
    assert c and s
    m.close()
    st.close()


def test_step_rejects_foreign_state(cuda):
    a = mb.Model(32, 16, 4, 2, 1, mb.F16)
    b = mb.Model(64, 16, 4, 2, 1, mb.F16)
    st = b.create_state(1)
    tok = np.zeros((1, 32), np.float32)
    out = np.zeros_like(tok)
    assert mb.lib().mamba_step(a.handle, st.handle, tok.ctypes.data, out.ctypes.data) == -1
    assert "state" in mb.last_error()


def test_graph_replayed_decode_equals_plain_launches(cuda, monkeypatch):
    """Decode steps replayed from the captured CUDA graph give the same bits as
    steps launched one kernel at a time (MAMBA_STEP_GRAPH=0)."""
    rng = np.random.default_rng(107)
    cfg = mb.MambaConfig(96, 16, 4, 2, 3, mb.F16)
    layers = [mb.random_layer_weights(cfg, rng) for _ in range(3)]
    blob = mb.make_weight_blob(cfg, layers)
    monkeypatch.setenv("MAMBA_STEP_GRAPH", "0")
    plain = mb.Model(96, 16, 4, 2, 3, mb.F16)
    monkeypatch.setenv("MAMBA_STEP_GRAPH", "1")
    graphed = mb.Model(96, 16, 4, 2, 3, mb.F16)
    plain.load_weights(blob)
    graphed.load_weights(blob)
    sp, sg = plain.create_state(5), graphed.create_state(5)
    toks = rng.standard_normal((12, 5, 96)).astype(np.float32)
    for t in range(12):
        assert np.array_equal(sp.step(toks[t]), sg.step(toks[t])), t
    # device API with fixed buffers reuses the graph; a new buffer re-captures
    dev_in = torch.from_numpy(toks[0]).cuda()
    out_a, out_b = torch.empty_like(dev_in), torch.empty_like(dev_in)
    sg.step_device(dev_in.data_ptr(), out_a.data_ptr())
    sp.step_device(dev_in.data_ptr(), out_b.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)


def test_decode_with_tcgen05_projections_matches_cublas(cuda, monkeypatch):
    """MAMBA_TC_LINEAR=1 runs the decode projections (batch rows <= 512) on
    the library's tcgen05 linear kernel; the steps agree with the cuBLAS
    model within the FP16 tolerance."""
    rng = np.random.default_rng(108)
    cfg = mb.MambaConfig(256, 16, 4, 2, 2, mb.F16)
    layers = [mb.random_layer_weights(cfg, rng) for _ in range(2)]
    blob = mb.make_weight_blob(cfg, layers)
    monkeypatch.setenv("MAMBA_TC_LINEAR", "0")
    ref = mb.Model(256, 16, 4, 2, 2, mb.F16)
    monkeypatch.setenv("MAMBA_TC_LINEAR", "1")
    tc = mb.Model(256, 16, 4, 2, 2, mb.F16)
    ref.load_weights(blob)
    tc.load_weights(blob)
    sr, st = ref.create_state(40), tc.create_state(40)
    toks = rng.standard_normal((6, 40, 256)).astype(np.float32)
    for t in range(6):
        a, b = sr.step(toks[t]), st.step(toks[t])
        assert oracle.normwise_rel_err(b - toks[t], a - toks[t]) < 2e-3, t
    h = rng.standard_normal((2, 50, 256)).astype(np.float32)
    assert oracle.normwise_rel_err(tc.forward(h) - h, ref.forward(h) - h) < 2e-3
    assert mb.device_status() == 0


def test_chunked_host_forward_matches_device_forward(cuda, monkeypatch):
    """mamba_forward with the batch cut into row chunks (uploads, compute and
    downloads overlapped on separate streams) gives the rows of the
    single-call device forward (per-row results may take other kernel paths
    at the smaller batch, so within the FP16 tolerance)."""
    rng = np.random.default_rng(109)
    cfg = mb.MambaConfig(128, 16, 4, 2, 2, mb.F16)
    layers = [mb.random_layer_weights(cfg, rng) for _ in range(2)]
    blob = mb.make_weight_blob(cfg, layers)
    monkeypatch.setenv("MAMBA_HOST_CHUNKS", "3")
    m = mb.Model(128, 16, 4, 2, 2, mb.F16)
    m.load_weights(blob)
    h = rng.standard_normal((7, 200, 128)).astype(np.float32)
    out = m.forward(h)  # 3 chunks of 3, 3 and 1 rows
    dh = torch.from_numpy(h).cuda()
    dout = torch.empty_like(dh)
    m.forward_device(dh.data_ptr(), dout.data_ptr(), 7, 200)
    torch.cuda.synchronize()
    ref = dout.cpu().numpy()
    assert oracle.normwise_rel_err(out - h, ref - h) < 2e-3
    ref_cpu = block_ref.model_forward(h, layers, cfg, block_ref.F16)
    assert oracle.normwise_rel_err(out - h, ref_cpu - h) < 2e-3


def test_edge_layer_host_forward_is_bitwise_the_device_forward(cuda):
    """A 4-layer stack with a 84 MB host input: mamba_forward runs the first
    and last two layers per row chunk (5 rows, uploads and downloads
    overlapped) and the middle layers on the whole batch.  Every op is
    row-independent and the chunks take the same kernels as the whole batch
    here (over 512 rows per GEMM, at least one 128-channel scan CTA per SM),
    so the output equals the single-call device forward bit for bit."""
    m = mb.Model(2048, 16, 4, 2, 4, mb.F16)
    m.init_random(11)
    h = np.random.default_rng(110).standard_normal((40, 256, 2048)).astype(np.float32)
    out = m.forward(h)
    dh = torch.from_numpy(h).cuda()
    dout = torch.empty_like(dh)
    m.forward_device(dh.data_ptr(), dout.data_ptr(), 40, 256)
    torch.cuda.synchronize()
    assert mb.device_status() == 0
    assert np.array_equal(out, dout.cpu().numpy())
    assert not np.array_equal(out, h)


def test_save_weights_round_trip(cuda):
    """mamba_save_weights writes a blob that reproduces the model bit for bit
    when loaded into a second model; its projections are the FP16 values the
    GEMMs use, so saving a loaded blob of FP16-exact weights gives it back."""
    a = mb.Model(96, 16, 4, 2, 2, mb.F16)
    a.init_random(11)
    blob = a.save_weights()
    assert blob.nbytes == mb.lib().mamba_weights_blob_size(ctypes.byref(a.cfg))
    b = mb.Model(96, 16, 4, 2, 2, mb.F16)
    b.load_weights(blob)
    h = np.random.default_rng(1).standard_normal((2, 33, 96)).astype(np.float32)
    assert np.array_equal(a.forward(h), b.forward(h))
    assert np.array_equal(b.save_weights(), blob)
    layers = mb.weights_from_blob(a.cfg, blob)
    assert np.array_equal(layers[1]["A"], np.tile(-np.arange(1, 17, dtype=np.float32), (192, 1)))
    w = layers[0]["in_proj"]
    assert np.array_equal(w, w.astype(np.float16).astype(np.float32))
    assert mb.lib().mamba_save_weights(a.handle, blob.ctypes.data, blob.nbytes - 4) == -1
    assert "size" in mb.last_error()


def test_fused_conv_forward_equals_unfused(cuda, monkeypatch):
    """The forward with in_proj and the causal conv fused in one kernel
    (MAMBA_CONV_FUSE=1) gives the same bits as the forward with them
    separate (the default)."""
    rng = np.random.default_rng(110)
    cfg = mb.MambaConfig(128, 16, 4, 2, 2, mb.F16)
    layers = [mb.random_layer_weights(cfg, rng) for _ in range(2)]
    blob = mb.make_weight_blob(cfg, layers)
    monkeypatch.setenv("MAMBA_CONV_FUSE", "0")
    sep = mb.Model(128, 16, 4, 2, 2, mb.F16)
    monkeypatch.setenv("MAMBA_CONV_FUSE", "1")
    fused = mb.Model(128, 16, 4, 2, 2, mb.F16)
    sep.load_weights(blob)
    fused.load_weights(blob)
    h = rng.standard_normal((3, 333, 128)).astype(np.float32)
    a, b = sep.forward(h), fused.forward(h)
    assert np.array_equal(a, b)
    ref = block_ref.model_forward(h, layers, cfg, block_ref.F16)
    assert oracle.normwise_rel_err(b - h, ref - h) < 2e-3

"""CPU tests of the oracle: pinned to the reference's own outputs.

The golden vectors in tests/golden/ were written by the reference's
selective_scan_cpu (tests/golden/make_golden.py); the restatement must
reproduce them bit for bit.  The reference test suite's checks
(Tests/test_numerical.cpp:16-61, Tests/test_selective_scan.cpp:26-35) are
re-run as known-answer tests.
"""
import glob
import os

import numpy as np
import pytest

import oracle
from oracle import block_ref

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load_golden(path):
    with open(path, "rb") as f:
        raw = f.read()
    assert raw[:8] == b"MGOLD01\0"
    L, D, N, _ = np.frombuffer(raw[8:24], np.int32)
    arr = np.frombuffer(raw[24:], np.float32)
    sizes = [L * D, L * D, L * N, L * N, D * N, D, L * D, D * N]
    shapes = [(L, D), (L, D), (L, N), (L, N), (D, N), (D,), (L, D), (D, N)]
    out, off = [], 0
    for s, sh in zip(sizes, shapes):
        out.append(arr[off:off + s].reshape(sh).copy())
        off += s
    assert off == arr.size
    names = ["x", "delta", "B", "C", "A", "Dskip", "y", "state"]
    return dict(zip(names, out))


CASES = sorted(glob.glob(os.path.join(GOLDEN, "*.bin")))


def test_golden_cases_present():
    names = {os.path.basename(c)[:-4] for c in CASES}
    assert {"ref_test_selective_scan", "ref_test_impulse", "ref_test_zero_input",
            "ref_bench_dist", "scan_workload_slice", "edge_branches"} <= names


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[:-4] for c in CASES])
def test_restatement_matches_reference_golden_bitwise(path):
    g = load_golden(path)
    y, h = oracle.selective_scan(g["x"], g["delta"], g["B"], g["C"], g["A"], g["Dskip"])
    assert np.array_equal(y, g["y"])
    assert np.array_equal(h, g["state"])


@pytest.mark.parametrize("path", CASES, ids=[os.path.basename(c)[:-4] for c in CASES])
def test_general_scan_matches_golden_bitwise(path):
    """The batched/strided restatement evaluates the same operations per
    element, so it must also be bit-identical (here in [batch, D, L] layout)."""
    g = load_golden(path)
    L, D = g["x"].shape
    xt = np.ascontiguousarray(g["x"].T)[None]          # [1, D, L]
    dt = np.ascontiguousarray(g["delta"].T)[None]
    Bt = np.ascontiguousarray(g["B"].T)[None]          # [1, N, L]
    Ct = np.ascontiguousarray(g["C"].T)[None]
    y, h = oracle.scan(xt.transpose(0, 2, 1), dt.transpose(0, 2, 1), Bt.transpose(0, 2, 1),
                       Ct.transpose(0, 2, 1), g["A"], g["Dskip"], nthreads=2)
    assert np.array_equal(y[0], g["y"])
    assert np.array_equal(h[0], g["state"])


def test_reference_library_matches_golden():
    if oracle.ref_lib() is None:
        pytest.skip("reference oracle library not built (no reference checkout)")
    for path in CASES:
        g = load_golden(path)
        y, h = oracle.selective_scan(g["x"], g["delta"], g["B"], g["C"], g["A"], g["Dskip"],
                                     use_reference=True)
        assert np.array_equal(y, g["y"]) and np.array_equal(h, g["state"]), path


def test_kat_last_y():
    """Tests/test_selective_scan.cpp prints last_y = -0.453731 for seed 42."""
    g = load_golden(os.path.join(GOLDEN, "ref_test_selective_scan.bin"))
    y, _ = oracle.selective_scan(g["x"], g["delta"], g["B"], g["C"], g["A"], g["Dskip"])
    assert np.all(np.isfinite(y))
    assert "%.6f" % y[-1, -1] == "-0.453731"


def test_kat_zero_input():
    """Tests/test_numerical.cpp:38-51: zero input gives exactly zero output."""
    g = load_golden(os.path.join(GOLDEN, "ref_test_zero_input.bin"))
    y, _ = oracle.selective_scan(g["x"], g["delta"], g["B"], g["C"], g["A"], g["Dskip"])
    assert np.count_nonzero(np.abs(y) > 1e-7) == 0


def test_kat_impulse_decay():
    """Tests/test_numerical.cpp:16-36: |y| on channel 0 never grows."""
    g = load_golden(os.path.join(GOLDEN, "ref_test_impulse.bin"))
    y, _ = oracle.selective_scan(g["x"], g["delta"], g["B"], g["C"], g["A"], g["Dskip"])
    assert y[0, 0] != 0
    a = np.abs(y[:, 0])
    assert np.all(a[1:] <= a[:-1] + 1e-6)


def test_kat_associativity():
    """Tests/test_numerical.cpp:53-61."""
    a, b, c = (0.9, 0.1), (0.8, 0.2), (0.7, 0.3)
    left = oracle.affine_compose(a, oracle.affine_compose(b, c))
    right = oracle.affine_compose(oracle.affine_compose(a, b), c)
    assert abs(left[0] - right[0]) <= 1e-5 + 1e-4 * abs(right[0])
    assert abs(left[1] - right[1]) <= 1e-5 + 1e-4 * abs(right[1])


def _rand_scan_inputs(rng, bsz, L, D, N):
    x = rng.standard_normal((bsz, L, D)).astype(np.float32)
    dr = rng.normal(-4.6, 0.5, (bsz, L, D)).astype(np.float32)
    B = rng.standard_normal((bsz, L, N)).astype(np.float32)
    C = rng.standard_normal((bsz, L, N)).astype(np.float32)
    A = np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))
    Dk = np.ones(D, np.float32)
    return x, dr, B, C, A, Dk


def test_chunk_summaries_compose_to_full_scan():
    """Splitting time into chunks, composing (P, H) summaries and rescanning
    each chunk from its entering state reproduces the single sequential scan
    (the carry algebra used across chunks and across GPUs)."""
    rng = np.random.default_rng(0)
    bsz, L, D, N = 2, 97, 24, 16
    x, dr, B, C, A, Dk = _rand_scan_inputs(rng, bsz, L, D, N)
    bias = rng.normal(0, 0.3, D).astype(np.float32)
    z = rng.standard_normal((bsz, L, D)).astype(np.float32)
    h0 = rng.standard_normal((bsz, D, N)).astype(np.float32) * 0.1
    y_full, h_full = oracle.scan(x, dr, B, C, A, Dk, z=z, dt_bias=bias, h0=h0)
    bounds = [0, 13, 40, 41, 97]
    Ps, Hs = [], []
    for t0, t1 in zip(bounds[:-1], bounds[1:]):
        P, H = oracle.scan_chunk_summary(x, dr, B, A, dt_bias=bias, t0=t0, t1=t1)
        Ps.append(P.reshape(-1))
        Hs.append(H.reshape(-1))
    h_in, h_fin = oracle.scan_chunk_combine(np.stack(Ps), np.stack(Hs), h0=h0)
    assert oracle.normwise_rel_err(h_fin.reshape(bsz, D, N), h_full) < 1e-5
    ys = []
    for g, (t0, t1) in enumerate(zip(bounds[:-1], bounds[1:])):
        sl = slice(t0, t1)
        y, h = oracle.scan(x[:, sl], dr[:, sl], B[:, sl], C[:, sl], A, Dk, z=z[:, sl],
                           dt_bias=bias, h0=h_in[g].reshape(bsz, D, N))
        ys.append(y)
    assert oracle.normwise_rel_err(np.concatenate(ys, axis=1), y_full) < 1e-5
    assert oracle.normwise_rel_err(h, h_full) < 1e-5


def test_gate_restatement():
    rng = np.random.default_rng(1)
    x, dr, B, C, A, Dk = _rand_scan_inputs(rng, 1, 33, 8, 4)
    z = rng.standard_normal((1, 33, 8)).astype(np.float32)
    y0, _ = oracle.scan(x, dr, B, C, A, Dk)
    y1, _ = oracle.scan(x, dr, B, C, A, Dk, z=z)
    silu = z / (np.float32(1) + np.exp(-z))
    np.testing.assert_allclose(y1, y0 * silu, rtol=1e-6, atol=1e-7)


def test_ssm_step_equals_scan_bitwise():
    """T single-token updates (state_update.metal semantics with softplus
    always applied) reproduce the sequential scan exactly."""
    rng = np.random.default_rng(2)
    bsz, L, D, N = 3, 20, 16, 16
    x, dr, B, C, A, Dk = _rand_scan_inputs(rng, bsz, L, D, N)
    z = rng.standard_normal((bsz, L, D)).astype(np.float32)
    bias = rng.normal(0, 0.3, D).astype(np.float32)
    y_scan, h_scan = oracle.scan(x, dr, B, C, A, Dk, z=z, dt_bias=bias)
    st = np.zeros((bsz, D, N), np.float32)
    ys = [oracle.ssm_step(x[:, t], dr[:, t], B[:, t], C[:, t], A, Dk, st, z=z[:, t], dt_bias=bias)
          for t in range(L)]
    assert np.array_equal(np.stack(ys, 1), y_scan)
    assert np.array_equal(st, h_scan)


def test_conv_step_equals_full_conv():
    rng = np.random.default_rng(3)
    bsz, L, D, K = 2, 11, 10, 4
    x = rng.standard_normal((bsz, L, D)).astype(np.float32)
    w = rng.uniform(-0.5, 0.5, (D, K)).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, D).astype(np.float32)
    y_full = oracle.causal_conv1d(x, w, b, silu=True)
    st = np.zeros((bsz, D, K - 1), np.float32)
    ys = [oracle.causal_conv1d_step(x[:, t], w, b, st, silu=True) for t in range(L)]
    assert np.array_equal(np.stack(ys, 1), y_full)
    # state holds the last K-1 inputs, oldest first
    assert np.array_equal(st, x[:, L - K + 1:].transpose(0, 2, 1))


def test_block_step_matches_block_forward():
    """Decode over T tokens from zero state equals the full-sequence block
    graph on the same tokens (CPU reference, both activation types)."""
    from mamba_b200 import MambaConfig, random_layer_weights
    for act in (block_ref.F32, block_ref.F16):
        cfg = MambaConfig(32, 16, 4, 2, 2, act)
        rng = np.random.default_rng(4)
        layers = [random_layer_weights(cfg, rng) for _ in range(cfg.n_layer)]
        bsz, L = 2, 9
        h = rng.standard_normal((bsz, L, cfg.d_model)).astype(np.float32)
        y_fwd = block_ref.model_forward(h, layers, cfg, act)
        state = block_ref.new_state(cfg, bsz)
        y_step = np.stack([block_ref.model_step(h[:, t], layers, state, cfg, act)
                           for t in range(L)], 1)
        tol = 1e-5 if act == block_ref.F32 else 2e-3
        assert oracle.normwise_rel_err(y_step, y_fwd) < tol


def test_layer_major_decode_equals_token_steps():
    """block_ref.model_decode (projections batched over the tokens of a layer)
    gives the outputs and the final states of model_step called token by
    token; only the BLAS summation order of the batched products differs."""
    from mamba_b200 import MambaConfig, random_layer_weights
    cfg = MambaConfig(48, 16, 4, 2, 3, block_ref.F16)
    rng = np.random.default_rng(9)
    layers = [random_layer_weights(cfg, rng) for _ in range(cfg.n_layer)]
    bsz, T = 3, 7
    h = rng.standard_normal((bsz, T, cfg.d_model)).astype(np.float32)
    s_tok = block_ref.new_state(cfg, bsz)
    y_tok = np.stack([block_ref.model_step(h[:, t], layers, s_tok, cfg, block_ref.F16) for t in range(T)], 1)
    s_lay = block_ref.new_state(cfg, bsz)
    y_lay = block_ref.model_decode(h, layers, cfg, block_ref.F16, state=s_lay)
    assert oracle.normwise_rel_err(y_lay - h, y_tok - h) < 1e-4
    for a, b in zip(s_lay[1], s_tok[1]):
        assert oracle.normwise_rel_err(a, b) < 1e-4


def test_weight_blob_round_trip():
    """weights_from_blob reads back exactly what make_weight_blob wrote (views
    into the blob, layer by layer, in the documented tensor order)."""
    import mamba_b200 as mb
    cfg = mb.MambaConfig(40, 5, 3, 3, 2, mb.F16)
    rng = np.random.default_rng(10)
    layers = [mb.random_layer_weights(cfg, rng) for _ in range(2)]
    blob = mb.make_weight_blob(cfg, layers)
    back = mb.weights_from_blob(cfg, blob)
    for a, b in zip(layers, back):
        assert set(a) == set(b)
        for k in a:
            assert np.array_equal(a[k], b[k]), k
    with pytest.raises(ValueError):
        mb.weights_from_blob(mb.MambaConfig(40, 5, 3, 3, 3, mb.F16), blob)


def _propagate_loop(carries):
    """Pure-Python restatement of propagate_tile_carries_f32
    (prefix_scan.metal:19-40) with the documented [tiles, width, 2] layout:
    each tile's pair is replaced by the composition of the tiles before it."""
    c = np.array(carries, np.float32, copy=True)
    nt, width = c.shape[:2]
    total = np.empty((width, 2), np.float32)
    for p in range(width):
        acc = (np.float32(1), np.float32(0))
        for t in range(nt):
            a, b = c[t, p]
            c[t, p] = acc
            acc = (np.float32(a * acc[0]), np.float32(np.float32(a * acc[1]) + b))
        total[p] = acc
    return c, total


def test_tile_carries_restatement():
    rng = np.random.default_rng(5)
    for nt, width in [(1, 3), (7, 5), (33, 17), (0, 4)]:
        car = np.stack([rng.uniform(0.5, 1.0, (nt, width)), rng.standard_normal((nt, width))], -1)
        car = car.astype(np.float32)
        ex, tot = oracle.propagate_tile_carries(car)
        ex_loop, tot_loop = _propagate_loop(car)
        assert np.array_equal(ex, ex_loop) and np.array_equal(tot, tot_loop)
        if nt:
            assert np.array_equal(ex[0], np.tile(np.float32([1, 0]), (width, 1)))
        else:
            assert np.array_equal(tot, np.tile(np.float32([1, 0]), (width, 1)))


def test_tile_carries_of_chunk_summaries_give_final_state():
    """Chunk summaries (P, H) of a scan, laid out as [tiles, B*D*N, 2] pairs
    and propagated, give every chunk's entering state (from zero) and, as the
    total, the scan's final state."""
    rng = np.random.default_rng(6)
    bsz, L, D, N = 2, 64, 8, 16
    x, dr, B, C, A, Dk = _rand_scan_inputs(rng, bsz, L, D, N)
    _, h_full = oracle.scan(x, dr, B, C, A, Dk)
    bounds = [0, 16, 32, 48, 64]
    pairs = []
    for t0, t1 in zip(bounds[:-1], bounds[1:]):
        P, H = oracle.scan_chunk_summary(x, dr, B, A, t0=t0, t1=t1)
        pairs.append(np.stack([P.reshape(-1), H.reshape(-1)], -1))
    ex, tot = oracle.propagate_tile_carries(np.stack(pairs))
    assert oracle.normwise_rel_err(tot[:, 1].reshape(bsz, D, N), h_full) < 1e-5
    _, h_mid = oracle.scan(x[:, :32], dr[:, :32], B[:, :32], C[:, :32], A, Dk)
    assert oracle.normwise_rel_err(ex[2, :, 1].reshape(bsz, D, N), h_mid) < 1e-5


def test_gated_silu_mul_restatement():
    rng = np.random.default_rng(7)
    g = (rng.standard_normal(1001) * 4).astype(np.float32)
    u = rng.standard_normal(1001).astype(np.float32)
    want = g / (np.float32(1) + np.exp(-g)) * u
    np.testing.assert_allclose(oracle.gated_silu_mul(g, u), want, rtol=1e-6, atol=1e-7)

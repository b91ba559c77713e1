"""bench.py -- selective-scan HBM GB/s and Mamba block-forward tokens/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stack|scan]

Workloads (synthetic inputs, random-init weights; no datasets involved):
  stack (default)  48-layer Mamba stack forward, d_model 2048, expand 2
                   (d_inner 4096), d_state 16, d_conv 4, dt_rank 128,
                   batch 64, L 4096, FP16 activations/weights, FP32 state and
                   residual.  The batch is split across the N ranks (no
                   collective); value = tokens/s of the whole job.  The scan
                   kernel's HBM GB/s is measured live with CUDA events over
                   the timed region and reported in `roofline`.
  block            one Mamba block forward, d_model 768, d_inner 1536, batch 8,
                   L 2048, FP16; value = tokens/s (batch-sharded at N > 1).
  decode           incremental decode through mamba_step on a 64-layer stack,
                   d_model 2560, d_inner 5120, dt_rank 160, batch 256, 1024
                   sequential single-token steps from zero state (CUDA-graph
                   replayed); value = tokens/s, plus per-step latency.
  scan             standalone long selective scan, batch 1, d_inner 2048,
                   d_state 16, L 131072; x, B, C, z FP16, delta FP32; the
                   sequence is split across the N ranks with one all-gather
                   of the (P, H) chunk carries; value = algorithmic GB/s.

  mlp              fused SwiGLU up-projection silu(x Wg^T) * (x Wu^T) on the
                   tensor cores (mamba_gated_mlp_up), 262144 tokens (batch 64
                   x L 4096), d 2048, h 4096, FP16 in/out, FP32 accumulation;
                   tokens split across ranks; value = TFLOP/s of the job.

One process per GPU; for N > 1 launch with torchrun (RANK/LOCAL_RANK/
WORLD_SIZE/MASTER_* from the environment).  Rank 0 prints one JSON line.
`--impl reference` times the reference's CPU implementation of the same
path on this host (the reference's own selective_scan_cpu, compiled from
its sources into oracle/_ref, inside the CPU block restatement).
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "mamba-metal_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

STACK = dict(d_model=2048, d_state=16, d_conv=4, expand=2, n_layer=48, batch=64, seqlen=4096)
BLOCK = dict(d_model=768, d_state=16, d_conv=4, expand=2, n_layer=1, batch=8, seqlen=2048)
DECODE = dict(d_model=2560, d_state=16, d_conv=4, expand=2, n_layer=64, batch=256, decode_steps=1024)
SCAN = dict(batch=1, d_inner=2048, d_state=16, seqlen=131072)
MLP = dict(tokens=262144, d=2048, h=4096)
METRIC = "selective-scan HBM GB/s (% peak) and block fwd tokens/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(kernel):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.index = vis.split(",")[local_rank] if vis else str(local_rank)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", self.index], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU block reference timing (cpu_baseline leg and --impl reference arm)
# ---------------------------------------------------------------------------
def cpu_stack_tokens_per_s(budget_s, use_reference_scan, tokens=256, seed=0):
    """Times the CPU restatement of the stack workload's layer on one
    sequence of `tokens` tokens; per-token throughput of the full 48-layer
    stack is extrapolated from the measured per-layer time.  Uses every host
    thread (torchrun sets OMP_NUM_THREADS=1, so the BLAS pool is resized)."""
    import oracle  # noqa: F401  (CPU checker, only in this leg)
    from oracle import block_ref
    import mamba_b200 as mb
    from threadpoolctl import threadpool_limits
    with threadpool_limits(limits=os.cpu_count() or 1):
        return _cpu_stack(budget_s, use_reference_scan, tokens, seed, oracle, block_ref, mb)


def _cpu_stack(budget_s, use_reference_scan, tokens, seed, oracle, block_ref, mb):
    cfg = mb.MambaConfig(STACK["d_model"], STACK["d_state"], STACK["d_conv"], STACK["expand"],
                         STACK["n_layer"], mb.F16)
    rng = np.random.default_rng(seed)
    w = mb.random_layer_weights(cfg, rng)
    h = rng.standard_normal((1, tokens, cfg.d_model)).astype(np.float32)
    scan_impl = "reference" if use_reference_scan else "oracle"
    block_ref.block_forward(h, w, cfg, block_ref.F16, scan_impl=scan_impl)  # warm-up
    t0 = time.perf_counter()
    layers = 0
    while True:
        h = block_ref.block_forward(h, w, cfg, block_ref.F16, scan_impl=scan_impl)
        layers += 1
        if time.perf_counter() - t0 > budget_s or layers >= cfg.n_layer:
            break
    dt = time.perf_counter() - t0
    per_layer = dt / layers
    tps = tokens / (per_layer * cfg.n_layer)
    sample = ("1 sequence x %d tokens through %d of the 48 layers (CPU block restatement, "
              "%s scan), extrapolated to the 48-layer stack" %
              (tokens, layers, "reference selective_scan_cpu" if use_reference_scan else "oracle"))
    return tps, sample


def cpu_block_forward(h, layers, cfg):
    """The CPU block restatement over every layer on host FP32 input h
    [1, T, d_model]; returns (output, seconds).  All host threads (torchrun
    sets OMP_NUM_THREADS=1, so the BLAS pool is resized)."""
    from oracle import block_ref  # CPU checker, only in this leg
    from threadpoolctl import threadpool_limits
    with threadpool_limits(limits=os.cpu_count() or 1):
        t0 = time.perf_counter()
        ref = block_ref.model_forward(h, layers, cfg, block_ref.F16)
        return ref, time.perf_counter() - t0


def run_reference_arm(args, world, rank):
    """--impl reference: the reference's CPU implementation on this host."""
    if rank != 0:
        return
    import oracle
    cores = os.cpu_count() or 1
    if oracle.ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable": "reference CPU oracle not built"}))
        return
    if args.workload == "scan":
        vals = []
        L = 16384
        rng = np.random.default_rng(0)
        D, N = SCAN["d_inner"], SCAN["d_state"]
        x = rng.standard_normal((1, L, D)).astype(np.float16).astype(np.float32)
        dr = rng.normal(-4.6, 0.5, (1, L, D)).astype(np.float32)
        B = rng.standard_normal((1, L, N)).astype(np.float16).astype(np.float32)
        C = rng.standard_normal((1, L, N)).astype(np.float16).astype(np.float32)
        A = np.tile(-np.arange(1, N + 1, dtype=np.float32), (D, 1))
        Dk = np.ones(D, np.float32)
        nbytes = L * D * (2 + 4 + 2 + 2) + L * N * 2 * 2
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            oracle.ref_scan_batched(x, dr, B, C, A, Dk, nthreads=cores)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                vals.append(nbytes / dt / 1e9)
        v = statistics.median(vals)
        unit = "GB/s"
        sample = "L=16384 slice of the L=131072 sequence (all 2048 channels)"
        cfgd = {"workload": "selective scan batch 1, d_inner 2048, d_state 16, L 131072",
                "dtype_in": "x,B,C,z fp16 / delta fp32"}
    else:
        vals = []
        for i in range(args.warmup + args.steps):
            tps, sample = cpu_stack_tokens_per_s(budget_s=8.0, use_reference_scan=True, tokens=128)
            if i >= args.warmup:
                vals.append(tps)
        v = statistics.median(vals)
        unit = "tokens/s"
        cfgd = stack_config_dict(world)
    line = {"metric": METRIC, "impl": "reference", "value": v, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "data": "synthetic", "dtype": "f32", "config": cfgd,
            "cpu_baseline": {"value": v, "unit": unit, "cores": cores, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def stack_config_dict(world):
    return {"workload": "mamba stack forward: 48 layers, d_model 2048, d_inner 4096, "
                        "d_state 16, d_conv 4, dt_rank 128, batch 64, L 4096",
            "global_batch": STACK["batch"], "seq_len": STACK["seqlen"],
            "parallelism": "batch-sharded dp%d (no collective)" % world,
            "l2": "inputs larger than L2 (activations are GBs per layer)"}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_stack(args, world, rank, local, C=STACK):
    import torch
    import mamba_b200 as mb
    n_layer = args.layers or C["n_layer"]
    gb = args.batch or C["batch"]
    L = args.seqlen or C["seqlen"]
    if gb % world:
        raise SystemExit("global batch %d not divisible by %d ranks" % (gb, world))
    b = gb // world
    M, D, N = C["d_model"], C["d_model"] * C["expand"], C["d_state"]
    model = mb.Model(M, N, C["d_conv"], C["expand"], n_layer, mb.F16)
    model.init_random(1234)
    # All work of the timed region on one explicit stream: the model's calls
    # (set_stream) and the CUDA events that time them.
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    model.set_stream(stream.cuda_stream)
    g = torch.Generator(device="cuda")
    g.manual_seed(1000 + rank)
    x = torch.randn((b, L, M), device="cuda", dtype=torch.float32, generator=g)
    out = torch.empty_like(x)

    for _ in range(args.warmup):
        model.forward_device(x.data_ptr(), out.data_ptr(), b, L, stream.cuda_stream)
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    model.profile(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        model.forward_device(x.data_ptr(), out.data_ptr(), b, L, stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    prof = model.profile_read()
    model.profile(False)
    barrier(world)
    t_ms = max_over_ranks(e0.elapsed_time(e1), world)

    tokens = gb * L * args.steps
    value = tokens / (t_ms / 1e3)
    scan_ms, scan_calls, scan_kernels = prof["scan"]
    scan_ms = max_over_ranks(scan_ms, world)
    per_launch_s = scan_ms / scan_calls / 1e3
    # algorithmic bytes of one scan launch: x, delta, z read and y written
    # (FP16, 2 B each) per (b,t,d); B and C (FP16) per (b,t,n); A, D, dt_bias.
    scan_bytes = b * L * D * 8 + b * L * 2 * N * 2 + D * N * 4 + 2 * D * 4
    achieved = scan_bytes / per_launch_s / 1e9
    peak, peak_src = peaks()
    kernels = sum(v[2] for v in prof.values())
    breakdown = {k: round(v[0] / max(v[1], 1), 4) for k, v in prof.items()}
    # DRAM traffic per launch: the committed ncu figure for the batch-64
    # stack launch, scaled by the (b, t, d) units of this launch.
    traffic = None
    if C is STACK and committed_traffic("selective_scan_stack"):
        traffic = committed_traffic("selective_scan_stack") * (b * L) / (C["batch"] * C["seqlen"])
    # The scan's compute ceiling: 18 special-function (XU) operations per
    # (b, t, d) (16 state exponentials, softplus, SiLU) at 16 per clock per
    # SM, at the median SM clock sampled during the timed region.
    xu_ops = 18.0 * b * L * D
    sm_mhz = (clk or {}).get("sm_mhz") or 1965.0
    xu_peak = 16.0 * torch.cuda.get_device_properties(local).multi_processor_count * sm_mhz * 1e6
    xu = {"ops_per_launch": xu_ops, "achieved_ops_per_s": xu_ops / per_launch_s, "peak_ops_per_s": xu_peak,
          "frac": xu_ops / per_launch_s / xu_peak, "sm_mhz": sm_mhz}

    # end to end through the reference C API (mamba_forward, host FP32
    # buffers in pinned memory; H2D and D2H inside the timed region)
    e2e = None
    if not args.no_e2e:
        hin = torch.empty((b, L, M), dtype=torch.float32, pin_memory=True)
        hin.copy_(x.cpu())
        hout = torch.empty_like(hin).pin_memory()
        model.forward_ptr(hin.data_ptr(), hout.data_ptr(), b, L)  # warm
        barrier(world)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            model.forward_ptr(hin.data_ptr(), hout.data_ptr(), b, L)
        f1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        te = max_over_ranks(f0.elapsed_time(f1), world)
        e2e = {"value": tokens / (te / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": b * L * M * 4 * world, "d2h_bytes_per_step": b * L * M * 4 * world,
               "api": "mamba_forward (host FP32, pinned)"}

    # Parity and the CPU baseline on the same weights: the CPU block
    # restatement runs all layers over the first `ptok` tokens of the rank's
    # first row (every op is causal in time, so these outputs of the
    # full-size GPU forward depend on nothing else) and is timed.
    cpu = parity = None
    if rank == 0 and C is STACK and not args.no_parity:
        ptok = 256
        cfg = mb.MambaConfig(M, N, C["d_conv"], C["expand"], n_layer, mb.F16)
        layers = mb.weights_from_blob(cfg, model.save_weights())
        h = x[:1, :ptok].cpu().numpy()
        got = out[:1, :ptok].cpu().numpy()
        ref, dt = cpu_block_forward(h, layers, cfg)
        err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref - h)))
        parity = {"normwise_rel_err": err, "tolerance": 2e-3, "pass": err < 2e-3,
                  "checked": "row 0, tokens 0..%d, all %d layers, of the timed forward's output, against "
                             "the CPU block reference on the same weights (mamba_save_weights)" % (ptok - 1, n_layer)}
        if world == 1 and not args.no_cpu_baseline:
            cpu = {"value": ptok / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": "1 sequence x %d tokens through all %d layers (CPU block restatement with the "
                             "oracle scan, numpy BLAS on all host threads), same weights as the GPU run"
                             % (ptok, n_layer)}
        del layers

    if rank == 0:
        if C is STACK:
            cfgd = stack_config_dict(world)
        else:
            cfgd = {"workload": "mamba block forward: %d layer, d_model %d, d_inner %d, d_state %d, d_conv %d, "
                                "dt_rank %d, batch %d, L %d" % (C["n_layer"], M, D, N, C["d_conv"], (M + 15) // 16,
                                                                C["batch"], C["seqlen"]),
                    "global_batch": C["batch"], "seq_len": C["seqlen"],
                    "parallelism": "batch-sharded dp%d (no collective)" % world,
                    "l2": "activations exceed L2 between steps only partly; reported as measured"}
        if n_layer != C["n_layer"] or gb != C["batch"] or L != C["seqlen"]:
            cfgd["reduced"] = {"n_layer": n_layer, "batch": gb, "seqlen": L}
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f16 activations/weights, f32 state+residual, f32 scan arithmetic",
                "data": "synthetic (random-init weights, N(0,1) inputs)", "config": cfgd,
                "roofline": {"kernel": "selective_scan (fused, gated)", "bound": "hbm",
                             "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_source": peak_src,
                             "traffic": traffic,
                             "algorithmic_bytes_per_launch": scan_bytes,
                             "avg_launch_ms": per_launch_s * 1e3,
                             "xu_ceiling": xu},
                "op_ms_per_layer": breakdown,
                "gpu_launches": kernels,
                "parity": parity,
                "cpu_baseline": cpu, "e2e": e2e, "clocks": clk}
        print(json.dumps(line))


def run_decode(args, world, rank, local):
    import torch
    import mamba_b200 as mb
    C = DECODE
    n_layer = args.layers or C["n_layer"]
    gb = args.batch or C["batch"]
    K = args.decode_steps or C["decode_steps"]
    if gb % world:
        raise SystemExit("global batch %d not divisible by %d ranks" % (gb, world))
    b = gb // world
    M, D, N = C["d_model"], C["d_model"] * C["expand"], C["d_state"]
    model = mb.Model(M, N, C["d_conv"], C["expand"], n_layer, mb.F16)
    model.init_random(4321)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    model.set_stream(stream.cuda_stream)
    st = model.create_state(b)
    g = torch.Generator(device="cuda")
    g.manual_seed(500 + rank)
    toks = torch.randn((K, b, M), device="cuda", dtype=torch.float32, generator=g)
    cur = torch.empty((b, M), device="cuda")
    out = torch.empty_like(cur)

    def step(i):
        cur.copy_(toks[i % K])
        st.step_device(cur.data_ptr(), out.data_ptr(), stream.cuda_stream)

    for i in range(args.warmup):
        step(i)
    # per-operation times from a few profiled (graph-free) steps
    model.profile(True)
    for i in range(2):
        step(i)
    prof = model.profile_read()
    model.profile(False)
    st.reset()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(world)
    t_ms = max_over_ranks(e0.elapsed_time(e1), world)
    peak, peak_src = peaks()
    ssm_ms = prof["scan"][0] / max(prof["scan"][1], 1)
    ssm_bytes = b * D * N * 4 * 2 + b * D * 2 * 4 + b * 2 * N * 2 + D * N * 4 + 2 * D * 4
    if rank == 0:
        line = {"metric": METRIC, "value": gb * K / (t_ms / 1e3), "unit": "tokens/s", "n_gpus": world,
                "steps": K, "warmup": args.warmup, "ms_per_step": t_ms / K, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": "f16 activations/weights, f32 conv/ssm state", "data": "synthetic",
                "config": {"workload": "decode: %d layers, d_model %d, d_inner %d, d_state %d, dt_rank %d, "
                                       "batch %d, %d steps from zero state" % (n_layer, M, D, N, (M + 15) // 16,
                                                                               gb, K),
                           "parallelism": "batch-sharded dp%d (weights replicated)" % world},
                "roofline": {"kernel": "ssm_step (decode state update)", "bound": "hbm",
                             "achieved": ssm_bytes / (ssm_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                             "frac": ssm_bytes / (ssm_ms / 1e3) / 1e9 / peak, "peak_source": peak_src,
                             "algorithmic_bytes_per_launch": ssm_bytes, "avg_launch_ms": ssm_ms,
                             "traffic": None},
                "op_ms_per_layer": {k: round(v[0] / max(v[1], 1), 4) for k, v in prof.items()},
                "gpu_launches": 2 * n_layer * K, "clocks": clk}
        print(json.dumps(line))


def run_scan(args, world, rank, local):
    import torch
    import mamba_b200 as mb
    from mamba_b200.seqpar import NcclComm, sequence_parallel_scan_nccl
    Lg = args.seqlen or SCAN["seqlen"]
    if Lg % world:
        raise SystemExit("seqlen not divisible by ranks")
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    L = Lg // world
    D, N = SCAN["d_inner"], SCAN["d_state"]
    # Every rank draws the whole sequence from one seed (for the parity check
    # against a one-GPU scan) and scans its own time slice.
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    xf = torch.randn((1, Lg, D), device="cuda", generator=g).half()
    zf = torch.randn((1, Lg, D), device="cuda", generator=g).half()
    drf = (torch.randn((1, Lg, D), device="cuda", generator=g) * 0.5 - 4.6).float()
    Bf = torch.randn((1, Lg, N), device="cuda", generator=g).half()
    Cf = torch.randn((1, Lg, N), device="cuda", generator=g).half()
    s = slice(rank * L, (rank + 1) * L)
    x, z, dr, B, C = (t[:, s].contiguous() for t in (xf, zf, drf, Bf, Cf))
    A = -torch.arange(1, N + 1, device="cuda", dtype=torch.float32).repeat(D, 1).contiguous()
    Dk = torch.ones(D, device="cuda")
    comm = NcclComm() if world > 1 else None
    y = torch.empty_like(x)
    ws = None

    def step():
        if world == 1:
            return mb.selective_scan(x, dr, A, B, C, D=Dk, z=z, return_final_state=True, y=y)
        return sequence_parallel_scan_nccl(comm, x, dr, A, B, C, D=Dk, z=z, y=y, workspace=ws, stream=stream)

    if world > 1:
        need = mb.lib().mamba_selective_scan_seqpar_workspace(
            ctypes_byref(mb._scan_args(x, dr, A, B, C, Dk, z, None, None, y, None, 0)), world)
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device="cuda")
    for _ in range(args.warmup):
        step()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        _, h_last = step()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(world)
    t_ms = max_over_ranks(e0.elapsed_time(e1), world)
    # parity: this rank's slice (and, on the last rank, the final state)
    # against the one-GPU scan of the whole sequence
    yf, hf = mb.selective_scan(xf, drf, A, Bf, Cf, D=Dk, z=zf, return_final_state=True)
    torch.cuda.synchronize()
    ref = yf[:, s].float()
    err_y = float((y.float() - ref).abs().max() / ref.abs().max())
    err_h = float((h_last - hf).abs().max() / hf.abs().max()) if rank == world - 1 else 0.0
    err = max_over_ranks(max(err_y, err_h), world)
    if comm is not None:
        comm.close()
    nbytes = Lg * D * (2 + 4 + 2 + 2) + Lg * N * 2 * 2 + D * N * 4 + D * 4
    value = nbytes * args.steps / (t_ms / 1e3) / 1e9
    peak, peak_src = peaks()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "x,B,C,z,y f16; delta f32; f32 state", "data": "synthetic",
                "config": {"workload": "selective scan batch 1, d_inner 2048, d_state 16, L %d" % Lg,
                           "parallelism": ("sequence-sharded over %d ranks: mamba_selective_scan_seqpar "
                                           "(ncclAllGather of the slice carries, %d NCCL ranks)" % (world, world))
                           if world > 1 else "one GPU"},
                "roofline": {"bound": "hbm", "achieved": value / world, "peak": peak, "unit": "GB/s",
                             "frac": value / world / peak, "peak_source": peak_src, "traffic": None},
                "parity": {"normwise_rel_err": err, "tolerance": 2e-3, "pass": err < 2e-3,
                           "checked": "each rank's slice of y and the last rank's final state against the "
                                      "one-GPU scan of the whole sequence (max over ranks)"},
                # chunked scan: summary + combine + output kernels; sharded:
                # slice summary (2), compose (1), rescan (3), plus NCCL's
                "gpu_launches": args.steps * (3 if world == 1 else 6),
                "clocks": clk}
        print(json.dumps(line))


def ctypes_byref(obj):
    import ctypes
    return ctypes.byref(obj)


def run_mlp(args, world, rank, local):
    import torch
    import mamba_b200 as mb
    T = args.batch * 4096 if args.batch else MLP["tokens"]
    d, h = MLP["d"], MLP["h"]
    if T % world:
        raise SystemExit("tokens not divisible by ranks")
    t = T // world
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    g = torch.Generator(device="cuda")
    g.manual_seed(900 + rank)
    x = torch.randn((t, d), device="cuda", generator=g).half()
    w = (torch.randn((2 * h, d), device="cuda", generator=g) * 0.02).half()
    out = torch.empty((t, h), device="cuda", dtype=torch.float16)

    def step():
        mb.gated_mlp_up(x, w, out=out, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(world)
    assert mb.device_status() == 0
    t_ms = max_over_ranks(e0.elapsed_time(e1), world)
    flop = 2.0 * T * d * 2 * h
    value = flop * args.steps / (t_ms / 1e3) / 1e12
    e2e = None
    if not args.no_e2e:
        hx = torch.empty((t, d), dtype=torch.float16, pin_memory=True)
        hx.copy_(x.cpu())
        hout = torch.empty((t, h), dtype=torch.float16, pin_memory=True)
        xs = torch.empty_like(x)
        for _ in range(2):
            xs.copy_(hx, non_blocking=True)
            mb.gated_mlp_up(xs, w, out=out, stream=stream.cuda_stream)
            hout.copy_(out, non_blocking=True)
        torch.cuda.synchronize()
        barrier(world)
        e0.record(stream)
        for _ in range(args.steps):
            xs.copy_(hx, non_blocking=True)
            mb.gated_mlp_up(xs, w, out=out, stream=stream.cuda_stream)
            hout.copy_(out, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        te = max_over_ranks(e0.elapsed_time(e1), world)
        e2e = {"value": flop * args.steps / (te / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": t * d * 2, "d2h_bytes_per_step": t * h * 2,
               "api": "mamba_gated_mlp_up (pinned host FP16 in/out)"}
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak = float(pk.get("bf16_tflops", 1590.0))
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16 operands/output, f32 accumulation",
                "data": "synthetic",
                "config": {"workload": "gated MLP up-projection (SwiGLU fused): tokens %d, d %d, h %d" % (T, d, h),
                           "parallelism": "token-sharded dp%d" % world,
                           "l2": "x (%.1f GB) and out larger than L2" % (T * d * 2 / 1e9)},
                "roofline": {"kernel": "gated_mlp_up (tcgen05)", "bound": "tensor", "achieved": value / world,
                             "peak": peak, "unit": "TFLOP/s", "frac": value / world / peak,
                             "peak_source": "measured" if pk else "fallback", "traffic": None},
                "gpu_launches": args.steps, "e2e": e2e, "clocks": clk}
        print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stack", choices=["stack", "block", "decode", "scan", "mlp"])
    ap.add_argument("--decode-steps", type=int, default=0, help="decode workload: steps timed")
    ap.add_argument("--layers", type=int, default=0, help="override n_layer (reduced runs)")
    ap.add_argument("--batch", type=int, default=0, help="override global batch")
    ap.add_argument("--seqlen", type=int, default=0, help="override L")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the CPU parity check of the stack output")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.gpus != world and world > 1:
        print("warning: --gpus %d but WORLD_SIZE %d" % (args.gpus, world), file=sys.stderr)
    if args.gpus > 1 and world == 1:
        raise SystemExit("launch N>1 with torchrun (one process per GPU)")
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        return
    world, rank, local = dist_setup()
    try:
        if args.workload == "scan":
            run_scan(args, world, rank, local)
        elif args.workload == "mlp":
            run_mlp(args, world, rank, local)
        elif args.workload == "decode":
            run_decode(args, world, rank, local)
        elif args.workload == "block":
            run_stack(args, world, rank, local, C=BLOCK)
        else:
            run_stack(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

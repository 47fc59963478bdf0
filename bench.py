"""Benchmark: SelectiveScanFused at batch 8, d_inner 5120, seqlen 2048, d_state 16 (fp32).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

One step = one selective scan over the whole per-GPU batch (inputs resident in
HBM). With N GPUs (one process per GPU, launched by torch.distributed.run)
each rank scans its own batch-8 shard of a batch-8N job: the op shards by
batch with no exchange, so the scaling is weak. After the timed steps the
output shards are gathered to rank 0 through NCCL (the op's one collective),
timed on its own (gather_ms). Rank 0 prints one JSON line.

value     — scan elements (batch*d_inner*seqlen*d_state, all ranks) per second,
            timed with CUDA events over K steps, max over ranks.
e2e       — the same metric end to end through the ONNX Runtime custom-op
            entry (RegisterCustomOps -> CreateKernelV2 -> KernelComputeV2,
            driven by the CUDA-EP host of tests/fake_ort, ORT itself not being
            installed) with host buffers: pinned host inputs -> H2D -> op ->
            D2H of the output, pipelined per batch entry on two streams.
roofline  — the scan kernel's algorithmic HBM bytes per launch / its launch
            duration, against the measured copy bandwidth.
cpu_baseline — the reference's own C++ plugin (oracle/_ref, OpenMP, all host
            threads) on the same workload (all 8 batch entries).
--impl reference runs that reference plugin alone, as the reference arm.

    python bench.py --workload mamba130m [--gpus N] [--steps K] [--warmup W]

Mamba-130m forward (24 blocks, fp32) at batch 1 x seqlen 1024 per GPU with
every selective scan on SelectiveScanFusedExact; one step = one CUDA-graph
replay of the forward; value in tokens/s (all ranks; each rank runs its own
replica, no collective). Its cpu_baseline (and --impl reference) is the same
forward on the host: torch CPU GEMMs with the reference's C++ plugin doing
the scans.

    python bench.py --workload scan-b64 [--gpus N] [--steps K]

SelectiveScanFused on a fixed total batch of 64 x 5120 x 4096 sharded by batch
over the N GPUs (strong scaling); value from the compute time alone, the NCCL
gather of the output to rank 0 timed separately (gather_ms).

    python bench.py --workload mamba130m-decode [--gpus N] [--steps K]

Single-token decode of the same model after a 1024-token prefill: one step =
one CUDA-graph replay of the decode step (scans through h0/h_last), value in
tokens/s. The reference has no decode path (--impl reference says so).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "mamba-onnx_b200")]

OP = "SelectiveScanFused"
BATCH, DIM, SEQLEN, NSTATE = 8, 5120, 2048, 16
SEED = 1
METRIC = "scan elements/s (B*D*N*L)"
UNIT = "scan elements/s"
WORKLOAD = (f"{OP} fp32, batch {BATCH} x d_inner {DIM} x seqlen {SEQLEN}, d_state {NSTATE} "
            f"per GPU (Mamba-2.8B layer shape)")


def algorithmic_bytes(B, D, L, N=NSTATE, fused=True):
    """Bytes the op must move once: read u, delta, (z), write out; read B, C, A, D."""
    return 4 * B * D * L * (3 + (1 if fused else 0)) + 8 * B * L * N + 4 * D * N + 4 * D


def sfu_ops(B, D, L, fused=True, exact=False):
    """Transcendentals: softplus (exp + log) and silu (exp) per (b,d,l); exp per element if exact."""
    return (3 * B * D * L if fused else 0) + (B * D * L * NSTATE if exact else 0)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks (NVML)

class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU every 10 ms on a thread."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, torch_device):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nv = pynvml
            # NVML ignores CUDA_VISIBLE_DEVICES: find the GPU by its UUID.
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            try:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
            except Exception:  # noqa: BLE001
                self.h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception as e:  # noqa: BLE001 - NVML unavailable: report no samples
            self.nv, self.err = None, str(e)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.get_reasons(self.h)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self.nv:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.nv:
            self.t.join()

    def summary(self):
        d = {"sm_mhz": statistics.median(self.samples) if self.samples else None,
             "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
             "samples": len(self.samples)}
        if self.nv is None:
            d["error"] = self.err
        return d


# ---------------------------------------------------------------- inputs

def device_inputs(torch, device, seed):
    """Benchmark distributions drawn on the device: u, z, B, C ~ N(0,1);
    delta = N(0, 0.5^2) + log(expm1(dt)), dt log-uniform [1e-3, 1e-1] per channel;
    A[d, n] = -(n+1); D = 1."""
    g = torch.Generator(device=device).manual_seed(seed)
    kw = dict(device=device, generator=g)
    B, D, L = BATCH, DIM, SEQLEN
    u = torch.randn(B, D, L, **kw)
    z = torch.randn(B, D, L, **kw)
    Bm = torch.randn(B, L, NSTATE, **kw)
    Cm = torch.randn(B, L, NSTATE, **kw)
    lo, hi = float(np.log(1e-3)), float(np.log(1e-1))
    dt = torch.exp(torch.rand(D, **kw) * (hi - lo) + lo)
    delta = torch.randn(B, D, L, **kw) * 0.5 + torch.log(torch.expm1(dt))[None, :, None]
    A = -torch.arange(1, NSTATE + 1, device=device, dtype=torch.float32).repeat(D, 1)
    Dv = torch.ones(D, device=device)
    return u, delta, A, Bm, Cm, Dv, z


# ---------------------------------------------------------------- CPU baseline

def reference_inputs(entries):
    """Host copies of `entries` batch entries of the workload, drawn with the
    benchmark distributions from a seeded Philox stream."""
    g = np.random.Generator(np.random.Philox(SEED))
    D, L = DIM, SEQLEN
    u = g.standard_normal((entries, D, L), dtype=np.float32)
    z = g.standard_normal((entries, D, L), dtype=np.float32)
    Bm = g.standard_normal((entries, L, NSTATE), dtype=np.float32)
    Cm = g.standard_normal((entries, L, NSTATE), dtype=np.float32)
    dt = np.exp(g.uniform(np.log(1e-3), np.log(1e-1), D)).astype(np.float32)
    delta = (g.standard_normal((entries, D, L), dtype=np.float32) * np.float32(0.5)
             + np.log(np.expm1(dt.astype(np.float64))).astype(np.float32)[None, :, None])
    A = -np.tile(np.arange(1, NSTATE + 1, dtype=np.float32), (D, 1))
    Dv = np.ones(D, np.float32)
    return u, delta, A, Bm, Cm, Dv, z


def reference_timer(n_threads):
    """(fn, kind, threads): one call of the reference's C++ plugin (oracle/_ref,
    OpenMP) over the whole per-GPU workload (batch 8 x 5120 x 2048), or of the
    scalar port when the plugin was not built."""
    from oracle import oracle

    u, delta, A, Bm, Cm, Dv, z = reference_inputs(BATCH)
    out = np.empty_like(u)
    if oracle.ref_available():
        return (lambda: oracle.ref_run(OP, u, delta, A, Bm, Cm, Dv, z, n_threads=n_threads,
                                       out=out)), "reference", n_threads
    return (lambda: oracle.scan_f32ref(OP, u, delta, A, Bm, Cm, Dv, z)), "port", 1


def reference_sample(n_threads, reps, budget_s=30.0):
    """The reference C++ plugin on the full per-GPU workload (host arrays):
    up to `reps` timed calls after one warm-up, stopping once `budget_s`
    seconds of timed work have accumulated."""
    fn, kind, n_threads = reference_timer(n_threads)
    fn()  # warm-up (page-in, thread pool)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
        if sum(times) > budget_s:
            break
    elems = BATCH * DIM * SEQLEN * NSTATE
    return {"value": elems / statistics.median(times), "unit": UNIT, "cores": n_threads,
            "kind": kind,
            "sample": f"the full workload ({BATCH}x{DIM}x{SEQLEN}) per call, median of "
                      f"{len(times)} calls after 1 warm-up, {n_threads} OpenMP threads"}


def run_reference_arm(args, rank):
    """The reference's C++ plugin on the host cores, one call over the whole
    per-GPU workload per step: W warm-up calls, then K timed calls."""
    if rank != 0:
        return
    from oracle import oracle

    fn, kind, threads = reference_timer(oracle.host_threads())
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    sec = (time.perf_counter() - t0) / args.steps
    value = BATCH * DIM * SEQLEN * NSTATE / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sec, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "op": OP, "batch_per_gpu": BATCH, "d_inner": DIM,
                   "seqlen": SEQLEN, "d_state": NSTATE,
                   "step": "one reference plugin call on the whole batch 8 x 5120 x 2048"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"the full workload per step, mean of {args.steps} calls "
                                   f"after {args.warmup} warm-up calls"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 2000; 20 for --impl reference, whose step is "
                         "one ~0.1-0.2 s host call)")
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu-case", action="store_true",
                    help="for profilers: build the inputs, run warmup+steps calls, print nothing timed")
    ap.add_argument("--case", default=None, metavar="OP:B:D:L",
                    help="with --ncu-case: another op and shape (benchmark-configuration "
                         "distributions; non-fused ops draw delta per element)")
    ap.add_argument("--workload", choices=["scan", "scan-b64", "mamba130m", "mamba130m-decode"],
                    default="scan")
    ap.add_argument("--gemm-case", default=None, metavar="M:N:K",
                    help="profiling helper: warmup + steps calls of the tensor-core 3xTF32 "
                         "GEMM on random [M,K] x [N,K] operands; nothing timed")
    args = ap.parse_args()
    if args.case and not args.ncu_case:
        ap.error("--case is a profiling helper: use it with --ncu-case")
    args.warmup = max(3, args.warmup)
    if args.steps is None:
        args.steps = 20 if args.impl == "reference" else 2000
    if args.workload == "mamba130m":
        return run_model(args)
    if args.workload == "mamba130m-decode":
        return run_decode(args)
    if args.workload == "scan-b64":
        return run_scan_b64(args)
    if args.ncu_case and args.case:
        return run_case(args)
    if args.gemm_case:
        return run_gemm_case(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference_arm(args, rank)

    import torch
    import torch.distributed as dist

    from mamba_onnx import cuda

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()

    # CPU baseline first (rank 0, one GPU only): it must not overlap the GPU timing.
    cpu = None
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.ncu_case):
        from oracle import oracle

        cpu = reference_sample(oracle.host_threads(), reps=5)

    u, delta, A, Bm, Cm, Dv, z = device_inputs(torch, device, SEED + rank)
    out = torch.empty_like(u)
    stream = torch.cuda.current_stream(device)
    ws_bytes = cuda.workspace_size(OP, BATCH, DIM, SEQLEN)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    # one emit launch, or aggregate + carry + emit when the plan splits sequences
    launches_per_step = 1 if ws_bytes == 0 else 3

    def step():
        cuda.selective_scan(OP, u, delta, A, Bm, Cm, Dv, z, out=out, workspace=ws, stream=stream)

    if args.ncu_case:
        for _ in range(args.warmup + args.steps):
            step()
        torch.cuda.synchronize()
        print(json.dumps({"ncu_case": WORKLOAD, "launches_per_call": launches_per_step,
                          "calls": args.warmup + args.steps}))
        return

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    elems_per_step = BATCH * DIM * SEQLEN * NSTATE
    value = world * elems_per_step / (ms_per_step * 1e-3)

    # ---- the op's one collective: every rank's output shard to rank 0 (NCCL)
    gather = None
    if world > 1:
        gather = gather_to_rank0(torch, dist, out, world, rank, device, stream)

    # ---- end to end through the custom-op entry, host buffers (pinned), per-entry pipeline
    e2e = end_to_end(torch, device, args, world)

    if rank == 0:
        hbm_peak, peak_kind = measured_peaks()
        algo = algorithmic_bytes(BATCH, DIM, SEQLEN)
        achieved = algo / (ms_per_step * 1e-3) / 1e9
        traffic = None
        tf = ROOT / "profiles" / "scan_fused_8x5120x2048.traffic.json"
        if tf.exists():
            traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "op": OP, "batch_per_gpu": BATCH,
                       "global_batch": BATCH * world, "d_inner": DIM, "seqlen": SEQLEN,
                       "d_state": NSTATE,
                       "parallelism": (f"batch-sharded x{world}; the output gathered to rank 0 "
                                       "by NCCL after the timed steps (gather_ms)"
                                       if world > 1 else "one GPU"),
                       "l2": "inputs 1.34 GB per GPU, larger than L2; no flush"},
            "nccl_ranks": world if world > 1 else None,
            "gather": gather,
            "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": traffic,
                         "per": "op call (aggregate + carry + emit launches when the plan splits)",
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_launch": algo,
                         "sfu_ops_per_launch": sfu_ops(BATCH, DIM, SEQLEN)},
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def gather_to_rank0(torch, dist, out, world, rank, device, stream, reps=5):
    """Gather every rank's [8, 5120, 2048] output shard into a preallocated
    [8N, 5120, 2048] tensor on rank 0 (torch.distributed.gather over NCCL,
    mamba_onnx.distributed.gather_output); one warm-up gather, then `reps`
    timed ones, CUDA events, max over ranks. The result is checked against
    rank 0's own shard and one remote shard's checksum."""
    from mamba_onnx.distributed import gather_output, shard_plan

    plan = shard_plan(BATCH * world, DIM, world, rank)
    full = torch.empty(BATCH * world, DIM, SEQLEN, device=device) if rank == 0 else None
    gather_output(out, plan, out=full)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        gather_output(out, plan, out=full)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # rank 1's checksum against what landed in its slice on rank 0
    s1 = torch.tensor([float(out.double().sum().item())], device=device, dtype=torch.float64)
    sums = [torch.zeros_like(s1) for _ in range(world)]
    dist.all_gather(sums, s1)
    ok = None
    if rank == 0:
        ok = bool(torch.equal(full[:BATCH], out)) and all(
            float(full[r * BATCH:(r + 1) * BATCH].double().sum().item()) == float(sums[r].item())
            for r in range(world))
    moved = (world - 1) * out.numel() * 4
    del full
    return {"gather_ms": ms, "bytes_to_rank0": moved, "GBps_into_rank0": moved / (ms * 1e-3) / 1e9,
            "reps": reps, "collective": "torch.distributed.gather (NCCL) into a preallocated "
                                        "rank-0 tensor", "checked": ok}


def end_to_end(torch, device, args, world):
    """Host -> device, the op, device -> host per step, through the ONNX Runtime
    custom-op entry of libmamba_ops_cuda.so (RegisterCustomOps, CreateKernelV2
    once, KernelComputeV2 per batch entry) on the CUDA-EP host of tests/fake_ort."""
    sys.path.insert(0, str(ROOT / "tests"))
    import mamba_onnx
    from fake_ort import ort_shim

    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    sess = ort_shim.InferenceSession(ort_shim.make_model(OP, True), opts,
                                     providers=["CUDAExecutionProvider"])
    B, D, L = BATCH, DIM, SEQLEN
    gen = torch.Generator().manual_seed(7)
    host = {
        "u": torch.randn(B, D, L, generator=gen).pin_memory(),
        "delta": (torch.randn(B, D, L, generator=gen) * 0.5 - 3.0).pin_memory(),
        "z": torch.randn(B, D, L, generator=gen).pin_memory(),
        "B": torch.randn(B, L, NSTATE, generator=gen).pin_memory(),
        "C": torch.randn(B, L, NSTATE, generator=gen).pin_memory(),
        "A": (-torch.arange(1, NSTATE + 1, dtype=torch.float32).repeat(D, 1)).pin_memory(),
        "D": torch.ones(D).pin_memory(),
    }
    host_out = torch.empty(B, D, L).pin_memory()
    dev = {k: torch.empty_like(v, device=device) for k, v in host.items()}
    dev_out = torch.empty(B, D, L, device=device)
    streams = [torch.cuda.Stream(device), torch.cuda.Stream(device)]
    main = torch.cuda.current_stream(device)

    def one_step():
        for s in streams:
            s.wait_stream(main)
        with torch.cuda.stream(streams[0]):
            dev["A"].copy_(host["A"], non_blocking=True)
            dev["D"].copy_(host["D"], non_blocking=True)
        streams[1].wait_stream(streams[0])
        for b in range(B):
            s = streams[b % 2]
            with torch.cuda.stream(s):
                for k in ("u", "delta", "z", "B", "C"):
                    dev[k][b].copy_(host[k][b], non_blocking=True)
                # inputs in the op's order u, delta, A, B, C, D, z (cc:167-186)
                sess.run_device([dev["u"][b:b + 1], dev["delta"][b:b + 1], dev["A"],
                                 dev["B"][b:b + 1], dev["C"][b:b + 1], dev["D"],
                                 dev["z"][b:b + 1]], dev_out[b:b + 1], stream=s)
                host_out[b].copy_(dev_out[b], non_blocking=True)
        for s in streams:
            main.wait_stream(s)

    for _ in range(2):
        one_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(1, args.e2e_steps)
    e0.record(main)
    for _ in range(n):
        one_step()
    e1.record(main)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / n
    sess.close()
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    h2d = sum(v.numel() * 4 for v in host.values())
    d2h = host_out.numel() * 4
    return {"value": world * B * D * L * NSTATE / (ms * 1e-3), "unit": UNIT,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms,
            "steps": n, "path": "ONNX Runtime custom-op entry: RegisterCustomOps -> "
                                "CreateKernelV2 -> KernelComputeV2 per batch entry "
                                "(tests/fake_ort CUDA-EP host)",
            "pipeline": "per batch entry on 2 streams, pinned host buffers"}


# ---------------------------------------------------------------- Mamba-130m forward

MODEL_BATCH, MODEL_SEQLEN = 1, 1024
MODEL_METRIC, MODEL_UNIT = "Mamba-130m forward tokens/s", "tokens/s"
MODEL_WORKLOAD = ("Mamba-130m forward (24 blocks, d_model 768, d_inner 1536, d_state 16, "
                  "vocab 50280), fp32, batch 1 x seqlen 1024 per GPU, every selective scan on "
                  "SelectiveScanFusedExact; in_proj, out_proj and the LM head on the "
                  "tensor-core 3xTF32 GEMM (fp32-accurate), x_proj and dt_proj on this "
                  "package's fp32 kernels")


def model_cpu_sample(n_threads, budget_s=30.0):
    """The same forward on the host: torch CPU GEMMs, the reference C++ plugin
    (oracle/_ref, OpenMP) for each layer's scan; delta_bias is added to delta
    before the plugin call (the plugin has no bias input)."""
    import torch

    from mamba_onnx.model import MambaLM, mamba_130m
    from oracle import oracle

    torch.set_num_threads(n_threads)
    model = MambaLM(mamba_130m()).init_random(0)
    ids = torch.randint(0, model.cfg.vocab_size, (MODEL_BATCH, MODEL_SEQLEN),
                        generator=torch.Generator().manual_seed(SEED))
    kind = "reference" if oracle.ref_available() else "port"

    def host_scan(op, u, delta, A, B, C, D, z, delta_bias=None, h0=None, h_last=None):
        if delta_bias is not None:
            delta = delta + delta_bias[None, :, None]
        arrs = [t.detach().contiguous().numpy() for t in (u, delta, A, B, C, D, z)]
        if kind == "reference":
            out = oracle.ref_run(op, *arrs, n_threads=n_threads)
        else:
            out = oracle.scan_f32ref(op, *arrs)
        return torch.from_numpy(out)

    model(ids[:, :64], scan=host_scan)  # warm-up (thread pools, page-in)
    times = []
    while not times or (sum(times) < budget_s and len(times) < 3):
        t0 = time.perf_counter()
        model(ids, scan=host_scan)
        times.append(time.perf_counter() - t0)
    tokens = MODEL_BATCH * MODEL_SEQLEN
    return {"value": tokens / statistics.median(times), "unit": MODEL_UNIT, "cores": n_threads,
            "kind": kind,
            "sample": f"the full forward (batch {MODEL_BATCH} x {MODEL_SEQLEN}), median of "
                      f"{len(times)} runs after a 64-token warm-up; torch CPU GEMMs and the "
                      f"reference plugin's scans on {n_threads} threads"}


def run_model(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import oracle

        cpu = model_cpu_sample(oracle.host_threads())
        print(json.dumps({
            "impl": "reference", "metric": MODEL_METRIC, "value": cpu["value"],
            "unit": MODEL_UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * MODEL_SEQLEN / cpu["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random init, Mamba's initialisation)",
            "config": {"workload": MODEL_WORKLOAD, "batch_per_gpu": MODEL_BATCH,
                       "seqlen": MODEL_SEQLEN},
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": MODEL_UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return

    import torch
    import torch.distributed as dist

    from mamba_onnx import cuda
    from mamba_onnx import model as M
    from mamba_onnx.model import SCAN_OP, MambaLM, mamba_130m

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle

        cpu = model_cpu_sample(oracle.host_threads())

    B, L = MODEL_BATCH, MODEL_SEQLEN
    model = MambaLM(mamba_130m()).init_random(0).to(device)
    ids, logits, graph = model.capture(B, L)
    g = torch.Generator(device=device).manual_seed(SEED + rank)
    ids.copy_(torch.randint(0, model.cfg.vocab_size, (B, L), device=device, generator=g))
    stream = torch.cuda.current_stream(device)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(device) as clocks:
        ms = timed(graph.replay, args.steps)
    if world > 1:
        dist.barrier()
    ms_per_step = max_over_ranks(ms)
    value = world * B * L / (ms_per_step * 1e-3)

    # end to end: token ids from pinned host memory, the last position's
    # logits back to pinned host memory, every step
    host_ids = ids.cpu().pin_memory()
    host_last = torch.empty(B, model.cfg.vocab_size).pin_memory()

    def e2e_step():
        ids.copy_(host_ids, non_blocking=True)
        graph.replay()
        host_last.copy_(logits[:, -1], non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(timed(e2e_step, max(3, args.e2e_steps)))

    # the 24 scans of one forward alone (same shapes, one CUDA graph)
    D, N = model.cfg.d_inner, model.cfg.d_state
    sg = torch.Generator(device=device).manual_seed(3)
    u, z = (torch.randn(B, D, L, device=device, generator=sg) for _ in range(2))
    delta = torch.randn(B, D, L, device=device, generator=sg) * 0.1
    Bm, Cm = (torch.randn(B, L, N, device=device, generator=sg) for _ in range(2))
    layer = model.layers[0]
    A = -torch.exp(layer.A_log.detach())
    scan_args = (SCAN_OP, u, delta, A, Bm, Cm, layer.D.detach(), z)
    out = torch.empty_like(u)
    ws = torch.empty(max(1, cuda.workspace_size(SCAN_OP, B, D, L)), dtype=torch.uint8,
                     device=device)

    def scans():
        for _ in range(model.cfg.n_layer):
            cuda.selective_scan(*scan_args, delta_bias=layer.dt_proj_bias.detach(), out=out,
                                workspace=ws)

    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        scans()
    stream.wait_stream(side)
    sgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(sgraph):
        scans()
    sgraph.replay()
    torch.cuda.synchronize()
    scan_ms = timed(sgraph.replay, 20)
    launches_per_scan = 3 if cuda.workspace_size(SCAN_OP, B, D, L) > 0 else 1
    out_proj_reduce = 1 if cuda.gemm_workspace_size(model.cfg.d_model, L, D) > 0 else 0

    # the same forward run eagerly, its 24 scans through the ONNX Runtime
    # custom-op entry (CreateKernelV2 once per op, KernelComputeV2 per call)
    # on the CUDA-EP host of tests/fake_ort, as an ORT session would run them
    sys.path.insert(0, str(ROOT / "tests"))
    from fake_ort import ort_shim

    ort_scan = ort_shim.OrtScan()
    x_ids = ids.clone()
    for _ in range(2):
        model(x_ids, scan=ort_scan)
    torch.cuda.synchronize()
    ort_ms = max_over_ranks(timed(lambda: model(x_ids, scan=ort_scan), max(3, args.e2e_steps)))
    ort_scan.close()

    if rank == 0:
        hbm_peak, peak_kind = measured_peaks()
        algo = model.cfg.n_layer * algorithmic_bytes(B, D, L)
        achieved = algo / (scan_ms * 1e-3) / 1e9
        line = {
            "metric": MODEL_METRIC, "value": value, "unit": MODEL_UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random init with Mamba's initialisation, uniform token ids)",
            "config": {"workload": MODEL_WORKLOAD, "batch_per_gpu": B, "global_batch": B * world,
                       "seqlen": L, "parallelism": f"replica per GPU x{world}, no collective",
                       "step": "one CUDA-graph replay of the forward",
                       "l2": "weights 0.52 GB > L2; no flush"},
            "e2e": {"value": world * B * L / (e2e_ms * 1e-3), "unit": MODEL_UNIT,
                    "h2d_bytes_per_step": host_ids.numel() * 8,
                    "d2h_bytes_per_step": host_last.numel() * 4, "ms_per_step": e2e_ms,
                    "path": "pinned token ids -> graph replay -> last-position logits to host"},
            # this package's kernels per forward: per block the RMSNorm that
            # writes in_proj's tf32 operand, in_proj, conv + SiLU, x_proj,
            # dt_proj (unless on cuBLAS), the scan, y's tf32 split, out_proj
            # (and its split-K reduction); then the final RMSNorm (to the LM
            # head's operand) and the LM head
            "gpu_launches": (model.cfg.n_layer * (6 + (M.DT_PROJ == "kernel") + launches_per_scan
                                                  + out_proj_reduce) + 2) * args.steps,
            "scan_ms_per_step": scan_ms,
            "ort_entry": {"ms_per_step": ort_ms, "value": world * B * L / (ort_ms * 1e-3),
                          "unit": MODEL_UNIT,
                          "path": "eager forward (no CUDA graph), every scan through "
                                  "RegisterCustomOps -> CreateKernelV2 -> KernelComputeV2 on "
                                  "the tests/fake_ort CUDA-EP host"},
            "roofline": {"bound": "hbm", "kernel": f"the {model.cfg.n_layer} {SCAN_OP} calls of "
                         f"one forward (1x{D}x{L} each)", "achieved": achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": achieved / hbm_peak, "traffic": None,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_step": algo},
            "clocks": clocks.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        del graph, sgraph
        dist.destroy_process_group()


def run_case(args):
    """Profiling helper: warmup + steps calls of one op on one shape, nothing timed."""
    import torch

    from mamba_onnx import cuda

    op, B, D, L = args.case.split(":")
    B, D, L = int(B), int(D), int(L)
    fused = "Fused" in op
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(SEED)
    kw = dict(device=device, generator=g)
    u = torch.randn(B, D, L, **kw)
    z = torch.randn(B, D, L, **kw) if fused else None
    Bm, Cm = torch.randn(B, L, NSTATE, **kw), torch.randn(B, L, NSTATE, **kw)
    lo, hi = float(np.log(1e-3)), float(np.log(1e-1))
    if fused:
        dt = torch.exp(torch.rand(D, **kw) * (hi - lo) + lo)
        delta = torch.randn(B, D, L, **kw) * 0.5 + torch.log(torch.expm1(dt))[None, :, None]
    else:
        delta = torch.exp(torch.rand(B, D, L, **kw) * (hi - lo) + lo)
    A = -torch.arange(1, NSTATE + 1, device=device, dtype=torch.float32).repeat(D, 1)
    Dv = torch.ones(D, device=device)
    out = torch.empty_like(u)
    ws_bytes = cuda.workspace_size(op, B, D, L)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    for _ in range(args.warmup + args.steps):
        cuda.selective_scan(op, u, delta, A, Bm, Cm, Dv, z, out=out, workspace=ws)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_case": args.case, "launches_per_call": 3 if ws_bytes else 1,
                      "calls": args.warmup + args.steps}))


def run_gemm_case(args):
    """Profiling helper: warmup + steps calls of gemm_tf32x3 on one shape, nothing timed."""
    import torch

    from mamba_onnx import cuda

    M, N, K = (int(v) for v in args.gemm_case.split(":"))
    device = torch.device("cuda", 0)
    g = torch.Generator(device=device).manual_seed(SEED)
    a = cuda.split_tf32(torch.randn(M, K, device=device, generator=g))
    b = cuda.split_tf32(torch.randn(N, K, device=device, generator=g))
    c = torch.empty(M, N, device=device)
    for _ in range(args.warmup + args.steps):
        cuda.gemm_tf32x3(a, b, c)
    torch.cuda.synchronize()
    print(json.dumps({"gemm_case": args.gemm_case, "calls": args.warmup + args.steps}))


B64_BATCH, B64_SEQLEN, B64_SEED = 64, 4096, 3
B64_WORKLOAD = (f"SelectiveScanFused fp32, total batch {B64_BATCH} x d_inner {DIM} x seqlen "
                f"{B64_SEQLEN}, d_state {NSTATE}, sharded by batch across the GPUs; the output "
                f"gathered to rank 0 by NCCL (timed separately)")


def run_scan_b64(args):
    """Strong scaling of the scan over a fixed batch of 64 (one shard per rank)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            from oracle import oracle

            cpu = reference_sample(oracle.host_threads(), 3)
            print(json.dumps({"impl": "reference", "metric": METRIC, "value": cpu["value"],
                              "unit": UNIT, "n_gpus": args.gpus, "cpu_baseline": cpu,
                              "config": {"workload": B64_WORKLOAD,
                                         "step": "one reference plugin call on 8x5120x2048 "
                                                 "(one GPU's shard at 8 GPUs)"},
                              "e2e": {"value": cpu["value"], "unit": UNIT,
                                      "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return
    import torch
    import torch.distributed as dist

    from mamba_onnx import cuda
    from mamba_onnx.distributed import gather_output, shard_plan

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    plan = shard_plan(B64_BATCH, DIM, world, rank)
    if plan.axis != 0 or len(set(plan.sizes)) != 1:
        raise SystemExit("scan-b64 needs a GPU count that divides 64")
    nb, D, L = plan.length, DIM, B64_SEQLEN
    # every batch entry from its own seed, so a rank's shard equals the slice
    # of the single-GPU tensors
    u = torch.empty(nb, D, L, device=device)
    z, delta = torch.empty_like(u), torch.empty_like(u)
    Bm = torch.empty(nb, L, NSTATE, device=device)
    Cm = torch.empty_like(Bm)
    g = torch.Generator(device=device)
    g.manual_seed(B64_SEED)
    lo, hi = float(np.log(1e-3)), float(np.log(1e-1))
    dt = torch.exp(torch.rand(D, device=device, generator=g) * (hi - lo) + lo)
    bias = torch.log(torch.expm1(dt))[:, None]
    for i in range(nb):
        g.manual_seed(B64_SEED * 1000003 + plan.start + i)
        for t in (u[i], z[i], delta[i], Bm[i], Cm[i]):
            t.normal_(generator=g)
        delta[i].mul_(0.5).add_(bias)
    A = -torch.arange(1, NSTATE + 1, device=device, dtype=torch.float32).repeat(D, 1)
    Dv = torch.ones(D, device=device)
    out = torch.empty_like(u)
    ws = torch.empty(max(1, cuda.workspace_size(OP, nb, D, L)), dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        cuda.selective_scan(OP, u, delta, A, Bm, Cm, Dv, z, out=out, workspace=ws, stream=stream)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(device) as clocks:
        ms = max_over_ranks(timed(step, args.steps))
    gather_ms = None
    if world > 1:
        full = torch.empty(B64_BATCH, D, L, device=device) if rank == 0 else None
        gather_output(out, plan, out=full)  # warm-up
        torch.cuda.synchronize()
        dist.barrier()
        gather_ms = max_over_ranks(timed(lambda: gather_output(out, plan, out=full), 5))
        del full
    if rank == 0:
        hbm_peak, peak_kind = measured_peaks()
        algo = algorithmic_bytes(nb, D, L)
        achieved = algo / (ms * 1e-3) / 1e9
        total = B64_BATCH * D * L * NSTATE
        line = {
            "metric": METRIC, "value": total / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": B64_WORKLOAD, "op": OP, "global_batch": B64_BATCH,
                       "batch_per_gpu": nb, "d_inner": D, "seqlen": L, "d_state": NSTATE,
                       "parallelism": f"batch-sharded x{world}; NCCL gather of out to rank 0",
                       "l2": f"inputs {algo / 1e9:.2f} GB per GPU, larger than L2; no flush"},
            "gather_ms": gather_ms,
            "gather_bytes_to_rank0": (B64_BATCH - nb) * D * L * 4 if world > 1 else 0,
            "compute_plus_gather_ms": ms + (gather_ms or 0.0),
            "e2e": {"value": None, "note": "host-buffer end to end is measured on the default "
                                           "workload (this one holds up to 21.5 GB per GPU)"},
            "gpu_launches": (3 if ws.numel() > 1 else 1) * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "per": "rank's op call",
                         "peak_source": f"{peak_kind} hbm_gbs"},
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


DECODE_BATCH, DECODE_PROMPT = 1, 1024
DECODE_WORKLOAD = ("Mamba-130m single-token decode (24 blocks, fp32), batch 1 per GPU after a "
                   "1024-token prefill; each step one CUDA-graph replay of the step (every scan "
                   "is SelectiveScanFusedExact with seqlen 1 through h0/h_last)")


def run_decode(args):
    """Decode tokens/s: one step = one token for each sequence of the batch."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference has no decode path (its op always starts from a zero "
                              "state); see --workload mamba130m for the reference forward"}))
        return
    import torch
    import torch.distributed as dist

    from mamba_onnx import model as M
    from mamba_onnx.model import MambaLM, mamba_130m

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    B = DECODE_BATCH
    model = MambaLM(mamba_130m()).init_random(0).to(device)
    g = torch.Generator(device=device).manual_seed(SEED + rank)
    prompt = torch.randint(0, model.cfg.vocab_size, (B, DECODE_PROMPT), device=device, generator=g)
    _, state = model.prefill(prompt)
    ids, logits, g_state, graph = model.capture_step(B)
    model.copy_state(g_state, state)
    ids.copy_(prompt[:, -1])
    stream = torch.cuda.current_stream(device)

    def timed(fn, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(device) as clocks:
        ms = max_over_ranks(timed(graph.replay, args.steps))

    # end to end: next token ids from pinned host memory, greedy token back
    host_ids = ids.cpu().pin_memory()
    host_next = torch.empty(B, dtype=torch.int64).pin_memory()

    def e2e_step():
        ids.copy_(host_ids, non_blocking=True)
        graph.replay()
        host_next.copy_(torch.argmax(logits, dim=-1), non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(timed(e2e_step, max(3, args.e2e_steps * 10)))
    if rank == 0:
        print(json.dumps({
            "metric": "Mamba-130m decode tokens/s", "value": world * B / (ms * 1e-3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (random init with Mamba's initialisation)",
            "config": {"workload": DECODE_WORKLOAD, "batch_per_gpu": B, "global_batch": B * world,
                       "prompt": DECODE_PROMPT,
                       "parallelism": f"replica per GPU x{world}, no collective"},
            "e2e": {"value": world * B / (e2e_ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": host_ids.numel() * 8,
                    "d2h_bytes_per_step": host_next.numel() * 8, "ms_per_step": e2e_ms,
                    "path": "pinned token ids -> graph replay -> argmax token to host"},
            # this package's kernels per token: the persistent decoding kernel
            # (every block and the LM head in one launch), or per block
            # RMSNorm + in_proj, the convolution step, x_proj, the fused
            # dt_proj + scan step and out_proj + residual, then the final
            # RMSNorm + LM head
            "gpu_launches": (1 if M.DECODE == "persistent" else model.cfg.n_layer * 5 + 1)
                            * args.steps,
            "decode": M.DECODE,
            "clocks": clocks.summary()}), flush=True)
    if world > 1:
        del graph
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

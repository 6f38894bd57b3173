"""Benchmark of the quantized matmul path on B200.

Workload (one "step"): quantization::matmul of fp32 activations x [8192 x 8192]
~N(0,1) with INT8 per-column weights W [K=8192 x N=65536] (~N(0,0.02) before
quantization), i.e. the prefill INT8 GEMM M=8192 K=8192 N=65536.  The step is
the full path: per-row activation quantizer + tcgen05 GEMM with the fused
fp32 rescale epilogue.  On N GPUs the weight is column-sharded (N/p columns
per GPU, no data exchange inside the step) and each GPU then all-gathers the
output shards over NCCL so every GPU holds the full [M, N] result.

Metric: int8 TOPS (2*M*N*K ops / step time).  x is 256 MiB, W 512 MiB and y
2 GiB, all larger than the 126 MB L2, so no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the ZYRON reference's own CPU implementation
(oracle/_ref/libzyron_ref.so, compiled from the reference's sources; falls
back to the C restatement in oracle/ when that library is absent) on a
bounded row sample of the same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import hashlib
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_ROWS, K_DIM, N_COLS = 8192, 8192, 65536
WORKLOAD = "prefill_int8_gemm_M8192_K8192_N65536"
METRIC = "int8 qmatmul throughput (quantization::matmul, prefill INT8 GEMM)"
UNIT = "TOPS"
# The reference parallelises over rows only (one std::thread per row chunk),
# so a bounded CPU sample is one row per host thread: every thread busy, one
# row (K x N = 537 M scalar MACs) each, about 2 s per step.


def ops(m, n, k):
    return 2.0 * m * n * k


# --------------------------------------------------------------------------
# clocks sampled during the timed region (NVML reads only)
# --------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: no clock record
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv is not None:
            self.t.join()

    def summary(self):
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


# --------------------------------------------------------------------------
# reference CPU timing (oracle/_ref or the oracle port) -- checker side only
# --------------------------------------------------------------------------
# Inputs shared by both arms: numpy PCG64 streams that either arm can
# regenerate on the host.  x is one stream (any prefix of rows is the same);
# W is stored transposed per 256-column block, block b drawn from
# PCG64(seed).jumped(b), so a rank generates only its own column shard.
X_SEED, W_SEED, W_BLOCK = 0, 1, 256
OUTPUT_CHECK_ROWS = 16
INPUTS_NOTE = ("x: numpy PCG64(0) standard normal fp32 [M, K]; W: N(0, 0.02) fp32, 256-column blocks of W^T from "
               "PCG64(1).jumped(block); the same values in both arms")


def synthetic_x(M, K):
    """x ~ N(0, 1), fp32 [M, K]."""
    return np.random.Generator(np.random.PCG64(X_SEED)).standard_normal((M, K), dtype=np.float32)


def synthetic_wT(K, N, c0, n):
    """Columns c0 .. c0+n of W ~ N(0, 0.02) as W^T, fp32 [n, K]."""
    out = np.empty((n, K), dtype=np.float32)
    for b in range(c0 // W_BLOCK, (c0 + n + W_BLOCK - 1) // W_BLOCK):
        blk = np.random.Generator(np.random.PCG64(W_SEED).jumped(b)).standard_normal((W_BLOCK, K),
                                                                                   dtype=np.float32)
        lo, hi = max(c0, b * W_BLOCK), min(c0 + n, (b + 1) * W_BLOCK)
        out[lo - c0:hi - c0] = blk[lo - b * W_BLOCK:hi - b * W_BLOCK]
    out *= np.float32(0.02)
    return out


def output_digest(y_rows):
    """sha256 of the first output rows' fp32 bytes: both arms print it for the
    same inputs, and bit-exact results give the same digest."""
    return hashlib.sha256(np.ascontiguousarray(y_rows, dtype=np.float32).tobytes()).hexdigest()


def reference_cpu_timer(zyq: bytes, x_rows: np.ndarray):
    """Returns (time_one_call, threads, kind) for quantization::matmul of
    x_rows against the .zyq weight, on the host cores."""
    from oracle import oracle as O

    if O.ref_available():
        R = O.RefMatrix.load_bytes(zyq)
        threads = O.ref_set_threads(os.cpu_count() or 1)

        def call():
            t0 = time.perf_counter()
            R.matmul(x_rows)
            return time.perf_counter() - t0

        return call, threads, "reference", R
    # oracle port (single thread)
    K = int(np.frombuffer(zyq[12:20], dtype="<u8")[0])
    N = int(np.frombuffer(zyq[20:28], dtype="<u8")[0])
    scales = np.frombuffer(zyq[36:36 + 4 * N], dtype=np.float32)
    payload = np.frombuffer(zyq[36 + 4 * N + 8:], dtype=np.uint8)

    def call():
        t0 = time.perf_counter()
        O.matmul(x_rows, 1, payload, scales, N)
        return time.perf_counter() - t0

    return call, 1, "port", None


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    K, N = K_DIM, N_COLS
    from oracle import oracle as O

    # the inputs of our arm: the same x rows and W (quantized by the reference)
    x = synthetic_x(max(64, OUTPUT_CHECK_ROWS), K)
    w = np.ascontiguousarray(synthetic_wT(K, N, 0, N).T)
    if O.ref_available():
        zyq = O.RefMatrix.quantize(w, O.INT8).save_bytes()
    else:
        pay, sc = O.quantize_weights(w, O.INT8)
        zyq = O.zyq_bytes(1, K, N, sc, pay)
    del w
    threads = O.ref_set_threads(os.cpu_count() or 1) if O.ref_available() else 1
    rows = max(1, min(64, threads))
    call, threads, kind, keep = reference_cpu_timer(zyq, x[:rows])
    for _ in range(args.warmup):
        call()
    times = [call() for _ in range(args.steps)]
    t = sum(times) / len(times)
    value = ops(rows, N, K) / t / 1e12
    # untimed: the first output rows, for the digest our arm prints too
    if keep is not None:
        y_chk = keep.matmul(x[:OUTPUT_CHECK_ROWS])
    else:
        pay, sc = np.frombuffer(zyq[36 + 4 * N + 8:], dtype=np.uint8), np.frombuffer(zyq[36:36 + 4 * N], np.float32)
        y_chk = O.matmul(x[:OUTPUT_CHECK_ROWS], 1, pay, sc, N)[3]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "M": M_ROWS, "K": K, "N": N, "weight": "int8 per-column",
                   "sample_rows_per_step": rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{rows} of {M_ROWS} rows x K={K} x N={N} per step, "
                                   f"ZYRON quantization::matmul on {threads} host threads "
                                   f"(os.cpu_count()={os.cpu_count()})"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "inputs": INPUTS_NOTE,
        "output_check": {"rows": OUTPUT_CHECK_ROWS, "sha256": output_digest(y_chk)},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import zyron_b200 as zb
    from zyron_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)

    M, K, N = args.shape
    assert N % world == 0
    n_loc = N // world
    c0 = rank * n_loc

    # Inputs generated on the host from the streams the reference arm uses
    # too: x is the same on every rank, each rank quantizes its own column
    # shard of W on the device.
    x = torch.from_numpy(synthetic_x(M, K)).to(dev)
    w_f32 = torch.from_numpy(synthetic_wT(K, N, c0, n_loc)).to(dev).t().contiguous()
    int4 = args.weight_type == "int4"
    W = zb.quantize(w_f32, zb.Type.Int4 if int4 else zb.Type.Int8)
    del w_f32
    torch.cuda.empty_cache()
    y = torch.empty((M, n_loc), dtype=torch.float32, device=dev)
    ws_bytes = L.zq_matmul_workspace_bytes(W.handle, M)
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=dev)
    ws_ptr = (ws.data_ptr() + 255) & ~255
    peer_out = None
    if world > 1:
        # Every rank ends a step with the full [M, N] output: the matmul
        # epilogue stores each finished tile into all ranks' outputs over
        # NVLink (zq_matmul_multi); a one-element all-reduce then marks the
        # step complete on every rank.
        from zyron_b200.sharded import PeerOutputs, sharded_matmul_gathered

        peer_out = PeerOutputs(M, N, dev)

    result = [y]

    def step():
        if world == 1:
            _lib.check(L.zq_matmul(W.handle, C.c_void_p(x.data_ptr()), M, None, C.c_void_p(y.data_ptr()),
                                   C.c_void_p(ws_ptr), ws_bytes, sp))
            return
        result[0] = sharded_matmul_gathered(x, W, peer_out, workspace=(ws_ptr, ws_bytes), stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()

    sampler = ClockSampler(local_rank)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    ms = e0.elapsed_time(e1) / args.steps
    # the first output rows of the last step (the full gathered rows at N > 1)
    digest = output_digest(result[0][:OUTPUT_CHECK_ROWS].cpu().numpy())

    # GEMM kernel alone (activation codes precomputed), same stream: the
    # dominant kernel's average launch duration for the roofline.
    Kp = L.zq_weight_padded_k(W.handle)
    codes = torch.empty((M, Kp), dtype=torch.int8, device=dev)
    rs = torch.empty((M,), dtype=torch.float32, device=dev)
    _lib.check(L.zq_quantize_rows(C.c_void_p(x.data_ptr()), M, K, C.c_void_p(codes.data_ptr()), Kp,
                                  C.c_void_p(rs.data_ptr()), sp))

    def gemm_only():
        _lib.check(L.zq_matmul_codes(W.handle, C.c_void_p(codes.data_ptr()), C.c_void_p(rs.data_ptr()), M, None,
                                     C.c_void_p(y.data_ptr()), C.c_void_p(ws_ptr), ws_bytes, sp))

    def quant_only():
        _lib.check(L.zq_quantize_rows(C.c_void_p(x.data_ptr()), M, K, C.c_void_p(codes.data_ptr()), Kp,
                                      C.c_void_p(rs.data_ptr()), sp))

    def time_loop(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / n

    reps = max(args.steps, 10)
    gemm_ms = time_loop(gemm_only, reps)
    quant_ms = time_loop(quant_only, reps)
    code = zb.device_error(stream)

    # End to end through the public host entry point (zq_matmul_host):
    # pinned host x in, host y out, H2D + compute + D2H inside every step.
    x_h = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
    x_h.copy_(x.cpu())
    y_h = torch.empty((M, n_loc), dtype=torch.float32, pin_memory=True)

    def e2e_step():
        _lib.check(L.zq_matmul_host(W.handle, C.c_void_p(x_h.data_ptr()), M, None, C.c_void_p(y_h.data_ptr()), sp))

    e2e_ms = float("nan")
    if not args.no_e2e:
        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(max(1, min(args.warmup, 3))):
            e2e_step()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        b.record(stream)
        barrier()
        e2e_ms = a.elapsed_time(b) / e2e_steps

    # max over ranks
    if world > 1:
        t = torch.tensor([ms, gemm_ms, quant_ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, gemm_ms, quant_ms, e2e_ms = t.tolist()

    if rank != 0:
        return

    total_ops = ops(M, N, K)
    value = total_ops / (ms * 1e-3) / 1e12
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    if "bf16_tflops" in peaks:
        int8_peak = 2.0 * float(peaks["bf16_tflops"])
        peak_src = "measured: 2 x MEASURED_PEAKS bf16_tflops (burst); int8 dense MMA rate is twice bf16 on sm_100"
    else:
        int8_peak = 2.0 * 1590.0
        peak_src = "fallback: 2 x 1590 TFLOP/s bf16 (earlier pool measurement)"
    gemm_tops = ops(M, n_loc, K) / (gemm_ms * 1e-3) / 1e12
    # the committed DRAM figure is for the 1-GPU INT8 headline workload only
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemm_traffic.json")
    headline = (M, K, n_loc) == (M_ROWS, K_DIM, N_COLS) and args.weight_type == "int8"
    if headline and os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch_full_workload")

    cpu = None
    if world == 1 and not args.skip_cpu_baseline:
        try:
            zyq = W.save_bytes()
            from oracle import oracle as O

            rows = max(1, min(64, O.ref_set_threads(os.cpu_count() or 1) if O.ref_available() else 1))
            xs = x[:rows].cpu().numpy()
            call, threads, kind, _keep = reference_cpu_timer(zyq, xs)
            call()  # warm
            tc = min(call() for _ in range(2))
            cpu = {"value": ops(rows, N, K) / tc / 1e12, "unit": UNIT, "cores": threads,
                   "kind": kind,
                   "sample": f"{rows} of {M} rows x K={K} x N={N} (same weights), best of 2, "
                             f"ZYRON quantization::matmul on {threads} threads (os.cpu_count()={os.cpu_count()})"}
        except Exception as exc:  # report, never fail the bench on the baseline leg
            cpu = {"value": None, "unit": UNIT, "cores": None, "kind": None, "sample": f"failed: {exc}"}

    line = {
        "metric": METRIC.replace("int8", "int4").replace("INT8", "INT4") if int4 else METRIC, "value": value,
        "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD if (M, K, N) == (M_ROWS, K_DIM, N_COLS) and not int4
                   else f"prefill_{args.weight_type}_gemm_M{M}_K{K}_N{N}",
                   "M": M, "K": K, "N": N, "weight": f"{args.weight_type} per-column (device quantize)",
                   "x": "N(0,1) fp32", "w": "N(0,0.02) fp32 before quantization",
                   "parallelism": f"column-sharded x{world}" + (
                       " + all-gather of outputs fused into the matmul epilogue (NVLink peer stores)"
                       if world > 1 else ""),
                   "l2": "inputs larger than L2 (x 256 MiB, W 512 MiB, y 2 GiB); no flush"},
        "gpu_launches": (2 * args.steps),
        "clocks": sampler.summary(),
        "roofline": {"bound": "tensor",
                     "kernel": "gemm_i8_pair_kernel (tcgen05.mma.cta_group::2.kind::i8, 2-SM 256x256 tiles"
                               + (", packed INT4 tiles unpacked in shared memory)" if int4 else ")"),
                     "achieved": gemm_tops, "peak": int8_peak, "unit": UNIT, "frac": gemm_tops / int8_peak,
                     "peak_source": peak_src, "traffic": traffic,
                     "ms_per_launch": gemm_ms, "ops_per_launch": ops(M, n_loc, K)},
        "kernels_ms": {"quantize_rows": quant_ms, "gemm_i8": gemm_ms},
        "e2e": {"value": total_ops / (e2e_ms * 1e-3) / 1e12 / (1 if world == 1 else 1), "unit": UNIT,
                "ms_per_step": e2e_ms, "h2d_bytes_per_step": M * K * 4, "d2h_bytes_per_step": M * n_loc * 4,
                "api": "zq_matmul_host (pinned host x -> host y), per rank on its column shard"},
        "cpu_baseline": cpu,
        "device_error": code,
        "inputs": INPUTS_NOTE,
        "output_check": {"rows": OUTPUT_CHECK_ROWS, "sha256": digest,
                         "note": "sha256 of the first output rows; the reference arm prints the digest of its "
                                 "own result for the same inputs (INT8 weights)"},
    }
    if world > 1:
        line["e2e"]["value"] = ops(M, N, K) / (e2e_ms * 1e-3) / 1e12
        # What the gathered step is made of: every rank's GEMM on its own
        # column shard, and the (world-1)/world of the fp32 output each GPU
        # receives over NVLink from the peers' epilogues.
        recv = (world - 1) / world * M * N * 4
        link_gbs = 770.0  # measured peer-copy bandwidth per direction on this pool
        line["multi_gpu"] = {
            "gemm_only_ms_per_rank": gemm_ms, "quantize_ms_per_rank": quant_ms,
            "gemm_only_tops_per_rank": gemm_tops, "gemm_only_tops_all_ranks": ops(M, N, K) / (gemm_ms * 1e-3) / 1e12,
            "gather_ms_beyond_compute": max(ms - gemm_ms - quant_ms, 0.0),
            "nvlink_bytes_received_per_gpu": recv, "nvlink_gbs_received_per_gpu": recv / (ms * 1e-3) / 1e9,
            "link_floor_ms": recv / (link_gbs * 1e9) * 1e3, "frac_of_link_floor": recv / (link_gbs * 1e9) / (ms * 1e-3),
            "link_floor_basis": "770 GB/s per direction per GPU (measured peer copy)",
            "barriers_per_step": 2}
    if world == 1 and not args.no_secondary:
        line["secondary"] = secondary_block(args)
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# secondary workloads (not the default line): decode GEMV and LM decode
# --------------------------------------------------------------------------
def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured: MEASURED_PEAKS hbm_gbs"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback: 6.65 TB/s (earlier pool measurement)"


def decode_cases(args, kinds=(("default", 0),), min_region_s=0.25):
    """Decode GEMV M in {1, 8}, K=4096, N=11008, INT8 and INT4 weights
    ~N(0,0.02), x ~N(0,1).  For each case and decode kernel: the matmul kernel
    alone on precomputed codes (zq_matmul_codes) and the whole zq_matmul call.
    Weight copies rotate so the streamed bytes exceed 2 x L2; launches are
    replayed from a CUDA graph (device back to back), for at least
    `min_region_s` per measurement, with the SM clocks sampled meanwhile."""
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda:0")
    K, N = 4096, 11008
    peak, peak_src = hbm_peak()
    s = torch.cuda.Stream()
    cases = {}
    launches = 0
    for qt in (1, 2):
        payload = K * N if qt == 1 else K * N // 2
        copies = max(3, int(2 * 126e6 / payload) + 2)
        g = torch.Generator(device=dev)
        g.manual_seed(2 + qt)
        Ws = []
        for _ in range(copies):
            w = torch.randn((K, N), generator=g, device=dev).mul_(0.02)
            Ws.append(zb.quantize(w, zb.Type(qt)))
            del w
        torch.cuda.empty_cache()
        Kp = L.zq_weight_padded_k(Ws[0].handle)
        for M in (1, 8):
            x = torch.randn((M, K), generator=g, device=dev)
            q = torch.empty((M, Kp), dtype=torch.int8, device=dev)
            rs = torch.empty(M, device=dev)
            y = torch.empty((M, N), device=dev)
            wsb = L.zq_matmul_workspace_bytes(Ws[0].handle, M)
            ws = torch.empty(wsb + 256, dtype=torch.uint8, device=dev)
            wp = (ws.data_ptr() + 255) & ~255
            res = {}
            with torch.cuda.stream(s):
                sp = C.c_void_p(s.cuda_stream)
                _lib.check(L.zq_quantize_rows(C.c_void_p(x.data_ptr()), M, K, C.c_void_p(q.data_ptr()), Kp,
                                              C.c_void_p(rs.data_ptr()), sp))

                def kernel_only(i):
                    _lib.check(L.zq_matmul_codes(Ws[i % copies].handle, C.c_void_p(q.data_ptr()),
                                                 C.c_void_p(rs.data_ptr()), M, None, C.c_void_p(y.data_ptr()),
                                                 C.c_void_p(wp), wsb, sp))

                def full_call(i):
                    _lib.check(L.zq_matmul(Ws[i % copies].handle, C.c_void_p(x.data_ptr()), M, None,
                                           C.c_void_p(y.data_ptr()), C.c_void_p(wp), wsb, sp))

                for kname, kind in kinds:
                    for W in Ws:
                        W.set_decode_kernel(kind)
                    res[kname] = {}
                    for name, fn in (("kernel", kernel_only), ("matmul_call", full_call)):
                        for i in range(copies):
                            fn(i)
                        s.synchronize()
                        reps = 10 * copies
                        graph = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(graph, stream=s):
                            for i in range(reps):
                                fn(i)
                        for _ in range(args.warmup):
                            graph.replay()
                        s.synchronize()
                        # replays for about min_region_s of device time
                        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
                        a.record(s)
                        graph.replay()
                        b.record(s)
                        s.synchronize()
                        n_rep = max(args.steps, int(min_region_s * 1e3 / max(a.elapsed_time(b), 1e-3)) + 1)
                        sampler = ClockSampler(0)
                        with sampler:
                            a.record(s)
                            for _ in range(n_rep):
                                graph.replay()
                            b.record(s)
                            s.synchronize()
                        launches += n_rep * reps * (1 if name == "kernel" else 2)
                        us = a.elapsed_time(b) / (n_rep * reps) * 1e3
                        byts = payload + 4 * N + M * Kp + 4 * M * N
                        res[kname][name] = {"us": us, "GBs": byts / us / 1e3, "frac_of_hbm": byts / us / 1e3 / peak,
                                            "bytes": byts, "clocks": sampler.summary()}
                        del graph
                for W in Ws:
                    W.set_decode_kernel(0)
            cases[f"{'int8' if qt == 1 else 'int4'}_M{M}"] = res
        del Ws
        torch.cuda.empty_cache()
    return cases, peak, peak_src, launches


def run_gemv_workload(args):
    """Decode GEMV M in {1, 8}, K=4096, N=11008 through both decode kernels
    (see decode_cases), the host entry point, and the reference's CPU
    matmul."""
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda:0")
    K, N = 4096, 11008
    if args.once:
        # profiling aid: three eager zq_matmul calls per case and decode
        # kernel, in the order int8 M=1, M=8, int4 M=1, M=8, each with the
        # tensor-core kernel first, then the dp4a GEMV; no timing
        g = torch.Generator(device=dev)
        g.manual_seed(2)
        for qt in (1, 2):
            W = zb.quantize(torch.randn((K, N), generator=g, device=dev).mul_(0.02), zb.Type(qt))
            for M in (1, 8):
                x = torch.randn((M, K), generator=g, device=dev)
                for kind in (1, 2):
                    W.set_decode_kernel(kind)
                    for _ in range(3):
                        y = zb.matmul(x, W)
                W.set_decode_kernel(0)
        torch.cuda.synchronize()
        print(json.dumps({"workload": "decode_gemv_K4096_N11008", "once": True, "checksum": float(y.abs().sum())}))
        return
    cases, peak, peak_src, launches = decode_cases(args, kinds=(("tensor_core", 1), ("cuda_core", 2)),
                                                   min_region_s=0.05)
    # end to end through the host entry point (M=1, INT8): pinned host x in, host y out
    W0 = zb.quantize(torch.randn((K, N), device=dev).mul_(0.02), zb.Type.Int8)
    xh = torch.randn((1, K)).pin_memory()
    yh = torch.empty((1, N)).pin_memory()
    for _ in range(args.warmup):
        _lib.check(L.zq_matmul_host(W0.handle, C.c_void_p(xh.data_ptr()), 1, None, C.c_void_p(yh.data_ptr()), None))
    t0 = time.perf_counter()
    for _ in range(args.steps * 10):
        _lib.check(L.zq_matmul_host(W0.handle, C.c_void_p(xh.data_ptr()), 1, None, C.c_void_p(yh.data_ptr()), None))
    e2e_us = (time.perf_counter() - t0) / (args.steps * 10) * 1e6
    cpu = None
    if not args.skip_cpu_baseline:
        zyq = W0.save_bytes()
        call, threads, kind, _keep = reference_cpu_timer(zyq, xh.numpy())
        call()
        tc = min(call() for _ in range(3))
        cpu = {"value": (K * N) / tc / 1e9, "unit": "GB/s", "cores": 1, "kind": kind,
               "sample": f"M=1 x K={K} x N={N} INT8, best of 3 (the reference splits work over rows, so M=1 runs on "
                         f"one thread whatever the thread count)"}
    # the default dispatch (ZQ_DECODE_AUTO) runs the dp4a GEMV for M <= 4 and
    # the tensor-core kernel above; the headline is the kernel it picks
    for key, c in cases.items():
        c["default"] = "cuda_core" if key.endswith("_M1") else "tensor_core"
    head = cases["int8_M1"]["cuda_core"]["kernel"]
    line = {"metric": "decode GEMV weight-stream bandwidth (quantization::matmul, M=1 INT8)", "value": head["GBs"],
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["us"] / 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "decode_gemv_K4096_N11008", "M": [1, 8], "types": ["int8", "int4"],
                       "l2": "weights rotate over enough copies to stream > 2 x L2 per pass"},
            "gpu_launches": launches, "clocks": head["clocks"],
            "roofline": {"bound": "hbm", "kernel": "gemv_kernel<int8, M=1> (dp4a, warp per column)",
                         "achieved": head["GBs"], "peak": peak,
                         "unit": "GB/s", "frac": head["frac_of_hbm"], "peak_source": peak_src,
                         "bytes_per_launch": head["bytes"]},
            "cases": cases,
            "e2e": {"value": (K * N) / e2e_us / 1e3, "unit": "GB/s", "us_per_step": e2e_us,
                    "h2d_bytes_per_step": 4 * K, "d2h_bytes_per_step": 4 * N, "api": "zq_matmul_host"},
            "cpu_baseline": cpu}
    print(json.dumps(line), flush=True)


def run_kernels_workload(args):
    """The HBM-bound helper kernels of the path at sizes larger than L2, each
    timed with CUDA events: the activation quantizer (x 8192 x 8192 fp32),
    the device weight quantizer (W 8192 x 16384 fp32 -> INT8 / INT4 panel) and
    dequantize() of the INT8 panel.  GB/s are algorithmic bytes (every input read once, every output
    written once)."""
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda:0")
    peak, peak_src = hbm_peak()
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    M, K, N = 8192, 8192, 16384

    def timed(fn, reps=None):
        reps = reps or max(args.steps, 1)
        for _ in range(max(args.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps * 1e3  # us

    cases = {}

    def add(name, us, nbytes):
        cases[name] = {"us": us, "GBs": nbytes / us / 1e3, "frac_of_hbm": nbytes / us / 1e3 / peak}

    x = torch.randn((M, K), generator=g, device=dev)
    q = torch.empty((M, K), dtype=torch.int8, device=dev)
    rs = torch.empty((M,), device=dev)
    add("quantize_rows (activations 8192 x 8192)",
        timed(lambda: _lib.check(L.zq_quantize_rows(C.c_void_p(x.data_ptr()), M, K, C.c_void_p(q.data_ptr()), K,
                                                    C.c_void_p(rs.data_ptr()), None))),
        4 * M * K + M * K + 4 * M)
    w = torch.randn((K, N), generator=g, device=dev).mul_(0.02)
    holder = {}

    def quant8():
        holder["w8"] = zb.quantize(w, zb.Type.Int8)

    add("zq_weight_quantize INT8 call (8192 x 16384; allocates the panel)", timed(quant8, 3),
        2 * 4 * K * N + K * N + 4 * N)

    def quant4():
        holder["w4"] = zb.quantize(w, zb.Type.Int4)

    add("zq_weight_quantize INT4 call (8192 x 16384; allocates the panel)", timed(quant4, 3), 2 * 4 * K * N + K * N // 2 + 4 * N)
    W8, W4 = holder["w8"], holder["w4"]
    out = torch.empty((K, N), device=dev)

    def deq():
        _lib.check(L.zq_dequantize(W8.handle, C.c_void_p(out.data_ptr()), None))

    add("dequantize INT8 (8192 x 16384 -> fp32)", timed(deq), K * N + 4 * N + 4 * K * N)
    del out
    torch.cuda.empty_cache()
    # INT4 against INT8 weights in the prefill GEMM on the same shape: the
    # INT4 kernel streams the packed panel and unpacks it in shared memory
    gm = 8192
    xg = torch.randn((gm, K), generator=g, device=dev)
    yg = torch.empty((gm, N), device=dev)
    Kp = L.zq_weight_padded_k(W8.handle)
    codes = torch.empty((gm, Kp), dtype=torch.int8, device=dev)
    rsg = torch.empty((gm,), device=dev)
    _lib.check(L.zq_quantize_rows(C.c_void_p(xg.data_ptr()), gm, K, C.c_void_p(codes.data_ptr()), Kp,
                                  C.c_void_p(rsg.data_ptr()), None))
    gemm = {}
    for name, W in (("int8", W8), ("int4", W4)):
        wsb = L.zq_matmul_workspace_bytes(W.handle, gm)
        ws = torch.empty(wsb + 256, dtype=torch.uint8, device=dev)
        wp = (ws.data_ptr() + 255) & ~255
        us = timed(lambda: _lib.check(L.zq_matmul_codes(W.handle, C.c_void_p(codes.data_ptr()),
                                                        C.c_void_p(rsg.data_ptr()), gm, None,
                                                        C.c_void_p(yg.data_ptr()), C.c_void_p(wp), wsb, None)), 10)
        gemm[name] = {"us": us, "TOPS": 2.0 * gm * N * K / us / 1e6}
    gemm["int4_over_int8"] = gemm["int4"]["TOPS"] / gemm["int8"]["TOPS"]
    line = {"metric": "helper kernels of the path (HBM-bound)", "value": cases["quantize_rows (activations 8192 x 8192)"]["GBs"],
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32->int8", "data": "synthetic",
            "config": {"workload": "helper_kernels", "x": [M, K], "W": [K, N]},
            "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s", "peak_source": peak_src}, "cases": cases,
            "gemm_M8192_K8192_N16384": gemm}
    print(json.dumps(line), flush=True)


def run_small_workload(args):
    """The two small matmul configurations: INT8 M=64 K=512 N=512 and INT4
    M=128 K=2048 N=2048, x ~N(0,1), w ~N(0,0.02).  Calls are replayed from a
    CUDA graph; the reference's CPU matmul is timed on the same inputs."""
    import numpy as np
    import torch

    import zyron_b200 as zb
    from zyron_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda:0")
    s = torch.cuda.Stream()
    out = {}
    for name, qt, M, K, N, seed in (("int8_M64_K512_N512", 1, 64, 512, 512, 0),
                                    ("int4_M128_K2048_N2048", 2, 128, 2048, 2048, 1)):
        rng = np.random.default_rng(seed)
        x = rng.standard_normal((M, K)).astype(np.float32)
        w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        W = zb.quantize(torch.from_numpy(w).to(dev), zb.Type(qt))
        xd = torch.from_numpy(x).to(dev)
        y = torch.empty((M, N), device=dev)
        if args.once:
            # profiling aid: three eager zq_matmul calls, no timing
            for _ in range(3):
                y = zb.matmul(xd, W)
            torch.cuda.synchronize()
            out[name] = {"checksum": float(y.abs().sum())}
            continue
        wsb = L.zq_matmul_workspace_bytes(W.handle, M)
        ws = torch.empty(wsb + 256, dtype=torch.uint8, device=dev)
        wp = (ws.data_ptr() + 255) & ~255
        with torch.cuda.stream(s):
            sp = C.c_void_p(s.cuda_stream)

            def call():
                _lib.check(L.zq_matmul(W.handle, C.c_void_p(xd.data_ptr()), M, None, C.c_void_p(y.data_ptr()),
                                       C.c_void_p(wp), wsb, sp))

            for _ in range(3):
                call()
            s.synchronize()
            reps = 50
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                for _ in range(reps):
                    call()
            for _ in range(args.warmup):
                graph.replay()
            s.synchronize()
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record(s)
            for _ in range(args.steps):
                graph.replay()
            b.record(s)
            s.synchronize()
            us = a.elapsed_time(b) / (args.steps * reps) * 1e3
        res = {"us_per_call": us, "TOPS": 2.0 * M * N * K / us / 1e6}
        if not args.skip_cpu_baseline:
            zyq = W.save_bytes()
            call_ref, threads, kind, _keep = reference_cpu_timer(zyq, x)
            call_ref()
            tc = min(call_ref() for _ in range(3))
            res["cpu_baseline"] = {"us_per_call": tc * 1e6, "TOPS": 2.0 * M * N * K / tc / 1e12, "cores": threads,
                                   "kind": kind}
        out[name] = res
    if args.once:
        print(json.dumps({"workload": "small_matmuls", "once": True, "cases": out}), flush=True)
        return
    line = {"metric": "small quantized matmul configurations (quantization::matmul)",
            "value": out["int4_M128_K2048_N2048"]["TOPS"], "unit": "TOPS", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic", "config": {"workload": "small_matmuls"}, "cases": out}
    print(json.dumps(line), flush=True)


QLM_WORKLOAD = "qlm_decode_d768_L12_H12_KV4_F3072_V16384_prompt64_new512"


def qlm_measure(args, cpu_baseline=True):
    """QuantizedLanguageModel decode: d_model 768, 12 layers, 12 heads, 4 KV
    heads, GELU FFN 3072, tied vocab 16384, INT8, batch 1, 64-token uniform
    prompt, 512 greedy tokens.  The model is LanguageModel(config, 0)
    quantized to INT8, initialised by the library with the reference's
    generator and seeds (the image equals the reference's byte for byte).
    Per-token time = (generate(512) - generate(1)) / 511, best of 3, with the
    SM clocks sampled meanwhile."""
    import tempfile

    import torch

    from zyron_b200.qlm import Config, GenerationConfig, QuantizedLanguageModel, init_zyqmodel

    cfg = Config(vocab_size=16384, hidden_size=768, num_layers=12, num_heads=12, num_kv_heads=4,
                 intermediate_size=3072, max_sequence_length=576)
    img = init_zyqmodel(cfg, seed=0)
    lm = QuantizedLanguageModel.load_bytes(img)
    prompt = np.random.default_rng(0).integers(0, 16384, 64).tolist()
    lm.generate(prompt, GenerationConfig(max_new_tokens=512, top_k=1))  # builds the graphs
    s = torch.cuda.Stream()

    def timed(n):
        best = None
        for _ in range(max(1, args.warmup // 3)):
            lm.generate(prompt, GenerationConfig(max_new_tokens=n, top_k=1), stream=s)
        for _ in range(3):
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record(s)
            lm.generate(prompt, GenerationConfig(max_new_tokens=n, top_k=1), stream=s)
            b.record(s)
            s.synchronize()
            t = a.elapsed_time(b) / 1e3
            best = t if best is None else min(best, t)
        return best

    sampler = ClockSampler(0)
    with sampler:
        t1 = timed(1)
        t512 = timed(512)
    per_tok = (t512 - t1) / 511
    weight_bytes = 12 * (768 * (768 + 256 + 256 + 768 + 3072) + 3072 * 768) + 768 * 16384
    peak, peak_src = hbm_peak()
    cpu = None
    if cpu_baseline:
        from oracle import oracle as O

        if O.ref_available():
            with tempfile.TemporaryDirectory() as d:
                path = os.path.join(d, "m.zyqmodel")
                with open(path, "wb") as f:
                    f.write(img)
                h = C.c_void_p()
                if O.ref().ref_qlm_load(path.encode(), C.byref(h)) == 0:
                    threads = O.ref_set_threads(os.cpu_count() or 1)
                    ids = np.asarray(prompt, dtype=np.uint64)
                    out = np.zeros(ids.size + 4, dtype=np.uint64)
                    n = C.c_size_t()
                    t0 = time.perf_counter()
                    O.ref().ref_qlm_generate_greedy(h, C.c_void_p(ids.ctypes.data), ids.size, 2,
                                                    C.c_void_p(out.ctypes.data), C.byref(n))
                    tc = (time.perf_counter() - t0) / 2
                    O.ref().ref_qlm_free(h)
                    cpu = {"value": 1.0 / tc, "unit": "tok/s", "cores": threads, "kind": "reference",
                           "sample": "2 greedy tokens after the 64-token prompt (the reference recomputes the whole "
                                     "prefix for every token; later tokens cost more)"}
    return {"tok_s": 1.0 / per_tok, "ms_per_token": per_tok * 1e3, "generate_512_tok_s": 512.0 / t512,
            "prefill_ms": t1 * 1e3, "clocks": sampler.summary(),
            "roofline": {"bound": "hbm", "achieved": weight_bytes / per_tok / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": weight_bytes / per_tok / 1e9 / peak, "peak_source": peak_src,
                         "note": "weight bytes per token / time per token; the 88 MB of weights fit in L2"},
            "launches_per_token": 2 + 5 * 12, "cpu_baseline": cpu}


def run_qlm_workload(args):
    """The LM decode workload on its own line (see qlm_measure)."""
    from zyron_b200.qlm import Config, GenerationConfig, QuantizedLanguageModel, init_zyqmodel

    if args.once:
        # profiling aid: one 4-token generation after the 64-token prompt
        cfg = Config(vocab_size=16384, hidden_size=768, num_layers=12, num_heads=12, num_kv_heads=4,
                     intermediate_size=3072, max_sequence_length=576)
        lm = QuantizedLanguageModel.load_bytes(init_zyqmodel(cfg, seed=0))
        prompt = np.random.default_rng(0).integers(0, 16384, 64).tolist()
        toks = lm.generate(prompt, GenerationConfig(max_new_tokens=4, top_k=1))
        print(json.dumps({"workload": "qlm_decode_d768_L12", "once": True, "tokens": list(map(int, toks))}))
        return
    r = qlm_measure(args, cpu_baseline=not args.skip_cpu_baseline)
    line = {"metric": "quantized-LM decode tok/s (QuantizedLanguageModel::generate, greedy)", "value": r["tok_s"],
            "unit": "tok/s", "n_gpus": 1, "steps": 512, "warmup": args.warmup, "ms_per_step": r["ms_per_token"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": QLM_WORKLOAD,
                       "weights": "LanguageModel(config, 0) quantized to INT8 (the reference's init)"},
            "clocks": r["clocks"], "roofline": r["roofline"],
            "e2e": {"value": r["generate_512_tok_s"], "unit": "tok/s",
                    "note": "whole generate call incl. 64-token prefill", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "prefill_ms": r["prefill_ms"], "cpu_baseline": r["cpu_baseline"]}
    print(json.dumps(line), flush=True)


def secondary_block(args):
    """The decode GEMV (weight GB/s) and LM decode (tok/s) figures of the
    metric, measured after the headline in the same process, each with its
    own clock record."""
    out = {}
    try:
        cases, peak, peak_src, launches = decode_cases(args)
        out["decode_gemv_K4096_N11008"] = {
            "unit": "GB/s", "peak": peak, "peak_source": peak_src,
            "dispatch": "zq_matmul default: dp4a GEMV with the quantizer fused for M <= 4, tcgen05 decode kernel "
                        "for 5-16 rows",
            "bytes": "payload + 4N scales + M*Kp codes + 4MN outputs per launch; weights rotate over > 2 x L2",
            "cases": {k: v["default"] for k, v in cases.items()}, "gpu_launches": launches}
    except Exception as exc:  # report, never lose the headline
        out["decode_gemv_K4096_N11008"] = {"error": repr(exc)}
    try:
        out[QLM_WORKLOAD] = qlm_measure(args, cpu_baseline=not args.skip_cpu_baseline)
    except Exception as exc:
        out[QLM_WORKLOAD] = {"error": repr(exc)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["prefill", "gemv", "small", "qlm", "kernels"], default="prefill",
                    help="prefill (default line), gemv (decode GEMV), small (64x512x512 INT8 and "
                         "128x2048x2048 INT4) or qlm (LM decode)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg (profiling runs)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the decode GEMV and LM decode figures after the headline (profiling runs)")
    ap.add_argument("--once", action="store_true",
                    help="gemv / small / qlm workloads: a few untimed calls of the kernels (for ncu captures)")
    ap.add_argument("--weight-type", choices=["int8", "int4"], default="int8",
                    help="prefill workload: weight type (the headline configuration is INT8)")
    ap.add_argument("--shape", type=lambda v: tuple(int(t) for t in v.split(",")),
                    default=(M_ROWS, K_DIM, N_COLS), help="M,K,N override for small profiling cases")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world == 1 and args.gpus > 1:
        raise SystemExit("--gpus > 1 must be launched with torch.distributed.run (one process per GPU)")

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.workload == "gemv":
        run_gemv_workload(args)
        return
    if args.workload == "qlm":
        run_qlm_workload(args)
        return
    if args.workload == "kernels":
        run_kernels_workload(args)
        return
    if args.workload == "small":
        run_small_workload(args)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

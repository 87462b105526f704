#!/usr/bin/env python3
"""Benchmark of the Q8_0 / Q4_0 GGML_OP_MUL_MAT hot path on B200.

Workload (a "step" = one pass over it):
    fc1  Q4_0 weight [4096 out x 1024 in],  x = N(0,1)        [4096 tokens x 1024]
    fc2  Q4_0 weight [1024 out x 4096 in],  x = GELU(N(0,1))  [4096 tokens x 4096]
    kv   Q8_0 weight [1024 out x 1024 in],  x = N(0,1)        [1374 tokens x 1024]
each = activation quantize (fp32 -> Q8_0) + tcgen05 int8 block GEMM, weights
~ N(0, 0.02) quantized once (ggml reference quantizer) and packed once on the
device (the buffer-type upload), as a model's weights are.
Metric: effective TOPS = sum 2*M*N*K / device time (int8 MACs count 2 ops).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b2q|reference]

N > 1 runs under torchrun, one rank per GPU, each an independent replica of the
workload (the path has no exchange step): "scaling": "weak", value = all ranks'
ops / max-over-ranks device time.  --impl reference times the CPU
implementation of the same path (the oracle's vectorised port of ggml's CPU
mul_mat; ggml itself is absent from the reference checkout) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "sam-3d-objects-ggml_b200"))
sys.path.insert(0, os.path.join(REPO, "oracle"))

import numpy as np  # noqa: E402

METRIC = "Q8_0/Q4_0 mul_mat effective TOPS"
UNIT = "TOPS"
INT8_SPEC_TOPS = 4500.0  # B200 dense int8 tensor peak (public spec)
WORKLOAD = [
    # name, wtype, M (tokens), N (out), K (in), gelu input
    ("fc1_q4_0", 2, 4096, 4096, 1024, False),
    ("fc2_q4_0", 2, 4096, 1024, 4096, True),
    ("kv_q8_0", 8, 1374, 1024, 1024, False),
]
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


# What the parity of this path is pinned to (ggml v0.21.0 itself is absent from
# the reference checkout, so the arithmetic is checked against an oracle that
# restates it; these are the oracle's external anchors and its gaps).
PARITY_PIN = {
    "pinned": ["Q8_0 / Q4_0 weight quantizers and the reference activation quantizer: gguf-py 0.19.0 bytes",
               "Q4_0 weight quantizer: the reference's own cpp_ggml/scripts/gguf_schema.py quantize_q4_0, byte "
               "for byte (edge blocks, fc1 / fc2 shapes)",
               "int32 block dots: numpy from the gguf-py bytes", "Q4_K dequantizer: gguf-py",
               "reference regression test criteria (matmul_backend_test.cpp) through the C ABI from C++"],
    "unpinned": ["B2Q_ACT_X86 activation rounding (127/amax, ties to even), the variant this line uses",
                 "ggml's x86 fp32 lane order of the block dot", "the ggml_gelu fp16 table",
                 "the rounding of ggml_norm's variance"],
    "reason": "no ggml source or binary in the reference checkout or this machine (empty submodule)",
}


def ops_of(M, N, K):
    return 2.0 * M * N * K


def max_over_ranks(ms: float, dist=None, device="cpu") -> float:
    """The job's time is its slowest rank's: MAX all-reduce of a per-rank time
    (identity on one process).  NCCL needs a device tensor, gloo a host one."""
    import torch
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if dist is not None and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def config_dict():
    return {
        "workload": "configs[1]: fc1 Q4_0 4096x1024->4096, fc2 Q4_0 4096x4096->1024 (GELU in), "
                    "kv Q8_0 1374x1024->1024; activation quantize + int8 block GEMM each",
        "weights": "N(0,0.02) -> ggml reference quantizer, packed once on device",
        "activations": "N(0,1) fp32 (fc2: GELU-tanh of N(0,1)), seed 1234",
        "act_quantizer": "ggml-cpu x86 from_float semantics (B2Q_ACT_X86)",
        "l2": "flushed between steps (256 MiB write, outside the per-step events)",
        "parallelism": "replicas (one independent workload per GPU)",
    }


def synth_blocks(wtype: int, w: np.ndarray | None, n: int, k: int, seed: int = 0) -> np.ndarray:
    """Synthetic GGUF weight rows (uint8 [n, row bytes]).  Q8_0 / Q4_0: the
    fp32 matrix w quantized blockwise here in numpy with ggml's reference
    quantizers (Q8_0: d = amax/127, inverse 1/d, round half away from zero;
    Q4_0: the first signed element of largest magnitude sets d = max/-8,
    q = min(15, trunc(x*id + 8.5)), as cpp_ggml/scripts/gguf_schema.py:27-52
    restates it); Q4_K: seeded random blocks with finite fp16 d / dmin, since
    any such bytes are a valid weight."""
    if wtype == 12:  # Q4_K
        rng = np.random.default_rng(seed)
        nb = k // 256
        b = rng.integers(0, 256, size=(n, nb, 144), dtype=np.uint8)
        b[:, :, 0:2] = np.abs(rng.standard_normal((n, nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(n, nb, 2)
        b[:, :, 2:4] = np.abs(rng.standard_normal((n, nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(n, nb, 2)
        return b.reshape(n, nb * 144)
    blk = w.reshape(n, k // 32, 32).astype(np.float32)
    one = np.float32(1)
    if wtype == 8:  # Q8_0
        d = np.abs(blk).max(-1) / np.float32(127)
        inv = np.where(d > 0, one / np.where(d > 0, d, one), np.float32(0)).astype(np.float32)
        v = (blk * inv[..., None]).astype(np.float32)
        # roundf: half away from zero (|v| + 0.5 is exact in float64)
        q = (np.sign(v) * np.floor(np.abs(v).astype(np.float64) + 0.5)).astype(np.int8)
        out = np.empty((n, k // 32, 34), np.uint8)
        out[:, :, :2] = d.astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
        out[:, :, 2:] = q.view(np.uint8)
        return out.reshape(n, -1)
    idx = np.abs(blk).argmax(-1)
    mx = np.take_along_axis(blk, idx[..., None], -1)[..., 0]
    d = mx / np.float32(-8)
    inv = np.where(d != 0, one / np.where(d != 0, d, one), np.float32(0)).astype(np.float32)
    v = (blk * inv[..., None]).astype(np.float32) + np.float32(8.5)
    q = np.minimum(15, np.trunc(v)).astype(np.uint8)
    out = np.empty((n, k // 32, 18), np.uint8)
    out[:, :, :2] = d.astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
    out[:, :, 2:] = q[:, :, :16] | (q[:, :, 16:] << 4)
    return out.reshape(n, -1)


def make_inputs(seed=1234):
    from_gelu = None
    rng = np.random.default_rng(seed)
    out = []
    for name, wtype, M, N, K, gelu in WORKLOAD:
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        if gelu:
            x64 = x.astype(np.float64)
            x = (0.5 * x64 * (1.0 + np.tanh(0.7978845608028654 * (x64 + 0.044715 * x64 ** 3)))).astype(np.float32)
        out.append((name, wtype, M, N, K, synth_blocks(wtype, w, N, K), x))
    del from_gelu
    return out


# --------------------------------------------------------------------- clocks
# The sampler runs in a child process: a thread of this process gets the GIL
# too rarely while the timed loop enqueues its launches (one sample in a 44 ms
# region was seen).  The child prints "<wall time> <SM MHz> <reason bits>"
# every period; the parent keeps the samples inside its timed window.
_SAMPLER_CODE = r"""
import sys, time, pynvml
pynvml.nvmlInit()
uuid, period = sys.argv[1], float(sys.argv[2])
try:
    h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
except Exception:
    h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[3]))
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
while True:
    try:
        print(time.time(), pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
              pynvml.nvmlDeviceGetCurrentClocksEventReasons(h), flush=True)
    except Exception:
        pass
    time.sleep(period)
"""


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML (in a child process)
    during the `with` block."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons, self.max_mhz, self.error = [], 0, None, ""
        self._proc = None
        try:
            import subprocess
            import torch
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
            self._proc = subprocess.Popen([sys.executable, "-c", _SAMPLER_CODE, uuid, str(period_s),
                                           str(device_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                          text=True)
            first = self._proc.stdout.readline().split()  # the child is sampling once it prints this
            if len(first) != 2 or first[0] != "max":
                raise RuntimeError("sampler did not start")
            self.max_mhz = int(first[1])
        except Exception as e:  # noqa: BLE001
            self.error = f"nvml unavailable: {e}"
            if self._proc is not None:
                self._proc.kill()
            self._proc = None

    def __enter__(self):
        self._t0 = time.time()
        return self

    def __exit__(self, *a):
        t1 = time.time()
        if self._proc is None:
            return
        time.sleep(0.01)  # the child's samples up to t1 are written
        self._proc.kill()
        out, _ = self._proc.communicate()
        for line in out.splitlines():
            f = line.split()
            if len(f) == 3 and self._t0 <= float(f[0]) <= t1:
                self.samples.append(int(f[1]))
                self.reasons |= int(f[2])

    def summary(self):
        if self.max_mhz is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": self.error}
        rs = [v for k, v in self.REASONS.items() if self.reasons & k and k != 0x1]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": rs, "samples": len(self.samples),
                "source": "nvml in a child process, sampled every 2 ms during the timed region"}


# -------------------------------------------------------------------- GPU arm
def run_gpu(args, rank, world, local_rank):
    import torch
    import b2q

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    stream = torch.cuda.current_stream()
    inputs = make_inputs()
    if args.only:
        inputs = [t for t in inputs if t[0] == args.only]
        if not inputs:
            raise SystemExit(f"--only: no workload entry named {args.only}")
    gemms = []
    for name, wtype, M, N, K, wq, x in inputs:
        w_raw = torch.from_numpy(wq).to(dev)
        packed = b2q.weight_pack(wtype, w_raw, K)
        x_host = torch.from_numpy(x).pin_memory()
        x_dev = x_host.to(dev)
        act = b2q._empty_aligned(b2q.act_prepared_size(M, K), dev)
        y_dev = torch.empty((M, N), dtype=torch.float32, device=dev)
        y_host = torch.empty((M, N), dtype=torch.float32).pin_memory()
        ws = b2q.workspace(M, N, K, True, dev)
        gemms.append(dict(name=name, wtype=wtype, M=M, N=N, K=K, packed=packed, x_host=x_host,
                          x_dev=x_dev, act=act, y_dev=y_dev, y_host=y_host, ws=ws))
        del w_raw
    flush = torch.empty(L2_FLUSH_BYTES if not args.only else 1, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()

    def step(evs=None):
        for i, g in enumerate(gemms):
            b2q.act_prepare(g["x_dev"], out=g["act"], stream=stream)
            if evs is not None:
                evs[2 * i + 1].record(stream)
            b2q.mul_mat_prepared(g["packed"], g["N"], g["K"], g["act"], g["M"], out=g["y_dev"],
                                 stream=stream)
            if evs is not None:
                evs[2 * i + 2].record(stream)

    launches_per_step = 2 * len(gemms)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()

    nev = 1 + 2 * len(gemms)
    all_evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for s in range(args.steps):
            flush.zero_()
            all_evs[s][0].record(stream)
            step(all_evs[s])
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    status = b2q.device_status(clear=True)
    if status:
        raise RuntimeError(f"device status 0x{status:x}")

    # Hot-L2 figures (reported beside the flushed ones, not used for `value`):
    # each GEMM re-run back to back on its already-quantized input.
    hot_us = []
    for g in gemms:
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for _ in range(3):
            b2q.mul_mat_prepared(g["packed"], g["N"], g["K"], g["act"], g["M"], out=g["y_dev"], stream=stream)
        ev[0].record(stream)
        for _ in range(20):
            b2q.mul_mat_prepared(g["packed"], g["N"], g["K"], g["act"], g["M"], out=g["y_dev"], stream=stream)
        ev[1].record(stream)
        torch.cuda.synchronize()
        hot_us.append(ev[0].elapsed_time(ev[1]) / 20 * 1e3)

    step_ms = [e[0].elapsed_time(e[-1]) for e in all_evs]
    quant_ms = [[e[2 * i].elapsed_time(e[2 * i + 1]) for e in all_evs] for i in range(len(gemms))]
    gemm_ms = [[e[2 * i + 1].elapsed_time(e[2 * i + 2]) for e in all_evs] for i in range(len(gemms))]
    total_ms = sum(step_ms)
    step_ops = sum(ops_of(g["M"], g["N"], g["K"]) for g in gemms)

    max_total_ms = max_over_ranks(total_ms, dist, dev)
    value = world * step_ops * args.steps / (max_total_ms * 1e-3) / 1e12

    # ---- end to end through the public C ABI, host buffers, copies inside the timing
    e2e_steps = 0 if args.no_e2e else max(1, min(args.steps, 20))
    h2d = sum(g["x_host"].numel() * 4 for g in gemms)
    d2h = sum(g["y_host"].numel() * 4 for g in gemms)

    # Copies run on their own streams so that the upload of one GEMM's input,
    # another GEMM's compute and the download of a third GEMM's output overlap
    # (the H2D and D2H copy engines and the SMs are separate).  The device
    # input and output buffers are doubled and alternate by step, so a step's
    # uploads need not wait for the previous step's GEMMs; events keep each
    # buffer's reuse ordered.
    h2d_stream, d2h_stream = torch.cuda.Stream(), torch.cuda.Stream()
    ev = lambda: torch.cuda.Event()  # noqa: E731
    for g in gemms:
        g["x_devs"] = [g["x_dev"], torch.empty_like(g["x_dev"])]
        g["y_devs"] = [g["y_dev"], torch.empty_like(g["y_dev"])]
        g["uploaded"] = ev()
        g["computed"], g["downloaded"] = [ev(), ev()], [ev(), ev()]
        for b in range(2):
            g["computed"][b].record(stream)
            g["downloaded"][b].record(stream)
    e2e_parity = [0]

    def e2e_step():
        b = e2e_parity[0]
        e2e_parity[0] ^= 1
        for g in gemms:
            h2d_stream.wait_event(g["computed"][b])  # the GEMM two steps back has read this x buffer
            with torch.cuda.stream(h2d_stream):
                g["x_devs"][b].copy_(g["x_host"], non_blocking=True)
            g["uploaded"].record(h2d_stream)
            stream.wait_event(g["uploaded"])
            stream.wait_event(g["downloaded"][b])  # this y buffer's previous result has left
            b2q.mul_mat_packed(g["packed"], g["N"], g["K"], g["x_devs"][b], out=g["y_devs"][b], ws=g["ws"],
                               stream=stream)
            g["computed"][b].record(stream)
            d2h_stream.wait_event(g["computed"][b])
            with torch.cuda.stream(d2h_stream):
                g["y_host"].copy_(g["y_devs"][b], non_blocking=True)
            g["downloaded"][b].record(d2h_stream)

    for _ in range(min(args.warmup, 3) if e2e_steps else 0):
        e2e_step()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    h2d_stream.wait_event(e0)
    for _ in range(e2e_steps):
        e2e_step()
    for g in gemms:  # the timed region ends when every download has landed
        for b in range(2):
            stream.wait_event(g["downloaded"][b])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    e2e_max_ms = max_over_ranks(e2e_ms, dist, dev)
    e2e_value = (world * step_ops * e2e_steps / (e2e_max_ms * 1e-3) / 1e12) if e2e_steps else None

    gemm_total_ms = sum(sum(v) for v in gemm_ms)
    gemm_ops = step_ops * args.steps
    achieved = gemm_ops / (gemm_total_ms * 1e-3) / 1e12
    breakdown = []
    for i, g in enumerate(gemms):
        gm = statistics.median(gemm_ms[i])
        qm = statistics.median(quant_ms[i])
        o = ops_of(g["M"], g["N"], g["K"])
        breakdown.append({"name": g["name"], "M": g["M"], "N": g["N"], "K": g["K"],
                          "gemm_us_median": round(gm * 1e3, 2), "quantize_us_median": round(qm * 1e3, 2),
                          "gemm_tops": round(o / (gm * 1e-3) / 1e12, 1),
                          "gemm_frac_of_int8_spec": round(o / (gm * 1e-3) / 1e12 / INT8_SPEC_TOPS, 4),
                          "gemm_us_hot_l2": round(hot_us[i], 2)})
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    traffic = None
    try:
        traffic = json.load(open(os.path.join(REPO, "profiles", "gemm_traffic.json")))
    except Exception:
        pass
    # Denominator: the public B200 dense int8 tensor peak.  MEASURED_PEAKS.json
    # has no int8 entry; a back-to-back tcgen05 kind::i8 loop on this pool's
    # B200s ran at 4583 TOPS sustained (profiles/int8_peak.json), within 2% of it.
    peak, peak_source = INT8_SPEC_TOPS, "B200 dense int8 spec (MEASURED_PEAKS.json has no int8 entry)"
    roofline = {
        "bound": "tensor", "kernel": "gemm_tc_kernel (tcgen05 kind::i8 + per-block scale epilogue)",
        "achieved": round(achieved, 1), "peak": peak, "unit": "TOPS",
        "frac": round(achieved / peak, 4),
        "peak_source": peak_source,
        "frac_of_int8_spec": round(achieved / INT8_SPEC_TOPS, 4),
        "traffic": traffic.get("bytes_per_step") if isinstance(traffic, dict) else None,
    }
    if peaks.get("bf16_tflops"):
        roofline["frac_of_2x_measured_bf16"] = round(achieved / (2 * peaks["bf16_tflops"]), 4)

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(max_total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8 (int8 x int8 -> int32 per block, fp32 scale epilogue)",
        "data": "synthetic", "config": config_dict(), "roofline": roofline, "parity_pin": PARITY_PIN,
        "e2e": {"value": round(e2e_value, 2) if e2e_value else None, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "path": "b2q_mul_mat_packed per GEMM; pinned host x -> device -> pinned host y, uploads and "
                        "downloads on their own streams, overlapped with other GEMMs' compute; device x / y "
                        "buffers doubled and alternated by step"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(), "breakdown": breakdown,
    }
    if not args.only and not args.no_mlp:
        result["mlp_branch"] = mlp_branch(b2q, gemms, flush, stream, dev)
        result["q4_k"] = q4_k_side(b2q, gemms, flush, stream, dev)
        result["ss_block"] = ss_block_side(b2q, flush, stream, dev,
                                           cpu=(rank == 0 and world == 1 and not args.no_cpu_baseline))
        result["ss_step"] = ss_step_side(b2q, stream, dev, cpu=(rank == 0 and world == 1 and not args.no_cpu_baseline))
        result["slat_linears"] = slat_side(b2q, stream, dev)
        result["f16"] = f16_side(b2q, flush, stream, dev, peaks)
        result["attention"] = attention_side(b2q, stream, dev, peaks)
        result["slat_sparse"] = slat_sparse_side(b2q, flush, stream, dev, peaks)
    if not args.only and not args.no_colpar:
        result["colpar"] = colpar_side(args, rank, world, dev, dist)
    if args.only:
        result["config"]["workload"] = f"single GEMM {args.only} (profiling case)"
        result["config"]["l2"] = "not flushed (profiling case)"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(inputs, budget_s=args.cpu_budget)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return result


# ------------------------------------------------------ fused MLP (next row)
def mlp_branch(b2q, gemms, flush, stream, dev, iters=10):
    """The SS block's feed-forward branch on the fc1 and fc2 weights of the
    workload (cpp_ggml/src/ss_flow_graph.cpp:376-387):
        x += gate * fc2(gelu(fc1(modulate(norm(x), scale, shift)) + b1)) + b2
    from the fp32 residual stream x to its in-place update, run as ggml runs
    it (one kernel per op) and fused (pre-norm + quantize, fc1 + GELU +
    quantize, fc2 + gate + residual: 3 launches).  Reported beside the headline
    (its ops are not part of `value`); L2 flushed before each iteration, CUDA
    events on the launching stream."""
    import torch
    by = {g["name"]: g for g in gemms}
    f1, f2 = by.get("fc1_q4_0"), by.get("fc2_q4_0")
    if f1 is None or f2 is None or f1["N"] != f2["K"] or f1["M"] != f2["M"] or f1["K"] != f2["N"]:
        return None
    M, H, C = f1["M"], f1["N"], f2["N"]
    g = torch.Generator(device=dev).manual_seed(7)
    b1 = torch.randn(H, device=dev, generator=g)
    b2 = torch.randn(C, device=dev, generator=g)
    sc = torch.randn(C, device=dev, generator=g) * 0.1
    sh = torch.randn(C, device=dev, generator=g) * 0.1
    gate = torch.randn(C, device=dev, generator=g) * 0.1
    x0 = torch.randn(M, C, device=dev, generator=g)
    x = x0.clone()
    hn = torch.empty((M, C), dtype=torch.float32, device=dev)
    hid = torch.empty((M, H), dtype=torch.float32, device=dev)
    act1 = b2q._empty_aligned(b2q.act_prepared_size(M, C), dev)
    act2 = b2q._empty_aligned(b2q.act_prepared_size(M, H), dev)
    y = torch.empty((M, C), dtype=torch.float32, device=dev)

    def unfused():
        b2q.norm_modulate(x, 1e-6, sc, sh, out=hn, stream=stream)
        b2q.act_prepare(hn, out=act1, stream=stream)
        b2q.mul_mat_prepared(f1["packed"], H, C, act1, M, bias=b1, out=hid, stream=stream)
        b2q.gelu(hid, out=hid, stream=stream)
        b2q.act_prepare(hid, out=act2, stream=stream)
        b2q.mul_mat_prepared(f2["packed"], C, H, act2, M, bias=b2, out=y, stream=stream)
        torch.mul(y, gate, out=y)
        torch.add(x, y, out=x)

    def fused():
        b2q.norm_modulate_q8(x, 1e-6, sc, sh, out=act1, stream=stream)
        b2q.mul_mat_prepared_gelu_q8(f1["packed"], H, C, act1, M, bias=b1, out=act2, stream=stream)
        b2q.mul_mat_prepared_gate_residual(f2["packed"], C, H, act2, M, x, bias=b2, gate=gate, out=x,
                                           stream=stream)

    def timed(fn):
        for _ in range(3):
            fn()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(iters)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            fn()
            e1.record(stream)
        torch.cuda.synchronize()
        return statistics.median(e0.elapsed_time(e1) * 1e3 for e0, e1 in evs)

    u, f = timed(unfused), timed(fused)

    def hot(fn, n=20):  # one kernel back to back, hot L2
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return round(e0.elapsed_time(e1) / n * 1e3, 2)

    kernels = {
        "norm_modulate_q8": hot(lambda: b2q.norm_modulate_q8(x0, 1e-6, sc, sh, out=act1, stream=stream)),
        "fc1_bias": hot(lambda: b2q.mul_mat_prepared(f1["packed"], H, C, act1, M, bias=b1, out=hid,
                                                     stream=stream)),
        "fc1_bias_gelu_q8": hot(lambda: b2q.mul_mat_prepared_gelu_q8(f1["packed"], H, C, act1, M, bias=b1,
                                                                     out=act2, stream=stream)),
        "gelu": hot(lambda: b2q.gelu(hid, out=hid, stream=stream)),
        "act_prepare_hidden": hot(lambda: b2q.act_prepare(hid, out=act2, stream=stream)),
        "fc2_bias": hot(lambda: b2q.mul_mat_prepared(f2["packed"], C, H, act2, M, bias=b2, out=y,
                                                     stream=stream)),
        "fc2_bias_gate_residual": hot(lambda: b2q.mul_mat_prepared_gate_residual(
            f2["packed"], C, H, act2, M, x0, bias=b2, gate=gate, out=y, stream=stream)),
    }
    # one update of the same stream, both ways, compared bit for bit
    x.copy_(x0)
    unfused()
    xu = x.clone()
    x.copy_(x0)
    fused()
    torch.cuda.synchronize()
    return {"shape": {"M": M, "C": C, "hidden": H, "weights": "Q4_0"},
            "unfused_us": round(u, 2), "fused_us": round(f, 2), "speedup": round(u / f, 3),
            "launches": {"unfused": 8, "fused": 3},
            "kernels_us_hot_l2": kernels,
            "fused_equals_unfused": bool(torch.equal(x, xu)),
            "path": "unfused: norm_modulate -> act_prepare -> mul_mat_prepared(+b1) -> gelu -> act_prepare -> "
                    "mul_mat_prepared(+b2) -> mul(gate) -> add(residual); fused: norm_modulate_q8 -> "
                    "mul_mat_prepared_gelu_q8(+b1) -> mul_mat_prepared_gate_residual(+b2, gate, in place)"}


# ------------------------------------------------ Q4_K (the shipped format)
def q4_k_side(b2q, gemms, flush, stream, dev, iters=10):
    """The fc1 and fc2 GEMMs of the workload with Q4_K weights (the 4-bit
    format the reference ships, cpp_ggml/models/MODEL_CARD.md:54-74) against
    Q8_K activations: GEMM and quantize time with the L2 flushed, beside the
    headline (not part of `value`).  Weights are seeded random valid Q4_K
    blocks."""
    import torch
    out = []
    for g in gemms:
        if g["name"] not in ("fc1_q4_0", "fc2_q4_0") or g["K"] % 256:
            continue
        M, N, K = g["M"], g["N"], g["K"]
        packed = b2q.weight_pack(b2q.TYPE_Q4_K, torch.from_numpy(synth_blocks(12, None, N, K, seed=N + K)).to(dev), K)
        act = b2q.act_prepare(g["x_dev"], b2q.ACT_Q8_K, stream=stream)
        y = torch.empty((M, N), dtype=torch.float32, device=dev)

        def timed(fn):
            for _ in range(3):
                fn()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(iters)]
            for e0, e1 in evs:
                flush.zero_()
                e0.record(stream)
                fn()
                e1.record(stream)
            torch.cuda.synchronize()
            return statistics.median(e0.elapsed_time(e1) * 1e3 for e0, e1 in evs)

        gu = timed(lambda: b2q.mul_mat_prepared_q4_k(packed, N, K, act, M, out=y, stream=stream))
        qu = timed(lambda: b2q.act_prepare(g["x_dev"], b2q.ACT_Q8_K, out=act, stream=stream))
        o = ops_of(M, N, K)
        out.append({"name": g["name"].replace("q4_0", "q4_k"), "M": M, "N": N, "K": K,
                    "gemm_us_median": round(gu, 2), "quantize_us_median": round(qu, 2),
                    "gemm_tops": round(o / (gu * 1e-6) / 1e12, 1)})
    return {"kernel": "gemm_q4k_kernel (three int8 planes, per-super-block fold)", "gemms": out}


# ------------------------------------------------- SS-flow DiT block step
SS_BLOCK = dict(B=2, T=4096, C=1024, H=16, n_cond=1374)  # BASELINE configs[2] and the 1374 condition tokens


def ss_block_side(b2q, flush, stream, dev, cpu=False, iters=10):
    """One SS-flow DiT block (sam-3d-objects-ggml_b200/ss_block.py) at the
    BASELINE block config: pre-norms, qkv, RMS-norm heads, attention, output
    projection with gate + residual, fused MLP; Q8_0 weights, every kernel
    libb2q's (attention: the tensor-core fp16 core).  Reported beside the headline.  With cpu=True the same block's
    CPU time is estimated from the oracle port's quantized mul_mats (all host
    threads) plus torch's CPU attention, each at full size."""
    import torch
    import ss_block
    B, T, C, H = SS_BLOCK["B"], SS_BLOCK["T"], SS_BLOCK["C"], SS_BLOCK["H"]
    rng = np.random.default_rng(99)
    weights = {name: synth_blocks(8, (rng.standard_normal(sh) * 0.02).astype(np.float32), *sh)
               for name, sh in ss_block.SsBlock.shapes(C, 4 * C).items()}
    blk = ss_block.SsBlock(dev, weights, C=C, heads=H, wtype=8, seed=5)
    gen = torch.Generator(device=dev).manual_seed(5)
    x0 = torch.randn(B * T, C, device=dev, generator=gen)
    nc = SS_BLOCK["n_cond"]
    cond = torch.randn(B * nc, C, device=dev, generator=gen)
    x = x0.clone()
    for _ in range(3):
        x.copy_(x0)
        blk.forward(x, B, T, cond, nc)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for e0, e1 in evs:
        x.copy_(x0)
        flush.zero_()
        e0.record(stream)
        blk.forward(x, B, T, cond, nc)
        e1.record(stream)
    torch.cuda.synchronize()
    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)
    M = B * T
    lin_ops = sum(ops_of(B * nc if name == "xkv" else M, n, k)
                  for name, (n, k) in ss_block.SsBlock.shapes(C, 4 * C).items())
    attn_flops = 4 * B * H * T * (T + nc) * (C // H)
    out = {"config": dict(SS_BLOCK, weights="Q8_0", mlp_ratio=4), "block_ms": round(ms, 4),
           "linear_int_ops": lin_ops, "attention_flops": attn_flops,
           "path": "libb2q: norm_modulate_q8, layer_norm_q8, act_prepare, mul_mat_prepared, qkv_heads, "
                   "rows_to_heads, mul_mat_prepared_gate_residual, mul_mat_prepared_gelu_q8; "
                   "b2q_attention_f16_q8 (self and cross attention cores on tensor cores, the to_out Q8_0 "
                   "quantize in their epilogue)",
           "not_included": "the 4-token pose group, the adaLN projection (both are in ss_step)"}
    if cpu:
        out["cpu"] = cpu_block_seconds(weights, B, T, C, H, nc)
        out["speedup_vs_cpu"] = round(out["cpu"]["seconds"] * 1e3 / ms, 1)
    return out


def cpu_block_seconds(weights, B, T, C, H, n_cond):
    """CPU time of the same block's heavy parts: the oracle port's quantized
    mul_mats (ggml CPU semantics, vectorised, all host threads) on the full
    token count, and torch's fp32 CPU attention.  Norms and elementwise steps
    are not timed (a lower bound)."""
    import torch
    import oracle as O
    thr = host_threads()
    torch.set_num_threads(thr)
    rng = np.random.default_rng(7)
    M = B * T
    t0 = time.perf_counter()
    for name, w in weights.items():
        k = 4 * C if name == "fc2" else C
        rows = B * n_cond if name == "xkv" else M
        O.mul_mat(8, w, rng.standard_normal((rows, k)).astype(np.float32), O.ACT_X86, nthreads=thr, fast=True)
    t1 = time.perf_counter()
    q = torch.randn(B, H, T, C // H)
    kc = torch.randn(B, H, n_cond, C // H)
    torch.nn.functional.scaled_dot_product_attention(q, q, q)
    torch.nn.functional.scaled_dot_product_attention(q, kc, kc)
    t2 = time.perf_counter()
    return {"seconds": round(t2 - t0, 3), "linears_s": round(t1 - t0, 3), "attention_s": round(t2 - t1, 3),
            "threads": thr, "kind": "port (linears) + torch CPU attention"}


SS_FLOW = dict(C=1024, heads=16, n_blocks=24, n_shape=4096, in_ch=8, mlp_ratio=4)


def _random_q8_rows(rng, n, k):
    """Valid Q8_0 GGUF rows of N(0, 0.02)-like magnitude (random codes, fp16 scales)."""
    nb = k // 32
    out = np.empty((n, nb, 34), np.uint8)
    out[:, :, :2] = (rng.random((n, nb), dtype=np.float32) * 2e-4 + 3e-4).astype(np.float16).view(np.uint8).reshape(
        n, nb, 2)
    out[:, :, 2:] = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int8).view(np.uint8)
    return out.reshape(n, nb * 34)


def cpu_ss_step(blocks_timed=2, cfg=SS_FLOW, n_cond=1374):
    """One SS-flow sampling step of configs[4] on the host cores, every op of the
    reference graph (cpp_ggml/src/ss_flow_graph.cpp:56-419, session.cpp:
    1199-1245) at the full token count: timestep / d embeddings, the adaLN
    projection of all blocks, the F32 input layers, per block both token groups
    (pre-norm + modulate, qkv, per-head RMS norm, self-attention including the
    pose group's attention over the shape keys, output projection with gate and
    residual, cross-attention with its affine LayerNorm and K/V projection of the
    condition tokens, MLP with GELU), the output layers and the CFG blend +
    Euler update.  Quantized linears: the oracle port of ggml's CPU mul_mat
    (AVX-512 VNNI, all host threads); attention: torch's fp32 CPU SDPA; the rest
    numpy fp32.  `blocks_timed` blocks run at full size (blocks are identical in
    work), and the step is reported both as measured pieces and as
    fixed parts + n_blocks x the measured mean block time."""
    import torch
    import oracle as O
    thr = host_threads()
    torch.set_num_threads(thr)
    C, H, T = cfg["C"], cfg["heads"], cfg["n_shape"]
    D, hid, nb, B, eps = C // H, C * cfg["mlp_ratio"], cfg["n_blocks"], 2, np.float32(1e-6)
    f32 = np.float32
    rng = np.random.default_rng(17)
    mm = lambda w, x: O.mul_mat(8, w, np.ascontiguousarray(x, f32), O.ACT_X86, nthreads=thr, fast=True)  # noqa: E731
    vec = lambda n, s=0.02: (rng.standard_normal(n) * s).astype(f32)  # noqa: E731
    silu = lambda x: (x / (f32(1) + np.exp(-x))).astype(f32)  # noqa: E731
    W = {"t0": _random_q8_rows(rng, C, 256), "t2": _random_q8_rows(rng, C, C),
         "d0": _random_q8_rows(rng, C, 256), "d2": _random_q8_rows(rng, C, C),
         "adaln": _random_q8_rows(rng, nb * 6 * C, C), "out": _random_q8_rows(rng, cfg["in_ch"], C)}
    for i in range(blocks_timed):
        for g in ("s", "p"):
            for name, (n, k) in {"qkv": (3 * C, C), "out": (C, C), "xq": (C, C), "xkv": (2 * C, C),
                                 "xout": (C, C), "fc1": (hid, C), "fc2": (C, hid)}.items():
                W[f"{i}.{g}.{name}"] = _random_q8_rows(rng, n, k)
    xs = rng.standard_normal((T, cfg["in_ch"])).astype(f32)
    cond2 = np.concatenate([rng.standard_normal((n_cond, C)).astype(f32), np.zeros((n_cond, C), f32)])
    w_in = (rng.standard_normal((C, cfg["in_ch"])) * 0.3).astype(f32)
    pe = (rng.standard_normal((T, C)) * 0.5).astype(f32)

    def heads(x, n, g=None):
        x = x.reshape(B, n, H, D)
        if g is not None:
            ms = ((x * x).astype(np.float64).sum(-1, keepdims=True) / D).astype(f32)
            x = (x * (f32(1) / np.sqrt(ms + eps))).astype(f32) * g.reshape(H, D)
        return torch.from_numpy(np.ascontiguousarray(x.transpose(0, 2, 1, 3)))

    def attend(q, k, v):
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v)
        return o.permute(0, 2, 1, 3).reshape(-1, C).numpy()

    t_start = time.perf_counter()
    half = 128
    freqs = np.exp(f32(-np.log(10000.0)) * np.arange(half, dtype=f32) / f32(half)).astype(f32)

    def embed(e, s):
        ang = (f32(s) * freqs).astype(f32)
        emb = np.concatenate([np.cos(ang), np.sin(ang)]).astype(f32)[None]
        return mm(W[f"{e}2"], silu(mm(W[f"{e}0"], emb) + vec(C))) + vec(C)

    mod = embed("t", 412.5) + embed("d", 0.0)
    six_all = (mm(W["adaln"], silu(mod)) + vec(nb * 6 * C))[0]
    hs = np.tile(((xs @ w_in.T).astype(f32) + vec(C) + pe)[None], (B, 1, 1)).reshape(B * T, C).astype(f32)
    hp = (rng.standard_normal((B * 4, C)) * 0.5).astype(f32)
    cond_rows = cond2
    t_fixed_a = time.perf_counter() - t_start
    block_s = []
    for i in range(blocks_timed):
        tb = time.perf_counter()
        six = six_all[i * 6 * C:(i + 1) * 6 * C]
        sh_msa, sc_msa, g_msa, sh_mlp, sc_mlp, g_mlp = (six[j * C:(j + 1) * C] for j in range(6))
        qkv = {}
        for g, x, n in (("s", hs, T), ("p", hp, 4)):
            y = mm(W[f"{i}.{g}.qkv"], O.norm_modulate(x, 1e-6, sc_msa, sh_msa)) + vec(3 * C)
            qkv[g] = (heads(y[:, :C], n, 1 + vec(C, 0.1)), heads(y[:, C:2 * C], n, 1 + vec(C, 0.1)),
                      heads(y[:, 2 * C:], n))
        qs, ks, vs = qkv["s"]
        qp, kp, vp = qkv["p"]
        o_s = attend(qs, ks, vs)
        o_p = attend(qp, torch.cat([kp, ks], 2), torch.cat([vp, vs], 2))
        hs = hs + (mm(W[f"{i}.s.out"], o_s) + vec(C)) * g_msa
        hp = hp + (mm(W[f"{i}.p.out"], o_p) + vec(C)) * g_msa
        new = []
        for g, x, n in (("s", hs, T), ("p", hp, 4)):
            h = O.norm_modulate(x, 1e-6) * (1 + vec(C, 0.1)) + vec(C, 0.1)
            q = heads(mm(W[f"{i}.{g}.xq"], h) + vec(C), n)
            kv = mm(W[f"{i}.{g}.xkv"], cond_rows) + vec(2 * C)
            o = attend(q, heads(kv[:, :C], n_cond), heads(kv[:, C:], n_cond))
            x = x + mm(W[f"{i}.{g}.xout"], o) + vec(C)
            h = O.gelu(mm(W[f"{i}.{g}.fc1"], O.norm_modulate(x, 1e-6, sc_mlp, sh_mlp)) + vec(hid))
            new.append((x + (mm(W[f"{i}.{g}.fc2"], h) + vec(C)) * g_mlp).astype(f32))
        hs, hp = new
        block_s.append(time.perf_counter() - tb)
    tc = time.perf_counter()
    v = mm(W["out"], O.norm_modulate(hs, 1e-6)) + vec(cfg["in_ch"])
    vc, vu = v[:T], v[T:]
    xs_new = xs + f32(0.04) * (vc + f32(7.0) * (vc - vu))
    assert np.isfinite(xs_new).all()
    t_fixed_b = time.perf_counter() - tc
    fixed = t_fixed_a + t_fixed_b
    mean_block = float(np.mean(block_s))
    return {"step_s": round(fixed + nb * mean_block, 2), "measured_s": round(fixed + sum(block_s), 2),
            "fixed_s": round(fixed, 3), "block_s": [round(b, 3) for b in block_s], "threads": thr,
            "sample": f"embeddings, adaLN of all {nb} blocks, input and output layers, CFG / Euler update, and "
                      f"{blocks_timed} of {nb} blocks (both token groups, every op) timed at the full "
                      f"2 x {T} + 2 x 4 tokens with {n_cond} condition tokens; step = fixed + {nb} x mean block",
            "kind": "port (oracle mul_mat, all host threads) + torch fp32 CPU attention + numpy fp32"}


def ss_step_side(b2q, stream, dev, cpu=False, iters=5):
    """One Euler / CFG sampling step of the full 24-block SS-flow DiT
    (sam-3d-objects-ggml_b200/ss_flow.py) at BASELINE configs[4]: 4096 shape
    tokens + 4 pose tokens, 1374 condition tokens, C 1024, Q8_0 random-init
    weights generated on the device, both CFG branches in one batched pass.
    Timed as a CUDA-graph replay (and eagerly, for the launch overhead) with
    CUDA events; the step streams ~1 GB of weights, far above L2, so no flush.
    The CPU figure is a timed run of the same step on the host cores
    (cpu_ss_step): every op, with a measured subset of the identical blocks."""
    import torch
    import ss_flow
    cfg = SS_FLOW
    C, nc = cfg["C"], SS_BLOCK["n_cond"]
    specs = ss_flow.param_specs(C, cfg["n_blocks"], cfg["n_shape"], cfg["in_ch"], cfg["mlp_ratio"])
    params = ss_flow.random_params(specs, dev, b2q.TYPE_Q8_0, seed=11)
    wbytes = sum(int(v.numel()) for n, v in params.items() if v.dtype == torch.uint8)
    flow = ss_flow.SsFlow(dev, params, **cfg)
    del params
    gen = torch.Generator(device=dev).manual_seed(13)
    smp = ss_flow.SsSampler(flow, torch.randn(nc, C, device=dev, generator=gen), nc, seed=12)
    t, dt = ss_flow.euler_schedule()[0]
    t_model = t * 1000.0

    def timed(n):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for e0, e1 in evs:
            e0.record(stream)
            smp.step(t_model, dt)
            e1.record(stream)
        torch.cuda.synchronize()
        return statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)

    smp.step(t_model, dt)
    eager_ms = timed(3)
    smp.capture(cfg=True)
    for _ in range(2):
        smp.step(t_model, dt)
    graph_ms = timed(iters)
    finite = bool(torch.isfinite(smp.xs).all().item())
    B, T, M = 2, cfg["n_shape"], 2 * cfg["n_shape"]
    hid = C * cfg["mlp_ratio"]
    per_group = lambda m: (ops_of(m, 3 * C, C) + 3 * ops_of(m, C, C) + ops_of(m, hid, C)  # noqa: E731
                           + ops_of(m, C, hid))
    lin_ops = cfg["n_blocks"] * (per_group(M) + per_group(B * 4) + 2 * ops_of(B * nc, 2 * C, C))
    out = {"config": dict(cfg, n_cond=nc, cfg_branches=B, weights="Q8_0 (random codes and fp16 scales)",
                          graph="whole step (forward + CFG blend + Euler update) in one CUDA graph"),
           "step_ms": round(graph_ms, 3), "step_ms_eager": round(eager_ms, 3),
           "weights_bytes": wbytes, "linear_int_ops": lin_ops,
           "linear_tops_effective": round(lin_ops / (graph_ms * 1e-3) / 1e12, 1),
           "state_finite": finite,
           "path": "ss_flow.SsSampler: libb2q for every quantized linear, norm, quantize, head layout and "
                   "fused epilogue and the attention cores (b2q_attention_f16_q8); torch for the K<=8 F32 input layers, "
                   "timestep cos/sin/SiLU and the Euler update"}
    if cpu:
        out["cpu"] = cpu_ss_step()
        out["speedup_vs_cpu"] = round(out["cpu"]["step_s"] * 1e3 / graph_ms, 1)
    del smp, flow
    torch.cuda.empty_cache()
    return out


F16_CASES = {"f16_fc1": (4096, 4096, 1024), "f16_fc2": (4096, 1024, 4096)}
# SS block attention cores (B = 2 CFG branches, 16 heads, D = 64): self over the
# 4096 shape tokens, cross to the 1374 condition tokens.
ATTN_CASES = {"attn_self": (2, 16, 4096, 4096), "attn_cross": (2, 16, 4096, 1374)}


def _attn_inputs(dev, B, H, Tq, Tk, seed=41):
    import torch
    gen = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, H, Tq, 64, device=dev, generator=gen).half()
    k = torch.randn(B, H, Tk, 64, device=dev, generator=gen).half()
    v = torch.randn(B, H, Tk, 64, device=dev, generator=gen).half()
    o = torch.empty(B * Tq, H * 64, device=dev, dtype=torch.half)
    return q, k, v, o


def run_attn_case(args):
    """Profiling case: --steps b2q_attention_f16 calls of one shape (after
    --warmup); prints the median CUDA-event time per call."""
    import torch
    import b2q
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H, Tq, Tk = ATTN_CASES[args.only]
    q, k, v, o = _attn_inputs(dev, B, H, Tq, Tk)
    for _ in range(args.warmup):
        b2q.attention_f16(q, k, v, out=o)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in evs:
        e0.record()
        b2q.attention_f16(q, k, v, out=o)
        e1.record()
    torch.cuda.synchronize()
    us = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3
    flops = 4.0 * B * H * Tq * Tk * 64
    return {"case": args.only, "B": B, "H": H, "Tq": Tq, "Tk": Tk, "D": 64, "us_median_hot_l2": round(us, 2),
            "tflops": round(flops / (us * 1e-6) / 1e12, 1), "launches_per_call": 1,
            "device_status": b2q.device_status(clear=True)}


def attention_side(b2q, stream, dev, peaks, iters=20):
    """The SS block's attention cores on their own: b2q_attention_f16 (tcgen05
    S = Q K^T and P V, fp16 P, fp32 softmax) against torch SDPA on the same
    fp16 tensors (cuDNN's flash kernel, the library path it replaces).  Both are
    timed as CUDA-graph replays of `iters` calls, so host launch cost (SDPA's is
    above its kernel time) is out of both numbers.  Inputs (q 16 MB, k / v up
    to 16 MB each) stay in L2 between calls, as they do in the block."""
    import torch
    out = {"kernel": "attention_f16_kernel (tcgen05 kind::f16, fp32 TMEM S and O, fp16 P in TMEM as the P V "
                     "MMA's A operand, 1/2 of the exps on the FMA pipe)",
           "timing": "CUDA-graph replay of back-to-back calls, both sides",
           "cases": []}

    def timed(fn):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / iters * 1e3
    for name, (B, H, Tq, Tk) in ATTN_CASES.items():
        q, k, v, o = _attn_inputs(dev, B, H, Tq, Tk)
        mine = timed(lambda: b2q.attention_f16(q, k, v, out=o))
        sdpa = timed(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v))
        flops = 4.0 * B * H * Tq * Tk * 64
        peak = peaks.get("bf16_tflops")
        out["cases"].append({"name": name, "B": B, "H": H, "Tq": Tq, "Tk": Tk, "D": 64, "us": round(mine, 2),
                             "tflops": round(flops / (mine * 1e-6) / 1e12, 1),
                             "frac_of_measured_bf16": round(flops / (mine * 1e-6) / 1e12 / peak, 4) if peak else None,
                             "torch_sdpa_us": round(sdpa, 2), "speedup_vs_sdpa": round(sdpa / mine, 3)})
        del q, k, v, o
    out["status"] = b2q.device_status(clear=True)
    return out


def run_f16_case(args):
    """Profiling case: --steps F16 mul_mats of one shape (after --warmup), no
    side measurements; prints the median CUDA-event time per call."""
    import torch
    import b2q
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M, N, K = F16_CASES[args.only]
    gen = torch.Generator(device=dev).manual_seed(31)
    w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).half()
    x = torch.randn(M, K, device=dev, generator=gen)
    y = torch.empty(M, N, device=dev)
    ws = b2q._empty_aligned(b2q.lib().b2q_mul_mat_workspace_bytes(b2q.TYPE_F16, M, N, K, 0), dev)
    for _ in range(args.warmup):
        b2q.mul_mat(b2q.TYPE_F16, w, x, out=y, ws=ws)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in evs:
        e0.record()
        b2q.mul_mat(b2q.TYPE_F16, w, x, out=y, ws=ws)
        e1.record()
    torch.cuda.synchronize()
    us = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3
    return {"case": args.only, "M": M, "N": N, "K": K, "us_median_hot_l2": round(us, 2),
            "tflops": round(ops_of(M, N, K) / (us * 1e-6) / 1e12, 1), "launches_per_call": 2}


def f16_side(b2q, flush, stream, dev, peaks, iters=10):
    """F16-weight mul_mat (b2q_mul_mat with B2Q_TYPE_F16: fp16 rounding of the
    activations + the tcgen05 kind::f16 GEMM) at the fc1 / fc2 shapes, L2
    flushed between runs.  Tensor-bound: reported against the measured dense
    bf16 rate (fp16 runs at the same rate on the tensor cores)."""
    import torch
    gen = torch.Generator(device=dev).manual_seed(31)
    out = {"kernel": "gemm_f16_kernel (tcgen05 kind::f16, fp32 TMEM accumulators)", "gemms": []}
    peak = peaks.get("bf16_tflops")
    for name, M, N, K in (("fc1_f16", 4096, 4096, 1024), ("fc2_f16", 4096, 1024, 4096)):
        w = (torch.randn(N, K, device=dev, generator=gen) * 0.02).half()
        x = torch.randn(M, K, device=dev, generator=gen)
        y = torch.empty(M, N, device=dev)
        ws = b2q._empty_aligned(b2q.lib().b2q_mul_mat_workspace_bytes(b2q.TYPE_F16, M, N, K, 0), dev)
        for _ in range(3):
            b2q.mul_mat(b2q.TYPE_F16, w, x, out=y, ws=ws, stream=stream)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            b2q.mul_mat(b2q.TYPE_F16, w, x, out=y, ws=ws, stream=stream)
            e1.record(stream)
        torch.cuda.synchronize()
        us = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3
        tflops = ops_of(M, N, K) / (us * 1e-6) / 1e12
        row = {"name": name, "M": M, "N": N, "K": K, "us_incl_fp16_rounding": round(us, 2),
               "tflops": round(tflops, 1)}
        if peak:
            row["frac_of_measured_bf16"] = round(tflops / peak, 4)
        out["gemms"].append(row)
    return out


SLAT = dict(C=1024, n_blocks=24, grid=64, occupancy=0.03, n_cond=1374, fixed_tokens=(8192, 20480))


def slat_tokens(seed: int = 3):
    """BASELINE configs[3] token count: 3% of the 64^3 cells sampled without
    replacement, downsampled to 32^3 (coarse = unique(coord // 2))."""
    g = SLAT["grid"]
    rng = np.random.default_rng(seed)
    n_fine = int(round(SLAT["occupancy"] * g ** 3))
    idx = rng.choice(g ** 3, n_fine, replace=False)
    x, y, z = idx // (g * g), (idx // g) % g, idx % g
    return n_fine, int(np.unique((x // 2) * 1024 + (y // 2) * 32 + z // 2).size)


def neighbour_table(keys: np.ndarray, g: int) -> np.ndarray:
    """27-neighbour table (offset-major, -1 = missing) of the sorted cell keys
    (x * g + y) * g + z of a g^3 grid."""
    n = keys.size
    xyz = np.stack([keys // (g * g), (keys // g) % g, keys % g], 1)
    idx = np.full((27, n), -1, np.int32)
    o = 0
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                q = xyz + np.array([dx, dy, dz])
                inside = np.all((q >= 0) & (q < g), 1)
                qk = (q[:, 0] * g + q[:, 1]) * g + q[:, 2]
                pos = np.clip(np.searchsorted(keys, qk), 0, n - 1)
                hit = inside & (keys[pos] == qk)
                idx[o, hit] = pos[hit]
                o += 1
    return idx


def slat_grid_tables(seed: int = 3):
    """The configs[3] sparse grid (3% of 64^3 sampled without replacement):
    the 27-neighbour tables of the fine cells and of their 2x-downsampled
    coarse cells, and the downsample mapping (coarse row per fine cell,
    divisors |children| + 1)."""
    g = SLAT["grid"]
    rng = np.random.default_rng(seed)
    n = int(round(SLAT["occupancy"] * g ** 3))
    keys = np.sort(rng.choice(g ** 3, n, replace=False))
    x, y, z = keys // (g * g), (keys // g) % g, keys % g
    ck = ((x // 2) * (g // 2) + y // 2) * (g // 2) + z // 2
    ckeys, rows = np.unique(ck, return_inverse=True)
    counts = (np.bincount(rows, minlength=ckeys.size) + 1).astype(np.float32)
    return neighbour_table(keys, g), neighbour_table(ckeys, g // 2), rows.astype(np.int32), counts


def run_ss_step_case(args):
    """Profiling case: the configs[4] SS-flow step run eagerly (no graph, so a
    profiler sees every kernel), --warmup steps, then --steps steps inside the
    NVTX range "ss_step"; prints the median CUDA-event time per step."""
    import torch
    import b2q
    import ss_flow
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = SS_FLOW
    C, nc = cfg["C"], SS_BLOCK["n_cond"]
    specs = ss_flow.param_specs(C, cfg["n_blocks"], cfg["n_shape"], cfg["in_ch"], cfg["mlp_ratio"])
    flow = ss_flow.SsFlow(dev, ss_flow.random_params(specs, dev, b2q.TYPE_Q8_0, seed=11), **cfg)
    gen = torch.Generator(device=dev).manual_seed(13)
    smp = ss_flow.SsSampler(flow, torch.randn(nc, C, device=dev, generator=gen), nc, seed=12)
    t, dt = ss_flow.euler_schedule()[0]
    for _ in range(args.warmup):
        smp.step(t * 1000.0, dt)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.nvtx.range_push("ss_step")
    for e0, e1 in evs:
        e0.record()
        smp.step(t * 1000.0, dt)
        e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)
    return {"case": "ss_step", "step_ms_eager": round(ms, 3), "steps": args.steps}


SPARSE_CASES = ("sparse_conv_fine", "sparse_conv_fine_planned")


def run_sparse_case(args):
    """Profiling case: --steps sparse convolutions (128 -> 128 channels on the
    configs[3] fine cells), dense or planned, after --warmup; hot L2."""
    import torch
    import b2q
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    idx, _, _, _ = slat_grid_tables()
    tokens, C, cout = idx.shape[1], 128, 128
    gen = torch.Generator(device=dev).manual_seed(41)
    x16 = torch.randn(tokens, C, device=dev, generator=gen).half()
    w16 = (torch.randn(cout, 27 * C, device=dev, generator=gen) / (27 * C) ** 0.5).half()
    b16 = (torch.randn(cout, device=dev, generator=gen) * 0.1).half()
    y16 = torch.empty(tokens, cout, device=dev, dtype=torch.float16)
    table = torch.from_numpy(idx).to(dev)
    if args.only.endswith("planned"):
        plan = b2q.sparse_conv_plan(table)
        ws = b2q._empty_aligned(b2q.lib().b2q_sparse_conv_f16_planned_workspace_bytes(tokens, C, cout), dev)
        fn = lambda: b2q.sparse_conv_f16_planned(x16, w16, b16, plan, out=y16, ws=ws)  # noqa: E731
    else:
        ws = b2q._empty_aligned(b2q.lib().b2q_sparse_conv_f16_workspace_bytes(tokens, C, cout), dev)
        fn = lambda: b2q.sparse_conv_f16(x16, w16, b16, table, out=y16, ws=ws)  # noqa: E731
    for _ in range(args.warmup):
        fn()
    # Ten calls per event pair: a single call of a few microseconds would time
    # the host's submission, not the device.
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in evs:
        e0.record()
        for _ in range(10):
            fn()
        e1.record()
    torch.cuda.synchronize()
    us = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3 / 10
    return {"case": args.only, "tokens": tokens, "C": C, "Cout": cout, "us_per_call_hot_l2": round(us, 2),
            "calls_per_event_pair": 10}


def slat_sparse_side(b2q, flush, stream, dev, peaks, iters=10):
    """The SLat sparse stages at the configs[3] grid: the F16 submanifold
    convolution (gather of the 27 neighbour rows + kind::f16 GEMM) on the fine
    cells at 128 -> 128 channels and on the coarse cells at 256 -> 256, and
    the F16 scatter-mean (2x downsample) of 128 channels.  L2 flushed between
    runs; CUDA events."""
    import torch
    idx, cidx, rows, counts = slat_grid_tables()
    fine, coarse = idx.shape[1], cidx.shape[1]
    gen = torch.Generator(device=dev).manual_seed(41)

    def timed(fn):
        fn()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            fn()
            e1.record(stream)
        torch.cuda.synchronize()
        return statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) * 1e3

    out = {"grid": f"{SLAT['grid']}^3 at {SLAT['occupancy']:.0%}", "fine_cells": fine, "coarse_cells": coarse,
           "conv": []}
    idx_d = torch.from_numpy(idx).to(dev)
    for name, tokens, C, cout, table in (("fine_128_128", fine, 128, 128, idx_d),
                                         ("coarse_256_256", coarse, 256, 256, torch.from_numpy(cidx).to(dev))):
        x16 = torch.randn(tokens, C, device=dev, generator=gen).half()
        w16 = (torch.randn(cout, 27 * C, device=dev, generator=gen) / (27 * C) ** 0.5).half()
        b16 = (torch.randn(cout, device=dev, generator=gen) * 0.1).half()
        y16 = torch.empty(tokens, cout, device=dev, dtype=torch.float16)
        ws = b2q._empty_aligned(b2q.lib().b2q_sparse_conv_f16_workspace_bytes(tokens, C, cout), dev)
        us = timed(lambda: b2q.sparse_conv_f16(x16, w16, b16, table, out=y16, ws=ws, stream=stream))
        plan = b2q.sparse_conv_plan(table, stream=stream)
        wsp = b2q._empty_aligned(b2q.lib().b2q_sparse_conv_f16_planned_workspace_bytes(tokens, C, cout), dev)
        us_p = timed(lambda: b2q.sparse_conv_f16_planned(x16, w16, b16, plan, out=y16, ws=wsp, stream=stream))
        flops = 2.0 * tokens * cout * 27 * C
        valid = int((table >= 0).sum().item())
        row = {"name": name, "tokens": tokens, "C": C, "Cout": cout, "us": round(us, 2),
               "tflops_dense_27": round(flops / (us * 1e-6) / 1e12, 1),
               "valid_neighbour_fraction": round(valid / (27 * tokens), 3),
               "gather_bytes": tokens * 27 * C * 2, "launches": 3,
               "us_planned": round(us_p, 2), "launches_planned": 4,
               "tflops_useful_planned": round(2.0 * valid * cout * C / (us_p * 1e-6) / 1e12, 1)}
        out["conv"].append(row)
    x16 = torch.randn(fine, 128, device=dev, generator=gen).half()
    rows_d, counts_d = torch.from_numpy(rows).to(dev), torch.from_numpy(counts).to(dev)
    o16 = torch.empty(coarse, 128, device=dev, dtype=torch.float16)
    ws = b2q._empty_aligned(b2q.lib().b2q_sparse_scatter_mean_workspace_bytes(fine, coarse), dev)
    us = timed(lambda: b2q.sparse_scatter_mean_f16(x16, rows_d, counts_d, coarse, out=o16, ws=ws, stream=stream))
    plan = b2q.sparse_scatter_plan(rows_d, coarse, stream=stream)
    us_planned = timed(lambda: b2q.sparse_scatter_mean_f16_planned(x16, plan, counts_d, coarse, out=o16,
                                                                   stream=stream))
    out["scatter_mean"] = {"fine": fine, "coarse": coarse, "C": 128, "us": round(us, 2), "launches": 6,
                           "us_planned": round(us_planned, 2), "launches_planned": 1,
                           "bytes": fine * 256 + coarse * 256 + fine * 8}
    return out


def slat_side(b2q, stream, dev, iters=3):
    """the SLat flow transformer's linears over 24 blocks
    with Q4_0 weights (random codes and fp16 scales generated on the device)
    at the sampled sparse token count and at 8192 / 20480 tokens.  One pass =
    for every block: qkv, out, cross q, cross kv (on the condition tokens),
    cross out, fc1, fc2, each with its activation quantize (ggml mul_mat
    semantics: every mul_mat quantizes its fp32 input).  The weights (216 MB)
    and activations exceed L2, so no flush."""
    import torch
    import ss_flow
    C, nbk, nc = SLAT["C"], SLAT["n_blocks"], SLAT["n_cond"]
    shapes = ss_flow.linear_shapes(C, 4 * C)
    specs = [(f"b{i}.{name}", "q", shp, (0.0, 0.02)) for i in range(nbk) for name, shp in shapes.items()]
    raw = ss_flow.random_params(specs, dev, b2q.TYPE_Q4_0, seed=21)
    W = {name: b2q.weight_pack(b2q.TYPE_Q4_0, raw[name], shp[1]) for name, _, shp, _ in specs}
    del raw
    n_fine, n_coarse = slat_tokens()
    gen = torch.Generator(device=dev).manual_seed(22)
    cond = torch.randn(nc, C, device=dev, generator=gen)
    out = {"config": dict(SLAT, weights="Q4_0 (random codes and fp16 scales)", sampled_fine_cells=n_fine),
           "runs": []}
    for M in (n_coarse,) + SLAT["fixed_tokens"]:
        x = torch.randn(M, C, device=dev, generator=gen)
        xh = torch.randn(M, 4 * C, device=dev, generator=gen)
        y = torch.empty(M * 4 * C, device=dev)
        act = b2q._empty_aligned(b2q.act_prepared_size(M, 4 * C), dev)
        act_c = b2q._empty_aligned(b2q.act_prepared_size(nc, C), dev)

        def one_pass():
            for i in range(nbk):
                for name, (n, k) in shapes.items():
                    src, m = (cond, nc) if name == "xkv" else ((xh, M) if name == "fc2" else (x, M))
                    a = act_c if name == "xkv" else act
                    b2q.act_prepare(src, out=a, stream=stream)
                    b2q.mul_mat_prepared(W[f"b{i}.{name}"], n, k, a, m, out=y[:m * n].view(m, n), stream=stream)

        one_pass()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
        for e0, e1 in evs:
            e0.record(stream)
            one_pass()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)
        ops = nbk * sum(ops_of(nc if name == "xkv" else M, n, k) for name, (n, k) in shapes.items())
        out["runs"].append({"tokens": M, "source": "sampled" if M == n_coarse else "fixed",
                            "ms_24_blocks": round(ms, 3), "int_ops": ops,
                            "tops_incl_quantize": round(ops / (ms * 1e-3) / 1e12, 1),
                            "launches": nbk * len(shapes) * 2})
    del W
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------- column-parallel (multi-GPU)
COLPAR_SHAPE = ("slat_qkv_q4_0", 2, 20480, 3072, 1024)  # name, wtype, M tokens, N out, K in
COLPAR_Q8_SHAPE = ("slat_fc1_q4_0", 2, 20480, 4096, 1024)  # fc1 -> GELU -> Q8_0: the next layer's input
NVLINK_PEER_GBS = 770.0  # measured peer copy per direction per GPU on this pool's B200s


def colpar_side(args, rank, world, dev, dist=None):
    """One large SLat linear split by output rows over the ranks (the
    column-parallel variant of BASELINE configs[4]); every rank needs the whole
    output.  Two exchanges, each timed fused (the GEMM epilogue stores each
    finished tile into every rank's buffer over NVLink, overlapping the
    remaining tiles' math) against GEMM + NCCL all-gather + transpose:
      fp32: the qkv linear's fp32 output, 4 bytes per value;
      q8:   fc1 with GELU + Q8_0 in the epilogue, so what crosses the links is
            the next layer's prepared input, 1.125 bytes per value.
    Each iteration ends with a one-element all-reduce so that every rank's work
    of the iteration is complete; both variants pay it.  Rank 0 checks the
    gathered bytes against a single-GPU run of the whole weight."""
    import torch
    import b2q
    import colpar

    stream = torch.cuda.current_stream()
    tick = torch.zeros(1, device=dev)
    iters = max(5, min(args.steps, 30))

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / iters, dist, dev)

    def sync_tick():
        if dist:
            dist.all_reduce(tick)

    out = {"n_gpus": world, "iterations": iters, "nvlink_peer_gbs_per_direction": NVLINK_PEER_GBS,
           "sync": "one-element all_reduce per iteration (both variants)"}
    for kind, (name, wtype, M, N, K) in (("fp32", COLPAR_SHAPE), ("q8", COLPAR_Q8_SHAPE)):
        rng = np.random.default_rng(4321 if kind == "fp32" else 4322)  # same weights and inputs on every rank
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        wq = synth_blocks(wtype, w, N, K)
        start, stop = colpar.slices(N, world)[rank]
        n = stop - start
        equal = all(b - a == n for a, b in colpar.slices(N, world))
        packed = b2q.weight_pack(wtype, torch.from_numpy(wq[start:stop]).to(dev), K)
        act = b2q.act_prepare(torch.from_numpy(x).to(dev))
        bias = torch.from_numpy((rng.standard_normal(N) * 0.1).astype(np.float32)).to(dev)
        if kind == "fp32":
            bufs = colpar.PeerBuffers(M, N)
            slice_out = torch.empty((M, n), dtype=torch.float32, device=dev)
            gathered = torch.empty((world * M, n), dtype=torch.float32, device=dev) if equal else None
            full_out = torch.empty((M, N), dtype=torch.float32, device=dev)

            def fused():
                colpar.fused(packed, n, K, act, M, bufs, start, stream=stream)
                sync_tick()

            def baseline():
                if dist:
                    colpar.nccl_baseline(packed, n, K, act, M, N, slice_out, gathered, full_out, stream=stream)
                else:
                    b2q.mul_mat_prepared(packed, n, K, act, M, out=full_out, stream=stream)
                sync_tick()
            value_bytes = 4.0
        else:
            bufs = colpar.activation_buffers(M, N)
            ld = (M + 3) // 4 * 4
            local = b2q._empty_aligned(b2q.act_prepared_size(M, n), dev)
            gcodes = torch.empty((world * M, n), dtype=torch.int8, device=dev) if equal else None
            gscales = torch.empty((world * (n // 32), ld), dtype=torch.float32, device=dev) if equal else None
            full_act = b2q._empty_aligned(b2q.act_prepared_size(M, N), dev)
            b_slice = bias[start:stop]

            def fused():
                colpar.fused_gelu_q8(packed, n, K, act, M, bufs, start, bias=b_slice, stream=stream)
                sync_tick()

            def baseline():
                if dist:
                    colpar.nccl_baseline_gelu_q8(packed, n, K, act, M, N, local, gcodes, gscales, full_act,
                                                 bias=b_slice, stream=stream)
                else:
                    b2q.mul_mat_prepared_gelu_q8(packed, n, K, act, M, bias=b_slice, out=full_act, stream=stream)
                sync_tick()
            value_bytes = 1.125
        ms_fused = timed(fused)
        ms_base = timed(baseline) if (equal or world == 1) else None
        ok = None
        if rank == 0:  # the fused result against one GPU running the whole weight
            full_packed = b2q.weight_pack(wtype, torch.from_numpy(wq).to(dev), K)
            got = bufs.to_tensor(dev)
            if kind == "fp32":
                ok = bool(torch.equal(got, b2q.mul_mat_prepared(full_packed, N, K, act, M)))
            else:
                want = b2q.mul_mat_prepared_gelu_q8(full_packed, N, K, act, M, bias=bias)
                gc, gs = colpar.split_views(got, M, N)
                wc, wsc = colpar.split_views(want, M, N)
                ok = bool(torch.equal(gc, wc) and torch.equal(gs[:, :M], wsc[:, :M]))
            del full_packed
        status = b2q.device_status(clear=True)
        if dist:
            dist.barrier()
        bufs.close()
        ops = 2.0 * M * N * K
        bytes_in = M * N * value_bytes * (world - 1) / world  # each rank receives the others' slices
        link_ms = bytes_in / (NVLINK_PEER_GBS * 1e9) * 1e3
        out[kind] = {
            "workload": f"{name}: M={M} tokens, K={K} -> N={N}, weight rows split over {world} rank(s), every "
                        f"rank ends with the whole output ({'fp32' if kind == 'fp32' else 'GELU + Q8_0 prepared'})",
            "fused_ms": round(ms_fused, 4), "fused_tops": round(ops / (ms_fused * 1e-3) / 1e12, 2),
            "nccl_baseline_ms": None if ms_base is None else round(ms_base, 4),
            "speedup_vs_nccl": None if ms_base is None else round(ms_base / ms_fused, 3),
            "nvlink_bytes_in_per_rank": int(bytes_in),
            "nvlink_gbs_in_per_rank": round(bytes_in / (ms_fused * 1e-3) / 1e9, 1) if world > 1 else 0.0,
            # the time the gathered bytes need at the measured peer bandwidth, as a share of the fused time
            "nvlink_bound_frac": round(link_ms / ms_fused, 3) if world > 1 else 0.0,
            "parity_rank0_bitwise_vs_single_gpu": ok, "device_status": status,
            "path": ("b2q_mul_mat_prepared_peers" if kind == "fp32" else "b2q_mul_mat_prepared_gelu_q8_peers")
                    + " (CUDA-IPC peer pointers, P2P stores from the epilogue); baseline: the single-rank "
                    "kernel on the slice + all_gather_into_tensor + transpose copy",
        }
        del packed, act
    out["mlp"] = colpar_mlp(args, rank, world, dev, dist, timed, sync_tick)
    return out


COLPAR_MLP = (20480, 1024, 4096)  # tokens, model width C, hidden width (SLat feed-forward, Q4_0)


def colpar_mlp(args, rank, world, dev, dist, timed, sync_tick):
    """The SLat feed-forward branch sharded over the ranks end to end:
    fc1 (C -> hidden, GELU + Q8_0) column-parallel with the Q8_0 exchange into
    every rank's fc2 input, then fc2 (hidden -> C) column-parallel with the
    fp32 gather into every rank's output -- two fused exchanges per step, the
    ranks synchronised between them (fc2 reads what the peers wrote).  Rank 0's
    output is checked bit for bit against one GPU running both whole weights."""
    import torch
    import b2q
    import colpar

    M, C, H = COLPAR_MLP
    rng = np.random.default_rng(4323)  # same weights and inputs on every rank
    w1 = synth_blocks(2, (rng.standard_normal((H, C)) * 0.02).astype(np.float32), H, C)
    w2 = synth_blocks(2, (rng.standard_normal((C, H)) * 0.02).astype(np.float32), C, H)
    x = rng.standard_normal((M, C)).astype(np.float32)
    b1 = torch.from_numpy((rng.standard_normal(H) * 0.1).astype(np.float32)).to(dev)
    b2 = torch.from_numpy((rng.standard_normal(C) * 0.1).astype(np.float32)).to(dev)
    s1, e1 = colpar.slices(H, world)[rank]
    s2, e2 = colpar.slices(C, world)[rank]
    p1 = b2q.weight_pack(2, torch.from_numpy(w1[s1:e1]).to(dev), C)
    p2 = b2q.weight_pack(2, torch.from_numpy(w2[s2:e2]).to(dev), H)
    act = b2q.act_prepare(torch.from_numpy(x).to(dev))
    hid = colpar.activation_buffers(M, H)  # every rank's fc2 input
    ybuf = colpar.PeerBuffers(M, C)        # every rank's output
    hid_t = hid.local_tensor(dev)  # this rank's copy, as the fc2 operand (no copy)
    stream = torch.cuda.current_stream()

    def step():
        colpar.fused_gelu_q8(p1, e1 - s1, C, act, M, hid, s1, bias=b1[s1:e1], stream=stream)
        sync_tick()  # every rank's fc1 tiles have landed before any rank's fc2 reads them
        colpar.fused(p2, e2 - s2, H, hid_t, M, ybuf, s2, bias=b2[s2:e2], stream=stream)
        sync_tick()

    ms = timed(step)
    ok = None
    if rank == 0:
        f1 = b2q.weight_pack(2, torch.from_numpy(w1).to(dev), C)
        f2 = b2q.weight_pack(2, torch.from_numpy(w2).to(dev), H)
        h_ref = b2q.mul_mat_prepared_gelu_q8(f1, H, C, act, M, bias=b1)
        y_ref = b2q.mul_mat_prepared(f2, C, H, h_ref, M, bias=b2)
        ok = bool(torch.equal(ybuf.to_tensor(dev), y_ref))
        del f1, f2, h_ref, y_ref
    status = b2q.device_status(clear=True)
    if dist:
        dist.barrier()
    del hid_t
    hid.close()
    ybuf.close()
    ops = 2.0 * M * C * H * 2
    bytes_in = M * (H * 1.125 + C * 4.0) * (world - 1) / world
    return {"workload": f"SLat MLP, {M} tokens: fc1 {C} -> {H} (GELU + Q8_0, exchanged as Q8_0), fc2 {H} -> {C} "
                        f"(fp32, gathered), Q4_0 weights, both split by output rows over {world} rank(s)",
            "ms": round(ms, 4), "tops": round(ops / (ms * 1e-3) / 1e12, 2),
            "nvlink_bytes_in_per_rank": int(bytes_in),
            "parity_rank0_bitwise_vs_single_gpu": ok, "device_status": status,
            "path": "b2q_mul_mat_prepared_gelu_q8_peers, rank sync, b2q_mul_mat_prepared_peers, rank sync"}


def run_colpar(args, rank, world, local_rank):
    """--colpar: only the column-parallel measurement, as its own JSON line."""
    import datetime
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    d = None
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        d = dist
    side = colpar_side(args, rank, world, dev, d)
    if d:
        dist.destroy_process_group()
    q8 = side["q8"]
    return {
        "metric": "column-parallel fc1 (GELU + Q8_0 exchange) effective TOPS, output on every rank",
        "value": q8["fused_tops"], "unit": UNIT, "n_gpus": world, "steps": side["iterations"],
        "warmup": 3, "ms_per_step": q8["fused_ms"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "i8", "data": "synthetic",
        "config": {"workload": q8["workload"], "parallelism": f"column-parallel tp{world}"},
        "colpar": side,
    }


# -------------------------------------------------------------------- CPU arm
def host_threads() -> int:
    """Every core this process may run on.  Passed to the oracle explicitly:
    torchrun sets OMP_NUM_THREADS=1 in each rank, which would otherwise leave
    the CPU arm (rank 0 alone) on one core."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_sample_run(inputs, frac):
    """Oracle (vectorised port of ggml's CPU mul_mat) over the first `frac` of
    each GEMM's token rows; returns (ops, seconds, threads)."""
    import oracle as O
    ops, secs, thr = 0.0, 0.0, host_threads()
    for name, wtype, M, N, K, wq, x in inputs:
        rows = max(1, int(round(M * frac)))
        xs = np.ascontiguousarray(x[:rows])
        t0 = time.perf_counter()
        O.mul_mat(wtype, wq, xs, O.ACT_X86, nthreads=thr, fast=True)
        secs += time.perf_counter() - t0
        ops += ops_of(rows, N, K)
    return ops, secs, thr


def pick_frac(inputs, target_s):
    ops, secs, _ = cpu_sample_run(inputs, 0.01)
    full_ops = sum(ops_of(M, N, K) for _, _, M, N, K, _, _ in inputs)
    rate = ops / max(secs, 1e-6)
    return min(1.0, max(0.01, target_s * rate / full_ops))


def cpu_baseline(inputs, budget_s=15.0):
    """Bounded sample of the same workload on the host cores: whole passes over
    the workload (or the leading fraction of each GEMM's token rows when one
    pass exceeds the budget), repeated until ~budget_s of CPU work."""
    import oracle as O
    frac = pick_frac(inputs, budget_s)
    ops, secs, reps, thr = 0.0, 0.0, 0, 1
    while secs < budget_s and reps < 1000:
        o, s, thr = cpu_sample_run(inputs, frac)
        ops, secs, reps = ops + o, secs + s, reps + 1
    return {"value": round(ops / secs / 1e12, 4), "unit": UNIT, "cores": thr, "kind": "port",
            "isa": O.isa(),
            "sample": f"{reps} pass(es) over the first {frac:.3f} of each GEMM's token rows "
                      f"(fc1, fc2, kv), {secs:.1f} s, oracle port of ggml CPU mul_mat incl. "
                      f"activation quantize"}


def run_reference(args):
    inputs = make_inputs()
    per_step_s = min(3.0, 150.0 / max(1, args.steps + args.warmup))
    frac = pick_frac(inputs, per_step_s)
    for _ in range(args.warmup):
        cpu_sample_run(inputs, frac)
    tot_ops, tot_s, thr = 0.0, 0.0, 1
    for _ in range(args.steps):
        o, s, thr = cpu_sample_run(inputs, frac)
        tot_ops += o
        tot_s += s
    import oracle as O
    value = tot_ops / tot_s / 1e12
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tot_s / args.steps * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "i8", "data": "synthetic",
        "config": config_dict(),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": thr, "kind": "port",
                         "isa": O.isa(),
                         "sample": f"first {frac:.3f} of each GEMM's token rows per step"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "ggml (the reference's arithmetic) is an empty submodule in the reference checkout; "
                "timed is the oracle's vectorised C port of ggml's CPU Q8_0/Q4_0 mul_mat, all host threads",
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b2q", "reference"], default="b2q")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-mlp", action="store_true", help="skip the fused-MLP side measurement")
    ap.add_argument("--only", default=None, help="run one workload entry (profiling case)")
    ap.add_argument("--no-colpar", action="store_true", help="skip the column-parallel side measurement")
    ap.add_argument("--colpar", action="store_true",
                    help="column-parallel SLat linear (one GEMM split over the ranks, all-gathered output)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return
    if args.only in ATTN_CASES:
        res = run_attn_case(args)
    elif args.only in F16_CASES:
        res = run_f16_case(args)
    elif args.only in SPARSE_CASES:
        res = run_sparse_case(args)
    elif args.only == "ss_step":
        res = run_ss_step_case(args)
    else:
        res = run_colpar(args, rank, world, local_rank) if args.colpar else run_gpu(args, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()

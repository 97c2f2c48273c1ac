"""Benchmark: the BitLinear hot path of one BitNet-b1.58-2B-shaped decode token.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("bitnet2b_decode_bitlinear_sweep", BASELINE config 2 shapes): one
step runs every BitLinear of one decode token -- 30 layers x {Q,K,V fused,
O, gate/up fused, down}, each an absmax int8 quantisation of a distinct f32
activation vector followed by the I2_S ternary matvec (210 weight tensors,
521,011,200 packed bytes, all distinct and resident in HBM).  The working set
is 4x the 126 MB L2, so no L2 flush is needed between steps.  The metric is
BASELINE's "I2_S matvec HBM GB/s": algorithmic bytes (packed weights + scale +
f32 activations in + f32 outputs) per second.

`value` is the sustained streaming rate (SURVEY's "sustains" reading: back to
back over distinct weight buffers larger than L2): the 210 matvecs, each with
its own input, as one persistent launch per step (wl_dev_i2s_stream_run:
quantise all inputs, then stream every weight once), CUDA events on the
launching stream, max over ranks.  `decode_chain` times the same 210 matvecs in
decode order as 120 dependent launches (QKV and gate/up fused; every kernel
waits for the previous one, quantises its input in-kernel, and prefetches its
weights before that wait) -- the latency-bound batch-1 decode figure.
`e2e` runs the same 210 matvecs through the drop-in host-buffer C ABI
(wl_bitlinear_i2s_matvec_f32, one call per BitLinear as the reference's
linear_matvec_f32 is called), host->device copy of each input and
device->host copy of each output inside the timed region.

Multi-GPU (torchrun, N > 1): every rank runs its own copy of the sweep (a
replica; independent decode streams), no collective on the data path;
value = N x bytes / max-over-ranks time ("scaling": "weak").

`--impl reference` times the reference's x86 kernel (the oracle port of
bitlinear_i2s_matvec_f32_sse2_i8, single-threaded like the reference's x86
I2_S path) on this host over a bounded sample of the same sweep.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "I2_S matvec HBM GB/s"
UNIT = "GB/s"
WORKLOAD = "bitnet2b_decode_bitlinear_sweep"
SEED = 0x5EED + 2
LAYERS = 30
D_MODEL, D_FF, D_KV = 2560, 6912, 640
VOCAB = 128256
# fused launch groups per layer: (in_dim, [out_dims])
GROUPS = [(D_MODEL, [D_MODEL, D_KV, D_KV]), (D_MODEL, [D_MODEL]), (D_MODEL, [D_FF, D_FF]),
          (D_FF, [D_MODEL])]


def algorithmic_bytes(in_dim: int, out_dim: int) -> int:
    """Packed weights + f32 scale + f32 input + f32 output of one matvec."""
    return in_dim // 4 * out_dim + 4 + 4 * in_dim + 4 * out_dim


def sweep_bytes() -> int:
    return LAYERS * sum(algorithmic_bytes(k, n) for k, ns in GROUPS for n in ns)


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ GPU arm
def make_i2s_weights(torch, dev, rng: np.random.Generator):
    """All 210 BitNet-2B BitLinear weights, generated on the device (seeded)."""
    from project_willamette_b200.synth import _BYTE_LUT
    lut = torch.from_numpy(_BYTE_LUT).to(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(int(rng.integers(0, 2**62)))
    layers = []
    for _ in range(LAYERS):
        groups = []
        for in_dim, outs in GROUPS:
            ws = []
            for n in outs:
                raw = torch.randint(0, 256, (n * in_dim // 4,), dtype=torch.uint8, device=dev,
                                    generator=g)
                ws.append((lut[raw.long()], float(np.float32(rng.uniform(0.01, 0.1))), n))
            x = torch.randn(in_dim, device=dev, generator=g, dtype=torch.float32)
            groups.append((in_dim, ws, x))
        layers.append(groups)
    return layers


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist
    import project_willamette_b200 as wl
    from project_willamette_b200 import _abi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    L = wl.lib()
    rc = L.wl_init(local)
    if rc:
        raise RuntimeError(L.wl_last_error().decode())

    def ck(rc):
        if rc:
            raise RuntimeError(L.wl_last_error().decode())

    rng = np.random.default_rng(SEED + rank)
    layers = make_i2s_weights(torch, dev, rng)
    stream = torch.cuda.Stream(device=dev)
    found = torch.zeros(1, dtype=torch.int32, device=dev)

    # Per launch group: a fused-input weight array (decode-order chain) and the
    # same weights as stream ops (persistent streaming launch).
    groups, sops, outs = [], [], []
    for lgroups in layers:
        for in_dim, ws, x in lgroups:
            arr = (_abi.WlI2sDevWeight * len(ws))()
            for i, (packed, s, n) in enumerate(ws):
                ck(L.wl_dev_i2s_scan_code3(packed.data_ptr(), packed.numel(), found.data_ptr(),
                                           stream.cuda_stream))
                torch.cuda.synchronize()
                y = torch.empty(n, dtype=torch.float32, device=dev)
                outs.append(y)
                arr[i].packed, arr[i].w_scale, arr[i].out_dim = packed.data_ptr(), s, n
                arr[i].y, arr[i].acc = y.data_ptr(), None
                arr[i].flags = 0 if int(found.item()) else _abi.WL_I2S_NO_CODE3
                op = _abi.WlI2sStreamOp()
                op.packed, op.w_scale, op.in_dim, op.out_dim = packed.data_ptr(), s, in_dim, n
                op.x, op.y, op.acc, op.flags = x.data_ptr(), y.data_ptr(), None, 0
                sops.append(op)
            groups.append((in_dim, x, arr, len(ws)))
    ops_arr = (_abi.WlI2sStreamOp * len(sops))(*sops)
    plan = C.c_void_p()
    ck(L.wl_i2s_stream_plan_create(ops_arr, len(sops), C.byref(plan)))

    def stream_step(h: int) -> int:
        ck(L.wl_dev_i2s_stream_run(plan, h))
        return 2

    def chain_step(h: int) -> int:
        for in_dim, x, arr, nw in groups:
            ck(L.wl_dev_i2s_matvec_fused_f32(arr, nw, in_dim, x.data_ptr(), h))
        return len(groups)

    def capture(fn):
        with torch.cuda.stream(stream):
            n = fn(stream.cuda_stream)  # eager run: first-use paths
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                fn(torch.cuda.current_stream().cuda_stream)
        return g, n

    def timed(g, steps, clocks=None):
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 3)):
                g.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ctx = clocks if clocks is not None else _Null()
            with ctx:
                e0.record(stream)
                for _ in range(steps):
                    g.replay()
                e1.record(stream)
                torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    g_stream, launches_per_step = capture(stream_step)
    g_chain, chain_launches = capture(chain_step)
    clk = ClockSampler(local)
    ms_total = timed(g_stream, args.steps, clk)
    chain_steps = max(1, args.steps // 4)
    ms_chain = timed(g_chain, chain_steps)

    # Isolated per-launch duration of the per-op kernel (events around each
    # launch of one eager decode-order step; no overlap between launches).
    iso = []
    with torch.cuda.stream(stream):
        for in_dim, x, arr, nw in groups:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ck(L.wl_dev_i2s_matvec_fused_f32(arr, nw, in_dim, x.data_ptr(), stream.cuda_stream))
            b.record(stream)
            iso.append((a, b, sum(algorithmic_bytes(in_dim, arr[i].out_dim) for i in range(nw))))
        torch.cuda.synchronize()
    iso_ms = sum(a.elapsed_time(b) for a, b, _ in iso)
    iso_bytes = sum(nb for _, _, nb in iso)

    bytes_step = sweep_bytes()
    ms_step = ms_total / args.steps
    value = world * bytes_step / (ms_step * 1e-3) / 1e9
    achieved = bytes_step / (ms_step * 1e-3) / 1e9  # one stream launch per step
    ms_chain_step = ms_chain / chain_steps
    pk = peaks()

    # ---- lm-head (Q6_K 128256 x 2560, batch 1 and 64) and prefill GEMM (config 3)
    lm = lm_head_bench(torch, dev, L, stream, rng, reps=max(20, min(args.steps, 200)))
    gemm = gemm_bench(torch, dev, L, stream, rng)

    # ---- e2e through the host-buffer C ABI
    e2e = e2e_bench(torch, layers, wl, rng, steps=max(1, min(args.steps, 20)))
    if world > 1:
        t = torch.tensor([e2e["seconds_per_step"]], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e["seconds_per_step"] = float(t.item())
    e2e_value = world * bytes_step / e2e["seconds_per_step"] / 1e9

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(seconds=args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xternary->i32", "data": "synthetic (seeded; BASELINE distributions)",
            "config": {"workload": WORKLOAD, "layers": LAYERS, "d_model": D_MODEL, "d_ff": D_FF,
                       "kv_dim": D_KV, "matvecs_per_step": LAYERS * 7,
                       "bytes_per_step": bytes_step, "batch": 1,
                       "mode": "sustained: 210 independent matvecs, one persistent launch",
                       "l2": "inputs larger than L2 (521 MB of distinct weights per step)",
                       "parallelism": f"replicas x{world}" if world > 1 else "single"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": TRAFFIC_PER_STEP_BYTES,
                         "peak_source": pk["source"], "kernel": "i2s_stream_kernel"},
            "decode_chain": {
                "gbs": round(world * bytes_step / (ms_chain_step * 1e-3) / 1e9, 2),
                "ms_per_step": round(ms_chain_step, 5), "launches_per_step": chain_launches,
                "note": "decode order: 120 dependent fused quantise+matvec kernels (PDL)",
                "isolated_launch_gbs": round(iso_bytes / (iso_ms * 1e-3) / 1e9, 2)},
            "e2e": {"value": round(e2e_value, 3), "unit": UNIT,
                    "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                    "api": "wl_bitlinear_i2s_matvec_f32 (host buffers, one call per BitLinear)"},
            "gpu_launches": launches_per_step * args.steps,
            "lm_head": lm,
            "prefill_gemm": gemm,
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del g_stream, g_chain
    L.wl_i2s_stream_plan_destroy(plan)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# Measured DRAM traffic of the sweep per step (ncu, see profiles/); None until
# captured.
TRAFFIC_PER_STEP_BYTES = None


def lm_head_bench(torch, dev, L, stream, rng, reps: int) -> dict:
    """Q6_K tied lm-head + greedy argmax, 128256 x 2560, batch 1 (config 4)."""
    from project_willamette_b200 import synth
    raw = torch.from_numpy(synth.q6k_rows(rng, D_MODEL, VOCAB)).to(dev)
    packed = torch.empty(L.wl_q6k_packed_bytes(D_MODEL, VOCAB), dtype=torch.uint8, device=dev)
    assert L.wl_dev_q6k_repack(raw.data_ptr(), D_MODEL, VOCAB, packed.data_ptr(),
                               stream.cuda_stream) == 0
    del raw
    h = torch.randn(D_MODEL, device=dev)
    ids = torch.zeros(1, dtype=torch.int32, device=dev)
    scratch = torch.zeros(L.wl_q6k_scratch_bytes(1), dtype=torch.uint8, device=dev)
    s = stream.cuda_stream

    def once():
        rc = L.wl_dev_q6k_lm_head(packed.data_ptr(), D_MODEL, VOCAB, h.data_ptr(), 1, None,
                                  ids.data_ptr(), scratch.data_ptr(), s)
        if rc:
            raise RuntimeError(L.wl_last_error().decode())

    with torch.cuda.stream(stream):
        for _ in range(3):
            once()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            once()
        b.record(stream)
        torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / reps
    alg = 269337600 + 4 * D_MODEL + 4
    # batch 64 (config 4), same exact arithmetic
    H = torch.randn(64, D_MODEL, device=dev)
    ids64 = torch.zeros(64, dtype=torch.int32, device=dev)
    scratch64 = torch.zeros(L.wl_q6k_scratch_bytes(64), dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        def once64():
            rc = L.wl_dev_q6k_lm_head(packed.data_ptr(), D_MODEL, VOCAB, H.data_ptr(), 64, None,
                                      ids64.data_ptr(), scratch64.data_ptr(), s)
            if rc:
                raise RuntimeError(L.wl_last_error().decode())
        once64()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(5):
            once64()
        b.record(stream)
        torch.cuda.synchronize()
    us64 = a.elapsed_time(b) * 1e3 / 5
    return {"us_per_call": round(us, 2), "gbs": round(alg / (us * 1e-6) / 1e9, 1),
            "algorithmic_bytes": alg, "vocab": VOCAB, "batch": 1, "exact_logits": True,
            "batch64_us_per_call": round(us64, 1),
            "batch64_gflops": round(2 * 64 * D_MODEL * VOCAB / (us64 * 1e-6) / 1e9, 1)}


def int8_peak_tops() -> dict:
    """Dense int8 tensor peak: MEASURED_PEAKS.json has the cuBLAS bf16 figure;
    B200's dense int8 rate is twice its dense bf16 rate."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return {"tops": 2.0 * float(json.load(f)["bf16_tflops"]),
                    "source": "2 x measured bf16 (burst)"}
    except Exception:
        return {"tops": 4500.0, "source": "nominal dense int8"}


def gemm_bench(torch, dev, L, stream, rng) -> dict:
    """prefill GEMM, M in {2048, 512, 128} x the three
    BitNet-2B weight shapes, one tcgen05 GEMM per call (bit-exact path)."""
    from project_willamette_b200 import _abi, synth
    pk = int8_peak_tops()
    shapes = [(2560, 6912), (2560, 2560), (6912, 2560)]  # (K, N)
    rows = []
    s = stream.cuda_stream
    with torch.cuda.stream(stream):
        for M in (2048, 512, 128):
            for K, N in shapes:
                packed = torch.from_numpy(synth.i2s_packed(rng, K, N)).to(dev)
                x = torch.randn(M, K, device=dev)
                y = torch.empty(M, N, device=dev)
                ws = torch.empty(L.wl_i2s_gemm_workspace_bytes(M, K), dtype=torch.uint8, device=dev)
                scale = float(np.float32(rng.uniform(0.01, 0.1)))

                def once():
                    rc = L.wl_dev_i2s_gemm_f32(packed.data_ptr(), scale, K, N, M, x.data_ptr(),
                                               y.data_ptr(), None, ws.data_ptr(),
                                               _abi.WL_I2S_NO_CODE3, s)
                    if rc:
                        raise RuntimeError(L.wl_last_error().decode())

                for _ in range(3):
                    once()
                reps = 50
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for _ in range(reps):
                    once()
                b.record(stream)
                torch.cuda.synchronize()
                us = a.elapsed_time(b) * 1e3 / reps
                tops = 2.0 * M * N * K / (us * 1e-6) / 1e12
                rows.append({"M": M, "N": N, "K": K, "us": round(us, 2), "tops": round(tops, 1),
                             "frac": round(tops / pk["tops"], 4)})
    return {"peak_tops": pk["tops"], "peak_source": pk["source"],
            "note": "per call: quantise + tcgen05 GEMM (2 kernels); ops = 2*M*N*K",
            "cases": rows}


def e2e_bench(torch, layers, wl, rng, steps: int) -> dict:
    """The 210 matvecs through the host-buffer drop-in entry point."""
    calls = []
    for groups in layers:
        for in_dim, ws, _ in groups:
            for packed, s, n in ws:
                host = packed.cpu().numpy()
                t = wl.TensorView.i2s("w", in_dim, n, host, s)
                x = rng.standard_normal(in_dim).astype(np.float32)
                y = np.empty(n, np.float32)
                calls.append((t, x, y))
    h2d = sum(c[1].nbytes for c in calls)
    d2h = sum(c[2].nbytes for c in calls)
    for t, x, y in calls:  # first use uploads and caches the weights
        wl.bitlinear_i2s_matvec_f32(t, x, y)
    t0 = time.perf_counter()
    for _ in range(steps):
        for t, x, y in calls:
            wl.bitlinear_i2s_matvec_f32(t, x, y)
    dt = (time.perf_counter() - t0) / steps
    wl.release_weights()
    return {"seconds_per_step": dt, "h2d": h2d, "d2h": d2h}


# ------------------------------------------------------------------ CPU arms
def _one_layer_sample(rng):
    from project_willamette_b200 import synth
    mats = []
    for in_dim, outs in GROUPS:
        for n in outs:
            mats.append((synth.i2s_packed(rng, in_dim, n), synth.i2s_scale(rng), in_dim, n,
                         synth.activations(rng, in_dim)))
    return mats


def cpu_baseline(seconds: float) -> dict:
    """The oracle's SSE2-i8 matvec (reference x86 default, 1 thread), one
    BitNet-2B layer's 7 matvecs repeated for about `seconds`."""
    import oracle
    rng = np.random.default_rng(SEED)
    mats = _one_layer_sample(rng)
    layer_bytes = sum(algorithmic_bytes(k, n) for _, _, k, n, _ in mats)
    for p, s, k, n, x in mats:
        oracle.i2s_matvec_sse2_i8(p, s, k, n, x)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < seconds:
        for p, s, k, n, x in mats:
            oracle.i2s_matvec_sse2_i8(p, s, k, n, x)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": round(layer_bytes * reps / dt / 1e9, 3), "unit": UNIT, "cores": 1,
            "kind": "port", "cpu": _cpu_model(), "host_threads": os.cpu_count(),
            "sample": f"{reps} x one BitNet-2B layer (7 I2_S matvecs, {layer_bytes} B), "
                      f"bitlinear_sse2.rs:313 restated, single thread as the reference's x86 "
                      f"I2_S path"}


def _cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    rng = np.random.default_rng(SEED)
    mats = _one_layer_sample(rng)
    layer_bytes = sum(algorithmic_bytes(k, n) for _, _, k, n, _ in mats)

    def step():
        for p, s, k, n, x in mats:
            oracle.i2s_matvec_sse2_i8(p, s, k, n, x)

    for _ in range(max(args.warmup, 1)):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = layer_bytes / dt / 1e9
    sample = (f"each step = one BitNet-2B layer's 7 I2_S matvecs ({layer_bytes} B) of the "
              f"{LAYERS}-layer sweep; oracle port of bitlinear_sse2.rs:313 (x86 default), "
              f"1 thread (the reference's x86 I2_S path is single-threaded)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xternary->i32",
        "data": "synthetic (seeded; BASELINE distributions)",
        "config": {"workload": WORKLOAD, "layers": LAYERS, "d_model": D_MODEL, "d_ff": D_FF,
                   "kv_dim": D_KV, "batch": 1},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": 1, "kind": "port",
                         "sample": sample, "cpu": _cpu_model()},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()

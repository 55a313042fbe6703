#!/usr/bin/env python
"""Throughput benchmark: ViT-L DINOv2+DPT at 518x518, int8 path, 64 images per
GPU, images/s on N B200s of one node.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N

One step = one batch of `--batch` random-u8 518x518 BGR8 images (seeded per
image) through the whole network (GPU preprocessing -> encoder -> DPT head),
one replica per GPU, no collectives on the data path (images are
independent; "scaling": "weak").

  value    images/s with the images already in HBM: dav2_infer_device_bgr8_batch
           on a CUDA stream, timed with CUDA events (max over ranks);
  e2e      the same through dav2_infer_bgr8_batch with pinned host buffers:
           host->device copy of the BGR8 batch and device->host copy of the
           depth maps inside the timed region (host clock, max over ranks);
  roofline the dominant operation of one step (largest share of the
           executor's live per-operation event timing, dav2_profile_operations)
           with its algorithmic tensor work per launch, against the tensor peak
           of its operand type: int8 = cuBLAS int8 GEMM measured in this run
           (torch._int_mm, 8192^3); f16 = MEASURED_PEAKS.json's sustained bf16
           figure, else the pool's stated fallback (1.4 PFLOP/s sustained);
           `ops` lists the same for every GEMM-family operation;
  cpu_baseline (rank 0, N=1) the reference's CPU path — its PyTorch-CPU fp32
           forward, restated in oracle/torch_graph.py — on one image, all
           host cores.
--impl reference times only that CPU path (rank 0), one image per step.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "depth-anything-v2_b200"), str(ROOT / "oracle")]

METRIC = "ViT-L 518^2 images/s (full graph, int8 path)"
GFLOP_PER_IMAGE = 1304.2  # ViT-L @518 (torch.utils.flop_counter on the reference model)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--encoder", default="vitl")
    ap.add_argument("--size", type=int, default=518)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--precision", choices=["int8", "fp16"], default="int8")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-only", action="store_true", help="print the per-operation profile and exit")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def model_path(encoder: str, rank: int, world: int) -> Path:
    """Seeded random-init weights (seed 0, N(0,0.02)) as a .dav2 file, written
    once per node (rank 0 writes, the others wait at the barrier)."""
    from dav2_b200 import dav2file

    path = Path(tempfile.gettempdir()) / f"dav2_bench_{encoder}_seed0.dav2"
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        dav2file.write_dav2(tmp, dav2file.random_state_dict(encoder, seed=0), encoder)
        tmp.rename(path)
    return path


def images(n, size, seed0):
    import numpy as np

    return np.stack([np.random.default_rng(seed0 + i).integers(0, 256, (size, size, 3), dtype=np.uint8)
                     for i in range(n)])


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        rows = [l.split(",") for l in Path(self.file.name).read_text().splitlines() if l.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def int8_peak_tops(torch):
    """Dense int8 tensor throughput of this GPU: cuBLAS s8 x s8 -> s32 via
    torch._int_mm, 8192^3, best of 10 (burst)."""
    n = 8192
    a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def f16_peak_tflops():
    """Dense 16-bit tensor peak for an operation timed inside a long step:
    MEASURED_PEAKS.json (driver-written) sustained bf16 figure, else the
    pool's stated fallback."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            d = json.loads(f.read_text())
            for k in ("bf16_tflops_sustained", "bf16_tflops"):
                if d.get(k):
                    return float(d[k]), f"MEASURED_PEAKS.json {k} (of measured)"
        except (ValueError, OSError):
            pass
    return 1400.0, "fallback 1.4 PFLOP/s sustained bf16 (of fallback; MEASURED_PEAKS.json absent)"


def hbm_peak_gbs():
    """HBM copy bandwidth: MEASURED_PEAKS.json (driver-written) else the pool's
    stated fallback."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        try:
            d = json.loads(f.read_text())
            if d.get("hbm_gbs"):
                return float(d["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
        except (ValueError, OSError):
            pass
    return 6650.0, "fallback 6.65 TB/s (of fallback; MEASURED_PEAKS.json absent)"


def op_bytes(encoder, batch, size, int8):
    """Algorithmic HBM bytes per launch of the bandwidth-bound operations the
    executor profiles by name: every tensor read once and written once."""
    from dav2_b200.dav2file import ARCH

    d, heads, blocks, _, f, oc = ARCH[encoder]
    p = size // 14
    r = batch * (p * p + 1)
    code = 1 if int8 else 2  # int8 codes (+ f32 row scale) or f16 values
    out = {
        "ln1": r * d * 4 + r * d * code + (r * 4 if int8 else 0),
        "ln2": r * d * 4 + r * d * code + (r * 4 if int8 else 0),
    }
    if int8:
        out["quantize hidden"] = r * 4 * d * 2 + r * 4 * d + r * 4
        out["quantize attention"] = r * d * 2 + r * d + r * 4
    # align-corners bilinear on channels-last f16 maps (channels padded to 64)
    fp = -(-f // 64) * 64
    l4 = (p + 2 - 3) // 2 + 1
    sizes = [(l4, p), (p, 2 * p), (2 * p, 4 * p), (4 * p, 8 * p)]
    out["fusion resize"] = sum(batch * (a * a + b * b) * fp * 2 for a, b in sizes) / len(sizes)
    hp = -(-(f // 2) // 64) * 64
    out["head resize"] = batch * ((8 * p) ** 2 + size * size) * hp * 2
    return out


def op_work(encoder, batch, size):
    """Algorithmic tensor ops per launch of each GEMM-family operation name
    (2*M*N*K), for the operations the executor profiles by name."""
    from dav2_b200.dav2file import ARCH

    d, heads, blocks, _, f, oc = ARCH[encoder]
    p = size // 14
    t = p * p + 1
    r = batch * t
    return {
        "qkv": 2 * r * 3 * d * d, "proj": 2 * r * d * d, "fc1": 2 * r * 4 * d * d, "fc2": 2 * r * 4 * d * d,
        "attention": batch * heads * 4 * t * t * 64,
    }


def cpu_baseline(encoder, size, seconds_cap=40.0):
    """The reference's CPU path (PyTorch CPU fp32 forward, oracle/torch_graph.py)
    on one image with all host threads."""
    import numpy as np
    import torch

    import torch_graph
    from dav2_b200 import dav2file

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = torch_graph.to_torch(dav2file.random_state_dict(encoder, seed=0))
    x = np.random.default_rng(0).standard_normal((1, 3, size, size)).astype(np.float32)
    t0 = time.perf_counter()
    torch_graph.forward(w, x, encoder)
    first = time.perf_counter() - t0
    best = first
    if first * 2 < seconds_cap:
        t0 = time.perf_counter()
        torch_graph.forward(w, x, encoder)
        best = min(best, time.perf_counter() - t0)
    return {"value": round(1.0 / best, 4), "unit": "images/s", "cores": threads, "kind": "port",
            "sample": f"1 image {encoder} {size}x{size}, fp32 PyTorch-CPU restatement of the reference forward "
                      f"(oracle/torch_graph.py), best of {1 if first * 2 >= seconds_cap else 2} runs"}


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    import numpy as np
    import torch

    import torch_graph
    from dav2_b200 import dav2file

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = torch_graph.to_torch(dav2file.random_state_dict(args.encoder, seed=0))
    x = np.random.default_rng(0).standard_normal((1, 3, args.size, args.size)).astype(np.float32)
    for _ in range(args.warmup):
        torch_graph.forward(w, x, args.encoder)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        torch_graph.forward(w, x, args.encoder)
    dt = time.perf_counter() - t0
    value = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "images/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.encoder} {args.size}x{args.size} full graph, 1 image per step (bounded "
                               f"sample of the 64-image batch)", "precision": "fp32 (the reference CPU path)",
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 4), "unit": "images/s", "cores": threads, "kind": "port",
                         "sample": "1 image per step, PyTorch-CPU fp32 restatement of the reference forward "
                                   "(oracle/torch_graph.py)"},
        "e2e": {"value": round(value, 4), "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import numpy as np
    import torch

    import dav2_b200
    from dav2_b200 import capi

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    lib = dav2_b200.load()
    path = model_path(args.encoder, rank, world)
    barrier()
    flags = capi.FLAGS[args.precision]
    opts = capi.CreateOptions(ctypes.sizeof(capi.CreateOptions), 1, capi.ENCODERS[args.encoder], local, flags, None)
    ctx = ctypes.c_void_p()
    rc = lib.dav2_create(str(path).encode(), ctypes.byref(opts), ctypes.byref(ctx))
    if rc != 0:
        raise RuntimeError(f"dav2_create: {lib.dav2_last_error().decode()}")

    B, S = args.batch, args.size
    host = images(B, S, seed0=rank * B)
    pinned_in = torch.from_numpy(host).pin_memory()
    dev_in = pinned_in.cuda()
    pinned_out = torch.empty((B, S, S), dtype=torch.float32).pin_memory()
    dev_out = torch.empty((B, S, S), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > 126 MB L2

    def device_step():
        r = lib.dav2_infer_device_bgr8_batch(ctx, dev_in.data_ptr(), B, S, S, S * 3, S * S * 3, S, dev_out.data_ptr(),
                                             ctypes.c_void_p(stream.cuda_stream))
        if r != 0:
            raise RuntimeError(f"dav2_infer_device_bgr8_batch: {lib.dav2_last_error().decode()}")

    def host_step():
        r = lib.dav2_infer_bgr8_batch(ctx, pinned_in.data_ptr(), B, S, S, S * 3, S * S * 3, S,
                                      pinned_out.data_ptr(), B * S * S)
        if r != 0:
            raise RuntimeError(f"dav2_infer_bgr8_batch: {lib.dav2_last_error().decode()}")

    # per-operation live profile (also builds the plan)
    buf = ctypes.create_string_buffer(1 << 20)
    if lib.dav2_profile_operations(ctx, B, S, S, buf, len(buf)) != 0:
        raise RuntimeError(lib.dav2_last_error().decode())
    prof = json.loads(buf.value.decode())
    if args.profile_only:
        if rank == 0:
            agg = {}
            for o in prof["ops"]:
                a = agg.setdefault(o["name"], [0, 0.0])
                a[0] += 1
                a[1] += o["ms"]
            for name, (n, ms) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
                print(f"{name:28s} {n:4d} {ms:9.3f} ms {100 * ms / prof['total_ms']:5.1f}%")
            print("total", prof["total_ms"])
        return

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            device_step()
        torch.cuda.synchronize()
        launches0 = ctypes.c_uint64()
        lib.dav2_get_kernel_launch_count(ctx, ctypes.byref(launches0))
        barrier()
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(args.steps):
                flush.zero_()
                device_step()
            end.record(stream)
            torch.cuda.synchronize()
        barrier()
        dev_ms = max_over_ranks(start.elapsed_time(end))
        launches1 = ctypes.c_uint64()
        lib.dav2_get_kernel_launch_count(ctx, ctypes.byref(launches1))
        # end to end through the host-buffer entry point
        host_step()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host_step()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        barrier()
    out = pinned_out.numpy()
    assert np.isfinite(out).all()

    value = B * world * args.steps / (dev_ms * 1e-3)
    e2e = B * world * args.steps / e2e_s
    line = None
    if rank == 0:
        peak = int8_peak_tops(torch) if args.precision == "int8" else None
        work = op_work(args.encoder, B, S)
        agg = {}
        for o in prof["ops"]:
            a = agg.setdefault(o["name"], [0, 0.0])
            a[0] += 1
            a[1] += o["ms"]
        shares = {k: round(v[1] / prof["total_ms"], 4) for k, v in sorted(agg.items(), key=lambda kv: -kv[1][1])}
        f16_peak, f16_src = f16_peak_tflops()
        traffic_by_op = {}
        tfile = ROOT / "profiles" / "traffic.txt"
        if tfile.exists():
            for l in tfile.read_text().splitlines():
                if l.startswith(f"{args.encoder} b{B} ") and ":" in l:
                    traffic_by_op[l.split(":")[0].split(" ", 2)[2]] = int(l.split(":")[1].split()[0])

        def roofline_of(name):
            per_launch_ms = agg[name][1] / agg[name][0]
            achieved = work[name] / (per_launch_ms * 1e-3) / 1e12
            int8 = args.precision == "int8" and name != "attention"
            pk = peak if int8 else f16_peak
            return {"bound": "tensor",
                    "kernel": f"attention_tc f16 ({name})" if name == "attention" else
                              f"gemm_tc {'int8' if int8 else 'f16'} ({name})",
                    "achieved": round(achieved, 1), "peak": round(pk, 1) if pk else None, "unit": "TFLOP/s",
                    "frac": round(achieved / pk, 3) if pk else None, "traffic": traffic_by_op.get(name),
                    "peak_source": ("cuBLAS int8 GEMM (torch._int_mm 8192^3, burst) measured in this run; "
                                    "MEASURED_PEAKS.json has no int8 figure") if int8 else f16_src,
                    "per_launch_ms": round(per_launch_ms, 4), "launches_per_step": agg[name][0]}

        hbm_pk, hbm_src = hbm_peak_gbs()
        mem = op_bytes(args.encoder, B, S, args.precision == "int8")
        hbm_ops = {}
        for k, nbytes in mem.items():
            if k in agg:
                gbs = nbytes / (agg[k][1] / agg[k][0] * 1e-3) / 1e9
                hbm_ops[k] = {"achieved": round(gbs, 1), "peak": hbm_pk, "unit": "GB/s", "frac": round(gbs / hbm_pk, 3),
                              "bytes_per_launch": int(nbytes)}
        known = [k for k in shares if k in work]
        dom = max(known, key=lambda k: agg[k][1])
        roof = roofline_of(dom)
        roof["ops"] = {k: {kk: v for kk, v in roofline_of(k).items() if kk in ("achieved", "peak", "frac")}
                       for k in known}
        roof["hbm_ops"] = hbm_ops
        roof["hbm_peak_source"] = hbm_src
        roof["op_shares"] = shares
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(args.encoder, S)
        clk = clocks.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8" if args.precision == "int8" else "f16",
            "data": "synthetic (random u8 BGR8 images, seeded per image; random-init N(0,0.02) weights)",
            "config": {"workload": f"{args.encoder} {S}x{S} full graph (GPU preprocessing + encoder + DPT head), "
                                   f"{B} images per GPU per step",
                       "encoder": args.encoder, "image": f"{S}x{S}", "batch_per_gpu": B,
                       "precision": f"{args.precision} (int8 linears/projections/resize layers, f16 attention "
                                    f"and refinement convolutions, f32/s32 accumulation)" if args.precision == "int8"
                       else "fp16",
                       "parallelism": f"replicas x{world} (independent images, no collectives)",
                       "l2": "256 MiB buffer written between timed steps (inside the timed region); per-step "
                             "working set ~15 GB"},
            "e2e": {"value": round(e2e, 2), "unit": "images/s", "h2d_bytes_per_step": int(B * S * S * 3),
                    "d2h_bytes_per_step": int(B * S * S * 4)},
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": {k: clk[k] for k in ("sm_mhz", "sm_max_mhz", "reasons")},
            "gpu_launches": int(launches1.value - launches0.value),
            "effective_tflops": round(value / world * GFLOP_PER_IMAGE / 1e3, 1),
        }
        print(json.dumps(line), flush=True)
    lib.dav2_destroy(ctx)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

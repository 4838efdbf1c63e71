"""Benchmark of the decision.js hot path on B200: requests/sec of BASELINE config 2.

Workload (per GPU, weak scaling): the EmbeddingGemma-300M-architecture encoder (24 layers, d 768, 3 query heads /
1 KV head of 256, GeGLU 1152, q8 group-32 weights, random init, vocab 262144), 64 packed texts x 256 token ids
(uniform over the vocabulary) per step, mean-pooled embeddings out. A request is one text.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

value      device-resident passes (ids and bounds already in HBM; dc_forward_encoder_device), CUDA events on the
           library's stream around each step, L2 flushed (256 MiB write) before each step outside the timed span;
           requests of all ranks / max over ranks of the summed step time.
e2e        the same metric through the public API (Decision.embed_raw: host ids -> pinned -> H2D, forward, D2H of
           the pooled embeddings), host clock, max over ranks.
roofline   the dominant kernel (the tcgen05 dequantizing GEMM): algorithmic flops of its launches / their CUDA-event
           time in the timed region, against the measured sustained bf16 tensor peak.
cpu_baseline  the CPU oracle (C restatement of the reference's WGSL kernels, all host threads) on a bounded sample
           of the same workload, rank 0 at N=1.
--impl reference  times that CPU restatement of the reference as the reference arm (rank 0 only).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TEXTS, TOKENS = 64, 256
WORKLOAD = ("BASELINE config 2: EmbeddingGemma-300M-architecture encoder, random-init, q8 g32 f16 scales, 24 layers, "
            "d768, 3q/1kv heads of 256, GeGLU 1152, vocab 262144; 64 packed texts x 256 tokens per GPU per step, "
            "mean-pooled embeddings")
METRIC, UNIT = "requests/sec", "requests/s"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def recorded_traffic():
    """Per-launch DRAM bytes of the GEMM from the committed ncu summary (profiles/qgemm_*), if present."""
    p = os.path.join(ROOT, "profiles", "qgemm_encoder_config2.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class Clocks:
    """SM clock and throttle-reason samples during the timed region: an NVML polling thread (every ~2 ms, so even a
    short timed region gets many samples), or nvidia-smi at 200 ms when NVML is unavailable. Reads only."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.thread = None
        self.samples, self.reasons, self.max = [], set(), None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(self.device)
        bus = getattr(p, "pci_bus_id", None)
        if bus is not None:
            dom, dev = getattr(p, "pci_domain_id", 0), getattr(p, "pci_device_id", 0)
            for fmt in ("%08x:%02x:%02x.0", "%04x:%02x:%02x.0"):
                try:
                    return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId((fmt % (dom, bus, dev)).encode())
                except pynvml.NVMLError:
                    pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def start(self):
        try:
            nv, h = self._nvml_handle()
        except Exception:
            nv = None
        if nv is not None:
            import threading
            bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                    "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                    "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                    "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
            self.max = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.stop_flag = False

            def run():
                while not self.stop_flag:
                    try:
                        self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.reasons.update(n for n, b in bits.items() if r & b)
                    except Exception:
                        return
                    time.sleep(0.002)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join(timeout=5)
            sm = self.samples
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max,
                    "reasons": sorted(self.reasons), "samples": len(sm), "source": "nvml"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(self.NAMES, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


def cpu_sample(model_dir, n_texts, seed=99):
    """The oracle on n_texts texts of 256 tokens (all host threads): returns (requests/s, seconds, threads)."""
    import __graft_entry__ as ge
    oracle = ge.load_oracle()
    threads = oracle.threads()
    oracle.build()
    from decision_js_b200 import synth
    w = oracle.Weights(model_dir)
    seqs = synth.encoder_requests(n_texts, TOKENS, w.cfg["vocab"], seed=seed)
    t0 = time.perf_counter()
    oracle.encoder_embed(w, np.concatenate(seqs), [len(s) for s in seqs])
    dt = time.perf_counter() - t0
    return n_texts / dt, dt, threads


def reference_arm(args, rank, world):
    if rank != 0:
        return
    import __graft_entry__ as ge
    ge.load_package()
    from decision_js_b200 import synth
    model_dir = synth.cached_model("encoder")
    n_texts = int(os.environ.get("DECISION_REF_TEXTS", "2"))
    for _ in range(args.warmup):
        cpu_sample(model_dir, n_texts, seed=1)
    total, threads = 0.0, 1
    for k in range(args.steps):
        _, dt, threads = cpu_sample(model_dir, n_texts, seed=100 + k)
        total += dt
    value = n_texts * args.steps / total
    sample = f"{n_texts} texts x {TOKENS} tokens through all 24 layers per step (of the {TEXTS}-text GPU step)"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 math",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": TEXTS * args.gpus, "seq_len": TOKENS,
                       "parallelism": "host CPU"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("the reference (TypeScript + WGSL on WebGPU) cannot run here: no JS runtime and no WebGPU/Dawn; "
                     "this arm times the C restatement of its portable WGSL kernels on the host cores")}
    print(json.dumps(line), flush=True)


def sweep(args):
    """the quantized matmul over M in {1,16,64,256,1024,4096} x (N,K) in {(768,768), (1152,768),
    (3072,1024), (8192,3072)}, q8 and q4, through dc_qmatmul (the form it picks). One JSON line per shape. The
    timed unit is a CUDA graph of R back-to-back launches, each on its own copy of the weights, with R copies
    together larger than 3x L2 (so every launch streams its weights from HBM, as the layers of a forward pass
    do): per-launch time = graph time / R, CUDA events, median of `steps` replays after `warmup`. Algorithmic
    GB/s against the measured HBM copy bandwidth for M <= 64, TFLOP/s against the measured bf16 tensor peak for
    larger M."""
    import torch
    import __graft_entry__ as ge
    ge.load_package()
    from decision_js_b200 import synth
    from decision_js_b200._lib import Context
    hbm, tf_burst, tf_sus, src = peaks()
    ctx = Context(int(os.environ.get("LOCAL_RANK", "0")))
    stream = torch.cuda.ExternalStream(ctx.stream)
    l2 = 126 << 20
    only = tuple(int(v) for v in args.only.split(",")) if args.only else None  # M,N,K,bits
    for bits in (8, 4):
        for (N, K) in ((768, 768), (1152, 768), (3072, 1024), (8192, 3072)):
            if only and (only[1], only[2], only[3]) != (N, K, bits):
                continue
            wbytes = N * K * bits // 8 + N * K // 16
            R = max(8, min(512, -(-3 * l2 // wbytes)))
            X0, codes0, S0 = synth.config1_inputs(seed=N + K + bits, M=1, N=N, K=K, bits=bits)
            dW0 = torch.from_numpy(codes0).cuda()
            dS0 = torch.from_numpy(S0.view(np.int16)).cuda()
            # R copies of the same quantized weights (values do not change the timing; copies defeat L2)
            dWs = [dW0.clone() for _ in range(R)]
            dSs = [dS0.clone() for _ in range(R)]
            for M in (1, 16, 64, 256, 1024, 4096):
                if only and M != only[0]:
                    continue
                X = (torch.randn(M, K, generator=torch.Generator().manual_seed(M)) ).half().view(torch.int16).cuda()
                dY = torch.empty((M, N), dtype=torch.int16, device="cuda")
                def run(i):
                    ctx.call("qmatmul", X, dWs[i], dSs[i], dY, M, N, K, bits, 0)
                for i in range(max(args.warmup, 3)):
                    run(i % R)
                ctx.sync()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(g, stream=stream):
                        for i in range(R):
                            run(i)
                    for _ in range(max(args.warmup, 3)):
                        g.replay()
                    times = []
                    for _ in range(args.steps):
                        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        a.record(stream)
                        g.replay()
                        b.record(stream)
                        times.append((a, b))
                    torch.cuda.synchronize()
                us = 1e3 * float(np.median([a.elapsed_time(b) for a, b in times])) / R
                del g
                byts = wbytes + 2 * M * K + 2 * M * N
                flops = 2.0 * M * N * K
                gbs, tfl = byts / (us * 1e-6) / 1e9, flops / (us * 1e-6) / 1e12
                hbm_bound = M <= 64
                line = {"metric": "qmatmul", "bits": bits, "M": M, "N": N, "K": K, "us": us,
                        "GBps": gbs, "TFLOPs": tfl, "bound": "hbm" if hbm_bound else "tensor",
                        "frac": gbs / hbm if hbm_bound else tfl / tf_burst,
                        "peak": hbm if hbm_bound else tf_burst,
                        "peak_source": f"{src} ({'copy' if hbm_bound else 'bf16 burst'})",
                        "timing": f"graph of {R} launches on distinct weight copies ({R * wbytes / 2**20:.0f} MiB > 3x L2)"}
                print(json.dumps(line), flush=True)
            del dWs, dSs
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="BASELINE config 5: the quantized matmul shape sweep")
    ap.add_argument("--only", default="", help="with --sweep: one shape, 'M,N,K,bits' (e.g. for a profiler capture)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.sweep:
        return sweep(args)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    import __graft_entry__ as ge
    pkg = ge.load_package()
    from decision_js_b200 import synth
    from decision_js_b200._lib import K_ATTN, K_NORM, K_OTHER, K_QGEMM, K_QGEMV, check, lib

    if rank == 0:
        model_dir = synth.cached_model("encoder", device=f"cuda:{local}")
    barrier()
    model_dir = synth.cached_model("encoder", device=f"cuda:{local}")
    dec = pkg.Decision.load(model_dir, devices=[local], tokensPerPass=TEXTS * TOKENS)
    mdl = dec.models[0]
    ctx = mdl.ctx
    vocab = int(mdl.cfg("vocab"))
    seqs = synth.encoder_requests(TEXTS, TOKENS, vocab, seed=1000 + rank)
    ids = torch.tensor(np.concatenate(seqs), dtype=torch.int32, device="cuda")
    bounds = torch.tensor([[i * TOKENS, (i + 1) * TOKENS] for i in range(TEXTS)], dtype=torch.int32, device="cuda")
    out = torch.empty((TEXTS, int(mdl.cfg("hidden"))), dtype=torch.float32, device="cuda")
    T = TEXTS * TOKENS
    stream = torch.cuda.ExternalStream(ctx.stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def step():
        check(lib().dc_forward_encoder_device(mdl.h, ids.data_ptr(), bounds.data_ptr(), T, TEXTS, out.data_ptr()))

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    ctx.sync()
    # ---------------- timed region (device-resident)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    clocks = Clocks(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    with torch.cuda.stream(stream):
        for k in range(args.steps):
            flush.zero_()  # L2 flush, outside the timed span
            evs[k][0].record(stream)
            step()
            evs[k][1].record(stream)
    ctx.sync()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    total_ms = sum(a.elapsed_time(b) for a, b in evs)

    # ---------------- per-kernel breakdown: the same steps again with every launch bracketed by CUDA events on
    # the library's stream (the brackets add gaps, so this pass is not the timed one)
    ctx.profile(True)
    with torch.cuda.stream(stream):
        for k in range(args.steps):
            flush.zero_()
            step()
    ctx.sync()
    prof = {k: ctx.profile_read(v) for k, v in
            {"qgemm": K_QGEMM, "qgemv": K_QGEMV, "attention": K_ATTN, "norm": K_NORM, "other": K_OTHER}.items()}
    ctx.profile(False)
    launches = sum(p["launches"] for p in prof.values())

    # ---------------- e2e through the public API
    host_seqs = [np.asarray(s, np.int32) for s in seqs]
    for _ in range(args.warmup):
        dec.embed_raw(host_seqs)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        res = dec.embed_raw(host_seqs)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    barrier()
    assert len(res) == TEXTS and np.isfinite(np.stack(res)).all()

    # ---------------- reduce over ranks
    t = torch.tensor([total_ms, e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms, max_e2e = float(t[0]), float(t[1])
    if rank == 0:
        hbm, tf_burst, tf_sus, src = peaks()
        q = prof["qgemm"]
        achieved = q["flops"] / (q["ms"] * 1e-3) / 1e12 if q["ms"] > 0 else 0.0
        n_q = max(q["launches"], 1)
        attn_flops = 4.0 * TEXTS * TOKENS * TOKENS * 3 * 256 * 24
        kernels = {k: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps}
                   for k, v in prof.items()}
        kernels["qgemm"]["tflops"] = achieved
        if prof["attention"]["ms"] > 0:
            kernels["attention"]["tflops"] = attn_flops * args.steps / (prof["attention"]["ms"] * 1e-3) / 1e12
        traffic = recorded_traffic()
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            n = int(os.environ.get("DECISION_CPU_TEXTS", "4"))
            v, dt, threads = cpu_sample(model_dir, n)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"{n} texts x {TOKENS} tokens through all 24 layers ({dt:.1f} s) with the C oracle"}
        line = {
            "metric": METRIC, "value": TEXTS * world * args.steps / (max_ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random-init weights in the reference's format, uniform token ids)",
            "config": {"workload": WORKLOAD, "global_batch": TEXTS * world, "seq_len": TOKENS,
                       "tokens_per_gpu_step": T, "parallelism": f"dp{world} (replicas, requests sharded, no collective)",
                       "l2": "flushed before each timed step (256 MiB write, outside the timed span)"},
            "roofline": {"bound": "tensor", "kernel": "qgemm (TMA + tcgen05 dequantizing GEMM, prefill form)",
                         "achieved": achieved, "peak": tf_sus, "unit": "TFLOP/s", "frac": achieved / tf_sus,
                         "peak_source": f"{src} bf16 sustained", "frac_of_burst": achieved / tf_burst,
                         "traffic": traffic, "algorithmic_bytes_per_launch": q["bytes"] / n_q,
                         "flops_per_launch": q["flops"] / n_q, "launches": q["launches"]},
            "kernels": kernels,
            "cpu_baseline": cpu,
            "e2e": {"value": TEXTS * world * args.steps / max_e2e, "unit": UNIT,
                    "h2d_bytes_per_step": T * 4 + TEXTS * 8, "d2h_bytes_per_step": TEXTS * 768 * 4},
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    dec.destroy()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the decision.js hot path on B200: requests/sec of BASELINE config 2 (the default line).

Workload (per GPU, weak scaling): the EmbeddingGemma-300M-architecture encoder (24 layers, d 768, 3 query heads /
1 KV head of 256, GeGLU 1152, q8 group-32 weights, random init, vocab 262144), 64 packed texts x 256 token ids
(uniform over the vocabulary) per step, mean-pooled embeddings out. A request is one text. `--config 3` and
`--config 4` measure the two decoder configurations the same way (a request is one tree, 512 or 1024 tokens: a
trunk and three 4-token question branches, each read out over 10 answer ids).

  python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--config 2|3|4]
  python bench.py --sweep [--only M,N,K,bits]

value      device-resident passes (inputs already in HBM; dc_forward_encoder_device / dc_forward_decoder_device),
           CUDA events on the library's stream around each step, L2 flushed (256 MiB write) before each step
           outside the timed span; requests of all ranks / max over ranks of the summed step time.
e2e        the same metric through the public API (Decision.embed_raw / Decision.run: host ids -> pinned -> H2D,
           forward, D2H of the pooled embeddings or readout logits), host clock, max over ranks.
e2e (N>1)  one global batch of requests x N through the public API sharded over the ranks (multi.run_sharded: each
           rank runs its token-balanced shard, the results are gathered on every host in request order), so the
           host gather is inside the timed span.
roofline   the dominant kernel (the tcgen05 dequantizing GEMM): algorithmic flops of its launches / their CUDA-event
           time, against the measured bf16 tensor peak: the burst figure when the timed region ran at the maximum
           SM clock, the sustained (power-capped) one otherwise. The per-kernel times (`kernels`, and the GEMM's
           time behind `roofline.achieved`) come from a second, event-bracketed pass of the same steps that runs
           every launch directly (no CUDA graph), so their sum exceeds the graph-replayed step time; the shares are
           indicative.
matmul     the decode-shape and BASELINE config 1 matmuls timed as --sweep times them (a CUDA graph of launches on
           weight copies larger than L2): q8/q4 1 x 8192 x 3072 and q8 16/64 x 8192 x 3072 in algorithmic GB/s
           against the measured HBM copy bandwidth, q8 256 x 1152 x 768 in TFLOP/s.
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


class EncoderLoad:
    """BASELINE config 2 (the default line): the EmbeddingGemma-300M-architecture encoder, 64 packed texts x 256
    tokens per GPU per step, mean-pooled embeddings out; a request is one text."""
    config = 2
    requests, tokens, layers = 64, 256, 24
    workload = ("BASELINE config 2: EmbeddingGemma-300M-architecture encoder, random-init, q8 g32 f16 scales, 24 "
                "layers, d768, 3q/1kv heads of 256, GeGLU 1152, vocab 262144; 64 packed texts x 256 tokens per GPU "
                "per step, mean-pooled embeddings")

    @classmethod
    def model_dir(cls, device="cpu"):
        from decision_js_b200 import synth
        return synth.cached_model("encoder", device=device)

    def __init__(self, pkg, local, rank):
        import torch
        from decision_js_b200 import synth
        from decision_js_b200._lib import check, lib
        self._check, self._lib = check, lib
        self.dec = pkg.Decision.load(self.model_dir(f"cuda:{local}"), devices=[local],
                                     tokensPerPass=self.requests * self.tokens)
        self.mdl = self.dec.models[0]
        vocab, self.hidden = int(self.mdl.cfg("vocab")), int(self.mdl.cfg("hidden"))
        self.seqs = [np.asarray(s, np.int32) for s in
                     synth.encoder_requests(self.requests, self.tokens, vocab, seed=1000 + rank)]
        self.T = self.requests * self.tokens
        self.ids = torch.tensor(np.concatenate(self.seqs), dtype=torch.int32, device="cuda")
        self.bounds = torch.tensor([[i * self.tokens, (i + 1) * self.tokens] for i in range(self.requests)],
                                   dtype=torch.int32, device="cuda")
        self.out = torch.empty((self.requests, self.hidden), dtype=torch.float32, device="cuda")
        self.h2d = self.T * 4 + self.requests * 8
        self.d2h = self.requests * self.hidden * 4
        self.attn_flops = 4.0 * self.T * self.tokens * 3 * 256 * self.layers  # QK^T and PV, all keys visible

    def device_step(self):
        self._check(self._lib().dc_forward_encoder_device(self.mdl.h, self.ids.data_ptr(), self.bounds.data_ptr(),
                                                          self.T, self.requests, self.out.data_ptr()))

    def e2e_step(self):
        res = self.dec.embed_raw(self.seqs)
        assert len(res) == self.requests and np.isfinite(np.stack(res)).all()

    def global_batch(self, world):
        """The same requests x world texts on every rank, with their token counts (for the sharded e2e)."""
        vocab = int(self.mdl.cfg("vocab"))
        seqs = [np.asarray(s, np.int32) for s in
                synth_mod().encoder_requests(self.requests * world, self.tokens, vocab, seed=2000)]
        return seqs, [len(s) for s in seqs]

    def api_call(self, batch):
        return self.dec.embed_raw(batch)

    @classmethod
    def cpu_sample(cls, n, seed=99):
        """The C oracle on n texts of the workload (all host threads): (requests/s, seconds, threads, sample)."""
        import __graft_entry__ as ge
        oracle = ge.load_oracle()
        oracle.build()
        from decision_js_b200 import synth
        w = oracle.Weights(cls.model_dir())
        seqs = synth.encoder_requests(n, cls.tokens, w.cfg["vocab"], seed=seed)
        t0 = time.perf_counter()
        oracle.encoder_embed(w, np.concatenate(seqs), [len(s) for s in seqs])
        dt = time.perf_counter() - t0
        return n / dt, dt, oracle.threads(), (f"{n} texts x {cls.tokens} tokens through all {cls.layers} layers "
                                               f"({dt:.1f} s) with the C oracle")


class DecoderLoad:
    """BASELINE configs 3 and 4: causal prefill of packed D13BEngine trees (a trunk and three 4-token question
    branches per request), next-token logits read at the three question positions over a 10-token answer subset;
    a request is one tree."""
    PRESETS = {
        3: dict(requests=32, tokens=512, layers=28, sample_layers=4, over={},
                workload=("BASELINE config 3: 0.6B dense decoder, random-init, q8 g32 f16 scales, 28 layers, d1024, "
                          "16q/8kv heads of 128, SwiGLU 3072, vocab 151936; 32 requests x 512 tokens (causal, 3 "
                          "questions each, 10 answer ids) per GPU per step")),
        4: dict(requests=16, tokens=1024, layers=32, sample_layers=2,
                over=dict(hidden=3072, intermediate=8192, heads=24, kv_heads=8, vocab=65536, eps=1e-5, layers=32,
                          bits=4),
                workload=("BASELINE config 4: 3B dense decoder, random-init, q4 g32 f16 scales, 32 layers, d3072, "
                          "24q/8kv heads of 128, SwiGLU 8192, vocab 65536; 16 requests x 1024 tokens (causal, 3 "
                          "questions each, 10 answer ids) per GPU per step")),
    }

    def __init__(self, pkg, local, rank, config):
        import torch
        from decision_js_b200 import forest, synth
        from decision_js_b200._lib import check, lib
        self._check, self._lib = check, lib
        p = self.PRESETS[config]
        self.config, self.workload = config, p["workload"]
        self.requests, self.tokens, self.layers = p["requests"], p["tokens"], p["layers"]
        self.dec = pkg.Decision.load(self.model_dir(config, device=f"cuda:{local}"), devices=[local],
                                     tokensPerPass=self.requests * self.tokens)
        self.mdl = self.dec.models[0]
        vocab = int(self.mdl.cfg("vocab"))
        heads, D = int(self.mdl.cfg("heads")), int(self.mdl.cfg("head_dim"))
        self.trees = synth.decoder_trees(self.requests, self.tokens, vocab, seed=1000 + rank)
        ids, pos, rng, leaves, leaf_ids = forest(self.trees)
        flat = np.array(leaf_ids, np.int32)
        self.T, self.L, self.nids = int(ids.size), int(leaves.size), int(flat.shape[1])
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.ids, self.pos, self.rng, self.leaves, self.flat = dev(ids), dev(pos), dev(rng), dev(leaves), dev(flat)
        self.out = torch.empty((self.L, self.nids), dtype=torch.float32, device="cuda")
        self.h2d = self.T * (4 + 4 + 16) + self.L * 4 + self.L * self.nids * 4
        self.d2h = self.L * self.nids * 4
        visible = float(((rng[:, 1] - rng[:, 0]) + (rng[:, 3] - rng[:, 2])).sum())
        self.attn_flops = 4.0 * heads * D * visible * self.layers  # QK^T and PV over the visible keys only

    @classmethod
    def model_dir(cls, config, device="cpu", layers=None):
        from decision_js_b200 import synth
        over = dict(cls.PRESETS[config]["over"])
        if layers is not None:
            over["layers"] = layers
        return synth.cached_model("decoder", device=device, **over)

    def device_step(self):
        self._check(self._lib().dc_forward_decoder_device(
            self.mdl.h, self.ids.data_ptr(), self.pos.data_ptr(), self.rng.data_ptr(), self.T,
            self.leaves.data_ptr(), self.flat.data_ptr(), self.L, self.nids, self.out.data_ptr()))

    def e2e_step(self):
        res = self.dec.run(self.trees)
        assert len(res) == self.requests and all(np.isfinite(s).all() for r in res for s in r)

    def global_batch(self, world):
        """The same requests x world trees on every rank, with their token counts (for the sharded e2e)."""
        vocab = int(self.mdl.cfg("vocab"))
        trees = synth_mod().decoder_trees(self.requests * world, self.tokens, vocab, seed=2000)
        return trees, [len(t["trunk"]) + sum(len(b) for b in t["branches"]) for t in trees]

    def api_call(self, batch):
        return self.dec.run(batch)

    @classmethod
    def cpu_sample(cls, config, n, seed=99, device="cpu"):
        """The C oracle on n requests of the workload through the first `sample_layers` layers of the same
        architecture (all host threads), scaled to all layers by the layer ratio (the embedding gather and the
        readout, a small part, are scaled with them): (requests/s, seconds, threads, sample)."""
        import __graft_entry__ as ge
        from decision_js_b200 import forest, synth
        oracle = ge.load_oracle()
        oracle.build()
        p = cls.PRESETS[config]
        k, L = p["sample_layers"], p["layers"]
        w = oracle.Weights(cls.model_dir(config, device=device, layers=k))  # `device` only writes the weights
        trees = synth.decoder_trees(n, p["tokens"], w.cfg["vocab"], seed=seed)
        ids, pos, rng, leaves, leaf_ids = forest(trees)
        t0 = time.perf_counter()
        oracle.decoder_logits(w, ids, pos, rng, leaves, np.array(leaf_ids, np.int32))
        dt = time.perf_counter() - t0
        full = dt * L / k
        return n / full, full, oracle.threads(), (
            f"{n} request(s) x {p['tokens']} tokens through {k} of the {L} layers ({dt:.1f} s) with the C oracle, "
            f"scaled by {L}/{k}")


def synth_mod():
    from decision_js_b200 import synth
    return synth


def cpu_sample(config, n, seed=99, device="cpu"):
    return EncoderLoad.cpu_sample(n, seed) if config == 2 else DecoderLoad.cpu_sample(config, n, seed, device)


def reference_arm(args, rank, world):
    if rank != 0:
        return
    import __graft_entry__ as ge
    ge.load_package()
    if args.config == 2:
        requests, tokens, workload = EncoderLoad.requests, EncoderLoad.tokens, EncoderLoad.workload
    else:
        p = DecoderLoad.PRESETS[args.config]
        requests, tokens, workload = p["requests"], p["tokens"], p["workload"]
    n = int(os.environ.get("DECISION_REF_REQUESTS", "2" if args.config == 2 else "1"))
    for _ in range(args.warmup if args.config == 2 else 1):
        cpu_sample(args.config, n, seed=1)
    total, threads, sample = 0.0, 1, ""
    for k in range(args.steps):
        _, dt, threads, sample = cpu_sample(args.config, n, seed=100 + k)
        total += dt
    value = n * args.steps / total
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 storage, f32 math",
            "data": "synthetic",
            "config": {"workload": workload, "global_batch": requests * args.gpus, "seq_len": tokens,
                       "parallelism": "host CPU"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"per step: {sample} (of the {requests}-request GPU step)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": ("the reference (TypeScript + WGSL on WebGPU) cannot run here: no JS runtime and no WebGPU/Dawn; "
                     "this arm times the C restatement of its portable WGSL kernels on the host cores")}
    print(json.dumps(line), flush=True)


class MatmulTimer:
    """Per-launch time of dc_qmatmul at one shape: a CUDA graph of R back-to-back launches, each on its own copy of
    the weights, with R copies together larger than 3x L2 (every launch streams its weights from HBM, as the layers
    of a forward pass do); per-launch time = graph time / R, CUDA events on the library's stream, median of `steps`
    replays after `warmup`."""

    def __init__(self, ctx):
        import torch
        from decision_js_b200._lib import lib
        self.ctx = ctx
        lib().dc_static_weights(ctx.h, 1)  # the weights are uploaded before and never written, as in a model pass
        self.stream = torch.cuda.ExternalStream(ctx.stream)
        self.weights = {}

    def load(self, N, K, bits):
        """R device copies of one seeded quantized weight (the values do not change the timing)."""
        import torch
        from decision_js_b200 import synth
        if (N, K, bits) not in self.weights:
            self.weights.clear()
            wbytes = N * K * bits // 8 + N * K // 16
            R = max(8, min(512, -(-3 * (126 << 20) // wbytes)))
            _, codes0, S0 = synth.config1_inputs(seed=N + K + bits, M=1, N=N, K=K, bits=bits)
            dW0 = torch.from_numpy(codes0).cuda()
            dS0 = torch.from_numpy(S0.view(np.int16)).cuda()
            self.weights[(N, K, bits)] = (wbytes, [dW0.clone() for _ in range(R)], [dS0.clone() for _ in range(R)])
        return self.weights[(N, K, bits)]

    def time(self, M, N, K, bits, steps, warmup, direct=False):
        """(us per launch, R, weight bytes per launch). direct: dc_qmatmul_f16 on f16 copies of the weights made
        by dc_dequant (the reference's direct path), with the f16 bytes as the weight bytes."""
        import torch
        wbytes, dWs, dSs = self.load(N, K, bits)
        R = len(dWs)
        X = torch.randn(M, K, generator=torch.Generator().manual_seed(M)).half().view(torch.int16).cuda()
        dY = torch.empty((M, N), dtype=torch.int16, device="cuda")
        if direct:
            W16s = []
            for i in range(R):
                w16 = torch.empty((N, K), dtype=torch.int16, device="cuda")
                self.ctx.call("dequant", dWs[i], dSs[i], w16, N, K, bits)
                W16s.append(w16)
            wbytes = 2 * N * K

            def run(i):
                self.ctx.call("qmatmul_f16", X, W16s[i], dY, M, N, K, 0)
        else:
            def run(i):
                self.ctx.call("qmatmul", X, dWs[i], dSs[i], dY, M, N, K, bits, 0)

        for i in range(max(warmup, 3)):
            run(i % R)
        self.ctx.sync()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(self.stream):
            with torch.cuda.graph(g, stream=self.stream):
                for i in range(R):
                    run(i)
            for _ in range(max(warmup, 3)):
                g.replay()
            times = []
            for _ in range(steps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(self.stream)
                g.replay()
                b.record(self.stream)
                times.append((a, b))
            torch.cuda.synchronize()
        us = 1e3 * float(np.median([a.elapsed_time(b) for a, b in times])) / R
        del g
        return us, R, wbytes

    def line(self, M, N, K, bits, steps, warmup, hbm, tf_burst, src, direct=False):
        us, R, wbytes = self.time(M, N, K, bits, steps, warmup, direct)
        byts = wbytes + 2 * M * K + 2 * M * N
        flops = 2.0 * M * N * K
        gbs, tfl = byts / (us * 1e-6) / 1e9, flops / (us * 1e-6) / 1e12
        hbm_bound = M <= 64
        return {"bits": bits, "M": M, "N": N, "K": K, "us": us, "GBps": gbs, "TFLOPs": tfl,
                "bound": "hbm" if hbm_bound else "tensor", "frac": gbs / hbm if hbm_bound else tfl / tf_burst,
                "peak": hbm if hbm_bound else tf_burst,
                "peak_source": f"{src} ({'copy' if hbm_bound else 'bf16 burst'})",
                "algorithmic_bytes": byts, "flops": flops,
                "timing": f"graph of {R} launches on distinct weight copies ({R * wbytes / 2**20:.0f} MiB > 3x L2)"}


# The matmuls the default line reports beside the requests/s: the q8 decode shape of the HBM target, its q4
# twin, two more decode-range token counts, and BASELINE config 1's single q8 linear.
LINE_MATMULS = [("q8_decode_1x8192x3072", 1, 8192, 3072, 8), ("q8_decode_16x8192x3072", 16, 8192, 3072, 8),
                ("q8_decode_64x8192x3072", 64, 8192, 3072, 8), ("q4_decode_1x8192x3072", 1, 8192, 3072, 4),
                ("q8_config1_256x1152x768", 256, 1152, 768, 8)]


def sweep(args):
    """the quantized matmul over M in {1,16,64,256,1024,4096} x (N,K) in {(768,768), (1152,768),
    (3072,1024), (8192,3072)}, q8 and q4, through dc_qmatmul (the form it picks). One JSON line per shape. The
    timed unit is a CUDA graph of R back-to-back launches, each on its own copy of the weights, with R copies
    together larger than 3x L2 (so every launch streams its weights from HBM, as the layers of a forward pass
    do): per-launch time = graph time / R, CUDA events, median of `steps` replays after `warmup`. Algorithmic
    GB/s against the measured HBM copy bandwidth for M <= 64, TFLOP/s against the measured bf16 tensor peak for
    larger M."""
    if args.direct and not args.only:
        raise SystemExit("bench.py: --direct needs --only M,N,K,bits")
    import __graft_entry__ as ge
    ge.load_package()
    from decision_js_b200._lib import Context
    hbm, tf_burst, tf_sus, src = peaks()
    ctx = Context(int(os.environ.get("LOCAL_RANK", "0")))
    timer = MatmulTimer(ctx)
    only = tuple(int(v) for v in args.only.split(",")) if args.only else None  # M,N,K,bits
    if args.direct:
        # the direct form (dc_qmatmul_f16 on weights dequantized once) on one shape, any N and K
        M, N, K, bits = only
        line = {"metric": "qmatmul_f16", **timer.line(M, N, K, bits, args.steps, args.warmup, hbm, tf_burst, src,
                                                       direct=True),
                "weights": f"f16, dequantized once from q{bits} by dc_dequant"}
        print(json.dumps(line), flush=True)
        ctx.close()
        return
    for bits in (8, 4):
        for (N, K) in ((768, 768), (1152, 768), (3072, 1024), (8192, 3072)):
            if only and (only[1], only[2], only[3]) != (N, K, bits):
                continue
            for M in ((only[0],) if only else (1, 16, 64, 256, 1024, 4096)):
                line = {"metric": "qmatmul", **timer.line(M, N, K, bits, args.steps, args.warmup, hbm, tf_burst, src),
                        "weights": "static (dc_static_weights: a launch starts on its weights while the one before "
                                   "drains)"}
                print(json.dumps(line), flush=True)
            timer.weights.clear()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-matmuls", action="store_true", help="skip the decode/config-1 matmul keys of the line")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4],
                    help="BASELINE config: 2 the encoder (default), 3 the 0.6B q8 decoder, 4 the 3B q4 decoder")
    ap.add_argument("--sweep", action="store_true", help="BASELINE config 5: the quantized matmul shape sweep")
    ap.add_argument("--only", default="", help="with --sweep: one shape, 'M,N,K,bits' (e.g. for a profiler capture)")
    ap.add_argument("--direct", action="store_true",
                    help="with --sweep --only: time the direct form (dc_qmatmul_f16 on f16 weights) on that shape")
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
    from decision_js_b200._lib import K_ATTN, K_NORM, K_OTHER, K_QGEMM, K_QGEMV, lib

    # rank 0 writes the synthetic model first (the others then find it written)
    if rank == 0:
        EncoderLoad.model_dir(f"cuda:{local}") if args.config == 2 else DecoderLoad.model_dir(args.config,
                                                                                                f"cuda:{local}")
    barrier()
    w = EncoderLoad(pkg, local, rank) if args.config == 2 else DecoderLoad(pkg, local, rank, args.config)
    ctx = w.mdl.ctx
    stream = torch.cuda.ExternalStream(ctx.stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        w.device_step()
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
            w.device_step()
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
            w.device_step()
    ctx.sync()
    prof = {k: ctx.profile_read(v) for k, v in
            {"qgemm": K_QGEMM, "qgemv": K_QGEMV, "attention": K_ATTN, "norm": K_NORM, "other": K_OTHER}.items()}
    ctx.profile(False)
    launches = sum(p["launches"] for p in prof.values())

    # ---------------- e2e through the public API: at N > 1 one global batch sharded over the ranks, the results
    # gathered on every host (multi.run_sharded), so the gather is inside the timed span
    if world > 1:
        from decision_js_b200 import multi
        batch, sizes = w.global_batch(world)

        def e2e_step():
            res = multi.run_sharded(batch, sizes, w.api_call)
            assert len(res) == len(batch)
    else:
        e2e_step = w.e2e_step
    for _ in range(args.warmup):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    barrier()

    # ---------------- the decode-shape and config-1 matmuls (rank 0; no collective inside)
    matmuls = None
    if rank == 0 and not args.no_matmuls:
        hbm, tf_burst, tf_sus, src = peaks()
        timer = MatmulTimer(ctx)
        matmuls = {name: timer.line(M, N, K, bits, args.steps, args.warmup, hbm, tf_burst, src)
                   for name, M, N, K, bits in LINE_MATMULS}
        timer.weights.clear()
        lib().dc_static_weights(ctx.h, 0)

    # ---------------- reduce over ranks
    t = torch.tensor([total_ms, e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms, max_e2e = float(t[0]), float(t[1])
    if rank == 0:
        hbm, tf_burst, tf_sus, src = peaks()
        # the burst peak applies when the timed region held the maximum SM clock, the sustained (power-capped)
        # one when the clock sagged under the power cap
        at_max = bool(clk.get("sm_mhz") and clk.get("sm_max_mhz") and clk["sm_mhz"] >= 0.97 * clk["sm_max_mhz"])
        peak = tf_burst if at_max else tf_sus
        peak_src = (f"{src} bf16 {'burst' if at_max else 'sustained'} (timed region median SM clock "
                    f"{clk.get('sm_mhz')} of {clk.get('sm_max_mhz')} MHz)")
        q = prof["qgemm"]
        achieved = q["flops"] / (q["ms"] * 1e-3) / 1e12 if q["ms"] > 0 else 0.0
        n_q = max(q["launches"], 1)
        kernels = {k: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps}
                   for k, v in prof.items()}
        kernels["qgemm"]["tflops"] = achieved
        if prof["attention"]["ms"] > 0:
            kernels["attention"]["tflops"] = w.attn_flops * args.steps / (prof["attention"]["ms"] * 1e-3) / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            n = int(os.environ.get("DECISION_CPU_REQUESTS", "4" if args.config == 2 else "1"))
            v, dt, threads, sample = cpu_sample(args.config, n, device=f"cuda:{local}")
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
        line = {
            "metric": METRIC, "value": w.requests * world * args.steps / (max_ms * 1e-3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random-init weights in the reference's format, uniform token ids)",
            "config": {"workload": w.workload, "global_batch": w.requests * world, "seq_len": w.tokens,
                       "tokens_per_gpu_step": w.T, "parallelism": f"dp{world} (replicas, requests sharded, no collective)",
                       "l2": "flushed before each timed step (256 MiB write, outside the timed span)"},
            "roofline": {"bound": "tensor", "kernel": "qgemm (TMA + tcgen05 dequantizing GEMM, prefill form)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": peak_src, "frac_of_burst": achieved / tf_burst,
                         "frac_of_sustained": achieved / tf_sus,
                         "traffic": recorded_traffic() if args.config == 2 else None,
                         "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum, mean over the four "
                                            "GEMM launches of one encoder layer (profiles/qgemm_encoder_config2.md)"
                                            if args.config == 2 else None),
                         "algorithmic_bytes_per_launch": q["bytes"] / n_q,
                         "flops_per_launch": q["flops"] / n_q, "launches": q["launches"],
                         "timing": "event-bracketed, non-graph pass of the same steps (see kernels)"},
            "kernels": kernels,
            "kernels_timing": ("a second pass of the same steps with every launch bracketed by CUDA events and run "
                               "directly (no CUDA graph): the sum exceeds the timed step, shares are indicative"),
            "matmul": matmuls,
            "cpu_baseline": cpu,
            "e2e": {"value": w.requests * world * args.steps / max_e2e, "unit": UNIT,
                    "h2d_bytes_per_step": w.h2d, "d2h_bytes_per_step": w.d2h},
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    w.dec.destroy()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

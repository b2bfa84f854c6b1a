"""Benchmark: JumpReLU SAE fwd + bwd + Adam tokens/s on B200.

Workload (N = 1): d_in = 1536, F = 49152 (32x), one 32768-token microbatch of
bf16 synthetic superposition activations (50 of 49152 unit directions per
token, Exponential(1) magnitudes, N(0, 0.05^2) noise, per-token norm
LogNormal(log 60, 0.4)), K = 50, lambda = 1e-3, mu = 1e-2, lr = 2e-4, fp32
master weights and Adam state. Thresholds are calibrated once (untimed) so
that the mean L0 is ~50, the trained-like state the metric is quoted at, and
a proportional threshold nudge after every step (the trainer's L0
controller) keeps it there.

A step is the reference loop body: forward, backward, global clip, Adam with
the fused decoder/encoder renormalisation, with the loop's stats read-back
before the optimizer step.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
                    [--workload atlas|sharded|inference] [--layers 35]

Under torchrun every rank trains its own SAE (one layer per GPU, the atlas
layout): no data-path collective, weak scaling; the timing is the max over
ranks. `--layers 35` runs the 35-layer atlas configuration instead (layers
round-robin over the GPUs, K timed steps per layer). `--workload sharded`
trains one wide SAE (d_in = 4096, F = 131072, K = 64, LogNormal(log 80, 0.4)
norms) with its dictionary split over the ranks and three cross-rank sums per
step (strong scaling), with a per-phase time breakdown. `--impl reference`
times the reference's fp32 CPU step (its torch-operator restatement in
oracle/torch_step.py) on a bounded sample on this host's cores (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT, ROOT / "event-aware-sae-trainer_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

METRIC = "SAE fwd+bwd+Adam tokens/s at d=1536×49152 L0≈50; % bf16 TC / HBM peak"
PUBLISHED_TOK_S = 250_000.0   # reference README: 250k-273k tokens/s (H100), same metric/config
D_IN, N_FEAT, TOKENS, K_TARGET = 1536, 49152, 32768, 50
LAMBDA, MU, LR = 1e-3, 1e-2, 2e-4
NORM_MU, NORM_SIGMA = math.log(60.0), 0.4
POOL_BATCHES = 4
# DRAM bytes (read + write) per launch of the tile GEMMs at d=1536, F=49152, 32768
# tokens. Encoder storing pre at the entries only (the default): a one-pass ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum) of a 32768-token launch of
# this bench. Encoder storing all of pre, and the grad_feat GEMM: a 4096-token
# launch scaled by 8 (their traffic is dominated by the [F, B] pre tensor, which
# grows with the tokens).
TRAFFIC_ENCODER_GEMM = 1.533931520e9 + 0.630690048e9
TRAFFIC_ENCODER_GEMM_FULL_PRE = 8 * (0.204492e9 + 0.418109e9)
TRAFFIC_GRAD_GEMM = 8 * (0.604495e9 + 0.014044e9)
WORKLOAD = ("d_in=1536 F=49152 32768-token microbatch, L0~50, bf16 activations / "
            "fp32 master+Adam (Gemma-4-E2B residual shape)")


def _peaks():
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"],
                "bf16_sustained": d["bf16_tflops_sustained"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "src": "fallback"}


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    read every 10 ms on a side thread (read-only queries), so that a timed
    region of a few tens of milliseconds still gets samples; nvidia-smi
    (-lms 200) where NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int, period_s: float = 0.01):
        self.index = index
        self.period = period_s
        self.proc = None
        self.thread = None
        self.rows = []          # (sm_mhz, sm_max_mhz, {reason names})
        self.error = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = getattr(torch.cuda.get_device_properties(self.index), "uuid", None)
        if uuid is not None:
            for key in (f"GPU-{uuid}", f"GPU-{uuid}".encode()):
                try:
                    return pynvml, pynvml.nvmlDeviceGetHandleByUUID(key)
                except Exception:
                    pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _sample(self, nv, h):
        bits = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.rows.append((float(sm), float(smax), {k for k, b in bits.items() if r & b}))

    def sample(self):
        """One sample from the calling thread (e.g. once the timed work is
        queued and the GPU is still running it)."""
        if getattr(self, "nvml", None) is not None:
            try:
                self._sample(*self.nvml)
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"

    def _poll(self, nv, h):
        try:
            while not self.stop.is_set():
                self._sample(nv, h)
                self.stop.wait(self.period)
        except Exception as e:      # reported in the summary
            self.error = f"{type(e).__name__}: {e}"

    def __enter__(self):
        import threading
        self.stop = threading.Event()
        try:
            nv, h = self._nvml_handle()
            self.nvml = (nv, h)
            # one sample from this thread as the region starts and one as it
            # ends, so that a region shorter than the poll thread's first
            # wake-up still has a record
            self._sample(nv, h)
            self.thread = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.thread.start()
            return self
        except Exception as e:
            self.error = f"{type(e).__name__}: {e}"
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            try:
                self._sample(*self.nvml)
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for line in (out or "").strip().splitlines():
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9 and p[1].replace(".", "").isdigit():
                    self.rows.append((float(p[1]), float(p[2]),
                                      {n for i, n in enumerate(self.NAMES) if p[5 + i] == "Active"}))
        return False

    def summary(self):
        src = "nvml" if self.thread is not None else "nvidia-smi"
        if self.error:
            src += f" ({self.error})"
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "source": src}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted(set().union(*(r[2] for r in self.rows))),
                "samples": len(self.rows), "source": src}


# ------------------------------------------------------------- CPU reference
def host_threads() -> int:
    """Cores this process may run on (its affinity set)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


CPU_SAMPLE_TOKENS = 2048


class CpuReferenceSampler:
    """The reference trainer's fp32 CPU step (oracle/torch_step.py: its torch-
    operator restatement, pinned to the reference's own outputs) on a bounded
    sample of the 32768-token workload, timed on the host cores.

    One sample = 1/k of one optimizer step (k = 32768 / S): the forward and
    backward of one S-token microbatch over the whole dictionary (exact
    gradient accumulation makes the step k such microbatches) plus the clip
    norm, Adam and both renorms over 1/k of the features (those are passes
    over the parameters, linear in their count). A sample's tokens/s is S over
    its measured time: nothing is extrapolated. All host threads are used
    (torchrun sets OMP_NUM_THREADS=1, so the count is set explicitly), and the
    thresholds are calibrated so that the mean L0 is ~50, as on the GPU."""

    def __init__(self, sample_tokens: int = 0, seed: int = 0):
        import torch

        from oracle import sae_oracle as O
        from oracle.torch_step import TorchReferenceStep
        self.threads = host_threads()
        torch.set_num_threads(self.threads)
        self.S = int(sample_tokens or CPU_SAMPLE_TOKENS)
        self.k = TOKENS // self.S
        self.xs = [torch.from_numpy(O.superposition_batch(self.S, D_IN, N_FEAT, K_TARGET, NORM_MU,
                                                          NORM_SIGMA, seed=seed + i))
                   for i in range(2)]
        self.ref = TorchReferenceStep(D_IN, N_FEAT, seed=0, lr=LR, ste_bandwidth=0.2,
                                      lambda_l0=LAMBDA, al_mu=MU, target_l0=K_TARGET)
        with torch.no_grad():
            self.ref.b_dec.copy_(self.xs[0].mean(0))
            pre = torch.addmm(self.ref.b_enc, self.xs[0][:256] - self.ref.b_dec,
                              self.ref.W_enc.t())
            q = torch.quantile(pre.flatten(), 1.0 - K_TARGET / N_FEAT).item()
            self.ref.log_threshold.fill_(math.log(max(q, 1e-6)))
        self.ref.microbatch(self.xs[0], self.k, True)          # gradients exist for the slice
        self.opt_slice = self.ref.slice_features(N_FEAT // self.k)
        self.description = (
            f"per step: 1/{self.k} of the 32768-token optimizer step, timed as is: one "
            f"{self.S}-token fwd+bwd microbatch over all {N_FEAT} features + clip norm, Adam and "
            f"both renorms over {N_FEAT // self.k} features; the reference's fp32 CPU step "
            "restated with torch CPU operators (oracle/torch_step.py, pinned to the reference's "
            f"own outputs), {self.threads} threads, thresholds calibrated to L0~{K_TARGET}")

    def sample(self, i: int):
        """(seconds, l0) of one sample."""
        t0 = time.perf_counter()
        out = self.ref.microbatch(self.xs[i % 2], self.k, True)
        self.opt_slice.optimizer_step()
        return time.perf_counter() - t0, out["l0"]


CFG1 = dict(d=256, F=8192, tokens=4096)


def cpu_cfg1_full_step(steps: int = 3, warmup: int = 1):
    """One full, unscaled step of the CPU benchmark configuration (d=256,
    F=8192, one 4096-token microbatch, log_threshold = log 0.05, b_dec =
    mean(x)) with the same torch restatement: (tokens/s, ms per step, l0)."""
    import torch

    from oracle import sae_oracle as O
    from oracle.torch_step import TorchReferenceStep
    torch.set_num_threads(host_threads())
    d, F, n = CFG1["d"], CFG1["F"], CFG1["tokens"]
    x = torch.from_numpy(O.superposition_batch(n, d, F, 50, math.log(16.0), 0.3, seed=0))
    ref = TorchReferenceStep(d, F, seed=0, lr=1e-4, ste_bandwidth=0.2, lambda_l0=1e-3,
                             al_mu=1e-2, target_l0=50)
    with torch.no_grad():
        ref.b_dec.copy_(x.mean(0))
        ref.log_threshold.fill_(math.log(0.05))
    times, l0 = [], None
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        out = ref.step([x])
        if i >= warmup:
            times.append(time.perf_counter() - t0)
        l0 = out["l0"]
    t = statistics.mean(times)
    return n / t, t * 1e3, l0


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sampler = CpuReferenceSampler()
    times, l0s = [], []
    for i in range(args.warmup + args.steps):
        t, l0 = sampler.sample(i)
        if i >= args.warmup:
            times.append(t)
            l0s.append(l0)
    step_s = statistics.mean(times)
    value = sampler.S / step_s
    c1_tok_s, c1_ms, c1_l0 = cpu_cfg1_full_step()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "d_in": D_IN, "n_features": N_FEAT,
                   "tokens_per_step": TOKENS, "cpu_sample_tokens": sampler.S,
                   "sample_fraction_of_step": 1.0 / sampler.k, "l0_measured": statistics.mean(l0s)},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": sampler.threads,
                         "kind": "port", "sample": sampler.description, "extrapolated": False},
        "cfg1_full_step": {"workload": "d_in=256 F=8192, one 4096-token microbatch, "
                                       "log_threshold = log 0.05 (one full unscaled "
                                       "fwd+bwd+clip+Adam+renorm step)",
                           "tokens_per_s": c1_tok_s, "ms_per_step": c1_ms, "l0": c1_l0},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# -------------------------------------------------------------- GPU arm
WORKLOADS = {
    # the metric's configuration; under torchrun one layer's SAE per GPU (atlas)
    "atlas": dict(d=D_IN, F=N_FEAT, tokens=TOKENS, k=K_TARGET, norm_mu=NORM_MU,
                  norm_sigma=NORM_SIGMA, lr=LR, description=WORKLOAD),
    # one wide SAE, dictionary split over the GPUs (strong scaling)
    "sharded": dict(d=4096, F=131072, tokens=32768, k=64, norm_mu=math.log(80.0),
                    norm_sigma=0.4, lr=LR,
                    description=("wide SAE d_in=4096 F=131072, 32768-token microbatch, K=64, "
                                 "dictionary split evenly over the GPUs, all-reduce of the "
                                 "partial x_hat + L0 counts, b_dec gradient and clip norm")),
}


INFER = dict(d=2304, F=65536, tokens=65536, k=80, norm_mu=math.log(60.0), norm_sigma=0.4,
             description=("encode + gathered decode inference: d_in=2304 F=65536, 65536 bf16 "
                          "tokens, per-feature log-thresholds ~ N(c, 0.3^2) with c set so the "
                          "mean L0 is ~80 (80 active directions per token)"))


def run_inference(args):
    """Inference configuration: encoder GEMM + JumpReLU gate + gathered decode
    (sae_b200_encode_decode), reported as tokens/s with the encoder GEMM (the
    dominant kernel) against the bf16 tensor peak; the gathered decode is
    reported as a gather rate (its row bytes include L2 hits, so it is not an
    HBM fraction). Under torchrun every rank runs its own replica."""
    import torch
    import torch.distributed as dist

    import sae_b200
    from sae_b200 import _lib as L
    from sae_b200 import atlas

    wl = INFER
    d, F, tokens = wl["d"], wl["F"], wl["tokens"]
    tokens = args.tokens or tokens
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))
    sae = sae_b200.make_shard_sae(d, F, 0, 1, seed=11 + rank, device=dev)
    pool = [sae_b200.superposition_batch(tokens, d, F, wl["k"], wl["norm_mu"], wl["norm_sigma"],
                                         seed=31 + 100 * rank + 7 * i, device=dev)
            for i in range(2)]
    with torch.no_grad():
        sae.b_dec.copy_(pool[0].float().mean(0))
        g = torch.Generator(device=dev).manual_seed(3)
        z = 0.3 * torch.randn(F, generator=g, device=dev)
        lo, hi = math.log(0.01), math.log(100.0)       # bisection on the common scale c
        for _ in range(30):
            c = 0.5 * (lo + hi)
            sae.log_threshold.copy_(z + c)
            _, cnt = sae.reconstruct(pool[0][:8192])
            if cnt.float().mean().item() > wl["k"]:
                lo = c
            else:
                hi = c
        sae.log_threshold.copy_(z + hi)
    x_hat = torch.empty(tokens, d, device=dev)
    counts = torch.empty(tokens, device=dev, dtype=torch.int32)
    model = sae._model_struct(need_shadows=True)
    ws = torch.empty(L.workspace_bytes(tokens, d, F, 0), device=dev, dtype=torch.uint8)
    stream = torch.cuda.current_stream().cuda_stream

    def step(x, out=x_hat):
        L.call("sae_b200_encode_decode", model, L.ptr(x), L.DTYPE_BF16, tokens, L.ptr(ws),
               ws.numel(), L.ptr(out), L.ptr(counts), None, stream)

    for i in range(args.warmup):
        step(pool[i % 2])
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    for e in sum(ev, []):
        e.record()    # creates the CUDA events before the library records them
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0s = []
    launches0 = L.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record()
        for i in range(args.steps):
            L.set_kernel_timer(L.KERNEL_ENCODER_GEMM, ev[i][0], ev[i][1])
            L.set_kernel_timer(L.KERNEL_DECODE, ev[i][2], ev[i][3])
            step(pool[i % 2])
        clocks.sample()
        t1.record()
        torch.cuda.synchronize()
    L.set_kernel_timer(L.KERNEL_ENCODER_GEMM)
    L.set_kernel_timer(L.KERNEL_DECODE)
    launches = L.launch_count() - launches0
    l0 = counts.float().mean().item()
    ms = atlas.max_over_ranks(t0.elapsed_time(t1) / args.steps, device=dev)
    enc_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    dec_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in ev)
    clock = clocks.summary()
    # end to end: every step copies its pinned host batch in and its x_hat (fp32) back
    # to pinned host memory. Double-buffered: batch i+1 goes up on one side stream and
    # x_hat of step i comes down on another while step i+1 computes (PCIe is duplex and
    # each direction has its own copy engine).
    host = [b.cpu().pin_memory() for b in pool]
    out_host = [torch.empty(tokens, d, dtype=torch.float32).pin_memory() for _ in range(2)]
    xb = [torch.empty_like(pool[0]) for _ in range(2)]
    xh = [x_hat, torch.empty_like(x_hat)]
    cur = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(3, args.steps)

    def h2d(j, src):
        up.wait_stream(cur)       # the step that last read xb[j] has been queued before
        with torch.cuda.stream(up):
            xb[j].copy_(src, non_blocking=True)
            in_ready[j].record(up)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    h2d(0, host[0])
    for i in range(e2e_steps):
        j = i % 2
        cur.wait_event(in_ready[j])
        if i + 1 < e2e_steps:
            h2d(1 - j, host[(i + 1) % 2])
        if i >= 2:
            cur.wait_event(out_done[j])    # x_hat of step i - 2 has reached the host
        step(xb[j], xh[j])
        computed[j].record(cur)
        down.wait_event(computed[j])
        with torch.cuda.stream(down):
            out_host[j].copy_(xh[j], non_blocking=True)
            out_done[j].record(down)
    cur.wait_stream(down)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = atlas.max_over_ranks(e0.elapsed_time(e1) / e2e_steps, device=dev)
    if rank == 0:
        peaks = _peaks()
        rows = tokens * l0 * d * 2
        dec_bytes = rows + tokens * d * 4 + tokens * ((F + 31) // 32) * 4 + tokens * l0 * 2
        dec_gbs = dec_bytes / (dec_ms / 1e3) / 1e9
        enc_tf = 2.0 * tokens * d * F / (enc_ms / 1e3) / 1e12
        timed_s = ms * args.steps / 1e3
        long_region = timed_s >= 2.0
        peak = peaks["bf16_sustained"] if long_region else peaks["bf16"]
        line = {
            "metric": "SAE encode+sparse-decode tokens/s at d=2304x65536 L0~80",
            "value": world * tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic superposition activations (seeded, on device)",
            "config": {"workload": wl["description"], "d_in": d, "n_features": F,
                       "tokens_per_step": tokens, "l0_measured": l0,
                       "parallelism": f"replicas only: {world} independent GPU(s)",
                       "l2": "inputs alternate between two 302 MB batches, each larger than "
                             "the 126 MB L2"},
            "roofline": {"bound": "tensor", "kernel": "encoder GEMM + JumpReLU gate "
                                                      "(tc2_tile_gemm<EncodeEpiT>)",
                         "achieved": enc_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": enc_tf / peak,
                         "peak_source": (f"bf16_tflops_sustained ({peaks['src']}): timed region "
                                         f"{timed_s:.2f} s" if long_region else
                                         f"bf16_tflops burst ({peaks['src']}): timed region "
                                         f"{timed_s:.2f} s"),
                         "frac_of_sustained": enc_tf / peaks["bf16_sustained"],
                         "frac_of_burst": enc_tf / peaks["bf16"],
                         "traffic": None, "per_launch_flop": 2.0 * tokens * d * F,
                         "launch_ms": enc_ms},
            "kernels": {"encoder_gemm_ms": enc_ms, "encoder_gemm_tflops": enc_tf,
                        "decode_ms": dec_ms,
                        # algorithmic bytes of the decode over its time: the gathered rows
                        # are partly L2 hits, so this is a gather rate, not DRAM throughput
                        "decode_gather_gbs": dec_gbs,
                        "decode_algorithmic_bytes": dec_bytes,
                        "decode_bytes_note": "B*L0*d*2 gathered bf16 decoder rows + B*d*4 "
                                             "x_hat + B*F/8 mask + B*L0*2 pre values",
                        "decode_row_gbs": rows / (dec_ms / 1e3) / 1e9},
            "clocks": clock,
            "e2e": {"value": world * tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": world * tokens * d * 2,
                    "d2h_bytes_per_step": world * tokens * d * 4},
            "gpu_launches": int(launches),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def calibrate(sae, pool, target_l0, n_features_total):
    """Untimed set-up that mirrors the trainer's preflight (2576-2640): b_dec =
    mean activation, then one uniform threshold at the pre-activation quantile
    that gives the target L0 (the metric is quoted at L0 ~ 50)."""
    import torch

    with torch.no_grad():
        sae.b_dec.copy_(pool[0].float().mean(0))
        probe = pool[0][:4096]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            pre = sae.encode_pre(probe)
        flat = pre.float().flatten()
        idx = torch.randint(0, flat.numel(), (8_000_000,), device=flat.device,
                            generator=torch.Generator(device=flat.device).manual_seed(0))
        q = torch.quantile(flat[idx], 1.0 - target_l0 / n_features_total).item()
        sae.log_threshold.fill_(math.log(max(q, 1e-3)))
        sae.mark_weights_dirty()
    return q


def threshold_nudge(sae, l0, target):
    """The trainer's L0 controller writes log_threshold after every step
    (compute_threshold_nudge, sae_scheduler.py:876-959, applied at
    sae_trainer_rolling.py:3334-3338); here a plain proportional version keeps
    the benchmark at the L0 its metric is quoted for."""
    import torch
    nudge = max(-0.05, min(0.05, 0.5 * math.log(max(l0, 1e-3) / target)))
    with torch.no_grad():
        sae.log_threshold.add_(nudge)


def run_b200(args):
    import torch
    import torch.distributed as dist

    import sae_b200
    from sae_b200 import _lib as L
    from sae_b200 import atlas

    wl = WORKLOADS[args.workload]
    d, F_total, tokens, k_target = wl["d"], wl["F"], wl["tokens"], wl["k"]
    tokens = args.tokens or tokens
    F_total = args.features or F_total
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))
    sharded = args.workload == "sharded"
    if sharded:
        # every rank holds the same batches (replicated input), its slice of the dictionary
        data_seed = 17
        F = F_total // world
        sae = sae_b200.make_shard_sae(d, F_total, rank, world, seed=5, device=dev)
    else:
        data_seed = 17 + 100 * rank      # atlas layout: one layer's SAE per GPU
        F = F_total
        torch.manual_seed(1000 + rank)
        sae = sae_b200.make_sae(d, F, seed=rank).to(dev)
    gen_k = k_target
    if args.l0:
        # an L0 other than the workload's (e.g. early training, before the
        # controller has brought L0 down): the thresholds are calibrated to it
        k_target = args.l0
    pool = [sae_b200.superposition_batch(tokens, d, F_total, gen_k, wl["norm_mu"],
                                         wl["norm_sigma"], seed=data_seed + 7 * i, device=dev)
            for i in range(POOL_BATCHES)]
    sae.ste_bandwidth = args.ste_bandwidth
    thr = calibrate(sae, pool, k_target, F_total)
    opt = sae_b200.B200Adam(sae_b200.reference_param_groups(sae, wl["lr"]), lr=wl["lr"],
                            betas=(0.9, 0.999), sae=sae, renorm=True)
    if sharded:
        fs = sae_b200.ShardedFusedStep(sae, opt, max_tokens=tokens, grad_feat=args.grad_feat,
                                       exchange=args.exchange)
    else:
        fs = sae_b200.FusedStep(sae, opt, max_tokens=tokens, grad_feat=args.grad_feat,
                                pre_store=args.pre_store)

    aux_dead, aux_k = None, 0
    if args.aux_dead > 0 and not sharded:
        # a fixed dead set (the revival controller's aux_dead_mask) and the trainer's
        # legacy eff_k = max(8, min(AUX_K=128, K // 2)) (sae_trainer_rolling.py:449-456)
        gen = torch.Generator(device="cpu").manual_seed(99)
        n_dead = int(args.aux_dead * F)
        aux_dead = torch.randperm(F, generator=gen)[:n_dead].sort().values.to(dev)
        aux_k = max(8, min(128, k_target // 2))

    def step(i, x):
        out = fs.step(x, lambda_l0=LAMBDA, al_mu=MU, target_l0=k_target,
                      wenc_dampen=lambda l0: 1.0, aux_dead=aux_dead, aux_k=aux_k)
        threshold_nudge(sae, out["l0"], k_target)
        return out

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        return atlas.max_over_ranks(v, device=dev)

    # ---------------- device-resident timing (value)
    for i in range(args.warmup):
        step(i, pool[i % POOL_BATCHES])
    n_ev = args.steps
    k_start = [torch.cuda.Event(enable_timing=True) for _ in range(2 * n_ev)]
    k_stop = [torch.cuda.Event(enable_timing=True) for _ in range(2 * n_ev)]
    d_start = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    d_stop = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    a_start = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    a_stop = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    x_start = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    x_stop = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
    for e in k_start + k_stop + d_start + d_stop + a_start + a_stop + x_start + x_stop:
        e.record()
    if sharded:
        fs.timing = {}       # per-phase events of the timed steps (forward, backward, ...)
    barrier()
    launches0 = L.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stats = []
    with ClockSampler(local) as clocks:
        ev0.record()
        for i in range(args.steps):
            L.set_kernel_timer(L.KERNEL_ENCODER_GEMM, k_start[2 * i], k_stop[2 * i])
            L.set_kernel_timer(L.KERNEL_GRAD_GEMM, k_start[2 * i + 1], k_stop[2 * i + 1])
            L.set_kernel_timer(L.KERNEL_DECODE, d_start[i], d_stop[i])
            L.set_kernel_timer(L.KERNEL_ADAM, a_start[i], a_stop[i])
            L.set_kernel_timer(L.KERNEL_EXCHANGE, x_start[i], x_stop[i])
            stats.append(step(i, pool[(args.warmup + i) % POOL_BATCHES]))
        clocks.sample()
        ev1.record()
        barrier()
    for k in (L.KERNEL_ENCODER_GEMM, L.KERNEL_GRAD_GEMM, L.KERNEL_DECODE, L.KERNEL_ADAM,
              L.KERNEL_EXCHANGE):
        L.set_kernel_timer(k)
    phases = None
    if sharded:
        phases = {k: statistics.mean(a.elapsed_time(b) for a, b in v)
                  for k, v in fs.timing.items()}
        fs.timing = None
    launches = (L.launch_count() - launches0)
    dec_ms = statistics.mean(d_start[i].elapsed_time(d_stop[i]) for i in range(n_ev))
    xch_ms = (statistics.mean(x_start[i].elapsed_time(x_stop[i]) for i in range(n_ev))
              if sharded and world > 1 and args.exchange == "p2p" else None)
    adam_ms = statistics.mean(a_start[i].elapsed_time(a_stop[i]) for i in range(n_ev))
    # mean entry counts of the timed microbatches (active, and active + in-band)
    nnz_mean = statistics.mean(s["nnz"] for s in stats)
    pairs_mean = statistics.mean(s.get("csr_pairs", s["nnz"]) for s in stats)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms)
    enc_ms = statistics.mean(k_start[2 * i].elapsed_time(k_stop[2 * i]) for i in range(n_ev))
    grad_ms = statistics.mean(k_start[2 * i + 1].elapsed_time(k_stop[2 * i + 1])
                              for i in range(n_ev))
    clock = clocks.summary()
    status = L.device_status()
    job_tokens = tokens if sharded else world * tokens
    value = job_tokens / (ms / 1e3)   # max-over-ranks time, all ranks' tokens
    l0_timed = statistics.mean(s["l0"] for s in stats)

    # ---------------- end to end from host memory (e2e)
    host = [b.cpu().pin_memory() for b in pool]
    side = torch.cuda.Stream(device=dev)
    bufs = [torch.empty_like(pool[0]) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(3, args.steps)    # the same K steps as the device-resident timing

    def h2d(j, src):
        with torch.cuda.stream(side):
            side.wait_stream(torch.cuda.current_stream())
            if sharded and world > 1:
                # the replicated batch: each rank copies its 1/N of the rows over PCIe and
                # the ranks all-gather the rest over NVLink
                lo, hi = tokens * rank // world, tokens * (rank + 1) // world
                bufs[j][lo:hi].copy_(src[lo:hi], non_blocking=True)
                dist.all_gather_into_tensor(bufs[j], bufs[j][lo:hi].clone())
            else:
                bufs[j].copy_(src, non_blocking=True)
            ready[j].record(side)

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    h2d(0, host[0])
    for i in range(e2e_steps):
        j = i % 2
        torch.cuda.current_stream().wait_event(ready[j])
        if i + 1 < e2e_steps:
            h2d(1 - j, host[(i + 1) % POOL_BATCHES])
        step(i, bufs[j])    # includes the stats read-back (loss, l0, grad norm) to the host
    e1.record()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    e2e_value = job_tokens / (e2e_ms / 1e3)

    if rank == 0:
        peaks = _peaks()
        gemm_flop = 2.0 * tokens * d * F
        enc_tf = gemm_flop / (enc_ms / 1e3) / 1e12
        grad_tf = gemm_flop / (grad_ms / 1e3) / 1e12
        traffic_scale = (d * F) / (D_IN * N_FEAT) * (tokens / TOKENS)
        gemm_bwd = fs.grad_feat == "gemm"   # the backward in effect at the end ("auto" may switch)
        entries = fs.pre_store == "entries" and not gemm_bwd and aux_dead is None
        dom_ms, dom_tf, dom_name, dom_traffic = (
            (enc_ms, enc_tf, "encoder tile GEMM (tcgen05 cta_group::2) + JumpReLU epilogue",
             TRAFFIC_ENCODER_GEMM if entries else TRAFFIC_ENCODER_GEMM_FULL_PRE)
            if (enc_ms >= grad_ms or not gemm_bwd) else
            (grad_ms, grad_tf, "grad_feat tile GEMM (tcgen05 cta_group::2) + STE epilogue",
             TRAFFIC_GRAD_GEMM))
        # The burst peak applies to a kernel timed inside a sub-second region; the
        # sustained (seconds-long, power-capped) peak only to a long timed region.
        timed_s = ms * args.steps / 1e3
        long_region = timed_s >= 2.0
        peak = peaks["bf16_sustained"] if long_region else peaks["bf16"]
        adam_bytes = 30.0 * (2 * d * F + 2 * F + d)
        dense_per_token = (4 if gemm_bwd else 2) * d * F_total
        step_flop = float(dense_per_token) * tokens
        line = {
            "metric": METRIC if not sharded else
            "wide-SAE fwd+bwd+Adam tokens/s at d=4096x131072 L0~64 (dictionary-sharded)",
            "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if sharded else "weak",
            "vs_baseline": None if sharded else value / PUBLISHED_TOK_S, "dtype": "bf16",
            "data": "synthetic superposition activations (seeded, on device)",
            "config": {"workload": wl["description"],
                       "model": f"JumpReLU SAE d_in={d} F={F_total}",
                       "d_in": d, "n_features": F_total, "features_per_gpu": F,
                       "tokens_per_step": tokens, "global_batch": job_tokens, "seq_len": None,
                       "parallelism": (f"dictionary split over {world} GPU(s), "
                                       + ("NVLink peer exchange of the partial x_hat"
                                          if args.exchange == "p2p" and world > 1 else
                                          "NCCL all-reduce of the partial x_hat")
                                       if sharded else
                                       f"atlas: {world} independent SAE(s), one per GPU"),
                       "l0_target": k_target, "l0_measured": l0_timed,
                       "ste_bandwidth": args.ste_bandwidth,
                       "entries_per_token": pairs_mean / tokens,
                       "aux_loss": ({"dead_fraction": args.aux_dead, "k": aux_k}
                                    if aux_dead is not None else None),
                       "threshold_calibrated": thr,
                       "threshold_control": "proportional log-threshold nudge after each step "
                                            "(the trainer's L0 controller)",
                       "l2": "inputs rotate over a 4-batch pool; every step's Adam pass "
                             f"streams {30 * (2 * d * F + 2 * F + d) / 1e9:.1f} GB of parameters, "
                             "gradients and moments, which flushes the 126 MB L2",
                       "dense_gemm_flop_per_token": dense_per_token,
                       "backward": ("dense tcgen05 grad_feat GEMM + STE epilogue, sparse CSR "
                                    "weight gradients: 4*d*F dense FLOP/token" if gemm_bwd else
                                    "sampled: grad_feat dot products on the active and in-band "
                                    "entries only, fused with the STE and the sparse weight "
                                    "gradients: 2*d*F dense FLOP/token (the encoder)")},
            "roofline": {"bound": "tensor", "kernel": dom_name,
                         "achieved": dom_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": dom_tf / peak,
                         "peak_source": (f"bf16_tflops_sustained ({peaks['src']}): timed region "
                                         f"{timed_s:.2f} s" if long_region else
                                         f"bf16_tflops burst ({peaks['src']}): timed region "
                                         f"{timed_s:.2f} s"),
                         "frac_of_sustained": dom_tf / peaks["bf16_sustained"],
                         "frac_of_burst": dom_tf / peaks["bf16"],
                         "traffic": dom_traffic * traffic_scale,
                         "traffic_note": ("ncu dram__bytes_read.sum + dram__bytes_write.sum "
                                          "of one 32768-token d=1536 F=49152 launch (pre stored "
                                          "at the entries only)" if entries else
                                          "ncu dram__bytes_read.sum + dram__bytes_write.sum of a "
                                          "4096-token d=1536 F=49152 launch, scaled by 8")
                                         + ("" if traffic_scale == 1 else
                                            f", scaled by tokens and d*F (x{traffic_scale:.3g})"),
                         "pre_store": "entries" if entries else "full",
                         "per_launch_flop": gemm_flop, "launch_ms": dom_ms},
            "kernels": ({"encoder_gemm_ms": enc_ms, "encoder_gemm_tflops": enc_tf,
                         "grad_gemm_ms": grad_ms, "grad_gemm_tflops": grad_tf} if gemm_bwd else
                        {"encoder_gemm_ms": enc_ms, "encoder_gemm_tflops": enc_tf,
                         "sampled_backward_ms": grad_ms,
                         # go rows of every entry + xc rows of the active ones, bf16, through L2
                         "sampled_backward_row_gbs":
                             (pairs_mean + nnz_mean) * d * 2 / (grad_ms / 1e3) / 1e9}) |
                       {"decode_ms": dec_ms,
                        # gathered bf16 decoder rows (L2 hits included)
                        "decode_row_gbs": nnz_mean * d * 2 / (dec_ms / 1e3) / 1e9,
                        "adam_ms": adam_ms,
                        # 30 B per parameter (p, g, m, v read; p, m, v written; bf16 copy)
                        "adam_gbs": adam_bytes / (adam_ms / 1e3) / 1e9,
                        "adam_frac_hbm": adam_bytes / (adam_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                        "hbm_peak_source": f"hbm_gbs ({peaks['src']})"} |
                       {"step_dense_tflops": step_flop / (ms / 1e3) / 1e12},
            "clocks": clock,
            "phases_ms": (None if phases is None else
                          {**{k: round(v, 4) for k, v in phases.items()},
                           "encoder_gemm": round(enc_ms, 4), "decode_partial": round(dec_ms, 4),
                           "exchange_p2p": None if xch_ms is None else round(xch_ms, 4),
                           "sampled_backward": round(grad_ms, 4),
                           "note": ("CUDA events on rank 0: forward = encoder + decode "
                                    "partial + exchange + loss terms; backward = this "
                                    "shard's sampled backward; bdec_allreduce, norm "
                                    "(sum of squares + its all-reduce + clip) and adam as "
                                    "named; the step's remainder is host time (the one "
                                    "stats read-back per microbatch)")}),
            "e2e": {"value": e2e_value, "unit": "tokens/s",
                    "h2d_bytes_per_step": (tokens if sharded else world * tokens) * d * 2,
                    "d2h_bytes_per_step": world * 2 * 64,
                    "note": ("whole job: each rank copies 1/N of the pinned host batch over "
                             "PCIe and the ranks all-gather the replicated batch over NVLink"
                             if sharded and world > 1 else
                             "whole job: every rank copies its pinned host batch") +
                            " (on a side stream overlapped with the previous step, as the "
                            "trainer's double buffer) and reads its stats back every step"},
            "gpu_launches": int(launches),
            "device_status": status,
        }
        if args.cpu_baseline and world == 1 and not sharded:
            sampler = CpuReferenceSampler()
            times = [sampler.sample(i)[0] for i in range(4)][1:]   # one warm-up sample
            cpu_s = statistics.mean(times)
            line["cpu_baseline"] = {
                "value": sampler.S / cpu_s, "unit": "tokens/s", "cores": sampler.threads,
                "kind": "port", "sample": sampler.description + f"; mean of {len(times)} samples",
                "extrapolated": False}
        print(json.dumps(line), flush=True)
    if sharded:
        fs.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


ATLAS_POOL_BATCHES = 16   # per-layer activation pool: 16 shards x 32768 tokens


def run_atlas_layers(args):
    """The 35-layer atlas configuration: independent SAEs (d=1536, F=49152,
    K=50), layer l with its own seed-derived pool of 16 x 32768 tokens whose
    norms are LogNormal(log(20 + 3 l), 0.4), placed round-robin on the GPUs
    (layer l on rank l mod N, sae_b200.atlas) and trained one after another on
    each GPU, as the reference's atlas loop trains them one after another
    (run_atlas_rolling, sae_trainer_rolling.py:4040-4180). Per layer: set-up
    (pool, init, threshold calibration; untimed), W warm-up steps, K timed
    steps on device-resident batches (value), then K steps fed from pinned
    host memory (e2e). A rank's time is the sum of its layers' timed regions;
    the job's is the slowest rank's, so the 35 / ceil(35 / N) bound of the
    round-robin placement shows in the value."""
    import torch
    import torch.distributed as dist

    import sae_b200
    from sae_b200 import _lib as L
    from sae_b200 import atlas

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=600))
    d, F, tokens, k = D_IN, N_FEAT, TOKENS, K_TARGET
    mine = atlas.layers_for_rank(args.layers, world, rank)
    side = torch.cuda.Stream(device=dev)
    per_layer = []
    launches0 = L.launch_count()
    with ClockSampler(local) as clocks:
        for layer in mine:
            norm_mu = math.log(20.0 + 3.0 * layer)
            pool = [sae_b200.superposition_batch(tokens, d, F, k, norm_mu, 0.4,
                                                 seed=100_000 * (layer + 1) + i, device=dev)
                    for i in range(ATLAS_POOL_BATCHES)]
            sae = sae_b200.make_shard_sae(d, F, 0, 1, seed=layer, device=dev)
            sae.ste_bandwidth = 0.2
            calibrate(sae, pool, k, F)
            opt = sae_b200.B200Adam(sae_b200.reference_param_groups(sae, LR), lr=LR,
                                    betas=(0.9, 0.999), sae=sae, renorm=True)
            fs = sae_b200.FusedStep(sae, opt, max_tokens=tokens)

            def step(x):
                out = fs.step(x, lambda_l0=LAMBDA, al_mu=MU, target_l0=k)
                threshold_nudge(sae, out["l0"], k)
                return out

            for i in range(args.warmup):
                step(pool[i % ATLAS_POOL_BATCHES])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            outs = [step(pool[(args.warmup + i) % ATLAS_POOL_BATCHES]) for i in range(args.steps)]
            e1.record()
            torch.cuda.synchronize()
            dev_ms = e0.elapsed_time(e1)
            # the same K steps fed from pinned host memory, double-buffered on a side stream
            host = [b.cpu().pin_memory() for b in pool]
            bufs = [torch.empty_like(pool[0]) for _ in range(2)]
            ready = [torch.cuda.Event() for _ in range(2)]

            def h2d(j, src):
                with torch.cuda.stream(side):
                    side.wait_stream(torch.cuda.current_stream())
                    bufs[j].copy_(src, non_blocking=True)
                    ready[j].record(side)

            torch.cuda.synchronize()
            h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            h0.record()
            h2d(0, host[0])
            for i in range(args.steps):
                j = i % 2
                torch.cuda.current_stream().wait_event(ready[j])
                if i + 1 < args.steps:
                    h2d(1 - j, host[(i + 1) % ATLAS_POOL_BATCHES])
                step(bufs[j])
            h1.record()
            torch.cuda.synchronize()
            per_layer.append({"layer": layer, "device_ms": dev_ms, "e2e_ms": h0.elapsed_time(h1),
                              "l0": statistics.mean(o["l0"] for o in outs)})
            del fs, opt, sae, pool, host, bufs
            torch.cuda.empty_cache()
    launches = L.launch_count() - launches0
    status = L.device_status()
    rank_ms = sum(p["device_ms"] for p in per_layer)
    rank_e2e_ms = sum(p["e2e_ms"] for p in per_layer)
    job_ms = atlas.max_over_ranks(rank_ms, device=dev)
    job_e2e_ms = atlas.max_over_ranks(rank_e2e_ms, device=dev)
    job_tokens = args.layers * args.steps * tokens
    busiest = -(-args.layers // world)
    if rank == 0:
        value = job_tokens / (job_ms / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": job_ms / (busiest * args.steps), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": value / PUBLISHED_TOK_S, "dtype": "bf16",
            "data": "synthetic superposition activations (seeded per layer, on device)",
            "config": {"workload": (f"{args.layers}-layer atlas: independent d_in={d} F={F} "
                                    f"K={k} SAEs, 32768-token microbatches, per-layer pools "
                                    f"of {ATLAS_POOL_BATCHES} x 32768 tokens with norms "
                                    "LogNormal(log(20 + 3 layer), 0.4), round-robin over "
                                    "the GPUs, trained layer after layer on each GPU"),
                       "layers": args.layers, "steps_per_layer": args.steps,
                       "layers_on_busiest_gpu": busiest,
                       "ideal_speedup": atlas.ideal_speedup(args.layers, world),
                       "parallelism": f"atlas: layer l on GPU l mod {world}, no collective",
                       "timed": "per layer, the K steps only (set-up and warm-up untimed); "
                                "a rank's time is the sum over its layers, the job's the "
                                "slowest rank's",
                       "rank0_layers": per_layer},
            "clocks": clocks.summary(),
            "e2e": {"value": job_tokens / (job_e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": world * tokens * d * 2,
                    "d2h_bytes_per_step": world * 2 * 64,
                    "note": "every step's batch copied from pinned host memory on a side "
                            "stream overlapped with the previous step; stats read back "
                            "every step"},
            "gpu_launches": int(launches),
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["inference"], default="atlas",
                    help="atlas: the metric's d=1536 F=49152 SAE, one per GPU (default); "
                         "sharded: one d=4096 F=131072 SAE split over the GPUs; inference: "
                         "encode + gathered decode at d=2304 F=65536")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--exchange", choices=["nccl", "p2p"], default="p2p",
                    help="sharded workload: sum the shards' partial x_hat with an NCCL "
                         "all-reduce, or with the fused NVLink peer exchange (default)")
    ap.add_argument("--aux-dead", type=float, default=0.0,
                    help="atlas workload: also run the dead-feature aux loss with this fraction "
                         "of the dictionary marked dead (the trainer turns it on after 250 "
                         "silent steps)")
    ap.add_argument("--ste-bandwidth", type=float, default=0.2,
                    help="STE band half-width epsilon (the scheduler adapts it up to 0.5); "
                         "the sampled backward's work grows with the band's population")
    ap.add_argument("--l0", type=float, default=0.0,
                    help="calibrate the thresholds to this mean L0 instead of the workload's "
                         "(e.g. an early-training state); not the metric's configuration")
    ap.add_argument("--layers", type=int, default=0,
                    help="atlas workload: train this many independent layer SAEs (35 for the "
                         "atlas configuration) round-robin over the GPUs, --steps timed steps "
                         "each, instead of one SAE per GPU")
    ap.add_argument("--tokens", type=int, default=0,
                    help="tokens per step (default: the workload's); smaller values are for "
                         "profiler captures, not for the reported metric")
    ap.add_argument("--features", type=int, default=0,
                    help="dictionary size (default: the workload's); other values are for "
                         "profiler captures of a small case, not for the reported metric")
    ap.add_argument("--pre-store", choices=["entries", "full"], default="entries",
                    help="encoder stores pre only in the 32-token words holding a backward "
                         "entry (default), or all of it")
    ap.add_argument("--grad-feat", choices=["sampled", "gemm", "auto"], default="sampled",
                    help="backward: grad_feat on the active + in-band entries only (default), "
                         "or the dense tcgen05 grad_feat GEMM")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.layers > 0:
        if args.workload != "atlas":
            ap.error("--layers applies to the atlas workload")
        return run_atlas_layers(args)
    if args.workload == "inference":
        return run_inference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())

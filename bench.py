#!/usr/bin/env python
"""Benchmark of the attention hot path on BASELINE config 4.

Workload (one "step"): 256 independent sequences, each with one Gated DeltaNet
layer decode step (config-0 shapes: 16/16 heads, d=128, f32 state) and one
gated-GQA layer decode step over a 32768-token f32 KV cache (8 q heads, 2 kv
heads, d=256, RoPE on 64 dims, theta 1e7).  The cache grows by one token per
step.  Sequences are sharded evenly over the N GPUs (strong scaling, no
inter-GPU traffic on the data path).  Inputs: seeded synthetic N(0,1) data of
those shapes (no checkpoints or datasets are needed).

value   = layer-steps/s over all GPUs (256 seqs x 2 layers per step),
          inputs resident in HBM, CUDA events, max over ranks.
e2e     = the same metric through the public C-ABI calls with the per-step
          inputs copied from pinned host memory and the outputs copied back
          inside the timed region (pipelined as a serving loop would be: the
          next step's inputs go up and the previous step's outputs come back
          on two copy streams while the current step computes).
roofline: the dominant kernel (GQA flash-decode) -- algorithmic bytes per
          launch over its CUDA-event duration, against MEASURED_PEAKS.json.
cpu_baseline: the CPU oracle (restatement of the reference, which is Rust/Burn
          and cannot be built here) timed on a bounded sample, rank 0, N=1.

--impl reference runs that CPU implementation alone on the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen-3.5_b200"))

# ---- workload constants (dims from text_config.rs) ----
NSEQ = 256
HK = HV = 16
DK = 128
CONV = 2 * HK * DK + HV * DK  # 6144
KCONV = 4
HQ, HKV, D, ROT = 8, 2, 256, 64
L0 = 32768
L2_BYTES = 126 << 20  # B200 L2
THETA = 1e7

GDN_BYTES_PER_SEQ = (2 * HV * DK * DK * 4          # state read + write
                     + 2 * CONV * (KCONV - 1) * 4  # conv state read + write
                     + CONV * 4 + HV * DK * 4 + 2 * HV * 4  # mixed_qkv, z, beta, g
                     + HV * DK * 4)                # out
GDN_BYTES_SHARED = CONV * KCONV * 4 + DK * 4     # conv weight + norm weight (read once per launch)


def gqa_bytes_per_seq(L):
    """Algorithmic bytes of one GQA decode step of one sequence whose cache
    holds L tokens before the append: K and V read for L+1 tokens, the new
    k/v written, q_gate/k_new/v_new/cos/sin read, output written."""
    return (2 * HKV * (L + 1) * D * 4 + 2 * HKV * D * 4 + HQ * 2 * D * 4 + 2 * HKV * D * 4 + 2 * ROT * 4
            + HQ * D * 4)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons; only samples
    stamped inside [mark_start, mark_end] (the timed region) are summarised."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.t0 = self.t1 = None
        self.out = ""

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)  # let the sampler start before the timed region
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out = self.proc.communicate(timeout=5)[0]
            except Exception:
                self.proc.kill()

    def summary(self):
        import datetime
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk, cmax = float(f[2]), float(f[3])
            except ValueError:
                continue
            mx = max(mx, cmax)
            if self.t0 is not None and not (self.t0 - 0.06 <= ts <= (self.t1 or ts) + 0.06):
                continue
            sm.append(clk)
            for n, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx or None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- CPU (oracle) leg
def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def host_mem_available():
    """Bytes of host memory available to this process (MemAvailable), or None."""
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except (OSError, ValueError, IndexError):
        pass
    return None


def cpu_cache_bytes(nseq, steps):
    return nseq * 2 * HKV * (L0 + steps + 1) * D * 4


def cpu_fit_seqs(want, steps, reserve=4 << 30):
    """The largest sequence count <= want (halving) whose caches fit in the
    host memory available now, with a margin."""
    avail = host_mem_available()
    n = want
    if avail is None:
        return n
    while n > 1 and cpu_cache_bytes(n, steps) * 1.1 + reserve > avail:
        n //= 2
    return n


class CpuBatch:
    """The CPU oracle (the reference's attention math restated in C) on nseq
    DISTINCT config-4 sequences: each has its own 32768-token KV cache, which
    grows by one token per step, and its own Gated DeltaNet state.  One step()
    is one config-4 step of those sequences: a GDN decode and a GQA decode of
    the whole batch, the oracle threaded over sequences and heads."""

    def __init__(self, nseq, threads, max_steps, seed=123):
        import concurrent.futures as cf
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # test infrastructure: the checker / CPU baseline only
        self.oracle = oracle
        oracle.set_threads(threads)
        self.nseq, self.threads = nseq, threads
        f = np.float32
        cap = L0 + max_steps + 1
        self.K = np.empty((nseq, HKV, cap, D), f)
        self.V = np.empty((nseq, HKV, cap, D), f)

        def fill(i):  # sequence i's cache, from its own generator (threads release the GIL)
            gen = np.random.default_rng([seed, i])
            for h in range(HKV):
                gen.standard_normal((L0, D), dtype=f, out=self.K[i, h, :L0])
                gen.standard_normal((L0, D), dtype=f, out=self.V[i, h, :L0])

        with cf.ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(fill, range(nseq)))
        rng = np.random.RandomState(seed)
        self.S = (0.02 * rng.randn(nseq, HV, DK, DK)).astype(f)
        self.conv_w = (0.5 * rng.randn(CONV, KCONV)).astype(f)
        self.norm_w = np.ones(DK, f)
        self.cst = np.zeros((nseq, CONV, KCONV - 1), f)
        self.w0 = np.zeros(D, f)
        self.lens = np.full(nseq, L0, np.int32)
        self.rng = rng

    def step(self):
        """One config-4 step over the batch; returns the seconds spent inside
        the two oracle calls (input generation is outside)."""
        o, f, rng, n = self.oracle, np.float32, self.rng, self.nseq
        x = rng.randn(n, CONV).astype(f)
        z = rng.randn(n, HV * DK).astype(f)
        g = (-np.log1p(np.exp(rng.randn(n, HV)))).astype(f)
        beta = (1 / (1 + np.exp(-rng.randn(n, HV)))).astype(f)
        qg = rng.randn(n, HQ, 2 * D).astype(f)
        kn = rng.randn(n, HKV, D).astype(f)
        vn = rng.randn(n, HKV, D).astype(f)
        cos, sin = o.rope_tables(self.lens.astype(np.int64), rot=ROT, theta=THETA)
        t0 = time.perf_counter()
        o.gdn_decode(x, z, beta, g, self.conv_w, self.norm_w, self.cst, self.S, HK, HV, inplace=True)
        o.gqa_decode(qg, kn, vn, self.w0, self.w0, cos, sin, self.K, self.V, self.lens, rot=ROT, inplace=True)
        return time.perf_counter() - t0


def cpu_sample(threads, nseq=32, min_s=10.0, max_steps=60):
    """Bounded CPU baseline beside the GPU run: whole config-4 steps of nseq
    distinct sequences, repeated until about min_s seconds of oracle time."""
    nseq = cpu_fit_seqs(nseq, max_steps + 1)
    w = CpuBatch(nseq, threads, max_steps + 1)
    w.step()  # warm
    el, n = 0.0, 0
    while n < max_steps and el < min_s:
        el += w.step()
        n += 1
    desc = (f"{n} config-4 steps of {nseq} distinct sequences (each step: 1 GDN decode + 1 GQA decode at "
            f"L~32768 per sequence), {threads} thread(s), {el:.1f} s")
    return 2 * nseq * n / el, desc, nseq


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    nsteps = args.warmup + args.steps
    nseq = cpu_fit_seqs(args.ref_seqs_full, nsteps)
    w = CpuBatch(nseq, threads, nsteps)
    for _ in range(args.warmup):
        w.step()
    tot = 0.0
    for _ in range(args.steps):
        tot += w.step()
    value = 2 * nseq * args.steps / tot
    desc = (f"{args.steps} timed config-4 steps of {nseq} distinct sequences, each with its own 32K KV cache "
            f"and GDN state (1 GDN decode + 1 GQA decode per sequence per step), {threads} thread(s), "
            f"{tot:.1f} s")
    config = {"workload": "config4: %d seqs x (GDN decode + GQA decode @32K ctx) per step" % nseq,
              "seqs": nseq, "kv_len_start": L0, "parallelism": "host cores",
              "cpu": cpu_model()}
    if nseq < args.ref_seqs_full:
        config["note"] = (f"{args.ref_seqs_full} sequences need {cpu_cache_bytes(args.ref_seqs_full, nsteps) / 1e9:.1f}"
                          f" GB of host memory, more than is available; {nseq} distinct sequences were timed instead")
    elif nseq != NSEQ:
        config["note"] = f"--ref-seqs-full {nseq}: a smaller batch than config 4's {NSEQ} sequences"
    line = {
        "impl": "reference", "metric": "attn layer-steps/s", "value": value, "unit": "layer-steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * tot / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
        "cpu_baseline": {"value": value, "unit": "layer-steps/s", "cores": threads, "kind": "port",
                         "cpu": cpu_model(), "sample": desc},
        "e2e": {"value": value, "unit": "layer-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is Rust/Burn over wgpu; neither cargo nor a graphics stack exists here, so its "
                "attention math runs as the C restatement in oracle/ on the host cores",
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU leg
def run_gpu(args):
    import torch
    import torch.distributed as dist

    import q35attn

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    NSEQ = args.seqs
    if NSEQ % world:
        raise SystemExit("world size must divide the number of sequences")
    B = NSEQ // world
    K, W = args.steps, args.warmup
    nsteps = W + K
    cap = L0 + 2 * nsteps + 16
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def randn(*shape, scale=1.0):
        t = torch.empty(*shape, device=dev, dtype=torch.float32)
        t.normal_(0.0, scale, generator=gen)
        return t

    # persistent state / caches (resident in HBM)
    S = randn(B, HV, DK, DK, scale=0.02)
    cst = randn(B, CONV, KCONV - 1, scale=0.5)
    conv_w = randn(CONV, KCONV, scale=0.5)
    norm_w = torch.ones(DK, device=dev)
    Kc = torch.empty(B, HKV, cap, D, device=dev)
    Vc = torch.empty(B, HKV, cap, D, device=dev)
    Kc[:, :, :L0].normal_(generator=gen)
    Vc[:, :, :L0].normal_(generator=gen)
    lens = torch.full((B,), L0, dtype=torch.int32, device=dev)
    qn_w = torch.zeros(D, device=dev)
    kn_w = torch.zeros(D, device=dev)
    ws = q35attn.GqaWorkspace(B, HQ, HKV, cap, max_len=cap, device=dev)

    # per-step inputs, resident (device leg)
    x = randn(nsteps, B, CONV)
    z = randn(nsteps, B, HV * DK)
    g = -torch.nn.functional.softplus(randn(nsteps, B, HV))
    beta = torch.sigmoid(randn(nsteps, B, HV))
    qg = randn(nsteps, B, HQ, 2 * D)
    kn = randn(nsteps, B, HKV, D)
    vn = randn(nsteps, B, HKV, D)
    pos = torch.arange(L0, L0 + 2 * nsteps + 1, device=dev, dtype=torch.float32)
    inv_freq = torch.exp(torch.arange(0, ROT, 2, device=dev, dtype=torch.float32) * (-np.log(THETA) / ROT))
    fr = pos[:, None] * inv_freq[None, :]
    cos_t = torch.cat([fr.cos(), fr.cos()], -1).contiguous()
    sin_t = torch.cat([fr.sin(), fr.sin()], -1).contiguous()
    cos_b = cos_t[:, None, :].expand(-1, B, -1).contiguous()
    sin_b = sin_t[:, None, :].expand(-1, B, -1).contiguous()
    out_gdn = torch.empty(B, HV * DK, device=dev)
    out_gqa = torch.empty(B, HQ * D, device=dev)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)

    def step(i, ev=None):
        q35attn.gdn_decode(x[i], z[i], beta[i], g[i], conv_w, norm_w, cst, S, out_gdn, num_k_heads=HK,
                           num_v_heads=HV, stream=stream)
        if ev is not None:
            ev[0].record(stream)
        q35attn.gqa_decode(qg[i], kn[i], vn[i], qn_w, kn_w, cos_b[i], sin_b[i], Kc, Vc, lens, out_gqa, workspace=ws,
                           max_len=cap, stream=stream)
        if ev is not None:
            ev[1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident leg
    for i in range(W):
        step(i)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    gdn_evs = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    L_start = L0 + W
    barrier()
    q35attn.launch_count(reset=True)
    with ClockSampler(local) as clk:
        clk.mark_start()
        t0.record(stream)
        for k in range(K):
            gdn_evs[k].record(stream)
            step(W + k, evs[k])
        t1.record(stream)
        torch.cuda.synchronize(dev)
        clk.mark_end()
    launches = q35attn.launch_count()
    barrier()
    elapsed = max_over_ranks(t0.elapsed_time(t1) / 1000.0)
    gqa_ms = [evs[k][0].elapsed_time(evs[k][1]) for k in range(K)]
    gdn_ms = [gdn_evs[k].elapsed_time(evs[k][0]) for k in range(K)]
    gqa_avg = statistics.mean(gqa_ms) / 1000.0
    gdn_avg = statistics.mean(gdn_ms) / 1000.0
    gqa_alg = sum(B * gqa_bytes_per_seq(L_start + k) for k in range(K)) / K
    gdn_alg = B * GDN_BYTES_PER_SEQ + GDN_BYTES_SHARED
    value = 2 * NSEQ * K / elapsed
    peak, peak_kind = load_peaks()
    gqa_gbs = gqa_alg / gqa_avg / 1e9
    gdn_gbs = gdn_alg / gdn_avg / 1e9
    step_bytes_all = (gqa_alg + gdn_alg) * world
    if lens.min().item() != L0 + W + K or ws.status() != 0:
        raise SystemExit(f"bench self-check failed: lens {lens.min().item()}..{lens.max().item()}, "
                         f"status {ws.status()}")

    # ---- end-to-end leg through the public API, host buffers
    nE = K
    h_x = torch.empty(nE, B, CONV, pin_memory=True)
    h_z = torch.empty(nE, B, HV * DK, pin_memory=True)
    h_b = torch.empty(nE, B, HV, pin_memory=True)
    h_g = torch.empty(nE, B, HV, pin_memory=True)
    h_qg = torch.empty(nE, B, HQ, 2 * D, pin_memory=True)
    h_kn = torch.empty(nE, B, HKV, D, pin_memory=True)
    h_vn = torch.empty(nE, B, HKV, D, pin_memory=True)
    h_cos = torch.empty(nE, B, ROT, pin_memory=True)
    h_sin = torch.empty(nE, B, ROT, pin_memory=True)
    for hbuf, src in ((h_x, x), (h_z, z), (h_b, beta), (h_g, g), (h_qg, qg), (h_kn, kn), (h_vn, vn)):
        hbuf.copy_(src[:nE].cpu())
    h_cos.copy_(cos_b[W + K:W + K + nE].cpu())
    h_sin.copy_(sin_b[W + K:W + K + nE].cpu())
    h_out_gdn = torch.empty(nE, B, HV * DK, pin_memory=True)
    h_out_gqa = torch.empty(nE, B, HQ * D, pin_memory=True)
    def dev_inputs():
        return [torch.empty(B, CONV, device=dev), torch.empty(B, HV * DK, device=dev), torch.empty(B, HV, device=dev),
                torch.empty(B, HV, device=dev), torch.empty(B, HQ, 2 * D, device=dev),
                torch.empty(B, HKV, D, device=dev), torch.empty(B, HKV, D, device=dev),
                torch.empty(B, ROT, device=dev), torch.empty(B, ROT, device=dev)]
    # Pipelined like a serving loop: step i+1's inputs go up on `up` into the
    # other input buffer while step i computes on `stream`, and step i's outputs
    # come back on `down` from the other output buffer.  Events order every
    # reuse of a buffer; all copies are inside the timed region.
    d_in = [dev_inputs(), dev_inputs()]
    d_out = [(torch.empty_like(out_gdn), torch.empty_like(out_gqa)) for _ in range(2)]
    h_bufs = [h_x, h_z, h_b, h_g, h_qg, h_kn, h_vn, h_cos, h_sin]
    h2d = sum(t[0].numel() * 4 for t in h_bufs)
    d2h = (h_out_gdn[0].numel() + h_out_gqa[0].numel()) * 4
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()
    in_ready = [ev() for _ in range(nE)]   # step i's inputs are on the device
    computed = [ev() for _ in range(nE)]   # step i's kernels are done (its inputs and outputs are free to reuse)
    fetched = [ev() for _ in range(nE)]    # step i's outputs are on the host

    def upload(i):
        if i >= 2:
            up.wait_event(computed[i - 2])  # step i-2 has finished reading this input buffer
        with torch.cuda.stream(up):
            for dbuf, hbuf in zip(d_in[i % 2], h_bufs):
                dbuf.copy_(hbuf[i], non_blocking=True)
        in_ready[i].record(up)

    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up.wait_event(e0)
    upload(0)
    for i in range(nE):
        if i + 1 < nE:
            upload(i + 1)
        di, (og, oq) = d_in[i % 2], d_out[i % 2]
        stream.wait_event(in_ready[i])
        if i >= 2:
            stream.wait_event(fetched[i - 2])  # step i-2's outputs have left this output buffer
        q35attn.gdn_decode(di[0], di[1], di[2], di[3], conv_w, norm_w, cst, S, og, num_k_heads=HK,
                           num_v_heads=HV, stream=stream)
        q35attn.gqa_decode(di[4], di[5], di[6], qn_w, kn_w, di[7], di[8], Kc, Vc, lens, oq,
                           workspace=ws, max_len=cap, stream=stream)
        computed[i].record(stream)
        down.wait_event(computed[i])
        with torch.cuda.stream(down):
            h_out_gdn[i].copy_(og, non_blocking=True)
            h_out_gqa[i].copy_(oq, non_blocking=True)
        fetched[i].record(down)
    stream.wait_event(fetched[nE - 1])
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_elapsed = max_over_ranks(e0.elapsed_time(e1) / 1000.0)
    e2e_value = 2 * NSEQ * nE / e2e_elapsed
    if not (torch.isfinite(h_out_gqa).all() and torch.isfinite(h_out_gdn).all()):
        raise SystemExit("non-finite outputs")

    extras = None
    if world > 1 and not args.no_extras:
        del x, z, g, beta, qg, kn, vn
        cp = run_single_seq_cp(dev, world, rank)
        extras = {"single_seq_context_parallel": cp}
    if rank == 0 and world == 1 and not args.no_extras:
        del x, z, g, beta, qg, kn, vn
        extras = run_extras(dev)
        extras["single_seq_context_parallel"] = run_single_seq_cp(dev, 1, 0)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, desc, _ = cpu_sample(threads, nseq=args.ref_seqs)
        cpu = {"value": v, "unit": "layer-steps/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
               "sample": desc}

    if rank == 0:
        traffic = None
        tp = os.path.join(ROOT, "profiles", "gqa_decode_traffic.json")
        if os.path.exists(tp):
            try:
                with open(tp) as f:
                    tj = json.load(f)
                traffic = tj["bytes_per_seq_step"] * B
            except Exception:
                traffic = None
        line = {
            "metric": "attn layer-steps/s", "value": value, "unit": "layer-steps/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": 1000.0 * elapsed / K, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config4: 256 seqs x (GDN decode + GQA decode @32K ctx) per step",
                       "seqs": NSEQ, "seqs_per_gpu": B, "kv_len_start": L0, "gdn_heads": [HK, HV, DK],
                       "gqa_heads": [HQ, HKV, D], "parallelism": f"seq-sharded x{world}",
                       "l2": "inputs larger than L2 (KV cache %.1f GB per GPU)" % (Kc.numel() * 8 / 1e9)},
            "hbm_gbs": step_bytes_all * K / elapsed / 1e9,
            "hbm_frac_measured": step_bytes_all * K / elapsed / 1e9 / world / peak,
            "hbm_frac_nominal_8tbs": step_bytes_all * K / elapsed / 1e9 / world / 8000.0,
            "roofline": {"bound": "hbm", "kernel": "gqa_decode", "achieved": gqa_gbs, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": gqa_gbs / peak, "traffic": traffic,
                         "alg_bytes_per_launch": gqa_alg, "avg_launch_ms": gqa_avg * 1e3},
            "gdn_kernel": {"achieved": gdn_gbs, "unit": "GB/s", "frac": gdn_gbs / peak,
                           "alg_bytes_per_launch": gdn_alg, "avg_launch_ms": gdn_avg * 1e3},
            "e2e": {"value": e2e_value, "unit": "layer-steps/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "configs": extras,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------- side measurements
def run_extras(dev, reps=3):
    """Per-step latency of BASELINE configs 0, 1 and 2 and of the single
    32K-context sequence on one GPU.  Decode loops are captured in one CUDA
    graph per configuration (each replay = the config's full step count), so
    the numbers exclude host launch overhead; the eager per-step time of
    config 0 is reported beside it."""
    import torch

    import q35attn
    res = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)

    def randn(*shape, scale=1.0):
        t = torch.empty(*shape, device=dev, dtype=torch.float32)
        t.normal_(0.0, scale, generator=gen)
        return t

    def timed_graph(fn, reps):
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            fn()  # warm (also configures kernel attributes outside capture)
        torch.cuda.synchronize(dev)
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=st):
            fn()
        gph.replay()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            gph.replay()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / 1000.0 / reps

    # config 0: GDN decode, B=1, 256 steps
    n0 = 256
    x, z = randn(n0, 1, CONV), randn(n0, 1, HV * DK)
    g = -torch.nn.functional.softplus(randn(n0, 1, HV))
    beta = torch.sigmoid(randn(n0, 1, HV))
    S, cst = randn(1, HV, DK, DK, scale=0.02), randn(1, CONV, KCONV - 1, scale=0.5)
    conv_w, norm_w = randn(CONV, KCONV, scale=0.5), torch.ones(DK, device=dev)
    o = torch.empty(1, HV * DK, device=dev)

    def cfg0():
        for i in range(n0):
            q35attn.gdn_decode(x[i], z[i], beta[i], g[i], conv_w, norm_w, cst, S, o, num_k_heads=HK, num_v_heads=HV)
    t = timed_graph(cfg0, reps) / n0
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    cfg0()
    b.record()
    torch.cuda.synchronize(dev)
    t_eager = a.elapsed_time(b) / 1000.0 / n0
    by0 = GDN_BYTES_PER_SEQ + GDN_BYTES_SHARED
    res["config0_gdn_decode_b1"] = {"us_per_step_graph": t * 1e6, "us_per_step_eager": t_eager * 1e6,
                                    "layer_steps_per_s": 1.0 / t, "alg_bytes_per_step": by0,
                                    "achieved_gbs": by0 / t / 1e9}

    # config 1 and the single 32K sequence: GQA decode, B=1
    for name, L0c, n1 in (("config1_gqa_decode_b1_L4096", 4096, 128), ("single_seq_gqa_decode_L32768", 32768, 64)):
        cap = L0c + n1 * (reps + 2) + 1
        Kc, Vc = torch.empty(1, HKV, cap, D, device=dev), torch.empty(1, HKV, cap, D, device=dev)
        Kc[:, :, :L0c].normal_(generator=gen)
        Vc[:, :, :L0c].normal_(generator=gen)
        lens = torch.full((1,), L0c, dtype=torch.int32, device=dev)
        qg, kn, vn = randn(n1, 1, HQ, 2 * D), randn(n1, 1, HKV, D), randn(n1, 1, HKV, D)
        cs, sn = randn(n1, 1, ROT), randn(n1, 1, ROT)
        w0 = torch.zeros(D, device=dev)
        o1 = torch.empty(1, HQ * D, device=dev)
        ws = q35attn.GqaWorkspace(1, HQ, HKV, cap, device=dev)

        def cfg1():
            for i in range(n1):
                q35attn.gqa_decode(qg[i], kn[i], vn[i], w0, w0, cs[i], sn[i], Kc, Vc, lens, o1, workspace=ws,
                                   max_len=cap)
        t = timed_graph(cfg1, reps) / n1
        Lmid = L0c + n1 * 2 + n1 * reps // 2
        by1 = gqa_bytes_per_seq(Lmid)
        res[name] = {"us_per_step_graph": t * 1e6, "layer_steps_per_s": 1.0 / t, "alg_bytes_per_step": by1,
                     "achieved_gbs": by1 / t / 1e9, "status": ws.status()}
        del Kc, Vc

    # GDN decode at the config-4 batch (256 sequences): column-split sweep
    Bs = 256
    xs, zs = randn(Bs, CONV), randn(Bs, HV * DK)
    gs = -torch.nn.functional.softplus(randn(Bs, HV))
    bs = torch.sigmoid(randn(Bs, HV))
    Ss, cs_ = randn(Bs, HV, DK, DK, scale=0.02), randn(Bs, CONV, KCONV - 1, scale=0.5)
    os_ = torch.empty(Bs, HV * DK, device=dev)
    sweep = {}
    for split in (-1, 1, 2, 4, 8):
        def gdn_b():
            for _ in range(10):
                q35attn.gdn_decode(xs, zs, bs, gs, conv_w, norm_w, cs_, Ss, os_, num_k_heads=HK, num_v_heads=HV,
                                   split=split)
        t = timed_graph(gdn_b, reps) / 10
        byb = Bs * GDN_BYTES_PER_SEQ + GDN_BYTES_SHARED
        sweep[str(split)] = {"us": t * 1e6, "achieved_gbs": byb / t / 1e9}
    res["gdn_decode_b256_split_sweep"] = sweep
    del Ss

    # config 2: GDN chunked prefill, T=8192
    T2 = 8192
    xp, zp = randn(1, T2, CONV), randn(1, T2, HV * DK)
    gp = -torch.nn.functional.softplus(randn(1, T2, HV))
    bp = torch.sigmoid(randn(1, T2, HV))
    S2, c2 = torch.zeros(1, HV, DK, DK, device=dev), torch.zeros(1, CONV, KCONV - 1, device=dev)
    op = torch.empty(1, T2, HV * DK, device=dev)
    wsp = q35attn.gdn_prefill_workspace(1, T2, HK, HV, device=dev)

    def cfg2():
        q35attn.gdn_prefill(xp, zp, bp, gp, conv_w, norm_w, c2, S2, op, num_k_heads=HK, num_v_heads=HV,
                            workspace=wsp)
    t = timed_graph(cfg2, reps)
    by2 = 271.6e6
    fl2 = 23.97e9
    res["config2_gdn_prefill_T8192"] = {"ms": t * 1e3, "tokens_per_s": T2 / t, "alg_bytes": by2,
                                        "achieved_gbs": by2 / t / 1e9, "alg_gflop": fl2 / 1e9,
                                        "achieved_tflops": fl2 / t / 1e12}
    del xp, zp, gp, bp, op, wsp

    # GQA prefill over the config-3 prompt (T = 1024, empty cache); lens is
    # reset inside the graph so every replay prefills the same prompt
    T3 = 1024
    qg3, kn3, vn3 = randn(1, T3, HQ, 2 * D), randn(1, T3, HKV, D), randn(1, T3, HKV, D)
    w03 = torch.zeros(D, device=dev)
    inv = 1.0 / (THETA ** (torch.arange(0, ROT, 2, device=dev, dtype=torch.float32) / ROT))
    ang = torch.arange(T3, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
    cos3 = torch.cat([ang.cos(), ang.cos()], -1)[None].contiguous()
    sin3 = torch.cat([ang.sin(), ang.sin()], -1)[None].contiguous()
    K3, V3 = torch.zeros(1, HKV, T3 + 64, D, device=dev), torch.zeros(1, HKV, T3 + 64, D, device=dev)
    lens3, out3 = torch.zeros(1, dtype=torch.int32, device=dev), torch.empty(1, T3, HQ * D, device=dev)
    ws3 = q35attn.GqaPrefillWorkspace(1, HQ, HKV, T3 + 64, T3)

    def cfg3_gqa():
        lens3.zero_()
        q35attn.gqa_prefill(qg3, kn3, vn3, w03, w03, cos3, sin3, K3, V3, lens3, out3, workspace=ws3)
    t = timed_graph(cfg3_gqa, reps)
    fl3 = 2 * 2 * (T3 * T3 / 2) * D * HQ
    res["config3_gqa_prefill_T1024"] = {"us": t * 1e6, "causal_gflop": fl3 / 1e9, "achieved_tflops": fl3 / t / 1e12}
    del qg3, kn3, vn3, K3, V3, ws3

    # Q8F decode GEMV (kernels.rs:103-165) at the 2B projection shapes; the
    # timed calls rotate over enough weight copies to exceed L2 (126 MB)
    gemv = {}
    for name, ind, outd in (("in_proj_qkv", 2048, 6144), ("o_proj", 2048, 2048), ("down_proj", 6144, 2048),
                            ("lm_head", 2048, 248320)):
        wbytes = ind * outd + ind * (outd // 64) * 4
        ncopy = max(1, -(-(256 << 20) // wbytes))
        ws_ = [torch.randint(-2**31, 2**31 - 1, (ind, outd // 4), dtype=torch.int32, device=dev)
               for _ in range(ncopy)]
        ss_ = [torch.rand(ind, outd // 64, device=dev) * 0.01 for _ in range(ncopy)]
        xg, yg = randn(ind), torch.empty(outd, device=dev)
        calls = 64

        def gcall():
            for i in range(calls):
                q35attn.q8_gemv(xg, ws_[i % ncopy], ss_[i % ncopy], yg, mode=0)
        tg = timed_graph(gcall, reps) / calls
        by = wbytes + 4 * (ind + outd)
        gemv[name] = {"in": ind, "out": outd, "us": tg * 1e6, "alg_bytes": by, "achieved_gbs": by / tg / 1e9,
                      "weight_copies": ncopy}
        del ws_, ss_
    res["q8_gemv"] = gemv

    # Q8F prefill GEMM (Linear::forward at seq_len > 1) at the config-3 prompt
    # shapes, on the tensor cores; three bf16 products per output (hi/lo splits)
    gemm = {}
    for name, ind, outd in (("in_proj_qkv", 2048, 6144), ("o_proj", 2048, 2048), ("down_proj", 6144, 2048),
                            ("up_proj", 2048, 6144)):
        wq = torch.randint(-2**31, 2**31 - 1, (ind, outd // 4), dtype=torch.int32, device=dev)
        sq = torch.rand(ind, outd // 64, device=dev) * 0.01
        xq, yq = randn(1024, ind), torch.empty(1024, outd, device=dev)

        def qcall():
            for _ in range(8):
                q35attn.q8_gemm(xq, wq, sq, yq)
        tq = timed_graph(qcall, reps) / 8
        fl = 2.0 * 1024 * ind * outd
        gemm[name] = {"T": 1024, "in": ind, "out": outd, "us": tq * 1e6, "tflops": fl / tq / 1e12,
                      "tensor_tflops_3_products": 3 * fl / tq / 1e12}
        del wq, sq, xq, yq
    res["q8_gemm_prefill"] = gemm

    # config 3: the 2B hybrid stack (24 layers, random Q8F weights), a
    # 1024-token random prompt, then 512 greedy decode steps (CUDA graph)
    import q35attn.stack as qs
    st3 = qs.HybridStack(qs.QWEN35_2B, capacity=1024 + 512 + 16, seed=0, device=dev)
    ids3 = torch.randint(0, qs.QWEN35_2B.vocab, (1024,), dtype=torch.int32, device=dev, generator=gen)
    st3.prefill(ids3)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    st3.prefill(ids3)
    b.record()
    torch.cuda.synchronize(dev)
    pre_ms = a.elapsed_time(b)
    core_ms, step_ms = st3.profile_decode_step()
    st3.prefill(ids3)
    st3.capture()
    st3.prefill(ids3)
    a.record()
    st3.decode(512)
    b.record()
    torch.cuda.synchronize(dev)
    dec_ms = a.elapsed_time(b)
    res["config3_stack_2b"] = {"prompt": 1024, "decode_steps": 512, "prefill_ms": pre_ms,
                               "decode_tok_s": 512 / dec_ms * 1e3, "decode_ms_per_token": dec_ms / 512,
                               "attention_core_share_eager": core_ms / step_ms, "gemv_mode": st3.gemv_mode,
                               "weights_gb": st3.weight_bytes() / 1e9,
                               "decode_weight_gbs": st3.weight_bytes() / (dec_ms / 512) / 1e6}
    del st3
    return res


def run_single_seq_cp(dev, world, rank, steps=64, warmup=3):
    """BASELINE config 4's single 32K-context sequence, one decode step of a
    GDN layer and a GQA layer, across all ranks: GDN heads-parallel, GQA KV
    length split; each rank stores its GDN head outputs and GQA softmax
    partials into every peer's receive buffer and merges what it received
    (q35attn.PeerExchange, one kernel, bounded waits, no collective in the
    step).  With one rank the same step is the single-GPU path (all heads,
    q35_gqa_decode over the whole cache, no exchange) -- the figure the
    multi-GPU ones are compared with.  Consecutive steps rotate over several
    independent sequences, each a full 32K context sharded the same way, so
    that what one step reads was last read more than an L2 (126 MB) ago.  The
    timed steps replay as one CUDA graph.  Returns the per-step time (max over
    ranks)."""
    import torch
    import torch.distributed as dist

    import q35attn
    from q35attn.parallel import PeerExchange, ShardPlan

    plan = ShardPlan(world, rank, HK, HV, L0)
    lo, hi = plan.kv_tokens
    n_loc = hi - lo
    tail = plan.holds_tail
    shard_bytes = 2 * HKV * n_loc * D * 4
    nring = max(1, -(-(2 * L2_BYTES) // shard_bytes))
    # the tail rank appends one key per step of a sequence: the eager warm-up steps plus a warm and a timed replay
    cap = n_loc + (-(-(warmup + 2 * steps) // nring) + 2 if tail else 0) + 1
    gen = torch.Generator(device=dev)
    gen.manual_seed(777 + rank)

    def randn(*shape, scale=1.0):
        t = torch.empty(*shape, device=dev, dtype=torch.float32)
        t.normal_(0.0, scale, generator=gen)
        return t

    hk_l, hv_l = HK // world, HV // world
    c_loc = 2 * hk_l * DK + hv_l * DK
    seqs = []
    for _ in range(nring):
        seqs.append(dict(K=randn(1, HKV, cap, D), V=randn(1, HKV, cap, D),
                         lens=torch.full((1,), n_loc, dtype=torch.int32, device=dev),
                         S=randn(1, hv_l, DK, DK, scale=0.02), cst=randn(1, c_loc, KCONV - 1, scale=0.5)))
    ws = q35attn.GqaWorkspace(1, HQ, HKV, cap, device=dev)
    conv_w = randn(c_loc, KCONV, scale=0.5)
    norm_w = torch.ones(DK, device=dev)
    w0 = torch.zeros(D, device=dev)
    nst = steps + warmup
    x, z = randn(nst, 1, c_loc), randn(nst, 1, hv_l * DK)
    g = -torch.nn.functional.softplus(randn(nst, 1, hv_l))
    beta = torch.sigmoid(randn(nst, 1, hv_l))
    qg, kn, vn = randn(nst, 1, HQ, 2 * D), randn(nst, 1, HKV, D), randn(nst, 1, HKV, D)
    cs, sn = randn(nst, 1, ROT), randn(nst, 1, ROT)
    part = torch.empty(1, HQ, D + 2, device=dev)
    out_l = torch.empty(1, hv_l * DK, device=dev)
    gdn_all = torch.empty(1, world * hv_l * DK, device=dev)
    out = torch.empty(1, HQ * D, device=dev)
    xchg = None
    if world > 1:
        # receive buffers mapped by CUDA IPC (handles gathered once over the group)
        def gather_handles(h):
            lst = [None] * world
            dist.all_gather_object(lst, h)
            return lst
        xchg = PeerExchange(world, rank, 1, hv_l * DK, HQ, gather_handles)

    def step(i):
        sq = seqs[i % nring]
        q35attn.gdn_decode(x[i], z[i], beta[i], g[i], conv_w, norm_w, sq["cst"], sq["S"], out_l, num_k_heads=hk_l,
                           num_v_heads=hv_l)
        if xchg is None:
            q35attn.gqa_decode(qg[i], kn[i], vn[i], w0, w0, cs[i], sn[i], sq["K"], sq["V"], sq["lens"], out,
                               workspace=ws, max_len=cap)
            return
        q35attn.gqa_decode_partial(qg[i], kn[i] if tail else None, vn[i] if tail else None, w0, w0, cs[i], sn[i],
                                   sq["K"], sq["V"], sq["lens"], part, workspace=ws, max_len=cap)
        xchg(out_l, part, qg[i], gdn_all, out)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[dev.index])

    # eager warm-up on a side stream, then the timed steps captured once in a CUDA graph (with an exchange: GDN
    # heads, GQA partial and its split combine, peer exchange + merge); every rank replays the same exchanges
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(warmup):
            step(i)
    torch.cuda.synchronize(dev)
    barrier()
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=side):
        for i in range(warmup, nst):
            step(i)
    gph.replay()
    torch.cuda.synchronize(dev)
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    gph.replay()
    b.record()
    torch.cuda.synchronize(dev)
    del gph
    status = (xchg.status() if xchg is not None else 0) | ws.status()
    t = a.elapsed_time(b) / 1000.0 / steps
    if world > 1:
        tt = torch.tensor([t], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
        xchg.close(barrier=barrier)
    if status:
        raise SystemExit(f"single-sequence step reported device status {status}")
    if not (torch.isfinite(out).all() and torch.isfinite(gdn_all if world > 1 else out_l).all()):
        raise SystemExit("single-sequence step: non-finite outputs")
    by = gqa_bytes_per_seq(L0 + (warmup + steps + steps // 2) // nring) + GDN_BYTES_PER_SEQ + GDN_BYTES_SHARED
    res = {"us_per_step": t * 1e6, "layer_steps_per_s": 2.0 / t, "alg_bytes_per_step_all_gpus": by,
           "achieved_gbs_all_gpus": by / t / 1e9, "sequences_rotated": nring,
           "l2": f"{nring} sequences of {shard_bytes / 1e6:.1f} MB KV per GPU rotated (> 2 x 126 MB L2)"}
    if world > 1:
        res.update({"collectives_per_step": 0,
                    "exchange": "epoch-tagged peer-memory stores over NVLink, one kernel per step (q35_cp_exchange)",
                    "partitioning": f"GDN heads {HV}/{world} per rank, GQA KV length {L0}/{world} per rank"})
    else:
        res["path"] = "one GPU: GDN decode (all heads) + q35_gqa_decode over the whole cache"
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--ref-seqs", type=int, default=32,
                    help="distinct sequences in the bounded CPU sample beside the GPU run")
    ap.add_argument("--ref-seqs-full", type=int, default=NSEQ,
                    help="distinct sequences timed by --impl reference (fewer only if host memory is short)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seqs", type=int, default=NSEQ, help="total sequences (256 = config 4; smaller for ncu)")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 0/1/2 side measurements")
    ap.add_argument("--prefill-tokens", type=int, default=0,
                    help="only run the config-2 GDN prefill at this prompt length (profiling aid)")
    ap.add_argument("--gqa-prefill-tokens", type=int, default=0,
                    help="only run the GQA prefill (8/2 heads, empty cache) at this prompt length (profiling aid)")
    ap.add_argument("--gqa-decode-len", type=int, default=0,
                    help="profiling aid: GQA decode of one sequence with this many cached tokens, 64 steps per "
                         "CUDA-graph replay (config 1: 4096; single 32K sequence: 32768)")
    ap.add_argument("--gemv-fused", choices=["gdn_front", "gqa_front", "mlp"], default="",
                    help="profiling aid: one fused decode projection launch of the 2B stack, timed alone")
    ap.add_argument("--gemv", type=str, default="",
                    help="IN,OUT: only run the Q8F GEMV of that shape (profiling aid)")
    ap.add_argument("--config3-steps", type=int, default=0,
                    help="only run config 3 (2B hybrid stack, 1024-token prompt) with this many graph decode steps")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)
    if args.prefill_tokens > 0:
        return run_prefill_only(args)
    if args.gqa_prefill_tokens > 0 or args.gemv or args.gemv_fused or args.gqa_decode_len:
        return run_kernel_only(args)
    if args.config3_steps > 0:
        return run_config3_only(args)
    return run_gpu(args)


def run_config3_only(args):
    """Config 3 alone: the 2B hybrid stack (random Q8F weights), a 1024-token
    random prompt, then --config3-steps greedy decode steps replayed from a CUDA
    graph (--warmup prefills first).  One JSON line; a profiling aid."""
    import torch

    import q35attn.stack as qs
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    st = qs.HybridStack(qs.QWEN35_2B, capacity=1024 + args.config3_steps + 16, seed=0, device=dev)
    ids = torch.randint(0, qs.QWEN35_2B.vocab, (1024,), dtype=torch.int32, device=dev, generator=gen)
    for _ in range(args.warmup):
        st.prefill(ids)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    st.prefill(ids)
    b.record()
    torch.cuda.synchronize(dev)
    pre = a.elapsed_time(b)
    st.capture()
    st.prefill(ids)
    a.record()
    toks = st.decode(args.config3_steps)
    b.record()
    torch.cuda.synchronize(dev)
    dec = a.elapsed_time(b)
    print(json.dumps({"case": "config3_stack_2b", "prompt": 1024, "decode_steps": args.config3_steps,
                      "prefill_ms": pre, "decode_ms_per_token": dec / args.config3_steps,
                      "decode_tok_s": args.config3_steps / dec * 1e3, "first_tokens": toks[:8].tolist()}))
    return 0


def run_kernel_only(args):
    """--gqa-prefill-tokens T: the GQA prefill of a T-token prompt into an
    empty cache (config-3 head shapes); --gemv IN,OUT: one Q8F GEMV (mode 0);
    --gemv-fused SHAPE: one fused decode projection (norm in front, mode 1);
    --gqa-decode-len L: 64 GQA decode steps of one sequence per call (a graph).
    --warmup untimed calls, then --steps calls timed with CUDA events; one JSON
    line.  A profiling aid, not the bench line."""
    import torch

    import q35attn
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    if args.gemv:
        ind, outd = (int(v) for v in args.gemv.split(","))
        w = torch.randint(-2**31, 2**31 - 1, (ind, outd // 4), dtype=torch.int32, device=dev, generator=gen)
        sc = torch.rand(ind, outd // 64, device=dev, generator=gen) * 0.01
        x, y = torch.randn(ind, device=dev, generator=gen), torch.empty(outd, device=dev)

        def call():
            q35attn.q8_gemv(x, w, sc, y, mode=0)
        case, size = "q8_gemv", {"in": ind, "out": outd}
        alg = ind * outd + ind * (outd // 64) * 4 + 4 * (ind + outd)
    elif args.gqa_decode_len:
        # one sequence, L cached tokens, 64 decode steps per graph replay (BASELINE config 1 at L=4096, the single
        # 32K-context sequence at L=32768); --steps replays are timed
        L0c, n1 = args.gqa_decode_len, 64
        cap = L0c + n1 * (args.steps + args.warmup + 2) + 1
        Kc, Vc = torch.empty(1, HKV, cap, D, device=dev), torch.empty(1, HKV, cap, D, device=dev)
        Kc[:, :, :L0c].normal_(generator=gen)
        Vc[:, :, :L0c].normal_(generator=gen)
        lens = torch.full((1,), L0c, dtype=torch.int32, device=dev)
        qg = torch.randn(n1, 1, HQ, 2 * D, device=dev, generator=gen)
        kn, vn = torch.randn(n1, 1, HKV, D, device=dev, generator=gen), torch.randn(n1, 1, HKV, D, device=dev,
                                                                                    generator=gen)
        cs, sn = torch.randn(n1, 1, ROT, device=dev, generator=gen), torch.randn(n1, 1, ROT, device=dev, generator=gen)
        w0, o1 = torch.zeros(D, device=dev), torch.empty(1, HQ * D, device=dev)
        ws = q35attn.GqaWorkspace(1, HQ, HKV, cap, device=dev)

        def steps64():
            for i in range(n1):
                q35attn.gqa_decode(qg[i], kn[i], vn[i], w0, w0, cs[i], sn[i], Kc, Vc, lens, o1, workspace=ws,
                                   max_len=cap)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            steps64()
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            steps64()

        def call():
            graph.replay()
        case, size = "gqa_decode_b1", {"L0": L0c, "decode_steps_per_call": n1}
        Lmid = L0c + n1 * (args.warmup + 1) + n1 * args.steps // 2
        alg = n1 * (2 * HKV * (Lmid + 1) * D * 4 + 24576)
    elif args.gemv_fused:
        # the fused decode projections of the 2B stack: RMSNorm(x + residual) in front, mode 1 rows
        outs, swiglu = {"gdn_front": ([6144, 2048], False), "gqa_front": ([4096, 512, 512], False),
                        "mlp": ([6144, 6144], True)}[args.gemv_fused]
        ind = 2048
        W = [(torch.randint(-2**31, 2**31 - 1, (ind, o // 4), dtype=torch.int32, device=dev, generator=gen),
              torch.rand(ind, o // 64, device=dev, generator=gen) * 0.01) for o in outs]
        x, res, nw = (torch.randn(ind, device=dev, generator=gen) for _ in range(3))
        h = torch.empty(ind, device=dev)
        fg = q35attn.ops.FusedGemv(x, W, [torch.empty(o, device=dev) for o in outs], residual=res, norm_w=nw,
                                   sum_out=h, swiglu=swiglu, mode=1)

        def call():
            fg()
        case, size = "q8_gemv_fused", {"shape": args.gemv_fused, "in": ind, "outs": outs}
        alg = sum(ind * o + ind * (o // 64) * 4 for o in outs) + 4 * (4 * ind + sum(outs))
    else:
        T = args.gqa_prefill_tokens
        qg = torch.randn(1, T, HQ, 2 * D, device=dev, generator=gen)
        kn, vn = torch.randn(1, T, HKV, D, device=dev, generator=gen), torch.randn(1, T, HKV, D, device=dev,
                                                                                    generator=gen)
        w0 = torch.zeros(D, device=dev)
        inv = 1.0 / (THETA ** (torch.arange(0, ROT, 2, device=dev, dtype=torch.float32) / ROT))
        ang = torch.arange(T, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        cos = torch.cat([ang.cos(), ang.cos()], -1)[None].contiguous()
        sin = torch.cat([ang.sin(), ang.sin()], -1)[None].contiguous()
        K, V = torch.zeros(1, HKV, T + 64, D, device=dev), torch.zeros(1, HKV, T + 64, D, device=dev)
        lens, out = torch.zeros(1, dtype=torch.int32, device=dev), torch.empty(1, T, HQ * D, device=dev)
        ws = q35attn.GqaPrefillWorkspace(1, HQ, HKV, T + 64, T)

        def call():
            lens.zero_()
            q35attn.gqa_prefill(qg, kn, vn, w0, w0, cos, sin, K, V, lens, out, workspace=ws)
        case, size = "gqa_prefill", {"tokens": T}
        alg = None
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        call()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / args.steps
    line = {"case": case, **size, "steps": args.steps, "warmup": args.warmup, "ms_per_call": ms}
    if args.gqa_decode_len:
        line["us_per_step"] = ms * 1e3 / 64
    if alg:
        line["achieved_gbs"] = alg / ms / 1e6
    print(json.dumps(line))
    return 0


def run_prefill_only(args):
    """Config-2 shapes (B=1, 16 heads, conv 4) at --prefill-tokens tokens:
    --warmup untimed calls, then --steps calls timed with CUDA events.  Prints
    one JSON line; it is a profiling aid, not the bench line."""
    import torch

    import q35attn
    dev = torch.device("cuda:0")
    T = args.prefill_tokens
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)

    def randn(*shape, scale=1.0):
        t = torch.empty(*shape, device=dev, dtype=torch.float32)
        t.normal_(0.0, scale, generator=gen)
        return t

    x, z = randn(1, T, CONV), randn(1, T, HV * DK)
    g = -torch.nn.functional.softplus(randn(1, T, HV))
    beta = torch.sigmoid(randn(1, T, HV))
    conv_w, norm_w = randn(CONV, KCONV, scale=0.5), torch.ones(DK, device=dev)
    S, cst = torch.zeros(1, HV, DK, DK, device=dev), torch.zeros(1, CONV, KCONV - 1, device=dev)
    out = torch.empty(1, T, HV * DK, device=dev)
    ws = q35attn.gdn_prefill_workspace(1, T, HK, HV, device=dev)

    def call():
        q35attn.gdn_prefill(x, z, beta, g, conv_w, norm_w, cst, S, out, num_k_heads=HK, num_v_heads=HV,
                            workspace=ws)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        call()
    b.record()
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / args.steps
    print(json.dumps({"case": "gdn_prefill", "tokens": T, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_call": ms, "tokens_per_s": T / ms * 1e3,
                      "launches_per_call": 3}))
    return 0


if __name__ == "__main__":
    sys.exit(main())

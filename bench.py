"""Benchmark of the per-denoising-step attention path on B200.

Default workload (the metric's config): LLaDA-8B attention
stack, 32 layers x 32 MHA heads x head_dim 128, bf16; batch 16 varlen
sequences, prompt ~ U[256, 1024] + 128-token generation block; every layer
recomputes non-causal attention over the whole sequence (a dense denoising
step). Synthetic seeded N(0,1) q/k/v per layer (random init; no checkpoint).

One "step" = the attention path of one denoising step: 32 varlen attention
launches (one per layer), each over distinct q/k/v buffers (the per-step
working set is far larger than the 126 MB L2, so no L2 flush is needed).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: the 32 heads are sharded over the ranks (tensor
parallel head sharding, fixed total work -> "strong" scaling); the primary
number has no collective (attention needs none); the ``tp_layer`` block adds
the row-parallel o_proj and its all-reduce per layer, timed three ways: the
GEMM alone, cuBLAS GEMM + NCCL all-reduce, and the fused
dllm_oproj_allreduce kernel (GEMM tiles pushed over NVLink peer memory).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.join(REPO, "dllm-serve_b200")
for _p in (REPO, PKG_ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "non-causal attn TFLOP/s & step tokens/s at LLaDA-8B shape, 1/2/4/8 B200, % roofline"
LAYERS, HEADS, KV_HEADS, HEAD_DIM, HIDDEN = 32, 32, 32, 128, 4096  # LAYERS: --layers
BATCH, GEN = 16, 128


def workload_lengths(seed: int = 2) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    prompts = torch.randint(256, 1025, (BATCH,), generator=g).tolist()
    return [p + GEN for p in prompts]


def attn_flops(lens, heads=HEADS, d=HEAD_DIM) -> float:
    return 4.0 * sum(L * L for L in lens) * heads * d


def config_block(lens, world):
    return {
        "workload": "c2: LLaDA-8B attention stack, dense denoising step",
        "model": "LLaDA-8B attention shape (32 layers, 32 MHA heads x 128, hidden 4096)",
        "layers": LAYERS,
        "global_batch": BATCH,
        "seq_len": f"prompt U[256,1024] + gen {GEN}: {min(lens)}-{max(lens)} (sum {sum(lens)})",
        "tokens_per_step": sum(lens),
        "parallelism": f"tp{world} head-sharded" if world > 1 else "single GPU",
        "l2": "inputs larger than L2: distinct q/k/v per layer "
              f"({3 * sum(lens) * HEADS * HEAD_DIM * 2 * LAYERS / world / 1e9:.1f} GB per step per GPU)",
    }


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes of a kernel from a committed ncu summary, if any."""
    p = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(name)
    return None


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """Polls the GPU's SM clock, power and clock-event reasons (read-only NVML
    queries) every 20 ms while the timed region runs; falls back to
    ``nvidia-smi -lms 100`` when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, gpu_index: int, period_s: float = 0.02):
        self.gpu_index = gpu_index
        self.period = period_s
        self.samples = []
        self.err = None
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - report, never fail the bench
            self.err = f"nvml unavailable: {e}"
            return self
        self._stop = threading.Event()

        def loop():
            nv, h = self._nv, self._h
            while not self._stop.is_set():
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    pw = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, pw, rs))
                except Exception as e:  # noqa: BLE001
                    self.err = str(e)
                    return
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
            try:
                self._nv.nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"]}
        nv = self._nv
        reasons = set()
        for _, _, rs in self.samples:
            for name, const in self.REASONS:
                if hasattr(nv, const) and rs & getattr(nv, const):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples), "power_w_max": max(s[1] for s in self.samples),
                "source": "NVML, 20 ms period, during the timed region"}


def physical_gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own attention module on the host cores
# (oracle/reference_module.py: the installed dllmserve package under
# baseline/_ref with CPU stand-ins for its flash-attn/Triton callees), or the
# oracle's restatement of it when that package is absent
# ---------------------------------------------------------------------------
def cpu_dense_layer_fn(heads):
    """(fn(q, k, v, lens), kind, what): one dense diffusion step of one layer
    on the host, fp32."""
    from oracle import attention_ref as O

    scale = HEAD_DIM ** -0.5
    try:
        from oracle import reference_module as RM

        R = RM.load()

        def fn(q, k, v, lens):
            return RM.dense_layer_forward(R, q, k, v, lens, heads, heads, HEAD_DIM, scale)

        return fn, "reference", "the reference's dllmserve.layers.attention.Attention.forward " \
                                "(installed package; flash-attn/Triton callees replaced by CPU stand-ins)"
    except ImportError:
        def fn(q, k, v, lens):
            metas = [O.SeqMeta(state=0, num_tokens=L, prompt_len=L - GEN) for L in lens]
            return O.diffusion_layer(q, k, v, metas, None, None, [[]] * len(lens), scale, heads, heads)

        return fn, "port", "oracle restatement of the reference's diffusion layer"


def cpu_reference_sample(lens, budget_s: float, heads=HEADS, seed=7):
    """Times one dense diffusion step of one layer of the workload on the
    host cores (as many sequences as fit the time budget). Returns
    (tflops, seconds, sample_desc, cores, n_seq, kind)."""
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    fn, kind, what = cpu_dense_layer_fn(heads)
    g = torch.Generator().manual_seed(seed)
    n_seq = len(lens)
    # shrink the sample (sequences of one layer) to the time budget
    probe = [lens[0]]
    N = sum(probe)
    q, k, v = (torch.randn(N, heads, HEAD_DIM, generator=g) for _ in range(3))
    t0 = time.perf_counter()
    fn(q, k, v, probe)
    per_flop = (time.perf_counter() - t0) / attn_flops(probe, heads)
    total = attn_flops(lens, heads)
    while n_seq > 1 and per_flop * attn_flops(lens[:n_seq], heads) > budget_s:
        n_seq -= 1
    sample = lens[:n_seq]
    N = sum(sample)
    q, k, v = (torch.randn(N, heads, HEAD_DIM, generator=g) for _ in range(3))
    t0 = time.perf_counter()
    fn(q, k, v, sample)
    dt = time.perf_counter() - t0
    fl = attn_flops(sample, heads)
    desc = (f"{what}: 1 of {LAYERS} layers, {n_seq} of {len(lens)} sequences ({fl / total * 100:.0f}% of one "
            f"layer's FLOPs), fp32 on host, torch threads={cores}")
    return fl / dt / 1e12, dt, desc, cores, n_seq, kind


def run_reference_arm(args, lens):
    """The reference's CPU attention path on the host cores (rank 0 only).
    One step = one dense diffusion step of one layer of the workload (a
    bounded sample of the 32-layer step); ms_per_step is that measured time,
    and the full 32-layer step is extrapolated in a separate field."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    # size each step so the whole run stays within a few minutes
    budget = max(0.5, 150.0 / max(1, args.steps + args.warmup))
    _, _, desc, _, n_seq, kind = cpu_reference_sample(lens, budget)
    fn, _, _ = cpu_dense_layer_fn(HEADS)
    sample = lens[:n_seq]
    g = torch.Generator().manual_seed(11)
    N = sum(sample)
    q, k, v = (torch.randn(N, HEADS, HEAD_DIM, generator=g) for _ in range(3))
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        fn(q, k, v, sample)
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    dt = sum(times) / len(times)
    tflops = attn_flops(sample) / dt / 1e12
    full_step_s = dt * (attn_flops(lens) / attn_flops(sample)) * LAYERS
    line = {
        "impl": "reference", "metric": METRIC, "value": tflops, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic seeded N(0,1) q/k/v",
        "config": config_block(lens, 1),
        "step": "one dense diffusion step of one layer (" + str(n_seq) + " of " + str(len(lens))
                + " sequences): a bounded sample of the 32-layer step",
        "step_tokens_per_s": sum(lens) / full_step_s,
        "extrapolated_full_step_ms": full_step_s * 1e3,
        "cpu_baseline": {"value": tflops, "unit": "TFLOP/s", "cores": cores, "kind": kind,
                         "sample": desc + "; step_tokens_per_s from the 32-layer extrapolation"},
        "e2e": {"value": tflops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_cpu_baselines(args):
    """``--cpu-baselines``: the reference's CPU attention path on the host
    cores for configs 1, 3, 4 and 5 (config 2 is the ``--impl reference``
    arm): the reference's own ``Attention.forward`` (installed package under
    baseline/_ref; flash-attn/Triton callees replaced by CPU stand-ins), fp32,
    one layer per measurement on a bounded sample of each workload's
    sequences (the same seeded prompt lengths as ``--workload``). Sparse
    configs time a dense step, a compute-cache step (state 1: attention,
    selection and cache store) and a reuse step (state 2) of that layer;
    per-layer times are also extrapolated to the whole batch and all layers
    (labelled as such). Prints one JSON line (rank 0 only)."""
    import platform

    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    try:
        from oracle import reference_module as RM

        R = RM.load()
    except ImportError as e:
        print(json.dumps({"impl": "reference", "unavailable": f"reference package not installed: {e}"}))
        return 0
    budget = args.cpu_budget
    scale = HEAD_DIM ** -0.5

    def timed(fn):
        fn()  # first call: allocations, lazy imports
        t0, n = time.perf_counter(), 0
        while True:
            fn()
            n += 1
            if time.perf_counter() - t0 > budget / 3 or n >= 20:
                return (time.perf_counter() - t0) / n

    g = torch.Generator().manual_seed(7)
    out = {"impl": "reference", "kind": "reference", "cores": cores, "cpu": _cpu_model(),
           "host": platform.node(), "dtype": "f32",
           "what": "the reference's dllmserve.layers.attention.Attention.forward on the host cores "
                   "(installed package; flash-attn/Triton callees replaced by CPU stand-ins), one layer"}
    # config 1: the whole config (one layer, one 64 + 32-token sequence, 32/32 heads)
    q, k, v = (torch.randn(96, HEADS, HEAD_DIM, generator=g) for _ in range(3))
    t = timed(lambda: RM.dense_layer_forward(R, q, k, v, [96], HEADS, HEADS, HEAD_DIM, scale))
    out["c1"] = {"ms": t * 1e3, "tflops": attn_flops([96]) / t / 1e12,
                 "sample": "the whole config: one layer, one sequence of 64 + 32 tokens, 32/32 heads x 128"}
    for wl in ("c3", "c4", "c5"):
        layers, Hq, Hkv, B, (plo, phi), gen, ratio, desc = SPARSE_WORKLOADS[wl]
        gw = torch.Generator().manual_seed(40 + int(wl[1]))
        prompts = torch.randint(plo, phi + 1, (B,), generator=gw).tolist()
        lens = [p + gen for p in prompts]
        # sample: the first n sequences, as many as fit the budget (probe with one)
        probe = lens[:1]
        qp, kp, vp = (torch.randn(sum(probe), h, HEAD_DIM, generator=g) for h in (Hq, Hkv, Hkv))
        t0 = time.perf_counter()
        RM.dense_layer_forward(R, qp, kp, vp, probe, Hq, Hkv, HEAD_DIM, scale)
        per_flop = (time.perf_counter() - t0) / attn_flops(probe, Hq)
        n = 1
        while n < B and per_flop * attn_flops(lens[:n + 1], Hq) < budget / 6:
            n += 1
        sl, sp = lens[:n], prompts[:n]
        N = sum(sl)
        q, k, v = (torch.randn(N, h, HEAD_DIM, generator=g) for h in (Hq, Hkv, Hkv))
        t_dense = timed(lambda: RM.dense_layer_forward(R, q, k, v, sl, Hq, Hkv, HEAD_DIM, scale))
        cyc = RM.SparseLayerCycle(R, sp, gen, Hq, Hkv, HEAD_DIM, ratio, True)
        t_state = {}
        for st in (1, 2):  # state 1 fills the cache that state 2 reads
            rows = cyc.rows(st)
            qs_, ks_, vs_ = (torch.randn(rows, h, HEAD_DIM, generator=g) for h in (Hq, Hkv, Hkv))
            t_state[st] = timed(lambda: cyc.forward(st, qs_, ks_, vs_))
        full = attn_flops(lens, Hq) / attn_flops(sl, Hq)  # dense / state-1 work scales with sum L^2
        out[wl] = {
            "desc": desc, "sample": f"{n} of {B} sequences (lengths {sl}), 1 of {layers} layers",
            "dense_ms_per_layer": t_dense * 1e3, "dense_tflops": attn_flops(sl, Hq) / t_dense / 1e12,
            "state1_ms_per_layer": t_state[1] * 1e3, "state2_ms_per_layer": t_state[2] * 1e3,
            "n_keep": cyc.n_keep,
            "extrapolated_full_step_ms": {"dense": t_dense * full * layers * 1e3,
                                          "state1": t_state[1] * full * layers * 1e3,
                                          "state2": t_state[2] * (B / n) * layers * 1e3,
                                          "note": f"x {layers} layers; dense and state 1 scaled by the batch's "
                                                  "sum L^2, state 2 by the sequence count"},
        }
    print(json.dumps(out), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, lens):
    import torch.distributed as dist

    from dllmserve_b200 import _native, ops
    from dllmserve_b200.layers.attention import Attention
    from dllmserve_b200.tp import head_slice, row_parallel_oproj
    from dllmserve_b200.utils.context import reset_context, set_context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=dev)
    _native.lib()

    h0, h1, kv0, kv1 = head_slice(HEADS, KV_HEADS, rank, world)
    Hq, Hk = h1 - h0, kv1 - kv0
    N = sum(lens)
    cu_host = [0]
    for L in lens:
        cu_host.append(cu_host[-1] + L)
    cu = torch.tensor(cu_host, dtype=torch.int32, device=dev)
    max_q = max(lens)
    scale = HEAD_DIM ** -0.5
    flops_step_local = attn_flops(lens, Hq) * LAYERS
    flops_step_total = attn_flops(lens, HEADS) * LAYERS

    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    qs = [torch.randn(N, Hq, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(LAYERS)]
    ks = [torch.randn(N, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(LAYERS)]
    vs = [torch.randn(N, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(LAYERS)]
    outs = [torch.empty(N, Hq, HEAD_DIM, device=dev, dtype=torch.bfloat16) for _ in range(2)]

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.current_stream()

    # ---------------- device-resident timing (value) ----------------
    for _ in range(args.warmup):
        for l in range(LAYERS):
            ops.varlen_attention(qs[l], ks[l], vs[l], cu, cu, max_q, scale, out=outs[l & 1])
    torch.cuda.synchronize()
    if ops.read_device_status(dev) != 0:
        raise RuntimeError("attention kernel reported a device error during warm-up")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(LAYERS * args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ops.LAUNCHES[0]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(physical_gpu_index(local_rank)) as clk:
        t_start.record(stream)
        i = 0
        for _ in range(args.steps):
            for l in range(LAYERS):
                ev[i][0].record(stream)
                ops.varlen_attention(qs[l], ks[l], vs[l], cu, cu, max_q, scale, out=outs[l & 1])
                ev[i][1].record(stream)
                i += 1
        t_end.record(stream)
        torch.cuda.synchronize()
    barrier()
    launches = ops.LAUNCHES[0] - launches0
    ms_total = max_over_ranks(t_start.elapsed_time(t_end))
    ms_step = ms_total / args.steps
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    mean_launch_ms = max_over_ranks(sum(launch_ms) / len(launch_ms))
    clocks = clk.summary()

    value = flops_step_total / (ms_step * 1e-3) / 1e12
    tokens_per_s = N / (ms_step * 1e-3)
    peaks, peak_kind = load_peaks()
    # Denominator: the measured burst cuBLAS bf16 GEMM figure (a kernel timed
    # in isolation); the sustained (seconds-long, power-capped) figure and the
    # burst figure scaled to the sampled median SM clock are reported beside it.
    burst = peaks.get("bf16_tflops", peaks.get("bf16_tflops_sustained"))
    sustained = peaks.get("bf16_tflops_sustained", burst)
    achieved = (flops_step_local / LAYERS) / (mean_launch_ms * 1e-3) / 1e12
    sm_mhz, sm_max = (clocks or {}).get("sm_mhz"), (clocks or {}).get("sm_max_mhz")
    at_clock = burst * min(1.0, sm_mhz / sm_max) if sm_mhz and sm_max else None
    roof = {"kernel": "dllm::attn_fwd_kernel", "bound": "tensor", "achieved": achieved,
            "peak": burst, "unit": "TFLOP/s", "frac": achieved / burst,
            "peak_kind": f"{peak_kind} bf16 dense, burst (cuBLAS GEMM timed alone)",
            "frac_of_sustained": achieved / sustained,
            "frac_of_burst_at_sampled_clock": (achieved / at_clock) if at_clock else None,
            # ncu capture of a full 32-head layer; a rank's launch covers Hq/world heads
            "traffic": (None if profile_traffic("attn_fwd_c2") is None
                        else profile_traffic("attn_fwd_c2") * Hq / HEADS),
            "algorithmic_per_launch": f"{flops_step_local / LAYERS / 1e9:.1f} GFLOP (4*sum(L^2)*Hq*D)",
            "mean_launch_ms": mean_launch_ms}

    # ---------------- KV-cache store (paged, random slot permutation) ----------------
    kv_block = None
    if not args.skip_extras:
        row = Hk * HEAD_DIM
        pages = (N + 255) // 256 + 8
        num_slots = pages * 256
        kc = torch.zeros(pages, 256, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        slot = torch.randperm(num_slots, device=dev, generator=gen)[:N].to(torch.int32)
        for _ in range(3):
            ops.store_kvcache(ks[0], vs[0], kc, vc, slot)
        reps = 20
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        for r in range(reps):
            l = r % LAYERS
            ops.store_kvcache(ks[l], vs[l], kc, vc, slot)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        byts = 2 * N * row * 2 * 2 + 4 * N
        gbs = byts / (ms * 1e-3) / 1e9
        hbm = peaks.get("hbm_gbs", 6650.0)
        kv_block = {"kernel": "dllm::kv_copy_kernel (store)", "ms": ms, "GB/s": gbs,
                    "frac_of_hbm": gbs / hbm, "bytes_per_launch": byts, "rows": N,
                    "row_bytes": row * 2}

    # ---------------- rotary embedding of q and k (the op before attention) ----------------
    rope_block = None
    if not args.skip_extras:
        from dllmserve_b200.layers.rotary_embedding import RotaryEmbedding

        rope = RotaryEmbedding(HEAD_DIM, HEAD_DIM, 4096, 500000.0).to(dev)
        pos = torch.cat([torch.arange(L, device=dev) for L in lens])
        qo, ko = torch.empty_like(qs[0]), torch.empty_like(ks[0])
        for _ in range(3):
            ops.rope_neox(pos, qs[0], ks[0], rope.cos_sin_cache, query_out=qo, key_out=ko)
        reps = 20
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        for r in range(reps):
            l = r % LAYERS
            ops.rope_neox(pos, qs[l], ks[l], rope.cos_sin_cache, query_out=qo, key_out=ko)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        byts = N * (Hq + Hk) * HEAD_DIM * 2 * 2 + 8 * N  # q, k read + written, positions
        gbs = byts / (ms * 1e-3) / 1e9
        hbm = peaks.get("hbm_gbs", 6650.0)
        rope_block = {"kernel": "dllm::rope_kernel", "ms": ms, "GB/s": gbs, "frac_of_hbm": gbs / hbm,
                      "bytes_per_launch": byts, "tokens": N}

    # ---------------- RoPE fused into a reuse-step attention launch ----------------
    rope_fused = None
    if not args.skip_extras:
        # config-3 reuse step: 8 sequences, 32-token block, 304 cached rows each
        B3, blk, nkeep, L3 = 8, 32, 304, 16
        n3 = B3 * blk
        pages3 = (B3 * nkeep + 255) // 256 + 1
        kc3 = torch.randn(pages3, 256, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen)
        vc3 = torch.randn(pages3, 256, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen)
        paged3 = dict(k_cache=kc3, v_cache=vc3,
                      slots=torch.arange(B3 * nkeep, dtype=torch.int32, device=dev),
                      cu_seqlens_slots=torch.arange(0, B3 * nkeep + 1, nkeep, dtype=torch.int32, device=dev))
        cq3 = torch.arange(0, n3 + 1, blk, dtype=torch.int32, device=dev)
        q3 = [torch.randn(n3, Hq, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(L3)]
        k3 = [torch.randn(n3, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(L3)]
        v3 = [torch.randn(n3, Hk, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(L3)]
        pos3 = torch.cat([torch.arange(nkeep, nkeep + blk) for _ in range(B3)]).to(dev)
        out3 = torch.empty(n3, Hq, HEAD_DIM, device=dev, dtype=torch.bfloat16)
        qo3, ko3 = torch.empty_like(q3[0]), torch.empty_like(k3[0])
        cs = rope.cos_sin_cache

        def r_unfused():
            for l in range(L3):
                ops.rope_neox(pos3, q3[l], k3[l], cs, query_out=qo3, key_out=ko3)
                ops.varlen_attention(qo3, ko3, v3[l], cq3, cq3, blk, scale, out=out3, **paged3)

        def r_fused():
            for l in range(L3):
                ops.varlen_attention(q3[l], k3[l], v3[l], cq3, cq3, blk, scale, out=out3,
                                     rope=(pos3, cs), **paged3)

        def r_attn():
            for l in range(L3):
                ops.varlen_attention(q3[l], k3[l], v3[l], cq3, cq3, blk, scale, out=out3, **paged3)

        r_unfused()
        ref3 = out3.clone()
        r_fused()
        same = bool(torch.equal(out3, ref3))
        us = {}
        for tag, fn in (("rope_then_attention", r_unfused), ("fused", r_fused), ("attention_only", r_attn)):
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            for _ in range(3):
                graph.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record(stream)
            for _ in range(20):
                graph.replay()
            b.record(stream)
            torch.cuda.synchronize()
            us[tag] = a.elapsed_time(b) * 1000 / (20 * L3)
            del graph
        rope_fused = {"workload": f"config-3 reuse-step layer: {B3} x {blk}-token blocks, {nkeep} cached rows, "
                                  f"{Hq}/{Hk} heads, CUDA graph of {L3} layers",
                      "us_per_layer": us, "fused_equals_unfused": same,
                      "fused_entry": "dllm_attn_varlen_rope_fwd (opt-in; the layer uses rope_then_attention)"}

    # ---------------- TP layer: attention + o_proj + all-reduce ----------------
    tp_block = None
    if not args.skip_extras:
        from dllmserve_b200.tp import OprojAllReduce

        w = (torch.randn(HIDDEN, Hq * HEAD_DIM, device=dev, generator=gen) * 0.02).to(torch.bfloat16)
        steps_tp = max(1, min(args.steps, 20))
        # The fused path must not take the whole line down: the ranks agree on
        # whether every rank could set it up, and a device error it raises is
        # recorded and cleared (the other paths' numbers stand).
        fused, fused_problem = None, None
        try:
            fused = OprojAllReduce(N, HIDDEN, device=dev)
        except Exception as e:  # noqa: BLE001 - reported in the line
            fused_problem = f"setup failed: {e}"
        fused_ok = max_over_ranks(0.0 if fused is not None else 1.0) == 0.0
        if not fused_ok and fused_problem is None:
            fused_problem = "setup failed on another rank"

        def fused_status_clean(where):
            nonlocal fused_ok, fused_problem
            st = max_over_ranks(float(ops.read_device_status(dev, reset=False)))
            if st != 0.0:
                fused_ok = False
                fused_problem = f"device status {int(st)} after {where}"
                ops.read_device_status(dev, reset=True)
            return fused_ok

        def tp_gemm_only():  # no collective: what the all-reduce adds is measured against this
            for l in range(LAYERS):
                o = ops.varlen_attention(qs[l], ks[l], vs[l], cu, cu, max_q, scale, out=outs[l & 1])
                torch.nn.functional.linear(o.view(N, Hq * HEAD_DIM), w)

        def tp_nccl():
            for l in range(LAYERS):
                o = ops.varlen_attention(qs[l], ks[l], vs[l], cu, cu, max_q, scale, out=outs[l & 1])
                row_parallel_oproj(o.view(N, Hq * HEAD_DIM), w, rank=rank)

        def tp_fused():
            for l in range(LAYERS):
                o = ops.varlen_attention(qs[l], ks[l], vs[l], cu, cu, max_q, scale, out=outs[l & 1])
                fused(o.view(N, Hq * HEAD_DIM), w)

        def time_tp(fn):
            for _ in range(2):
                fn()
            barrier()
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(steps_tp):
                fn()
            b.record(stream)
            torch.cuda.synchronize()
            barrier()
            return max_over_ranks(a.elapsed_time(b) / steps_tp)

        ms_gemm = time_tp(tp_gemm_only)
        ms_nccl = time_tp(tp_nccl)
        if ops.read_device_status(dev, reset=False) != 0:
            raise RuntimeError("a kernel reported a device error before the fused o_proj path")
        ms_fused, fused_err = None, None
        o = ops.varlen_attention(qs[0], ks[0], vs[0], cu, cu, max_q, scale, out=outs[0])
        if fused_ok:
            # one call first: a peer that never writes ends within the kernel's wait limit
            fused(o.view(N, Hq * HEAD_DIM), w)
            torch.cuda.synchronize()
        if fused_status_clean("a first call"):
            ms_fused = time_tp(tp_fused)
        if fused_ok and fused_status_clean("the timed calls"):
            # the fused path's result against GEMM + NCCL on the first layer's inputs
            y_ref = row_parallel_oproj(o.view(N, Hq * HEAD_DIM), w, rank=rank)
            y_f = fused(o.view(N, Hq * HEAD_DIM), w)
            torch.cuda.synchronize()
            fused_err = max_over_ranks(float((y_f.float() - y_ref.float()).abs().max()))
        if not fused_ok:
            ms_fused = None
        if fused is not None:
            fused.close()
            del fused
        best = ms_nccl if ms_fused is None else min(ms_nccl, ms_fused)
        tp_block = {"ms_per_step": best, "step_tokens_per_s": N / (best * 1e-3),
                    "ms_per_step_by_path": {"attention_gemm_no_collective": ms_gemm,
                                            "attention_gemm_nccl_allreduce": ms_nccl,
                                            "attention_fused_oproj_allreduce": ms_fused},
                    "us_per_layer_by_path": {"attention_gemm_no_collective": ms_gemm * 1e3 / LAYERS,
                                             "attention_gemm_nccl_allreduce": ms_nccl * 1e3 / LAYERS,
                                             "attention_fused_oproj_allreduce":
                                                 None if ms_fused is None else ms_fused * 1e3 / LAYERS},
                    "allreduce_share_nccl_path": (ms_nccl - ms_gemm) / ms_nccl,
                    "fused_vs_nccl_max_abs_diff": fused_err,
                    "fused_problem": fused_problem,
                    "includes": "per layer: attention on the rank's heads + o_proj [tokens, Hq*128] x "
                                "[4096, Hq*128]^T bf16 + all-reduce of [tokens, 4096] bf16; the nccl path "
                                "is cuBLAS + NCCL, the fused path one dllm_oproj_allreduce launch",
                    "steps": steps_tp}

    # ---------------- config-3 sparse diffusion block (r=0.5, head_select) ----------------
    sparse_block = None
    if not args.skip_extras:
        sparse_block = sparse_cycle("c3", args.steps, args.warmup)

    # ---------------- e2e through the public API, host buffers ----------------
    e2e = None
    if not args.skip_extras:
        class _Seq:  # dense sequence as the model runner hands it to the layer
            sparse_state = None

            def __init__(self, L):
                self.num_tokens = L
                self.num_prompt_tokens = L - GEN

        seqs = [_Seq(L) for L in lens]
        attn = Attention(Hq, HEAD_DIM, scale, Hk, causal=False)
        host_q = [qs[i].cpu().pin_memory() for i in range(2)]
        host_k = [ks[i].cpu().pin_memory() for i in range(2)]
        host_v = [vs[i].cpu().pin_memory() for i in range(2)]
        host_o = [torch.empty(N, Hq * HEAD_DIM, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        dq = [torch.empty_like(qs[0]) for _ in range(2)]
        dk = [torch.empty_like(ks[0]) for _ in range(2)]
        dv = [torch.empty_like(vs[0]) for _ in range(2)]
        h2d_s = torch.cuda.Stream(dev)
        d2h_s = torch.cuda.Stream(dev)
        e2e_steps = max(1, min(args.steps, 5))

        def e2e_step():
            set_context(True, cu_seqlens_k=cu, is_diffusion=True, seqs=seqs,
                        slot_mapping=[[] for _ in seqs])
            done = [None, None]
            for l in range(LAYERS):
                j = l & 1
                with torch.cuda.stream(h2d_s):
                    if done[j] is not None:
                        h2d_s.wait_event(done[j])
                    dq[j].copy_(host_q[j], non_blocking=True)
                    dk[j].copy_(host_k[j], non_blocking=True)
                    dv[j].copy_(host_v[j], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(h2d_s)
                stream.wait_event(ready)
                o = attn(dq[j].view(N, -1), dk[j].view(N, -1), dv[j].view(N, -1))
                fin = torch.cuda.Event()
                fin.record(stream)
                done[j] = fin
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(fin)
                    o.record_stream(d2h_s)
                    host_o[j].copy_(o, non_blocking=True)
            stream.wait_stream(d2h_s)
            stream.wait_stream(h2d_s)
            reset_context()

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(stream)
        h2d_s.wait_stream(stream)
        for _ in range(e2e_steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_e2e = max_over_ranks(a.elapsed_time(b) / e2e_steps)
        h2d = LAYERS * (qs[0].numel() + ks[0].numel() + vs[0].numel()) * 2 + (BATCH + 1) * 4
        d2h = LAYERS * N * Hq * HEAD_DIM * 2
        e2e = {"value": flops_step_total / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
               "api": "dllmserve_b200.layers.attention.Attention.forward per layer with "
                      "set_context per step; q/k/v H2D from pinned host, output D2H",
               "steps": e2e_steps}

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        tf, dt, desc, cores, _, kind = cpu_reference_sample(lens, budget_s=12.0)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": cores, "kind": kind, "sample": desc,
               "seconds": dt}

    if ops.read_device_status(dev) != 0:
        raise RuntimeError("a kernel reported a device error")

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) bf16 q/k/v per layer (random init, no checkpoint)",
            "config": config_block(lens, world),
            "step_tokens_per_s": tokens_per_s,
            "e2e": e2e, "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": launches, "kv_store": kv_block, "rope": rope_block,
            "rope_fused_reuse": rope_fused, "tp_layer": tp_block, "sparse_cycle_c3": sparse_block,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# sparse diffusion-block cycle (configs 3, 4, 5) through the public layer API
# ---------------------------------------------------------------------------
SPARSE_WORKLOADS = {
    # name: (layers, Hq, Hkv, batch, prompt (lo, hi), gen, ratio, description)
    "c3": (32, 32, 32, 8, (512, 512), 128, 0.5,
           "c3: LLaDA-8B head_select r=0.5, B=8, 512+128 tokens"),
    "c4": (28, 28, 4, 32, (128, 768), 256, 0.5,
           "c4: Dream-7B GQA 28/4 head_select r=0.5, B=32, U[128,768]+256 tokens"),
    "c5": (32, 32, 32, 8, (4096, 4096), 512, 0.25,
           "c5: LLaDA-8B long context head_select r=0.25, B=8, 4096+512 tokens"),
}


def run_sparse_cycle(args):
    """``--workload c3|c4|c5``: prints the sparse_cycle() line of the workload."""
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)
    line = sparse_cycle(args.workload, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return 0


def sparse_cycle(workload, steps, warmup):
    """One diffusion block = 32 denoising steps with SparseConfig(delay_step=1,
    block 32): state 0 (dense), state 1 (dense + select/store), 30 x state 2
    (block queries over cached + fresh keys), timed against 32 dense steps,
    eagerly (each step builds a new Context and launches from Python, as the
    reference's model runner does) and as per-state CUDA graphs. Every layer
    is the public Attention module; q/k/v are synthetic per layer. Runs on
    this rank's head slice under an initialised process group."""
    import torch.distributed as dist

    from dllmserve_b200 import _native, ops
    from dllmserve_b200.layers.attention import Attention
    from dllmserve_b200.sparse.state import PerRequestSparseState, SparseConfig, num_keep
    from dllmserve_b200.tp import head_slice
    from dllmserve_b200.utils.context import reset_context, set_context

    layers, Hq_all, Hkv_all, B, (plo, phi), gen, ratio, desc = SPARSE_WORKLOADS[workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local_rank)
    _native.lib()
    h0, h1, k0, k1 = head_slice(Hq_all, Hkv_all, rank, world)
    Hq, Hkv = h1 - h0, k1 - k0
    g = torch.Generator().manual_seed(40 + int(workload[1]))
    prompts = torch.randint(plo, phi + 1, (B,), generator=g).tolist()
    lens = [p + gen for p in prompts]
    blk = 32
    cfg = SparseConfig(enabled=True, default_block_len=blk, retention_ratio=ratio, pool_kernel=3,
                       delay_step=1, head_select=True)

    class Seq:
        def __init__(self, prompt, L, sparse):
            self.num_prompt_tokens = prompt
            self.num_tokens = L
            self.sparse_state = PerRequestSparseState(0, cfg, dev) if sparse else None

    n_keeps = [num_keep(L - blk, ratio) for L in lens]
    pages_per = [(n + 255) // 256 for n in n_keeps]
    total_pages = sum(pages_per) + 4
    slots, pg = [], 0
    for n, npg in zip(n_keeps, pages_per):
        lst = []
        for j in range(npg):
            lst.extend(range((pg + j) * 256, (pg + j) * 256 + min(256, n - j * 256)))
        pg += npg
        slots.append(torch.tensor(lst, dtype=torch.int32, device=dev))
    N_full = sum(lens)
    gd = torch.Generator(device=dev).manual_seed(1000 + rank)
    mk = lambda h: torch.randn(N_full, h, HEAD_DIM, device=dev, dtype=torch.bfloat16, generator=gd)
    qs = [mk(Hq) for _ in range(layers)]
    ks = [mk(Hkv) for _ in range(layers)]
    vs = [mk(Hkv) for _ in range(layers)]
    attn = []
    for _ in range(layers):
        a = Attention(Hq, HEAD_DIM, HEAD_DIM ** -0.5, Hkv, causal=False)
        a.k_cache = torch.zeros(total_pages, 256, Hkv, HEAD_DIM, device=dev, dtype=torch.bfloat16)
        a.v_cache = torch.zeros_like(a.k_cache)
        attn.append(a)

    from dllmserve_b200.utils.context import Context, use_context

    def rows_of(seqs):
        return sum(s.num_tokens if (s.sparse_state is None or s.sparse_state.cache_state != 2)
                   else s.sparse_state.compute_block_boundaries(s.num_prompt_tokens, s.num_tokens)[1]
                   for s in seqs)

    def make_ctx(seqs):
        return Context(is_prefill=True, is_diffusion=True, seqs=seqs,
                       slot_mapping=[(sl if s.sparse_state is not None and s.sparse_state.cache_state
                                      else []) for s, sl in zip(seqs, slots)])

    views = {}  # rows -> per-layer [rows, heads*D] views of q/k/v: the step's inputs, made in warm-up

    def layer_inputs(rows):
        v = views.get(rows)
        if v is None:
            v = views[rows] = [(qs[l][:rows].view(rows, -1), ks[l][:rows].view(rows, -1),
                                vs[l][:rows].view(rows, -1)) for l in range(layers)]
        return v

    def step(seqs, ctx=None):
        rows = rows_of(seqs)
        use_context(ctx if ctx is not None else make_ctx(seqs))
        for l, (q, k, v) in enumerate(layer_inputs(rows)):
            attn[l](q, k, v)
        reset_context()
        return rows

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def timed(fn, reps):
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    dense_seqs = [Seq(p, L, False) for p, L in zip(prompts, lens)]
    for _ in range(max(1, warmup)):
        step(dense_seqs)
    dense_ms = timed(lambda: step(dense_seqs), max(1, min(steps, 10)))

    sparse_seqs = [Seq(p, L, True) for p, L in zip(prompts, lens)]

    def rewind():
        for s in sparse_seqs:  # restart at the same block so every cycle sees the same shapes
            s.sparse_state.current_block_idx = 0
            s.sparse_state.step_in_block = 0
            s.sparse_state.cache_state = 0

    def advance():
        for s in sparse_seqs:
            s.sparse_state.advance_step()

    # eager: every step builds its context (metadata H2D) and launches from Python
    per_state = {0: [], 1: [], 2: []}
    cycles = max(1, min(steps // 32, 3))
    for _ in range(blk):  # warm-up cycle, also fills the caches
        step(sparse_seqs)
        advance()
    rewind()
    cycle_ms = []
    for _ in range(cycles):
        tot = 0.0
        for _ in range(blk):
            st = sparse_seqs[0].sparse_state.cache_state
            ms = timed(lambda: step(sparse_seqs), 1)
            per_state[st].append(ms)
            tot += ms
            advance()
        rewind()
        cycle_ms.append(tot)

    # graphs: one context + one captured 32-layer step per cache state, replayed
    # 1 x state 0, 1 x state 1, 30 x state 2 per block (identical device work)
    graphs, ctxs = {}, {}
    side = torch.cuda.Stream(dev)
    for st in (0, 1, 2):
        for s in sparse_seqs:
            s.sparse_state.cache_state = st
            s.sparse_state.step_in_block = st
        ctxs[st] = make_ctx(sparse_seqs)
        # One eager step on the capture stream: builds and caches the plan
        # outside capture and gives the stream its scheduler workspace, so the
        # captured attention launches hand out units dynamically.
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step(sparse_seqs, ctxs[st])
        torch.cuda.synchronize()
        g_ = torch.cuda.CUDAGraph()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(g_, stream=side):
                step(sparse_seqs, ctxs[st])
        torch.cuda.current_stream().wait_stream(side)
        graphs[st] = g_
    rewind()
    order = [0, 1] + [2] * (blk - 2)
    graph_cycle_ms = statistics.median(
        [timed(lambda: [graphs[st].replay() for st in order], 1) for _ in range(max(2, cycles))])
    graph_dense = torch.cuda.CUDAGraph()
    ctx_d = make_ctx(dense_seqs)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(dense_seqs, ctx_d)  # plan + the capture stream's scheduler workspace
    torch.cuda.synchronize()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph_dense, stream=side):
            step(dense_seqs, ctx_d)
    torch.cuda.current_stream().wait_stream(side)
    graph_dense_ms = timed(lambda: graph_dense.replay(), max(2, min(steps, 10)))
    graph_state_ms = {st: timed(lambda: graphs[st].replay(), 3) for st in (0, 1, 2)}
    if ops.read_device_status(dev) != 0:
        raise RuntimeError("a kernel reported a device error")
    sparse_step_ms = statistics.median(cycle_ms) / blk
    line = {
        "workload": workload, "desc": desc, "n_gpus": world,
        "parallelism": f"tp{world} head-sharded" if world > 1 else "single GPU",
        "layers": layers, "heads": [Hq_all, Hkv_all], "batch": B, "seq_lens": [min(lens), max(lens)],
        "tokens_dense_step": N_full, "retention_ratio": ratio, "n_keep": [min(n_keeps), max(n_keeps)],
        "eager": {"dense_ms_per_step": dense_ms, "sparse_ms_per_step": sparse_step_ms,
                  "sparse_speedup_vs_dense": dense_ms / sparse_step_ms},
        "state_ms": {k: (statistics.median(v) if v else None) for k, v in per_state.items()},
        "graph": {"dense_ms_per_step": graph_dense_ms,
                  "sparse_ms_per_step": graph_cycle_ms / blk,
                  "sparse_speedup_vs_dense": graph_dense_ms / (graph_cycle_ms / blk),
                  "state_ms": graph_state_ms,
                  "note": "per-state 32-layer steps captured as CUDA graphs and replayed "
                          "1x state 0, 1x state 1, 30x state 2 per block"},
        "dense_attn_tflops": attn_flops(lens, Hq_all) * layers / (graph_dense_ms * 1e-3) / 1e12,
        "dense_step_tokens_per_s": N_full / (graph_dense_ms * 1e-3),
        "note": "attention path only (per layer: selection/store, cache gather, varlen attention); "
                "each layer's q/k/v are [rows, heads*128] views made once per row count in warm-up "
                "(inputs, as a model's projections hand them over); eager steps build a new Context "
                "and step plan every step; timed with CUDA events, max over ranks",
    }
    for st in graphs.values():
        del st
    graphs.clear()
    del graph_dense
    return line


def run_kernels_case(args):
    """Small profiling case: each native kernel launched 3 times on inputs
    larger than L2 (one c2 layer for attention, the KV store, RoPE and the
    fused o_proj GEMM at tp=1, config-5 shapes for scoring/top-k and for the
    reuse-state attention)."""
    from dllmserve_b200 import _native, ops

    _native.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(3)
    lens = workload_lengths()
    N = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=dev)
    rnd = lambda *shape: torch.randn(*shape, device=dev, dtype=torch.bfloat16, generator=g)
    q, k, v = rnd(N, HEADS, HEAD_DIM), rnd(N, KV_HEADS, HEAD_DIM), rnd(N, KV_HEADS, HEAD_DIM)
    for _ in range(3):
        ops.varlen_attention(q, k, v, cu, cu, max(lens))
    pages = (N + 255) // 256 + 8
    kc = torch.zeros(pages, 256, KV_HEADS, HEAD_DIM, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slot = torch.randperm(pages * 256, device=dev, generator=g)[:N].to(torch.int32)
    for _ in range(3):
        ops.store_kvcache(k, v, kc, vc, slot)
    from dllmserve_b200.layers.rotary_embedding import RotaryEmbedding

    rope = RotaryEmbedding(HEAD_DIM, HEAD_DIM, 4096, 500000.0).to(dev)
    pos = torch.cat([torch.arange(L, device=dev) for L in lens])
    for _ in range(3):
        ops.rope_neox(pos, q, k, rope.cos_sin_cache)
    del q, k, v
    # config 5: B=8, L=4096+512, block 32 at the start of the generation, r=0.25
    B5, L5, blk = 8, 4608, 32
    q5, k5, v5 = rnd(B5 * L5, HEADS, HEAD_DIM), rnd(B5 * L5, KV_HEADS, HEAD_DIM), rnd(B5 * L5, KV_HEADS, HEAD_DIM)
    n_keep = min(max(1, int((L5 - blk) * 0.25)), L5 - blk)
    desc = torch.tensor([[b * L5, L5, 4096, blk, n_keep, b * n_keep, 0, 3] for b in range(B5)],
                        dtype=torch.int32, device=dev)
    pages5 = (B5 * n_keep + 255) // 256 + 8
    kc5 = torch.zeros(pages5, 256, KV_HEADS, HEAD_DIM, device=dev, dtype=torch.bfloat16)
    vc5 = torch.zeros_like(kc5)
    slots5 = torch.randperm(pages5 * 256, device=dev, generator=g)[:B5 * n_keep].to(torch.int32)
    for _ in range(3):
        ops.select_kv_store(q5, k5, v5, desc, L5 - blk, True, kc5, vc5, slots5)
    del q5, k5, v5
    # config 5 reuse state (split kernel, paged cache): B=8, 32 block queries,
    # 1,144 cached rows (runs of whole pages, as the block manager allocates) + 32 fresh keys
    B3, n3 = 8, n_keep
    q3, k3, v3 = rnd(B3 * 32, HEADS, HEAD_DIM), rnd(B3 * 32, KV_HEADS, HEAD_DIM), rnd(B3 * 32, KV_HEADS, HEAD_DIM)
    cq = torch.arange(0, B3 * 32 + 1, 32, dtype=torch.int32, device=dev)
    cc = torch.arange(0, B3 * n3 + 1, n3, dtype=torch.int32, device=dev)
    ppseq = (n3 + 255) // 256
    page_order = torch.randperm(pages5, device=dev, generator=g)[:B3 * ppseq]
    slot3 = torch.cat([torch.cat([torch.arange(256, device=dev) + 256 * int(p) for p in page_order[b * ppseq:(b + 1) * ppseq]])[:n3]
                       for b in range(B3)]).to(torch.int32)
    for _ in range(3):
        ops.varlen_attention(q3, k3, v3, cq, cq, 32, k_cache=kc5, v_cache=vc5, slots=slot3,
                             cu_seqlens_slots=cc)
    del q3, k3, v3, kc5, vc5
    # row-parallel o_proj of one config-2 layer through the fused kernel on
    # one rank (dllm_oproj_allreduce at tp=1: the GEMM with its direct epilogue)
    from dllmserve_b200.tp import OprojAllReduce

    x = rnd(N, HEADS * HEAD_DIM)
    w = rnd(HIDDEN, HEADS * HEAD_DIM) * 0.02
    fused = OprojAllReduce(N, HIDDEN, device=dev)
    for _ in range(3):
        fused(x, w)
    torch.cuda.synchronize()
    fused.close()
    if ops.read_device_status(dev) != 0:
        raise RuntimeError("a kernel reported a device error")
    print(json.dumps({"kernels_case": "ok", "launches": ops.LAUNCHES[0]}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-extras", action="store_true",
                    help="only the primary timed loop (used for profiling runs)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5"], default="c2",
                    help="c2 = the headline dense step; c3/c4/c5 = sparse diffusion-block cycle")
    ap.add_argument("--kernels-case", action="store_true",
                    help="run each native kernel 3x on a small case (for ncu captures)")
    ap.add_argument("--cpu-baselines", action="store_true",
                    help="time the reference's CPU path for configs 1, 3, 4 and 5 (one JSON line)")
    ap.add_argument("--cpu-budget", type=float, default=6.0,
                    help="seconds of CPU time per --cpu-baselines measurement")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="layers per step (32 = the workload; fewer only for profiling runs)")
    args = ap.parse_args()
    globals()["LAYERS"] = args.layers
    lens = workload_lengths()
    if args.kernels_case:
        return run_kernels_case(args)
    if args.cpu_baselines:
        return run_cpu_baselines(args)
    if args.workload != "c2" and args.impl == "ours":
        return run_sparse_cycle(args)
    if args.impl == "reference":
        return run_reference_arm(args, lens)
    return run_ours(args, lens)


if __name__ == "__main__":
    sys.exit(main())

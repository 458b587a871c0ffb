"""Benchmark of the d3 prefill hot path on B200 (one JSON line on rank 0).

Headline workload (BASELINE config 3a, "question-blocks/s at 4k state"): the
question pass of one full-attention layer — 16 question blocks of 64 tokens
attending to a 4096-token state plus their own block, 32 query heads, 4 KV
heads, head_dim 128, bf16 — through the sm_100a prefix-bidirectional kernel.
A step = one such pass; value = question blocks per second over all ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

* value / ms_per_step: device time of K attention launches back to back (CUDA
  events on their stream around all K), inputs resident in HBM in eight sets
  used in turn (q, k_q, v_q, a copy of the state K/V and the output: 151 MB,
  larger than L2, so no step finds its inputs there); max over ranks.
  ms_per_launch_alone: one launch event-timed alone after an L2 flush (it
  carries the ~6 us fixed cost of an event-timed launch).
* e2e: the same metric through the public API ``QuestionPipeline`` (which
  calls ``prefix_bidir_attention`` per batch) with every step's question inputs
  (q, k_q, v_q) copied from pinned host memory and its output copied back
  inside the timed region; consecutive steps overlap on three streams (copy
  in, attention, copy out), the L2 is flushed on the compute stream before
  every pass; device-timed from the first copy in to the last copy out. The
  state K/V is the resident snapshot (computed once per request in the
  state-once design).
* extra: state pass, config 3b (16384-token state + 255 blocks of 48), the
  W8A8 GEMM at config 2 (e4m3 and int8) with the act-quant kernel, the fused
  producers (add + RMSNorm + quant, sigmoid gate + quant) against their
  unfused two-kernel form, and the readout, each launch event-timed alone
  after an L2 flush, reported in TFLOP/s or GB/s.
* cpu_baseline: the CPU oracle's question pass (a restatement of
  ops.sdpa_questions in fp32) on all host threads, over a bounded sample.

Multi-GPU (torchrun, NCCL): rank 0 builds the state K/V and broadcasts it to
every rank (the one exchange step, reported separately); each rank then runs
its own 16 question blocks per step (weak scaling, no collective per step).
``--impl reference`` times the reference algorithm's CPU path (the oracle port)
on rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CFG3A = dict(B=16, H=32, Hkv=4, L=64, D=128, S=4096)
CFG3B = dict(B=255, H=32, Hkv=4, L=48, D=128, S=16384)
CFG5 = dict(B=255, H=32, Hkv=4, L=64, D=128, S=16384)
METRIC = "question-blocks/s at 4k state"
L2_FLUSH_BYTES = 256 << 20


def headline_config(world: int) -> dict:
    """The `config` of the headline line, the same for both arms (ours and the reference's)."""
    cfg = CFG3A
    return {"workload": "cfg3a question pass: 16 blocks x 64 tokens over a 4096-token state, "
                        "H32/Hkv4/D128 bf16, one layer, per rank",
            "question_blocks_per_rank": cfg["B"], "state_tokens": cfg["S"], "block_tokens": cfg["L"],
            "parallelism": f"dp{world} (question-block sharding, state KV broadcast once)",
            "l2": f"inputs larger than L2 on the GPU: {ROTATE_SETS} rotating sets of q/k_q/v_q, state K/V "
                  "and output (151 MB), the K steps back to back in one timed region; inputs far larger "
                  "than the CPU caches on the host"}


ROTATE_SETS = 8  # headline input sets used in turn: 8 x 18.9 MB > the 126 MB L2


def attn_flops(B, H, L, D, S, **_):
    """4*H*D*sum_b Lq*(S+Lq) (matmul FLOPs of QK^T and PV)."""
    return 4.0 * H * D * B * L * (S + L)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str) -> float | None:
    """dram_bytes_per_launch recorded from an ncu capture in profiles/<name>."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """SM clock and throttle reasons sampled every 2 ms (NVML) during a region.

    Falls back to `nvidia-smi -lms 200` when NVML is unavailable.
    """

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, float, int]] = []  # (sm_mhz, max_mhz, reasons bitmask)
        self._stop = None
        self._thread = None
        self._proc = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self._stop = threading.Event()

            def run():
                while not self._stop.is_set():
                    try:
                        sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        rs = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
                        self.samples.append((sm, mx, rs))
                    except Exception:  # noqa: BLE001
                        pass
                    time.sleep(0.002)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception:  # noqa: BLE001 - no NVML: nvidia-smi at its minimum period
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                     "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                    text=True)
            except OSError:
                self._proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self._proc is not None:
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            for line in out.splitlines():
                parts = [p.strip() for p in line.split(",")]
                try:
                    self.samples.append((float(parts[0]), float(parts[1]), int(parts[2], 16)))
                except (ValueError, IndexError):
                    continue

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted(name for name, bit in self.REASONS.items() if any(r & bit for _, _, r in self.samples))
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": reasons,
                "samples": len(self.samples), "source": "nvml" if self._thread is not None else "nvidia-smi"}


def make_question_inputs(cfg, seed, device, with_state=True):
    g = torch.Generator().manual_seed(seed)
    B, H, Hkv, L, D, S = (cfg[k] for k in ("B", "H", "Hkv", "L", "D", "S"))
    # model layout: q/k/v come out of the projections as [B, L, heads, D]
    q = torch.randn(B, L, H, D, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
    kq = torch.randn(B, L, Hkv, D, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
    vq = torch.randn(B, L, Hkv, D, generator=g).to(torch.bfloat16).permute(0, 2, 1, 3)
    out = {"q": q, "kq": kq, "vq": vq}
    if with_state:
        out["ks"] = torch.randn(S, Hkv, D, generator=g).to(torch.bfloat16).permute(1, 0, 2)
        out["vs"] = torch.randn(S, Hkv, D, generator=g).to(torch.bfloat16).permute(1, 0, 2)
    if device is not None:
        out = {k: v.to(device) for k, v in out.items()}
    return out


def act_quant_steady(x, mode, stream, copies=6, launches=24):
    """Per-launch device time (ms) of config 2's act quant in a steady stream of
    launches: `copies` inputs of x's shape (together larger than L2) used in
    turn, so no launch finds its input in L2, timed back to back between two
    events (no flush kernels in between, the launch cost overlaps the previous
    launch as it does in the backbone)."""
    from d3_turbo_trt_b200.model import quant
    xs = [x.clone() for _ in range(copies)]
    for i in range(2 * copies):
        quant.quantize_rows(xs[i % copies], mode)
    torch.cuda.synchronize()
    torch.cuda._sleep(int(2e6 * 2))
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(launches):
        quant.quantize_rows(xs[i % copies], mode)
    b.record(stream)
    torch.cuda.synchronize()
    del xs
    return a.elapsed_time(b) / launches


def time_steps(fn, steps, warmup, stream, flush, host_bound=False):
    """Per-step device time (ms) of fn() with an L2 flush before every step.

    A bounded spin kernel (torch.cuda._sleep) is queued first so the host has
    enqueued every step before the GPU reaches the first event: the events then
    see device time only, not the Python launch overhead. ``host_bound=True``
    (the end-to-end measurement) skips it and synchronises after every step,
    so host work inside the step is part of the measured time.
    """
    for _ in range(warmup):
        flush()
        fn()
    torch.cuda.synchronize()
    if not host_bound:
        torch.cuda._sleep(int(2e6 * (1 + 0.2 * steps)))  # ~1 ms + 0.1 ms per step at ~2 GHz
    times = []
    for _ in range(steps):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        times.append((a, b))
        if host_bound:
            stream.synchronize()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


def _fp32(inp):
    return {k: v.float() for k, v in inp.items()}


def cpu_baseline_questions(cfg, target_s=10.0):
    """The reference's CPU question pass (ops.sdpa_questions' call pattern: one torch SDPA per
    block over state + own keys, fp32, oracle.attention.questions_sdpa) on all host threads;
    blocks/s over a bounded sample."""
    from oracle import attention as oattn

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    one = dict(cfg, B=1)
    inp = _fp32(make_question_inputs(one, 99, None))
    fn = lambda: oattn.questions_sdpa(inp["q"], inp["ks"], inp["vs"], inp["kq"], inp["vq"], [one["L"]],
                                      one["D"] ** -0.5)
    fn()  # warm-up
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= target_s:
            break
    return {"value": n / el, "unit": "question-blocks/s", "cores": threads, "kind": "port",
            "sample": f"{n} question blocks of config 3a ({one['L']} tokens vs a {one['S']}-token state, "
                      f"H{one['H']}/Hkv{one['Hkv']}/D{one['D']}), torch SDPA per block in fp32 (the reference's "
                      f"sdpa_questions pattern), {el:.1f} s"}


def run_reference(args):
    """--impl reference: the reference algorithm's CPU path (oracle port) on rank 0."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import attention as oattn

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = CFG3A["B"]  # every step is the whole config-3a pass (16 blocks), as on the GPU
    one = dict(CFG3A, B=sample)
    inp = _fp32(make_question_inputs(one, 7, None))
    fn = lambda: oattn.questions_sdpa(inp["q"], inp["ks"], inp["vs"], inp["kq"], inp["vq"], [one["L"]] * sample,
                                      one["D"] ** -0.5)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    el = time.perf_counter() - t0
    value = sample * args.steps / el
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "question-blocks/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": headline_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "question-blocks/s", "cores": threads, "kind": "port",
                         "sample": f"the whole config-3a pass ({sample} blocks) per step: one torch SDPA per block "
                                   "over state + own keys in fp32, the call pattern of the reference's "
                                   "ops.sdpa_questions (d3trt/model/ops.py:127-171), all host threads"},
        "e2e": {"value": value, "unit": "question-blocks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true", help="skip the secondary workloads")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import torch.distributed as dist
    import d3_turbo_trt_b200 as d3b
    from d3_turbo_trt_b200 import _lib, dist as d3dist
    from d3_turbo_trt_b200.kernels import prefix_bidir as pb
    from d3_turbo_trt_b200.model import quant

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        # NCCL may print its banner on stdout when the communicator comes up (with
        # NCCL_DEBUG set); stdout carries only the JSON line, so it goes to stderr.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev,
                                    pg_options=d3dist.nccl_options())
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    stream = torch.cuda.current_stream(dev)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush = lambda: flush_buf.fill_(1)
    peaks = load_peaks()
    cfg = CFG3A
    scale = cfg["D"] ** -0.5

    # ---- state K/V: built on rank 0, broadcast over NCCL (the exchange step) ----
    state = make_question_inputs(cfg, 1, dev if rank == 0 else None, with_state=True)
    ks = torch.empty(cfg["S"], cfg["Hkv"], cfg["D"], dtype=torch.bfloat16, device=dev)
    vs = torch.empty_like(ks)
    if rank == 0:
        ks.copy_(state["ks"].permute(1, 0, 2))
        vs.copy_(state["vs"].permute(1, 0, 2))
    bcast_ms = None
    if world > 1:
        d3dist.broadcast_state_kv([(ks, vs)], src=0)  # first call also sets up the NCCL communicator
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        dist.barrier()
        t0.record(stream)
        d3dist.broadcast_state_kv([(ks, vs)], src=0)  # timed: the per-request exchange (8 MiB K+V)
        t1.record(stream)
        torch.cuda.synchronize()
        bcast_ms = t0.elapsed_time(t1)
    ks_v, vs_v = ks.permute(1, 0, 2), vs.permute(1, 0, 2)  # [Hkv, S, D] token-major views

    # ---- this rank's question blocks ----
    inp = make_question_inputs(cfg, 100 + rank, dev, with_state=False)
    lens = [cfg["L"]] * cfg["B"]
    out = torch.empty(cfg["B"], cfg["H"], cfg["L"], cfg["D"], dtype=torch.bfloat16, device=dev)
    step = lambda: pb.prefix_bidir_attention(inp["q"], ks_v, vs_v, inp["kq"], inp["vq"], lens, scale=scale, out=out)
    # Input sets used in turn (copies of the state K/V included), together larger
    # than L2: no timed step finds its inputs there, so the K steps run back to
    # back in one timed region with no flush kernels between them.
    sets = [(inp["q"], ks_v, vs_v, inp["kq"], inp["vq"], out)]
    for _ in range(ROTATE_SETS - 1):
        kc, vc = ks.clone(), vs.clone()
        sets.append((inp["q"].clone(), kc.permute(1, 0, 2), vc.permute(1, 0, 2), inp["kq"].clone(),
                     inp["vq"].clone(), torch.empty_like(out)))
    assert sets[1][0].stride() == inp["q"].stride()

    def step_set(i: int) -> None:
        q_i, k_i, v_i, kq_i, vq_i, o_i = sets[i % ROTATE_SETS]
        pb.prefix_bidir_attention(q_i, k_i, v_i, kq_i, vq_i, lens, scale=scale, out=o_i)

    for i in range(max(args.warmup, 3)):
        step_set(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # a bounded spin first, so the host has queued every step before the GPU
        # reaches the first event: the events see device time only
        torch.cuda._sleep(int(2e6 * (1 + 0.2 * args.steps)))
        t_begin.record(stream)
        for i in range(args.steps):
            step_set(i)
        t_end.record(stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    total_ms = t_begin.elapsed_time(t_end)
    # the same launch timed alone after an L2 flush (carries the fixed cost of an event-timed launch)
    alone_ms = statistics.median(time_steps(step, 20, 3, stream, flush))
    del sets
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = cfg["B"] * world / (ms_per_step / 1e3)
    flops = attn_flops(**cfg)
    achieved_tflops = flops / (ms_per_step / 1e3) / 1e12  # per GPU (each rank runs one launch per step)

    # ---- e2e through the public API with host buffers ----
    # QuestionPipeline: each step copies its q/k_q/v_q from pinned host memory,
    # runs the question pass and copies the output back; consecutive steps
    # overlap on three streams (copy in, compute, copy out). The L2 flush runs
    # on the compute stream before every pass.
    from d3_turbo_trt_b200.kernels.pipeline import QuestionPipeline
    depth = 2
    host = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in
            (("q", inp["q"].contiguous()), ("kq", inp["kq"].contiguous()), ("vq", inp["vq"].contiguous()))}
    for k in host:
        host[k].copy_(inp[k].contiguous().cpu())
    host_outs = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(depth)]
    host_out = host_outs[0]
    pipe = QuestionPipeline(ks_v, vs_v, scale=scale, depth=depth, before_compute=flush)
    lens_list = [cfg["L"]] * cfg["B"]
    for i in range(max(args.warmup, 3)):
        pipe.submit(host["q"], host["kq"], host["vq"], lens_list, host_outs[i % depth])
    pipe.synchronize()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    e0.record(cur)
    pipe.wait_stream(cur)
    for i in range(args.steps):
        pipe.submit(host["q"], host["kq"], host["vq"], lens_list, host_outs[i % depth])
    pipe.join(cur)
    e1.record(cur)
    pipe.synchronize()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = host_out.numel() * host_out.element_size()

    extra = {}
    if not args.no_extra:
        extra = secondary(dev, stream, flush, peaks, quant, pb, d3b)
        if world == 1:
            extra["cfg4_e2e_64_layers"] = cfg4_e2e(dev, stream, flush, peaks)
    # config 5 at every N: the request split over the ranks (strong) and 64 independent requests
    cfg5 = cfg5_strong(dev, stream, flush, peaks, pb, d3dist, rank, world)
    cfg5_dp = dp_requests(dev, stream, flush, pb, rank, world)
    if world > 1:
        dist.barrier()

    if rank == 0:
        # the CPU baseline is a single-process figure: measured at N = 1 only
        cpu = None if (args.no_cpu or world > 1) else cpu_baseline_questions(cfg)
        traffic = profile_traffic("prefix_bidir_cfg3a.md")  # per launch, from the committed ncu summary
        peak = peaks["bf16_tflops"]
        line = {
            "metric": METRIC, "value": value, "unit": "question-blocks/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q/k/v)",
            "config": headline_config(world),
            "roofline": {"bound": "tensor", "achieved": achieved_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved_tflops / peak, "traffic": traffic,
                         "kernel": "prefix_bidir_dual_kernel<128,bf16>",
                         "algorithmic_flops_per_launch": flops,
                         "peak_source": f"{peaks['source']} bf16 dense (burst)"},
            "e2e": {"value": cfg["B"] * world / (e2e_ms / 1e3), "unit": "question-blocks/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "api": "d3_turbo_trt_b200.kernels.pipeline.QuestionPipeline (prefix_bidir_attention per step)",
                    "overlap": f"{depth} batches in flight: copy in / attention / copy out on separate streams",
                    "l2": "flushed on the compute stream before every pass"},
            "gpu_launches": args.steps,
            "ms_per_launch_alone": alone_ms,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "state_kv_broadcast_ms": bcast_ms,
            "cfg5_strong_scaling": cfg5,
            "cfg5_dp_requests": cfg5_dp,
            "extra": extra,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cfg5_strong(dev, stream, flush, peaks, pb, d3dist, rank, world, layers=4):
    """Config 5, one request split over the ranks: 255 question blocks of 64 tokens over a
    16384-token state, H32/Hkv4/D128, through `layers` full-attention layers (the reference
    runs the state once, then the question blocks, layer by layer: d3trt/model/core.py:146-181).

    Rank 0 runs every layer's state pass (dense attention over the 16384 state tokens) and
    posts that layer's K/V broadcast (one 32 MiB buffer) right behind it, so layer l crosses
    NVLink while layer l+1's state pass runs. Every rank then runs its contiguous,
    length-sorted shard of the blocks through the layers, each layer once its K/V has landed
    (rank 0 holds them already). Device-timed from a common start (barrier), max over ranks:
    the state pass on rank 0, the broadcast still in flight when it ends, and the question
    phase after it. blocks/s = 255 / (question phase), the phase counted from the end of
    the state pass to the last rank's last question pass (so an exposed broadcast counts)."""
    import torch.distributed as dist

    cfg = CFG5
    S, H, Hkv, D, L, nb = cfg["S"], cfg["H"], cfg["Hkv"], cfg["D"], cfg["L"], cfg["B"]
    ex = d3dist.StateKVExchange(layers, S, Hkv, D, dtype=torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(55)
    if rank == 0:
        ex.buffers.normal_(generator=gen)
        q_state = torch.randn(1, S, H, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
        st_out = torch.empty(1, H, S, D, dtype=torch.bfloat16, device=dev)
    else:
        ex.buffers.zero_()
    lengths = [L] * nb
    order = d3dist.length_order(lengths)
    lo, hi = d3dist.shard_bounds(nb, world, rank)
    mine = [order[i] for i in range(lo, hi)]
    q = torch.randn(len(mine), L, H, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    kq = torch.randn(len(mine), L, Hkv, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    vq = torch.randn(len(mine), L, Hkv, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    out = torch.empty(len(mine), H, L, D, dtype=torch.bfloat16, device=dev)
    lens = [lengths[i] for i in mine]

    def request():
        ev = {k: torch.cuda.Event(enable_timing=True) for k in ("start", "state", "last_kv", "end")}
        flush()
        if world > 1:
            dist.barrier()
        ev["start"].record(stream)
        for layer in range(layers):
            if rank == 0:
                k, v = ex.kv(layer)
                pb.state_attention(q_state, k[None], v[None], scale=D ** -0.5, out=st_out)
            ex.post(layer)
        ev["state"].record(stream)
        for layer in range(layers):
            if rank != 0:
                ex.wait(layer)
            if layer == layers - 1:
                ev["last_kv"].record(stream)
            k, v = ex.kv(layer)
            pb.prefix_bidir_attention(q, k, v, kq, vq, lens, scale=D ** -0.5, out=out)
        ev["end"].record(stream)
        if rank == 0:
            for layer in range(layers):
                ex.wait(layer)
        torch.cuda.synchronize()
        return {k: ev["start"].elapsed_time(e) for k, e in ev.items() if k != "start"}

    for _ in range(2):
        request()
    runs = [request() for _ in range(5)]
    state_ms = statistics.median(r["state"] for r in runs)  # rank 0's is the one that counts
    end_ms = statistics.median(r["end"] for r in runs)
    kv_ms = statistics.median(r["last_kv"] for r in runs)
    t = torch.tensor([state_ms if rank == 0 else 0.0, end_ms, kv_ms if rank != 0 else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    state_ms, end_ms, kv_ms = (float(x) for x in t.tolist())
    question_ms = end_ms - state_ms
    bcast_exposed = max(0.0, kv_ms - state_ms) if world > 1 else 0.0
    # the 32 MiB layer broadcast on its own, for reference (all ranks, same order)
    bcast_alone = None
    if world > 1:
        ex.post(0)
        ex.wait(0)
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ex.post(0)
        ex.wait(0)
        b.record(stream)
        torch.cuda.synchronize()
        bt = torch.tensor([a.elapsed_time(b)], device=dev)
        dist.all_reduce(bt, op=dist.ReduceOp.MAX)
        bcast_alone = float(bt.item())
    fl = attn_flops(**cfg) * layers
    return {"workload": f"{nb} blocks x {L} tokens over a {S}-token state, H{H}/Hkv{Hkv}/D{D} bf16, "
                        f"{layers} full-attention layers, blocks split over {world} rank(s)",
            "value": nb / (question_ms / 1e3), "unit": "question-blocks/s (per request, all layers)",
            "question_phase_ms": question_ms, "state_pass_ms_rank0": state_ms,
            "broadcast_exposed_ms": bcast_exposed, "broadcast_32MiB_alone_ms": bcast_alone,
            "broadcast_gbs_alone": (2 * S * Hkv * D * 2) / bcast_alone / 1e6 if bcast_alone else None,
            "question_tflops_total": fl / question_ms / 1e9, "blocks_per_rank": len(mine),
            "timing": "device events from a common barrier, median of 5 requests, max over ranks; "
                      "L2 flushed before each request", "scaling": "strong"}


def dp_requests(dev, stream, flush, pb, rank, world, n_req=64):
    """Config 5's independent requests spread data-parallel: 64 requests, each one
    full-attention layer's state pass over 16384 tokens and its 255 x 64-token question
    pass, ceil/floor(64 / N) per rank, no communication. Device-timed, max over ranks."""
    import torch.distributed as dist

    cfg = CFG5
    S, H, Hkv, D, L, nb = cfg["S"], cfg["H"], cfg["Hkv"], cfg["D"], cfg["L"], cfg["B"]
    lo, hi = (rank * n_req) // world, ((rank + 1) * n_req) // world
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    kv = torch.randn(2, S, Hkv, D, generator=gen, device=dev, dtype=torch.bfloat16)
    ks, vs = kv[0].permute(1, 0, 2), kv[1].permute(1, 0, 2)
    q_state = torch.randn(1, S, H, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    st_out = torch.empty(1, H, S, D, dtype=torch.bfloat16, device=dev)
    q = torch.randn(nb, L, H, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    kq = torch.randn(nb, L, Hkv, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    vq = torch.randn(nb, L, Hkv, D, generator=gen, device=dev, dtype=torch.bfloat16).permute(0, 2, 1, 3)
    out = torch.empty(nb, H, L, D, dtype=torch.bfloat16, device=dev)
    lens = [L] * nb

    def one():
        flush()
        pb.state_attention(q_state, ks[None], vs[None], scale=D ** -0.5, out=st_out)
        pb.prefix_bidir_attention(q, ks, vs, kq, vq, lens, scale=D ** -0.5, out=out)

    one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(hi - lo):
        one()
    b.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    return {"workload": f"{n_req} independent requests, each a {S}-token state pass and {nb} x {L}-token "
                        f"question pass (one full-attention layer, H{H}/Hkv{Hkv}/D{D} bf16), spread over "
                        f"{world} rank(s), no communication",
            "value": n_req / (ms / 1e3), "unit": "requests/s", "ms": ms,
            "requests_per_rank_max": -(-n_req // world), "scaling": "strong",
            "timing": "device events, max over ranks, L2 flushed before each request"}


class _RandomWeights(dict):
    """The 64-layer backbone's parameters, generated on the GPU when the backbone reads them
    (by the model's own names), so the bf16 weights never coexist: each one is quantised to
    FP8 by the backbone and dropped. N(0, 1/sqrt(fan_in)) projections, small norm weights."""

    def __init__(self, config, vocab, dev, seed=4):
        super().__init__()
        self.c, self.vocab, self.dev = config, vocab, dev
        self.gen = torch.Generator(device=dev).manual_seed(seed)

    def _n(self, *shape, std):
        return (torch.randn(*shape, generator=self.gen, device=self.dev, dtype=torch.float32) * std).to(torch.bfloat16)

    def __getitem__(self, name):
        c = self.c
        H, I = c.hidden_size, c.intermediate_size
        if name == "embed_tokens.weight":
            return self._n(self.vocab, H, std=1.0)
        if name.endswith("norm.weight") and "linear_attn" not in name:
            return self._n(c.head_dim if ("q_norm" in name or "k_norm" in name) else H, std=0.1)
        leaf = name.split(".")[-2] if name.endswith(".weight") else name.split(".")[-1]
        shapes = {"q_proj": (2 * c.num_attention_heads * c.head_dim, H), "k_proj": (c.num_key_value_heads * c.head_dim, H),
                  "v_proj": (c.num_key_value_heads * c.head_dim, H), "o_proj": (H, c.num_attention_heads * c.head_dim),
                  "in_proj_qkv": (c.conv_dim, H), "in_proj_z": (c.value_dim, H),
                  "in_proj_b": (c.linear_num_value_heads, H), "in_proj_a": (c.linear_num_value_heads, H),
                  "out_proj": (H, c.value_dim), "gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}
        if leaf in shapes:
            n, k = shapes[leaf]
            return self._n(n, k, std=k ** -0.5)
        if leaf == "conv1d":
            return self._n(c.conv_dim, 1, c.linear_conv_kernel_dim, std=0.5)
        if leaf == "dt_bias":
            return torch.ones(c.linear_num_value_heads, dtype=torch.bfloat16, device=self.dev)
        if leaf == "A_log":
            return torch.log(torch.rand(c.linear_num_value_heads, generator=self.gen, device=self.dev) * 1.95 + 0.05
                             ).to(torch.bfloat16)
        if leaf == "norm":  # the GDN output's gated norm
            return (1 + self._n(c.linear_value_head_dim, std=0.1).float()).to(torch.bfloat16)
        raise KeyError(name)


def cfg4_e2e(dev, stream, flush, peaks):
    """Config 4: the state-once prefill of a random-init 64-layer d3 backbone end to end
    (d3trt/model/core.py:146-181 on this library's kernels, model/backbone.py): hidden 5120,
    MLP 17408, 16 full-attention layers (32 q / 4 kv heads, head_dim 128), 48 Gated DeltaNet
    layers (16 / 48 heads), every Linear W8A8 FP8, bf16 RMSNorm; token ids uniform over a
    151k vocabulary; a 4096-token state and 255 question blocks of 48 tokens; the 255-way
    fp32 readout (N(0, 0.02)) at each block's last token. Both GDN scans run on this
    library's chunked forms (the state pass with the inter-chunk recurrence, the question
    pass with one shared state). Timed on the device: state pass, question pass, readout;
    end to end: token ids from pinned host memory and probabilities back to it."""
    from d3_turbo_trt_b200.model.backbone import BackboneConfig, D3Backbone
    from d3_turbo_trt_b200.model.batching import QuestionBatcher

    cfg = BackboneConfig()
    vocab, S, nb, L, n_opt = 151_936, 4096, 255, 48, 255
    gdn_state = "ours"
    t0 = time.perf_counter()
    bb = D3Backbone(cfg, _RandomWeights(cfg, vocab, dev), device=dev, mode="fp8", gdn_state=gdn_state)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(44)
    state_ids = torch.randint(0, vocab, (1, S), generator=g).pin_memory()
    q_ids = torch.randint(0, vocab, (nb, L), generator=g)
    pieces = q_ids.tolist()  # the request's question pieces as the backend holds them (token lists)
    batcher = QuestionBatcher(dev, pad_id=0, stream=stream)
    lengths = [L] * nb
    readout = (torch.randn(n_opt, cfg.hidden_size, generator=g) * 0.02).to(dev)
    counts = torch.full((nb,), n_opt, dtype=torch.int32, device=dev)
    host_probs = torch.empty(nb, n_opt, dtype=torch.float32, pin_memory=True)

    def request():
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        flush()
        ev[0].record(stream)
        s_ids = state_ids.to(dev, non_blocking=True)
        qi, _ = batcher.build(pieces)  # padded ids + lengths: one pinned buffer, one copy
        ev[1].record(stream)
        snap = bb.state(s_ids)
        ev[2].record(stream)
        hidden = bb.questions(snap, qi, lengths, state_len=S)
        ev[3].record(stream)
        probs = bb.probabilities(hidden, readout, counts)
        host_probs.copy_(probs, non_blocking=True)
        ev[4].record(stream)
        torch.cuda.synchronize()
        return [ev[0].elapsed_time(e) for e in ev[1:]]

    request()  # warm-up (workspaces, tensor maps, FLA's autotune)
    runs = [request() for _ in range(2)]
    t_in, t_state, t_q, t_end = (statistics.median(r[i] for r in runs) for i in range(4))
    tokens = S + nb * L
    dense = 0
    for lw in bb.layers:
        for v in lw.values():
            if hasattr(v, "quant") and v.quant:
                dense += v.mod.in_features * v.mod.out_features
    gemm_flops = 2.0 * dense * tokens
    return {"workload": "64-layer d3 backbone (16 attention + 48 GDN layers, hidden 5120, W8A8 FP8), "
                        f"{S}-token state + {nb} x {L}-token question blocks + 255-way readout, random init",
            "value": nb / (t_end / 1e3), "unit": "question-blocks/s (end to end, one request)",
            "e2e_ms": t_end, "h2d_ms": t_in, "state_pass_ms": t_state - t_in, "question_pass_ms": t_q - t_state,
            "readout_and_copy_ms": t_end - t_q, "linear_params": dense, "gemm_tflop": gemm_flops / 1e12,
            "h2d_bytes": (state_ids.numel() + q_ids.numel()) * 8 + nb * 4, "d2h_bytes": host_probs.numel() * 4,
            "gdn_state_scan": gdn_state, "build_s": build_s,
            "timing": "device events, median of 2 requests after one warm-up, L2 flushed before each"}


FP8_SPEC_TFLOPS = 4500.0  # B200 dense e4m3 / int8, nominal


def model_gemms(dev, stream, flush):
    """The config-4 backbone's W8A8 projections at the question pass's 255 x 48 = 12240
    rows, e4m3 codes with per-row and per-channel scales, bf16 out: this library's kernel
    against torch._scaled_mm (a CUTLASS sm100 kernel) on the same operands."""
    from d3_turbo_trt_b200.model import quant

    g = torch.Generator(device=dev).manual_seed(12)
    M, out = 12240, {}
    for name, N, K in (("mlp_gate_or_up", 17408, 5120), ("mlp_down", 5120, 17408), ("attn_q_gate", 8192, 5120),
                       ("attn_k_or_v", 512, 5120), ("gdn_in_proj_qkv", 10240, 5120), ("gdn_out_proj", 5120, 6144)):
        a = (torch.randn(M, K, generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
        w = (torch.randn(N, K, generator=g, device=dev) * 0.5).to(torch.float8_e4m3fn)
        sa = torch.rand(M, generator=g, device=dev) + 0.5
        sw = torch.rand(N, generator=g, device=dev) + 0.5
        ours = statistics.median(time_steps(lambda: quant.scaled_mm(a, w, sa, sw, out_dtype=torch.bfloat16),
                                            10, 3, stream, flush))
        wt = w.t()
        lib = statistics.median(time_steps(lambda: torch._scaled_mm(a, wt, scale_a=sa[:, None], scale_b=sw[None, :],
                                                                    out_dtype=torch.bfloat16), 10, 3, stream, flush))
        fl = 2.0 * M * N * K
        out[name] = {"M": M, "N": N, "K": K, "ms": ours, "tflops": fl / ours / 1e9,
                     "frac_spec_4500": fl / ours / 1e9 / FP8_SPEC_TFLOPS, "torch_scaled_mm_ms": lib,
                     "speedup_vs_torch": lib / ours}
        del a, w, wt
    return out


def secondary(dev, stream, flush, peaks, quant, pb, d3b):
    """State pass, config 3b, W8A8 GEMM (config 2), act quant and readout."""
    res = {}
    bf16_peak = peaks["bf16_tflops"]
    # state pass of config 3a: [1, 32, 4096, 128] over [1, 4, 4096, 128]
    g = torch.Generator().manual_seed(3)
    S, H, Hkv, D = 4096, 32, 4, 128
    q = torch.randn(1, S, H, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    k = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    v = torch.randn(1, S, Hkv, D, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    t = statistics.median(time_steps(lambda: pb.state_attention(q, k, v, scale=D ** -0.5), 10, 3, stream, flush))
    fl = 4.0 * H * D * S * S
    res["state_pass_4k"] = {"ms": t, "tflops": fl / t / 1e9, "frac_bf16_peak": fl / t / 1e9 / bf16_peak}
    del q, k, v
    # config 3b: 16384-token state + 255 blocks of 48
    inp = make_question_inputs(CFG3B, 4, dev)
    lens = [48] * 255
    t = statistics.median(time_steps(lambda: pb.prefix_bidir_attention(
        inp["q"], inp["ks"], inp["vs"], inp["kq"], inp["vq"], lens, scale=D ** -0.5), 5, 3, stream, flush))
    fl = attn_flops(**CFG3B)
    res["cfg3b_question_pass"] = {"ms": t, "blocks_per_s": 255 / (t / 1e3), "tflops": fl / t / 1e9,
                                  "frac_bf16_peak": fl / t / 1e9 / bf16_peak}
    del inp
    # config 3a's blocks and state at the model's own attention shape (24 query heads, 4 KV
    # heads, head_dim 256: the D = 256 kernel, whose O accumulator alone fills 256 TMEM columns)
    c256 = dict(CFG3A, H=24, D=256)
    inp = make_question_inputs(c256, 5, dev)
    t = statistics.median(time_steps(lambda: pb.prefix_bidir_attention(
        inp["q"], inp["ks"], inp["vs"], inp["kq"], inp["vq"], [c256["L"]] * c256["B"], scale=256 ** -0.5),
        10, 3, stream, flush))
    fl = attn_flops(**c256)
    res["cfg3a_question_pass_h24_d256"] = {"ms": t, "blocks_per_s": c256["B"] / (t / 1e3), "tflops": fl / t / 1e9,
                                       "frac_bf16_peak": fl / t / 1e9 / bf16_peak}
    del inp
    # config 2: W8A8 [4096, 5120] x [13824, 5120]^T
    M, K, N = 4096, 5120, 13824
    x = torch.randn(M, K, generator=g)
    cols = torch.randperm(K, generator=g)[: K // 100]
    x[:, cols] *= 20.0
    x = x.to(torch.bfloat16).to(dev)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(dev)
    gemm_flops = 2.0 * M * N * K
    fp8_peak = 2 * bf16_peak  # dense e4m3 / int8 rate is twice bf16 on B200
    for mode in ("fp8", "int8"):
        layer = quant.QuantLinear(K, N, mode=mode, dtype=torch.bfloat16, device=dev)
        layer.load_full(w)
        qa, sa = quant.quantize_rows(x, mode)
        tg = statistics.median(time_steps(lambda: quant.scaled_mm(qa, layer.weight, sa, layer.weight_scale,
                                                                   out_dtype=torch.bfloat16), 10, 3, stream, flush))
        tq = statistics.median(time_steps(lambda: quant.quantize_rows(x, mode), 10, 3, stream, flush))
        tq_run = act_quant_steady(x, mode, stream)
        tl = statistics.median(time_steps(lambda: layer(x), 10, 3, stream, flush))
        qbytes = M * K * 2 + M * K + M * 4
        res[f"w8a8_{mode}_cfg2"] = {
            "gemm_ms": tg, "gemm_tflops": gemm_flops / tg / 1e9, "frac_dense_peak": gemm_flops / tg / 1e9 / fp8_peak,
            "frac_spec_4500": gemm_flops / tg / 1e9 / FP8_SPEC_TFLOPS,
            "act_quant_ms": tq, "act_quant_gbs": qbytes / tq / 1e6, "act_quant_frac_hbm": qbytes / tq / 1e6 / peaks["hbm_gbs"],
            "act_quant_steady_ms": tq_run, "act_quant_steady_gbs": qbytes / tq_run / 1e6,
            "act_quant_steady_frac_hbm": qbytes / tq_run / 1e6 / peaks["hbm_gbs"],
            "act_quant_steady_note": "launches back to back over 6 rotating inputs (252 MB > L2), no flush; "
                                     "act_quant_ms is one launch after an L2 flush, event-timed alone",
            "quant_linear_ms": tl}
        if mode == "fp8":
            ts = statistics.median(time_steps(lambda: torch._scaled_mm(
                qa, layer.weight.t(), scale_a=sa, scale_b=layer.weight_scale[None, :], out_dtype=torch.bfloat16),
                10, 3, stream, flush))
            res["w8a8_fp8_cfg2"]["torch_scaled_mm_ms"] = ts
        else:
            ti = statistics.median(time_steps(lambda: torch._int_mm(qa, layer.weight.t()), 10, 3, stream, flush))
            res["w8a8_int8_cfg2"]["torch_int_mm_ms"] = ti
            # the same output as torch._int_mm (raw int32 accumulators, no scales): like for like
            t32 = statistics.median(time_steps(lambda: quant.scaled_mm(qa, layer.weight, None, None,
                                                                        out_dtype=torch.int32), 10, 3, stream, flush))
            res["w8a8_int8_cfg2"]["gemm_i32_out_ms"] = t32
        del layer, qa, sa
    res["fp8_int8_peak_tflops"] = fp8_peak
    del x, w
    res["w8a8_fp8_model_shapes"] = model_gemms(dev, stream, flush)
    # launch-bound regime: back-to-back config-1-sized question passes, eager wrapper calls
    # against replays of a captured CUDA graph (events around the whole loop: host gaps count)
    from d3_turbo_trt_b200.kernels.graphs import QuestionPassGraph
    c1 = dict(B=8, H=8, Hkv=2, L=32, D=64, S=512)
    ks1 = torch.randn(c1["Hkv"], c1["S"], c1["D"], generator=g).to(torch.bfloat16).to(dev)
    vs1 = torch.randn(c1["Hkv"], c1["S"], c1["D"], generator=g).to(torch.bfloat16).to(dev)
    q1 = torch.randn(c1["B"], c1["H"], c1["L"], c1["D"], generator=g).to(torch.bfloat16).to(dev)
    kq1 = torch.randn(c1["B"], c1["Hkv"], c1["L"], c1["D"], generator=g).to(torch.bfloat16).to(dev)
    vq1 = torch.randn(c1["B"], c1["Hkv"], c1["L"], c1["D"], generator=g).to(torch.bfloat16).to(dev)
    lens1 = [c1["L"]] * c1["B"]
    gp = QuestionPassGraph(ks1, vs1, rows=c1["B"], width=c1["L"], heads=c1["H"], scale=c1["D"] ** -0.5)
    gp.q.copy_(q1); gp.k_q.copy_(kq1); gp.v_q.copy_(vq1); gp.set_lengths(lens1)
    calls = 200

    def loop_us(fn):
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(calls):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / calls

    eager_us = loop_us(lambda: pb.prefix_bidir_attention(q1, ks1, vs1, kq1, vq1, lens1, scale=c1["D"] ** -0.5))
    graph_us = loop_us(gp.replay)
    kern_us = statistics.median(time_steps(gp.replay, 10, 3, stream, flush)) * 1e3
    res["question_pass_call_cost_cfg1"] = {"eager_us_per_call": eager_us, "graph_replay_us_per_call": graph_us,
                                           "kernel_us": kern_us,
                                           "workload": "config 1 pass (8 blocks x 32 over a 512-token state, D64)"}
    del gp
    # fused producers at config 2 rows (4096 x 5120): residual add + RMSNorm + fp8 quant of
    # the normed rows in one kernel, against the same two steps as separate kernels
    from d3_turbo_trt_b200.model import fused
    r = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    dl = torch.randn(M, K, generator=g).to(torch.bfloat16).to(dev)
    w1 = (1 + torch.randn(K, generator=g) * 0.1).to(dev)
    tf = statistics.median(time_steps(lambda: fused.add_rmsnorm_quant(r, dl, w1, 1e-6, "fp8"), 10, 3, stream, flush))
    tu = statistics.median(time_steps(
        lambda: quant.quantize_rows(fused.add_rmsnorm(r, dl, w1, 1e-6)[1], "fp8"), 10, 3, stream, flush))
    nbytes = M * K * (2 + 2 + 2 + 1) + M * 4 + K * 4  # read residual, delta; write hidden, codes, scale
    res["add_rmsnorm_fp8_quant_cfg2"] = {"fused_ms": tf, "unfused_ms": tu, "fused_gbs": nbytes / tf / 1e6,
                                         "fused_frac_hbm": nbytes / tf / 1e6 / peaks["hbm_gbs"]}
    del r, dl
    # sigmoid gate + fp8 quant for o_proj: 4096 tokens x 32 heads x 128
    Tt, Hh, Dd = 4096, 32, 128
    at = torch.randn(1, Hh, Tt, Dd, generator=g).to(torch.bfloat16).to(dev).permute(0, 2, 1, 3)
    gt = torch.randn(1, Tt, Hh, 2 * Dd, generator=g).to(torch.bfloat16).to(dev)[..., Dd:]
    tf = statistics.median(time_steps(lambda: fused.sigmoid_gate_quant(at, gt, "fp8"), 10, 3, stream, flush))
    tu = statistics.median(time_steps(
        lambda: quant.quantize_rows(fused.sigmoid_gate(at, gt).reshape(Tt, Hh * Dd), "fp8"), 10, 3, stream, flush))
    nbytes = Tt * Hh * Dd * (2 + 2 + 1) + Tt * 4
    res["sigmoid_gate_fp8_quant_4k_tokens"] = {"fused_ms": tf, "unfused_ms": tu, "fused_gbs": nbytes / tf / 1e6,
                                               "fused_frac_hbm": nbytes / tf / 1e6 / peaks["hbm_gbs"]}
    del at, gt
    # state snapshot of the 64-layer model at a 4096-token state, packed into one arena block
    res["state_snapshot_4k_64_layers"] = snapshot_line(dev, stream, flush, peaks)
    # one GDN layer's question pass (255 blocks x 48 tokens, 48 value heads), against the
    # reference's GPU library kernels on the inputs the reference builds for them
    res["gdn_question_pass_255x48"] = gdn_line(dev, stream, flush)
    res["gdn_state_pass_4096x48"] = gdn_state_line(dev, stream, flush)
    # readout: 255 blocks x 5120 x 255 options
    hidden = torch.randn(255, 5120, generator=g).to(torch.bfloat16).to(dev)
    ro = (torch.randn(255, 5120, generator=g) * 0.02).to(dev)
    counts = torch.full((255,), 255, dtype=torch.int32, device=dev)
    t = statistics.median(time_steps(lambda: d3b.probabilities_tensor(hidden, ro, counts, temperature=1.0), 10, 3,
                                     stream, flush))
    res["readout_255x5120x255"] = {"ms": t}
    return res


def gdn_line(dev, stream, flush):
    """d3b_gated_delta_rule on one GDN layer's question pass; FLA's fused recurrent and chunk
    kernels (the reference's GPU paths, core.py:360-372) timed on the repeated q/k and the
    per-row copy of the state they are called with (the copy itself timed apart)."""
    from d3_turbo_trt_b200.model import gdn
    from d3_turbo_trt_b200.profile import gdn_question_inputs

    x = gdn_question_inputs(dev)
    B, T, H, K = x["q"].shape
    HV, V = x["v"].shape[2:]
    out = torch.empty_like(x["v"])
    h0 = x["h0"].expand(B, -1, -1, -1)
    t_ours = statistics.median(time_steps(lambda: gdn.gated_delta_rule(
        x["q"], x["k"], x["v"], g=x["g"], beta=x["beta"], initial_state=h0, out=out, algo="chunk"),
        5, 3, stream, flush))
    t_rec = statistics.median(time_steps(lambda: gdn.gated_delta_rule(
        x["q"], x["k"], x["v"], g=x["g"], beta=x["beta"], initial_state=h0, out=out, algo="recurrent"),
        5, 3, stream, flush))
    line = {"ours_chunk_ms": t_ours, "ours_recurrent_ms": t_rec,
            "workload": f"{B} blocks x {T} tokens, {H} q/k heads -> {HV} value heads, K=V={K}, shared initial state"}
    t_copy = statistics.median(time_steps(lambda: h0.contiguous(), 5, 3, stream, flush))
    line["reference_state_copy_ms"] = t_copy
    try:
        from fla.ops.gated_delta_rule import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule
    except Exception as exc:  # noqa: BLE001 - the library is optional on the box
        line["fla"] = f"unavailable: {type(exc).__name__}"
        return line
    rep = HV // H
    qr, kr = x["q"].repeat_interleave(rep, 2), x["k"].repeat_interleave(rep, 2)
    init = h0.contiguous()
    kw = dict(g=x["g"], beta=x["beta"], initial_state=init, output_final_state=False, use_qk_l2norm_in_kernel=True)
    line["fla_fused_recurrent_ms"] = statistics.median(time_steps(
        lambda: fused_recurrent_gated_delta_rule(qr, kr, x["v"], **kw), 5, 3, stream, flush))
    line["fla_chunk_ms"] = statistics.median(time_steps(
        lambda: chunk_gated_delta_rule(qr, kr, x["v"], **kw), 5, 3, stream, flush))
    o_ref, _ = fused_recurrent_gated_delta_rule(qr, kr, x["v"], **kw)
    o, _ = gdn.gated_delta_rule(x["q"], x["k"], x["v"], g=x["g"], beta=x["beta"], initial_state=h0,
                                algo="recurrent")
    line["max_abs_diff_recurrent_vs_fla_recurrent"] = float((o.float() - o_ref.float()).abs().max())
    o_chk, _ = chunk_gated_delta_rule(qr, kr, x["v"], **kw)
    o, _ = gdn.gated_delta_rule(x["q"], x["k"], x["v"], g=x["g"], beta=x["beta"], initial_state=h0, algo="chunk")
    line["max_abs_diff_chunk_vs_fla_chunk"] = float((o.float() - o_chk.float()).abs().max())
    return line


def gdn_state_line(dev, stream, flush):
    """One GDN layer's state pass (config 4): one row of 4096 tokens, 16 q/k heads feeding 48
    value heads, K = V = 128, final state; the inter-chunk form against FLA's chunked kernel
    (the reference's GPU path for ops.chunk_gated_delta_rule) on the same inputs."""
    from d3_turbo_trt_b200.model import gdn

    g = torch.Generator().manual_seed(5)
    B, T, H, HV, K, V = 1, 4096, 16, 48, 128, 128
    q = torch.randn(B, T, H, K, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B, T, H, K, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, T, HV, V, generator=g).to(torch.bfloat16).to(dev)
    gl = (-torch.rand(B, T, HV, generator=g) * 0.5).to(dev)
    beta = torch.sigmoid(torch.randn(B, T, HV, generator=g)).to(torch.bfloat16).to(dev)
    kw = dict(g=gl, beta=beta, initial_state=None, output_final_state=True, use_qk_l2norm_in_kernel=True)
    line = {"workload": f"{B} row x {T} tokens, {H} q/k heads -> {HV} value heads, K=V={K}, final state",
            "ours_chunk_state_ms": statistics.median(time_steps(
                lambda: gdn.chunk_gated_delta_rule(q, k, v, **kw), 5, 3, stream, flush))}
    try:
        from fla.ops.gated_delta_rule import chunk_gated_delta_rule
    except Exception as exc:  # noqa: BLE001 - the library is optional on the box
        line["fla"] = f"unavailable: {type(exc).__name__}"
        return line
    qr, kr = q.repeat_interleave(HV // H, 2), k.repeat_interleave(HV // H, 2)
    line["fla_chunk_ms"] = statistics.median(time_steps(lambda: chunk_gated_delta_rule(qr, kr, v, **kw), 5, 3,
                                                        stream, flush))
    o_ref, s_ref = chunk_gated_delta_rule(qr, kr, v, **kw)
    o, s_ours = gdn.chunk_gated_delta_rule(q, k, v, **kw)
    line["max_abs_diff_vs_fla_chunk"] = float((o.float() - o_ref.float()).abs().max())
    line["max_abs_diff_final_state_vs_fla_chunk"] = float((s_ours - s_ref.float()).abs().max())
    return line


def snapshot_line(dev, stream, flush, peaks):
    """Packing a state snapshot (cache format): one copy launch over 128 tensors, bytes held
    against the reference's list of views, and the pinned-host round trip of the packed block."""
    from d3_turbo_trt_b200.model.snapshot import SnapshotArena, SnapshotLayout, copy_segments, pack_snapshot
    from d3_turbo_trt_b200.profile import state_snapshot

    snap = state_snapshot(dev)
    layout = SnapshotLayout.of(snap)
    storages = {}
    for e in snap:
        for t in (getattr(e, f) for f in e.__slots__):
            storages[t.untyped_storage().data_ptr()] = t.untyped_storage().nbytes()
    arena = SnapshotArena(2 * layout.nbytes + (1 << 20), dev)
    block = arena.allocate(layout.nbytes)
    table = layout.table(snap, arena.buffer.data_ptr() + block.offset)
    tk = statistics.median(time_steps(lambda: copy_segments(table, dev), 10, 3, stream, flush))
    del block
    tcall = statistics.median(time_steps(lambda: pack_snapshot(snap, arena), 10, 3, stream, flush, host_bound=True))
    packed = pack_snapshot(snap, arena)
    host = packed.to_host()
    view = packed.block.bytes_view()[: layout.nbytes]
    t_d2h = statistics.median(time_steps(lambda: host.host.copy_(view, non_blocking=True), 5, 2, stream, flush))
    del packed, view
    t_h2d = statistics.median(time_steps(lambda: host.restore(arena), 5, 2, stream, flush, host_bound=True))
    moved = 2 * layout.tensor_bytes  # read + write, the measure of the copy peak
    return {"tensors": len(layout.slots), "tensor_bytes": layout.tensor_bytes, "block_bytes": layout.nbytes,
            "reference_held_bytes": sum(storages.values()), "pack_kernel_ms": tk,
            "pack_kernel_gbs": moved / tk / 1e6, "pack_kernel_frac_hbm": moved / tk / 1e6 / peaks["hbm_gbs"],
            "pack_call_ms": tcall, "to_host_ms": t_d2h, "restore_ms": t_h2d,
            "host_copy_gbs": layout.nbytes / max(t_d2h, t_h2d) / 1e6}


if __name__ == "__main__":
    main()

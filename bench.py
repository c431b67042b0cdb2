#!/usr/bin/env python
"""Benchmark: fused draft-block verification on B200 (config 1 of the benchmark plan).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dspine|reference]

One step = one dsv_verify_logits launch over the whole ragged batch: temperature / top-k /
top-p / softmax of every verify row of the target and of the draft, the capped chain rejection,
the residual bonus draw and the accept-compact of tokens and KV slots.  Inputs are seeded
synthetic logits (dspine_b200.workloads), resident in HBM for ``value``; ``e2e`` times the public
call on inputs in pinned host memory (verify.verify_logits_host: only the logit rows an outcome
can depend on cross to the device, in widening windows of verify positions) with the outputs
read back every step.  The kernel drops rows after a known rejection, so the roofline is taken
on the bytes it read (its own counter) with the fraction on every row's bytes beside it.

Multi-GPU: verification has no exchange step (requests are independent), so each rank runs an
independent replica on its own requests (weak scaling); no collective touches the data path.
The only collectives are the barrier around the timed region and the max/sum of the results.

``--impl reference`` times the reference algorithm on the host cores instead: the CPU
restatement under oracle/ (the reference itself is Python/Triton and cannot run on the GPU box)
on the same config's whole batch, with every host thread.
"""

from __future__ import annotations

import argparse
import json
import re
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "verified draft tokens/s at B=64, block 16, V=151936"
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

WORKLOADS = {
    "config1": "ragged continuous batch: 64 requests, verify length U{1..16}, V=151936, bf16 "
               "logits N(0,2.5^2)+8 spike, draft = target + N(0,1); T U[0,1.5] (25% 0), "
               "top_k {off,1,20,50}, top_p U[0.8,1]; accept-compact of tokens + int32 KV slots",
    "config0": "4 requests x 16, V=151936, fp32 logits, 2 greedy + 2 T=1",
    "config4": "256 requests, SPS-capped verify lengths + early stop 0.3, V=151936, bf16",
    "config2": "fused draft LM head + top-8 + logsumexp, Qwen3-8B draft shapes: hidden bf16 "
               "[1024, 4096] ~ N(0,1), W bf16 [151936, 4096] ~ N(0, 0.02^2); logits never written",
    "config3": "vocab-parallel TP head, TP = --gpus: hidden bf16 [512, 5120] (32 requests x 16), "
               "W [151936, 5120] ~ N(0, 0.02^2) sharded contiguously; per rank fused top-20 + "
               "logsumexp, one all-gather, replicated merge and greedy accept on every rank",
    "fp8": "FP8 coarse retrieval + BF16 rescore + top-16 (layers/fp8/coarse.py), the optimized "
           "V=248320 / H=5120 head: hidden bf16 [960, 5120] (64 requests x 15) ~ N(0,1), "
           "W bf16 [248320, 5120] ~ N(0, 0.02^2) quantized to e4m3 once; per step quantize, "
           "FP8 GEMM, top-128, rescore, top-16",
}
HEAD_SHAPES = {"config2": (1024, 4096, 8, 64), "config3": (512, 5120, 20, 32)}  # rows, H, k, B
FP8_SHAPE = (960, 5120, 248320)  # rows, H, vocab
VOCAB = 151936
HEAD_METRIC = {"config2": "fused LM head + top-8 + logsumexp: hidden rows/s (1024 x 4096 x 151936)",
               "config3": "vocab-parallel TP head top-20 + logsumexp + accept: draft rows/s "
                          "(512 x 5120 x 151936)"}

# NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("dspine", "reference"), default="dspine")
    p.add_argument("--config", choices=tuple(WORKLOADS), default="config1")
    p.add_argument("--no-cpu-baseline", action="store_true",
                   help="skip the CPU baseline leg (it is reported by default at N=1)")
    p.add_argument("--kernel", default=None,
                   help="time one library kernel alone (the workloads of the ncu summaries)")
    p.add_argument("--no-tp-head", action="store_true",
                   help="at N > 1, skip the config-3 TP head timed beside the replicas")
    p.add_argument("--requests", type=int, default=None,
                   help="config1 with this many requests instead of 64 (small ncu cases; not a "
                        "benchmark line)")
    p.add_argument("--no-other-configs", action="store_true",
                   help="at N = 1, skip configs 0, 4, 2 and the FP8 head measured after config 1")
    return p.parse_args()


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def measured_hbm_peak():
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(config: str):
    """DRAM bytes per verification call from the committed ncu summary, or (None, []).

    The summary holds one `dram_bytes_per_launch_<kernel>: N` line per captured kernel; the
    call's traffic is their sum, reported with the kernels it covers."""
    f = ROOT / "profiles" / f"rows_kernel_{config}.md"
    if not f.exists():
        return None, []
    total, kernels = 0.0, []
    for line in f.read_text().splitlines():
        m = re.match(r"\s*dram_bytes_per_launch_(\w+):\s*([0-9.eE+]+)", line)
        if m:
            kernels.append("dsv::" + m.group(1))
            total += float(m.group(2))
    return (total if kernels else None), kernels


def make_batch(config: str, rank: int, device, requests=None):
    """The config's batch.  Every replica verifies the same seeded batch, so that the time of
    N replicas measures the machine (HBM, clocks, launch) rather than the cost spread between
    differently seeded batches.  `requests` (config 1 only) draws a smaller batch with the same
    distributions: the small case of an ncu capture."""
    from dspine_b200 import workloads
    fn = getattr(workloads, config)
    seed = {"config0": 0, "config1": 1, "config4": 4}[config]
    if requests:
        if config != "config1":
            raise SystemExit("--requests applies to config1 only")
        return fn(seed=seed, device=device, B=requests)
    return fn(seed=seed, device=device)


class ClockSampler:
    """Polls NVML for SM clock and clock-event reasons of one GPU while running."""

    def __init__(self, torch_device):
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            props = torch.cuda.get_device_properties(torch_device)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            try:
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(torch_device.index or 0)
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # no NVML: report no clocks rather than fail the bench
            log(f"clock sampling unavailable: {e}")
            self._nvml = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((mhz, int(bits)))
            except Exception:
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        bits = 0
        for _, b in self.samples:
            bits |= b
        reasons = sorted(name for bit, name in _REASONS.items() if bits & bit and bit != 0x1)
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


def cpu_port_time(batch, n_requests=None, nthreads=None):
    """Seconds of one oracle run (the CPU restatement) over the first n requests."""
    import oracle as O

    def np_f32(t):
        return t.detach().float().cpu().numpy()

    def np_i(t):
        return t.detach().cpu().numpy()
    n = batch.B if n_requests is None else min(n_requests, batch.B)
    tgt = np_f32(batch.target_logits)
    drf = None if batch.draft_logits is None else np_f32(batch.draft_logits)
    args = (np_i(batch.candidates)[:n], tgt, np_i(batch.target_rows)[:n], drf,
            None if batch.draft_rows is None else np_i(batch.draft_rows)[:n],
            np_f32(batch.temperature)[:n], np_i(batch.top_k)[:n], np_f32(batch.top_p)[:n],
            np_i(batch.verify_lens)[:n], np_f32(batch.uniforms)[:n],
            np_f32(batch.uniform_final)[:n], np_i(batch.prefix_lens)[:n])
    tokens = int(batch.verify_lens[:n].sum())

    def once():
        t0 = time.perf_counter()
        O.verify_logits(*args, nthreads=nthreads)
        return time.perf_counter() - t0
    return once, tokens


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return  # the CPU reference arm runs once, on rank 0
    import torch
    cores = host_cores()
    torch.set_num_threads(cores)
    batch = make_batch(args.config, 0, "cpu")
    n = batch.B  # the whole batch of this arm's config: every request, every row
    once, tokens = cpu_port_time(batch, n, nthreads=cores)
    for _ in range(args.warmup):
        once()
    times = [once() for _ in range(args.steps)]
    step_s = sum(times) / len(times)
    value = tokens / step_s
    sample = (f"all {n} requests of {args.config} ({tokens} verified tokens) per step, "
              f"oracle port with {cores} OpenMP threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32+i64", "data": "synthetic",
        "config": {"workload": f"{args.config}: {WORKLOADS[args.config]}",
                   "requests": n, "same_config": True, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_dspine(args):
    import torch
    rank, local_rank, world = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU fallback)")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)

    from dspine_b200 import _lib, verify

    lib = _lib.load()
    batch = make_batch(args.config, rank, dev, args.requests)
    kw = batch.kwargs()
    B = batch.B
    out = verify.new_outputs(B, dev)
    comp = verify.CompactOutputs.allocate(B, dev)
    ws = verify.workspace_for(B, dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def step():
        verify.verify_logits(**kw, outputs=out, slots=batch.slots, slot_rows=batch.slot_rows,
                             compact=comp, workspace=ws)

    # the timed steps call the same C entry point with arguments validated once (the Python
    # checks would otherwise sit between the start event and the launch)
    _, _, _, cargs, _keep = verify._prepare(
        kw["candidates"], kw["target_logits"], kw["target_rows"], kw["temperature"], kw["top_k"],
        kw["top_p"], kw["verify_lens"], kw["uniforms"], kw["uniform_final"], kw["prefix_lens"],
        kw.get("draft_logits"), kw.get("draft_rows"), out, batch.slots, batch.slot_rows, comp)
    c_stream = torch.cuda.current_stream(dev).cuda_stream

    def step_timed():
        _lib.call("dsv_verify_logits", *cargs, ws.buf.data_ptr(), ws.nbytes, c_stream)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        step()
    torch.cuda.synchronize(dev)
    if ws.error_word() != 0:
        raise SystemExit("device error word set during warm-up")

    # ---- device-timed steps (inputs resident in HBM, L2 flushed before each step) ----
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches0 = lib.dsv_launch_count()
    read0 = ws.bytes_read()
    sampler = ClockSampler(dev)
    barrier()
    with sampler:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step_timed()
            ends[i].record()
        barrier()
    launches = lib.dsv_launch_count() - launches0
    bytes_read = (ws.bytes_read() - read0) / args.steps  # per launch (bf16 streaming path)
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    tokens = batch.verified_tokens()
    if dist is not None:
        t = torch.tensor([total_ms, float(tokens), float(launches)], dtype=torch.float64, device=dev)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_ms, all_tokens, all_launches = float(tmax[0]), float(t[1]), int(t[2])
    else:
        all_tokens, all_launches = float(tokens), launches
    ms_per_step = total_ms / args.steps
    value = all_tokens / (ms_per_step * 1e-3)

    # ---- end to end: the public call on pinned host inputs (verify.verify_logits_host: it
    # copies to the device the logit rows the outcome can depend on, in widening windows of
    # verify positions, verifies, compacts and reads the outputs back), every step ----
    inputs = {**kw, "slots": batch.slots, "slot_rows": batch.slot_rows}
    host_in = {k: v.cpu().pin_memory() for k, v in inputs.items() if v is not None}
    e2e_steps = max(3, min(args.steps, 20))
    h2d_total = d2h_total = 0
    windows = ()

    def e2e_step():
        nonlocal h2d_total, d2h_total, windows
        host_out, _, info = verify.verify_logits_host(**host_in, device=dev)
        h2d_total += info.h2d_bytes
        d2h_total += info.d2h_bytes
        windows = info.windows
        return host_out

    check = e2e_step()
    for got, want in zip(check, out):
        if not torch.equal(got, want.cpu()):
            raise SystemExit("host-input verification differs from the device-input call")
    h2d_total = d2h_total = 0
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    h2d = h2d_total / e2e_steps
    d2h = d2h_total / e2e_steps
    if dist is not None:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    e2e_value = all_tokens / (e2e_ms * 1e-3)
    if ws.error_word() != 0:
        raise SystemExit("device error word set during the timed region")

    tp_head = None
    if dist is not None and args.config == "config1" and not args.no_tp_head:
        tp_head = tp_head_report(dev, dist, rank, world, args.steps, args.warmup)

    line = None
    if rank == 0:
        alg_bytes = batch.algorithmic_bytes()
        # verification drops rows that cannot change an outcome: the roofline is taken on the
        # bytes it read (counted by the kernels)
        read_bytes = bytes_read if bytes_read > 0 else float(alg_bytes)
        deciding = batch.deciding_bytes(out[0])
        kernel_ms = statistics.mean(step_ms)
        achieved = read_bytes / (kernel_ms * 1e-3) / 1e9
        peak, peak_src = measured_hbm_peak()
        traffic, traffic_kernels = profiled_traffic(args.config)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32+i64", "data": "synthetic",
            "config": {"workload": f"{args.config}: {WORKLOADS[args.config]}",
                       "requests_per_gpu": B, "vocab": batch.V,
                       "verified_tokens_per_gpu": tokens,
                       "logits_dtype": str(batch.target_logits.dtype).replace("torch.", ""),
                       "parallelism": f"dp{world} (independent replicas)",
                       "l2": "flushed before every timed step (256 MiB memset, untimed)"},
            "clocks": sampler.summary(),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "call": "verify.verify_logits_host (pinned host inputs; logit rows copied in "
                            "widening windows of verify positions, outputs read back)",
                    "windows": list(windows),
                    "all_input_bytes": sum(v.numel() * v.element_size() for v in host_in.values())},
            "gpu_launches": all_launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "traffic_kernels": traffic_kernels, "peak_source": peak_src,
                         "kernel": "dsv::rows_kernel (the whole dsv_verify_logits call: rows and chain tasks)",
                         "bytes_read_per_launch": read_bytes,
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "frac_on_algorithmic_bytes": alg_bytes / (kernel_ms * 1e-3) / 1e9 / peak,
                         "deciding_bytes_per_launch": deciding,
                         "bytes_basis": "rows read (rows that cannot change an outcome are "
                                        "dropped; all rows of the batch: algorithmic_bytes, "
                                        "rows the outcome depends on: deciding_bytes)",
                         "kernel_ms": kernel_ms},
        }
        if tp_head is not None:
            line["tp_head"] = tp_head
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(batch)
        return line
    return None


def cpu_baseline(batch):
    """Oracle port over the whole workload on every host core, repeated for ~10 s."""
    cores = host_cores()
    once, tokens = cpu_port_time(batch, None, nthreads=cores)
    t, reps = 0.0, 0
    while reps < 1 or (t < 10.0 and reps < 10):
        t += once()
        reps += 1
    return {"value": tokens * reps / t, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"whole workload ({tokens} verified tokens) x {reps} runs, "
                      f"oracle port with {cores} OpenMP threads"}


def measured_tensor_peak():
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["bf16_tflops"]), "measured (burst)"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def head_inputs(config, rank, world, device):
    """Seeded synthetic hidden states and this rank's contiguous weight shard.  Every rank
    draws the same full weight on its GPU (one seeded generator) and keeps its rows, so the
    shards of all ranks partition one weight."""
    import torch
    rows, H, k, _ = HEAD_SHAPES[config]
    g = torch.Generator(device=device).manual_seed(2 if config == "config2" else 3)
    hidden = torch.randn(rows, H, generator=g, device=device).to(torch.bfloat16)
    start, end = VOCAB * rank // world, VOCAB * (rank + 1) // world
    full = (torch.randn(VOCAB, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    shard = full[start:end].contiguous()
    del full
    torch.cuda.empty_cache()
    return hidden, shard, start, end


def head_cpu_time(config, n_rows, cores):
    """torch CPU reference: matmul + topk + logsumexp over a row subset (the whole vocab)."""
    import torch
    torch.set_num_threads(cores)
    rows, H, k, _ = HEAD_SHAPES[config]
    g = torch.Generator(device="cpu").manual_seed(5)
    x = torch.randn(n_rows, H, generator=g).to(torch.bfloat16)
    w = (torch.randn(VOCAB, H, generator=g) * 0.02).to(torch.bfloat16)

    def once():
        t0 = time.perf_counter()
        logits = torch.matmul(x, w.T)
        torch.topk(logits.float(), k, dim=1)
        torch.logsumexp(logits.float(), dim=1)
        return time.perf_counter() - t0
    return once


def tp_head_report(dev, dist, rank, world, steps, warmup):
    """Config 3's vocab-parallel head at TP = world, timed in the same run as the verification
    replicas: per step the shard's fused head (top-20 + logsumexp), ONE all-gather of the packed
    candidate block, the replicated merge and the greedy accept, captured in a CUDA graph and
    replayed back to back (max over ranks).  Beside it: the unsharded head on one GPU (TP = 1),
    the all-gather of the same block alone, and whether every rank's merged ids and accept
    outputs equal each other's and the TP = 1 result."""
    import torch
    from dspine_b200 import accept, lmhead
    rows, H, k, B = HEAD_SHAPES["config3"]
    hidden, shard, start, end = head_inputs("config3", rank, world, dev)
    _, full, _, _ = head_inputs("config3", 0, 1, dev)
    group = lmhead.TorchGroup()
    head = lmhead.TPHead(shard, start, end, VOCAB, group)
    g = torch.Generator(device="cpu").manual_seed(9)
    cand = torch.randint(0, VOCAB, (B, 16), generator=g).to(dev)
    caps = torch.randint(1, 17, (B,), generator=g, dtype=torch.int32).to(dev)
    outs = accept.new_outputs(B, dev)
    outs1 = accept.new_outputs(B, dev)
    full_out = (torch.empty(rows, k, dtype=torch.int64, device=dev),
                torch.empty(rows, k, dtype=torch.float32, device=dev),
                torch.empty(rows, dtype=torch.float32, device=dev))
    res = {}

    def step_tp():
        ids, _, _ = head.topk_lse(hidden, k)
        accept.accept_greedy(cand, ids[:, 0].view(B, 16), caps, outputs=outs)
        res["ids"] = ids

    def step_one():
        lmhead.lmhead_topk(hidden, full, k, out=full_out)
        accept.accept_greedy(cand, full_out[0][:, 0].view(B, 16), caps, outputs=outs1)

    words = rows * k * 3 + rows
    words += words & 1
    block = torch.zeros(words, dtype=torch.int32, device=dev)
    gathered = torch.empty(world * words, dtype=torch.int32, device=dev)

    def step_ag():
        dist.all_gather_into_tensor(gathered, block)

    def barrier():
        dist.barrier(device_ids=[dev.index])
        torch.cuda.synchronize(dev)

    def timed(fn, graph_it):
        for _ in range(max(warmup, 3)):
            fn()
        barrier()
        run = fn
        graph = None
        if graph_it:
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream(dev).wait_stream(side)
            barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fn()
            barrier()
            run = graph.replay
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            run()
        e1.record()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del graph
        return float(t[0])

    tp_ms = timed(step_tp, True)
    ag_ms = timed(step_ag, True)
    one_ms = timed(step_one, False)
    step_tp()
    step_one()
    torch.cuda.synchronize(dev)
    same_as_tp1 = torch.equal(res["ids"], full_out[0]) and all(
        torch.equal(a, b) for a, b in zip(outs, outs1))
    digest = torch.cat([res["ids"].view(-1), *(o.view(-1).to(torch.int64) for o in outs)])
    everyone = torch.empty((world, digest.numel()), dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(everyone.view(-1), digest)
    across = bool((everyone == everyone[0:1]).all())
    flags = torch.tensor([0.0 if same_as_tp1 else 1.0], dtype=torch.float64, device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    return {"tp": world, "workload": "config3: 512 draft rows x H 5120 x V 151936, top-20 + "
                                     "logsumexp + greedy accept of 32 requests",
            "ms_per_step": tp_ms, "tp1_ms_per_step": one_ms, "speedup_vs_tp1": one_ms / tp_ms,
            "allgather_us": ag_ms * 1e3, "allgather_share": ag_ms / tp_ms,
            "allgather_bytes_per_rank": words * 4,
            "identical_across_ranks": across, "identical_to_tp1": bool(flags[0] == 0.0),
            "rows_per_s": rows / (tp_ms * 1e-3)}


def run_head(args):
    """Configs 2 and 3: the fused LM head (and, for config 3, the vocab-parallel TP head)."""
    import torch
    from dspine_b200 import lmhead, _lib, accept
    rank, local_rank, world = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU fallback)")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    rows, H, k, B = HEAD_SHAPES[args.config]
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    tp = world if args.config == "config3" else 1
    lib = _lib.load()
    hidden, shard, start, end = head_inputs(args.config, rank if tp > 1 else 0, tp, dev)
    group = lmhead.TorchGroup() if tp > 1 else None
    g = torch.Generator(device="cpu").manual_seed(9)
    cand = torch.randint(0, VOCAB, (B, 16), generator=g).to(dev)
    caps = torch.randint(1, 17, (B,), generator=g, dtype=torch.int32).to(dev)
    outs = accept.new_outputs(B, dev)

    if tp > 1:
        head = lmhead.TPHead(shard, start, end, VOCAB, group)

        def step():
            ids, vals, lse = head.topk_lse(hidden, k)
            accept.accept_greedy(cand, ids[:, 0].view(B, 16), caps, outputs=outs)
            return ids
    else:
        out = (torch.empty(rows, k, dtype=torch.int64, device=dev),
               torch.empty(rows, k, dtype=torch.float32, device=dev),
               torch.empty(rows, dtype=torch.float32, device=dev))

        def step():
            lmhead.lmhead_topk(hidden, shard, k, out=out)
            if args.config == "config3":
                accept.accept_greedy(cand, out[0][:, 0].view(B, 16), caps, outputs=outs)
            return out[0]

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    # config 3: the step (shard head, all-gather, merge, accept) is a handful of short
    # launches; it is captured once in a CUDA graph and replayed, so host launch overhead
    # does not pace the GPU (every rank captures the same collective sequence)
    graph = None
    run = step
    per_step = None
    if args.config == "config3":
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        barrier()
        graph = torch.cuda.CUDAGraph()
        c0 = lib.dsv_launch_count()
        with torch.cuda.graph(graph):
            graph_res = step()
        per_step = lib.dsv_launch_count() - c0
        barrier()

        def run():
            graph.replay()
            return graph_res
    # the K steps run back to back between one pair of events (the weight shard is larger
    # than L2 at every TP size, so consecutive steps cannot reuse it from L2)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    launches0 = lib.dsv_launch_count()
    sampler = ClockSampler(dev)
    with sampler:
        t_start.record()
        for i in range(args.steps):
            run()
        t_end.record()
        barrier()
    launches = lib.dsv_launch_count() - launches0
    if per_step is not None:
        launches = per_step * args.steps  # replays enqueue the captured kernels
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [total_ms / args.steps]
    if dist is not None:
        t = torch.tensor([total_ms, float(launches)], dtype=torch.float64, device=dev)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        total_ms, all_launches = float(tmax[0]), int(t[1])
    else:
        all_launches = launches
    ms_per_step = total_ms / args.steps
    value = rows / (ms_per_step * 1e-3)

    # end to end: hidden states from pinned host memory, top-k/lse (and accept) read back
    host_x = hidden.cpu().pin_memory()
    res = run()
    host_ids = torch.empty(res.shape, dtype=res.dtype).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        hidden.copy_(host_x, non_blocking=True)
        r = run()
        host_ids.copy_(r, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if dist is not None:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t[0])
    err = lmhead.workspace_for(rows, end - start, k, dev).error_word()
    if err:
        raise SystemExit(f"device error word {err:#x}")

    line = None
    if rank == 0:
        flops = 2.0 * rows * (end - start) * H          # this rank's share
        kernel_ms = statistics.mean(step_ms)
        achieved = flops / (kernel_ms * 1e-3) / 1e12
        peak, src = measured_tensor_peak()
        line = {
            "metric": HEAD_METRIC[args.config], "value": value, "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong" if tp > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": f"{args.config}: {WORKLOADS[args.config]}",
                       "rows": rows, "hidden": H, "vocab": VOCAB, "k": k, "tp": tp,
                       "cuda_graph": graph is not None or per_step is not None,
                       "parallelism": f"tp{tp}" if tp > 1 else "dp1",
                       "l2": "inputs larger than L2 (weight shard streamed every step)"},
            "clocks": sampler.summary(),
            "e2e": {"value": rows / (e2e_ms * 1e-3), "unit": "rows/s",
                    "h2d_bytes_per_step": host_x.numel() * 2,
                    "d2h_bytes_per_step": host_ids.numel() * host_ids.element_size()},
            "gpu_launches": all_launches,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "peak_source": src, "kernel": "dsv::lm::lmhead_kernel (+ merge)",
                         "flops_per_launch": flops, "kernel_ms": kernel_ms},
        }
    del graph  # graphs holding NCCL calls go before the process group
    if dist is not None:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            cores = host_cores()
            n_rows = 16
            once = head_cpu_time(args.config, n_rows, cores)
            once()
            t = min(once() for _ in range(2))
            line["cpu_baseline"] = {"value": n_rows / t, "unit": "rows/s", "cores": cores,
                                    "kind": "port",
                                    "sample": f"{n_rows} rows x full vocab: torch CPU matmul + "
                                              f"topk + logsumexp, {cores} threads"}
        return line
    return None


def fp8_cpu_time(n_rows, cores, vocab=None):
    """torch CPU port of retrieve_and_rescore (layers/fp8/coarse.py:41-113, gather.py) on
    n_rows hidden rows over the whole vocabulary: e4m3 quantization with per-row scales, the
    coarse product in fp32 over dequantized codes (vocabulary chunks), stable top-128, the
    BF16 rescore and the 16 selection rounds.  Returns once() -> seconds of one step."""
    import torch
    torch.set_num_threads(cores)
    _, H, V = FP8_SHAPE
    V = vocab or V
    chunk = 16384
    g = torch.Generator().manual_seed(17)

    def quantize(t):
        amax = t.float().abs().amax(dim=1, keepdim=True)
        sc = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
        return (t.float() / sc).clamp(-448.0, 448.0).to(torch.float8_e4m3fn), sc[:, 0]

    w = torch.empty(V, H, dtype=torch.bfloat16)
    w8 = torch.empty(V, H, dtype=torch.float8_e4m3fn)
    sw = torch.empty(V)
    for s0 in range(0, V, chunk):
        blk = (torch.randn(min(chunk, V - s0), H, generator=g) * 0.02).bfloat16()
        w[s0:s0 + blk.shape[0]] = blk
        w8[s0:s0 + blk.shape[0]], sw[s0:s0 + blk.shape[0]] = quantize(blk)
    x = torch.randn(n_rows, H, generator=g).bfloat16()

    def once():
        t0 = time.perf_counter()
        xq, sx = quantize(x)
        xf = xq.float()
        coarse = torch.empty(n_rows, V, dtype=torch.bfloat16)
        for s0 in range(0, V, chunk):
            s1 = min(V, s0 + chunk)
            coarse[:, s0:s1] = ((xf @ w8[s0:s1].float().T) * sx[:, None] * sw[None, s0:s1]).bfloat16()
        ids = torch.argsort(coarse.float(), dim=1, descending=True, stable=True)[:, :128]
        scores = (w[ids].float() * x.float()[:, None]).sum(-1).bfloat16()
        # 16 best by (stored score desc, token asc), ascending tokens
        by_id = torch.argsort(ids, dim=1)
        sv, si = scores.gather(1, by_id), ids.gather(1, by_id)
        best = torch.argsort(sv.float(), dim=1, descending=True, stable=True)[:, :16]
        si.gather(1, best).sort(dim=1)
        return time.perf_counter() - t0
    return once


def run_fp8(args):
    """FP8 coarse retrieval (one GPU; under torchrun every rank runs an independent replica)."""
    import torch
    from dspine_b200 import _lib
    from dspine_b200.layers.fp8 import coarse as C
    rank, local_rank, world = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU fallback)")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    rows, H, V = FP8_SHAPE
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(7)
    hidden = torch.randn(rows, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    local = C.FullVFP8Coarse(torch, w)
    wq, sw = local.weight8.view(torch.uint8), local.weight_scale.reshape(-1)

    def step():
        return local.retrieve_and_rescore(hidden)[0]

    def timed(fn, n):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / n

    # K steps back to back (the 1.27 GB e4m3 head is larger than L2: it streams every step)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    launches0 = lib.dsv_launch_count()
    sampler = ClockSampler(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.synchronize(dev)
    launches = lib.dsv_launch_count() - launches0
    ms_per_step = t0.elapsed_time(t1) / args.steps
    # the dominant kernel alone, and the reference's library call for the same GEMM
    xq, sx = C.quantize_rows(hidden)
    gemm_ms = timed(lambda: C.coarse_scores(xq, sx, wq, sw), args.steps)
    flops = 2.0 * rows * V * H
    ref_ms = None
    try:
        sxt, swt = sx.reshape(-1, 1).contiguous(), local.weight_scale
        ref_ms = timed(lambda: torch.ops.aten._scaled_mm.default(
            xq.view(torch.float8_e4m3fn), local.weight8_t, sxt, swt, bias=None, scale_result=None,
            out_dtype=torch.bfloat16, use_fast_accum=False), args.steps)
    except Exception as exc:  # the library call is a yardstick only
        log(f"torch._scaled_mm unavailable: {exc!r}")
    # end to end: hidden rows from pinned host memory, the 16 tokens of every row read back
    host_x = hidden.cpu().pin_memory()
    host_ids = torch.empty(rows, 16, dtype=torch.int64).pin_memory()

    def e2e_step():
        hidden.copy_(host_x, non_blocking=True)
        host_ids.copy_(step(), non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e2e_ms = timed(e2e_step, max(3, min(args.steps, 20)))
    if local.error_word():
        raise SystemExit(f"device error word {local.error_word():#x}")
    if rank != 0:
        return
    achieved = flops / (gemm_ms * 1e-3) / 1e12
    peak = flops / (ref_ms * 1e-3) / 1e12 if ref_ms else None
    traffic = None   # DRAM bytes of one full launch, scaled from a smaller ncu capture
    prof = ROOT / "profiles" / "fp8_retrieval_v248320_h5120.md"
    if prof.exists():
        m = re.search(r"full_launch_dram_bytes_coarse8_kernel:\s*([0-9]+)", prof.read_text())
        traffic = float(m.group(1)) if m else None
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cores = host_cores()
        n_cpu = 2
        once = fp8_cpu_time(n_cpu, cores)
        once()
        t = min(once() for _ in range(2))
        cpu = {"value": n_cpu / t, "unit": "rows/s", "cores": cores, "kind": "port",
               "sample": f"{n_cpu} rows x full vocabulary: torch CPU port (e4m3 quantization, "
                         f"fp32 coarse product, stable top-128, bf16 rescore, top-16), {cores} threads"}
    line = {
        "metric": "FP8 coarse retrieval + rescore + top-16: hidden rows/s (960 x 5120 x 248320)",
        "value": rows / (ms_per_step * 1e-3), "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e4m3 GEMM (fp32 accumulate) + bf16 rescore", "data": "synthetic",
        "config": {"workload": f"fp8: {WORKLOADS['fp8']}", "rows": rows, "hidden": H, "vocab": V,
                   "candidates": 128, "parallelism": "dp1 (replicas)",
                   "l2": "inputs larger than L2 (e4m3 head streamed every step)"},
        "clocks": sampler.summary(),
        "e2e": {"value": rows / (e2e_ms * 1e-3), "unit": "rows/s",
                "h2d_bytes_per_step": host_x.numel() * 2, "d2h_bytes_per_step": host_ids.numel() * 8},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if peak else None, "traffic": traffic,
                     "traffic_source": "ncu capture at V=32768 scaled by vocabulary rows",
                     "peak_source": "torch._scaled_mm (cuBLASLt FP8, same shapes) timed in this run",
                     "kernel": "dsv::lm::coarse8_kernel", "flops_per_launch": flops,
                     "kernel_ms": gemm_ms},
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def run_fp8_reference(args):
    """The CPU port of retrieve_and_rescore on every host core (rank 0 only)."""
    rank, _, _ = dist_env()
    if rank != 0:
        return
    cores = host_cores()
    n_rows = 2
    once = fp8_cpu_time(n_rows, cores)
    for _ in range(min(args.warmup, 1)):
        once()
    times = [once() for _ in range(min(args.steps, 3))]
    step_s = sum(times) / len(times)
    value = n_rows / step_s
    print(json.dumps({
        "impl": "reference",
        "metric": "FP8 coarse retrieval + rescore + top-16: hidden rows/s (960 x 5120 x 248320)",
        "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": len(times),
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 codes, fp32 product, bf16 rescore",
        "data": "synthetic",
        "config": {"workload": f"fp8: {WORKLOADS['fp8']}", "sample_rows": n_rows,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": f"{n_rows} rows x full vocabulary per step: torch CPU port"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_head_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    cores = host_cores()
    n_rows = 16
    once = head_cpu_time(args.config, n_rows, cores)
    for _ in range(min(args.warmup, 1)):
        once()
    times = [once() for _ in range(min(args.steps, 3))]
    step_s = sum(times) / len(times)
    value = n_rows / step_s
    print(json.dumps({
        "impl": "reference", "metric": HEAD_METRIC[args.config], "value": value, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{args.config}: {WORKLOADS[args.config]}", "sample_rows": n_rows,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": f"{n_rows} rows x full vocab per step: torch CPU matmul + "
                                   f"topk + logsumexp"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---- single kernels (--kernel NAME): the workloads the committed ncu summaries capture ------

def kernel_workload(name, dev):
    """(launch, algorithmic bytes per launch or None, description) of one library kernel on a
    seeded workload of the benchmark's sizes (V = 151936)."""
    import torch
    from dspine_b200 import lmhead, logits, verify
    from dspine_b200.kernels import dspine as kd
    from dspine_b200.layers.fp8 import gather
    from dspine_b200.sampling import rejection
    from dspine_b200.sampling.sparse import accept as sparse
    from dspine_b200.sampling.sparse.target import build_sparse_target
    V = VOCAB
    g = torch.Generator(device=dev).manual_seed(11)
    B = 64

    def softmax_rows(n):
        return torch.softmax(torch.randn(n, V, generator=g, device=dev) * 2.5, -1)

    def chain_inputs():
        cand = torch.randint(0, V, (B, 16), generator=g, device=dev)
        lens = torch.randint(1, 17, (B,), generator=g, device=dev, dtype=torch.int32)
        u = torch.rand(B, 15, generator=g, device=dev)
        uf = torch.rand(B, generator=g, device=dev)
        prefix = torch.zeros(B, dtype=torch.int32, device=dev)
        return cand, lens, u, uf, prefix

    if name == "chain_probs":
        p = softmax_rows(B * 16).view(B, 16, V)
        q = softmax_rows(B * 15).view(B, 15, V)
        cand, lens, u, uf, prefix = chain_inputs()
        out = verify.new_outputs(B, dev)

        def launch():
            rejection.sample_capped_chain_from_probs(
                candidates=cand, target_probs=p, draft_probs=q, verify_lens=lens, uniforms=u,
                uniform_final=uf, prefix_lens=prefix, outputs=out)
        return launch, B * 2 * V * 4, "dsv_chain_from_probs: 64 requests, bonus p and q rows fp32"
    if name == "sparse_accept":
        p = softmax_rows(B * 16)
        cand, lens, u, uf, prefix = chain_inputs()
        qid = torch.randint(0, V, (B, 15, 16), generator=g, device=dev)
        qv = torch.softmax(torch.randn(B, 15, 16, generator=g, device=dev), -1)
        out = verify.new_outputs(B, dev)

        def launch():
            sparse.accept_sparse(torch, candidates=cand, dense_p=p, packed=None, q_ids=qid,
                                 q_values=qv, verify_lens=lens, uniforms=u, uniform_final=uf,
                                 prefix_lens=prefix, outputs=out)
        return launch, B * V * 4, "dsv_accept_sparse: 64 requests, dense p rows fp32, sparse q"
    if name == "compress":
        p = softmax_rows(1024)
        p = p * (p > 2e-6)

        def launch():
            sparse.compress_probs(torch, p, capacity=32)
        return launch, 1024 * V * 4, "dsv_compress_probs: 1024 rows fp32"
    if name in ("target_probs", "sparse_target"):
        x = (torch.randn(B * 16, V, generator=g, device=dev) * 2.5).to(torch.bfloat16)
        T = torch.rand(B, generator=g, device=dev) + 0.5
        k = torch.full((B,), 20, dtype=torch.int32, device=dev)
        tp = torch.full((B,), 0.9, device=dev)
        if name == "target_probs":
            out = torch.empty(B * 16, V, device=dev)

            def launch():
                logits.target_probs(x, T, k, tp, rows_per_request=16, out=out)
            return launch, B * 16 * V * (2 + 4), "dsv_target_probs: 1024 bf16 rows -> fp32 p"
        from types import SimpleNamespace
        info = SimpleNamespace(temperatures=T, top_ks=k, top_ps=tp, max_top_k=20,
                               need_min_p_sampling=False, is_any_greedy=False)

        def launch():
            build_sparse_target(x, info, block_size=16, capacity=32)
        # each logit read once (k 20 < capacity 32: no row overflows, so no dense row is written)
        return launch, B * 16 * V * 2, "dsv_sparse_target: 1024 bf16 rows, k 20, top-p 0.9"
    if name == "serial_sample":
        K, T = 16, 16
        n = B * (T - 1)
        table = torch.randn(n, K, K, generator=g, device=dev)
        inv_t, top_p, min_p = (torch.full((B,), v, device=dev) for v in (1.0, 0.9, 0.0))
        top_k, greedy = (torch.full((B,), v, dtype=torch.int32, device=dev) for v in (8, 0))
        u = torch.rand(n, generator=g, device=dev)
        cand = torch.randint(0, V, (n, K), generator=g, device=dev)
        gt = torch.randint(0, V, (n,), generator=g, device=dev)
        ot = torch.empty(n, dtype=torch.int64, device=dev)
        oq = torch.empty(n, K, device=dev)

        def launch():
            kd.serial_sample_chain(table, inv_t, top_k, top_p, min_p, greedy, u, cand, gt, ot,
                                   oq, T)
        return launch, None, "dsv_serial_sample_chain: 64 requests x 15 rows, K 16"
    if name == "serial_table":
        K, T, H, R = 16, 16, 4096, 512
        m, n = B * T, B * (T - 1)
        raw = torch.randn(m, H, generator=g, device=dev).to(torch.bfloat16)
        norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
        cand = torch.randint(0, V, (n, K), generator=g, device=dev)
        ids = torch.randint(0, V, (m,), generator=g, device=dev)
        lm = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        tg = (torch.randn(V, R, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        tsv = (torch.randn(V, 2 * R, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        packed = torch.randn(m, R, generator=g, device=dev).to(torch.bfloat16)
        rms = torch.rand(m, generator=g, device=dev)
        gate_b = torch.zeros(R, device=dev, dtype=torch.bfloat16)

        def launch():
            kd.serial_table(raw, norm_w, cand, ids, lm, tg, tsv, packed, rms, gate_b, T)
        return launch, n * K * (H + 3 * R) * 2, "dsv_serial_table: 960 drafted rows, K 16, H 4096, R 512"
    if name == "rescore16":
        rows, C, H = 960, 128, 5120
        w = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        ids = torch.randint(0, V, (rows, C), generator=g, device=dev)
        hid = torch.randn(rows, H, generator=g, device=dev).to(torch.bfloat16)

        def launch():
            gather.rescore_select16(torch, w, ids, hid)
        return launch, rows * C * H * 2, "dsv_rescore_select16: 960 rows x 128 candidates, H 5120"
    if name == "merge":
        rows, S, k = 512, 8, 20
        vals = torch.randn(S, rows, k, generator=g, device=dev).sort(-1, descending=True).values
        ids = torch.randint(0, V, (S, rows, k), generator=g, device=dev)
        lse = torch.randn(S, rows, generator=g, device=dev)

        def launch():
            lmhead.merge_shards(vals, ids, lse, k, pad_id=V)
        return launch, None, "dsv_tp_merge: 512 rows, 8 shards x 20"
    if name == "topk_ids":
        x = (torch.randn(794, V, generator=g, device=dev) * 2.5).to(torch.bfloat16)
        out = torch.empty(794, 16, dtype=torch.int64, device=dev)

        def launch():
            kd.topk_ids(x, 16, out=out)
        return launch, 794 * V * 2, "dsv_topk_ids: 794 bf16 rows, k 16"
    if name == "adjust":
        from types import SimpleNamespace
        from dspine_b200.sampling.compact import adjust_logits
        x = (torch.randn(B, 16, V, generator=g, device=dev) * 2.5).to(torch.bfloat16)
        words = (V + 31) // 32
        info = SimpleNamespace(
            acc_additive_penalties=torch.randn(B, V, generator=g, device=dev),
            acc_scaling_penalties=1 + torch.rand(B, V, generator=g, device=dev),
            grammar_mask=SimpleNamespace(vocab_mask=torch.randint(
                -2**31, 2**31 - 1, (B, words), generator=g, device=dev, dtype=torch.int64).to(torch.int32)),
            logit_bias=torch.randn(B, V, generator=g, device=dev))

        def launch():
            adjust_logits(x, info, None)
        # per element of the rows: the logit read and written; penalties and bias rows per request
        return launch, B * 16 * V * 4 + B * V * 12, "dsv_adjust_logits: 64 x 16 bf16 rows, every adjustment"
    if name in ("coarse8", "fp8_step"):
        from dspine_b200.layers.fp8 import coarse as C
        rows, H, Vf = FP8_SHAPE
        if name == "coarse8":
            Vf = 32768  # the capture size: a 32768-row slice of the head (168 MB e4m3 > L2)
        hidden = torch.randn(rows, H, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn(Vf, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        head = C.FullVFP8Coarse(torch, w)
        del w
        if name == "fp8_step":
            def launch():
                head.retrieve_and_rescore(hidden)
            return launch, None, "FullVFP8Coarse.retrieve_and_rescore: 960 x 5120 hidden, V 248320"
        xq, xs = C.quantize_rows(hidden)
        wq, ws = head.weight8.view(torch.uint8), head.weight_scale.reshape(-1)

        def launch():
            C.coarse_scores(xq, xs, wq, ws)
        # a tensor-core GEMM (2 x 960 x 32768 x 5120 = 322 GFLOP): no HBM roofline line
        return launch, None, "dsv_fp8_coarse_scores: 960 x 5120 x 32768 e4m3"
    raise SystemExit(f"unknown kernel {name}")


KERNELS = ("chain_probs", "sparse_accept", "compress", "target_probs", "sparse_target",
           "serial_sample", "serial_table", "rescore16", "merge", "topk_ids", "adjust",
           "coarse8", "fp8_step")


def run_kernel(args):
    """One library kernel timed alone: K launches between CUDA events on the launching stream,
    L2 flushed before each (memory-bound kernels report GB/s against the measured HBM copy)."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    launch, nbytes, what = kernel_workload(args.kernel, dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        flush.zero_()
        launch()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        launch()
        e1.record()
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1))
    ms = statistics.mean(times)
    line = {"kernel": args.kernel, "workload": what, "ms_per_launch": ms,
            "ms_median": statistics.median(times), "steps": args.steps}
    if nbytes is not None:
        peak, src = measured_hbm_peak()
        gbs = nbytes / (ms * 1e-3) / 1e9
        line.update({"algorithmic_bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": peak,
                     "frac": gbs / peak, "peak_source": src})
    print(json.dumps(line), flush=True)


def other_configs(args):
    """The plan's other configurations measured in the same run (one GPU): configs 0 and 4 of
    the verification, the fused LM head (config 2) and the FP8 head, each with its own metric
    (20 timed steps, 3 warm-up steps, no CPU leg)."""
    import copy
    out = {}
    for name in ("config0", "config4", "config2", "fp8"):
        a = copy.copy(args)
        a.config, a.steps, a.warmup = name, 20, 3
        a.no_cpu_baseline = a.no_tp_head = True
        try:
            if name == "fp8":
                line = run_fp8(a)
            elif name in HEAD_SHAPES:
                line = run_head(a)
            else:
                line = run_dspine(a)
        except Exception as e:  # one failed extra must not lose the headline line
            out[name] = {"error": repr(e)[:200]}
            continue
        roof = line.get("roofline") or {}
        metric = line["metric"] if name in HEAD_SHAPES or name == "fp8" else \
            f"verified draft tokens/s, {name} ({line['config']['requests_per_gpu']} requests, V={VOCAB})"
        out[name] = {"metric": metric, "value": line["value"], "unit": line["unit"],
                     "ms_per_step": line["ms_per_step"], "e2e": line["e2e"]["value"],
                     "roofline": {k: roof.get(k) for k in ("bound", "achieved", "peak", "unit",
                                                           "frac")},
                     "clocks": line.get("clocks"), "workload": line["config"]["workload"]}
    return out


def main():
    args = parse_args()
    if args.kernel:
        run_kernel(args)
        return
    line = None
    if args.config == "fp8":
        run_fp8_reference(args) if args.impl == "reference" else (line := run_fp8(args))
    elif args.config in HEAD_SHAPES:
        run_head_reference(args) if args.impl == "reference" else (line := run_head(args))
    elif args.impl == "reference":
        run_reference(args)
    else:
        line = run_dspine(args)
        if (line is not None and args.config == "config1" and dist_env()[2] == 1
                and not args.no_other_configs):
            line["other_configs"] = other_configs(args)
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

"""Decode-step throughput of the CKL decoder on B200: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload cfg5|cfg1|cfg3|cfg4|vector] [--requests-per-gpu R]

Default workload: BASELINE config 5 (scale-out decoder: 4 layers, hidden 1024, 16 heads x 64,
SwiGLU 4096, vocab 32000, 2048-token prompts in the KV cache, greedy decode).  Requests are
sharded across GPUs with no collective in the step; each GPU holds 512 requests, so 8 GPUs
run the full 4096-request configuration (weak scaling; the full configuration's 279 GB KV
cache does not fit one GPU).  Weights are seeded random (reference draw order, seed 4),
prompts uniform over the vocabulary; the prompts are prefilled on the GPU (batched prefill).
Every timed step is one complete decode step (all layers, LM head, greedy argmax, KV append)
for every request on the GPU.

Timing: W warm-up steps, then K graph launches bracketed by a barrier and a synchronize on
both sides, CUDA events on the invocation stream, max over ranks.  The KV cache (34.9 GB per
GPU) is far larger than L2, so no flush is needed between steps.  Every phase (warm-up, timed,
end to end, median, profile, parity) restarts at the end of the prompt, so the measured
positions are the configuration's own (2047 onwards, inside its 2080-row capacity).  ``e2e``
repeats K steps through the public API with the step's tokens copied host->device from pinned
memory and the generated tokens copied back every step.  ``roofline`` reports the attention
kernel (the dominant, HBM-bound kernel) from per-node CUDA events over one extra profiled step.
``parity`` replays the first steps through the reference's own kernel bodies (generated, naive,
unfused) on the same state and compares tokens and logits; ``library_faults`` is the kernel
library's fault word after the run (must be 0).  At one GPU the line also carries
``small_configs`` (3, 4 and 2: time per step, speed-up over the naive
graph, parity), ``small_batches`` (config 5's model with 1, 4 and 16 requests: latency-oriented
decode, with the attention's fraction of the copy bandwidth) and, at every GPU count, ``full_job`` (config 5's 4096 requests in waves of one
shard per GPU).  ``--impl reference`` times the reference's own CPU decoder (its NumPy
algorithm, restated in oracle/) on a bounded sample of requests on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "composable-kernel-language_b200" / "python"))

WORKLOADS = {
    # name: (batch per GPU, hidden, heads, layers, ffn, vocab, context, steps, seed, eps)
    "cfg5": (512, 1024, 16, 4, 4096, 32000, 2048, 32, 4, 1e-6),
    "cfg1": (1, 64, 4, 2, 256, 512, 16, 16, 0, 1e-6),
    "cfg3": (64, 256, 8, 2, 1024, 512, 16, 16, 2, 1e-6),
    "cfg4": (256, 64, 4, 8, 256, 512, 16, 16, 3, 1e-6),
    # dst = (src + 0.5) + 0.5 over 2^28 float32 elements per GPU, seed 1.
    "vector": (1 << 28, 0, 0, 0, 0, 0, 0, 0, 1, 0.5),
}
PEAKS = ROOT / "MEASURED_PEAKS.json"


# DRAM bytes per algorithmic byte of one attention launch, from an ncu capture of the same
# kernel on the 32-request cfg5 shard at position 2047 (read 537.03 MB + write 4.03 MB for
# 537.13 MB of K/V rows, q and context).  The traffic grows with the rows read, so the ratio
# scales it to the bench workload.
ATTENTION_TRAFFIC_RATIO = (537.028608e6 + 4.029952e6) / 537.133056e6


def peaks():
    if PEAKS.exists():
        data = json.loads(PEAKS.read_text())
        return data["hbm_gbs"], "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples for this rank's GPU while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, ordinal: int):
        self.ordinal, self.samples, self.process = ordinal, [], None

    def __enter__(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--id={self.ordinal}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.process = None
        return self

    def _read(self):
        for line in self.process.stdout:
            self.samples.append([v.strip() for v in line.split(",")])

    def __exit__(self, *exc):
        if self.process:
            self.process.terminate()
            try:
                self.process.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.process.kill()
            self.thread.join(timeout=5)

    def summary(self):
        rows = [r for r in self.samples if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            for name, value in zip(names, r[5:9]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def distributed():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    group = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        group = dist
    return world, rank, local, group


def reduce_max(group, value: float) -> float:
    if group is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    group.all_reduce(t, op=group.ReduceOp.MAX)
    return float(t.item())


def barrier(group):
    if group is not None:
        group.barrier()


# ---- CPU leg: the reference algorithm on the host --------------------------------------
def host_threads() -> int:
    """Let NumPy's BLAS use every host thread (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    cores = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(cores)
    except ImportError:
        pass
    return cores


def cpu_vector_rate(workload, budget_s: float, min_steps: int, max_steps: int,
                    sample: int = 1 << 26):
    """Elements/s of the NumPy vector pipeline (oracle restatement) on `sample` elements."""
    from oracle import vector_pipeline as ref

    src = ref.make_source(sample, workload[8])
    out = np.empty_like(src)
    times = []
    begin = time.perf_counter()
    while len(times) < max_steps and (len(times) < min_steps or time.perf_counter() - begin < budget_s):
        t0 = time.perf_counter()
        ref.pipeline(src, workload[9], out)
        times.append(time.perf_counter() - t0)
    return sample / statistics.mean(times), len(times), sample


def cpu_rate(args, workload, budget_s, min_steps, max_steps, sample):
    if args.workload == "vector":
        return cpu_vector_rate(workload, budget_s, min_steps, max_steps)
    return cpu_decode_rate(workload, budget_s, min_steps, max_steps, sample)


def cpu_decode_rate(workload, budget_s: float, min_steps: int, max_steps: int, sample: int):
    """Tokens/s of the NumPy decoder (oracle restatement) on `sample` requests."""
    from oracle import decoder as ref

    host_threads()

    b, h, a, l, f, v, ctx, steps, seed, eps = workload
    config = ref.Config(batch=sample, hidden=h, heads=a, layers=l, ffn=f, vocab=v, context=ctx,
                        steps=max(steps, max_steps + 1))
    arrays, rng = ref.make_weights(config, seed)
    arrays.update(ref.empty_state(config))
    prompts = ref.make_prompts(config, rng)
    # The KV prefix the prompt would leave: random values (the step's cost does not depend
    # on them), position at the last prompt token, as after a prefill.
    fill = np.random.default_rng(seed + 1)
    p0 = ctx - 1
    for name in ("kc", "vc"):
        arrays[name][:, :, :, :p0] = fill.standard_normal(arrays[name][:, :, :, :p0].shape,
                                                          dtype=np.float32)
    arrays["position"][0] = p0
    arrays["tokens"] = prompts[-1].copy()
    times = []
    begin = time.perf_counter()
    while len(times) < max_steps and (len(times) < min_steps or time.perf_counter() - begin < budget_s):
        t0 = time.perf_counter()
        ref.decode_step(arrays, config, eps)
        times.append(time.perf_counter() - t0)
    return sample / statistics.mean(times), len(times), sample


def cpu_baseline(args, workload) -> dict:
    """The NumPy restatement of the reference algorithm on a bounded sample, all host threads
    and one thread."""
    if args.workload == "vector":
        rate, done, sample = cpu_vector_rate(workload, 10.0, 3, 40)
        return {"value": rate, "unit": "elements/s", "cores": 1, "kind": "port",
                "sample": f"{sample} elements, {done} passes of (src + b) + b, NumPy (one thread)"}
    sample = min(8, workload[0])
    rate, done, sample = cpu_decode_rate(workload, 15.0, 3, 40, sample)
    cores = host_threads()
    from threadpoolctl import threadpool_limits
    with threadpool_limits(1):
        rate1, done1, _ = cpu_decode_rate(workload, 8.0, 2, 20, sample)
    host_threads()
    return {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
            "value_one_thread": rate1,
            "sample": f"{sample} requests at position {workload[6] - 1}, {done} decode steps of "
                      f"the NumPy decoder (reference algorithm) with {cores} host threads; "
                      f"{done1} steps with one thread give value_one_thread"}


def reference_arm(args, workload, world, rank):
    if rank != 0:
        return 0
    sample = 8 if workload[0] >= 8 else workload[0]
    steps = max(args.steps, 1)
    # Warm-up steps, then `steps` timed steps of the bounded sample.
    cpu_rate(args, workload, 0.0, args.warmup, args.warmup, sample) if args.warmup else None
    rate, done, sample = cpu_rate(args, workload, 1e9, steps, steps, sample)
    vector = args.workload == "vector"
    cores = 1 if vector else host_threads()
    unit = "elements/s" if vector else "tokens/s"
    what = (f"{sample} elements, {done} pipeline passes, NumPy (one thread)" if vector else
            f"{sample} requests at position {workload[6] - 1}, {done} decode steps, NumPy with "
            f"{cores} host threads")
    line = {
        "impl": "reference", "metric": metric_name(args.workload), "value": rate,
        "unit": unit, "n_gpus": args.gpus, "steps": done, "warmup": args.warmup,
        "ms_per_step": 1000.0 * sample / rate, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, workload, world),
        "cpu_baseline": {"value": rate, "unit": unit, "cores": cores, "kind": "port",
                         "sample": what},
        "e2e": {"value": rate, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def metric_name(workload: str) -> str:
    return "decode tokens/s" if workload != "vector" else "vector pipeline elements/s"


def workload_config(args, workload, world):
    b, h, a, l, f, v, ctx, steps, seed, eps = workload
    if args.workload == "vector":
        return {"workload": "vector pipeline (BASELINE config 2): dst = (src + b) + b, fused "
                            "into one launch", "elements_per_gpu": b, "total_elements": b * world,
                "bias": eps, "seed": seed, "parallelism": f"elements x{world}, no collective",
                "l2": "no flush: 2 GiB of src + dst per GPU exceed the 126 MB L2"}
    return {"workload": f"{args.workload} decoder (BASELINE config "
                        f"{ {'cfg5': 5, 'cfg1': 1, 'cfg3': 3, 'cfg4': 4}[args.workload]}), "
                        f"{b} requests per GPU, request-sharded",
            "requests_per_gpu": b, "total_requests": b * world, "layers": l, "hidden": h,
            "heads": a, "head_dim": h // a, "ffn": f, "vocab": v, "context": ctx,
            "seed": seed, "epsilon": eps, "parallelism": f"requests x{world}, no collective",
            "l2": "no flush: per-GPU KV cache and weights exceed the 126 MB L2"
            if args.workload == "cfg5" else "small working set, L2-resident (latency-bound)"}


# ---- GPU leg ----------------------------------------------------------------------------
def vector_arm(args, workload, world, rank, local, group):
    """the two-launch vector pipeline, fused into one streaming launch."""
    import ckl
    from ckl.workloads import vector_pipeline

    n, seed, bias = workload[0], workload[8], workload[9]
    device = ckl.Device(local)
    spec = ckl.BufferSpec((n,), ckl.f32)
    src, dst = device.empty(spec), device.empty(spec)
    # Each GPU's slice of the job: U(-1, 1) from the seed, offset by the rank.
    host = np.random.default_rng(seed + rank).uniform(-1.0, 1.0, n).astype(np.float32)
    src.copy_from_host(host)
    compiled = vector_pipeline.lower(n).compile(target=ckl.NVIDIATarget("sm_100a"),
                                                fuse_pointwise=True)
    inv = compiled.bind(src, dst, float(bias))
    nodes = inv.node_count
    clocks = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        inv.run(mode="graph")
    barrier(group)
    inv.synchronize()
    elapsed_ms = inv.time_launches(args.steps, mode="graph")
    inv.synchronize()
    barrier(group)
    elapsed_ms = reduce_max(group, elapsed_ms)
    value = n * world * args.steps / (elapsed_ms / 1000.0)

    # End to end: the step's source copied in from pinned memory, the result copied out.
    pinned_in, pinned_out = ckl.cuda.PinnedHostBuffer(4 * n), ckl.cuda.PinnedHostBuffer(4 * n)
    np.frombuffer(pinned_in.view(), dtype=np.float32)[:] = host
    barrier(group)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        inv.copy_in_async(src, pinned_in.pointer, 4 * n)
        inv.launch(mode="graph")
        inv.copy_out_async(dst, pinned_out.pointer, 4 * n)
        inv.synchronize()
    e2e_s = reduce_max(group, time.perf_counter() - t0)
    e2e = n * world * args.steps / e2e_s
    clocks.__exit__(None, None, None)

    per_node = inv.profile_nodes(3)
    hbm, peak_kind = peaks()
    launch_ms = per_node[0] / 3 if per_node else None
    roofline = None
    if launch_ms:
        algorithmic = 8 * n  # read src, write dst
        achieved = algorithmic / (launch_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "kernel": inv.node_names[0], "achieved": achieved,
                    "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                    "traffic": None, "algorithmic_bytes_per_launch": algorithmic,
                    "launch_ms": launch_ms}
    line = None
    if rank == 0:
        line = {
            "metric": metric_name(args.workload), "value": value, "unit": "elements/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: U(-1, 1) float32 (seed 1 + rank)",
            "config": workload_config(args, workload, world),
            "roofline": roofline,
            "e2e": {"value": e2e, "unit": "elements/s", "h2d_bytes_per_step": 4 * n * world,
                    "d2h_bytes_per_step": 4 * n * world},
            "gpu_launches": nodes * args.steps,
            "graph_nodes_per_step": nodes,
            "clocks": clocks.summary(),
        }
    return line



def restart(sess, position: int, tokens: np.ndarray) -> None:
    """Put the session back at the end of its prompt (position, last prompt tokens): every
    measured phase decodes the same cache positions, inside the configuration's capacity."""
    sess.write("position", np.array([position], np.int32))
    sess.write("tokens", tokens)


def library_faults() -> int:
    from ckl import _native

    return _native.library_faults()


def gpu_arm(args, workload, world, rank, local, group):
    import ckl
    from ckl.workloads import session as S

    b, h, a, l, f, v, ctx, steps, seed, eps = workload
    # The configuration's own capacity (context + its step count); every phase restarts at
    # the end of the prompt, so the cache only grows when one phase has more steps than that.
    phase_steps = max(args.steps, args.warmup, PARITY_STEPS, NAIVE_STEPS + 1)
    shape = S.DecoderShape(batch=b, hidden=h, heads=a, layers=l, ffn=f, vocab=v, context=ctx,
                           steps=max(steps, phase_steps))
    arrays, rng = S.make_weights(shape, seed)
    from ckl.workloads.sharding import shard_prompts

    # Prompts for the whole job, sliced: a request's prompt does not depend on the GPU count.
    all_prompts = rng.integers(0, v, (ctx, b * world), dtype=np.int32)
    prompts = shard_prompts(all_prompts, world, rank)
    cache = (l, b, a, shape.capacity, h // a)
    arrays.update(tokens=prompts[0].copy(), position=np.zeros(1, np.int32),
                  history=np.full((shape.capacity, b), -1, np.int32),
                  kc=(cache, np.float32), vc=(cache, np.float32),
                  logits=np.zeros((b, v), np.float32))
    device = ckl.Device(local)
    t_setup = time.perf_counter()
    sess = S.DecoderSession(device, arrays, epsilon=eps, attention_scale=(h // a) ** -0.5,
                            tails=False, tensor_cores=args.projections == "tensor",
                            whole_step=args.whole_step == "on")
    t_prefill = time.perf_counter()
    if args.prefill in ("batched", "graph"):
        sess.prefill(prompts, batched=args.prefill == "batched")
        sess.invocation.synchronize()
    else:
        sess.write("tokens", prompts[-1])
        sess.write("position", np.array([ctx - 1], np.int32))
    prefill_s = time.perf_counter() - t_prefill
    setup_s = time.perf_counter() - t_setup
    p0, last_tokens = ctx - 1, prompts[-1].copy()
    inv = sess.invocation
    nodes = inv.node_count
    clocks = ClockSampler(local).__enter__()
    for _ in range(args.warmup):
        inv.run(mode="graph")
    restart(sess, p0, last_tokens)
    barrier(group)
    inv.synchronize()
    elapsed_ms = inv.time_launches(args.steps, mode="graph")
    inv.synchronize()
    barrier(group)
    elapsed_ms = reduce_max(group, elapsed_ms)
    value = b * world * args.steps / (elapsed_ms / 1000.0)

    # End to end through the public API: per step, tokens host->device from pinned memory,
    # the step, generated tokens device->host, wait for them.
    restart(sess, p0, last_tokens)
    pinned_in = ckl.cuda.PinnedHostBuffer(4 * b)
    pinned_out = ckl.cuda.PinnedHostBuffer(4 * b)
    tokens_buf = sess.buffers["tokens"]
    host_tokens = np.frombuffer(pinned_in.view(), dtype=np.int32)
    host_tokens[:] = last_tokens
    out_tokens = np.frombuffer(pinned_out.view(), dtype=np.int32)
    barrier(group)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        inv.copy_in_async(tokens_buf, pinned_in.pointer, 4 * b)
        inv.launch(mode="graph")
        inv.copy_out_async(tokens_buf, pinned_out.pointer, 4 * b)
        inv.synchronize()
        host_tokens[:] = out_tokens
    e2e_s = reduce_max(group, time.perf_counter() - t0)
    e2e = b * world * args.steps / e2e_s
    # Median step: the same steps timed one at a time (device time of each, CUDA events).
    restart(sess, p0, last_tokens)
    barrier(group)
    inv.synchronize()
    single = sorted(inv.time_launches(1, mode="graph") for _ in range(args.steps))
    median_ms = reduce_max(group, statistics.median(single))
    clocks.__exit__(None, None, None)

    # Per-kernel device time of one more (profiled, ordinary-mode) step at the first measured
    # position (attention over `ctx` cache rows).
    restart(sess, p0, last_tokens)
    position = p0
    per_node = inv.profile_nodes(1)
    names = inv.node_names
    attention_kernels = ("ckl.fused.attention", "ckl.fused.attention_split")
    attention_kernel = next((n for n in names if n in attention_kernels), attention_kernels[0])
    attention = [t for n, t in zip(names, per_node) if n == attention_kernel]
    hbm, peak_kind = peaks()
    roofline = None
    if attention:
        n_rows = position + 1
        algorithmic = 2 * b * a * n_rows * (h // a) * 4 + 2 * b * h * 4
        launch_ms = statistics.mean(attention)
        achieved = algorithmic / (launch_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "kernel": attention_kernel, "achieved": achieved,
                    "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / hbm,
                    "frac_of": "measured copy bandwidth (read + write stream); a read-only "
                               "stream such as attention's K/V rows can exceed it",
                    "traffic": algorithmic * ATTENTION_TRAFFIC_RATIO,
                    "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                      "32-request shard at position 2047, scaled by algorithmic "
                                      "bytes",
                    "algorithmic_bytes_per_launch": algorithmic,
                    "launch_ms": launch_ms, "launches_profiled": len(attention),
                    "kv_rows_per_head": n_rows}
    share = {}
    for n, t in zip(names, per_node):
        share[n] = share.get(n, 0.0) + t
    total = sum(per_node)
    naive, parity = reference_path(sess, elapsed_ms / args.steps, group, p0, last_tokens)
    faults = library_faults()
    if faults:
        raise RuntimeError(f"kernel library fault word {faults:#x} after the measured steps")
    line = None
    if rank == 0:
        line = {
            "metric": metric_name(args.workload), "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "median_step_us": median_ms * 1000.0,
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded random weights (reference draw order), uniform prompts",
            "config": workload_config(args, workload, world),
            "roofline": roofline,
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 4 * b * world,
                    "d2h_bytes_per_step": 4 * b * world},
            "gpu_launches": nodes * args.steps,
            "graph_nodes_per_step": nodes,
            "kernel_share": {k: round(t / total, 4) for k, t in sorted(share.items(),
                                                                       key=lambda kv: -kv[1])},
            "parity_check": parity["passed"],
            "parity": parity,
            "library_faults": faults,
            "naive_graph": naive,
            "measured_positions": [p0, p0 + phase_steps - 1],
            "cache_capacity": shape.capacity,
            "prefill": args.prefill,
            "projections": args.projections,
            "whole_step": args.whole_step,
            "prefill_setup_s": round(setup_s, 2),
            "prefill_s": round(prefill_s, 3),
            "clocks": clocks.summary(),
        }
    if args.workload == "cfg5" and not args.no_full_job:
        job = full_job(args, sess, workload, world, rank, group)
        if line is not None:
            line["full_job"] = job
    return line


NAIVE_STEPS = 3
PARITY_STEPS = 4
FULL_JOB_REQUESTS = 4096  # BASELINE config 5's whole job
FULL_JOB_STEPS = 8


def reference_path(sess, ms_per_step, group, p0, tokens, rounds=1, steps=NAIVE_STEPS):
    """The reference's own code path on this GPU, timed and used as the parity check.

    Every kernel is generated from its ``workloads.py`` body (naive FP32 code, no library, no
    fusion), the unfused 21L+6-node DAG with the reference's may-alias edges replayed as an
    inferred CUDA graph on the session's buffers.  It stands in for the reference's
    MLIR-compiled graph, which needs an LLVM/MLIR toolchain absent here.  Parity: from the same
    state (end of the prompt), `PARITY_STEPS` steps of the measured program and of this one
    must give the same greedy tokens and logits within 1e-4 relative / 1e-5 absolute.  Its
    time per step is the median over `rounds` rounds of `steps` graph launches from the end of
    the prompt (the small configurations use the protocol of their own measurement)."""
    import ckl
    from ckl.workloads import decoder

    t0 = time.perf_counter()
    program = sess.lowered.compile(target=ckl.NVIDIATarget("sm_100a"), fuse_pointwise=False,
                                   fuse_library=False, library=False)
    compile_s = time.perf_counter() - t0
    arguments = [sess.buffers[name] for name in decoder.ARGUMENTS[:-2]]
    naive = program.bind(*arguments, float(sess.epsilon), float(sess.attention_scale))
    runs = {}
    for label, invocation in (("measured", sess.invocation), ("reference", naive)):
        restart(sess, p0, tokens)
        for _ in range(PARITY_STEPS):
            invocation.run(mode="graph")
        runs[label] = (sess.read("history")[p0:p0 + PARITY_STEPS], sess.read("logits"))
    (ours, our_logits), (theirs, their_logits) = runs["measured"], runs["reference"]
    scale = np.maximum(np.abs(their_logits), 1e-30)
    excess = np.abs(our_logits - their_logits) - (1e-5 + 1e-4 * np.abs(their_logits))
    parity = {"passed": bool(np.array_equal(ours, theirs) and np.all(excess <= 0)),
              "steps": PARITY_STEPS, "positions": [p0, p0 + PARITY_STEPS - 1],
              "tokens_equal": bool(np.array_equal(ours, theirs)),
              "logits_max_abs_diff": float(np.max(np.abs(our_logits - their_logits))),
              "logits_max_rel_diff": float(np.max(np.abs(our_logits - their_logits) / scale)),
              "against": "the reference's kernel bodies compiled naively (generated, unfused, "
                         "reference DAG) on the same GPU and state",
              "tolerance": "tokens exact; logits 1e-4 relative + 1e-5 absolute (last step)"}
    restart(sess, p0, tokens)
    naive.run(mode="graph")
    naive.synchronize()
    timings = []
    for _ in range(rounds):
        restart(sess, p0, tokens)
        naive.synchronize()
        barrier(group)
        timings.append(reduce_max(group, naive.time_launches(steps, mode="graph")) / steps)
    naive_ms = statistics.median(timings)
    return ({"ms_per_step": naive_ms, "steps": steps, "rounds": rounds,
             "graph_nodes_per_step": naive.node_count, "speedup": naive_ms / ms_per_step,
             "compile_s": round(compile_s, 2),
             "what": "reference kernel bodies compiled naively (ckl codegen + NVRTC, sm_100a), "
                     "reference DAG, inferred graph, same buffers and GPU"}, parity)


def full_job(args, sess, workload, world, rank, group):
    """BASELINE config 5's whole job (4096 requests) at this run's GPU count, in waves of the
    per-GPU shard: each wave prefills its requests' prompts (batched) and decodes
    `FULL_JOB_STEPS` steps; device time of the decode steps is max over ranks per wave."""
    b, h, a, l, f, v, ctx, steps, seed, eps = workload
    waves = max(1, FULL_JOB_REQUESTS // (b * world))
    rng = np.random.default_rng([seed, 4096])
    inv = sess.invocation
    decode_ms, prefill_s = 0.0, 0.0
    for wave in range(waves):
        prompts_all = rng.integers(0, v, (ctx, b * world), dtype=np.int32)
        prompts = np.ascontiguousarray(prompts_all[:, rank * b:(rank + 1) * b])
        sess.write("history", np.full(sess.shapes["history"][0], -1, np.int32))
        barrier(group)
        t0 = time.perf_counter()
        sess.prefill(prompts, batched=True)
        inv.synchronize()
        prefill_s += reduce_max(group, time.perf_counter() - t0)
        barrier(group)
        decode_ms += reduce_max(group, inv.time_launches(FULL_JOB_STEPS, mode="graph"))
    requests = waves * b * world
    tokens = requests * FULL_JOB_STEPS
    return {"requests": requests, "waves": waves, "requests_per_gpu_per_wave": b,
            "decode_steps_per_wave": FULL_JOB_STEPS,
            "decode_tokens_per_s": tokens / (decode_ms / 1000.0),
            "decode_s": decode_ms / 1000.0, "prefill_s": prefill_s,
            "job_tokens_per_s": tokens / (decode_ms / 1000.0 + prefill_s),
            "what": "strong scaling of the fixed 4096-request job: waves of one shard per GPU, "
                    "batched prefill of each wave's 2048-token prompts, then decode steps; "
                    "prompts seeded per wave"}


SMALL_ROUNDS, SMALL_STEPS, SMALL_WARMUP = 5, 16, 20


def small_decoder(name, local):
    """One latency-bound BASELINE decoder config on this GPU: CUDA-event time per step (median
    of `SMALL_ROUNDS` rounds of `SMALL_STEPS` graph launches from the end of the prompt), the
    reference's naive code path on the same state and its parity check."""
    import ckl
    from ckl.workloads import session as S

    b, h, a, l, f, v, ctx, steps, seed, eps = WORKLOADS[name]
    shape = S.DecoderShape(batch=b, hidden=h, heads=a, layers=l, ffn=f, vocab=v, context=ctx,
                           steps=max(steps, SMALL_STEPS, SMALL_WARMUP))
    arrays, rng = S.make_weights(shape, seed)
    prompts = S.make_prompts(shape, rng)
    arrays.update(S.initial_state(shape))
    arrays["tokens"] = prompts[0].copy()
    sess = S.DecoderSession(ckl.Device(local), arrays, epsilon=eps,
                            attention_scale=(h // a) ** -0.5, tails=False)
    sess.prefill(prompts, batched=True)
    p0, last = ctx - 1, prompts[-1].copy()
    inv = sess.invocation
    for _ in range(SMALL_WARMUP):
        inv.run(mode="graph")
    rounds = []
    for _ in range(SMALL_ROUNDS):
        restart(sess, p0, last)
        inv.synchronize()
        rounds.append(inv.time_launches(SMALL_STEPS, mode="graph") / SMALL_STEPS)
    ms = statistics.median(rounds)
    naive, parity = reference_path(sess, ms, None, p0, last, rounds=SMALL_ROUNDS,
                                   steps=SMALL_STEPS)
    return {"ms_per_step": ms, "us_per_step": 1000.0 * ms, "tokens_per_s": b / (ms / 1000.0),
            "graph_nodes_per_step": inv.node_count, "naive_ms_per_step": naive["ms_per_step"],
            "speedup_vs_naive_graph": naive["speedup"], "parity_check": parity["passed"],
            "parity": parity, "requests": b, "positions": [p0, p0 + SMALL_STEPS - 1],
            "timing": f"median of {SMALL_ROUNDS} rounds of {SMALL_STEPS} graph launches, CUDA "
                      f"events, after {SMALL_WARMUP} warm-up steps"}


def small_vector(local, steps: int):
    """BASELINE config 2 on this GPU: the fused pipeline against the reference's own two
    generated launches through the temporary (same buffers), bitwise parity of the results."""
    import ckl
    from ckl.workloads import vector_pipeline

    n, seed, bias = WORKLOADS["vector"][0], WORKLOADS["vector"][8], WORKLOADS["vector"][9]
    device = ckl.Device(local)
    spec = ckl.BufferSpec((n,), ckl.f32)
    src, dst = device.empty(spec), device.empty(spec)
    src.copy_from_host(np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32))
    lowered = vector_pipeline.lower(n)
    target = ckl.NVIDIATarget("sm_100a")
    fused = lowered.compile(target=target, fuse_pointwise=True).bind(src, dst, float(bias))
    naive = lowered.compile(target=target, fuse_pointwise=False, library=False).bind(
        src, dst, float(bias))
    results, times = {}, {}
    for label, inv in (("fused", fused), ("naive", naive)):
        for _ in range(3):
            inv.run(mode="graph")
        times[label] = inv.time_launches(steps, mode="graph") / steps
        out = np.empty(n, np.float32)
        dst.copy_to_host(out)
        results[label] = out
    same = results["fused"].tobytes() == results["naive"].tobytes()
    return {"ms_per_step": times["fused"], "elements_per_s": n / (times["fused"] / 1000.0),
            "achieved_gbs": 8 * n / (times["fused"] / 1000.0) / 1e9,
            "naive_ms_per_step": times["naive"], "speedup_vs_naive_graph":
                times["naive"] / times["fused"], "parity_check": bool(same),
            "parity": {"passed": bool(same), "against": "the reference program's two generated "
                       "launches through its temporary, same GPU and buffers",
                       "tolerance": "bitwise"}, "elements": n}


def small_configs(args, local):
    out = {}
    for name in ("cfg1", "cfg3", "cfg4"):
        out[name] = small_decoder(name, local)
    out["vector"] = small_vector(local, max(args.steps, 3))
    return out


SMALL_BATCHES = (1, 4, 16)


def small_batch(local, requests: int):
    """BASELINE config 5's model with a few requests on this GPU (latency-oriented decode): the
    KV prefix of 2048 rows is left zero (the per-step work does not depend on its values),
    every step decodes from position 2047.  Time per step is the median of `SMALL_ROUNDS`
    rounds of `SMALL_STEPS` graph launches; the attention kernel's fraction of the measured
    copy bandwidth comes from one per-node profiled step; the reference's naive path is timed
    on the same state and replayed as the parity check."""
    import ckl
    from ckl.workloads import session as S

    _, h, a, l, f, v, ctx, _, seed, eps = WORKLOADS["cfg5"]
    shape = S.DecoderShape(batch=requests, hidden=h, heads=a, layers=l, ffn=f, vocab=v,
                           context=ctx, steps=max(SMALL_STEPS, SMALL_WARMUP, PARITY_STEPS) + 8)
    arrays, rng = S.make_weights(shape, seed)
    last = rng.integers(0, v, requests, dtype=np.int32)
    cache = (l, requests, a, shape.capacity, h // a)
    arrays.update(tokens=last.copy(), position=np.array([ctx - 1], np.int32),
                  history=np.full((shape.capacity, requests), -1, np.int32),
                  kc=(cache, np.float32), vc=(cache, np.float32),
                  logits=np.zeros((requests, v), np.float32))
    sess = S.DecoderSession(ckl.Device(local), arrays, epsilon=eps,
                            attention_scale=(h // a) ** -0.5, tails=False)
    p0 = ctx - 1
    inv = sess.invocation
    for _ in range(SMALL_WARMUP):
        inv.run(mode="graph")
    rounds = []
    for _ in range(SMALL_ROUNDS):
        restart(sess, p0, last)
        inv.synchronize()
        rounds.append(inv.time_launches(SMALL_STEPS, mode="graph") / SMALL_STEPS)
    ms = statistics.median(rounds)
    restart(sess, p0, last)
    per_node = inv.profile_nodes(1)
    names = inv.node_names
    attention = [t for n, t in zip(names, per_node)
                 if n in ("ckl.fused.attention", "ckl.fused.attention_split")]
    hbm, _ = peaks()
    frac = None
    if attention:
        algorithmic = 2 * requests * a * ctx * (h // a) * 4 + 2 * requests * h * 4
        frac = algorithmic / (statistics.mean(attention) / 1000.0) / 1e9 / hbm
    naive, parity = reference_path(sess, ms, None, p0, last)
    projections = ("streamed few-row FFMA" if "ckl.fused.norm_linear" in names else
                   "tensor cores" if "ckl.fused.panel_gate_up" in names else "FFMA")
    return {"ms_per_step": ms, "tokens_per_s": requests / (ms / 1000.0),
            "attention_frac_of_copy": frac, "attention_nodes": len(attention),
            "projections": projections, "graph_nodes_per_step": inv.node_count,
            "naive_ms_per_step": naive["ms_per_step"],
            "speedup_vs_naive_graph": naive["speedup"], "parity_check": parity["passed"],
            "parity": parity, "positions": [p0, p0 + SMALL_STEPS - 1],
            "timing": f"median of {SMALL_ROUNDS} rounds of {SMALL_STEPS} graph launches, CUDA "
                      f"events, after {SMALL_WARMUP} warm-up steps; zero KV prefix"}


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--workload", choices=tuple(WORKLOADS), default="cfg5")
    parser.add_argument("--requests-per-gpu", type=int)
    parser.add_argument("--context", type=int, help="override the prompt length (profiling)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--whole-step", choices=("on", "off"), default="on",
                        help="small decoders: the whole decode step as one kernel (on) or the "
                             "per-layer fused graph (off)")
    parser.add_argument("--no-full-job", action="store_true",
                        help="cfg5: skip the 4096-request full job (waves of one shard per GPU)")
    parser.add_argument("--no-small-configs", action="store_true",
                        help="cfg5 at one GPU: skip the cfg1/cfg3/cfg4/vector lines")
    parser.add_argument("--projections", choices=("tensor", "ffma"), default="tensor",
                        help="batched projections on tcgen05 tensor cores (3xTF32) or FFMA")
    parser.add_argument("--prefill", choices=("batched", "graph", "synthetic"), default="batched",
                        help="batched: chunked prefill of all prompt positions (library graph); "
                             "graph: one teacher-forced decode step per prompt token; synthetic: "
                             "zero KV prefix and position at the last prompt token (profiling)")
    args = parser.parse_args()
    if args.warmup < 0 or args.steps < 1:
        parser.error("steps must be positive and warmup nonnegative")
    workload = list(WORKLOADS[args.workload])
    if args.requests_per_gpu:
        workload[0] = args.requests_per_gpu
    if args.context:
        workload[6] = args.context
    workload = tuple(workload)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        return reference_arm(args, workload, world, int(os.environ.get("RANK", "0")))
    world, rank, local, group = distributed()
    arm = vector_arm if args.workload == "vector" else gpu_arm
    line = arm(args, workload, world, rank, local, group)
    if rank == 0:
        if world == 1 and args.workload == "cfg5" and not args.no_small_configs:
            line["small_configs"] = small_configs(args, local)
            if not args.requests_per_gpu:
                line["small_batches"] = {str(r): small_batch(local, r) for r in SMALL_BATCHES}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args, workload)
        print(json.dumps(line), flush=True)
    if group is not None:
        group.barrier()
        group.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

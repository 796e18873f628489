#!/usr/bin/env python
"""Benchmark of the GDN decode hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (the default is the one the headline metric is quoted on):
  decode  config 2: indexed decode, 256 sequences per GPU, T=1, pool of 1024 fp32 slots [32,128,128]
  verify  config 3: MTP verify, 64 sequences per GPU, T=4, accepted ~ U{1..4}
  commit  config 3's explicit commit: copy_state of each sequence's accepted slot to its home slot
  sample  config 3's greedy draft verification (greedy_verify): 64 requests x 3 drafts, 4 fp32
          logits rows each over a 151,936-token vocabulary
  conv    config 2 with the causal conv1d state update before the decode (conv_decode: the conv
          kernel, then the decode, in one call): bf16 conv state of width 4 per sequence; the
          pipeline it replaces (vLLM's conv kernel, then decode) is timed beside it when vLLM is
          importable
  copy    config 4: gather 512 slots of a 2048-slot layer pool, scatter them to a permuted set
  stacked config 5: 48 layers of T=4 verify over 2048 sequences sharded across the ranks (strong
          scaling), replayed as one CUDA graph per step; run it with a few --steps (~0.2 s each)
A step is one launch of the op over that batch.  Under torchrun every rank runs the same
per-GPU workload on its own slot shard (weak scaling, no data-path collective); the
rank-local device times are combined as their maximum.  Rank 0 prints one JSON line.
The default (decode) line also carries `extra`: configs 3 (verify) and 4 (copy) and both decode
configs on a bf16 state pool, each timed the same way after the headline (--no-extras skips them).

--impl reference times the CPU oracle port (oracle/, all host threads) on the same workload and
metric; under torchrun only rank 0 runs it.  When a GPU and the reference harness
(oracle/_ref/libref_harness.so) are present it also times the reference's own CUDA kernel at the
BASELINE geometry (HV=32) on configs 2 and 3 (`reference_gpu_kernel`).
"""

from __future__ import annotations

import argparse
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "GDN decode tokens/s and state HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 1024 * 1024


# ---------------------------------------------------------------------------------------------
# process setup
# ---------------------------------------------------------------------------------------------
def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--workload", choices=("decode", "verify", "decode_bf16", "verify_bf16", "commit", "sample", "conv",
                                          "copy", "stacked"),
                   default="decode")
    p.add_argument("--e2e-steps", type=int, default=200,
                   help="steps of the end-to-end (host buffers) measurement, independent of --steps")
    p.add_argument("--decode-kernel", choices=("auto", "stream", "rowreg"), default="auto",
                   help="decode kernel variant (all compute the same results)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline budget (rank 0, N=1)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-compare", action="store_true",
                   help="conv workload: skip the vLLM conv + decode comparison pipeline")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the secondary configs (3, 4, bf16 pool) that the default decode line also reports")
    args = p.parse_args(argv)
    if args.warmup < 3:
        p.error("--warmup must be at least 3")
    if args.steps < 1:
        p.error("--steps must be positive")
    return args


class Dist:
    """Rank bookkeeping; a gloo group carries the host barriers and the max-over-ranks timing."""

    def __init__(self, gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}: launch N>1 under torchrun")
        self.group = None
        if self.world > 1:
            import torch.distributed as dist

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group("gloo", rank=self.rank, world_size=self.world, timeout=timedelta(seconds=120))
            self.group = dist

    def barrier(self):
        if self.group is not None:
            self.group.barrier()

    def max(self, value: float) -> float:
        if self.group is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64)
        self.group.all_reduce(t, op=self.group.ReduceOp.MAX)
        return float(t.item())

    def sum(self, value: float) -> float:
        if self.group is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64)
        self.group.all_reduce(t, op=self.group.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.group is not None:
            self.group.destroy_process_group()


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "source": "fallback"}


def ncu_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    entry = json.loads(path.read_text()).get(workload)
    return None if entry is None else entry.get("bytes_per_launch")


class ClockSampler:
    """nvidia-smi clock / throttle sampling around the timed region."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.window = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def mark(self, start: float, end: float):
        self.window = (start, end)

    def summary(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for rec in csv.reader(io.StringIO(out)):
            if len(rec) < 10:
                continue
            rec = [r.strip() for r in rec]
            try:
                stamp = time.mktime(time.strptime(rec[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                stamp += float("0." + rec[0].split(".")[1]) if "." in rec[0] else 0.0
                rows.append((stamp, float(rec[2]), float(rec[3]), rec[5], rec[6:10]))
            except (ValueError, IndexError):
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        start, end = self.window if self.window else (rows[0][0], rows[-1][0])
        inside = [r for r in rows if start - 0.15 <= r[0] <= end + 0.15]
        scope = "timed region"
        if not inside:
            inside, scope = rows, "whole run (timed region shorter than the 100 ms sampling interval)"
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": reasons, "samples": len(inside), "scope": scope}


# ---------------------------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------------------------
def timed_launches(fn, steps: int, warmup: int, dist: Dist, stream):
    """W untimed calls, then K timed calls bracketed by barrier + synchronize.

    One CUDA event pair brackets the whole timed region on the launching stream; the average
    step duration is the region time over K.  (Event pairs around every launch were measured
    to add 3-5 us per step and to slow the neighbouring kernels, so they are not used.)
    """
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    begin.record(stream)
    for _ in range(steps):
        fn()
    finish.record(stream)
    torch.cuda.synchronize()
    wall1 = time.time()
    dist.barrier()
    total_ms = begin.elapsed_time(finish)
    return total_ms, total_ms / steps, (wall0, wall1)


class Workload:
    """One timed unit of the bench: `fn` runs one step; the byte and unit counts feed the roofline."""

    def __init__(self, fn, bytes_per_launch, touched, units_per_step, unit, config, *, case=None,
                 launches_per_step=1, kernels_per_step=None, dtype="fp32", cleanup=None):
        self.fn = fn
        self.bytes_per_launch = bytes_per_launch
        self.touched = touched
        self.units_per_step = units_per_step
        self.unit = unit
        self.config = config
        self.case = case
        self.launches_per_step = launches_per_step
        self.kernels_per_step = launches_per_step if kernels_per_step is None else kernels_per_step
        self.dtype = dtype
        self.cleanup = cleanup


def build_workload(name: str, args, dist: Dist, device, stream) -> Workload:
    import torch

    from lightdelta_b200 import workloads

    seed = 1000 * dist.rank
    if name in ("decode", "verify", "decode_bf16", "verify_bf16"):
        one_token = name in ("decode", "decode_bf16")
        bf16_pool = name.endswith("_bf16")
        case = workloads.config2(device, seed=2 + seed) if one_token else workloads.config3(device, seed=3 + seed)
        if bf16_pool:
            # The same batches on a bf16 state pool (fp32 recurrence, each stored step rounded).
            case.pool = case.pool.to(torch.bfloat16)
        op_args = case.op_args()
        requests, width = case.slots.shape
        hv, h = case.num_v_heads, case.num_k_heads
        itemsize = 2 if bf16_pool else 4
        op = torch.ops.lightdelta.decode_bf16_state if bf16_pool else torch.ops.lightdelta.decode

        def fn():
            op(*op_args)

        config = {"workload": f"config{'2' if one_token else '3'}_{name}", "sequences_per_gpu": requests,
                  "tokens_per_sequence": width, "num_k_heads": h, "num_v_heads": hv, "head_dim": 128,
                  "pool_slots": case.pool.shape[0], "state_dtype": "bf16" if bf16_pool else "fp32",
                  "activation_dtype": "bf16", "decode_kernel": args.decode_kernel}
        return Workload(fn, workloads.decode_algorithmic_bytes(requests, width, case.tokens, h, hv,
                                                               state_itemsize=itemsize),
                        requests * (1 + width) * hv * workloads.SLOT_HEAD_BYTES * itemsize // 4, case.tokens,
                        "tokens/s", config, case=case, dtype="fp32 (bf16 state pool)" if bf16_pool else "fp32")
    if name == "commit":
        # Config 3's explicit commit: after verify, copy each sequence's accepted step state to
        # its home slot (the first of its candidate slots) with the pool-to-pool copy op.
        # Four independent config-3 batches on one 1025-slot pool, used in turn, so that the
        # slots one step reads were last touched four steps earlier (> 126 MB L2 in between).
        first = workloads.config3(device, seed=3 + seed, pool_slots=1025)
        pool = first.pool
        sets = []
        for k in range(4):
            verify = first if k == 0 else workloads.config3(device, seed=3 + seed + 17 * k, pool_slots=1025,
                                                            pool=pool)
            src = verify.slots.gather(1, (verify.accepted - 1).long()[:, None]).flatten().contiguous()
            sets.append((src, verify.slots[:, 0].contiguous()))
        turn = [0]

        def fn():
            src, dst = sets[turn[0] % 4]
            turn[0] += 1
            torch.ops.lightdelta.copy_state(pool, src, dst)

        moved_per_set = [int((src != dst).sum().item()) for src, dst in sets]
        moved = sum(moved_per_set) / 4
        config = {"workload": "config3_commit_copy", "sequences_per_gpu": first.slots.shape[0],
                  "slots_copied_per_step": moved, "pool_slots": pool.shape[0], "batches_in_turn": 4,
                  "note": "a sequence whose accepted slot is its home slot copies nothing"}
        return Workload(fn, moved * 2 * first.num_v_heads * workloads.SLOT_HEAD_BYTES,
                        sum(moved_per_set) * 2 * first.num_v_heads * workloads.SLOT_HEAD_BYTES,
                        first.slots.shape[0], "sequences/s", config, dtype="fp32 (bit copy)")
    if name == "conv":
        case = workloads.config2(device, seed=2 + seed)
        conv = workloads.make_conv_state(case, case.pool.shape[0], seed=7 + seed)
        fused_args = workloads.conv_decode_args(case, conv)
        requests, width = case.slots.shape
        hv, h = case.num_v_heads, case.num_k_heads
        dim = case.qkv.shape[1]
        conv_width = conv.weight.shape[1]
        # Per token, besides the decode's bytes: the conv reads the window ((width - 1) bf16
        # positions of every channel) and the pre-conv row, writes the shifted state
        # (width - 2 + 1 positions) and the post-conv row.
        conv_bytes = case.tokens * dim * 2 * ((conv_width - 1) + (conv_width - 1) + 2)

        def fn():
            torch.ops.lightdelta.conv_decode(*fused_args)

        config = {"workload": "config2_conv_decode", "sequences_per_gpu": requests, "tokens_per_sequence": width,
                  "num_k_heads": h, "num_v_heads": hv, "conv_width": conv_width, "conv_state_dtype": "bf16",
                  "conv_layout": "[slots, dim, L]", "launches_per_step": "conv update + decode",
                  "vllm_pipeline": None if args.no_compare else unfused_conv_decode_us(case, conv, stream)}
        # The two kernels (conv update, decode) are accounted together as one step.
        return Workload(fn, workloads.decode_algorithmic_bytes(requests, width, case.tokens, h, hv) + conv_bytes,
                        requests * 2 * hv * workloads.SLOT_HEAD_BYTES, case.tokens, "tokens/s", config,
                        kernels_per_step=2)
    if name == "sample":
        sampling = workloads.sampling_case(device, seed=6 + seed)
        turn = [0]

        def fn():
            buffer = turn[0] % len(sampling.logits)
            turn[0] += 1
            torch.ops.lightdelta.greedy_verify(*sampling.op_args(buffer))

        rows, vocab = sampling.logits[0].shape
        config = {"workload": "config3_greedy_verify", "requests_per_gpu": sampling.requests,
                  "draft_tokens": sampling.sampled.shape[1] - 1, "logits_rows": rows, "vocab": vocab,
                  "logits_dtype": "fp32", "logits_buffers_in_turn": len(sampling.logits)}
        w = Workload(fn, sampling.bytes_per_launch(), sampling.bytes_per_launch() * len(sampling.logits),
                     sampling.requests, "requests/s", config, dtype="fp32 logits, int32 tokens")
        w.sampling = sampling
        return w
    if name == "stacked":
        from lightdelta_b200 import sharding

        total_sequences, layers, width = 2048, 48, 4
        local = len(sharding.shard_range(total_sequences, dist.rank, dist.world))
        free, _ = torch.cuda.mem_get_info(device)
        activations = layers * local * width * 40 * 1024  # proj + out + temporaries per token-layer
        wl = workloads.stacked_workload(device, local, layers=layers, width=width, seed=5 + seed,
                                        max_pool_bytes=max(0, free - activations - (8 << 30)))
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                for c in wl.layers:
                    torch.ops.lightdelta.decode(*c.op_args())
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for c in wl.layers:
                torch.ops.lightdelta.decode(*c.op_args())
        torch.cuda.synchronize()

        def fn():
            graph.replay()

        config = {"workload": "config5_stacked_verify", "layers": layers, "sequences_total": total_sequences,
                  "sequences_per_gpu": local, "tokens_per_sequence": width, "num_k_heads": 16, "num_v_heads": 32,
                  "physical_layer_pools": len(wl.pools),
                  "pool_slots_per_layer": wl.pools[0].shape[0], "cuda_graph": "one graph of 48 decode launches",
                  "decode_kernel": args.decode_kernel}
        return Workload(fn, wl.step_bytes() // layers, wl.step_bytes(), local * width, "tokens/s", config,
                        launches_per_step=layers, cleanup=graph.reset)
    if name == "copy":
        pool = torch.empty(2048, 32, 128, 128, device=device)
        pool.normal_(0.0, 0.02)
        gather_idx, scatter_idx = workloads.config4_indices(device, seed=4 + seed)
        packed = torch.empty(512, 32, 128, 128, device=device)
        valid = torch.ones(512, device=device, dtype=torch.bool)

        def fn():
            torch.ops.lightdelta.gather_state(pool, gather_idx, valid, packed)
            torch.ops.lightdelta.scatter_state(packed, scatter_idx, pool)

        bytes_per_launch = 512 * 32 * workloads.SLOT_HEAD_BYTES * 2  # per op: read + write 512 slots
        config = {"workload": "config4_copy", "pool_slots": 2048, "slots_per_step": 512,
                  "ops_per_step": ["gather_state", "scatter_state"], "num_v_heads": 32, "head_dim": 128}
        return Workload(fn, bytes_per_launch, bytes_per_launch * 2, 512, "slots/s", config, launches_per_step=2,
                        dtype="fp32 (bit copy)")
    raise ValueError(name)


# Secondary results of the default (config 2) line: BASELINE configs 3 and 4 and the bf16 pool.
EXTRA_WORKLOADS = ("verify", "copy", "decode_bf16", "verify_bf16")


def measure(w: Workload, steps: int, warmup: int, dist: Dist, stream, peaks: dict) -> dict:
    total_ms, launch_ms, window = timed_launches(w.fn, steps, warmup, dist, stream)
    max_ms = dist.max(total_ms)
    min_ms = -dist.max(-total_ms)
    kernel_ms = launch_ms / w.launches_per_step
    achieved = w.bytes_per_launch / (kernel_ms * 1e-3) / 1e9
    return {"total_ms": total_ms, "max_ms": max_ms, "min_ms": min_ms, "kernel_ms": kernel_ms, "achieved_gbs": achieved,
            "frac": achieved / peaks["hbm_gbs"], "window": window,
            "value": dist.sum(w.units_per_step) * steps / (max_ms * 1e-3),
            "state_gbs": dist.sum(w.bytes_per_launch * w.launches_per_step * steps / (total_ms * 1e-3) / 1e9)}


def run_ours(args, dist: Dist) -> dict | None:
    import torch

    from lightdelta_b200 import capi, ops  # noqa: F401

    capi.set_decode_kernel(args.decode_kernel)
    torch.cuda.set_device(dist.local_rank)
    device = torch.device("cuda", dist.local_rank)
    stream = torch.cuda.current_stream(device)
    sampler = ClockSampler(device.index if device.index is not None else 0)
    peaks = measured_peaks()

    w = build_workload(args.workload, args, dist, device, stream)
    m = measure(w, args.steps, args.warmup, dist, stream, peaks)
    sampler.mark(*m["window"])
    clocks = sampler.summary()
    case = w.case

    e2e = None
    if args.workload in ("decode", "verify"):
        e2e = run_e2e(case, args, dist, stream, m["kernel_ms"] * 1000)
    cpu = cpu_torch = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline and args.workload in ("decode", "verify"):
        cpu = cpu_baseline(case, args.cpu_seconds)
        cpu_torch = torch_reference_baseline(case, args.cpu_seconds)
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline and args.workload == "sample":
        cpu = sampling_cpu_baseline(w.sampling, args.cpu_seconds)
    if w.cleanup is not None:
        w.cleanup()

    main = {"unit": w.unit, "config": w.config, "dtype": w.dtype, "touched": w.touched,
            "bytes_per_launch": w.bytes_per_launch, "kernels_per_step": w.kernels_per_step}
    extra = None
    if args.workload == "decode" and not args.no_extras:
        del w, case
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        extra = {}
        for name in EXTRA_WORKLOADS:
            xw = build_workload(name, args, dist, device, stream)
            steps = max(args.steps, 50)
            xm = measure(xw, steps, args.warmup, dist, stream, peaks)
            extra[name] = {"workload": xw.config["workload"], "value": xm["value"], "unit": xw.unit,
                           "ms_per_launch": xm["kernel_ms"], "launches_per_step": xw.launches_per_step,
                           "algorithmic_bytes_per_launch": xw.bytes_per_launch, "achieved_gbs": xm["achieved_gbs"],
                           "frac": xm["frac"], "peak_gbs": peaks["hbm_gbs"], "dtype": xw.dtype, "steps": steps,
                           "traffic": ncu_traffic(name)}
            del xw
            torch.cuda.synchronize()
            torch.cuda.empty_cache()

    if dist.rank != 0:
        return None
    result = {
        "metric": METRIC,
        "value": m["value"],
        "unit": main["unit"],
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": m["max_ms"] / args.steps,
        "rank_ms_per_step": {"min": m["min_ms"] / args.steps, "max": m["max_ms"] / args.steps},
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "stacked" else "weak",
        "vs_baseline": None,
        "dtype": main["dtype"],
        "data": "synthetic (seeded, BASELINE config shapes and distributions)",
        "impl": "ours",
        "config": {**main["config"], "parallelism": f"slot-sharded x{dist.world}, no collective",
                   "l2": f"no flush: the {main['touched'] / 1e9:.2f} GB touched per step exceeds the 126 MB L2"},
        "state_gbs": m["state_gbs"],
        "hbm_frac_of_8tbs_per_gpu": m["state_gbs"] / dist.world / NOMINAL_HBM_GBS,
        "roofline": {
            "bound": "hbm",
            "achieved": m["achieved_gbs"],
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": m["frac"],
            "peak_source": peaks["source"],
            "traffic": ncu_traffic(args.workload),
            "algorithmic_bytes_per_launch": main["bytes_per_launch"],
            "kernel_ms": m["kernel_ms"],
        },
        "e2e": e2e,
        "cpu_baseline": cpu,
        "cpu_baseline_reference_torch": cpu_torch,
        "gpu_launches": main["kernels_per_step"] * args.steps,
        "clocks": clocks,
    }
    if extra is not None:
        result["extra"] = extra
    return result


def gpu_local_cpus(device_index: int):
    """Host CPUs attached to the GPU's NUMA node (NVML), or None if unknown."""
    try:
        import pynvml
        import torch

        props = torch.cuda.get_device_properties(device_index)
        bus_id = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus_id.encode())
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, 16)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))
        return cpus or None
    except Exception:  # noqa: BLE001 -- affinity is an optimisation only
        return None


def run_e2e(case, args, dist: Dist, stream, kernel_us: float) -> dict:
    """Same metric through the public op with host buffers.  Every step copies its activations
    and request metadata from pinned host memory, runs torch.ops.lightdelta.decode and reads the
    output back to pinned host memory.  A step's inputs (the projection rows, the a/b rows, slots,
    cu and accepted counts) sit in one pinned staging buffer, so one copy carries them; the op
    reads views of the device copy.  Two buffer sets let the copies of one step overlap the
    kernel of the neighbouring step (H2D, compute and D2H on three streams); the state pool is
    shared, so the kernels still run strictly in order.  After the timed region the same H2D and
    D2H copies are timed alone (`copies_alone`): a step cannot be shorter than the slowest of them
    and the kernel, so `bound` names which one sets the rate on this box."""
    import torch

    device = case.pool.device
    saved_affinity = os.sched_getaffinity(0)
    local = gpu_local_cpus(device.index or 0)
    if local:
        os.sched_setaffinity(0, local)
    try:
        proj = case.qkv.as_strided((case.tokens, case.qkv.stride(0)), (case.qkv.stride(0), 1))
        ba = case.b.as_strided((case.tokens, case.b.stride(0)), (case.b.stride(0), 1))
        parts = [("proj", proj), ("ba", ba), ("slots", case.slots), ("cu", case.cu), ("accepted", case.accepted)]
        offsets, size = {}, 0
        for name, t in parts:
            offsets[name] = size
            size += -(-t.numel() * t.element_size() // 256) * 256  # 256-byte aligned sections
        qkv_width, hv = case.qkv.shape[1], case.num_v_heads

        def views(buf):
            out = {}
            for name, t in parts:
                nbytes = t.numel() * t.element_size()
                out[name] = buf[offsets[name]:offsets[name] + nbytes].view(t.dtype).view(t.shape)
            return out

        host = [torch.empty(size, dtype=torch.uint8).pin_memory() for _ in range(2)]
        for b in range(2):
            hv_views = views(host[b])
            for name, t in parts:
                hv_views[name].copy_(t.cpu())
        dev = [torch.empty(size, dtype=torch.uint8, device=device) for _ in range(2)]
        out_h = [torch.empty(case.out.shape, dtype=case.out.dtype).pin_memory() for _ in range(2)]
        out_d = [torch.empty_like(case.out) for _ in range(2)]
        args_of = []
        for b in range(2):
            d = views(dev[b])
            args_of.append((d["proj"][:, :qkv_width], d["ba"][:, hv:], d["ba"][:, :hv], case.a_log, case.dt_bias,
                            d["slots"], d["cu"], d["accepted"], case.pool,
                            d["proj"][:, qkv_width:].view(case.tokens, hv, 128), case.weight, out_d[b], case.eps))
        h2d = size
        d2h = out_h[0].numel() * out_h[0].element_size()
        s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_h2d = [torch.cuda.Event() for _ in range(2)]
        ev_kernel = [torch.cuda.Event() for _ in range(2)]
        ev_d2h = [torch.cuda.Event() for _ in range(2)]
        for b in range(2):
            ev_kernel[b].record(stream)
            ev_d2h[b].record(stream)
        decode = torch.ops.lightdelta.decode

        def step(i: int):
            b = i & 1
            s_in.wait_event(ev_kernel[b])              # step i-2 has finished reading dev[b]
            with torch.cuda.stream(s_in):
                dev[b].copy_(host[b], non_blocking=True)
            ev_h2d[b].record(s_in)
            stream.wait_event(ev_h2d[b])
            stream.wait_event(ev_d2h[b])               # step i-2's output has been read back
            decode(*args_of[b])
            ev_kernel[b].record(stream)
            s_out.wait_event(ev_kernel[b])
            with torch.cuda.stream(s_out):
                out_h[b].copy_(out_d[b], non_blocking=True)
            ev_d2h[b].record(s_out)

        steps = args.e2e_steps
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        dist.barrier()
        begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        begin.record(stream)
        s_in.wait_stream(stream)
        host0 = time.perf_counter()
        for i in range(steps):
            step(i)
        host_us = (time.perf_counter() - host0) * 1e6 / steps
        stream.wait_stream(s_out)
        finish.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        max_ms = dist.max(begin.elapsed_time(finish))

        # After the timed region: the same copies alone (20 each, on their streams), so the line says
        # what the host path of this box delivers and whether it or the kernel bounds a step.
        def copy_us(stream_, dst, src):
            first, last = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream_):
                dst.copy_(src, non_blocking=True)
                first.record(stream_)
                for _ in range(20):
                    dst.copy_(src, non_blocking=True)
                last.record(stream_)
            torch.cuda.synchronize()
            return first.elapsed_time(last) * 1000 / 20

        h2d_us = copy_us(s_in, dev[0], host[0])
        d2h_us = copy_us(s_out, out_h[0], out_d[0])
    finally:
        os.sched_setaffinity(0, saved_affinity)
    return {"value": case.tokens * steps * dist.world / (max_ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "ms_per_step": max_ms / steps, "host_enqueue_us_per_step": host_us,
            "copies_alone": {"h2d_us": h2d_us, "h2d_gbs": h2d / (h2d_us * 1e3), "d2h_us": d2h_us,
                             "d2h_gbs": d2h / (d2h_us * 1e3),
                             "kernel_us": kernel_us,
                             "bound": "host copies" if max(h2d_us, d2h_us) > kernel_us else "kernel"},
            "api": "torch.ops.lightdelta.decode; inputs from one pinned staging buffer per step (one H2D copy), "
                   "output to pinned memory; double-buffered so copies overlap the neighbouring step's kernel",
            "host_cpus": len(local) if local else None}


# ---------------------------------------------------------------------------------------------
# CPU baseline / reference arm (the oracle port; never the product path)
# ---------------------------------------------------------------------------------------------
def host_workload(case, requests: int | None = None):
    """Host copy of a decode case restricted to `requests` sequences, with the pool compacted to
    the slots they use (slot 0 kept as the null slot)."""
    import numpy as np
    import torch

    R, W = case.slots.shape
    r = R if requests is None else max(1, min(R, requests))
    slots = case.slots[:r].cpu().numpy()
    used = sorted(set(slots.flatten().tolist()) - {0})
    remap = {s: i + 1 for i, s in enumerate(used)}
    pool = case.pool[torch.as_tensor([0] + used, device=case.pool.device, dtype=torch.long)].cpu().numpy()
    tokens = int(case.cu[r].item())

    def bf16(t):
        return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)

    return dict(
        qkv=bf16(case.qkv[:tokens]), a=bf16(case.a[:tokens]), b=bf16(case.b[:tokens]),
        a_log=case.a_log.cpu().numpy(), dt_bias=case.dt_bias.cpu().numpy(),
        slots=np.vectorize(lambda s: remap.get(int(s), 0), otypes=[np.int32])(slots),
        cu=case.cu[: r + 1].cpu().numpy(), accepted=case.accepted[:r].cpu().numpy(), pool=pool,
        gate=bf16(case.gate[:tokens]), weight=bf16(case.weight), out=np.zeros((tokens, case.num_v_heads, 128), np.uint16),
        num_k_heads=case.num_k_heads, tokens=tokens, requests=r,
    )


def oracle_step(w):
    import oracle

    oracle.decode(w["qkv"], w["a"], w["b"], w["a_log"], w["dt_bias"], w["slots"], w["cu"], w["accepted"], w["pool"],
                  w["gate"], w["weight"], w["out"], num_k_heads=w["num_k_heads"], threads=w["threads"])


def cpu_baseline(case, seconds: float) -> dict:
    import oracle

    w = host_workload(case)
    w["threads"] = oracle.default_threads()
    oracle_step(w)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle_step(w)
        reps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    return {"value": w["tokens"] * reps / elapsed, "unit": "tokens/s", "cores": w["threads"], "kind": "port",
            "sample": f"full batch ({w['requests']} sequences, {w['tokens']} tokens) x {reps} repetitions, "
                      f"{elapsed:.1f} s, C oracle with OpenMP"}


def _torch_reference_step(case, requests: int | None = None):
    """One step of the reference's own CPU implementation (oracle/ref_torch.py: its post_conv_gdn,
    compiled unmodified, with GDNBackend's packed gather and commit) on a host copy of `case`
    (the C port's host workload), and that workload."""
    import numpy as np
    import torch

    from oracle import ref_torch

    w = host_workload(case, requests)

    def bf16(x):
        return torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).view(torch.bfloat16)

    args = dict(qkv=bf16(w["qkv"]), a=bf16(w["a"]), b=bf16(w["b"]), a_log=torch.from_numpy(w["a_log"]),
                dt_bias=torch.from_numpy(w["dt_bias"]), slots=torch.from_numpy(w["slots"]),
                cu=torch.from_numpy(w["cu"]), accepted=torch.from_numpy(w["accepted"]),
                pool=torch.from_numpy(w["pool"]), gate=bf16(w["gate"]), weight=bf16(w["weight"]),
                out=torch.zeros(w["out"].shape, dtype=torch.bfloat16))

    def step():
        ref_torch.packed_decode(**args, num_k_heads=w["num_k_heads"])

    return step, w


TORCH_UNAVAILABLE = {"unavailable": "oracle/_ref/torch_path not built (python oracle/build_ref.py where the "
                                    "reference exists)"}


def torch_reference_baseline(case, seconds: float, requests: int | None = None) -> dict:
    """The reference's own CPU implementation on the same host workload as the C port, repeated for
    ~`seconds` on every host thread this process may use."""
    import torch

    import oracle
    from oracle import ref_torch

    if not ref_torch.available():
        return dict(TORCH_UNAVAILABLE)
    step, w = _torch_reference_step(case, requests)
    saved_threads = torch.get_num_threads()
    torch.set_num_threads(oracle.default_threads())
    try:
        step()  # warm-up
        reps, t0 = 0, time.perf_counter()
        while True:
            step()
            reps += 1
            elapsed = time.perf_counter() - t0
            if elapsed >= seconds:
                break
        threads = torch.get_num_threads()
    finally:
        torch.set_num_threads(saved_threads)
    return {"value": w["tokens"] * reps / elapsed, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"{w['requests']} sequences ({w['tokens']} tokens) per step x {reps} steps, {elapsed:.1f} s, "
                      f"the reference's post_conv_gdn (python/lightdelta/reference/gdn.py:70-128) with "
                      f"GDNBackend's packed gather and commit (backend.py:30-91), torch {torch.__version__} CPU"}


def torch_reference_configs(device, runs: int = 5) -> dict:
    """BASELINE configs 1-3 through the reference's own CPU implementation, each the median of `runs`
    timed steps after one warm-up, on every host thread this process may use."""
    import statistics

    import torch

    import oracle
    from lightdelta_b200 import workloads
    from oracle import ref_torch

    if not ref_torch.available():
        return dict(TORCH_UNAVAILABLE)
    cases = (("config1", lambda: workloads.make_decode_case(1, 1, 2, device=device, seed=1)),
             ("config2", lambda: workloads.config2(device, seed=2)),
             ("config3", lambda: workloads.config3(device, seed=3)))
    saved_threads = torch.get_num_threads()
    torch.set_num_threads(oracle.default_threads())
    result = {}
    try:
        for name, build in cases:
            step, w = _torch_reference_step(build())
            step()  # warm-up
            times = []
            for _ in range(runs):
                t0 = time.perf_counter()
                step()
                times.append(time.perf_counter() - t0)
            median = statistics.median(times)
            result[name] = {"tokens_per_s": w["tokens"] / median, "median_ms": median * 1e3, "runs": runs,
                            "sequences": w["requests"], "tokens": w["tokens"]}
        result.update(cores=torch.get_num_threads(), torch=torch.__version__, kind="reference")
    finally:
        torch.set_num_threads(saved_threads)
    return result


def unfused_conv_decode_us(case, conv, stream) -> dict | None:
    """Device time per step of the pipeline conv_decode replaces: vLLM's causal_conv1d_update
    (Triton) then lightdelta::decode, as vllm_layer.py:199-220 runs them; None without vLLM."""
    import torch

    try:
        from vllm.model_executor.layers.mamba.ops.causal_conv1d import causal_conv1d_update
    except Exception:  # noqa: BLE001
        return None
    x = case.qkv.clone()
    state = conv.state.clone()
    pool = case.pool.clone()
    out = torch.empty_like(case.out)
    slots0 = case.slots[:, 0].contiguous()

    def step():
        y = causal_conv1d_update(x, state, conv.weight, None, "silu", conv_state_indices=slots0, validate_data=False)
        torch.ops.lightdelta.decode(y, case.a, case.b, case.a_log, case.dt_bias, case.slots, case.cu, case.accepted,
                                    pool, case.gate, case.weight, out, 1e-6)

    for _ in range(20):
        step()
    torch.cuda.synchronize()
    begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = 500
    begin.record(stream)
    for _ in range(steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    vllm_us = begin.elapsed_time(end) * 1000 / steps
    width = case.slots.shape[1]

    def ours():
        torch.ops.lightdelta.conv_update(x, state, conv.weight, None, slots0, None, case.cu, width)

    for _ in range(20):
        ours()
    torch.cuda.synchronize()
    begin.record(stream)
    for _ in range(steps):
        ours()
    end.record(stream)
    torch.cuda.synchronize()
    return {"us_per_step": vllm_us, "conv_update_alone_us": begin.elapsed_time(end) * 1000 / steps,
            "pipeline": "vLLM causal_conv1d_update (Triton) + lightdelta::decode, same inputs"}


def sampling_cpu_baseline(sampling, seconds: float) -> dict:
    """The C oracle of greedy verification on one logits buffer, repeated for ~`seconds`."""
    import oracle

    host = {k: getattr(sampling, k).cpu().numpy() for k in
            ("cu_num_logits", "query_start_loc", "input_ids", "num_draft_tokens", "seq_lens", "prefill_len")}
    logits = sampling.logits[0].float().cpu().numpy()
    steps = sampling.sampled.shape[1] - 1
    threads = oracle.default_threads()

    def step():
        oracle.greedy_verify(logits, host["cu_num_logits"], host["query_start_loc"], host["input_ids"],
                             host["num_draft_tokens"], host["seq_lens"], host["prefill_len"], steps, threads)

    step()
    reps, t0 = 0, time.perf_counter()
    while True:
        step()
        reps += 1
        elapsed = time.perf_counter() - t0
        if elapsed >= seconds:
            break
    return {"value": sampling.requests * reps / elapsed, "unit": "requests/s", "cores": threads, "kind": "port",
            "sample": f"one {logits.shape[0]}x{logits.shape[1]} fp32 logits batch x {reps} repetitions, "
                      f"{elapsed:.1f} s, C oracle (argmax + prefix check) with OpenMP"}


def reference_gpu_kernel(steps: int, warmup: int) -> dict:
    """The reference's own CUDA kernel (oracle/_ref/libref_harness.so: csrc/gdn_decode.cu compiled
    unmodified, its kernel template launched at value-head ratio 2 = the BASELINE geometry) on
    configs 2 and 3, timed like our arm: back-to-back in-place launches on a pool larger than L2,
    one CUDA event pair over the timed launches."""
    import torch

    from lightdelta_b200 import workloads
    from oracle import ref_kernel

    if not torch.cuda.is_available():
        return {"unavailable": "no GPU visible"}
    if not ref_kernel.available():
        return {"unavailable": "oracle/_ref/libref_harness.so not built (python oracle/build_ref.py)"}
    device = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(device)
    peak = measured_peaks()["hbm_gbs"]
    result = {"kernel": "gdn_decode_post_conv_mtp_kernel<float, 2, false> (csrc/gdn_decode.cu:130-354), "
                        "grid (requests, HV) x 256 threads as the stock launcher (csrc/gdn_decode.cu:407-418)",
              "peak_gbs": peak}
    for name, builder in (("config2_decode", workloads.config2), ("config3_verify", workloads.config3)):
        case = builder(device)
        op_args = case.op_args()
        requests, width = case.slots.shape

        def fn():
            ref_kernel.decode(*op_args)

        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        begin, finish = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        count = max(steps, 50)
        begin.record(stream)
        for _ in range(count):
            fn()
        finish.record(stream)
        torch.cuda.synchronize()
        us = begin.elapsed_time(finish) * 1000 / count
        algorithmic = workloads.decode_algorithmic_bytes(requests, width, case.tokens, case.num_k_heads,
                                                         case.num_v_heads)
        achieved = algorithmic / (us * 1e-6) / 1e9
        result[name] = {"us_per_launch": us, "tokens_per_s": case.tokens / (us * 1e-6), "achieved_gbs": achieved,
                        "frac": achieved / peak, "launches": count}
        del case, op_args
        torch.cuda.empty_cache()
    return result


def reference_copy(args, dist: Dist) -> dict:
    """Config 4 on the host: the reference's CPU state I/O is torch indexing -- GDNBackend's packed
    gather is index_select into the packed buffer and its commit index_copy_ into the pool
    (python/lightdelta/backend.py:40-44, :87-91; its gather_state / scatter_state ops are CUDA-only).
    One step gathers 128 distinct slots of a 257-slot pool and scatters them to 128 others (2 MiB
    slots, 0.5 GiB moved per op), on every host thread this process may use."""
    import torch

    import oracle

    slots = 128
    threads = oracle.default_threads()
    saved_threads = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        gen = torch.Generator().manual_seed(4)
        pool = torch.empty(2 * slots + 1, 32, 128, 128)
        pool.normal_(0.0, 0.02, generator=gen)
        perm = torch.randperm(2 * slots, generator=gen) + 1
        gather_idx, scatter_idx = perm[:slots], perm[slots:]
        packed = torch.empty(slots, 32, 128, 128)

        def step():
            torch.index_select(pool, 0, gather_idx, out=packed)
            pool.index_copy_(0, scatter_idx, packed)

        for _ in range(args.warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        elapsed = time.perf_counter() - t0
    finally:
        torch.set_num_threads(saved_threads)
    value = slots * args.steps / elapsed
    sample = (f"{slots} of config 4's 512 slots per step from a {2 * slots + 1}-slot pool (2 MiB slots), torch "
              f"index_select + index_copy_ (backend.py:40-44, :87-91), torch {torch.__version__} on {threads} threads")
    return {
        "metric": METRIC, "value": value, "unit": "slots/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (bit copy)", "data": "synthetic (seeded)",
        "impl": "reference",
        "config": {"workload": "config4_copy", "pool_slots": 2 * slots + 1, "slots_per_step": slots,
                   "ops_per_step": ["index_select", "index_copy_"], "num_v_heads": 32, "head_dim": 128,
                   "parallelism": "rank 0 host CPU only"},
        "cpu_baseline": {"value": value, "unit": "slots/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "slots/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference(args, dist: Dist) -> dict | None:
    if dist.rank != 0:
        return None
    import torch

    import oracle
    from lightdelta_b200 import workloads

    if args.workload in ("decode_bf16", "verify_bf16"):
        return {"impl": "reference",
                "unavailable": "the reference supports only an fp32 state pool (csrc/gdn_decode.cu:375-377)"}
    if args.workload == "copy":
        return reference_copy(args, dist)
    if args.workload not in ("decode", "verify"):
        return {"impl": "reference", "unavailable": f"the {args.workload} workload has no reference CPU arm in this "
                                                    "harness (the decode, verify and copy workloads do)"}
    device = torch.device("cuda", dist.local_rank) if torch.cuda.is_available() else torch.device("cpu")
    case = workloads.config2(device, seed=2) if args.workload == "decode" else workloads.config3(device, seed=3)
    threads = oracle.default_threads()
    # Size each step so that warmup + steps finish in about a minute.
    probe = host_workload(case, 8)
    probe["threads"] = threads
    t0 = time.perf_counter()
    oracle_step(probe)
    per_request = (time.perf_counter() - t0) / probe["requests"]
    budget = 60.0 / (args.steps + args.warmup)
    requests = max(1, min(case.slots.shape[0], int(budget / max(per_request, 1e-9))))
    w = host_workload(case, requests)
    w["threads"] = threads
    for _ in range(args.warmup):
        oracle_step(w)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle_step(w)
    elapsed = time.perf_counter() - t0
    value = w["tokens"] * args.steps / elapsed
    sample = (f"{w['requests']} of {case.slots.shape[0]} sequences ({w['tokens']} tokens) per step, "
              f"C oracle port with OpenMP on {threads} host threads")
    return {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed * 1e3 / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded, BASELINE config shapes and distributions)",
        "impl": "reference",
        "config": {"workload": f"config{'2' if args.workload == 'decode' else '3'}_{args.workload}",
                   "sequences_per_gpu": case.slots.shape[0], "tokens_per_sequence": case.slots.shape[1],
                   "parallelism": "rank 0 host CPU only"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_torch": torch_reference_baseline(case, args.cpu_seconds),
        "reference_torch_configs": torch_reference_configs(device),
        "reference_gpu_kernel": reference_gpu_kernel(args.steps, args.warmup),
    }


def main(argv=None) -> int:
    args = parse_args(argv)
    dist = Dist(args.gpus)
    try:
        result = run_reference(args, dist) if args.impl == "reference" else run_ours(args, dist)
        if result is not None:
            print(json.dumps(result), flush=True)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Benchmark of the fused-MLP hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

A step is one pass of the fused MLP over one batch: M rows of the configured workload (default
`mgn_node`: MeshGraphNet node MLP, 1,048,576 rows, 256->128->128->128 + LayerNorm, fp16 -- the
second benchmark config, the one the headline metric is quoted on that fits one GPU).

Multi-GPU (torchrun, one process per GPU): rows are independent, so the M rows of the config are
split into contiguous, tile-aligned row ranges, one per rank (strong scaling, the default for
N > 1: global M fixed, as the benchmark configs specify). `--split weak` instead gives every rank
its own M-row slice of an N*M-row job. There is no collective on the data path; NCCL is used only
for the barrier and the max-over-ranks of the timing.

Reported:
  value       rows/s over all ranks, inputs already resident in HBM, CUDA-event timed
  e2e         same metric through the public API with the host->device copy of x (pinned) and
              the device->host copy of the output inside every timed step (plain chains through
              gp_fused_mlp_host, which overlaps the copies of neighbouring row chunks with the
              kernels; composed blocks copy, run and copy back in sequence)
  roofline    the fused kernel against the measured HBM bandwidth (the path is HBM-bound:
              768 B/row vs 131,072 FLOP/row, arithmetic intensity 171 < ridge 253)
  cpu_baseline the CPU oracle (the reference's PyTorch fp32 model, restated) on a bounded sample
  clocks      nvidia-smi samples taken during the timed region

`--impl reference` times the reference's CPU implementation (PyTorch fp32 model, restated in
oracle/) on this host with all cores, on the same config and metric.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from gpu_pipes_b200 import _lib as L  # noqa: E402
from gpu_pipes_b200 import workloads as W  # noqa: E402

L2_BYTES = 126 * 2**20
# DRAM bytes (read + write) per row of one launch of the dominant kernel: constants taken from
# ncu captures of that kernel (dram__bytes_read.sum + dram__bytes_write.sum over the captured
# launch, divided by its rows; for mgn_mp the edge kernel only). Not measured by this script:
# the line marks them as such. Traffic grows in proportion to the rows.
NCU_TRAFFIC_PER_ROW = {"mgn_node": 752.7e6 / 1048576, "nerf": 144.1e6 / 1048576,
                       "gc_edge": 497.7e6 / 131072, "dlrm_interact": 507.5e6 / 65536,
                       "mgn_mp": 744.5e6 / 1048576}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--config", default="mgn_node", choices=sorted(W.WORKLOADS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--split", default=None, choices=["strong", "weak"],
                   help="multi-GPU row split: strong (default; the config's M rows shared by the "
                        "ranks) or weak (M rows per rank)")
    p.add_argument("--m", type=int, default=0, help="override rows per GPU (testing only)")
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--cpu-seconds", type=float, default=8.0)
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--flush", action="store_true",
                   help="time workloads smaller than 2 x L2 step by step around an L2 flush instead "
                        "of rotating over copies of their inputs")
    p.add_argument("--no-graph", action="store_true",
                   help="time per-step library calls instead of CUDA-graph replays of captured steps")
    p.add_argument("--kernel-only", action="store_true",
                   help="time the kernel only (no e2e, CPU baseline or clock sampling); for ncu")
    return p.parse_args()


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# The kernel that dominates each config's step (the one the roofline line describes).
KERNEL_OF = {
    "mgn_node": "mlp_resident_kernel", "mgn_edge": "mlp_resident_pair_kernel",
    "mgn_linears": "mlp_resident_pair_kernel", "test_mlp": "mlp_resident_kernel",
    "dlrm_bot": "mlp_stream_kernel", "nerf": "mlp_stream_kernel", "gc_edge": "mlp_stream_pair_kernel",
    "bert_ffn": "mlp_gemm_pair_kernel", "dlrm_top": "mlp_gemm_pair_kernel",
    "bert_addln": "mlp_stream_kernel", "dlrm_interact": "dlrm_interaction_kernel",
    "nerf_full": "mlp_stream_kernel (one fused chain: trunk, alpha side output, rgb branch)",
    "mgn_mp": "mlp_resident_pair_kernel (edge update: gather4 of node rows, segment sum) + mlp_resident_kernel (node update)",
}


def cpu_oracle_rate(w, seconds: float) -> dict:
    """The CPU oracle on whole 65,536-row chunks for about `seconds` (at least one chunk)."""
    from oracle import mlp_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    layers, ln = W.make_weights(w)
    x = W.make_input_chunk(w, 0)
    O.workload_forward(w, W.make_input(w, 0, 256), layers, ln)  # warm-up
    rows, t0 = 0, time.perf_counter()
    while True:
        O.workload_forward(w, x, layers, ln)
        rows += W.rows_of(w, x)
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": rows / dt, "unit": "rows/s", "cores": torch.get_num_threads(),
            "cpu_count": os.cpu_count(), "kind": "port",
            "sample": f"{rows} rows of {w.name} in {rows // W.CHUNK_ROWS} x 65,536-row chunks, "
                      f"fp32 PyTorch on the host ({dt:.1f} s)"}


def split_mode(args, world: int) -> str:
    return args.split or "strong"  # at N = 1 both modes run the config's M rows


def run_reference(args, w, rank: int):
    """Reference arm: the reference's PyTorch fp32 model (restated in oracle/) on the CPU."""
    if rank != 0:
        return
    from oracle import mlp_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    layers, ln = W.make_weights(w)
    # every step runs the config's full M rows (the same work as one step of the GPU arm) unless
    # that would take the whole run past about three minutes; then a bounded sample
    x_cal = W.make_input(w, 0, 4096)
    O.workload_forward(w, x_cal, layers, ln)
    t0 = time.perf_counter()
    O.workload_forward(w, x_cal, layers, ln)
    per_row = (time.perf_counter() - t0) / 4096
    budget = 180.0 / max(1, args.steps + args.warmup)
    rows = int(min(w.m, max(256, budget / max(per_row, 1e-9))))
    if rows < w.m:
        rows = max(256, rows // 256 * 256)  # whole tiles (and whole 16-edge node groups for mgn_mp)
    x = W.make_input(w, 0, rows)
    for _ in range(args.warmup):
        O.workload_forward(w, x, layers, ln)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.workload_forward(w, x, layers, ln)
    dt = time.perf_counter() - t0
    val = rows * args.steps / dt
    line = {
        "impl": "reference", "metric": "fused-MLP rows/s", "value": val, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": split_mode(args, args.gpus), "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w.name, "rows_per_step": rows, "global_rows": w.m,
                   "same_rows_as_gpu_arm": rows == w.m, "chain": w.widths,
                   "description": w.description},
        "tflops": val * w.flop_per_row / 1e12,
        "cpu_baseline": {"value": val, "unit": "rows/s", "cores": torch.get_num_threads(),
                         "cpu_count": os.cpu_count(), "kind": "port",
                         "sample": f"{rows} rows per step of {w.name} ({'all' if rows == w.m else 'a sample'} "
                                   f"of the config's {w.m}), PyTorch fp32 on the host"},
        "e2e": {"value": val, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    base = W.WORKLOADS[args.config]
    w = base.with_m(args.m) if args.m else base

    if args.impl == "reference":
        run_reference(args, w, rank)
        return

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
    from gpu_pipes_b200 import cuda_ext

    # ---- data. strong: the config's M rows in contiguous 256-row-aligned ranges, one per rank
    # (weights replicated); weak: rank r owns rows [r*M, (r+1)*M) of an N*M-row job
    split = split_mode(args, world)
    if split == "strong":
        row0, n_rows = W.shard_rows(w.m, world, rank, tile=256)
        rows_total = w.m
    else:
        row0, n_rows = rank * w.m, w.m
        rows_total = w.m * world
    x_host = W.make_input(w.with_m(row0 + n_rows), row0, n_rows).pin_memory()
    w = w.with_m(n_rows)
    layers, ln = W.make_weights(w)
    x = x_host.to(dev)
    wd = [(a.to(dev), b.to(dev)) for a, b in layers]
    lnd = None if ln is None else tuple(t.to(dev) for t in ln)
    out = torch.empty(w.m, w.n_out, dtype=w.dtype, device=dev)
    stream = torch.cuda.current_stream(dev)

    # Inputs + outputs smaller than twice the L2 would be served from L2 on the next step. Such
    # workloads rotate over R copies of x and out (R * (x + out) >= 4 x 126 MB), so a step's rows
    # were last touched R - 1 steps earlier, with at least three L2 capacities of other traffic
    # in between, and come from HBM; the steps then run back to back like the large workloads.
    # `--flush` times them one by one around a 256 MB L2-flushing write instead.
    io_bytes = w.m * w.bytes_per_row
    small = io_bytes < 2 * L2_BYTES
    flush = small and args.flush
    n_rot = 1
    if small and not flush:
        n_rot = int(min(256, max(2, -(-4 * L2_BYTES // max(io_bytes, 1)))))
    xs = [x] + [x.clone() for _ in range(n_rot - 1)]
    outs = [out] + [torch.empty_like(out) for _ in range(n_rot - 1)]
    it = [0]

    def step():
        i = it[0] % n_rot
        it[0] += 1
        cuda_ext.run_workload_out(w, xs[i], wd, lnd, outs[i])

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    graph = None
    graph_launches = 0
    if not args.no_graph:
        # One captured step per input copy, after the warm-up (the workspaces are at size, so the
        # capture allocates nothing). A replay enqueues the step's kernels with no host work, so
        # a small step (MGN node on one of 8 GPUs: ~23 us) is not bounded by the ~19 us of host
        # time per library call. The library path itself is what `e2e` measures.
        graphs = []
        n0 = L.launch_count()
        for _ in range(n_rot):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            graphs.append(g)
        graph_launches = (L.launch_count() - n0) / n_rot
        # and all n_rot steps in one graph, so consecutive small steps also skip the per-graph
        # launch; the per-copy graphs cover a remainder of fewer than n_rot steps
        whole = None
        if n_rot > 1:
            whole = torch.cuda.CUDAGraph()
            with torch.cuda.graph(whole):
                for _ in range(n_rot):
                    step()
        torch.cuda.synchronize()
        graph = graphs[0]

        def run_steps(k):
            done = 0
            if whole is not None:
                while k - done >= n_rot:
                    whole.replay()
                    done += n_rot
            for i in range(k - done):
                graphs[i % n_rot].replay()

        git = [0]

        def step():  # noqa: F811
            graphs[git[0] % n_rot].replay()
            git[0] += 1

        for _ in range(max(3, n_rot)):
            step()
        torch.cuda.synchronize()

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    flush_buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if flush else None

    sampler = ClockSampler(local)
    if not args.kernel_only:
        sampler.start()
        time.sleep(0.25)
    launches0 = L.launch_count()
    barrier()
    if flush:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for e0, e1 in evs:
            flush_buf.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        barrier()
        ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    else:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        if graph is not None:
            run_steps(args.steps)
        else:
            for _ in range(args.steps):
                step()
        ev1.record(stream)
        barrier()
        ms = ev0.elapsed_time(ev1)
    launches = L.launch_count() - launches0
    if graph is not None:  # replays enqueue the captured kernels without calling the library
        launches = int(round(graph_launches * args.steps))
    clocks = sampler.stop() if not args.kernel_only else None
    if dist is not None:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    value = rows_total / (ms_step / 1e3)

    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"workload": w.name, "rows_per_gpu": w.m, "ms_per_step": ms_step,
                              "rows_per_s": value, "gpu_launches": launches}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return

    # ---- end to end through the public API: pinned host x -> device -> kernel -> host out
    out_host = torch.empty(w.m, w.n_out, dtype=w.dtype).pin_memory()
    x_dev2 = torch.empty_like(x)

    def e2e_step():
        if not w.block:
            # plain chains: the pipelined host-buffer entry point (chunked H2D / kernel / D2H on
            # three streams)
            cuda_ext.run_workload_host(w, x_host, wd, lnd, out_host)
            return
        x_dev2.copy_(x_host, non_blocking=True)
        cuda_ext.run_workload_out(w, x_dev2, wd, lnd, out)
        out_host.copy_(out, non_blocking=True)

    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_value = rows_total / (e_ms / args.e2e_steps / 1e3)

    status = L.device_status(local)
    hbm_gbs, tflops_peak, tflops_sus, peak_src = measured_peaks()
    alg_bytes = w.m * w.bytes_per_row  # per launch
    alg_flops = w.m * w.flop_per_row   # per launch
    tr = NCU_TRAFFIC_PER_ROW.get(w.name)
    if w.bound == "hbm":
        achieved, peak, unit = alg_bytes / (ms_step / 1e3) / 1e9, hbm_gbs, "GB/s"
        peak_note = f"{peak_src} hbm_gbs"
    else:
        long_run = ms > 1000.0
        achieved = alg_flops / (ms_step / 1e3) / 1e12
        peak, unit = (tflops_sus if long_run else tflops_peak), "TFLOP/s"
        peak_note = f"{peak_src} bf16_tflops" + ("_sustained (timed region > 1 s)" if long_run else " (burst)")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_oracle_rate(w, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": "fused-MLP rows/s", "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": split, "vs_baseline": None,
            "dtype": "f16" if w.dtype == torch.float16 else "bf16", "data": "synthetic",
            "config": {"workload": w.name, "rows_per_gpu": w.m, "global_rows": rows_total,
                       "chain": w.widths, "tail": ["none", "layernorm", "residual+layernorm"][w.tail],
                       "description": w.description,
                       "l2": ("L2 flushed (256 MB write) between timed steps: x %d MB + out %d MB "
                              "per GPU < 2 x 126 MB" % (w.m * w.in_width * 2 >> 20, w.m * w.n_out * 2 >> 20)
                              if flush else
                              "steps rotate over %d copies of x and out (x %d MB + out %d MB per GPU "
                              "each; >= 4 x 126 MB in all), so every step reads its rows from HBM" % (
                                  n_rot, w.m * w.in_width * 2 >> 20, w.m * w.n_out * 2 >> 20)
                              if n_rot > 1 else
                              "inputs larger than L2 (x %d MB + out %d MB per GPU)" % (
                                  w.m * w.in_width * 2 >> 20, w.m * w.n_out * 2 >> 20)),
                       "parallelism": f"rows sharded over {world} GPU(s), weights replicated",
                       "launch": "CUDA graph replays of the captured steps" if graph is not None
                                 else "library calls per step"},
            "tflops": value * w.flop_per_row / 1e12,
            "roofline": {"bound": w.bound, "achieved": achieved, "peak": peak, "unit": unit,
                         "frac": achieved / peak,
                         "traffic": None if tr is None else tr * w.m,
                         "traffic_source": None if tr is None else
                             "constant per row from an ncu capture of this kernel (not measured by this run)",
                         "peak_source": f"{peak_note} (MEASURED_PEAKS.json)",
                         "kernel": KERNEL_OF.get(w.name, "mlp_stream_kernel"),
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "algorithmic_flops_per_launch": alg_flops},
            "e2e": {"value": e2e_value, "unit": "rows/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "gpu_launches": launches,
            "clocks": clocks,
            "device_status": status,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

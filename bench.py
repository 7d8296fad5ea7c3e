"""Throughput of the hot path on B200s — one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 2): the batched decision forward of a ModernBERT-base encoder + Laya decision
head with every projection in Q8_0, 64 questions × 512 tokens per GPU (synthetic, seeded; laya_b200/workloads.py).
A step is one forward over one such batch.  Inference shards by request: each rank runs its own batch with no
collective on the data path (weak scaling); torch.distributed only brackets the timed region and takes the max of
the per-rank times.

`value` is device-resident throughput (inputs already in HBM, laya_decision_forward_device); `e2e` is the same
through the host-pointer C ABI (laya_decision_forward), host↔device copies of each step's inputs and outputs inside
the timed region.  `--impl reference` times the CPU restatement of the reference's path (oracle/) on the host cores.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS, SEQ = 64, 512
TOKENS = ROWS * SEQ
WORKLOAD = "config2_q8_0_decision_forward"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample-rows", type=int, default=1, help="rows of 512 tokens in one CPU step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def config_block(world):
    return {"workload": WORKLOAD, "rows_per_gpu": ROWS, "seq_len": SEQ, "tokens_per_gpu_step": TOKENS,
            "geometry": "ModernBERT-base 22x768 (12x64, GeGLU 1152) + 2 head layers", "weights": "Q8_0 (config 2)",
            "l2": "inputs larger than L2 (Q8_0 weights ~150 MB + 0.5 GB activations per step)",
            "parallelism": f"request-sharded x{world}, no collective"}


# --------------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([v.strip() for v in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm = [float(s[1]) for s in self.samples if len(s) >= 9 and s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if len(s) >= 9 and s[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            if len(s) >= 9:
                for n, v in zip(names, s[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------------------------------- CPU arms
def oracle_step_seconds(rows, seed=1):
    """One bounded CPU sample: the oracle's Q8_0 decision forward over `rows` × 512 tokens of the same workload."""
    import numpy as np
    import oracle
    from laya_b200 import workloads
    from oracle.model import EncoderConfig, Item, OracleModel
    oracle.build()
    w, q8 = workloads.decision_weights(seed=0)
    om = OracleModel(EncoderConfig(), w, workloads.dequantized(q8))
    items = workloads.decision_batch(rows=rows, length=SEQ, seed=seed)
    its = [Item(np.asarray(it.token_ids), list(it.marker_positions), it.type) for it in items]
    t0 = time.perf_counter()
    om.forward(its)
    return time.perf_counter() - t0, oracle.lib().lo_num_threads()


def cpu_baseline(rows):
    secs, cores = oracle_step_seconds(rows)
    return {"value": rows * SEQ / secs, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{rows} x {SEQ} tokens, one full 22-layer Q8_0 decision forward ({secs:.1f} s)"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    rows = args.cpu_sample_rows
    times = []
    cores = None
    for i in range(args.warmup + args.steps):
        s, cores = oracle_step_seconds(rows, seed=1 + i)
        if i >= args.warmup:
            times.append(s)
    per = statistics.mean(times)
    value = rows * SEQ / per
    line = {"impl": "reference", "metric": "Q8_0 encode tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1000,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config_block(world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"{rows} x {SEQ} tokens per step, CPU restatement of the reference path"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------------- GPU arm
def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def load_traffic():
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    import laya_b200
    from laya_b200 import workloads

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))

    w, q8 = workloads.decision_weights(seed=0)                    # the same weights on every rank
    model = laya_b200.DecisionModel(laya_b200.base_desc(max_tokens=TOKENS, max_items=ROWS, max_markers=ROWS * 8),
                                    w, q8, device=local)
    del w, q8
    items = workloads.decision_batch(rows=ROWS, length=SEQ, seed=1 + rank)
    ids, seg_len, qtype, counts, markers = model.pack(items)
    n_mark = int(counts.sum())
    stream = torch.cuda.Stream()
    model.ctx.set_stream(stream.cuda_stream)
    dev = [torch.from_numpy(v).cuda() for v in (ids, seg_len, qtype, counts, markers)]
    logits = torch.zeros(n_mark, dtype=torch.float32, device="cuda")
    act = torch.zeros(ROWS * 2, dtype=torch.float32, device="cuda")
    L = laya_b200.lib()

    def step_device():
        laya_b200.api.check(L.laya_decision_forward_device(
            model.ctx.handle, dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), ROWS, int(ids.size),
            dev[3].data_ptr(), dev[4].data_ptr(), n_mark, logits.data_ptr(), act.data_ptr()))

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step_device()
    model.ctx.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- timed region: device-resident
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    launches0 = model.ctx.launches()
    model.ctx.set_profiling(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            step_device()
        e1.record(stream)
    e1.synchronize()
    launches = model.ctx.launches() - launches0
    gemm_ms, gemm_ops, gemm_n = model.ctx.profile()
    model.ctx.set_profiling(False)
    model.ctx.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps

    # ---- timed region: end to end through the host-pointer C ABI (pinned host buffers)
    pin = [torch.from_numpy(v).pin_memory() for v in (ids, seg_len, qtype, counts, markers)]
    host_logits = torch.zeros(n_mark, dtype=torch.float32).pin_memory()
    host_act = torch.zeros(ROWS * 2, dtype=torch.float32).pin_memory()

    def step_host():
        laya_b200.api.check(L.laya_decision_forward(
            model.ctx.handle, pin[0].data_ptr(), pin[1].data_ptr(), pin[2].data_ptr(), ROWS, pin[3].data_ptr(),
            pin[4].data_ptr(), host_logits.data_ptr(), host_act.data_ptr()))

    for _ in range(max(1, args.warmup // 2)):
        step_host()
    barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for _ in range(args.steps):
        step_host()
    h1.record(stream)
    h1.synchronize()
    barrier()
    e2e_ms = h0.elapsed_time(h1) / args.steps
    h2d = sum(int(v.nbytes) for v in (ids, seg_len, qtype, counts, markers))
    d2h = n_mark * 4 + ROWS * 2 * 4

    # max over ranks
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = float(t[0]), float(t[1])

    if rank == 0:
        peaks, source = load_peaks()
        bf16 = peaks.get("bf16_tflops", 1590.0)
        i8_peak = 2.0 * bf16          # int8 dense rate is twice bf16 on B200; measured bf16 × 2
        achieved = gemm_ops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
        traffic = load_traffic().get("q8_gemm", {}).get("dram_bytes_per_launch")
        line = {
            "metric": "Q8_0 encode tokens/s", "value": world * TOKENS / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config_block(world),
            "e2e": {"value": world * TOKENS / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "roofline": {"kernel": "q8_gemm_kernel (Q8_0 tcgen05 kind::i8 product + per-block rescale)",
                         "bound": "tensor", "achieved": achieved, "peak": i8_peak, "unit": "TOP/s",
                         "frac": achieved / i8_peak, "peak_source": f"2 x {source} bf16 burst ({bf16} TFLOP/s)",
                         "traffic": traffic, "launches": gemm_n,
                         "share_of_step": (gemm_ms / gemm_n) * (gemm_n / args.steps) / ms if gemm_n else None},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_sample_rows)
        print(json.dumps(line), flush=True)
    model.ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

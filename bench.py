"""Throughput of the hot path on B200s — one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload all|train|q8|f32|decoder]

Headline workload (config 3, the data-parallel fine-tune): per GPU 32 ModernBERT-base rows with valid lengths
U{256..1024} (padding is not work: rows are concatenated), the Laya decision head, the RLCD objective with 4 noise
groups, a global-norm clip and AdamW over fp32 masters — one step = forward + objective + backward + clip + AdamW +
zero-grad (laya_b200/workloads.py, seeded, data seed 1000 + rank).  Products are bf16 tensor-core tiles; the default
forward is the accurate one (bf16 hi/lo products, fp32-accurate activations: the parity-checked path).  With N GPUs
every rank trains its own rows and the gradients are summed over NCCL in 25 MB buckets while the backward runs
(weak scaling); torch.distributed only exchanges the NCCL id, brackets the timed region and takes the max of the
per-rank times.

Nested `q8_0_encode` (config 2): the batched decision forward with every projection in Q8_0, 64 rows × 512 tokens per
GPU, sharded by request with no collective.

Nested `mica_prefill` (config 5): the Mica hybrid decoder (32 Qwen3.5 layers, [DeltaNet ×3, full] ×8, h 2560) with
every projection and the tied token table in Q8_0, a prefill of 8 rows × 2048 token ids per GPU and the logits of 26
label ids at each row's last position; replicas sharded by request with no collective.  Beside it,
`mica_shared_prefix`: the same prompts served as one multi-question request whose shared prefix is read once into a
decoder state and cloned per question (MicaJudge.Predict), the effective prompt tokens/s.

Nested `systemone_f32`: the decision forward's fp32-accurate path (the reference's PackedMatrix products, here split
bf16 products) on a bf16 checkpoint of ModernBERT-large geometry, config 2's 64 × 512 batch.

`value` is device-resident throughput (inputs staged in HBM before the timed region); `e2e` is the same step through
the host-pointer C ABI with the step's inputs copied from pinned host memory and its result (the loss; the logits)
read back inside the timed region.  `--impl reference` times the CPU restatement of the reference's path (oracle/)
on the host cores.
"""
import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# config 3 (fine-tune)
TR_ROWS, TR_MIN, TR_MAX, TR_GROUPS = 32, 256, 1024, 4   # rows per GPU: --train-rows
TR_WORKLOAD = "config3_dp_finetune_step"
# config 2 (Q8_0 encode)
ROWS, SEQ = 64, 512
TOKENS = ROWS * SEQ
Q8_WORKLOAD = "config2_q8_0_decision_forward"
# config 5 (Mica decoder prefill)
DEC_ROWS, DEC_LEN, DEC_LABELS = 8, 2048, 26
DEC_TOKENS = DEC_ROWS * DEC_LEN
DEC_SHARED = 1792   # prompt tokens the questions of one Mica request share (the shared-prefix nested line)
DEC_WORKLOAD = "config5_mica_hybrid_decoder_prefill"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="all", choices=["all", "train", "q8", "f32", "decoder"])
    ap.add_argument("--dec-tokens", type=int, default=128, help="tokens of the decoder's CPU sample")
    ap.add_argument("--dec-layers", type=int, default=32, help="decoder layers (fewer only for small captures)")
    ap.add_argument("--delta-rule", default="chunked", choices=["chunked", "per-token"],
                    help="decoder prefill: the delta rule in 64-token tensor-core chunks (default) or the per-token "
                         "sweep in the reference's floating-point order")
    ap.add_argument("--forward", default="accurate", choices=["accurate", "bf16"],
                    help="forward mode of the headline training step")
    ap.add_argument("--no-bf16-forward", action="store_true", help="skip the extra BF16-forward measurement")
    ap.add_argument("--cpu-sample-rows", type=int, default=1, help="rows of 512 tokens in one Q8_0 CPU step")
    ap.add_argument("--cpu-train-tokens", type=int, default=256, help="tokens of the CPU fine-tune sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config4", action="store_true",
                    help="skip the nested config-4 (ModernBERT-large, 4 x 8192 tokens) measurement of the default run")
    ap.add_argument("--train-config", type=int, default=3, choices=[3, 4],
                    help="3: ModernBERT-base, 32 rows x U{256..1024}; 4: ModernBERT-large, 4 rows x 8192 tokens")
    ap.add_argument("--train-rows", type=int, default=None, help="rows per GPU of the fine-tune step")
    ap.add_argument("--train-layers", type=int, default=None, help="encoder layers (fewer only for small captures)")
    ap.add_argument("--kernel", choices=["q8_gemm", "bf16_gemm", "mma_peak"],
                    help="time one product alone at the workload's shapes (profiling captures), not the step")
    ap.add_argument("--case", default="wqkv",
                    help="q8_gemm: wqkv|wo|wi|mlp_wo; bf16_gemm: fwd_split|dx|dw (the Wqkv projection, 20480 tokens)")
    ap.add_argument("--reps", type=int, default=20)
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# fine-tune geometries: (hidden, intermediate, layers, heads, rows per GPU, min length, max length)
TRAIN_CONFIGS = {3: (768, 1152, 22, 12, TR_ROWS, TR_MIN, TR_MAX), 4: (1024, 2624, 28, 16, 4, 8192, 8192)}
GEOMETRY = {3: "ModernBERT-base 22x768 (12x64, GeGLU 1152, local 128 / global every 3rd) + 2 head layers",
            4: "ModernBERT-large 28x1024 (16x64, GeGLU 2624, local 128 / global every 3rd) + 2 head layers"}


def train_shape(args):
    H, I, layers, heads, rows, lo, hi = TRAIN_CONFIGS[args.train_config]
    return (H, I, args.train_layers or layers, heads, args.train_rows or rows, lo, hi)


def train_config(world, tokens, forward, rows=TR_ROWS, which=3, lens=(TR_MIN, TR_MAX)):
    return {"workload": TR_WORKLOAD if which == 3 else "config4_large_long_context_finetune_step", "rows_per_gpu": rows,
            "valid_len": f"U{{{lens[0]}..{lens[1]}}}" if lens[0] != lens[1] else str(lens[0]),
            "tokens_per_gpu_step": tokens,
            "geometry": GEOMETRY[which],
            "optimizer": "RLCD (4 groups) + clip 1.0 + AdamW, fp32 masters, bf16 products",
            "forward": forward, "l2": "inputs larger than L2 (0.66 GB fp32 parameters + ~30 GB tape per step)",
            "parallelism": f"dp{world}, NCCL allreduce in 25 MB buckets overlapped with the backward" if world > 1
            else "dp1"}


def q8_config(world):
    return {"workload": Q8_WORKLOAD, "rows_per_gpu": ROWS, "seq_len": SEQ, "tokens_per_gpu_step": TOKENS,
            "geometry": "ModernBERT-base 22x768 (12x64, GeGLU 1152) + 2 head layers", "weights": "Q8_0 (config 2)",
            "l2": "inputs larger than L2 (Q8_0 weights ~150 MB + 0.5 GB activations per step)",
            "parallelism": f"request-sharded x{world}, no collective"}


def dec_config(world, layers=32):
    return {"workload": DEC_WORKLOAD, "rows_per_gpu": DEC_ROWS, "seq_len": DEC_LEN, "tokens_per_gpu_step": DEC_TOKENS,
            "geometry": f"Qwen3.5 hybrid {layers} layers ([DeltaNet x3, full] blocks), h 2560, I 9216, vocab 151936, "
                        "DeltaNet 16x128 k/v heads, attention 16q/4kv x128, quarter RoPE theta 1e7",
            "labels": DEC_LABELS, "weights": "Q8_0 projections + tied Q8_0 token table (config 5)",
            "l2": "inputs larger than L2 (6.9 GB of fp16-held weight codes and ~2 GB of activations per step)",
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
def cpu_products():
    """Switch the oracle's products to the AVX-512 restatements of the reference's panel kernels when this CPU has
    them (same bits as the scalar definitions); returns the phrase the baseline's `sample` carries."""
    import oracle
    oracle.build()
    if oracle.set_fast(True):
        return "products by AVX-512 restatements of PackedMatrixQ8_0.Panel512 (VNNI) and PackedMatrix's panel kernel"
    return "products by the scalar restatement (this CPU has no AVX-512 VNNI)"


def q8_cpu_seconds(rows, seed=1):
    """One bounded CPU sample: the oracle's Q8_0 decision forward over `rows` × 512 tokens of the same workload."""
    import numpy as np
    import oracle
    from laya_b200 import workloads
    from oracle.model import EncoderConfig, Item, OracleModel
    cpu_products()
    w, q8 = workloads.decision_weights(seed=0)
    om = OracleModel(EncoderConfig(), w, workloads.dequantized(q8))
    items = workloads.decision_batch(rows=rows, length=SEQ, seed=seed)
    its = [Item(np.asarray(it.token_ids), list(it.marker_positions), it.type) for it in items]
    t0 = time.perf_counter()
    om.forward(its)
    return time.perf_counter() - t0, oracle.lib().lo_num_threads()


def q8_cpu_baseline(rows):
    secs, cores = q8_cpu_seconds(rows)
    return {"value": rows * SEQ / secs, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{rows} x {SEQ} tokens, one full 22-layer Q8_0 decision forward ({secs:.1f} s); {cpu_products()}"}


def f32_cpu_seconds(tokens, seed=1):
    """One bounded CPU sample of the fp32 decision forward: the oracle's fp32 restatement (PackedMatrix products)
    over one row of `tokens` tokens of the ModernBERT-large bf16 checkpoint."""
    import numpy as np
    import oracle
    from laya_b200 import workloads
    from oracle.model import EncoderConfig, Item, OracleModel
    cpu_products()
    w = workloads.bf16_checkpoint_weights(**LARGE, seed=0)
    om = OracleModel(EncoderConfig(**LARGE), w)
    items = workloads.decision_batch(rows=1, length=tokens, seed=seed)
    its = [Item(np.asarray(it.token_ids), list(it.marker_positions), it.type) for it in items]
    t0 = time.perf_counter()
    om.forward(its)
    return time.perf_counter() - t0, oracle.lib().lo_num_threads()


F32_CPU_TOKENS = 512


def f32_cpu_baseline(tokens=F32_CPU_TOKENS):
    secs, cores = f32_cpu_seconds(tokens)
    return {"value": tokens / secs, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"1 x {tokens} tokens, one full 28-layer fp32 decision forward ({secs:.1f} s); {cpu_products()}"}


def dec_cpu_baseline(tokens, reps=1):
    """A bounded CPU sample of config 5: the oracle's Q8_0 restatement of Qwen35Model.Forward over one row of `tokens`
    ids through one [DeltaNet x3, full] block of the workload's weights, scaled to the 32-layer model (x8)."""
    import numpy as np
    import oracle
    from laya_b200 import workloads
    from oracle.decoder import DecoderConfig, OracleDecoder, mica_config
    products = cpu_products()
    kinds = workloads.MICA_KINDS[:4]
    q8, vec = workloads.decoder_q8_weights(kinds, seed=0)
    base = mica_config()
    cfg = DecoderConfig(**{**base.__dict__, "layers": 4, "kinds": kinds})
    stacks = {}
    for i, k in enumerate(kinds):
        p = f"layers.{i}."
        groups = [[p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"], [p + "mlp.down_proj.weight"]]
        if k == "full":
            a = p + "self_attn."
            groups += [[a + "q_proj.weight", a + "k_proj.weight", a + "v_proj.weight"], [a + "o_proj.weight"]]
        else:
            a = p + "linear_attn."
            groups += [[a + n + ".weight" for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")],
                       [a + "out_proj.weight"]]
        for g in groups:
            stacks["|".join(g)] = (np.concatenate([q8["model." + n][0] for n in g], 0),
                                   np.concatenate([q8["model." + n][1] for n in g], 0).astype(np.float32))
    qe, de = q8["model.embed_tokens.weight"]
    stacks["embed"] = (qe, de.astype(np.float32))
    om = OracleDecoder(cfg, vec, precision="q8_0", q8=stacks)
    seqs, labels = workloads.decoder_batch(rows=1, length=tokens, seed=5)
    times = []
    for _ in range(reps + 1):
        t0 = time.perf_counter()
        _, last = om.forward(seqs[0], record=False)
        om.logits(last, labels)
        times.append(time.perf_counter() - t0)
    secs = statistics.mean(times[1:]) * 8.0
    return {"value": tokens / secs, "unit": "tokens/s", "cores": oracle.lib().lo_num_threads(), "kind": "port",
            "sample": f"1 row x {tokens} tokens through one [DeltaNet x3, full] block of the config-5 Q8_0 weights "
                      f"({secs / 8:.2f} s), scaled x8 to the 32-layer model, plus the 26 label logits; CPU "
                      f"restatement of the reference's Qwen35Model Q8_0 forward, {products}"}


class CpuTrainStep:
    """A bounded CPU sample of the fine-tune step: the oracle's fp32 restatement of TrainableDecisionModel (PyTorch
    autograd on the host cores) over one row of the workload, the RLCD objective and AdamW over every parameter."""

    def __init__(self, tokens):
        import numpy as np
        import torch
        from laya_b200 import workloads
        from oracle.model import EncoderConfig
        from oracle.train import TorchTrainModel
        torch.set_num_threads(os.cpu_count() or 1)
        self.cores = torch.get_num_threads()
        self.tokens = tokens
        self.w = workloads.training_weights(seed=0)
        self.model = TorchTrainModel(EncoderConfig(), self.w)
        self.state = {k: (np.zeros(v.size, np.float32), np.zeros(v.size, np.float32)) for k, v in self.w.items()
                      if k != "temperature"}
        self.steps = 0

    def run(self, seed):
        """(seconds of forward + objective + backward over one row, seconds of clip + AdamW over every parameter)."""
        import torch
        from laya_b200 import workloads
        from oracle.train import adamw_step, clip_by_global_norm, rlcd
        items, draws = workloads.training_batch(rows=1, min_len=self.tokens, max_len=self.tokens, seed=seed,
                                                groups=TR_GROUPS)
        oi = [{"ids": it.token_ids, "markers": list(it.marker_positions), "qtype": it.question_type} for it in items]
        t0 = time.perf_counter()
        self.model.zero_grad()
        logits = self.model.forward(oi, training=True, seed=seed)
        k = items[0].options
        _, _, _, _, grads = rlcd([l.detach().numpy() for l in logits], [it.target for it in items],
                                 [it.question_type for it in items], 0.4, [[draws[g, :k]] for g in range(TR_GROUPS)])
        sum((l * torch.from_numpy(g)).sum() for l, g in zip(logits, grads)).backward()
        g = self.model.grads()
        t1 = time.perf_counter()
        clip_by_global_norm(list(g.values()), 1.0)
        self.steps += 1
        for name, p in self.model.p.items():
            data = p.detach().numpy().reshape(-1)
            m, v = self.state[name]
            adamw_step(data, g[name].reshape(-1), m, v, self.steps, 2.5e-5 if name.startswith("encoder.") else 1e-4)
        return t1 - t0, time.perf_counter() - t1

    def rate(self, fb, opt):
        """tokens/s with the optimizer amortised as the workload runs it: one clip + AdamW per step of
        TR_ROWS rows (mean valid length (TR_MIN + TR_MAX) / 2)."""
        step_tokens = TR_ROWS * (TR_MIN + TR_MAX) / 2
        return self.tokens / (fb + opt * self.tokens / step_tokens)

    def sample(self, fb, opt):
        return (f"1 row x {self.tokens} tokens: fp32 forward + RLCD + backward ({fb:.2f} s), plus clip + AdamW over "
                f"all {sum(v.size for v in self.w.values()) / 1e6:.0f}M parameters ({opt:.2f} s) amortised over a "
                f"{TR_ROWS}-row step's {TR_ROWS * (TR_MIN + TR_MAX) // 2} tokens; CPU restatement (PyTorch autograd, "
                f"numpy AdamW) of the reference's Laya.Training path")


def train_cpu_baseline(tokens):
    c = CpuTrainStep(tokens)
    c.run(0)   # warm-up
    fb, opt = c.run(1)
    return {"value": c.rate(fb, opt), "unit": "tokens/s", "cores": c.cores, "kind": "port", "sample": c.sample(fb, opt)}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    if args.workload == "q8":
        rows = args.cpu_sample_rows
        times, cores = [], None
        for i in range(args.warmup + args.steps):
            s, cores = q8_cpu_seconds(rows, seed=1 + i)
            if i >= args.warmup:
                times.append(s)
        per = statistics.mean(times)
        value = rows * SEQ / per
        line = {"impl": "reference", "metric": "Q8_0 encode tokens/s", "value": value, "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1000,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic", "config": q8_config(world),
                "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                                 "sample": f"{rows} x {SEQ} tokens per step, CPU restatement of the reference path; "
                                           f"{cpu_products()}"},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.workload == "f32":
        b = f32_cpu_baseline()
        line = {"impl": "reference", "metric": "decision forward tokens/s, fp32-accurate path on a bf16 checkpoint",
                "value": b["value"], "unit": "tokens/s", "n_gpus": world, "steps": 1, "warmup": 0,
                "ms_per_step": F32_CPU_TOKENS / b["value"] * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "systemone_f32_modernbert_large", "rows_per_gpu": ROWS, "seq_len": SEQ},
                "cpu_baseline": b,
                "e2e": {"value": b["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    if args.workload == "decoder":
        vals = [dec_cpu_baseline(args.dec_tokens) for _ in range(max(1, args.steps // 5))]
        b = vals[-1]
        value = statistics.mean(v["value"] for v in vals)
        line = {"impl": "reference", "metric": "Mica prefill tokens/s", "value": value, "unit": "tokens/s",
                "n_gpus": world, "steps": len(vals), "warmup": 1, "ms_per_step": DEC_TOKENS / value * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic", "config": dec_config(world),
                "cpu_baseline": {**b, "value": value},
                "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    c = CpuTrainStep(args.cpu_train_tokens)
    fbs, opts = [], []
    for i in range(args.warmup + args.steps):
        fb, opt = c.run(i)
        if i >= args.warmup:
            fbs.append(fb)
            opts.append(opt)
    fb, opt = statistics.mean(fbs), statistics.mean(opts)
    value = c.rate(fb, opt)
    line = {"impl": "reference", "metric": "fine-tune tokens/s (fwd+bwd+AdamW)", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": args.cpu_train_tokens / value * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": train_config(world, args.cpu_train_tokens, "fp32 (CPU restatement)"),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": c.cores, "kind": "port",
                             "sample": c.sample(fb, opt)},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "all" and not args.no_cpu_baseline:
        line["q8_0_encode"] = {"metric": "Q8_0 encode tokens/s", **q8_cpu_baseline(args.cpu_sample_rows)}
        line["mica_prefill"] = {"metric": "Mica prefill tokens/s", **dec_cpu_baseline(args.dec_tokens)}
        line["systemone_f32"] = {"metric": "decision forward tokens/s, fp32-accurate path on a bf16 checkpoint",
                                 **f32_cpu_baseline()}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------------------------------- GPU arm
def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def measured_i8_peak():
    """The int8 tensor rate of this device, measured now (laya_mma_peak, kind::i8, M 128 x N 256): TOP/s."""
    import ctypes
    import torch
    import laya_b200
    L = laya_b200.lib()
    nsm = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    reps = 20000
    ms, cyc = ctypes.c_double(), ctypes.c_double()
    laya_b200.api.check(L.laya_mma_peak(2, 256, reps, ctypes.byref(ms), ctypes.byref(cyc)))
    return nsm * reps * 4 * 2.0 * 128 * 256 * 32 / (ms.value / 1e3) / 1e12


I8_SOURCE = "measured int8 tensor rate of this device in this run (laya_mma_peak kind::i8, M128 N256)"


def load_traffic():
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


class Dist:
    def __init__(self, rank, world, local):
        import torch
        import torch.distributed as dist
        self.rank, self.world, self.local = rank, world, local
        self.dist = dist if world > 1 else None
        self.torch = torch
        torch.cuda.set_device(local)
        if world > 1:
            dist.init_process_group("nccl", init_method="env://", device_id=torch.device("cuda", local),
                                    timeout=datetime.timedelta(seconds=180))

    def barrier(self):
        if self.dist:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def reduce(self, values, op):
        t = self.torch.tensor(values, dtype=self.torch.float64, device="cuda")
        if self.dist:
            self.dist.all_reduce(t, op=op(self.dist))
        return [float(v) for v in t]

    def broadcast_bytes(self, b):
        if not self.dist:
            return b
        obj = [b]
        self.dist.broadcast_object_list(obj, src=0)
        return obj[0]


def train_measure(args, d, forward_mode, with_e2e=True, with_profile=True):
    """Times the fine-tune step on this rank; returns a dict of per-rank measurements (rank 0 formats the line)."""
    import numpy as np
    import torch
    import laya_b200
    from laya_b200 import workloads
    from laya_b200.workloads import mix
    rank, world, local = d.rank, d.world, d.local
    H, I, layers, heads, rows, lo, hi = train_shape(args)
    w = workloads.training_weights(hidden=H, intermediate=I, layers=layers, seed=0)   # the same weights on every rank
    tr = laya_b200.Trainer(laya_b200.base_desc(hidden=H, intermediate=I, heads=heads, layers=layers,
                                               max_tokens=rows * hi, max_items=rows, max_markers=rows * 8),
                           laya_b200.train_desc(max_segment=hi, forward_mode=forward_mode), device=local)
    if world > 1:
        uid = d.broadcast_bytes(laya_b200.Trainer.unique_id() if rank == 0 else None)
        tr.comm_init(uid, rank, world)
    stream = torch.cuda.Stream()
    tr.set_stream(stream.cuda_stream)
    tr.load(w)
    del w
    # two batches per rank staged on the device before the timed region (data seed 1000 + rank)
    sets = [workloads.training_batch(rows=rows, min_len=lo, max_len=hi, seed=1000 + rank + 64 * i,
                                     groups=TR_GROUPS) for i in range(2)]
    batches = [tr.batch(items, draws) for items, draws in sets]
    tokens = [sum(len(it.token_ids) for it in items) for items, _ in sets]
    options = [sum(it.options for it in items) for items, _ in sets]

    def step(b, i):
        tr.forward(b, training=True, seed=mix(42, i + 1), fetch=False)
        tr.objective(b, sigma=0.4, groups=TR_GROUPS, fetch=False)
        tr.backward(b)
        tr.clip_and_step(1.0, fetch_norm=False)
        tr.zero_grads()

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(batches[i % 2], i)
    tr.synchronize()
    out = {}
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    d.barrier()
    n0 = tr.launches()
    if with_profile:
        tr.set_profiling(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    done_tokens = 0
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(args.steps):
            step(batches[i % 2], args.warmup + i)
            done_tokens += tokens[i % 2]
        e1.record(stream)
    e1.synchronize()
    out["launches"] = tr.launches() - n0
    if with_profile:
        out["prof"] = [tr.profile(k) for k in range(3)]
        tr.set_profiling(False)
    tr.synchronize()
    d.barrier()
    out["clocks"] = sampler.stop()
    out["ms"] = e0.elapsed_time(e1) / args.steps
    out["tokens"] = done_tokens
    out["tokens_per_step"] = done_tokens / args.steps

    if with_e2e:
        # end to end: each step's batch from pinned host memory (ids, segments, markers, targets, draws), the loss
        # read back (laya_train_objective with a host result synchronises the step)
        L = laya_b200.lib()
        host = []
        for items, draws in sets:
            ids = np.concatenate([np.asarray(it.token_ids, np.int64) for it in items]).astype(np.int32)
            arrs = [ids, np.array([len(it.token_ids) for it in items], np.int32),
                    np.array([it.question_type for it in items], np.int32),
                    np.array([it.options for it in items], np.int32),
                    np.concatenate([np.asarray(it.marker_positions, np.int32) for it in items]),
                    np.concatenate([it.target for it in items]).astype(np.float32),
                    np.ascontiguousarray(draws, np.float64)]
            host.append([torch.from_numpy(a).pin_memory() for a in arrs])
        h2d = [sum(int(a.nbytes) for a in hs) for hs in host]
        staged = laya_b200.Batch(tr)
        res = torch.zeros(4, dtype=torch.float64).pin_memory()
        rl = laya_b200.RlcdDesc(TR_GROUPS, 0.4, 1.0, 0.75, 1.0, 1.0)
        import ctypes

        def step_host(i):
            hs = host[i % 2]
            laya_b200.api.check(L.laya_batch_set(tr.handle, staged.handle, hs[0].data_ptr(), hs[1].data_ptr(),
                                                 hs[2].data_ptr(), rows, hs[3].data_ptr(), hs[4].data_ptr(),
                                                 hs[5].data_ptr(), hs[6].data_ptr(), TR_GROUPS))
            laya_b200.api.check(L.laya_train_forward(tr.handle, staged.handle, 1, ctypes.c_uint64(mix(42, i + 1)),
                                                     None))
            laya_b200.api.check(L.laya_train_objective(tr.handle, staged.handle, ctypes.byref(rl), res.data_ptr(),
                                                       None))
            laya_b200.api.check(L.laya_train_backward(tr.handle, staged.handle, None))
            laya_b200.api.check(L.laya_train_clip_and_step(tr.handle, ctypes.c_double(1.0), None))
            laya_b200.api.check(L.laya_train_zero_grads(tr.handle))

        for i in range(max(1, args.warmup // 2)):
            step_host(i)
        tr.synchronize()
        d.barrier()
        h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for i in range(args.steps):
            step_host(i)
        h1.record(stream)
        h1.synchronize()
        d.barrier()
        out["e2e_ms"] = h0.elapsed_time(h1) / args.steps
        out["h2d"] = sum(h2d[i % 2] for i in range(args.steps)) / args.steps
        out["d2h"] = 4 * 8
        out["loss"] = float(res[0])
        staged.close()
    for b in batches:
        b.close()
    tr.synchronize()
    tr.close()
    return out


def q8_measure(args, d):
    import numpy as np
    import torch
    import laya_b200
    from laya_b200 import workloads
    rank, world, local = d.rank, d.world, d.local
    w, q8 = workloads.decision_weights(seed=0)                    # the same weights on every rank
    model = laya_b200.DecisionModel(laya_b200.base_desc(max_tokens=TOKENS, max_items=ROWS, max_markers=ROWS * 8),
                                    w, q8, device=local)
    del w, q8
    items = workloads.decision_batch(rows=ROWS, length=SEQ, seed=1 + rank)
    return decision_timing(args, d, model, items)


LARGE = dict(hidden=1024, intermediate=2624, layers=28, heads=16, vocab=50368)   # ModernBERT-large (config 4)


def f32_measure(args, d):
    """The decision forward's fp32-accurate path (LAYA_PRECISION_F32) on a bf16 checkpoint of ModernBERT-large
    geometry (the released English / TypedDecisions checkpoints' encoder) with the decision head, config 2's batch."""
    import laya_b200
    from laya_b200 import workloads
    w = workloads.bf16_checkpoint_weights(**LARGE, seed=0)
    desc = laya_b200.base_desc(max_tokens=TOKENS, max_items=ROWS, max_markers=ROWS * 8,
                               precision=laya_b200.PRECISION_F32, **LARGE)
    model = laya_b200.DecisionModel(desc, w, device=d.local)
    del w
    items = workloads.decision_batch(rows=ROWS, length=SEQ, seed=1 + d.rank)
    return decision_timing(args, d, model, items)


def decision_timing(args, d, model, items):
    """Device-resident and host-pointer timings of the batched decision forward over `items`."""
    import numpy as np
    import torch
    import laya_b200
    local = d.local
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
    out = {}
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    d.barrier()
    launches0 = model.ctx.launches()
    model.ctx.set_profiling(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            step_device()
        e1.record(stream)
    e1.synchronize()
    out["launches"] = model.ctx.launches() - launches0
    out["gemm"] = model.ctx.profile()
    model.ctx.set_profiling(False)
    model.ctx.synchronize()
    d.barrier()
    out["clocks"] = sampler.stop()
    out["ms"] = e0.elapsed_time(e1) / args.steps

    pin = [torch.from_numpy(v).pin_memory() for v in (ids, seg_len, qtype, counts, markers)]
    host_logits = torch.zeros(n_mark, dtype=torch.float32).pin_memory()
    host_act = torch.zeros(ROWS * 2, dtype=torch.float32).pin_memory()

    def step_host():
        laya_b200.api.check(L.laya_decision_forward(
            model.ctx.handle, pin[0].data_ptr(), pin[1].data_ptr(), pin[2].data_ptr(), ROWS, pin[3].data_ptr(),
            pin[4].data_ptr(), host_logits.data_ptr(), host_act.data_ptr()))

    for _ in range(max(1, args.warmup // 2)):
        step_host()
    d.barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for _ in range(args.steps):
        step_host()
    h1.record(stream)
    h1.synchronize()
    d.barrier()
    out["e2e_ms"] = h0.elapsed_time(h1) / args.steps
    out["h2d"] = sum(int(v.nbytes) for v in (ids, seg_len, qtype, counts, markers))
    out["d2h"] = n_mark * 4 + ROWS * 2 * 4
    model.ctx.close()
    return out


def dec_measure(args, d):
    import numpy as np
    import torch
    import laya_b200
    from laya_b200 import workloads
    rank, world, local = d.rank, d.world, d.local
    kinds = workloads.MICA_KINDS[:args.dec_layers]
    model = laya_b200.Qwen35Model(laya_b200.decoder_desc(kinds, max_tokens=DEC_TOKENS, max_seqs=DEC_ROWS),
                                  device=local)
    q8, vec = workloads.decoder_q8_weights(kinds, seed=0)          # the same weights on every rank
    for name, (q, dd) in q8.items():
        model.upload_q8_0(name, q, dd)
    for name, v in vec.items():
        model.upload(name, v)
    del q8, vec
    seqs, labels = workloads.decoder_batch(rows=DEC_ROWS, length=DEC_LEN, n_labels=DEC_LABELS, seed=5 + rank)
    ids = np.concatenate(seqs).astype(np.int32)
    lens = [len(s) for s in seqs]
    stream = torch.cuda.Stream()
    model.set_stream(stream.cuda_stream)
    model.set_chunked_delta_rule(args.delta_rule == "chunked")
    ids_dev = torch.from_numpy(ids).cuda()
    hidden = torch.zeros((DEC_ROWS, 2560), dtype=torch.float32, device="cuda")
    logits = torch.zeros((DEC_ROWS, DEC_LABELS), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step_device():
        model.forward_device(ids_dev.data_ptr(), lens, labels, hidden.data_ptr(), logits.data_ptr())

    for _ in range(args.warmup):
        step_device()
    model.synchronize()
    out = {}
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    d.barrier()
    launches0 = model.launches()
    model.set_profiling(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_device()
    e1.record(stream)
    e1.synchronize()
    out["launches"] = model.launches() - launches0
    out["prof"] = [model.profile(k) for k in range(3)]
    model.set_profiling(False)
    model.synchronize()
    d.barrier()
    out["clocks"] = sampler.stop()
    out["ms"] = e0.elapsed_time(e1) / args.steps
    out["finite"] = bool(torch.isfinite(logits).all().item())

    pin_ids = torch.from_numpy(ids).pin_memory()
    lens_np = np.asarray(lens, np.int32)
    lab_np = np.asarray(labels, np.int32)
    host_hidden = torch.zeros((DEC_ROWS, 2560), dtype=torch.float32).pin_memory()
    host_logits = torch.zeros((DEC_ROWS, DEC_LABELS), dtype=torch.float32).pin_memory()
    L = laya_b200.lib()

    def step_host():
        laya_b200.api.check(L.laya_decoder_forward(
            model.handle, pin_ids.data_ptr(), lens_np.ctypes.data, DEC_ROWS, lab_np.ctypes.data, DEC_LABELS,
            host_hidden.data_ptr(), host_logits.data_ptr()))

    step_host()
    d.barrier()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for _ in range(args.steps):
        step_host()
    h1.record(stream)
    h1.synchronize()
    d.barrier()
    out["e2e_ms"] = h0.elapsed_time(h1) / args.steps
    out["h2d"] = int(ids.nbytes + lens_np.nbytes + lab_np.nbytes)
    out["d2h"] = int(host_hidden.numel() * 4 + host_logits.numel() * 4)
    out["shared"] = shared_prefix_measure(args, d, model, stream, labels)
    model.close()
    return out


def shared_prefix_measure(args, d, model, stream, labels):
    """A multi-question Mica request as MicaJudge.Predict serves it (MicaJudge.cs:166-229): the questions' common
    prefix read once into a state (Readout = false), then every question's remainder in one batched pass, each from
    its own clone of the prefix state, with the label logits.  The same prompts as the prefill step (DEC_ROWS
    questions of DEC_LEN tokens), DEC_SHARED of them shared.  Timed per request through the host-pointer C ABI."""
    import numpy as np
    import torch
    import laya_b200
    rng = np.random.default_rng(11 + d.rank)
    prefix = rng.integers(0, 151936, DEC_SHARED).astype(np.int64)
    rests = [rng.integers(0, 151936, DEC_LEN - DEC_SHARED).astype(np.int64) for _ in range(DEC_ROWS)]

    def request():
        state = model.new_state(DEC_LEN)
        model.read(prefix, state)
        branches = [laya_b200.Qwen35Sequence(r, state if i == DEC_ROWS - 1 else state.clone())
                    for i, r in enumerate(rests)]
        model.forward_sequences(branches, labels)
        for q in branches:
            q.state.close()
        return branches

    for _ in range(max(1, args.warmup)):
        request()
    d.barrier()
    launches0 = model.launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        out = request()
    e1.record(stream)
    e1.synchronize()
    d.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    return {"ms": ms, "launches": (model.launches() - launches0) // args.steps,
            "finite": all(bool(np.isfinite(q.logits).all()) for q in out)}


def run_ours(args):
    import torch
    rank, world, local = dist_env()
    d = Dist(rank, world, local)
    peaks, source = load_peaks()
    traffic = load_traffic()
    bf16_sus = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1590.0))
    SUM = lambda dist: dist.ReduceOp.SUM
    MAX = lambda dist: dist.ReduceOp.MAX
    line = None
    if args.workload in ("all", "train"):
        mode = 0 if args.forward == "accurate" else 1
        r = train_measure(args, d, mode)
        ms, e2e_ms = d.reduce([r["ms"], r["e2e_ms"]], MAX)
        step_tokens, h2d = d.reduce([r["tokens_per_step"], r["h2d"]], SUM)   # all ranks, per step
        alt = None
        if args.workload == "all" and not args.no_bf16_forward:
            ra = train_measure(args, d, 1 - mode, with_e2e=False, with_profile=False)
            alt = (d.reduce([ra["ms"]], MAX)[0], d.reduce([ra["tokens_per_step"]], SUM)[0])
        if rank == 0:
            (g_ms, g_fl, g_n), (af_ms, af_fl, af_n), (ab_ms, ab_fl, ab_n) = r["prof"]
            g_ach = g_fl / (g_ms / 1e3) / 1e12 if g_ms else 0.0
            step_flops = (g_fl + af_fl + ab_fl) / args.steps
            fwd = "accurate (bf16 hi/lo tensor-core products, fp32-accurate forward)" if mode == 0 else \
                "bf16 (bf16-operand forward)"
            value = step_tokens / (ms / 1e3)
            line = {
                "metric": "fine-tune tokens/s (fwd+bwd+AdamW)", "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": train_config(world, r["tokens_per_step"], fwd, train_shape(args)[4], args.train_config,
                                       train_shape(args)[5:]),
                "e2e": {"value": step_tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": r["d2h"] * world,
                        "ms_per_step": e2e_ms},
                "roofline": {"kernel": "gemm_bf16_kernel (tcgen05 bf16 products: forward, dX, split-K dW)",
                             "bound": "tensor", "achieved": g_ach, "peak": bf16_sus, "unit": "TFLOP/s",
                             "frac": g_ach / bf16_sus,
                             "peak_source": f"{source} bf16 sustained (kernels timed inside a long step)",
                             "traffic": traffic.get("bf16_gemm", {}).get("dram_bytes_per_launch"),
                             "launches": g_n, "share_of_step": g_ms / args.steps / ms,
                             "flops_per_launch": g_fl / g_n if g_n else None},
                "attention": {"kernels": "tcgen05 flash forward, dK/dV and dQ (head_dim 64)",
                              "fwd_tflops": af_fl / (af_ms / 1e3) / 1e12 if af_ms else None,
                              "bwd_tflops": ab_fl / (ab_ms / 1e3) / 1e12 if ab_ms else None,
                              "share_of_step": (af_ms + ab_ms) / args.steps / ms},
                "step_roofline": {"algorithmic_tflop_per_step": step_flops / 1e12,
                                  "achieved": step_flops / (ms / 1e3) / 1e12, "peak": bf16_sus, "unit": "TFLOP/s",
                                  "frac": step_flops / (ms / 1e3) / 1e12 / bf16_sus,
                                  "note": "products 2MNK (fwd) + 4MNK (bwd); attention 4·hidden per visible pair "
                                          "fwd, 2x bwd; no credit for the accurate forward's extra passes"},
                "gpu_launches": r["launches"],
                "clocks": r["clocks"],
                "loss_last_e2e_step": r["loss"],
            }
            if alt:
                line["bf16_forward" if mode == 0 else "accurate_forward"] = {
                    "value": alt[1] / (alt[0] / 1e3), "unit": "tokens/s", "ms_per_step": alt[0]}
        if args.workload == "all" and args.train_config == 3 and not args.no_config4 and world == 1:
            # config 4 (ModernBERT-large, 4 rows of 8192 tokens) beside the headline on one GPU: a few timed steps
            import copy
            a4 = copy.copy(args)
            a4.train_config, a4.train_layers, a4.train_rows = 4, None, None
            a4.steps, a4.warmup = max(2, min(args.steps, 4)), 2
            try:
                r4 = train_measure(a4, d, mode, with_e2e=False, with_profile=False)
                ms4 = d.reduce([r4["ms"]], MAX)[0]
                tok4 = d.reduce([r4["tokens_per_step"]], SUM)[0]
                c4 = {"metric": "fine-tune tokens/s (fwd+bwd+AdamW)", "value": tok4 / (ms4 / 1e3),
                      "unit": "tokens/s", "ms_per_step": ms4, "steps": a4.steps, "warmup": a4.warmup,
                      "config": train_config(world, r4["tokens_per_step"], fwd if rank == 0 else "", 4, 4, (8192, 8192))}
            except Exception as e:   # reported, not fatal: the headline line stands on its own
                c4 = {"error": f"{type(e).__name__}: {e}"}
            if rank == 0 and line is not None:
                line["config4_long_context"] = c4
            if not args.no_cpu_baseline and world == 1:   # the CPU sample: rank 0 at N = 1 only
                line["cpu_baseline"] = train_cpu_baseline(args.cpu_train_tokens)
    if args.workload in ("all", "q8"):
        r = q8_measure(args, d)
        ms, e2e_ms = d.reduce([r["ms"], r["e2e_ms"]], MAX)
        if rank == 0:
            gemm_ms, gemm_ops, gemm_n = r["gemm"]
            i8_peak = measured_i8_peak()
            achieved = gemm_ops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else 0.0
            q = {
                "metric": "Q8_0 encode tokens/s", "value": world * TOKENS / (ms / 1e3), "unit": "tokens/s",
                "n_gpus": world, "ms_per_step": ms, "dtype": "int8", "scaling": "weak", "config": q8_config(world),
                "e2e": {"value": world * TOKENS / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                        "d2h_bytes_per_step": r["d2h"], "ms_per_step": e2e_ms},
                "roofline": {"kernel": "q8_gemm_kernel (Q8_0 product: exact fp16-held codes on tcgen05 kind::f16, "
                                       "per-block rescale)",
                             "bound": "tensor", "achieved": achieved, "peak": i8_peak, "unit": "TOP/s",
                             "frac": achieved / i8_peak, "peak_source": I8_SOURCE,
                             "traffic": traffic.get("q8_gemm", {}).get("dram_bytes_per_launch"), "launches": gemm_n,
                             "share_of_step": gemm_ms / args.steps / ms},
                "gpu_launches": r["launches"], "clocks": r["clocks"]}
            if not args.no_cpu_baseline and world == 1:   # the CPU sample: rank 0 at N = 1 only
                q["cpu_baseline"] = q8_cpu_baseline(args.cpu_sample_rows)
            if line is None:
                q.update({"steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "vs_baseline": None, "data": "synthetic"})
                line = q
            else:
                line["q8_0_encode"] = q
    if args.workload in ("all", "f32"):
        r = f32_measure(args, d)
        ms, e2e_ms = d.reduce([r["ms"], r["e2e_ms"]], MAX)
        if rank == 0:
            g_ms, g_ops, g_n = r["gemm"]
            bf16 = peaks.get("bf16_tflops", 1590.0)
            H, I, Ls = LARGE["hidden"], LARGE["intermediate"], LARGE["layers"]
            # two bf16 passes per product (bf16 weights): executed = 2 x algorithmic
            executed = g_ops / (g_ms / 1e3) / 1e12 if g_ms > 0 else 0.0
            q = {"metric": "decision forward tokens/s, fp32-accurate path on a bf16 checkpoint",
                 "value": world * TOKENS / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "ms_per_step": ms,
                 "dtype": "bf16 split (fp32-accurate)", "scaling": "weak",
                 "config": {"workload": "systemone_f32_modernbert_large", "rows_per_gpu": ROWS, "seq_len": SEQ,
                            "geometry": f"ModernBERT-large encoder ({Ls} layers, h {H}, 16x64, GeGLU I {I}) + "
                                        "2 head layers + scorer + act head",
                            "weights": "bf16 values (a bf16 checkpoint), products x_hi.W + x_lo.W",
                            "parallelism": f"request-sharded x{world}, no collective"},
                 "e2e": {"value": world * TOKENS / (e2e_ms / 1e3), "unit": "tokens/s",
                         "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"], "ms_per_step": e2e_ms},
                 "roofline": {"kernel": "gemm_bf16_kernel (split product, two passes)", "bound": "tensor",
                              "achieved": executed / 2, "executed": executed, "peak": bf16, "unit": "TFLOP/s",
                              "frac": executed / bf16, "peak_source": f"{source} bf16 burst",
                              "launches": g_n, "share_of_step": g_ms / args.steps / ms},
                 "gpu_launches": r["launches"], "clocks": r["clocks"]}
            if not args.no_cpu_baseline and world == 1:   # the CPU sample: rank 0 at N = 1 only
                q["cpu_baseline"] = f32_cpu_baseline()
            if line is None:
                q.update({"steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "vs_baseline": None, "data": "synthetic"})
                line = q
            else:
                line["systemone_f32"] = q
    if args.workload in ("all", "decoder"):
        r = dec_measure(args, d)
        ms, e2e_ms, sp_ms = d.reduce([r["ms"], r["e2e_ms"], r["shared"]["ms"]], MAX)
        if rank == 0:
            (g_ms, g_ops, g_n), (r_ms, r_ops, r_n), (a_ms, a_ops, a_n) = r["prof"]
            i8_peak = measured_i8_peak()
            achieved = g_ops / (g_ms / 1e3) / 1e12 if g_ms > 0 else 0.0
            q = {
                "metric": "Mica prefill tokens/s", "value": world * DEC_TOKENS / (ms / 1e3), "unit": "tokens/s",
                "n_gpus": world, "ms_per_step": ms, "dtype": "int8", "scaling": "weak",
                "config": dec_config(world, args.dec_layers),
                "e2e": {"value": world * DEC_TOKENS / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                        "d2h_bytes_per_step": r["d2h"], "ms_per_step": e2e_ms},
                "roofline": {"kernel": "q8_gemm_kernel (Q8_0 products: exact fp16-held codes on tcgen05 kind::f16, "
                                       "per-block rescale)",
                             "bound": "tensor", "achieved": achieved, "peak": i8_peak, "unit": "TOP/s",
                             "frac": achieved / i8_peak, "peak_source": I8_SOURCE,
                             "traffic": traffic.get("q8_gemm_dec", {}).get("dram_bytes_per_launch"), "launches": g_n,
                             "share_of_step": g_ms / args.steps / ms},
                "delta_rule": {"kernel": "delta_chunk_kernel (gated delta rule in 64-token chunks, tcgen05 "
                                         "fp32-accurate products, one CTA per sequence x value head)"
                                         if args.delta_rule == "chunked" else
                                         "delta_rule_kernel (per-token sweep, one CTA per sequence x value head)",
                               "ms_per_step": r_ms / args.steps,
                               "share_of_step": r_ms / args.steps / ms,
                               "gflops": r_ops / (r_ms / 1e3) / 1e9 if r_ms else None},
                "attention": {"kernel": "attn_prep + attention_tc_kernel (tcgen05 fp16, causal GQA, two query heads per CTA, sigmoid gate)",
                              "ms_per_step": a_ms / args.steps, "share_of_step": a_ms / args.steps / ms,
                              "tflops": a_ops / (a_ms / 1e3) / 1e12 if a_ms else None},
                "gpu_launches": r["launches"], "clocks": r["clocks"], "logits_finite": r["finite"]}
            q["mica_shared_prefix"] = {
                "metric": "Mica prompt tokens/s, shared prefix read once into a state (MicaJudge.Predict)",
                "value": world * DEC_TOKENS / (sp_ms / 1e3), "unit": "tokens/s", "ms_per_request": sp_ms,
                "requests_per_s": world / (sp_ms / 1e3),
                "config": {"questions": DEC_ROWS, "prompt_tokens": DEC_LEN, "shared_prefix": DEC_SHARED,
                           "path": "laya_decoder_state_create + forward_states(read prefix) + state_clone x"
                                   f"{DEC_ROWS - 1} + forward_states(all remainders, label logits), host buffers"},
                "vs_prefill_every_prompt_ms": e2e_ms, "gpu_launches_per_request": r["shared"]["launches"],
                "logits_finite": r["shared"]["finite"]}
            if not args.no_cpu_baseline and world == 1:   # the CPU sample: rank 0 at N = 1 only
                q["cpu_baseline"] = dec_cpu_baseline(args.dec_tokens)
            if line is None:
                q.update({"steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "vs_baseline": None, "data": "synthetic"})
                line = q
            else:
                line["mica_prefill"] = q
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        d.barrier()
        torch.distributed.destroy_process_group()


# --------------------------------------------------------------------------------------------------- one product
def run_mma_peak():
    """The tensor-core rate per MMA form and width on this device (laya_mma_peak): one CTA per SM issuing back-to-back
    M 128 x N MMAs from fixed shared-memory (or, TS, tensor-memory) operands.  One JSON line per (form, N)."""
    import ctypes
    import torch
    import laya_b200
    torch.cuda.set_device(0)
    L = laya_b200.lib()
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    forms = {"bf16": (0, 16), "f16": (1, 16), "i8": (2, 32), "bf16_ts": (3, 16), "bf16_mn": (4, 16),
             "bf16_ts_mn": (5, 16)}
    reps = 20000
    for name, (form, k) in forms.items():
        for n in (64, 128, 256):
            ms, cyc = ctypes.c_double(), ctypes.c_double()
            laya_b200.api.check(L.laya_mma_peak(form, n, reps, ctypes.byref(ms), ctypes.byref(cyc)))
            ops = nsm * reps * 4 * 2.0 * 128 * n * k
            print(json.dumps({"kernel": "mma_peak", "form": name, "M": 128, "N": n, "K": k,
                              "tops": ops / (ms.value / 1e3) / 1e12, "cycles_per_mma": cyc.value,
                              "ops_per_clk_per_sm": 2.0 * 128 * n * k / cyc.value, "ms": ms.value}), flush=True)


def run_kernel(args):
    """One product alone at a workload shape, CUDA events over --reps launches (the command ncu captures)."""
    import torch
    import laya_b200
    if args.kernel == "mma_peak":
        return run_mma_peak()
    torch.cuda.set_device(0)
    ctx = laya_b200.Context(laya_b200.base_desc(max_tokens=512, max_items=4, max_markers=16))
    st = torch.cuda.current_stream()
    ctx.set_stream(st.cuda_stream)
    L = laya_b200.lib()
    if args.kernel == "q8_gemm":
        N, K = {"wqkv": (2304, 768), "wo": (768, 768), "wi": (2304, 768), "mlp_wo": (768, 1152),
                "dec_in": (8224, 2560), "dec_qkv": (5120, 2560), "dec_gate_up": (18432, 2560),
                "dec_down": (2560, 9216), "dec_out": (2560, 2048)}[args.case]
        M = DEC_TOKENS if args.case.startswith("dec_") else TOKENS
        qx = torch.randint(-127, 128, (M, K), device="cuda").to(torch.float16)
        qw = torch.randint(-127, 128, (N, K), device="cuda").to(torch.float16)
        ldx, ldw = (M + 127) // 128 * 128, (N + 127) // 128 * 128
        dx = torch.rand((K // 32, ldx), device="cuda") * 0.01
        dw = torch.rand((K // 32, ldw), device="cuda") * 0.002
        out = torch.empty((M, N), device="cuda")
        f = lambda: L.laya_q8_0_gemm_device(ctx.handle, qx.data_ptr(), dx.data_ptr(), ldx, M, qw.data_ptr(),
                                            dw.data_ptr(), ldw, N, K, None, out.data_ptr(), N)
        flops = 2.0 * M * N * K
        desc = f"q8_gemm_kernel store epilogue, config-{5 if args.case.startswith('dec_') else 2} {args.case}: " \
               f"M={M} N={N} K={K}"
    else:
        T, H = 20480, 768
        bf = torch.bfloat16
        if args.case == "fwd_split":     # y = x·Wᵀ from hi/lo parts (accurate forward), fp32 out
            M, N, K = T, 3 * H, H
            A, Al = torch.randn(M, K, device="cuda").to(bf), torch.randn(M, K, device="cuda").to(bf) * 1e-3
            B, Bl = torch.randn(N, K, device="cuda").to(bf), torch.randn(N, K, device="cuda").to(bf) * 1e-3
            out = torch.zeros(M, N, device="cuda")
            f = lambda: L.laya_gemm_bf16_split_device(ctx.handle, M, N, K, A.data_ptr(), Al.data_ptr(), K, 0,
                                                      B.data_ptr(), Bl.data_ptr(), K, 0, None, 1, out.data_ptr(), N)
        elif args.case == "dx":          # dx = dy·W, W read N-contiguous, fp32 out
            M, N, K = T, H, 3 * H
            A = torch.randn(M, K, device="cuda").to(bf)
            B = torch.randn(K, N, device="cuda").to(bf)
            out = torch.zeros(M, N, device="cuda")
            f = lambda: L.laya_gemm_bf16_device(ctx.handle, M, N, K, A.data_ptr(), K, 0, B.data_ptr(), N, 1, None, 1,
                                                out.data_ptr(), N)
        else:                            # dW += dyᵀ·x, both read N-contiguous, K = tokens, split-K reduce-add
            M, N, K = 3 * H, H, T
            A = torch.randn(K, M, device="cuda").to(bf)
            B = torch.randn(K, N, device="cuda").to(bf)
            out = torch.zeros(M, N, device="cuda")
            f = lambda: L.laya_gemm_bf16_device(ctx.handle, M, N, K, A.data_ptr(), M, 1, B.data_ptr(), N, 1, None, 2,
                                                out.data_ptr(), N)
        flops = 2.0 * M * N * K
        desc = f"gemm_bf16_kernel {args.case}: M={M} N={N} K={K}"
    for _ in range(3):
        laya_b200.api.check(f())
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.reps):
        laya_b200.api.check(f())
    e1.record()
    e1.synchronize()
    ctx.synchronize()
    ms = e0.elapsed_time(e1) / args.reps
    print(json.dumps({"kernel": desc, "ms": ms, "tflops": flops / (ms / 1e3) / 1e12, "reps": args.reps}), flush=True)
    ctx.close()


def main():
    args = parse()
    if args.kernel:
        run_kernel(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Benchmark of the XingLing-0.68B token loop on B200.

Workload (per GPU): the XingLing-0.68B shape in fp32 with seeded N(0, 0.02)
weights (gains 1.0), a 32-id prompt (uniform ids, seed 0), then 128 greedy
decode tokens (top_p 0, repetition penalty 1.0).  One step = that prefill +
128 decode tokens.  The headline `value` is decode tokens/s from CUDA events
on the engine's stream around each decode step (inputs resident in HBM;
weights 2.75 GB per token, far above the 126 MB L2, so no flush is needed);
`e2e` is the same metric through the public API (llm_cpp_engine
next_token(int)), wall clock, including the per-token host->device copy of
the step inputs from pinned memory and the device->host read of the result.
`roofline` is the dominant kernel, the persistent decode kernel (one launch
per token, all of a greedy decode step's kernel time), timed by CUDA event
nodes around it inside the decode graph in one more step right after the
timed region (the timed steps run without the nodes).  Also reported: the
whole decode step against the same roofline, the same 128 ids through the
device-side loop (`generate`, one call per prefill), prefill of a 512-id
prompt (seed 1),
the reference's own CPU path on the host cores, `replica_batch` (64
sequences, prompt lengths uniform in [16, 512] with seed 5, 128 sampled
tokens each, spread over the N replicas, each replica decoding waves of 8
sequences with one batched step per token, and the same sequences one at a
time beside it) and at N > 1 the tensor-parallel decode latency (prompt 64,
seed 4, greedy 256).

  python bench.py [--gpus N --steps K --warmup W]          # this engine
  python bench.py --impl reference [...]                   # reference CPU path
N > 1 runs one engine per GPU (replicas, weak scaling) under torchrun.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "xingling-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for _p in (PKG, ORACLE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import xl_synth as S  # noqa: E402

PROMPT, DECODE, PREFILL_N = 32, 128, 512
ENGINE_OPTS: dict[str, int] = {}  # --opt KEY=VALUE, applied to every engine the bench creates


def apply_opts(eng):
    for k, v in ENGINE_OPTS.items():
        eng.set_option(k, v)
    return eng


REF_DECODE_SAMPLE = 128  # the reference arm times the whole decode workload each step
WEIGHT_DIR = os.environ.get("XL_BENCH_WEIGHTS", os.path.join(tempfile.gettempdir(), "xl_weights", "full"))
METRIC = "decode tokens/s, XingLing-0.68B fp32, batch 1"


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def decode_bytes_per_token(shape: S.ModelShape, ctx: float) -> float:
    """Algorithmic HBM bytes of one decode token: every Linear weight, bias and
    gain, the tied LM head (whole embedding table), one embedding row, the
    final gain, and K and V of `ctx` cached positions in every layer."""
    H, F, V, L = shape.hidden, shape.ffn, shape.vocab, shape.layers
    per_layer = 4 * (4 * H * H + 4 * H + 3 * F * H + 2 * F + H + 2 * H)
    return L * per_layer + 4 * V * H + 4 * H + 4 * H + 2 * L * 4 * H * ctx


def traffic_per_launch() -> float | None:
    """DRAM bytes (read + write) of one persistent decode launch at the bench's
    workload, from the Nsight Compute capture summarised in
    profiles/decode_persistent_kernel.md (its `traffic_per_launch_full` line)."""
    p = os.path.join(ROOT, "profiles", "decode_persistent_kernel.md")
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_per_launch_full:"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def prefill_flops(shape: S.ModelShape, n: int) -> float:
    H, F, L, V = shape.hidden, shape.ffn, shape.layers, shape.vocab
    linear = 2.0 * n * (4 * H * H + 3 * F * H) * L
    attn = 4.0 * 64 * shape.heads * L * n * (n + 1) / 2
    return linear + attn + 2.0 * H * V


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = tempfile.mktemp(prefix="xl_clocks_", suffix=".csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sms, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10 or (self.uuid and parts[1] != self.uuid):
                    continue
                try:
                    sm, mx = float(parts[2]), float(parts[3])
                except ValueError:
                    continue
                sms.append(sm)
                smax = mx
                for name, val in zip(names, parts[6:10]):
                    if val.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sms)}


# ---------------------------------------------------------------------------
def cpu_worker(args) -> None:
    """CPU baseline in its own process (CUDA_VISIBLE_DEVICES=""): the reference's
    CPU path (oracle/_ref) when built, else the oracle port; prefill of the
    32-id prompt, then greedy decode for up to `budget` seconds."""
    import numpy as np

    import oracle

    shape = S.FULL
    kind = "reference" if oracle.ref_available() else "port"
    model = oracle.Ref(shape) if kind == "reference" else oracle.Port(shape)
    model.load(args.weights)
    ids = S.prompt_ids(0, PROMPT, shape.vocab)

    def pick(logits):
        if kind == "reference":  # the reference's sample_cpu, greedy settings
            return oracle.ref_sample(logits, 0.7, 0.0, 1.0, [], 0)[0]
        return int(np.argmax(logits))

    t0 = time.perf_counter()
    tok = pick(model.prefill(ids))
    t_prefill = time.perf_counter() - t0
    n, t_dec = 0, 0.0
    while n < DECODE and t_dec < args.budget:
        t0 = time.perf_counter()
        tok = pick(model.decode(tok))
        t_dec += time.perf_counter() - t0
        n += 1
    print(json.dumps({"value": n / t_dec, "unit": "tokens/s", "cores": int(os.environ.get("OMP_NUM_THREADS", "1")),
                      "kind": kind, "prefill_ms": 1e3 * t_prefill,
                      "sample": f"prefill {PROMPT} ids + {n} greedy decode tokens of the {DECODE}-token workload"}))
    sys.stdout.flush()
    os._exit(0)  # the reference's Embedding destructor exits the process on GPU-less hosts


def run_cpu_baseline(budget: float) -> dict | None:
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS=str(host_cores()))
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    try:
        r = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-worker", "--budget", str(budget),
                            "--weights", WEIGHT_DIR], env=env, capture_output=True, text=True, timeout=600)
        for line in r.stdout.splitlines()[::-1]:
            if line.startswith("{"):
                return json.loads(line)
        sys.stderr.write(r.stdout[-2000:] + r.stderr[-2000:])
    except subprocess.TimeoutExpired:
        pass
    return None


def library_record(path: str) -> dict:
    """The library the reference arm timed: its resolved path, size and hash,
    and whether this process has it mapped (from /proc/self/maps)."""
    import hashlib

    real = os.path.realpath(path)
    rec = {"path": os.path.relpath(real, ROOT), "bytes": os.path.getsize(real),
           "sha256_16": hashlib.sha256(open(real, "rb").read()).hexdigest()[:16],
           "what": "the reference's src/*.cu compiled from its sources by oracle/Makefile, behind oracle/ref_harness.cpp"
           if real.endswith("libxlref.so") else "the oracle's C restatement (oracle/xl_oracle.c)"}
    try:
        with open("/proc/self/maps") as f:
            rec["mapped"] = any(line.rstrip().endswith(real) for line in f)
    except OSError:
        rec["mapped"] = None
    return rec


# ---------------------------------------------------------------------------
def reference_arm(args) -> None:
    """The reference's own CPU implementation (oracle/_ref, else the oracle port),
    all host threads, same metric: each step = prefill of the 32-id prompt and a
    bounded sample of REF_DECODE_SAMPLE greedy decode tokens."""
    if env_int("RANK", 0) != 0:
        return
    os.environ["CUDA_VISIBLE_DEVICES"] = ""
    os.environ.setdefault("OMP_NUM_THREADS", str(host_cores()))
    import numpy as np

    import oracle

    shape = S.FULL
    S.write_weight_tree(WEIGHT_DIR, shape)
    kind = "reference" if oracle.ref_available() else "port"
    model = oracle.Ref(shape) if kind == "reference" else oracle.Port(shape)
    model.load(WEIGHT_DIR)
    ids = S.prompt_ids(0, PROMPT, shape.vocab)

    def pick(logits):
        if kind == "reference":
            return oracle.ref_sample(logits, 0.7, 0.0, 1.0, [], 0)[0]
        return int(np.argmax(logits))

    def step():
        tok = pick(model.prefill(ids))
        t = 0.0
        for _ in range(REF_DECODE_SAMPLE):
            t0 = time.perf_counter()
            tok = pick(model.decode(tok))
            t += time.perf_counter() - t0
        return t

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    dec = sum(step() for _ in range(args.steps))
    wall = time.perf_counter() - t0
    value = args.steps * REF_DECODE_SAMPLE / dec
    cores = int(os.environ["OMP_NUM_THREADS"])
    lib = oracle.REF_SO if kind == "reference" else oracle.PORT_SO
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decode: prompt {PROMPT} ids (seed 0) + greedy tokens, XingLing-0.68B fp32",
                   "model": "XingLing-0.68B", "prompt": PROMPT, "decode_tokens_per_step": REF_DECODE_SAMPLE,
                   "device": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": f"per step: prefill {PROMPT} + {REF_DECODE_SAMPLE} of the {DECODE} decode tokens"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "library": library_record(lib),
    }
    print(json.dumps(line))
    sys.stdout.flush()
    os._exit(0)


# ---------------------------------------------------------------------------
def xl_arm(args) -> None:
    import torch
    import torch.distributed as dist

    import llm_cpp_engine

    rank, world, local = env_int("RANK", 0), env_int("WORLD_SIZE", 1), env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    shape = S.FULL
    if local == 0:
        S.write_weight_tree(WEIGHT_DIR, shape)
    barrier()
    if args.tp_only:
        if world < 2:
            raise SystemExit("--tp-only needs two or more ranks")
        tp_info = tp_latency(args, llm_cpp_engine, dist, rank, world, local, max_over_ranks)
        if rank == 0:
            print(json.dumps({"metric": "tensor-parallel decode latency", "tp": tp_info}))
            sys.stdout.flush()
        dist.destroy_process_group()
        return
    eng = apply_opts(llm_cpp_engine.InferenceEngine(f"cuda:{local}"))
    eng.load(WEIGHT_DIR)
    eng.load(WEIGHT_DIR)  # the second load reads the tree from the page cache
    load_s = eng.last_load_s()
    ids = S.prompt_ids(0, PROMPT, shape.vocab)

    def step():
        w0 = time.perf_counter()
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        pre_dev = eng.last_device_ms()
        w1 = time.perf_counter()
        dec_dev, kern = 0.0, []
        for _ in range(DECODE):
            tok = eng.next_token(tok, top_p=0.0, repetition_penalty=1.0)
            dec_dev += eng.last_device_ms()
            kern.append(eng.last_kernel_ms())
        w2 = time.perf_counter()
        return pre_dev, dec_dev, w1 - w0, w2 - w1, kern

    for _ in range(args.warmup):
        step()
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    with Clocks(uuid) as clk:
        barrier()
        torch.cuda.synchronize()
        launches0 = llm_cpp_engine.kernel_launches()
        t0 = time.perf_counter()
        res = [step() for _ in range(args.steps)]
        torch.cuda.synchronize()
        barrier()
        wall = time.perf_counter() - t0
        launches = llm_cpp_engine.kernel_launches() - launches0
    clocks = clk.summary()

    dec_dev_s = max_over_ranks(sum(r[1] for r in res) / 1e3)
    step_dev_s = max_over_ranks(sum(r[0] + r[1] for r in res) / 1e3)
    dec_wall_s = max_over_ranks(sum(r[3] for r in res))
    wall = max_over_ranks(wall)
    tokens = world * args.steps * DECODE
    value = tokens / dec_dev_s
    e2e = tokens / dec_wall_s

    pk, pk_kind = peaks()
    hbm = float(pk["hbm_gbs"])
    # whole decode step vs the HBM roofline (context grows 32 -> 160 over a step)
    ctx_mean = PROMPT + (DECODE - 1) / 2.0
    step_bytes = decode_bytes_per_token(shape, ctx_mean)
    step_gbs = step_bytes * (args.steps * DECODE) / (sum(r[1] for r in res) / 1e3) / 1e9

    # the dominant kernel: the persistent decode kernel, one launch per token at
    # context PROMPT + i, timed by event nodes around it in the decode graph
    # (a separate pass, so that the headline steps above run without them)
    eng.set_option("kernel_events", 1)
    kres = [step() for _ in range(2)][1:]
    eng.set_option("kernel_events", 0)
    kern_ms = [k for r in kres for k in r[4]]
    if min(kern_ms) <= 0:
        raise RuntimeError("persistent decode kernel times missing (decode path not persistent?)")
    kern_bytes = [decode_bytes_per_token(shape, PROMPT + i) for _ in kres for i in range(DECODE)]
    kern_avg_ms = sum(kern_ms) / len(kern_ms)
    kern_gbs = sum(kern_bytes) / (sum(kern_ms) / 1e3) / 1e9

    # the same decode workload through the device-side loop: one generate call
    # for the 128 ids after each prefill (wall clock around the call, and the
    # device time from the call's own CUDA events)
    gen_wall, gen_dev = [], []
    for i in range(max(3, args.steps) + 1):
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        w0 = time.perf_counter()
        out = eng.generate(tok, DECODE, top_p=0.0, repetition_penalty=1.0)
        if i > 0:
            gen_wall.append(time.perf_counter() - w0)
            gen_dev.append(eng.last_device_ms())
        if len(out) != DECODE:
            raise RuntimeError("generate returned fewer ids than asked")
    gen_info = {"api": "llm_cpp_engine.InferenceEngine.generate", "tokens_per_call": DECODE,
                "e2e_tokens_per_s": DECODE / statistics.median(gen_wall),
                "device_tokens_per_s": DECODE / (statistics.median(gen_dev) / 1e3),
                "h2d_bytes_per_call": 64 + 4 * DECODE, "d2h_bytes_per_call": 64 + 4 * DECODE + 80,
                "timing": "median over calls; wall clock around the call / CUDA events inside it"}

    # prefill of the 512-id prompt (seed 1)
    pids = S.prompt_ids(1, PREFILL_N, shape.vocab)
    for _ in range(2):
        eng.next_token(pids, top_p=0.0, repetition_penalty=1.0)
    pre_dev, pre_wall = [], []
    for _ in range(max(3, args.steps)):
        w0 = time.perf_counter()
        eng.next_token(pids, top_p=0.0, repetition_penalty=1.0)
        pre_wall.append(time.perf_counter() - w0)
        pre_dev.append(eng.last_device_ms())
    pre_ms = statistics.median(pre_dev)
    flops = prefill_flops(shape, PREFILL_N)
    tf32_peak, tf32_kind = measure_tf32_peak(torch), "measured: cuBLAS fp32 GEMM on TF32 tensor cores, 8192^3, best of 10"
    if tf32_peak is None:
        tf32_peak, tf32_kind = float(pk.get("bf16_tflops", 1590.0)) / 2.0, "half of the measured dense bf16 peak"

    batch_info = replica_batch(eng, rank, world, max_over_ranks, barrier)
    tp_info = None
    if world > 1:
        try:  # a sub-measurement: a failure here is reported in the line, not lost with it
            tp_info = tp_latency(args, llm_cpp_engine, dist, rank, world, local, max_over_ranks)
        except Exception as e:  # noqa: BLE001
            tp_info = {"tp": world, "error": repr(e)[:300]}
    del eng  # this rank's engine (its own graphs and streams) before the process group goes
    if world > 1:
        barrier()
        dist.destroy_process_group()

    if rank != 0:
        return
    cpu = run_cpu_baseline(args.cpu_budget) if world == 1 else None
    h2d = 4 * PROMPT + 36 + DECODE * 32
    d2h = (DECODE + 1) * 80
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * step_dev_s / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,0.02) fp32 weights (gains 1.0), uniform random prompt ids",
        "config": {"workload": f"decode: prompt {PROMPT} ids (seed 0) + {DECODE} greedy tokens, batch 1, per GPU",
                   "model": "XingLing-0.68B", "prompt": PROMPT, "decode_tokens": DECODE,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (2.75 GB of weights per token vs 126 MB L2)",
                   "value_timing": "CUDA events on the engine stream around each decode step; max over ranks"},
        "roofline": {"bound": "hbm", "kernel": "decode_persistent_kernel (16 layers + LM head, one launch per token)",
                     "achieved": kern_gbs, "peak": hbm, "unit": "GB/s", "frac": kern_gbs / hbm,
                     "traffic": traffic_per_launch(), "peak_kind": pk_kind,
                     "bytes_per_launch": sum(kern_bytes) / len(kern_bytes), "avg_launch_ms": kern_avg_ms},
        "step_roofline": {"bound": "hbm", "achieved": step_gbs, "peak": hbm, "unit": "GB/s", "frac": step_gbs / hbm,
                          "bytes_per_token": step_bytes, "mean_ctx": ctx_mean,
                          "ms_per_token": 1e3 * (sum(r[1] for r in res) / 1e3) / (args.steps * DECODE)},
        "prefill": {"prompt": PREFILL_N, "device_ms": pre_ms, "ttft_ms": 1e3 * statistics.median(pre_wall),
                    "tokens_per_s": PREFILL_N / (pre_ms / 1e3), "tflops": flops / (pre_ms / 1e3) / 1e12,
                    "tf32_peak_tflops": tf32_peak, "tf32_peak_kind": tf32_kind,
                    "frac_of_tf32": flops / (pre_ms / 1e3) / 1e12 / tf32_peak,
                    "hbm_floor_ms": 1e3 * decode_bytes_per_token(shape, 0) / (hbm * 1e9)},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "llm_cpp_engine.InferenceEngine.next_token"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    tree_bytes = sum(os.path.getsize(os.path.join(dp, f)) for dp, _, fs in os.walk(WEIGHT_DIR) for f in fs)
    line["load"] = {"seconds": load_s, "bytes": tree_bytes, "GB_per_s": tree_bytes / load_s / 1e9,
                    "what": "file reads + host-to-device copies of the raw-fp32 tree (page cache), 4 workers"}
    line["generate"] = gen_info
    line["replica_batch"] = batch_info
    if tp_info is not None:
        line["tp"] = tp_info
    print(json.dumps(line))
    sys.stdout.flush()


def measure_tf32_peak(torch) -> float | None:
    """Dense TF32 tensor-core throughput of this GPU (TFLOP/s): a cuBLAS fp32
    GEMM with TF32 allowed, 8192^3, best of 10 by CUDA events.  The prefill's
    roofline denominator (its 3xTF32 GEMMs run on the same tensor-core kind)."""
    try:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = True
        n = 8192
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        c = torch.empty(n, n, device="cuda")
        for _ in range(3):
            torch.matmul(a, b, out=c)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b, out=c)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        torch.backends.cuda.matmul.allow_tf32 = prev
        del a, b, c
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / (best / 1e3) / 1e12
    except Exception:  # noqa: BLE001
        return None


def tp_latency(args, llm_cpp_engine, dist, rank, world, local, max_over_ranks) -> dict:
    """Tensor-parallel decode across all ranks: prompt 64 (seed 4), greedy 256,
    on the persistent path (the split projections' partial sums exchanged over
    NVLink inside the kernel) and on the per-op path (NCCL all-reduces) for
    comparison."""
    out = tp_latency_path(llm_cpp_engine, dist, rank, world, local, max_over_ranks, 0, trace=args.tp_only)
    if args.tp_per_op:
        per_op = tp_latency_path(llm_cpp_engine, dist, rank, world, local, max_over_ranks, 1)
        out["per_op_ms_per_token"] = per_op["ms_per_token"]
        out["per_op_first_tokens"] = per_op["first_tokens"]
        out["per_op_gpu_launches"] = per_op["gpu_launches"]
    return out


PHASE_KINDS = ["QKV", "attention", "out-projection", "W1/V", "W2"]


def phase_summary(raw: bytes, sms: int, layers: int) -> dict:
    """Per-phase times (us) of one persistent decode step from its phase_trace
    stamps ([CTA][phase][start, staged, end, producer first, producer last],
    %globaltimer ns): per phase kind, the mean over layers of the median CTA's
    staging (start -> staged) and consume (staged -> end) times, and of the
    phase total (median CTA end of the phase minus that of the phase before)."""
    import numpy as np

    a = np.frombuffer(raw, dtype=np.uint64).reshape(sms, 5 * layers + 1, 5).astype(np.float64)

    def med(col):
        v = col[col > 0]
        return float(np.median(v)) if v.size else float("nan")

    ends = [med(a[:, ph, 2]) for ph in range(5 * layers + 1)]
    out = {}
    for k, name in enumerate(PHASE_KINDS + ["LM head"]):
        phs = [5 * layers] if k == 5 else [5 * l + k for l in range(layers)]
        stg, con, tot = [], [], []
        for ph in phs:
            ok = (a[:, ph, 0] > 0) & (a[:, ph, 1] > 0) & (a[:, ph, 2] > 0)
            if ok.any():
                stg.append(float(np.median(a[ok, ph, 1] - a[ok, ph, 0])) / 1e3)
                con.append(float(np.median(a[ok, ph, 2] - a[ok, ph, 1])) / 1e3)
            if ph > 0:
                tot.append((ends[ph] - ends[ph - 1]) / 1e3)
        out[name] = {"staging_us": float(np.mean(stg)) if stg else None,
                     "consume_us": float(np.mean(con)) if con else None,
                     "phase_us": float(np.mean(tot)) if tot else None}
    out["step_us"] = (ends[-1] - med(a[:, 0, 0])) / 1e3
    return out


def tp_latency_path(llm_cpp_engine, dist, rank, world, local, max_over_ranks, path, trace=False) -> dict:
    id_holder = [llm_cpp_engine.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(id_holder, src=0)
    eng = apply_opts(llm_cpp_engine.InferenceEngine(f"cuda:{local}", tp=world, rank=rank, nccl_id=id_holder[0]))
    eng.set_option("decode_path", path)
    eng.set_option("kernel_events", 1)  # the persistent kernel's own time, apart from the NCCL steps
    eng.load(WEIGHT_DIR)
    ids = S.prompt_ids(4, 64, S.FULL.vocab)
    n_dec = 256

    def run():
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        dev = kern = 0.0
        toks = [tok]
        for _ in range(n_dec):
            tok = eng.next_token(tok, top_p=0.0, repetition_penalty=1.0)
            dev += eng.last_device_ms()
            kern += max(0.0, eng.last_kernel_ms())
            toks.append(tok)
        return dev, kern, toks

    run()
    dist.barrier()
    n0 = llm_cpp_engine.kernel_launches()
    dev, kern, toks = run()
    launches = llm_cpp_engine.kernel_launches() - n0
    dev = max_over_ranks(dev)
    kern = max_over_ranks(kern)
    gen = None
    if path == 0:
        # the same workload through the device-side loop: one generate call per rank, no host round trip
        # between steps (CUDA events around the call's steps, max over ranks)
        tok = eng.next_token(ids, top_p=0.0, repetition_penalty=1.0)
        dist.barrier()
        gen_ids = eng.generate(tok, n_dec, top_p=0.0, repetition_penalty=1.0)
        gms = max_over_ranks(eng.last_device_ms())
        gen = {"api": "llm_cpp_engine.InferenceEngine.generate", "ms_per_token": gms / n_dec,
               "tokens_per_s": n_dec / (gms / 1e3), "same_ids_as_next_token": list(gen_ids) == toks[1:]}
    phases = None
    if trace and path == 0:
        # Phase timeline of one more step (the kernel stamps %globaltimer itself), rank 0's.
        import torch

        eng.set_option("phase_trace", 1)
        tok = toks[-1]
        for _ in range(4):
            tok = eng.next_token(tok, top_p=0.0, repetition_penalty=1.0)
        sms = torch.cuda.get_device_properties(local).multi_processor_count
        raw = eng.phase_trace(sms * (5 * S.FULL.layers + 1) * 5)
        phases = phase_summary(raw, sms, S.FULL.layers)
        phases["context"] = 64 + n_dec + 4
    del eng
    out = {"tp": world, "prompt": 64, "decode_tokens": n_dec, "ms_per_token": dev / n_dec,
           "tokens_per_s": n_dec / (dev / 1e3), "first_tokens": toks[:8], "decode_path": path,
           "persistent_kernel_ms_per_token": kern / n_dec if path == 0 else None, "gpu_launches": launches}
    if gen is not None:
        out["generate"] = gen
    if phases is not None:
        out["phase_timeline_rank0"] = phases
    return out


def replica_batch(eng, rank, world, max_over_ranks, barrier) -> dict:
    """64 independent sequences over the ranks' replicas: prompt lengths uniform
    in [16, 512] and ids uniform (seed 5), 128 sampled tokens each (T 0.7,
    top_p 0.9, repetition penalty 1.1, Philox seed 5000 + sequence).  Each
    replica decodes its sequences in waves of BatchDecoder.size (one batched
    step advances every sequence of the wave by one token, over one read of the
    weights); the same sequences decoded one at a time on the engine are timed
    beside it.  Reports the box's aggregate decode tokens/s over prefill +
    decode time."""
    import numpy as np
    import llm_cpp_engine

    rng = np.random.default_rng(5)
    lens = rng.integers(16, 513, size=64)
    seqs = [[int(t) for t in rng.integers(0, S.FULL.vocab, size=int(n))] for n in lens]
    mine = list(range(rank, 64, world))
    samp = dict(temperature=0.7, top_p=0.9, repetition_penalty=1.1)
    bd = llm_cpp_engine.BatchDecoder(eng)
    B = llm_cpp_engine.BatchDecoder.size
    barrier()
    dev_ms, w0 = 0.0, time.perf_counter()
    for w in range(0, len(mine), B):
        wave = mine[w:w + B]
        toks = []
        for b, j in enumerate(wave):
            bd.seed(b, 5000 + j)
            toks.append(bd.prefill(b, seqs[j], **samp))
            dev_ms += eng.last_device_ms()
        while len(toks) < B:  # a short last wave repeats its first sequence in the idle slots
            b = len(toks)
            bd.seed(b, 5000 + wave[0])
            toks.append(bd.prefill(b, seqs[wave[0]], **samp))
            dev_ms += eng.last_device_ms()
        for _ in range(DECODE):
            toks = bd.step(toks, **samp)
            dev_ms += bd.last_device_ms()
    wall = time.perf_counter() - w0
    dev_s = max_over_ranks(dev_ms / 1e3)
    wall = max_over_ranks(wall)
    # the same sequences one at a time on the engine
    barrier()
    seq_ms = 0.0
    for j in mine:
        eng.seed(5000 + j)
        tok = eng.next_token(seqs[j], **samp)
        seq_ms += eng.last_device_ms()
        for _ in range(DECODE):
            tok = eng.next_token(tok, **samp)
            seq_ms += eng.last_device_ms()
    seq_s = max_over_ranks(seq_ms / 1e3)
    tokens = 64 * DECODE
    return {"sequences": 64, "prompt_len": "uniform [16, 512], seed 5", "decode_tokens_each": DECODE,
            "sampling": "T 0.7, top_p 0.9, rp 1.1", "replicas": world, "batch_per_replica": B,
            "tokens_per_s": tokens / dev_s, "e2e_tokens_per_s": tokens / wall,
            "sequential_tokens_per_s": tokens / seq_s,
            "timing": "device time of every prefill and decode step; max over ranks"}


def ncu_case(args) -> None:
    """Short fixed workloads for Nsight Compute captures (no timing output):
    decode-full: XingLing-0.68B, prefill 32 + 4 decode steps;
    decode-sampled: XingLing-0.68B, prefill 32 + 4 decode steps sampled (T 0.7, top_p 0.9, rp 1.1);
    batch-sampled: XingLing-0.68B, 8 sequences (prompts of 32 ids) + 3 batched decode steps, sampled;
    decode-wide: 2 full-width layers, vocab 8192 (weights 276 MB > L2), prefill 32 + 3 decode steps;
    prefill-512: XingLing-0.68B, one prefill of 512 ids.
    --decode-path selects the persistent (0) or per-op (1) decode kernels."""
    import llm_cpp_engine

    shape = S.WIDE2 if args.ncu_case == "decode-wide" else S.FULL
    wdir = WEIGHT_DIR if shape is S.FULL else WEIGHT_DIR + "_wide2"
    S.write_weight_tree(wdir, shape)
    eng = apply_opts(llm_cpp_engine.InferenceEngine("cuda:0", **shape.engine_kwargs()))
    eng.load(wdir)
    eng.set_option("decode_path", args.decode_path)
    if args.ncu_case == "prefill-512":
        eng.next_token(S.prompt_ids(1, PREFILL_N, shape.vocab), top_p=0.0, repetition_penalty=1.0)
        return
    samp = dict(temperature=0.7, top_p=0.9, repetition_penalty=1.1) if "sampled" in args.ncu_case else \
        dict(top_p=0.0, repetition_penalty=1.0)
    if args.ncu_case == "batch-sampled":
        bd = llm_cpp_engine.BatchDecoder(eng)
        toks = [bd.prefill(b, S.prompt_ids(10 + b, PROMPT, shape.vocab), **samp) for b in range(bd.size)]
        for _ in range(3):
            toks = bd.step(toks, **samp)
        print("ncu case done", args.ncu_case, toks)
        return
    eng.seed(3)
    tok = eng.next_token(S.prompt_ids(0, PROMPT, shape.vocab), **samp)
    for _ in range(3 if args.ncu_case == "decode-wide" else 4):
        tok = eng.next_token(tok, **samp)
    print("ncu case done", args.ncu_case, tok)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["xl", "reference"], default="xl")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--ncu-case", choices=["decode-full", "decode-sampled", "batch-sampled", "decode-wide", "prefill-512"],
                    default=None)
    ap.add_argument("--decode-path", type=int, default=0, choices=[0, 1])
    ap.add_argument("--tp-only", action="store_true", help="only the tensor-parallel decode latency (torchrun, N>1)")
    ap.add_argument("--tp-per-op", type=int, default=1, choices=[0, 1],
                    help="also time the per-op tensor-parallel path (NCCL all-reduces) beside the persistent one")
    ap.add_argument("--opt", action="append", default=[], metavar="KEY=VALUE",
                    help="engine option (InferenceEngine.set_option) for every engine the bench creates")
    ap.add_argument("--cpu-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--budget", type=float, default=15.0, help=argparse.SUPPRESS)
    ap.add_argument("--weights", default=WEIGHT_DIR, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    for kv in args.opt:
        k, _, v = kv.partition("=")
        ENGINE_OPTS[k] = int(v)
    if args.ncu_case:
        ncu_case(args)
    elif args.cpu_worker:
        cpu_worker(args)
    elif args.impl == "reference":
        reference_arm(args)
    else:
        xl_arm(args)


if __name__ == "__main__":
    main()

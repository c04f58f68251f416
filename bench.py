"""Benchmark: embedded tokens/s of the packed embedding forward on B200.

Workload (the one the headline metric is quoted on):
Qwen3-Embedding-0.6B-shaped decoder, bf16, random-init safetensors weights
(seed 0); per rank a batch of 128 sequences, lengths U[32, 2048] + EOS, token
ids U[0, 151642] (seed 1 + rank).  One step = one forward + last-token pooling
+ L2 over that batch.  Weak scaling: every rank (one per GPU) encodes its own
batch; value = all ranks' tokens / max-over-ranks time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value` is measured with the inputs resident in HBM (ffwd_b200_encode_device)
and CUDA events on the backend's stream; `e2e` goes through the reference's
public API (ffwd_encode_batch of libffwd_b200_api.so) with host token ids,
H2D / D2H inside the timed region.  `--impl reference` times the reference's
own CPU path (oracle/_ref, OpenBLAS f32) on a bounded sample of the workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from ffwd_b200 import synth  # noqa: E402

CONFIG = "qwen3-0.6b"
METRIC = "embedded tokens/s"
UNIT = "tokens/s"


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


def workload(rank: int):
    spec = synth.CONFIGS[CONFIG]
    seqs = synth.token_batch(CONFIG, seed=1 + rank)
    return spec, seqs


def flops_per_token(spec, seqs):
    """Algorithmic FLOPs (2 x MAC), attention causal-exact, token-weighted."""
    H, I, L = spec.hidden, spec.intermediate, spec.n_layers
    q = spec.n_heads * spec.head_dim
    kv = spec.n_kv_heads * spec.head_dim
    lin = 2.0 * L * (H * (q + 2 * kv) + q * H + 3 * H * I)
    lens = np.array([len(s) for s in seqs], np.float64)
    attn = L * 4.0 * q * ((lens * (lens + 1) / 2).sum()) / lens.sum()
    return lin + attn, lin, attn


# ------------------------------------------------------------------ clocks


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        loaded = [v for v in sm if mx and v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ distributed


class Dist:
    """Rank plumbing of a torchrun launch (RANK / LOCAL_RANK / WORLD_SIZE /
    MASTER_* from the environment): NCCL with one rank per GPU, or gloo on CPU
    tensors (host-side tests).  Only the barrier and the max / sum of per-rank
    scalars cross ranks; the data path has no collective."""

    def __init__(self, backend: str = "nccl"):
        self.world = env_int("WORLD_SIZE", 1)
        self.rank = env_int("RANK", 0)
        self.local = env_int("LOCAL_RANK", 0)
        self.backend = backend
        self.pg = False
        self._gloo = None

    def init(self, torch):
        if self.world > 1:
            import torch.distributed as dist
            if self.backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(self.backend)
            self.pg = True

    def _device(self):
        return "cuda" if self.backend == "nccl" else "cpu"

    def barrier(self, torch):
        if self.pg:
            import torch.distributed as dist
            dist.barrier()

    def max(self, torch, v: float) -> float:
        if not self.pg:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=self._device())
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, torch, v: float) -> float:
        if not self.pg:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=self._device())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def cpu_barrier(self):
        """Barrier over a gloo group: waiting ranks spin on the host, not on a
        collective kernel that would hold SMs of their GPU."""
        if self.pg:
            import torch.distributed as dist
            if self._gloo is None:
                self._gloo = dist.new_group(backend="gloo")
            dist.barrier(group=self._gloo)

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()


# ------------------------------------------------------------------ CPU reference


def cpu_info():
    """CPU model name, logical and physical core counts of this host."""
    name = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    logical = os.cpu_count() or 1
    try:
        import psutil
        physical = psutil.cpu_count(logical=False) or logical
    except Exception:
        physical = logical
    return {"model": name, "nproc": logical, "physical_cores": physical}


def cpu_reference_sample(model_dir, seqs, budget_s, repeats=5, min_seqs=2):
    """Time the reference CPU path on the leading sequences of the batch (at
    least min_seqs of them) sized so `repeats` runs take about budget_s.
    Returns (median tokens/s, tokens, median seconds, n_seqs, threads, outputs
    of the sample, [tokens/s of every run])."""
    from oracle.ref import RefModel
    threads = os.cpu_count() or 1
    ref = RefModel(model_dir, threads=threads)
    probe = [seqs[0][:64]]
    ref.encode_batch(probe)  # warm-up: page in the weights
    t0 = time.perf_counter()
    ref.encode_batch(probe)
    per_tok = (time.perf_counter() - t0) / len(probe[0])
    per_run = budget_s / repeats
    n, tok = 0, 0
    while n < len(seqs):
        L = len(seqs[n])
        # attention grows with L; scale the probe rate by length / 4096 beyond the linear part
        est = per_tok * (tok + L) * (1.0 + (tok + L) / 4096.0)
        if n >= min_seqs and est > per_run:
            break
        tok += L
        n += 1
    sample = seqs[:n]
    rates, times, outs = [], [], None
    for _ in range(repeats):
        t0 = time.perf_counter()
        outs = ref.encode_batch(sample)
        dt = time.perf_counter() - t0
        times.append(dt)
        rates.append(tok / dt)
    ref.close()
    return (statistics.median(rates), tok, statistics.median(times), n, threads, outs, rates)


def parity_rows(gpu_rows, ref_rows):
    """Row-by-row agreement of GPU pooled rows with the reference CPU path."""
    a = np.asarray(gpu_rows, np.float64)
    b = np.asarray(ref_rows, np.float64)
    cos = (a * b).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1))
    return {"rows": int(len(a)), "min_cos": float(cos.min()),
            "max_abs": float(np.abs(a - b).max()), "gate_cos": 0.999,
            "ok": bool(np.isfinite(a).all() and cos.min() >= 0.999)}


def run_reference(args, dist):
    if dist.rank != 0:
        return 0
    spec, seqs = workload(0)
    d = synth.ensure_model(spec)
    from oracle import ref as oref
    if not oref.available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libffwd_ref.so not built (make -C oracle)"}))
        return 0
    from oracle.ref import RefModel
    threads = os.cpu_count() or 1
    ref = RefModel(d, threads=threads)
    # Size one step (a bounded sample) from a probe so K + W steps take minutes.
    probe = [seqs[0][:64]]
    ref.encode_batch(probe)
    t0 = time.perf_counter()
    ref.encode_batch(probe)
    per_tok = (time.perf_counter() - t0) / 64
    budget = max(2.0, 150.0 / (args.steps + args.warmup))
    n, tok = 0, 0
    while n < len(seqs):
        L = len(seqs[n])
        if n > 0 and per_tok * (tok + L) * (1.0 + (tok + L) / 4096.0) > budget:
            break
        tok += L
        n += 1
    sample = seqs[:n]
    for _ in range(args.warmup):
        ref.encode_batch(sample)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ref.encode_batch(sample)
        times.append(time.perf_counter() - t0)
    ref.close()
    info = cpu_info()
    total = sum(times)
    value = tok * len(times) / total
    sample_desc = (f"first {n} of the 128 seeded sequences ({tok} tokens) per step, "
                   f"reference CPU path (OpenBLAS f32, bf16 weights widened) on {threads} threads")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": 0,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded ids, random-init weights)",
        "config": {"workload": "Qwen3-Embedding-0.6B bf16, 128 seqs U[32,2048]+EOS, last-token+L2",
                   "sample_tokens_per_step": tok},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": sample_desc, "cpu_model": info["model"],
                         "nproc": info["nproc"], "physical_cores": info["physical_cores"],
                         "median_step_tokens_per_s": tok / statistics.median(times)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ ours


# DRAM bytes (read + write) per token of one gate/up GEMM launch, from an ncu
# capture of that kernel (profiles/gemm_gate_up_qwen3_0.6b.md gives the
# command and the raw figures); roofline.traffic scales it by the step's
# tokens.  Refresh it whenever the kernel changes.
GATE_UP_DRAM_BYTES_PER_TOKEN = 7976.4


def run_ours(args, dist):
    import torch
    from ffwd_b200 import native

    dist.init(torch)
    dev = dist.local if dist.world > 1 else 0
    torch.cuda.set_device(dev)
    spec, seqs = workload(dist.rank)
    if dist.rank == 0:
        d = synth.ensure_model(spec)
    dist.barrier(torch)
    d = synth.ensure_model(spec)

    peaks = {}
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peaks = json.load(open(pk))
    peak_tflops = peaks.get("bf16_tflops")
    peak_kind = "measured (burst)" if peak_tflops else "fallback"
    peak_tflops = peak_tflops or 1590.0

    m = native.B200Model(d, gemm_mode="bf16", devices=[dev])
    lens = np.array([len(s) for s in seqs], np.int32)
    offs = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T, B, H = int(offs[-1]), len(seqs), spec.hidden
    ids = np.concatenate(seqs).astype(np.int32)
    d_ids = torch.from_numpy(ids).to(f"cuda:{dev}")
    d_out = torch.empty((B, H), dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.ExternalStream(m.stream(), device=f"cuda:{dev}")

    def step():
        m.encode_device(d_ids.data_ptr(), offs, d_out.data_ptr(), sync=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---------------- device-resident timed region
    clocks = ClockSampler(dev)
    dist.barrier(torch)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.4)
    n0 = native.launch_count()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    launches = native.launch_count() - n0
    torch.cuda.synchronize()
    dist.barrier(torch)
    clk = clocks.stop()
    local_s = e0.elapsed_time(e1) / 1000.0
    value, max_s, total_tokens = whole_job_rate(dist, torch, T, args.steps, local_s)
    ms_per_step = 1000.0 * max_s / args.steps

    # ---------------- per-kernel timing (CUDA events on the backend's stream)
    reps = 10
    ops = {0: "gemm_qkv_qknorm_rope", 1: "attention_varlen_causal", 2: "gemm_o_resid",
           3: "rmsnorm", 4: "gemm_gate_up_swiglu", 5: "gemm_down_resid", 6: "rmsnorm"}
    op_ms = {}
    for op in (0, 1, 2, 3, 4, 5):
        m.run_op(op, layer=0, reps=2)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        m.run_op(op, layer=0, reps=reps)
        b.record(stream)
        b.synchronize()
        op_ms[ops[op]] = a.elapsed_time(b) / reps
    q = spec.n_heads * spec.head_dim
    kv = spec.n_kv_heads * spec.head_dim
    gu_flops = 2.0 * T * (2 * spec.intermediate) * H
    gu_s = op_ms["gemm_gate_up_swiglu"] / 1000.0
    achieved = gu_flops / gu_s / 1e12
    traffic_per_tok = GATE_UP_DRAM_BYTES_PER_TOKEN
    fpt, lin_fpt, attn_fpt = flops_per_token(spec, seqs)
    kernels = {
        "gemm_qkv_qknorm_rope": 2.0 * T * (q + 2 * kv) * H,
        "gemm_o_resid": 2.0 * T * H * q,
        "gemm_gate_up_swiglu": gu_flops,
        "gemm_down_resid": 2.0 * T * H * spec.intermediate,
        "attention_varlen_causal": 4.0 * q * float((lens.astype(np.float64) *
                                                   (lens + 1) / 2).sum()),
    }
    kernel_report = {k: {"ms": round(op_ms[k], 4),
                         "tflops": round(kernels[k] / (op_ms[k] / 1000.0) / 1e12, 1),
                         "frac_of_peak": round(kernels[k] / (op_ms[k] / 1000.0) / 1e12
                                               / peak_tflops, 3)}
                     for k in kernels}
    kernel_report["rmsnorm"] = {"ms": round(op_ms["rmsnorm"], 4),
                                "gbs": round(T * H * 6 / (op_ms["rmsnorm"] / 1000.0) / 1e9, 1)}
    model_tflops = T * fpt / (ms_per_step / 1000.0) / 1e12

    # ---------------- where one step's time goes (CUDA events, same stream)
    def timed(fn, reps=1):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        b.synchronize()
        return a.elapsed_time(b) / reps

    def layer_stack():
        for li in range(spec.n_layers):
            for op in range(7):
                m.run_op(op, layer=li)

    embed_ms = timed(lambda: m.run_op(7), reps)
    pool_ms = timed(lambda: m.run_op(8), reps)
    layer_stack()
    stack_ms = timed(layer_stack, 2)
    ops_sum_ms = spec.n_layers * sum(op_ms[ops[o]] for o in (0, 1, 2, 4, 5)) \
        + spec.n_layers * 2 * op_ms["rmsnorm"]
    step_split = {
        "step_ms": round(ms_per_step, 3),
        "embedding_ms": round(embed_ms, 3),
        "layer_stack_ms": round(stack_ms, 3),
        "per_op_sum_ms": round(ops_sum_ms, 3),
        "pool_ms": round(pool_ms, 3),
        "host_and_gaps_ms": round(ms_per_step - embed_ms - stack_ms - pool_ms, 3),
        "note": "layer_stack re-issues the 28 x 7 layer launches back to back; per_op_sum is "
                "28 x the per-op times measured in isolation; host_and_gaps = step - embedding "
                "- layer stack - pool (host work list, H2D of ids/offsets/items, sync)",
    }
    gpu_rows = d_out.cpu().numpy()

    # ---------------- attention by sequence length: uniform-length batches of
    # about the bench's token count (layer 0 of the same model), CUDA events
    attn_by_len = {}
    rng = np.random.default_rng(7)
    for Lb in (256, 512, 1024, 2048, 8192):
        nb = max(1, T // Lb)
        ids_b = torch.from_numpy(rng.integers(0, 151642, size=nb * Lb).astype(np.int32)).to(
            f"cuda:{dev}")
        offs_b = (np.arange(nb + 1) * Lb).astype(np.int32)
        out_b = torch.empty((nb, H), dtype=torch.float32, device=f"cuda:{dev}")
        m.encode_device(ids_b.data_ptr(), offs_b, out_b.data_ptr(), sync=True)
        m.run_op(1, layer=0, reps=2)
        a_ms = timed(lambda: m.run_op(1, layer=0), reps)
        fl = 4.0 * q * nb * Lb * (Lb + 1) / 2
        attn_by_len[f"L{Lb}"] = {"ms": round(a_ms, 4), "tflops": round(fl / (a_ms / 1e3) / 1e12, 1),
                                 "frac_of_peak": round(fl / (a_ms / 1e3) / 1e12 / peak_tflops, 3)}
    kernel_report["attention_by_length"] = attn_by_len

    # ---------------- end to end through the public API (host buffers)
    os.environ["FFWD_B200_DEVICES"] = str(dev)
    m.close()
    del m
    api = native.FfwdApi(d, gemm_mode="bf16")
    ins = (native.ffwd_input_t * B)()
    keep = [np.ascontiguousarray(s, dtype=np.int32) for s in seqs]
    for i, a in enumerate(keep):
        ins[i].ids = a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
        ins[i].n_tokens = len(a)
    out = np.zeros((B, H), np.float32)
    for _ in range(max(1, args.warmup)):
        assert api.encode_batch_into(ins, B, out.ctypes.data) == 0
    dist.barrier(torch)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        assert api.encode_batch_into(ins, B, out.ctypes.data) == 0
    e2e_local = time.perf_counter() - t0
    e2e_max = dist.max(torch, e2e_local)
    e2e_value = total_tokens * args.steps / e2e_max
    # attention work list: pairs of 128-row query blocks per key/value head
    # (AttnItem, 6 ints), plus the ids and row offsets
    rep = spec.n_heads // spec.n_kv_heads
    n_items = int(sum((L + 127) // 128 for L in lens)) * spec.n_kv_heads * ((rep + 1) // 2)
    h2d = T * 4 + (B + 1) * 4 + n_items * 24
    d2h = B * H * 4 + 4

    # p50 micro-batch latency, server packing (length-sorted, <= 32 inputs,
    # <= 16384 tokens; tools/server/handlers.c:51-120, models.c:269-276)
    order = sorted(range(B), key=lambda i: len(seqs[i]))
    batches, cur, ctok = [], [], 0
    for i in order:
        L = len(seqs[i])
        if cur and (len(cur) >= 32 or ctok + L > 16384):
            batches.append(cur)
            cur, ctok = [], 0
        cur.append(i)
        ctok += L
    if cur:
        batches.append(cur)
    lat = []
    for bi, bidx in enumerate(batches):
        sub = (native.ffwd_input_t * len(bidx))()
        for j, i in enumerate(bidx):
            sub[j] = ins[i]
        o = np.zeros((len(bidx), H), np.float32)
        api.encode_batch_into(sub, len(bidx), o.ctypes.data)  # warm this shape
        t0 = time.perf_counter()
        assert api.encode_batch_into(sub, len(bidx), o.ctypes.data) == 0
        lat.append((time.perf_counter() - t0) * 1000.0)
    api.close()

    # ---------------- CPU baseline and parity (rank 0): the reference CPU path on
    # the leading sequences of this rank's batch, its rows compared with ours.
    cpu, parity = None, None
    if dist.rank == 0 and not args.no_cpu:
        from oracle import ref as oref
        if oref.available():
            budget = args.cpu_budget if dist.world == 1 else 4.0
            reps = 5 if dist.world == 1 else 1
            v, tok, dt, n, thr, ref_rows, rates = cpu_reference_sample(d, seqs, budget, reps)
            parity = parity_rows(gpu_rows[:n], ref_rows)
            parity["sequences"] = f"first {n} of the bench batch ({tok} tokens), 28 layers, " \
                                  "vocab 151669, vs the reference CPU path (oracle/_ref)"
            if dist.world == 1:
                info = cpu_info()
                cpu = {"value": v, "unit": UNIT, "cores": thr, "kind": "reference",
                       "sample": f"first {n} of the 128 seeded sequences ({tok} tokens, "
                                 f"median {dt:.1f} s of {reps} runs), reference CPU path "
                                 f"(OpenBLAS f32) via oracle/_ref",
                       "runs_tokens_per_s": [round(r, 1) for r in rates],
                       "cpu_model": info["model"], "nproc": info["nproc"],
                       "physical_cores": info["physical_cores"]}
        else:
            parity = {"ok": False, "error": "oracle/_ref/libffwd_ref.so not built"}

    # ---------------- the reference's own CUDA backend on the same GPU (N = 1):
    # libffwd/cuda.cu built unmodified for sm_100a (cuBLAS / cuBLASLt GEMMs;
    # attention through cuDNN SDPA, its default for this shape, and through its
    # built-in mma.sync flash kernel), in a process of its own.
    gpu_ref = None
    if dist.world == 1 and not args.no_gpu_ref:
        gpu_ref = gpu_reference_arms(d, args, gpu_rows, e2e_value)

    # ---------------- the library's own multi-GPU sharder (N > 1): rank 0 encodes
    # all ranks' batches in one ffwd_encode_batch call over devices 0..N-1 while
    # the other ranks wait on a CPU (gloo) barrier, so no collective kernel
    # occupies their GPUs.
    sharded = None
    if dist.world > 1 and not args.no_sharded:
        if dist.rank == 0:
            sharded = sharded_leg(d, spec, dist.world, args)
        dist.cpu_barrier()
    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded token ids, random-init bf16 safetensors weights)",
            "config": {
                "workload": "Qwen3-Embedding-0.6B bf16 (28 layers, hidden 1024, 16/8 heads x 128, "
                            "SwiGLU 3072), 128 seqs/GPU U[32,2048]+EOS, last-token pooling + L2",
                "tokens_per_gpu_step": T, "sequences_per_gpu_step": B,
                "parallelism": f"dp{dist.world} (sequence sharding, no collective)",
                "l2": "inputs larger than L2 (weights 1.2 GB, activations > 1 GB per step)",
            },
            "p50_batch_latency_ms": statistics.median(lat) if lat else None,
            "model_tflops": model_tflops,
            "gflop_per_token": fpt / 1e9,
            "roofline": {
                "kernel": "gemm_gate_up_swiglu (tcgen05, fused SwiGLU epilogue)",
                "bound": "tensor", "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
                "frac": achieved / peak_tflops, "peak_source": peak_kind,
                "flops_per_launch": gu_flops,
                "traffic": traffic_per_tok * T,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                  "gate/up launch, per token, scaled to this step's tokens",
            },
            "kernels": kernel_report,
            "step_split": step_split,
            "parity": parity,
            "sharded_e2e": sharded,
            "gpu_reference": gpu_ref,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "ffwd_encode_batch (libffwd_b200_api.so)"},
            "gpu_launches": launches,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    dist.close()
    if parity is not None and not parity.get("ok"):
        sys.stderr.write(f"parity check failed: {parity}\n")
        return 1
    return 0


def gpu_reference_arms(d, args, gpu_rows, e2e_value):
    """Time the reference CUDA backend (oracle/_ref/libffwd_refcuda.so, built by
    `make -C oracle cuda`) on this rank's batch through ffwd_cuda_encode_batch
    with host buffers, once per attention route, each in a child process."""
    import tempfile
    from oracle import refcuda
    if not refcuda.available():
        return {"unavailable": "oracle/_ref/libffwd_refcuda.so not built (make -C oracle cuda)"}
    arms = {}
    steps = max(1, min(args.steps, 5))
    for name, env in (("cudnn_sdpa", {}), ("builtin_flash", {"FFWD_CUDA_SDPA": "0"})):
        fd, npy = tempfile.mkstemp(suffix=".npy")
        os.close(fd)
        try:
            r = subprocess.run([sys.executable, "-m", "oracle.refcuda", d, str(steps), "2", "1", npy],
                               cwd=ROOT, env={**os.environ, **env}, capture_output=True,
                               text=True, timeout=600)
            lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
            if r.returncode != 0 or not lines:
                arms[name] = {"error": (r.stderr or r.stdout)[-300:]}
                continue
            arm = json.loads(lines[-1])
            rows = np.load(npy)
            a = np.asarray(gpu_rows, np.float64)
            bb = rows.astype(np.float64)
            cos = (a * bb).sum(1) / (np.linalg.norm(a, axis=1) * np.linalg.norm(bb, axis=1))
            arm["min_cos_vs_ours"] = float(cos.min())
            arm["ours_e2e_over_this"] = e2e_value / arm["value"]
            arm["attention_route"] = (
                "built-in kernels (cuDNN unavailable)" if "using built-in" in r.stderr
                else "cuDNN SDPA" if name == "cudnn_sdpa" else "attn_stream_tc128 (mma.sync)")
            arms[name] = arm
        except subprocess.TimeoutExpired:
            arms[name] = {"error": "timed out"}
        finally:
            if os.path.exists(npy):
                os.unlink(npy)
    arms["note"] = ("reference libffwd/cuda.cu + cuda_sdpa.cu unmodified, nvcc 12.9 sm_100a, "
                    "ffwd_cuda_encode_batch on the same 128 sequences, host ids in / rows out, "
                    "wall clock of the synchronous call, --gpu-gemm-mode bf16, bf16 weights")
    return arms


# --configs: every BASELINE model family on one GPU, ours beside the reference's
# own CUDA backend.  (config, gemm mode, sequences per call, spec overrides)
SWEEP = [
    ("minilm", "f32", None, {}),
    ("bge-base", "f32", None, {}),
    ("bge-base-bf16", "bf16", None, {}),
    ("xlmr-large", "bf16", None, {}),
    ("qwen3-0.6b", "bf16", None, {}),
    # Qwen3-Embedding-8B shape at 4 of its 36 layers (writing the full random
    # model would take minutes per box); a micro-batch of 4 documents x 8192.
    ("qwen3-8b", "bf16", 4, {"n_layers": 4}),
]


def config_sweep(args):
    """One JSON line per BASELINE config: tokens/s through ffwd_b200_encode_batch
    (host ids in, host rows out, wall clock of the synchronous call, the same
    contract as the reference's ffwd_cuda_encode_batch) and the reference CUDA
    backend's tokens/s on the same batch in a child process, with the minimum
    row cosine between the two."""
    import tempfile
    from ffwd_b200 import native
    from oracle import refcuda
    steps = max(1, args.steps)
    for name, mode, batch, over in SWEEP:
        spec = synth.spec(name, **over) if over else synth.CONFIGS[name]
        d = synth.ensure_model(spec)
        seqs = synth.token_batch(name, seed=1, batch=batch)
        tokens = sum(len(q) for q in seqs)
        m = native.B200Model(d, gemm_mode=mode, devices=[0])
        for _ in range(2):
            ours = m.encode_batch(seqs)
        t0 = time.perf_counter()
        for _ in range(steps):
            ours = m.encode_batch(seqs)
        dt = (time.perf_counter() - t0) / steps
        m.close()
        line = {"config": spec.name, "gemm_mode": mode, "sequences": len(seqs),
                "tokens_per_call": tokens, "ours": {"value": tokens / dt, "unit": UNIT,
                                                    "ms_per_call": 1000.0 * dt}}
        if refcuda.available():
            fd, npy = tempfile.mkstemp(suffix=".npy")
            os.close(fd)
            try:
                r = subprocess.run([sys.executable, "-m", "oracle.refcuda", d, str(steps), "2",
                                    "1", npy, name, mode, str(len(seqs))], cwd=ROOT,
                                   capture_output=True, text=True, timeout=900)
                out = [l for l in r.stdout.splitlines() if l.startswith("{")]
                if r.returncode != 0 or not out:
                    line["reference_cuda"] = {"error": (r.stderr or r.stdout)[-300:]}
                else:
                    ref = json.loads(out[-1])
                    rows = np.load(npy).astype(np.float64)
                    a = ours.astype(np.float64)
                    cos = (a * rows).sum(1) / (np.linalg.norm(a, axis=1) *
                                               np.linalg.norm(rows, axis=1))
                    line["reference_cuda"] = {"value": ref["value"], "unit": UNIT,
                                              "ms_per_call": ref["ms_per_call"]}
                    line["ours_over_reference_cuda"] = (tokens / dt) / ref["value"]
                    line["min_cos_vs_reference_cuda"] = float(cos.min())
            except subprocess.TimeoutExpired:
                line["reference_cuda"] = {"error": "timed out"}
            finally:
                if os.path.exists(npy):
                    os.unlink(npy)
        else:
            line["reference_cuda"] = {"unavailable": "oracle/_ref/libffwd_refcuda.so not built"}
        print(json.dumps(line), flush=True)
    return 0


def sharded_leg(d, spec, world, args):
    """ffwd_encode_batch of all ranks' batches (world x 128 sequences) through
    the public API with FFWD_B200_DEVICES=0..world-1: the library's LPT
    sharder, one host thread and stream per GPU, rows copied into the
    caller's buffer."""
    from ffwd_b200 import native
    os.environ["FFWD_B200_DEVICES"] = ",".join(str(i) for i in range(world))
    seqs = []
    for r in range(world):
        seqs += synth.token_batch(CONFIG, seed=1 + r)
    api = native.FfwdApi(d, gemm_mode="bf16")
    ins, keep = native._pack_inputs(seqs)
    out = np.zeros((len(seqs), spec.hidden), np.float32)
    for _ in range(2):
        assert api.encode_batch_into(ins, len(seqs), out.ctypes.data) == 0
    steps = max(1, args.steps)
    t0 = time.perf_counter()
    for _ in range(steps):
        assert api.encode_batch_into(ins, len(seqs), out.ctypes.data) == 0
    dt = (time.perf_counter() - t0) / steps
    st = api.shard_stats()
    api.close()
    tokens = sum(len(q) for q in seqs)
    ms = [x[2] for x in st]
    return {"value": tokens / dt, "unit": UNIT, "n_devices": world, "sequences": len(seqs),
            "tokens_per_call": tokens, "ms_per_call": 1000.0 * dt, "calls": steps,
            "per_device": [{"seqs": a, "tokens": b, "ms": round(c, 2)} for a, b, c in st],
            "imbalance_max_over_mean": max(ms) / (sum(ms) / len(ms)) if ms else None,
            "api": "ffwd_encode_batch (libffwd_b200_api.so), FFWD_B200_DEVICES=0..N-1, host "
                   "buffers, wall clock of the synchronous call"}


def whole_job_rate(dist, torch, tokens_per_step: int, steps: int, local_s: float):
    """Weak-scaling aggregate: all ranks' tokens over the slowest rank's time.
    Returns (tokens/s, max seconds over ranks, total tokens per step)."""
    max_s = dist.max(torch, local_s)
    total = dist.sum(torch, float(tokens_per_step))
    return total * steps / max_s, max_s, total


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-gpu-ref", action="store_true",
                    help="skip timing the reference CUDA backend (N = 1)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the multi-GPU sharder leg (N > 1)")
    ap.add_argument("--configs", action="store_true",
                    help="instead of the headline: every BASELINE config on GPU 0, beside "
                         "the reference's own CUDA backend, one JSON line each")
    args = ap.parse_args()
    if args.configs:
        return config_sweep(args)
    if args.warmup < 3:
        args.warmup = 3
    dist = Dist()
    if args.impl == "reference":
        return run_reference(args, dist)
    return run_ours(args, dist)


if __name__ == "__main__":
    sys.exit(main())

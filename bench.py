#!/usr/bin/env python
"""bench.py — decode+prefill tok/s of the int8 forward engine: the Llama-3-8B shape, 64 sequences of 512 prompt tokens
+ 256 greedy tokens, sharded by sequence across 1/2/4/8 GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config c5|c4|c3|c2]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One step is one batch of the workload through the engine's C ABI: `seqs` sequences in all (64) of `prompt` (512)
seeded random prompt tokens, split evenly over the ranks; each rank prefills its sequences in blocks (b200fwd_run),
then makes `gen` (256) greedy tokens each on the device (b200fwd_generate_greedy); then the ranks all-gather every
sequence's generated ids (NCCL, the one collective on the data path). Weights: N(0, 0.02), quantized to int8 with one
float32 scale per group of 32, made on the device and replicated on every GPU (8.4 GB; far larger than L2, so every
step reads them from HBM). The total work is fixed as N grows (strong scaling).

value: tokens processed (prompt positions 0..510 and the 256 greedy positions of every sequence) / the device time
of the step (CUDA events around the engine's calls and the all-gather, max over ranks). e2e: the same through the
host-buffer calls, by the host clock around each step, host-to-device copies of the prompts and device-to-host reads
of the generated ids inside. roofline: the dominant kernel (the int8 matmul) timed alone at the decode step's shapes
with CUDA events, algorithmic bytes over its duration against the measured HBM copy bandwidth. c4_matmul: the matmul
alone at the 8B projection shapes at M = 1, 8, 64, 512 tokens; c3_decode_attention and c2_prefill_attention: the
decode attention and the tensor-core prefill attention at their own configurations. cpu_baseline: the oracle (a C++ restatement of the
reference's WASM-SIMD path, built for the host's own CPU, every host thread) on a bounded sample of the workload.

--impl reference: the reference's CPU path on this host (the oracle port: the reference's AssemblyScript kernels
cannot be built or run here), every host thread, one sequence of the same model per step.
"""
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
sys.path.insert(0, str(ROOT / "pyodide-llm_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import numpy as np  # noqa: E402

METRIC = "decode+prefill tok/s, 8B-shape int8 (64 seq x (512 prompt + 256 greedy), sharded across the GPUs)"
HEADER = (4096, 14336, 32, 32, 8, -128256, 8192)
THETA = 500000.0
BOS = 1


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--seqs", type=int, default=64, help="sequences in all (split evenly over the ranks)")
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--gen", type=int, default=256)
    p.add_argument("--block", type=int, default=64, help="prompt positions per prefill call")
    p.add_argument("--cpu-prompt", type=int, default=16)
    p.add_argument("--cpu-gen", type=int, default=8)
    p.add_argument("--model", default="llama3-8b", choices=["llama3-8b", "stories15m"])
    p.add_argument("--config", default="c5", choices=["c5", "c4", "c3", "c2"],
                   help="c5: the end-to-end line (default); c4: only the int8 matmul sweep over the 8B projection "
                        "shapes at M = 1, 8, 64, 512; c3: only decode attention over 64 sequences with contexts "
                        "U[512, 8192]; c2: only causal prefill attention on the tensor cores, 4 x 2048 tokens, 8 heads "
                        "of 64 (all three also part of the c5 line)")
    p.add_argument("--matmul", default=None, metavar="ROWSxN",
                   help="time the int8 matmul alone (b200k_matmul_q8s) at ROWSxN with --seqs tokens, one matrix of "
                        "random weights on the device: the small case the kernel profiles are captured on")
    return p.parse_args()


def model_of(args):
    if args.model == "stories15m":
        return (288, 768, 6, 6, 6, 32000, 256), 10000.0
    return HEADER, THETA


def cpu_model():
    sys.path.insert(0, str(ROOT / "oracle"))
    from build_oracle import cpu_model as model

    return model()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class Clocks:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = str(index), [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.index], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def cpu_sample(ckpt_host, plan, args, threads):
    """The oracle on one sequence: cpu_prompt prompt tokens (one block) then cpu_gen greedy steps. tok/s."""
    import oracle

    oracle.use_native()
    t0 = time.perf_counter()
    eng = oracle.OracleEngine(ckpt_host, plan, half_keys=1, threads=threads)
    setup = time.perf_counter() - t0
    rng = np.random.default_rng(7)
    vocab = abs(HEADER[5]) if args.model == "llama3-8b" else 32000
    prompt = [BOS] + [int(t) for t in rng.integers(0, vocab, args.cpu_prompt - 1)]
    t0 = time.perf_counter()
    eng.forward_many(prompt[:-1], 0)
    token = prompt[-1]
    for s in range(args.cpu_gen):
        token = int(np.argmax(eng.forward(token, len(prompt) - 1 + s)))
    dt = time.perf_counter() - t0
    eng.close()
    return (args.cpu_prompt + args.cpu_gen) / dt, dt, setup


def workload_prompts(seqs, prompt, vocab):
    """every sequence's prompt (seeded: the same workload at every GPU count), each starting with BOS"""
    rng = np.random.default_rng(1000)
    prompts = rng.integers(0, vocab, size=(seqs, prompt), dtype=np.int32)
    prompts[:, 0] = BOS
    return prompts


def shard(seqs, world, rank):
    """the sequences rank `rank` of `world` takes: an even split (every rank the same count, so that the all-gather
    of the generated ids has equal parts)"""
    if seqs % world:
        raise SystemExit(f"{seqs} sequences do not split evenly over {world} GPUs")
    per = seqs // world
    return slice(rank * per, (rank + 1) * per)


def gather_ids(ids, world, device):
    """every rank's generated ids [per rank][steps] gathered on every rank in rank order [seqs][steps] (NCCL
    all-gather over NVLink; the one collective on the data path). Returns the gathered device tensor."""
    import torch
    import torch.distributed as dist

    local = torch.from_numpy(np.ascontiguousarray(ids, np.int32)).to(device, non_blocking=True)
    if world == 1:
        return local
    out = torch.empty((world * local.shape[0], local.shape[1]), dtype=torch.int32, device=device)
    dist.all_gather_into_tensor(out, local)
    return out


def max_over_ranks(x, world, device):
    """the largest of every rank's x (the job's time is its slowest rank's)"""
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def workload_config(args, world):
    """the bench line's `config`, the same for both arms"""
    S, P, G = args.seqs, args.prompt, args.gen
    return {"workload": f"{args.model} int8 end to end: {S} sequences x ({P} prompt tokens prefilled in blocks of "
                        f"{args.block} positions + {G} greedy tokens), sharded by sequence over {world} GPU(s), "
                        f"the generated ids all-gathered",
            "model": args.model, "global_batch": S, "seq_len": P + G, "prompt": P, "generated": G,
            "tokens_per_sequence": P - 1 + G,
            "parallelism": f"dp{world} (independent sequences, weights replicated)", "kv": "float16",
            "activations": "7-bit + bias 64 (relaxed)", "float_order": "exact (the reference's)",
            "l2": "inputs larger than L2: 8.4 GB of weights read per step"}


def reference_arm(args):
    """bench.py --impl reference: the oracle port of the reference's CPU path, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch

    from b200fwd import synthetic

    header, theta = model_of(args)
    torch.set_num_threads(host_threads())
    file = synthetic.make(header, seed=0, device="cpu")
    plan = synthetic.plan_for(header, file, theta)
    ckpt = file.numpy()
    threads = host_threads()
    times = []
    for i in range(args.warmup + args.steps):
        v, dt, _ = cpu_sample(ckpt, plan, args, threads)
        if i >= args.warmup:
            times.append(dt)
    per = float(np.mean(times))
    value = (args.cpu_prompt + args.cpu_gen) / per
    sample = (f"1 sequence per step: {args.cpu_prompt} prompt tokens in one block + {args.cpu_gen} greedy steps, "
              f"the whole {args.model} int8 model")
    out = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
           "config": workload_config(args, args.gpus),
           "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample,
                            "cpu": cpu_model(), "build": "g++ -O3 -march=native -ffp-contract=off"},
           "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference's AssemblyScript/WASM kernels cannot be built here (no node, no asc); the oracle "
                   "is their C++ restatement, pinned to the reference's bit-exact checks"}
    print(json.dumps(out), flush=True)
    return 0


# measured DRAM bytes / algorithmic bytes of the decode-shape matmul launches (ncu, one launch each): q8_gemm_tc at
# 28672 x 4096 136.25 / 139.76 MB, q8_gemm_lanes at 4096 x 14336 67.91 / 68.14 MB; weighted by the bytes each kernel
# moves in a decode pass at 64 tokens (w1|w3 and the classifier on the first, q|k|v, o and w2 on the second: 5096 and
# 3793 MB)
TRAFFIC_RATIO = (5096 * (136.25 / 139.76) + 3793 * (67.91 / 68.14)) / (5096 + 3793)


def matmul_roofline(eng, M, peaks, reps=3):
    """The int8 matmul (the dominant kernel) alone, as the engine launches it at the decode step's M tokens: every
    layer's q|k|v, o, w1|w3 and w2, then the classifier (8.9 GB of weights, far beyond L2), back to back on the
    engine's stream, timed with CUDA events (b200fwd_time_matmuls), right after the timed steps on the same engine."""
    ms, nbytes, launches = eng.time_matmuls(M, reps)
    per_launch_s = ms / 1e3 / launches
    per_launch_bytes = nbytes / launches
    achieved = per_launch_bytes / per_launch_s / 1e9
    peak = float(peaks["hbm_gbs"])
    return {"kernel": "q8_gemm_tc + q8_gemm_lanes (int8 group-32 matmul, tcgen05, exact order)" if M >= 2 else
            "matvec_kernel (int8 group-32 matmul, exact order)", "bound": "hbm",
            "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            # DRAM bytes per launch: ncu (dram__bytes_read.sum + dram__bytes_write.sum) on one launch of each
            # kernel at 64 tokens read and wrote 0.975 and 0.997 of its algorithmic bytes (every byte once); their
            # byte-weighted ratio over this pass's launches
            "traffic": TRAFFIC_RATIO * per_launch_bytes,
            "traffic_source": "ncu, 28672x4096 (q8_gemm_tc) and 4096x14336 (q8_gemm_lanes) at 64 tokens, scaled",
            "M": M, "per_launch_us": per_launch_s * 1e6, "launches_per_pass": launches,
            "algorithmic_bytes_per_launch": per_launch_bytes, "pass_ms": ms}


C4_SHAPES = {"qkv": "6144x4096", "o": "4096x4096", "w13": "28672x4096", "w2": "4096x14336"}


def c4_sweep(eng, peaks, counts=(1, 8, 64, 512), reps=2):
    """The int8 matmul at the 8B projection shapes (q|k|v 6144x4096, o 4096x4096, w1|w3 28672x4096, w2 4096x14336)
    at M tokens, each shape over all 32 layers' copies in turn so that no launch finds its weights in L2
    (b200fwd_time_matmul_kinds), on the engine's activations. M <= 64: HBM-bound (bytes = rows n 9/8 + M n 9/8 +
    4 M rows); M = 512: ops = 2 M rows n against twice the measured bf16 tensor rate (the int8 rate), and the exact
    epilogue's CUDA-core floor (3 float32 operations per row, token and group of 32 at 128 lanes x SM clock)."""
    hbm = float(peaks["hbm_gbs"])
    int8_tops = 2.0 * float(peaks["bf16_tflops"])
    sm_hz = float(peaks.get("sm_max_mhz", 1965.0)) * 1e6
    out = {}
    for m in counts:
        kinds = eng.time_matmul_kinds(m, reps)
        row = {}
        for k, shape in C4_SHAPES.items():
            us, nbytes = kinds[k]
            rows, n = (int(v) for v in shape.split("x"))
            gbs = nbytes / (us * 1e-6) / 1e9
            e = {"us": round(us, 2), "gb_s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4)}
            if m >= 512:
                tops = 2.0 * m * rows * n / (us * 1e-6) / 1e12
                floor_us = 3.0 * m * rows * (n // 32) / (148 * 128 * sm_hz) * 1e6
                e.update({"tops": round(tops, 1), "int8_tensor_frac": round(tops / int8_tops, 4),
                          "fp32_epilogue_floor_us": round(floor_us, 2)})
            row[shape] = e
        out[f"M={m}"] = row
    return {"what": "int8 group-32 matmul (exact order) per launch, every layer's copy in turn (no L2 hits)",
            "kernel": "matvec_kernel (CUDA cores) for one token, q8_gemm_tc (tcgen05) from 2",
            "peak_hbm_gbs": hbm, "int8_tops_peak": int8_tops, "table": out}


def c3_decode_attention(peaks, reps=5):
    """Decode attention at the Llama-3-8B shape (b200k_attention_batch, exact order): 64 sequences, one query token
    each, contexts drawn from U[512, 8192] (seed 2), 32 query / 8 key-value heads of 128, float16 cache N(0, 1)
    (2.1 GB with the unused tails; 1.14 GB read, far above L2). Bytes: every sequence's keys and values read once
    (sum of contexts x 8 x 128 x 2 x 2) + the queries read and the outputs written; HBM-bound."""
    import ctypes

    import torch

    from b200fwd import abi

    lib = abi.load()
    nh, nkv, hs, seqs = 32, 8, 128, 64
    kvd = nkv * hs
    ctx = np.random.default_rng(2).integers(512, 8193, seqs).astype(np.int32)
    P = int(ctx.max())
    g = torch.Generator(device="cuda").manual_seed(2)
    kc = torch.randn((seqs, P, kvd), generator=g, device="cuda", dtype=torch.float32).half()
    vc = torch.randn((seqs, P, kvd), generator=g, device="cuda", dtype=torch.float32).half()
    q = torch.randn((seqs, nh * hs), generator=g, device="cuda", dtype=torch.float32)
    out = torch.empty_like(q)
    att = torch.empty((seqs, nh, P), device="cuda", dtype=torch.float32)
    seq = torch.arange(seqs, dtype=torch.int32, device="cuda")
    pos = torch.from_numpy(ctx - 1).to("cuda")
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream

    def launch():
        abi.check(lib.b200k_attention_batch(ptr(out), ptr(q), ptr(kc), ptr(vc), ptr(att), ptr(seq), ptr(pos), seqs,
                                            P * kvd, P, nh, nkv, hs, 1, ctypes.c_void_p(stream)), "attention_batch")

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        launch()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / reps
    nbytes = float(ctx.sum()) * kvd * 2 * 2 + 2 * seqs * nh * hs * 4
    hbm = float(peaks["hbm_gbs"])
    gbs = nbytes / (us * 1e-6) / 1e9
    res = {"what": "decode attention, 64 sequences x 1 token, contexts U[512, 8192] seed 2, 32/8 heads of 128, "
                   "float16 cache, exact order (b200k_attention_batch)", "us": us, "bytes": nbytes,
           "gb_s": gbs, "hbm_frac": gbs / hbm, "peak_hbm_gbs": hbm, "sum_context": int(ctx.sum()),
           "tokens_per_s": seqs / (us * 1e-6)}
    del kc, vc, att
    torch.cuda.empty_cache()
    return res


def c2_prefill_attention(peaks, reps=20):
    """Causal attention of whole prompts on the tensor cores (b200k_prefill_attention: RoPE + float16 conversion,
    then the tcgen05 flash-attention kernel): 4 sequences of 2048 tokens, 8 heads = 8 kv heads of 64, RoPE theta
    1e4, Q/K/V N(0, 1) (seed 1). FLOPs: the causal QK^T and PV, 4 B H d S (S + 1) / 2 = 17.18 G, against the measured
    dense bf16 tensor rate (the float16 rate is the same)."""
    import ctypes

    import torch

    from b200fwd import abi
    from b200fwd import checkpoint as ck

    lib = abi.load()
    B, S, H, D = 4, 2048, 8, 64
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn((B, S, H, D), generator=g, device="cuda") for _ in range(3))
    cos, sin = ck.rope_tables(S, D, 10000.0)
    cos_t = torch.from_numpy(np.ascontiguousarray(cos, np.float32)).cuda()
    sin_t = torch.from_numpy(np.ascontiguousarray(sin, np.float32)).cuda()
    size = ctypes.c_uint64()
    abi.check(lib.b200k_prefill_attention_scratch(B, S, H, H, D, ctypes.byref(size)))
    scratch = torch.empty(int(size.value) + 256, dtype=torch.uint8, device="cuda")
    out = torch.empty_like(q)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def launch():
        abi.check(lib.b200k_prefill_attention(ptr(out), ptr(q), ptr(k), ptr(v), ptr(cos_t), ptr(sin_t), B, S, H, H,
                                              D, ptr(scratch), stream), "prefill_attention")

    for _ in range(3):
        launch()
    abi.check(lib.b200k_prefill_attention_check(ptr(scratch), B, S, H, H, D, stream))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        launch()
    b.record()
    torch.cuda.synchronize()
    abi.check(lib.b200k_prefill_attention_check(ptr(scratch), B, S, H, H, D, stream))
    us = a.elapsed_time(b) * 1e3 / reps
    flops = 4.0 * B * H * D * S * (S + 1) / 2
    tf = flops / (us * 1e-6) / 1e12
    peak = float(peaks["bf16_tflops"])
    return {"what": "causal prefill attention, 4 x 2048 tokens, 8/8 heads of 64, RoPE 1e4, float16 tensor cores "
                    "(kind::f16, float32 accumulate), within 1e-3 of float64", "us": us, "flops": flops,
            "tflops": tf, "tensor_frac": tf / peak, "peak_tflops": peak,
            "note": "time of the whole call: the RoPE/float16 prologue and the flash-attention kernel"}


def c2_arm(args):
    """bench.py --config c2: prefill attention alone (one GPU)."""
    import torch

    torch.cuda.set_device(0)
    peaks, which = measured_peaks()
    res = c2_prefill_attention(peaks)
    res["peak_source"] = which
    print(json.dumps({"config": "c2", **res}), flush=True)
    return 0


def c3_arm(args):
    """bench.py --config c3: decode attention alone (one GPU)."""
    import torch

    torch.cuda.set_device(0)
    peaks, which = measured_peaks()
    res = c3_decode_attention(peaks)
    res["peak_source"] = which
    print(json.dumps({"config": "c3", **res}), flush=True)
    return 0


def c4_arm(args):
    """bench.py --config c4: the matmul sweep alone on the 8B-shape engine (one GPU)."""
    import torch

    from b200fwd import synthetic
    from b200fwd.forward import Engine

    torch.cuda.set_device(0)
    header, theta = model_of(args)
    file = synthetic.make(header, seed=0, device="cuda")
    plan = synthetic.plan_for(header, file, theta)
    eng = Engine(file.data_ptr(), plan, checkpoint_on_device=True, size=file.numel(), half_keys=True, slots=1,
                 max_tokens=512, capacity=512)
    del file
    torch.cuda.empty_cache()
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, abs(header[5]), 512).astype(np.int32)
    eng.run(np.zeros(512, np.int32), tokens, np.arange(512, dtype=np.int32))  # activations of a real block
    peaks, which = measured_peaks()
    res = c4_sweep(eng, peaks)
    res["peak_source"] = which
    print(json.dumps({"config": "c4", **res}), flush=True)
    eng.release()
    return 0


def b200_arm(args):
    import ctypes

    import torch
    import torch.distributed as dist

    from b200fwd import abi, synthetic
    from b200fwd.forward import Engine

    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    header, theta = model_of(args)
    vocab = abs(header[5])
    mine = shard(args.seqs, world, rank)
    S, P, G = mine.stop - mine.start, args.prompt, args.gen
    file = synthetic.make(header, seed=0, device="cuda")
    plan = synthetic.plan_for(header, file, theta)
    ckpt_host = file.cpu().numpy() if rank == 0 else None
    eng = Engine(file.data_ptr(), plan, checkpoint_on_device=True, size=file.numel(), half_keys=True, slots=S,
                 max_tokens=S * args.block, capacity=P + G, device=local)
    del file
    torch.cuda.empty_cache()
    prompts = workload_prompts(args.seqs, P, vocab)[mine]
    stream = eng.stream()
    st = torch.cuda.ExternalStream(stream)
    slots_all = np.arange(S, dtype=np.int32)

    def step(events=None):
        """one batch: prefill positions 0..P-2 in blocks, then G greedy steps from the last prompt token"""
        torch.cuda.nvtx.range_push("prefill")
        for b0 in range(0, P - 1, args.block):
            n = min(args.block, P - 1 - b0)
            sl = np.repeat(slots_all, n)
            tk = prompts[:, b0:b0 + n].reshape(-1)
            ps = np.tile(np.arange(b0, b0 + n, dtype=np.int32), S)
            if events is not None:
                events.append(torch.cuda.Event(enable_timing=True))
                events[-1].record(st)
            eng.run(sl, tk, ps)
            if events is not None:
                events.append(torch.cuda.Event(enable_timing=True))
                events[-1].record(st)
        torch.cuda.nvtx.range_pop()
        if events is not None:
            events.append(torch.cuda.Event(enable_timing=True))
            events[-1].record(st)
        torch.cuda.nvtx.range_push("decode")
        ids = eng.generate_greedy(slots_all, prompts[:, P - 1], np.full(S, P - 1, np.int32), G)
        torch.cuda.nvtx.range_pop()
        if events is not None:
            events.append(torch.cuda.Event(enable_timing=True))
            events[-1].record(st)
            events.append(torch.cuda.Event(enable_timing=True))
            events[-1].record()
        every = gather_ids(ids, world, "cuda")
        if events is not None:
            events.append(torch.cuda.Event(enable_timing=True))
            events[-1].record()
        return every.cpu().numpy() if rank == 0 else None

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    launches0 = eng.launch_count()
    wall, device_ms, prefill_ms, decode_ms, gather_ms = [], [], [], [], []
    torch.cuda.nvtx.range_push("timed")  # lets a profiler keep to the timed steps (ncu --nvtx-include timed/)
    with Clocks(local) as clocks:
        for _ in range(args.steps):
            ev = []
            t0 = time.perf_counter()
            step(ev)
            torch.cuda.synchronize()
            wall.append(time.perf_counter() - t0)
            pairs = [ev[i].elapsed_time(ev[i + 1]) for i in range(0, len(ev), 2)]
            prefill_ms.append(sum(pairs[:-2]))
            decode_ms.append(pairs[-2])
            gather_ms.append(pairs[-1])
            device_ms.append(sum(pairs))
    torch.cuda.nvtx.range_pop()
    barrier()
    launches = eng.launch_count() - launches0

    def worst(x):
        return max_over_ranks(x, world, "cuda")

    ms_step = worst(np.mean(device_ms))
    wall_step = worst(np.mean(wall))
    pre = worst(np.mean(prefill_ms))
    dec = worst(np.mean(decode_ms))
    gat = worst(np.mean(gather_ms))
    tokens = args.seqs * (P - 1 + G)
    result = None
    if rank == 0:
        peaks, which = measured_peaks()
        roof = matmul_roofline(eng, S, peaks)
        roof["peak_source"] = which
        c4 = c4_sweep(eng, peaks)
        c3 = c3_decode_attention(peaks)
        c2 = c2_prefill_attention(peaks)
        cpu_v, cpu_dt, _ = cpu_sample(ckpt_host, plan, args, host_threads())
        # the same oracle on one thread, a shorter sample (4 prompt tokens + 2 greedy steps)
        one = argparse.Namespace(**{**vars(args), "cpu_prompt": 4, "cpu_gen": 2})
        cpu1_v, cpu1_dt, _ = cpu_sample(ckpt_host, plan, one, 1)
        del ckpt_host
        # each engine call copies its token table (4 x max_tokens int32) from pinned memory; greedy 2 more words;
        # the generated ids go to the device for the all-gather
        runs = -(-(P - 1) // args.block)
        h2d = (runs + 1) * 16 * S * args.block + 8 + S * G * 4
        d2h = S * G * 4 + 4 + args.seqs * G * 4  # the ids and the not-finite flag; rank 0 reads every sequence's ids
        clk = clocks.summary()
        result = {
            "metric": METRIC, "value": tokens / (ms_step / 1e3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": workload_config(args, world),
            "prefill_tok_s": args.seqs * (P - 1) / (pre / 1e3), "decode_tok_s": args.seqs * G / (dec / 1e3),
            "gather_ms": gat, "per_gpu_sequences": S,
            "e2e": {"value": tokens / wall_step, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": roof,
            "cpu_baseline": {"value": cpu_v, "unit": "tok/s", "cores": host_threads(), "kind": "port",
                             "sample": f"1 sequence: {args.cpu_prompt} prompt tokens (one block) + {args.cpu_gen} "
                                       f"greedy steps of the same model ({cpu_dt:.1f} s); the reference's CPU path "
                                       f"holds one sequence, so this is unbatched against the GPU's 64",
                             "cpu": cpu_model(), "build": "g++ -O3 -march=native -ffp-contract=off"},
            "cpu_baseline_1thread": {"value": cpu1_v, "unit": "tok/s", "cores": 1, "kind": "port",
                                     "sample": f"1 sequence: 4 prompt tokens (one block) + 2 greedy steps of the same "
                                               f"model ({cpu1_dt:.1f} s)"},
            "c4_matmul": c4,
            "c3_decode_attention": c3,
            "c2_prefill_attention": c2,
            "gpu_launches": launches // max(1, args.steps) * args.steps,
            "clocks": clk,
        }
    eng.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def matmul_arm(args):
    """One matrix (rows x n int8, scales, --seqs tokens of activations) and --warmup + --steps launches of
    b200k_matmul_q8s on it, timed with CUDA events; prints one line. Holds rows * n * 1.2 bytes on the device."""
    import ctypes

    import torch

    from b200fwd import abi

    rows, n = (int(v) for v in args.matmul.lower().split("x"))
    count = args.seqs
    lib = abi.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    ngp = (n // 32 + 3) // 4 * 4
    w = torch.randint(-127, 128, (rows, n), dtype=torch.int8, device="cuda", generator=g)
    ws = torch.rand((rows, ngp), device="cuda", generator=g) * 0.019 + 0.001
    xq = torch.randint(-63, 64, (count, n), dtype=torch.int8, device="cuda", generator=g)
    xs = torch.rand((count, ngp), device="cuda", generator=g) * 0.1
    out = torch.empty((count, rows), device="cuda")
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())

    def launch():
        abi.check(lib.b200k_matmul_q8s(ptr(out), ptr(xq), ptr(xs), ptr(w), ptr(ws), ngp, n, rows, count, rows, n, ngp,
                                       None), "matmul_q8s")

    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        launch()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    nbytes = rows * n * 9 / 8 + count * n * 9 / 8 + 4 * count * rows
    ms = float(np.median(times))
    print(json.dumps({"matmul": f"{rows}x{n}", "tokens": count, "ms_per_call": ms,
                      "gb_s": nbytes / (ms / 1e3) / 1e9, "note": "per call: the scale copy, the matmul, the "
                      "error-word read; weights in L2 after the first call (one matrix)"}), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    if args.matmul:
        return matmul_arm(args)
    if args.config == "c4":
        return c4_arm(args)
    if args.config == "c3":
        return c3_arm(args)
    if args.config == "c2":
        return c2_arm(args)
    return b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())

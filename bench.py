"""Decode benchmark: TinyLlama-1.1B-shaped FP32 batch-1 greedy decode.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token: embedding, 22 decoder layers, final norm, LM
head and argmax over seeded synthetic weights (N(0, 0.02) Irwin-Hall
deviates, norms 1.0, seed 0) after a 32-token seeded prompt.  Weights
stream 4.14 GB per step, far above the 126 MB L2, so no flush is needed
between steps.

Our arm prints one JSON line with
  value    device-resident tokens/s: K steps chained on the device (the
           next token never leaves HBM), CUDA events on the engine's stream;
  e2e      the same K steps through the public C API
           (infernt_engine_forward_token -> InferenceEngine::forward_token):
           token and position in as kernel arguments, next token out by a
           4-byte device-to-host copy, one host sync per step;
  roofline the dominant kernel, the persistent decode kernel (one launch
           runs the K chained steps): algorithmic bytes of K steps over its
           CUDA-event time, against the measured HBM copy bandwidth; traffic
           from the ncu summary under profiles/;
  cpu_baseline  the CPU oracle (oracle/, scalar C, all host threads) on a
           bounded sample of the same decode, rank 0 at N=1 only.
With N > 1 (torchrun, one process per GPU) every rank decodes its own
sequence on a full replica (data parallel, no collective on the data path);
value = all ranks' tokens / max-over-ranks device time.

--impl reference runs the reference's own build (INFERNT sources compiled
unchanged for sm_100 into oracle/_ref/libinfernt_ref.so, cuBLAS FP32) on
the same workload through its InferenceEngine::forward_token +
sample_next_token loop, rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_TOKENS = 32
SEED = 0
STD = 0.02
T4_PUBLISHED_TOKS = 53.10  # reference README.md:355 (TinyLlama FP32 b=1 decode, Tesla T4)
METRIC = "decode tok/s (TinyLlama-1.1B FP32 batch-1 greedy)"


def env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), \
        int(os.environ.get("LOCAL_RANK", "0"))


def max_over_ranks(torch, x, device):
    """The largest value of x over all ranks (x itself without a process
    group): timings are reported as the slowest rank's."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_tokens_per_s(world, steps, ms_max):
    """Whole-job throughput: every rank decodes `steps` tokens of its own
    sequence; the job takes the slowest rank's time."""
    return world * steps / (ms_max / 1e3)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes_per_step(cfg, ctx_mean):
    """Bytes one decode step must move: every projection weight and the LM
    head once, the embedding row, the norm weights, and the K/V rows read by
    attention (2 * L * Nkv * ctx * D floats) plus the appended rows."""
    wbytes = 4 if cfg.weight_dtype == 0 else 2
    H, L = cfg.hidden_size, cfg.num_layers
    b = cfg.weight_params * wbytes
    b += H * 4 + (2 * L + 1) * H * 4
    b += 2 * L * cfg.num_key_value_heads * cfg.head_dim * 4 * (ctx_mean + 1)
    return b


class ClockSampler:
    """nvidia-smi clock / throttle sampling around a timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = "/tmp/infernt_clocks_%d_%d.csv" % (os.getpid(), gpu_index)

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q,
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def time_dominant_kernel(torch, ib, eng, cfg, launches=66):
    """RMSNorm + gate/up GEMV + SiLU (the largest per-layer weight read:
    2 * I * H weights) launched alone, cycling through the layers' weights
    so nothing is served from L2; CUDA events on the launching stream."""
    H, I, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_layers
    w = eng.weight_ptrs()
    x = torch.randn(H, device="cuda")
    nw = torch.ones(H, device="cuda")
    out = torch.empty(I, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def launch(l):
        lw = w[3 + 9 * l:]
        ib.call("infernt_rmsnorm_gate_up_silu", out.data_ptr(), lw[6], lw[7], I, H, cfg.weight_dtype,
                x.data_ptr(), nw.data_ptr(), cfg.rms_norm_eps, sp)

    for l in range(min(L, 6)):
        launch(l)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(launches):
        launch(i % L)
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / launches
    wbytes = 4 if cfg.weight_dtype == 0 else 2
    alg = 2 * I * H * wbytes + H * 8 + I * 4
    return ms, alg


def cpu_baseline(cfg, budget_s=12.0):
    import oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    t0 = time.time()
    m = O.LlamaOracle(cfg, seed=SEED, std=STD)
    gen_s = time.time() - t0
    prompt = O.prompt(PROMPT_TOKENS, SEED, 3, cfg.vocab_size)
    n, t1 = 0, time.time()
    tok = int(prompt[0])
    while n < 64 and (n < 2 or time.time() - t1 < budget_s):
        tok, _ = m.decode_token(int(prompt[n]) if n < PROMPT_TOKENS else tok, n)
        n += 1
    el = time.time() - t1
    return {"value": round(n / el, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": "%d decode steps at positions 0..%d of the same seeded model (oracle/oracle.c, "
                      "double accumulation, %d threads; weight generation %.1f s not timed)"
                      % (n, n - 1, threads, gen_s)}


def measure_batched_b1_exchanges(torch, ib, rank, world, pos, steps):
    """The same 8B-shaped decode (bf16 weights, seed 1, batch 1) through the
    batched engine: one kernel per op captured in a CUDA graph, tensor
    parallel over the ranks, its O and down sums crossing the ranks by the
    peer-memory exchange and then by ncclAllReduce (the NCCL baseline);
    seeded KV rows for `pos` positions, `steps` timed steps each (CUDA
    events, max over ranks)."""
    import torch.distributed as dist
    cfg = ib.LLAMA3_8B.with_(weight_dtype=ib.DTYPE_BF16, max_seq_len=pos + 2 * steps + 16)
    nid = [ib.nccl_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(nid, src=0)
    eng = ib.BatchEngine(cfg, 1, seed=1, std=STD, rank=rank, world=world, nccl_id=nid[0] if world > 1 else None)
    eng.fill_kv(0, 7, pos)
    out = {"engine": "infernt_batch_engine (bgemm tcgen05 projections, T = 1), CUDA graph per step",
           "positions": [pos, pos + 2 * steps]}
    tok, p = [5], [pos]
    for mode in (["peer", "nccl"] if world > 1 else ["single"]):
        if world > 1:
            eng.set_tp_exchange(mode == "peer")
            dist.barrier()
        toks, _ = eng.decode(tok, p, 3)
        tok, p = [int(toks[-1][0])], [p[0] + 3]
        if world > 1:
            dist.barrier()
        toks, ms = eng.decode(tok, p, steps)
        tok, p = [int(toks[-1][0])], [p[0] + steps]
        ms_max = max_over_ranks(torch, ms, "cuda")
        out[mode] = {"ms_per_step": round(ms_max / steps, 5), "tok_s": round(steps / (ms_max / 1e3), 2)}
    eng.close()
    return out


def run_ours(args):
    import torch
    import infernt_b200 as ib
    rank, world, local = env_rank()
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    cfg = ib.TINYLLAMA
    K, W = args.steps, args.warmup
    assert PROMPT_TOKENS + W + K <= cfg.max_seq_len, "steps + warmup exceed max_seq_len"
    prompt = ib.prompt(PROMPT_TOKENS, SEED + rank, 3, cfg.vocab_size)

    eng = ib.Engine(cfg, seed=SEED, std=STD)

    def prefill():
        eng.reset()
        t = None
        for pos, tok in enumerate(prompt):
            t = eng.forward_token(tok, pos)
        return t

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # ---- device-resident value: K chained steps
    first = prefill()
    toks_w, _ = eng.decode_chain(first, PROMPT_TOKENS, W)
    start_tok, start_pos = toks_w[-1] if W else first, PROMPT_TOKENS + W
    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    toks, ms = eng.decode_chain(start_tok, start_pos, K)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms_max = max_over_ranks(torch, ms, "cuda")
    value = job_tokens_per_s(world, K, ms_max)

    # ---- end to end through the public C API (same positions)
    first = prefill()
    t = first
    for i in range(W):
        t = eng.forward_token(t, PROMPT_TOKENS + i)
    barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    e2e_toks = []
    for i in range(K):
        t = eng.forward_token(t, start_pos + i)
        e2e_toks.append(t)
    b.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(torch, a.elapsed_time(b), "cuda")
    e2e_value = job_tokens_per_s(world, K, e2e_ms)
    same_tokens = e2e_toks == toks

    # ---- roofline of the dominant kernel: the persistent decode kernel runs
    # the whole chain of K steps in one launch (all of the timed GPU time),
    # so its algorithmic bytes per launch are K steps' worth
    mode = eng.mode
    hbm, src = peaks()
    ctx_mean = start_pos + K / 2.0
    step_bytes = algorithmic_bytes_per_step(cfg, ctx_mean)
    launch_bytes = step_bytes * K
    achieved = launch_bytes / (ms / 1e3) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "decode_mega_kernel_f32_tinyllama_traffic.txt")
    if os.path.exists(tfile):
        for line in open(tfile):
            if line.startswith("decode_mega_kernel_f32_tinyllama_per_step"):
                traffic = int(line.split("=")[1].split()[0]) * K
    # the largest per-layer projection launched alone (standalone C entry point)
    k_ms, k_bytes = time_dominant_kernel(torch, ib, eng, cfg)
    # the persistent kernel takes the first step's token and position as
    # launch parameters: one launch runs the K chained steps (the kernel
    # sequence sets them with a one-thread kernel first)
    launches = 1 if mode == ib.MODE_PERSISTENT else K * eng_kernels(cfg) + 1

    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms_max / K, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / T4_PUBLISHED_TOKS, 3), "dtype": "f32",
        "data": "synthetic: seeded weights N(0,0.02) (Irwin-Hall, include/infernt_seed.h), norms 1.0, "
                "32-token seeded prompt",
        "config": {"workload": "tinyllama-1.1b-fp32-b1-greedy-decode", "hidden": 2048, "layers": 22,
                   "q_heads": 32, "kv_heads": 4, "head_dim": 64, "intermediate": 5632, "vocab": 32000,
                   "prompt_tokens": PROMPT_TOKENS, "positions": [start_pos, start_pos + K],
                   "execution": {0: "eager", 1: "graph", 2: "persistent"}[mode],
                   "parallelism": "replicas (one sequence per GPU)" if world > 1 else "single GPU",
                   "l2": "no flush: 4.14 GB of weights streamed per step >> 126 MB L2",
                   "global_batch": world, "seq_len": start_pos + K},
        "e2e": {"value": round(e2e_value, 3), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 68, "api": "infernt_engine_forward_token (C ABI) -> "
                "InferenceEngine::forward_token", "tokens_match_device_chain": same_tokens},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "decode_mega_kernel<float> (persistent decode, %d steps per launch)"
                     % K if mode == ib.MODE_PERSISTENT else "decode step (kernel sequence)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": src + " (MEASURED_PEAKS.json hbm_gbs)"
                     if src == "measured" else src, "traffic": traffic,
                     "algorithmic_bytes_per_launch": launch_bytes, "algorithmic_bytes_per_step": step_bytes,
                     "avg_launch_ms": round(ms, 4)},
        "standalone_gate_up_kernel": {"kernel": "gemv_tma_kernel<float,SwiGLU> (C entry point, launched alone)",
                                      "achieved_gbs": round(k_bytes / (k_ms / 1e3) / 1e9, 1),
                                      "avg_launch_ms": round(k_ms, 5), "bytes_per_launch": k_bytes},
        "clocks": clocks,
    }
    eng.close()
    if not args.no_llama8b:
        # the 8B-shaped tensor-parallel decode over the same ranks (the
        # collective path), after the replicas' measurement
        result["llama8b_tp"] = measure_llama8b_tp(torch, ib, rank, world, local)
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(cfg)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


# The first 64 greedy tokens of the Llama-3-8B-shaped decode below (seed 1,
# 512-token seeded prompt) on one GPU (measure_llama8b_tp with world 1, one
# B200): the tensor-parallel runs are checked against them.
LLAMA8B_TP1_TOKENS = [
    74325, 29784, 116036, 13841, 78160, 8054, 87554, 99912,
    22201, 48487, 46054, 9760, 14993, 95613, 68450, 32004,
    70506, 91286, 65530, 36762, 2697, 47189, 77848, 86374,
    55866, 72738, 96966, 15700, 126896, 31724, 91417, 15059,
    58308, 55092, 104689, 42894, 83670, 30557, 66623, 24200,
    115946, 28298, 125357, 86034, 2520, 25757, 128182, 115911,
    38943, 92207, 83477, 105780, 56659, 92537, 66869, 121544,
    53370, 20360, 72045, 110362, 68328, 62196, 45986, 33142,
]


def measure_llama8b_tp(torch, ib, rank, world, local, steps=61, warmup=3):
    """Llama-3-8B-shaped bf16 greedy decode, batch 1, tensor-parallel over
    the ranks already in the process group (tp = world): seeded weights
    (seed 1), a 512-token seeded prompt, `warmup` chained steps, then `steps`
    chained steps timed with CUDA events on every rank, max over ranks.  The
    O and down all-reduces and the argmax agreement run inside the
    persistent kernel over NVLink peer memory.  Returns ms/step, tok/s, the
    per-GPU HBM fraction, whether every rank produced the same tokens and
    how many of the first 64 generated tokens equal the one-GPU run's."""
    import torch.distributed as dist
    multi = world > 1
    prompt_len = 512
    cfg = ib.LLAMA3_8B.with_(max_seq_len=prompt_len + warmup + steps + 8)
    eng = ib.TPEngine(cfg, rank, world, seed=1, std=STD)
    if multi:
        handles = [None] * world
        dist.all_gather_object(handles, eng.xchg_handle())
        eng.set_peers(handles)
        dist.barrier()
    t = None
    for pos, tok in enumerate(ib.prompt(prompt_len, 1, 3, cfg.vocab_size)):
        if multi:
            dist.barrier()  # the ranks' kernels wait on one another: launch them together
        t = eng.forward_token(tok, pos)
    if multi:
        dist.barrier()
    toks_w, _ = eng.decode_chain(t, prompt_len, warmup)
    if multi:
        dist.barrier()
    torch.cuda.synchronize()
    toks, ms = eng.decode_chain(toks_w[-1], prompt_len + warmup, steps)
    ms_max = max_over_ranks(torch, ms, "cuda")
    gen = [t] + toks_w + toks
    if multi:
        every = [None] * world
        dist.all_gather_object(every, gen)
        agree = all(g == every[0] for g in every)
    else:
        agree = True
    ref = LLAMA8B_TP1_TOKENS
    match = None
    if ref is not None:
        match = next((i for i, (a, b) in enumerate(zip(gen, ref)) if a != b), min(len(gen), len(ref)))
    # per-GPU algorithmic bytes per step: this rank's bf16 weight shards, its
    # KV rows read by attention (FP32), the embedding row
    H, L, D = cfg.hidden_size, cfg.num_layers, cfg.head_dim
    d = eng.dims
    per_layer = (d[0] * D + 2 * d[1] * D) * H + H * d[0] * D + 2 * d[2] * H + H * d[3]
    wbytes = 2 * (L * per_layer + d[5] * H)
    ctx_mean = prompt_len + warmup + steps / 2.0
    bytes_gpu = wbytes + 2 * L * d[1] * D * 4 * (ctx_mean + 1) + H * 4
    hbm, src = peaks()
    eng.close()
    nccl_side = measure_batched_b1_exchanges(torch, ib, rank, world, prompt_len + warmup, steps)
    return {"workload": "llama3-8b-bf16-b1-tp%d" % world, "parallelism": "tp%d" % world,
            "kernel_sequence_engine": nccl_side,
            "ms_per_step": round(ms_max / steps, 5), "tok_s": round(steps / (ms_max / 1e3), 2),
            "steps": steps, "positions": [prompt_len + warmup, prompt_len + warmup + steps],
            "bytes_per_gpu_per_step": bytes_gpu,
            "hbm_frac_per_gpu": round(bytes_gpu / (ms_max / steps / 1e3) / 1e9 / hbm, 4),
            "tokens_agree_across_ranks": agree,
            "tokens_match_tp1": (match == 64) if match is not None else None,
            "tokens_matching_tp1": match, "tokens": gen[:64],
            "all_reduce": "in-kernel over NVLink peer memory (tagged words), after O and down",
            "kernel": "decode_mega_kernel<bf16> (persistent, one launch per chain)"}


def eng_kernels(cfg):
    return 5 * cfg.num_layers + 1


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    import oracle as O
    import infernt_b200 as ib  # configuration presets only
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libinfernt_ref.so not built "
                          "(the reference checkout was absent when build() ran)"}))
        return
    cfg = ib.TINYLLAMA
    K, W = args.steps, args.warmup
    prompt = [int(t) for t in O.prompt(PROMPT_TOKENS, SEED, 3, cfg.vocab_size)]
    eng = O.RefEngine(cfg, seed=SEED, std=STD)
    t = None
    for pos, tok in enumerate(prompt):
        t = eng.forward_token(tok, pos)
    toks, _ = eng.decode_loop(t, PROMPT_TOKENS, W)
    start_tok = toks[-1] if W else t
    start_pos = PROMPT_TOKENS + W
    sampler = ClockSampler(0)
    sampler.start()
    toks, ms = eng.decode_loop(start_tok, start_pos, K)
    clocks = sampler.stop()
    value = K / (ms / 1e3)
    eng.close()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": 1,
        "steps": K, "warmup": W, "ms_per_step": round(ms / K, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / T4_PUBLISHED_TOKS, 3), "dtype": "f32",
        "data": "synthetic: seeded weights N(0,0.02), norms 1.0, 32-token seeded prompt",
        "config": {"workload": "tinyllama-1.1b-fp32-b1-greedy-decode", "prompt_tokens": PROMPT_TOKENS,
                   "positions": [start_pos, start_pos + K], "parallelism": "single GPU"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": 1, "kind": "reference",
                         "sample": "the reference's own build (src/, cuda/, gemm/ compiled unchanged for "
                                   "sm_100, cuBLAS FP32) driven through InferenceEngine::forward_token + "
                                   "sample_next_token on one B200; it has no CPU path"},
        "clocks": clocks,
    }), flush=True)


def run_layer_ops(args):
    """Single-layer decode microbench at the TinyLlama shape (FP32): one token
    at position 4095 with the KV cache filled with N(0,1) values for 4095
    positions; every op of the layer launched through its C entry point.

    Each op is timed as --steps launches back to back on one stream between
    two CUDA events (after --warmup launches), cycling through enough copies
    of its weights / KV cache (over 256 MB per cycle, twice the L2) that every
    launch reads them from HBM; the per-launch time is the interval over the
    launch count, so it holds the kernel and the gap to the next launch, not
    the host's call into the library.  Each op's algorithmic bytes (weights,
    inputs, outputs, K/V rows read) over that time, against the measured HBM
    bandwidth.  "cold_us" is the same op launched once after a 256 MB L2
    flush, events around it (a spin kernel ahead keeps the host's enqueue
    time out): launch and drain included."""
    import torch
    import infernt_b200 as ib
    torch.cuda.set_device(0)
    H, I, Nq, Nkv, D, V = 2048, 5632, 32, 4, 64, 32000
    pos, max_seq, eps, theta = 4095, 4096, 1e-5, 10000.0
    qs, kvs = Nq * D, Nkv * D
    f32 = 0
    g = torch.Generator(device="cuda").manual_seed(SEED)

    def randn(*shape, std=1.0):
        return torch.randn(*shape, device="cuda", generator=g) * std

    def copies(nbytes):
        return max(1, min(64, -(-(256 << 20) // max(nbytes, 1))))

    x, nw = randn(H), torch.ones(H, device="cuda")
    qkv, attn, act, hid, y = (torch.zeros(n, device="cuda") for n in (qs + 2 * kvs, qs, I, H, H))
    logits = randn(V)
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    splits = torch.cuda.get_device_properties(0).multi_processor_count // Nkv
    ws = torch.zeros(ib.lib().infernt_attention_workspace_bytes(Nq, Nkv, D, splits), dtype=torch.uint8,
                     device="cuda")
    nqkv, no, ngu, nd = (copies(b) for b in ((qs + 2 * kvs) * H * 4, H * qs * 4, 2 * I * H * 4, H * I * 4))
    nkv = copies(2 * Nkv * max_seq * D * 4)
    WQ = [(randn(qs, H, std=STD), randn(kvs, H, std=STD), randn(kvs, H, std=STD)) for _ in range(nqkv)]
    WO = [randn(H, qs, std=STD) for _ in range(no)]
    WGU = [(randn(I, H, std=STD), randn(I, H, std=STD)) for _ in range(ngu)]
    WD = [randn(H, I, std=STD) for _ in range(nd)]
    KV = [(randn(Nkv, max_seq, D), randn(Nkv, max_seq, D)) for _ in range(nkv)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    P = lambda t: t.data_ptr()  # noqa: E731
    ops = [
        ("rmsnorm", 3 * H * 4, 1, lambda i: ib.call("infernt_rmsnorm", P(y), P(x), P(nw), 1, H, eps, sp)),
        ("qkv_rmsnorm_gemv", (qs + 2 * kvs) * H * 4 + 2 * H * 4 + (qs + 2 * kvs) * 4, nqkv,
         lambda i: ib.call("infernt_rmsnorm_gemv", P(qkv), P(WQ[i][0]), qs, P(WQ[i][1]), kvs, P(WQ[i][2]), kvs, H,
                           f32, P(x), P(nw), eps, sp)),
        ("rope", 2 * (qs + kvs) * 4, 1, lambda i: ib.call("infernt_rope", P(qkv), P(qkv) + qs * 4, 1, Nq, Nkv, D,
                                                          pos, theta, sp)),
        ("kv_cache_append", 4 * kvs * 4, 1,
         lambda i: ib.call("infernt_kv_cache_append", P(KV[0][0]), P(KV[0][1]), P(qkv) + qs * 4,
                           P(qkv) + (qs + kvs) * 4, Nkv, D, max_seq, pos, sp)),
        ("attention_decode", 2 * Nkv * (pos + 1) * D * 4 + (qs + 2 * kvs) * 4 + qs * 4, nkv,
         lambda i: ib.call("infernt_attention_decode", P(attn), P(qkv), P(KV[i][0]), P(KV[i][1]), Nq, Nkv, D,
                           max_seq, pos, theta, splits, P(ws), sp)),
        ("o_gemv_residual", H * qs * 4 + qs * 4 + 2 * H * 4, no,
         lambda i: ib.call("infernt_gemv_residual", P(hid), P(x), P(WO[i]), H, qs, f32, P(attn), sp)),
        ("gate_up_rmsnorm_silu", 2 * I * H * 4 + 2 * H * 4 + I * 4, ngu,
         lambda i: ib.call("infernt_rmsnorm_gate_up_silu", P(act), P(WGU[i][0]), P(WGU[i][1]), I, H, f32, P(hid),
                           P(nw), eps, sp)),
        ("down_gemv_residual", H * I * 4 + I * 4 + 2 * H * 4, nd,
         lambda i: ib.call("infernt_gemv_residual", P(y), P(hid), P(WD[i]), H, I, f32, P(act), sp)),
        ("residual_add", 3 * H * 4, 1, lambda i: ib.call("infernt_residual_add", P(y), P(hid), P(x), H, sp)),
        ("argmax", V * 4 + 4, 1, lambda i: ib.call("infernt_argmax", P(tok), P(logits), V, sp)),
    ]
    hbm, src = peaks()
    res = {}
    n = max(args.steps, 1)
    for name, nbytes, ncopy, op in ops:
        for i in range(args.warmup):
            op(i % ncopy)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2000000)
        a.record(stream)
        for i in range(n):
            op(i % ncopy)
        b.record(stream)
        b.synchronize()
        ms = a.elapsed_time(b) / n
        # one launch after an L2 flush, launch and drain included
        flush.zero_()
        c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2000000)
        c.record(stream)
        op(0)
        d.record(stream)
        d.synchronize()
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"us": round(ms * 1e3, 2), "bytes": nbytes, "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
                     "copies_cycled": ncopy, "cold_us": round(c.elapsed_time(d) * 1e3, 2)}
    total_us = sum(r["us"] for r in res.values())
    total_bytes = sum(r["bytes"] for r in res.values())
    print(json.dumps({
        "metric": "single-layer decode ops at position 4095 (TinyLlama shape, FP32)", "unit": "us",
        "value": round(total_us, 2), "higher_is_better": False, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "dtype": "f32", "data": "synthetic: torch.randn seeded 0 (weights x0.02), "
        "KV cache N(0,1) for 4095 positions, logits N(0,1)",
        "config": {"workload": "tinyllama-layer-ops-pos4095", "position": pos, "attention_splits": splits,
                   "l2": "launches cycle through over 256 MB of weight / KV copies (HBM reads every launch); "
                         "cold_us after a 256 MB flush"},
        "ops": res, "layer_bytes": total_bytes,
        "layer_gbs": round(total_bytes / (total_us / 1e6) / 1e9, 1),
        "peak": {"hbm_gbs": hbm, "source": src},
    }), flush=True)


def run_llama8b_tp(args):
    """Llama-3-8B-shaped bf16 greedy decode, batch 1, tensor-parallel over
    the torchrun ranks (one per GPU; 1 without torchrun): seeded weights
    (seed 1), a 512-token seeded prompt, then --steps chained decode steps
    timed with CUDA events on each rank, max over ranks.  The O and down
    all-reduces and the argmax exchange run inside the persistent kernel over
    NVLink peer memory; torch.distributed only swaps the exchange-region
    handles and lines the ranks up.  value: the sequence's tokens/s (strong
    scaling: the same sequence on more GPUs)."""
    import datetime
    import torch
    import torch.distributed as dist
    import infernt_b200 as ib
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    prompt_len = 512
    cfg = ib.LLAMA3_8B.with_(max_seq_len=prompt_len + args.warmup + args.steps + 8)
    seed = 1
    eng = ib.TPEngine(cfg, rank, world, seed=seed, std=STD)
    if world > 1:
        handles = [None] * world
        dist.all_gather_object(handles, eng.xchg_handle())
        eng.set_peers(handles)
        dist.barrier()
    prompt = ib.prompt(prompt_len, seed, 3, cfg.vocab_size)
    t = None
    for pos, tok in enumerate(prompt):
        t = eng.forward_token(tok, pos)
    toks_w, _ = eng.decode_chain(t, prompt_len, args.warmup)
    start_tok, start_pos = toks_w[-1], prompt_len + args.warmup
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    toks, ms = eng.decode_chain(start_tok, start_pos, args.steps)
    clocks = sampler.stop()
    ms_max = max_over_ranks(torch, ms, "cuda")
    K = args.steps
    value = K / (ms_max / 1e3)
    # per-GPU algorithmic bytes per token: this rank's weight shards (bf16),
    # its KV rows read by attention, the embedding row
    H, L, D = cfg.hidden_size, cfg.num_layers, cfg.head_dim
    d = eng.dims
    per_layer = (d[0] * D + 2 * d[1] * D) * H + H * d[0] * D + 2 * d[2] * H + H * d[3]
    wbytes = 2 * (L * per_layer + d[5] * H)
    ctx_mean = start_pos + K / 2.0
    kv = 2 * L * d[1] * D * 4 * (ctx_mean + 1)
    bytes_gpu = wbytes + kv + H * 4
    hbm, src = peaks()
    achieved = bytes_gpu * K / (ms_max / 1e3) / 1e9
    result = {
        "metric": "decode tok/s (Llama-3-8B shape, bf16 weights, batch 1, tensor parallel)", "value": round(value, 3),
        "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": round(ms_max / K, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 weights, f32 math",
        "data": "synthetic: seeded weights N(0,0.02) seed 1, norms 1.0, 512-token seeded prompt",
        "config": {"workload": "llama3-8b-bf16-b1-tp%d" % world, "hidden": H, "layers": L, "q_heads": 32,
                   "kv_heads": 8, "head_dim": D, "intermediate": cfg.intermediate_size, "vocab": cfg.vocab_size,
                   "prompt_tokens": prompt_len, "positions": [start_pos, start_pos + K],
                   "parallelism": "tp%d" % world, "l2": "no flush: %.2f GB of weights per GPU per step"
                   % (wbytes / 1e9)},
        "roofline": {"bound": "hbm", "kernel": "decode_mega_kernel<bf16> (persistent, per GPU)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": src, "bytes_per_gpu_per_step": bytes_gpu},
        "clocks": clocks,
    }
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_batched(args, longctx=False, tp=False):
    """TinyLlama-shaped bf16 decode of 64 concurrent sequences (contexts
    uniform in [512, 2048], seeded), data-parallel over the torchrun ranks;
    with longctx, the Llama-3-8B shape (bf16) with 16 sequences of 32768
    positions each, the KV caches seeded instead of prefilled:
    rank r decodes sequences [64 r / N, 64 (r + 1) / N) with its own weight
    replica, no collective on the data path.  The projections run on the
    tensor cores (tcgen05), the KV caches are bf16.  Each sequence's first
    `context` KV rows are seeded values (the bench times decode, not the
    prompt).  value: tokens/s of the whole job; timed with CUDA events, max
    over ranks.  With tp (the long-context shape only), every rank holds all
    16 sequences and 1/N of every layer (tensor parallelism: heads, FFN rows,
    vocabulary rows; NCCL all-reduce of the O and down sums, all-gather of
    the argmax candidates)."""
    import datetime
    import torch
    import torch.distributed as dist
    import numpy as np
    import infernt_b200 as ib
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    K, W = args.steps, args.warmup
    if longctx:
        n_seq, seed = 16, 1
        ctx = np.full(n_seq, 32768)
        cfg = ib.LLAMA3_8B.with_(weight_dtype=ib.DTYPE_BF16, max_seq_len=32768 + W + 2 * K + 64)
    else:
        n_seq, seed = 64, 0
        ctx = np.random.default_rng(1234).integers(512, 2049, size=n_seq)
        cfg = ib.TINYLLAMA.with_(weight_dtype=ib.DTYPE_BF16, max_seq_len=2048 + W + K + 16)
    if tp:
        lo, hi = 0, n_seq
        nid = [ib.nccl_unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(nid, src=0)
        eng = ib.BatchEngine(cfg, n_seq, seed=seed, std=STD, rank=rank, world=world, nccl_id=nid[0])
    else:
        lo, hi = n_seq * rank // world, n_seq * (rank + 1) // world
    mine = ctx[lo:hi]
    T = hi - lo
    page = getattr(args, "paged", 0)
    if not tp:
        if page:
            # paged caches: each sequence's pages drawn from a shuffled pool
            # that holds exactly the positions the run reaches
            need = [-(-(int(c) + W + K + 16) // page) for c in mine]
            order = np.random.default_rng(99).permutation(sum(need)).tolist()
            eng = ib.BatchEngine(cfg, T, seed=seed, std=STD, pages=(page, sum(need)))
            at = 0
            for b in range(T):
                eng.set_pages(b, order[at:at + need[b]])
                at += need[b]
        else:
            eng = ib.BatchEngine(cfg, T, seed=seed, std=STD)
    tokens = ib.prompt(n_seq, seed, 3, cfg.vocab_size)[lo:hi]
    prefill = None
    if longctx and getattr(args, "real_prefill", False):
        # the prompts run through the engine's prefill (tensor-core chunks) and
        # each sequence decodes from the token its prompt produced
        pf_ms = 0.0
        for b in range(T):
            prompt = ib.prompt(int(mine[b]), 5000 + lo + b, 3, cfg.vocab_size)
            nxt, _, ms_b = eng.prefill(b, prompt)
            tokens[b] = nxt
            pf_ms += ms_b
        pf_max = max_over_ranks(torch, pf_ms, "cuda")
        prefill = {"ms": round(pf_max, 1), "prompt_tokens": int(np.sum(ctx)),
                   "tok_s": round(float(np.sum(ctx)) / (pf_max / 1e3), 1),
                   "api": "infernt_batch_engine_prefill, one sequence after another" +
                          (" (tensor parallel: every rank its shards, ncclAllReduce of each chunk's O and down "
                           "rows)" if tp and world > 1 else "")}
    else:
        for b in range(T):
            eng.fill_kv(b, 1000 + lo + b, int(mine[b]))
    positions = [int(c) for c in mine]
    toks_w, _ = eng.decode(tokens, positions, W)
    tokens = [int(t) for t in toks_w[-1]]
    positions = [p + W for p in positions]
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    toks, ms = eng.decode(tokens, positions, K)
    clocks = sampler.stop()
    ms_max = max_over_ranks(torch, ms, "cuda")
    value = n_seq * K / (ms_max / 1e3)
    shards = world if tp else 1
    nccl_baseline = None
    if tp and world > 1:
        # the same steps with the sums crossing the ranks by ncclAllReduce
        eng.set_tp_exchange(False)
        tk = [int(t) for t in toks[-1]]
        ps = [p + K for p in positions]
        tw, _ = eng.decode(tk, ps, 2)
        tk, ps = [int(t) for t in tw[-1]], [p + 2 for p in ps]
        dist.barrier()
        tn, ms_n = eng.decode(tk, ps, K)
        ms_n = max_over_ranks(torch, ms_n, "cuda")
        nccl_baseline = {"exchange": "ncclAllReduce after O and down", "ms_per_step": round(ms_n / K, 5),
                         "tok_s": round(n_seq * K / (ms_n / 1e3), 1)}
        eng.set_tp_exchange(True)
        positions = ps
        toks = tn
    # end to end through the synchronous step entry point: host token and
    # position arrays in, next tokens out, every step
    tokens = [int(t) for t in toks[-1]]
    positions = [p + K for p in positions]
    ne = 16
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(ne):
        tokens = eng.step(tokens, positions)
        positions = [p + 1 for p in positions]
    e2e_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(torch, e2e_s * 1e3, "cuda") / 1e3
    # algorithmic bytes per GPU per step: bf16 weights, the embedding rows,
    # the K/V rows read (bf16) and the rows appended
    H, L, D, nkv = cfg.hidden_size, cfg.num_layers, cfg.head_dim, cfg.num_key_value_heads
    wbytes = 2 * cfg.weight_params / shards + T * H * 4
    ctx_mean = float(np.mean(mine)) + W + K / 2.0
    kv_bytes = L * nkv * D * 2 * 2 * T * (ctx_mean + 1) / shards
    bytes_gpu = wbytes + kv_bytes
    hbm, src = peaks()
    achieved = bytes_gpu * K / (ms_max / 1e3) / 1e9
    flops = 2.0 * T * cfg.weight_params / shards
    sp = eng.splits()
    if longctx:
        metric = "decode tok/s (Llama-3-8B shape, bf16 weights, 16 sequences at 32768 positions)"
        data = ("synthetic: seeded weights N(0,0.02) seed 1, norms 1.0; every sequence's 32768 KV rows "
                "seeded (the prefill is timed by --workload prefill); seeded first tokens")
        workload = "llama8b-bf16-16seq-ctx32768-%s%d" % ("tp" if tp else "dp", world)
    else:
        metric = "decode tok/s (TinyLlama-1.1B shape, bf16 weights, 64 concurrent sequences)"
        data = ("synthetic: seeded weights N(0,0.02) seed 0, norms 1.0; per-sequence contexts uniform in "
                "[512, 2048] (numpy seed 1234) with seeded KV rows; seeded first tokens")
        workload = "tinyllama-bf16-64seq-dp%d" % world
    # kernels of a step: embedding + norm, per layer Q|K|V projection, the
    # attention (with the Q|K|V finishing), O, norm, gate/up, SwiGLU, down,
    # norm; the LM head and the argmax (groups of 16 query heads add the
    # Q|K|V finishing and the merge per layer)
    per_layer = 8 if cfg.num_attention_heads // cfg.num_key_value_heads <= 8 else 10
    if tp and world > 1:
        per_layer += 2  # the pushes of the two sums into the ranks' regions
    result = {
        "metric": metric,
        "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_max / K, 5), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "parallelism_detail": ("tensor parallel: heads, FFN rows and vocabulary rows split over the ranks, NCCL "
                               "all-reduce after O and down" if tp else "data parallel: sequences split over ranks"),
        "dtype": "bf16 weights and projection inputs, f32 accumulation, bf16 KV",
        "data": data,
        "gpu_launches": K * (per_layer * cfg.num_layers + (5 if tp and world > 1 else 3)),
        "config": {"workload": workload, "sequences": n_seq, "per_gpu": T,
                   "contexts_mean": round(float(np.mean(ctx)), 1),
                   "parallelism": ("tp%d" if tp else "dp%d") % world,
                   "splits_qkv_o_gateup_down_lm_attn": sp,
                   "kv_layout": ("paged: pages of %d positions from a shuffled pool, block table per sequence"
                                 % page if page else "contiguous [sequence][kv head][max_seq][head_dim]"),
                   "l2": "no flush: %.2f GB of weights + %.2f GB of KV per GPU per step"
                   % (wbytes / 1e9, kv_bytes / 1e9)},
        "e2e": {"value": round(n_seq * ne / e2e_s, 1), "unit": "tok/s",
                "h2d_bytes_per_step": 8 * T, "d2h_bytes_per_step": 4 * T,
                "api": "infernt_batch_engine_step (C ABI), host arrays in and out"},
        "roofline": {"bound": "hbm", "kernel": "whole step (bgemm tcgen05 projections + batch.cu kernels)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": src, "bytes_per_gpu_per_step": bytes_gpu,
                     "tensor_tflops": round(flops * K / (ms_max / 1e3) / 1e12, 1)},
        "clocks": clocks,
    }
    if nccl_baseline:
        result["nccl_baseline"] = nccl_baseline
        result["parallelism_detail"] = ("tensor parallel: heads, FFN rows and vocabulary rows split over the ranks; "
                                        "O and down sums pushed into every rank's region over NVLink (peer-memory "
                                        "exchange), ncclAllReduce reported beside it")
    if prefill:
        result["prefill"] = prefill
        result["data"] = ("synthetic: seeded weights N(0,0.02) seed 1, norms 1.0; every sequence's 32768-token "
                          "seeded prompt prefilled by the engine (time under 'prefill'), then decoded from "
                          "the token it produced")
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_serving(args):
    """Continuous batching of TinyLlama-shaped bf16 requests through the
    server C ABI (infernt_server_*: iteration-level scheduler, paged KV
    caches, prefill per admitted request on the tensor cores, one batched
    decode step of every running request per iteration): 256 requests with
    seeded prompts of uniform length in [512, 2048] and uniform
    max_new_tokens in [16, 512] (numpy seed 4321), 64 slots, pages of 32
    positions, a pool of 80% of the positions the slots could hold at
    max_seq_len.  value: generated tokens per second over the whole run
    (prefills, decode steps and host scheduling inside the host-timed
    region: the call a user makes, so it is also the e2e figure).  Beside
    it, static batching of the same requests on the contiguous batched
    engine and the same kernels: waves of 64, each prompt prefilled, then
    every wave decoded until its longest request is done.  With N ranks
    each serves its own share of the requests on a full replica (replicas,
    no collective); value = all ranks' generated tokens / the slowest
    rank's time."""
    import datetime
    import torch
    import torch.distributed as dist
    import numpy as np
    import infernt_b200 as ib
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    slots, page = 64, 32
    n_req = 256
    rng = np.random.default_rng(4321)
    plen = rng.integers(512, 2049, size=n_req)
    new = rng.integers(16, 513, size=n_req)
    lo, hi = n_req * rank // world, n_req * (rank + 1) // world
    cfg = ib.TINYLLAMA.with_(weight_dtype=ib.DTYPE_BF16, max_seq_len=2048 + 512 + 16)
    prompts = [ib.prompt(int(plen[i]), 7000 + i, 3, cfg.vocab_size) for i in range(lo, hi)]
    n_pages = int(0.8 * slots * cfg.max_seq_len / page)
    srv = ib.Server(cfg, slots, page, n_pages, seed=SEED, std=STD)
    # warm-up: graph capture, prefill scratch, staging caches
    for i in range(args.warmup):
        srv.submit(prompts[i % len(prompts)][:512], 8)
    srv.run()
    w0 = srv.stats()
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ids = [srv.submit(prompts[i], int(new[lo + i])) for i in range(hi - lo)]
    srv.run()
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    clocks = sampler.stop()
    st = srv.stats()
    outs = [srv.result(r) for r in ids]
    assert all(o[1] == "finished" and len(o[0]) == int(new[lo + i]) for i, o in enumerate(outs))
    srv.close()
    gen = int(np.sum(new[lo:hi]))
    secs_max = max_over_ranks(torch, secs * 1e3, "cuda") / 1e3
    total_gen = int(np.sum(new))
    value = total_gen / secs_max
    steps = st["steps"] - w0["steps"]
    dec = st["decode_tokens"] - w0["decode_tokens"]
    # static batching on the contiguous engine: waves of `slots` requests
    eng = ib.BatchEngine(cfg, slots, seed=SEED, std=STD)
    eng.prefill(0, prompts[0][:512])
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    for w0i in range(0, hi - lo, slots):
        wave = list(range(w0i, min(hi - lo, w0i + slots)))
        toks = [0] * slots
        pos = [0] * slots
        for j, i in enumerate(wave):
            toks[j], _, _ = eng.prefill(j, prompts[i])
            pos[j] = len(prompts[i])
        longest = max(int(new[lo + i]) for i in wave)
        if longest > 1:
            eng.decode(toks, pos, longest - 1)
    torch.cuda.synchronize()
    static_s = max_over_ranks(torch, (time.perf_counter() - t1) * 1e3, "cuda") / 1e3
    eng.close()
    result = {
        "metric": "served tok/s (TinyLlama-1.1B shape, bf16, continuous batching of 256 requests)",
        "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": int(steps),
        "warmup": args.warmup, "ms_per_step": round(secs_max * 1e3 / max(1, steps), 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 weights and projection inputs, f32 accumulation, bf16 KV",
        "data": ("synthetic: seeded weights N(0,0.02) seed 0, norms 1.0; 256 seeded prompts, lengths uniform "
                 "in [512, 2048], max_new_tokens uniform in [16, 512] (numpy seed 4321), greedy"),
        "config": {"workload": "tinyllama-bf16-serving-256req-64slots", "slots": slots, "page_size": page,
                   "pool_pages": n_pages, "requests": n_req, "parallelism": "replicas%d" % world,
                   "prompt_tokens": int(np.sum(plen)), "generated_tokens": total_gen,
                   "l2": "no flush: 2.07 GB of weights per step"},
        "serving": {"decode_steps": int(steps), "mean_running": round(dec / max(1, steps), 1),
                    "preemptions": st["preemptions"] - w0["preemptions"],
                    "prefill_tokens": st["prefill_tokens"] - w0["prefill_tokens"],
                    "rank0_generated": gen},
        "static_batching": {"tok_s": round(total_gen / static_s, 1), "s": round(static_s, 3),
                            "how": "contiguous batched engine, waves of 64 requests, each wave decoded "
                                   "until its longest request finishes"},
        "e2e": {"value": round(value, 1), "unit": "tok/s", "h2d_bytes_per_step": 8 * slots,
                "d2h_bytes_per_step": 4 * slots,
                "api": "infernt_server_submit / infernt_server_run (C ABI); host-timed, prefills included"},
        "gpu_launches": None,
        "clocks": clocks,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def prefill_flops(cfg, n, start=0):
    """Algorithmic FLOPs of prefilling n prompt tokens at positions [start,
    start + n): every projection (2 per weight element per token), causal
    attention (q.k and p.v: 4 Nq D per key, token at position p reads p + 1
    keys) and the LM head of the last token."""
    H, L, D, I = cfg.hidden_size, cfg.num_layers, cfg.head_dim, cfg.intermediate_size
    nq, nkv, V = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.vocab_size
    qs = nq * D
    proj = L * ((qs + 2 * nkv * D) * H + H * qs + 2 * I * H + H * I)
    keys = n * start + n * (n + 1) // 2
    return 2.0 * n * proj + 4.0 * nq * D * keys * L + 2.0 * V * H, 2.0 * n * proj, 4.0 * nq * D * keys * L


def run_prefill(args):
    """Prompt prefill of the long-context configuration: Llama-3-8B shape,
    bf16 weights, 16 sequences of 32768 seeded random prompt tokens each,
    data-parallel over the torchrun ranks (rank r prefills sequences [16 r /
    N, 16 (r + 1) / N)).  A step is the prefill of one whole prompt through
    the batched engine (infernt_batch_engine_prefill: chunks of 4096 tokens,
    tensor-core projections and causal attention, every K/V row written, the
    last token's LM head and argmax); the rank's sequences are taken in turn.
    value: prompt tokens/s of the whole job (max over ranks of the CUDA-event
    time); roofline: algorithmic FLOPs over the time against the measured
    sustained bf16 tensor peak, and the dominant kernel (the gate/up
    projection of one chunk, infernt_pgemm_bf16) timed alone."""
    import datetime
    import torch
    import torch.distributed as dist
    import numpy as np
    import infernt_b200 as ib
    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    K, W = args.steps, args.warmup
    n_seq, n_tok, chunk, seed = 16, 32768, 4096, 1
    cfg = ib.LLAMA3_8B.with_(weight_dtype=ib.DTYPE_BF16, max_seq_len=n_tok + 64)
    lo, hi = n_seq * rank // world, n_seq * (rank + 1) // world
    T = hi - lo
    eng = ib.BatchEngine(cfg, T, seed=seed, std=STD)
    prompts = [np.asarray(ib.prompt(n_tok, 1000 + lo + b, 3, cfg.vocab_size), dtype=np.int32) for b in range(T)]
    for i in range(W):
        eng.prefill(i % T, prompts[i % T], chunk=chunk)
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = 0.0
    t0 = time.perf_counter()
    first = []
    for i in range(K):
        nxt, _, m = eng.prefill(i % T, prompts[i % T], chunk=chunk)
        ms += m
        first.append(nxt)
    wall_s = time.perf_counter() - t0
    clocks = sampler.stop()
    ms_max = max_over_ranks(torch, ms, "cuda")
    wall_max = max_over_ranks(torch, wall_s * 1e3, "cuda") / 1e3
    value = world * K * n_tok / (ms_max / 1e3)
    flops, f_proj, f_attn = prefill_flops(cfg, n_tok)
    achieved = flops * K / (ms_max / 1e3) / 1e12
    peak_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peak_path):
        peak, src = float(json.load(open(peak_path))["bf16_tflops_sustained"]), "measured (sustained)"
    else:
        peak, src = 1400.0, "fallback (sustained)"
    # the dominant kernel alone: the gate/up projection (SwiGLU epilogue) of
    # one 4096-token chunk, as the prefill runs it
    H, I = cfg.hidden_size, cfg.intermediate_size
    g = torch.Generator(device="cuda").manual_seed(3)
    Wg = (torch.randn(2 * I, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(chunk, H, device="cuda", generator=g).to(torch.bfloat16)
    Y = torch.empty(chunk, I, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(3):
        ib.call("infernt_pgemm_swiglu_bf16", Wg.data_ptr(), I, H, X.data_ptr(), chunk, Y.data_ptr(), I, None,
                st.cuda_stream)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    reps = 10
    ev[0].record(st)
    for _ in range(reps):
        ib.call("infernt_pgemm_swiglu_bf16", Wg.data_ptr(), I, H, X.data_ptr(), chunk, Y.data_ptr(), I, None,
                st.cuda_stream)
    ev[1].record(st)
    torch.cuda.synchronize()
    gemm_ms = ev[0].elapsed_time(ev[1]) / reps
    gemm_tflops = 2.0 * chunk * 2 * I * H / (gemm_ms / 1e3) / 1e12
    del Wg, X, Y
    n_chunks = (n_tok + chunk - 1) // chunk
    per_layer = 8  # Q|K|V, RoPE + append, attention, O, norm, gate/up + SwiGLU, down, norm
    result = {
        "metric": "prefill tok/s (Llama-3-8B shape, bf16 weights, 32768-token prompts)",
        "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_max / K, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 weights, projection inputs, queries and probabilities; f32 accumulation; bf16 KV",
        "data": "synthetic: seeded weights N(0,0.02) seed 1, norms 1.0; seeded random prompts of 32768 token ids",
        "gpu_launches": K * (n_chunks * (per_layer * cfg.num_layers + 1) + 2),
        "config": {"workload": "llama8b-bf16-prefill-32768-16seq-dp%d" % world, "sequences": n_seq,
                   "per_gpu": T, "prompt_tokens": n_tok, "chunk": chunk, "parallelism": "dp%d" % world,
                   "step": "one whole prompt", "l2": "no flush: 15 GB of weights per chunk pass"},
        "e2e": {"value": round(world * K * n_tok / wall_max, 1), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * n_tok + 8, "d2h_bytes_per_step": 8,
                "api": "infernt_batch_engine_prefill (C ABI): host prompt in, next token out"},
        "roofline": {"bound": "tensor", "kernel": "whole prefill (pgemm tcgen05 projections + pf_attn_tc)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_source": src,
                     "flops_per_step": flops, "projection_flops": f_proj, "attention_flops": f_attn,
                     "dominant_kernel": {"name": "pgemm_kernel<swiglu> (gate/up + SwiGLU, 4096 x 28672 x 4096)",
                                         "ms": round(gemm_ms, 4), "achieved": round(gemm_tflops, 1),
                                         "frac": round(gemm_tflops / float(json.load(open(peak_path))["bf16_tflops"])
                                                       if os.path.exists(peak_path) else gemm_tflops / 1590.0, 4),
                                         "peak": "burst bf16"}},
        "first_tokens": first[:4],
        "clocks": clocks,
    }
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)


def run_profile_case(args):
    """A run sized for profilers (one GPU), no JSON line.

    Default: the TinyLlama-1.1B shape (or, with --shape llama3-8b, the
    Llama-3-8B shape) with --layers decoder layers (the per-layer matrices
    keep their full size; --vocab shrinks the embedding and LM head), seeded
    N(0, 0.02) weights.  Launch order on the device: --prompt single-step
    launches (the prompt), then one warm-up chain and one measured chain of
    --steps steps, so a profiler that skips --prompt + 1 launches of the
    decode kernel captures the measured chain.

    --batched T: the batched engine instead (bf16, T sequences with contexts
    uniform in [512, 2048], numpy seed 1234, seeded KV rows): --steps timed
    steps, then one more step between cudaProfilerStart and cudaProfilerStop,
    for a profiler started with --profile-from-start off.

    --prefill N: the batched engine's prompt prefill (bf16, one sequence):
    the first --start KV rows seeded, then a prompt of N seeded tokens at
    positions [start, start + N) in chunks of --chunk, twice (a warm-up
    prefill, then the measured one).  Per chunk and layer the launch order is
    pgemm (Q|K|V), pf_qkv_rope, pf_attn, pgemm (O), bt_resid_norm, pgemm
    (gate/up with SwiGLU), pgemm (down), bt_resid_norm."""
    import numpy as np
    import torch
    import infernt_b200 as ib
    torch.cuda.set_device(0)
    if args.prefill:
        base = ib.TINYLLAMA if args.shape == "tinyllama" else ib.LLAMA3_8B
        cfg = base.with_(num_layers=args.layers, weight_dtype=ib.DTYPE_BF16,
                         max_seq_len=args.start + args.prefill + 8)
        if args.vocab:
            cfg = cfg.with_(vocab_size=args.vocab)
        eng = ib.BatchEngine(cfg, 1, seed=1)
        if args.start:
            eng.fill_kv(0, 77, args.start)
        prompt = ib.prompt(args.prefill, 1000, 3, cfg.vocab_size)
        eng.prefill(0, prompt, start_pos=args.start, chunk=args.chunk)
        nxt, _, ms = eng.prefill(0, prompt, start_pos=args.start, chunk=args.chunk)
        print("prefill tokens=%d start=%d layers=%d chunk=%d: %.3f ms, %.0f tok/s, next token %d"
              % (args.prefill, args.start, args.layers, args.chunk, ms, args.prefill * 1e3 / ms, nxt))
        eng.close()
        return
    if args.batched:
        T = args.batched
        base = ib.TINYLLAMA if args.shape == "tinyllama" else ib.LLAMA3_8B
        cfg = base.with_(num_layers=args.layers, weight_dtype=ib.DTYPE_BF16, max_seq_len=2048 + 2 * args.steps + 8)
        if args.vocab:
            cfg = cfg.with_(vocab_size=args.vocab)
        eng = ib.BatchEngine(cfg, T, seed=0)
        ctx = np.random.default_rng(1234).integers(512, 2049, size=T)
        for b in range(T):
            eng.fill_kv(b, 1000 + b, int(ctx[b]))
        tokens = [5 + b for b in range(T)]
        pos = [int(c) for c in ctx]
        toks, _ = eng.decode(tokens, pos, args.steps)
        tokens, pos = [int(t) for t in toks[-1]], [p + args.steps for p in pos]
        toks, ms = eng.decode(tokens, pos, args.steps)
        tokens, pos = [int(t) for t in toks[-1]], [p + args.steps for p in pos]
        print("batched T=%d layers=%d: %.4f ms/step, %.0f tok/s, splits %s"
              % (T, args.layers, ms / args.steps, T * args.steps * 1e3 / ms, eng.splits()))
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        eng.step(tokens, pos)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        eng.close()
        return
    base = ib.TINYLLAMA if args.shape == "tinyllama" else ib.LLAMA3_8B.with_(max_seq_len=1024)
    cfg = base.with_(num_layers=args.layers)
    if args.vocab:
        cfg = cfg.with_(vocab_size=args.vocab)
    if args.bf16:
        cfg = cfg.with_(weight_dtype=ib.DTYPE_BF16)
    eng = ib.Engine(cfg, seed=0)
    t = 5
    for pos in range(args.prompt):
        t = eng.forward_token(t, pos)
    eng.decode_chain(t, args.prompt, args.steps)
    toks, ms = eng.decode_chain(t, args.prompt, args.steps)
    wbytes = cfg.weight_params * (2 if args.bf16 else 4)
    print("layers=%d steps=%d mode=%d: %.4f ms/step, %.0f tok/s, weights %.3f GB -> %.1f GB/s"
          % (args.layers, args.steps, eng.mode, ms / args.steps, args.steps * 1e3 / ms, wbytes / 1e9,
             wbytes / (ms / args.steps / 1e3) / 1e9))
    eng.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "layer-ops", "llama8b-tp", "batched", "longctx", "longctx-tp",
                                           "prefill", "serving", "profile-case"],
                    default="decode",
                    help="decode: the TinyLlama decode benchmark; layer-ops: every op of one layer "
                         "at position 4095, timed alone; llama8b-tp: the 8B-shaped bf16 decode, "
                         "tensor-parallel over the torchrun ranks; batched: 64 TinyLlama-shaped bf16 "
                         "sequences on the tensor cores, data-parallel over the torchrun ranks; "
                         "longctx: 16 8B-shaped bf16 sequences at 32768 positions, decode only, "
                         "data-parallel over the torchrun ranks; longctx-tp: the same 16 sequences, "
                         "tensor-parallel over the torchrun ranks; prefill: the 32768-token prompts of "
                         "those sequences (one prompt per step), data-parallel over the torchrun ranks; "
                         "serving: continuous batching of 256 TinyLlama-shaped bf16 requests over paged KV "
                         "(infernt_server_*), static batching beside it; "
                         "profile-case: a run sized for profilers (see run_profile_case), no JSON line")
    ap.add_argument("--paged", type=int, default=0,
                    help="batched / longctx: page size of paged KV caches (0: contiguous caches)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-llama8b", action="store_true",
                    help="decode: skip the Llama-3-8B-shaped tensor-parallel measurement")
    ap.add_argument("--real-prefill", action="store_true",
                    help="longctx: prefill every sequence's 32768-token prompt with the engine (reported "
                         "separately) instead of seeding its KV rows")
    pc = ap.add_argument_group("profile-case")
    pc.add_argument("--layers", type=int, default=4)
    pc.add_argument("--prompt", type=int, default=2)
    pc.add_argument("--bf16", action="store_true", help="bf16 weights (FP32 activations)")
    pc.add_argument("--shape", choices=["tinyllama", "llama3-8b"], default="tinyllama")
    pc.add_argument("--vocab", type=int, default=0, help="vocabulary size (0: the shape's own)")
    pc.add_argument("--batched", type=int, default=0, help="sequences of a batched-engine run (0: b=1 decode)")
    pc.add_argument("--prefill", type=int, default=0, help="prompt tokens of a prefill run (0: decode)")
    pc.add_argument("--start", type=int, default=0, help="prefill: seeded KV rows before the prompt")
    pc.add_argument("--chunk", type=int, default=4096, help="prefill: tokens per chunk")
    args = ap.parse_args()
    if args.workload == "profile-case":
        return run_profile_case(args)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.workload == "layer-ops":
        run_layer_ops(args)
    elif args.workload == "llama8b-tp":
        run_llama8b_tp(args)
    elif args.workload == "batched":
        run_batched(args)
    elif args.workload == "longctx":
        run_batched(args, longctx=True)
    elif args.workload == "longctx-tp":
        run_batched(args, longctx=True, tp=True)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "serving":
        run_serving(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

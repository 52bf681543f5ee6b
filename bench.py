#!/usr/bin/env python
"""Decode throughput of the Llama-3-8B-shaped model (BASELINE metric:
"decode tok/s (Llama-8B shape, bs1) at 1/2/4/8 B200; GEMV % of HBM peak").

A step is one decode step of the whole batch (32 layers + lm_head + greedy
argmax) replayed from the captured CUDA graph.  Workload:
random-init fp16 weights ~N(0, 0.02) (seeded), a 512-token uniform random
prompt (prefilled untimed), then W warm-up and K timed decode steps at batch B,
context 512+W .. 512+W+K.  Each step streams ~15 GB of weights, far more than
the 126 MB L2, so no flush is needed.

  value    device-resident greedy loop (b2_model_generate_greedy), CUDA events
           on the model's stream, max over ranks
  e2e      the public step API b2_model_decode_step: host token/position in
           (H2D from pinned memory), fp32 logits [B, V] and next ids out (D2H),
           every step
  roofline the dominant kernel (gate/up GEMV with SwiGLU epilogue) timed on its
           launch stream, algorithmic bytes / avg launch time vs measured HBM peak
  cpu_baseline  the reference's CPU forward (src/model/forward_cpu.cpp, no KV
           cache: a decode token recomputes every position) on the host's
           cores, one decoder layer at the bench's context as the sample

N > 1 runs Megatron tensor parallelism (one process per GPU under torchrun),
the decode-step reductions over NVLink peer memory (or NCCL with --exchange
nccl); before the timed region a 2-layer sharded model is checked against the
same model unsharded ("tp_parity").  `--impl reference` times the reference's
CPU path instead.
"""
import argparse
import datetime as dt
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "serving-engine_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "decode tok/s (Llama-8B shape, bs1) at 1/2/4/8 B200; GEMV % of HBM peak"
LLAMA8B = dict(vocab=128256, hidden=4096, inter=14336, layers=32, nq=32, nkv=8, head_dim=128, eps=1e-5,
               theta=500000.0)
# BASELINE's model shapes (random-init; the metric's default is llama3-8b)
MODELS = {
    "llama3-8b": LLAMA8B,
    "llama3-70b": dict(vocab=128256, hidden=8192, inter=28672, layers=80, nq=64, nkv=8, head_dim=128, eps=1e-5,
                       theta=500000.0),
    "tinyllama-1.1b": dict(vocab=32000, hidden=2048, inter=5632, layers=22, nq=32, nkv=4, head_dim=64, eps=1e-5,
                           theta=10000.0),
}


def weight_gb(c):
    lin = c["layers"] * ((c["nq"] + 2 * c["nkv"]) * c["head_dim"] * c["hidden"] + c["hidden"] * c["nq"] *
                         c["head_dim"] + 3 * c["inter"] * c["hidden"]) + 2 * c["vocab"] * c["hidden"]
    return 2.0 * lin / 1e9


def model_cfg(args):
    c = dict(MODELS[args.model])
    if args.layers:
        c["layers"] = args.layers
    return c
PROMPT = 512
PAGE = 16  # KV block size of the paged mode (the reference runner's default)
SEED_W, SEED_P = 1234, 42
FALLBACK_HBM = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy burst)"
    except Exception:
        return FALLBACK_HBM, "fallback (6.65 TB/s, earlier measurement on this pool)"


def ncu_traffic(kernel_tag):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/ (or None)."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for fn in sorted(os.listdir(d)):
        if not fn.endswith(".md"):
            continue
        try:
            with open(os.path.join(d, fn)) as f:
                for line in f:
                    if line.startswith(f"traffic_bytes_per_launch[{kernel_tag}]:"):
                        return float(line.split(":", 1)[1].strip())
        except OSError:
            pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms in the background."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        self.windows = []

    def mark(self, t0, t1):
        self.windows.append((t0, t1))

    def stop(self):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except Exception:
                self.p.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(", ") for r in self.f.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.f.name)
        samples = []
        for r in rows:
            try:
                ts = dt.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
                samples.append((ts, float(r[1]), float(r[2]), r[3], r[5:9]))
            except Exception:
                continue
        inside = [s for s in samples if any(a - 0.15 <= s[0] <= b + 0.15 for a, b in self.windows)] or samples
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in inside for i, v in enumerate(s[4]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": max(s[2] for s in inside),
                "reasons": reasons, "samples": len(inside)}


# ---------------------------------------------------------------------------
# CPU: the reference's src/cpu path
# ---------------------------------------------------------------------------

class RefLayerSample:
    """The reference's CPU decode at this bench's widths, as a bounded sample.

    The reference's CPU path (src/model/forward_cpu.cpp:58-174) has no KV
    cache: to decode the token after a context of c tokens it recomputes the
    whole forward over c + 1 positions.  One sample is one of its L decoder
    layers over those c + 1 positions (embedding, the layer, final norm) on
    all host threads, through the oracle port (oracle/b2oracle.c, pinned
    bit-exact to the reference's own build by tests/test_oracle.py and
    split across threads by output row only, so every value is the
    reference's).  The lm_head is timed once for the LAST position only
    (the reference computes all c + 1 rows of logits): a decode token then
    costs L x layer + head, which flatters the reference."""

    def __init__(self, c, ctx1):
        import numpy as np
        import oracle as O
        self.threads = os.cpu_count() or 1
        O.set_threads(self.threads)
        self.O, self.L, self.ctx1 = O, c["layers"], ctx1
        cfg1 = O.Config(**{**c, "layers": 1}, tied=True)
        self.cfg1 = cfg1
        self.W = O.seeded_weights(cfg1, SEED_W)
        self.ids = np.random.default_rng(SEED_P).integers(0, cfg1.vocab, ctx1).astype(np.int64)
        self.row = np.ones((1, cfg1.hidden), np.float32)
        self.kind = "port"

    def layer(self):
        """Seconds for one decoder layer of the recompute over ctx1 positions."""
        a = time.perf_counter()
        self.O.forward(self.cfg1, self.W, self.ids, logit_row0=self.ctx1)
        return time.perf_counter() - a

    def head(self):
        """Seconds for the lm_head of one position."""
        a = time.perf_counter()
        self.O.matmul_transB(self.row, self.W["embed"])
        return time.perf_counter() - a

    def describe(self):
        return (f"one decoder layer of the reference CPU forward (no KV cache: full recompute) over the "
                f"{self.ctx1} positions a decode token at context {self.ctx1 - 1} recomputes, "
                f"{self.cfg1.hidden}-wide, on {self.threads} host threads (oracle port, bit-identical to the "
                f"reference, split by output row); tok/s = 1 / ({self.L} x layer + lm_head of the last position "
                f"only: the reference computes all {self.ctx1} logit rows, so this flatters it)")


def cpu_baseline_single(c, ctx1):
    """cpu_baseline of the GPU arm: two layer samples and one lm_head sample."""
    smp = RefLayerSample(c, ctx1)
    lay = min(smp.layer() for _ in range(2))
    head = smp.head()
    step = smp.L * lay + head
    return {"value": 1.0 / step, "unit": "tok/s", "cores": smp.threads, "kind": smp.kind,
            "sample": smp.describe(), "layer_s": lay, "head_s": head, "token_s": step}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU decode at the bench's model and
    context.  Each warm-up and timed step runs one layer sample (all host
    threads); ms_per_step is that sample's time, tok/s counts the model's L
    layers at the timed per-layer cost plus the last row's lm_head."""
    if rank != 0:
        return
    c = model_cfg(args)
    ctx1 = args.prompt + args.warmup + args.steps // 2 + 1
    smp = RefLayerSample(c, ctx1)
    head = min(smp.head() for _ in range(2))
    for _ in range(args.warmup):
        smp.layer()
    layer_times = [smp.layer() for _ in range(args.steps)]
    lay = statistics.mean(layer_times)
    token_s = smp.L * lay + head
    value = 1.0 / token_s
    sample = smp.describe() + f"; each of the {args.steps} timed steps runs one layer sample"
    cfg = config_dict(args, world)
    cfg["workload"] = (f"{args.model}-shaped bs1 decode at context {ctx1 - 1} on the reference's CPU path: each "
                       f"step times one of its {smp.L} decoder layers over the {ctx1}-position recompute "
                       f"(ms_per_step); tok/s = 1 / ({smp.L} x the mean layer time + one lm_head row)")
    cfg["global_batch"] = 1
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": lay * 1e3,
           "ms_per_token": token_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic: seeded random-init weights ~N(0,0.02) rounded to fp16, uniform "
                                   "random prompt ids",
           "config": cfg,
           "cpu_baseline": {"value": value, "unit": "tok/s", "cores": smp.threads, "kind": smp.kind,
                            "sample": sample, "layer_s": lay, "head_s": head},
           "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def config_dict(args, world):
    c = model_cfg(args)
    if args.paged:
        wl = (f"{args.model}-shaped decode over a paged KV cache ({PAGE}-position blocks scattered over a pool), "
              f"batch {args.batch}, prompts of {args.prompt // 2}..{args.prompt * 3 // 2} tokens (mixed), then "
              f"{args.warmup}+{args.steps} decode steps")
    else:
        wl = (f"{args.model}-shaped decode, batch {args.batch}, {args.prompt}-token prompt then "
              f"{args.warmup}+{args.steps} decode steps")
    return {"workload": wl,
            "model": f"{args.model}-shape random-init (H{c['hidden']} L{c['layers']} {c['nq']}/{c['nkv']} heads "
                     f"D{c['head_dim']} FFN{c['inter']} V{c['vocab']}, theta {c['theta']:g})",
            "global_batch": args.batch, "prompt_len": args.prompt,
            "ctx_range": [args.prompt + args.warmup, args.prompt + args.warmup + args.steps],
            "parallelism": f"tp{world}",
            "tp_exchange": (args.exchange if world > 1 else None),
            "weights": ("fp16" if args.weights == "fp16" else
                        "fp8 e4m3 per-row copies for the decode GEMVs (b2_model_quantize_weights)"
                        if args.weights == "fp8" else
                        "4-bit copies, fp32 scale per 128 weights, for the batch-1/2 decode GEMVs "
                        "(b2_model_quantize_weights)"),
            "l2": f"inputs larger than L2: every step streams the model's {weight_gb(c):.1f} GB of fp16 weights "
                  f"(half that as fp8; divided over the tensor-parallel ranks; L2 126 MB)"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def tp_parity(args, rank, world):
    """Sharded-path correctness for N > 1, checked before the timed region.

    A 2-layer model at the bench's widths runs tensor-parallel over the N
    ranks (same exchange as the timed run): prefill of a 16-token prompt, 9
    greedy tokens from the device loop, then the same positions teacher-forced
    through b2_model_decode_step with the logits gathered from every rank.
    Rank 0 runs the identical model unsharded (tp = 1) on its own GPU and
    compares: logits max-abs <= 2e-2 and cosine >= 0.9999 at every position,
    and every sharded greedy id equal to the unsharded argmax unless that row's
    top-1 / top-2 margin is below 0.05.  The unsharded model is the one the
    -m gpu tests check against the reference's CPU forward at these widths."""
    import numpy as np
    import torch.distributed as dist

    import b2engine as b2
    c = model_cfg(args)
    S0, n, L2, seed = 16, 9, 2, SEED_W + 1

    def build(r, t, nid):
        m = b2.Model(c["vocab"], c["hidden"], c["inter"], L2, c["nq"], c["nkv"], c["head_dim"], eps=c["eps"],
                     theta=c["theta"], tied=False, max_batch=1, max_seq=64, tp_rank=r, tp_size=t, nccl_id=nid)
        m.init_random(seed, 0.02)
        return m

    obj = [b2.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    ms = build(rank, world, obj[0])
    if args.exchange == "p2p":
        handles = [None] * world
        dist.all_gather_object(handles, ms.p2p_handle())
        ms.p2p_open(handles)
    prompt = np.random.default_rng(SEED_P + 1).integers(0, c["vocab"], (1, S0))
    lg_s = [ms.prefill(prompt)[0].copy()]
    gen = ms.generate_greedy(n)[:, 0].copy()
    ms.reset()
    ms.prefill(prompt, want_logits=False)
    for i in range(n - 1):
        lg, _ = ms.decode_step([gen[i]], [S0 + i])
        lg_s.append(lg[0].copy())
    ms.close()
    res = None
    if rank == 0:
        mu = build(0, 1, None)
        lg_u = [mu.prefill(prompt)[0].copy()]
        for i in range(n - 1):
            lg, _ = mu.decode_step([gen[i]], [S0 + i])
            lg_u.append(lg[0].copy())
        mu.close()
        max_abs, cos_min, greedy_ok, ties = 0.0, 1.0, True, 0
        for i in range(n):
            a, b = np.asarray(lg_s[i], np.float64), np.asarray(lg_u[i], np.float64)
            max_abs = max(max_abs, float(np.max(np.abs(a - b))))
            cos_min = min(cos_min, float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30)))
            if int(gen[i]) != int(np.argmax(b)):
                srt = np.sort(b)[::-1]
                if srt[0] - srt[1] < 0.05:
                    ties += 1
                else:
                    greedy_ok = False
        ok = max_abs <= 2e-2 and cos_min >= 0.9999 and greedy_ok
        res = {"ok": ok, "max_abs": max_abs, "cos_min": cos_min, "greedy_ok": greedy_ok, "near_tie_flips": ties,
               "greedy_tokens": n, "positions": n, "layers": L2, "tp": world, "exchange": args.exchange,
               "reference": "the same seeded 2-layer model unsharded (tp=1) on rank 0's GPU"}
        log(f"[rank 0] tp parity: {res}")
    dist.barrier()
    return res


def run_b2(args, rank, world, local):
    import numpy as np
    import torch
    import torch.distributed as dist

    import b2engine as b2

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    parity = tp_parity(args, rank, world) if world > 1 and not args.no_tp_parity else None
    nccl_id = None
    if world > 1:
        obj = [b2.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    B, K, W = args.batch, args.steps, args.warmup
    max_seq = max(4096, 2 * args.prompt + 2 * (W + K) + 8)
    c = model_cfg(args)
    kv_blocks = 0
    if args.paged:  # pool with room for every sequence's blocks, scattered
        kv_blocks = B * ((args.prompt * 3 // 2 + 2 * (W + K) + 8 + PAGE - 1) // PAGE)
    m = b2.Model(c["vocab"], c["hidden"], c["inter"], c["layers"], c["nq"], c["nkv"], c["head_dim"], eps=c["eps"],
                 theta=c["theta"], tied=False, max_batch=B, max_seq=max_seq, tp_rank=rank, tp_size=world,
                 nccl_id=nccl_id, kv_blocks=kv_blocks, block_size=PAGE)
    m.init_random(SEED_W, 0.02)
    if args.weights != "fp16":  # decode GEMVs on quantised copies (prefill stays fp16)
        m.quantize_weights(args.weights)
    if world > 1 and args.exchange == "p2p":
        # decode-step partial sums over NVLink peer memory (fused into the
        # GEMVs) instead of NCCL all-reduces
        handles = [None] * world
        dist.all_gather_object(handles, m.p2p_handle())
        m.p2p_open(handles)
    prompt = np.random.default_rng(SEED_P).integers(0, c["vocab"], (B, args.prompt))
    if args.paged:
        # mixed lengths: sequence b's prompt is lens[b] tokens, its blocks a
        # random scatter over the pool; prefilled one sequence at a time
        prng = np.random.default_rng(SEED_P + 7)
        lens = [int(x) for x in prng.integers(args.prompt // 2, args.prompt * 3 // 2 + 1, B)]
        perm = list(prng.permutation(kv_blocks))
        per_seq = kv_blocks // B
        tables = np.array([perm[b * per_seq:(b + 1) * per_seq] for b in range(B)], np.int32)
        firsts = np.zeros(B, np.int64)
        m.prefill_paged(prompt[0, :lens[0]], tables[0])  # first call: workspace allocation, module load
        torch.cuda.synchronize()
        t = time.time()
        for b in range(B):
            firsts[b] = m.prefill_paged(prompt[b, :lens[b]], tables[b])[0]
        prefill_s = time.time() - t
        # the device loop continues every sequence from its own position
        m.decode_step_paged(firsts, [n + 1 for n in lens], tables)
        log(f"[rank {rank}] paged prefill of {B} prompts of {min(lens)}..{max(lens)} tokens in "
            f"{prefill_s * 1e3:.1f} ms")
    else:
        m.prefill(prompt, want_logits=False)  # first call: workspace allocation, module load
        m.reset()
        torch.cuda.synchronize()
        t = time.time()
        m.prefill(prompt, want_logits=False)
        prefill_s = time.time() - t
        log(f"[rank {rank}] prefill {B}x{args.prompt} tokens in {prefill_s * 1e3:.1f} ms")
    stream = torch.cuda.ExternalStream(m.stream, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    clocks = ClockSampler(uuid)
    time.sleep(0.3)

    # warm-up: W device-resident steps
    m.generate_greedy(W, fetch=False)
    m.sync()
    pos0 = args.prompt + W
    if args.paged:  # next position of each sequence after the warm-up and timed loops
        pos_b = np.array([n + 1 + W + K for n in lens])

    # value: K device-resident steps, CUDA events on the model's stream
    barrier()
    torch.cuda.synchronize()
    m.sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.time()
    e0.record(stream)
    m.generate_greedy(K, fetch=False)
    e1.record(stream)
    e1.synchronize()
    w1 = time.time()
    torch.cuda.synchronize()
    barrier()
    clocks.mark(w0, w1)
    ms = max_over_ranks(e0.elapsed_time(e1))
    next_tok = m.read("tokens", np.int64, B)

    # per-kernel launch durations (dominant kernel for the roofline)
    ctx_mid = pos0 + K // 2
    try:  # the fused-GEMV step; the batched tensor-core step has no per-kind kernel
        ktimes = {k: m.time_kernel(k, B, reps=2) for k in b2.Model.KERNELS}
    except b2.B2Error:
        ktimes = {}
    kbytes = {k: m.kernel_bytes(k, B, ctx_mid) for k in b2.Model.KERNELS}

    # e2e: public step API with host buffers, same contexts as the timed loop
    barrier()
    torch.cuda.synchronize()
    tok = next_tok.copy()
    # the step's logits land in one page-locked host buffer, reused every step
    lg_host = torch.empty((B, c["vocab"]), dtype=torch.float32, pin_memory=True)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w2 = time.time()
    e2.record(stream)
    for i in range(K):
        if args.paged:
            tok, _ = m.decode_step_paged(tok, pos_b + i + 1, tables)
        else:
            _, tok = m.decode_step(tok, [pos0 + i] * B, want_logits=True, want_next=True, logits_out=lg_host)
    e3.record(stream)
    e3.synchronize()
    w3 = time.time()
    barrier()
    clocks.mark(w2, w3)
    ms_e2e = max_over_ranks(e2.elapsed_time(e3))
    ck = clocks.stop()

    trace = None
    if not args.no_trace:
        # per-launch device timestamps of a few live steps (b2_model_trace_step)
        L = c["layers"]
        layouts = [  # launch sequences of the step forms, in launch order
            # fused-GEMV step
            ["step_begin"] + ["qkv", "attention", "o_proj", "gate_up", "down"] * L + ["lm_head", "step_end"],
            # batched step: skinny projections and the kernels that sum their partials
            ["step_begin"] + ["qkv", "qkv_sum_rope", "attention", "o_proj", "o_sum_norm", "gate_up", "swiglu",
                              "down", "down_sum_norm"] * L + ["lm_head", "logits_argmax", "step_end"],
        ]
        runs = np.stack([m.trace_step(B) for _ in range(5)])
        t = np.median(runs, axis=0)
        names = next((n for n in layouts if len(n) == len(t)), [f"k{i}" for i in range(len(t))])
        agg, prev = {}, 0
        for i, (a, e) in enumerate(t):
            g = agg.setdefault(names[i] if i < len(names) else f"k{i}", [0, 0.0, 0.0])
            g[0] += 1
            g[1] += (e - a) / 1e3
            g[2] += (a - prev) / 1e3
            prev = e
        trace = {"step_span_us": float(t[-1, 1] - t[0, 0]) / 1e3,
                 "per_kernel": {k: {"launches": n, "mean_us": d / n, "mean_gap_before_us": gp / n}
                                for k, (n, d, gp) in agg.items()},
                 "how": "b2_model_trace_step: %globaltimer at the first CTA past its programmatic-launch wait and "
                        "at the last CTA's end, median of 5 steps, rank 0"}

    if rank == 0:
        peak, peak_src = measured_peak()
        step_ms = ms / K
        step_bytes = m.step_bytes(B, ctx_mid)
        step_gbs = step_bytes / (step_ms * 1e-3) / 1e9
        if ktimes:
            dom = "gate_up"
            achieved, dom_bytes, dom_ms, dom_name = (kbytes[dom] / (ktimes[dom] * 1e-3) / 1e9, kbytes[dom],
                                                     ktimes[dom], f"gemv {dom}")
        else:
            achieved, dom_bytes, dom_ms, dom_name = step_gbs, step_bytes, step_ms, "whole decode step (batched)"
        launches = m.step_launches(B)
        out = {
            "metric": METRIC, "value": B * K / (ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": {"fp16": "f16", "fp8": "f16 activations, fp8 e4m3 weights (per-row fp32 scales)",
                      "int4": "f16 activations, 4-bit weights (fp32 scale per 128)"}[args.weights],
            "data": "synthetic: seeded random-init fp16 weights ~N(0,0.02), uniform random prompt ids",
            "config": config_dict(args, world),
            "e2e": ({"value": B * K / (ms_e2e * 1e-3), "unit": "tok/s",
                     "h2d_bytes_per_step": 12 * B + 4 * int(tables.size), "d2h_bytes_per_step": 8 * B,
                     "ms_per_step": ms_e2e / K,
                     "api": "b2_model_decode_step_paged (host tokens, sequence lengths and block tables in, "
                            "next ids out)"} if args.paged else
                    {"value": B * K / (ms_e2e * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 12 * B,
                     "d2h_bytes_per_step": 4 * B * c["vocab"] + 8 * B, "ms_per_step": ms_e2e / K,
                     "api": "b2_model_decode_step (host token + position in, fp32 logits into a reused page-locked "
                            "host buffer + next id out)"}),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": ncu_traffic("gate_up") if ktimes and args.weights == "fp16" else None,
                         "kernel": dom_name, "bytes_per_launch": dom_bytes, "launch_ms": dom_ms,
                         "peak_source": peak_src},
            "step_roofline": {"bytes_per_step": step_bytes, "achieved": step_gbs, "peak": peak, "unit": "GB/s",
                              "frac": step_gbs / peak},
            "kernels_ms_per_launch": {k: round(v, 5) for k, v in ktimes.items()},
            "gpu_launches": launches * K,
            "prefill": {"tokens": B * args.prompt, "ms": prefill_s * 1e3, "tok_s": B * args.prompt / prefill_s,
                        "how": "b2_model_prefill wall time (host ids in, tensor-core GEMMs + flash prefill, "
                               "synchronised), second call"},
            "clocks": ck,
        }
        if trace:
            out["trace"] = trace
        if parity is not None:
            out["tp_parity"] = parity
        if world == 1 and not args.no_cpu_baseline and args.model == "llama3-8b" and args.weights == "fp16":
            try:
                out["cpu_baseline"] = cpu_baseline_single(c, ctx_mid + 1)
            except Exception as ex:  # reported, never fatal
                out["cpu_baseline"] = {"value": None, "error": str(ex)[:200]}
        print(json.dumps(out), flush=True)
    m.close()


# ---------------------------------------------------------------------------
# kernel microbenchmarks (BASELINE configs 2 and 3, prefill projections)
# ---------------------------------------------------------------------------

def _events_time(fn, iters, flush=None, back_to_back=10):
    """Median per-call milliseconds over `iters` samples timed with CUDA
    events on the current stream.  With `flush`, one call per sample, the
    flush (an L2-sized memset) enqueued first: the call is queued behind it,
    so the host's launch work never leaves the device idle inside the timed
    interval.  Without, `back_to_back` calls per sample (the device time of
    a call, not the host's time to issue it)."""
    import torch
    times = []
    for _ in range(iters):
        reps = 1
        if flush is not None:
            flush()
        else:
            reps = back_to_back
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) / reps)
    return statistics.median(times)


def run_op(args):
    import numpy as np  # noqa: F401
    import torch

    import b2engine as b2
    torch.cuda.set_device(0)
    peak_hbm, hbm_src = measured_peak()
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak_tf = float(peaks.get("bf16_tflops", 1590.0))
    flush_buf = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")  # 512 MB > 4x L2

    def flush():
        flush_buf.zero_()

    st = b2.stream_ptr()
    warm, iters = max(args.warmup, 3), max(args.steps, 1)
    out = {"metric": None, "n_gpus": 1, "steps": iters, "warmup": warm, "data": "synthetic ~N(0,1)"}
    if args.op == "attention":
        # split-KV decode attention: fp16 q [B,32,128], K/V [B,ctx,8,128] token-major, GQA 4:1
        nq, nkv, D = 32, 8, 128
        cases = []
        shapes = [(B, ctx) for B in (1, 8, 32) for ctx in (512, 4096, 32768)]
        if args.seq:  # one case: --batch B --seq ctx
            shapes = [(args.batch, args.seq)]
        for B, ctx in shapes:
            g = torch.Generator(device="cuda").manual_seed(B * 100003 + ctx)
            q = torch.randn(B, nq, D, generator=g, device="cuda").half()
            k = torch.randn(B, ctx, nkv, D, generator=g, device="cuda").half()
            v = torch.randn(B, ctx, nkv, D, generator=g, device="cuda").half()
            lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
            o = torch.empty_like(q)
            split = torch.empty(B * nq * 132 * (D + 2) + 4096, dtype=torch.float32, device="cuda")
            kv = b2.KVView(k.data_ptr(), ctx * nkv * D, D, nkv * D, 1)
            vv = b2.KVView(v.data_ptr(), ctx * nkv * D, D, nkv * D, 1)

            def fn():
                b2.call("b2_decode_gqa_split", q.data_ptr(), kv, vv, lens.data_ptr(), o.data_ptr(), B, nq, nkv, D,
                        ctx, split.data_ptr(), split.numel(), st)
            for _ in range(warm):
                fn()
            ms = _events_time(fn, iters, flush)
            nbytes = 4.0 * B * ctx * nkv * D + 4.0 * B * nq * D
            gbs = nbytes / (ms * 1e-3) / 1e9
            cases.append({"B": B, "ctx": ctx, "us": ms * 1e3, "bytes": nbytes, "GBs": gbs, "frac": gbs / peak_hbm})
            del q, k, v, o, split
        out.update({"metric": "split-KV decode attention achieved HBM GB/s (fp16, Hq 32 / Hkv 8, D 128)",
                    "value": max(c["GBs"] for c in cases), "unit": "GB/s", "higher_is_better": True,
                    "dtype": "f16", "config": {"workload": "BASELINE split-KV decode attention microbench",
                                               "l2": "512 MB buffer written between timed calls"},
                    "cases": cases, "peak": peak_hbm, "peak_source": hbm_src})
    elif args.op == "flash_prefill":
        nq, nkv, D = 32, 8, 128
        cases = []
        for S in ([args.seq] if args.seq else [2048, 8192]):
            g = torch.Generator(device="cuda").manual_seed(S)
            q = torch.randn(S, nq, D, generator=g, device="cuda").bfloat16()
            k = torch.randn(S, nkv, D, generator=g, device="cuda").bfloat16()
            v = torch.randn(S, nkv, D, generator=g, device="cuda").bfloat16()
            o = torch.empty_like(q)
            for rope in (500000.0, 0.0):
                def fn():
                    b2.call("b2_flash_prefill_gqa_ex", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), S, nq,
                            nkv, D, 1, 1, rope, 0, st)
                for _ in range(warm):
                    fn()
                ms = _events_time(fn, iters)
                flop = 2.0 * S * S * D * nq
                tf = flop / (ms * 1e-3) / 1e12
                cases.append({"S": S, "rope_theta": rope, "us": ms * 1e3, "flop": flop, "TFLOPs": tf,
                              "frac": tf / peak_tf})
            assert b2.device_status() == 0
        out.update({"metric": "causal flash prefill TFLOP/s (bf16, tcgen05, Hq 32 / Hkv 8, D 128)",
                    "value": max(c["TFLOPs"] for c in cases), "unit": "TFLOP/s", "higher_is_better": True,
                    "dtype": "bf16", "config": {"workload": "BASELINE causal flash prefill, batch 1",
                                                "flop": "2*S^2*D*Hq (causal half of 4*S^2*D*Hq)"},
                    "cases": cases, "peak": peak_tf, "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops)"})
    elif args.op == "gemv":
        # the decode GEMV's weight forms on the gate|up shape at batch 1:
        # fp16, FP8 rows (b2_gemv_fp8), 4-bit groups of 128 (b2_gemv_int4),
        # all quantised by the library from one seeded fp16 matrix
        N, K = 28672, 4096
        g = torch.Generator(device="cuda").manual_seed(7)
        w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
        x = torch.randn(1, K, generator=g, device="cuda").half()
        y = torch.empty(1, N, dtype=torch.float16, device="cuda")
        q8 = torch.empty(N, K, dtype=torch.uint8, device="cuda")
        s8 = torch.empty(N, dtype=torch.float32, device="cuda")
        q4 = torch.empty(N, K // 2, dtype=torch.uint8, device="cuda")
        s4 = torch.empty(N, K // 128, dtype=torch.float32, device="cuda")
        b2.call("b2_quantize_fp8_rows", w.data_ptr(), N, K, q8.data_ptr(), s8.data_ptr(), st)
        b2.call("b2_quantize_int4_rows", w.data_ptr(), N, K, q4.data_ptr(), s4.data_ptr(), st)
        forms = [
            ("fp16", 2.0 * N * K, lambda: b2.call("b2_gemv", w.data_ptr(), x.data_ptr(), y.data_ptr(), N, K, st)),
            ("fp8", 1.0 * N * K + 4.0 * N,
             lambda: b2.call("b2_gemv_fp8", q8.data_ptr(), s8.data_ptr(), x.data_ptr(), y.data_ptr(), 1, N, K, 0, st)),
            ("int4", 0.5 * N * K + 4.0 * N * K / 128,
             lambda: b2.call("b2_gemv_int4", q4.data_ptr(), s4.data_ptr(), x.data_ptr(), y.data_ptr(), 1, N, K, 0,
                             st)),
        ]
        cases = []
        for name, nbytes, fn in forms:
            for _ in range(warm):
                fn()
            ms = _events_time(fn, iters, flush)
            gbs = nbytes / (ms * 1e-3) / 1e9
            cases.append({"weights": name, "N": N, "K": K, "us": ms * 1e3, "bytes": nbytes, "GBs": gbs,
                          "frac": gbs / peak_hbm})
        assert b2.device_status() == 0
        out.update({"metric": "decode GEMV achieved HBM GB/s by weight form (batch 1, N 28672, K 4096)",
                    "value": max(c["GBs"] for c in cases), "unit": "GB/s", "higher_is_better": True,
                    "dtype": "f16 activations", "config": {"workload": "Llama-3-8B gate|up GEMV shape, batch 1",
                                                          "l2": "512 MB buffer written between timed calls"},
                    "cases": cases, "peak": peak_hbm, "peak_source": hbm_src})
    elif args.op == "gemm":
        cases = []
        for (M, K, N) in [(512, 4096, 6144), (2048, 4096, 6144), (2048, 4096, 28672), (2048, 14336, 4096),
                          (8192, 4096, 6144)]:
            A = torch.randn(M, K, device="cuda").half()
            Bw = torch.randn(N, K, device="cuda").half()
            C = torch.empty(M, N, device="cuda").half()

            def fn():
                b2.call("b2_matmul_transB", A.data_ptr(), Bw.data_ptr(), C.data_ptr(), M, K, N, st)
            for _ in range(warm):
                fn()
            ms = _events_time(fn, iters)
            tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            cases.append({"M": M, "K": K, "N": N, "us": ms * 1e3, "TFLOPs": tf, "frac": tf / peak_tf})
            del A, Bw, C
        assert b2.device_status() == 0
        out.update({"metric": "prefill projection GEMM TFLOP/s (fp16 in, fp32 accumulate, tcgen05)",
                    "value": max(c["TFLOPs"] for c in cases), "unit": "TFLOP/s", "higher_is_better": True,
                    "dtype": "f16", "config": {"workload": "Llama-3-8B prefill projection shapes"},
                    "cases": cases, "peak": peak_tf, "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops)"})
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", default="b2", choices=["b2", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tp-parity", action="store_true",
                    help="skip the sharded-vs-unsharded check run before the timed region at N > 1")
    ap.add_argument("--trace", action="store_true",
                    help="(the default) add a per-kernel device trace of five steps, taken after the timed region")
    ap.add_argument("--no-trace", action="store_true", help="leave the per-kernel trace out")
    ap.add_argument("--op", default=None, choices=["attention", "flash_prefill", "gemm", "gemv"],
                    help="kernel microbenchmark instead of the decode metric (1 GPU)")
    ap.add_argument("--seq", type=int, default=0,
                    help="--op flash_prefill: one sequence length; --op attention: one context (with --batch)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="tensor-parallel decode reduction: fused peer-memory exchange or NCCL all-reduce")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt length (512 for the metric)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder depth override (reduced only for small profiler captures; 0 = the model's)")
    ap.add_argument("--weights", default="fp16", choices=["fp16", "fp8", "int4"],
                    help="decode GEMV weights: fp16 (the metric), per-row FP8 E4M3 copies "
                         "(b2_model_quantize_weights; batches the GEMV step takes), or 4-bit copies "
                         "with a scale per 128 weights (batch 1-2)")
    ap.add_argument("--paged", action="store_true",
                    help="paged KV cache (16-position blocks scattered over a pool), mixed prompt lengths "
                         "prompt/2 .. 3*prompt/2, prefilled one sequence at a time")
    ap.add_argument("--model", default="llama3-8b", choices=sorted(MODELS),
                    help="model shape (the metric is quoted on llama3-8b)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.op:
        if rank == 0:
            run_op(args)
        return
    if world > 1:
        # one node: NCCL's bootstrap goes over loopback (its default pick, the
        # first non-loopback interface, may not route between local processes);
        # the data path is NVLink either way
        os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=dt.timedelta(seconds=300))
    try:
        run_b2(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

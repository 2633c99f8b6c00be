"""Benchmark of the MoE quantized-expert layer.

Workload: one MoE layer at Qwen3-30B-A3B shape -- hidden 2048, 128 experts,
top-8, moe_intermediate 768, SwiGLU, q4_0 experts from N(0, 0.02), f32
router N(0, 0.02), x ~ N(0, 1) -- over a batch of M decode tokens per GPU
(default M=64; --tokens). A step is one hale_moe_forward over the batch.
Metric: decode tokens/s through the layer (BASELINE: "decode tok/s ...;
q4_0 MoE GEMV achieved HBM GB/s").

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens M]
  python bench.py --impl reference ...   # the reference's CPU path (oracle port)

Multi-GPU (torchrun): the layer is split over the N GPUs by expert
parallelism -- each rank holds E/N experts and brings its own M tokens
(per-GPU tokens fixed -> weak scaling); a step is one hale_moe_forward_ep
per rank (records and y rows stored into peer memory over NVLink), timed
with CUDA events, max over ranks. The line says whether every rank's output
equals the 1-GPU layer bit for bit, and carries beside it the replicas time
(every GPU all experts) and the host-driven NCCL all-to-all-v exchange.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

SEED = 2026
E, H, I, K_TOP = 128, 2048, 768, 8
WORKLOAD = "moe_layer_qwen3_30b_a3b_q4_0"
# DRAM bytes (read + write) of one expert_gate_up_ws_kernel<q4_0, 4, 1> launch on this
# bench's seeded 64-token step (126 distinct experts), from one ncu --set full capture:
# dram__bytes_read.sum 224.354 MB + dram__bytes_write.sum 4.644 MB. Reported only for
# that token count.
NCU_GATE_UP_TRAFFIC = {64: 224354048 + 4643840}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--impl", default="hale", choices=["hale", "reference"])
    p.add_argument("--no-sweep", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-ep", action="store_true", help="skip the host-driven NCCL exchange measurement at N > 1")
    p.add_argument("--no-decode", action="store_true",
                   help="skip the whole-model decode figures (config-2 shapes) carried in the N=1 line")
    p.add_argument("--decode", action="store_true",
                   help="whole-model decode tok/s (BASELINE config 2 shapes; --batch sequences) instead of the layer")
    p.add_argument("--layers", type=int, default=48, help="--decode: decoder layers")
    p.add_argument("--prompt", type=int, default=64, help="--decode: positions filled before timing")
    p.add_argument("--batch", type=int, default=1,
                   help="--decode: sequences decoded together (one row each per hale_decoder_step)")
    return p.parse_args()


def config(m, n):
    par = ("dp1" if n == 1 else
           f"ep{n} (experts split over {n} GPUs, {E // n} each; records and y rows over NVLink peer memory)")
    return {"workload": WORKLOAD, "hidden": H, "experts": E, "top_k": K_TOP,
            "moe_intermediate": I, "expert_dtype": "q4_0", "router_dtype": "f32",
            "tokens_per_gpu": m, "global_batch": m * n, "parallelism": par,
            "inputs": "seeded synthetic: weights N(0,0.02), x N(0,1)",
            "l2": "flushed between timed steps (256 MiB write, untimed)"}


# ---------------------------------------------------------------------------
# host data
# ---------------------------------------------------------------------------
def make_layer(fmt):
    return fmt.SyntheticLayer(SEED, E, H, I, fmt.Q4_0)


def encode_all(ld):
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(min(16, os.cpu_count() or 4)) as ex:
        return list(ex.map(ld.expert_encoded, range(E)))


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def oracle_tok_s(ld, encoded, m, budget_s=8.0):
    """The oracle (C restatement of the reference CPU path, OpenMP over rows
    like rayon) on a bounded sample of the same tokens -> tokens/s."""
    from oracle import oracle as O
    fmt = __import__("importlib").import_module("hale-token_b200.formats")
    # every core this process may run on (torchrun sets OMP_NUM_THREADS=1)
    O.set_num_threads(len(os.sched_getaffinity(0)), native=True)
    experts = [O.ExpertWeights(fmt.Q4_0, H, I, *encoded[e]) for e in range(E)]
    renc = fmt.encode(fmt.F32, ld.router)
    x = ld.tokens(m)
    O.moe_forward(fmt.F32, renc, experts, K_TOP, True, x[:1], native=True)  # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        take = min(m, 8)
        O.moe_forward(fmt.F32, renc, experts, K_TOP, True, x[:take], native=True)
        done += take
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, done, dt, O.num_threads(native=True)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device, self.rows, self.proc = device, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        reasons = set()
        sm = []
        smax = None
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                smax = float(r[2])
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def measure_ep(hale, fmt, ctx, ld, encoded, router, world, rank, m, args, flush, barrier, max_over_ranks):
    """The layer split over `world` ranks by expert parallelism: this rank
    holds experts [rank*E/world, (rank+1)*E/world) and its own m tokens; a step
    is one ep.moe_forward_ep (dispatch, NCCL all-to-all-v of the records,
    local experts, y rows back, combine). Device time per step by CUDA events
    on the current stream, L2 flushed before each step, max over ranks."""
    import importlib

    import torch
    ep = importlib.import_module("hale-token_b200.ep")
    epr = E // world
    pool = hale.Pool(ctx, fmt.Q4_0, H, I, 1, epr)
    for le in range(epr):
        pool.upload(0, le, fmt.pack_record(*encoded[rank * epr + le]))
    layer = hale.moe_layer(0, router, fmt.F32, E, K_TOP, True)
    backend = ep.CudaEpBackend(ctx, pool, layer, H, rank, world)
    exch = ep.Exchange(device=f"cuda:{torch.cuda.current_device()}")
    x = torch.from_numpy(ld.tokens(m, seed=1000 + rank)).cuda()
    for _ in range(max(args.warmup, 3)):
        ep.moe_forward_ep(backend, exch, x)
    ctx.check()
    stream = torch.cuda.current_stream()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        flush.zero_()
        a.record(stream)
        ep.moe_forward_ep(backend, exch, x)
        b.record(stream)
    torch.cuda.synchronize()
    barrier()
    ctx.check()
    ms = max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in evs])))
    return {"tok_s": world * m / (ms / 1e3), "ms_per_step": ms, "n_ranks": world, "experts_per_rank": epr,
            "tokens_per_rank": m, "exchange": "NCCL all-to-all-v via torch.distributed (counts, q8 rows, "
            "scales, route metadata; y rows back)", "bit_exact_vs_1gpu": "tests/test_gpu_ep*.py"}


def measure_ep_p2p(hale, fmt, ctx, ld, encoded, router, full_pool, world, rank, m, args, flush, barrier,
                   max_over_ranks, all_true, uid, clocks):
    """The layer split over `world` GPUs by expert parallelism, one
    hale_moe_forward_ep per step: this rank holds experts [rank*E/world,
    (rank+1)*E/world) and brings its own m tokens; records and y rows move by
    stores into peer memory. Device time per step by CUDA events on the
    launch stream, L2 flushed before each step, max over ranks. Also: the
    same call end to end from pinned host buffers (copies in the timed
    region), and whether every rank's output equals hale_moe_forward over the
    full pool on one GPU bit for bit."""
    import torch
    epr = E // world
    pool = hale.Pool(ctx, fmt.Q4_0, H, I, 1, epr)
    for le in range(epr):
        pool.upload(0, le, fmt.pack_record(*encoded[rank * epr + le]))
    layer = hale.moe_layer(0, router, fmt.F32, E, K_TOP, True)
    comm = hale.Comm(ctx, world, rank, uid, H, E, K_TOP, m)
    stream = torch.cuda.current_stream()
    try:
        x = torch.from_numpy(ld.tokens(m, seed=1000 + rank)).cuda()
        out = torch.empty((m, H), dtype=torch.float32, device="cuda")
        launches0 = ctx.launches
        for _ in range(max(args.warmup, 3)):
            hale.moe_forward_ep(ctx, comm, pool, layer, x, out)
        ctx.check()
        per_call = (ctx.launches - launches0) // max(args.warmup, 3)
        # parity with the 1-GPU layer, on this rank's tokens
        want = torch.empty_like(out)
        hale.moe_forward(ctx, full_pool, layer, x, want)
        ctx.check()
        exact = bool(torch.equal(out.view(torch.int32), want.view(torch.int32)))
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        clocks.start()
        time.sleep(0.3)
        # the timed steps, repeated (untimed) until the clock sampler has seen
        # the GPU under load for a while
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            hale.moe_forward_ep(ctx, comm, pool, layer, x, out)
            b.record(stream)
        torch.cuda.synchronize()
        t_end = time.perf_counter() + 0.5
        while time.perf_counter() < t_end:
            for _ in range(20):
                hale.moe_forward_ep(ctx, comm, pool, layer, x, out)
            torch.cuda.synchronize()
        clk = clocks.stop()
        barrier()
        ctx.check()
        ms = max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in evs])))
        # end to end: pinned x in, the call, out back, synchronised
        xh = torch.from_numpy(ld.tokens(m, seed=1000 + rank)).pin_memory()
        oh = torch.empty((m, H), dtype=torch.float32).pin_memory()
        xd = torch.empty_like(x)
        for _ in range(3):
            xd.copy_(xh, non_blocking=True)
            hale.moe_forward_ep(ctx, comm, pool, layer, xd, out)
            oh.copy_(out, non_blocking=True)
            torch.cuda.synchronize()
        barrier()
        e2e_t = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            xd.copy_(xh, non_blocking=True)
            hale.moe_forward_ep(ctx, comm, pool, layer, xd, out)
            oh.copy_(out, non_blocking=True)
            torch.cuda.synchronize()
            e2e_t.append(time.perf_counter() - t0)
        barrier()
        e2e_s = max_over_ranks(float(np.mean(e2e_t)))
        exact_all = all_true(exact)
    finally:
        comm.close()
    return {"ms": ms, "per_call_launches": per_call, "bit_exact": exact_all, "clocks": clk,
            "e2e": {"value": world * m / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": world * m * H * 4,
                    "d2h_bytes_per_step": world * m * H * 4, "ms_per_step": e2e_s * 1e3,
                    "timing": "host wall clock around x H2D (pinned), hale_moe_forward_ep, out D2H and a "
                              "synchronize on every rank; max over ranks"}}


def build_decoder(hale, fmt, ctx, L, n_seqs, max_batch, max_len):
    """A Qwen3-30B-A3B-shaped decoder: hidden 2048, 32 q /
    4 kv heads of 128, q/k norms, 128 experts top-8 of intermediate 768 in
    q4_0, vocab 151936, bf16 attention, embedding and lm_head. Synthetic
    weights: one layer's 128 expert records uploaded to every layer (each
    layer its own copy in HBM), random bf16 dense weights N(0, 0.02), norms
    1.0."""
    Hd, nh, nkv, hd, V = 2048, 32, 4, 128, 151936
    rng = np.random.default_rng(SEED)

    def bf16(rows, cols):
        a = (rng.standard_normal((rows, cols), dtype=np.float32) * 0.02).view(np.uint32)
        return (fmt.BF16, rows, cols, ((a + 0x7FFF + ((a >> 16) & 1)) >> 16).astype(np.uint16).view(np.uint8))

    ld = make_layer(fmt)
    encoded = encode_all(ld)
    pool = hale.Pool(ctx, fmt.Q4_0, Hd, I, L, E)
    records = [fmt.pack_record(*encoded[e]) for e in range(E)]
    for l in range(L):
        for e in range(E):
            pool.upload(l, e, records[e])
    ones_h, ones_d = np.ones(Hd, np.float32), np.ones(hd, np.float32)
    router = (fmt.F32, E, Hd, fmt.encode(fmt.F32, ld.router))
    layers = []
    for l in range(L):
        layers.append(dict(input_norm=ones_h, post_norm=ones_h, q_norm=ones_d, k_norm=ones_d,
                           q=bf16(nh * hd, Hd), k=bf16(nkv * hd, Hd), v=bf16(nkv * hd, Hd), o=bf16(Hd, nh * hd),
                           router=router))
    dims = dict(hidden=Hd, n_layers=L, n_heads=nh, n_kv_heads=nkv, head_dim=hd, vocab=V, n_experts=E, top_k=K_TOP,
                normalize_topk=1, eps=1e-6, rope_theta=1e6)
    dec = hale.Decoder(ctx, dims, layers, bf16(V, Hd), bf16(V, Hd), ones_h, pool, max_len, n_seqs=n_seqs,
                       max_batch=max_batch)
    shape = {"layers": L, "hidden": Hd, "heads": nh, "kv_heads": nkv, "head_dim": hd, "vocab": V, "experts": E,
             "top_k": K_TOP, "moe_intermediate": I}
    bytes_per_token = {"expert": 2 * I * fmt.row_bytes(fmt.Q4_0, Hd) + Hd * fmt.row_bytes(fmt.Q4_0, I),
                       "attn": ((nh + 2 * nkv) * hd * Hd + Hd * nh * hd) * 2, "router": E * Hd * 4,
                       "lm_head": V * Hd * 2}
    return dec, pool, shape, bytes_per_token


def decode_measure(hale, ctx, dec, shape, bpt, B, prompt, steps, warmup, seq0=0):
    """Whole-model decode of B sequences (seq0 .. seq0+B-1): each first
    prefills a `prompt`-token random prompt in batched steps (timed: prefill
    tok/s); then a step is one token of every sequence -> logits for each,
    timed with CUDA events (device time, no L2 flush: the per-step working
    set is 3.5 GB and up). B = 1 steps go through hale_decoder_forward (one
    captured CUDA graph replayed), B > 1 through hale_decoder_step."""
    import torch
    L, V = shape["layers"], shape["vocab"]
    rng = np.random.default_rng(SEED + B)
    chunk = max(B, min(prompt, 512))
    logits = torch.empty((B, V), dtype=torch.float32, device="cuda")
    max_len = prompt + steps + warmup + 6
    toks = rng.integers(0, V, size=(B, max_len))
    stream = torch.cuda.current_stream()
    pre_ms, pre_tokens = 0.0, 0
    for b in range(B):
        for s0 in range(0, prompt, chunk):
            s1 = min(prompt, s0 + chunk)
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dec.step(toks[b, s0:s1], np.arange(s0, s1), np.full(s1 - s0, seq0 + b), logits=logits[:1],
                     last_logits_only=True)
            e.record(stream)
            torch.cuda.synchronize()
            if b > 0 or s0 > 0 or B == 1:   # the very first step warms the kernels
                pre_ms += a.elapsed_time(e)
                pre_tokens += s1 - s0
    pos = prompt
    seq_ids = np.arange(seq0, seq0 + B)

    def one_step(p):
        if B == 1 and seq0 == 0:
            dec.forward(int(toks[0, p]), p, logits[0])
        else:
            dec.step(toks[:, p], np.full(B, p), seq_ids, logits=logits)

    for _ in range(warmup):
        one_step(pos)
        pos += 1
    ctx.check()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    for a, b in evs:
        a.record(stream)
        one_step(pos)
        b.record(stream)
        pos += 1
    torch.cuda.synchronize()
    ctx.check()
    ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    # per-kernel device time of eager steps (hale_ctx_profile: CUDA events around each launch)
    n_prof = min(3, max(1, steps))
    ctx.profile(True)
    for _ in range(n_prof):
        dec.step(toks[:, pos], np.full(B, pos), seq_ids, logits=logits)
        pos += 1
    names = ("embed", "rmsnorm", "fgemv", "lm_head", "qk_rope", "attention", "router", "expert_gate_up",
             "expert_down", "moe_token", "silu_mul")
    kernels = {}
    for nm in names:
        cnt, tot = ctx.profile_read(nm)
        if cnt:
            kernels[nm] = {"launches_per_step": cnt / n_prof, "us_per_step": tot * 1e3 / n_prof}
    ctx.profile(False)
    # distinct experts a step reads: expected over B tokens' independent top-8 picks
    distinct = E * (1 - (1 - K_TOP / E) ** B)
    per_step_bytes = L * (distinct * bpt["expert"] + bpt["attn"] + bpt["router"]) + bpt["lm_head"]
    return {"tok_s": B * 1e3 / ms, "ms_per_step": ms, "batch": B, "positions_before_timing": prompt,
            "steps": steps, "warmup": warmup,
            "timing": ("CUDA events around each step; steps after the first replay one captured CUDA graph "
                       "(token and position through device memory)") if B == 1 else
                      "CUDA events around each hale_decoder_step of B rows (one per sequence)",
            "algorithmic_bytes_per_step": per_step_bytes, "achieved_gbs": per_step_bytes / (ms / 1e3) / 1e9,
            "kernels": kernels,
            "kernels_timing": "eager hale_decoder_step calls with per-launch CUDA events (adds event overhead)",
            "prefill": {"tok_s": pre_tokens / (pre_ms / 1e3) if pre_ms > 0 else None, "prompt": prompt,
                        "rows_per_step": chunk, "timed_tokens": pre_tokens,
                        "timing": "CUDA events around batched hale_decoder_step calls (first one untimed at B > 1)"}}


def run_decode(args):
    """bench.py --decode: the decode figures alone, as their own line."""
    import importlib

    import torch
    hale = importlib.import_module("hale-token_b200")
    fmt = importlib.import_module("hale-token_b200.formats")
    torch.cuda.set_device(0)
    ctx = hale.Context(0)
    B = max(1, args.batch)
    max_len = args.prompt + args.steps + args.warmup + 6
    dec, pool, shape, bpt = build_decoder(hale, fmt, ctx, args.layers, B, max(B, min(args.prompt, 512)), max_len)
    r = decode_measure(hale, ctx, dec, shape, bpt, B, args.prompt, args.steps, args.warmup)
    line = {"metric": "decode_tok_s_full_model", "value": r["tok_s"], "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 experts, bf16 dense, f32 activations",
            "data": "synthetic", "config": dict(workload=f"qwen3_30b_a3b_decode_b{B}", batch=B, **shape),
            "decode": r}
    emit(line)
    dec.close()
    ctx.close()


def decode_block(hale, fmt, ctx, steps, warmup):
    """The whole-model decode figures carried in the headline line (BASELINE
    config 2 shapes, 48 layers): batch 1 and batch 16 at position 512."""
    prompt, L = 512, 48
    max_len = prompt + steps + warmup + 8
    dec, pool, shape, bpt = build_decoder(hale, fmt, ctx, L, 17, 512, max_len)
    try:
        b1 = decode_measure(hale, ctx, dec, shape, bpt, 1, prompt, steps, warmup)
        b16 = decode_measure(hale, ctx, dec, shape, bpt, 16, prompt, steps, warmup, seq0=1)
        # generate() through the public call: a fresh 512-token prompt, the
        # reference's default SamplingParams (0.7 / 0.9 / 40, seed 42)
        n_new = 16
        ptoks = np.random.default_rng(SEED + 99).integers(0, shape["vocab"], prompt).tolist()
        toks, pre_ms, dec_ms = dec.generate(ptoks, hale.SamplingParams(0.7, 0.9, 40, 1.0), 42, n_new)
        ctx.check()
        gen = {"prompt_tokens": prompt, "generated_tokens": len(toks), "prefill_ms": pre_ms, "decode_ms": dec_ms,
               "prefill_tok_s": prompt / (pre_ms / 1e3) if pre_ms > 0 else None,
               "decode_tok_s": (len(toks) - 1) / (dec_ms / 1e3) if dec_ms > 0 and len(toks) > 1 else None,
               "timing": "hale_decoder_generate's CUDA events (GenerationStats: decode rate excludes the first "
                         "token); each round samples on the device and reads the token back for the stop check"}
    finally:
        dec.close()
        del pool
    return {"metric": "decode_tok_s_full_model", "unit": "tok/s",
            "config": dict(workload="qwen3_30b_a3b_decode", **shape), "b1": b1, "b16": b16, "generate": gen}


def decode_ep_block(hale, fmt, ctx, world, rank, uid, barrier, max_over_ranks, layers=4, global_batch=32,
                    prompt=256, steps=16, warmup=3):
    """Whole-model decode across the N GPUs (BASELINE config 3's shapes:
    Mixtral-8x7B -- hidden 4096, 32 q / 8 kv heads of 128, 8 experts top-2 of
    intermediate 14336 in q8_0, vocab 32000, bf16 attention, embedding and
    lm_head -- at `layers` decoder layers instead of 32). Experts are split
    over the ranks (hale_decoder_set_comm: every MoE layer is one
    hale_moe_forward_ep); attention is data-parallel: the global batch of
    sequences is divided evenly and each rank decodes its own. Each sequence
    first prefills a `prompt`-token random prompt (one step each), then a
    step is one token of every sequence; CUDA events, max over ranks.
    Synthetic weights: dense N(0, 0.02) from the same seed on every rank,
    this rank's experts encoded from the seeded layer, one layer's records in
    every layer (each its own HBM copy), norms 1.0."""
    import torch
    from concurrent.futures import ThreadPoolExecutor
    Hd, nh, nkv, hd, V, Ex, kx, Ix = 4096, 32, 8, 128, 32000, 8, 2, 14336
    epr, B = Ex // world, global_batch // world
    rng = np.random.default_rng([SEED, 3])

    def bf16(rows, cols):
        out = np.empty((rows, cols), np.uint16)
        for r0 in range(0, rows, 4096):
            a = (rng.standard_normal((min(4096, rows - r0), cols), dtype=np.float32) * 0.02).view(np.uint32)
            out[r0:r0 + 4096] = ((a + 0x7FFF + ((a >> 16) & 1)) >> 16).astype(np.uint16)
        return (fmt.BF16, rows, cols, out.reshape(-1).view(np.uint8))

    ld = fmt.SyntheticLayer(SEED + 3, Ex, Hd, Ix, fmt.Q8_0)
    with ThreadPoolExecutor(4) as ex:
        recs = list(ex.map(lambda e: fmt.pack_record(*ld.expert_encoded(e)), range(rank * epr, (rank + 1) * epr)))
    pool = hale.Pool(ctx, fmt.Q8_0, Hd, Ix, layers, epr)
    for l in range(layers):
        for le in range(epr):
            pool.upload(l, le, recs[le])
    del recs
    ones = np.ones(Hd, np.float32)
    router = (fmt.F32, Ex, Hd, fmt.encode(fmt.F32, ld.router))
    lys = [dict(input_norm=ones, post_norm=ones, q=bf16(nh * hd, Hd), k=bf16(nkv * hd, Hd), v=bf16(nkv * hd, Hd),
                o=bf16(Hd, nh * hd), router=router) for _ in range(layers)]
    dims = dict(hidden=Hd, n_layers=layers, n_heads=nh, n_kv_heads=nkv, head_dim=hd, vocab=V, n_experts=Ex,
                top_k=kx, normalize_topk=1, eps=1e-5, rope_theta=1e6)
    max_len = prompt + steps + warmup + 2
    dec = hale.Decoder(ctx, dims, lys, bf16(V, Hd), bf16(V, Hd), ones, pool, max_len, n_seqs=B, max_batch=prompt)
    comm = hale.Comm(ctx, world, rank, uid, Hd, Ex, kx, prompt)
    stream = torch.cuda.current_stream()
    try:
        dec.set_comm(comm)
        toks = np.random.default_rng([SEED, 4, rank]).integers(0, V, size=(B, max_len))
        logits = torch.empty((B, V), dtype=torch.float32, device="cuda")
        barrier()
        for b in range(B):
            dec.step(toks[b, :prompt], np.arange(prompt), np.full(prompt, b), logits=logits[:1],
                     last_logits_only=True)
        pos = prompt
        seqs = np.arange(B)
        for _ in range(warmup):
            dec.step(toks[:, pos], np.full(B, pos), seqs, logits=logits)
            pos += 1
        ctx.check()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize()
        for a, b in evs:
            a.record(stream)
            dec.step(toks[:, pos], np.full(B, pos), seqs, logits=logits)
            b.record(stream)
            pos += 1
        torch.cuda.synchronize()
        ctx.check()
        ms = max_over_ranks(float(np.mean([a.elapsed_time(b) for a, b in evs])))
    finally:
        dec.set_comm(None)
        comm.close()
        dec.close()
    return {"metric": "decode_tok_s_full_model_ep", "tok_s": world * B / (ms / 1e3), "ms_per_step": ms,
            "unit": "tok/s", "steps": steps, "warmup": warmup,
            "config": {"workload": "mixtral_8x7b_decode_ep", "layers": layers, "layers_of_model": 32,
                       "hidden": Hd, "heads": nh, "kv_heads": nkv, "head_dim": hd, "vocab": V, "experts": Ex,
                       "top_k": kx, "moe_intermediate": Ix, "expert_dtype": "q8_0",
                       "global_batch": global_batch, "sequences_per_rank": B, "positions_before_timing": prompt,
                       "parallelism": f"ep{world} experts, data-parallel attention"},
            "timing": "CUDA events around each rank's hale_decoder_step (one row per sequence), max over ranks"}


def ep_decode_fits(world):
    """Config 3's 8 experts and global batch of 32 divide over `world` ranks."""
    return 8 % world == 0 and 32 % world == 0


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return
    fmt = __import__("importlib").import_module("hale-token_b200.formats")
    ld = make_layer(fmt)
    encoded = encode_all(ld)
    m = args.tokens
    vals = []
    for _ in range(args.warmup):
        oracle_tok_s(ld, encoded, m, budget_s=0.5)
    for _ in range(args.steps):
        v, done, dt, cores = oracle_tok_s(ld, encoded, m, budget_s=2.0)
        vals.append(v)
    v = float(np.median(vals))
    ms = m / v * 1e3
    line = {
        "metric": "decode_tok_s_moe_layer", "value": v, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 weights x i8 activations, f32 accumulate",
        "data": "synthetic", "config": config(m, world), "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"each step: >=2 s of the layer over up to 8 of the {m} tokens, repeated; "
                                   f"oracle/hale_oracle.c -O2 -march=native, OpenMP {cores} threads on {cpu_model()}"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "Rust reference cannot be built here (no cargo); the C restatement of its CPU path stands in",
    }
    emit(line)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def main():
    args = parse()
    if args.decode:
        run_decode(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import importlib

    import torch
    import torch.distributed as dist

    hale = importlib.import_module("hale-token_b200")
    fmt = importlib.import_module("hale-token_b200.formats")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ctx = hale.Context(local)
    ld = make_layer(fmt)
    encoded = encode_all(ld)
    pool = hale.Pool(ctx, fmt.Q4_0, H, I, 1, E)
    for e in range(E):
        pool.upload(0, e, fmt.pack_record(*encoded[e]))
    router = torch.from_numpy(fmt.encode(fmt.F32, ld.router)).cuda()
    layer = hale.moe_layer(0, router, fmt.F32, E, K_TOP, True)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def measure(m, steps, warmup, with_profile=False, graph=False):
        """Device time per layer call (CUDA events on the launch stream, L2
        flushed before each step). graph=True replays a captured CUDA graph
        of the call; with_profile=True also records per-kernel events."""
        x = torch.from_numpy(ld.tokens(m, seed=1000 + rank)).cuda()
        out = torch.empty((m, H), dtype=torch.float32, device="cuda")
        idx = torch.empty((m, K_TOP), dtype=torch.int32, device="cuda")
        for _ in range(warmup):
            hale.moe_forward(ctx, pool, layer, x, out, idx)
        ctx.check()
        g = None
        if graph:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                with torch.cuda.graph(g, stream=side):
                    hale.moe_forward(ctx, pool, layer, x, out, idx, stream=side)
            torch.cuda.current_stream().wait_stream(side)
            for _ in range(warmup):
                g.replay()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        launches0 = ctx.launches
        barrier()
        torch.cuda.synchronize()
        if with_profile:
            ctx.profile(True)
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            if g is not None:
                g.replay()
            else:
                hale.moe_forward(ctx, pool, layer, x, out, idx)
            b.record(stream)
        torch.cuda.synchronize()
        barrier()
        prof = {}
        if with_profile:
            ctx.profile(False)
            for kname in ("router", "expert_gate_up", "expert_down", "moe_token"):
                prof[kname] = ctx.profile_read(kname)
        ctx.check()
        ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
        distinct = int(np.unique(idx.cpu().numpy()).size)
        # kernels of this library launched in the timed region (a graph
        # replay launches the captured 3 kernels per step)
        launched = (ctx.launches - launches0) if g is None else 3 * steps
        del g
        return ms, prof, launched, distinct

    def all_true(flag):
        if world == 1:
            return bool(flag)
        t = torch.tensor([1 if flag else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        return bool(t.item())

    m = args.tokens
    ep_p2p = None
    clocks = Clocks(local)
    if world > 1:
        # ---- headline at N > 1: the layer split over the N GPUs (EP) -------
        uid = [hale.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ep_p2p = measure_ep_p2p(hale, fmt, ctx, ld, encoded, router, pool, world, rank, m, args, flush, barrier,
                                max_over_ranks, all_true, uid[0], clocks)
        ms_max = ep_p2p["ms"]
        value = world * m / (ms_max / 1e3)
        launches = ep_p2p["per_call_launches"] * args.steps
        clk = ep_p2p["clocks"]
        # replicas (every GPU all experts, its own batch) beside it
        ms_dp, _, _, distinct = measure(m, args.steps, max(args.warmup, 3), graph=True)
        ms = ms_dp
    else:
        # ---- headline: CUDA-graph replay of the layer call --------------------
        clocks.start()
        time.sleep(0.3)
        ms, _, launches, distinct = measure(m, args.steps, max(args.warmup, 3), graph=True)
        clk = clocks.stop()
        ms_max = max_over_ranks(ms)
        value = world * m / (ms_max / 1e3)
    # eager calls with per-kernel events (roofline of the dominant kernel)
    ms_eager, prof, _, _ = measure(m, args.steps, 3, with_profile=True)

    # ---- roofline of the dominant kernel (gate/up GEMV) --------------------
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak_gbs = peaks.get("hbm_gbs", 6650.0)
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    q4_row = fmt.row_bytes(fmt.Q4_0, H)
    gate_up_bytes = distinct * 2 * I * q4_row                 # weights of the touched experts
    gate_up_bytes += m * H + m * (H // 32) * 8               # quantized activations read
    n_gu, t_gu = prof.get("expert_gate_up", (0, 0.0))
    gu_ms = t_gu / max(n_gu, 1)
    achieved = gate_up_bytes / (gu_ms / 1e3) / 1e9 if gu_ms > 0 else None
    layer_bytes = distinct * fmt.row_bytes(fmt.Q4_0, H) * 2 * I + distinct * H * fmt.row_bytes(fmt.Q4_0, I)
    layer_bytes += E * H * 4 + 2 * m * H * 4
    roofline = {"bound": "hbm", "kernel": "expert_gate_up", "achieved": achieved, "peak": peak_gbs,
                "unit": "GB/s", "frac": (achieved / peak_gbs) if achieved else None,
                "traffic": NCU_GATE_UP_TRAFFIC.get(m) if world == 1 else None,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch"
                if world == 1 and m in NCU_GATE_UP_TRAFFIC else None,
                "peak_source": peak_src, "algorithmic_bytes_per_launch": gate_up_bytes,
                "avg_launch_ms": gu_ms, "distinct_experts": distinct,
                "timing": "per-kernel CUDA events over an eager timed loop of the same steps",
                "layer": {"algorithmic_bytes": layer_bytes, "ms": ms,
                          "achieved_gbs": layer_bytes / (ms / 1e3) / 1e9,
                          "frac": layer_bytes / (ms / 1e3) / 1e9 / peak_gbs}}
    kern = {k: {"launches": n, "avg_ms": (t / n if n else None)} for k, (n, t) in prof.items()}

    # ---- end to end through the public call with host buffers ---------------
    if ep_p2p is not None:
        e2e = ep_p2p["e2e"]
    else:
        xh = torch.from_numpy(ld.tokens(m, seed=1000 + rank)).pin_memory()
        oh = torch.empty((m, H), dtype=torch.float32).pin_memory()
        for _ in range(3):
            hale.moe_forward_host(ctx, pool, layer, xh, oh)
        barrier()
        e2e_t = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            hale.moe_forward_host(ctx, pool, layer, xh, oh)   # H2D, layer, D2H, sync
            e2e_t.append(time.perf_counter() - t0)
        barrier()
        e2e_s = max_over_ranks(float(np.mean(e2e_t)))
        e2e = {"value": world * m / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": m * H * 4,
               "d2h_bytes_per_step": m * H * 4, "ms_per_step": e2e_s * 1e3,
               "timing": "host wall clock around hale_moe_forward_host (pinned buffers), max over ranks"}

    # ---- sweep of the other config-1 batch sizes (one GPU) ------------------
    sweep = {}
    if not args.no_sweep and world == 1:
        for mm in (1, 8, 64, 512):
            s_ms, _, _, s_distinct = measure(mm, max(5, args.steps // 2), 3, graph=True)
            s_ms = max_over_ranks(s_ms)
            lb = s_distinct * (2 * I * q4_row + H * fmt.row_bytes(fmt.Q4_0, I)) + E * H * 4 + 2 * mm * H * 4
            sweep[str(mm)] = {"ms_per_step": s_ms, "tok_s": world * mm / (s_ms / 1e3),
                              "distinct_experts": s_distinct,
                              "layer_hbm_gbs": lb / (s_ms / 1e3) / 1e9}

    # ---- whole-model decode across the N GPUs (config 3 shapes, reduced) -------
    decode_ep = None
    if world > 1 and not args.no_decode and ep_decode_fits(world):
        uid2 = [hale.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid2, src=0)
        decode_ep = decode_ep_block(hale, fmt, ctx, world, rank, uid2[0], barrier, max_over_ranks)

    # ---- the host-driven NCCL exchange (hale_ep_* halves), for comparison -----
    ep_line = None
    if world > 1 and not args.no_ep:
        ep_line = measure_ep(hale, fmt, ctx, ld, encoded, router, world, rank, m, args, flush, barrier,
                             max_over_ranks)

    # ---- CPU baseline (rank 0, N=1 only) --------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, done, dt, cores = oracle_tok_s(ld, encoded, m, budget_s=10.0)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"{done} tokens of the same layer in {dt:.1f} s (batches of 8); "
                         f"oracle/hale_oracle.c -O2 -march=native, OpenMP {cores} threads, {cpu_model()}"}

    # ---- whole-model decode, BASELINE config 2 shapes (rank 0, N=1 only) ----
    decode = None
    if rank == 0 and world == 1 and not args.no_decode:
        decode = decode_block(hale, fmt, ctx, steps=16, warmup=3)

    if rank == 0:
        line = {
            "metric": "decode_tok_s_moe_layer", "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_0 weights x i8 activations, int32 block dots, f32 accumulate",
            "data": "synthetic", "config": config(m, world), "roofline": roofline,
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "kernels": kern,
            "ms_per_step_eager": ms_eager,
            "timing": ("device: CUDA events around CUDA-graph replays of hale_moe_forward" if world == 1 else
                       "device: CUDA events around each rank's hale_moe_forward_ep, max over ranks"),
            "clocks": clk, "sweep": sweep,
        }
        if decode is not None:
            line["decode"] = decode
        if decode_ep is not None:
            line["decode_ep"] = decode_ep
        if ep_p2p is not None:
            line["bit_exact_vs_1gpu"] = ep_p2p["bit_exact"]
            line["launches_per_call"] = ep_p2p["per_call_launches"]
            line["replicas"] = {"tok_s": world * m / (ms / 1e3), "ms_per_step": ms,
                                "note": "every GPU all experts and its own batch (no exchange); this rank's time"}
        if ep_line is not None:
            line["ep_host_nccl"] = ep_line
        emit(line)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def emit(line):
    """The one JSON line, on the process's original stdout."""
    os.write(_JSON_FD, (json.dumps(line) + "\n").encode())


_JSON_FD = 1

if __name__ == "__main__":
    # stdout carries exactly one JSON line: everything else written to fd 1
    # (library banners such as NCCL's version line, warnings) goes to stderr
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    main()

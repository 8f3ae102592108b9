"""Batch-one Qwen3 decode benchmark on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config qwen3-8b] [--context 4096]

Workload (N=1): the Qwen3-8B shape (seeded random-init bf16 weights, drawn on
the GPU), batch 1, decoding at a 4096-token context: the KV cache holds 4096
seeded random positions (the decode step's work does not depend on their
values), then K timed greedy steps each attend over 4096+i positions. One
step = the captured decode graph (embed -> 36 layers -> final norm -> LM head
-> argmax, position += 1). Weights (15.1 GB) are far larger than L2, so every
step streams them from HBM.

* value      device-timed tok/s (CUDA events around K graph replays), max over ranks
* e2e        the same K steps through the engine's state API with host buffers:
             per step a pinned host->device token copy, the replay, a
             device->host token copy and a stream sync (what generate() does)
* roofline   dominant kernel (gate/up + SwiGLU GEMV) timed live with CUDA
             events over all layers' weights, algorithmic bytes / duration
* step_roofline  whole-step algorithmic bytes (weights + KV) / step time
* cpu_baseline   the reference's eager path (Transformers Qwen3ForCausalLM,
             bf16, DynamicCache) decoding at the same shape on the host cores
* --impl reference  times only that CPU path (rank 0; other ranks exit 0)

* repeats    further windows of the same K steps: every window's tok/s,
             the median and the spread
* parity     correctness gate before timing (every N): the 0.6B golden
             prompts of the reference's eager path (tokens up to the
             golden file's first exact tie, top-64 logits within 0.0625),
             and at N > 1 one 8B-shaped layer tensor parallel vs one GPU;
             the run exits 3 after printing its line if the gate fails
* configs    the other BASELINE configurations (N = 1): 8B at 32k, 4B with
             a real 4096-token prefill + 256 steps, 0.6B with a 32-token
             prompt + 128 steps, the attention op sweep; and at every N the
             speculative line (8B target tensor parallel over the N GPUs,
             0.6B draft replica per rank, k = 4, synthetic p = 0.7 drafts,
             context 8192)

Multi-GPU (N>1, launched by torchrun): tensor parallelism over the N GPUs
(KV heads, FFN columns and vocabulary sharded; the o-proj and down partial
sums reduced over NVLink peer memory inside their GEMV epilogues). `value`
is the one sequence's tok/s (strong scaling); `step_roofline` uses the bytes
each GPU streams per step.
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

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tok/s and % of HBM roofline (1/2/4/8 B200) vs reference CPU"


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of this GPU's SM clock, power and throttle reasons
    every 50 ms. ``start`` returns once the first sample has arrived; ``mark``
    is called where the timed region begins and ``stop`` waits for one more
    sample after it ends, so the record is the samples that bracket the timed
    region (the last one before it, every one inside, the first one after),
    however short the region is."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 50

    def __init__(self, device_index: int):
        self.proc = None
        self.path = None
        self.first = 0
        try:
            props = torch.cuda.get_device_properties(device_index)
            ident = str(getattr(props, "uuid", ""))
            self.ident = ident if ident.startswith("GPU-") else (f"GPU-{ident}" if ident else str(device_index))
        except Exception:
            self.ident = str(device_index)

    def _rows(self):
        rows = []
        with open(self.path) as f:
            for line in f:
                if not line.endswith("\n"):
                    break  # a sample still being written
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 8:
                    rows.append(parts)
        return rows

    def _wait_rows(self, n: int, limit_s: float) -> int:
        deadline = time.monotonic() + limit_s
        while True:
            k = len(self._rows())
            if k >= n or time.monotonic() > deadline or self.proc.poll() is not None:
                return k
            time.sleep(0.01)

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="qb_clocks_", suffix=".csv")
            os.close(fd)
            self.fh = open(self.path, "w", buffering=1)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.ident, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.INTERVAL_MS)],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        self._wait_rows(1, 10.0)
        self.mark()

    def mark(self):
        """The timed region starts now: keep the newest sample and all later ones."""
        if self.proc is not None:
            self.first = max(len(self._rows()) - 1, 0)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        self._wait_rows(len(self._rows()) + 1, 2.0)  # one sample taken after the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        rows = self._rows()[self.first:]
        os.unlink(self.path)
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons if rows else ["unsampled"], "samples": len(rows),
                "interval_ms": self.INTERVAL_MS,
                "power_w_max": max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)}


# ------------------------------------------------------------------ CPU arm
def cpu_reference_decode(cfg, context: int, budget_s: float, max_steps: int = 64):
    """Time the reference's eager path (HF Qwen3ForCausalLM, bf16, SDPA,
    DynamicCache greedy loop) at this shape on the host cores: a KV cache of
    ``context`` random positions, then greedy steps until ``budget_s``."""
    from transformers import DynamicCache

    from oracle import hf_eager

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    t0 = time.perf_counter()
    model = hf_eager.build_hf_model(cfg, None)
    gen = torch.Generator().manual_seed(0)
    block = (torch.randn(1 << 20, generator=gen) * 0.02).to(torch.bfloat16)
    with torch.no_grad():
        for p in model.parameters():
            flat = p.data.view(-1)
            for s in range(0, flat.numel(), block.numel()):
                n = min(block.numel(), flat.numel() - s)
                flat[s:s + n].copy_(block[:n])
        for name, p in model.named_parameters():
            if "norm" in name:
                p.data.fill_(1.0)
    cache = DynamicCache()
    shape = (1, cfg.n_kv_heads, context, cfg.head_dim)
    for layer in range(cfg.n_layers):
        k = torch.randn(shape, generator=gen).to(torch.bfloat16)
        v = torch.randn(shape, generator=gen).to(torch.bfloat16)
        cache.update(k, v, layer)
    setup = time.perf_counter() - t0
    tok = torch.tensor([[1]])
    steps, times = 0, []
    with torch.inference_mode():
        t_start = time.perf_counter()
        while steps < max_steps:
            ts = time.perf_counter()
            res = model(input_ids=tok, past_key_values=cache, use_cache=True, logits_to_keep=1)
            cache = res.past_key_values
            tok = res.logits[:, -1:].float().argmax(-1)
            times.append(time.perf_counter() - ts)
            steps += 1
            if time.perf_counter() - t_start > budget_s and steps >= 2:
                break
    total = sum(times)
    return {"value": steps / total, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": (f"Transformers {__import__('transformers').__version__} Qwen3ForCausalLM eager bf16 "
                       f"(the reference's eager path, dryft/OPTIMIZATION_GUIDE.md:316-368), {cfg.name} shape, "
                       f"{steps} greedy DynamicCache steps at context {context}..{context + steps - 1}, "
                       f"median {1000 * statistics.median(times):.1f} ms/token; setup {setup:.0f}s untimed"),
            "median_ms_per_token": 1000 * statistics.median(times)}


# ------------------------------------------------------------------ GPU arm
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def profiled_traffic(name):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch from the
    committed ncu summary ``profiles/<name>.md`` (None if absent)."""
    try:
        with open(os.path.join(ROOT, "profiles", name + ".md")) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1])
    except OSError:
        pass
    return None


def time_dominant_kernel(engine, reps_per_layer=2):
    """Gate/up + SwiGLU GEMV (about half of a step's bytes) launched alone over
    every layer's weights in turn: the launches are captured once as a CUDA
    graph and the replay is timed with CUDA events on its stream, so the
    figure is device time, not Python launch rate. Returns (average seconds
    per launch, algorithmic bytes per launch)."""
    from hackthenorth_b200 import ops

    cfg = engine.cfg
    layers = engine.weights.layers
    x = torch.randn(cfg.hidden, device=engine.device).to(torch.bfloat16)
    for lw in layers[:3]:
        ops.norm_projection(x, lw["post_norm"], lw["gu"], cfg.rms_eps, swiglu=True)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n = 0
    with torch.cuda.graph(graph):
        for _ in range(reps_per_layer):
            for lw in layers:
                ops.norm_projection(x, lw["post_norm"], lw["gu"], cfg.rms_eps, swiglu=True)
                n += 1
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ops.check_device_errors(engine.device)
    sec = e0.elapsed_time(e1) / 1000.0 / n
    del graph
    gu = layers[0]["gu"]
    nbytes = gu.numel() * gu.element_size() + cfg.hidden * 2 * 2 + (gu.shape[0] // 2) * 2
    return sec, nbytes


def build_engine(cfg, world, dev, seed=0, cpu_weights=False):
    """This rank's engine: tensor parallel under torchrun, else one GPU.
    ``cpu_weights``: draw the weights with the CPU generator (the golden
    vectors' weights), else on the GPU."""
    from hackthenorth_b200.engine import Engine

    if world > 1:
        from hackthenorth_b200 import tp

        return tp.engine_from_random(cfg, seed=seed, init_device="cpu" if cpu_weights else None)
    return Engine.from_random(cfg, seed=seed, device=str(dev), init_device="cpu" if cpu_weights else str(dev))


def timed_steps(state, steps, first_token, ctx, world):
    """K graph replays from position ``ctx``, bracketed by a barrier and a
    synchronize on both sides, CUDA events on the replay stream; the slowest
    rank's seconds."""
    state.token.fill_(first_token)
    state.position.fill_(ctx)
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        state.step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    sec = e0.elapsed_time(e1) / 1000.0
    state.check()
    return max_over_ranks(sec, world)


def warm_state(state, warmup, first_token, ctx):
    state.token.fill_(first_token)
    state.position.fill_(ctx)
    if not state.captured:
        state.capture()
    for _ in range(warmup):
        state.step()
    state.check()


def prefill_decode_line(cfg, world, dev, ctx, n_decode, warmup, peak_gbs, note):
    """A configuration line: a real batched prefill of a seeded random prompt
    of ``ctx`` tokens (timed after one untimed prefill of the same prompt),
    then ``n_decode`` greedy decode steps from position ``ctx`` timed as one
    window (graph replays; warm-up steps first, whose K/V slots the timed
    steps overwrite)."""
    engine = build_engine(cfg, world, dev)
    st = engine.new_state(ctx, n_decode + 1, capacity=ctx + n_decode + warmup + 8)
    prompt = torch.randint(0, cfg.vocab, (ctx,), generator=torch.Generator().manual_seed(1)).to(dev)
    st.prefill(prompt)
    st.check()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    st.prefill(prompt)
    p1.record()
    torch.cuda.synchronize()
    st.check()
    prefill_ms = p0.elapsed_time(p1)
    first = st.read_token()[0]
    warm_state(st, warmup, first, ctx)
    sec = timed_steps(st, n_decode, first, ctx, world)
    mean_ctx = int(round(ctx + (n_decode - 1) / 2.0))
    step_bytes = cfg.step_bytes(mean_ctx) // world
    line = {"tok_s": round(n_decode / sec, 2), "ms_per_step": round(1000.0 * sec / n_decode, 4),
            "steps": n_decode, "prefill_tokens": ctx, "prefill_ms": round(prefill_ms, 3),
            "roofline": {"bytes_per_step": step_bytes, "achieved_GBps": round(step_bytes / (sec / n_decode) / 1e9, 1),
                         "peak": peak_gbs, "frac": round(step_bytes / (sec / n_decode) / 1e9 / peak_gbs, 4),
                         "roofline_tok_s": round(peak_gbs * 1e9 / step_bytes, 1)},
            "workload": note}
    import gc

    del st, engine
    gc.collect()  # engine and state refer to each other
    torch.cuda.empty_cache()
    return line


def seeded_kv(state, cfg, ctx, dev, seed=2):
    gen = torch.Generator(device=dev).manual_seed(seed)
    for t in (state.keys, state.values):
        for l in range(cfg.n_layers):
            t[l, ..., :ctx, :].normal_(generator=gen)  # [Hkv, cap, D] or [B, Hkv, cap, D]


GOLDEN_FILES = ("qwen3_0p6b_greedy.json", "qwen3_0p6b_greedy_notie.json")
LOGIT_ATOL = 0.0625


def gather_logits(t, world):
    """The full logit row from this rank's vocabulary shard (every rank)."""
    if world == 1:
        return t.float().cpu()
    import torch.distributed as dist

    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t.contiguous())
    return torch.cat(parts, dim=-1).float().cpu()


def parity_check(world, rank, dev):
    """Correctness gate run before timing (every N): the engine (tensor
    parallel over the N GPUs) against the committed golden vectors of the
    reference's eager path, and at N > 1 against this engine on one GPU.

    * 0.6B shape, CPU-drawn seed-0 weights, each golden prompt: the plain
      greedy stream equals the golden tokens up to the golden file's first
      exact top-1/top-2 tie (all 128 for the tie-free prompt), and every
      teacher-forced step's logits at the golden top-64 ids lie within
      LOGIT_ATOL of the native values.
    * N > 1: one Qwen3-8B-shaped layer (full vocabulary) over a seeded N(0, 1)
      cache at context 4096: the tensor-parallel step's logits (gathered from
      the vocabulary shards) against the same step on rank 0's GPU alone, max
      abs within LOGIT_ATOL, mean within 0.01, same greedy token unless the
      one-GPU logits hold a near tie.
    Returns (report, ok); every rank takes the same collective steps."""
    import dataclasses

    from hackthenorth_b200.config import QWEN3_0P6B, QWEN3_8B

    report = {"tolerance": {"logit_max_abs": LOGIT_ATOL, "tp_vs_one_gpu_mean_abs": 0.01}}
    ok = True
    threads = torch.get_num_threads()
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // world))
    engine = build_engine(QWEN3_0P6B, world, dev, seed=0, cpu_weights=True)
    torch.set_num_threads(threads)
    for name in GOLDEN_FILES:
        path = os.path.join(ROOT, "tests", "golden", name)
        if not os.path.exists(path):
            continue
        with open(path) as f:
            g = json.load(f)
        prompt, gold = g["prompt"], g["tokens"]
        st = engine.new_state(len(prompt), len(gold), keep_logits=True)
        st.prefill(torch.tensor(prompt, dtype=torch.int64, device=dev))
        rows = [gather_logits(st.logits, world)]
        for t in gold[:-1]:
            st.token.fill_(t)
            st.step()
            rows.append(gather_logits(st.logits, world))
        st.check()
        worst = 0.0
        for row, s in zip(rows, g["steps"]):
            ids = torch.tensor(s["top_ids"])
            worst = max(worst, float((row[ids] - torch.tensor(s["top_vals"])).abs().max()))
        free = [s[0] for s in engine.generate([prompt], len(gold), draft_tokens=0)]
        engine.state.check()
        upto = next((i for i, s in enumerate(g["steps"]) if s["margin"] == 0.0), len(gold))
        same = free[:upto] == gold[:upto]
        first_diff = next((i for i, (a, b) in enumerate(zip(free, gold)) if a != b), None)
        report[name] = {"tokens_required_equal": upto, "tokens_equal": same, "first_difference": first_diff,
                        "top64_logit_max_abs": round(worst, 5)}
        ok = ok and same and worst <= LOGIT_ATOL
        del st
    import gc

    del engine
    gc.collect()
    torch.cuda.empty_cache()
    if world > 1:
        from hackthenorth_b200.engine import Engine

        cfg1 = dataclasses.replace(QWEN3_8B, n_layers=1)
        ctx = 4096
        gen = torch.Generator(device=dev).manual_seed(4)
        kfull = torch.randn(1, cfg1.n_kv_heads, ctx, cfg1.head_dim, generator=gen, device=dev).to(torch.bfloat16)
        vfull = torch.randn(1, cfg1.n_kv_heads, ctx, cfg1.head_dim, generator=gen, device=dev).to(torch.bfloat16)
        hl = cfg1.n_kv_heads // world
        tpe = build_engine(cfg1, world, dev, seed=3)
        st = tpe.new_state(ctx, 4, keep_logits=True)
        st.keys[:, :, :ctx] = kfull[:, rank * hl:(rank + 1) * hl]
        st.values[:, :, :ctx] = vfull[:, rank * hl:(rank + 1) * hl]
        st.token.fill_(17)
        st.position.fill_(ctx)
        st.step()
        st.check()
        tp_logits = gather_logits(st.logits, world)
        tp_tok = st.read_token()[0]
        del st, tpe
        gc.collect()  # releases the TP graph (it holds NCCL calls) and the weights
        torch.cuda.empty_cache()
        flag = torch.ones(1, dtype=torch.int32, device=dev)
        if rank == 0:
            one = Engine.from_random(cfg1, seed=3, device=str(dev), init_device=str(dev))
            s1 = one.new_state(ctx, 4, keep_logits=True)
            s1.keys[:, :, :ctx] = kfull
            s1.values[:, :, :ctx] = vfull
            s1.token.fill_(17)
            s1.position.fill_(ctx)
            s1.step()
            s1.check()
            ref = s1.logits.float().cpu()
            one_tok = s1.read_token()[0]
            d = (tp_logits - ref).abs()
            top2 = ref.topk(2).values
            tok_ok = tp_tok == one_tok or float(top2[0] - top2[1]) <= LOGIT_ATOL
            good = float(d.max()) <= LOGIT_ATOL and float(d.mean()) <= 0.01 and tok_ok
            report["tp_vs_one_gpu"] = {"workload": f"qwen3-8b shape, 1 layer, context {ctx}, seeded N(0,1) K/V",
                                       "logit_max_abs": round(float(d.max()), 5),
                                       "logit_mean_abs": round(float(d.mean()), 6),
                                       "token_tp": tp_tok, "token_one_gpu": one_tok, "ok": good}
            flag.fill_(1 if good else 0)
            del s1, one
            gc.collect()
            torch.cuda.empty_cache()
        import torch.distributed as dist

        dist.broadcast(flag, src=0)
        ok = ok and bool(flag.item())
    report["ok"] = ok
    return report, ok


def run_ours(args):
    from hackthenorth_b200 import build as qbuild
    from hackthenorth_b200.config import get_config

    world, rank, local = dist_setup(args.gpus)
    qbuild.build()
    cfg = get_config(args.config)
    import dataclasses

    if args.layers:
        # Profiling only: fewer layers of the same shapes (keeps each kernel's
        # launch identical, and the device footprint small enough for ncu).
        cfg = dataclasses.replace(cfg, n_layers=args.layers)
    if args.shard_of > 1:
        # Profiling only: one rank's shapes under N-way tensor parallelism (its
        # query/KV heads, FFN columns and vocabulary rows) on one GPU without
        # the cross-rank exchange, so a 1-GPU profiler sees the per-rank kernels.
        n = args.shard_of
        if world > 1 or cfg.n_kv_heads % n or cfg.ffn % n or cfg.vocab % n:
            raise SystemExit("--shard-of N runs on one GPU and needs KV heads, FFN and vocabulary divisible by N")
        cfg = dataclasses.replace(cfg, name=f"{cfg.name}-tp{n}-rank", n_heads=cfg.n_heads // n,
                                  n_kv_heads=cfg.n_kv_heads // n, ffn=cfg.ffn // n, vocab=cfg.vocab // n)
    dev = torch.device(f"cuda:{local}")
    peak_gbs, peak_kind = load_peaks()
    B = args.batch
    if B > 1 and (world > 1 or args.real_prefill):
        raise SystemExit("--batch > 1 runs on one GPU over seeded K/V (no --real-prefill)")
    full = not args.layers and B == 1 and not args.real_prefill and args.shard_of <= 1

    parity, parity_ok = (None, True)
    if full and not args.no_parity:
        parity, parity_ok = parity_check(world, rank, dev)

    engine = build_engine(cfg, world, dev)
    torch.cuda.empty_cache()
    ctx = args.context
    total_steps = args.warmup + args.steps
    state = engine.new_state(ctx, total_steps + 2, capacity=ctx + 2 * total_steps + 8, batch=B)
    prefill_ms = None
    if args.real_prefill:
        # the configuration's random prompt (seed 1) prefilled as dense blocks
        # (tensor parallel under torchrun), timed with CUDA events after one
        # untimed prefill of the same prompt; the max over ranks
        prompt = torch.randint(0, cfg.vocab, (ctx,), generator=torch.Generator().manual_seed(1)).to(dev)
        state.prefill(prompt)
        state.check()
        torch.cuda.synchronize()
        barrier(world)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        state.prefill(prompt)
        p1.record()
        torch.cuda.synchronize()
        state.check()
        prefill_ms = max_over_ranks(p0.elapsed_time(p1), world)
        first_token = state.read_token()[0]
    else:
        seeded_kv(state, cfg, ctx, dev)
        first_token = 1
    warm_state(state, args.warmup, first_token, ctx)
    stream = torch.cuda.current_stream()

    # Clocks are sampled across the first window and the repeats (the same K
    # steps timed again in further windows; the line's value is the first
    # window, as the contract asks, and the spread shows how stable it is).
    clocks = ClockSampler(local)
    clocks.start()
    clocks.mark()
    t_dev = timed_steps(state, args.steps, first_token, ctx, world)
    windows = [t_dev] + [timed_steps(state, args.steps, first_token, ctx, world) for _ in range(args.repeats)]
    clk = clocks.stop()
    rates = [B * args.steps / t for t in windows]

    # e2e: the same steps with host buffers (pinned H2D of the token, replay,
    # D2H of the result, sync) — the per-token loop of generate().
    state.position.fill_(ctx)
    host_in = torch.tensor([first_token] * B, dtype=torch.int64).pin_memory()
    host_out = torch.empty(B, dtype=torch.int64).pin_memory()
    torch.cuda.synchronize()
    barrier(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for _ in range(args.steps):
        state.token.copy_(host_in, non_blocking=True)
        state.step()
        host_out.copy_(state.token, non_blocking=True)
        stream.synchronize()
        host_in.copy_(host_out)
    f1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_s = f0.elapsed_time(f1) / 1000.0
    state.check()

    kern_s, kern_bytes = time_dominant_kernel(engine)
    kern_s = max_over_ranks(kern_s, world)

    if args.trace and B == 1:
        # One more step with the kernels' own timestamps (after the timed
        # windows; the trace drops and re-captures the step graph).
        from hackthenorth_b200.trace import StepTrace

        tr = StepTrace(state)
        warm_state(state, 2, first_token, ctx)
        timed_steps(state, 1, first_token, ctx, world)
        summ = tr.summary()
        tr.close()
        path = args.trace if world == 1 else f"{args.trace}.rank{rank}"
        with open(path, "w") as f:
            json.dump({"config": cfg.name, "context": ctx, "n_gpus": world, "rank": rank, **summ}, f)

    # The public API end to end (one GPU, batch one): Engine.generate on the
    # configuration's seeded random prompt of `ctx` tokens; decode rate from
    # the first yielded token to the last (prefill excluded), host ints out.
    # Default generate speculates with prompt lookup (the reference's
    # default); draft_tokens=0 is plain decode with replays running ahead.
    gen_rates = {}
    if world == 1 and full:
        prompt = torch.randint(0, cfg.vocab, (ctx,), generator=torch.Generator().manual_seed(1)).tolist()
        n_gen = args.steps + 1
        for label, kw in (("default", {}), ("plain", {"draft_tokens": 0})):
            for _ in engine.generate([prompt], 4, **kw):  # warm-up: shape-keyed state, graph capture
                pass
            for _ in engine.generate([prompt], n_gen, **kw):
                pass
            t_first = None
            for i, _tok in enumerate(engine.generate([prompt], n_gen, **kw)):
                if i == 0:
                    t_first = time.perf_counter()
            gen_rates[label] = (n_gen - 1) / (time.perf_counter() - t_first)
            engine.state.check()

    t_e2e = max_over_ranks(e2e_s, world)
    ms_step = 1000.0 * t_dev / args.steps
    value = B * args.steps / t_dev  # B sequences; with N GPUs one sequence sharded across them
    mean_ctx = ctx + (args.steps - 1) / 2.0
    wbytes = cfg.weight_bytes_per_token()
    # weights once per step, K/V of every sequence; per GPU under tensor parallelism
    step_bytes = (wbytes + B * (cfg.step_bytes(int(round(mean_ctx))) - wbytes)) // world
    achieved = kern_bytes / kern_s / 1e9
    launches_per_step = (5 * cfg.n_layers + 1 + (1 if world > 1 else 0) if B == 1
                         else 6 * cfg.n_layers + 2)  # batched: + rope rows per layer, + position update
    out = {
        "metric": METRIC if B == 1 else f"batch-{B} decode tok/s (all sequences) and % of HBM roofline",
        "value": round(value, 3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": ("synthetic (seeded random-init weights N(0,0.02); context = a real prefill of a seeded "
                 "random prompt)" if prefill_ms is not None else
                 "synthetic (seeded random-init weights N(0,0.02); KV cache of seeded N(0,1) positions)"),
        "config": {"workload": f"{cfg.name}-shaped batch-{B} greedy decode at context {ctx}",
                   "model": cfg.name, "global_batch": B, "seq_len": ctx, "context": ctx,
                   "parallelism": "none" if world == 1 else (
                       f"tp{world} (NCCL all-reduce after o-proj and down)" if os.environ.get("QB_TP_NCCL") == "1"
                       else f"tp{world} (peer-memory reduction fused into the o-proj and down epilogues over NVLink)"),
                   "l2": "inputs larger than L2 (weights stream %.1f GB per step)" % (cfg.weight_bytes_per_token() / 1e9)},
        "repeats": {"windows": len(windows), "steps_each": args.steps,
                    "tok_s": [round(r, 2) for r in rates], "median_tok_s": round(statistics.median(rates), 2),
                    "spread_pct": round(100.0 * (max(rates) - min(rates)) / statistics.median(rates), 2)},
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel<EPI_SWIGLU> (post-norm + gate/up + SwiGLU)",
                     "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                     "frac": round(achieved / peak_gbs, 4), "peak_source": peak_kind,
                     "bytes_per_launch": kern_bytes, "us_per_launch": round(kern_s * 1e6, 2),
                     "timing": "CUDA events around a replayed graph of the kernel over every layer's weights",
                     "traffic": profiled_traffic("gemv_swiglu_qwen3-8b") if (cfg.name == "qwen3-8b" and world == 1) else None,
                     "traffic_source": "ncu capture, profiles/gemv_swiglu_qwen3-8b.md"},
        "step_roofline": {"bytes_per_step": step_bytes, "achieved": round(step_bytes / (t_dev / args.steps) / 1e9, 1),
                          "peak": peak_gbs, "unit": "GB/s",
                          "frac": round(step_bytes / (t_dev / args.steps) / 1e9 / peak_gbs, 4),
                          "roofline_tok_s": round(B * peak_gbs * 1e9 / step_bytes, 1)},
        "e2e": {"value": round(args.steps / t_e2e, 3), "unit": "tok/s",
                "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
                "d2h_bytes_per_step": host_out.numel() * host_out.element_size()},
        "e2e_generate": None if not gen_rates else {
            "value": round(gen_rates["default"], 3), "unit": "tok/s",
            "plain_value": round(gen_rates["plain"], 3),
            "how": "Engine.generate(prompt of the context length) yielding host token ids; first to last yield. "
                   "value: the default generate (prompt-lookup speculation, as the reference's); plain_value: "
                   "draft_tokens=0, replays %d ahead of the consumer through a pinned device-to-host token ring"
                   % engine.STREAM_DEPTH},
        "gpu_launches": launches_per_step * args.steps,
        "prefill_ms": None if prefill_ms is None else round(prefill_ms, 3),
        "profile_only": bool(args.layers) or args.shard_of > 1,
        "clocks": clk,
        "parity": parity,
    }
    if B > 1:
        # the dominant kernels of a batched step are the rows GEMVs: the step's
        # own bytes over its time are the roofline figure
        out["roofline"] = dict(out["step_roofline"], bound="hbm", kernel="whole batched step (rows kernels)",
                               traffic=None, peak_source=peak_kind)

    configs = {}
    if full and world == 1 and cfg.name == "qwen3-8b" and not args.no_configs:
        # BASELINE configurations beside the headline, each as its own line
        long_ctx = 32768
        del state
        torch.cuda.empty_cache()
        st = engine.new_state(long_ctx, total_steps + 2, capacity=long_ctx + 2 * total_steps + 8)
        seeded_kv(st, cfg, long_ctx, dev)
        warm_state(st, args.warmup, 1, long_ctx)
        sec = timed_steps(st, args.steps, 1, long_ctx, world)
        sb = cfg.step_bytes(int(round(long_ctx + (args.steps - 1) / 2.0)))
        configs["qwen3-8b@32k"] = {
            "tok_s": round(args.steps / sec, 2), "ms_per_step": round(1000.0 * sec / args.steps, 4),
            "steps": args.steps,
            "roofline": {"bytes_per_step": sb, "achieved_GBps": round(sb / (sec / args.steps) / 1e9, 1),
                         "peak": peak_gbs, "frac": round(sb / (sec / args.steps) / 1e9 / peak_gbs, 4),
                         "roofline_tok_s": round(peak_gbs * 1e9 / sb, 1)},
            "workload": "qwen3-8b shape, batch 1, KV cache of 32768 seeded N(0,1) positions, greedy decode"}
        del st
    import gc

    del engine
    state = engine = None
    gc.collect()  # engine and state refer to each other
    torch.cuda.empty_cache()
    if full and world == 1 and cfg.name == "qwen3-8b" and not args.no_configs:
        from hackthenorth_b200.config import QWEN3_0P6B, QWEN3_4B

        cs = ClockSampler(local)
        cs.start()
        configs["qwen3-4b"] = prefill_decode_line(
            QWEN3_4B, world, dev, 4096, 256, args.warmup, peak_gbs,
            "qwen3-4b shape, batched prefill of a seeded random 4096-token prompt, then 256 greedy decode steps "
            "(KV cache 4096 -> 4352)")
        configs["qwen3-0.6b"] = prefill_decode_line(
            QWEN3_0P6B, world, dev, 32, 128, args.warmup, peak_gbs,
            "qwen3-0.6b shape, 32-token seeded random prompt, then 128 greedy decode steps")
        configs["attention"] = {"cases": attention_cases(args.warmup, peak_gbs),
                                "workload": "decode attention op, GQA 32/8, D 128, bf16 N(0,1) Q/K/V, batch 1; "
                                            "us = device time per call from a replayed graph of the calls"}
        configs["clocks"] = cs.stop()
    if full and not args.no_spec:
        configs["speculative"] = speculative_line(args, world, rank, local)
    if configs:
        out["configs"] = configs
    if world == 1 and not args.no_cpu_baseline and B == 1:
        torch.cuda.empty_cache()
        out["cpu_baseline"] = cpu_reference_decode(cfg, ctx, budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import gc

        import torch.distributed as dist

        # The decode graph holds NCCL calls: release it (and the communicator)
        # before the process group goes away.
        state = engine = None
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    if not parity_ok:
        raise SystemExit(3)


def attention_cases(warmup, peak_gbs, only=None):
    """Decode-attention op sweep (GQA 32/8, D 128, bf16 N(0,1), batch 1):
    KV lengths 512..131072, 1 query row and the 5-row causal verify variant.
    Each timed launch reads a different KV buffer (>= 256 MB cycled), so the
    K/V bytes come from HBM. "us" is device time per call (the timed calls
    replayed as one CUDA graph); "us_host" the same calls issued one by one
    from Python. Returns the per-case list."""
    from hackthenorth_b200 import ops

    gen = torch.Generator(device="cuda").manual_seed(2)
    cases = []
    for L in (512, 4096, 32768, 131072):
        for queries in (1, 5):
            if only and (L, queries) not in only:
                continue
            per_call = 2 * 8 * L * 128 * 2
            nbuf = max(2, min(64, -(-(256 << 20) // per_call)))
            kv = [(torch.randn(8, L, 128, generator=gen, device="cuda").to(torch.bfloat16),
                   torch.randn(8, L, 128, generator=gen, device="cuda").to(torch.bfloat16)) for _ in range(nbuf)]
            q = torch.randn(queries, 32, 128, generator=gen, device="cuda").to(torch.bfloat16)
            pos = torch.arange(L - queries, L, device="cuda")
            for k, v in kv[:2]:
                ops.grouped_attention(q, k, v, pos)
            torch.cuda.synchronize()
            reps = max(warmup + 3, 40 if L <= 4096 else 10)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # host-driven: one op call per launch from Python (tensor maps encoded per call)
            e0.record()
            for i in range(reps):
                k, v = kv[i % nbuf]
                ops.grouped_attention(q, k, v, pos)
            e1.record()
            torch.cuda.synchronize()
            ops.check_device_errors()
            host_sec = e0.elapsed_time(e1) / 1000.0 / reps
            # device time: the same calls captured once as a CUDA graph and replayed
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for i in range(reps):
                    k, v = kv[i % nbuf]
                    ops.grouped_attention(q, k, v, pos)
            graph.replay()
            torch.cuda.synchronize()
            replays = 3
            e0.record()
            for _ in range(replays):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ops.check_device_errors()
            sec = e0.elapsed_time(e1) / 1000.0 / (replays * reps)
            del graph
            nbytes = per_call + 2 * q.numel() * 2 + queries * 8
            cases.append({"kv_len": L, "queries": queries, "us": round(sec * 1e6, 2),
                          "GBps": round(nbytes / sec / 1e9, 1), "frac": round(nbytes / sec / 1e9 / peak_gbs, 4),
                          "us_host": round(host_sec * 1e6, 2)})
            del kv
            torch.cuda.empty_cache()
    return cases


def run_attention_sweep(args):
    """The attention op sweep alone: one JSON line with a per-case list."""
    from hackthenorth_b200 import build as qbuild

    qbuild.build()
    torch.cuda.set_device(0)
    peak_gbs, peak_kind = load_peaks()
    only = None
    if args.att_cases:
        only = {tuple(int(x) for x in c.split(":")) for c in args.att_cases.split(",")}
    cases = attention_cases(args.warmup, peak_gbs, only)
    print(json.dumps({"op": "grouped_attention", "metric": "decode attention us and GB/s of K/V reads",
                      "peak_gbs": peak_gbs, "peak_source": peak_kind, "dtype": "bf16",
                      "config": {"q_heads": 32, "kv_heads": 8, "head_dim": 128}, "cases": cases}), flush=True)


def speculative_line(args, world, rank, local, ctx=8192):
    """Speculative decoding line (not the headline): the 8B target verifies
    k = 4 draft tokens per cycle (tensor parallel over the ranks under
    torchrun), the 0.6B draft model runs its k decode steps every cycle on each
    rank (a replica; timed, its tokens unused), and each draft token is the
    target's greedy token for the current prefix with seeded Bernoulli(0.7)
    probability, else uniform (expected 2.773 emitted per cycle). Every rank
    takes the same cycles; the line reports the slowest rank's time.

    The target's greedy continuation comes from its plain decode path. The
    verify pass sums in a different order, so at a near tie of the plain
    logits it may pick the other token; the emitted stream then leaves the
    precomputed continuation, and the harness recomputes the continuation from
    that point with plain decode steps (untimed), recording the plain top-2
    margin there. Only the draft + verify cycles are timed (CUDA events on the
    stream, plus the host read of each cycle's predictions)."""
    from hackthenorth_b200.config import QWEN3_0P6B, get_config
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.speculate import SyntheticDraft

    dev = torch.device(f"cuda:{local}")
    cfg = get_config(args.config)
    k, n_out = 4, 256
    if world > 1:
        from hackthenorth_b200 import tp

        target = tp.engine_from_random(cfg, seed=0)  # this rank's shard
    else:
        target = Engine.from_random(cfg, seed=0, device=str(dev), init_device=str(dev))
    draft = Engine.from_random(QWEN3_0P6B, seed=0, device=str(dev), init_device=str(dev))
    cap = ctx + 2 * n_out + 2 * k + 8
    ts = target.new_state(ctx, n_out + 1, draft_tokens=k, capacity=cap, keep_logits=True)
    ds = draft.new_state(ctx, n_out + 1, draft_tokens=k, capacity=cap)
    gen = torch.Generator(device=dev).manual_seed(2)
    for st, c in ((ts, cfg), (ds, QWEN3_0P6B)):
        for t in (st.keys, st.values):
            for l in range(c.n_layers):
                t[l, :, :ctx].normal_(generator=gen)
    first = 1
    ts.capture()
    ds.capture()

    def margin():
        """Top-2 margin of the last step's logits (over all vocabulary shards)."""
        top2 = ts.logits.float().topk(2).values
        if world > 1:
            import torch.distributed as dist

            parts = [torch.empty_like(top2) for _ in range(world)]
            dist.all_gather(parts, top2)
            top2 = torch.cat(parts).topk(2).values
        return float(top2[0] - top2[1])

    def plain_from(token, position, count):
        """Plain greedy continuation and each step's top-2 margin (untimed)."""
        ts.token.fill_(token)
        ts.position.fill_(position)
        toks, margins = [], []
        for _ in range(count):
            ts.step()
            toks += ts.read_token()
            margins.append(margin())
        return toks, margins

    # warm-up of both graphs and the plain timing
    plain_from(first, ctx, 3)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    plain, plain_margins = plain_from(first, ctx, n_out)
    plain_s = max_over_ranks(time.perf_counter() - t0, world)
    ts.check()

    split_ms = [0.0, 0.0]  # draft steps, verify (+ host read) per run

    def run_spec(timed):
        drafter = SyntheticDraft([], cfg.vocab, p=0.7, seed=3, draft_length=k)
        ref, margins = list(plain), list(plain_margins)
        out, cur, cycles, spent, anchors = [], first, 0, 0.0, []
        split_ms[0] = split_ms[1] = 0.0
        ts.token.fill_(first)
        ts.position.fill_(ctx)
        stream = torch.cuda.current_stream()
        while len(out) < n_out:
            drafter.reference = ref
            e0, em, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            ds.position.fill_(ctx + len(out))  # the draft model follows the accepted prefix
            for _ in range(k):
                ds.step()
            em.record(stream)
            proposal = drafter.propose(len(out), k)
            emitted = ts.verify(cur, proposal)
            e1.record(stream)
            e1.synchronize()
            spent += e0.elapsed_time(e1) / 1000.0
            split_ms[0] += e0.elapsed_time(em)
            split_ms[1] += em.elapsed_time(e1)
            cycles += 1
            base = len(out)
            out += emitted
            cur = emitted[-1]
            bad = next((j for j, tok in enumerate(emitted) if base + j >= len(ref) or ref[base + j] != tok), None)
            if bad is not None and len(out) < n_out:
                # re-anchor: the plain continuation after the emitted prefix (untimed)
                if base + bad < len(margins):
                    anchors.append(round(margins[base + bad], 4))
                pos = int(ts.position.item())
                tail, tail_m = plain_from(cur, pos, n_out - len(out) + k + 1)
                ref = out + tail
                margins = margins[:len(out)] + tail_m
                ts.token.fill_(cur)
                ts.position.fill_(pos)
        return out[:n_out], cycles, spent, anchors

    run_spec(False)  # warm-up (captures the verify graph)
    torch.cuda.synchronize()
    barrier(world)
    spec, cycles, spec_s, anchors = run_spec(True)
    ts.check()
    ds.check()
    spec_s = max_over_ranks(spec_s, world)
    split_ms[0] = max_over_ranks(split_ms[0], world)
    split_ms[1] = max_over_ranks(split_ms[1], world)
    reduction = ("NCCL all-reduce of fp32 partial rows" if os.environ.get("QB_TP_NCCL") == "1"
                 else "peer-memory reduction fused into the o-proj and down epilogues over NVLink")
    par = f"tp{world} target ({reduction}), draft replica per rank" if world > 1 else "none"
    line = {
        "metric": "speculative decode tok/s (target verify k=4 + 0.6B draft steps, synthetic p=0.7 drafts)",
        "value": round(n_out / spec_s, 3), "unit": "tok/s", "n_gpus": world, "higher_is_better": True,
        "mode": "speculative", "dtype": "bf16",
        "data": "synthetic (seeded random-init weights; KV prefix of seeded N(0,1) values; drafts = target "
                "greedy continuation with Bernoulli(0.7), else uniform, seed 3)",
        "config": {"workload": f"{cfg.name} target, qwen3-0.6b draft, context {ctx}, k={k}, {n_out} tokens",
                   "parallelism": par},
        "emitted_per_cycle": round(n_out / cycles, 3), "expected_emitted_per_cycle": 2.773, "cycles": cycles,
        "plain_tok_s": round(n_out / plain_s, 3), "speedup_vs_plain": round(plain_s / spec_s, 3),
        "draft_ms_per_cycle": round(split_ms[0] / cycles, 3), "verify_ms_per_cycle": round(split_ms[1] / cycles, 3),
        "reanchors": len(anchors), "reanchor_plain_top2_margins": anchors,
        "tokens_equal_plain_greedy": spec == plain,
        "timing": "sum of per-cycle CUDA-event times (draft steps + verify + the host read of its predictions), "
                  "max over ranks; re-anchoring after a near-tie disagreement is untimed",
    }
    # the verify and decode graphs hold NCCL calls under tensor parallelism:
    # release them before the caller tears the process group down
    import gc

    ts = ds = target = draft = None
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return line


def run_speculative(args):
    """The speculative line alone (target tensor parallel under torchrun)."""
    from hackthenorth_b200 import build as qbuild

    world, rank, local = dist_setup(args.gpus)
    qbuild.build()
    line = speculative_line(args, world, rank, local, ctx=args.context)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from hackthenorth_b200.config import get_config

    cfg = get_config(args.config)
    budget = max(10.0, min(120.0, 2.0 * args.steps))
    cb = cpu_reference_decode(cfg, args.context, budget_s=budget, max_steps=args.warmup + args.steps)
    out = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(cb["value"], 4),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(cb["median_ms_per_token"], 2),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"{cfg.name}-shaped batch-1 greedy decode at context {args.context}",
                   "model": cfg.name, "global_batch": 1, "seq_len": args.context, "context": args.context,
                   "parallelism": "none (host CPU)"},
        "cpu_baseline": cb,
        "e2e": {"value": round(cb["value"], 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--config", default="qwen3-8b")
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--repeats", type=int, default=4,
                    help="further timed windows of K steps after the first (median and spread reported)")
    ap.add_argument("--no-parity", action="store_true", help="skip the correctness gate run before timing")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the other BASELINE configurations (0.6B, 4B, 8B@32k, attention sweep)")
    ap.add_argument("--no-spec", action="store_true", help="skip the speculative-decoding configuration")
    ap.add_argument("--op", choices=("decode", "attention", "speculative"), default="decode",
                    help="attention: the decode-attention op sweep; speculative: verify + draft cycles "
                         "(neither is the headline line)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: override the layer count (the line is marked profile_only)")
    ap.add_argument("--att-cases", default="",
                    help="--op attention: only these KV_LEN:QUERIES cases, comma separated (e.g. 4096:5)")
    ap.add_argument("--trace", default="",
                    help="write a per-launch timeline of one decode step (the kernels' %%globaltimer stamps) "
                         "to this JSON path (per rank under torchrun: PATH.rankR)")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="profiling only: one rank's shapes under N-way tensor parallelism, on one GPU "
                         "without the exchange (the line is marked profile_only)")
    ap.add_argument("--real-prefill", action="store_true",
                    help="fill the context with a real prefill of a seeded random prompt (timed, reported as "
                         "prefill_ms) instead of seeded random K/V values")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences decoded together (1..8, one GPU; the line's value is their total tok/s)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.op == "attention":
        run_attention_sweep(args)
    elif args.op == "speculative":
        run_speculative(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

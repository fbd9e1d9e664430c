"""Benchmark: beam decode tokens/s on the Llama-3-8B shape (W=16), with the
paged-attention kernel's HBM roofline.

Workload: random-init Llama-3-8B-shaped model in bf16,
8 prompts x 1024 uniform-random token ids, beam width 16, 128 new tokens,
page size 16.  A "step" is one beam decode step over all 8 x 16 beams
(forward over 32 layers with cascade attention, log-softmax + top-2W,
global top-W per prompt, trie update, copy-on-write forks).  ``--warmup W``
decode steps run untimed after the prefill, then ``--steps K`` are timed with
CUDA events (barrier + synchronize on both sides); W + K <= 127 (the 128th
token comes from the prefill).  Every step streams the 15 GB of weights, far
more than L2, so no flush is needed between steps.

Multi-GPU (torchrun, one process per GPU): tensor parallel over the N GPUs
(default; the same 8 prompts, heads / MLP columns / vocabulary sharded, NCCL
all-reduces; strong scaling; value = the job's beam tokens / max-over-ranks
time), or ``--parallel replicas`` (every rank decodes its own 8 prompts, weak
scaling, no collective on the data path).  ``BENCH_WATCHDOG_S`` > 0 dumps
every thread's Python stack if a rank is still running after that many
seconds (diagnosis of a stuck collective).

``--impl reference`` times the CPU restatement of the reference engine (the
oracle; the reference's own GPU path needs FlashInfer 0.2.8, and its Python
tree cannot travel to the GPU box) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "beam decode tokens/s, Llama-3-8B-shape W=16; paged attn HBM GB/s vs peak"
# DRAM bytes per algorithmic byte of the attention launch, from one ncu capture of the
# beam-tile kernel on a cfg3 decode state (bench.py --op tiles3 --pool-pages 8192: dram
# read+write 45.31 MB for 52.63 MB of planned K/V + Q/O; pages listed at two cascade levels
# are read from L2 the second time); traffic scales with the tokens read
TRAFFIC_RATIO = (45.306112 + 0.00384) / 52.625408
TRAFFIC_SOURCE = ("scaled: ncu dram__bytes_read+write of attn_tile_kernel on a cfg3 decode state "
                  "(bench.py --op tiles3) x this launch's algorithmic bytes")
PROMPTS, PROMPT_LEN, BEAM, NEW_TOKENS, PAGE = 8, 1024, 16, 128, 16
MODEL_NAME, KERNEL = "LLAMA3_8B", "cascade"
WORKLOAD = ("cfg3: Llama-3-8B shape, 8 prompts x 1024 tokens, beam width 16, 128 new tokens, "
            "page size 16, cascade attention")
# the BASELINE configs the decode bench can run (--config); cfg3 is the default
CONFIGS = {
    "cfg3": dict(PROMPTS=8, PROMPT_LEN=1024, BEAM=16, NEW_TOKENS=128, MODEL_NAME="LLAMA3_8B",
                 KERNEL="cascade", WORKLOAD=WORKLOAD),
    "cfg4": dict(PROMPTS=1, PROMPT_LEN=4096, BEAM=32, NEW_TOKENS=256, MODEL_NAME="LLAMA3_8B",
                 KERNEL="auto",
                 WORKLOAD="cfg4: Llama-3-8B shape, 1 prompt x 4096 tokens, beam width 32, 256 new "
                          "tokens, page size 16, tree-vs-cascade picker (kernel_type auto); "
                          "random-init logits reparent most beams every step (churn reported)"),
    "cfg5": dict(PROMPTS=4, PROMPT_LEN=2048, BEAM=16, NEW_TOKENS=128, MODEL_NAME="LLAMA3_70B",
                 KERNEL="cascade",
                 WORKLOAD="cfg5: Llama-3-70B shape, 4 prompts x 2048 tokens, beam width 16, 128 "
                          "new tokens, page size 16, cascade attention"),
}


def use_config(name):
    globals().update(CONFIGS[name])


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            out = ""
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def write_kernel_trace(prof, path, rank, steps):
    """Per-kernel device time of the timed steps (CUPTI activity records via
    torch.profiler, graph-replayed kernels included), one table per rank.  A
    traced run is for the table only: its step time is not a bench value."""
    import collections
    tot = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if str(e.device_type).endswith("CUDA"):
            t = tot[e.name[:100]]
            t[0] += 1
            t[1] += e.device_time_total
    allt = sum(v[1] for v in tot.values()) or 1.0
    with open(f"{path}.rank{rank}.txt", "w") as f:
        f.write(f"timed steps {steps}; kernel time per step {allt / steps:.0f} us\n")
        f.write("us/step | launches/step | share | kernel\n")
        for name, (n, us) in sorted(tot.items(), key=lambda kv: -kv[1][1]):
            f.write(f"{us / steps:9.1f} | {n / steps:6.1f} | {100 * us / allt:5.1f}% | {name}\n")


def run_b200(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist

    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from beam_engine_b200 import configs as model_configs
    from beam_engine_b200.configs import param_count
    from beam_engine_b200.llama import BeamLlama

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = dict(getattr(model_configs, MODEL_NAME))
    tp_mode = world > 1 and args.parallel == "tp"
    tp = None
    if tp_mode:
        from beam_engine_b200.parallel import TensorParallel
        tp = TensorParallel()
    # tensor parallel: every rank builds the same full weights and keeps its shard;
    # replicas: independent models and prompts per rank
    seed = 1234 if tp_mode else 1234 + rank
    model = BeamLlama(cfg, None, dtype=torch.bfloat16, device=dev, seed=seed, tp=tp)
    if tp_mode and args.tp_comm == "peer":
        model.enable_peer_allreduce()   # fused peer-memory all-reduce + add + RMSNorm
    gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=PAGE,
                              max_num_pages=args.pages, kernel_type=KERNEL)
    g = torch.Generator().manual_seed(0 if tp_mode else rank)
    prompts = [torch.randint(0, cfg["vocab_size"], (PROMPT_LEN,), generator=g).tolist()
               for _ in range(PROMPTS)]
    W, K = args.warmup, args.steps
    total_steps = NEW_TOKENS - 1
    if W + K > total_steps:
        raise SystemExit(f"warmup + steps must be <= {total_steps}")
    ev = {}
    clocks = Clocks(local_rank)
    attn_events = []
    launches = {"n": 0}
    plan_bytes = []
    plan_stats = []
    plan_kind = set()
    plan_seq = []                      # kind of every timed step's plan, in order
    timing = {"on": False}
    gen.time_attention = True          # per-layer attention events recorded inside the step graph

    def plan_hook(nq, inf):
        if timing["on"]:
            # every planned token is read once per KV head: K and V, q in, o out
            plan_bytes.append(inf.total_tokens * 2 * model.Hkv * model.D * 2
                              + 2 * nq * model.Hq * model.D * 2)
            tiles = hasattr(inf, "n_pieces")
            if tiles:
                plan_stats.append((nq, inf.n_tiles, inf.n_pieces, inf.n_part_pieces,
                                   inf.n_entries))
            else:
                plan_stats.append((nq, inf.n_work, inf.n_work_wide, inf.n_parts, inf.n_merge))
            plan_kind.add("tiles" if tiles else "items")
            plan_seq.append("tiles" if tiles else "items")
            # per layer: 2 add_rmsnorm, rope_append, silu_mul + attention (one beam-tile
            # launch, or tcgen05 wide + all-heads narrow + LSE merge); final norm; fused
            # log-softmax / top-k; the copy-on-write fork list at the head of the step
            launches["n"] += cfg["num_hidden_layers"] * (4 + (1 if tiles else 3)) + 1 + 1 + 1

    gen.plan_hook = plan_hook
    orig_after = gen._after_update

    churn = []

    def after_hook(state):
        orig_after(state)
        if timing["on"]:   # share of new beams whose parent is shared with a sibling or gone
            cp = np.asarray(state.last_child_ptr)
            kids = int(cp[-1])
            if kids:
                churn.append(1.0 - int((np.diff(cp) > 0).sum()) / kids)

    gen._after_update = after_hook

    def on_step(i):
        if i == W:
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            clocks.start()
            if args.kernel_trace:
                from torch.profiler import ProfilerActivity, profile
                ev["prof"] = profile(activities=[ProfilerActivity.CUDA])
                ev["prof"].__enter__()
            ev["start"] = torch.cuda.Event(enable_timing=True)
            ev["start"].record()
            timing["on"] = True
            gen.attn_times = attn_events
        if i == W + K:
            ev["end"] = torch.cuda.Event(enable_timing=True)
            ev["end"].record()
            torch.cuda.synchronize()
            timing["on"] = False
            gen.attn_times = None
            if world > 1:
                dist.barrier()
            ev["clocks"] = clocks.stop()
            if args.kernel_trace:
                ev["prof"].__exit__(None, None, None)
                write_kernel_trace(ev["prof"], args.kernel_trace, rank, K)

    # -- timed decode run (inputs resident: model, pages) ------------------
    gen.generate_ids(prompts, BEAM, max_new_tokens=W + K + 1, on_step=on_step)
    ms = ev["start"].elapsed_time(ev["end"])
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    replicas = 1 if tp_mode else world         # independent beam searches in the job
    tokens = PROMPTS * BEAM * K * replicas
    value = tokens / (ms_max / 1e3)
    # attention roofline: algorithmic bytes / launch duration, live events
    attn_ms = list(attn_events)
    L = cfg["num_hidden_layers"]
    bytes_total = sum(b * L for b in plan_bytes)
    attn_total_ms = sum(attn_ms)
    hbm, tflops, src = peaks()
    achieved = bytes_total / (attn_total_ms / 1e3) / 1e9 if attn_total_ms else 0.0
    step_bytes = (param_count(cfg) - cfg["vocab_size"] * cfg["hidden_size"]) * 2
    if args.no_e2e:
        return dict(value=value, ms_per_step=ms_max / K, churn=float(np.mean(churn)) if churn else None,
                    captures_ms=[round(x * 1e3, 1) for x in gen.graph_captures],
                    regrowth=gen.graph_regrowth,
                    picks=({k: gen.picks.count(k) for k in set(gen.picks)} if gen.picks else None),
                    attn_us=attn_total_ms / max(len(attn_ms), 1) * 1e3,
                    achieved=achieved, plan_avg=[float(np.mean([p[i] for p in plan_stats])) for i in range(5)])
    # -- end-to-end: the public API call from host token ids to host beams ----
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    gen2_t0 = torch.cuda.Event(enable_timing=True)
    gen2_t1 = torch.cuda.Event(enable_timing=True)
    h2d0 = gen.h2d_bytes
    d2h0 = gen.d2h_bytes
    gen2_pre = torch.cuda.Event(enable_timing=True)

    def mark_prefill_done(i):   # decode step 0 starts: prefill + root expansion are queued
        if i == 0:
            gen2_pre.record()

    gen2_t0.record()
    t0 = time.perf_counter()
    out = gen.generate_ids(prompts, BEAM, max_new_tokens=NEW_TOKENS, on_step=mark_prefill_done)
    gen2_t1.record()
    torch.cuda.synchronize()
    e2e_ms = gen2_t0.elapsed_time(gen2_t1)
    prefill_ms = gen2_t0.elapsed_time(gen2_pre)
    wall_ms = (time.perf_counter() - t0) * 1e3
    t = torch.tensor([e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    e2e_tokens = PROMPTS * BEAM * NEW_TOKENS * replicas
    steps_e2e = NEW_TOKENS
    assert len(out) == PROMPTS and all(len(o) == 1 for o in out)
    res = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "beam tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_max / K, 4),
        "higher_is_better": True,
        "scaling": "strong" if tp_mode else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded uniform token ids, random-init N(0,0.02) weights)",
        "config": {"workload": WORKLOAD,
                   "model": f"{MODEL_NAME} shape (random init)", "global_batch": PROMPTS * BEAM * replicas,
                   "seq_len": PROMPT_LEN,
                   "parallelism": (f"tp{world}" + ("-peer" if args.tp_comm == "peer" else "")
                                   if tp_mode else (f"replicas x{world}" if world > 1 else "tp1")),
                   "l2": f"no flush needed: each step reads {step_bytes / 1e9:.1f} GB of weights "
                         "(> 126 MB L2)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4),
                     "traffic": round(TRAFFIC_RATIO * bytes_total / max(len(attn_ms), 1)),
                     "traffic_source": TRAFFIC_SOURCE,
                     "kernel": ("be_attn_tiles_run per layer (one beam-tile tcgen05 launch, "
                                "pieces merged on chip by clusters or by the merge kernel)"
                                if plan_kind == {"tiles"} else
                                "be_attn_run_fixed_2s per layer (tcgen05 prefix tiles, all-heads "
                                "suffix tiles on a second stream, LSE merge)")
                               + ", timed by event nodes inside the step graph",
                     "peak_source": src,
                     "avg_launch_us": round(attn_total_ms / max(len(attn_ms), 1) * 1e3, 2),
                     "bytes_per_launch": round(bytes_total / max(len(attn_ms), 1)),
                     "plan_avg": dict(zip(("queries", "tiles", "pieces", "partial_pieces",
                                           "entries") if plan_kind == {"tiles"} else
                                          ("queries", "work_items", "wide_items", "partial_rows",
                                           "merged_queries"),
                                          [round(float(np.mean([p[i] for p in plan_stats])), 1)
                                           for i in range(5)])) if plan_stats else None},
        "step_roofline": {"bytes_per_step": step_bytes, "achieved_gbs":
                          round(step_bytes / (ms_max / K / 1e3) / 1e9, 1),
                          "frac": round(step_bytes / (ms_max / K / 1e3) / 1e9 / hbm, 4)},
        "e2e": {"value": round(e2e_tokens / (e2e_ms / 1e3), 2), "unit": "beam tokens/s",
                "h2d_bytes_per_step": int((gen.h2d_bytes - h2d0) / steps_e2e),
                "d2h_bytes_per_step": int((gen.d2h_bytes - d2h0) / steps_e2e),
                "includes": f"prefill of {PROMPTS} x {PROMPT_LEN} prompt tokens + {NEW_TOKENS - 1} "
                            "decode steps, host ids in, host beams out", "wall_ms": round(wall_ms, 1),
                "prefill_ms": round(prefill_ms, 2)},
        "sequence_tokens_per_s": round(value / BEAM, 2),
        "gpu_launches": launches["n"],
        "graph_captures": [round(x * 1e3, 1) for x in gen.graph_captures],   # ms, whole run
        "churn": round(float(np.mean(churn)), 3) if churn else None,
        "kernel_picks": ({k: gen.picks.count(k) for k in set(gen.picks)} if gen.picks else None),
        "clocks": ev.get("clocks"),
    }
    if len(plan_kind) > 1:
        # mixed steps (kernel_type auto): the beam-tile and the work-item kernels separately
        # (each graph step records one plan, then one attention event pair per layer)
        by = {} if len(attn_ms) == len(plan_seq) * L else None
        for kind in sorted(plan_kind) if by is not None else []:
            idx = [i for i, k_ in enumerate(plan_seq) if k_ == kind]
            ms = sum(sum(attn_ms[i * L:(i + 1) * L]) for i in idx)
            b = sum(plan_bytes[i] * L for i in idx)
            a = b / (ms / 1e3) / 1e9 if ms else 0.0
            by[kind] = {"steps": len(idx), "avg_launch_us": round(ms / max(len(idx) * L, 1) * 1e3, 2),
                        "achieved": round(a, 1), "frac": round(a / hbm, 4)}
        res["roofline"]["by_kind"] = by
        res["roofline"]["kernel"] = ("mixed: be_attn_tiles_run (beam-tile kernel) on exact cascade "
                                     "steps, the work-item kernels on tree steps (see by_kind); "
                                     "timed by event nodes inside the step graph")
        res["roofline"]["plan_avg"] = None
    return res


class CpuDecodeSample:
    """The oracle (CPU restatement of the reference engine) on one cfg3 decode
    step's state: 128 beams, cascade over 8 x 1024-token prefixes plus 1-4 page
    suffixes, one decoder layer's weights (every layer of the 8B shape has the
    same shape and cost) and the lm_head.  ``layer()`` runs one decoder layer
    over all beams (RMSNorm, q/k/v, cascade attention, o_proj, SwiGLU MLP);
    ``head()`` the final log-softmax + top-2W.  A full step is 32 layers + head."""

    def __init__(self, threads=None):
        import numpy as np
        import torch
        from beam_engine_b200.configs import LLAMA3_8B
        self.threads = threads or os.cpu_count()
        torch.set_num_threads(self.threads)
        cfg = LLAMA3_8B
        rng = np.random.default_rng(0)
        H, F, D, Hq, Hkv, V = (cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"],
                               cfg["num_attention_heads"], cfg["num_key_value_heads"],
                               cfg["vocab_size"])
        self.L, self.D, self.Hq = cfg["num_hidden_layers"], D, Hq
        N = self.N = PROMPTS * BEAM
        P = PROMPTS * 64 + N * 4 + 8
        self.pool = rng.standard_normal((P, 2, PAGE, Hkv, D), dtype=np.float32)
        lv0 = dict(qo_indptr=[i * BEAM for i in range(PROMPTS + 1)],
                   kv_indptr=[i * 64 for i in range(PROMPTS + 1)],
                   kv_indices=list(range(PROMPTS * 64)), kv_last_page_len=[PAGE] * PROMPTS)
        kvp, kvi, last, nxt = [0], [], [], PROMPTS * 64
        for b in range(N):
            n = 1 + b % 4
            kvi += list(range(nxt, nxt + n))
            nxt += n
            kvp.append(len(kvi))
            last.append(1 + b % PAGE)
        lv1 = dict(qo_indptr=list(range(N + 1)), kv_indptr=kvp, kv_indices=kvi,
                   kv_last_page_len=last)
        self.levels = [lv0, lv1]

        def w(*sh):
            return rng.standard_normal(sh, dtype=np.float32) * np.float32(0.02)
        self.wq, self.wk, self.wv, self.wo = w(Hq * D, H), w(Hkv * D, H), w(Hkv * D, H), w(H, Hq * D)
        self.wg, self.wu, self.wd = w(F, H), w(F, H), w(H, F)
        self.lm = w(V, H)
        self.x = rng.standard_normal((N, H), dtype=np.float32)
        self.ones = np.ones(H, np.float32)
        self.h = self.x

    def layer(self):
        import numpy as np
        from oracle.attention import cascade_attention
        from oracle.llama import rmsnorm, silu
        N, D, Hq = self.N, self.D, self.Hq
        x = self.x
        h = rmsnorm(x, self.ones, 1e-5)
        q = (h @ self.wq.T).reshape(N, Hq, D)
        _k = h @ self.wk.T
        _v = h @ self.wv.T
        a = cascade_attention(q, self.pool, self.levels, PAGE, D ** -0.5).astype(np.float32)
        x2 = x + a.reshape(N, -1) @ self.wo.T
        h = rmsnorm(x2, self.ones, 1e-5)
        m = silu(h @ self.wg.T) * (h @ self.wu.T)
        self.h = h
        return x2 + m.astype(np.float32) @ self.wd.T

    def head(self):
        import numpy as np
        logits = self.h @ self.lm.T
        lp = logits - logits.max(-1, keepdims=True)
        lp = lp - np.log(np.exp(lp).sum(-1, keepdims=True))
        return np.argpartition(-lp, 2 * BEAM, axis=-1)[:, :2 * BEAM]

    def timed(self, fn, n):
        out = []
        for _ in range(n):
            t0 = time.perf_counter()
            fn()
            out.append(time.perf_counter() - t0)
        return out


SAMPLE_TEXT = ("one decoder layer of a cfg3 decode step per sample (128 beams: q/k/v, cascade over "
               "8 x 1024-token prefixes + 1-4 page suffixes, o_proj, SwiGLU MLP), numpy oracle fp32; "
               "a full step = 32 layers + lm_head/log-softmax/top-2W (timed once)")


def cpu_baseline_sample(threads=None, layers_timed=2):
    """cpu_baseline of the decode bench line: ``layers_timed`` decoder layers
    and one head of the oracle, one full step extrapolated from them."""
    smp = CpuDecodeSample(threads)
    smp.layer()                                   # warm-up (page faults, BLAS threads)
    lay = smp.timed(smp.layer, layers_timed)
    head = smp.timed(smp.head, 1)[0]
    step_s = statistics.mean(lay) * smp.L + head
    return {"value": round(smp.N / step_s, 3), "unit": "beam tokens/s", "cores": smp.threads,
            "kind": "port",
            "sample": f"{layers_timed} timed layers + 1 head; " + SAMPLE_TEXT,
            "step_s": round(step_s, 3)}


def run_reference(args, rank, world):
    """--impl reference: the CPU restatement of the reference engine, every
    warm-up and timed step one bounded sample (one decoder layer over the full
    cfg3 decode state).  ms_per_step is the measured time of one sample; value
    is the beam-token throughput of a full step built from the measured layer
    and head times (32 layers + head), reported with that full-step time."""
    if rank != 0:
        return None
    smp = CpuDecodeSample()
    head = smp.timed(smp.head, 1)[0]
    smp.timed(smp.layer, max(args.warmup, 0))
    lay = smp.timed(smp.layer, max(args.steps, 1))
    layer_s = statistics.mean(lay)
    step_s = layer_s * smp.L + head
    value = smp.N / step_s
    base = {"value": round(value, 3), "unit": "beam tokens/s", "cores": smp.threads, "kind": "port",
            "sample": f"{len(lay)} timed samples after {args.warmup} warm-up; " + SAMPLE_TEXT}
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "beam tokens/s", "n_gpus": world,
        "steps": len(lay), "warmup": args.warmup, "ms_per_step": round(layer_s * 1e3, 2),
        "step_is": "one bounded sample (one decoder layer over all 128 beams)",
        "full_step_ms": round(step_s * 1e3, 1), "head_ms": round(head * 1e3, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD,
                   "model": f"{MODEL_NAME} shape (random init)", "global_batch": PROMPTS * BEAM,
                   "seq_len": PROMPT_LEN, "parallelism": "cpu"},
        "cpu_baseline": base,
        "e2e": {"value": round(value, 3), "unit": "beam tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_op_bench(args):
    """cfg2: op-level cascade attention, append and fork
    microbench, bf16, Hq 32 / Hkv 8 / D 128 / page 16; shared prefix 2048
    tokens, W = 16 suffixes of U[1, 256] tokens, page ids a seeded permutation
    of the pool.  Each timed iteration is preceded by a 256 MB L2 flush;
    durations are CUDA events on the launching stream (median of --iters)."""
    import numpy as np
    import torch
    from beam_engine_b200 import _lib
    from beam_engine_b200.cascade import MultiLevelCascadeAttentionWrapper
    from beam_engine_b200.page_table import PageTable
    dev = torch.device("cuda", 0)
    Hq, Hkv, D, ps, W, prefix = 32, 8, 128, 16, 16, 2048
    P = args.pool_pages
    g = torch.Generator().manual_seed(0)
    perm = torch.randperm(P, generator=g)
    suf = torch.randint(1, 257, (W,), generator=g).tolist()
    npre = prefix // ps
    off = npre
    kvp, kvi, last = [0], [], []
    for L in suf:
        n = -(-L // ps)
        kvi += perm[off:off + n].tolist()
        off += n
        kvp.append(len(kvi))
        last.append(L - (n - 1) * ps)
    levels = [dict(qo_indptr=[0, W], kv_indptr=[0, npre], kv_indices=perm[:npre].tolist(),
                   kv_last_page_len=[ps]),
              dict(qo_indptr=list(range(W + 1)), kv_indptr=kvp, kv_indices=kvi, kv_last_page_len=last)]
    layers = args.op_layers
    pt = PageTable(1, ps, P, Hkv, D, device=dev, store_dtype=torch.bfloat16)
    pt.kv_cache.normal_(generator=torch.Generator(device=dev).manual_seed(1))
    P2 = min(P, 4096)        # all-layer pool for the fused append / fork launches
    ptL = PageTable(layers, ps, P2, Hkv, D, device=dev, store_dtype=torch.bfloat16)
    q = torch.randn((W, Hq, D), device=dev).to(torch.bfloat16)
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=dev)
    w = MultiLevelCascadeAttentionWrapper(2, ws)
    t = lambda a: torch.tensor(np.asarray(a, np.int32))  # noqa: E731
    w.plan([t(x["qo_indptr"]) for x in levels], [t(x["kv_indptr"]) for x in levels],
           [t(x["kv_indices"]) for x in levels], [t(x["kv_last_page_len"]) for x in levels],
           Hq, Hkv, D, ps, causal=True, sm_scale=D ** -0.5, split_tokens=args.split)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    hbm, _, src = peaks()

    def timeit(fn, iters):
        """Differential timing: (flush + op) x iters minus flush x iters, both
        enqueued behind a GPU sleep so host launch gaps are not timed."""
        for _ in range(3):
            fn()

        def run(with_op):
            torch.cuda.synchronize()
            torch.cuda._sleep(2_000_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iters):
                flush.zero_()
                if with_op:
                    fn()
            e.record()
            torch.cuda.synchronize()
            return s.elapsed_time(e)
        base = min(run(False) for _ in range(3))
        tot = min(run(True) for _ in range(3))
        return max(tot - base, 0.0) / iters * 1e3
    out = torch.empty_like(q)
    attn_us = timeit(lambda: w.run(q, pt.kv_cache_at_layer[0], out=out), args.iters)
    kv_tokens = prefix + sum(suf)
    attn_bytes = kv_tokens * 2 * Hkv * D * 2 + 2 * W * Hq * D * 2
    pre_bytes = prefix * 2 * Hkv * D * 2
    # append: one token per beam at (tail page, L % 16), one layer and all layers
    pages = torch.tensor([kvi[kvp[b + 1] - 1] for b in range(W)], dtype=torch.int32, device=dev)
    pos = torch.tensor([L % ps for L in suf], dtype=torch.int32, device=dev)
    kk = torch.randn((layers, W, Hkv, D), device=dev).to(torch.bfloat16)
    vv = torch.randn((layers, W, Hkv, D), device=dev).to(torch.bfloat16)
    ar = torch.arange(W + 1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    pagesL = pages % P2

    def app(nl):
        tab, pg, npg = (pt, pages, P) if nl == 1 else (ptL, pagesL, P2)
        _lib.check(L.be_append_paged_kv(kk.data_ptr(), vv.data_ptr(), Hkv * D, W * Hkv * D,
                                        ar.data_ptr(), pos.data_ptr(), pg.data_ptr(),
                                        ar.data_ptr(), W, tab.kv_cache.data_ptr(),
                                        tab.kv_cache.stride(0), nl, npg, ps, Hkv, D, _lib.BE_BF16,
                                        None))
    app1_us = timeit(lambda: app(1), args.iters)
    appL_us = timeit(lambda: app(layers), args.iters)
    app_bytes = W * 2 * Hkv * D * 2 * 2          # read + write, K and V
    # fork: beams remapped by a random parent vector; a parent with c children
    # copies its partial tail page c - 1 times
    parent = torch.randint(0, W, (W,), generator=g).tolist()
    src_p, dst_p, lens = [], [], []
    fresh = iter(perm[off:].tolist())
    for p_ in sorted(set(parent)):
        c = parent.count(p_)
        tail = suf[p_] - (-(-suf[p_] // ps) - 1) * ps
        if tail < ps:
            for _ in range(c - 1):
                src_p.append(kvi[kvp[p_ + 1] - 1])
                dst_p.append(next(fresh))
                lens.append(tail)
    sd = torch.tensor(src_p or [0], dtype=torch.int32, device=dev)
    dd = torch.tensor(dst_p or [0], dtype=torch.int32, device=dev)
    ld = torch.tensor(lens or [0], dtype=torch.int32, device=dev)
    sdL, ddL = sd % P2, (dd % P2 + P2 // 2) % P2

    def fork(nl):
        tab, a, b, npg = (pt, sd, dd, P) if nl == 1 else (ptL, sdL, ddL, P2)
        _lib.check(L.be_fork_tail_copy(tab.kv_cache.data_ptr(), tab.kv_cache.stride(0), nl, npg, ps,
                                       Hkv, D, _lib.BE_BF16, a.data_ptr(), b.data_ptr(),
                                       ld.data_ptr(), len(src_p), None))
    fork1_us = timeit(lambda: fork(1), args.iters) if src_p else 0.0
    forkL_us = timeit(lambda: fork(layers), args.iters) if src_p else 0.0
    fork_bytes = sum(lens) * Hkv * D * 2 * 2 * 2   # K+V, read + write
    # bandwidth sweep (all layers, one launch): append of SWEEP_TOK tokens to distinct
    # (page, slot) positions, and SWEEP_COPIES copy-on-write tail copies
    SWEEP_TOK = min(8192, P2 * ps // 2)
    sw_i = torch.arange(SWEEP_TOK, dtype=torch.int32, device=dev)
    sw_pages = (sw_i // ps).contiguous()
    sw_pos = (sw_i % ps).contiguous()
    sw_ind = torch.arange(SWEEP_TOK + 1, dtype=torch.int32, device=dev)
    sw_k = torch.randn((layers, SWEEP_TOK, Hkv, D), device=dev).to(torch.bfloat16)
    sw_v = torch.randn((layers, SWEEP_TOK, Hkv, D), device=dev).to(torch.bfloat16)
    # batch b = token i with its own one-page table entry: kv_indices[kv_indptr[i] + pos // ps]
    # = page, so kv_indices is the per-token page list and kv_indptr[i] = i - pos // ps
    sw_indptr = (sw_i - sw_pos // ps).contiguous()

    def app_sweep():
        _lib.check(L.be_append_paged_kv(sw_k.data_ptr(), sw_v.data_ptr(), Hkv * D,
                                        SWEEP_TOK * Hkv * D, sw_i.data_ptr(), sw_pos.data_ptr(),
                                        sw_pages.data_ptr(), sw_indptr.data_ptr(), SWEEP_TOK,
                                        ptL.kv_cache.data_ptr(), ptL.kv_cache.stride(0), layers,
                                        P2, ps, Hkv, D, _lib.BE_BF16, None))
    appS_us = timeit(app_sweep, max(3, args.iters // 4))
    appS_bytes = SWEEP_TOK * 2 * Hkv * D * 2 * 2 * layers
    n_cp = min(65535 // (2 * layers), P2 // 2)
    sw_src = torch.randperm(P2 // 2, generator=g)[:n_cp].to(torch.int32).to(dev)
    sw_dst = (torch.randperm(P2 // 2, generator=g)[:n_cp] + P2 // 2).to(torch.int32).to(dev)
    sw_len = torch.randint(1, ps, (n_cp,), generator=g).to(torch.int32).to(dev)

    def fork_sweep():
        _lib.check(L.be_fork_tail_copy(ptL.kv_cache.data_ptr(), ptL.kv_cache.stride(0), layers, P2,
                                       ps, Hkv, D, _lib.BE_BF16, sw_src.data_ptr(),
                                       sw_dst.data_ptr(), sw_len.data_ptr(), n_cp, None))
    forkS_us = timeit(fork_sweep, max(3, args.iters // 4))
    forkS_bytes = int(sw_len.sum().item()) * Hkv * D * 2 * 2 * 2 * layers
    inf = w._plan.tinfo if w.tiles else w._plan.info
    plan_desc = (dict(kind="tiles", tiles=inf.n_tiles, pieces=inf.n_pieces,
                      entries=inf.n_entries, rows=inf.tile_rows) if w.tiles else
                 dict(kind="items", work=inf.n_work, wide=inf.n_work_wide, parts=inf.n_parts))

    def rl(b, us):
        a = b / (us / 1e6) / 1e9 if us else 0.0
        return {"us": round(us, 2), "bytes": b, "gbs": round(a, 1), "frac": round(a / hbm, 4)}
    return {
        "config": {"workload": "cfg2 op microbench", "pool_pages": P, "layers_for_multi": layers,
                   "prefix": prefix, "beams": W, "suffix_tokens": suf, "l2": "256 MB flush per iter"},
        "peak_gbs": hbm, "peak_source": src,
        "cascade_attention": dict(rl(attn_bytes, attn_us), prefix_bytes=pre_bytes, plan=plan_desc),
        "append_1layer": rl(app_bytes, app1_us),
        f"append_{layers}layers_1launch": rl(app_bytes * layers, appL_us),
        "fork_1layer": dict(rl(fork_bytes, fork1_us), copies=len(src_p)),
        f"fork_{layers}layers_1launch": rl(fork_bytes * layers, forkL_us),
        "append_sweep": dict(rl(appS_bytes, appS_us), tokens=SWEEP_TOK, layers=layers),
        "fork_sweep": dict(rl(forkS_bytes, forkS_us), copies=n_cp, layers=layers),
    }


def run_op_picker(args):
    """--op picker: fits the tree-vs-cascade picker's work-item cost model
    (picker.fit_work_item_model) to cascade runs on the work-item kernels over
    a sweep of cfg2-like states: one shared prefix of P tokens and W beams with
    suffixes of U[1, S] tokens, Hq 32 / Hkv 8 / D 128, page size 16, bf16, page
    ids a seeded permutation of the pool.  Each run is preceded by a 256 MB L2
    flush; times are CUDA events (differential against the flush alone)."""
    import numpy as np
    import torch
    from beam_engine_b200.cascade import MultiLevelCascadeAttentionWrapper
    from beam_engine_b200.page_table import PageTable
    from beam_engine_b200.picker import PickerModel, fit_work_item_model
    dev = torch.device("cuda", 0)
    Hq, Hkv, D, ps = 32, 8, 128, 16
    P = min(args.pool_pages, 16384)
    pt = PageTable(1, ps, P, Hkv, D, device=dev, store_dtype=torch.bfloat16)
    pt.kv_cache.normal_(generator=torch.Generator(device=dev).manual_seed(1))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ws = torch.empty(128 << 20, dtype=torch.uint8, device=dev)
    hbm, _, src = peaks()
    t = lambda a: torch.tensor(np.asarray(a, np.int32))  # noqa: E731

    def timeit(fn, iters):
        for _ in range(3):
            fn()

        def run(with_op):
            torch.cuda.synchronize()
            torch.cuda._sleep(2_000_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iters):
                flush.zero_()
                if with_op:
                    fn()
            e.record()
            torch.cuda.synchronize()
            return s.elapsed_time(e)
        base = min(run(False) for _ in range(3))
        return max(min(run(True) for _ in range(3)) - base, 0.0) / iters * 1e3

    samples = []
    g = torch.Generator().manual_seed(0)
    for prefix in (256, 1024, 2048, 4096):
        for W in (4, 16, 32, 64):
            for smax in (16, 256):
                perm = torch.randperm(P, generator=g).tolist()
                suf = torch.randint(1, smax + 1, (W,), generator=g).tolist()
                npre = prefix // ps
                off, kvp, kvi, last = npre, [0], [], []
                for L in suf:
                    n = -(-L // ps)
                    kvi += perm[off:off + n]
                    off += n
                    kvp.append(len(kvi))
                    last.append(L - (n - 1) * ps)
                lv = [([0, W], [0, npre], perm[:npre], [ps]), (list(range(W + 1)), kvp, kvi, last)]
                w = MultiLevelCascadeAttentionWrapper(2, ws)
                w.plan([t(x[0]) for x in lv], [t(x[1]) for x in lv], [t(x[2]) for x in lv],
                       [t(x[3]) for x in lv], Hq, Hkv, D, ps, causal=True, sm_scale=D ** -0.5)
                w._plan_items()                   # the work-item kernels the model describes
                q = torch.randn((W, Hq, D), device=dev).to(torch.bfloat16)
                out = torch.empty_like(q)
                us = timeit(lambda: w.run(q, pt.kv_cache_at_layer[0], out=out), args.iters)
                inf = w._plan.info
                samples.append(dict(prefix=prefix, beams=W, suffix_max=smax, us=round(us, 2),
                                    n_work=inf.n_work, n_work_wide=inf.n_work_wide,
                                    n_parts=inf.n_parts, total_tokens=inf.total_tokens,
                                    hkv=Hkv, hq=Hq, d=D, elt=2))
    base = PickerModel(num_sms=torch.cuda.get_device_properties(dev).multi_processor_count,
                       hbm_gbs=hbm)
    fit = fit_work_item_model(samples, base)
    err = [abs(fit.cascade_us(_Counts(s), Hkv, Hq, D) - s["us"]) / s["us"] for s in samples]
    return {"op": "picker", "peak_gbs": hbm, "peak_source": src, "samples": samples,
            "fit": {k: round(getattr(fit, k), 3) for k in
                    ("num_sms", "hbm_gbs", "t_launch_us", "t_wide_cta_us", "t_narrow_cta_us")},
            "rel_err_median": round(float(np.median(err)), 4),
            "rel_err_max": round(float(np.max(err)), 4)}


class _Counts:
    """A work-item plan's counts from one picker sample (what cascade_us reads)."""

    def __init__(self, s):
        self.n_work, self.n_work_wide = s["n_work"], s["n_work_wide"]
        self.n_parts, self.total_tokens = s["n_parts"], s["total_tokens"]


def run_op_tiles(args):
    """Decode attention of one layer at a cfg3 decode state, on the beam-tile
    kernel: 8 prompts x 1024 tokens, 16 beams each, after `--op-steps` random
    selection steps (half the beams of a prompt fork, half die), Hq 32 / Hkv 8 /
    D 128, page size 16, bf16, one layer's pool of `--pool-pages` pages; 256 MB
    L2 flush before every timed launch, CUDA events, median of --iters."""
    import numpy as np
    import torch
    from beam_engine_b200 import _lib
    from beam_engine_b200.beam_state import BeamState
    from beam_engine_b200.cascade import target_pieces, tile_plan_host
    from beam_engine_b200.page_table import PageTable, dtype_code
    dev = torch.device("cuda", 0)
    # --op-tp N: one rank's share of the heads under N-way tensor parallelism
    Hq, Hkv, D, ps = 32 // args.op_tp, 8 // args.op_tp, 128, 16
    pt = PageTable(1, ps, args.pool_pages, Hkv, D, device=dev, store_dtype=torch.bfloat16)
    rng = np.random.default_rng(0)
    bs = BeamState(BEAM, pt)
    for _ in range(PROMPTS):
        bs.add_root_sequence(rng.integers(0, 1000, PROMPT_LEN).tolist())
    bs.update_native(bs.leaves, np.arange(PROMPTS + 1, dtype=np.int32) * BEAM,
                     rng.integers(0, 1000, PROMPTS * BEAM).astype(np.int32),
                     -rng.random(PROMPTS * BEAM))
    for _ in range(args.op_steps):
        n = len(bs.leaves)
        cnt = np.zeros(n, np.int32)
        for p_ in range(PROMPTS):
            c = np.zeros(BEAM, np.int32)
            c[: BEAM // 2] = 2
            rng.shuffle(c)
            cnt[p_ * BEAM:(p_ + 1) * BEAM] = c
        ptr = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        bs.update_native(bs.leaves, ptr, rng.integers(0, 1000, int(ptr[-1])).astype(np.int32),
                         -rng.random(int(ptr[-1])))
    pt.kv_cache.normal_(generator=torch.Generator(device=dev).manual_seed(1))
    levels = bs.cascade_levels()
    n = len(bs.leaves)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    info, plan = tile_plan_host(levels, n, ps, Hq, Hkv, num_sms=sms, cluster=args.cluster,
                                pieces=args.op_pieces or target_pieces(sms, Hkv))
    plan_d = torch.from_numpy(np.ascontiguousarray(plan)).to(dev)
    slots = max(1, info.n_part_pieces) * Hkv * info.tile_rows
    po = torch.empty(slots * D, dtype=torch.bfloat16, device=dev)
    pl = torch.empty(slots, dtype=torch.float32, device=dev)
    q = torch.randn((n, Hq, D), device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    pool = pt.kv_cache_at_layer[0]
    L = _lib.lib()

    def run():
        _lib.check(L.be_attn_tiles_run(plan_d.data_ptr(), info.n_pieces, info.n_tiles,
                                       info.n_part_pieces, info.tile_rows, ps, q.data_ptr(),
                                       q.stride(0), pool.data_ptr(), pool.shape[0], Hq, Hkv, D,
                                       dtype_code(pool.dtype), D ** -0.5, out.data_ptr(),
                                       out.stride(0), None, po.data_ptr(), pl.data_ptr(),
                                       info.cluster, 0, None))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        run()
    ts = []
    for _ in range(args.iters):
        flush.zero_()
        s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_.record()
        run()
        e_.record()
        torch.cuda.synchronize()
        ts.append(s_.elapsed_time(e_) * 1e3)
    us = statistics.median(ts)
    byts = info.total_tokens * 2 * Hkv * D * 2 + 2 * n * Hq * D * 2
    hbm, _, src = peaks()
    return {"config": {"workload": "cfg3 decode attention, one layer", "beams": n,
                       "heads": [Hq, Hkv],
                       "selection_steps": args.op_steps, "l2": "256 MB flush per iter"},
            "plan": {"tiles": info.n_tiles, "pieces": info.n_pieces, "entries": info.n_entries,
                     "tile_rows": info.tile_rows, "cluster": info.cluster},
            "us": round(us, 2), "bytes": byts, "gbs": round(byts / us / 1e3, 1),
            "frac": round(byts / us / 1e3 / hbm, 4), "peak_gbs": hbm, "peak_source": src}


def run_op_allreduce(args, rank, world, local_rank):
    """--op allreduce (under torchrun): one decode-step reduction, 128 rows x 4096
    bf16 (1 MiB), as the fused peer all-reduce + add + RMSNorm and as NCCL's
    all_reduce, `--iters` calls back to back, eagerly and replayed from a CUDA
    graph; device time per call by CUDA events, max over ranks."""
    import torch
    import torch.distributed as dist
    from beam_engine_b200._lib import check, lib
    from beam_engine_b200.page_table import stream_ptr
    from beam_engine_b200.parallel import PeerAllReduce, TensorParallel
    dev = torch.device("cuda", local_rank)
    tp = TensorParallel()
    n, H = 128, 4096
    comm = PeerAllReduce(tp, n * H * 2, dev)
    x = torch.randn(n, H, device=dev).bfloat16()
    w = torch.ones(H, device=dev).bfloat16()
    h = torch.empty_like(x)
    for slot in (0, 1):
        comm.slot_view(slot, (n, H), torch.bfloat16).normal_()
    t = torch.randn(n, H, device=dev).bfloat16()

    def peer(k):
        for i in range(k):
            check(lib().be_comm_allreduce_rmsnorm(comm.ptr, i & 1, x.data_ptr(), w.data_ptr(),
                                                  h.data_ptr(), n, H, 1e-6, 2, stream_ptr(dev)),
                  "allreduce")

    def nccl(k):
        for _ in range(k):
            dist.all_reduce(t)

    def timed(f, graph):
        k = args.iters
        torch.cuda.synchronize()
        dist.barrier()
        if graph:
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                f(4)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                f(k)
            run = g.replay
        else:
            def run():
                f(k)
        run()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        us = torch.tensor([e0.elapsed_time(e1) * 1e3 / k], device=dev)
        dist.all_reduce(us, op=dist.ReduceOp.MAX)
        return round(float(us.item()), 2)

    res = {"op": "allreduce", "rows": n, "hidden": H, "bytes": n * H * 2, "n_gpus": world,
           "calls": args.iters, "us_per_call": {}}
    for name, f in (("peer", peer), ("nccl", nccl)):
        for graph in (False, True):
            res["us_per_call"][name + ("_graph" if graph else "")] = timed(f, graph)
    torch.cuda.synchronize()
    dist.barrier()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--pages", type=int, default=4096)
    ap.add_argument("--config", default="cfg3", choices=sorted(CONFIGS),
                    help="decode workload (BASELINE configs); the driver's line is cfg3")
    ap.add_argument("--parallel", default="tp", choices=["tp", "replicas"],
                    help="N > 1: tensor parallel over the N GPUs (default) or N independent replicas")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp-comm", default="peer", choices=["nccl", "peer"],
                    help="tensor-parallel all-reduce: NCCL, or the fused peer-memory kernel")
    ap.add_argument("--op", default=None, choices=["cfg2", "tiles3", "allreduce", "picker"],
                    help="op-level microbench instead of the decode benchmark")
    ap.add_argument("--pool-pages", type=int, default=65536)
    ap.add_argument("--op-steps", type=int, default=60,
                    help="--op tiles3: random selection steps before the timed launches")
    ap.add_argument("--cluster", type=int, default=-1,
                    help="--op tiles3: cluster size (-1: the planner's choice, 0: merge kernel)")
    ap.add_argument("--op-layers", type=int, default=32)
    ap.add_argument("--op-pieces", type=int, default=0,
                    help="--op tiles3: pieces per KV head (0: the planner's target)")
    ap.add_argument("--op-tp", type=int, default=1, choices=[1, 2, 4, 8],
                    help="--op tiles3: heads of one rank under this tensor parallelism")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--split", type=int, default=0)
    ap.add_argument("--kernel-trace", default=None, metavar="PATH",
                    help="write per-kernel device time of the timed steps to PATH.rank<r>.txt "
                         "(torch.profiler; the traced run's numbers are not bench values)")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end pass and print a short line (for profiling)")
    args = ap.parse_args()
    use_config(args.config)
    wd = float(os.environ.get("BENCH_WATCHDOG_S", "0") or 0)
    if wd > 0:
        import faulthandler
        faulthandler.dump_traceback_later(wd, repeat=True, exit=False)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.op == "allreduce":
        import datetime
        import torch
        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=180))
        res = run_op_allreduce(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(res), flush=True)
        sys.stdout.flush()
        os._exit(0)
    if args.op:
        fn = {"tiles3": run_op_tiles, "picker": run_op_picker}.get(args.op, run_op_bench)
        print(json.dumps(fn(args)), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if rank == 0:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        # NVLS off: multicast objects outlive a failed rank on this kind of box
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(local_rank)
        # a short process-group timeout turns a stuck collective into an error
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank),
                                timeout=datetime.timedelta(seconds=180))
    res = run_b200(args, rank, world, local_rank)
    if rank == 0:
        if not args.no_cpu_baseline and not args.no_e2e and world == 1 and args.config == "cfg3":
            res["cpu_baseline"] = cpu_baseline_sample()
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        # destroy_process_group() can block on communicators that captured CUDA
        # graphs still reference; the process is done, so leave without it
        os._exit(0)


if __name__ == "__main__":
    main()

"""Benchmark: Qwen3-8B-shaped W4A16 MTP verify step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload per GPU (independent replicas, weak scaling): 32 sequences with 8192-token
synthetic prompts, MTP depth k=2 -> 96 verify rows per step, page size 16,
random-init Qwen3-8B-shaped weights (hidden 4096, 36 layers, 32 Q / 8 KV heads,
head_dim 128, SwiGLU 12288, vocab 151936), W4A16 group-128 for every linear incl.
the tied LM head.  The prompts' K/V pages are filled with seeded random values
(prefill is not part of the verify path); drafts are seeded random token ids.

A step = one verify pass: embedding, 36 decoder layers over the 96 rows (fused
QKV / O / gate-up / down W4 linears, QK-norm + RoPE + KV append, paged attention
over ~8.2K keys per sequence), final norm, LM head, row argmax, greedy accept and
rollback.  `value` times K such steps on device-resident inputs with CUDA events
(max over ranks); `e2e` times K steps of the public engine call
MTPVerifyEngine.verify_step with host drafts in, host accept results out.
Random drafts are almost never accepted by a random model, so `e2e_accepting` times
the same call with drafts the model accepts: its own greedy continuation, computed
untimed beforehand.

--impl reference times the reference's own CPU kernels (oracle/_ref/libecpu.so,
built from the reference sources) on a bounded sample of the same workload on the
host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "verified tok/s/GPU, Qwen3-8B W4A16 MTP verify; quant-GEMM HBM GB/s vs peak"
SEQS, PROMPT, K_DRAFT, PAGE = 32, 8192, 2, 16
GEN_HEADROOM = 512
# the committed ncu summary of one attn_pages launch whose DRAM traffic the bench line scales
ATTN_PROFILE = ROOT / "profiles" / "attn_pages_qwen3_8b_16seq_8k.md"


def attn_traffic_capture() -> dict | None:
    """DRAM read + write bytes of the attn_pages launch in ATTN_PROFILE (dram__bytes_read.sum +
    dram__bytes_write.sum, as written there) and the K/V bytes of that launch (its title
    line's "<seqs> seqs x <keys> keys", 8 KV heads x 128 bf16, K and V)."""
    import re
    try:
        text = ATTN_PROFILE.read_text()
    except OSError:
        return None
    unit = {"KB": 1e3, "MB": 1e6, "GB": 1e9}
    got = {}
    for name in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
        m = re.search(re.escape(name) + r"\s+([0-9.]+)\s+(KB|MB|GB)", text)
        if not m:
            return None
        got[name] = float(m.group(1)) * unit[m.group(2)]
    m = re.search(r"(\d+) seqs x (\d+) keys", text)
    if not m:
        return None
    kv = int(m.group(1)) * int(m.group(2)) * 8 * 128 * 2 * 2
    return {"bytes": got["dram__bytes_read.sum"] + got["dram__bytes_write.sum"], "kv_bytes": kv,
            "source": f"{ATTN_PROFILE.relative_to(ROOT)} ({m.group(1)} seqs x {m.group(2)} keys), "
                      "scaled to this launch by its K/V bytes"}


def bench_config(layers: int, world: int, seqs: int = SEQS, prompt: int = PROMPT) -> dict:
    """The workload both arms report (BASELINE configs[3] unless a reduced case is asked for)."""
    full = (seqs, prompt, layers) == (32, 8192, 36)
    return {
        "workload": ("Qwen3-8B-shaped W4A16 g128 MTP verify step (BASELINE configs[3])" if full else
                     f"reduced profiling case: {layers} layers, {seqs} seqs x {prompt} tokens"),
        "seqs_per_gpu": seqs, "prompt_len": prompt, "layers": layers, "draft_k": K_DRAFT,
        "rows_per_step": seqs * (K_DRAFT + 1),
        "page_size": PAGE, "parallelism": f"replicas x{world}",
        "l2": "inputs larger than L2 (about 40 GB KV + 4 GB weights read per step)",
    }


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons, every 20 ms, from the start of
    the first timed region to the end of the last (the device step, e2e and cycle legs)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
            return
        # nvidia-smi takes a moment to start; the timed region begins once it is sampling
        t0 = time.perf_counter()
        while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 5.0:
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
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
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------

def reduce_over_ranks(maxes: list[float], sums: list[float], device=None) -> tuple[list[float], list[float]]:
    """Job-level figures of a replicated run: every rank's times reduced by MAX (the job
    lasts as long as its slowest replica) and its counts by SUM.  Every rank makes the
    same two collective calls; a single process returns its inputs unchanged."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(maxes), list(sums)
    t_max = torch.tensor(list(maxes) or [0.0], dtype=torch.float64, device=device)
    t_sum = torch.tensor(list(sums) or [0.0], dtype=torch.float64, device=device)
    dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    dist.all_reduce(t_sum, op=dist.ReduceOp.SUM)
    return t_max.tolist()[:len(maxes)], t_sum.tolist()[:len(sums)]


def greedy_rollout(eng, n_tokens: int, k: int):
    """Drafts that the model accepts: run n_tokens steps without drafts (each appends the
    model's greedy next token), record every running sequence's continuation, then rewind
    each sequence to where it started.  Its pages stay allocated; the next steps rewrite
    the same positions.  Returns a function that gives, for the engine's current state,
    each sequence's next k tokens of that continuation (fewer near its end)."""
    run = list(eng.sched.running)
    base = {s.seq_id: (len(s.tokens), len(s.outputs), s.num_computed) for s in run}
    for _ in range(n_tokens):
        eng.verify_step({})
    traj = {s.seq_id: list(s.tokens[base[s.seq_id][0] - 1:]) for s in run}  # [pending, t1, t2, ...]
    for s in run:
        nt, no, nc = base[s.seq_id]
        del s.tokens[nt:]
        del s.outputs[no:]
        s.num_computed = nc

    def drafts() -> dict[int, list[int]]:
        out = {}
        for s in run:
            j = len(s.tokens) - base[s.seq_id][0]  # index of the pending token in traj
            out[s.seq_id] = traj[s.seq_id][j + 1:j + 1 + k]
        return out

    return drafts


def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    from pilm_b200 import bindings
    from pilm_b200.engine import MTPVerifyEngine
    from pilm_b200.qwen3 import QWEN3_8B, PagedKVCache, Qwen3Verifier, Qwen3Weights, attention_bytes

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    bindings.init()
    shape = QWEN3_8B
    if args.layers:  # reduced-depth case for profiling captures
        from dataclasses import replace
        shape = replace(shape, layers=args.layers)
    SEQS, PROMPT = args.seqs, args.prompt
    seed = 1234 + rank
    weights = Qwen3Weights.synthetic(shape, seed, dev)
    pages_per_seq = (PROMPT + GEN_HEADROOM + PAGE - 1) // PAGE
    num_blocks = SEQS * pages_per_seq + 1
    kv = PagedKVCache(shape, num_blocks, dev, fill="random", seed=seed)
    max_rows = SEQS * (K_DRAFT + 1)
    ver = Qwen3Verifier(weights, kv, max_rows=max_rows, max_pos=PROMPT + GEN_HEADROOM + 64, device=dev)
    eng = MTPVerifyEngine(ver, num_blocks=num_blocks, max_model_len=PROMPT + GEN_HEADROOM + 64)
    g = torch.Generator().manual_seed(seed)
    for _ in range(SEQS):
        sid = eng.add_request(torch.randint(0, shape.vocab, (PROMPT,), generator=g).tolist(),
                              max_new_tokens=GEN_HEADROOM)
        eng.admit_prefilled(sid)
    # state after prefill: the first generated token is pending (verify row 0) at
    # position 8192, the first slot of a fresh page, so k=2 drafts fit (engine.py:399-401)
    for s in eng.sched.running:
        t = int(torch.randint(0, shape.vocab, (1,), generator=g))
        s.tokens.append(t)
        s.outputs.append(t)

    def drafts_for_step():
        return {s.seq_id: torch.randint(0, shape.vocab, (K_DRAFT,), generator=g).tolist() for s in eng.sched.running}

    # ---- device-resident verify step (value) -------------------------------------
    from pilm_b200.qwen3 import VerifyGraph
    seqs = list(eng.sched.running)
    d0 = drafts_for_step()
    for s in seqs:
        s.tokens.extend(d0[s.seq_id])
        eng.pages.allocate(s, 1 + K_DRAFT, eng.max_pages)
    starts = [s.num_computed for s in seqs]
    batch = eng.build_batch(seqs, starts, [1 + K_DRAFT] * len(seqs))
    stream = torch.cuda.current_stream()
    graph = VerifyGraph(ver, len(seqs), batch.total_q, batch.max_q_len, eng.max_pages, eng.max_model_len)
    graph.load(batch)
    graph.capture()

    def step():
        graph.replay()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    if world > 1:
        dist.barrier()
    sampler.start()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    rows_per_step = batch.total_q
    (ms_max,), _ = reduce_over_ranks([ms], [], dev)
    # per-kernel timings for the rooflines (CUDA events, same stream, back-to-back launches)
    timeline = graph_timeline(graph) if args.timeline else None
    op_ms = {"attention": ver.time_attention(graph.batch)}
    op_ms["attention_total"] = op_ms["attention"] * shape.layers
    op_ms.update(ver.time_linears(rows_per_step))

    # ---- end to end through the engine API (e2e) -----------------------------------
    for s in seqs:  # undo the resident step's draft rows
        del s.tokens[s.num_computed + 1:]
    h2d = 0
    e2e_steps = 0 if args.no_e2e else args.steps
    # at least one page of warm-up steps, so every verify-row count the page-boundary cap
    # produces (k+1 rows per sequence down to 1) has its graph captured before timing
    for _ in range(max(args.warmup, PAGE) if e2e_steps else 0):
        eng.verify_step(drafts_for_step())
    # the drafts a caller hands in are ready before its call: generate them up front
    step_drafts = [drafts_for_step() for _ in range(e2e_steps)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_rows = 0
    t0 = time.perf_counter()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for d in step_drafts:
        rows_before = eng.stats["verified_rows"]
        eng.verify_step(d)
        e2e_rows += eng.stats["verified_rows"] - rows_before
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end) / max(1, e2e_steps)
    wall_ms = (time.perf_counter() - t0) * 1e3 / max(1, e2e_steps)
    (e2e_ms_max,), (e2e_rows_all,) = reduce_over_ranks([e2e_ms], [float(e2e_rows)], dev)
    maxp = max(len(s.pages) for s in eng.sched.running)

    def run_cycle(linears: str) -> dict:
        from pilm_b200.mtp import MTPDrafter, MTPWeights
        mw = MTPWeights.synthetic(shape, seed + 17, dev, linears=linears)
        eng.drafter, eng.draft_k, eng.graphs, eng.pending = MTPDrafter(mw, weights, SEQS, dev), K_DRAFT, {}, {}
        for _ in range(max(args.warmup, PAGE)):
            eng.verify_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        c_tokens = c_att = c_acc = 0
        c_rows = 0
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(e2e_steps):
            rows_before = eng.stats["verified_rows"]
            for r in eng.verify_step():
                c_tokens += 1 + r.accepted
                c_att += len(r.drafts)
                c_acc += r.accepted
            c_rows += eng.stats["verified_rows"] - rows_before
        c1.record(stream)
        torch.cuda.synchronize()
        (c_ms,), (c_rows_all, c_tokens_all) = reduce_over_ranks([c0.elapsed_time(c1) / e2e_steps],
                                                                [float(c_rows), float(c_tokens)], dev)
        eng.graphs = {}
        return {
            "verified_tok_s": round(c_rows_all / e2e_steps / (c_ms * 1e-3), 2),
            "accepted_tok_s": round(c_tokens_all / e2e_steps / (c_ms * 1e-3), 2),
            "ms_per_cycle": round(c_ms, 4),
            "draft_k": K_DRAFT,
            "draft_linears": linears,
            "draft_linear_bytes": mw.linear_bytes,
            "accept_rate": round(c_acc / max(1, c_att), 4),
            "call": "pilm_b200.engine.MTPVerifyEngine.verify_step() with the GPU MTP drafter "
                    "(verify + k draft steps in one captured step; host accept results and drafts out)",
        }

    # ---- the speculative cycle: verify + k MTP draft steps on the GPU (cycle) --------
    # The engine drafts each sequence's next tokens with the GPU drafter inside the same
    # captured step; verify_step() then verifies them.  Synthetic weights: the random
    # drafter rarely agrees with the random model, so accepted tok/s sits near the
    # 1-token-per-step floor; the timing is what a real checkpoint's cycle costs.  Both
    # draft-module options: the W4A16 one (cycle) and the reference's default bf16 one.
    cycle = cycle_bf16 = None
    if e2e_steps and not args.no_draft:
        cycle = run_cycle("w4a16")
        cycle_bf16 = run_cycle("bf16")

    def run_accepting() -> dict:
        """The verify step with drafts that the model accepts: the drafts are the target
        model's own greedy continuation, computed beforehand (untimed) by steps without
        drafts, after which every sequence is rewound to where it started (its pages are
        kept: the timed steps rewrite the same positions with the same K/V).  The timed
        steps then run the accept, bonus-token and context-advance path with k accepted
        drafts per sequence wherever the page-boundary cap allows k."""
        eng.drafter, eng.draft_k, eng.graphs, eng.pending = None, 0, {}, {}
        n_warm = max(args.warmup, PAGE)
        ideal_drafts = greedy_rollout(eng, (n_warm + e2e_steps) * (K_DRAFT + 1) + 2, K_DRAFT)
        eng.graphs = {}

        for _ in range(n_warm):
            eng.verify_step(ideal_drafts())
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a_rows = a_tokens = a_att = a_acc = 0
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(e2e_steps):
            d = ideal_drafts()
            rows_before = eng.stats["verified_rows"]
            for r in eng.verify_step(d):
                a_tokens += 1 + r.accepted
                a_att += len(r.drafts)
                a_acc += r.accepted
            a_rows += eng.stats["verified_rows"] - rows_before
        a1.record(stream)
        torch.cuda.synchronize()
        (a_ms,), (a_rows_all, a_tokens_all) = reduce_over_ranks([a0.elapsed_time(a1) / e2e_steps],
                                                                [float(a_rows), float(a_tokens)], dev)
        eng.graphs = {}
        return {
            "verified_tok_s": round(a_rows_all / e2e_steps / (a_ms * 1e-3), 2),
            "accepted_tok_s": round(a_tokens_all / e2e_steps / (a_ms * 1e-3), 2),
            "ms_per_step": round(a_ms, 4),
            "draft_k": K_DRAFT,
            "accept_rate": round(a_acc / max(1, a_att), 4),
            "drafts": "the target model's own greedy continuation (computed untimed beforehand)",
            "call": "pilm_b200.engine.MTPVerifyEngine.verify_step (host drafts -> host accept results)",
        }

    accepting = run_accepting() if e2e_steps and not args.no_accepting else None
    clocks = sampler.stop()
    # each rank's own timings on stderr (the JSON line carries the max over ranks)
    print(json.dumps({"rank": rank, "world": world, "ms_per_step": round(ms, 4),
                      "e2e_ms_per_step": round(e2e_ms, 4) if e2e_steps else None,
                      "e2e_host_wall_ms_per_step": round(wall_ms, 4) if e2e_steps else None}),
          file=sys.stderr, flush=True)
    h2d = 4 * (3 * rows_per_step + SEQS * maxp + 2 * SEQS + 1) + 0
    d2h = 4 * 2 * SEQS

    if rank != 0:
        return None

    # ---- roofline of the dominant kernel (paged attention) -------------------------
    pk = peaks()
    ctx = batch.context_lens.tolist()
    att_bytes = attention_bytes(shape, ctx, [1 + K_DRAFT] * SEQS)
    att_ms = op_ms.get("attention")
    att_gbs = att_bytes / (att_ms * 1e-3) / 1e9 if att_ms else None
    lin_bytes = weights.linear_bytes
    lin_ms = op_ms.get("linear_total")
    lin_gbs = lin_bytes / (lin_ms * 1e-3) / 1e9 if lin_ms else None
    step_bytes = att_bytes * shape.layers + lin_bytes + 2 * rows_per_step * shape.hidden * 2
    # DRAM traffic of one attn_pages launch: the committed ncu capture of the same kernel on
    # a 16-sequence case, scaled by this launch's K/V bytes, with which the kernel's traffic
    # grows (it reads each K/V byte once)
    kv_bytes = sum(ctx) * shape.n_kv_heads * shape.head_dim * 2 * 2
    cap = attn_traffic_capture()
    traffic = round(cap["bytes"] * kv_bytes / cap["kv_bytes"]) if cap else None
    # the CPU baseline runs at N = 1 only: at N > 1 the host's cores serve every rank
    cpu = cpu_baseline_sample(args) if not args.no_cpu and world == 1 else None
    value = rows_per_step * world / (ms_max * 1e-3)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "verified tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_max, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations x int4 weights, fp32 accumulate",
        "data": "synthetic (seeded random-init weights, random prompt KV pages, random drafts)",
        "config": bench_config(shape.layers, world, SEQS, PROMPT),
        "per_gpu": round(value / world, 2),
        "e2e": {
            "value": round(e2e_rows_all / max(1, e2e_steps) / (e2e_ms_max * 1e-3), 2) if e2e_steps else None,
            "unit": "verified tok/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "ms_per_step": round(e2e_ms_max, 4),
            "host_wall_ms_per_step": round(wall_ms, 4),
            "call": "pilm_b200.engine.MTPVerifyEngine.verify_step (host drafts -> host accept results)",
        },
        "cycle": cycle,
        "cycle_bf16_drafter": cycle_bf16,
        "e2e_accepting": accepting,
        "roofline": {
            "kernel": "attn_pages (+ attn_merge_pages), per layer",
            "bound": "hbm",
            "achieved": round(att_gbs, 1) if att_gbs else None,
            "peak": pk["hbm_gbs"],
            "peak_source": pk["source"],
            "unit": "GB/s",
            "frac": round(att_gbs / pk["hbm_gbs"], 4) if att_gbs else None,
            "traffic": traffic,
            "traffic_source": cap["source"] if cap else None,
            "algorithmic_bytes_per_launch": att_bytes,
            "avg_launch_ms": round(att_ms, 5) if att_ms else None,
        },
        "quant_gemm": {
            "bytes_per_step": lin_bytes,
            "ms_per_step": round(lin_ms, 4) if lin_ms else None,
            "achieved_gbs": round(lin_gbs, 1) if lin_gbs else None,
            "frac_of_peak": round(lin_gbs / pk["hbm_gbs"], 4) if lin_gbs else None,
            "rows": rows_per_step,
        },
        "step_roofline": {
            "algorithmic_bytes": step_bytes,
            "achieved_gbs": round(step_bytes / (ms_max * 1e-3) / 1e9, 1),
            "frac": round(step_bytes / (ms_max * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
        },
        "op_ms_per_step": {k: round(v, 4) for k, v in op_ms.items()},
        "gpu_launches": graph.launches * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "acceptance": {"attempts": eng.stats["attempts"], "accepts": eng.stats["accepts"]},
    }
    if timeline:
        line["timeline"] = timeline
    return line


# ---------------------------------------------------------------------------------------
# CPU baseline: the reference's own C kernels on the host cores
# ---------------------------------------------------------------------------------------

def _ref_linear_ms(lib, M, N, K, threads_note) -> float:
    import numpy as np
    from oracle import reflib
    rng = np.random.default_rng(N + K)
    x = rng.integers(0, 65535, (M, K), dtype=np.uint16) & 0x3FFF | 0x3C00  # finite bf16 values
    qw = rng.integers(0, 256, (N, (K + 1) // 2), dtype=np.uint8)
    s = (rng.random((N, (K + 127) // 128), dtype=np.float32) * 0.01).astype(np.float32)
    out = np.zeros((M, N), np.uint16)  # pages touched before the timed call
    d = reflib.LinearDesc(M, N, K)
    args = (ctypes.byref(d), x.ctypes.data, qw.ctypes.data, s.ctypes.data, out.ctypes.data, 1)
    assert lib.ekernel_linear_w4a16g128_bf16(*args) == 0  # untimed warm-up: thread pool, caches
    t0 = time.perf_counter()
    rc = lib.ekernel_linear_w4a16g128_bf16(*args)
    assert rc == 0
    return (time.perf_counter() - t0) * 1e3


def cpu_baseline_sample(args) -> dict | None:
    """Bounded sample of the reference's CPU verify step: one Qwen3-8B decoder layer's seven
    W4 g128 linears (q, k, v, o, gate, up, down) and the LM head at M = 96 verify rows, each
    timed on its second call (the first warms the thread pool and caches), through the
    reference's ekernel_linear_w4a16g128_bf16 (oracle/_ref/libecpu.so, OpenMP over all host
    threads), plus one layer of the reference's attention for the 32 sequences.  The
    attention runs FullAttention.forward's arithmetic over the paged cache as the reference
    does it, block gather by torch.cat included (attention.py:98-139), through the oracle's
    restatement of that module (oracle/model.py attend): the reference's Python modules are
    not on the GPU box.  The sample is one of 36 layers and is extrapolated to the step."""
    from oracle import reflib
    if not reflib.available():
        return None
    import torch
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    torch.set_num_threads(threads)
    lib = reflib.lib()
    M = SEQS * (K_DRAFT + 1)
    H, I, V = 4096, 12288, 151936
    t0 = time.perf_counter()
    t_layer = 0.0
    for (N, K) in ((4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (I, H), (I, H), (H, I)):
        t_layer += _ref_linear_ms(lib, M, N, K, threads)
    t_head = _ref_linear_ms(lib, M, V, H, threads)
    t_att = _cpu_attention_layer_ms()
    sample_s = time.perf_counter() - t0
    step_ms = 36 * (t_layer + t_att) + t_head
    return {
        "value": round(M / (step_ms * 1e-3), 3),
        "unit": "verified tok/s",
        "cores": threads,
        "kind": "reference",
        "isa": reflib.isa_name(),
        "extrapolated": True,
        "layers_sampled": 1,
        "sample_s": round(sample_s, 3),
        "extrapolated_step_ms": round(step_ms, 1),
        "sample": (f"1 of 36 layers (q/k/v/o/gate/up/down W4 g128 linears at M={M} through the reference "
                   f"ekernel_linear_w4a16g128_bf16: {t_layer:.0f} ms; the reference's paged attention "
                   f"arithmetic over 32 seqs x {PROMPT + K_DRAFT + 1} keys: {t_att:.0f} ms) + LM head "
                   f"({t_head:.0f} ms), timed in {sample_s:.1f} s and extrapolated to a {step_ms / 1e3:.1f} s step"),
    }


_ATT_CACHE = {}


def _cpu_attention_layer_ms() -> float:
    """One layer of the reference attention for all sequences on the host: each sequence's
    pages gathered from the paged cache by torch.cat, GQA expansion, bf16 scores, causal
    mask over the verify rows, fp32 softmax, bf16 P.V (attention.py:98-139, restated in
    oracle/model.py attend), over a page pool shaped like the bench's."""
    import torch
    from oracle import model as om
    nkv, nh, hd, q = 8, 32, 128, K_DRAFT + 1
    ctx = PROMPT + q
    pages = (ctx + PAGE - 1) // PAGE
    if "kv" not in _ATT_CACHE:
        g = torch.Generator().manual_seed(0)
        nb = SEQS * pages + 1
        _ATT_CACHE["kv"] = (torch.randn((nb, PAGE, nkv, hd), generator=g).to(torch.bfloat16),
                            torch.randn((nb, PAGE, nkv, hd), generator=g).to(torch.bfloat16))
        _ATT_CACHE["q"] = torch.randn((q, nh, hd), generator=g).to(torch.bfloat16)
        _ATT_CACHE["tables"] = [list(range(1 + b * pages, 1 + (b + 1) * pages)) for b in range(SEQS)]
    kc, vc = _ATT_CACHE["kv"]
    cfg = om.Qwen3Config(n_heads=nh, n_kv_heads=nkv, head_dim=hd, block_size=PAGE)
    t0 = time.perf_counter()
    for b in range(SEQS):
        om.attend(cfg, _ATT_CACHE["q"], None, kc, vc, _ATT_CACHE["tables"][b], ctx, True)
    return (time.perf_counter() - t0) * 1e3


def run_reference(args, rank: int, world: int = 1) -> dict | None:
    """The reference arm: rank 0 times cpu_baseline_sample --steps times (after --warmup
    untimed samples); each step is one bounded sample, and `value` is the median sample's
    extrapolated verified tok/s.  ms_per_step is the measured wall time of one sample, so
    steps x ms_per_step is the timed region; extrapolated_step_ms is the full step."""
    if rank != 0:
        return None
    from oracle import reflib
    if not reflib.available():
        return {"impl": "reference", "unavailable": "oracle/_ref/libecpu.so was not built (reference sources absent)"}
    for _ in range(max(0, args.warmup)):  # untimed warm-up samples
        cpu_baseline_sample(args)
    samples = []
    for _ in range(max(1, args.steps)):
        samples.append(cpu_baseline_sample(args))
    samples.sort(key=lambda c: c["value"])
    cpu = samples[len(samples) // 2]
    value = cpu["value"]
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "verified tok/s",
        "n_gpus": 0,
        "steps": len(samples),
        "warmup": max(0, args.warmup),
        "ms_per_step": round(statistics.mean(c["sample_s"] for c in samples) * 1e3, 1),
        "extrapolated": True,
        "layers_sampled": 1,
        "extrapolated_step_ms": cpu["extrapolated_step_ms"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 activations x int4 weights, fp32 accumulate (AVX2)",
        "data": "synthetic",
        "config": bench_config(36, world),
        "cpu_baseline": dict(cpu),
        "e2e": {"value": value, "unit": "verified tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------------------
# BASELINE configs 1-3 (python bench.py --config N): one JSON line each
# ---------------------------------------------------------------------------------------

CONFIGS = {
    1: dict(name="Qwen3-0.6B-shaped W8A32 (fp32 activations) MTP verify, BASELINE configs[0]", shape="0.6B",
            fmt="w8a32", seqs=1, k=1, prompt=(128, 128), gen=128, sampling=None),
    2: dict(name="Qwen3-1.7B-shaped W4A16 g128 MTP verify, BASELINE configs[1]", shape="1.7B", fmt="w4a16g128",
            seqs=1, k=3, prompt=(512, 512), gen=256, sampling=None),
    3: dict(name="Qwen3-1.7B-shaped W4A16 g128 MTP verify under continuous batching with rejection sampling "
                 "(T 0.8, top-p 0.95), BASELINE configs[2]", shape="1.7B", fmt="w4a16g128", seqs=64, k=3,
            prompt=(128, 2048), gen=256, sampling=(0.8, 0.95), pool_pages=16384),
}


def _config_prompts(cfg, seed):
    import numpy as np
    lo, hi = cfg["prompt"]
    rng = np.random.default_rng(seed)
    return [int(v) for v in rng.integers(lo, hi + 1, cfg["seqs"])]


def cpu_baseline_config(cfg, lens) -> dict | None:
    """The reference's CPU verify step for configs 1-3 on the host cores: its own linears
    (oracle/_ref/libecpu.so: ekernel_linear_w8a32 for config 1, ekernel_linear_w4a16g128_bf16
    otherwise, q/k/v/o/gate/up/down per layer as the reference issues them) plus its paged
    attention arithmetic (oracle/model.py attend, the torch.cat page gather of
    attention.py:98-139) and the LM head.  Configs 1 and 2 run every layer on distinct
    weights (the whole forward, timed on its second run); config 3 (256 rows) samples one
    layer and extrapolates to 28."""
    from oracle import reflib
    if not reflib.available():
        return None
    import numpy as np
    import torch
    from oracle import model as om
    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    torch.set_num_threads(threads)
    lib = reflib.lib()
    H, I, V, L = (1024, 3072, 151936, 28) if cfg["shape"] == "0.6B" else (2048, 6144, 151936, 28)
    nh, nkv, hd = 16, 8, 128
    M = sum(1 + cfg["k"] for _ in lens)
    fp32 = cfg["fmt"] == "w8a32"
    shapes = [(nh * hd, H), (nkv * hd, H), (nkv * hd, H), (H, nh * hd), (I, H), (I, H), (H, I)]
    rng = np.random.default_rng(7)
    layers = 1 if cfg["seqs"] > 1 else L

    def weights(N, K):
        if fp32:
            return (rng.integers(-127, 128, (N, K), dtype=np.int8), rng.random(N, dtype=np.float32) * 0.01)
        return (rng.integers(0, 256, (N, K // 2), dtype=np.uint8), rng.random((N, K // 128), dtype=np.float32) * 0.01)

    W = [[weights(N, K) for (N, K) in shapes] for _ in range(layers)]
    head = weights(V, H)
    fn = lib.ekernel_linear_w8a32 if fp32 else lib.ekernel_linear_w4a16g128_bf16

    def xin(K):
        if fp32:
            return rng.standard_normal((M, K), dtype=np.float32)
        return (rng.integers(0, 65535, (M, K), dtype=np.uint16) & 0x3FFF) | 0x3C00

    X = {K: xin(K) for K in {H, I, nh * hd}}
    outs = {N: np.zeros((M, N), np.float32 if fp32 else np.uint16) for N in {nh * hd, nkv * hd, H, I, V}}

    def linear(w, N, K):
        d = reflib.LinearDesc(M, N, K)
        assert fn(ctypes.byref(d), X[K].ctypes.data, w[0].ctypes.data, w[1].ctypes.data, outs[N].ctypes.data, 1) == 0

    ocfg = om.Qwen3Config(n_heads=nh, n_kv_heads=nkv, head_dim=hd, block_size=PAGE,
                          dtype="float32" if fp32 else "bfloat16")
    dt = torch.float32 if fp32 else torch.bfloat16
    q = torch.randn((1 + cfg["k"], nh, hd)).to(dt)
    pages = [(c + PAGE - 1) // PAGE for c in lens]
    kc = torch.randn((sum(pages) + 1, PAGE, nkv, hd)).to(dt)
    vc = torch.randn((sum(pages) + 1, PAGE, nkv, hd)).to(dt)
    tables, off = [], 1
    for p in pages:
        tables.append(list(range(off, off + p)))
        off += p

    def attention():
        for b, c in enumerate(lens):
            om.attend(ocfg, q, None, kc, vc, tables[b], c, True)

    def forward():
        t_lin = t_att = 0.0
        for li in range(layers):
            t0 = time.perf_counter()
            for w, (N, K) in zip(W[li], shapes):
                linear(w, N, K)
            t1 = time.perf_counter()
            attention()
            t2 = time.perf_counter()
            t_lin += t1 - t0
            t_att += t2 - t1
        t0 = time.perf_counter()
        linear(head, V, H)
        return t_lin, t_att, time.perf_counter() - t0

    forward()  # warm-up: thread pool, pages of the outputs
    t_lin, t_att, t_head = forward()
    scale = L / layers
    step_s = scale * (t_lin + t_att) + t_head
    what = "all 28 layers" if layers == L else f"1 of {L} layers, extrapolated to {L}"
    return {
        "value": round(M / step_s, 3), "unit": "verified tok/s", "cores": threads, "kind": "reference",
        "isa": reflib.isa_name(), "extrapolated": layers != L, "layers_sampled": layers,
        "sample": (f"{what}: {'W8A32' if fp32 else 'W4A16 g128'} linears at M={M} through the reference library "
                   f"({t_lin * 1e3:.0f} ms), its paged attention arithmetic over {len(lens)} seqs "
                   f"({t_att * 1e3:.0f} ms), LM head ({t_head * 1e3:.0f} ms): a {step_s * 1e3:.0f} ms step"),
    }


def run_config(args) -> dict:
    """Configs 1-3 on one GPU: the verify step from a captured graph on device-resident
    inputs (value), end to end through MTPVerifyEngine.verify_step with host drafts (e2e),
    the step's HBM roofline and the reference CPU path."""
    import torch
    from pilm_b200 import bindings
    from pilm_b200.engine import MTPVerifyEngine
    from pilm_b200.qwen3 import (QWEN3_0_6B, QWEN3_1_7B, PagedKVCache, Qwen3Verifier, Qwen3VerifierF32,
                                 Qwen3Weights, Qwen3WeightsF32, VerifyGraph)
    cfg = CONFIGS[args.config]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bindings.init()
    shape = QWEN3_0_6B if cfg["shape"] == "0.6B" else QWEN3_1_7B
    fp32 = cfg["fmt"] == "w8a32"
    seed, k, B = 4321, cfg["k"], cfg["seqs"]
    lens = _config_prompts(cfg, seed)
    headroom = cfg["gen"] + 32
    max_len = max(lens) + headroom + 64
    num_blocks = cfg.get("pool_pages") or sum((n + headroom + PAGE - 1) // PAGE for n in lens) + 1
    if fp32:
        weights = Qwen3WeightsF32.synthetic(shape, seed, dev)
        kv = PagedKVCache(shape, num_blocks, dev, dtype=torch.float32)
        ver = Qwen3VerifierF32(weights, kv, max_rows=B * (k + 1), max_pos=max_len, device=dev)
    else:
        weights = Qwen3Weights.synthetic(shape, seed, dev)
        kv = PagedKVCache(shape, num_blocks, dev, fill="random", seed=seed)
        ver = Qwen3Verifier(weights, kv, max_rows=B * (k + 1), max_pos=max_len, device=dev)
    T_, P_ = cfg["sampling"] or (0.0, 1.0)
    eng = MTPVerifyEngine(ver, num_blocks=num_blocks, max_model_len=max_len, temperature=T_, top_p=P_,
                          sample_seed=seed)
    g = torch.Generator().manual_seed(seed)
    for n in lens:
        sid = eng.add_request(torch.randint(0, shape.vocab, (n,), generator=g).tolist(), max_new_tokens=cfg["gen"])
        eng.admit_prefilled(sid)
    for s in eng.sched.running:  # the pending first generated token
        t = int(torch.randint(0, shape.vocab, (1,), generator=g))
        s.tokens.append(t)
        s.outputs.append(t)

    def drafts_for_step():
        return {s.seq_id: torch.randint(0, shape.vocab, (k,), generator=g).tolist() for s in eng.sched.running}

    # ---- device-resident step: every sequence verifies k drafts (as many as its page allows)
    from pilm_b200.engine import draft_limit
    seqs = list(eng.sched.running)
    counts = []
    for s in seqs:
        n = draft_limit(s.num_computed, PAGE, cfg["gen"], k)
        s.tokens.extend(torch.randint(0, shape.vocab, (n,), generator=g).tolist())
        eng.pages.allocate(s, 1 + n, eng.max_pages)
        counts.append(1 + n)
    batch = eng.build_batch(seqs, [s.num_computed for s in seqs], counts)
    graph = VerifyGraph(ver, B, batch.total_q, batch.max_q_len, eng.max_pages, eng.max_model_len,
                        sampling=cfg["sampling"])
    uni = torch.rand((batch.total_q, 2), generator=g).to(dev) if cfg["sampling"] else None
    graph.load(batch, uni)
    graph.capture()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    sampler = ClockSampler(0)
    sampler.start()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    rows = batch.total_q
    timeline = graph_timeline(graph) if args.timeline else None
    for s in seqs:
        del s.tokens[s.num_computed + 1:]
    # ---- end to end through the engine
    for _ in range(max(args.warmup, PAGE)):
        eng.verify_step(drafts_for_step())
    step_drafts = [drafts_for_step() for _ in range(args.steps)]
    torch.cuda.synchronize()
    r0 = eng.stats["verified_rows"]
    a0, t0c = eng.stats["accepts"], eng.stats["attempts"]
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for d in step_drafts:
        eng.verify_step(d)
    c1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    e2e_ms = c0.elapsed_time(c1) / args.steps
    e2e_rows = eng.stats["verified_rows"] - r0
    # ---- roofline: weights + K/V read + appended K/V + logits written, per step
    ctx = sum(len(s.tokens) for s in seqs)
    kv_bytes = ctx * kv.bytes_per_token
    act = 4 if fp32 else 2
    step_bytes = weights.linear_bytes + kv_bytes + rows * shape.vocab * act + rows * shape.hidden * act
    pk = peaks()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    flops = 2 * rows * (weights.linear_bytes / (1.0 if fp32 else 0.53125))
    cpu = None if args.no_cpu else cpu_baseline_config(cfg, [s.num_computed + 1 for s in seqs])
    return {
        "metric": METRIC, "config_id": args.config,
        "value": round(rows / (ms * 1e-3), 2), "unit": "verified tok/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32 activations x int8 weights" if fp32 else "bf16 activations x int4 weights, fp32 accumulate",
        "data": "synthetic (seeded random-init weights, random prompt KV pages, random drafts)",
        "config": {"workload": cfg["name"], "seqs": B, "prompt_lens": f"{min(lens)}-{max(lens)}", "draft_k": k,
                   "rows_per_step": rows, "page_size": PAGE, "kv_pool_pages": num_blocks,
                   "verification": (f"rejection sampling T={cfg['sampling'][0]} top-p={cfg['sampling'][1]}"
                                    if cfg["sampling"] else "greedy"),
                   "l2": "inputs larger than L2" if step_bytes > L2_BYTES else "inputs fit in L2 (small model)"},
        "e2e": {"value": round(e2e_rows / args.steps / (e2e_ms * 1e-3), 2), "unit": "verified tok/s",
                "ms_per_step": round(e2e_ms, 4),
                "call": "pilm_b200.engine.MTPVerifyEngine.verify_step (host drafts -> host accept results)",
                "accept_rate": round((eng.stats["accepts"] - a0) / max(1, eng.stats["attempts"] - t0c), 4)},
        "step_roofline": {"algorithmic_bytes": step_bytes, "weight_bytes": weights.linear_bytes,
                          "kv_bytes": kv_bytes, "achieved_gbs": round(gbs, 1), "peak": pk["hbm_gbs"],
                          "peak_source": pk["source"], "frac": round(gbs / pk["hbm_gbs"], 4),
                          "tflops": round(flops / (ms * 1e-3) / 1e12, 2)},
        "gpu_launches": graph.launches * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
        **({"timeline": timeline} if timeline else {}),
    }


# ---------------------------------------------------------------------------------------
# op sweep: each hot-path kernel alone, over the shapes the configurations use
# ---------------------------------------------------------------------------------------

SWEEP_M = (1, 2, 3, 4, 8, 16, 32, 64, 128, 256)
SWEEP_KN = ((4096, 6144), (4096, 4096), (4096, 24576), (12288, 4096), (4096, 151936))
L2_BYTES = 126 * 2 ** 20


def run_prefill(args) -> None:
    """Prefill of one long prompt through MTPVerifyEngine.prefill (not the verify metric):
    chunks of --prefill-chunk tokens crossing page boundaries, against the reference's
    page-aligned chunks (engine.py:218).  One JSON line per schedule: wall time of the
    whole prefill (host scheduling included), prompt tokens/s, the first token, and a
    per-op split from a third run with the verifier's CUDA events on."""
    import torch

    from pilm_b200 import bindings
    from pilm_b200.engine import MTPVerifyEngine
    from pilm_b200.qwen3 import QWEN3_8B, PagedKVCache, Qwen3Verifier, Qwen3Weights

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    bindings.init()
    shape = QWEN3_8B
    P = args.prefill
    weights = Qwen3Weights.synthetic(shape, 1234, dev)
    prompt = torch.randint(0, shape.vocab, (P,), generator=torch.Generator().manual_seed(5)).tolist()
    nb = (P + GEN_HEADROOM) // PAGE + 2
    schedules = [(args.prefill_chunk, False)] + ([(PAGE * 32, True)] if args.prefill_aligned else [])
    for chunk, aligned in schedules:
        kv = PagedKVCache(shape, nb, dev)
        ver = Qwen3Verifier(weights, kv, max_rows=chunk, max_pos=P + GEN_HEADROOM, device=dev)

        def once():
            eng = MTPVerifyEngine(ver, num_blocks=nb, max_model_len=P + GEN_HEADROOM,
                                  max_num_batched_tokens=chunk, page_aligned_chunks=aligned)
            sid = eng.add_request(prompt, max_new_tokens=8)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            first = eng.prefill()[sid]
            torch.cuda.synchronize()
            return time.perf_counter() - t0, first, len(eng.sched.seqs[sid].pages)

        cold, _, _ = once()  # scratch buffers, kernel attributes
        t, first, npages = once()
        ver.op_timing, ver.op_events = True, []
        once()
        ops = {k: round(v, 2) for k, v in ver.collect_op_times().items() if k != "attention"}
        ver.op_timing = False
        print(json.dumps({"prefill_tokens": P, "chunk": chunk, "page_aligned": aligned, "ms": round(t * 1e3, 1),
                          "cold_ms": round(cold * 1e3, 1), "tok_s": round(P / t, 1), "first_token": first,
                          "pages": npages, "op_ms": ops, "model": "Qwen3-8B W4A16 g128 (synthetic weights)"}),
              flush=True)
        del ver, kv
        torch.cuda.empty_cache()


def graph_timeline(graph, replays: int = 3) -> dict:
    """Where a captured step's time goes, on the device: CUPTI kernel records (torch.profiler)
    of `replays` graph replays, the middle one kept.  Kernels overlap at programmatic
    dependent launches, so each kernel is charged only the part of its span after every
    earlier kernel has ended (its share of the critical path); the shares add up to the
    step.  Taken outside the timed region."""
    import re
    from collections import Counter, defaultdict

    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(replays):
            graph.replay()
        torch.cuda.synchronize()
    evs = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                 if e.device_type == torch.autograd.DeviceType.CUDA)
    n = len(evs) // replays
    step = evs[n * (replays // 2):n * (replays // 2 + 1)]
    if not step:
        return {}

    def short(name: str) -> str:
        name = name.replace("void ", "").replace("(anonymous namespace)::", "").replace("pilm::", "")
        m = re.match(r"[\w:]+", name)
        return m.group(0) if m else name[:40]

    crit, span, cnt = defaultdict(float), defaultdict(float), Counter()
    gaps, prev_end = 0.0, step[0][0]
    for s0, e0, name in step:
        k = short(name)
        span[k] += e0 - s0
        cnt[k] += 1
        gaps += max(0.0, s0 - prev_end)
        crit[k] += max(0.0, e0 - max(s0, prev_end))
        prev_end = max(prev_end, e0)
    total = step[-1][1] - step[0][0]
    return {"step_ms": round(total / 1e3, 4), "kernels": len(step), "idle_ms": round(gaps / 1e3, 4),
            "critical_ms": {k: round(crit[k] / 1e3, 4) for k in sorted(crit, key=lambda k: -crit[k])},
            "launches": {k: cnt[k] for k in sorted(crit, key=lambda k: -crit[k])},
            "span_ms": {k: round(span[k] / 1e3, 4) for k in sorted(crit, key=lambda k: -crit[k])},
            "how": "CUPTI kernel records of one graph replay (torch.profiler); a kernel's critical time is "
                   "its span after every earlier kernel has ended"}


def _graph_ms(body, calls: int, iters: int = 5) -> float:
    """ms per call: body() issues `calls` launches; it is captured once as a CUDA graph and
    replayed `iters` times between two CUDA events after a warm-up replay."""
    import torch
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        body()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        body()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / (iters * calls)


def run_sweep(args) -> None:
    """One JSON line per case.  Linears on the Qwen3-8B projection shapes (K, N): W4A16 g128
    (reference packing, and the k-pair layout the model keeps its weights in) and W8A32 at
    every M of SWEEP_M, bf16 weights (the draft module's default) at M <= 64; enough
    weight copies are cycled that each call reads
    its weights from HBM (copies x bytes > 2 x L2).  Paged attention: q_len 2-5 at 1K, 8K
    and 32K keys, 32 Q / 8 KV heads, batch sized to about 1 GB of K/V per call.  Accept:
    row top-2 + greedy accept over 256 sequences x 5 rows x 151936 bf16 logits."""
    import torch

    from pilm_b200 import bindings
    from pilm_b200 import ckernel as ck
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    bindings.init()
    pk = peaks()
    peak = pk["hbm_gbs"]
    g = torch.Generator(device=dev).manual_seed(7)

    def emit(d):
        d["peak_gbs"], d["peak_source"] = peak, pk["source"]
        print(json.dumps(d), flush=True)

    only = set(args.sweep.split(",")) if args.sweep != "all" else {"linear", "attention", "accept"}
    m_list = [int(v) for v in args.sweep_m.split(",")] if args.sweep_m else SWEEP_M
    kns = [tuple(int(t) for t in v.split("x")) for v in args.sweep_kn.split(",")] if args.sweep_kn else SWEEP_KN
    fmts = (args.sweep_formats.split(",") if args.sweep_formats
            else ("w4a16g128", "w4a16g128_kpairs", "w8a32", "bf16"))
    if "linear" in only:
        for K, N in kns:
            for fmt in fmts:
                if fmt == "bf16":
                    wbytes = 2 * N * K
                    mk = lambda: ((torch.randn((N, K), device=dev, generator=g) * 0.02).to(torch.bfloat16), None)
                elif fmt.startswith("w4a16g128"):
                    wbytes = N * K // 2 + 4 * N * (K // 128)
                    mk = lambda: (torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g),
                                  torch.rand((N, K // 128), device=dev, generator=g) * 0.01 + 1e-4)
                else:
                    wbytes = N * K + 4 * N
                    mk = lambda: (torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g),
                                  torch.rand((N,), device=dev, generator=g) * 0.01 + 1e-4)
                copies = max(1, -(-2 * L2_BYTES // wbytes))
                ws = [mk() for _ in range(copies)]
                kp = fmt.endswith("_kpairs")  # the model's load-time layout (a nibble permutation)
                calls = max(copies, 8)
                for M in m_list:
                    if fmt == "bf16" and M > 64:
                        continue  # the draft module's shapes: M = sequences per step
                    if fmt == "bf16":
                        x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
                        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
                        io = 2 * M * K + 2 * M * N
                        fn = lambda i: ck.linear_bf16(x, ws[i % copies][0], out=y)
                    elif fmt.startswith("w4a16g128"):
                        x = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
                        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
                        io = 2 * M * K + 2 * M * N
                        fn = lambda i: ck.linear_w4a16g128_bf16(x, ws[i % copies][0], ws[i % copies][1], out=y,
                                                                kpairs=kp)
                    else:
                        x = torch.randn((M, K), device=dev, generator=g)
                        y = torch.empty((M, N), dtype=torch.float32, device=dev)
                        io = 4 * M * K + 4 * M * N
                        fn = lambda i: ck.linear_w8a32(x, ws[i % copies][0], ws[i % copies][1], out=y)

                    def body():
                        for i in range(calls):
                            fn(i)
                    ms = _graph_ms(body, calls)
                    gbs = (wbytes + io) / (ms * 1e-3) / 1e9
                    emit({"sweep": "linear", "format": fmt, "M": M, "K": K, "N": N, "us": round(ms * 1e3, 2),
                          "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                          "tflops": round(2 * M * N * K / (ms * 1e-3) / 1e12, 2)})
                del ws
                torch.cuda.empty_cache()
    if "attention" in only:
        from pilm_b200.qwen3 import QWEN3_8B, attention_bytes, attention_slices
        s = QWEN3_8B
        ctx_list = [int(v) for v in args.sweep_ctx.split(",")] if args.sweep_ctx else [1024, 8192, 32768]
        q_list = [int(v) for v in args.sweep_q.split(",")] if args.sweep_q else [2, 3, 4, 5, 16]
        for ctx in ctx_list:
            B = max(1, (2 ** 30) // (ctx * s.n_kv_heads * s.head_dim * 4))
            pages = -(-(ctx + 8) // 16)
            nb = B * pages + 1
            kc = torch.randn((nb, 16, s.n_kv_heads, s.head_dim), device=dev, generator=g).to(torch.bfloat16)
            vc = torch.randn((nb, 16, s.n_kv_heads, s.head_dim), device=dev, generator=g).to(torch.bfloat16)
            perm = (torch.randperm(nb - 1, device=dev, generator=g) + 1).to(torch.int32)
            table = perm[:B * pages].view(B, pages).contiguous()
            for q_len in q_list:
                T = B * q_len
                i32 = dict(dtype=torch.int32, device=dev)
                cu = torch.arange(0, T + 1, q_len, **i32)
                ctxs = torch.full((B,), ctx, **i32)
                q = torch.randn((T, s.n_heads * s.head_dim), device=dev, generator=g).to(torch.bfloat16)
                out = torch.empty_like(q)
                desc = ck.attn_desc(num_seqs=B, total_q=T, max_q_len=q_len, n_heads=s.n_heads,
                                    n_kv_heads=s.n_kv_heads, head_dim=s.head_dim, block_size=16, num_blocks=nb,
                                    max_blocks_per_seq=pages, max_context=ctx, qkv_stride=s.qkv_rows,
                                    rope_rows=0, rot_dim=s.rot_dim, eps=s.eps, add_one=0, output_gate=0)

                def body():
                    for _ in range(4):
                        ck.paged_attention_verify(desc, q, kc, vc, table, cu, ctxs, None, out)
                ms = _graph_ms(body, 4)
                nbytes = attention_bytes(s, [ctx] * B, [q_len] * B)
                gbs = nbytes / (ms * 1e-3) / 1e9
                emit({"sweep": "attention", "q_len": q_len, "ctx": ctx, "seqs": B, "heads": [s.n_heads, s.n_kv_heads],
                      "us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)})
                cut = attention_slices(cu.cpu().numpy(), ctxs.cpu().numpy(), s.n_heads // s.n_kv_heads)
                if q_len * s.n_heads // s.n_kv_heads > 16 and cut is not None:
                    # the same pass cut into 16-row slices for the whole-page kernel
                    seq, cu_v, ctx_v, span = cut
                    table_v = table.index_select(0, torch.tensor(seq, dtype=torch.int64, device=dev)).contiguous()
                    cu_v, ctx_v = torch.tensor(cu_v, **i32), torch.tensor(ctx_v, **i32)
                    desc_v = ck.attn_desc(num_seqs=len(seq), total_q=T, max_q_len=span, n_heads=s.n_heads,
                                          n_kv_heads=s.n_kv_heads, head_dim=s.head_dim, block_size=16, num_blocks=nb,
                                          max_blocks_per_seq=pages, max_context=ctx, qkv_stride=s.qkv_rows,
                                          rope_rows=0, rot_dim=s.rot_dim, eps=s.eps, add_one=0, output_gate=0)

                    def body_v():
                        for _ in range(4):
                            ck.paged_attention_verify(desc_v, q, kc, vc, table_v, cu_v, ctx_v, None, out)
                    ms = _graph_ms(body_v, 4)
                    gbs = nbytes / (ms * 1e-3) / 1e9
                    emit({"sweep": "attention_sliced", "q_len": q_len, "ctx": ctx, "seqs": B, "slices": len(seq),
                          "heads": [s.n_heads, s.n_kv_heads], "us": round(ms * 1e3, 2), "gbs": round(gbs, 1),
                          "frac": round(gbs / peak, 4)})
            del kc, vc
            torch.cuda.empty_cache()
    if "accept" in only:
        B, k, V = 256, 4, 151936
        T = B * (k + 1)
        i32 = dict(dtype=torch.int32, device=dev)
        logits = torch.randn((T, V), device=dev, generator=g).to(torch.bfloat16)
        ids = torch.randint(0, V, (T,), device=dev, generator=g).to(torch.int32)
        cu = torch.arange(0, T + 1, k + 1, **i32)
        top1, acc, nxt = torch.empty(T, **i32), torch.empty(B, **i32), torch.empty(B, **i32)
        ctx0 = torch.full((B,), 4096, **i32)
        ctxs = ctx0.clone()

        def body():
            for _ in range(4):
                ctxs.copy_(ctx0)
                ck.argmax_top2(logits, top1)
                ck.verify_accept_greedy(B, ids, top1, cu, acc, nxt, ctxs)
        ms = _graph_ms(body, 4)
        nbytes = T * V * 2
        gbs = nbytes / (ms * 1e-3) / 1e9
        emit({"sweep": "accept", "seqs": B, "k": k, "vocab": V, "us": round(ms * 1e3, 2), "gbs": round(gbs, 1),
              "frac": round(gbs / peak, 4)})
        # rejection sampling (T 0.8, top-p 0.95) over the same bf16 logits: three reads of every
        # row for its nucleus statistics (max, bin histogram, gather of the cut's bin), then
        # two reads of one row per sequence to sample
        uni = torch.rand((T, 2), device=dev, generator=g)

        def body_rs():
            for _ in range(4):
                ctxs.copy_(ctx0)
                ck.verify_accept_rejection(B, logits, ids, cu, uni, 0.8, 0.95, acc, nxt, ctxs)
        ms = _graph_ms(body_rs, 4)
        nbytes = (3 * T + 2 * B) * V * 2
        gbs = nbytes / (ms * 1e-3) / 1e9
        emit({"sweep": "accept_rejection", "seqs": B, "k": k, "vocab": V, "temperature": 0.8, "top_p": 0.95,
              "us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end engine leg (profiling runs)")
    ap.add_argument("--timeline", action="store_true",
                    help="add the step's per-kernel critical-path times (CUPTI records of one graph replay, "
                         "taken after the timed region)")
    ap.add_argument("--no-draft", action="store_true", help="skip the verify + GPU draft cycle leg")
    ap.add_argument("--no-accepting", action="store_true",
                    help="skip the leg whose drafts are accepted (the model's own greedy continuation)")
    ap.add_argument("--seqs", type=int, default=SEQS, help="sequences per GPU (default: the BASELINE config)")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="prompt tokens per sequence")
    ap.add_argument("--layers", type=int, default=0, help="decoder layers (0 = all 36); profiling only")
    ap.add_argument("--sweep", default=None,
                    help="per-kernel op sweep instead of the bench line: all, or any of linear,attention,accept")
    ap.add_argument("--sweep-m", default=None, help="linear sweep: comma-separated M values (default: all)")
    ap.add_argument("--sweep-kn", default=None, help="linear sweep: comma-separated KxN shapes (default: Qwen3-8B)")
    ap.add_argument("--sweep-formats", default=None,
                    help="linear sweep: comma-separated formats of w4a16g128,w4a16g128_kpairs,w8a32,bf16")
    ap.add_argument("--sweep-ctx", default=None, help="attention sweep: comma-separated context lengths")
    ap.add_argument("--sweep-q", default=None, help="attention sweep: comma-separated rows per sequence")
    ap.add_argument("--config", type=int, default=0, choices=[0, 1, 2, 3],
                    help="BASELINE configs[0..2] (configs 1-3) on one GPU instead of the config-4 bench line")
    ap.add_argument("--prefill", type=int, default=0,
                    help="time the prefill of one prompt of this many tokens instead of the bench line")
    ap.add_argument("--prefill-chunk", type=int, default=2048, help="prefill: tokens per pass (cross-page chunks)")
    ap.add_argument("--prefill-aligned", action="store_true",
                    help="prefill: also time the reference's page-aligned chunk schedule")
    args = ap.parse_args()
    if args.prefill:
        run_prefill(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.config:
        print(json.dumps(run_config(args)), flush=True)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    line = run_ours(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

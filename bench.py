#!/usr/bin/env python
"""Decode and prefill throughput of the SLM.use token loop on B200.

Workload ("C2"): the 86M-class looped hybrid
(d 768, 12 heads × 64, FFN 3072, vocab 32000, window 4096, layout S | LS | S,
fp32, N(0, 0.02) random init, seed 0) at R = 4 loops.  A 4096-id uniform
random prompt is read in 256-token chunks, so every sliding-window ring is
full; then greedy decode.  One bench step = one decoded token (one m = 1
advance through prelude, R loops of the core and coda, tied logits, and the
on-device pick).

Printed on one JSON line (rank 0):
  value     decode tok/s over all ranks, inputs resident on the device
            (`slm_decode`: ids stay on the GPU), CUDA events on the library's
            stream, max over ranks;
  e2e       the same decode through the per-token C ABI (`slm_step` with a
            host id + `slm_sample` returning a host id), host clock;
  prefill   tok/s of the 4096-token prompt (feed + logits read back);
  extra     R = 8 and R = 16 decode with the sampling of configs[2]; C4,
            the G-layer variant (S | LS | SG) after a 16384-id prompt; C5,
            64 sequences (2048-id prompts) split over the ranks and decoded
            as one batch per GPU (aggregate tok/s, max over ranks);
  roofline  the decode step's kernel (one persistent kernel per token) against
            measured HBM bandwidth, and the m = 1 GEMV op on its own;
  cpu_baseline  the CPU oracle (a C++ restatement of the reference's CPU
            backend) on a bounded sample, rank 0 only, N = 1 only.
  ref_cuda_baseline  the reference's own CUDA kernels (kernels/slm.cu built
            from source) under a C++ restatement of its host side, on the same
            GPU with its own bench protocol; 32 decode steps per loop count
            after the same 4096-id prompt, and C4 (16384-id prompt, 16
            decode steps); rank 0, N = 1 only.

--impl reference runs only the CPU oracle on the host cores (rank 0), since
the reference itself (Rust) cannot be built on this image.

Multi-GPU (torchrun): each rank decodes its own sequence on its own GPU, no
collective on the data path ("weak" scaling); NCCL only for the barrier and
the max-over-ranks of the timed region.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
MODEL_BYTES_NOTE = "inputs larger than L2: 640 MB of weights and KV read per token at R=4"
# DRAM bytes (read + write) of one k_decode_mega launch from an ncu capture of
# this bench (profiles/k_decode_mega_R4.md), by loop count.
# DRAM bytes (read + write) of one R = 4 step, ncu dram__bytes of one launch
# (profiles/k_decode_mega_R4.md); no capture exists for other loop counts.
MEGA_TRAFFIC = {4: 444.9e6}


def load_pkg():
    if "slm_b200" in sys.modules:
        return sys.modules["slm_b200"]
    pkg = ROOT / "slm.use_b200"
    spec = importlib.util.spec_from_file_location("slm_b200", pkg / "__init__.py",
                                                  submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["slm_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def prompt_for(rank: int, vocab: int, n: int) -> np.ndarray:
    """The prompt of rank r: n uniform ids from seed r (each rank decodes its own sequence)."""
    return np.random.default_rng(rank).integers(0, vocab, n).astype(np.uint32)


def c5_partition(n_seq: int, rank: int, world: int) -> list[int]:
    """configs[4]'s sequences of rank r: q = r, r + world, r + 2·world, … (round robin,
    each sequence on exactly one rank; no collective on the data path)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return list(range(rank, n_seq, world))


def max_over_ranks(values, dist=None, device=None):
    """Element-wise max of per-rank timings (the slowest rank sets the job's time)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return list(values)
    import torch
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def model_dir(cfg: dict, seed: int) -> Path:
    """The synthetic model for (cfg, seed), written once.  Each process writes
    into its own temporary folder and publishes it with an atomic rename, so
    ranks that start together never read a half-written file."""
    import shutil

    import slm_b200.synthetic as syn  # noqa: F401  (package registered by load_pkg)
    tag = hashlib.sha1(json.dumps([cfg, seed], sort_keys=True).encode()).hexdigest()[:12]
    root = Path(os.environ.get("SLM_BENCH_DIR", str(ROOT / "_bench_models")))
    folder = root / tag
    if (folder / "done").exists():
        return folder
    tmp = root / f".{tag}.{os.getpid()}"
    syn.write_model(tmp, cfg, seed)
    (tmp / "done").write_text("ok")
    try:
        os.rename(tmp, folder)
    except OSError:  # another process published it first
        shutil.rmtree(tmp, ignore_errors=True)
    return folder


# ---------------------------------------------------------------------------
# Algorithmic bytes per decoded token (fp32), full window
# ---------------------------------------------------------------------------

def decode_bytes(cfg: dict, loops: int) -> dict:
    d, h, f, v, w = cfg["d_model"], cfg["n_heads"], cfg["hidden"], cfg["vocab_size"], cfg["window"]
    dh = d // h
    s_par = 3 * d * d + d * d + 2 * f * d + f * d + 2 * d
    l_par = 4 * d * d + h * d + d * d + 2 * f * d + f * d + 2 * d + h + dh
    n_s = cfg["prelude"].count("S") + cfg["coda"].count("S") + loops * cfg["core"].count("S")
    n_l = loops * cfg["core"].count("L")
    weights = 4 * (cfg["prelude"].count("S") * s_par + cfg["coda"].count("S") * s_par
                   + loops * (cfg["core"].count("S") * s_par + cfg["core"].count("L") * l_par)
                   + d * d + v * d + d)
    kv = n_s * 2 * h * w * dh * 4
    gla = n_l * 2 * h * dh * dh * 4
    return {"weights": weights, "kv": kv, "gla_state": gla, "total": weights + kv + gla}


def prefill_flops(cfg: dict, loops: int, n: int) -> float:
    """Algorithmic fp32 flops of reading an n-token prompt (S | LS | S layouts):
    the linears of every token, attention over each token's window, the GLA
    recurrence, and the logits of the last token."""
    d, h, f, v, w = cfg["d_model"], cfg["n_heads"], cfg["hidden"], cfg["vocab_size"], cfg["window"]
    dh = d // h
    s_lin = 3 * d * d + d * d + 2 * f * d + f * d
    l_lin = 4 * d * d + h * d + d * d + 2 * f * d + f * d
    n_s = cfg["prelude"].count("S") + cfg["coda"].count("S") + loops * cfg["core"].count("S")
    n_l = loops * cfg["core"].count("L")
    lin = n_s * s_lin + n_l * l_lin + (d * d if cfg["core"] else 0)
    spans = sum(min(p + 1, w) for p in range(n))
    return 2.0 * lin * n + n_s * 4.0 * d * spans + n_l * 4.0 * h * dh * dh * n + 2.0 * v * d


# ---------------------------------------------------------------------------
# Clocks during the timed region
# ---------------------------------------------------------------------------

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU oracle (the reference's CPU path restated) — baseline only
# ---------------------------------------------------------------------------

def cpu_measure(folder: Path, loops: int, steps: int, warmup: int, budget_s: float) -> dict:
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O

    cores = O.lib().orc_threads(os.cpu_count() or 1)
    model = O.Model(folder)
    se = model.session(loops)
    se.fill(4096, seed=0)
    tok = 1
    for _ in range(warmup):
        se.step(tok)
        tok = int(np.argmax(se.logits()))
    done, t0 = 0, time.perf_counter()
    while done < steps:
        se.step(tok)
        tok = int(np.argmax(se.logits()))
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dec_s = time.perf_counter() - t0
    # One 256-token prompt chunk whose queries all see a full window.
    pre = model.session(loops)
    pre.fill(3840, seed=1)
    ids = np.random.default_rng(0).integers(0, model.cfg["vocab_size"], 256)
    t1 = time.perf_counter()
    pre.feed(ids, 256)
    pre.logits()
    pre_s = time.perf_counter() - t1
    return {"decode_tok_s": done / dec_s, "decode_steps": done, "prefill_tok_s": 256 / pre_s, "cores": cores,
            "sample": f"{done} greedy decode steps at position 4096 (full window, R={loops}) from a seeded "
                      f"filled state; prefill: one 256-token chunk at positions 3840-4095"}


# ---------------------------------------------------------------------------
# The reference CUDA backend on the same GPU — baseline only
# ---------------------------------------------------------------------------

def ref_cuda_measure(cases, device: int) -> dict | None:
    """The reference's own kernels (kernels/slm.cu from source, JIT-compiled
    compute_60 PTX) under the C++ restatement of its host side, with its bench
    protocol (src/main.rs:200-223): prefill = feed + logits read, decode =
    logits read + host pick + step per token, host clock.

    cases: (name, model folder, prompt ids, loops, greedy, decode steps)."""
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    from oracle import ref_cuda as RC

    if not RC.available():
        return None
    backend = RC.Backend(device)
    out = {}
    models = {}
    for name, folder, prompt, loops, greedy, steps in cases:
        if folder not in models:
            models[folder] = RC.Model(backend, folder)
            # Warm-up, as the library's arm has: first launches and pool growth.
            w = models[folder].session(loops)
            w.feed(prompt[:512], 256)
            w.step(int(np.argmax(w.logits())))
            w.logits()
            w.close()
        se = models[folder].session(loops)
        t0 = time.perf_counter()
        se.feed(prompt, 256)
        logits = se.logits()
        pre_s = time.perf_counter() - t0
        st = [O.rng_new(0)]
        hist = [int(t) for t in prompt[-256:]]

        def pick(lg):
            if greedy:
                return int(np.argmax(lg))
            return O.pick(lg, np.array(hist[-256:], dtype=np.uint32), 0.8, 40, 1.0, 1.1, 256, st)

        tok = pick(logits)
        for _ in range(2):
            se.step(tok)
            tok = pick(se.logits())
        l0, s0 = backend.counts()
        t0 = time.perf_counter()
        for _ in range(steps):
            se.step(tok)
            tok = pick(se.logits())
            hist.append(tok)
        dec_s = time.perf_counter() - t0
        l1, s1 = backend.counts()
        out[name] = {"decode_tok_s": steps / dec_s, "prefill_tok_s": len(prompt) / pre_s, "decode_steps": steps,
                     "prompt": len(prompt), "launches_per_token": (l1 - l0) / steps,
                     "host_syncs_per_token": (s1 - s0) / steps,
                     "sampling": "greedy" if greedy else
                     "T=0.8 top-k 40 repeat-penalty 1.1 (window 256) seed 0, host pick"}
        se.close()
    for m in models.values():
        m.close()
    backend.close()
    return out


# ---------------------------------------------------------------------------
# Device timeline of the persistent decode step (--trace)
# ---------------------------------------------------------------------------

def phase_kinds(cfg: dict, loops: int, fused: bool = True, attn_o: bool | None = None) -> list[str]:
    """Phase names of the persistent step, in plan order (model.cpp build_plan).
    fused: each MLP is one phase ("mlp"); else gate/up ("up") and down.
    attn_o (default: fused): S and L blocks run o in their attention / GLA phase."""
    attn_o = fused if attn_o is None else attn_o
    mlp = ["mlp"] if fused else ["up", "down"]
    o = [] if attn_o else ["o"]
    names = {"S": ["S1", "attn"] + o + mlp, "L": ["L1", "gla"] + o + mlp, "G": ["G1", "gattn", "o"] + mlp}
    out = [n for k in cfg["prelude"] for n in names[k]]
    if cfg["core"]:
        out.append("inject")
        out += [n for _ in range(loops) for k in cfg["core"] for n in names[k]]
    out += [n for k in cfg["coda"] for n in names[k]]
    return out + ["logits"]


def trace_kinds(tr: np.ndarray, cfg: dict, loops: int) -> list[str] | None:
    """Phase names for a traced step of either plan shape (None if neither fits)."""
    for fused, attn_o in ((True, True), (True, False), (False, False)):
        kinds = phase_kinds(cfg, loops, fused, attn_o)
        if len(kinds) == tr.shape[0]:
            return kinds
    return None


def traced_step(se, greedy) -> np.ndarray:
    """Three traced persistent steps; the last one's timeline [phase][cta][8]."""
    se.set_trace(True)
    tok = int(se.sample(greedy))
    for _ in range(3):
        tok = int(se.decode(tok, 1, greedy)[0])
    se.set_trace(False)
    return se.trace().astype(np.int64)


def attention_phases(tr: np.ndarray, cfg: dict, loops: int) -> dict | None:
    """The persistent step's window-attention phases (attention and the o
    projection fused) at a full window: their K/V and o bytes over what each
    adds to the step (its last CTA arrival minus the previous phase's; the
    phases overlap, so first start to last arrival would count time that the
    previous phase's stragglers take)."""
    kinds = trace_kinds(tr, cfg, loops)
    if kinds is None:
        return None
    spans = [int(tr[p, :, 1].max() - tr[p - 1, :, 1].max()) for p in range(1, tr.shape[0]) if kinds[p] == "attn"]
    h, dh, d = cfg["n_heads"], cfg["d_model"] // cfg["n_heads"], cfg["d_model"]
    per = 2 * h * cfg["window"] * dh * 4 + d * d * 4
    return {"phases": len(spans), "bytes_per_phase": per, "us_per_phase": sum(spans) / len(spans) / 1000.0,
            "achieved": per * len(spans) / (sum(spans) * 1e-9) / 1e9}


def write_trace(tr: np.ndarray, cfg: dict, loops: int, path: str) -> None:
    """Per-phase sums of a traced step, grouped by phase kind, as a markdown
    table.  Step span: each phase's last CTA arrival minus the previous
    phase's (the first phase: minus the step's first start), i.e. what the
    phase adds to the step; phases overlap, since a CTA starts the next phase
    when its own part of this one is done.  Per CTA (medians over the CTAs,
    summed over the phases of the kind): duration from the CTA's start of the
    phase to its arrival, the input prologue (waiting for and building the
    input vector), work on its tiles, waits for tiles to land, and epilogues
    (output adds, the o tail of mixer phases).  globaltimer ticks are 32 ns
    to 1 µs depending on the GPU, so single values are coarse; the sums over
    148 CTAs' medians are not."""
    kinds = trace_kinds(tr, cfg, loops)
    if kinds is None:
        return
    t0 = tr[0, :, 0].min()
    st, en = tr[:, :, 0] - t0, tr[:, :, 1] - t0
    rows: dict = {}
    prev_end = 0.0
    for p in range(tr.shape[0]):
        r = rows.setdefault(kinds[p], [0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0])
        r[0] += 1
        r[1] += en[p].max() - prev_end
        prev_end = en[p].max()
        r[2] += float(np.median(tr[p, :, 1] - tr[p, :, 0]))
        r[3] += float(np.median(tr[p, :, 3]))
        r[4] += float(np.median(tr[p, :, 4]))
        r[5] += float(np.median(tr[p, :, 2]))
        r[6] += float(np.median(tr[p, :, 5]))
    lines = [f"Total step (trace run): {en[-1].max() / 1000:.1f} us over {tr.shape[0]} phases", "",
             "| phase kind | count | step span µs (sum) | per-CTA duration µs (median, sum) | input prologue µs"
             " (median, sum) | tile work µs (median, sum) | tile waits µs (median, sum) | epilogues µs (median, sum) |",
             "|---|---|---|---|---|---|---|---|"]
    for k, r in sorted(rows.items(), key=lambda kv: -kv[1][1]):
        lines.append(f"| {k} | {r[0]} | {r[1] / 1000:.1f} | {r[2] / 1000:.1f} | {r[3] / 1000:.1f} | "
                     f"{r[4] / 1000:.1f} | {r[5] / 1000:.1f} | {r[6] / 1000:.1f} |")
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_text("\n".join(lines) + "\n")


# ---------------------------------------------------------------------------
# The B200 arm
# ---------------------------------------------------------------------------

def queue_behind_sleep(torch, stream, ms: float = 3.0) -> None:
    """Holds `stream` in a device-side sleep of about `ms` (at the B200's
    1965 MHz maximum clock), so the launches the host issues next are all
    queued before the GPU reaches them: events recorded after the sleep time
    the kernels back to back, not the host's per-call overhead (a Python
    ctypes call per op costs more than the op's two short kernels)."""
    with torch.cuda.stream(stream):
        torch.cuda._sleep(int(ms * 1e-3 * 1.965e9))


def run_b200(args, rank: int, world: int, local: int) -> dict | None:
    import torch
    import torch.distributed as dist

    slm = load_pkg()
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.BASE
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if local == 0:
        folder = model_dir(cfg, 0)
    if world > 1:
        dist.barrier()
    folder = model_dir(cfg, 0)

    ctx = slm.Context(local)
    t_load = time.perf_counter()
    model = slm.Model(ctx, folder)
    load_s = time.perf_counter() - t_load  # file read, pinned upload, bf16x3 splits and layouts
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    V = cfg["vocab_size"]
    greedy = slm.Sampling()
    prompt = prompt_for(rank, V, args.prompt)

    def events():
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # Warm-up: load modules, capture the step graph once.
    w = model.session(args.loops)
    w.feed(prompt[:512])
    w.decode(w.sample(greedy), 8, greedy)
    w.close()

    se = model.session(args.loops)
    clocks = Clocks(local)
    with clocks:
        # Prefill (feed + logits read, src/main.rs:200-205).
        a, b = events()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        a.record(stream)
        se.feed(prompt, 256)
        logits = se.logits()
        b.record(stream)
        torch.cuda.synchronize(dev)
        prefill_host_s = time.perf_counter() - t0
        prefill_ms = a.elapsed_time(b)
        tok = int(np.argmax(logits))

        # Decode, device-resident ids.
        se.decode(tok, args.warmup, greedy)
        tok = int(se.sample(greedy))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = events()
        a.record(stream)
        out = se.decode(tok, args.steps, greedy)
        b.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        dec_ms = a.elapsed_time(b)

        # End to end through the per-token C ABI with host ids.
        tok = int(out[-1])
        for _ in range(min(args.warmup, 4)):
            se.step(tok)
            tok = se.sample(greedy)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            se.step(tok)
            tok = se.sample(greedy)
        e2e_s = time.perf_counter() - t0
        torch.cuda.synchronize(dev)

        # Dominant kernel: the m = 1 GEMV on a 32000 × 768 matrix (the tied
        # logits head, the largest decode weight); four copies rotate so each
        # launch streams its matrix from HBM, not L2.
        ops = slm.Ops(ctx)
        mats = [ops.upload(np.random.default_rng(9 + i).standard_normal(V * cfg["d_model"], dtype=np.float32))
                for i in range(4)]
        xv = ops.upload(np.ones(cfg["d_model"], dtype=np.float32))
        yv = ops.zeros(V)
        for i in range(8):
            ops.linear(yv, mats[i % 4], V, cfg["d_model"], xv, 1)
        reps = 40
        a, b = events()
        queue_behind_sleep(torch, stream)
        a.record(stream)
        for i in range(reps):
            ops.linear(yv, mats[i % 4], V, cfg["d_model"], xv, 1)
        b.record(stream)
        torch.cuda.synchronize(dev)
        gemv_us = a.elapsed_time(b) * 1000.0 / reps
        for mbuf in mats:
            mbuf.close()

        # Decode attention on its own (the m = 1 op, k_attn_split + combine):
        # one query per head over a full window of a 4352-slot ring; six
        # caches rotate (160 MB) so each call streams its K/V from HBM.
        H, dh = cfg["n_heads"], cfg["d_model"] // cfg["n_heads"]
        W, cap = cfg["window"], cfg["window"] + 256
        rng = np.random.default_rng(5)
        caches = [(ops.upload(rng.standard_normal(H * cap * dh, dtype=np.float32)),
                   ops.upload(rng.standard_normal(H * cap * dh, dtype=np.float32))) for _ in range(6)]
        qa, ya, sa = ops.upload(np.ones(H * dh, dtype=np.float32)), ops.zeros(H * dh), ops.zeros(1)

        def attend(i):
            ops.attend(ya, sa, qa, caches[i % 6][0], caches[i % 6][1], pos=cap + 100, m=1, reach=W, gap=0, cap=cap,
                       heads=H, key_heads=H, dh=dh, scale=1.0 / math.sqrt(dh))

        for i in range(6):
            attend(i)
        a, b = events()
        queue_behind_sleep(torch, stream)
        a.record(stream)
        for i in range(36):
            attend(i)
        b.record(stream)
        torch.cuda.synchronize(dev)
        attn_us = a.elapsed_time(b) * 1000.0 / 36

        # Prefill attention on its own (the tensor-core pass k_attn_tc and the
        # slice merge k_attn_combine64): a 256-query chunk at positions
        # 3840-4095 over the same rings, every query seeing all positions up to
        # its own; the six rings rotate, so each call streams its K/V from HBM.
        qp, yp = ops.upload(rng.standard_normal(256 * H * dh, dtype=np.float32)), ops.zeros(256 * H * dh)

        def attend_chunk(i):
            ops.attend(yp, sa, qp, caches[i % 6][0], caches[i % 6][1], pos=W - 256, m=256, reach=W, gap=0, cap=cap,
                       heads=H, key_heads=H, dh=dh, scale=1.0 / math.sqrt(dh))

        for i in range(6):
            attend_chunk(i)
        a, b = events()
        queue_behind_sleep(torch, stream)
        a.record(stream)
        for i in range(24):
            attend_chunk(i)
        b.record(stream)
        torch.cuda.synchronize(dev)
        pattn_us = a.elapsed_time(b) * 1000.0 / 24
        qp.close()
        yp.close()
        for kb, vb in caches:
            kb.close()
            vb.close()

    extra = {}
    legs = set(args.extras.split(",")) if args.extras else (set() if args.quick else {"R8", "R16", "C4", "C5", "BF16"})
    if "BF16" in legs:
        # The same decode with the persistent step streaming bf16 copies of
        # the weights (f32 arithmetic and caches): a separate line, never the
        # headline (logits differ by the weights' rounding).
        sb = model.session(args.loops)
        sb.set_bf16(True)
        sb.feed(prompt, 256)
        tb = int(np.argmax(sb.logits()))
        sb.decode(tb, args.warmup, greedy)
        tb = int(sb.sample(greedy))
        torch.cuda.synchronize(dev)
        a, b = events()
        a.record(stream)
        sb.decode(tb, args.steps, greedy)
        b.record(stream)
        torch.cuda.synchronize(dev)
        bf_ms = a.elapsed_time(b) / args.steps
        bf_bytes = decode_bytes(cfg, args.loops)
        bf_total = bf_bytes["total"] - bf_bytes["weights"] / 2
        extra["BF16"] = {"decode_tok_s": 1000.0 / bf_ms, "ms_per_step": bf_ms, "loops": args.loops,
                         "bytes_per_token": bf_total, "achieved_gbs": bf_total / (bf_ms / 1000.0) / 1e9,
                         "weights": "bf16 copies (round to nearest even), f32 arithmetic, caches and state",
                         "sampling": "greedy"}
        sb.close()
    if legs & {"R8", "R16"}:
        c3 = slm.Sampling(temperature=0.8, top_k=40, repeat_penalty=1.1, repeat_window=256)
        for loops in (8, 16):
            if f"R{loops}" not in legs:
                continue
            s2 = model.session(loops)
            torch.cuda.synchronize(dev)
            a, b = events()
            a.record(stream)
            s2.feed(prompt, 256)
            lg = s2.logits()
            b.record(stream)
            torch.cuda.synchronize(dev)
            pre_ms = a.elapsed_time(b)
            st = [slm.rng_seed(0)]
            hist = list(prompt[-256:])
            first = s2.sample(c3, hist, st)
            hist.append(first)
            s2.decode(first, 8, c3, hist, st)
            n2 = min(args.steps, 256)
            a, b = events()
            a.record(stream)
            s2.decode(first, n2, c3, hist, st)
            b.record(stream)
            torch.cuda.synchronize(dev)
            extra[f"R{loops}"] = {"decode_tok_s": n2 / (a.elapsed_time(b) / 1000.0),
                                  "prefill_tok_s": len(prompt) / (pre_ms / 1000.0), "decode_steps": n2,
                                  "prompt": len(prompt),
                                  "sampling": "T=0.8 top-k 40 repeat-penalty 1.1 (window 256) seed 0"}
            s2.close()
            # configs[2] as written: a 2048-id prompt, then 512 sampled steps
            # (the window fills up to 2560 positions).
            s3 = model.session(loops)
            p3 = prompt_for(rank, V, 2048)
            torch.cuda.synchronize(dev)
            a, b = events()
            a.record(stream)
            s3.feed(p3, 256)
            s3.logits()
            b.record(stream)
            torch.cuda.synchronize(dev)
            pre3 = a.elapsed_time(b)
            st = [slm.rng_seed(0)]
            hist = list(p3[-256:])
            first = s3.sample(c3, hist, st)
            hist.append(first)
            a, b = events()
            a.record(stream)
            s3.decode(first, 512, c3, hist, st)
            b.record(stream)
            torch.cuda.synchronize(dev)
            extra[f"R{loops}"]["configs2"] = {"decode_tok_s": 512 / (a.elapsed_time(b) / 1000.0),
                                              "prefill_tok_s": 2048 / (pre3 / 1000.0), "prompt": 2048,
                                              "decode_steps": 512}
            s3.close()

    if "C4" in legs:
        # configs[3] ("C4"): the G-layer variant (S | LS | SG, the fixture's
        # global options), 16384-id prompt, then 256 greedy decodes.
        gcfg = syn.GLOBAL
        gfolder = model_dir(gcfg, 0)
        gmodel = model.__class__(ctx, gfolder)
        gprompt = prompt_for(rank, V, 16384)
        # Warm-up, as the R = 4 arm has: first launches of this model's shapes.
        w3 = gmodel.session(args.loops)
        w3.feed(gprompt[:512], 256)
        w3.logits()
        w3.close()
        s3 = gmodel.session(args.loops)
        torch.cuda.synchronize(dev)
        a, b = events()
        a.record(stream)
        s3.feed(gprompt, 256)
        lg = s3.logits()
        b.record(stream)
        torch.cuda.synchronize(dev)
        pre_ms = a.elapsed_time(b)
        first = int(np.argmax(lg))
        s3.decode(first, 8, greedy)
        first = int(s3.sample(greedy))
        n3 = 256
        a, b = events()
        a.record(stream)
        s3.decode(first, n3, greedy)
        b.record(stream)
        torch.cuda.synchronize(dev)
        extra["C4"] = {"decode_tok_s": n3 / (a.elapsed_time(b) / 1000.0), "prefill_tok_s": 16384 / (pre_ms / 1000.0),
                       "decode_steps": n3, "prompt": 16384, "layout": "S|LS|SG", "loops": args.loops,
                       "decode_path": "persistent kernel" if s3.mega else "captured graph",
                       "sampling": "greedy"}
        s3.close()
        gmodel.close()

    if "C5" in legs:
        # configs[4] ("C5"): 64 independent sequences (2048-id prompts, seeds
        # 0..63) partitioned over the ranks, each rank's share decoded as one
        # batch (weights read once per step), 256 greedy steps; the total is
        # fixed, so this part scales strongly.
        n_seq = args.c5_sequences
        mine = c5_partition(n_seq, rank, world)
        sessions = []
        firsts = []
        for q in mine:
            sq = model.session(args.loops)
            sq.feed(prompt_for(q, V, 2048), 256)
            firsts.append(int(np.argmax(sq.logits())))
            sessions.append(sq)
        bt = slm.Batch(sessions)
        warm = bt.decode(firsts, 4)
        nxt = warm[-1]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        a, b = events()
        a.record(stream)
        bt.decode(nxt, 256)
        b.record(stream)
        torch.cuda.synchronize(dev)
        c5_ms = a.elapsed_time(b)
        c5_ms = max_over_ranks([c5_ms], dist, dev)[0]
        if args.profile_c5:
            # Two more batched steps, after the timed region, inside a profiler
            # range (for `ncu --profile-from-start off`).
            torch.cuda.cudart().cudaProfilerStart()
            bt.decode(nxt, 2)
            torch.cuda.synchronize(dev)
            torch.cuda.cudart().cudaProfilerStop()
        extra["C5"] = {"value": n_seq * 256 / (c5_ms / 1000.0), "unit": "tok/s (all ranks)", "sequences": n_seq,
                       "per_rank": len(mine), "prompt": 2048, "decode_steps": 256, "loops": args.loops,
                       "scaling": "strong", "ms_per_step": c5_ms / 256, "sampling": "greedy",
                       "path": "slm_batch_decode (one graph-replayed step for the rank's sequences)"}
        bt.close()
        for sq in sessions:
            sq.close()

    attn_phase = None
    if se.mega:
        tr = traced_step(se, greedy)
        attn_phase = attention_phases(tr, cfg, args.loops)
        if args.trace:
            write_trace(tr, cfg, args.loops, args.trace)

    step_kernels = se.step_kernels
    mega = se.mega
    res = {"dec_ms": dec_ms, "e2e_s": e2e_s, "prefill_ms": prefill_ms, "prefill_host_s": prefill_host_s,
           "gemv_us": gemv_us, "attn_us": attn_us, "pattn_us": pattn_us, "attn_phase": attn_phase, "clocks": clocks.summary(), "extra": extra, "step_kernels": step_kernels, "mega": mega, "load_s": load_s,
           "device": ctx.name, "state_bytes": se.state_bytes()}
    res["dec_ms"], res["e2e_s"], res["prefill_ms"] = max_over_ranks([dec_ms, e2e_s, prefill_ms], dist, dev)
    se.close()
    model.close()
    ctx.close()
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--loops", type=int, default=4)
    ap.add_argument("--prompt", type=int, default=4096)
    ap.add_argument("--quick", action="store_true", help="skip the extra legs (R=8/16, C4, C5)")
    ap.add_argument("--profile-c5", action="store_true", help="bracket two C5 batched steps (after the timed "
                    "region) with cudaProfilerStart/Stop, for ncu --profile-from-start off")
    ap.add_argument("--c5-sequences", type=int, default=64, help="sequences of the C5 leg (configs[4]: 64; "
                    "64/N on one GPU reproduces one rank's share at N GPUs)")
    ap.add_argument("--extras", default="", help="comma list of extra legs to run (R8,R16,C4,C5); default all, "
                    "none with --quick")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-ref-cuda", action="store_true", help="skip the reference CUDA baseline")
    ap.add_argument("--trace", default="", help="write the persistent step's phase timeline (markdown) here")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    load_pkg()
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.BASE
    byts = decode_bytes(cfg, args.loops)
    workload = (f"C2 decode: 86M-class S|LS|S (d768, 12x64, FFN 3072, V32000, window 4096) fp32, R={args.loops}, "
                f"{args.prompt}-id prompt in 256-chunks then greedy decode at a full window")
    config = {"workload": workload, "model": "86M-class looped hybrid (synthetic)", "loops": args.loops,
              "prompt": args.prompt, "global_batch": world, "seq_len": args.prompt,
              "parallelism": f"independent sequences, 1 per GPU x{world}", "l2": MODEL_BYTES_NOTE}

    if args.impl == "reference":
        if rank != 0:
            return
        folder = model_dir(cfg, 0)
        c = cpu_measure(folder, args.loops, args.steps, args.warmup, budget_s=120.0)
        line = {"metric": f"decode tok/s, R={args.loops}, 4096 ctx full", "value": c["decode_tok_s"],
                "unit": "tok/s", "n_gpus": world, "steps": c["decode_steps"], "warmup": args.warmup,
                "ms_per_step": 1000.0 / c["decode_tok_s"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic (N(0,0.02) init, seed 0)",
                "config": config, "impl": "reference",
                "cpu_baseline": {"value": c["decode_tok_s"], "unit": "tok/s", "cores": c["cores"], "kind": "port",
                                 "sample": c["sample"]},
                "e2e": {"value": c["decode_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "prefill": {"value": c["prefill_tok_s"], "unit": "tok/s"},
                "note": "the reference (Rust) has no toolchain here; this arm runs the C++ restatement of its "
                        "CPU backend (oracle/slm_oracle.cpp) on all host cores"}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    res = run_b200(args, rank, world, local)
    cpu = refc = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_measure(model_dir(cfg, 0), args.loops, 64, 2, budget_s=20.0)
    if rank == 0 and world == 1 and not args.no_ref_cuda:
        prompt = prompt_for(0, cfg["vocab_size"], args.prompt)
        cases = [(f"R{args.loops}", model_dir(cfg, 0), prompt, args.loops, True, 32)]
        if not args.quick:
            cases += [(f"R{r}", model_dir(cfg, 0), prompt, r, False, 32) for r in (8, 16)]
            cases.append(("C4", model_dir(syn.GLOBAL, 0), prompt_for(0, cfg["vocab_size"], 16384), args.loops,
                          True, 16))
        refc = ref_cuda_measure(cases, local)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = peaks.get("hbm_gbs") or 6650.0
    peak_src = "measured" if peaks.get("hbm_gbs") else "fallback"
    K = args.steps
    value = world * K / (res["dec_ms"] / 1000.0)
    gemv_bytes = (cfg["vocab_size"] * cfg["d_model"] + cfg["d_model"] + cfg["vocab_size"]) * 4
    gemv_gbs = gemv_bytes / (res["gemv_us"] * 1e-6) / 1e9
    step_gbs = byts["total"] / (res["dec_ms"] / 1000.0 / K) / 1e9
    H, dh = cfg["n_heads"], cfg["d_model"] // cfg["n_heads"]
    attn_gbs = (2 * H * cfg["window"] * dh * 4 + 2 * H * dh * 4) / (res["attn_us"] * 1e-6) / 1e9
    pre_flops = prefill_flops(cfg, args.loops, args.prompt)
    line = {
        "metric": f"decode tok/s, R={args.loops}, 4096 ctx full", "value": value, "unit": "tok/s",
        "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": res["dec_ms"] / K,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (N(0,0.02) random init, uniform random ids, seed 0 / rank)", "config": config,
        "e2e": {"value": world * K / res["e2e_s"], "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 8,
                "how": "per token slm_step(host id) + slm_sample -> host id, host clock; the id goes in the "
                       "persistent kernel's launch parameters, the picked id and the error word come back in "
                       "one 8-byte copy"},
        "prefill": {"value": world * args.prompt / (res["prefill_ms"] / 1000.0), "unit": "tok/s",
                    "e2e_value": world * args.prompt / res["prefill_host_s"], "prompt": args.prompt,
                    "tflops_fp32": pre_flops / (res["prefill_ms"] / 1000.0) / 1e12,
                    "flops_per_token": pre_flops / args.prompt},
        # The m = 1 step is one persistent kernel (k_decode_mega), so its
        # average launch duration is the decode time per token (CUDA events
        # over the K launches; inter-launch gaps included).
        "roofline": {"bound": "hbm", "kernel": "k_decode_mega (one m=1 token step, R=%d)" % args.loops,
                     "achieved": step_gbs, "peak": hbm, "unit": "GB/s", "frac": step_gbs / hbm,
                     "bytes_per_launch": byts["total"], "traffic": MEGA_TRAFFIC.get(args.loops),
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one R=4 launch "
                                        "(profiles/k_decode_mega_R4.md)" if args.loops in MEGA_TRAFFIC else
                                        "not captured for this loop count"),
                     "peak_source": peak_src,
                     "gemv": {"kernel": "k_gemv<1,STORE> (32000x768 fp32, m=1)", "achieved": gemv_gbs,
                              "frac": gemv_gbs / hbm, "how": "40 launches queued behind a device sleep, CUDA "
                              "events around them"},
                     "attention": {"kernel": "k_attn_split (m=1, 12 heads x 4096 positions of a 4352-slot ring, "
                                             "K and V from HBM; the last slice of each head merges)",
                                   "achieved": attn_gbs, "frac": attn_gbs / hbm, "how": "36 calls (one launch "
                                   "each) queued behind a device sleep, CUDA events around them"}},
        "clocks": res["clocks"],
        # Greedy persistent decode runs up to 4096 steps per launch.
        "gpu_launches": (math.ceil(K / int(os.environ.get("SLM_MEGA_STEPS", "4096"))) if res["mega"]
                         else K * (res["step_kernels"] + 1)),
        "extra": res["extra"],
        "device": res["device"],
        "state_mib": res["state_bytes"] / 2**20,
        "model_load": {"seconds": res["load_s"],
                       "weights_mb": (model_dir(cfg, 0) / "model.safetensors").stat().st_size / 1e6,
                       "how": "slm_model_load: safetensors read, f32 upload through pinned double buffers, "
                              "derived layouts (bf16x3 parts, transposed down, per-head o) on the device"},
    }
    if res.get("pattn_us"):
        # Algorithmic work of the chunk: QKᵀ and P·V over every visible
        # position, 2 flops per multiply-add; the pass runs each fp32 product
        # as three bf16 products, so its tensor work is three times that.
        span = sum(p + 1 for p in range(cfg["window"] - 256, cfg["window"]))
        fl = 4.0 * span * dh * H
        bf16_peak = peaks.get("bf16_tflops") or 1590.0
        ach = 3 * fl / (res["pattn_us"] * 1e-6) / 1e12
        line["roofline"]["prefill_attention"] = {
            "kernel": "k_attn_tc + k_attn_combine64 (256 queries at positions 3840-4095, 12 heads, each over all "
                      "positions up to its own: 6 slices x 2 query tiles x 12 heads)",
            "bound": "tensor", "achieved": ach, "peak": bf16_peak, "unit": "TFLOP/s (bf16 products)",
            "frac": ach / bf16_peak, "fp32_tflops": fl / (res["pattn_us"] * 1e-6) / 1e12,
            "us_per_call": res["pattn_us"], "flops_fp32_per_call": fl,
            "peak_source": "measured" if peaks.get("bf16_tflops") else "fallback",
            "how": "24 calls (two launches each) queued behind a device sleep, CUDA events around them; six "
                   "K/V rings rotate (160 MB)"}
    if res.get("attn_phase"):
        ap = res["attn_phase"]
        line["roofline"]["attention_in_step"] = {
            "kernel": "k_decode_mega window-attention + o phases (12 heads x 4096 positions, 12 splits per head, "
                      "then the 768x768 o projection)",
            "achieved": ap["achieved"], "frac": ap["achieved"] / hbm, "us_per_phase": ap["us_per_phase"],
            "bytes_per_phase": ap["bytes_per_phase"], "how": "globaltimer trace of one step (each attention phase's "
            "last CTA arrival minus the previous phase's)"}
    if cpu:
        line["cpu_baseline"] = {"value": cpu["decode_tok_s"], "unit": "tok/s", "cores": cpu["cores"], "kind": "port",
                                "sample": cpu["sample"], "prefill_tok_s": cpu["prefill_tok_s"]}
    if refc:
        line["ref_cuda_baseline"] = {
            "value": refc[f"R{args.loops}"]["decode_tok_s"], "unit": "tok/s", "same_gpu": True,
            "what": "the reference's kernels/slm.cu built from source (compute_60 PTX, JIT) under a C++ "
                    "restatement of src/cuda.rs + src/model.rs, its own bench protocol (host clock, logits "
                    "read back and host pick every token)",
            "cases": refc}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

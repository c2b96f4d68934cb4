"""Benchmark: CCPE+WCA reuse-prefill tok/s (and decode tok/s) on B200.

Workload (kernel microbenchmark config): per GPU 8 requests, 32 query / 8 KV
heads x 128, 4096 tokens in 8 chunks of 512 (chunk 3 recomputed, the rest
reused), CoPE npos 64, paged KV blocks of 16 with shuffled physical ids, WCA
15 % with profile K = K + N(0, 0.05).  Synthetic seeded data.

One step = one reuse-prefill layer of every request: SLIDE baseline write,
WCA calibration scoring + top-k, fused WCA blend+scatter of the active rows,
WCA commit (cosine gate + promotion), CCPE attention of the active rows over
all 4096 keys through the paged slots.  ``value`` = prompt tokens / s with
inputs resident in HBM; ``e2e`` repeats the step with the per-layer snapshot
and the fresh rows copied from pinned host memory and the outputs copied back.

``--impl reference`` times the reference algorithm on the host cores (the
numpy restatement of the reference's CPU path) on whole requests of the same
workload (every active row; a step is one eighth of a request).
Multi-GPU (torchrun): requests are sharded by rank, no data-path collective.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "CCPE+WCA reuse-prefill tok/s"
WORKLOAD = "c2-kernel-microbench: B=8/GPU, Hq=32, Hkv=8, D=128, S=4096 (8x512), npos=64, block=16, WCA=15%"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--requests", type=int, default=8)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batched-attention", action="store_true",
                    help="with --per-request-streams: one attention launch for all requests "
                         "after their WCA / SLIDE chains")
    ap.add_argument("--no-c3", action="store_true",
                    help="skip the RAG slice with shared chunks (run at one GPU by default)")
    ap.add_argument("--no-c4", action="store_true",
                    help="skip the multi-session chat slice (run at one GPU by default)")
    ap.add_argument("--c5", action="store_true",
                    help="also run the C5 tensor-parallel slice at one GPU (it runs by "
                         "default whenever there are several ranks)")
    ap.add_argument("--per-request-streams", action="store_true",
                    help="one launch per request and stage, each request on its own stream "
                         "(default: every stage of the step as one launch for all requests, "
                         "seven launches per step; e2e always uses the per-request streams)")
    args = ap.parse_args()
    args.batched = not args.per_request_streams
    return args


def peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ----------------------------------------------------------- accounting
# DRAM bytes of one batched prefill launch of the C2 step (8 requests), from
# an ncu capture of that launch (dram__bytes_read.sum + dram__bytes_write.sum);
# None until captured for the current kernel
# dram__bytes_read.sum + dram__bytes_write.sum of one batched C2 attention
# launch, from the ncu --set full capture summarised in
# profiles/cope_prefill_sm100_batch_c2_step.md (362.21 MB + 50.31 MB)
PREFILL_DRAM_BYTES_PER_LAUNCH = 412519168


def attention_flops(work, visible_only: bool = False) -> float:
    """Algorithmic FLOPs of the attention launches of one step.

    QK over every causal cell, PV over every visible cell (association
    policy), plus the q.E table.  Counting QK over every causal cell follows
    the reference's computation, whose gates count all causal keys.  The
    kernel skips the key tiles whose cells no row of a CTA sees and whose
    gates feed no seen key's count, so it issues less than this.  With
    `visible_only`, QK and PV count the visible cells only: the lower bound
    that any implementation must compute.
    """
    c = work.cfg
    total = 0.0
    for r in work.requests:
        qpos = r.active.cpu().numpy()
        causal = (qpos + 1).astype(np.float64)
        sel = r.q_sel.cpu().numpy().astype(bool)
        fixed = r.reused.cpu().numpy()
        dyn_prefix = np.cumsum(~fixed)  # dynamic keys with position <= p
        visible = np.where(sel, dyn_prefix[qpos] + 1, causal)
        qk_cells = visible.sum() if visible_only else causal.sum()
        total += 2 * c.head_dim * c.q_heads * (qk_cells + visible.sum())
        total += 2 * len(qpos) * c.q_heads * c.npos * c.head_dim
    return total


def hot_bytes(work) -> dict:
    c = work.cfg
    rec = c.kv_heads * c.head_dim * 2  # bytes of K (or V) of one token
    out = {}
    n = c.seq
    a = sum(r.a for r in work.requests) / len(work.requests)
    out["slide_scatter"] = 2 * 2 * n * rec  # read dense K,V + write paged K,V
    out["slide_gather"] = 2 * 2 * n * rec  # read paged K,V + write dense K,V
    out["slide_relocate"] = 2 * 2 * n * rec  # read and write paged K,V
    out["wca_initialize"] = 2 * n * rec  # read cached K + calib K
    out["wca_update"] = 3 * 2 * a * rec  # old + fresh + fused (K and V)
    out["decode_attention"] = (n + 1) * 2 * rec + c.q_heads * c.head_dim * 2 + (n + 1) * 8
    return out


def hbm_report(work, kernel_ms: dict, dec_ms: float, peak_gbs: float) -> dict:
    """Per HBM-bound kernel: algorithmic bytes of one launch per request x the
    requests, over the CUDA-event time of those launches back to back."""
    hb = hot_bytes(work)
    n = len(work.requests)
    out = {}
    for name, ms in kernel_ms.items():
        if name in hb:
            gbs = hb[name] * n / (ms * 1e-3) / 1e9
            out[name] = {"us_per_request": ms * 1e3 / n, "gbs": gbs, "frac": gbs / peak_gbs}
        else:  # the top-k selections: latency bound, no byte roofline
            out[name] = {"us_per_request": ms * 1e3 / n}
    gbs = hb["decode_attention"] * n / (dec_ms * 1e-3) / 1e9  # scatter of the new rows included
    out["decode_step"] = {"us": dec_ms * 1e3, "gbs": gbs, "frac": gbs / peak_gbs}
    out["peak_gbs"] = peak_gbs
    return out


# --------------------------------------------------------------- clocks
class Clocks:
    """SM clock, its maximum and the active clock-event (throttle) reasons,
    sampled about every millisecond from a background thread through NVML --
    the counters `nvidia-smi --query-gpu=clocks.sm,clocks_event_reasons.*`
    prints -- so that even a timed region of a few milliseconds has samples.
    `mark()` opens and closes the window of the timed steps."""

    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
        self.samples: list[tuple[float, float, int]] = []
        self.window: list[float] = []
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            try:  # the NVML device of this CUDA ordinal, by UUID
                uuid = str(torch.cuda.get_device_properties(device).uuid)
                self.h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nv = None
            return
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def _loop(self) -> None:
        nv, h = self.nv, self.h
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((time.perf_counter(), sm, rs))
            except Exception:
                pass
            time.sleep(0.001)

    def mark(self) -> None:
        self.window.append(time.perf_counter())

    def stop(self) -> dict:
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"],
                    "samples": 0}
        self._stop.set()
        self.thread.join(2)
        t0, t1 = (self.window + [0.0, float("inf")])[:2] if len(self.window) >= 2 else (0.0, float("inf"))
        inside = [x for x in self.samples if t0 <= x[0] <= t1]
        use = inside if inside else self.samples
        reasons = sorted({name for _, _, rs in use for name, bit in self.REASONS.items()
                          if rs & bit})
        return {"sm_mhz": statistics.median(x[1] for x in use) if use else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(use), "samples_in_timed_steps": len(inside),
                "source": "nvml, 1 ms"}


# ------------------------------------------------------------- CPU legs
class CpuRequest:
    """The reference algorithm for one request on the host (the numpy
    restatement of the reference's CPU path), split into SLICES equal steps:
    slice 0 runs the SLIDE baseline write, WCA initialize + select + update,
    the write-back of the fused rows and the logical gather; slice s then runs
    the CCPE attention of active rows s, s + SLICES, ...  The SLICES slices
    together are one whole request: every active row, nothing extrapolated."""

    SLICES = 8

    def __init__(self, work, b: int, threads: int):
        r = work.requests[b]
        c = work.cfg
        f32 = lambda t: t.float().cpu().numpy()  # noqa: E731
        self.cached_k, self.cached_v = f32(r.cached_k), f32(r.cached_v)
        self.calib_k = f32(r.calib_k)
        self.q_all, self.fresh_k, self.fresh_v = f32(r.q_all), f32(r.fresh_k), f32(r.fresh_v)
        self.cache_shape = (work.cache.shape[0], c.kv_heads, c.block, 2 * c.head_dim)
        self.slots = r.slots.cpu().numpy()
        self.E = work.E.float().cpu().numpy()
        self.key_chunk = r.key_chunk.cpu().numpy()
        self.offsets = r.offsets.cpu().numpy()
        self.fixed = r.fixed.cpu().numpy()
        self.reused, self.mandatory = r.reused.cpu().numpy(), r.mandatory.cpu().numpy()
        self.fraction = c.fraction
        self.tokens = c.seq
        self.threads = threads

    def layer_state(self) -> None:
        from oracle import slide as oslide
        from oracle import wca as owca

        cache = np.zeros(self.cache_shape, np.float32)
        oslide.scatter(cache, None, None, self.slots, self.cached_k, self.cached_v)
        st = owca.OracleWCA(correction_fraction=self.fraction).initialize(
            self.cached_k, self.calib_k, self.reused, self.mandatory)
        self.active = st.active
        self.sel_prev = np.nonzero(st.selected & ~self.mandatory)[0]
        upd = st.update(2, self.cached_k, self.cached_v, self.fresh_k[self.active],
                        self.fresh_v[self.active])
        oslide.scatter(cache, None, None, self.slots[self.active],
                       upd["fused_k"].astype(np.float32), upd["fused_v"].astype(np.float32))
        self.k, self.v = oslide.gather(cache, None, None, self.slots)

    def attention(self, rows: np.ndarray) -> None:
        from oracle import cope as ocope

        active = self.active

        def part(idx):
            return ocope.cope_attention(
                self.q_all[active[idx]], self.k, self.v, self.E, active[idx],
                visibility_fn=lambda a_, b_: ocope.association_mask(a_, b_, self.fixed,
                                                                    self.sel_prev),
                chunk_reset=(self.key_chunk, self.offsets[:, active[idx]]), chunk=16)

        groups = [g for g in np.array_split(rows, max(1, self.threads)) if len(g)]
        with ThreadPoolExecutor(max_workers=self.threads) as pool:
            list(pool.map(part, groups))

    def step(self, s: int) -> float:
        """Slice s % SLICES of the request; returns its seconds."""
        t0 = time.perf_counter()
        k = s % self.SLICES
        if k == 0:
            self.layer_state()
        self.attention(np.arange(k, len(self.active), self.SLICES))
        return time.perf_counter() - t0

    def describe(self, requests: int) -> str:
        return (f"{requests} whole request(s) of the workload (request 0, {self.tokens} tokens: "
                f"SLIDE write, WCA initialize/select/update, gather, CCPE attention of all "
                f"{len(self.active)} active rows), each timed as {self.SLICES} slices; "
                f"nothing extrapolated; {self.threads} host threads")


def cpu_requests(work, requests: int, threads: int):
    """Seconds per request of the reference algorithm over `requests` whole
    requests, and the sample description."""
    cpu = CpuRequest(work, 0, threads)
    total = sum(cpu.step(s) for s in range(requests * CpuRequest.SLICES))
    return total / requests, cpu.describe(requests)


def run_reference(args):
    """--impl reference: the reference algorithm on host cores (numpy port).
    A step is one slice (1/8) of a whole request; the timed steps are rounded
    up to whole requests, so at least one request is timed unextrapolated."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    from cacheslide_b200.reuse import SyntheticWorkload, WorkloadConfig

    threads = os.cpu_count() or 1
    cfg = WorkloadConfig(requests=1, seq=args.seq)
    # inputs are built on the host; nothing of this package runs on this arm
    work = SyntheticWorkload(cfg, torch.device("cpu"))
    cpu = CpuRequest(work, 0, threads)
    cpu.layer_state()  # warm-up: the request's WCA / SLIDE part (no attention)
    slices = CpuRequest.SLICES
    requests = max(1, -(-args.steps // slices))
    times = [cpu.step(s) for s in range(requests * slices)]
    per_req = sum(times) / requests
    value = cfg.seq / per_req
    desc = cpu.describe(requests)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": len(times), "warmup": 1,
        "ms_per_step": statistics.mean(times) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": desc, "sample_fraction": 1.0,
                   "per": "one host process (rank 0), whatever the number of GPUs"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ C5 slice
def c5_slice(args, dev, rank: int, world: int) -> dict:
    """The C5 layout (Llama-3-70B, 8 KV / 64 query heads split over the
    ranks, 8 requests x 64K tokens in 32 chunks of 2K, WCA 10 %, npos 128):
    one reuse-prefill layer with its collectives -- the WCA row-sum
    all-reduces and the o_proj all-reduce of [active rows, 8192] bf16 --
    timed per stage on the device, max over ranks."""
    import torch
    import torch.distributed as dist

    from cacheslide_b200.tp_step import ShardedReuseStep, TPWorkloadConfig

    cfg = TPWorkloadConfig()
    step = ShardedReuseStep(cfg, dev, None, rank, world)
    stream = torch.cuda.current_stream(dev)
    steps = max(1, min(args.steps, 5))
    for _ in range(2):
        step.run(stream)
    torch.cuda.synchronize(dev)
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    for i in range(steps):
        step.run(stream, marks[i])
    torch.cuda.synchronize(dev)
    step.check_status()
    names = ["slide_scatter", "wca_sharded", "attention", "o_proj_gemm", "o_proj_all_reduce"]
    per = [[m[j].elapsed_time(m[j + 1]) for j in range(5)] + [m[0].elapsed_time(m[5])]
           for m in marks]
    vals = torch.tensor([statistics.mean(x[j] for x in per) for j in range(6)],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms = vals.tolist()
    flops = step.attention_flops()
    ar_bytes = step.proj.numel() * step.proj.element_size()
    out = {
        "workload": "c5-llama70b-tp: 8 requests x 64K (32 x 2K chunks), Hq/Hkv 64/8 split over "
                    f"{world} rank(s) ({step.hq}/{step.hkv} per GPU), D=128, npos=128, WCA 10%",
        "ms_per_step": ms[5],
        "value": cfg.requests * cfg.seq / (ms[5] / 1e3),
        "unit": "tok/s (per TP group)",
        "stage_ms": dict(zip(names, ms[:5])),
        "collective_share": (ms[4] + 0.0) / ms[5],
        "attention_tflops_per_gpu": flops / (ms[2] / 1e3) / 1e12,
        "o_proj_all_reduce": {"bytes": ar_bytes, "ms": ms[4],
                              "bus_gbs": (2 * (world - 1) / world * ar_bytes / (ms[4] / 1e3) / 1e9
                                          if world > 1 else None)},
        "active_rows": sum(r.a for r in step.requests),
        "steps": steps,
        "note": "WCA stage includes its row-sum all-reduces and status agreements (host "
                "synchronising, as ShardedWCAState is); max over ranks per stage",
    }
    del step
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------ selective QKV layer
def qkv_layer(args, work, dev) -> dict:
    """The selective layer loop's QKV projection for the step's active rows
    (the 8 requests' ~1051 rows each, Mistral-7B projection 4096 -> 6144 with
    a rank-16 LoRA delta): rows gathered from the previous layer's output (a
    third of them) or the layer snapshot, one tensor-core launch; TFLOP/s
    against the measured bf16 peak."""
    import torch

    from cacheslide_b200.layer import SelectiveQKV

    g = torch.Generator(device=dev).manual_seed(11)
    hidden, n_out, rank = 4096, 6144, 16
    rows = sum(r.a for r in work.requests)
    n = rows * 3  # a prompt frame of which the active rows are a third
    active = torch.sort(torch.randperm(n, generator=g, device=dev)[:rows]).values
    previous = active[torch.randperm(rows, generator=g, device=dev)[: rows // 3]].sort().values
    fixed = torch.arange(n, device=dev)
    bf = torch.bfloat16
    prev_h = torch.randn(previous.numel(), hidden, generator=g, device=dev).to(bf)
    snap_h = torch.randn(n, hidden, generator=g, device=dev).to(bf)
    w = (torch.randn(n_out, hidden, generator=g, device=dev) / 64).to(bf)
    la = (torch.randn(rank, hidden, generator=g, device=dev) / 64).to(bf)
    lb = (torch.randn(n_out, rank, generator=g, device=dev) / 4).to(bf)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    layer = SelectiveQKV(prev_h, previous, snap_h, fixed, active, n, w, la, lb)
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        layer.run(stream.cuda_stream)
    layer.check()
    steps = max(1, min(args.steps, 10))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for i in range(steps):
        flush.fill_(i & 0xFF)
        ev[i][0].record(stream)
        layer.run(stream.cuda_stream)
        ev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    layer.check()
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    flops = 2.0 * rows * hidden * (n_out + rank) + 2.0 * rows * rank * n_out
    pk, kind = peaks()
    tf = flops / (ms / 1e3) / 1e12
    return {"rows": rows, "shape": f"{hidden} -> {n_out}, LoRA rank {rank}", "ms": ms,
            "tflops": tf, "frac": tf / float(pk.get("bf16_tflops", 1590.0)),
            "peak_kind": kind, "launches_timed": steps}


# ------------------------------------------------------------ C3 / C4 slices
def _turns(step, args, dev, decode_tokens: int) -> tuple[float, float, int]:
    """Mean device ms of the prefill and of the decode of a turn step (after
    two warm-up turns, L2 flushed before each), and the turns timed."""
    import torch

    stream = torch.cuda.current_stream(dev)
    s = stream.cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(2):
        step.prefill(s)
        step.decode(s)
    turns = max(1, min(args.steps, 5))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(turns)]
    torch.cuda.synchronize(dev)
    for i in range(turns):
        flush.fill_(i & 0xFF)
        ev[i][0].record(stream)
        step.prefill(s)
        ev[i][1].record(stream)
        step.decode(s)
        ev[i][2].record(stream)
    torch.cuda.synchronize(dev)
    step.check_status()
    pre = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    dec = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    return pre, dec, turns


def c3_slice(args, dev) -> dict:
    """The RAG slice (C3 shapes: Mistral-7B heads, 64 requests x 10 chunks of
    512 drawn Zipf(1.1) from a pool of 40 shared chunks + a 64-token
    question, WCA 15 %, 32 decode tokens)."""
    import torch

    from cacheslide_b200.rag import RagConfig, RagStep

    cfg = RagConfig()
    step = RagStep(cfg, dev)
    pre, dec, turns = _turns(step, args, dev, cfg.decode_tokens)
    out = {
        "workload": "c3-rag: 64 requests x 10 chunks of 512 (Zipf 1.1 over a pool of 40 "
                    "chunks resident once) + 64-token question, Hq=32, Hkv=8, D=128, npos=64, "
                    "WCA 15%, copy-on-write relocation of the selected chunk rows, 32 decoded",
        "prompt_tokens": step.prompt_tokens(),
        "shared_chunk_reads": step.shared_fraction(),
        "relocated_rows": sum(x.reloc_src.numel() for x in step.sessions),
        "prefill_ms": pre,
        "prefill_tok_s": step.prompt_tokens() / (pre / 1e3),
        "decode_ms_per_token": dec / cfg.decode_tokens,
        "decode_tok_s": cfg.requests * cfg.decode_tokens / (dec / 1e3),
        "batches_timed": turns,
    }
    del step
    torch.cuda.empty_cache()
    return out


def chained_slice(args, dev, layers: int = 8) -> dict:
    """Layers 2..L of one C2-shaped request, each on the rows the previous
    layer's WCA commit chose, with the row count left on the device (no host
    read between layers), against the same layers with the count read back
    to the host before each, the reference runtime's order (runtime.py:410)."""
    import torch

    from cacheslide_b200.chain import ChainedLayers
    from cacheslide_b200.reuse import ReuseStep, SyntheticWorkload, WorkloadConfig

    cfg = WorkloadConfig(requests=1, seq=args.seq, seed=77)
    work = SyntheticWorkload(cfg, dev)
    step = ReuseStep(work, batched=True)
    step.run()  # layer 1
    chain = ChainedLayers(step, layers=layers)
    out = {"workload": f"c2-shaped request, layers 2-{layers} on the previous commit's rows "
                       f"(WCA update + CCPE attention + commit per layer, 15%)",
           "layers_timed": layers - 1}
    for device in (True, False):
        times = []
        for rep in range(4):
            torch.cuda.synchronize(dev)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            t0 = time.perf_counter()
            e0.record()
            chain.run(device=device)
            e1.record()
            torch.cuda.synchronize(dev)
            wall = (time.perf_counter() - t0) * 1e3
            if rep > 0:  # the first pass is a warm-up
                times.append((e0.elapsed_time(e1), wall))
        step.check_status()
        key = "device_count" if device else "host_count"
        out[key] = {"ms_per_layer": sum(t[0] for t in times) / len(times) / (layers - 1),
                    "wall_ms_per_layer": sum(t[1] for t in times) / len(times) / (layers - 1),
                    "host_reads_per_layer": 0 if device else 1}
    del chain, step, work
    torch.cuda.empty_cache()
    return out


def c4_slice(args, dev) -> dict:
    """The multi-session chat slice (C4): 32 sessions at turn 8 of
    conversations adding 256-1024 tokens a turn plus 128 decoded tokens;
    a turn = WCA + SLIDE relocation of the selected history rows + blend +
    attention of the active rows, then 128 batched decode steps."""
    import torch

    from cacheslide_b200.chat import ChatConfig, ChatTurnStep

    cfg = ChatConfig()
    step = ChatTurnStep(cfg, dev)
    pre, dec, turns = _turns(step, args, dev, cfg.decode_tokens)
    reloc_rows = sum(x.reloc_src.numel() for x in step.sessions)
    out = {
        "workload": "c4-multi-session-chat: 32 sessions at turn 8 (+256-1024 tokens a turn, "
                    "128 decoded), Hq=32, Hkv=8, D=128, npos=64, WCA 15%, SLIDE relocation of "
                    "the selected history rows every turn",
        "prompt_tokens": step.prompt_tokens(),
        "new_tokens": step.new_tokens(),
        "relocated_rows": reloc_rows,
        "prefill_ms": pre,
        "prefill_tok_s": step.prompt_tokens() / (pre / 1e3),
        "decode_ms_per_token": dec / cfg.decode_tokens,
        "decode_tok_s": cfg.sessions * cfg.decode_tokens / (dec / 1e3),
        "turn_ms": pre + dec,
        "turns_timed": turns,
    }
    del step
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------ our arm
def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from cacheslide_b200 import _native as N
    from cacheslide_b200.reuse import ReuseStep, SyntheticWorkload, WorkloadConfig

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    cfg = WorkloadConfig(requests=args.requests, seq=args.seq, seed=1000 + rank)
    work = SyntheticWorkload(cfg, dev)
    step = ReuseStep(work, batched_attention=args.batched_attention, batched=args.batched)
    # a dedicated stream, current for every torch op below: on the legacy
    # default stream, events around the 8-stream fork/join of a step were
    # seen to under-count the step (456 us against a 1040 us host-synchronised
    # wall clock); on an ordinary stream the two agree
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    s = stream.cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(3, args.warmup)):
        step.run(s)
        step.decode(s)
    barrier()
    step.check_status()

    # ---- device-timed reuse-prefill steps (L2 flushed between steps)
    clocks = Clocks(torch.cuda.current_device()) if rank == 0 else None
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    barrier()
    # the clock sampler is a Python thread: a short GIL switch interval lets it
    # run about every millisecond while this thread queues the timed steps
    # (the steps are timed on the device; the launches stay ahead of the GPU)
    switch = sys.getswitchinterval()
    sys.setswitchinterval(2e-4)
    if clocks:
        clocks.mark()
    wall0 = time.perf_counter()
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        torch.cuda.nvtx.range_push("reuse_step")  # launch-list filter for ncu --nvtx
        ev[i][0].record(stream)
        step.run(s)
        ev[i][1].record(stream)
        torch.cuda.nvtx.range_pop()
    barrier()
    wall_ms = (time.perf_counter() - wall0) * 1e3  # host clock around the timed steps
    if clocks:
        clocks.mark()
    sys.setswitchinterval(switch)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = sum(step_ms)

    # ---- attention launches alone (roofline of the dominant kernel): one
    # launch for all requests of the step (the launch the step issues)
    att = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        att[i][0].record(stream)
        step.attention_all(s)
        att[i][1].record(stream)
    # ---- the HBM-bound kernels of a step, each launched for all requests back
    # to back on the timed stream after an L2 flush (achieved GB/s per kernel)
    hbm_ms = {}
    if args.batched:  # one launch for all requests
        kinds = {"slide_scatter": lambda: step.scatter_all(s),
                 "wca_initialize": lambda: step.initialize_all(s),
                 "wca_select": lambda: step.select_all(s),
                 "wca_update": lambda: step.update_all(s),
                 "wca_commit": lambda: step.commit_all(s)}
    else:  # one launch per request
        each = lambda f: lambda: [f(r, s) for r in work.requests]  # noqa: E731
        kinds = {"slide_scatter": each(step.baseline_write),
                 "wca_initialize": each(step._initialize),
                 "wca_select": each(step._select),
                 "wca_update": each(step.wca_update),
                 "wca_commit": each(step.wca_commit)}
    # SLIDE gather and relocation of every request's records (n per request):
    # gather into dense rows; relocate within a pool of twice the step's
    # blocks, from the request's slots to the same slots in the second half
    import ctypes

    lib = N.load()
    nblk = work.cache.shape[0]
    pool = torch.zeros((2 * nblk,) + tuple(work.cache.shape[1:]), dtype=work.cache.dtype,
                       device=dev)
    pool[:nblk].copy_(work.cache)
    pool_kv = N.paged_view(pool)
    slots_per_pool = nblk * cfg.block
    dst_slots = [(r.slots + slots_per_pool).contiguous() for r in work.requests]
    gk = torch.empty(cfg.seq, cfg.kv_heads, cfg.head_dim, dtype=cfg.dtype, device=dev)
    gv = torch.empty_like(gk)

    def gather_all():
        for r in work.requests:
            N.check(lib.cs_slide_gather(ctypes.byref(step.kv), r.slots.data_ptr(), cfg.seq,
                                        gk.data_ptr(), gv.data_ptr(), gk.stride(0),
                                        gk.stride(1), r.status_ptr, s), "cs_slide_gather")

    def relocate_all():
        for r, d in zip(work.requests, dst_slots):
            N.check(lib.cs_slide_relocate(ctypes.byref(pool_kv), r.slots.data_ptr(),
                                          d.data_ptr(), cfg.seq, r.status_ptr, s),
                    "cs_slide_relocate")

    kinds["slide_gather"] = gather_all
    kinds["slide_relocate"] = relocate_all
    for name, fn in kinds.items():
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            evs[i][0].record(stream)
            fn()
            evs[i][1].record(stream)
        torch.cuda.synchronize(dev)
        hbm_ms[name] = statistics.mean(a.elapsed_time(b) for a, b in evs)
    # ---- decode steps
    dec = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        torch.cuda.nvtx.range_push("decode_step")  # launch-list filter for ncu --nvtx
        dec[i][0].record(stream)
        step.decode(s)
        dec[i][1].record(stream)
        torch.cuda.nvtx.range_pop()
    barrier()
    clk = clocks.stop() if clocks else None
    step.check_status()
    att_ms = statistics.mean(a.elapsed_time(b) for a, b in att)
    dec_ms = statistics.mean(a.elapsed_time(b) for a, b in dec)

    # ---- e2e: snapshot + fresh rows from pinned host memory, outputs back
    host = []
    h2d = d2h = 0
    for r in work.requests:
        item = {}
        for name in ("cached_k", "cached_v", "q", "fk", "fv"):
            t = getattr(r, name)
            item[name] = t.cpu().pin_memory()
            h2d += t.numel() * t.element_size()
        item["out"] = torch.empty(r.out.shape, dtype=r.out.dtype).pin_memory()
        d2h += r.out.numel() * r.out.element_size()
        host.append(item)
    e2e_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
    barrier()
    items = {id(r): item for r, item in zip(work.requests, host)}

    def stage_in(r, rs):  # on the request's stream, before its launches
        for name in ("cached_k", "cached_v", "q", "fk", "fv"):
            getattr(r, name).copy_(items[id(r)][name], non_blocking=True)

    def stage_out(r, rs):  # on the request's stream, after its attention
        items[id(r)]["out"].copy_(r.out, non_blocking=True)

    for i in range(args.steps):
        flush.fill_(i & 0xFF)
        e2e_ev[i][0].record(stream)
        # per-request streams: each request's copies overlap the others' kernels
        step.run(s, before=stage_in, after=stage_out, batched=False)
        e2e_ev[i][1].record(stream)
    barrier()
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_ev)

    # ---- max over ranks
    vals = torch.tensor([total_ms, att_ms, dec_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, att_ms, dec_ms, e2e_ms = vals.tolist()
    tokens = args.requests * cfg.seq * world
    value = tokens * args.steps / (total_ms / 1e3)
    e2e_value = tokens * args.steps / (e2e_ms / 1e3)
    decode_value = args.requests * world / (dec_ms / 1e3)

    qkv = qkv_layer(args, work, dev) if rank == 0 else None
    c5 = c5_slice(args, dev, rank, world) if (world > 1 or args.c5) else None
    c4 = c4_slice(args, dev) if (world == 1 and not args.no_c4) else None
    c3 = c3_slice(args, dev) if (world == 1 and not args.no_c3) else None
    chained = chained_slice(args, dev) if (world == 1 and not args.no_c3) else None

    if rank == 0:
        pk, pk_kind = peaks()
        flops = attention_flops(work)  # per attention pass over this rank's requests
        flops_vis = attention_flops(work, visible_only=True)
        achieved = flops / (att_ms / 1e3) / 1e12
        peak = float(pk.get("bf16_tflops", 1590.0))
        cpu = None
        if not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            sec, desc = cpu_requests(work, 1, threads)
            cpu = {"value": cfg.seq / sec, "unit": "tok/s", "cores": threads, "kind": "port",
                   "sample": desc, "sample_fraction": 1.0}
        # batched: scatter, counts reset, initialize, select, update, commit,
        # attention; per request: those five WCA / SLIDE kernels and attention
        launches_per_step = 7 if args.batched else len(work.requests) * 6
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "wall_ms_per_step": wall_ms / args.steps,  # host clock, includes the L2 flushes
            "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init inputs of the C2 shapes)",
            "config": {"workload": WORKLOAD, "requests_per_gpu": args.requests,
                       "l2": "flushed (256 MB write) between timed steps",
                       "parallelism": f"request-sharded x{world}",
                       "schedule": ("batched: one launch per stage for all requests"
                                    if args.batched else
                                    "per-request streams" + (", one attention launch"
                                                             if args.batched_attention else "")),
                       "e2e_schedule": "per-request streams (each request's copies overlap "
                                       "the other requests' kernels)"},
            "decode": {"value": decode_value, "unit": "tok/s",
                       "ms_per_step": dec_ms, "note": "one token per request over 4097 keys"},
            "roofline": {"bound": "tensor",
                         "kernel": "cope_prefill_sm100_batch (all requests of a step per launch)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_kind": pk_kind,
                         "flops_per_launch": flops,
                         "visible_cell_flops_per_launch": flops_vis,
                         "visible_cell_tflops": flops_vis / (att_ms * 1e-3) / 1e12,
                         "ms_per_launch": att_ms,
                         "launches_timed": args.steps,
                         "traffic": PREFILL_DRAM_BYTES_PER_LAUNCH,
                         "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum of one "
                                         "batched C2 attention launch (8 requests; ncu --set full "
                                         "capture)"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "hot_bytes": hot_bytes(work),
            "hbm_kernels": hbm_report(work, hbm_ms, dec_ms, float(pk.get("hbm_gbs", 6650.0))),
        }
        if qkv is not None:
            line["selective_qkv"] = qkv
        if c5 is not None:
            line["c5_tp"] = c5
        if c4 is not None:
            line["c4_chat"] = c4
        if c3 is not None:
            line["c3_rag"] = c3
        if chained is not None:
            line["chained_layers"] = chained
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark of the attention hot path on B200 (one process per GPU).

Headline (BASELINE.json config 2 at T=4096): causal GQA prefill attention for the SmolLM2-135M shape (9 query /
3 KV heads, d=64), 30 independent layers' f16 Q/K/V ~ N(0,1) per step, fp32 accumulate, f32 output. One step =
one call of the C ABI (alpaca_attention) over the 30 layers, which the library runs as one persistent tcgen05
kernel. `value` is prefill attention TFLOP/s over all ranks (FLOPs = 2*H*d*T*(T+1) per layer); `tokens_per_s`
is 30*T / step time per rank, summed over ranks. Inputs (236 MB per step) exceed the 126 MB L2. The inputs come from
a SplitMix64 + Box-Muller generator (`synth_normal`), the same draws the reference arm times on the host.

The same JSON line carries the other measured legs, each with its own timing, clocks and roofline:
  e2e / e2e_f16_out  the headline step through the C ABI with pinned host buffers, copies inside the timed region
  chunked_prefill    alpaca.swift's own prefill loop: the config-2 prompt in 512-token chunks at moving start positions,
                     30 layers per chunk (calls short of work items split their KV range over the SMs)
  chunked_sessions   the same loop for 3 sessions at once: every session's next chunk in one ragged call per layer
  decode             config 3: split-KV decode (batch 64, one token each, contexts U[1,4096], 30 layers of f16 caches)
  rope_kv_append     the RoPE + KV-cache append upstream of the attention, config-2 shape
  decode_proj        the fused decode projections around the attention (norm + QKV, out + residual, gate/up + SiLU,
                     down + residual), one token through the 24 q8_0 layers of SmolLM2-1.7B
  cfg4               config 4: 8 x 4096 tokens at 15/5 heads (SmolLM2-360M), strong scaling: the 40 (sequence, KV-head)
                     units split over the ranks
  cfg5               config 5: the SmolLM2-1.7B ragged mixed batch (256 prefill sequences, lengths log-uniform in
                     [128, 8192], + 512 decode sequences over 1..8192-row caches, 32/32 heads), strong scaling: units of
                     (sequence, 8 KV heads) packed over the ranks longest-first; per rank one ragged prefill launch and
                     one ragged decode launch over a paged pool of 256-row blocks
Multi-GPU (torchrun): every rank runs its own units (no exchange step: (sequence, KV-head) units share nothing),
timing is the max over ranks, and NCCL only gathers per-rank output checksums after the timed regions.
`--impl reference` times the CPU restatement of alpaca.swift's reference attention (oracle/) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "prefill attn TFLOP/s + decode attn HBM GB/s; tokens/s at 1/2/4/8 B200"
H, KVH, D = 9, 3, 64
LAYERS = 30
T_PREFILL = 4096
SEED_CFG2 = 20260102
DEC_BATCH, DEC_CAP = 64, 4096
SESSIONS = 3             # sessions of the ragged chunk-loop leg
CFG4_SEQS, CFG4_H, CFG4_KVH = 8, 15, 5
CFG5_H = CFG5_KVH = 32
CFG5_UNIT_HEADS = 8      # KV heads per config-5 unit
CFG5_BLOCK_ROWS = 256
L2_BYTES = 126 * 2 ** 20


def flops_prefill(T: int, heads: int = H, d: int = D) -> float:
    return 2.0 * heads * d * T * (T + 1)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm_gbs": j["hbm_gbs"], "tflops": j["bf16_tflops"], "tflops_sustained": j["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


def profile_traffic(name: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md ("traffic_bytes_per_launch: N")."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


def host_cpu():
    model = None
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count(),
            "threads_available": len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()}


# ---------------------------------------------------------------------------------------------- synthetic data

_GOLD, _MIX1, _MIX2 = 0x9E3779B97F4A7C15, 0xBF58476D1CE4E5B9, 0x94D049BB133111EB


def _s64(x: int) -> int:
    return x - (1 << 64) if x >= 1 << 63 else x


def synth_normal(seed: int, shape, device="cpu"):
    """N(0,1) f32 draws: SplitMix64 over a counter (x_i = mix(seed + i * golden), i = 1, 2, ...) and Box-Muller on
    pairs, in torch int64 arithmetic (wrapping; right shifts masked to logical), on `device`."""
    import torch
    n = math.prod(shape)
    m = (n + 1) // 2
    i = torch.arange(1, 2 * m + 1, dtype=torch.int64, device=device)

    def lsr(z, k):
        return (z >> k) & ((1 << (64 - k)) - 1)

    z = i * _s64(_GOLD) + _s64(seed & (2 ** 64 - 1))
    z = (z ^ lsr(z, 30)) * _s64(_MIX1)
    z = (z ^ lsr(z, 27)) * _s64(_MIX2)
    z = z ^ lsr(z, 31)
    u = (lsr(z, 11).double() + 0.5) * (1.0 / 9007199254740992.0)
    del z, i
    r = torch.sqrt(-2.0 * torch.log(u[0::2]))
    t = (2.0 * math.pi) * u[1::2]
    out = torch.stack([r * torch.cos(t), r * torch.sin(t)], dim=1).reshape(-1)[:n]
    return out.float().reshape(shape)


def cfg2_layer(rank: int, layer: int, T: int, device="cpu"):
    """Layer `layer` of rank `rank` of the config-2 step: f16 Q [T, 9, 64] and K, V [T, 3, 64]."""
    s = SEED_CFG2 + 100000 * rank + 3 * layer
    return (synth_normal(s, (T, H, D), device).half(), synth_normal(s + 1, (T, KVH, D), device).half(),
            synth_normal(s + 2, (T, KVH, D), device).half())


DATA_CFG2 = (f"synthetic N(0,1): SplitMix64 + Box-Muller (synth_normal), seed {SEED_CFG2} + 100000*rank + 3*layer, "
             "rounded to f16")


def cfg2_config(T: int, layers: int, world: int) -> dict:
    return {"workload": f"config 2: SmolLM2-135M causal GQA prefill, T={T}, {layers} independent layers per step, "
                        "9/3 heads, d=64, f16 in / f32 out",
            "tokens": T, "layers": layers, "heads": H, "kv_heads": KVH, "head_dim": D, "batch_per_gpu": 1,
            "parallelism": f"independent sequences per GPU x{world}",
            "l2": "inputs 236 MB per step vs 126 MB L2 (no flush)"}


# ---------------------------------------------------------------------------------------------- timing

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        self.idx = ids[cuda_index] if cuda_index < len(ids) else str(cuda_index)
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.15)  # the first sample lands inside the timed region
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != gpus and world > 1:
        raise SystemExit(f"--gpus {gpus} but WORLD_SIZE {world}")
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # Communicator set-up (eager with device_id: inside init_process_group) may print a banner on stdout; keep
        # stdout for the one JSON result line.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
            pg = dist
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    return rank, world, local, pg


def max_over_ranks(x: float, pg) -> float:
    if pg is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg):
    import torch
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()


class Ctx:
    """What every leg needs: the process group, this rank's device and stream, the peaks and the arguments."""

    def __init__(self, args, rank, world, local, pg):
        import torch
        import alpaca_b200 as ab
        self.args, self.rank, self.world, self.local, self.pg = args, rank, world, local, pg
        self.torch, self.ab = torch, ab
        self.dev = torch.device("cuda", local)
        self.stream = torch.cuda.current_stream()
        self.pk = peaks()
        self._flush = None

    def flush_l2(self):
        if self._flush is None:
            self._flush = self.torch.empty(2 * L2_BYTES // 4, dtype=self.torch.float32, device=self.dev)
        self._flush.zero_()

    def timed(self, fn, steps: int, warmup: int, flush: bool = False):
        """Device time of one call of fn on this rank's stream, after `warmup` untimed calls: `steps` calls between
        CUDA events (flush: L2 written over before every call, outside the timed spans). Returns (ms this rank,
        ms max over ranks, clocks sampled during the timed calls)."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        self.ab.device_status()
        clocks = ClockSampler(self.local)
        clocks.start()
        barrier(self.pg)
        if flush:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for e0, e1 in evs:
                self.flush_l2()
                e0.record(self.stream)
                fn()
                e1.record(self.stream)
            barrier(self.pg)
            ms = sum(e0.elapsed_time(e1) for e0, e1 in evs) / steps
        else:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            for _ in range(steps):
                fn()
            e1.record(self.stream)
            barrier(self.pg)
            ms = e0.elapsed_time(e1) / steps
        clk = clocks.stop()
        self.ab.device_status()
        return ms, max_over_ranks(ms, self.pg), clk

    def graph(self, fn):
        """fn captured once into a CUDA graph (per-layer launches are launch-bound otherwise)."""
        torch = self.torch
        side = torch.cuda.Stream(device=self.dev)
        side.wait_stream(self.stream)
        with torch.cuda.stream(side):
            fn()
        self.stream.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g


# ---------------------------------------------------------------------------------------------- CPU baseline

def cpu_layer_rates(threads: int, T: int = T_PREFILL, min_seconds: float = 0.0):
    """The oracle (C restatement of CPUOps.attentionScores / softmax / attentionApply, CPUOps.swift:162-274) on layer
    0 of rank 0's config-2 inputs (the GPU arm's own first layer): a full layer (9 heads x T tokens) on `threads`
    threads, repeated until `min_seconds` have passed; returns (TFLOP/s, seconds per layer, layers timed)."""
    import numpy as np

    import oracle
    q, k, v = (x.float().numpy() for x in cfg2_layer(0, 0, T))
    out = np.zeros((T, H, D), np.float32)
    times = []
    while not times or sum(times) < min_seconds:
        t0 = time.perf_counter()
        oracle.attention(q, k, v, 0, threads=threads, out=out)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    return flops_prefill(T) / per / 1e12, per, len(times)


def cpu_single_thread(T: int = T_PREFILL):
    """One thread, as CPUOps runs (no concurrentPerform in its attention loops, CPUOps.swift:238-271), over head 0
    of layer 0 (all T tokens; rows are independent, so the rate of one head is the rate of the layer)."""
    import numpy as np

    import oracle
    q, k, v = (x.float().numpy() for x in cfg2_layer(0, 0, T))
    out = np.zeros((T, H, D), np.float32)
    t0 = time.perf_counter()
    oracle.attention(q, k, v, 0, threads=1, rows=(0, T), out=out)
    dt = time.perf_counter() - t0
    return {"value": flops_prefill(T, 1) / dt / 1e12, "unit": "TFLOP/s", "cores": 1, "seconds": dt,
            "sample": f"head 0 of layer 0 (all {T} tokens, exact FLOP count), 1 thread"}


# ---------------------------------------------------------------------------------------------- legs

def leg_cfg2(c: Ctx):
    """Config 2 (the headline): 30 layers x T tokens of rank-seeded inputs, one ABI call per step."""
    torch, ab, args = c.torch, c.ab, c.args
    T, L = args.tokens, args.layers
    q = torch.empty((L, T, H, D), dtype=torch.float16, device=c.dev)
    k = torch.empty((L, T, KVH, D), dtype=torch.float16, device=c.dev)
    v = torch.empty_like(k)
    for layer in range(L):
        q[layer], k[layer], v[layer] = cfg2_layer(c.rank, layer, T, c.dev)
    out = torch.empty((L, T, H, D), dtype=torch.float32, device=c.dev)
    desc = ab.make_desc(q, k, v, out, start_position=0)
    assert ab.workspace_bytes(desc, ab.Kernel.PREFILL_TC) == 0
    ms, ms_max, clk = c.timed(lambda: ab.launch(desc, ab.Kernel.PREFILL_TC, None, c.stream), args.steps, args.warmup)
    flops_rank = L * flops_prefill(T)
    spot = None
    if c.rank == 0:
        import oracle
        q0, k0, v0 = (x[0].float().cpu().numpy() for x in (q, k, v))
        rows = [0, 1, 129, T - 1, T + 5, 3 * T + T // 2 - 1, H * T - 1]
        ref = oracle.attention_rows(q0, k0, v0, 0, rows)
        sel = oracle.rows_mask(rows, T, H)
        spot = float(abs(out[0].cpu().numpy()[sel] - ref[sel]).max())
    return dict(q=q, k=k, v=v, out=out, ms=ms, ms_max=ms_max, clk=clk, flops_rank=flops_rank, spot=spot)


def leg_e2e(c: Ctx, q, k, v, out_dtype, job_flops):
    """The headline step through the public ABI from pinned host buffers: H2D of the step's Q/K/V and D2H of its
    output inside the timed region, every step, pipelined over chunks of layers on three streams."""
    torch, ab, args = c.torch, c.ab, c.args
    out = torch.empty(q.shape, dtype=out_dtype, device=c.dev)
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()
    n_units = q.shape[0]
    chunk = max(1, min(n_units, args.e2e_chunk if args.e2e_chunk > 0 else -(-n_units // 6)))
    bounds = [(c0, min(n_units, c0 + chunk)) for c0 in range(0, n_units, chunk)]
    descs = [ab.make_desc(q[a:b], k[a:b], v[a:b], out[a:b], start_position=0) for a, b in bounds]
    s_in, s_out = torch.cuda.Stream(c.dev), torch.cuda.Stream(c.dev)
    ev_in = [torch.cuda.Event() for _ in bounds]
    ev_comp = [torch.cuda.Event() for _ in bounds]
    ev_out = [torch.cuda.Event() for _ in bounds]
    started = [False]

    def e2e_step():
        for i, ((a, b), dsc) in enumerate(zip(bounds, descs)):
            with torch.cuda.stream(s_in):
                if started[0]:
                    s_in.wait_event(ev_comp[i])  # previous step's kernel has read these inputs
                q[a:b].copy_(hq[a:b], non_blocking=True)
                k[a:b].copy_(hk[a:b], non_blocking=True)
                v[a:b].copy_(hv[a:b], non_blocking=True)
                ev_in[i].record(s_in)
            c.stream.wait_event(ev_in[i])
            if started[0]:
                c.stream.wait_event(ev_out[i])  # previous step's output chunk has been read back
            ab.launch(dsc, ab.Kernel.PREFILL_TC, None, c.stream)
            ev_comp[i].record(c.stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp[i])
                hout[a:b].copy_(out[a:b], non_blocking=True)
                ev_out[i].record(s_out)
        started[0] = True
        c.stream.wait_event(ev_out[-1])

    s_in.wait_stream(c.stream)
    steps = max(3, min(args.steps, 10))
    ms, ms_max, clk = c.timed(e2e_step, steps, 2)
    ok = bool(torch.equal(hout[-1].to(c.dev), out[-1]))
    return {"value": job_flops / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms_max, "chunks_per_step": len(bounds),
            "out_dtype": "f16" if out_dtype == torch.float16 else "f32", "readback_matches_device": ok,
            "clocks": clk,
            "api": "alpaca_attention (C ABI via ctypes), one call per chunk of sequences; pinned host Q/K/V in, "
                   "context out, every step; copy-in / compute / copy-out on three streams"}


def leg_chunked(c: Ctx):
    """alpaca.swift's own prefill loop (MetalLlamaModel.swift:293-298): one session's 4096-token prompt in 512-token
    chunks at a moving start position, every chunk through the 30 layers before the next (240 calls per step, each
    one layer's chunk, replayed from a CUDA graph), config 2's heads and FLOPs. A chunk has 18 work items (9 heads x 2
    pairs of query tiles), so the library splits the KV range of the later chunks' items over the SMs and merges the
    parts; the workspace is the size the library asks for."""
    torch, ab, args = c.torch, c.ab, c.args
    T, L, CH = args.tokens, args.layers, 512
    g = torch.Generator(device=c.dev)
    g.manual_seed(20260108 + 1000 * c.rank)
    k = [torch.randn((T, KVH, D), generator=g, device=c.dev).half() for _ in range(L)]
    v = [torch.randn((T, KVH, D), generator=g, device=c.dev).half() for _ in range(L)]
    q = [torch.randn((T, H, D), generator=g, device=c.dev).half() for _ in range(L)]
    out = [torch.empty((T, H, D), dtype=torch.float32, device=c.dev) for _ in range(L)]
    descs = [ab.make_desc(q[l][c0:c0 + CH], k[l][:c0 + CH], v[l][:c0 + CH], out[l][c0:c0 + CH], start_position=c0)
             for c0 in range(0, T, CH) for l in range(L)]
    needs = [ab.workspace_bytes(d, ab.Kernel.PREFILL_TC) for d in descs]  # > 0: a split call (f16 queries)
    need = max(needs)
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=c.dev)  # stream-ordered calls share it
    launches = sum(2 if n > 0 else 1 for n in needs)  # a split call adds the merge kernel

    def step():
        for d in descs:
            ab.launch(d, ab.Kernel.PREFILL_TC, ws)

    gr = c.graph(step)
    ms, ms_max, clk = c.timed(gr.replay, args.steps, args.warmup)
    del gr
    import oracle
    rows = _spot_rows(T, H)
    ref = oracle.attention_rows(q[0].float().cpu().numpy(), k[0].float().cpu().numpy(), v[0].float().cpu().numpy(),
                                0, rows)
    sel = oracle.rows_mask(rows, T, H)
    spot = max_over_ranks(float(abs(out[0].cpu().numpy()[sel] - ref[sel]).max()), c.pg)
    flops = L * flops_prefill(T)
    return {"workload": f"alpaca's chunked prefill: a {T}-token prompt in {CH}-token chunks at moving start "
                        f"positions, {L} layers per chunk ({len(descs)} calls per step), 9/3 heads, d=64, f16 in / "
                        "f32 out; calls short of work items split their KV range over the SMs",
            "value": c.world * flops / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_max,
            "tokens_per_s": c.world * T / (ms_max * 1e-3), "scaling": "weak", "workspace_bytes": need,
            "l2": f"{L} layers' K/V and Q ({L * T * (H + 2 * KVH) * D * 2 / 1e6:.0f} MB) vs 126 MB L2 (no flush)",
            "split_calls_per_step": sum(1 for n in needs if n > 0),
            "clocks": clk, "spot_check_max_abs": spot, "gpu_launches": args.steps * launches}


def leg_chunked_sessions(c: Ctx):
    """The same chunk loop serving several sessions at once: SESSIONS prompts of the config-2 length, every session's
    next 512-token chunk in one ragged call per layer (packed queries, each session's own KV cache and start
    position), 30 layers per chunk. A call has 18 work items per session, fewer than the SMs, so the library splits
    the units' KV ranges too (each unit into as many parts as its own blocks allow)."""
    torch, ab, args = c.torch, c.ab, c.args
    T, L, CH, S = args.tokens, args.layers, 512, SESSIONS
    NC = T // CH
    g = torch.Generator(device=c.dev)
    g.manual_seed(20260109 + 1000 * c.rank)
    k = [torch.randn((S, T, KVH, D), generator=g, device=c.dev).half() for _ in range(L)]
    v = [torch.randn((S, T, KVH, D), generator=g, device=c.dev).half() for _ in range(L)]
    q = [torch.randn((NC, S * CH, H, D), generator=g, device=c.dev).half() for _ in range(L)]  # packed per chunk
    out = [torch.empty((NC, S * CH, H, D), dtype=torch.float32, device=c.dev) for _ in range(L)]
    offs = torch.arange(0, S + 1, dtype=torch.int32, device=c.dev) * CH
    starts = [torch.full((S,), j * CH, dtype=torch.int32, device=c.dev) for j in range(NC)]
    descs = [ab.make_varlen_desc(q[l][j], k[l], v[l], out[l][j], offs, starts[j], max_tokens=CH, max_ctx_len=T)
             for j in range(NC) for l in range(L)]
    need = max(ab.workspace_bytes(d, ab.Kernel.PREFILL_TC) for d in descs)
    ws = torch.empty(need, dtype=torch.uint8, device=c.dev)  # stream-ordered calls share it

    def step():
        for d in descs:
            ab.launch(d, ab.Kernel.PREFILL_TC, ws)

    gr = c.graph(step)
    ms, ms_max, clk = c.timed(gr.replay, args.steps, args.warmup)
    del gr
    import oracle
    rows = _spot_rows(T, H)
    sel = oracle.rows_mask(rows, T, H)
    spot = 0.0
    for s in (0, S - 1):  # first and last session of layer 0, their chunks put back in prompt order
        qs = torch.cat([q[0][j][s * CH:(s + 1) * CH] for j in range(NC)]).float().cpu().numpy()
        os_ = torch.cat([out[0][j][s * CH:(s + 1) * CH] for j in range(NC)]).cpu().numpy()
        ref = oracle.attention_rows(qs, k[0][s].float().cpu().numpy(), v[0][s].float().cpu().numpy(), 0, rows)
        spot = max(spot, float(abs(os_[sel] - ref[sel]).max()))
    spot = max_over_ranks(spot, c.pg)
    flops = S * L * flops_prefill(T)
    return {"workload": f"{S} sessions' {T}-token prompts in {CH}-token chunks, every session's next chunk in one "
                        f"ragged call per layer, {L} layers per chunk ({len(descs)} calls per step), 9/3 heads, d=64, "
                        "f16 in / f32 out; calls short of work items split their units' KV ranges over the SMs",
            "value": c.world * flops / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_max,
            "tokens_per_s": c.world * S * T / (ms_max * 1e-3), "scaling": "weak", "workspace_bytes": need,
            "l2": f"{L} layers' K/V and Q ({L * S * T * (H + 2 * KVH) * D * 2 / 1e6:.0f} MB) vs 126 MB L2 (no flush)",
            "clocks": clk, "spot_check_max_abs": spot,
            "gpu_launches": args.steps * len(descs) * 3}  # plan, prefill and merge kernels per call


def leg_decode(c: Ctx):
    torch, ab, args = c.torch, c.ab, c.args
    Kernel = ab.Kernel
    g = torch.Generator(device=c.dev)
    g.manual_seed(20260103 + 1000 * c.rank)
    gl = torch.Generator()
    gl.manual_seed(20260103)
    LAY = args.dec_layers
    lens = torch.randint(1, DEC_CAP + 1, (LAY, DEC_BATCH), generator=gl, dtype=torch.int32)
    lens_d = lens.to(c.dev)
    kc = torch.randn((LAY, DEC_BATCH, DEC_CAP, KVH, D), generator=g, device=c.dev).half()
    vc = torch.randn((LAY, DEC_BATCH, DEC_CAP, KVH, D), generator=g, device=c.dev).half()
    qd = torch.randn((LAY, DEC_BATCH, 1, H, D), generator=g, device=c.dev)
    od = torch.empty((LAY, DEC_BATCH, 1, H, D), dtype=torch.float32, device=c.dev)
    descs = [ab.make_desc(qd[l], kc[l], vc[l], od[l], ctx_lens=lens_d[l], max_ctx_len=DEC_CAP) for l in range(LAY)]
    wsb = max(ab.workspace_bytes(dd, Kernel.DECODE_SPLIT) for dd in descs)
    ws = torch.empty(wsb, dtype=torch.uint8, device=c.dev)

    def step():  # LAY layers x (split + combine), on the current stream
        for dd in descs:
            ab.launch(dd, Kernel.DECODE_SPLIT, ws)

    gr = c.graph(step)
    steps = max(5, args.steps)
    ms, ms_max, clk = c.timed(gr.replay, steps, max(3, args.warmup))
    del gr
    kv_bytes = float(lens.sum().item()) * KVH * D * 2 * 2
    qo_bytes = LAY * DEC_BATCH * H * D * 4 * 2
    byts = kv_bytes + qo_bytes
    gbs = byts / (ms * 1e-3) / 1e9

    # The decode step of each layer: RoPE + KV append of the new token at row ctx_len - 1, then the attention, as
    # two calls (alpaca_rope_kv_append + alpaca_attention) and fused (alpaca_attn_decode_rope).
    kn = torch.randn((LAY, DEC_BATCH, 1, KVH, D), generator=g, device=c.dev)
    vn = torch.randn((LAY, DEC_BATCH, 1, KVH, D), generator=g, device=c.dev)
    pos_d = (lens_d - 1).contiguous()
    rdescs = [ab.make_rope_desc(qd[l], kn[l], vn[l], kc[l], vc[l], theta=1e5, positions=pos_d[l]) for l in range(LAY)]

    def step_two_calls():
        for l in range(LAY):
            ab.rope_launch(rdescs[l])
            ab.launch(descs[l], Kernel.DECODE_SPLIT, ws)

    def step_fused():
        for l in range(LAY):
            ab.decode_rope(qd[l], kn[l], vn[l], kc[l], vc[l], od[l], theta=1e5, ctx_lens=lens_d[l],
                           max_ctx_len=DEC_CAP, workspace=ws)

    step_ms, step_clk = {}, {}
    for name, fn in (("two_calls", step_two_calls), ("fused", step_fused)):
        gr = c.graph(fn)
        _, step_ms[name], step_clk[name] = c.timed(gr.replay, steps, max(3, args.warmup))
        del gr
    w = c.world
    return {"workload": "config 3: batch 64 one-token decode, contexts U[1,4096], 9/3 heads, d=64, f16 KV, "
                        f"{LAY} layers (distinct caches, {kc.numel() * 4 / 1e9:.1f} GB) per step",
            "value": w * byts / (ms_max * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_max,
            "tokens_per_s": w * DEC_BATCH / (ms_max * 1e-3),  # one token per sequence per 30-layer step
            "bytes_per_step": byts, "l2": "caches 6 GB per step vs 126 MB L2 (no flush)",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": c.pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / c.pk["hbm_gbs"], "traffic": profile_traffic("decode_split_cfg3"),
                         "kernel": "alpaca::decode_split_kernel<64,3> + decode_combine_kernel per layer, "
                                   "replayed from a CUDA graph"},
            "clocks": clk, "gpu_launches": steps * LAY * 2,
            "decode_step": {
                "workload": f"config 3 decode step of {LAY} layers: per layer the RoPE + f16 KV append of each "
                            "sequence's new token (row ctx_len - 1), then the split-KV attention",
                "two_calls_ms_per_step": step_ms["two_calls"], "fused_ms_per_step": step_ms["fused"],
                "value": w * DEC_BATCH / (step_ms["fused"] * 1e-3), "unit": "tokens/s",
                "two_calls_tokens_per_s": w * DEC_BATCH / (step_ms["two_calls"] * 1e-3),
                "clocks": step_clk["fused"], "gpu_launches": steps * LAY * 2}}


def leg_rope(c: Ctx):
    """RoPE of q (in place) + rotated K / raw V appended to an f16 cache, for the config-2 prefill shape: 30 layers
    x T tokens x 9/3 heads x d=64 per step, each layer its own tensors (inputs > L2). HBM-bound; GB/s counts q read
    + written (f32), k and v read (f32) and the cache rows written (f16)."""
    torch, ab, args = c.torch, c.ab, c.args
    LAY, T = args.layers, args.tokens
    g = torch.Generator(device=c.dev)
    g.manual_seed(20260105 + 1000 * c.rank)
    q = torch.randn((LAY, T, H, D), generator=g, device=c.dev)
    k = torch.randn((LAY, T, KVH, D), generator=g, device=c.dev)
    v = torch.randn((LAY, T, KVH, D), generator=g, device=c.dev)
    kc = torch.zeros((LAY, T, KVH, D), dtype=torch.float16, device=c.dev)
    vc = torch.zeros_like(kc)
    descs = [ab.make_rope_desc(q[l], k[l], v[l], kc[l], vc[l], theta=1e5, start_position=0) for l in range(LAY)]

    def step():
        for dd in descs:
            ab.rope_launch(dd)

    gr = c.graph(step)
    steps = max(5, args.steps)
    ms, ms_max, clk = c.timed(gr.replay, steps, max(3, args.warmup))
    del gr
    byts = LAY * T * (H * D * 4 * 2 + KVH * D * 4 * 2 + KVH * D * 2 * 2)
    gbs = byts / (ms * 1e-3) / 1e9
    return {"workload": f"RoPE + KV append, config-2 shape: {LAY} layers x T={T} tokens, 9/3 heads, d=64, f32 q/k/v "
                        "in, f16 cache out, one call per layer replayed from a CUDA graph",
            "value": c.world * byts / (ms_max * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_max,
            "tokens_per_s": c.world * T / (ms_max * 1e-3),  # prompt tokens through all layers per second
            "bytes_per_step": byts, "l2": "850 MB per step vs 126 MB L2 (no flush)",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": c.pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / c.pk["hbm_gbs"], "traffic": profile_traffic("rope_kv_cfg2"),
                         "kernel": "alpaca::rope_kv_vec_kernel per layer"},
            "clocks": clk, "gpu_launches": steps * LAY}


PROJ_LAYERS, PROJ_HIDDEN, PROJ_FFN = 24, 2048, 8192  # SmolLM2-1.7B


def leg_proj(c: Ctx):
    """The fused decode projections around the attention of one token through the 24 layers of SmolLM2-1.7B (hidden
    2048, 32/32 heads of 64, FFN 8192) with q8_0 weights, as alpaca.swift's fused decode path issues them
    (MetalLlamaModel.swift:344-354): per layer Q/K/V with the attention norm, the out-projection added to the
    residual, gate + up with the FFN norm and SiLU, down added to the residual. 71.3 MB of weights per layer, 1.71 GB
    per step (>> L2), 96 launches per step replayed from a CUDA graph. HBM-bound: GB/s of weight bytes."""
    torch, ab, args = c.torch, c.ab, c.args
    Hd, F = PROJ_HIDDEN, PROJ_FFN
    g = torch.Generator(device=c.dev)
    g.manual_seed(20260107 + 1000 * c.rank)

    def q8(rows, k):  # random int8 weights with a fixed f16 scale per 32-weight block
        w = torch.randint(-127, 128, (rows, k // 32, 34), generator=g, device=c.dev, dtype=torch.int8).view(torch.uint8)
        w[:, :, 0:2] = torch.tensor([0.002], dtype=torch.float16).view(torch.uint8).to(c.dev)
        return w.reshape(rows, k // 32 * 34).contiguous()

    layers = []
    for _ in range(PROJ_LAYERS):
        layers.append(dict(q=q8(Hd, Hd), k=q8(Hd, Hd), v=q8(Hd, Hd), o=q8(Hd, Hd), gate=q8(F, Hd), up=q8(F, Hd),
                           down=q8(Hd, F), ga=torch.ones(Hd, device=c.dev), gf=torch.ones(Hd, device=c.dev)))
    x = torch.randn((1, Hd), generator=g, device=c.dev)
    qo, ko, vo = (torch.empty((1, Hd), device=c.dev) for _ in range(3))
    gate = torch.empty((1, F), device=c.dev)
    descs = []
    for L in layers:
        descs.append(ab.make_proj_desc([L["q"], L["k"], L["v"]], "q8_0", Hd, x, [qo, ko, vo], norm_weight=L["ga"]))
        descs.append(ab.make_proj_desc([L["o"]], "q8_0", Hd, qo, [x], add=True))  # the attention output stands in
        descs.append(ab.make_proj_desc([L["gate"], L["up"]], "q8_0", Hd, x, [gate], norm_weight=L["gf"],
                                       silu_gate=True))
        descs.append(ab.make_proj_desc([L["down"]], "q8_0", F, gate, [x], add=True))

    def step():
        for d in descs:
            ab.project_launch(d)

    gr = c.graph(step)
    steps = max(5, args.steps)
    ms, ms_max, clk = c.timed(gr.replay, steps, max(3, args.warmup))
    del gr
    wbytes = float(sum(t.numel() for L in layers for key, t in L.items() if key not in ("ga", "gf")))
    gbs = wbytes / (ms * 1e-3) / 1e9
    return {"workload": f"fused decode projections, SmolLM2-1.7B shape (hidden {Hd}, FFN {F}), q8_0 weights, one token "
                        f"through {PROJ_LAYERS} layers: QKV + norm, out-proj + residual, gate/up + norm + SiLU, down + "
                        "residual per layer, replayed from a CUDA graph",
            "value": c.world * wbytes / (ms_max * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_max,
            "tokens_per_s": c.world / (ms_max * 1e-3), "bytes_per_step": wbytes,
            "l2": f"{wbytes / 1e9:.2f} GB of weights per step vs 126 MB L2 (no flush)",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": c.pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / c.pk["hbm_gbs"], "traffic": profile_traffic("decode_proj_q8_1p7b"),
                         "kernel": "alpaca::proj_mma_kernel<q8_0> (int8 tensor-core form, one token) per projection; traffic: the "
                                   "gate + up launch"},
            "clocks": clk, "gpu_launches": steps * PROJ_LAYERS * 4}


def _spot_rows(T: int, heads: int):
    return sorted({0, 1, min(129, T - 1), T - 1, min(T + 5, heads * T - 1), heads * T - 1})


def leg_cfg4(c: Ctx):
    """Config 4: 8 sequences x 4096 tokens of the SmolLM2-360M shape (15/5 heads, d=64), strong scaling. The 40
    (sequence, KV-head) units (3 query heads each) are packed over the ranks longest-first; each rank holds its units'
    Q/K/V as [units, T, 3 | 1, 64] (generated from the unit's own seed, so no data moves) and runs them as one call."""
    torch, ab, args = c.torch, c.ab, c.args
    from alpaca_b200.partition import partition, units_for_batch
    T, G = args.tokens, CFG4_H // CFG4_KVH
    units = units_for_batch([T] * CFG4_SEQS, [0] * CFG4_SEQS, CFG4_H, CFG4_KVH)
    # --cfg4-ranks R (one process): time rank 0's share of an R-rank plan, the per-rank work of R GPUs on this one
    emulated = args.cfg4_ranks if (args.cfg4_ranks > 0 and c.world == 1) else 0
    plan = partition(units, emulated or c.world, tflops=c.pk["tflops"] * 0.45, hbm_gbs=c.pk["hbm_gbs"] * 0.7)
    mine = plan.ranks[0 if emulated else c.rank]
    U = len(mine)
    q = torch.empty((U, T, G, D), dtype=torch.float16, device=c.dev)
    k = torch.empty((U, T, 1, D), dtype=torch.float16, device=c.dev)
    v = torch.empty_like(k)
    for i, u in enumerate(mine):
        g = torch.Generator(device=c.dev)
        g.manual_seed(20260104 + 100 * u.seq + u.kv_head)
        q[i] = torch.randn((T, G, D), generator=g, device=c.dev).half()
        k[i] = torch.randn((T, 1, D), generator=g, device=c.dev).half()
        v[i] = torch.randn((T, 1, D), generator=g, device=c.dev).half()
    out = torch.empty((U, T, G, D), dtype=torch.float32, device=c.dev)
    in_bytes = (q.numel() + k.numel() + v.numel()) * 2
    # Identical copies of the rank's inputs and outputs, used in turn, so that the calls between two uses of a copy
    # touch more than the L2 holds: every call reads its inputs from HBM, and the calls run back to back as a
    # model's layers do (a flush before each call would also time a dirty L2's write-backs and the launch ramp).
    copy_bytes = in_bytes + out.numel() * 4
    n_copies = 1 + -(-(3 * L2_BYTES // 2) // copy_bytes)
    bufs = [(q, k, v, out)] + [(q.clone(), k.clone(), v.clone(), torch.empty_like(out)) for _ in range(n_copies - 1)]
    descs = [ab.make_desc(*b) for b in bufs]
    turn = [0]

    def call():
        ab.launch(descs[turn[0] % n_copies], ab.Kernel.PREFILL_TC, None, c.stream)
        turn[0] += 1

    ms, ms_max, clk = c.timed(call, args.steps, args.warmup)
    ab.launch(descs[0], ab.Kernel.PREFILL_TC, None, c.stream)  # copy 0's output for the spot check
    import oracle
    rows = _spot_rows(T, G)
    ref = oracle.attention_rows(q[0].float().cpu().numpy(), k[0].float().cpu().numpy(), v[0].float().cpu().numpy(),
                                0, rows)
    sel = oracle.rows_mask(rows, T, G)
    spot = max_over_ranks(float(abs(out[0].cpu().numpy()[sel] - ref[sel]).max()), c.pg)
    flops_rank = U * G * flops_prefill(T, 1)
    kt = flops_rank / (ms * 1e-3) / 1e12
    job = CFG4_SEQS * flops_prefill(T, CFG4_H)
    if emulated:
        return {"workload": f"config 4: rank 0's share of a {emulated}-rank plan ({U} (sequence, KV-head) units of 3 "
                            f"query heads x T={T}), one call, timed on one GPU",
                "emulated_ranks": emulated, "units": U, "value": kt, "unit": "TFLOP/s", "ms_per_step": ms_max,
                "l2": f"calls take turns over {n_copies} identical copies of the inputs and outputs "
                      f"({n_copies * copy_bytes / 1e6:.0f} MB vs 126 MB L2), back to back, no flush",
                "clocks": clk, "spot_check_max_abs": spot, "gpu_launches": args.steps}
    return {"workload": f"config 4: SmolLM2-360M causal GQA prefill, {CFG4_SEQS} sequences x T={T}, 15/5 heads, d=64; "
                        f"(sequence, KV-head) units split over {c.world} GPU(s), one call per rank",
            "value": job / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_max,
            "tokens_per_s": CFG4_SEQS * T / (ms_max * 1e-3), "scaling": "strong", "units_rank0": U,
            "plan_imbalance": plan.imbalance,
            "l2": (f"inputs {in_bytes / 1e6:.0f} MB + outputs {out.numel() * 4 / 1e6:.0f} MB per rank, used in turn "
                   f"from {n_copies} identical copies ({n_copies * copy_bytes / 1e6:.0f} MB vs 126 MB L2): every call "
                   "reads its inputs from HBM; calls back to back, no flush"),
            "roofline": {"bound": "tensor", "achieved": kt, "peak": c.pk["tflops"], "unit": "TFLOP/s",
                         "frac": kt / c.pk["tflops"], "traffic": None,
                         "kernel": "alpaca::prefill_kernel (tcgen05, persistent), rank 0's launch"},
            "clocks": clk, "spot_check_max_abs": spot, "gpu_launches": args.steps}


def leg_cfg5(c: Ctx):
    """Config 5: the SmolLM2-1.7B ragged mixed batch (32/32 heads, d=64): 256 prefill sequences with lengths
    log-uniform in [128, 8192] and 512 one-token decode sequences over caches of 1..8192 rows, strong scaling. Units
    of (sequence, 8 KV heads) are packed over the ranks longest-processing-time first; each rank keeps its units'
    K/V rows in one pool of 256-row blocks handed out in shuffled order (per-unit block tables, the serving layout),
    and runs one step as one ragged prefill launch over all its prefill units (packed queries) plus one ragged split
    decode over all its decode units."""
    import numpy as np
    torch, ab, args = c.torch, c.ab, c.args
    Kernel = ab.Kernel
    from alpaca_b200.partition import head_group_units, partition
    HG, R = CFG5_UNIT_HEADS, CFG5_BLOCK_ROWS
    rng = np.random.default_rng(20260105)
    pre_T = np.round(np.exp(rng.uniform(np.log(128), np.log(8192), 256))).astype(int)
    dec_L = rng.integers(1, 8192 + 1, 512)
    units = head_group_units(list(pre_T), [0] * 256, CFG5_KVH, HG) + \
        head_group_units([1] * 512, list(dec_L - 1), CFG5_KVH, HG, first_seq=256)
    plan = partition(units, c.world, tflops=c.pk["tflops"] * 0.45, hbm_gbs=c.pk["hbm_gbs"] * 0.7)
    mine = plan.ranks[c.rank]
    pre = [u for u in mine if u.seq < 256]
    dec = [u for u in mine if u.seq >= 256]
    Tp = [u.tokens for u in pre]
    Ld = [u.start + 1 for u in dec]
    nb_p = [-(-t // R) for t in Tp]
    nb_d = [-(-x // R) for x in Ld]
    total = max(1, sum(nb_p) + sum(nb_d))
    g = torch.Generator(device=c.dev)
    g.manual_seed(20260105 + 1000 * c.rank)
    order = torch.randperm(total, generator=torch.Generator().manual_seed(20260106 + c.rank)).to(torch.int32)
    kpool = torch.randn((total, R, HG, D), generator=g, device=c.dev).half()
    vpool = torch.randn((total, R, HG, D), generator=g, device=c.dev).half()
    nxt = 0

    def table(nbs):
        nonlocal nxt
        t = torch.zeros((max(1, len(nbs)), max([1] + nbs)), dtype=torch.int32)
        for i, nb in enumerate(nbs):
            t[i, :nb] = order[nxt:nxt + nb]
            nxt += nb
        return t.to(c.dev)

    tab_p, tab_d = table(nb_p), table(nb_d)
    n_pre = max(1, len(pre))
    offs = np.concatenate([[0], np.cumsum(Tp)]).astype(np.int32) if pre else np.zeros(2, np.int32)
    qp = torch.randn((max(1, int(offs[-1])), HG, D), generator=g, device=c.dev).half()
    op = torch.empty((qp.shape[0], HG, D), dtype=torch.float32, device=c.dev)
    offs_d = torch.from_numpy(offs).to(c.dev)
    starts_d = torch.zeros(n_pre, dtype=torch.int32, device=c.dev)
    max_T = max([1] + Tp)
    pdesc = ab.make_varlen_desc(qp, kpool, vpool, op, offs_d, starts_d, max_tokens=max_T,
                                max_ctx_len=tab_p.shape[1] * R, block_table=tab_p) if pre else None
    ws_p = torch.empty(max(16, ab.workspace_bytes(pdesc, Kernel.PREFILL_TC)) if pre else 16, dtype=torch.uint8,
                       device=c.dev)
    nd = max(1, len(dec))
    qd = torch.randn((nd, 1, HG, D), generator=g, device=c.dev)
    od = torch.empty((nd, 1, HG, D), dtype=torch.float32, device=c.dev)
    lens = torch.tensor(Ld if dec else [1], dtype=torch.int32, device=c.dev)
    ddesc = ab.make_desc(qd, kpool, vpool, od, ctx_lens=lens, max_ctx_len=tab_d.shape[1] * R,
                         block_table=tab_d) if dec else None
    ws_d = torch.empty(max(16, ab.workspace_bytes(ddesc, Kernel.DECODE_SPLIT)) if dec else 16, dtype=torch.uint8,
                       device=c.dev)

    def prefill():
        if pdesc is not None:
            ab.launch(pdesc, Kernel.PREFILL_TC, ws_p, c.stream)

    def decode():
        if ddesc is not None:
            ab.launch(ddesc, Kernel.DECODE_SPLIT, ws_d, c.stream)

    def step():
        prefill()
        decode()

    ms, ms_max, clk = c.timed(step, args.steps, args.warmup)
    ms_p, _, _ = c.timed(prefill, args.steps, 1)
    ms_d, _, _ = c.timed(decode, max(5, args.steps), 1)

    # spot checks: rows of this rank's first prefill unit and its first decode unit against the oracle
    import oracle
    spot = 0.0
    kp_h = vp_h = None
    if pre or dec:
        kp_h, vp_h = kpool.float().cpu().numpy(), vpool.float().cpu().numpy()

    def gather(pool_h, tab, i, rows):
        t = tab[i].cpu().numpy()
        return np.concatenate([pool_h[t[b]] for b in range(-(-rows // R))])[:rows]

    if pre:
        T0 = Tp[0]
        rows = _spot_rows(T0, HG)
        ref = oracle.attention_rows(qp[:T0].float().cpu().numpy(), gather(kp_h, tab_p, 0, T0),
                                    gather(vp_h, tab_p, 0, T0), 0, rows)
        sel = oracle.rows_mask(rows, T0, HG)
        spot = max(spot, float(abs(op[:T0].cpu().numpy()[sel] - ref[sel]).max()))
    if dec:
        L0 = Ld[0]
        ref = oracle.attention(qd[0].cpu().numpy(), gather(kp_h, tab_d, 0, L0), gather(vp_h, tab_d, 0, L0), L0 - 1,
                               length=L0)
        spot = max(spot, float(abs(od[0].cpu().numpy() - ref).max()))
    spot = max_over_ranks(spot, c.pg)

    job_flops = float(sum(flops_prefill(int(t), CFG5_H) for t in pre_T))
    flops_rank = float(sum(u.flops for u in pre))
    bytes_rank = float(sum(u.kv_bytes for u in dec)) + len(dec) * HG * D * 4 * 2
    tokens = float(pre_T.sum() + len(dec_L))
    kt = flops_rank / (ms_p * 1e-3) / 1e12 if pre else None
    gb = bytes_rank / (ms_d * 1e-3) / 1e9 if dec else None
    return {"workload": "config 5: SmolLM2-1.7B shape (32/32 heads, d=64) ragged mixed batch: 256 prefill sequences, "
                        "lengths log-uniform [128, 8192], + 512 decode sequences, contexts U[1, 8192]; units of "
                        f"(sequence, {HG} KV heads) LPT-packed over {c.world} GPU(s); per rank one ragged prefill "
                        "launch + one ragged split decode over a paged pool of 256-row blocks in shuffled order",
            "value": tokens / (ms_max * 1e-3), "unit": "tokens/s", "ms_per_step": ms_max, "scaling": "strong",
            "prefill_tokens": int(pre_T.sum()), "decode_tokens": len(dec_L), "plan_imbalance": plan.imbalance,
            "units_rank0": {"prefill": len(pre), "decode": len(dec)},
            "kv_gb_rank0": 2 * kpool.numel() * 2 / 1e9, "l2": "K/V pool of GBs per rank vs 126 MB L2 (no flush)",
            "prefill_ms_rank0": ms_p, "decode_ms_rank0": ms_d,
            "prefill_tflops_if_alone": job_flops / (ms_max * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "achieved": kt, "peak": c.pk["tflops"], "unit": "TFLOP/s",
                         "frac": kt / c.pk["tflops"] if kt else None, "traffic": None,
                         "kernel": "alpaca::prefill_kernel ragged form (tcgen05, persistent), rank 0's launch alone"},
            "decode_roofline": {"bound": "hbm", "achieved": gb, "peak": c.pk["hbm_gbs"], "unit": "GB/s",
                                "frac": gb / c.pk["hbm_gbs"] if gb else None, "traffic": None,
                                "kernel": "alpaca::decode_split_kernel<64,1> + combine, rank 0's launch alone"},
            "clocks": clk, "spot_check_max_abs": spot, "gpu_launches": args.steps * 4}


# ---------------------------------------------------------------------------------------------- our arm

def run_ours(args):
    import torch

    import alpaca_b200 as ab
    rank, world, local, pg = dist_setup(args.gpus)
    ab.load()
    c = Ctx(args, rank, world, local, pg)
    T, L = args.tokens, args.layers
    job_flops = world * L * flops_prefill(T)

    p2 = leg_cfg2(c)
    ms_max = p2["ms_max"]
    kernel_tflops = p2["flops_rank"] / (p2["ms"] * 1e-3) / 1e12

    gather_ms = None
    if pg is not None:  # NCCL gather of per-rank output checksums (outside the timed regions)
        cs = p2["out"].double().sum().reshape(1)
        allcs = [torch.zeros_like(cs) for _ in range(world)]
        t0 = time.perf_counter()
        pg.all_gather(allcs, cs)
        torch.cuda.synchronize()
        gather_ms = (time.perf_counter() - t0) * 1e3

    e2e = e2e16 = None
    if not args.no_e2e:
        e2e = leg_e2e(c, p2["q"], p2["k"], p2["v"], torch.float32, job_flops)
        e2e16 = leg_e2e(c, p2["q"], p2["k"], p2["v"], torch.float16, job_flops)
    del p2["q"], p2["k"], p2["v"], p2["out"]
    torch.cuda.empty_cache()
    chunked = leg_chunked(c) if not args.no_chunked else None
    torch.cuda.empty_cache()
    sessions = leg_chunked_sessions(c) if not args.no_sessions else None
    torch.cuda.empty_cache()
    decode = leg_decode(c) if not args.no_decode else None
    torch.cuda.empty_cache()
    rope_kv = leg_rope(c) if not args.no_rope else None
    torch.cuda.empty_cache()
    proj = leg_proj(c) if not args.no_proj else None
    torch.cuda.empty_cache()
    cfg4 = leg_cfg4(c) if not args.no_cfg4 else None
    torch.cuda.empty_cache()
    cfg5 = leg_cfg5(c) if not args.no_cfg5 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        oracle.build()
        thr = oracle.host_threads()
        tf, per, n = cpu_layer_rates(thr, T, args.cpu_seconds)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": thr, "kind": "port",
               "sample": f"{n} full T={T} layer(s) of config 2 (9 heads x {T} tokens, layer 0 of the GPU arm's "
                         f"inputs), {per:.2f} s each on {thr} threads",
               "single_thread": cpu_single_thread(T), **host_cpu()}

    if pg is not None:
        pg.barrier()
    if rank == 0:
        roof = {"bound": "tensor", "achieved": kernel_tflops, "peak": c.pk["tflops"], "unit": "TFLOP/s",
                "frac": kernel_tflops / c.pk["tflops"], "traffic": profile_traffic("prefill_sm100_cfg2"),
                "peak_source": f"{c.pk['source']}: MEASURED_PEAKS.json bf16_tflops (dense, burst)",
                "kernel": "alpaca::prefill_kernel (tcgen05, persistent)",
                "algorithmic_flops_per_launch": p2["flops_rank"]}
        line = {
            "metric": METRIC, "value": job_flops / (ms_max * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": DATA_CFG2,
            "config": cfg2_config(T, L, world),
            "tokens_per_s": world * L * T / (ms_max * 1e-3),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "e2e_f16_out": e2e16,
            "gpu_launches": args.steps,
            "clocks": p2["clk"],
            "spot_check_max_abs": p2["spot"],
            "chunked_prefill": chunked,
            "chunked_sessions": sessions,
            "decode": decode,
            "rope_kv_append": rope_kv,
            "decode_proj": proj,
            "cfg4": cfg4,
            "cfg5": cfg5,
            "gather_ms": gather_ms,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


# ---------------------------------------------------------------------------------------------- reference arm

def run_reference(args):
    """alpaca.swift's CPU attention (CPUOps.swift:162-274, restated in C in oracle/: Swift + Metal cannot run here)
    on this box's host cores, all threads, on the headline config: one step times one full T=4096 layer of the 30
    (the GPU arm's own layer-0 inputs); ms_per_step is that time x 30. Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    oracle.build()
    thr = oracle.host_threads()
    T, L = args.tokens, args.layers
    vals, pers = [], []
    for i in range(args.warmup + args.steps):
        tf, per, _ = cpu_layer_rates(thr, T)
        if i >= args.warmup:
            vals.append(tf)
            pers.append(per)
    value = statistics.median(vals)
    per = statistics.median(pers)
    single = cpu_single_thread(T)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * L * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": DATA_CFG2,
        "config": cfg2_config(T, L, world),
        "timed_ms_per_step": per * 1e3,
        "extrapolated_from": f"1 full T={T} layer of the {L} per step (ms_per_step = measured layer time x {L})",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": thr, "kind": "port",
                         "sample": f"one full T={T} layer per step (9 heads x {T} tokens), {per:.2f} s each",
                         "single_thread": single, **host_cpu()},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "alpaca.swift is Swift + Metal (no Swift toolchain or Apple GPU here); the reference's CPU attention "
                "(CPUOps.swift:162-274) runs as its C restatement in oracle/ on all host threads (f32 arithmetic on "
                "the same f16-rounded inputs); the single-thread figure is how CPUOps itself runs",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=T_PREFILL)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--dec-layers", type=int, default=LAYERS)
    for leg in ("decode", "rope", "proj", "cpu", "e2e", "cfg4", "cfg5", "chunked", "sessions"):
        ap.add_argument(f"--no-{leg}", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=0, help="sequences per ABI call in the e2e pipeline (0: 1/6 of them)")
    ap.add_argument("--cpu-seconds", type=float, default=3.0, help="minimum seconds of the all-thread CPU baseline")
    ap.add_argument("--cfg4-ranks", type=int, default=0,
                    help="with one process: the cfg4 leg times rank 0's share of this many ranks' plan")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

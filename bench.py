#!/usr/bin/env python3
"""Benchmark of the attention hot path on B200 (one process per GPU).

Headline (BASELINE.json config 2 at T=4096): causal GQA prefill attention for the SmolLM2-135M shape (9 query /
3 KV heads, d=64), 30 independent layers' f16 Q/K/V ~ N(0,1) per step, fp32 accumulate, f32 output. One step =
one call of the C ABI (alpaca_attention) over the 30 layers, which the library runs as one persistent tcgen05
kernel. `value` is prefill attention TFLOP/s over all ranks (FLOPs = 2*H*d*T*(T+1) per layer); `tokens_per_s`
is 30*T / step time per rank, summed over ranks. Inputs (236 MB per step) exceed the 126 MB L2.

Also measured in the same run and reported in the `decode` object: config 3 split-KV decode (batch 64, one token
each, contexts uniform in [1,4096], 30 layers of distinct f16 KV caches per step), as HBM GB/s.

Multi-GPU (torchrun): every rank runs its own independent sequences (weak scaling; (sequence, KV-head) units
share nothing), timing is the max over ranks, and NCCL only gathers per-rank output checksums after the timed
region. `--impl reference` times the CPU restatement of alpaca.swift's reference attention (oracle/) on the host
cores instead.
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
PAGED_BLOCK_ROWS = 256
DEC_BATCH, DEC_CAP = 64, 4096


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
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
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


# ---------------------------------------------------------------------------------------------- distributed

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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
        pg = dist
        # Communicator set-up may print a banner on stdout; keep stdout for the one JSON result line.
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
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


# ---------------------------------------------------------------------------------------------- CPU baseline

def cpu_prefill_sample(seconds_target: float, threads: int, T: int = T_PREFILL):
    """Times the oracle (C restatement of CPUOps.attentionScores/softmax/attentionApply) on a strided sample of
    one layer's (head, token) rows of config 2; returns (TFLOP/s, sample description, threads)."""
    import numpy as np

    import oracle
    q = oracle.f16_round(oracle.splitmix_normal(7, (T, H, D)))
    k = oracle.f16_round(oracle.splitmix_normal(8, (T, KVH, D)))
    v = oracle.f16_round(oracle.splitmix_normal(9, (T, KVH, D)))
    out = np.zeros((T, H, D), np.float32)
    # Rows are h*T + t. Blocks of `blk` consecutive rows at evenly spread offsets cover the causal range; each
    # block runs on all `threads` (the oracle interleaves a block's rows over its POSIX threads). FLOPs are
    # counted exactly per row (4*d*(t+1)), so the rate is exact for the sample.
    blk = max(1, threads) * 8
    done_flops, elapsed, nrows = 0.0, 0.0, 0
    for nblocks in (4, 16, 64, 256, 1024):
        if elapsed >= seconds_target:
            break
        starts = [int((i + 0.5) * (H * T - blk) / nblocks) for i in range(nblocks)]
        t0 = time.perf_counter()
        for r0 in starts:
            oracle.attention(q, k, v, 0, threads=threads, rows=(r0, r0 + blk), out=out)
        dt = time.perf_counter() - t0
        done_flops += sum(4.0 * D * (((r0 + i) % T) + 1) for r0 in starts for i in range(blk))
        elapsed += dt
        nrows += nblocks * blk
    tflops = done_flops / elapsed / 1e12
    return tflops, f"{nrows} (head, token) rows of one T={T} layer in blocks spread over the causal range, " \
                   f"{elapsed:.1f} s", threads


# ---------------------------------------------------------------------------------------------- our arm

def run_ours(args):
    import numpy as np
    import torch

    import alpaca_b200 as ab
    from alpaca_b200 import Kernel
    rank, world, local, pg = dist_setup(args.gpus)
    ab.load()
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    pk = peaks()
    T = args.tokens
    if args.workload == "cfg4":
        # config 4: 8 sequences x T tokens of the SmolLM2-360M shape, split by sequence over the ranks (strong
        # scaling: the job is fixed, each rank runs sequences rank, rank+N, ...)
        nh, nkv, total_seqs = 15, 5, 8
        L = len(range(rank, total_seqs, world))
        job_flops = total_seqs * flops_prefill(T, nh)
    else:
        nh, nkv, total_seqs = H, KVH, args.layers * world
        L = args.layers
        job_flops = world * L * flops_prefill(T, nh)
    flops_step = L * flops_prefill(T, nh)  # this rank

    # ---- inputs: L independent sequences (layers) per rank, seeded per rank
    g = torch.Generator(device=dev)
    g.manual_seed(20260102 + 1000 * rank)
    q = torch.randn((L, T, nh, D), generator=g, device=dev).half()
    k = torch.randn((L, T, nkv, D), generator=g, device=dev).half()
    v = torch.randn((L, T, nkv, D), generator=g, device=dev).half()
    out = torch.empty((L, T, nh, D), dtype=torch.float32, device=dev)
    desc = ab.make_desc(q, k, v, out, start_position=0)
    assert ab.workspace_bytes(desc, Kernel.PREFILL_TC) == 0

    def step():
        ab.launch(desc, Kernel.PREFILL_TC, None, stream)

    ms_max = ms = float("nan")
    clk = None
    if not args.no_prefill:
        for _ in range(args.warmup):
            step()
        ab.device_status()
        clocks = ClockSampler(local)
        clocks.start()
        barrier(pg)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        barrier(pg)
        clk = clocks.stop()
        ab.device_status()
        ms = ev0.elapsed_time(ev1) / args.steps
        ms_max = max_over_ranks(ms, pg)
    value = job_flops / (ms_max * 1e-3) / 1e12
    tokens_per_s = total_seqs * T / (ms_max * 1e-3)
    kernel_tflops = flops_step / (ms * 1e-3) / 1e12  # one launch per step on this rank

    # ---- correctness spot check of the timed output vs the oracle (rank 0, a few rows of layer 0)
    spot = None
    if rank == 0 and not args.no_prefill:
        import oracle
        q0, k0, v0 = (x[0].float().cpu().numpy() for x in (q, k, v))
        o0 = out[0].cpu().numpy()
        rows = [0, 1, 129, T - 1, T + 5, 3 * T + T // 2 - 1, nh * T - 1]
        ref = oracle.attention_rows(q0, k0, v0, 0, rows)
        sel = oracle.rows_mask(rows, T, nh)
        spot = float(np.abs(o0[sel] - ref[sel]).max())

    # ---- NCCL gather of per-rank output checksums (outside the timed region)
    gather_ms = None
    if pg is not None:
        cs = out.double().sum().reshape(1)
        allcs = [torch.zeros_like(cs) for _ in range(world)]
        t0 = time.perf_counter()
        pg.all_gather(allcs, cs)
        torch.cuda.synchronize()
        gather_ms = (time.perf_counter() - t0) * 1e3

    # ---- e2e: host buffers (pinned), H2D of the step's inputs + kernel + D2H of the output, every step.
    # The step is pipelined over chunks of sequences (layers): chunk i's H2D (copy-in stream), ABI call (compute
    # stream) and D2H (copy-out stream) overlap the neighbouring chunks' work, as a caller streaming layers would.
    # Events order each chunk's copy -> compute -> copy, and guard device-buffer reuse by the next step.
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        hout = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
        d2h = hout.numel() * hout.element_size()
        n_units = q.shape[0]
        chunk = max(1, min(n_units, args.e2e_chunk if args.e2e_chunk > 0 else -(-n_units // 6)))
        bounds = [(c0, min(n_units, c0 + chunk)) for c0 in range(0, n_units, chunk)]
        descs = [ab.make_desc(q[a:b], k[a:b], v[a:b], out[a:b], start_position=0) for a, b in bounds]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
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
                stream.wait_event(ev_in[i])
                if started[0]:
                    stream.wait_event(ev_out[i])  # previous step's output chunk has been read back
                ab.launch(dsc, Kernel.PREFILL_TC, None, stream)
                ev_comp[i].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_comp[i])
                    hout[a:b].copy_(out[a:b], non_blocking=True)
                    ev_out[i].record(s_out)
            started[0] = True

        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(2):
            e2e_step()
        stream.wait_event(ev_out[-1])
        torch.cuda.synchronize()
        barrier(pg)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_stream(stream)
        for _ in range(e2e_steps):
            e2e_step()
        stream.wait_event(ev_out[-1])
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(pg)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, pg)
        # the last step's result must be the device result (checked on one chunk of rows)
        e2e_ok = bool(torch.equal(hout[-1].to(dev), out[-1]))
        e2e = {"value": job_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "chunks_per_step": len(bounds),
               "readback_matches_device": e2e_ok,
               "api": "alpaca_attention (C ABI via ctypes), one call per chunk of sequences; pinned host Q/K/V "
                      "in, f32 context out, every step; copy-in / compute / copy-out on three streams"}
        del hq, hk, hv, hout

    # ---- decode (config 3)
    decode = run_decode(args, ab, torch, dev, stream, rank, world, pg, pk) if not args.no_decode else None

    # ---- RoPE + KV-cache append (the step upstream of attention), config-2 prefill shape
    rope_kv = run_rope(args, ab, torch, dev, stream, rank, world, pg, pk) if not args.no_rope else None

    # ---- CPU baseline (rank 0 at N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        tf, sample, cores = cpu_prefill_sample(args.cpu_seconds, oracle.host_threads(), T)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}

    if pg is not None:
        pg.barrier()
    if rank == 0:
        roof = {"bound": "tensor", "achieved": kernel_tflops, "peak": pk["tflops"], "unit": "TFLOP/s",
                "frac": kernel_tflops / pk["tflops"], "traffic": profile_traffic("prefill_sm100_cfg2"),
                "peak_source": f"{pk['source']}: MEASURED_PEAKS.json bf16_tflops (dense, burst)",
                "kernel": "alpaca::prefill_kernel (tcgen05, persistent)",
                "algorithmic_flops_per_launch": flops_step}
        in_mb = (q.numel() + k.numel() + v.numel()) * 2 / 1e6
        if args.workload == "cfg4":
            cfg = {"workload": f"config 4: SmolLM2-360M causal GQA prefill, 8 sequences x T={T}, 15/5 heads, d=64, "
                               f"split by sequence over {world} GPU(s)", "tokens": T, "sequences": total_seqs,
                   "heads": nh, "kv_heads": nkv, "head_dim": D, "parallelism": f"sequence-sharded x{world}",
                   "l2": f"inputs {in_mb:.0f} MB per rank per step (no flush)"}
            scaling = "strong"
        else:
            cfg = {"workload": f"config 2: SmolLM2-135M causal GQA prefill, T={T}, {L} independent layers "
                               f"per step, 9/3 heads, d=64, f16 in / f32 out", "tokens": T, "layers": L,
                   "heads": nh, "kv_heads": nkv, "head_dim": D, "batch_per_gpu": 1,
                   "parallelism": f"independent sequences per GPU x{world}",
                   "l2": f"inputs {in_mb:.0f} MB per step vs 126 MB L2 (no flush)"}
            scaling = "weak"
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "f16", "data": "synthetic N(0,1) (torch.randn seeded per rank)",
            "config": cfg,
            "tokens_per_s": tokens_per_s,
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": 0 if args.no_prefill else args.steps,
            "clocks": clk,
            "decode": decode,
            "rope_kv_append": rope_kv,
            "spot_check_max_abs": spot,
            "gather_ms": gather_ms,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


def run_cfg5(args):
    """Config 5: SmolLM2-1.7B shape (32/32 heads, d=64) ragged mixed batch — 256 prefill sequences with lengths
    log-uniform in [128, 8192] and 512 one-token decode sequences over f16 caches of 1..8192 rows — whole sequences
    packed over the ranks longest-processing-time first. Per rank one step = one prefill call per sequence (spread
    over 4 streams) + one ragged decode call, captured in a CUDA graph and replayed. With --paged every sequence's
    K/V rows live in one shared pool of 256-row blocks in shuffled order (per-sequence block tables), the serving
    layout, instead of a buffer per prefill sequence and a decode cache padded to the longest context."""
    import numpy as np
    import torch

    import alpaca_b200 as ab
    from alpaca_b200 import Kernel
    from alpaca_b200.partition import Unit, partition
    rank, world, local, pg = dist_setup(args.gpus)
    ab.load()
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    pk = peaks()
    NH = NKV = 32
    rng = np.random.default_rng(20260105)
    pre_T = np.round(np.exp(rng.uniform(np.log(128), np.log(8192), 256))).astype(int)
    dec_L = rng.integers(1, 8192 + 1, 512)
    units = [Unit(i, 0, int(t), 0, NH) for i, t in enumerate(pre_T)] + \
            [Unit(256 + i, 0, 1, int(l) - 1, NH) for i, l in enumerate(dec_L)]
    plan = partition(units, world, tflops=pk["tflops"] * 0.4, hbm_gbs=pk["hbm_gbs"] * 0.6)
    mine = plan.ranks[rank]
    my_pre = [int(pre_T[u.seq]) for u in mine if u.seq < 256]
    my_dec = [int(dec_L[u.seq - 256]) for u in mine if u.seq >= 256]
    g = torch.Generator(device=dev)
    g.manual_seed(20260105 + 1000 * rank)
    nd = len(my_dec)
    cap = max(my_dec) if nd else 1
    kv_bytes = 0
    if args.paged:
        # one pool of R-row blocks for every sequence of this rank, handed out in a shuffled order
        R = PAGED_BLOCK_ROWS
        nb_pre = [-(-T // R) for T in my_pre]
        nb_dec = [-(-L // R) for L in my_dec]
        total = max(1, sum(nb_pre) + sum(nb_dec))
        order = torch.randperm(total, generator=torch.Generator().manual_seed(20260106 + rank)).to(torch.int32)
        kpool = torch.randn((total, R, NKV, D), generator=g, device=dev, dtype=torch.float16)
        vpool = torch.randn((total, R, NKV, D), generator=g, device=dev, dtype=torch.float16)
        kv_bytes = 2 * kpool.numel() * 2
        nxt = 0
        pre = []
        for T, nb in zip(my_pre, nb_pre):
            tab = order[nxt:nxt + nb].reshape(1, nb).to(dev).contiguous()
            nxt += nb
            q = torch.randn((T, NH, D), generator=g, device=dev).half()
            o = torch.empty((T, NH, D), dtype=torch.float32, device=dev)
            pre.append((q, tab, o, ab.make_desc(q, kpool, vpool, o, block_table=tab)))
        mb = max(nb_dec) if nd else 1
        dtab = torch.zeros((max(nd, 1), mb), dtype=torch.int32)
        for i, nb in enumerate(nb_dec):
            dtab[i, :nb] = order[nxt:nxt + nb]
            nxt += nb
        dtab = dtab.to(dev)
        dk, dv = kpool, vpool
    else:
        # prefill: each sequence in its own buffers
        pre = []
        for T in my_pre:
            q = torch.randn((T, NH, D), generator=g, device=dev).half()
            k = torch.randn((T, NKV, D), generator=g, device=dev).half()
            v = torch.randn((T, NKV, D), generator=g, device=dev).half()
            o = torch.empty((T, NH, D), dtype=torch.float32, device=dev)
            kv_bytes += 2 * k.numel() * 2
            pre.append((q, k, v, o, ab.make_desc(q, k, v, o)))
        # decode: one ragged batch
        dk = torch.randn((max(nd, 1), cap, NKV, D), generator=g, device=dev).half()
        dv = torch.randn((max(nd, 1), cap, NKV, D), generator=g, device=dev).half()
        kv_bytes += 2 * dk.numel() * 2
        dtab = None
    dq = torch.randn((max(nd, 1), 1, NH, D), generator=g, device=dev)
    do = torch.empty((max(nd, 1), 1, NH, D), dtype=torch.float32, device=dev)
    lens = torch.tensor(my_dec if nd else [1], dtype=torch.int32, device=dev)
    ddesc = ab.make_desc(dq, dk, dv, do, ctx_lens=lens, max_ctx_len=cap, block_table=dtab)
    ws = torch.empty(max(16, ab.workspace_bytes(ddesc, Kernel.DECODE_SPLIT)), dtype=torch.uint8, device=dev)
    streams = [torch.cuda.Stream(device=dev) for _ in range(4)]

    def step():
        cur = torch.cuda.current_stream()
        ev = torch.cuda.Event()
        ev.record(cur)
        order = sorted(range(len(pre)), key=lambda i: -my_pre[i])  # longest first across the streams
        for n, i in enumerate(order):
            st = streams[n % len(streams)]
            st.wait_event(ev)
            ab.launch(pre[i][-1], Kernel.PREFILL_TC, None, st)
        if nd:
            ab.launch(ddesc, Kernel.DECODE_SPLIT, ws, cur)
        for st in streams:
            done = torch.cuda.Event()
            done.record(st)
            cur.wait_event(done)

    side = torch.cuda.Stream(device=dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    ab.device_status()
    clocks = ClockSampler(local)
    clocks.start()
    barrier(pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    e1.record(stream)
    barrier(pg)
    clk = clocks.stop()
    ab.device_status()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ms, pg)
    del graph
    job_flops = float(sum(flops_prefill(int(t), NH) for t in pre_T))
    job_kv_bytes = float(sum(int(l) * NKV * D * 4 for l in dec_L))
    tokens = float(pre_T.sum() + len(dec_L))
    if pg is not None:
        pg.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": tokens / (ms_max * 1e-3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic N(0,1) (torch.randn seeded per rank), lengths seeded",
            "config": {"workload": "config 5: SmolLM2-1.7B shape (32/32 heads, d=64) ragged mixed batch: 256 prefill "
                                   "sequences, lengths log-uniform [128, 8192], + 512 decode sequences, contexts "
                                   "U[1, 8192]; whole sequences LPT-packed over the GPUs",
                       "prefill_tokens": int(pre_T.sum()), "decode_tokens": len(dec_L),
                       "parallelism": f"sequence-sharded x{world}", "plan_imbalance": plan.imbalance,
                       "kv_layout": (f"paged: one pool of {PAGED_BLOCK_ROWS}-row blocks per GPU, shuffled block "
                                     f"order, per-sequence block tables" if args.paged else
                                     "contiguous: a buffer per prefill sequence, decode cache padded to the "
                                     "longest context"),
                       "kv_gb_rank0": kv_bytes / 1e9},
            "prefill_tflops_if_alone": job_flops / (ms_max * 1e-3) / 1e12,
            "decode_kv_gbs_if_alone": job_kv_bytes / (ms_max * 1e-3) / 1e9,
            "gpu_launches": args.steps * (len(pre) + (2 if nd else 0)),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


def run_rope(args, ab, torch, dev, stream, rank, world, pg, pk):
    """RoPE of q (in place) + rotated K / raw V appended to an f16 cache, for the config-2 prefill shape: 30 layers
    x T tokens x 9/3 heads x d=64 per step, each layer its own tensors (inputs > L2). HBM-bound; GB/s counts q read
    + written (f32), k and v read (f32) and the cache rows written (f16)."""
    LAYERS, T = args.layers, args.tokens
    g = torch.Generator(device=dev)
    g.manual_seed(20260105 + 1000 * rank)
    q = torch.randn((LAYERS, T, H, D), generator=g, device=dev)
    k = torch.randn((LAYERS, T, KVH, D), generator=g, device=dev)
    v = torch.randn((LAYERS, T, KVH, D), generator=g, device=dev)
    kc = torch.zeros((LAYERS, T, KVH, D), dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    descs = [ab.make_rope_desc(q[l], k[l], v[l], kc[l], vc[l], theta=1e5, start_position=0) for l in range(LAYERS)]

    def step():
        for dd in descs:
            ab.rope_launch(dd)

    side = torch.cuda.Stream(device=dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    steps = max(5, args.steps)
    barrier(pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    barrier(pg)
    ms = e0.elapsed_time(e1) / steps
    ms_max = max_over_ranks(ms, pg)
    del graph
    byts = LAYERS * T * (H * D * 4 * 2 + KVH * D * 4 * 2 + KVH * D * 2 * 2)
    gbs = byts / (ms * 1e-3) / 1e9
    return {"workload": f"RoPE + KV append, config-2 shape: {LAYERS} layers x T={T} tokens, 9/3 heads, d=64, f32 q/k/v "
                        "in, f16 cache out, one call per layer replayed from a CUDA graph",
            "value": world * byts / (ms_max * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_max,
            "tokens_per_s": world * T / (ms_max * 1e-3),  # prompt tokens through all layers per second
            "bytes_per_step": byts,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / pk["hbm_gbs"], "traffic": profile_traffic("rope_kv_cfg2"),
                         "kernel": "alpaca::rope_kv_vec_kernel per layer"},
            "gpu_launches": steps * LAYERS}


def run_decode(args, ab, torch, dev, stream, rank, world, pg, pk):
    from alpaca_b200 import Kernel
    g = torch.Generator(device=dev)
    g.manual_seed(20260103 + 1000 * rank)
    gl = torch.Generator()
    gl.manual_seed(20260103)
    LAYERS = args.dec_layers
    lens = torch.randint(1, DEC_CAP + 1, (LAYERS, DEC_BATCH), generator=gl, dtype=torch.int32)
    lens_d = lens.to(dev)
    kc = torch.randn((LAYERS, DEC_BATCH, DEC_CAP, KVH, D), generator=g, device=dev).half()
    vc = torch.randn((LAYERS, DEC_BATCH, DEC_CAP, KVH, D), generator=g, device=dev).half()
    qd = torch.randn((LAYERS, DEC_BATCH, 1, H, D), generator=g, device=dev)
    od = torch.empty((LAYERS, DEC_BATCH, 1, H, D), dtype=torch.float32, device=dev)
    descs = [ab.make_desc(qd[l], kc[l], vc[l], od[l], ctx_lens=lens_d[l], max_ctx_len=DEC_CAP)
             for l in range(LAYERS)]
    wsb = max(ab.workspace_bytes(dd, Kernel.DECODE_SPLIT) for dd in descs)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)

    def step():  # 30 layers x (split + combine), on the current stream
        for dd in descs:
            ab.launch(dd, Kernel.DECODE_SPLIT, ws)

    # The per-layer launches are captured once in a CUDA graph and replayed (launch-bound otherwise).
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step()
    stream.wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(3, args.warmup)):
        graph.replay()
    ab.device_status()
    steps = max(5, args.steps)
    barrier(pg)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    barrier(pg)
    ab.device_status()
    ms = e0.elapsed_time(e1) / steps
    ms_max = max_over_ranks(ms, pg)
    del graph
    kv_bytes = float(lens.sum().item()) * KVH * D * 2 * 2
    qo_bytes = LAYERS * DEC_BATCH * H * D * 4 * 2
    byts = kv_bytes + qo_bytes
    gbs = byts / (ms * 1e-3) / 1e9

    # The decode step of each layer: RoPE + KV append of the new token at row ctx_len - 1, then the attention, as
    # two calls (alpaca_rope_kv_append + alpaca_attention) and fused (alpaca_attn_decode_rope).
    kn = torch.randn((LAYERS, DEC_BATCH, 1, KVH, D), generator=g, device=dev)
    vn = torch.randn((LAYERS, DEC_BATCH, 1, KVH, D), generator=g, device=dev)
    pos_d = (lens_d - 1).contiguous()
    rdescs = [ab.make_rope_desc(qd[l], kn[l], vn[l], kc[l], vc[l], theta=1e5, positions=pos_d[l])
              for l in range(LAYERS)]

    def step_two_calls():
        for l in range(LAYERS):
            ab.rope_launch(rdescs[l])
            ab.launch(descs[l], Kernel.DECODE_SPLIT, ws)

    def step_fused():
        for l in range(LAYERS):
            ab.decode_rope(qd[l], kn[l], vn[l], kc[l], vc[l], od[l], theta=1e5, ctx_lens=lens_d[l],
                           max_ctx_len=DEC_CAP, workspace=ws)

    step_ms = {}
    for name, fn in (("two_calls", step_two_calls), ("fused", step_fused)):
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        for _ in range(max(3, args.warmup)):
            gr.replay()
        barrier(pg)
        e0.record(stream)
        for _ in range(steps):
            gr.replay()
        e1.record(stream)
        barrier(pg)
        ab.device_status()
        step_ms[name] = max_over_ranks(e0.elapsed_time(e1) / steps, pg)
        del gr
    decode_step = {
        "workload": f"config 3 decode step of {LAYERS} layers: per layer the RoPE + f16 KV append of each sequence's "
                    "new token (row ctx_len - 1), then the split-KV attention",
        "two_calls_ms_per_step": step_ms["two_calls"], "fused_ms_per_step": step_ms["fused"],
        "value": world * DEC_BATCH / (step_ms["fused"] * 1e-3), "unit": "tokens/s",
        "two_calls_tokens_per_s": world * DEC_BATCH / (step_ms["two_calls"] * 1e-3),
        "gpu_launches": steps * LAYERS * 2,
    }
    return {"workload": "config 3: batch 64 one-token decode, contexts U[1,4096], 9/3 heads, d=64, f16 KV, "
                        f"{LAYERS} layers (distinct caches, {kc.numel() * 4 / 1e9:.1f} GB) per step",
            "value": world * byts / (ms_max * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_max,
            "tokens_per_s": world * DEC_BATCH / (ms_max * 1e-3),  # one token per sequence per 30-layer step
            "bytes_per_step": byts,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / pk["hbm_gbs"], "traffic": profile_traffic("decode_split_cfg3"),
                         "kernel": "alpaca::decode_split_kernel<64,3> + decode_combine_kernel per layer, "
                                   "replayed from a CUDA graph"},
            "gpu_launches": steps * LAYERS * 2,
            "decode_step": decode_step}


# ---------------------------------------------------------------------------------------------- reference arm

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    oracle.build()
    thr = oracle.host_threads()
    T = args.tokens
    vals = []
    for i in range(args.warmup + args.steps):
        tf, sample, cores = cpu_prefill_sample(args.ref_seconds, thr, T)
        if i >= args.warmup:
            vals.append(tf)
    value = statistics.median(vals)
    full_step_s = LAYERS * flops_prefill(T) / (value * 1e12)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": full_step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) (SplitMix64 Box-Muller)",
        "config": {"workload": f"config 2: SmolLM2-135M causal GQA prefill, T={T}, {LAYERS} independent layers "
                               f"per step, 9/3 heads, d=64 (CPU reference restatement, sampled rows)",
                   "tokens": T, "layers": LAYERS},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "alpaca.swift is Swift + Metal (no Swift toolchain or Apple GPU here); the reference's CPU "
                "attention (CPUOps.swift:162-274) runs as its C restatement in oracle/ on all host threads; ms_per_step "
                "is the extrapolated time of a full 30-layer step",
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--paged", action="store_true",
                    help="cfg5: K/V of every sequence in one shuffled pool of 256-row blocks (block tables)")
    ap.add_argument("--workload", choices=["cfg2", "cfg4", "cfg5"], default="cfg2",
                    help="cfg2 (default headline, weak scaling), cfg4 (8 x 4096 at 15/5 heads, strong scaling) or "
                         "cfg5 (ragged mixed prefill + decode batch at 32/32 heads, strong scaling)")
    ap.add_argument("--tokens", type=int, default=T_PREFILL)
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-rope", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=0, help="sequences per ABI call in the e2e pipeline (0: 1/6 of them)")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--dec-layers", type=int, default=LAYERS)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=4.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cfg5":
        run_cfg5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

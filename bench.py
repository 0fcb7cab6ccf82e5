#!/usr/bin/env python
"""bench.py — MoE-layer tokens/s of the B200 MoE block (BASELINE metric), plus the decode
HBM bandwidth sub-metric and the other BASELINE configurations as sub-blocks of the line.

Headline workload (N=1, cfg3): one HunyuanImage-3.0 MoE block (H=4096, I=3072, 64 routed + 1
shared SwiGLU expert, top-8), GGUF Q4_0 expert weights, 4096 tokens per step, activations
~N(0,1), router bias ~N(0,0.5) (seeded synthetic data, random-init weights generated on the
device).  A step is one hymoe_forward over the 4096 tokens.

  value  tokens/s with inputs resident in HBM, device time by CUDA events, L2 flushed
         between steps (a 256 MiB write outside the timed events)
  e2e    the same call through the C ABI with pinned HOST buffers: H2D of x and the bias,
         compute, D2H of the output inside the timed region
  roofline  the dominant kernel (grouped gate_up GEMM): algorithmic FLOP per launch / its
         CUDA-event duration, against MEASURED_PEAKS.json bf16 burst (the kernel runs at the
         maximum SM clock inside a 3 ms step)
  parity  rows of the timed 4096-token call against the oracle (N=1), or every row of every
         rank against a single-GPU context of the same layer (N>1)
  cpu_baseline  the reference's own moe_forward_cpu (oracle/_ref, compiled from the
         reference sources) on the same sampled token rows, one host core as written
Sub-blocks: `cfg1` (F32 weights, 256 tokens; N=1), `cfg4` (8192 tokens split over the ranks,
Zipf(1.1) router bias, balanced placement; every N), `stack` (cfg5: 32 Q4_0 blocks layer by
layer on a 4160-token sequence; every N), `decode` (cfg2: Q8_0, 1/8/64 tokens; N=1).

--impl reference times the reference's CPU implementation with all host cores (token
sharded over processes; the MoE is per-token independent) on the same workload.
Under torchrun (N > 1) the layer runs expert-parallel: rank r owns 64/N experts (plus the
router and the shared expert) — by default those of its slots in a placement that balances
the experts' routed rows on a calibration batch (--placement contiguous: experts
[r*64/N, (r+1)*64/N)) — processes its own 4096 tokens, and token rows and results move over
NVLink peer memory inside the timed step (weak scaling: per-GPU tokens fixed).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "hunyuan-image-3-80b.cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

H, I, E, K = 4096, 3072, 64, 8
FLOP_PER_PAIR_GU = 2 * 2 * I * H      # gate_up, per (token, expert) row
FLOP_PER_PAIR_DN = 2 * H * I          # down
FLOP_ROUTER_PER_TOKEN = 2 * E * H
FFN_BYTES = {2: 2 * I * H // 32 * 18 + H * I // 32 * 18, 8: 2 * I * H // 32 * 34 + H * I // 32 * 34}
METRIC = "MoE-layer tokens/s (Q4_0, 4096 tok) at 1/2/4/8 B200; decode HBM GB/s"
CFG1_TOKENS = 256
CFG4_TOKENS = 8192
STACK_LAYERS, STACK_SEQ = 32, 4160
STACK_METRIC = "MoE-stack tokens/s (32 Q4_0 MoE blocks, 4160-token sequence, layer by layer)"
PARITY_ROWS = 12          # oracle-checked rows of the timed call (N=1)
PARITY_ROWS_EP = 4        # oracle-checked rows of rank 0's expert-parallel output (N>1)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=d["hbm_gbs"], tf=d["bf16_tflops"], tf_sus=d["bf16_tflops_sustained"],
                    src="measured")
    return dict(hbm=6650.0, tf=1590.0, tf_sus=1400.0, src="fallback")


def ncu_traffic():
    p = os.path.join(ROOT, "profiles", "ncu_summary.json")
    if os.path.exists(p):
        return json.load(open(p))
    return {}


class Clocks:
    """SM clock and clock-event reasons sampled through NVML every 2 ms during the timed region
    (a background thread; the device is found by its CUDA UUID, else its PCI bus id)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, dev: int):
        import threading
        self.samples, self.mask, self.max_mhz, self.err = [], 0, None, None
        self.stop_ev = threading.Event()
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            props = torch.cuda.get_device_properties(dev)
            h = None
            try:
                h = N.nvmlDeviceGetHandleByUUID("GPU-" + str(props.uuid))
            except Exception:
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                h = N.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons

            def loop():
                while not self.stop_ev.is_set():
                    self.samples.append(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                    self.mask |= int(get_reasons(h))
                    self.stop_ev.wait(0.002)
            self.t = threading.Thread(target=loop, daemon=True)
            self.t.start()
        except Exception as e:  # no NVML: report it instead of a number
            self.t, self.err = None, f"nvml unavailable: {e!r}"[:120]

    def stop(self) -> dict:
        if self.t is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err], "samples": 0}
        self.stop_ev.set()
        self.t.join()
        reasons = sorted(v for k, v in self.REASONS.items() if self.mask & k)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples)}


# --------------------------------------------------------------------------- GPU helpers

def _context(hymoe, torch, T: int, rank: int, world: int, local_rank: int, layers: int = 1):
    """A hymoe context for up to T tokens per call: expert parallel over the job's ranks (rank 0
    makes the NCCL id) or, on one GPU, the whole layer."""
    if world > 1:
        box = [hymoe.nccl_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(box, src=0)
        return hymoe.MoE(H, I, E, K, layers, T, device=local_rank, ep_rank=rank, ep_size=world,
                         nccl_id=box[0])
    return hymoe.MoE(H, I, E, K, layers, T, device=local_rank)


def _balance(m, hymoe, torch, xc, bias, wtype: int, seed: int, world: int, layer: int = 0):
    """Expert placement from a calibration batch xc (its own seed, not the timed tokens): each
    expert's routed rows over all ranks, balanced greedily over the ranks; then every rank
    loads the experts of its slots."""
    T = xc.shape[0]
    out = torch.empty_like(xc)
    idx = torch.empty(T, K, dtype=torch.int32, device=xc.device)
    m.forward_device(layer, xc.data_ptr(), out.data_ptr(), T, bias_ptr=bias.data_ptr(),
                     dbg=hymoe.Debug(None, None, None, idx.data_ptr()))
    torch.cuda.synchronize()
    cal = torch.bincount(idx.flatten().long(), minlength=E)
    torch.distributed.all_reduce(cal)
    place = hymoe.balance_placement(cal.cpu().tolist(), world)
    m.set_placement(layer, place)
    m.synth_layer(layer, wtype, seed, 0.02)
    return place


def _max_over_ranks(torch, dev, *vals):
    t = torch.tensor(list(vals), device=dev, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def _time_steps(torch, stream, step, steps: int, flush, world: int, local_rank: int, dev):
    """`steps` steps, each bracketed by CUDA events on `stream` (an L2 flush outside them when
    `flush` is given), clocks sampled meanwhile; returns (total device ms, max over ranks;
    clock record)."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    clocks = Clocks(local_rank)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for s in range(steps):
        if flush is not None:
            flush.zero_()
        ev[s][0].record(stream)
        step()
        ev[s][1].record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    if world > 1:
        ms = _max_over_ranks(torch, dev, ms)[0]
    return ms, clk


def _row_parity(torch, hymoe, ref1, x, out, idx, bias, world: int, dev) -> dict:
    """Expert-parallel rows against a single-GPU context `ref1` holding all E experts of the
    same seeded layer (the single-GPU path is pinned to the oracle by the N=1 line and the GPU
    tests): this rank's tokens through ref1, compared with the expert-parallel output `out`
    and top-K `idx` of the same tokens; summed over the ranks."""
    T = x.shape[0]
    out1 = torch.empty_like(x)
    lg1 = torch.empty(T, E, device=dev)
    idx1 = torch.empty(T, K, dtype=torch.int32, device=dev)
    ref1.forward_device(0, x.data_ptr(), out1.data_ptr(), T, bias_ptr=bias.data_ptr(),
                        dbg=hymoe.Debug(lg1.data_ptr(), None, None, idx1.data_ptr()))
    torch.cuda.synchronize()
    same_rows = (out1 == out).all(dim=1).sum()
    num = ((out.double() - out1.double()) ** 2).sum()
    den = (out1.double() ** 2).sum()
    srt = torch.sort(lg1, dim=1, descending=True).values
    gap = srt[:, K - 1] - srt[:, K]
    differ = (torch.sort(idx, dim=1).values != torch.sort(idx1, dim=1).values).any(dim=1)
    bad = (differ & (gap > 1e-4)).sum()
    ties = (differ & (gap <= 1e-4)).sum()
    t = torch.stack([same_rows.double(), torch.tensor(float(T), device=dev, dtype=torch.float64),
                     num, den, bad.double(), ties.double()])
    if world > 1:
        torch.distributed.all_reduce(t)
    same_rows, rows, num, den, bad, ties = t.tolist()
    rel = (num / den) ** 0.5 if den > 0 else 0.0
    return {"against": "single-GPU hymoe context holding all 64 experts of the same layer, every row of every rank",
            "rows": int(rows), "bit_identical_rows": int(same_rows), "rel_l2": rel, "rel_l2_tol": 1e-3,
            "topk_mismatches": int(bad), "near_ties_excluded": int(ties),
            "ok": int(bad) == 0 and rel <= 1e-3}


# --------------------------------------------------------------------------- GPU arm

def run_gpu(args, rank: int, world: int, local_rank: int):
    import numpy as np
    import torch
    import hymoe

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    T = args.tokens
    wtype = hymoe.TYPE_Q8_0 if args.wtype == "q8_0" else hymoe.TYPE_Q4_0
    m = _context(hymoe, torch, T, rank, world, local_rank)
    m.synth_layer(0, wtype, args.seed, 0.02)
    # A dedicated stream: torch's default stream has handle 0, which the C ABI reads as
    # "the context's own stream".  Every torch op and event below runs on this stream.
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    m.set_stream(stream.cuda_stream)
    g = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    x = torch.randn(T, H, device=dev, generator=g, dtype=torch.float32)
    if args.bias == "zipf":
        bias = torch.from_numpy(hymoe.zipf_router_bias(args.seed, E)).to(dev)
    else:
        gb = torch.Generator(device=dev).manual_seed(args.seed)
        bias = (torch.randn(E, device=dev, generator=gb) * 0.5).contiguous()
    out = torch.empty_like(x)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        m.forward_device(0, x.data_ptr(), out.data_ptr(), T, bias_ptr=bias.data_ptr())

    place = None
    if world > 1 and args.placement == "balanced":
        gc = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank + 500)
        xc = torch.randn(T, H, device=dev, generator=gc, dtype=torch.float32)
        place = _balance(m, hymoe, torch, xc, bias, wtype, args.seed, world)
        del xc

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # routing statistics of this workload (for the algorithmic FLOP count)
    dbg_idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    dbg = hymoe.Debug(None, None, None, dbg_idx.data_ptr())
    m.forward_device(0, x.data_ptr(), out.data_ptr(), T, bias_ptr=bias.data_ptr(), dbg=dbg)
    torch.cuda.synchronize()
    counts_t = torch.bincount(dbg_idx.flatten().long(), minlength=E)
    counts = counts_t.cpu().numpy()
    if world > 1:  # rows this rank's GEMMs process: its T shared rows + the pairs it receives
        torch.distributed.all_reduce(counts_t)
        el = E // world
        slot_of = place if place is not None else list(range(E))
        mine = [e for e in range(E) if slot_of[e] // el == rank]
        rows = T + int(counts_t[mine].sum())
    else:
        rows = T * K + T
    flop_gu = rows * FLOP_PER_PAIR_GU
    flop_dn = rows * FLOP_PER_PAIR_DN
    flop_total = flop_gu + flop_dn + T * FLOP_ROUTER_PER_TOKEN

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    # The sampler starts before the barrier: NVML initialisation takes a different time on
    # each rank, and a rank that enters the timed loop late makes its peers' first step wait.
    clocks = Clocks(local_rank)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    m.profile(True)
    for s in range(args.steps):
        flush.zero_()
        ev[s][0].record(stream)
        step()
        ev[s][1].record(stream)
    torch.cuda.synchronize()
    m.profile(False)
    prof = m.profile_read()
    clk = clocks.stop()
    if world > 1:
        torch.distributed.barrier()
    dev_ms = sum(a.elapsed_time(b) for a, b in ev)
    t_max = _max_over_ranks(torch, dev, dev_ms)[0] if world > 1 else dev_ms
    ms_per_step = t_max / args.steps
    value = world * T * args.steps / (t_max / 1e3)
    # `out` now holds the last timed step's output: the rows the parity below checks

    # ---- e2e through the C ABI with pinned host buffers
    xh = x.cpu().pin_memory()
    bh = bias.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    for _ in range(2):
        m.forward_device(0, xh.data_ptr(), oh.data_ptr(), T, bias_ptr=bh.data_ptr(), host=True)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e2e_ms = 0.0
    for s in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        m.forward_device(0, xh.data_ptr(), oh.data_ptr(), T, bias_ptr=bh.data_ptr(), host=True)
        b.record(stream)
        b.synchronize()
        e2e_ms += a.elapsed_time(b)
    # copy breakdown from separate profiled calls (events around every copy; not the timed loop)
    if world > 1:
        torch.distributed.barrier()
    m.profile(True)
    n_prof = 3
    for s in range(n_prof):
        m.forward_device(0, xh.data_ptr(), oh.data_ptr(), T, bias_ptr=bh.data_ptr(), host=True)
    m.profile(False)
    pe = m.profile_read()
    mine_e2e = {"rank": rank, "e2e_ms": round(e2e_ms / args.steps, 4),
                "copy_in_ms": round(pe["copy_in"][0] / n_prof, 4),
                "copy_out_ms": round(pe["copy_out"][0] / n_prof, 4),
                "copies_per_step": (pe["copy_in"][1] + pe["copy_out"][1]) // n_prof}
    e2e_ranks = [mine_e2e]
    if world > 1:
        e2e_ranks = [None] * world
        torch.distributed.all_gather_object(e2e_ranks, mine_e2e)
        e2e_ms = _max_over_ranks(torch, dev, e2e_ms)[0]
    e2e_value = world * T * args.steps / (e2e_ms / 1e3)

    pk = peaks()
    gu_ms, gu_n = prof["gate_up"]
    gu_launch_ms = gu_ms / max(gu_n, 1)
    achieved = flop_gu / (gu_launch_ms / 1e3) / 1e12
    tr = ncu_traffic().get("gate_up_q4_0_t4096", {})
    roofline = {"kernel": "gemm_tc_kernel<Q4_0> (grouped gate_up + SwiGLU)", "bound": "tensor",
                "achieved": round(achieved, 1), "peak": pk["tf"], "unit": "TFLOP/s",
                "frac": round(achieved / pk["tf"], 4),
                "peak_src": f"{pk['src']} bf16 burst (the step is 3 ms at the maximum SM clock; "
                            f"sustained {pk['tf_sus']})",
                "traffic": tr.get("dram_bytes_per_launch"),
                "algorithmic_flop_per_launch": flop_gu}
    phases = {k: round(v[0] / args.steps, 4) for k, v in prof.items() if v[1]}
    launches = sum(v[1] for v in prof.values())
    per_rank = None
    if world > 1:  # every rank's rows and phases: the slowest rank sets the step time
        per_rank = [None] * world
        torch.distributed.all_gather_object(per_rank, {"rank": rank, "rows": rows, "phases": phases})
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16",
        "data": f"synthetic (seeded; random-init {args.wtype.upper()} weights generated on device)",
        "config": {"workload": f"cfg3: one MoE block, {args.wtype.upper()} experts, {T} tokens/step/GPU, "
                               f"router bias {'Zipf(1.1) over a seeded expert permutation' if args.bias == 'zipf' else '~N(0,0.5)'}",
                   "model": "HunyuanImage-3.0 MoE block H=4096 I=3072 E=64+1 shared top-8",
                   "global_batch": T * world, "seq_len": T,
                   "parallelism": f"ep{world} (E/{world} experts per GPU; token rows and results over NVLink peer memory)" if world > 1 else "single",
                   "placement": ("greedy balance of each expert's routed rows on a calibration batch (own seed)"
                                 if place is not None else "contiguous (rank r owns experts [r*E/N, (r+1)*E/N))") if world > 1 else None,
                   "l2": "flushed between steps (256 MiB write outside the timed events)"},
        "tflops_total": round(flop_total / (ms_per_step / 1e3) / 1e12, 1),
        "frac_of_peak_total": round(flop_total / (ms_per_step / 1e3) / 1e12 / pk["tf"], 4),
        "phases_ms_per_step": phases,
        "roofline": roofline,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": xh.numel() * 4 + bh.numel() * 4,
                "d2h_bytes_per_step": oh.numel() * 4, "ms_per_step": round(e2e_ms / args.steps, 4),
                "note": "host-pointer calls run in token chunks whose copies overlap the compute; "
                        "copy_in/copy_out: the copies' summed device time per call on each rank, from "
                        "separate profiled calls after the timed loop",
                "ranks": e2e_ranks},
        "gpu_launches": launches,
        "clocks": clk,
        "expert_load": {"max": int(counts.max()), "min": int(counts.min()),
                        "mean": float(counts.mean())},
    }
    if per_rank is not None:
        res["ep_ranks"] = per_rank

    # ---- parity of the timed call's rows
    n_rows = min(T, PARITY_ROWS if world == 1 else PARITY_ROWS_EP)
    sample = np.sort(np.random.default_rng(args.seed + 77).choice(T, size=n_rows, replace=False))
    sel = torch.from_numpy(sample).to(dev)
    xs = x.index_select(0, sel).cpu().numpy()
    outs = out.index_select(0, sel).cpu().numpy()
    idxs = dbg_idx.index_select(0, sel).cpu().numpy()
    bias_np = bias.cpu().numpy()
    ref1 = None
    if world > 1:
        # every row of every rank against a single-GPU context of the same layer
        ref1 = hymoe.MoE(H, I, E, K, 1, CFG4_TOKENS, device=local_rank)
        ref1.synth_layer(0, wtype, args.seed, 0.02)
        ref1.set_stream(stream.cuda_stream)
        res["parity"] = _row_parity(torch, hymoe, ref1, x, out, dbg_idx, bias, world, dev)
        if args.cpu:  # and a few of rank 0's rows against the oracle
            if rank == 0:
                res["parity"]["oracle_rows"] = oracle_rows(args.seed, wtype, xs, outs, idxs, bias_np,
                                                           time_reference=False)[1]
            torch.distributed.barrier()
        res["parity"]["ok"] = res["parity"]["ok"] and res["parity"].get("oracle_rows", {}).get("ok", True)
    elif args.cpu:
        res["cpu_baseline"], res["parity"] = oracle_rows(args.seed, wtype, xs, outs, idxs, bias_np)
        res["parity"]["rows_of"] = f"the last timed {T}-token call (rows {sample.tolist()})"
    m.close()
    del x, out, flush

    if args.subblocks:
        res["cfg4"] = run_cfg4(args, rank, world, local_rank, stream, ref1)
        if ref1 is not None:
            ref1.close()
        if world == 1:
            res["cfg1"] = run_cfg1(args, local_rank, stream)
        res["stack"] = run_stack(args, rank, world, local_rank, sub=True)
    elif ref1 is not None:
        ref1.close()
    if args.decode and world == 1:
        res["decode"] = run_decode(args, local_rank)
    return res


def run_cfg4(args, rank: int, world: int, local_rank: int, stream, ref1=None) -> dict:
    """cfg4: one Q4_0 block on 8192 tokens in total, split evenly over the ranks (strong
    scaling), router bias Zipf(1.1) over a seeded expert permutation, experts placed by the
    balanced placement of a calibration batch.  At N>1 rank 0 also times the same 8192 tokens
    on its own GPU through a single-GPU context (the other ranks wait), which gives the
    sub-block's own scaling efficiency, and every rank's rows are compared with that context."""
    import torch
    import hymoe

    dev = torch.device("cuda", local_rank)
    per = CFG4_TOKENS // world
    wtype = hymoe.TYPE_Q4_0
    m = _context(hymoe, torch, per, rank, world, local_rank)
    m.synth_layer(0, wtype, args.seed, 0.02)
    m.set_stream(stream.cuda_stream)
    bias = torch.from_numpy(hymoe.zipf_router_bias(args.seed, E)).to(dev)
    g = torch.Generator(device=dev).manual_seed(args.seed * 1000 + 4242)
    xall = torch.randn(CFG4_TOKENS, H, device=dev, generator=g, dtype=torch.float32)
    x = xall[rank * per:(rank + 1) * per].contiguous()
    out = torch.empty_like(x)
    if world > 1:
        gc = torch.Generator(device=dev).manual_seed(args.seed * 1000 + 4243)
        xc = torch.randn(CFG4_TOKENS, H, device=dev, generator=gc, dtype=torch.float32)
        _balance(m, hymoe, torch, xc[rank * per:(rank + 1) * per].contiguous(), bias, wtype, args.seed, world)
        del xc
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        m.forward_device(0, x.data_ptr(), out.data_ptr(), per, bias_ptr=bias.data_ptr())

    for _ in range(args.warmup):
        step()
    idx = torch.empty(per, K, dtype=torch.int32, device=dev)
    m.forward_device(0, x.data_ptr(), out.data_ptr(), per, bias_ptr=bias.data_ptr(),
                     dbg=hymoe.Debug(None, None, None, idx.data_ptr()))
    torch.cuda.synchronize()
    steps = args.steps
    ms, clk = _time_steps(torch, stream, step, steps, flush, world, local_rank, dev)
    load = torch.bincount(idx.flatten().long(), minlength=E)
    if world > 1:
        torch.distributed.all_reduce(load)
    value = CFG4_TOKENS * steps / (ms / 1e3)
    res = {"metric": "MoE-layer tokens/s (Q4_0, 8192 tokens in total, Zipf(1.1) router bias)",
           "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
           "ms_per_step": round(ms / steps, 4), "scaling": "strong",
           "config": {"workload": f"cfg4: {CFG4_TOKENS} tokens split over {world} GPU(s) ({per} each), "
                                  "Zipf(1.1) bias over a seeded expert permutation",
                      "placement": "balanced on a calibration batch" if world > 1 else None,
                      "l2": "flushed between steps"},
           "expert_rows": {"max": int(load.max()), "min": int(load.min()), "mean": float(load.double().mean())},
           "clocks": clk}
    if world > 1 and ref1 is not None:
        ref1.set_stream(stream.cuda_stream)
        res["parity"] = _row_parity(torch, hymoe, ref1, x, out, idx, bias, world, dev)
        m.close()
        one = torch.zeros(1, device=dev, dtype=torch.float64)
        if rank == 0:
            o1 = torch.empty_like(xall)

            def step1():
                ref1.forward_device(0, xall.data_ptr(), o1.data_ptr(), CFG4_TOKENS, bias_ptr=bias.data_ptr())

            for _ in range(args.warmup):
                step1()
            ms1, _ = _time_steps(torch, stream, step1, steps, flush, 1, local_rank, dev)
            one[0] = CFG4_TOKENS * steps / (ms1 / 1e3)
        torch.distributed.broadcast(one, src=0)
        v1 = float(one.item())
        res["one_gpu_value"] = round(v1, 1)
        res["efficiency"] = round(value / (world * v1), 4)
    else:
        m.close()
    return res


def run_cfg1(args, local_rank: int, stream) -> dict:
    """cfg1: the reference's own weight type, F32 (stored on the device as F16 tiles for the
    fp16 tensor cores), 256 tokens, no router bias; timed like the headline, with the parity of
    8 sampled rows against the oracle on the F32 weights."""
    import numpy as np
    import torch
    import hymoe

    dev = torch.device("cuda", local_rank)
    T = CFG1_TOKENS
    m = hymoe.MoE(H, I, E, K, 1, T, device=local_rank)
    m.synth_layer(0, hymoe.TYPE_F32, args.seed, 0.02)
    m.set_stream(stream.cuda_stream)
    g = torch.Generator(device=dev).manual_seed(args.seed * 1000 + 256)
    x = torch.randn(T, H, device=dev, generator=g, dtype=torch.float32)
    out = torch.empty_like(x)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        m.forward_device(0, x.data_ptr(), out.data_ptr(), T)

    for _ in range(args.warmup):
        step()
    idx = torch.empty(T, K, dtype=torch.int32, device=dev)
    m.forward_device(0, x.data_ptr(), out.data_ptr(), T, dbg=hymoe.Debug(None, None, None, idx.data_ptr()))
    torch.cuda.synchronize()
    m.profile(True)
    ms, clk = _time_steps(torch, stream, step, args.steps, flush, 1, local_rank, dev)
    m.profile(False)
    prof = m.profile_read()
    m.close()
    pk = peaks()
    flop = T * (K + 1) * (FLOP_PER_PAIR_GU + FLOP_PER_PAIR_DN) + T * FLOP_ROUTER_PER_TOKEN
    tf = flop / (ms / args.steps / 1e3) / 1e12
    res = {"metric": "MoE-layer tokens/s (F32 weights, 256 tokens)",
           "value": round(T * args.steps / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": 1,
           "steps": args.steps, "ms_per_step": round(ms / args.steps, 4),
           "config": {"workload": "cfg1: one MoE block, F32 weights (F16 tiles on the device), 256 tokens, no bias",
                      "l2": "flushed between steps"},
           "tflops_total": round(tf, 1), "frac_of_peak_total": round(tf / pk["tf"], 4),
           "phases_ms_per_step": {k: round(v[0] / args.steps, 4) for k, v in prof.items() if v[1]},
           "clocks": clk}
    if args.cpu:
        sample = np.sort(np.random.default_rng(args.seed + 1).choice(T, size=8, replace=False))
        sel = torch.from_numpy(sample).to(dev)
        res["parity"] = oracle_rows(args.seed, hymoe.TYPE_F32, x.index_select(0, sel).cpu().numpy(),
                                    out.index_select(0, sel).cpu().numpy(),
                                    idx.index_select(0, sel).cpu().numpy(), None, time_reference=False)[1]
    return res


def run_stack(args, rank: int, world: int, local_rank: int, sub: bool = False) -> dict:
    """cfg5: 32 MoE blocks (Q4_0, random-init per layer from one seed) applied layer by layer to
    one 4160-token sequence, x <- x + MoE_l(RMSNorm(x)) with unit RMSNorm weights (the
    post-attention half of src/decoder_layer.cpp:34-42; eps 1e-5), in place
    (HYMOE_PRE_NORM, residual = out = x).  The sequence is split over the ranks, each of which
    holds E/N experts of every layer.  A step is the whole stack; `value` = sequence tokens per
    second (device time, max over ranks); `e2e` adds the upload of x and the download of the
    result through the host API.  As a sub-block of the default line (`sub`) it runs at most
    5 timed steps of about 0.1 s."""
    import numpy as np
    import torch
    import hymoe

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    L = STACK_LAYERS
    steps = min(args.steps, 5) if sub else args.steps
    per = (STACK_SEQ + world - 1) // world
    T = max(0, min(per, STACK_SEQ - rank * per))  # this rank's slice of the sequence
    m = _context(hymoe, torch, per, rank, world, local_rank, layers=L)
    ones = np.ones(H, np.float32)
    for l in range(L):
        m.synth_layer(l, hymoe.TYPE_Q4_0, args.seed, 0.02)
        m.set_norm(l, ones, 1e-5)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    m.set_stream(stream.cuda_stream)
    g = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    x0 = torch.randn(max(T, 1), H, device=dev, generator=g, dtype=torch.float32)[:T]
    x = torch.empty_like(x0)

    def stack(ptr):
        for l in range(L):
            m.forward_device(l, ptr, ptr, T, resid_ptr=ptr, pre_norm=True)

    for _ in range(args.warmup):
        x.copy_(x0)
        stack(x.data_ptr())
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    clocks = Clocks(local_rank)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    m.profile(True)
    for s in range(steps):
        x.copy_(x0)  # every step starts from the same sequence (outside the timed events)
        ev[s][0].record(stream)
        stack(x.data_ptr())
        ev[s][1].record(stream)
    torch.cuda.synchronize()
    m.profile(False)
    prof = m.profile_read()
    clk = clocks.stop()
    dev_ms = sum(a.elapsed_time(b) for a, b in ev)
    e2e_ms = 0.0
    xh = x0.cpu().pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    for s in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        x.copy_(xh, non_blocking=True)
        stack(x.data_ptr())
        oh.copy_(x, non_blocking=True)
        b.record(stream)
        b.synchronize()
        e2e_ms += a.elapsed_time(b)
    if world > 1:
        dev_ms, e2e_ms = _max_over_ranks(torch, dev, dev_ms, e2e_ms)
    m.close()
    ms = dev_ms / steps
    pk = peaks()
    flop = STACK_SEQ * L * ((K + 1) * (FLOP_PER_PAIR_GU + FLOP_PER_PAIR_DN) + FLOP_ROUTER_PER_TOKEN)
    tf = flop / (ms / 1e3) / 1e12 / world
    return {
        "metric": STACK_METRIC, "value": round(STACK_SEQ * steps / (dev_ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded; random-init Q4_0 weights of 32 layers generated on device)",
        "config": {"workload": f"cfg5: {L} MoE blocks layer by layer on a {STACK_SEQ}-token sequence "
                               f"({T} tokens on rank 0), x <- x + MoE(RMSNorm(x)), unit norm weights, no router bias",
                   "model": "HunyuanImage-3.0 MoE block H=4096 I=3072 E=64+1 shared top-8, 32 layers",
                   "global_batch": STACK_SEQ, "seq_len": STACK_SEQ,
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "l2": "weights of 32 layers (44 GB at N=1) far exceed L2"},
        "tflops_per_gpu": round(tf, 1),
        "frac_of_peak_per_gpu": round(tf / pk["tf_sus"], 4),
        "peak_src": f"{pk['src']} bf16 sustained (a 100 ms GEMM loop under the power cap)",
        "phases_ms_per_step": {k: round(v[0] / steps, 4) for k, v in prof.items() if v[1]},
        "e2e": {"value": round(STACK_SEQ * steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": xh.numel() * 4, "d2h_bytes_per_step": oh.numel() * 4,
                "ms_per_step": round(e2e_ms / steps, 4)},
        "gpu_launches": sum(v[1] for v in prof.values()),
        "clocks": clk,
    }


def run_decode(args, local_rank: int) -> dict:
    """cfg2: Q8_0 weights, T = 1/8/64 tokens per step, HBM-bound grouped GEMV/GEMM."""
    import torch
    import hymoe

    dev = torch.device("cuda", local_rank)
    m = hymoe.MoE(H, I, E, K, 1, 64, device=local_rank)
    m.synth_layer(0, hymoe.TYPE_Q8_0, args.seed, 0.02)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    m.set_stream(stream.cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    pk = peaks()
    res = {}
    for T in (1, 8, 64):
        g = torch.Generator(device=dev).manual_seed(args.seed + T)
        x = torch.randn(T, H, device=dev, generator=g)
        out = torch.empty_like(x)
        idx = torch.empty(T, K, dtype=torch.int32, device=dev)
        dbg = hymoe.Debug(None, None, None, idx.data_ptr())
        m.forward_device(0, x.data_ptr(), out.data_ptr(), T, dbg=dbg)
        torch.cuda.synchronize()
        distinct = int(torch.unique(idx).numel())
        nbytes = (distinct + 1) * FFN_BYTES[8] + E * H * 4 + 2 * T * H * 4
        # phase breakdown (eager launches, events per phase)
        m.profile(True)
        for _ in range(5):
            m.forward_device(0, x.data_ptr(), out.data_ptr(), T)
        torch.cuda.synchronize()
        m.profile(False)
        prof = m.profile_read()
        # timed: the decode loop replays a captured CUDA graph of the whole call
        for _ in range(max(args.warmup, 3)):
            m.forward_device(0, x.data_ptr(), out.data_ptr(), T, graph=True)
        steps = max(args.steps, 20)
        tot = 0.0
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            m.forward_device(0, x.data_ptr(), out.data_ptr(), T, graph=True)
            b.record(stream)
            b.synchronize()
            tot += a.elapsed_time(b)
        ms = tot / steps
        steps = 5  # phases above were recorded over 5 eager calls
        gbs = nbytes / (ms / 1e3) / 1e9
        res[f"T{T}"] = {"ms_per_step": round(ms, 4), "algorithmic_bytes": nbytes,
                        "distinct_experts": distinct, "achieved_GBps": round(gbs, 1),
                        "frac_hbm": round(gbs / pk["hbm"], 4),
                        "phases_ms": {k: round(v[0] / steps, 4) for k, v in prof.items() if v[1]}}
    m.close()
    res["peak_GBps"] = pk["hbm"]
    res["weights"] = "Q8_0"
    return res


# --------------------------------------------------------------------------- CPU reference

def _cpu_inputs(n_tokens: int, seed: int):
    """Full-shape Q4_0 layer as the reference consumes it (F32), restricted to the
    experts the sample tokens select; x ~N(0,1).  moe_forward_cpu has no router-bias
    input, so the CPU runs route without it; the per-token cost (shared + 8 experts) is
    the same either way."""
    sys.path.insert(0, ORACLE)
    import numpy as np
    import oracle as O
    orc = O.Oracle()
    x = O.synth_x(orc, seed, n_tokens, H)
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    _, _, _, ti = orc.router(x, rw, K)
    w = O.synth_layer_f32(orc, seed, 0, H, I, E, O.Q4_0, experts=np.unique(ti))
    return O, orc, x, w


def parity_stats(gpu: dict, ref_out, ref_idx, k: int, tol: float = 1e-3, gap: float = 1e-4) -> dict:
    """Bench-line parity of a GPU call against the reference on the same tokens: output
    relative L2 (tolerance 1e-3) and top-K agreement, tokens whose K-th/(K+1)-th logit gap is
    at most 1e-4 excluded as near ties (the reference's pre-softmax logits decide)."""
    import numpy as np
    out = np.asarray(gpu["out"], np.float64)
    ref = np.asarray(ref_out, np.float64)
    rel = float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-30))
    same = ties = bad = 0
    for t in range(ref.shape[0]):
        if np.array_equal(gpu["idx"][t], ref_idx[t]):
            same += 1
            continue
        srt = np.sort(gpu["logits"][t])[::-1]
        if srt[k - 1] - srt[k] <= gap:
            ties += 1
        else:
            bad += 1
    n = ref.shape[0]
    return {"tokens": n, "rel_l2": rel, "rel_l2_tol": tol, "topk_match": same / n,
            "near_ties_excluded": ties, "topk_mismatches": bad, "ok": bad == 0 and rel <= tol}


def oracle_rows(seed: int, wtype: int, xs, gpu_out, gpu_idx, bias, time_reference: bool = True):
    """Sampled rows of a timed GPU call against the CPU checkers, on the same seeded layer.
    parity: the oracle (the C restatement, bit-identical to the reference's moe_forward_cpu) with
    the call's router bias, against the GPU's rows and top-K.  cpu_baseline (time_reference):
    the reference's own moe_forward_cpu (oracle/_ref) on the same rows, one host core as written
    and without the bias it has no input for (same per-token cost); its output must equal the
    oracle's at bias 0 bit for bit.  Returns (cpu_baseline or None, parity)."""
    sys.path.insert(0, ORACLE)
    import numpy as np
    import oracle as O
    orc = O.Oracle()
    xs = np.ascontiguousarray(xs, np.float32)
    n = xs.shape[0]
    rw = orc.fill_normal(E * H, seed, O.stream_id(0, O.KIND_ROUTER), 0.02).reshape(E, H)
    logits, _, _, ti = orc.router(xs, rw, K, bias=bias)
    need = np.unique(ti)
    use_ref = time_reference and O.RefMoE.available()
    if time_reference:
        need = np.union1d(need, orc.router(xs, rw, K)[3])
    w = O.synth_layer_f32(orc, seed, 0, H, I, E, wtype, experts=need)
    o = orc.moe_forward(xs, *w, K, I, bias=bias)
    parity = parity_stats({"out": gpu_out, "idx": gpu_idx, "logits": logits}, o["out"], o["idx"], K)
    parity["against"] = ("oracle: C restatement of moe_forward_cpu (bit-identical to the reference at "
                         "bias 0) with the call's router bias")
    base = None
    if time_reference:
        if use_ref:
            ref = O.RefMoE()
            h = ref.weights(H, I, *w)
            t0 = time.perf_counter()
            r = ref.moe_forward(xs, h, E, H, I, K)
            dt = time.perf_counter() - t0
            ref.free(h)
            o0 = orc.moe_forward(xs, *w, K, I)
            parity["oracle_equals_reference_at_bias0"] = bool(np.array_equal(o0["out"], r["out"]))
            kind = "reference"
        else:
            one = O.Oracle(nthreads=1)
            t0 = time.perf_counter()
            one.moe_forward(xs, *w, K, I)
            dt = time.perf_counter() - t0
            kind = "port"
        base = {"value": round(n / dt, 3), "unit": "tokens/s", "cores": 1, "kind": kind,
                "sample": f"the same {n} token rows through moe_forward_cpu (src/attention.cpp:191-313), "
                          f"F32-dequantised weights, no router bias (the reference has none; same "
                          f"per-token cost), {dt:.2f} s; host has {os.cpu_count()} cores"}
    return base, parity


def run_reference(args, rank: int, world: int) -> dict | None:
    """Reference arm: the reference's CPU path with every host core (persistent workers
    forked after the weight build, each running moe_forward_cpu on its token slice)."""
    if rank != 0:
        return None
    P = len(os.sched_getaffinity(0))
    per = 2
    S = P * per
    O, orc, x, w = _cpu_inputs(S, args.seed)
    use_ref = O.RefMoE.available()
    if use_ref:
        ref = O.RefMoE()
        handle = ref.weights(H, I, *w)
    pipes = []
    for p in range(P):
        r_go, w_go = os.pipe()
        r_done, w_done = os.pipe()
        pid = os.fork()
        if pid == 0:
            os.close(w_go)
            os.close(r_done)
            xs = x[p * per:(p + 1) * per].copy()
            one = O.Oracle(nthreads=1)
            while True:
                b = os.read(r_go, 1)
                if not b or b == b"q":
                    os._exit(0)
                if use_ref:
                    ref.moe_forward(xs, handle, E, H, I, K)
                else:
                    one.moe_forward(xs, *w, K, I)
                os.write(w_done, b"d")
        os.close(r_go)
        os.close(w_done)
        pipes.append((pid, w_go, r_done))

    def step():
        t0 = time.perf_counter()
        for _, wg, _ in pipes:
            os.write(wg, b"g")
        for _, _, rd in pipes:
            os.read(rd, 1)
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        step()
    tot = sum(step() for _ in range(args.steps))
    for pid, wg, rd in pipes:
        os.write(wg, b"q")
        os.waitpid(pid, 0)
    value = S * args.steps / tot
    kind = "reference" if use_ref else "port"
    sample = (f"{S} tokens per step ({per} per process x {P} processes) of the cfg3 workload, "
              f"F32-dequantised Q4_0 weights, no router bias (moe_forward_cpu has none; same "
              f"per-token cost)")
    return {
        "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(tot / args.steps * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": "cfg3: one MoE block, Q4_0 experts (dequantised to F32 as the "
                               "reference holds them), router bias ~N(0,0.5)",
                   "model": "HunyuanImage-3.0 MoE block H=4096 I=3072 E=64+1 shared top-8",
                   "global_batch": S, "seq_len": S, "parallelism": f"{P} CPU processes"},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": P, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# --------------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hymoe", choices=["hymoe", "reference"])
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--bias", default="normal", choices=["normal", "zipf"])
    ap.add_argument("--no-cpu", dest="cpu", action="store_false")
    ap.add_argument("--no-decode", dest="decode", action="store_false")
    ap.add_argument("--no-subblocks", dest="subblocks", action="store_false",
                    help="skip the cfg1 / cfg4 / stack sub-blocks of the default line")
    # weights of the main (timed) workload: cfg3/cfg4 use Q4_0; q8_0 with --tokens 1..64 runs the
    # decode workload through the same path (used for kernel captures)
    ap.add_argument("--wtype", default="q4_0", choices=["q4_0", "q8_0"])
    ap.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                    help="expert placement across ranks (N > 1)")
    ap.add_argument("--stack", action="store_true",
                    help="cfg5 alone: 32 MoE blocks layer by layer on a 4160-token sequence")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    if world > 1:
        import datetime

        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                             device_id=torch.device("cuda", local_rank))
    res = run_stack(args, rank, world, local_rank) if args.stack else run_gpu(args, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Benchmark of the B200 router + expert-map path (one JSON line on rank 0).

Step = one pass of the fused router + expert-map build (kb_router_maps) over one batch of
T tokens of synthetic router logits (fp32 [T, 384] ~ N(0,1), bias ~ N(0, 0.1)); T = 65536
per GPU (the large-T configuration of the metric).  With N GPUs every rank routes its own
T tokens and the ranks all-gather their per-expert counts (the expert-parallel exchange
step) inside the same kernel (kb_router_maps_allgather: its tail stores the counts into the
peers' memory over NVLink and collects theirs); the work per GPU is fixed ("weak" scaling)
and value = N*T / step time.

  value     device-resident throughput: inputs already in HBM, steps replayed from CUDA
            graphs, four rotating 100 MB input sets (together > the 126 MB L2)
  e2e       the same op through the C ABI with pinned host buffers: H2D of the logits and
            D2H of every output inside the timed region
  roofline  algorithmic bytes of the router+map pass (1632 B/token + 6164 B/call) over its
            measured device time, against MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the reference's eager router + map path on the host cores (rank 0, N=1)
  kernels   (N=1) every kernel of the path at every benchmark T: us/call, GB/s, roofline
            fraction, and the reference's eager CPU time of the same call
  decode_chain  the 50-layer chain at T in {1, 32, 256, 8192}; with N GPUs the batch is
            token-sharded T/N per rank with the expert-parallel exchange in every layer
  ep_dispatch   one layer's expert-parallel round trip at 4096 tokens per GPU, checked bit
            for bit (ep_parity) before it is timed

--impl reference times the reference's eager CPU path alone (rank 0; other ranks exit).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "profiling-moe_b200"))

METRIC = "router+expert-map Mtok/s (50-layer non-GEMM decode us/token reported alongside)"
UNIT = "Mtok/s"
E, K = 384, 6
HIDDEN = 6144
BYTES_PER_TOKEN = 1536 + 24 + 24 + 24 + 24      # logits, ids, w, p2u, u2p
BYTES_PER_CALL = 384 * 4 + 385 * 8 + 384 * 4    # bias, offsets, counts


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--tokens", type=int, default=65536, help="tokens per GPU per step")
    p.add_argument("--impl", choices=["kolibri", "reference"], default="kolibri")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--chain-tokens", default="1,32,256,8192",
                   help="batch sizes of the 50-layer decode chain ('' = skip)")
    p.add_argument("--chain-layers", type=int, default=50)
    p.add_argument("--no-kernels", action="store_true",
                   help="skip the per-kernel table (configs 2/3, expansion, finalize, maps)")
    p.add_argument("--only-kernel", default="",
                   help="time one kernel of the per-kernel table alone (profiling runs)")
    p.add_argument("--only-T", type=int, default=0)
    p.add_argument("--no-ep", action="store_true",
                   help="skip the expert-parallel round trip")
    p.add_argument("--exchange", choices=["fused", "separate"], default="fused",
                   help="N > 1: count all-gather inside the router+maps kernel, or as a "
                        "second kernel")
    return p.parse_args()


# ------------------------------------------------------------------------------------
# Clock sampling during the timed region (NVML, every 2 ms)
# ------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device: torch.device):
        self.samples, self.reasons = [], 0
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            h = None
            try:
                props = torch.cuda.get_device_properties(device)
                bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.nv, self.h = pynvml, h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report no clocks rather than fail the bench
            self.err = str(e)

    def _reason_bits(self):
        f = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            self.nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(f(self.h))

    def _run(self):
        while not self.stop.is_set():
            self.sample_once()
            time.sleep(0.002)

    def sample_once(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= self._reason_bits()
        except Exception:
            pass

    def __enter__(self):
        if self.ok:
            self.stop = threading.Event()
            self.sample_once()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.sample_once()
            self.stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": self.err}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16 TFLOP/s of a cuBLAS GEMM burst on this pool (MEASURED_PEAKS.json), else the
    fallback figure."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def ncu_traffic(T: int):
    """DRAM bytes per call of the router+map kernels from the committed ncu summary."""
    p = REPO / "profiles" / "router_maps_dram.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    rec = d.get(str(T))
    return None if rec is None else float(rec["dram_bytes_per_call"])


# ------------------------------------------------------------------------------------
# CPU baseline / reference arm
# ------------------------------------------------------------------------------------
def cpu_reference_rate(T: int, steps: int, warmup: int, budget_s: float):
    from kolibri_b200 import workloads as wl
    from oracle import kolibri_oracle as orc  # CPU baseline leg only
    torch.set_num_threads(os.cpu_count() or 1)
    logits, bias = wl.router_inputs(T, seed=1)
    for _ in range(max(1, warmup)):
        orc.router_maps_eager_reference(logits, bias)
    times = []
    t_all = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        orc.router_maps_eager_reference(logits, bias)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    med = statistics.median(times)
    return {"value": T / med / 1e6, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{len(times)} reps of the eager router+map path at T={T} (median)",
            "ms_per_step": med * 1e3}


def cpu_kernel_times(entries: dict, budget_s: float = 120.0):
    """The reference's eager CPU path of every kernel of the per-kernel table, on the host
    cores, at the same T (median of up to 5 reps after one warm-up, each (kernel, T) capped
    at about 2 s): fills cpu_us_per_call / cpu_cores / cpu_kind into the entries in place."""
    from kolibri_b200 import workloads as wl
    from oracle import kolibri_oracle as orc  # CPU baseline leg only
    torch.set_num_threads(os.cpu_count() or 1)
    t_all = time.perf_counter()
    cache = {}

    def cached(key, make):
        if key not in cache:
            cache.clear()  # one input family at a time (bounded host memory)
            cache[key] = make()
        return cache[key]

    def inputs(name, T):
        if name.startswith("qk_norm_rope"):
            q, k, gq, gk, pos = cached(("qk", T), lambda: wl.qk_inputs(T))
            pos_ = None if name.endswith("rnope") else pos
            return lambda: orc.qk_norm_rope_ref(q, k, gq, gk, pos_, wl.EPS)
        if name in ("sandwich", "post_moe_pre_attn", "add_rms_norm"):
            ni = cached(("norm", T), lambda: wl.norm_inputs(T))
        if name == "sandwich":
            return lambda: orc.sandwich_ref(ni.attn_out, ni.residual, ni.g_post_attn,
                                            ni.g_pre_moe, wl.EPS)
        if name == "post_moe_pre_attn":
            return lambda: orc.post_moe_pre_attn_ref(ni.moe_out, ni.residual, ni.g_post_moe,
                                                     ni.g_pre_attn, wl.EPS)
        if name == "add_rms_norm":
            return lambda: orc.add_post_moe_norm_ref(ni.moe_out, ni.residual, ni.g_post_moe,
                                                     wl.EPS)
        if name.startswith("router_gemm"):   # the reference's eager gate GEMM + router
            def gate_inputs():
                g = torch.Generator().manual_seed(40)
                return (torch.randn(T, wl.HIDDEN, generator=g).to(torch.bfloat16),
                        (0.02 * torch.randn(wl.HIDDEN, wl.NUM_EXPERTS, generator=g)).to(
                            torch.bfloat16), 0.1 * torch.randn(wl.NUM_EXPERTS, generator=g))
            x, wg, b = cached(("gate", T), gate_inputs)
            return lambda: orc.router_eager_reference(orc.router_logits_ref(x, wg), b)
        logits, bias = cached(("router", T), lambda: wl.router_inputs(T, seed=1))
        if name == "router_maps":
            return lambda: orc.router_maps_eager_reference(logits, bias)
        ids, w, *_ = orc.router_maps_eager_reference(logits, bias)
        if name == "expert_maps":
            return lambda: orc.maps_eager_reference(ids)
        _, _, _, _, p2u, u2p = orc.router_maps_eager_reference(logits, bias)
        x = torch.randn(T, wl.HIDDEN).to(torch.bfloat16)
        if name == "expansion":
            return lambda: orc.expansion_ref(x, p2u.numpy())
        rows = torch.randn(T * wl.TOP_K, wl.HIDDEN).to(torch.bfloat16)
        return lambda: orc.finalize_ref(rows, u2p.numpy(), w)

    order = sorted(((name, T) for name, by_t in entries.items() for T in by_t),
                   key=lambda nt: (nt[0].startswith("qk"), nt[0] in ("sandwich", "post_moe_pre_attn",
                                                                      "add_rms_norm"), int(nt[1])))
    for name, T in order:
        rec = entries[name][T]
        if time.perf_counter() - t_all > budget_s:
            rec["cpu_us_per_call"] = None
            continue
        fn = inputs(name, int(T))
        fn()
        times = []
        t0 = time.perf_counter()
        while len(times) < 5 and time.perf_counter() - t0 < 2.0:
            a = time.perf_counter()
            fn()
            times.append(time.perf_counter() - a)
        rec["cpu_us_per_call"] = round(statistics.median(times) * 1e6, 1)
        rec["cpu_cores"] = torch.get_num_threads()
        rec["cpu_kind"] = "port"


def kernel_table(dev, stream, peak, only=None, only_T=0):
    """Per-kernel device timings (kolibri_b200.kbench) at every BASELINE token count."""
    from kolibri_b200 import kbench
    out = {}
    for name, Ts in kbench.KERNEL_T.items():
        if only and name != only:
            continue
        out[name] = {}
        for T in Ts:
            if only_T and T != only_T:
                continue
            out[name][str(T)] = kbench.run_kernel(name, dev, T, peak, stream,
                                                  measured_tensor_peak()[0])
            torch.cuda.empty_cache()
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cb = cpu_reference_rate(args.tokens, args.steps, args.warmup, budget_s=120.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(cb["value"], 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(cb["ms_per_step"], 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        # the same workload keys as the B200 arm's config (the rest of that dict describes
        # the device run: graph replays, L2 policy, the exchange)
        "config": {"workload": f"fused router+expert-maps, T={args.tokens} tokens per GPU, "
                               f"E=384, k=6", "tokens_per_gpu": args.tokens, "experts": E,
                   "top_k": K, "implementation": "eager CPU path on the host cores"},
        "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": round(cb["value"], 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------
# 50-layer decode chain (replicas only: every rank times its own copy at N>1)
# ------------------------------------------------------------------------------------
def _time_graph(g, stream, dev, steps, warmup, world, pg=None):
    """Device time of one replay of g (CUDA events on `stream`, max over ranks), in ms.  With
    N > 1 a device-side barrier of the peer group (pg) precedes the start event, so that no
    rank's first step waits for a rank whose host started later."""
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        if pg is not None and world > 1:
            pg.barrier(stream)
        a.record(stream)
        for _ in range(steps):
            g.replay()
        b.record(stream)
    torch.cuda.synchronize(dev)
    ms = a.elapsed_time(b) / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def decode_chain_times(dev, tokens, n_layers, stream, world=1, steps=20, warmup=3):
    """The 50-layer chain at every batch size.  One GPU: the per-stage graph with and without
    the gate GEMM, the one-launch kernel (T <= 4), and the token-sharded expert-parallel
    layer (self exchange).  N GPUs: batch T is sharded T/N tokens per rank and every layer
    runs the expert-parallel exchange over peer memory (config 4); a batch smaller than N
    (T = 1) runs as replicas (the one-launch kernel on every rank)."""
    from kolibri_b200 import decode_chain as dc
    from kolibri_b200.ep import PeerExpertParallel
    layers = dc.make_layers(n_layers, dev)
    out = {"layers": n_layers, "rnope_layers": sum(L.rnope for L in layers),
           "stages": "qk_norm_rope, sandwich, gate GEMM/GEMV, router+maps, expansion or the "
                     "expert-parallel exchange, post-MoE+pre-attn norm",
           "paths": {"with_gate_gemm": "CUDA graph of per-stage kernels; the gate GEMM and router "
                                       "are kb_router_gemm (tcgen05, routing in its epilogue), "
                                       "then kb_expert_maps",
                     "with_gate_cublas": "the same graph with the gate GEMM on cuBLAS "
                                         "(torch.matmul + fp32 cast + kb_router_maps), as the "
                                         "reference runs it",
                     "non_gemm_only": "the same graph without the gate GEMM",
                     "one_launch_with_gate_gemv": "kb_decode_chain: all layers in one "
                                                  "persistent launch (T <= 4)",
                     "ep_sharded": "T/N tokens per rank; per layer the per-stage kernels, "
                                   "tcgen05 gate GEMM, then the peer-memory count all-gather, "
                                   "dispatch to the 384/N expert owners, identity experts, "
                                   "combine back + finalize as the layer's MoE output"},
           "graph": True, "n_gpus": world, "by_T": {}}
    sharded = [T for T in tokens if T >= world and T % world == 0]
    ep = None
    if sharded:
        ep = PeerExpertParallel(E, K, HIDDEN, max_tokens=max(sharded) // world, device=dev)
    try:
        for T in tokens:
            rec = {}
            if world == 1:
                for key, gemm, gate in (("with_gate_gemm", True, "tcgen05"),
                                        ("with_gate_cublas", True, "cublas"),
                                        ("non_gemm_only", False, "tcgen05")):
                    ch = dc.DecodeChain(T, layers, dev, gate_gemm=gemm, expansion=True, gate=gate)
                    g = ch.capture(stream)
                    ms = _time_graph(g, stream, dev, steps, warmup, world)
                    rec[key] = {"us_per_step": round(ms * 1e3, 2),
                                "us_per_token": round(ms * 1e3 / T, 4),
                                "kb_launches_per_step": ch.launches_per_layer() * n_layers}
                    del g, ch
            if T <= dc.DecodeChain.MEGA_MAX_T and (world == 1 or T not in sharded):
                ch = dc.DecodeChain(T, layers, dev, gate_gemm=True, expansion=True)
                for _ in range(warmup):
                    ch.run_mega(stream)
                torch.cuda.synchronize(dev)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    a.record(stream)
                    for _ in range(steps):
                        ch.run_mega(stream)
                    b.record(stream)
                torch.cuda.synchronize(dev)
                ms = a.elapsed_time(b) / steps
                key = "one_launch_with_gate_gemv" if world == 1 else "replicas_one_launch"
                rec[key] = {"us_per_step": round(ms * 1e3, 2), "us_per_token": round(ms * 1e3 / T, 4),
                            "kb_launches_per_step": 1}
                del ch
            if T in sharded:
                ch = dc.DecodeChain(T // world, layers, dev, gate_gemm=True, ep=ep)
                g = ch.capture(stream)
                ms = _time_graph(g, stream, dev, max(3, steps // 2), warmup, world, ep.pg)
                rec["ep_sharded"] = {"us_per_step": round(ms * 1e3, 2),
                                     "us_per_token": round(ms * 1e3 / T, 4),
                                     "tokens_per_rank": T // world,
                                     "kb_launches_per_step": ch.launches_per_layer() * n_layers,
                                     "exchange_status": ep.pg.status()}
                del g, ch
            out["by_T"][str(T)] = rec
    finally:
        if ep is not None:
            ep.close()
    t1 = out["by_T"].get("1")
    if t1:
        best = t1.get("one_launch_with_gate_gemv") or t1.get("replicas_one_launch") or \
            t1.get("with_gate_gemm")
        out["us_per_token_bs1"] = best["us_per_token"]
    return out


# ------------------------------------------------------------------------------------
# Expert-parallel dispatch + combine (N > 1): count all-gather and token all-to-all
# ------------------------------------------------------------------------------------
def ep_round_trip(dev, world, rank, T=4096, H=HIDDEN, steps=10, warmup=3):
    """One MoE layer's expert-parallel round trip at T tokens per GPU: router + maps, count
    all-gather, dispatch to the owners, identity experts, combine back + finalize.  The timed
    path is the peer-memory exchange (kb_ep_*), replayed from a CUDA graph; before timing it
    is checked bit for bit against the one-GPU finalize(expand(x)) of the same routing and,
    with N > 1, against the collective exchange (ExpertParallel over NCCL), whose eager time
    is reported beside it."""
    import torch.distributed as dist
    from kolibri_b200 import ops
    from kolibri_b200 import workloads as wl
    from kolibri_b200.ep import ExpertParallel, PeerExpertParallel
    g = torch.Generator().manual_seed(31 + rank)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(dev)
    logits, bias = wl.router_inputs(T, seed=41 + rank)
    logits, bias = logits.to(dev), bias.to(dev)
    pep = PeerExpertParallel(E, K, H, max_tokens=T, device=dev)
    graph = None
    try:
        d = pep.dispatch(x, logits, bias)
        out = pep.combine(d, d.rows)
        _, w0, _, _, p2u0, u2p0 = ops.router_maps(logits, bias)
        local = ops.moe_finalize(ops.expand_rows(x, p2u0), u2p0, w0)
        torch.cuda.synchronize(dev)
        R = d.num_rows()
        ok = torch.equal(out, local) and pep.pg.status() == 0
        nccl_ms = None
        if world > 1:
            ref_ep = ExpertParallel(E, K)
            r = ref_ep.dispatch(x, logits, bias)
            rout = ref_ep.combine(r, r.rows)
            ok = ok and torch.equal(rout, local) and R == r.rows.shape[0] and \
                torch.equal(d.rows[:R], r.rows) and torch.equal(d.expert_offsets, r.expert_offsets)
            del r, rout
            for i in range(warmup + steps):     # the collective path, eager (host splits)
                if i == warmup:
                    torch.cuda.synchronize(dev)
                    dist.barrier()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                rr = ref_ep.dispatch(x, logits, bias)
                ref_ep.combine(rr, rr.rows)
            b.record()
            torch.cuda.synchronize(dev)
            t = torch.tensor([a.elapsed_time(b) / steps], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            nccl_ms = float(t.item())
            flag = torch.tensor([1 if ok else 0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            ok = bool(flag.item())
        # rows this rank sends to other ranks (dispatch) and gets back (combine)
        Er = E // world
        mine = d.gathered[rank].view(world, Er).sum(-1)
        sent = int(mine.sum().item()) - int(mine[rank].item())
        ops.reserve_workspace(T)
        s = torch.cuda.Stream(dev)
        obuf = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        with torch.cuda.stream(s):
            dd = pep.dispatch(x, logits, bias)
            pep.combine(dd, dd.rows, obuf)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            dd = pep.dispatch(x, logits, bias)
            pep.combine(dd, dd.rows, obuf)
        ms = _time_graph(graph, s, dev, steps, warmup, world, pep.pg)
        ok = ok and torch.equal(obuf, local) and pep.pg.status() == 0
        if world > 1:
            flag = torch.tensor([1 if ok else 0], device=dev)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            ok = bool(flag.item())
    finally:
        graph = None
        pep.close()
    remote = 2 * sent * H * 2      # rows out to the owners and back; no metadata travels
    res = {"tokens_per_gpu": T, "hidden": H, "experts_per_gpu": E // world, "ep_parity": ok,
           "us_per_step": round(ms * 1e3, 2),
           "stages": "router+maps, peer count all-gather, dispatch (expansion + pack + "
                     "all-to-all in one kernel), identity experts, combine back + finalize",
           "kb_launches_per_step": 5,
           "remote_bytes_per_gpu": remote,
           "remote_GBps_per_gpu": round(remote / (ms * 1e-3) / 1e9, 1) if world > 1 else None,
           "parity": "combine(dispatch(x)) == finalize(expand(x)) bit for bit"
                     + (", rows/segments == the NCCL collective path" if world > 1 else "")}
    if nccl_ms is not None:
        res["nccl_collective_path_us_per_step"] = round(nccl_ms * 1e3, 2)
    return res


# ------------------------------------------------------------------------------------
# B200 arm
# ------------------------------------------------------------------------------------
def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)

    from kolibri_b200 import _lib, ops
    from kolibri_b200 import workloads as wl

    if args.only_kernel == "decode_chain":  # the one-launch chain alone (profiling runs)
        from kolibri_b200 import decode_chain as dc
        ch = dc.DecodeChain(args.only_T or 1, dc.make_layers(args.chain_layers, dev), dev)
        for _ in range(4):
            ch.run_mega(torch.cuda.current_stream(dev))
        torch.cuda.synchronize(dev)
        if rank == 0:
            print(json.dumps({"decode_chain_calls": 4, "T": args.only_T or 1}), flush=True)
        return
    if args.only_kernel == "ep_exchange":  # the expert-parallel round trip alone (profiling)
        res = ep_round_trip(dev, world, rank, T=args.only_T or 4096, steps=3, warmup=1)
        if rank == 0:
            print(json.dumps({"ep_dispatch": res}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    if args.only_kernel:  # one kernel of the per-kernel table alone (profiling runs)
        peak, _ = measured_peak()
        tab = kernel_table(dev, torch.cuda.Stream(dev), peak, args.only_kernel, args.only_T)
        if rank == 0:
            print(json.dumps({"kernels": tab}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    T = args.tokens
    nsets = 4
    sets = []
    for s in range(nsets):
        logits, bias = wl.router_inputs(T, seed=1 + 100 * s + 1000 * rank)
        sets.append((logits.to(dev), bias.to(dev)))
    ids = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, dtype=torch.float32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int64, device=dev)
    p2u = torch.empty(T * K, dtype=torch.int32, device=dev)
    u2p = torch.empty(T * K, dtype=torch.int32, device=dev)
    gathered = torch.empty(world, E, dtype=torch.int32, device=dev)
    lib = _lib.load()
    # N > 1: the per-expert counts are all-gathered by a kernel over peer memory (no NCCL in
    # the step), so the whole step is captured in CUDA graphs at every N.
    counts_pg = None
    if world > 1:
        from kolibri_b200.ep import PeerGroup
        counts_pg = PeerGroup(E, K, 0, 16, device=dev)
    ws_bytes = lib.kb_router_maps_workspace_bytes(T, E, K)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(dev)

    def router_maps(lg, bs, cs):
        """One step: kb_router_maps, or with N > 1 kb_router_maps_allgather (the count
        all-gather fused into the same kernel's tail; --exchange separate: kb_router_maps
        followed by kb_ep_counts_allgather)."""
        if world > 1 and args.exchange == "separate":
            _lib.check(lib.kb_router_maps(lg.data_ptr(), bs.data_ptr(), ids.data_ptr(),
                                          w.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
                                          p2u.data_ptr(), u2p.data_ptr(), ws.data_ptr(), ws_bytes,
                                          T, E, K, 0, _lib.KB_MAPS_AUTO, cs), "kb_router_maps")
            _lib.check(lib.kb_ep_counts_allgather(counts_pg.addr, counts.data_ptr(),
                                                  gathered.data_ptr(), cs),
                       "kb_ep_counts_allgather")
        elif world > 1:
            _lib.check(lib.kb_router_maps_allgather(
                counts_pg.addr, lg.data_ptr(), bs.data_ptr(), ids.data_ptr(), w.data_ptr(),
                counts.data_ptr(), offsets.data_ptr(), p2u.data_ptr(), u2p.data_ptr(),
                ws.data_ptr(), ws_bytes, T, 0, _lib.KB_MAPS_AUTO, gathered.data_ptr(), cs),
                "kb_router_maps_allgather")
        else:
            _lib.check(lib.kb_router_maps(lg.data_ptr(), bs.data_ptr(), ids.data_ptr(),
                                          w.data_ptr(), counts.data_ptr(), offsets.data_ptr(),
                                          p2u.data_ptr(), u2p.data_ptr(), ws.data_ptr(), ws_bytes,
                                          T, E, K, 0, _lib.KB_MAPS_AUTO, cs), "kb_router_maps")

    def step(i):
        lg, bs = sets[i % nsets]
        router_maps(lg, bs, torch.cuda.current_stream(dev).cuda_stream)

    # Graphs: one per input set (router+maps, and the count all-gather for N>1).
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        for i in range(nsets):
            step(i)
    torch.cuda.synchronize(dev)
    graphs = []
    for i in range(nsets):
        gi = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gi, stream=stream):
            step(i)
        graphs.append(gi)
    del gi
    graph_all = torch.cuda.CUDAGraph()  # the nsets steps back to back in one graph
    with torch.cuda.graph(graph_all, stream=stream):
        for i in range(nsets):
            step(i)
    run = lambda i: graphs[i % nsets].replay()  # noqa: E731

    def run_steps(n):
        """n steps in order: whole groups of nsets from the combined graph, the rest singly."""
        i = 0
        if graph_all is not None:
            while i + nsets <= n:
                graph_all.replay()
                i += nsets
        while i < n:
            run(i)
            i += 1
    import ctypes
    path_c, launch_c, grid_c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.check(lib.kb_maps_describe(T, E, K, 1, _lib.KB_MAPS_AUTO, ctypes.byref(path_c),
                                    ctypes.byref(launch_c), ctypes.byref(grid_c)),
               "kb_maps_describe")
    launches_per_step = launch_c.value
    path_name = {1: "single-CTA", 2: "tile kernel, persistent multi-CTA", 3: "two-kernel",
                 4: "hybrid-router persistent", 5: "warp-router persistent"}[path_c.value]

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            run(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(dev)
    with clocks:
        with torch.cuda.stream(stream):
            if world > 1:
                counts_pg.barrier(stream)   # the ranks enter the timed region together
            start.record(stream)
            run_steps(args.steps)
            end.record(stream)
        torch.cuda.synchronize(dev)
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T / (ms * 1e-3) / 1e6

    # Roofline of the router+map pass (1 GPU: the whole step is that pass).
    peak, peak_kind = measured_peak()
    alg_bytes = BYTES_PER_TOKEN * T + BYTES_PER_CALL
    achieved = alg_bytes / (ms * 1e-3) / 1e9
    traffic = ncu_traffic(T)

    # e2e through the C ABI with host buffers.
    e2e = None
    if not args.no_e2e:
        lg_h = sets[0][0].cpu().pin_memory()
        bs_h = sets[0][1].cpu().pin_memory()
        lg_d = torch.empty_like(sets[0][0])
        bs_d = torch.empty_like(sets[0][1])
        outs = [ids, w, counts, offsets, p2u, u2p]
        outs_h = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
        h2d = lg_h.numel() * 4 + bs_h.numel() * 4
        d2h = sum(o.numel() * o.element_size() for o in outs)

        def e2e_step():
            cs = torch.cuda.current_stream(dev)
            lg_d.copy_(lg_h, non_blocking=True)
            bs_d.copy_(bs_h, non_blocking=True)
            router_maps(lg_d, bs_d, cs.cuda_stream)
            for o, oh in zip(outs, outs_h):
                oh.copy_(o, non_blocking=True)

        e_steps = max(3, min(args.steps, 50))
        with torch.cuda.stream(stream):
            for _ in range(3):
                e2e_step()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        with torch.cuda.stream(stream):
            if world > 1:
                counts_pg.barrier(stream)
            start.record(stream)
            for _ in range(e_steps):
                e2e_step()
            end.record(stream)
        torch.cuda.synchronize(dev)
        ems = start.elapsed_time(end) / e_steps
        if world > 1:
            t = torch.tensor([ems], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ems = float(t.item())
        e2e = {"value": round(world * T / (ems * 1e-3) / 1e6, 4), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(ems, 4), "steps": e_steps}

    # N > 1: the last step's all-gathered counts against NCCL's all-gather of the same counts.
    count_parity = None
    if world > 1:
        torch.cuda.synchronize(dev)
        nccl_counts = torch.empty(world, E, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(nccl_counts, counts)
        flag = torch.tensor([1 if (torch.equal(nccl_counts, gathered) and
                                   counts_pg.status() == 0) else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        count_parity = bool(flag.item())

    ep = ep_round_trip(dev, world, rank) if not args.no_ep else None

    kernels = None
    if not args.no_kernels and world == 1:
        kernels = kernel_table(dev, stream, peak)
        if rank == 0 and not args.no_cpu_baseline:
            cpu_kernel_times(kernels)

    chain = None
    if args.chain_tokens:
        chain = decode_chain_times(dev, [int(t) for t in args.chain_tokens.split(",") if t],
                                   args.chain_layers, stream, world=world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_reference_rate(T, steps=20, warmup=1, budget_s=20.0)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}

    # Every graph is released before the exchange buffers and the process group go.
    run = None
    graphs.clear()
    graph_all = None
    if world > 1:
        dist.barrier()
        counts_pg.close()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic",
        "config": {"workload": f"fused router+expert-maps, T={T} tokens per GPU, E=384, k=6",
                   "tokens_per_gpu": T, "experts": E, "top_k": K,
                   "l2": "4 rotating input sets of 100 MB (> 126 MB L2 together)",
                   "graph": True,
                   "steps_per_graph_replay": nsets,
                   "parallelism": f"token-sharded x{world}" + (
                       (" + per-expert count all-gather over peer memory, fused into the "
                        "router+maps kernel (kb_router_maps_allgather)")
                       if args.exchange == "fused" else
                       (" + per-expert count all-gather over peer memory "
                        "(kb_ep_counts_allgather after kb_router_maps)")
                       if world > 1 else "")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "algorithmic_bytes": alg_bytes, "peak_source": peak_kind,
                     "kernel": f"kb_router_maps ({path_name}, grid {grid_c.value})"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "decode_chain": chain,
        "kernels": kernels,
        "ep_dispatch": ep,
        "count_exchange_parity": count_parity,
        "gpu_launches": (launches_per_step + (1 if world > 1 and args.exchange == "separate"
                                              else 0)) * args.steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()

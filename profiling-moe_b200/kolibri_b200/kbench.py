"""Per-kernel timing of the hot-path entry points on the GPU (device-resident inputs).

Every measurement captures a CUDA graph of `reps` back-to-back calls that cycle through
`nsets` independent input sets, replays it after warm-up and divides the CUDA-event time of
the replays by the calls.  Where one set is smaller than twice the 126 MB L2, enough sets are
cycled that the data of consecutive calls do not share L2 (large T); at decode T everything
fits in L2 anyway and the figure is launch + SM time.

Algorithmic bytes per unit (the compulsory reads and writes of each kernel):
  qk_norm_rope      36 864 B/token (72 heads x 128 bf16 read + written) + 4 B position
                    + 512 B of gammas per call
  sandwich / post_moe_pre_attn (kb_residual_norm_pair)
                    49 152 B/token (2 rows read, 2 written) + 24 576 B of gammas per call
  add_rms_norm      36 864 B/token (2 rows read, 1 written) + 12 288 B of gamma per call
  expansion         rows x (12 288 written + 4 B p2u) + T x 12 288 read (each source row once)
  finalize          T*K x 12 288 read + T x 12 288 written + T*K x (4 B u2p + 4 B weight)
  router_maps       1632 B/token + 6164 B per call
  expert_maps       72 B/token + 4 616 B per call
  router_gemm       x read (12 288 B/token) + gate weight read once (E x H x 2 = 4 718 592 B
                    per call) + logits written (1536 B/token) + ids and weights (48 B/token);
                    2 x T x H x E flops.  Its roofline is the slower of bytes / HBM peak and
                    flops / tensor peak (the weight read bounds small T, the flops large T).
  router_gemm_cublas
                    the same work as the reference runs it: torch.matmul (cuBLAS, bf16 out),
                    the cast to fp32 and kb_router on the logits
"""
from __future__ import annotations

from typing import Callable, Dict, List

import torch

from . import _lib, ops
from . import workloads as wl

L2_BYTES = 126 * 1024 * 1024
ROW = wl.HIDDEN * 2                      # one bf16 hidden row
HEADS = wl.HQ + wl.HKV


def nsets_for(bytes_per_set: int, cap_bytes: int = 3 << 30) -> int:
    """Input sets to cycle so that consecutive calls' data exceed twice the L2 (at most 16)."""
    if bytes_per_set <= 0:
        return 1
    n = max(1, -(-2 * L2_BYTES // bytes_per_set))
    n = min(n, 16, max(1, cap_bytes // bytes_per_set))
    return int(n)


def time_calls(launch: Callable[[int], None], nsets: int, stream: torch.cuda.Stream,
               reps: int = 16, warmup: int = 3, iters: int = 10) -> float:
    """Microseconds per call of launch(i) (i cycles over the input sets), from a CUDA graph
    of `reps` calls replayed `iters` times after `warmup` replays."""
    reps = max(reps, nsets)
    with torch.cuda.stream(stream):
        for i in range(nsets):  # eager run first: library set-up, workspaces
            launch(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            launch(i % nsets)
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(iters):
            g.replay()
        b.record(stream)
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (iters * reps)
    del g
    return us


def _entry(us: float, T: int, nbytes: float, peak: float, nsets: int) -> dict:
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"us_per_call": round(us, 3), "tokens_per_s": round(T / (us * 1e-6), 1),
            "GBps": round(gbs, 1), "frac": round(gbs / peak, 4),
            "algorithmic_bytes": int(nbytes), "input_sets": nsets}


def bench_qk(dev, T: int, rnope: bool, peak: float, stream) -> dict:
    per_set = T * HEADS * 128 * 2 * 2
    n = nsets_for(per_set)
    sets = []
    for i in range(n):
        q, k, gq, gk, pos = wl.qk_inputs(T, seed=2 + 17 * i)
        sets.append([t.to(dev) for t in (q, k, gq, gk, pos)])
    outs = [(torch.empty_like(s[0]), torch.empty_like(s[1])) for s in sets]
    lib = _lib.load()
    inv = ops.rope_inv_freq(wl.ROPE_THETA, 128, dev)

    def launch(i):
        q, k, gq, gk, pos = sets[i]
        qo, ko = outs[i]
        _lib.check(lib.kb_qk_norm_rope(q.data_ptr(), qo.data_ptr(), k.data_ptr(), ko.data_ptr(),
                                       gq.data_ptr(), gk.data_ptr(),
                                       None if rnope else pos.data_ptr(),
                                       None if rnope else inv.data_ptr(), T, wl.HQ, wl.HKV, 128,
                                       wl.HQ * 128, wl.HKV * 128, wl.EPS,
                                       torch.cuda.current_stream(dev).cuda_stream),
                   "kb_qk_norm_rope")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * (HEADS * 128 * 2 * 2 + 4) + 512, peak, n)


def bench_pair(dev, T: int, which: str, peak: float, stream) -> dict:
    """which: 'sandwich' (attn_out, residual) or 'post_moe_pre_attn' (moe_out, h)."""
    per_set = T * ROW * 4
    n = nsets_for(per_set)
    sets = []
    for i in range(n):
        ni = wl.norm_inputs(T, seed=3 + 31 * i)
        if which == "sandwich":
            a, r, g1, g2 = ni.attn_out, ni.residual, ni.g_post_attn, ni.g_pre_moe
        else:
            a, r, g1, g2 = ni.moe_out, ni.residual, ni.g_post_moe, ni.g_pre_attn
        sets.append([t.to(dev) for t in (a, r, g1, g2)] +
                    [torch.empty(T, wl.HIDDEN, dtype=torch.bfloat16, device=dev) for _ in range(2)])
    lib = _lib.load()

    def launch(i):
        a, r, g1, g2, so, no = sets[i]
        _lib.check(lib.kb_residual_norm_pair(a.data_ptr(), r.data_ptr(), g1.data_ptr(),
                                             g2.data_ptr(), so.data_ptr(), no.data_ptr(), T,
                                             wl.HIDDEN, wl.EPS, _lib.KB_BF16,
                                             torch.cuda.current_stream(dev).cuda_stream),
                   "kb_residual_norm_pair")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * ROW * 4 + 2 * ROW, peak, n)


def bench_add_norm(dev, T: int, peak: float, stream) -> dict:
    per_set = T * ROW * 3
    n = nsets_for(per_set)
    sets = []
    for i in range(n):
        ni = wl.norm_inputs(T, seed=5 + 13 * i)
        sets.append([t.to(dev) for t in (ni.moe_out, ni.residual, ni.g_post_moe)] +
                    [torch.empty(T, wl.HIDDEN, dtype=torch.bfloat16, device=dev)])
    lib = _lib.load()

    def launch(i):
        a, b, g, o = sets[i]
        _lib.check(lib.kb_add_rms_norm(a.data_ptr(), b.data_ptr(), g.data_ptr(), o.data_ptr(),
                                       None, T, wl.HIDDEN, wl.EPS, _lib.KB_BF16,
                                       torch.cuda.current_stream(dev).cuda_stream),
                   "kb_add_rms_norm")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * ROW * 3 + ROW, peak, n)


def _routing(dev, T: int, seed: int):
    logits, bias = wl.router_inputs(T, seed=seed)
    ids, w, c, off, p2u, u2p = ops.router_maps(logits.to(dev), bias.to(dev))
    return w, p2u, u2p


def bench_expansion(dev, T: int, peak: float, stream) -> dict:
    K = wl.TOP_K
    per_set = T * ROW * (K + 1)
    n = nsets_for(per_set)
    sets = []
    for i in range(n):
        g = torch.Generator().manual_seed(40 + i)
        x = torch.randn(T, wl.HIDDEN, generator=g).to(torch.bfloat16).to(dev)
        _, p2u, _ = _routing(dev, T, 50 + i)
        sets.append((x, p2u, torch.empty(T * K, wl.HIDDEN, dtype=torch.bfloat16, device=dev)))
    lib = _lib.load()

    def launch(i):
        x, p2u, out = sets[i]
        _lib.check(lib.kb_expand_rows(x.data_ptr(), out.data_ptr(), p2u.data_ptr(), T, T * K,
                                      ROW, torch.cuda.current_stream(dev).cuda_stream),
                   "kb_expand_rows")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * K * (ROW + 4) + T * ROW, peak, n)


def bench_finalize(dev, T: int, peak: float, stream) -> dict:
    K = wl.TOP_K
    per_set = T * ROW * (K + 1)
    n = nsets_for(per_set)
    sets = []
    for i in range(n):
        g = torch.Generator().manual_seed(60 + i)
        rows = torch.randn(T * K, wl.HIDDEN, generator=g).to(torch.bfloat16).to(dev)
        w, _, u2p = _routing(dev, T, 70 + i)
        sets.append((rows, u2p, w, torch.empty(T, wl.HIDDEN, dtype=torch.bfloat16, device=dev)))
    lib = _lib.load()

    def launch(i):
        rows, u2p, w, out = sets[i]
        _lib.check(lib.kb_moe_finalize(rows.data_ptr(), u2p.data_ptr(), w.data_ptr(),
                                       out.data_ptr(), T, K, wl.HIDDEN, _lib.KB_BF16,
                                       torch.cuda.current_stream(dev).cuda_stream),
                   "kb_moe_finalize")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * K * ROW + T * ROW + T * K * 8, peak, n)


def bench_router_maps(dev, T: int, peak: float, stream) -> dict:
    E, K = wl.NUM_EXPERTS, wl.TOP_K
    per_set = T * 1632
    n = nsets_for(per_set)
    lib = _lib.load()
    sets = []
    for i in range(n):
        logits, bias = wl.router_inputs(T, seed=1 + 100 * i)
        sets.append((logits.to(dev), bias.to(dev)))
    outs = [torch.empty(T, K, dtype=torch.int32, device=dev), torch.empty(T, K, device=dev),
            torch.empty(E, dtype=torch.int32, device=dev),
            torch.empty(E + 1, dtype=torch.int64, device=dev),
            torch.empty(T * K, dtype=torch.int32, device=dev),
            torch.empty(T * K, dtype=torch.int32, device=dev)]
    wsb = lib.kb_router_maps_workspace_bytes(T, E, K)
    ws = torch.zeros(max(wsb, 256), dtype=torch.uint8, device=dev)

    def launch(i):
        lg, b = sets[i]
        _lib.check(lib.kb_router_maps(lg.data_ptr(), b.data_ptr(), *[o.data_ptr() for o in outs],
                                      ws.data_ptr(), wsb, T, E, K, 0, _lib.KB_MAPS_AUTO,
                                      torch.cuda.current_stream(dev).cuda_stream),
                   "kb_router_maps")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * 1632 + 6164, peak, n)


def bench_expert_maps(dev, T: int, peak: float, stream) -> dict:
    E, K = wl.NUM_EXPERTS, wl.TOP_K
    n = nsets_for(T * 72)
    lib = _lib.load()
    sets = []
    for i in range(n):
        logits, bias = wl.router_inputs(T, seed=1 + 7 * i)
        ids, *_ = ops.router_maps(logits.to(dev), bias.to(dev))
        sets.append(ids)
    outs = [torch.empty(E, dtype=torch.int32, device=dev),
            torch.empty(E + 1, dtype=torch.int64, device=dev),
            torch.empty(T * K, dtype=torch.int32, device=dev),
            torch.empty(T * K, dtype=torch.int32, device=dev)]
    wsb = lib.kb_expert_maps_workspace_bytes(T, E, K)
    ws = torch.zeros(max(wsb, 256), dtype=torch.uint8, device=dev)

    def launch(i):
        _lib.check(lib.kb_expert_maps(sets[i].data_ptr(), *[o.data_ptr() for o in outs],
                                      ws.data_ptr(), wsb, T, E, K, _lib.KB_MAPS_AUTO,
                                      torch.cuda.current_stream(dev).cuda_stream),
                   "kb_expert_maps")
    us = time_calls(launch, n, stream)
    return _entry(us, T, T * 72 + 384 * 4 + 385 * 8, peak, n)


def _gate_sets(dev, T: int):
    E, H = wl.NUM_EXPERTS, wl.HIDDEN
    per_set = T * H * 2 + E * H * 2
    n = nsets_for(per_set)
    sets = []
    for i in range(n):
        g = torch.Generator(device=dev).manual_seed(40 + i)
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        w = (0.02 * torch.randn(E, H, generator=g, device=dev)).to(torch.bfloat16)
        b = 0.1 * torch.randn(E, generator=g, device=dev)
        sets.append((x, w, b))
    return sets, n


def _gate_entry(us: float, T: int, peak: float, tflops_peak: float, nsets: int) -> dict:
    E, K, H = wl.NUM_EXPERTS, wl.TOP_K, wl.HIDDEN
    nbytes = T * H * 2 + E * H * 2 + T * E * 4 + T * K * 8
    flops = 2.0 * T * H * E
    t_hbm, t_tc = nbytes / (peak * 1e9), flops / (tflops_peak * 1e12)
    e = _entry(us, T, nbytes, peak, nsets)
    e.update({"TFLOPs": round(flops / (us * 1e-6) / 1e12, 2),
              "bound": "hbm" if t_hbm >= t_tc else "tensor",
              "frac": round(max(t_hbm, t_tc) / (us * 1e-6), 4), "flops": flops})
    return e


def bench_router_gemm(dev, T: int, peak: float, stream, tflops_peak: float) -> dict:
    E, K, H = wl.NUM_EXPERTS, wl.TOP_K, wl.HIDDEN
    sets, n = _gate_sets(dev, T)
    lib = _lib.load()
    logits = torch.empty(T, E, device=dev)
    ids = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, device=dev)
    wsb = lib.kb_router_gemm_workspace_bytes(T, H, E, K)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)

    def launch(i):
        x, wg, b = sets[i]
        _lib.check(lib.kb_router_gemm(x.data_ptr(), wg.data_ptr(), b.data_ptr(), logits.data_ptr(),
                                      ids.data_ptr(), w.data_ptr(), ws.data_ptr(), wsb, T, H, E, K,
                                      0, torch.cuda.current_stream(dev).cuda_stream),
                   "kb_router_gemm")
    us = time_calls(launch, n, stream)
    return _gate_entry(us, T, peak, tflops_peak, n)


def bench_router_gemm_cublas(dev, T: int, peak: float, stream, tflops_peak: float) -> dict:
    E, K = wl.NUM_EXPERTS, wl.TOP_K
    sets, n = _gate_sets(dev, T)
    lib = _lib.load()
    lbf = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
    logits = torch.empty(T, E, device=dev)
    ids = torch.empty(T, K, dtype=torch.int32, device=dev)
    w = torch.empty(T, K, device=dev)

    def launch(i):
        x, wg, b = sets[i]
        torch.matmul(x, wg.t(), out=lbf)
        logits.copy_(lbf)
        _lib.check(lib.kb_router(logits.data_ptr(), b.data_ptr(), ids.data_ptr(), w.data_ptr(),
                                 _lib.KB_F32, T, E, K, 0,
                                 torch.cuda.current_stream(dev).cuda_stream), "kb_router")
    us = time_calls(launch, n, stream)
    return _gate_entry(us, T, peak, tflops_peak, n)


# The BASELINE token counts of each kernel.
KERNEL_T: Dict[str, List[int]] = {
    "qk_norm_rope_swa": [1, 8, 64, 256, 4096],
    "qk_norm_rope_rnope": [1, 8, 64, 256, 4096],
    "sandwich": [1, 64, 1024, 16384],
    "post_moe_pre_attn": [1, 64, 1024, 16384],
    "add_rms_norm": [1, 64, 1024, 16384],
    "expansion": [1, 64, 4096],
    "finalize": [1, 64, 4096],
    "router_maps": [1, 128, 4096, 65536],
    "expert_maps": [1, 64, 4096, 65536],
    "router_gemm": [1, 32, 256, 4096, 8192],
    "router_gemm_cublas": [1, 32, 256, 4096, 8192],
}


def run_kernel(name: str, dev, T: int, peak: float, stream, tflops_peak: float = 1677.6) -> dict:
    if name == "qk_norm_rope_swa":
        return bench_qk(dev, T, False, peak, stream)
    if name == "qk_norm_rope_rnope":
        return bench_qk(dev, T, True, peak, stream)
    if name in ("sandwich", "post_moe_pre_attn"):
        return bench_pair(dev, T, name, peak, stream)
    if name == "add_rms_norm":
        return bench_add_norm(dev, T, peak, stream)
    if name == "expansion":
        return bench_expansion(dev, T, peak, stream)
    if name == "finalize":
        return bench_finalize(dev, T, peak, stream)
    if name == "router_maps":
        return bench_router_maps(dev, T, peak, stream)
    if name == "expert_maps":
        return bench_expert_maps(dev, T, peak, stream)
    if name == "router_gemm":
        return bench_router_gemm(dev, T, peak, stream, tflops_peak)
    if name == "router_gemm_cublas":
        return bench_router_gemm_cublas(dev, T, peak, stream, tflops_peak)
    raise ValueError(name)

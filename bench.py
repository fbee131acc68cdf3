#!/usr/bin/env python
"""Benchmark of the B200 Q8-activation projection backend (one JSON line on rank 0).

Default workload: the Q4_K decode GEMVs of a Qwen2.5-1.5B FFN,
W 8960x1536 and W 1536x8960, exact Q32.32 outputs (`matvec_q8act`), batch 1.  One step
is both projections over one activation each.  Weights rotate over enough device copies
that every step streams them from HBM (copies > 3x the 126 MB L2), the reference's own
bench does the same with 256 MB of cycled copies (src/engine/chart/tests.rs:884-887).

  value  — algorithmic bytes (weights + int8 codes + exponents + i64 outputs) per second,
           device-timed with CUDA events, inputs already resident in HBM;
  e2e    — the same metric through the public C ABI with host buffers
           (apx_matvec_q8act: H2D of codes/exponents, D2H of outputs, every step);
  roofline — the Q4_K GEMV kernel: algorithmic bytes per launch / mean launch time
           (CUDA events on the launching stream) against the measured HBM copy peak.

`--impl reference` times the CPU restatement of the reference kernel (oracle/, the
reference is Rust and cannot be built here) on all host threads, same metric: the
reference's AVX2 / AVX-VNNI two-row decode cores and, for prefill, its k-column Q8_0
AVX-VNNI GEMM (oracle/apx_oracle_x86.c), on a persistent host thread pool.
Multi-GPU: replicas (independent decode streams per GPU, weak scaling), time = max over
ranks.

The same line carries `prefill`: 512 f32 tokens through the device
quantizer and the exact int8 tensor-core GEMM against W 4864x896 and W 896x4864 (Q8_0), one
step = both projections; TOPS = 2·MACs per second, roofline against the dense int8 peak
(twice the measured bf16 GEMM peak); e2e through apx_matmat_f32 with host buffers.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GEMV HBM GB/s (% of 8 TB/s); pp512 int8 GEMM TOPS (% peak); 1/2/4/8 GPU"
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), "measured"
    return 6650.0, "fallback"


def int8_peak():
    """Dense int8 tensor peak in TOPS: twice the bf16 GEMM peak (the tensor cores' int8
    rate is twice their bf16 rate), from the measured bf16 figure when present."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if "bf16_tflops" in d:
            return 2.0 * d["bf16_tflops"], "2 x measured bf16 GEMM burst"
    return 2.0 * 1590.0, "2 x fallback bf16 GEMM burst"


PREFILL = [(8, 4864, 896), (8, 896, 4864)]
PREFILL_TOKENS = 512


def host_threads():
    """The host threads this process may run on (its CPU affinity set, which a container's
    cpuset can make smaller than the machine's count)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_isa():
    """The vector form the CPU arm runs in, and the host CPU's model name."""
    from oracle import oracle as O

    f = O.simd_features()
    isa = "AVX-VNNI" if f["avxvnni"] else ("AVX2" if f["avx2"] else "scalar")
    model = "unknown CPU"
    try:
        with open("/proc/cpuinfo") as fh:
            for ln in fh:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return f"{isa} on {model}"


def cpu_prefill_baseline(seconds=10.0, tokens=PREFILL_TOKENS):
    """The prefill contract on the host cores: the oracle's restatement of the reference's
    matmat_q8act, which runs the k-column Q8_0 GEMM with AVX-VNNI (kern/gemm.rs:498-580;
    else the per-column vector rows), over `tokens` tokens of each shape, TOPS."""
    from apeiron_b200 import synth
    from oracle import oracle as O

    threads = host_threads()
    work = []
    for m, (t, n_out, n_in) in enumerate(PREFILL):
        raw = synth.payload(t, n_out, n_in, 2000 + m)
        cs, ss = [], []
        for c in range(tokens):
            cc, ee = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, 3000 + 7 * m + c)))
            cs.append(cc)
            ss.append(O.exps_to_scales(ee))
        work.append((t, raw, n_out, n_in, np.stack(cs), np.stack(ss)))
    macs = sum(tokens * n_out * n_in for _, n_out, n_in in PREFILL)
    done, t0 = 0, time.perf_counter()
    while True:
        for t, raw, n_out, n_in, cs, ss in work:
            r = O.matmat_q8act_mt(t, raw, n_out, n_in, cs, ss, threads, simd=True)
            assert not isinstance(r, tuple)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 1000:
            break
    return {"value": 2.0 * macs * done / el / 1e12, "unit": "TOPS", "cores": threads,
            "kind": "port", "sample": f"{done} passes of {tokens} tokens x both shapes "
                                      f"({el:.1f} s), k-column GEMM restatement, {cpu_isa()}"}


def measure_prefill(be, lib, dev, stream, steps, warmup, pg, local, world):
    """device-timed prefill steps (f32 columns quantized inside the GEMM's prep
    kernel, then the exact GEMM; both shapes)."""
    import torch

    from apeiron_b200 import synth
    from oracle import oracle as O

    sp = stream.cuda_stream
    k = PREFILL_TOKENS
    per_copy = sum(n_out * n_in * 34 // 32 for _, n_out, n_in in PREFILL) * 2  # + GEMM view
    copies = max(2, int(np.ceil(3 * L2_BYTES / per_copy)))
    raws = [synth.payload(t, n_out, n_in, 2000 + m) for m, (t, n_out, n_in) in enumerate(PREFILL)]
    tensors = [[be.upload(t, raws[m], n_out, n_in) for m, (t, n_out, n_in) in enumerate(PREFILL)]
               for _ in range(copies)]
    bufs = []
    for m, (t, n_out, n_in) in enumerate(PREFILL):
        x = np.stack([synth.activation_f32(n_in, 3000 + 7 * m + c) for c in range(k)])
        bufs.append(dict(
            x=x, dx=torch.from_numpy(x).to(dev),
            q32=torch.zeros(k * n_out, dtype=torch.int64, device=dev),
            f32=torch.zeros(k * n_out, dtype=torch.float32, device=dev),
            status=torch.full((2 * k,), -1, dtype=torch.int64, device=dev)))

    def step(i, q32=False):
        for m, (t, n_out, n_in) in enumerate(PREFILL):
            b = bufs[m]
            assert lib.apx_matmat_f32_async(be.ctx, tensors[i % copies][m].handle, n_out,
                                            n_in, k, b["dx"].data_ptr(), n_in,
                                            b["q32"].data_ptr() if q32 else None,
                                            b["f32"].data_ptr(), b["status"].data_ptr(),
                                            sp) == 0

    # exactness of the timed configuration: every column's Q32.32 outputs of both shapes
    # against the oracle's per-column contract (threaded C port), before any timing
    with torch.cuda.stream(stream):
        for i in range(copies):
            step(i, q32=True)
    stream.synchronize()
    for m, (t, n_out, n_in) in enumerate(PREFILL):
        cs, es = zip(*(synth.quant_act_np(synth.f32_to_q32(bufs[m]["x"][c])) for c in range(k)))
        want = O.matmat_q8act_mt(t, raws[m], n_out, n_in, np.stack(cs),
                                 np.stack([O.exps_to_scales(e) for e in es]),
                                 host_threads())
        got = bufs[m]["q32"].cpu().numpy().reshape(k, n_out)
        assert np.array_equal(got, want), "prefill parity failure in bench workload"
        assert bool((bufs[m]["status"] == -1).all().item())

    G = min(steps, 200)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        for i in range(G):
            step(i)
    with torch.cuda.stream(stream):
        for i in range(warmup):
            step(i)
        gr.replay()
    stream.synchronize()
    barrier(pg, local)
    reps = max(1, steps // G)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(reps):
            gr.replay()
        t1.record(stream)
    stream.synchronize()
    barrier(pg, local)
    ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / (reps * G)
    macs = sum(k * n_out * n_in for _, n_out, n_in in PREFILL)
    tops = world * 2.0 * macs / (ms / 1e3) / 1e12

    # e2e: every step copies both shapes' pinned f32 inputs in and their f32 outputs out, around
    # the public f32 entry point (apx_matmat_f32_async); the copies run on streams of their own
    # and overlap the projections, the device buffers double-buffered by step parity
    hx = [torch.from_numpy(bufs[m]["x"]).pin_memory() for m in range(len(PREFILL))]
    hy = [torch.empty(k * n_out, dtype=torch.float32).pin_memory() for _, n_out, _ in PREFILL]
    dxs = [[bufs[m]["dx"] for m in range(len(PREFILL))],
           [torch.empty_like(bufs[m]["dx"]) for m in range(len(PREFILL))]]
    dys = [[bufs[m]["f32"] for m in range(len(PREFILL))],
           [torch.empty_like(bufs[m]["f32"]) for m in range(len(PREFILL))]]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = {n: [torch.cuda.Event() for _ in range(2)] for n in ("in_ready", "in_free", "out_free")}
    ev_out = [[torch.cuda.Event() for _ in PREFILL] for _ in range(2)]

    def e2e_step(i):
        par = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev["in_free"][par])
            for m in range(len(PREFILL)):
                dxs[par][m].copy_(hx[m], non_blocking=True)
            ev["in_ready"][par].record(s_in)
        with torch.cuda.stream(stream):
            stream.wait_event(ev["in_ready"][par])
            stream.wait_event(ev["out_free"][par])
            for m, (t, n_out, n_in) in enumerate(PREFILL):
                assert lib.apx_matmat_f32_async(be.ctx, tensors[i % copies][m].handle, n_out,
                                                n_in, k, dxs[par][m].data_ptr(), n_in, None,
                                                dys[par][m].data_ptr(),
                                                bufs[m]["status"].data_ptr(), sp) == 0
                ev_out[par][m].record(stream)
            ev["in_free"][par].record(stream)
        with torch.cuda.stream(s_out):
            for m in range(len(PREFILL)):
                s_out.wait_event(ev_out[par][m])
                hy[m].copy_(dys[par][m], non_blocking=True)
            ev["out_free"][par].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(pg, local)
    e_steps = 200
    ev_start = torch.cuda.Event()
    with torch.cuda.stream(stream):
        t0.record(stream)
        ev_start.record(stream)
    s_in.wait_event(ev_start)
    s_out.wait_event(ev_start)
    for i in range(e_steps):
        e2e_step(i)
    with torch.cuda.stream(stream):
        stream.wait_event(ev["out_free"][(e_steps - 1) % 2])
        t1.record(stream)
    torch.cuda.synchronize()
    barrier(pg, local)
    for m in range(len(PREFILL)):
        assert torch.equal(hy[m], dys[(e_steps - 1) % 2][m].cpu()), "e2e outputs differ"
        assert bool((bufs[m]["status"] == -1).all().item())
    e_s = max_over_ranks(t0.elapsed_time(t1), pg, local) / 1e3
    e2e = world * 2.0 * macs * e_steps / e_s / 1e12
    peak, src = int8_peak()
    return {
        "metric": "pp512 int8 GEMM TOPS", "value": tops, "unit": "TOPS",
        "ms_per_step": ms, "steps": reps * G, "warmup": warmup,
        "config": {"workload": "Q8_0 prefill, 512 f32 tokens x (W 4864x896, W 896x4864), "
                               "configs[2]; step = f32_to_fixed + quant_act fused into the GEMM's prep, "
                               "then the exact GEMM, both shapes",
                   "weight_copies": copies, "l2": "rotating weight copies, > 3x the 126 MB L2",
                   "exact": "Q32.32 outputs of every column bit-equal to the CPU oracle "
                            "(checked before timing)"},
        "roofline": {"bound": "tensor", "achieved": tops, "peak": peak, "unit": "TOPS",
                     "frac": tops / peak, "peak_source": src,
                     "note": "whole step (fused quantize-prep and GEMM launches); the exact "
                             "per-block scale fold on the integer pipes bounds it, not the "
                             "tensor cores"},
        "e2e": {"value": e2e, "unit": "TOPS", "ms_per_step": e_s * 1e3 / e_steps,
                "h2d_bytes_per_step": sum(4 * k * n_in for _, _, n_in in PREFILL),
                "d2h_bytes_per_step": sum(4 * k * n_out for _, n_out, _ in PREFILL),
                "note": "per step: both shapes' pinned f32 inputs -> device, "
                        "apx_matmat_f32_async on each, the f32 outputs -> pinned host; the "
                        "copies on their own streams, overlapping the projections (device "
                        "buffers double-buffered by step parity); CUDA events, max over ranks"},
        "gpu_launches_per_step": 2 * len(PREFILL),
    }


# one decode step of a Qwen2.5-0.5B-shaped Q4_K_M model, every linear layer
DECODE_LAYER = [(12, 896, 896), (12, 128, 896), (12, 128, 896), (12, 896, 896),   # q k v o
                (12, 4864, 896), (12, 4864, 896), (12, 896, 4864)]                # gate up down
DECODE_LAYERS = 24
DECODE_HEAD = (14, 151936, 896)                                                   # tied lm_head


def measure_decode_step(be, lib, dev, stream, steps, warmup, pg, local, world):
    """the 169 projections of one decode step (24 layers of q/k/v/o/gate/up/down in
    Q4_K, the Q6_K head) as two launches replayed from a CUDA graph: one step plan
    (apx_plan_run_async) for the 168 layer projections and the head on its own.  q/k/v/o and
    gate/up read resident activations of their width (attention and the residual stream are
    not on this path); each layer's down reads the hidden activation its FFN produces on the
    device (SwiGLU + quant_act in the gate/up finish).  Replicas at N > 1."""
    import ctypes as C

    import torch

    from apeiron_b200 import _abi, synth
    from oracle import oracle as O

    sp = stream.cuda_stream
    mats = DECODE_LAYER * DECODE_LAYERS + [DECODE_HEAD]
    per_step = sum(gemv_bytes(*m) for m in mats)
    raws = {}
    for i, (t, n_out, n_in) in enumerate(DECODE_LAYER + [DECODE_HEAD]):
        raws[i] = synth.payload(t, n_out, n_in, 6000 + i)
    nl = len(DECODE_LAYER)
    wbytes = sum(raws[i % nl].size if i < len(mats) - 1 else raws[nl].size
                 for i in range(len(mats)))
    copies = max(2, int(np.ceil(3 * L2_BYTES / wbytes)))
    tensors = []  # [copy][projection]: every layer its own upload
    for c in range(copies):
        tensors.append([be.upload(t, raws[nl if i == len(mats) - 1 else i % nl], n_out, n_in)
                        for i, (t, n_out, n_in) in enumerate(mats)])
    n_embd, n_ff = DECODE_LAYER[0][2], DECODE_LAYER[4][1]
    x = synth.activation_f32(n_embd, 7000 + n_embd)
    cx, ex = synth.quant_act_np(synth.f32_to_q32(x))
    pad = lib.apx_act_padded_len(n_embd)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    codes[:n_embd] = torch.from_numpy(cx).to(dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    exps[:ex.size] = torch.from_numpy(ex).to(dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_embd,
                                          desc.data_ptr(), sp) == 0
    hpad = lib.apx_act_padded_len(n_ff)
    hs = [(torch.zeros(hpad, dtype=torch.int8, device=dev),
           torch.full((hpad // 32,), 0xFF, dtype=torch.uint8, device=dev),
           torch.zeros(8, dtype=torch.int32, device=dev)) for _ in range(DECODE_LAYERS)]
    outs = [torch.zeros(m[1], dtype=torch.int64, device=dev) for m in mats]
    statuses = torch.full((len(mats) + DECODE_LAYERS, 2), -1, dtype=torch.int64, device=dev)
    acts = [_abi.PlanAct(codes.data_ptr(), exps.data_ptr(), desc.data_ptr(), -1, 0)]
    acts += [_abi.PlanAct(h[0].data_ptr(), h[1].data_ptr(), h[2].data_ptr(), layer, 0)
             for layer, h in enumerate(hs)]
    ffns = (_abi.PlanFfn * DECODE_LAYERS)(*[
        _abi.PlanFfn(0, 1 + layer, None, statuses[len(mats) + layer].data_ptr())
        for layer in range(DECODE_LAYERS)])
    plans = []
    for c in range(copies):
        projs = []
        for i, (t, n_out, n_in) in enumerate(mats[:-1]):
            layer, k = divmod(i, nl)
            ffn, role = (layer, k - 4) if k in (4, 5) else (-1, 0)
            projs.append(_abi.PlanProj(tensors[c][i].handle, n_out, n_in,
                                       1 + layer if k == 6 else 0, ffn, role, 0,
                                       outs[i].data_ptr(), None, statuses[i].data_ptr()))
        err = _abi.ApxErr()
        pl = lib.apx_plan_create(be.ctx, (_abi.PlanProj * len(projs))(*projs), len(projs),
                                 (_abi.PlanAct * len(acts))(*acts), len(acts), ffns,
                                 DECODE_LAYERS, C.byref(err))
        assert pl, f"apx_plan_create failed: {err.code}"
        plans.append(pl)
    head = len(mats) - 1

    def step(i):
        assert lib.apx_plan_run_async(plans[i % copies], sp) == 0
        t, n_out, n_in = mats[head]
        assert lib.apx_matvec_async(be.ctx, tensors[i % copies][head].handle, n_out, n_in,
                                    codes.data_ptr(), exps.data_ptr(), desc.data_ptr(),
                                    outs[head].data_ptr(), None, statuses[head].data_ptr(),
                                    sp) == 0

    with torch.cuda.stream(stream):
        step(0)
    stream.synchronize()
    assert bool((statuses == -1).all().item()), "refusal in the decode step"
    # exactness: layer 0's projections (down through the device FFN chain) and the head
    thr = host_threads()
    sc = O.exps_to_scales(ex)
    ys = {}
    for k in range(4):
        t, n_out, n_in = DECODE_LAYER[k]
        ys[k] = O.matvec_q8act_mt(t, raws[k], n_out, n_in, cx, sc, thr)
        assert np.array_equal(outs[k].cpu().numpy(), ys[k]), f"decode-step parity {k}"
    g = O.matvec_q8act_mt(12, raws[4], n_ff, n_embd, cx, sc, thr)
    u = O.matvec_q8act_mt(12, raws[5], n_ff, n_embd, cx, sc, thr)
    assert np.array_equal(outs[4].cpu().numpy(), g) and np.array_equal(outs[5].cpu().numpy(), u)
    _, hcodes, hscales = O.swiglu_quant(g, u, 0)
    assert np.array_equal(hs[0][0].cpu().numpy()[:n_ff], hcodes), "decode-step h codes"
    y = O.matvec_q8act_mt(12, raws[6], n_embd, n_ff, hcodes, hscales, thr)
    assert np.array_equal(outs[6].cpu().numpy(), y), "decode-step down (FFN chain) parity"
    t, n_out, n_in = DECODE_HEAD
    want = O.matvec_q8act_mt(t, raws[nl], n_out, n_in, cx, sc, thr)
    assert np.array_equal(outs[head].cpu().numpy(), want), "decode-step head parity"
    G = max(2, min(steps, 20))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        for i in range(G):
            step(i)
    with torch.cuda.stream(stream):
        for i in range(warmup):
            step(i)
        gr.replay()
    stream.synchronize()
    barrier(pg, local)
    reps = max(1, steps // G)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(reps):
            gr.replay()
        t1.record(stream)
    stream.synchronize()
    barrier(pg, local)
    ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / (reps * G)
    assert bool((statuses == -1).all().item()), "refusal while timed"
    # the plan alone and the head alone, back to back (the step's kernels)
    parts = {}
    for name, fn in (("plan", lambda i: lib.apx_plan_run_async(plans[i % copies], sp)),
                     ("head", lambda i: lib.apx_matvec_async(
                         be.ctx, tensors[i % copies][head].handle, mats[head][1], mats[head][2],
                         codes.data_ptr(), exps.data_ptr(), desc.data_ptr(),
                         outs[head].data_ptr(), None, statuses[head].data_ptr(), sp))):
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            for i in range(G):
                assert fn(i) == 0
        with torch.cuda.stream(stream):
            g2.replay()
            t0.record(stream)
            g2.replay()
            t1.record(stream)
        stream.synchronize()
        parts[name] = t0.elapsed_time(t1) / G
        del g2
    del gr

    # e2e: every step copies the f32 input vector in (pinned), quantizes it on the device into
    # the activation the plan and the head read, runs both, and copies the head's Q32.32 outputs
    # out on a stream of its own (overlapping the next step; the output double-buffered)
    hxv = torch.from_numpy(x).pin_memory()
    dxv = torch.empty(n_embd, dtype=torch.float32, device=dev)
    hy = torch.empty(mats[head][1], dtype=torch.int64).pin_memory()
    dys = [outs[head], torch.zeros_like(outs[head])]
    s_out = torch.cuda.Stream(device=dev)
    ev_ready = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        par = i % 2
        with torch.cuda.stream(stream):
            dxv.copy_(hxv, non_blocking=True)
            assert lib.apx_quant_f32_async(be.ctx, dxv.data_ptr(), n_embd, codes.data_ptr(),
                                           exps.data_ptr(), desc.data_ptr(), sp) == 0
            assert lib.apx_plan_run_async(plans[i % copies], sp) == 0
            stream.wait_event(ev_free[par])
            assert lib.apx_matvec_async(be.ctx, tensors[i % copies][head].handle,
                                        mats[head][1], mats[head][2], codes.data_ptr(),
                                        exps.data_ptr(), desc.data_ptr(), dys[par].data_ptr(),
                                        None, statuses[head].data_ptr(), sp) == 0
            ev_ready[par].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_ready[par])
            hy.copy_(dys[par], non_blocking=True)
            ev_free[par].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(pg, local)
    e_steps = max(4, min(steps, 400)) // 2 * 2
    ev_start = torch.cuda.Event()
    with torch.cuda.stream(stream):
        t0.record(stream)
        ev_start.record(stream)
    s_out.wait_event(ev_start)
    for i in range(e_steps):
        e2e_step(i)
    with torch.cuda.stream(stream):
        stream.wait_event(ev_free[(e_steps - 1) % 2])
        t1.record(stream)
    torch.cuda.synchronize()
    barrier(pg, local)
    e_ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / e_steps
    assert np.array_equal(hy.numpy(), want), "decode-step e2e head outputs differ"
    assert bool((statuses == -1).all().item()), "refusal in the e2e steps"
    for pl in plans:
        lib.apx_plan_destroy(pl)
    hbm, _ = peaks()
    gbs = world * per_step / (ms / 1e3) / 1e9
    plan_bytes = sum(gemv_bytes(*m) for m in mats[:-1])
    head_bytes = gemv_bytes(*mats[head])
    return {
        "metric": "decode step GB/s (all linear layers)", "value": gbs, "unit": "GB/s",
        "ms_per_step": ms, "steps": reps * G, "tokens_per_s": world * 1e3 / ms,
        "scaling": "weak",
        "config": {"workload": "Qwen2.5-0.5B-shaped Q4_K_M decode step, configs[3]: 24 layers "
                               "x (q 896x896, k/v 128x896, o 896x896, gate/up 4864x896, down "
                               "896x4864) Q4_K + tied lm_head 151936x896 Q6_K = 169 projections "
                               "in 2 launches: one step plan (168 layer projections; each "
                               "layer's down reads the hidden activation its FFN's SwiGLU + "
                               "quant_act produces on the device; the plan queues by dependency "
                               "level: gate/up, then q/k/v/o, then down) and the head; "
                               "q/k/v/o/gate/up read resident activations",
                   "bytes_per_step": per_step, "weight_copies": copies,
                   "l2": "rotating weight copies, >= 3x the 126 MB L2",
                   "exact": "layer 0's q/k/v/o/gate/up, its h codes and its down output (the "
                            "device FFN chain) and the head bit-equal to the CPU oracle (checked "
                            "before timing)"},
        "hbm_frac": gbs / world / hbm,
        "kernels": [{"kernel": "plan_kernel<Q4_K> (168 projections, 24 FFNs)",
                     "us": parts["plan"] * 1e3, "gbs": plan_bytes / (parts["plan"] / 1e3) / 1e9,
                     "frac": plan_bytes / (parts["plan"] / 1e3) / 1e9 / hbm},
                    {"kernel": "gemv_stream_kernel<Q6_K> (head 151936x896)",
                     "us": parts["head"] * 1e3, "gbs": head_bytes / (parts["head"] / 1e3) / 1e9,
                     "frac": head_bytes / (parts["head"] / 1e3) / 1e9 / hbm}],
        "gpu_launches_per_step": 2,
        "e2e": {"value": world * per_step / (e_ms / 1e3) / 1e9, "unit": "GB/s",
                "ms_per_step": e_ms, "h2d_bytes_per_step": 4 * n_embd,
                "d2h_bytes_per_step": 8 * mats[head][1],
                "note": "per step: the pinned f32 input vector -> device, quant_act on the "
                        "device (apx_quant_f32_async), the step plan and the head, the head's "
                        "Q32.32 outputs -> pinned host on a stream of their own (overlapping "
                        "the next step); CUDA events, max over ranks"},
    }


SHARDED = [(12, 28672, 8192), (12, 28672, 8192), (12, 8192, 28672)]  # gate, up, down


def measure_sharded(be, lib, dev, stream, steps, warmup, pg, rank, local, world):
    """configs[4] decode: the Llama-3-70B-shaped Q4_K FFN as a chain, row-sharded over the
    ranks (apeiron_b200/shard.py).  Each rank holds the same row range of gate and up and a row
    range of down.  Per step: GEMVs of this rank's gate and up rows (one grouped launch when
    their layouts allow), SwiGLU + quant_act of the slice (apx_swiglu_quant_shard_async) storing
    each 32-row block of h (int8 codes and an exponent byte) and the slice's descriptor into
    every rank's buffer by NVLink peer stores; a publication (flags, bounded wait) makes every
    rank's slice visible and merges the descriptors; down projects this rank's rows from the
    whole h with its outputs stored into every rank's buffer; a second publication.  Strong
    scaling: the same FFN at every N."""
    import ctypes as C

    import torch

    from apeiron_b200 import _abi, shard, synth
    from oracle import oracle as O

    sp = stream.cuda_stream
    dist = pg if world > 1 else None
    raws = [synth.payload(t, n_out, n_in, 4000 + m) for m, (t, n_out, n_in) in enumerate(SHARDED)]
    per_rank = sum(r.size for r in raws) / world
    copies = max(1, int(np.ceil(3 * L2_BYTES / per_rank)))
    shards = [[shard.RowShard(be, t, raws[m], n_out, n_in, rank, world, dist, f"cuda:{local}")
               for m, (t, n_out, n_in) in enumerate(SHARDED)] for _ in range(copies)]
    n_ff, n_embd = SHARDED[0][1], SHARDED[0][2]
    x = synth.activation_f32(n_embd, 5000)
    cx, ex = synth.quant_act_np(synth.f32_to_q32(x))
    pad = lib.apx_act_padded_len(n_embd)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    codes[:n_embd] = torch.from_numpy(cx).to(dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    exps[:ex.size] = torch.from_numpy(ex).to(dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    with torch.cuda.stream(stream):
        assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_embd,
                                          desc.data_ptr(), sp) == 0
    stream.synchronize()
    hg = shard.HiddenGather(lib, be.ctx, shards[0][0], shards[0][1])
    yg = shard.PeerGather(lib, be.ctx, [shards[0][2]])
    st_gu = torch.full((2, 2), -1, dtype=torch.int64, device=dev)
    merged_gu = torch.full((2, 2), -1, dtype=torch.int64, device=dev)
    st_y = torch.full((1, 2), -1, dtype=torch.int64, device=dev)
    merged_y = torch.full((1, 2), -1, dtype=torch.int64, device=dev)
    ffn_st = torch.full((2,), -1, dtype=torch.int64, device=dev)
    peers = [q for q in range(world) if q != rank]
    gq = torch.zeros(shards[0][0].rows, dtype=torch.int64, device=dev)
    uq = torch.zeros(shards[0][1].rows, dtype=torch.int64, device=dev)
    gu_handles = [(C.c_uint64 * 2)(row[0].tensor.handle, row[1].tensor.handle) for row in shards]
    gu_outs = (C.c_void_p * 2)(gq.data_ptr(), uq.data_ptr())
    gu_st = (C.c_void_p * 2)(st_gu[0].data_ptr(), st_gu[1].data_ptr())
    dests = []  # per parity: this rank's slice in its own buffer and in every peer's
    for par in (0, 1):
        own = hg.slice_dest(par, rank)
        ps = [hg.slice_dest(par, q) for q in peers]
        n = max(len(ps), 1)
        dests.append((own, len(ps), (C.c_void_p * n)(*[p[0] for p in ps]),
                      (C.c_void_p * n)(*[p[1] for p in ps]),
                      (C.c_void_p * n)(*[p[2] for p in ps])))

    def step(i):
        row = shards[i % copies]
        par = hg.next_parity()
        # gate and up of this rank's rows (Q32.32: the SwiGLU's inputs), one launch when their
        # layouts allow
        assert lib.apx_matvec_group_async(be.ctx, gu_handles[i % copies], 2, n_embd,
                                          codes.data_ptr(), exps.data_ptr(), desc.data_ptr(),
                                          gu_outs, None, gu_st, sp) == 0
        (oc, oe, od), npeer, pc, pe, pd = dests[par]
        assert lib.apx_swiglu_quant_shard_async(be.ctx, gq.data_ptr(), uq.data_ptr(), row[0].rows,
                                                0, None, oc, oe, od, npeer, pc, pe, pd,
                                                ffn_st.data_ptr(), sp) == 0
        assert hg.publish(st_gu, merged_gu, sp) == par
        ypar = yg.run([hg.activation(par)], st_y, merged_y, sp, shards=[row[2]])
        return par, ypar

    # exactness before timing: every rank's whole h and gathered y against the oracle's chain
    with torch.cuda.stream(stream):
        par, ypar = step(0)
    stream.synchronize()
    thr = max(1, host_threads() // world)
    sc = O.exps_to_scales(ex)
    g = O.matvec_q8act_mt(12, raws[0], n_ff, n_embd, cx, sc, thr, simd=True)
    u = O.matvec_q8act_mt(12, raws[1], n_ff, n_embd, cx, sc, thr, simd=True)
    _, hcodes, hscales = O.swiglu_quant(g, u, 0)
    hc, he, hd = hg.read(par)
    assert np.array_equal(hc, hcodes), "sharded h codes parity failure"
    assert np.array_equal(he, O.scales_to_exps(hscales)), "sharded h exponents parity failure"
    want = O.matvec_q8act_mt(12, raws[2], n_embd, n_ff, hcodes, hscales, thr, simd=True)
    assert np.array_equal(yg.read(0, ypar), want), "sharded FFN chain parity failure"
    for w in (merged_gu, merged_y):
        assert bool((w[:, 0] == -1).all().item()), "sharded refusal in bench workload"
    assert int(ffn_st[0].item()) == -1
    del raws
    barrier(pg, local)

    with torch.cuda.stream(stream):
        for i in range(max(warmup, 3) + 1):  # an even number of calls: parities in step
            step(1 + i)
    stream.synchronize()
    G = min(steps, 100) // 2 * 2 or 2
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(G):
            step(i)
    barrier(pg, local)
    reps = max(1, steps // G)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        t0.record(stream)
        for _ in range(reps):
            graph.replay()
        t1.record(stream)
    stream.synchronize()
    barrier(pg, local)
    ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / (reps * G)
    for w in (merged_gu, merged_y):
        assert bool((w[:, 0] == -1).all().item()), "sharded refusal while timed"
    del graph
    torch.cuda.synchronize()
    barrier(pg, local)  # no rank writes into another's buffers any more
    hg.close()
    yg.close()
    per_step = sum(gemv_bytes(*mat) for mat in SHARDED)
    gbs = per_step / (ms / 1e3) / 1e9
    hbm, _ = peaks()
    return {
        "metric": "70B FFN decode GB/s (row-sharded FFN chain, NVLink peer-store exchange)",
        "value": gbs, "unit": "GB/s", "n_gpus": world, "ms_per_step": ms, "steps": reps * G,
        "scaling": "strong",
        "config": {"workload": "Llama-3-70B-shaped Q4_K FFN decode, configs[4]: W_gate/W_up "
                               "28672x8192, W_down 8192x28672; step = gate and up of this "
                               "rank's rows (GEMV, one launch when their layouts allow), SwiGLU "
                               "+ quant_act of the slice storing h's int8 codes and exponent "
                               "bytes (and the slice's descriptor) into every rank's buffer, a "
                               "publication, down of this rank's rows from the whole h with its "
                               "outputs stored into every rank's buffer, a second publication",
                   "rows_per_rank": {"gate_up": shards[0][0].rows, "down": shards[0][2].rows},
                   "nvlink_bytes_per_rank": (shards[0][0].rows + shards[0][0].rows // 32 + 32)
                                            * (world - 1) + 8 * shards[0][2].rows * (world - 1),
                   "weight_copies": copies,
                   "l2": "rotating weight copies, >= 3x the 126 MB L2 per rank",
                   "timing": "CUDA graph",
                   "exact": "every rank's whole h and gathered y bit-equal to the CPU oracle's "
                            "chain (matvec_q8act, swiglu_quant, matvec_q8act), checked before "
                            "timing"},
        "hbm_frac_per_gpu": gbs / world / hbm,
        # gate and up share one launch when both plan as one resident wave (the GEMV planner:
        # row tiles x K-slots within two waves of 148 SMs x 48 units), as at N = 8
        "gpu_launches_per_step": 6 if shards[0][0].rows // 32 * (n_embd // 256) <= 148 * 48
                                 else 7,
    }


PREFILL70 = [(12, 28672, 8192), (12, 28672, 8192), (12, 8192, 28672)]  # gate, up, down


def cpu_prefill70_baseline(seconds=10.0, tokens=64):
    """configs[4]'s prefill on the host cores: the oracle's restatement of the reference's
    k-column Q4_K kernel (chart/kcols.rs:1406-1518, what matmat_q8act runs for multi-column Q4_K
    calls) over `tokens` tokens of the 28672x8192 gate matrix, TOPS."""
    from apeiron_b200 import synth
    from oracle import oracle as O

    threads = host_threads()
    t, n_out, n_in = PREFILL70[0]
    raw = synth.payload(t, n_out, n_in, 4000)
    cs, ss = [], []
    for c in range(tokens):
        cc, ee = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, 8000 + c)))
        cs.append(cc)
        ss.append(O.exps_to_scales(ee))
    cs, ss = np.stack(cs), np.stack(ss)
    done, t0 = 0, time.perf_counter()
    while True:
        r = O.matmat_q8act_mt(t, raw, n_out, n_in, cs, ss, threads, simd=True)
        assert not isinstance(r, tuple)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= 100:
            break
    macs = tokens * n_out * n_in * done
    return {"value": 2.0 * macs / el / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{done} passes of {tokens} tokens x W 28672x8192 Q4_K ({el:.1f} s), "
                      f"k-column Q4_K restatement, {cpu_isa()}"}


def measure_prefill70(be, lib, dev, stream, steps, warmup, pg, rank, local, world):
    """configs[4]'s prefill: the Llama-3-70B-shaped Q4_K projections over 512 f32 tokens each
    (x ~ N(0,1)): gate and up (W 28672x8192) on one 512-token input, down (W 8192x28672) on its
    own, each through the f32 prefill entry (fused quantize + digit-plane tensor-core GEMM).  At
    N > 1 every rank holds a 32-row-aligned slice of each matrix's rows (apeiron_b200/shard.py
    row_split) and an NCCL all-gather of every projection's f32 output slices gives each rank
    the whole outputs.  Strong scaling.

    Before timing, the FFN chain these projections make is checked on the device against the
    oracle's chain for 4 tokens: gate and up, SwiGLU + quant_act of every token's hidden vector
    in one launch (at N > 1 an all-gather of the hidden codes), down reading those codes."""
    import torch

    from apeiron_b200 import shard, synth
    from oracle import oracle as O

    sp = stream.cuda_stream
    k = PREFILL_TOKENS
    dist = pg if world > 1 else None
    raws = [synth.payload(t, n_out, n_in, 4000 + m) for m, (t, n_out, n_in) in enumerate(PREFILL70)]
    shards = [shard.RowShard(be, t, raws[m], n_out, n_in, rank, world, dist, f"cuda:{local}")
              for m, (t, n_out, n_in) in enumerate(PREFILL70)]
    n_embd, n_ff = PREFILL70[0][2], PREFILL70[0][1]
    rg, rd = shards[0].rows, shards[2].rows
    for sh in shards:  # equal slices: all-gathers of equal-sized chunks
        assert all(b - a == sh.rows for a, b in sh.splits)
    assert rg % 256 == 0, "hidden slices must fill whole padded activation blocks"
    x = np.stack([synth.activation_f32(n_embd, 8000 + c) for c in range(k)])
    xd_h = np.stack([synth.activation_f32(n_ff, 8600 + c) for c in range(k)])
    dx = torch.from_numpy(x).to(dev)
    dxd = torch.from_numpy(xd_h).to(dev)
    q32 = lambda n: torch.zeros(n, dtype=torch.int64, device=dev)
    st = lambda: torch.full((2 * k,), -1, dtype=torch.int64, device=dev)
    thr = max(1, host_threads() // world)
    r0, g0 = shards[2].r0, shards[0].r0

    # ---- the FFN chain, exactness only ----
    gate_s, up_s = q32(k * rg), q32(k * rg)
    sg, su, sf, sy = st(), st(), st(), st()
    hc = torch.zeros(k * n_ff, dtype=torch.int8, device=dev)
    he = torch.full((k * n_ff // 32,), 0xFF, dtype=torch.uint8, device=dev)
    hd = torch.zeros(8 * k, dtype=torch.int32, device=dev)
    yq_s = q32(k * rd)
    with torch.cuda.stream(stream):
        assert lib.apx_matmat_f32_async(be.ctx, shards[0].tensor.handle, rg, n_embd, k,
                                        dx.data_ptr(), n_embd, gate_s.data_ptr(), None,
                                        sg.data_ptr(), sp) == 0
        assert lib.apx_matmat_f32_async(be.ctx, shards[1].tensor.handle, rg, n_embd, k,
                                        dx.data_ptr(), n_embd, up_s.data_ptr(), None,
                                        su.data_ptr(), sp) == 0
        if world == 1:
            assert lib.apx_swiglu_quant_cols_async(be.ctx, gate_s.data_ptr(), up_s.data_ptr(), rg,
                                                   k, 0, None, hc.data_ptr(), he.data_ptr(),
                                                   hd.data_ptr(), sf.data_ptr(), sp) == 0
        else:
            hc_s = torch.zeros(k * rg, dtype=torch.int8, device=dev)
            he_s = torch.full((k * rg // 32,), 0xFF, dtype=torch.uint8, device=dev)
            hd_s = torch.zeros(8 * k, dtype=torch.int32, device=dev)
            hc_g = torch.zeros(world * k * rg, dtype=torch.int8, device=dev)
            he_g = torch.zeros(world * k * rg // 32, dtype=torch.uint8, device=dev)
            assert lib.apx_swiglu_quant_cols_async(be.ctx, gate_s.data_ptr(), up_s.data_ptr(), rg,
                                                   k, 0, None, hc_s.data_ptr(), he_s.data_ptr(),
                                                   hd_s.data_ptr(), sf.data_ptr(), sp) == 0
            pg.all_gather_into_tensor(hc_g, hc_s)
            pg.all_gather_into_tensor(he_g, he_s)
            # [rank][token][slice] -> [token][rank][slice]: every token's whole h
            hc.view(k, world, rg).copy_(hc_g.view(world, k, rg).transpose(0, 1))
            he.view(k, world, rg // 32).copy_(he_g.view(world, k, rg // 32).transpose(0, 1))
            assert lib.apx_act_describe_cols_async(be.ctx, hc.data_ptr(), he.data_ptr(), n_ff, k,
                                                   hd.data_ptr(), sp) == 0
        assert lib.apx_matmat_async(be.ctx, shards[2].tensor.handle, rd, n_ff, k, hc.data_ptr(),
                                    he.data_ptr(), hd.data_ptr(), yq_s.data_ptr(), None,
                                    sy.data_ptr(), sp) == 0
    stream.synchronize()
    for s_ in (sg, su, sf, sy):
        assert bool((s_[0::2] == -1).all().item()), "refusal in the prefill chain"
    ys = yq_s.cpu().numpy().reshape(k, rd)
    gq, uq = gate_s.cpu().numpy().reshape(k, rg), up_s.cpu().numpy().reshape(k, rg)
    hcn, hen = hc.cpu().numpy().reshape(k, n_ff), he.cpu().numpy().reshape(k, n_ff // 32)
    for c in (0, 1, k // 2, k - 1):
        cx, sx = O.quant_act(synth.f32_to_q32(x[c]))
        g = O.matvec_q8act_mt(12, raws[0], n_ff, n_embd, cx, sx, thr, simd=True)
        u = O.matvec_q8act_mt(12, raws[1], n_ff, n_embd, cx, sx, thr, simd=True)
        assert np.array_equal(gq[c], g[g0:g0 + rg]), f"gate parity failure, token {c}"
        assert np.array_equal(uq[c], u[g0:g0 + rg]), f"up parity failure, token {c}"
        _, hcodes, hscales = O.swiglu_quant(g, u, 0)
        assert np.array_equal(hcn[c], hcodes), f"h codes parity failure, token {c}"
        assert np.array_equal(hen[c], O.scales_to_exps(hscales)), f"h exponents, token {c}"
        want = O.matvec_q8act_mt(12, raws[2], n_embd, n_ff, hcodes, hscales, thr, simd=True)
        if not np.array_equal(ys[c], want[r0:r0 + rd]):
            bad = np.nonzero(ys[c] != want[r0:r0 + rd])[0]
            raise AssertionError(f"prefill chain parity failure, token {c}: {bad.size} rows, "
                                 f"first {bad[0]} gpu {ys[c][bad[0]]} oracle {want[r0 + bad[0]]}")
    del gate_s, up_s, hc, he, yq_s

    # ---- the timed step: the three projections (+ all-gathers of their output slices) ----
    ins = [(dx, n_embd), (dx, n_embd), (dxd, n_ff)]
    rows = [sh.rows for sh in shards]
    y_s = [torch.zeros(k * r, dtype=torch.float32, device=dev) for r in rows]
    yq = [q32(k * r) for r in rows]
    y_g = ([torch.zeros(world * k * r, dtype=torch.float32, device=dev) for r in rows]
           if world > 1 else y_s)
    sts = [st() for _ in rows]

    def step(check=False):
        # each projection's all-gather runs on NCCL's stream while the next projection computes
        # (the work's wait makes this stream wait for it only after that projection is queued)
        pending = None
        for m in range(3):
            xin, n_in = ins[m]
            assert lib.apx_matmat_f32_async(be.ctx, shards[m].tensor.handle, rows[m], n_in, k,
                                            xin.data_ptr(), n_in,
                                            yq[m].data_ptr() if check else None,
                                            y_s[m].data_ptr(), sts[m].data_ptr(), sp) == 0
            if pending is not None:
                pending.wait()
            if world > 1:
                pending = pg.all_gather_into_tensor(y_g[m], y_s[m], async_op=True)
        if pending is not None:
            pending.wait()

    with torch.cuda.stream(stream):
        step(check=True)
    stream.synchronize()
    for m, (t, n_out, n_in) in enumerate(PREFILL70):
        assert bool((sts[m][0::2] == -1).all().item()), f"refusal in projection {m}"
        got = yq[m].cpu().numpy().reshape(k, rows[m])
        gf = y_g[m].cpu().numpy().reshape(world, k, rows[m])
        xs = x if m < 2 else xd_h
        sr0 = shards[m].r0
        for c in ((0, k - 1) if m < 2 else (0, k // 3, k - 1)):
            cx, sx = O.quant_act(synth.f32_to_q32(xs[c]))
            want = O.matvec_q8act_mt(t, raws[m], n_out, n_in, cx, sx, thr, simd=True)
            assert np.array_equal(got[c], want[sr0:sr0 + rows[m]]), \
                f"projection {m} parity failure, token {c}"
            wf = (want.astype(np.float64) / 4294967296.0).astype(np.float32)
            whole = np.concatenate([gf[r, c] for r in range(world)])
            assert np.allclose(whole, wf, rtol=1e-6, atol=0), f"projection {m} f32, token {c}"
    del raws, yq
    barrier(pg, local)
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            step()
    stream.synchronize()
    barrier(pg, local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
    stream.synchronize()
    barrier(pg, local)
    ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / steps
    for m in range(3):
        assert bool((sts[m][0::2] == -1).all().item()), "refusal while timed"
    macs = sum(k * n_out * n_in for _, n_out, n_in in PREFILL70)
    tops = 2.0 * macs / (ms / 1e3) / 1e12

    # e2e: every step copies its pinned host inputs in and the assembled f32 outputs out, on
    # copy streams of their own so that the copies overlap the projections (a projection's
    # outputs go out while the next one runs, and the next step's inputs come in); the device
    # inputs and outputs are double-buffered by step parity.
    hx = [torch.from_numpy(x).pin_memory(), torch.from_numpy(xd_h).pin_memory()]
    hy = [torch.empty(y_g[m].numel(), dtype=torch.float32).pin_memory() for m in range(3)]
    d_in = [(dx, dxd), (torch.empty_like(dx), torch.empty_like(dxd))]
    y_s2 = [torch.zeros_like(v) for v in y_s]
    d_ys = [y_s, y_s2]
    d_yg = [y_g, [torch.zeros_like(v) for v in y_g] if world > 1 else y_s2]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in_ready = [torch.cuda.Event() for _ in range(2)]
    ev_in_free = [torch.cuda.Event() for _ in range(2)]
    ev_out_free = [torch.cuda.Event() for _ in range(2)]
    ev_out_ready = [[torch.cuda.Event() for _ in range(3)] for _ in range(2)]

    def e2e_step(i):
        par = i % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_in_free[par])
            d_in[par][0].copy_(hx[0], non_blocking=True)
            d_in[par][1].copy_(hx[1], non_blocking=True)
            ev_in_ready[par].record(s_in)
        with torch.cuda.stream(stream):
            stream.wait_event(ev_in_ready[par])
            stream.wait_event(ev_out_free[par])
            pending = None
            for m in range(3):
                xin, n_in = (d_in[par][0], n_embd) if m < 2 else (d_in[par][1], n_ff)
                assert lib.apx_matmat_f32_async(be.ctx, shards[m].tensor.handle, rows[m], n_in,
                                                k, xin.data_ptr(), n_in, None,
                                                d_ys[par][m].data_ptr(), sts[m].data_ptr(),
                                                sp) == 0
                if m == 2:
                    ev_in_free[par].record(stream)
                if pending is not None:  # the previous projection's gather, behind this one
                    pending.wait()
                    ev_out_ready[par][m - 1].record(stream)
                if world > 1:
                    pending = pg.all_gather_into_tensor(d_yg[par][m], d_ys[par][m],
                                                        async_op=True)
                else:
                    ev_out_ready[par][m].record(stream)
            if pending is not None:
                pending.wait()
                ev_out_ready[par][2].record(stream)
        with torch.cuda.stream(s_out):
            for m in range(3):
                s_out.wait_event(ev_out_ready[par][m])
                hy[m].copy_(d_yg[par][m], non_blocking=True)
            ev_out_free[par].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(pg, local)
    e_steps = max(4, steps // 2) // 2 * 2
    ev_start = torch.cuda.Event()
    with torch.cuda.stream(stream):
        t0.record(stream)
        ev_start.record(stream)
    s_in.wait_event(ev_start)
    s_out.wait_event(ev_start)
    for i in range(e_steps):
        e2e_step(i)
    with torch.cuda.stream(stream):
        stream.wait_event(ev_out_free[(e_steps - 1) % 2])
        t1.record(stream)
    torch.cuda.synchronize()
    barrier(pg, local)
    for m in range(3):  # the last step's host outputs are the assembled outputs
        assert torch.equal(hy[m], d_yg[(e_steps - 1) % 2][m].cpu()), "e2e outputs differ"
        assert bool((sts[m][0::2] == -1).all().item()), "refusal in the e2e steps"
    e_ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / e_steps
    peak, src = int8_peak()
    return {
        "metric": "70B FFN pp512 int8 TOPS (gate/up/down projections, row-sharded)",
        "value": tops, "unit": "TOPS", "n_gpus": world, "ms_per_step": ms, "steps": steps,
        "warmup": warmup, "scaling": "strong",
        "config": {"workload": "Llama-3-70B-shaped Q4_K FFN prefill, configs[4]: 512 f32 tokens "
                               "(N(0,1)) through gate and up (W 28672x8192) and 512 through down "
                               "(W 8192x28672), each by the f32 prefill entry (quantize + digit-"
                               "plane tensor-core GEMM); at N > 1 row shards and an NCCL all-"
                               "gather of every projection's f32 output slices (assembled "
                               "outputs [rank][token][row slice] on every rank)",
                   "rows_per_rank": {"gate_up": rg, "down": rd},
                   "l2": "digit planes of the three matrices (2.8 GB at N = 1) exceed the 126 MB "
                         "L2: every step streams them from HBM",
                   "exact": "2-3 tokens of every projection bit-equal (Q32.32) to the oracle, and "
                            "the FFN chain (gate, up, SwiGLU + quant_act, down) bit-equal for 4 "
                            "tokens, checked before timing"},
        "roofline": {"bound": "tensor", "achieved": tops / world, "peak": peak, "unit": "TOPS",
                     "frac": tops / world / peak, "peak_source": src,
                     "note": "algorithmic int8 ops per GPU; these Q4_K rows need four weight "
                             "digits (27-bit integer weights), so the GEMM runs 8 int8 MMAs "
                             "(4 weight x 2 activation digits) per algorithmic op: the tensor "
                             "pipe's own rate is 8x this"},
        "gpu_launches_per_step": 6,
        "e2e": {"value": 2.0 * macs / (e_ms / 1e3) / 1e12, "unit": "TOPS", "ms_per_step": e_ms,
                "h2d_bytes_per_step": int(x.nbytes + xd_h.nbytes),
                "d2h_bytes_per_step": int(sum(4 * y_g[m].numel() for m in range(3))),
                "note": "per step: pinned host inputs -> device, the three projections (+ "
                        "gathers), the assembled f32 outputs -> pinned host; the copies on "
                        "their own streams, overlapping the projections (device buffers double-"
                        "buffered by step parity); CUDA events, max over ranks"},
    }


def measure_gemv(be, lib, dev, stream, mat, steps, warmup, pg, local, world, seed=1100):
    """One projection's decode GEMV (configs[0]: Q8_0 4864x896) on its own: device-timed GB/s
    of algorithmic bytes over rotating weight copies (3x the L2), back-to-back launches replayed
    from a CUDA graph, checked against the oracle first; e2e through apx_matvec_q8act with host
    buffers (every copy's synchronous call warmed first)."""
    import ctypes as C

    import torch

    from apeiron_b200 import _abi, synth
    from oracle import oracle as O

    sp = stream.cuda_stream
    t, n_out, n_in = mat
    raw = synth.payload(t, n_out, n_in, seed)
    copies = max(4, int(np.ceil(3 * L2_BYTES / raw.size)))
    tensors = [be.upload(t, raw, n_out, n_in) for _ in range(copies)]
    x = synth.activation_f32(n_in, seed + 1)
    c, e = synth.quant_act_np(synth.f32_to_q32(x))
    pad = lib.apx_act_padded_len(n_in)
    codes = torch.zeros(pad, dtype=torch.int8, device=dev)
    codes[:n_in] = torch.from_numpy(c).to(dev)
    exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
    exps[:e.size] = torch.from_numpy(e).to(dev)
    desc = torch.zeros(8, dtype=torch.int32, device=dev)
    out = torch.zeros(n_out, dtype=torch.int64, device=dev)
    status = torch.full((2,), -1, dtype=torch.int64, device=dev)
    with torch.cuda.stream(stream):
        assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_in,
                                          desc.data_ptr(), sp) == 0

    def launch(i):
        assert lib.apx_matvec_async(be.ctx, tensors[i % copies].handle, n_out, n_in,
                                    codes.data_ptr(), exps.data_ptr(), desc.data_ptr(),
                                    out.data_ptr(), None, status.data_ptr(), sp) == 0

    with torch.cuda.stream(stream):
        launch(0)
    stream.synchronize()
    want = O.matvec_q8act(t, raw, n_out, n_in, c, O.exps_to_scales(e))
    assert np.array_equal(out.cpu().numpy(), want), "configs[0] parity failure"
    G = max(64, min(steps, 1000))
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=stream):
        for i in range(G):
            launch(i)
    with torch.cuda.stream(stream):
        for i in range(max(warmup, 3)):
            launch(i)
        gr.replay()
    stream.synchronize()
    barrier(pg, local)
    reps = max(1, steps // G)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(reps):
            gr.replay()
        t1.record(stream)
    stream.synchronize()
    barrier(pg, local)
    ms = max_over_ranks(t0.elapsed_time(t1), pg, local) / (reps * G)
    assert int(status[0].item()) == -1
    del gr
    nbytes = gemv_bytes(*mat)
    gbs = world * nbytes / (ms / 1e3) / 1e9
    # e2e: the synchronous drop-in with host buffers, every rotating copy warmed first
    hc, he = np.ascontiguousarray(c, dtype=np.int8), np.ascontiguousarray(e, dtype=np.uint8)
    ho = np.empty(n_out, dtype=np.int64)
    err = _abi.ApxErr()
    for i in range(copies):
        assert lib.apx_matvec_q8act(be.ctx, tensors[i].handle, n_out, n_in, hc.ctypes.data, n_in,
                                    he.ctypes.data, ho.ctypes.data, C.byref(err)) == 0
    assert np.array_equal(ho, want)
    n_e = 2000
    e0 = time.perf_counter()
    for i in range(n_e):
        lib.apx_matvec_q8act(be.ctx, tensors[i % copies].handle, n_out, n_in, hc.ctypes.data,
                             n_in, he.ctypes.data, ho.ctypes.data, C.byref(err))
    e_s = max_over_ranks(time.perf_counter() - e0, pg, local)
    hbm, src = peaks()
    return {
        "metric": "Q8_0 decode GEMV GB/s", "value": gbs, "unit": "GB/s", "ms_per_step": ms,
        "steps": reps * G, "scaling": "weak",
        "config": {"workload": "Q8_0 GEMV 4864x896 (Qwen2.5-0.5B FFN up), configs[0]; step = one "
                               "launch, resident activation",
                   "weight_copies": copies, "l2": "rotating weight copies, 3x the 126 MB L2",
                   "exact": "Q32.32 outputs bit-equal to the CPU oracle (checked before timing)"},
        "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / world / hbm, "kernel": f"gemv_kernel<Q8_0> {n_out}x{n_in}",
                     "algorithmic_bytes": nbytes, "peak_source": src,
                     "note": "back-to-back launches under programmatic dependent launch"},
        "e2e": {"value": world * nbytes * n_e / e_s / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": 16 + 32 + ((-(-n_in // 32) + 15) // 16) * 16 +
                                      ((n_in + 15) // 16) * 16,
                "d2h_bytes_per_step": ((8 * n_out + 15) // 16) * 16 + 16},
        "gpu_launches_per_step": 1,
    }


def gemv_config(name):
    """The headline's `config`: the workload alone, identical for both arms."""
    return {"workload": name,
            "l2": "every step streams its weights from memory (rotating copies larger than the "
                  "last-level cache)",
            "exact": "Q32.32 outputs bit-equal to the CPU oracle (checked before timing)"}


def gemv_bytes(t, n_out, n_in):
    from apeiron_b200 import synth
    qk, bb = synth.GEOM[t]
    w = n_out * (-(-n_in // qk)) * bb
    return w + n_in + (-(-n_in // 32)) + 8 * n_out


WORKLOADS = {
    1: ("Q8_0 GEMV 4864x896 (Qwen2.5-0.5B FFN up), configs[0]", [(8, 4864, 896)]),
    2: ("Q4_K GEMV 8960x1536 + 1536x8960 (Qwen2.5-1.5B FFN), configs[1]",
        [(12, 8960, 1536), (12, 1536, 8960)]),
}


class Clocks:
    """nvidia-smi sampling during the timed region (clocks, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
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
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
        pg = dist
    return world, rank, local, pg


def max_over_ranks(v, pg, local):
    if pg is None:
        return v
    import torch

    t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg, local):
    if pg is not None:
        import torch

        pg.barrier(device_ids=[local])
        torch.cuda.synchronize()


def cpu_data(mats, min_bytes=256 << 20):
    """Host copies of the workload cycled so every pass streams DRAM, as the reference's
    bench_pooled_shapes does with 256 MB of copies (src/engine/chart/tests.rs:835-911)."""
    from apeiron_b200 import synth
    from oracle import oracle as O

    base = []
    for t, n_out, n_in in mats:
        raw = synth.payload(t, n_out, n_in, 17 + n_out)
        c, e = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, 3)))
        base.append((t, raw, n_out, n_in, c, O.exps_to_scales(e)))
    per = sum(d[1].size for d in base)
    copies = max(1, -(-min_bytes // per))
    return [[(t, raw.copy(), n_out, n_in, c, s) for (t, raw, n_out, n_in, c, s) in base]
            for _ in range(copies)], copies


def cpu_passes(data, max_passes, max_seconds, min_seconds=0.0):
    """Timed passes of the oracle's threaded fused rows (restating the reference's AVX2
    chunked decode, src/engine/chart/ffn.rs:667-745) on every host thread: at least
    `max_passes` passes or `min_seconds`, whichever is longer, and at most `max_seconds`."""
    from oracle import oracle as O

    threads = host_threads()
    total = done = 0
    t0 = time.perf_counter()
    while done < max_passes or time.perf_counter() - t0 < min_seconds:
        for t, raw, n_out, n_in, c, s in data[done % len(data)]:
            r = O.matvec_q8act_mt(t, raw, n_out, n_in, c, s, threads, simd=True)
            assert not isinstance(r, tuple)
            total += gemv_bytes(t, n_out, n_in)
        done += 1
        if time.perf_counter() - t0 > max_seconds:
            break
    return total, done, time.perf_counter() - t0, threads


def cpu_chain_baseline(mats, seed0, seconds=5.0):
    """The CPU arm of a chain of projections (configs[3]'s decode step, configs[4]'s whole FFN):
    every projection its own host copy, so a pass streams DRAM as the device's does, one
    quantized activation per width, and every call the oracle's restatement of the reference's
    pooled decode (the vector two-row cores where the width allows, else the portable fast rows
    or the contract, as the reference picks them); GB/s of the same algorithmic bytes."""
    from apeiron_b200 import synth
    from oracle import oracle as O

    threads = host_threads()
    base = {m: synth.payload(m[0], m[1], m[2], seed0 + i) for i, m in enumerate(dict.fromkeys(mats))}
    data = [(t, base[(t, n_out, n_in)].copy(), n_out, n_in) for t, n_out, n_in in mats]
    acts = {}
    for n_in in {m[2] for m in mats}:
        c, e = synth.quant_act_np(synth.f32_to_q32(synth.activation_f32(n_in, seed0 + n_in)))
        acts[n_in] = (c, O.exps_to_scales(e))
    per_pass = sum(gemv_bytes(*m) for m in mats)

    def one_pass():
        for t, raw, n_out, n_in in data:
            r = O.matvec_q8act_mt(t, raw, n_out, n_in, *acts[n_in], threads, simd=True)
            assert not isinstance(r, tuple)

    one_pass()
    done, t0 = 0, time.perf_counter()
    while True:
        one_pass()
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": per_pass * done / el / 1e9, "unit": "GB/s", "cores": threads,
            "kind": "port", "sample": f"{done} passes of all {len(mats)} projections "
                                      f"({per_pass / 1e6:.0f} MB of distinct host copies per "
                                      f"pass) in {el:.1f} s, {cpu_isa()}"}


def cpu_gemv_baseline(mats, seconds=10.0):
    data, copies = cpu_data(mats)
    cpu_passes(data, 3, 2.0)
    total, done, el, threads = cpu_passes(data, 1 << 30, seconds)
    return {"value": total / el / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{done} passes of the workload over {copies} cycled host copies "
                      f"(>= 256 MB, streamed from DRAM) in {el:.1f} s, two-row "
                      f"decode cores, {cpu_isa()}"}


def run_reference(args, world, rank, local, pg):
    if rank != 0:
        return
    name, mats = WORKLOADS[args.config]
    data, copies = cpu_data(mats)
    cpu_passes(data, args.warmup, 10.0)
    # a timed window of at least 5 s whatever --steps is (a few ms per step on the host)
    total, done, el, threads = cpu_passes(data, args.steps, 60.0, min_seconds=5.0)
    v = total / el / 1e9
    sample = (f"{done} steps in {el:.1f} s (at least {args.steps} and 5 s, at most 60 s) over "
              f"{copies} cycled host copies (>= 256 MB, streamed from DRAM), two-row decode "
              f"cores, {cpu_isa()}")
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": done, "warmup": args.warmup, "ms_per_step": el * 1e3 / max(done, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int64",
            "data": "synthetic", "impl": "reference",
            "config": gemv_config(name),
            "arm": {"weight_copies": copies, "l2": "cycled host copies >= 256 MB",
                    "parallelism": f"{threads} host threads"},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if not args.no_prefill:
        pre = cpu_prefill_baseline(seconds=min(20.0, args.cpu_seconds * 2))
        line["prefill"] = {"metric": "pp512 int8 GEMM TOPS", "value": pre["value"],
                           "unit": "TOPS", "cpu_baseline": pre,
                           "e2e": {"value": pre["value"], "unit": "TOPS",
                                   "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_gemv0:
        g0 = cpu_gemv_baseline(WORKLOADS[1][1], seconds=min(10.0, args.cpu_seconds))
        line["gemv_q8_0"] = {"metric": "Q8_0 decode GEMV GB/s", "value": g0["value"],
                             "unit": "GB/s", "cpu_baseline": g0}
    if not args.no_prefill70:
        p70 = cpu_prefill70_baseline(seconds=min(20.0, args.cpu_seconds * 2))
        line["prefill_70b"] = {
            "metric": "70B FFN pp512 int8 TOPS (gate/up/down projections, row-sharded)",
            "value": p70["value"], "unit": "TOPS", "cpu_baseline": p70}
    for key, skip, metric, mats_, seed in (
            ("decode_step", args.no_decode, "decode step GB/s (all linear layers)",
             DECODE_LAYER * DECODE_LAYERS + [DECODE_HEAD], 6000),
            ("sharded", args.no_shard, "70B FFN decode GB/s (row-sharded FFN chain)", SHARDED, 4000)):
        if skip:
            continue
        try:
            cb = cpu_chain_baseline(mats_, seed, args.cpu_seconds / 2)
            line[key] = {"metric": metric, "value": cb["value"], "unit": "GB/s",
                         "cpu_baseline": cb}
        except Exception as exc:  # the headline line stands without it
            line[key] = {"unavailable": f"{type(exc).__name__}: {exc}"}
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local, pg):
    import ctypes as C

    import torch

    from apeiron_b200 import _abi, synth
    from apeiron_b200.chart import Backend

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    be = Backend(local)
    lib = be.lib
    name, mats = WORKLOADS[args.config]
    per_step = sum(gemv_bytes(*m) for m in mats)
    copies = max(4, int(np.ceil(3 * L2_BYTES / sum(
        synth.GEOM[t][1] * n_out * (-(-n_in // synth.GEOM[t][0])) for t, n_out, n_in in mats))))
    tensors = []  # [copy][mat]
    for m, (t, n_out, n_in) in enumerate(mats):
        raw = synth.payload(t, n_out, n_in, 1000 + m)
        for c in range(copies):
            if m == 0:
                tensors.append([])
            tensors[c].append(be.upload(t, raw, n_out, n_in))
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    acts = []
    for m, (t, n_out, n_in) in enumerate(mats):
        x = synth.activation_f32(n_in, 50 + m)
        c, e = synth.quant_act_np(synth.f32_to_q32(x))
        pad = lib.apx_act_padded_len(n_in)
        codes = torch.zeros(pad, dtype=torch.int8, device=dev)
        codes[:n_in] = torch.from_numpy(c).to(dev)
        exps = torch.full((pad // 32,), 0xFF, dtype=torch.uint8, device=dev)
        exps[:e.size] = torch.from_numpy(e).to(dev)
        desc = torch.zeros(8, dtype=torch.int32, device=dev)
        with torch.cuda.stream(stream):
            assert lib.apx_act_describe_async(be.ctx, codes.data_ptr(), exps.data_ptr(), n_in,
                                              desc.data_ptr(), sp) == 0
        out = torch.zeros(n_out, dtype=torch.int64, device=dev)
        acts.append((codes, exps, desc, out, c, e))
    status = torch.full((2,), -1, dtype=torch.int64, device=dev)

    def step(i):
        for m, (t, n_out, n_in) in enumerate(mats):
            codes, exps, desc, out, _, _ = acts[m]
            rc = lib.apx_matvec_async(be.ctx, tensors[i % copies][m].handle, n_out, n_in,
                                      codes.data_ptr(), exps.data_ptr(), desc.data_ptr(),
                                      out.data_ptr(), None, status.data_ptr(), sp)
            assert rc == 0

    # correctness of the timed configuration against the oracle (small, untimed)
    from oracle import oracle as O
    for m, (t, n_out, n_in) in enumerate(mats):
        with torch.cuda.stream(stream):
            step(0)
        stream.synchronize()
        codes, exps, desc, out, c, e = acts[m]
        raw = synth.payload(t, n_out, n_in, 1000 + m)
        want = O.matvec_q8act(t, raw, n_out, n_in, c, O.exps_to_scales(e))
        assert np.array_equal(out.cpu().numpy(), want), "parity failure in bench workload"
    assert int(status[0].item()) == -1

    # The timed steps are replayed from CUDA graphs (captured once, untimed), so the device
    # time is the kernels' and not the Python launch loop's.
    def capture(first, count, only=None):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            for i in range(first, first + count):
                if only is not None:
                    t, n_out, n_in = mats[only]
                    codes, exps, desc, out, _, _ = acts[only]
                    assert lib.apx_matvec_async(be.ctx, tensors[i % copies][only].handle, n_out,
                                                n_in, codes.data_ptr(), exps.data_ptr(),
                                                desc.data_ptr(), out.data_ptr(), None,
                                                status.data_ptr(), sp) == 0
                else:
                    step(i)
        return gr

    G = min(args.steps, 1000)
    g_main = capture(0, G)
    g_rem = capture(0, args.steps % G) if args.steps % G else None
    n_k = min(max(args.steps, 64), 1000)
    g_kernels = [capture(0, n_k, only=m) for m in range(len(mats))]
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
        g_main.replay()
    stream.synchronize()
    barrier(pg, local)
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(args.steps // G):
            g_main.replay()
        if g_rem is not None:
            g_rem.replay()
        t1.record(stream)
    stream.synchronize()
    barrier(pg, local)
    ms = t0.elapsed_time(t1)
    # each projection's kernel alone, n_k back-to-back launches over the rotating copies
    kms = []
    for g_kernel in g_kernels:
        k0e, k1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            g_kernel.replay()
            k0e.record(stream)
            g_kernel.replay()
            k1e.record(stream)
        stream.synchronize()
        kms.append(k0e.elapsed_time(k1e) / n_k)
    clk = clocks.stop()
    clk["timed_region_ms"] = ms
    ms_max = max_over_ranks(ms, pg, local)
    value = world * per_step * args.steps / (ms_max / 1e3) / 1e9
    assert int(status[0].item()) == -1

    # e2e through the synchronous C ABI (apx_matvec_q8act, the drop-in for matvec_q8act) with
    # host buffers: every call copies its activation in and its Q32.32 outputs back, then
    # returns; called through ctypes directly, as the engine's FFI binding would
    host = [(np.ascontiguousarray(a[4], dtype=np.int8), np.ascontiguousarray(a[5], dtype=np.uint8),
             np.empty(max(m[1], 1), dtype=np.int64)) for a, m in zip(acts, mats)]
    herr = _abi.ApxErr()
    hptr = C.byref(herr)
    fn = lib.apx_matvec_q8act

    def e2e_step(i):
        for m, (t, n_out, n_in) in enumerate(mats):
            hc, he, ho = host[m]
            if fn(be.ctx, tensors[i % copies][m].handle, n_out, n_in, hc.ctypes.data, hc.size,
                  he.ctypes.data, ho.ctypes.data, hptr):
                raise RuntimeError(f"apx_matvec_q8act failed: code {herr.code}")

    # every rotating copy once first: each tensor's synchronous call builds its cached graph on
    # its first call, so the timed loop measures the steady state
    for i in range(max(args.warmup, copies)):
        e2e_step(i)
    for m, (t, n_out, n_in) in enumerate(mats):  # the host outputs are the exact ones
        raw = synth.payload(t, n_out, n_in, 1000 + m)
        want = O.matvec_q8act(t, raw, n_out, n_in, acts[m][4], O.exps_to_scales(acts[m][5]))
        assert np.array_equal(host[m][2][:n_out], want), "parity failure on the e2e path"
    barrier(pg, local)
    e_steps = min(args.steps, 2000)
    e0 = time.perf_counter()
    for i in range(e_steps):
        e2e_step(args.warmup + i)
    e_s = time.perf_counter() - e0
    e_s = max_over_ranks(e_s, pg, local)
    e2e = world * per_step * e_steps / e_s / 1e9
    h2d = sum(16 + 32 + ((-(-n_in // 32) + 15) // 16) * 16 + ((n_in + 15) // 16) * 16
              for _, _, n_in in mats)
    d2h = sum(((8 * n_out + 15) // 16) * 16 + 16 for _, n_out, _ in mats)

    gemv0 = None
    if not args.no_gemv0:
        gemv0 = measure_gemv(be, lib, dev, stream, WORKLOADS[1][1][0], args.steps, args.warmup,
                             pg, local, world)
    prefill = None
    if not args.no_prefill:
        prefill = measure_prefill(be, lib, dev, stream, args.prefill_steps, args.warmup, pg,
                                  local, world)
    prefill70 = None
    if not args.no_prefill70:
        prefill70 = measure_prefill70(be, lib, dev, stream, args.prefill70_steps, args.warmup, pg,
                                      rank, local, world)
    decode = None
    if not args.no_decode:
        decode = measure_decode_step(be, lib, dev, stream, args.decode_steps, args.warmup, pg,
                                     local, world)
    sharded = None
    if not args.no_shard:
        sharded = measure_sharded(be, lib, dev, stream, args.shard_steps, args.warmup, pg, rank,
                                  local, world)
    if rank != 0:
        return
    hbm, src = peaks()
    # the roofline of the slowest kernel per byte of the step (the one that bounds it)
    rates = [gemv_bytes(*m) / (kms[i] / 1e3) / 1e9 for i, m in enumerate(mats)]
    slow = int(np.argmin(rates))
    t0m = mats[slow]
    kbytes = gemv_bytes(*t0m)
    achieved = rates[slow]
    traffic = None
    prof = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(prof):
        traffic = json.load(open(prof)).get(f"{t0m[0]}:{t0m[1]}x{t0m[2]}")
    fam = {8: "Q8_0", 12: "Q4_K", 14: "Q6_K"}
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
        "config": gemv_config(name),
        "arm": {"weight_copies": copies, "l2": "rotating device copies, 3x the 126 MB L2",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": traffic,
                     "kernel": f"gemv_kernel<{fam[t0m[0]]}> {t0m[1]}x{t0m[2]} (the step's slower "
                               f"kernel per byte)",
                     "share_of_step": kms[slow] / sum(kms),
                     "kernels": [{"shape": f"{m[1]}x{m[2]}", "us": kms[i] * 1e3,
                                  "gbs": rates[i], "frac": rates[i] / hbm}
                                 for i, m in enumerate(mats)],
                     "algorithmic_bytes": kbytes, "peak_source": src},
        "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": len(mats) * args.steps,
        "kernel_us": kms[slow] * 1e3,
        "clocks": clk,
    }
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_gemv_baseline(mats, seconds=args.cpu_seconds)
        if gemv0 is not None:
            gemv0["cpu_baseline"] = cpu_gemv_baseline(WORKLOADS[1][1], seconds=args.cpu_seconds / 2)
        if prefill is not None:
            prefill["cpu_baseline"] = cpu_prefill_baseline(seconds=args.cpu_seconds)
        if prefill70 is not None:
            prefill70["cpu_baseline"] = cpu_prefill70_baseline(seconds=args.cpu_seconds)
        for obj, mats_, seed in ((decode, DECODE_LAYER * DECODE_LAYERS + [DECODE_HEAD], 6000),
                                 (sharded, SHARDED, 4000)):
            if obj is None:
                continue
            try:
                obj["cpu_baseline"] = cpu_chain_baseline(mats_, seed, args.cpu_seconds / 2)
            except Exception as exc:  # the device numbers stand without it
                obj["cpu_baseline"] = {"unavailable": f"{type(exc).__name__}: {exc}"}
    if gemv0 is not None:
        line["gemv_q8_0"] = gemv0
        line["gpu_launches"] += gemv0["steps"]
    if prefill is not None:
        line["prefill"] = prefill
        line["gpu_launches"] += prefill["gpu_launches_per_step"] * prefill["steps"]
    if prefill70 is not None:
        line["prefill_70b"] = prefill70
        line["gpu_launches"] += prefill70["gpu_launches_per_step"] * prefill70["steps"]
    if decode is not None:
        line["decode_step"] = decode
        line["gpu_launches"] += decode["gpu_launches_per_step"] * decode["steps"]
    if sharded is not None:
        line["sharded"] = sharded
        line["gpu_launches"] += sharded["gpu_launches_per_step"] * sharded["steps"]
    print(json.dumps(line), flush=True)


def gemm_probe(args):
    """One k-column shape through the f32 prefill entry (apx_matmat_f32_async), its first token
    checked against the oracle, then `--steps` calls back to back (rotating two weight copies,
    CUDA events); prints one JSON line.  A small single-GPU case for ncu captures of the
    tensor-core GEMM."""
    import torch

    from apeiron_b200 import synth
    from apeiron_b200.chart import Backend
    from oracle import oracle as O

    t, n_out, n_in, k = (int(v) for v in args.gemm_probe.split(","))
    dev = torch.device("cuda:0")
    be = Backend(0)
    lib = be.lib
    route = {"auto": 0, "digits": 1, "fold": 2}[args.gemm_route]
    assert lib.apx_ctx_set_gemm_route(be.ctx, route) == 0
    stream = torch.cuda.Stream(device=dev)
    sp = stream.cuda_stream
    raws = [synth.payload(t, n_out, n_in, 600 + c) for c in range(2)]
    tens = [be.upload(t, r, n_out, n_in) for r in raws]
    x = np.stack([synth.activation_f32(n_in, 700 + c) for c in range(k)])
    dx = torch.from_numpy(x).to(dev)
    yq = torch.zeros(k * n_out, dtype=torch.int64, device=dev)
    y = torch.zeros(k * n_out, dtype=torch.float32, device=dev)
    st = torch.full((2 * k,), -1, dtype=torch.int64, device=dev)

    def call(i, q=False):
        assert lib.apx_matmat_f32_async(be.ctx, tens[i % 2].handle, n_out, n_in, k, dx.data_ptr(),
                                        n_in, yq.data_ptr() if q else None, y.data_ptr(),
                                        st.data_ptr(), sp) == 0

    with torch.cuda.stream(stream):
        call(0, q=True)
    stream.synchronize()
    c, e = O.quant_act(synth.f32_to_q32(x[0]))
    want = O.matvec_q8act_mt(t, raws[0], n_out, n_in, c, e, host_threads(), simd=True)
    assert np.array_equal(yq.cpu().numpy()[:n_out], want), "gemm probe parity failure"
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            call(i)
    stream.synchronize()
    steps = min(args.steps, 200)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        for i in range(steps):
            call(i)
        t1.record(stream)
    stream.synchronize()
    assert bool((st[0::2] == -1).all().item())
    us = t0.elapsed_time(t1) / steps * 1e3
    print(json.dumps({"probe": "gemm", "type": t, "n_out": n_out, "n_in": n_in, "tokens": k,
                      "route": args.gemm_route, "us_per_call": us,
                      "tops": 2.0 * k * n_out * n_in / us / 1e6}), flush=True)
    be.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-shard", action="store_true")
    ap.add_argument("--no-gemv0", action="store_true")
    ap.add_argument("--no-prefill70", action="store_true")
    ap.add_argument("--prefill70-steps", type=int, default=10)
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--decode-steps", type=int, default=200)
    ap.add_argument("--shard-steps", type=int, default=400)
    ap.add_argument("--prefill-steps", type=int, default=400)
    ap.add_argument("--gemm-probe", default=None,
                    help="TYPE,N_OUT,N_IN,TOKENS: time one prefill shape alone and exit (a small "
                         "case for profilers)")
    ap.add_argument("--gemm-route", default="auto", choices=["auto", "digits", "fold"],
                    help="the Q8_0 GEMM a --gemm-probe call takes (the bits are the same)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.gemm_probe:
        gemm_probe(args)
        return
    world, rank, local, pg = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank, local, pg)
        else:
            run_ours(args, world, rank, local, pg)
    finally:
        if pg is not None:
            pg.destroy_process_group()


if __name__ == "__main__":
    main()

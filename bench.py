#!/usr/bin/env python
"""Benchmark: Q8_0 LFM2-8B-A1B-shaped greedy decode on B200 (benchmark config 4).

One "step" = one greedy decode token (batch 1) through all 24 layers: 18 short-conv +
6 GQA attention layers, 2 dense FFNs, 22 MoE FFNs (32 experts, top-4), lm_head + argmax.
Weights are seeded random-init Q8_0 (no checkpoints exist here); the prompt is 512 seeded
uniform token ids, prefilled untimed; then W warm-up and K timed decode steps.

  value  -- tok/s of the device-resident decode loop (token fed back on the device, all
            inputs in HBM; each step streams 1.66 GB of weights, far above the 126 MB L2)
  e2e    -- tok/s through the public engine API (Lfm2CudaEngine.forward_argmax): each step
            copies its token/position host->device and reads the argmax back
  N > 1  -- N sequences, one per GPU, whole model per GPU (value = total tokens / max-over-ranks
            time); the expert-parallel model (32/N experts per GPU, NCCL exchange in every MoE
            layer) is measured beside it: prefill and decode (run_multi)

`--impl reference` times the reference algorithm's CPU implementation (the C restatement
of the JS CPU path in oracle/, all host threads) on a bounded slice of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
from __graft_entry__ import load_package  # noqa: E402

METRIC = "decode tok/s and MoE-layer HBM GB/s (Q8_0 LFM2-MoE) at 1/2/4/8 B200"
SEED = 1234
PROMPT = 512
THINK_ID = 124901  # LFM2 <think> (lfm2-engine.js:539); >= vocab 65536 here, so nothing to suppress


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _traffic():
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return {}
    return {}


class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _lfm2_model_bytes(spec) -> dict:
    """Algorithmic bytes per decode token (Q8_0 = 34 B / 32 weights)."""
    E, F, Fe, V, NE, k = spec.n_embd, spec.n_ff, spec.n_ff_exp, spec.n_vocab, spec.n_expert, spec.n_expert_used
    q8 = 34 / 32
    nq = spec.n_head * spec.head_dim
    nkv = spec.n_head_kv * spec.head_dim
    conv = (E * 3 * E + E * E) * q8
    attn = (E * (nq + 2 * nkv) + nq * E) * q8
    dense = 3 * E * F * q8
    router = E * NE * q8
    expert = 3 * E * Fe * q8
    gateup = k * 2 * E * Fe * q8 + 4 * E + 4 * k * Fe
    down = k * Fe * E * q8 + 4 * k * Fe + 8 * E
    moe_layer = router + k * expert + 3 * 4 * E
    n_attn = sum(1 for i in range(spec.n_layers) if spec.is_attn(i))
    n_moe = sum(1 for i in range(spec.n_layers) if spec.is_moe(i))
    weights = ((spec.n_layers - n_attn) * conv + n_attn * attn + (spec.n_layers - n_moe) * dense
               + n_moe * (router + k * expert) + E * V * q8)
    return dict(gateup=gateup, down=down, moe_layer=moe_layer, weights_per_token=weights)


def run_ours(args, ws, rank, local):
    import torch

    qq3 = load_package()
    qq3.build.build_all()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    if args.n_expert != spec.n_expert:
        # profiling knob: fewer experts per layer shrink the model on the device, while a decode
        # token still streams the same bytes (top-4 of any expert count)
        spec.n_expert = args.n_expert
    t0 = time.time()
    tensors = qq3.synth.build_tensors(spec)
    gen_s = time.time() - t0
    g = qq3.synth.MemoryGGUF(spec, tensors)
    max_ctx = args.prompt + args.warmup + 2 * args.steps + 16
    # sequence 1 only serves the clock-sampling soak, so sequence 0's state stays the true continuation
    t_up = time.time()
    eng = qq3.Lfm2CudaEngine(g, device=local, max_ctx=max_ctx, n_seq=2)
    torch.cuda.synchronize()
    upload_s = time.time() - t_up
    stream = torch.cuda.Stream(device=local)
    eng.ctx.set_stream(stream.cuda_stream)
    prompt = qq3.synth.uniform_tokens(args.prompt, SEED + rank, spec.n_vocab)
    suppress = THINK_ID if THINK_ID < spec.n_vocab else -1

    torch.cuda.synchronize()
    t_pf = time.perf_counter()
    eng.prefill(prompt[:-1].tolist())  # batched (tensor cores) from 64 tokens on
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pf
    pos = args.prompt - 1
    toks = eng.model.decode_loop(int(prompt[-1]), pos, args.warmup, suppress_id=suppress)
    pos += args.warmup
    cur = int(toks[-1]) if len(toks) else int(prompt[-1])
    pos_timed = pos

    # ---- value: device-resident greedy decode loop
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        # un-timed soak of the same loop on sequence 1 so that nvidia-smi sees the clocks under
        # this load (the 200 ms sampler needs ~1 s); sequence 0 is untouched
        t_soak = time.time()
        while time.time() - t_soak < 1.0:
            eng.model.decode_loop(cur, pos, args.steps, seq=1, suppress_id=suppress, want_tokens=False)
        e0.record(stream)
        out = eng.model.decode_loop(cur, pos, args.steps, suppress_id=suppress)
        e1.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    pos += args.steps
    cur = int(out[-1])

    # ---- e2e: public engine API, host token in / argmax out per step
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e2.record(stream)
    for _ in range(args.steps):
        cur = eng.forward_argmax(cur, pos, suppress)
        pos += 1
    e3.record(stream)
    torch.cuda.synchronize()
    ms_e2e = e2.elapsed_time(e3)

    # ---- per-phase trace of one step of the persistent kernel (after the timed regions): the
    # MoE-layer HBM rate of the shipped path (bytes of one routed FFN phase / its critical-path
    # time); with --trace the whole breakdown goes into the line
    phase_trace = None
    if eng.model.stat(qq3.runtime.QQ_STAT_STEP_KERNELS) == 1:
        eng.model.decode_trace(True)
        eng.model.decode_loop(cur, pos, 4, seq=1, suppress_id=suppress, want_tokens=False)
        stamps, kinds = eng.model.decode_trace(False, read=True)
        phase_trace = trace_summary(stamps, kinds, eng.model.decode_trace_sub())

    # ---- dominant kernel (expert gate/up GEMV) and whole MoE layer, timed alone over all layers
    nbytes = _lfm2_model_bytes(spec)
    ms_gateup = eng.model.bench_kernel(qq3.runtime.QQ_KERN_MOE_GATEUP, 3)
    ms_layer = eng.model.bench_kernel(qq3.runtime.QQ_KERN_MOE_LAYER, 3)
    moe_persist_gbs = moe_persist_us = None
    routed = (phase_trace or {}).get("by_kind", {}).get("fused/store/routed")
    if routed:
        moe_persist_us = routed["crit_us_per_phase"]
        moe_persist_gbs = round(nbytes["moe_layer"] / (moe_persist_us * 1e-6) / 1e9, 1)
    step_kernels = eng.model.stat(qq3.runtime.QQ_STAT_STEP_KERNELS)

    if dist:
        t = torch.tensor([ms, ms_e2e], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    peak, peak_kind = _peaks()
    tr = _traffic()
    # KV rows the 6 attention layers read per step, at the mean position of the timed steps
    n_attn = sum(1 for i in range(spec.n_layers) if spec.is_attn(i))
    kv_bytes = n_attn * spec.n_head_kv * spec.head_dim * 4 * 2 * (pos_timed + 1 + args.steps / 2)
    step_bytes = nbytes["weights_per_token"] + kv_bytes
    if step_kernels == 1:
        # the persistent step kernel is the only kernel of a step: its launch time is the step time
        step_ms = ms / args.steps
        roof = {"bound": "hbm", "kernel": "k_decode (persistent decode step: all 24 layers + lm_head + argmax)",
                "achieved": round(step_bytes / (step_ms * 1e-3) / 1e9, 1), "peak": peak, "peak_kind": peak_kind,
                "unit": "GB/s", "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / peak, 4),
                "traffic": tr.get("decode_step_bytes_per_launch"), "algorithmic_bytes": int(step_bytes),
                "avg_launch_ms": round(step_ms, 5)}
    else:
        achieved = nbytes["gateup"] / (ms_gateup * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "moe expert gate/up SwiGLU GEMV (4 experts x 2 x 2048x1792 Q8_0)",
                "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": tr.get("moe_gateup_bytes_per_launch"),
                "algorithmic_bytes": int(nbytes["gateup"]), "avg_launch_ms": round(ms_gateup, 5)}
    tok_s = ws * args.steps / (ms * 1e-3)
    e2e_tok_s = ws * args.steps / (ms_e2e * 1e-3)
    res = {
        "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xf32 (Q8_0 weights, f32 activations)",
        "data": "synthetic (seeded random-init Q8_0 weights, seeded uniform prompt ids)",
        "config": {"workload": "LFM2-8B-A1B-shaped Q8_0 greedy decode, batch 1 (benchmark config 4)",
                   "layers": "24 (18 short-conv, 6 GQA attention; 2 dense FFN 7168, 22 MoE 32x top-4 x 1792)",
                   "hidden": 2048, "vocab": 65536, "prompt": args.prompt, "global_batch": ws,
                   "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
                   "l2": "inputs larger than L2: each step streams 1.66 GB of weights"},
        # one MoE layer (router, gate/up, down, combine) as one phase of the persistent step: its
        # algorithmic bytes / its critical-path time in a traced step
        "moe_layer_hbm_gbs": moe_persist_gbs,
        "moe_layer_us": moe_persist_us,
        # the same layer as separate kernels, timed alone over all 22 layers
        "moe_layer_kernels_hbm_gbs": round(nbytes["moe_layer"] / (ms_layer * 1e-3) / 1e9, 1),
        "moe_gateup_kernel_gbs": round(nbytes["gateup"] / (ms_gateup * 1e-3) / 1e9, 1),
        "step_weight_gbs_per_gpu": round(nbytes["weights_per_token"] * args.steps / (ms * 1e-3) / 1e9, 1),
        "roofline": roof,
        "e2e": {"value": round(e2e_tok_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 12,
                "api": "Lfm2CudaEngine.forward_argmax -> qq_forward"},
        "gpu_launches": int(step_kernels * args.steps),
        "clocks": clk.summary(),
        "prefill": {"tokens": args.prompt - 1, "ms": round(prefill_s * 1e3, 2),
                    "tok_s": round((args.prompt - 1) / prefill_s, 1), "note": "untimed setup, host wall clock"},
        "phase_trace": phase_trace if args.trace else None,
        "setup_s": {"weight_generation": round(gen_s, 1), "engine_create": round(upload_s, 2),
                    "weight_upload_gbs": round(eng.uploadBytes / upload_s / 1e9, 2),
                    "note": "engine_create = streamed upload of the raw GGUF bytes (pinned ring) + model binding"},
    }
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_decode(g, spec, qq3.synth.uniform_tokens(args.prompt, SEED, spec.n_vocab),
                                         budget_s=args.cpu_seconds)
    if dist:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)
    eng.close()


PHASE_TYPES = {0: "embed", 1: "gemv", 2: "down4", 3: "attention", 4: "finish", 5: "fused"}
EPI_KINDS = {0: "store", 1: "resid", 2: "swiglu", 3: "conv", 4: "argmax"}


SUB_POINTS = ("input", "staged", "routed", "first_stage", "part1", "part2", "reduced", "published",
              "route_stage", "route_dots", "prod_routed", "prod_issue", "topk_start", "topk_ranks", "topk_done",
              "route_start")


def trace_summary(stamps, kinds, sub=None) -> dict:
    """Critical path of a traced persistent step: per phase, the end of its last CTA minus the end
    of the previous phase's last CTA, summed per phase kind (type/epilogue[/routed]).  With the
    sub-stamps, `timeline_us` gives per kind the time of each point of a phase (input wait over,
    staged, routed, first weight stage, first / second part done, reduction performed, output
    published) and of the phase end, measured from the end of the previous phase's last CTA:
    the median and the maximum over the CTAs that reach it, averaged over the phases of the kind."""
    stamps = stamps.astype(np.int64)
    t0 = int(stamps[:, 0].min())
    ends = stamps[:, 1:].max(axis=0) - t0
    out: dict = {}
    acc: dict = {}
    prev = 0
    for ph, k in enumerate(kinds):
        label = f"{PHASE_TYPES.get(int(k) & 255, '?')}/{EPI_KINDS.get((int(k) >> 8) & 255, '?')}" + \
                ("/routed" if (int(k) >> 16) & 1 else "")
        crit = int(ends[ph]) - prev
        e = out.setdefault(label, {"count": 0, "crit_us": 0.0})
        e["count"] += 1
        e["crit_us"] += crit / 1e3
        if sub is not None:
            a = acc.setdefault(label, {})
            pts = [(name, sub[:, ph, j].astype(np.int64)) for j, name in enumerate(SUB_POINTS)]
            pts.append(("end", stamps[:, ph + 1]))
            for name, col in pts:
                v = col[col > t0] - t0 - prev  # stamps of earlier steps are older than t0
                if v.size:
                    r = a.setdefault(name, [0.0, 0.0, 0])
                    r[0] += float(np.median(v)) / 1e3
                    r[1] += float(v.max()) / 1e3
                    r[2] += 1
        prev = int(ends[ph])
    for label, e in out.items():
        e["crit_us_per_phase"] = round(e["crit_us"] / e["count"], 2)
        e["crit_us"] = round(e["crit_us"], 1)
        if label in acc:
            e["timeline_us"] = {name: [round(r[0] / r[2], 2), round(r[1] / r[2], 2)]
                                for name, r in acc[label].items()}
    return {"step_us": round(int(ends[-1]) / 1e3, 1), "by_kind": out,
            "note": "one traced step (%globaltimer per CTA and phase, qq_decode_trace; timeline_us: "
                    "[median, max] over CTAs of each point, from the end of the previous phase)"}


def run_multi(args, ws, rank, local):
    """benchmark config 4 on N GPUs.  Decode (`value`): the N ranks serve N independent sequences
    (one each, the seeded 512-token prompt of rank r), each rank holding the whole model; the
    decode data path has no collective, per-GPU work is fixed (`scaling: weak`), value = N x K
    tokens / the max-over-ranks CUDA-event time.  Expert parallelism (`ep`): the same ranks also
    build the model with the experts split 32/N per rank and the library's NCCL exchange in every
    MoE layer, and time its prefill (each rank's 511 prompt tokens through the batched path) and
    its decode, with the CUDA-event split of one exchange."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    qq3 = load_package()
    qq3.build.build_all()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    t0 = time.time()
    # one rank writes the model to a GGUF file, every rank memory-maps it
    files = [None]
    if rank == 0:
        f = _model_file(SEED)
        files = [None if f is None else (str(f[0]), str(f[1]))]
    dist.broadcast_object_list(files, src=0)
    if files[0] is not None:
        g = qq3.gguf.GGUFReader.fromFile(files[0][0])
    else:
        g = qq3.synth.MemoryGGUF(spec, qq3.synth.build_tensors(spec))
    gen_s = time.time() - t0
    prompt = qq3.synth.uniform_tokens(args.prompt, SEED + rank, spec.n_vocab)
    suppress = THINK_ID if THINK_ID < spec.n_vocab else -1
    n_prof = 4
    max_ctx = args.prompt + args.warmup + 2 * args.steps + n_prof + 16

    def max_ms(v):
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    def ev():
        return torch.cuda.Event(enable_timing=True)

    # ---- decode of N independent sequences, whole model per rank
    ctx = qq3.runtime.Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    t_up = time.time()
    # sequence 1 only serves the clock-sampling soak, so sequence 0's state stays the true continuation
    eng = qq3.Lfm2CudaEngine(g, ctx=ctx, max_ctx=max_ctx, n_seq=2)
    upload_s = time.time() - t_up
    eng.prefill(prompt[:-1].tolist())
    pos = args.prompt - 1
    toks = eng.model.decode_loop(int(prompt[-1]), pos, args.warmup, suppress_id=suppress)
    pos += args.warmup
    cur = int(toks[-1])
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    with Clocks(local) as clk:
        t_soak = time.time()  # un-timed: nvidia-smi sees the clocks under this load (200 ms sampler)
        while time.time() - t_soak < 1.0:
            eng.model.decode_loop(cur, pos, args.steps, seq=1, suppress_id=suppress, want_tokens=False)
        e0.record(stream)
        out = eng.model.decode_loop(cur, pos, args.steps, suppress_id=suppress)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = max_ms(e0.elapsed_time(e1))
    pos += args.steps
    cur = int(out[-1])
    dist.barrier()
    torch.cuda.synchronize()
    e2, e3 = ev(), ev()
    e2.record(stream)
    for _ in range(args.steps):
        cur = eng.forward_argmax(cur, pos, suppress)
        pos += 1
    e3.record(stream)
    torch.cuda.synchronize()
    ms_e2e = max_ms(e2.elapsed_time(e3))
    step_kernels = eng.model.stat(qq3.runtime.QQ_STAT_STEP_KERNELS)
    eng.close()
    ctx.close()

    # ---- expert parallelism: experts split over the ranks, NCCL exchange in every MoE layer
    ctx_ep = qq3.runtime.Context(local)
    ctx_ep.set_stream(stream.cuda_stream)
    ctx_ep.comm_init_from_torch(timeout_ms=120000)
    eng_ep = qq3.Lfm2CudaEngine(g, ctx=ctx_ep, max_ctx=max_ctx, ep_world=ws)
    eng_ep.prefill(prompt[:-1].tolist())  # untimed: buffers, first-use set-up
    eng_ep.resetKVCache()
    dist.barrier()
    torch.cuda.synchronize()
    p0, p1 = ev(), ev()
    p0.record(stream)
    eng_ep.prefill(prompt[:-1].tolist())
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = max_ms(p0.elapsed_time(p1))
    eng_ep.resetKVCache()
    eng_ep.model.ep_profile(True)
    eng_ep.prefill(prompt[:-1].tolist())
    split_pf = eng_ep.model.ep_profile(False)
    pos = args.prompt - 1
    toks = eng_ep.model.decode_loop(int(prompt[-1]), pos, args.warmup, suppress_id=suppress)
    pos += args.warmup
    cur = int(toks[-1])
    dist.barrier()
    torch.cuda.synchronize()
    d0, d1 = ev(), ev()
    d0.record(stream)
    eng_ep.model.decode_loop(cur, pos, args.steps, suppress_id=suppress)
    d1.record(stream)
    torch.cuda.synchronize()
    ms_ep = max_ms(d0.elapsed_time(d1))
    pos += args.steps
    eng_ep.model.ep_profile(True)
    eng_ep.model.decode_loop(cur, pos, n_prof, suppress_id=suppress)
    split_dec = eng_ep.model.ep_profile(False)
    eng_ep.close()
    dist.barrier()
    ctx_ep.comm_destroy()
    ctx_ep.close()

    nbytes = _lfm2_model_bytes(spec)
    peak, peak_kind = _peaks()
    step_ms = ms / args.steps
    n_attn = sum(1 for i in range(spec.n_layers) if spec.is_attn(i))
    kv_bytes = n_attn * spec.n_head_kv * spec.head_dim * 4 * 2 * (args.prompt + args.warmup + args.steps / 2)
    step_bytes = nbytes["weights_per_token"] + kv_bytes
    tr = _traffic()

    def per_exchange(sp):
        n = max(sp["exchanges"], 1)
        return {k: round(sp[k] / n * 1e3, 2) for k in ("dispatch", "experts", "ret", "combine")} | {"exchanges": sp["exchanges"]}

    dec_split, pf_split = per_exchange(split_dec), per_exchange(split_pf)
    res = {
        "metric": METRIC, "value": round(ws * args.steps / (ms * 1e-3), 2), "unit": "tok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xf32 (Q8_0 weights, f32 activations)",
        "data": "synthetic (seeded random-init Q8_0 weights, seeded uniform prompt ids)",
        "config": {"workload": "LFM2-8B-A1B-shaped Q8_0 greedy decode, batch 1 per GPU (benchmark config 4)",
                   "layers": "24 (18 short-conv, 6 GQA attention; 2 dense FFN 7168, 22 MoE 32x top-4 x 1792)",
                   "hidden": 2048, "vocab": 65536, "prompt": args.prompt, "global_batch": ws,
                   "parallelism": f"{ws} sequences sharded over {ws} GPUs (whole model per GPU, no collective "
                                  f"in the decode data path); expert parallelism ep{ws} measured under 'ep'",
                   "l2": "inputs larger than L2: each step streams 1.66 GB of weights per GPU"},
        "roofline": {"bound": "hbm", "kernel": "k_decode (persistent decode step: all 24 layers + lm_head + argmax)",
                     "achieved": round(step_bytes / (step_ms * 1e-3) / 1e9, 1), "peak": peak, "peak_kind": peak_kind,
                     "unit": "GB/s", "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / peak, 4),
                     "traffic": tr.get("decode_step_bytes_per_launch"), "algorithmic_bytes": int(step_bytes),
                     "avg_launch_ms": round(step_ms, 5), "per": "GPU (max-over-ranks time)"},
        "e2e": {"value": round(ws * args.steps / (ms_e2e * 1e-3), 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": 12, "api": "Lfm2CudaEngine.forward_argmax -> qq_forward, on every rank"},
        "gpu_launches": int(step_kernels * args.steps),
        "clocks": clk.summary(),
        "ep": {"experts_per_gpu": spec.n_expert // ws,
               "prefill": {"tokens_per_gpu": args.prompt - 1, "ms": round(prefill_ms, 3),
                           "tok_s": round(ws * (args.prompt - 1) / (prefill_ms * 1e-3), 1),
                           "us_per_exchange": pf_split},
               "decode": {"tok_s": round(ws * args.steps / (ms_ep * 1e-3), 2), "ms_per_step": round(ms_ep / args.steps, 4),
                          "us_per_exchange": dec_split},
               "limiting_collective": max({"dispatch": dec_split["dispatch"], "combine (return)": dec_split["ret"]}.items(),
                                          key=lambda kv: kv[1])[0],
               "note": "max over ranks, CUDA events; one sequence per GPU; exchanges are NCCL send/recv on the "
                       "library's communicator"},
        "setup_s": {"model": round(gen_s, 1), "engine_create": round(upload_s, 2)},
    }
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


def _oracle():
    sys.path.insert(0, str(ROOT))
    from oracle import oracle as orc  # noqa: WPS433

    return orc


def _cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_decode(g, spec, prompt, steps=None, warmup: int = 0, budget_s: float = 12.0, single_s: float = 0.0,
               label: str = "LFM2-8B-A1B-shaped decode"):
    """The oracle (C restatement of the JS CPU path) on the host cores, on the same workload as
    the GPU arm: the whole prompt (all but its last token without logits, as generate() does),
    then greedy decode steps -- `steps` of them, or as many as fit in budget_s seconds -- timed on
    all host threads.  With single_s > 0 the decode then continues on one thread (the JS engine is
    single-threaded) for about that many seconds."""
    orc = _oracle()
    cores = os.cpu_count() or 1
    n_steps = steps if steps is not None else 4096
    m = orc.OracleModel(g, max_ctx=len(prompt) + warmup + n_steps + 64, threads=cores)
    t0 = time.perf_counter()
    for p, t in enumerate(prompt[:-1]):
        m.forward(int(t), p, True)
    prefill_s = time.perf_counter() - t0
    cur, pos = int(prompt[-1]), len(prompt) - 1
    for _ in range(warmup):
        cur = int(np.argmax(m.forward(cur, pos, False)))
        pos += 1
    n, t0 = 0, time.perf_counter()
    while True:
        cur = int(np.argmax(m.forward(cur, pos, False)))
        pos += 1
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and (el >= budget_s and n >= 2)) or n >= n_steps:
            break
    res = {"value": round(n / el, 4), "unit": "tok/s", "cores": cores, "kind": "port",
           "cpu_model": _cpu_model(), "nproc": cores,
           "sample": f"{label}: {len(prompt)}-token prompt ({len(prompt) - 1} prefill tokens in "
                     f"{prefill_s:.1f} s), {warmup} warm-up + {n} timed greedy steps at positions "
                     f"{len(prompt) - 1 + warmup}.., all {spec.n_layers} layers, f64-accumulating C restatement of "
                     f"the JS CPU path, {cores} threads"}
    if single_s > 0:
        orc.set_threads(1)
        k, t0 = 0, time.perf_counter()
        while True:
            cur = int(np.argmax(m.forward(cur, pos, False)))
            pos += 1
            k += 1
            el1 = time.perf_counter() - t0
            if el1 >= single_s and k >= 1:
                break
        orc.set_threads(cores)
        res["single_thread"] = {"value": round(k / el1, 4), "unit": "tok/s", "cores": 1,
                                "sample": f"{k} greedy steps on one thread, continuing the same decode"}
    return res


def _model_file(spec_seed: int) -> tuple[Path, Path] | None:
    """The config-4 model written to a GGUF file by a separate process (so that the timed CPU arm's
    process loads nothing but the oracle), plus its prompt ids, in the repository's scratch folder
    (git- and snapshot-ignored).  None when there is no room for the 8.9 GB file."""
    d = ROOT / "_scratch"
    d.mkdir(exist_ok=True)
    path = d / f"qq3_lfm2_8b_a1b_seed{spec_seed}.gguf"
    ids = path.with_suffix(".prompt.npy")
    if path.exists() and ids.exists():
        return path, ids
    st = os.statvfs(d)
    if st.f_bavail * st.f_frsize < 10 * 1024 ** 3:
        return None
    r = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--write-model", str(path)],
                       capture_output=True, text=True)
    if r.returncode == 0 and path.exists() and ids.exists():
        return path, ids
    for f in (path, ids):
        try:
            f.unlink()
        except OSError:
            pass
    return None


def write_model(path: str) -> None:
    qq3 = load_package()
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    tmp = Path(path + ".part")
    qq3.synth.write_gguf(spec, tmp)
    np.save(Path(path).with_suffix(".prompt.npy"), qq3.synth.uniform_tokens(PROMPT, SEED, spec.n_vocab))
    tmp.rename(path)


def run_reference(args, ws, rank):
    """The reference algorithm's CPU implementation on the host cores, on the GPU arm's workload:
    the same seeded model, the same 512-token prompt, then K timed greedy steps (after W warm-up
    steps) on all host threads, and a single-thread sample of the same decode."""
    if rank != 0:
        return
    qq3 = load_package()
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    files = _model_file(SEED)
    if files is not None:
        g = qq3.gguf.GGUFReader.fromFile(files[0])
        prompt = np.load(files[1])
        weights = "written by a separate process to a GGUF file, memory-mapped here"
    else:
        g = qq3.synth.MemoryGGUF(spec, qq3.synth.build_tensors(spec))
        prompt = qq3.synth.uniform_tokens(PROMPT, SEED, spec.n_vocab)
        weights = "generated in this process (no scratch directory had room for the GGUF file)"
    cb = cpu_decode(g, spec, prompt, steps=args.steps, warmup=args.warmup, single_s=args.cpu_seconds)
    res = {
        "metric": METRIC, "value": cb["value"], "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1000.0 / cb["value"], 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64 accumulate (JS numbers), f32 stores",
        "data": "synthetic (seeded random-init Q8_0 weights, seeded uniform prompt ids)", "impl": "reference",
        "config": {"workload": "LFM2-8B-A1B-shaped Q8_0 greedy decode, batch 1 (benchmark config 4)",
                   "layers": "24 (18 short-conv, 6 GQA attention; 2 dense FFN 7168, 22 MoE 32x top-4 x 1792)",
                   "hidden": 2048, "vocab": 65536, "prompt": len(prompt), "global_batch": 1,
                   "same_config": True, "weights": weights},
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)


def run_moe_block_ep(args, ws, rank, local):
    """benchmark config 3 on N GPUs: the LFM2-MoE block expert-parallel (experts sharded evenly,
    NCCL all-to-all dispatch and combine; qwenqwen3.js_b200/ep.py).  Each rank owns T token
    rows (weak scaling); one step = one EP forward of every rank's rows."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    qq3 = load_package()
    qq3.build.build_all()
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    prefix = "blk.2."
    names = {prefix + n for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                  "ffn_down_exps.weight", "exp_probs_b.bias")}
    tensors = qq3.synth.build_tensors(spec, only=names)
    ctx = qq3.runtime.Context(local)
    block = qq3.ep.EPMoEBlock(ctx, tensors, prefix, spec.n_expert, 4, rank, ws)
    T = args.tokens
    stream = torch.cuda.Stream(device=local)
    with torch.cuda.stream(stream):
        x = torch.from_numpy(qq3.synth.normal_f32(T * 2048, seed=T + 977 * rank).reshape(T, 2048)).cuda()
        for _ in range(args.warmup):
            block.forward(x)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            out = block.forward(x)
        e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    q8 = 34 / 32
    flops = ws * T * (2 * 2048 * 32 + 4 * 3 * 2 * 2048 * 1792)
    res = {"metric": "tokens/s through the LFM2-MoE block (expert-parallel)", "value": round(ws * T / (ms * 1e-3), 1),
           "unit": "tokens/s", "n_gpus": ws, "tokens_per_gpu": T, "ms_per_step": round(ms, 4),
           "tflops": round(flops / (ms * 1e-3) / 1e12, 2), "scaling": "weak", "steps": args.steps,
           "warmup": args.warmup, "parallelism": f"ep{ws}",
           "expert_bytes_per_gpu": int(spec.n_expert // ws * 3 * 2048 * 1792 * q8),
           "path": "route -> NCCL all-to-all (counts, rows, ids) -> grouped tcgen05 expert GEMMs -> "
                   "NCCL all-to-all back -> slot-order combine",
           "out_checksum": round(float(out.double().abs().sum()), 3)}
    if rank == 0:
        print(json.dumps(res), flush=True)
    block.close()
    dist.destroy_process_group()
    ctx.close()


def run_moe_block(args, ws, rank, local):
    """benchmark config 3: the isolated LFM2-MoE block on T tokens (also the small case the
    ncu captures use).  One step = one qq_moe_block call over T token rows."""
    import torch

    if ws > 1:
        run_moe_block_ep(args, ws, rank, local)
        return
    qq3 = load_package()
    qq3.build.build_all()
    torch.cuda.set_device(local)
    spec = qq3.synth.lfm2_8b_a1b(seed=SEED)
    names = {f"blk.2.{n}" for n in ("ffn_gate_inp.weight", "ffn_gate_exps.weight", "ffn_up_exps.weight",
                                    "ffn_down_exps.weight", "exp_probs_b.bias")}
    tensors = qq3.synth.build_tensors(spec, only=names)
    ctx = qq3.runtime.Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    L = qq3.runtime.LayerDesc()
    keep = []
    for name, (t, ne, raw) in tensors.items():
        suffix = name.split(".", 2)[2]
        slot = [k for k, v in qq3.runtime.SLOT_TENSOR_NAMES.items() if v == suffix][0]
        h = ctx.upload(raw, t, ne)
        keep.append(h)
        L.t[qq3.runtime.SLOT[slot]] = h.h.value
    L.is_moe = 1
    T = args.tokens
    x = torch.from_numpy(qq3.synth.normal_f32(T * 2048, seed=T).reshape(T, 2048)).cuda()
    out = torch.empty_like(x)
    rec = torch.empty((T, 40), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        ctx.moe_block(L, 32, 4, x, T, out, rec)
    ctx.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ctx.moe_block(L, 32, 4, x, T, out, rec)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ids = rec[:, :4].cpu().numpy().astype(np.int64)
    distinct = len(np.unique(ids))
    q8 = 34 / 32
    nbytes = 2048 * 32 * q8 + distinct * 3 * 2048 * 1792 * q8 + T * 2048 * 8
    flops = T * (2 * 2048 * 32 + 4 * 3 * 2 * 2048 * 1792)  # router + 4 experts x (gate, up, down) per token
    res = {"metric": "MoE-layer HBM GB/s (isolated LFM2-MoE block)", "value": round(nbytes / (ms * 1e-3) / 1e9, 1),
           "unit": "GB/s", "tokens": T, "distinct_experts": distinct, "ms_per_step": round(ms, 4),
           "tflops": round(flops / (ms * 1e-3) / 1e12, 2),
           "path": "per-token expert GEMVs" if T < 16 else "rows regrouped by expert, tcgen05 GEMMs",
           "steps": args.steps, "warmup": args.warmup,
           "note": "weights only re-read from HBM when the 375 MB of experts exceed L2 between steps"}
    if rank == 0:
        print(json.dumps(res), flush=True)
    for k in keep:
        k.free()
    ctx.close()


def run_batch_decode(args, ws, rank, local):
    """benchmark config 5, decode part: the Qwen3-8B-shaped dense model (36 layers, hidden 4096,
    32/8 heads of 128, FFN 12288, vocab 151936, untied output), 16 concurrent sequences, each
    prefilled with a seeded uniform prompt (untimed), then K greedy steps of all 16 sequences
    through the public engine API (Qwen3CudaEngine.forward_batch -> qq_forward_batch): each step
    copies 16 tokens and positions host->device and reads the 16 greedy ids back.  One step
    streams the 8.04 GB of layer and output weights once for all sequences plus every sequence's
    K/V rows (f32 cache)."""
    import torch

    qq3 = load_package()
    qq3.build.build_all()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:  # tensor-parallel: every rank holds its shards of the same model and sequences
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    spec = qq3.synth.qwen3_8b(seed=SEED)
    if args.layers:
        spec.n_layers = args.layers  # profiling knob: every layer streams the same bytes
    n = args.seqs
    prompt = args.prompt if args.prompt is not None else 4096
    g = qq3.synth.memory_model(spec)
    ctx = qq3.runtime.Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    if dist:
        ctx.comm_init_from_torch(timeout_ms=120000)
    max_ctx = prompt + args.warmup + args.steps + 1
    eng = qq3.Qwen3CudaEngine(g, ctx=ctx, max_ctx=max_ctx, n_seq=n, tp_world=ws)
    cur, pos = [], []
    t0 = time.time()
    for s in range(n):
        toks = qq3.synth.uniform_tokens(prompt, SEED + s, spec.n_vocab)
        if prompt > 1:
            eng.prefill(toks[:-1].tolist(), pos0=0, seq=s)
        cur.append(int(toks[-1]))
        pos.append(prompt - 1)
    ctx.synchronize()
    prefill_s = time.time() - t0
    if dist:
        t = torch.tensor([prefill_s], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_s = float(t[0])
    seqs = list(range(n))

    def step():
        _, am = eng.forward_batch(seqs, cur, pos, want_logits_array=False)
        for s in range(n):
            cur[s] = int(am[s])
            pos[s] += 1

    for _ in range(args.warmup):
        step()
    kv_pos = sum(pos) + n  # positions attended in the first timed step (grows by n per step)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if dist:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    L, E, F, V = spec.n_layers, spec.n_embd, spec.n_ff, spec.n_vocab
    nq, nkv = spec.n_head * spec.head_dim, spec.n_head_kv * spec.head_dim
    w_bytes = 34 / 32 * (L * (E * (2 * nq + 2 * nkv) + 3 * E * F) + E * V)
    kv_bytes = L * nkv * 4 * 2 * (kv_pos + n * (args.steps - 1) / 2)  # mean over the timed steps
    peak, kind = _peaks()
    gbs = (w_bytes + kv_bytes) / (ms * 1e-3) / 1e9
    res = {"metric": "decode tok/s (Qwen3-8B-shaped, 16 concurrent sequences)", "impl": "ours",
           "value": round(n / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
           "scaling": "strong" if ws > 1 else "weak", "parallelism": f"tp{ws}" if ws > 1 else "single GPU",
           "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "int8xf16",
           "data": "synthetic (seeded random-init Q8_0 weights, uniform prompt ids)",
           "config": {"workload": "qwen3-8b-batch-decode", "sequences": n, "prompt": prompt, "layers": L,
                      "path": "qq_forward_batch: tcgen05 GEMMs over the 16 rows, f32 KV cache",
                      "l2": "weights 8.04 GB + KV per step, far above the 126 MB L2"},
           "roofline": {"bound": "hbm", "achieved": round(gbs / ws, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / ws / peak, 4), "peak_kind": kind, "per": "GPU (each rank streams 1/N)",
                        "bytes_per_step": {"weights": round(w_bytes), "kv": round(kv_bytes)}},
           "prefill_s": round(prefill_s, 2), "clocks": clk.summary()}
    eng.close()
    if dist:
        dist.barrier()
        ctx.comm_destroy()
        dist.destroy_process_group()
    ctx.close()
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        # the reference serves one sequence per engine: one sequence, a short prompt (CPU time)
        res["cpu_baseline"] = cpu_decode(g, spec, qq3.synth.uniform_tokens(8, SEED, spec.n_vocab),
                                         budget_s=args.cpu_seconds, label="Qwen3-8B-shaped decode of one sequence")
    if rank == 0:
        print(json.dumps(res), flush=True)


def run_matmul(args, ws, rank, local):
    """benchmark config 2: one Q8_0 matmul Y[M][N] = X[M][K] . W^T (qq_q8_matmul). M = 1 runs the
    streamed GEMV, M >= 2 the tcgen05 tensor-core kernel."""
    import torch

    qq3 = load_package()
    qq3.build.build_all()
    torch.cuda.set_device(local)
    M, N, K = args.M, args.N, args.K
    ctx = qq3.runtime.Context(local)
    stream = torch.cuda.Stream(device=local)
    ctx.set_stream(stream.cuda_stream)
    W = ctx.upload(qq3.synth.q8_0_blocks(N * K, seed=N + K, mode=1), 8, [K, N])
    x = torch.from_numpy(qq3.synth.normal_f32(M * K, seed=M).reshape(M, K)).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        ctx.q8_matmul(W, x, M, y)
    ctx.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ctx.q8_matmul(W, x, M, y)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = 34 / 32 * N * K + 4 * M * K + 4 * M * N
    peak, kind = _peaks()
    res = {"metric": "Q8_0 matmul throughput", "value": round(2 * M * N * K / (ms * 1e-3) / 1e12, 2),
           "unit": "TFLOP/s", "M": M, "N": N, "K": K, "ms_per_step": round(ms, 5),
           "hbm_gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4),
           "peak_kind": kind, "path": "streamed GEMV" if M == 1 else "tcgen05 fp16 GEMM (TMEM accumulators)",
           "steps": args.steps, "warmup": args.warmup,
           "note": "weights are the same every step; M = 1 re-reads them from HBM only beyond the 126 MB L2"}
    if rank == 0:
        print(json.dumps(res), flush=True)
    W.free()
    ctx.close()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--case", choices=["decode", "moe-block", "matmul", "batch-decode"], default="decode")
    ap.add_argument("--M", type=int, default=4096, help="rows for --case matmul")
    ap.add_argument("--N", type=int, default=151936, help="output columns for --case matmul")
    ap.add_argument("--K", type=int, default=1024, help="inner dimension for --case matmul")
    ap.add_argument("--tokens", type=int, default=1, help="token rows for --case moe-block")
    ap.add_argument("--prompt", type=int, default=None,
                    help=f"prompt length (decode: {PROMPT}; batch-decode: 4096 per sequence)")
    ap.add_argument("--seqs", type=int, default=16, help="concurrent sequences for --case batch-decode")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers of the batch-decode model (profiling knob; default: all 36 of the configuration)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--n-expert", type=int, default=32,
                    help="experts per MoE layer (profiling knob: a token streams the same bytes for any count >= 4)")
    ap.add_argument("--trace", action="store_true",
                    help="add the per-phase critical-path breakdown of the persistent decode step")
    ap.add_argument("--write-model", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.write_model:
        write_model(args.write_model)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.prompt is None and args.case != "batch-decode":
        args.prompt = PROMPT
    ws, rank, local = _dist()
    if args.impl == "reference":
        run_reference(args, ws, rank)
    elif args.case == "moe-block":
        run_moe_block(args, ws, rank, local)
    elif args.case == "matmul":
        run_matmul(args, ws, rank, local)
    elif args.case == "batch-decode":
        run_batch_decode(args, ws, rank, local)
    elif ws > 1:
        run_multi(args, ws, rank, local)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()

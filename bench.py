"""Training-throughput benchmark: the 26M ZeroLLM model at seq 2048.

  python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

One step = zero_grad -> forward -> fused cross-entropy -> backward ->
(bucketed NCCL all-reduce for N > 1) -> AdamW, on one batch of 16 x 2048
synthetic token ids per GPU (uniform in [0, 6400); weights N(0, 0.02)).
N > 1 is data parallel with per-GPU batch fixed (weak scaling), launched as
one process per GPU by torch.distributed.run; the control plane (id
exchange, barriers, max over ranks) uses a gloo process group, gradients
move over the library's own NCCL communicator.

Prints one JSON line (rank 0).  `value` is measured with inputs resident in
HBM; `e2e` repeats the timing through the same public API with the step's
ids/targets copied from pinned host memory and the loss read back every
step.  `roofline` reports the dominant kernel of the step: its duration per
launch comes from CUDA events recorded around it inside training steps of the
same workload run right after the timed regions (event nodes of the step
graph, which would lengthen a timed step by ~2 %); the breakdown
(`kernels_ms`) times every kernel alone on the model's shapes.  `--impl reference` times the CPU
restatement of the reference step (the reference has no CPU path of its own)
on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train tokens/sec (26M model, seq 2048)"
# The scaled configuration (vocab 32000, d_model 2048, 24 layers, 16 heads of 128, FFN 8192, ~1.3 B
# parameters): `--model scaled`, per-GPU batch 8 x 2048, ids seeded 5 (+ rank).
SCALED = dict(vocab=32000, dim=2048, layers=24, heads=16, ffn=8192)
METRIC_SCALED = "train tokens/sec (1.3B scaled model, seq 2048)"


def flop_per_token(vocab, dim, layers, ffn, seq):
    """6 * N_gemm + 6 * L * S * d (causal attention, fwd + bwd)."""
    return 6 * (layers * (4 * dim * dim + 2 * dim * ffn) + vocab * dim) + 6 * layers * seq * dim
VOCAB, DIM, LAYERS, HEADS, FFN = 6400, 512, 6, 8, 2048


def peaks():
    p = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        p = {"hbm_gbs": float(j["hbm_gbs"]), "bf16_tflops": float(j["bf16_tflops"]),
             "bf16_tflops_sustained": float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), "source": "measured"}
    except Exception:
        pass
    return p


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
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
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- kernel breakdown
def kernel_breakdown(B, S, reps=5):
    """Times each kernel of the step alone at the model's shapes (CUDA events on the launching stream).
    Returns {name: {ms, launches_per_step, flop or bytes per launch}}."""
    import torch

    from zerollm_b200 import lib as L
    lib = L.load()
    T, d, F, V, H, Dh = B * S, DIM, FFN, VOCAB, HEADS, DIM // HEADS
    st = torch.cuda.current_stream()
    sp = C.c_void_p(st.cuda_stream)
    bf = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(0)

    def rnd(n, dt=bf, scale=1.0):
        return (torch.randn(int(n), device="cuda", generator=g) * scale).to(dt)

    ws = torch.empty(64 * 1024 * 1024, device="cuda")
    res = {}

    def timeit(name, fn, launches, work, kind):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(reps):
            fn()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        res[name] = {"ms": ms, "per_step": launches, "work": work, "kind": kind}

    KK = L.A_KMAJOR | L.B_KMAJOR
    # operand buffers large enough for every shape below: A up to [T, V], B up to [T, F]
    x, w = rnd(T * V), rnd(T * max(F, 3 * d), scale=0.02)
    out = torch.empty(T * V, device="cuda", dtype=bf)
    out32 = torch.empty(V * F, device="cuda")
    bias = torch.zeros(max(F, 3 * d), device="cuda")
    e = L.Epilogue()
    e.bias = bias.data_ptr()
    e.residual = x.data_ptr()
    e_res_elems = x.numel()

    # the model's FF1 product writes its ReLU mask as bits and the masked dF product reads them
    # (zl_gemm_bf16_relu_bits; in the step the dF product also adds the FF1 bias gradient's column sums)
    fbits = torch.empty(T * F // 32, device="cuda", dtype=torch.int32)
    bsum = torch.zeros(F, device="cuda")

    def gemm(Mm, Nn, Kk, layout, flags, o, bits_out=None, bits_in=None):
        if bits_out is not None:
            L.call("zl_gemm_bf16_relu_bits", x.data_ptr(), w.data_ptr(), o.data_ptr(), Mm, Nn, Kk, layout, flags,
                   C.byref(e), ws.data_ptr(), bits_out.data_ptr(), None, sp)
        elif bits_in is not None:
            L.call("zl_gemm_bf16_relu_bits", x.data_ptr(), w.data_ptr(), o.data_ptr(), Mm, Nn, Kk, layout,
                   flags | L.EPI_RELU_MASK, C.byref(L.Epilogue()), ws.data_ptr(), None, bits_in.data_ptr(), sp)
        else:
            L.call("zl_gemm_bf16", x.data_ptr(), w.data_ptr(), o.data_ptr(), Mm, Nn, Kk, layout, flags, C.byref(e),
                   ws.data_ptr(), sp)

    shapes = [
        ("gemm_fwd_qkv", T, 3 * d, d, KK, L.EPI_BIAS, out),
        ("gemm_fwd_out", T, d, d, KK, L.EPI_BIAS | L.EPI_RESIDUAL, out),
        ("gemm_fwd_ff1", T, F, d, KK, L.EPI_BIAS | L.EPI_RELU, out),
        ("gemm_fwd_ff2", T, d, F, KK, L.EPI_BIAS | L.EPI_RESIDUAL, out),
        ("gemm_fwd_head", T, V, d, KK, 0, out),
        ("gemm_dx_head", T, d, V, L.A_KMAJOR, 0, out),
        ("gemm_dw_head", V, d, T, 0, L.EPI_OUT_F32 | L.EPI_ACCUM, out32),
        ("gemm_dx_ff2", T, F, d, L.A_KMAJOR, 0, out),
        ("gemm_dw_ff2", d, F, T, 0, L.EPI_OUT_F32, out32),
        ("gemm_dx_ff1", T, d, F, L.A_KMAJOR, L.EPI_RESIDUAL, out),
        ("gemm_dw_ff1", F, d, T, 0, L.EPI_OUT_F32, out32),
        ("gemm_dx_out", T, d, d, L.A_KMAJOR, 0, out),
        ("gemm_dw_out", d, d, T, 0, L.EPI_OUT_F32, out32),
        ("gemm_dx_qkv", T, d, 3 * d, L.A_KMAJOR, L.EPI_RESIDUAL, out),
        ("gemm_dw_qkv", 3 * d, d, T, 0, L.EPI_OUT_F32, out32),
    ]
    for name, Mm, Nn, Kk, lay, fl, o in shapes:
        a_elems, b_elems, d_elems = Mm * Kk, Nn * Kk, Mm * Nn
        assert a_elems <= x.numel() and b_elems <= w.numel() and d_elems <= o.numel() and d_elems <= e_res_elems
        n_per_step = 1 if "head" in name else LAYERS
        bo = fbits if name == "gemm_fwd_ff1" else None
        bi = fbits if name == "gemm_dx_ff2" else None
        timeit(name, lambda Mm=Mm, Nn=Nn, Kk=Kk, lay=lay, fl=fl, o=o, bo=bo, bi=bi: gemm(Mm, Nn, Kk, lay, fl, o, bo, bi),
               n_per_step, 2.0 * Mm * Nn * Kk, "tensor")
    qkv = rnd(T * 3 * d, scale=0.5)
    ob, dob = rnd(T * d), rnd(T * d)
    lse = torch.empty(B * H * S, device="cuda")
    dqkv = torch.empty(T * 3 * d, device="cuda", dtype=bf)
    attn_flop = 2.0 * B * H * S * S * Dh  # causal forward (QK^T + PV over the lower triangle)
    timeit("attention_fwd", lambda: L.call("zl_attention_forward_bf16", qkv.data_ptr(), ob.data_ptr(), lse.data_ptr(),
                                           B, S, H, Dh, sp), LAYERS, attn_flop, "tensor")
    timeit("attention_bwd", lambda: L.call("zl_attention_backward_bf16", qkv.data_ptr(), ob.data_ptr(),
                                           dob.data_ptr(), lse.data_ptr(), dqkv.data_ptr(), ws.data_ptr(), B, S, H,
                                           Dh, None, None, sp), LAYERS, 2 * attn_flop, "tensor")
    g1 = torch.ones(F, device="cuda")
    y, mean, rstd = rnd(T * d), torch.empty(T, device="cuda"), torch.empty(T, device="cuda")
    timeit("norm_fwd", lambda: L.call("zl_norm_forward_bf16", 1, x.data_ptr(), g1.data_ptr(), None, y.data_ptr(),
                                      None, rstd.data_ptr(), T, d, 1e-5, sp), 2 * LAYERS + 1, 2.0 * T * d * 2, "hbm")
    dg = torch.zeros(F, device="cuda")
    timeit("norm_bwd", lambda: L.call("zl_norm_backward_bf16", 1, x.data_ptr(), y.data_ptr(), g1.data_ptr(), None,
                                      rstd.data_ptr(), out.data_ptr(), dg.data_ptr(), None, ws.data_ptr(), T, d, sp),
           2 * LAYERS + 1, 3.0 * T * d * 2, "hbm")
    logits = rnd(T * V)
    tg = torch.randint(0, V, (T,), device="cuda", dtype=torch.int32)
    lrow, lo = torch.empty(T, device="cuda"), torch.empty(1, device="cuda")
    timeit("cross_entropy", lambda: L.call("zl_cross_entropy_fused_bf16", logits.data_ptr(), tg.data_ptr(), T, V,
                                           1e-8, 1.0 / T, lrow.data_ptr(), lo.data_ptr(), sp), 1, 2.0 * T * V * 2,
           "hbm")
    NP = 25462272
    p, gr, m, v = (torch.zeros(NP, device="cuda") for _ in range(4))
    pb = torch.empty(NP, device="cuda", dtype=bf)
    timeit("adamw", lambda: L.call("zl_adamw_flat", p.data_ptr(), gr.data_ptr(), m.data_ptr(), v.data_ptr(),
                                   pb.data_ptr(), NP, 3e-4, 0.1, 0.9, 0.95, 1e-8, 0.1, 0.05, 1.0, sp), 1,
           NP * (28.0 + 2.0), "hbm")
    timeit("colsum_ff1", lambda: L.call("zl_colsum_bf16", x.data_ptr(), dg.data_ptr(), ws.data_ptr(), T, F, sp),
           LAYERS, 2.0 * T * F, "hbm")
    ids = torch.randint(0, V, (T,), device="cuda", dtype=torch.int32)
    tab = torch.zeros(V * d, device="cuda")
    timeit("embedding_fwd", lambda: L.call("zl_embedding_forward_bf16", ids.data_ptr(), tab.data_ptr(), None,
                                           y.data_ptr(), T, S, d, V, sp), 1, T * d * (4.0 + 2.0), "hbm")
    timeit("embedding_bwd", lambda: L.call("zl_embedding_backward_bf16", ids.data_ptr(), y.data_ptr(),
                                           tab.data_ptr(), T, d, V, sp), 1, T * d * (2.0 + 8.0), "hbm")
    del x, w, out, out32, p, gr, m, v, pb, logits
    torch.cuda.empty_cache()
    return res


def roofline_of(bd, pk, live=None):
    """The dominant kernel of the breakdown.  Its duration per launch is the in-step one (CUDA events
    recorded around the kernel inside the last timed step) when `live` has it, else the alone-timing."""
    total = {k: v["ms"] * v["per_step"] for k, v in bd.items()}
    dom = max(total, key=total.get)
    r = bd[dom]
    live = live or {}
    ms = live.get(dom, r["ms"])
    timing = ("CUDA events (event nodes of the step graph) around the kernel in training steps run right "
              "after the timed region on the same inputs, mean over a step's launches" if dom in live
              else "kernel timed alone with CUDA events")
    if r["kind"] == "tensor":
        ach = r["work"] / (ms * 1e-3) / 1e12
        peak, unit, bound = pk["bf16_tflops"], "TFLOP/s", "tensor"
    else:
        ach = r["work"] / (ms * 1e-3) / 1e9
        peak, unit, bound = pk["hbm_gbs"], "GB/s", "hbm"
    traffic = None
    tf = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if os.path.exists(tf):
        for ln in open(tf):
            f = ln.split()
            if len(f) >= 2 and f[0] == dom:
                traffic = float(f[1])
    return {"kernel": dom, "bound": bound, "achieved": round(ach, 2), "peak": peak, "unit": unit,
            "frac": round(ach / peak, 4), "traffic": traffic, "ms_per_launch": round(ms, 4),
            "ms_per_launch_alone": round(r["ms"], 4), "timing": timing,
            "share_of_kernel_time": round(total[dom] / sum(total.values()), 4), "peak_source": pk["source"]}


# ---------------------------------------------------------------------------- CPU baseline (oracle)
def host_cores():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def cpu_sample(B=1, S=2048, steps=1, threads=None):
    """fp32 training step(s) of the 26M model (baseline topology) on the CPU restatement, with an
    explicit OpenMP team size (default: every core this process may run on).  The size is set
    through the oracle itself, because a multi-process launcher exports OMP_NUM_THREADS=1."""
    from oracle import oracle as O
    import numpy as np
    want = threads or host_cores()
    used = O.set_threads(want)
    m = O.Model(max_seq=max(S, 2048))
    p = O.init_params(m, seed=0)
    mm, vv = np.zeros_like(p), np.zeros_like(p)
    ids = O.uniform_ids(B * (S + 1), 3, VOCAB).reshape(B, S + 1)
    inp, tgt = ids[:, :S].ravel().copy(), ids[:, 1:].ravel().copy()
    t0 = time.perf_counter()
    for i in range(steps):
        O.train_step(m, p, mm, vv, inp, tgt, B, S, step=i + 1)
    dt = time.perf_counter() - t0
    return {"value": round(B * S * steps / dt, 2), "unit": "tokens/s", "cores": used, "kind": "port",
            "sample": f"{steps} fp32 step(s) of {B}x{S} tokens, 26M model, oracle/liboracle.so (OpenMP, "
                      f"{used} threads)",
            "seconds": round(dt, 2)}


def cpu_single_thread():
    """The single-core figure beside the all-core one: one fp32 step of one 256-token sequence
    (a few seconds on one core; the seq-2048 step would take about a minute)."""
    r = cpu_sample(1, 256, 1, threads=1)
    r["seq_len"] = 256
    return r


def run_reference(args, rank, world):
    if rank != 0:
        return
    W, K = args.warmup, args.steps
    # bounded sample per step: one sequence of 2048 tokens (the CPU restatement; the reference has no CPU path)
    for _ in range(W):
        cpu_sample(1, 2048, 1)
    t0 = time.perf_counter()
    samples = []
    for _ in range(K):
        samples.append(cpu_sample(1, 2048, 1))
    dt = time.perf_counter() - t0
    tok = 2048 * K
    v = round(tok / dt, 2)
    one = cpu_single_thread()
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": K, "warmup": W,
            "ms_per_step": round(1e3 * dt / K, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "26M ZeroLLM train step, seq 2048, CPU sample of 1x2048 tokens per step",
                       "global_batch": 1, "seq_len": 2048, "parallelism": "cpu"},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": samples[0]["cores"], "kind": "port",
                             "sample": "1x2048 tokens per step, fp32 fwd+bwd+AdamW, oracle/liboracle.so",
                             "single_thread": one},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


# ---------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist

    from zerollm_b200 import Config, ZeroLLM, nccl_unique_id

    torch.cuda.set_device(local_rank)
    B, S = args.batch, args.seq
    T = B * S
    if world > 1:
        uid = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
    scaled = args.model == "scaled"
    if scaled:
        cfg = Config(vocab_size=SCALED["vocab"], embed_dim=SCALED["dim"], num_layers=SCALED["layers"],
                     num_heads=SCALED["heads"], ff_hidden_dim=SCALED["ffn"], max_seq_len=S)
    else:
        cfg = Config.baseline_26m()
    model = ZeroLLM(cfg, T, seed=0, init_std=0.02)
    model.set_optimizer(0.9, 0.95, 1e-8, 0.1)
    if world > 1:
        model.attach_nccl(uid[0], rank, world, 25 * 1024 * 1024)
    seed = (5 + rank) if scaled else (3 if world == 1 else 4 + rank)
    rng = np.random.default_rng(seed)
    ids = rng.integers(0, cfg.vocab_size, size=(B, S + 1), dtype=np.int32)
    h_inp = torch.from_numpy(np.ascontiguousarray(ids[:, :S])).reshape(-1).pin_memory()
    h_tgt = torch.from_numpy(np.ascontiguousarray(ids[:, 1:])).reshape(-1).pin_memory()
    d_inp, d_tgt = h_inp.cuda(), h_tgt.cuda()
    st = torch.cuda.current_stream()
    lr = 3e-4

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        model.train_step(d_inp, d_tgt, B, S, lr)
    barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.steps):
        model.train_step(d_inp, d_tgt, B, S, lr)
    e1.record(st)
    barrier()
    ck = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    launches = model.last_launches() * args.steps
    loss_now = model.loss_dev.item()

    # end-to-end through the public API: H2D of ids/targets from pinned memory + D2H of the loss per step
    h_loss = torch.empty(1, dtype=torch.float32).pin_memory()
    for _ in range(2):
        d_inp.copy_(h_inp, non_blocking=True)
        d_tgt.copy_(h_tgt, non_blocking=True)
        h_loss.copy_(model.train_step(d_inp, d_tgt, B, S, lr), non_blocking=True)
    barrier()
    t0 = time.perf_counter()
    e0.record(st)
    for _ in range(args.steps):
        d_inp.copy_(h_inp, non_blocking=True)
        d_tgt.copy_(h_tgt, non_blocking=True)
        h_loss.copy_(model.train_step(d_inp, d_tgt, B, S, lr), non_blocking=True)
    e1.record(st)
    barrier()
    wall = time.perf_counter() - t0
    ms_e2e = max_over_ranks(max(e0.elapsed_time(e1) / args.steps, 1e3 * wall / args.steps))
    # In-step kernel durations for the roofline, and the step's phases: the same steps again, with
    # timing-event nodes around each layer's attention kernels and at the step's start, after its last
    # backward kernel and after the gradient exchange has rejoined (every rank takes these steps).
    # The timed regions above run without them, since the nodes lengthen the step by ~2 %.
    model.set_kernel_timing(True)
    for _ in range(3):
        model.train_step(d_inp, d_tgt, B, S, lr)
    in_step = model.kernel_times()
    step_ms_t, exposed_ms = model.step_times()
    model.set_kernel_timing(False)
    in_step = (max_over_ranks(in_step[0]), max_over_ranks(in_step[1]))
    phases = {"step_ms": round(max_over_ranks(step_ms_t), 3),
              "exposed_exchange_ms": round(max_over_ranks(exposed_ms), 3),
              "timing": "event nodes in three extra steps after the timed regions, max over ranks; "
                        "exposed_exchange_ms = end of the last backward kernel to the rejoin of the "
                        "all-reduce side stream (AdamW not included in step_ms)"}
    csum = model.checksum()
    consistent = True
    if world > 1:
        allc = [None] * world
        dist.all_gather_object(allc, csum)
        consistent = all(c == allc[0] for c in allc)
    model.close()
    del model
    torch.cuda.empty_cache()

    bd, roof = None, None
    if rank == 0 and not args.no_breakdown and not scaled:
        bd = kernel_breakdown(B, S)
        roof = roofline_of(bd, peaks(), {"attention_fwd": in_step[0], "attention_bwd": in_step[1]} if in_step else None)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and not scaled:
        cpu = cpu_sample(1, 2048, 1)
        cpu["single_thread"] = cpu_single_thread()
    if rank != 0:
        return
    tokens = T * world
    value = tokens / (ms * 1e-3)
    pk = peaks()
    fpt = flop_per_token(cfg.vocab_size, cfg.embed_dim, cfg.num_layers, cfg.ff_hidden_dim, S)
    name = "1.3B scaled ZeroLLM" if scaled else "26M ZeroLLM"
    line = {
        "metric": METRIC_SCALED if scaled else METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic (uniform ids in [0,{cfg.vocab_size}), N(0,0.02) weights)",
        "config": {"workload": f"{name} training step (RMSNorm, RoPE, untied head), batch {B} x seq {S} per GPU",
                   "model": "zerollm-1.3b-scaled" if scaled else "zerollm-26m", "global_batch": B * world,
                   "seq_len": S, "parallelism": f"dp{world}",
                   "l2": "inputs larger than L2 (per-step working set of several GB)"},
        "mfu": round(value * fpt / world / (pk["bf16_tflops"] * 1e12), 4),
        "flop_per_token": fpt,
        "e2e": {"value": round(tokens / (ms_e2e * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": int(2 * T * 4), "d2h_bytes_per_step": 4},
        "gpu_launches": launches,
        "clocks": ck,
        "loss": round(loss_now, 4),
        "weights_identical_across_ranks": consistent,
    }
    if in_step:
        line["attention_ms_in_step"] = {"fwd": round(in_step[0], 4), "bwd": round(in_step[1], 4)}
        line["step_phases"] = phases
    if roof:
        line["roofline"] = roof
        line["kernels_ms"] = {k: round(v["ms"], 4) for k, v in bd.items()}
    if cpu:
        line["cpu_baseline"] = cpu
    emit(line)


_RESULT_OUT = None


def emit(line: dict) -> None:
    """Writes the result line to the process's original standard output."""
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def claim_stdout() -> None:
    """The result is one JSON line on standard output, but native libraries may write there too
    (NCCL prints a version banner when its debug level asks for one): from here on file descriptor 1
    points at standard error, and emit() writes to a copy of the original."""
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def main():
    claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="26m", choices=["26m", "scaled"])
    ap.add_argument("--batch", type=int, default=None, help="per-GPU batch (default 16; 8 for --model scaled)")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--no-breakdown", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--kernels-only", action="store_true",
                    help="time each kernel of the step alone at the model's shapes (batch --batch) and exit; "
                         "the small driver for per-kernel ncu captures")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.batch is None:
        args.batch = 8 if args.model == "scaled" else 16
    if args.kernels_only:
        import torch
        torch.cuda.set_device(0)
        bd = kernel_breakdown(args.batch, args.seq, reps=2)
        emit({"kernels_only": True, "batch": args.batch, "seq_len": args.seq,
              "kernels_ms": {k: round(v["ms"], 4) for k, v in bd.items()}})
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

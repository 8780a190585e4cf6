#!/usr/bin/env python3
"""Benchmark of the quantized decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): the Q4_K decode matvec sweep at batch 1 -- one y = W.x
over each matrix of a rotation set of 16 distinct 11008x4096 and 16 distinct
4096x4096 Q4_K matrices (557 MB > 4x the 126 MB L2, so every step streams its
weights from HBM).  The 32 independent matvecs of a step are one
GpuDispatch::matvec_lote, which the library runs as ONE launch
(sbk_matvec_batch: the weight streams of all 32 matrices split evenly over all
SMs), captured in a CUDA graph.  Weights are synthetic (uniform 4-bit codes /
6-bit scales, f16 d,dmin in U[1e-4,1e-3]), x ~ N(0,1), seeded.

Reported: `value` = algorithmic bytes (weights + x + y) per step / device time
per step, device-resident inputs; `e2e` = the same through the C ABI's
GpuDispatch surface (sb_matvec_batch: host x in, host y out, copies and the
sync inside the timed region); `roofline` for the matvec kernel against the
measured HBM copy bandwidth; `cpu_baseline` = the reference's AVX2 Q4_K kernel
(restated, all host cores) on a bounded sample.  With N > 1 (torchrun) every
rank runs its own rotation set on its own GPU (rows are independent: weak
scaling, no collective on the data path); `value` sums all ranks over the
slowest rank's time.

--impl reference times the reference's CPU implementation of the path (the
restated AVX2 kernel, all host threads) on the same workload, a bounded sample
per step, and prints the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_K matvec HBM GB/s (% of peak)"
UNIT = "GB/s"
SHAPES = [(11008, 4096), (4096, 4096)]  # BASELINE.json configs[1], Q4_K shapes
COPIES = 16
Q4K = 3


def algo_bytes(rows: int, cols: int) -> int:
    return rows * (cols // 256) * 144 + cols * 4 + rows * 4


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profile_traffic() -> int | None:
    """DRAM bytes (read + write) per launch of the step's kernel, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "q4k_mmv_batch_sweep.txt")
    if os.path.exists(p):
        with open(p) as f:
            for line in f:
                line = line.strip()
                if line.startswith("dram_bytes_per_launch:"):
                    return int(line.split(":", 1)[1].split()[0])
    return None


def bench_mats(rank: int):
    """The rotation set of one rank: COPIES distinct matrices of each shape, with their x."""
    from soso_b200 import synth
    mats = []
    for rows, cols in SHAPES:
        for k in range(COPIES):
            g = synth.rng("bench", rank, rows, cols, k)
            w = synth.random_weights(Q4K, rows, cols, g)
            x = synth.randn(cols, g)
            mats.append((rows, cols, w, x))
    return mats


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class Clocks:
    """nvidia-smi sampling during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.p = None

    def stop(self) -> dict | None:
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
            out, _ = self.p.communicate()
        sms, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [t.strip() for t in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": float(np.median(sms)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sms)}


def cpu_sample_gbs(seconds: float, threads: int) -> dict:
    """The reference's AVX2 Q4_K matvec (gemm.rs:842-894, restated in oracle/) on the
    host cores: both BASELINE shapes once per pass, as many passes as fit `seconds`."""
    import oracle
    from soso_b200 import synth
    mats = []
    for rows, cols in SHAPES:
        g = synth.rng("bench", "cpu", rows, cols)
        mats.append((synth.random_weights(Q4K, rows, cols, g), rows, cols, synth.randn(cols, g),
                     np.empty(rows, np.float32)))
    oracle.cpu_matvec(Q4K, mats[1][0], mats[1][1], mats[1][2], mats[1][3], threads, mats[1][4])  # warm
    t0, passes, nbytes = time.perf_counter(), 0, 0
    while True:
        for w, rows, cols, x, y in mats:
            oracle.cpu_matvec(Q4K, w, rows, cols, x, threads, y)
            nbytes += algo_bytes(rows, cols)
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": nbytes / el / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{passes} passes of Q4_K 11008x4096 + 4096x4096 matvec ({el:.1f} s)"}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# --------------------------------------------------------------- our arm
def run_ours(args) -> None:
    import torch

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        # (long enough for rank 0's one-GPU agreement run of a decode model while the others wait)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=480), device_id=dev)

    from soso_b200 import synth
    from soso_b200._lib import SbkMvOp, SbMatvecOp, SbView, c_f32p, c_u8p, last_error, lib
    L = lib()

    mats = bench_mats(rank)
    wd = [torch.from_numpy(m[2]).to(dev) for m in mats]
    xd = [torch.from_numpy(m[3]).to(dev) for m in mats]
    yd = [torch.empty(m[0], device=dev, dtype=torch.float32) for m in mats]
    step_bytes = sum(algo_bytes(m[0], m[1]) for m in mats)
    # the step is one GpuDispatch::matvec_lote of all 32 independent matvecs: one launch
    batch = (SbkMvOp * len(mats))()
    for i, ((rows, cols, _, _), w, x, y) in enumerate(zip(mats, wd, xd, yd)):
        batch[i] = SbkMvOp(w.data_ptr(), rows, cols, x.data_ptr(), y.data_ptr())
    launches_per_step = 1

    stream = torch.cuda.Stream(dev)

    def enqueue():
        s = torch.cuda.current_stream().cuda_stream
        rc = L.sbk_matvec_batch(Q4K, batch, len(mats), 1, s)
        if rc:
            raise RuntimeError(f"sbk_matvec_batch rc={rc}")

    with torch.cuda.stream(stream):
        enqueue()  # warm (sets smem attributes outside capture)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        enqueue()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    # keep the GPU busy a little longer so the sampler sees load if the region was short
    with torch.cuda.stream(stream):
        for _ in range(max(1, int(200.0 / max(ms / args.steps, 1e-3)))):
            graph.replay()
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # one matvec per launch (dependent-chain style), for reference: graph of PDL launches
    single = {}
    for (rows, cols) in SHAPES:
        idx = [i for i, m in enumerate(mats) if (m[0], m[1]) == (rows, cols)]
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            for i in idx:
                L.sbk_matvec(Q4K, wd[i].data_ptr(), rows, cols, xd[i].data_ptr(), yd[i].data_ptr(), 1,
                             stream.cuda_stream)
        torch.cuda.synchronize()
        with torch.cuda.graph(g1, stream=stream):
            for i in idx:
                L.sbk_matvec(Q4K, wd[i].data_ptr(), rows, cols, xd[i].data_ptr(), yd[i].data_ptr(), 1,
                             torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            g1.replay()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a0.record(stream)
            for _ in range(5):
                g1.replay()
            a1.record(stream)
        torch.cuda.synchronize()
        us = a0.elapsed_time(a1) * 1e3 / (5 * len(idx))
        single[f"{rows}x{cols}"] = {"us_per_launch": round(us, 2),
                                    "GBps": round(algo_bytes(rows, cols) / us / 1e3, 1)}
        del g1

    # e2e through the GpuDispatch surface: host x in, host y out, one wait per step
    views, keys, ops = [], [], (SbMatvecOp * len(mats))()
    hx = [np.ascontiguousarray(m[3]) for m in mats]
    hy = [np.empty(m[0], np.float32) for m in mats]
    import ctypes
    h = ctypes.c_void_p()
    if L.sb_create(local, ctypes.byref(h)) != 0:
        raise RuntimeError(last_error())
    ctx = h
    for i, (rows, cols, w, _) in enumerate(mats):
        views.append(SbView(w.ctypes.data_as(c_u8p), w.size, Q4K, rows * cols))
        keys.append(f"bench.{i}".encode())
    for i, (rows, cols, _, _) in enumerate(mats):
        ops[i] = SbMatvecOp(keys[i], ctypes.pointer(views[i]), rows, cols, hx[i].ctypes.data_as(c_f32p),
                            hy[i].ctypes.data_as(c_f32p))
    done = (ctypes.c_uint8 * len(mats))()
    for _ in range(max(1, args.warmup)):
        if L.sb_matvec_batch(ctx, ops, len(mats), done) != 1:
            raise RuntimeError(last_error())
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        L.sb_matvec_batch(ctx, ops, len(mats), done)
    e2e_s = time.perf_counter() - t0
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    L.sb_destroy(ctx)

    # the other BASELINE configs: C1 (Q8_0 matvec), the decode models (C3 dense, C4 MoE, C5
    # MLA+MoE; one model split over the ranks at N > 1), and the tcgen05 prefill GEMM on C5's
    # prefill shapes (N = 1)
    extra = {}
    if not args.no_decode:
        extra["c1_q8_0_matvec"] = q80_bench(dev)
        extra["decode"] = decode_bench(local, rank, "dense", world)
        extra["decode_moe"] = decode_bench(local, rank, "moe", world)
        extra["decode_mla"] = decode_bench(local, rank, "mla", world)
        if world == 1:
            extra["prefill"] = prefill_bench(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample_gbs(args.cpu_seconds, host_threads())

    if rank == 0:
        peaks = load_peaks()
        per_step_s = ms / 1e3 / args.steps
        value = world * step_bytes / per_step_s / 1e9
        per_launch_bytes = step_bytes / launches_per_step
        achieved = per_launch_bytes / (per_step_s / launches_per_step) / 1e9  # one launch per step
        traffic = profile_traffic()
        h2d = sum(m[1] * 4 for m in mats)
        d2h = sum(m[0] * 4 for m in mats)
        summary = {"q4k_GBps": round(value, 1), "q4k_frac": round(achieved / peaks["hbm_gbs"], 4)}
        for k, v in extra.items():
            if k.startswith("decode"):
                summary[k + "_tok_s"] = v["tok_per_s"]
                summary[k + "_frac"] = v["roofline"]["frac"]
                if "prefill" in v:
                    summary[k + "_prefill_ms"] = v["prefill"]["ms"]
                    summary[k + "_prefill_frac"] = v["prefill"]["frac_of_bf16_peak"]
                if "agreement_vs_1gpu" in v and v["agreement_vs_1gpu"]:
                    ag = v["agreement_vs_1gpu"]
                    summary[k + "_identical_vs_1gpu"] = ag["identical_frac"]
                    rd = ag.get("first_route_difference")
                    if rd:  # [position, router-logit gap there (whole run), first token divergence position]
                        summary[k + "_route_tie"] = [rd["position"], rd["router_gap_1gpu"],
                                                     rd["first_token_divergence_position"]]
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "summary": summary, "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "pct_of_peak": round(100.0 * value / world / peaks["hbm_gbs"], 1),
            "config": {
                "workload": f"Q4_K decode matvec sweep, batch 1: {COPIES}x 11008x4096 + {COPIES}x 4096x4096 "
                            "independent matvecs per step (BASELINE configs[1] Q4_K shapes) as one "
                            "matvec_lote (sbk_matvec_batch: one launch per step), CUDA graph",
                "rotation_bytes_per_gpu": int(sum(m[2].size for m in mats)),
                "l2": "inputs larger than L2 (557 MB rotation set per GPU, each matrix read once per step)",
                "parallelism": f"independent rotation sets per GPU x{world}",
            },
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic, "algorithmic_bytes_per_launch": int(per_launch_bytes),
                         "kernel": "sb::tcmv::tc_mmv_kernel<Q4K>"},
            "e2e": {"value": round(world * step_bytes / (e2e_s / args.steps) / 1e9, 1), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "sb_matvec_batch (GpuDispatch::matvec_lote), weights resident"},
            "gpu_launches": args.steps * launches_per_step,
            "single_matvec_launch": single,
            "clocks": clk,
        }
        for k, v in extra.items():
            line[k] = v
        if cpu:
            line["cpu_baseline"] = cpu
        # the same summary again as the line's last key: a reader that keeps only the end of a
        # long line still sees every config's tokens/s, roofline fraction and agreement
        line["summary_tail"] = summary
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        del graph
        dist.destroy_process_group()


def weight_bytes_per_token(cfg) -> float:
    """Weight bytes one decode token reads (reference layouts): every layer's attention and
    dense FFN or router + top_k routed experts + shared expert, and the output matrix; the
    same whatever the split over GPUs."""
    from soso_b200 import decode
    from soso_b200.formats import row_bytes
    H, total = cfg.hidden, 0.0
    for l in range(cfg.n_layers):
        for name, (rows, cols) in decode.shapes(cfg).items():
            if cfg.is_moe(l) and name.startswith("ffn_"):
                continue
            total += rows * row_bytes(cfg.dtypes[name], cols)
        if cfg.is_moe(l):
            total += cfg.n_exp * row_bytes(cfg.dtypes["ffn_gate_inp"], H)
            f = cfg.top_k * cfg.moe_ffn + cfg.shared_ffn
            total += 2 * f * row_bytes(cfg.dtypes["ffn_gate"], H)
            total += H * (cfg.top_k * row_bytes(cfg.dtypes["ffn_down"], cfg.moe_ffn)
                          + (row_bytes(cfg.dtypes["ffn_down"], cfg.shared_ffn) if cfg.shared_ffn else 0))
    return total + cfg.vocab * row_bytes(cfg.dtypes["output"], H)


def parallelism(cfg, world: int) -> str:
    """How the library splits a decode model over `world` GPUs (soso_b200.tp)."""
    from soso_b200 import tp
    parts = []
    parts.append(f"attention tp{world} (query heads)" if tp.attention_split(cfg, world) else
                 "attention whole on every rank")
    if cfg.ffn and cfg.ffn % 256 == 0:
        parts.append(f"dense FFN tp{world} (256-column blocks)")
    elif cfg.ffn:
        parts.append("dense FFN whole on every rank")
    if cfg.n_exp:
        parts.append(f"experts ep{world} (expert IDs split, router on every rank"
                     + (", shared expert on rank layer % world" if cfg.shared_ffn else "") + ")")
    parts.append("vocabulary rows split")
    return "; ".join(parts) + ("; partial sums and expert outputs exchanged through peer memory inside the "
                               "matvec kernels")


def decode_bench(device: int, rank: int, which: str = "dense", world: int = 1) -> dict:
    """Whole-token decode through the engine (sb_decode_greedy: one CUDA graph per token,
    tokens chained on the device), batch-1 greedy decode of 256 tokens after a 128-token
    random prompt.  which = "dense": BASELINE.json configs[2] (Qwen2.5-3B-style, Q4_K_M mix,
    fp16 KV at 4096); "moe": configs[3] (Qwen3-30B-A3B-style, 128 experts top-8, all Q4_K,
    fp16 KV at 2048).  Timed: the 256 generated tokens (wall clock around the call, which
    ends with a stream synchronize).  Bytes per token = weights read per token (attention,
    router, the top-k experts' matrices, output matrix) + the KV rows read at the average
    position."""
    from soso_b200 import decode, synth
    cfg = {"dense": decode.QWEN25_3B, "moe": decode.QWEN3_30B_A3B, "mla": decode.DEEPSEEK_V2_LITE}[which]
    group = None
    if world > 1:  # tensor-parallel across the ranks (one model, sharded by the library)
        from soso_b200 import tp
        group = (rank, world, tp.torch_all_gather())
    seed = f"{which}.{rank if group is None else 0}"
    # under expert parallelism a rank makes only the experts it holds (same bytes as whole)
    model = decode.synth_model(cfg, seed, held=(rank, world) if group and cfg.n_exp else None)
    sess = decode.DecodeSession(cfg, model, device=device, group=group)
    n_prompt = 512 if which == "mla" else 128  # configs[4]: a 512-token prefill, then decode
    prompt = synth.rng("prompt", which, 0 if group else rank).integers(0, cfg.vocab, n_prompt).astype(np.int32)
    sess.greedy(prompt[:8], 8)  # warm
    pf = None
    if group is None:
        # the prompt as one block on the tensor cores (sb_decode_prefill), timed over 3 runs
        sess.prefill(prompt)  # warm: buffers and weight maps
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            _, nxt = sess.prefill(prompt, logits=False)
            times.append(time.perf_counter() - t0)
        ms = 1e3 * sorted(times)[1]
        fl = prefill_flops(cfg, n_prompt)
        tf = fl / (ms / 1e3) / 1e12
        pf = {"tokens": n_prompt, "ms": round(ms, 3), "TFLOPs": round(tf, 1),
              "frac_of_bf16_peak": round(tf / load_bf16_peak(), 4), "flops": int(fl),
              "timing": "wall clock around sb_decode_prefill (tables and tokens up, every layer, last token's "
                        "logits and argmax down), median of 3"}
        first = np.array([nxt], np.int32)
    else:
        first = sess.greedy(prompt, n_prompt)[-1:]  # the prompt, one token per step
    n_gen = 256
    if group:
        group[2](b"go")  # start the timed region together
    t0 = time.perf_counter()
    toks = sess.greedy(first[-1:], n_gen, pos=n_prompt)
    dt = time.perf_counter() - t0
    if group:
        dt = max(float(v) for v in group[2](repr(dt).encode()))  # the slowest rank
    weights = weight_bytes_per_token(cfg)
    # cache bytes read per cached position: K and V rows (f16), or the latent row (f16) and the
    # rope keys (f32) of an MLA layer
    kv_per_pos = (cfg.n_layers * (cfg.kv_rank * 2 + cfg.kv_heads * cfg.qk_rope * 4) if cfg.mla
                  else cfg.n_layers * 2 * cfg.kv_dim * 2)
    avg_ctx = n_prompt + (n_gen + 1) / 2.0
    bytes_tok = weights + kv_per_pos * avg_ctx + cfg.hidden * 4
    peaks = load_peaks()
    hbm = peaks["hbm_gbs"] * (world if group else 1)  # a sharded model streams from every rank's HBM
    tps = n_gen / dt
    split_routes = None
    if group and rank == 0 and cfg.n_exp:
        # the experts the split model's routers chose at every position, with their gaps
        split_routes = [sess.route_trace(p) for p in range(n_prompt + n_gen)]
    sess.close()
    agree = None
    if group:
        # the same model and prompt unsharded on rank 0's GPU: token agreement of the split run,
        # and at a first divergence the unsharded top-1 / top-2 gap (a tie or not)
        full_toks = np.concatenate([first[-1:], toks])
        agree = group_agreement(cfg, which, prompt, full_toks, device, split_routes) if rank == 0 else None
        agree = group[2](json.dumps(agree).encode())[0]
        agree = json.loads(agree)
    desc = {"dense": "configs[2]: Qwen2.5-3B-style dense, 36 layers, hidden 2048, 16 q / 2 kv heads x 128, SwiGLU "
                     "11008, vocab 151936, Q4_K + Q6_K (ffn_down, output), fp16 KV ctx 4096",
            "moe": "configs[3]: Qwen3-30B-A3B-style MoE, 48 layers, hidden 2048, 32 q / 4 kv heads x 128, QK-norm, "
                   "128 experts x SwiGLU 768, softmax top-8, vocab 151936, all Q4_K, fp16 KV ctx 2048",
            "mla": "configs[4]: DeepSeek-V2-Lite-style MLA + MoE, 27 layers, hidden 2048, 16 heads, kv_lora 512, "
                   "qk_nope 128 + qk_rope 64, v_head 128, q-LoRA 512 (synthesized), layer 0 dense FFN 10944, then "
                   "64 experts top-6 x 1408 + shared 2816, vocab 102400, Q4_K (down projections Q8_0), latent "
                   "f16 cache ctx 2048"}[which]
    out = {"tok_per_s": round(tps, 1), "config": desc,
            "data": "synthetic random-init weights (seeded), random prompt",
            "prompt_tokens": n_prompt, "generated_tokens": n_gen,
            "ms_per_token": round(1e3 * dt / n_gen, 3), "bytes_per_token": int(bytes_tok),
            "roofline": {"bound": "hbm", "achieved_GBps": round(bytes_tok * tps / 1e9, 1),
                         "peak_GBps": hbm, "frac": round(bytes_tok * tps / 1e9 / hbm, 4),
                         "roofline_tok_per_s": round(hbm * 1e9 / bytes_tok, 1)},
            "timing": "wall clock around sb_decode_greedy(256 steps); graph launches chained on one stream"
                      + ("; max over ranks" if group else ""),
            "parallelism": parallelism(cfg, world) if group else "1 GPU",
            "last_tokens": toks[-4:].tolist()}
    if pf:
        out["prefill"] = pf
    if agree is not None:
        out["agreement_vs_1gpu"] = agree
    return out


def prefill_flops(cfg, n: int) -> float:
    """Useful FLOPs of a block prefill of n tokens from position 0: 2 x rows x cols per token
    of every matrix a token goes through (its routed experts only), the MLA re-expansion of
    the n latent rows, and the causal attention (heads x (dqk + dv) x 2 per (query, key))."""
    H, fl = cfg.hidden, 0.0
    for l in range(cfg.n_layers):
        if cfg.mla:
            qk = cfg.qk_nope + cfg.qk_rope
            fl += 2 * n * (cfg.q_rank * H + cfg.kv_rank * H + cfg.heads * qk * cfg.q_rank + H * cfg.q_dim)
            fl += 2 * n * (cfg.kv_heads * qk + cfg.kv_heads * cfg.v_dim) * cfg.kv_rank
            fl += cfg.heads * (qk + cfg.v_dim) * n * (n + 1)
        else:
            fl += 2 * n * (cfg.q_dim + 2 * cfg.kv_dim) * H + 2 * n * H * cfg.q_dim
            fl += cfg.heads * 2 * cfg.head_dim * n * (n + 1)
        if cfg.is_moe(l):
            fl += 2 * n * cfg.n_exp * H + 2 * n * cfg.top_k * 3 * cfg.moe_ffn * H + 2 * n * 3 * cfg.shared_ffn * H
        else:
            fl += 2 * n * 3 * cfg.ffn * H
    return fl + 2 * cfg.vocab * H


def load_bf16_peak() -> float:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f).get("bf16_tflops", 1590.0))
    return 1590.0


def group_agreement(cfg, which: str, prompt, split_toks, device: int, split_routes=None) -> dict:
    """The greedy chain of the split model against the same model on one GPU (rank 0's): the
    share of identical generated tokens, the first step where they differ and, there, the
    one-GPU top-1 / top-2 logit gap over the rms of the logits (a gap near the two runs'
    rounding difference is a tie, which either run may break).  For a MoE model also the first
    position where the two runs' routers chose different experts, with both runs' router-logit
    gaps between the k-th choice and the next expert there: a router near-tie broken the other
    way changes that token's hidden state and, through the KV rows, every later step."""
    from soso_b200 import decode
    model = decode.synth_model(cfg, f"{which}.0")  # every expert (the split run's rank 0 held its own)
    s = decode.DecodeSession(cfg, model, device=device)
    try:
        P = len(prompt)
        one = s.greedy(prompt, P + len(split_toks) - 1)[P - 1:]
        n = len(split_toks)
        same = one[:n] == split_toks
        first = None if same.all() else int(np.argmax(~same))
        route = None
        if split_routes is not None:
            # positions run on the same tokens by both: the prompt, then the common prefix
            last = P - 1 + (n - 1 if first is None else first)
            for pos in range(min(last + 1, len(split_routes))):
                ids1, gaps1 = s.route_trace(pos)
                ids2, gaps2 = split_routes[pos]
                diff = [l for l in ids1 if set(ids1[l].tolist()) != set(ids2[l].tolist())]
                if diff:
                    l = diff[0]
                    route = {"position": pos, "layer": l, "layers_differing": len(diff),
                             "router_gap_1gpu": round(gaps1[l], 6), "router_gap_split": round(gaps2[l], 6),
                             "first_token_divergence_position": None if first is None else P - 1 + first}
                    break
        gap = None
        if first is not None:
            # teacher forced on the common prefix: the logits of the step where the runs part
            orc_embed = decode_embed_rows(cfg, model)
            fed = np.concatenate([prompt, split_toks[:first]])
            for i, t in enumerate(fed):
                lg = s.token(orc_embed(int(t)), i)
            top = np.sort(lg.astype(np.float64))[-2:]
            gap = float((top[1] - top[0]) / np.sqrt(np.mean(lg.astype(np.float64) ** 2)))
        out = {"tokens": n, "identical_frac": round(float(same.mean()), 4), "first_divergence": first,
               "gap_at_divergence": gap}
        if split_routes is not None:
            out["first_route_difference"] = route
        return out
    finally:
        s.close()


def decode_embed_rows(cfg, model):
    """The embedding row of a token (Runtime::embed_token), dequantised by the library's
    embedding kernel (sbk_embed_row) on the current GPU."""
    import torch

    from soso_b200._lib import lib
    table = torch.from_numpy(model["token_embd"]).cuda()
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(cfg.hidden, dtype=torch.float32, device="cuda")

    def row(t: int) -> np.ndarray:
        tok.fill_(t)
        if lib().sbk_embed_row(table.data_ptr(), cfg.dtypes["token_embd"], cfg.vocab, cfg.hidden, tok.data_ptr(),
                               out.data_ptr(), 0, torch.cuda.current_stream().cuda_stream):
            raise RuntimeError("sbk_embed_row rejected")
        torch.cuda.synchronize()
        return out.cpu().numpy()
    return row


def q80_bench(dev) -> dict:
    """the Q8_0 4096x4096 matvec (.som blocks, f32 scale), batch 1, on
    the tensor-core kernel; a CUDA graph of launches over 32 distinct copies (604 MB > L2)."""
    import torch

    from soso_b200 import synth
    from soso_b200._lib import lib
    L = lib()
    rows, cols, copies, reps = 4096, 4096, 32, 5
    ws_ = [torch.from_numpy(synth.random_weights(2, rows, cols, synth.rng("c1", k))).to(dev) for k in range(copies)]
    x = torch.randn(cols, device=dev)
    y = torch.empty(rows, device=dev)
    s = torch.cuda.Stream(dev)

    def enq(st):
        for k in range(copies):
            if L.sbk_matvec(2, ws_[k].data_ptr(), rows, cols, x.data_ptr(), y.data_ptr(), 1, st):
                raise RuntimeError("sbk_matvec(Q8_0) rejected")
    with torch.cuda.stream(s):
        enq(s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        enq(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    nbytes = rows * cols // 32 * 36 + cols * 4 + rows * 4
    peaks = load_peaks()
    return {"config": "configs[0]: Q8_0 4096x4096 (.som 36-byte blocks), x f32, batch 1",
            "kernel": "sb::tcmv::tc_mmv_kernel<Q80> (one launch per matvec, PDL chain)",
            "us_per_matvec": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
            "frac_of_hbm": round(nbytes / us / 1e3 / peaks["hbm_gbs"], 4),
            "l2": f"{copies} distinct copies ({copies * rows * cols // 32 * 36 // 2**20} MiB) rotated"}


def prefill_bench(dev) -> dict:
    """The tcgen05 prefill GEMM (sbk_matmul, bf16 operands) on the
    Q4_K matrices of one configs[4] 512-token prefill layer: q_down, kv_down (512 x 2048),
    q_up (3072 x 512), the dense FFN gate/up (10944 x 2048) and an expert gate/up
    (1408 x 2048); each timed alone in a CUDA graph over 4 distinct copies."""
    import torch

    from soso_b200 import synth
    from soso_b200._lib import lib
    L = lib()
    peaks_tf = 1633.9
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peaks_tf = float(json.load(f).get("bf16_tflops", peaks_tf))
    n = 512
    out = {}
    tot_fl, tot_us = 0.0, 0.0
    for name, rows, cols in (("q_down|kv_down", 512, 2048), ("q_up", 3072, 512), ("ffn_gate|up", 10944, 2048),
                             ("expert_gate|up", 1408, 2048)):
        copies = 4
        ws_ = [torch.from_numpy(synth.random_weights(3, rows, cols, synth.rng("pf", name, k))).to(dev)
               for k in range(copies)]
        x = torch.randn(n, cols, device=dev)
        y = torch.empty(n, rows, device=dev)
        wsb = torch.empty(int(L.sbk_matmul_ws_bytes(n, cols)), dtype=torch.uint8, device=dev)
        s = torch.cuda.Stream(dev)

        def enq(st):
            for k in range(copies):
                if L.sbk_matmul(3, ws_[k].data_ptr(), rows, cols, n, x.data_ptr(), y.data_ptr(), wsb.data_ptr(), 0, 1,
                                st):
                    raise RuntimeError("sbk_matmul rejected")
        with torch.cuda.stream(s):
            enq(s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            enq(torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (10 * copies)
        fl = 2.0 * n * rows * cols
        tot_fl += fl
        tot_us += us
        out[f"{name} {rows}x{cols}"] = {"us": round(us, 1), "TFLOPs": round(fl / us / 1e6, 1)}
    return {"config": "configs[4] prefill, 512 tokens: Q4_K GEMMs of one layer, bf16 operands, f32 accumulation "
                      "in tensor memory (conversion of x to bf16 included)",
            "kernel": "sb::pf::pf_gemm_q4k_kernel (tcgen05.mma kind::f16, M=128 N=256)",
            "shapes": out, "TFLOPs": round(tot_fl / tot_us / 1e6, 1),
            "frac_of_bf16_peak": round(tot_fl / tot_us / 1e6 / peaks_tf, 4),
            "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops, burst)"}


# ---------------------------------------------------------- reference arm
def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import oracle
    from soso_b200 import synth
    threads = host_threads()
    mats = []
    for rows, cols in SHAPES:
        g = synth.rng("bench", "ref", rows, cols)
        mats.append((synth.random_weights(Q4K, rows, cols, g), rows, cols, synth.randn(cols, g),
                     np.empty(rows, np.float32)))
    step_bytes = sum(algo_bytes(r, c) for _, r, c, _, _ in mats)

    def step():
        for w, rows, cols, x, y in mats:
            oracle.cpu_matvec(Q4K, w, rows, cols, x, threads, y)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = step_bytes * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "Q4_K decode matvec sweep, batch 1: one 11008x4096 + one 4096x4096 per step "
                               "(bounded sample of BASELINE configs[1])",
                   "parallelism": f"{threads} host threads (row_strip)"},
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "reference AVX2 Q4_K matvec (gemm.rs:842-894) restated in C, "
                                   "row_strip-threaded (parallel.rs:22-31); one matvec per BASELINE shape per step"},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


NCU_CASES = {  # name -> (dtype, rows, cols, copies): small cases for ncu captures
    "q4k": (Q4K, 11008, 4096, 8),
    "q4k_4096": (Q4K, 4096, 4096, 16),
    "q6k": (13, 4096, 11008, 6),
    "q6k_lmhead": (13, 151936, 2048, 1),
    "q80": (2, 4096, 4096, 8),
}


def run_batch_case(launches: int) -> None:
    """The bench step's launch (one sbk_matvec_batch over the rank-0 rotation set), repeated
    `launches` times without a graph (for ncu); checks two outputs against the oracle."""
    import torch

    import oracle
    from soso_b200._lib import SbkMvOp, lib
    L = lib()
    dev = torch.device("cuda", 0)
    mats = bench_mats(0)
    wd = [torch.from_numpy(m[2]).to(dev) for m in mats]
    xd = [torch.from_numpy(m[3]).to(dev) for m in mats]
    yd = [torch.empty(m[0], device=dev, dtype=torch.float32) for m in mats]
    batch = (SbkMvOp * len(mats))()
    for i, ((rows, cols, _, _), w, x, y) in enumerate(zip(mats, wd, xd, yd)):
        batch[i] = SbkMvOp(w.data_ptr(), rows, cols, x.data_ptr(), y.data_ptr())
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(launches):
        rc = L.sbk_matvec_batch(Q4K, batch, len(mats), 0, s)
        if rc:
            raise SystemExit(f"sbk_matvec_batch rc={rc}")
    torch.cuda.synchronize()
    worst = 0.0
    for i in (0, len(mats) - 1):
        rows, cols, w, x = mats[i]
        t = oracle.matvec_f64(Q4K, w, rows, cols, x)
        y = yd[i].cpu().numpy()
        rms = float(np.sqrt(np.mean(t ** 2)))
        worst = max(worst, float(np.max(np.abs(y - t) / np.maximum(np.abs(t), 1e-3 * rms))))
    print(json.dumps({"case": "q4k_batch", "launches": launches, "matrices": len(mats),
                      "bytes_per_launch": sum(algo_bytes(m[0], m[1]) for m in mats), "max_rel_err": worst}))
    if worst > 1e-3:
        raise SystemExit(1)


def run_prefill_case(launches: int) -> None:
    """The tcgen05 prefill GEMM on configs[4]'s dense FFN gate shape (10944 x 2048, 512 tokens,
    bf16 operands), `launches` times without a graph (for ncu); checks one output row."""
    import torch

    import oracle
    from soso_b200 import synth
    from soso_b200._lib import lib
    L = lib()
    rows, cols, n = 10944, 2048, 512
    g = synth.rng("ncu", "prefill")
    w = synth.random_weights(Q4K, rows, cols, g)
    x = g.standard_normal((n, cols)).astype(np.float32)
    wd, xd = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    y = torch.empty(n, rows, device="cuda")
    ws = torch.empty(int(L.sbk_matmul_ws_bytes(n, cols)), dtype=torch.uint8, device="cuda")
    for _ in range(launches):
        if L.sbk_matmul(Q4K, wd.data_ptr(), rows, cols, n, xd.data_ptr(), y.data_ptr(), ws.data_ptr(), 0, 0,
                        torch.cuda.current_stream().cuda_stream):
            raise SystemExit("sbk_matmul rejected")
    torch.cuda.synchronize()
    t = oracle.matvec_f64(Q4K, w, rows, cols, x[7])
    err = float(np.max(np.abs(y[7].cpu().numpy() - t)) / np.sqrt(np.mean(t ** 2)))
    print(json.dumps({"case": "prefill", "launches": launches, "max_err_over_rms": err}))
    if err > 3e-2:
        raise SystemExit(1)


def run_decode_case(tokens: int) -> None:
    """A 4-layer slice of configs[2] (the dense decoder) through the whole-token engine:
    `tokens` greedy steps (eager warm-up, then graph replays) -- for an ncu launch list."""
    from soso_b200 import decode
    cfg = decode.DenseConfig(n_layers=4, hidden=2048, heads=16, kv_heads=2, head_dim=128, ffn=11008, vocab=151936,
                             ctx=4096)
    sess = decode.DecodeSession(cfg, decode.synth_model(cfg, "ncu"))
    toks = sess.greedy(np.arange(8, dtype=np.int32), tokens)
    sess.close()
    print(json.dumps({"case": "decode", "tokens": toks.tolist()}))


def run_decode_moe_case(tokens: int) -> None:
    """A 4-layer slice of configs[3] (the MoE decoder: 128 experts, top-8) through the
    whole-token engine: `tokens` greedy steps after an 8-token prompt -- for an ncu launch list."""
    import dataclasses

    from soso_b200 import decode
    cfg = dataclasses.replace(decode.QWEN3_30B_A3B, n_layers=4)
    sess = decode.DecodeSession(cfg, decode.synth_model(cfg, "ncu"))
    toks = sess.greedy(np.arange(8, dtype=np.int32), tokens)
    sess.close()
    print(json.dumps({"case": "decode_moe", "tokens": toks[-4:].tolist()}))


def run_prefill_engine_case(launches: int) -> None:
    """A 3-layer slice of configs[4] (MLA attention; the dense FFN layer, then two MoE layers)
    through the block prefill: `launches` prefills of a 512-token prompt -- for ncu captures
    of the table-driven GEMM (the grouped expert launches among them)."""
    import dataclasses

    from soso_b200 import decode, synth
    cfg = dataclasses.replace(decode.DEEPSEEK_V2_LITE, n_layers=3)
    sess = decode.DecodeSession(cfg, decode.synth_model(cfg, "ncu"))
    prompt = synth.rng("ncu", "pf").integers(0, cfg.vocab, 512).astype(np.int32)
    nxt = None
    for _ in range(launches):
        _, nxt = sess.prefill(prompt, logits=False)
    sess.close()
    print(json.dumps({"case": "prefill_engine", "prefills": launches, "next": nxt}))


def run_decode_mla_case(tokens: int) -> None:
    """A 3-layer slice of configs[4] (MLA attention; a dense FFN, then two MoE layers) through
    the whole-token engine: `tokens` greedy steps after a 64-token prompt -- for ncu captures
    of the MLA kernels."""
    import dataclasses

    from soso_b200 import decode
    cfg = dataclasses.replace(decode.DEEPSEEK_V2_LITE, n_layers=3)
    sess = decode.DecodeSession(cfg, decode.synth_model(cfg, "ncu"))
    toks = sess.greedy(np.arange(64, dtype=np.int32), 64 + tokens)
    sess.close()
    print(json.dumps({"case": "decode_mla", "tokens": toks[-4:].tolist()}))


def run_case(name: str, launches: int) -> None:
    """Plain launches of one kernel over a rotation of copies (for ncu); prints a check line."""
    import torch

    import oracle
    from soso_b200 import synth
    from soso_b200._lib import lib
    dt, rows, cols, copies = NCU_CASES[name]
    L = lib()
    dev = torch.device("cuda", 0)
    ws, xs = [], []
    for k in range(copies):
        g = synth.rng("case", name, k)
        ws.append(synth.random_weights(dt, rows, cols, g))
        xs.append(synth.randn(cols, g))
    wd = [torch.from_numpy(w).to(dev) for w in ws]
    xd = [torch.from_numpy(x).to(dev) for x in xs]
    yd = torch.empty(rows, device=dev, dtype=torch.float32)
    s = torch.cuda.current_stream().cuda_stream
    for i in range(launches):
        k = i % copies
        rc = L.sbk_matvec(dt, wd[k].data_ptr(), rows, cols, xd[k].data_ptr(), yd.data_ptr(), 0, s)
        if rc:
            raise SystemExit(f"sbk_matvec rc={rc}")
    torch.cuda.synchronize()
    k = (launches - 1) % copies
    t = oracle.matvec_f64(dt, ws[k], rows, cols, xs[k])
    y = yd.cpu().numpy()
    rms = float(np.sqrt(np.mean(t ** 2)))
    err = float(np.max(np.abs(y - t) / np.maximum(np.abs(t), 1e-3 * rms)))
    print(json.dumps({"case": name, "launches": launches, "max_rel_err": err}))
    if err > 1e-3:
        raise SystemExit(1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ncu-case", choices=sorted(NCU_CASES) + ["q4k_batch", "prefill", "decode", "decode_mla",
                                                               "decode_moe", "prefill_engine"], default=None)
    ap.add_argument("--launches", type=int, default=12)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    args = ap.parse_args()
    if args.ncu_case == "q4k_batch":
        run_batch_case(args.launches)
        return
    if args.ncu_case == "prefill":
        run_prefill_case(args.launches)
        return
    if args.ncu_case == "decode_mla":
        run_decode_mla_case(args.launches)
        return
    if args.ncu_case == "decode_moe":
        run_decode_moe_case(args.launches)
        return
    if args.ncu_case == "prefill_engine":
        run_prefill_engine_case(args.launches)
        return
    if args.ncu_case == "decode":
        run_decode_case(args.launches)
        return
    if args.ncu_case:
        run_case(args.ncu_case, args.launches)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

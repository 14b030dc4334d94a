"""Verified tokens/s of the Qwen3.5-27B-shape 4-bit decode / K-token verify step.

Workload: the full 64-layer stack (48 GatedDeltaNet + 16 attention layers,
MLX affine 4-bit weights, bf16 embedding, 4-bit lm_head), random-init
synthetic weights generated on the GPU, seeded recurrent state and a KV cache
of 1024 prior tokens; each step verifies K = 32 draft tokens (the headline)
and, reported alongside, K = 1 (plain decode).  One step = one pass of the
whole stack over the K tokens + lm_head argmax + accept length at positions
1024..1024+K-1: every step re-verifies its block at context 1024 (the
recurrent state carries on from step to step).

  python bench.py [--gpus N] [--steps S] [--warmup W] [--k 32] [--impl reference]
  python bench.py --batch 64 --k 8 [--ctx 4096]   # multi-sequence verify (one line, token-rows/s)

With N > 1 (one process per GPU under torch.distributed.run) the step runs
tensor-parallel over N GPUs (NCCL all-reduce of the row-parallel outputs), so
the total work is fixed and scaling is strong.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "inference-across-metal_b200"))

SEED = 20261201
CTX = 1024
METRIC = "verified tokens/sec, Qwen3.5-27B-shape 4-bit at K=1/32, and % of HBM roofline"
# dram__bytes_read.sum + dram__bytes_write.sum of one qmm_tc_kernel launch
# (34816 x 5120 weights, 32 tokens) over its weight bytes (104.09 MB / 100.27 MB)
TRAFFIC_PER_WEIGHT_BYTE = 104.090624 / 100.270080
WORKLOAD = "qwen3.5-27b-shape 64-layer (48 GDN + 16 attn) 4-bit verify, ctx 1024, batch 1"


def bench_config(K: int, world: int) -> dict:
    """The workload, shared by both arms' lines."""
    return {"workload": WORKLOAD, "K": K, "ctx": CTX, "batch": 1, "parallelism": f"tp{world}",
            "l2": "inputs larger than L2 (14.4 GB of weights streamed per step)"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """One ``nvidia-smi --query-gpu=... -lms 50`` process, started before the
    warm-up (so no process start falls inside the timed region) and stopped
    after it; the samples whose timestamps lie in the timed window [begin(),
    end()] are summarised."""
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)  # the first sample is out before any timing starts

    def begin(self):
        import datetime
        self.t0 = datetime.datetime.now()

    def end(self):
        import datetime
        self.t1 = datetime.datetime.now()

    def stop(self):
        import datetime
        rows = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except Exception:
                self.proc.kill()
                out = ""
            for line in out.splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 10:
                    continue
                try:
                    ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f")
                except ValueError:
                    continue
                rows.append((ts, f[1:]))
        inside = [r for ts, r in rows if self.t0 and self.t1 and self.t0 <= ts <= self.t1]
        if not inside and rows and self.t0:
            # a window shorter than the sampling period: the samples either side of it
            before = [r for ts, r in rows if ts <= self.t0][-1:]
            after = [r for ts, r in rows if self.t1 and ts >= self.t1][:1]
            inside = before + after
        sm = [float(r[1]) for r in inside if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in inside if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i in range(4) if len(r) > 5 + i and r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(inside), "sampling": "nvidia-smi -lms 50, timed window"}


# ---------------------------------------------------------------- CPU legs (oracle)
def oracle_sample(K: int, threads: int):
    """Time the CPU restatement (numpy fp32 with the multi-threaded C dequant
    helper, dequantisation included) on a bounded sample of the step at full
    size: one GDN layer, one attention layer and 1/16 of the lm_head.  Returns
    (tokens/s of the 64-layer step extrapolated x48/x16/x16, seconds the sample
    took, description)."""
    import numpy as np
    from oracle import fast as F
    from oracle import iam_oracle as O
    from oracle import synth_model as SM
    d = O.QWEN35_27B
    W = F.make_layer(SEED, d, 0)
    W.update(F.make_layer(SEED, d, 3))
    st = SM.make_state(SEED, d, CTX, CTX + K, layers=[0, 3])
    lm_rows = d.vocab // 16
    lm = F.gen_qweight(SEED, "lm_head", lm_rows, d.hidden)
    x = SM.hidden_input(SEED, d, K)
    with F.fast_dequant():
        t0 = time.perf_counter()
        O.gdn_block(x, W, "model.layers.0.", st.conv[0], st.S[0], d)
        t1 = time.perf_counter()
        O.attn_block(x, W, "model.layers.3.", st.k_cache[3], st.v_cache[3], CTX, d)
        t2 = time.perf_counter()
        O.argmax_first(O.qmm_affine4(O.rms_norm(x, np.ones(d.hidden, np.float32)), *lm))
        t3 = time.perf_counter()
    step = 48 * (t1 - t0) + 16 * (t2 - t1) + 16 * (t3 - t2)
    desc = (f"numpy fp32 oracle + C dequant, {threads} threads: 1 GDN layer {t1 - t0:.2f}s + 1 attention layer "
            f"{t2 - t1:.2f}s + 1/16 lm_head {t3 - t2:.2f}s at K={K}, ctx {CTX}, extrapolated x48/x16/x16 to "
            f"the 64-layer step")
    return K / step, t3 - t0, desc


def cpu_layers(threads: int, reps: int = 3) -> dict:
    """The single-layer workloads at K = 1 on the CPU restatement (numpy fp32
    with the multi-threaded C dequant, dequantisation included), median of
    `reps`: one GDN layer at full size (its mixer alone is the layer minus the
    MLP, timed on its own) and one attention + SwiGLU MLP layer at position
    CTX - 1 over CTX - 1 prior KV rows."""
    import numpy as np
    from oracle import fast as F
    from oracle import iam_oracle as O
    from oracle import synth_model as SM
    d = O.QWEN35_27B
    W = F.make_layer(SEED, d, 0)
    W.update(F.make_layer(SEED, d, 3))
    st = SM.make_state(SEED, d, CTX - 1, CTX, layers=[0, 3])
    x = SM.hidden_input(SEED, d, 1)
    g, a, m = [], [], []
    with F.fast_dequant():
        for _ in range(reps):
            conv, S = st.conv[0].copy(), st.S[0].copy()
            t0 = time.perf_counter()
            O.gdn_block(x, W, "model.layers.0.", conv, S, d)
            t1 = time.perf_counter()
            O.attn_block(x, W, "model.layers.3.", st.k_cache[3], st.v_cache[3], CTX - 1, d)
            t2 = time.perf_counter()
            O.mlp(O.rms_norm(x, W["model.layers.3.post_attention_layernorm.weight"], d.eps), W, "model.layers.3.")
            t3 = time.perf_counter()
            g.append(t1 - t0)
            a.append(t2 - t1)
            m.append(t3 - t2)
    med = statistics.median
    return {"gdn_layer_ms": 1e3 * med(g), "gdn_mixer_ms": 1e3 * (med(g) - med(m)), "attn_mlp_layer_ms": 1e3 * med(a),
            "threads": threads, "reps": reps,
            "kind": "port: numpy fp32 oracle + C dequant (OpenMP), dequantisation included"}


def gpu_layers(eng, K: int, pos: int) -> dict:
    """Median device time of the GDN and attention layers of one eager step
    (CUDA events around every launch; no overlap between launches)."""
    lay = eng.profile_layers(K, pos)
    med = statistics.median
    gdn = [x for x in lay if not x[0]]
    att = [x for x in lay if x[0]]
    return {"gdn_mixer_us": 1e3 * med([x[1] for x in gdn]), "gdn_layer_us": 1e3 * med([x[1] + x[2] for x in gdn]),
            "attn_mlp_layer_us": 1e3 * med([x[1] + x[2] for x in att]), "mlp_us": 1e3 * med([x[2] for x in lay]),
            "layers": [len(gdn), len(att)], "timing": "eager step, CUDA events around every launch, median over layers"}


def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of the path (the reference's own
    implementation is Swift + Metal + a binary MLX kernel and cannot run here).
    Each step is one bounded sample (oracle_sample); the line reports the
    sample's measured time per step and the 64-layer step time extrapolated
    from it, marked as extrapolated."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals, secs = [], []
    desc = ""
    for i in range(args.warmup + args.steps):
        v, sec, desc = oracle_sample(args.k, threads)
        if i >= args.warmup:
            vals.append(v)
            secs.append(sec)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * args.k / value,
        "extrapolated": True,
        "sample_ms_per_step": 1000.0 * statistics.median(secs),
        "sample_pieces": ["1 GDN layer x48", "1 attention layer x16", "1/16 of the lm_head x16"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(args.k, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU
def run_gpu(args, rank, world, local_rank):
    import numpy as np
    import torch
    import iam_b200 as I

    dist = None
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    K = args.k
    ksteps = args.warmup + args.steps
    max_ctx = CTX + (ksteps + 2) * max(K, 1) * 2 + 64
    dims = I.Dims.qwen35_27b(max_ctx=max_ctx, max_rows=max(32, K))
    if args.resident_gb:
        dims.resident_weight_bytes = int(args.resident_gb * 1e9)
    dims.comm_timeout_ms = 60000  # a peer that stops answering ends the run in a minute
    nccl_id = None
    if world > 1:
        obj = [I.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    eng = I.Engine(dims, device=local_rank, rank=rank, world=world, nccl_id=nccl_id)
    eng.init_synthetic(SEED)
    rng = np.random.default_rng(SEED)
    stream = torch.cuda.Stream()  # a real stream handle: the graphs and the events share it
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def device_run(kk: int):
        clk = ClockSampler(local_rank)
        clk.start()
        eng.state_init(SEED, CTX)
        toks = torch.from_numpy(rng.integers(0, dims.vocab, kk).astype(np.int32)).cuda()
        out = torch.zeros(kk, dtype=torch.int32, device="cuda")
        # every step verifies the block at positions CTX..CTX+kk-1 (the KV rows
        # of the block are rewritten each step), so each runs at context CTX
        for _ in range(args.warmup):
            eng.verify_device(toks.data_ptr(), kk, CTX, out.data_ptr(), sh)
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clk.begin()
        a.record(stream)
        for _ in range(args.steps):
            eng.verify_device(toks.data_ptr(), kk, CTX, out.data_ptr(), sh)
        b.record(stream)
        torch.cuda.synchronize()
        clk.end()
        ms = a.elapsed_time(b) / args.steps
        clocks = clk.stop()
        if dist is not None:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        barrier()
        return ms, clocks

    # Settle clocks before any timing: back-to-back steps for about a second
    # (the memory clock of an idle GPU ramps up under load).
    eng.state_init(SEED, CTX)
    _t = torch.zeros(K, dtype=torch.int32, device="cuda")
    t_end = time.perf_counter() + 1.0
    n_pre = 0
    while time.perf_counter() < t_end or n_pre < 10:
        for _ in range(10):
            eng.verify_device(_t.data_ptr(), K, CTX, None, sh)
        torch.cuda.synchronize()
        n_pre += 10
    ms32, clocks = device_run(K)
    ms1, _ = device_run(1) if K != 1 else (ms32, None)

    # end to end through the public C API: host tokens in, host argmax out
    eng.state_init(SEED, CTX)
    htoks = rng.integers(0, dims.vocab, K).astype(np.int32)
    for _ in range(args.warmup):
        eng.verify(htoks, CTX)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.verify(htoks, CTX)
    e2e_s = (time.perf_counter() - t0) / args.steps
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    # per-kernel-kind device time of one eager step (CUDA events on the engine stream)
    eng.state_init(SEED, CTX)
    lay1 = gpu_layers(eng, 1, CTX - 1)
    eng.state_init(SEED, CTX)
    layK = gpu_layers(eng, K, CTX)
    eng.state_init(SEED, CTX)
    prof1 = eng.profile_step(1, CTX)
    eng.state_init(SEED, CTX)
    prof = eng.profile_step(K, CTX)
    launches = eng.step_launches(K)
    step_bytes = eng.step_bytes(K, CTX)
    n_streamed = eng.streamed_layers()
    hbm, peak_kind = peaks()
    q = prof.get("qmm", {"ms": 0.0, "bytes": 0.0, "launches": 1})
    q_gbs = q["bytes"] / (q["ms"] / 1000.0) / 1e9 if q["ms"] > 0 else 0.0
    eng.close()

    if rank != 0:
        return
    step_gbs = step_bytes / (ms32 / 1000.0) / 1e9
    line = {
        "metric": METRIC,
        "value": K * 1000.0 / ms32,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms32,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": dict(bench_config(K, world), **({"resident_weight_gb": args.resident_gb,
                                                    "streamed_layers": n_streamed} if args.resident_gb else {})),
        "k1": {"value": 1000.0 / ms1, "unit": "tokens/s", "ms_per_step": ms1},
        "hbm_roofline_step": {"bytes_per_step_per_gpu": step_bytes, "achieved_gbs": step_gbs, "peak_gbs": hbm,
                              "frac": step_gbs / hbm, "peak_kind": peak_kind},
        "roofline": {"bound": "hbm", "kernel": "qmm_tc_kernel", "achieved": q_gbs, "peak": hbm, "unit": "GB/s",
                     "frac": q_gbs / hbm,
                     "traffic": TRAFFIC_PER_WEIGHT_BYTE * q["bytes"] / max(q["launches"], 1),
                     "traffic_note": "DRAM read+write per average launch: the weight bytes times the "
                                     "traffic / weight-bytes ratio of one ncu capture (34816 x 5120, 32 tokens)",
                     "peak_kind": peak_kind, "launches_per_step": q["launches"], "ms_per_step": q["ms"],
                     "timing": "eager step, CUDA events on the engine stream around each launch"},
        "layers": {
            "gdn_layer_decode_k1": {"workload": "one GatedDeltaNet layer, K=1, 27B dims (the mixer: norm, fused "
                                                "projections, conv + delta rule + gated norm, out_proj + residual)",
                                    "gpu_us": lay1["gdn_mixer_us"], "gpu_us_with_mlp": lay1["gdn_layer_us"]},
            "attn_mlp_layer_decode_k1": {"workload": "one full-attention layer + SwiGLU MLP, K=1, position 1023",
                                         "gpu_us": lay1["attn_mlp_layer_us"]},
            f"gdn_layer_verify_k{K}": {"gpu_us": layK["gdn_mixer_us"], "gpu_us_with_mlp": layK["gdn_layer_us"]},
            f"attn_mlp_layer_verify_k{K}": {"gpu_us": layK["attn_mlp_layer_us"]},
            "timing": lay1["timing"],
        },
        "kernels_ms": {k: round(v["ms"], 4) for k, v in prof.items()},
        "kernels_ms_k1": {k: round(v["ms"], 4) for k, v in prof1.items()},
        "e2e": {"value": K / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 4 * (K + 1),
                "d2h_bytes_per_step": 4 * (K + 1)},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
        "prewarm_steps": n_pre,
    }
    if world == 1 and not args.no_cpu:
        cl = cpu_layers(os.cpu_count() or 1)
        line["layers"]["gdn_layer_decode_k1"]["cpu_ms_median3"] = cl["gdn_mixer_ms"]
        line["layers"]["gdn_layer_decode_k1"]["cpu_ms_median3_with_mlp"] = cl["gdn_layer_ms"]
        line["layers"]["attn_mlp_layer_decode_k1"]["cpu_ms_median3"] = cl["attn_mlp_layer_ms"]
        line["layers"]["cpu"] = {"threads": cl["threads"], "reps": cl["reps"], "kind": cl["kind"]}
        v, secs, desc = oracle_sample(K, os.cpu_count() or 1)
        line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": desc}
    print(json.dumps(line), flush=True)


def profile_step(args):
    """One warm-up graph step and one measured step of the 64-layer engine at
    verify width --k (the workload of the ncu launch lists in profiles/)."""
    import numpy as np
    import torch
    import iam_b200 as I
    K = args.k
    d = I.Dims.qwen35_27b(max_ctx=CTX + 4 * K + 64, max_rows=max(K, 32))
    e = I.Engine(d)
    e.init_synthetic(SEED)
    e.state_init(SEED, CTX)
    toks = torch.from_numpy(np.random.default_rng(0).integers(0, d.vocab, K).astype(np.int32)).cuda()
    out = torch.zeros(K, dtype=torch.int32, device="cuda")
    st = torch.cuda.Stream()
    for i in range(2):
        e.verify_device(toks.data_ptr(), K, CTX if i == 0 else -1, out.data_ptr(), st.cuda_stream)
    torch.cuda.synchronize()
    print(json.dumps({"profile_step": K, "launches_per_step": e.step_launches(K)}))
    e.close()


MATRIX_OF_GRID_X = {40: "out_proj|o_proj|down", 272: "gate_up", 130: "in_proj", 112: "q|k|v", 1940: "lm_head"}


def kernel_kind(name: str, grid) -> str:
    """The kind a kernel record is summed under (per matrix for the matmuls)."""
    kind = next((k for k in ("qmm_gemv", "qmm_tc", "rms_norm", "gdn_fused", "attn_prep", "attn_decode_tc",
                              "attn_decode", "attn_combine", "finalize", "embed", "advance") if k in name), name[:40])
    if kind.startswith("qmm"):
        kind += " " + MATRIX_OF_GRID_X.get((grid or [0])[0], str(grid))
    return kind


def exposed_by_kind(events):
    """Kernel records (ts, dur in us; name; args.grid), sorted by start, of one
    step: per kind [launches, summed duration, exposed time], and the step's
    span.  A launch's exposed time is how far it extends the span past the
    end of every launch before it, so however the launches overlap the
    exposed times sum to the span less the gaps in which no kernel runs."""
    kinds = {}
    t0 = prev_end = events[0]["ts"]
    for x in events:
        s, dur = x["ts"], x["dur"]
        exposed = max(0.0, s + dur - max(s, prev_end))
        prev_end = max(prev_end, s + dur)
        r = kinds.setdefault(kernel_kind(x["name"], x.get("args", {}).get("grid")), [0, 0.0, 0.0])
        r[0] += 1
        r[1] += dur
        r[2] += exposed
    return kinds, prev_end - t0


def trace_step(args):
    """The kernels of graph steps as they run, with programmatic overlap:
    CUPTI's activity records (through torch.profiler) of three replays of the
    64-layer step at verify width --k, after warm-up.  Per kernel kind (and
    per matrix for the matmuls): launches, mean duration, and the exposed
    time -- how far each launch extends the step past the end of the
    launches before it (the sum is the step less its idle gaps).  One JSON
    line per kind;
    the trace file goes to --trace-out."""
    import numpy as np
    import torch
    from torch.profiler import ProfilerActivity, profile
    import iam_b200 as I
    K = args.k
    d = I.Dims.qwen35_27b(max_ctx=CTX + 256, max_rows=max(K, 32))
    e = I.Engine(d)
    e.init_synthetic(SEED)
    e.state_init(SEED, CTX)
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    toks = torch.from_numpy(np.random.default_rng(0).integers(0, d.vocab, K).astype(np.int32)).cuda()
    for _ in range(20):
        e.verify_device(toks.data_ptr(), K, CTX, None, st.cuda_stream)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(10):
        e.verify_device(toks.data_ptr(), K, CTX, None, st.cuda_stream)
    b.record(st)
    torch.cuda.synchronize()
    untraced = a.elapsed_time(b) / 10
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(3):
            e.verify_device(toks.data_ptr(), K, CTX, None, st.cuda_stream)
        torch.cuda.synchronize()
    prof.export_chrome_trace(args.trace_out)
    e.close()
    with open(args.trace_out) as f:
        ev = [x for x in json.load(f)["traceEvents"] if x.get("cat") == "kernel"]
    ev.sort(key=lambda x: x["ts"])
    n = len(ev) // 3
    kinds, span = exposed_by_kind(ev[n:2 * n])  # the middle replay
    print(json.dumps({"trace_step": K, "launches": n, "span_us": round(span, 1), "untraced_ms": round(untraced, 3)}))
    for kind, (cnt, tot, expo) in sorted(kinds.items(), key=lambda kv: -kv[1][2]):
        print(json.dumps({"kind": kind, "launches": cnt, "mean_us": round(tot / cnt, 2),
                          "exposed_us": round(expo, 1), "exposed_share": round(expo / span, 4)}))


def profile_small(args):
    """Two graph steps of a 4-layer full-width model (3 GDN + 1 attention
    layer, vocab 32768, context 1024: about 2.5 GB on the device) at verify
    width --k: the small case for per-kernel ncu captures of the GDN,
    attention, RMSNorm and matmul kernels at the 27B layer sizes."""
    import numpy as np
    import torch
    import iam_b200 as I
    K = args.k
    d = I.Dims.qwen35_27b(n_layers=4, vocab=32768, max_ctx=CTX + 4 * K + 64, max_rows=max(K, 32))
    e = I.Engine(d)
    e.init_synthetic(SEED)
    e.state_init(SEED, CTX)
    toks = torch.from_numpy(np.random.default_rng(0).integers(0, d.vocab, K).astype(np.int32)).cuda()
    out = torch.zeros(K, dtype=torch.int32, device="cuda")
    st = torch.cuda.Stream()
    for _ in range(2):
        e.verify_device(toks.data_ptr(), K, CTX, out.data_ptr(), st.cuda_stream)
    torch.cuda.synchronize()
    e.status()
    print(json.dumps({"profile_small": K, "launches_per_step": e.step_launches(K)}))
    e.close()


def run_batch(args, rank, world, local_rank):
    """Multi-sequence verify: --batch sequences x --k draft tokens per step,
    each sequence in its own slot (seeded GDN state, conv window, --ctx prior
    KV tokens); value = token-rows verified per second (whole job; tensor
    parallel over N GPUs, strong scaling)."""
    import numpy as np
    import torch
    import iam_b200 as I
    dist = None
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    n, K, ctx = args.batch, args.k, args.ctx
    steps = args.warmup + args.steps
    dims = I.Dims.qwen35_27b(max_ctx=ctx + (2 * steps + 2) * K + 64, max_rows=n * K, max_seqs=n)
    nccl_id = None
    if world > 1:
        obj = [I.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    eng = I.Engine(dims, device=local_rank, rank=rank, world=world, nccl_id=nccl_id)
    eng.init_synthetic(SEED)
    eng.state_init(SEED, ctx)
    rng = np.random.default_rng(SEED)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    htoks = rng.integers(0, dims.vocab, (n, K)).astype(np.int32)
    toks = torch.from_numpy(htoks.reshape(-1)).cuda()
    pos0 = torch.full((n,), ctx, dtype=torch.int32, device="cuda")
    out = torch.zeros(n * K, dtype=torch.int32, device="cuda")
    clk = ClockSampler(local_rank)
    clk.start()
    eng.verify_batch_device(toks.data_ptr(), n, K, pos0.data_ptr(), out.data_ptr(), None, sh)
    for _ in range(args.warmup - 1):
        eng.verify_batch_device(toks.data_ptr(), n, K, None, out.data_ptr(), None, sh)
    barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk.begin()
    a.record(stream)
    for _ in range(args.steps):
        eng.verify_batch_device(toks.data_ptr(), n, K, None, out.data_ptr(), None, sh)
    b.record(stream)
    torch.cuda.synchronize()
    clk.end()
    ms = a.elapsed_time(b) / args.steps
    clocks = clk.stop()
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    barrier()
    # end to end through the public C API: host tokens and positions in, argmax and accept lengths out
    pos = np.full(n, ctx + steps * K, np.int32)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        eng.verify_batch(htoks, pos)
        pos += K
    e2e_s = (time.perf_counter() - t0) / args.steps
    if dist is not None:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    byts = eng.step_bytes_batch(n, K, ctx)
    params = matmul_params(dims)
    eng.close()
    if rank != 0:
        return
    hbm, kind = peaks()
    tc = 1643.5
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            tc = float(json.load(f)["bf16_tflops"])
    rows = n * K
    gbs = byts / (ms / 1000.0) / 1e9
    tfs = 2.0 * params * rows / world / (ms / 1000.0) / 1e12
    line = {
        "metric": f"verified token-rows/sec, {n} sequences x K={K}, ctx {ctx}",
        "value": rows * 1000.0 / ms, "unit": "token-rows/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"qwen3.5-27b-shape 64-layer 4-bit multi-sequence verify, {n} x K={K}, ctx {ctx}",
                   "sequences": n, "K": K, "ctx": ctx, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (14.4 GB of weights, 19 GB of GDN state per step)"},
        "roofline": {"hbm": {"bytes_per_step_per_gpu": byts, "achieved_gbs": gbs, "peak_gbs": hbm,
                             "frac": gbs / hbm, "peak_kind": kind},
                     "tensor": {"achieved_tflops_per_gpu": tfs, "peak_tflops": tc, "frac": tfs / tc}},
        "e2e": {"value": rows / e2e_s, "unit": "token-rows/s", "h2d_bytes_per_step": 4 * (n + rows),
                "d2h_bytes_per_step": 4 * (n + rows)},
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def matmul_params(d) -> float:
    """Weights of every 4-bit matmul of one step (the FLOPs of a token are twice this)."""
    H, kd = d.hidden, d.gdn_k_heads * d.gdn_dk
    gdn = H * (2 * kd + d.gdn_v_heads * d.gdn_dv) + H * d.gdn_v_heads * d.gdn_dv + 2 * H * d.gdn_v_heads \
        + d.gdn_v_heads * d.gdn_dv * H
    attn = H * 2 * d.n_heads * d.head_dim + 2 * H * d.n_kv_heads * d.head_dim + d.n_heads * d.head_dim * H
    mlp = 3 * H * d.intermediate
    n_attn = d.n_layers // d.full_attn_interval
    return float((d.n_layers - n_attn) * gdn + n_attn * attn + d.n_layers * mlp + d.vocab * H)


def sweep(args):
    """Step time of the 64-layer verify against the verify width K (one engine,
    one graph per K, device-resident tokens, context 1024): one JSON line per K
    with the HBM fraction (step bytes / time) and the tensor fraction (2 x
    matmul weights x K / time against the dense bf16 peak)."""
    import numpy as np
    import torch
    import iam_b200 as I
    ks = [int(v) for v in args.sweep.split(",")]
    kmax = max(ks)
    ksteps = args.warmup + args.steps
    d = I.Dims.qwen35_27b(max_ctx=CTX + (ksteps + 2) * kmax + 64, max_rows=max(32, kmax))
    e = I.Engine(d)
    e.init_synthetic(SEED)
    hbm, kind = peaks()
    tc = 1643.5
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        with open(pp) as f:
            tc = float(json.load(f)["bf16_tflops"])
    params = matmul_params(d)
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    rng = np.random.default_rng(SEED)
    for K in ks:
        e.state_init(SEED, CTX)
        toks = torch.from_numpy(rng.integers(0, d.vocab, K).astype(np.int32)).cuda()
        out = torch.zeros(K, dtype=torch.int32, device="cuda")
        e.verify_device(toks.data_ptr(), K, CTX, out.data_ptr(), st.cuda_stream)
        for _ in range(args.warmup - 1):
            e.verify_device(toks.data_ptr(), K, -1, out.data_ptr(), st.cuda_stream)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        for _ in range(args.steps):
            e.verify_device(toks.data_ptr(), K, -1, out.data_ptr(), st.cuda_stream)
        b.record(st)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        byts = e.step_bytes(K, CTX)
        print(json.dumps({"sweep_k": K, "ms_per_step": round(ms, 4), "tokens_per_s": round(K * 1000.0 / ms, 1),
                          "hbm_frac": round(byts / (ms / 1000.0) / 1e9 / hbm, 4),
                          "tensor_frac": round(2.0 * params * K / (ms / 1000.0) / 1e12 / tc, 4),
                          "peaks": {"hbm_gbs": hbm, "bf16_tflops": tc, "kind": kind}}), flush=True)
    e.close()


def profile_qmm(args):
    """A few launches of W4A16 matmul shapes "N,K,M[,mlx];..." (random codes)
    for ncu: through the tensor-core kernel on packed weights, or, with a
    fourth field "mlx", through the mma.sync kernel on the MLX layout (the
    crossover pair)."""
    for spec in args.profile_qmm.split(";"):
        _profile_one_qmm(spec)


def _profile_one_qmm(spec):
    import torch
    import iam_b200 as I
    f = spec.split(",")
    N, K, M = (int(v) for v in f[:3])
    mlx = len(f) > 3 and f[3] == "mlx"
    g = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randint(-2**31, 2**31 - 1, (N, K // 8), dtype=torch.int32, device="cuda", generator=g)
    s = (torch.rand(N, K // 64, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (-8 * s.float()).to(torch.bfloat16)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    if mlx:
        for _ in range(4):
            I.qmm_affine4(w.data_ptr(), s.data_ptr(), b.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K)
    else:
        pk = torch.empty(I.qmm_packed_bytes(N, K), dtype=torch.uint8, device="cuda")
        I.qmm_pack_affine4(w.data_ptr(), s.data_ptr(), b.data_ptr(), pk.data_ptr(), N, K)
        for _ in range(4):
            I.qmm_affine4_packed(pk.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K)
    torch.cuda.synchronize()
    print(json.dumps({"profile_qmm": [N, K, M], "kernel": "mma.sync" if mlx else "tcgen05"}))


def qmm_sweep(args):
    """Warm per-launch time of the W4A16 matmul on packed weights, per shape
    and token count, on the GEMV kernel (the library's choice up to 16
    tokens) and on the tensor-core kernel: one JSON line each.  Enough copies
    of each matrix are cycled that every launch streams its weights from HBM
    (more than the 126 MB L2 between two uses of a copy); CUDA events on the
    launching stream around --steps launches after --warmup."""
    import torch
    import iam_b200 as I
    ms = [int(v) for v in args.qmm_ms.split(",")]
    hbm, kind = peaks()
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    for spec in args.qmm_sweep.split(";"):
        N, K = (int(v) for v in spec.split(","))
        g = torch.Generator(device="cuda").manual_seed(0)
        w = torch.randint(-2**31, 2**31 - 1, (N, K // 8), dtype=torch.int32, device="cuda", generator=g)
        sc = (torch.rand(N, K // 64, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        b = (-8 * sc.float()).to(torch.bfloat16)
        nb = I.qmm_packed_bytes(N, K)
        copies = max(2, -(-300_000_000 // nb))
        pk = [torch.empty(nb, dtype=torch.uint8, device="cuda") for _ in range(copies)]
        for p_ in pk:
            I.qmm_pack_affine4(w.data_ptr(), sc.data_ptr(), b.data_ptr(), p_.data_ptr(), N, K, st.cuda_stream)
        del w
        wbytes = N * K * (0.5 + 4 / 64)
        for M in ms:
            x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
            y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            for kern in ("gemv", "tcgen05"):
                if kern == "gemv" and M > 16:
                    continue
                os.environ["IAM_QMM_GEMV_MAX_M"] = "16" if kern == "gemv" else "0"
                for i in range(args.warmup):  # first calls: kernel attributes, workspace
                    I.qmm_affine4_packed(pk[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K,
                                         st.cuda_stream)
                torch.cuda.synchronize()
                # the timed launches replay as one CUDA graph (device time, as
                # inside the engine's step graph; no host launch gaps)
                g_ = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g_, stream=st):
                    for i in range(args.steps):
                        I.qmm_affine4_packed(pk[i % copies].data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K,
                                             st.cuda_stream)
                g_.replay()
                torch.cuda.synchronize()
                a, bb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(st)
                g_.replay()
                bb.record(st)
                torch.cuda.synchronize()
                del g_
                us = a.elapsed_time(bb) * 1000.0 / args.steps
                print(json.dumps({"qmm_sweep": [N, K, M], "kernel": kern, "us": round(us, 2),
                                  "gbs": round(wbytes / (us * 1e-6) / 1e9, 1),
                                  "hbm_frac": round(wbytes / (us * 1e-6) / 1e9 / hbm, 4), "peak_kind": kind}),
                      flush=True)
        os.environ.pop("IAM_QMM_GEMV_MAX_M", None)
        del pk
        torch.cuda.empty_cache()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--k", type=int, default=32)
    ap.add_argument("--impl", default="iam")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--profile-step", action="store_true", help="two graph steps at --k, for ncu launch lists")
    ap.add_argument("--trace-step", action="store_true", help="in-graph kernel timeline of the step at --k (CUPTI)")
    ap.add_argument("--trace-out", default="gpurun_out/trace_step.json", help="chrome trace file of --trace-step")
    ap.add_argument("--profile-small", action="store_true",
                    help="two graph steps of a 4-layer full-width model at --k, for per-kernel ncu captures")
    ap.add_argument("--profile-qmm", default=None,
                    help="N,K,M[,mlx];...: a few launches of each matmul (tensor-core, or mma.sync on the MLX layout), for ncu")
    ap.add_argument("--sweep", default=None, help="K1,K2,...: step time per verify width on one GPU")
    ap.add_argument("--qmm-sweep", default=None, help="N,K;...: warm matmul time per shape, token count and kernel")
    ap.add_argument("--qmm-ms", default="1,2,4,8,16,32", help="token counts of --qmm-sweep")
    ap.add_argument("--batch", type=int, default=0, help="sequences of a multi-sequence verify step (with --k)")
    ap.add_argument("--ctx", type=int, default=4096, help="prior KV tokens per sequence of --batch")
    ap.add_argument("--resident-gb", type=float, default=0.0,
                    help="HBM budget (GB) for the layers' 4-bit matrices; the rest stream from pinned host memory")
    args = ap.parse_args()
    if args.sweep:
        return sweep(args)
    if args.qmm_sweep:
        return qmm_sweep(args)
    if args.profile_step:
        return profile_step(args)
    if args.trace_step:
        return trace_step(args)
    if args.profile_small:
        return profile_small(args)
    if args.profile_qmm:
        return profile_qmm(args)
    args.warmup = max(args.warmup, 1)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        if args.impl != "reference":
            torch.cuda.set_device(local_rank)
        dist.init_process_group("gloo" if args.impl == "reference" else "nccl",
                                timeout=datetime.timedelta(seconds=300))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.batch:
            run_batch(args, rank, world, local_rank)
        else:
            run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

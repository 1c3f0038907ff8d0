#!/usr/bin/env python
"""Decode throughput of the B200 quantized decoder (tokens/s).

Workloads (synthetic random-weight models, linear weights N(0, 0.02)
quantized to GGUF Q4_K on the device, embeddings f16 N(0, 1), norms 1.0):
  * N = 1: Llama-3-8B shape, Q4_K, batch 1, context 4096 (then greedy decode);
  * N > 1: Llama-3-70B shape, Q4_K, tensor-parallel over N GPUs (column-split
    q/k/v/gate/up, row-split o/down, NCCL all-reduce), batch 1, context 8192.
The context's KV cache is filled with seeded pseudo-random rows instead of
running the prefill; a decode step's work does not depend on cached values.

value: greedy decode steps replayed as CUDA graphs with the next token fed back
on the device, timed with CUDA events on the decode stream, max over ranks.
e2e: the same steps through the public C-ABI call beacon_cuda_model_decode_step
with host buffers: token in (pinned staging), next token and the full logits
row out to the host every step, as the reference's CLI reads them
(crates/beacon-cli/src/main.rs:306-333).
roofline: the dominant kernel (fused gate/up dequant-GEMV, half of the weight
bytes of a step), timed over all layers (L2-cold) with CUDA events.
cpu_baseline / --impl reference: the CPU restatement of the reference path
(oracle/), row-parallel on all host cores, timed on a depth-truncated copy of
the same model (1 and 2 layers, full vocabulary) at the same context and
extrapolated to full depth: t = t1 + (L - 1) * (t2 - t1).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
for _p in (REPO, os.path.join(REPO, "beacon-ai_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

WORKLOADS = {
    "llama3-8b-q4k": dict(shape="LLAMA3_8B", context=4096, batch=1,
                          name="Llama-3-8B-shape decoder, Q4_K linears, f16 KV, batch {batch}, context 4096, "
                               "greedy decode"),
    "llama3-70b-q4k-tp": dict(shape="LLAMA3_70B", context=8192, batch=1,
                              name="Llama-3-70B-shape decoder, Q4_K linears, f16 KV, tensor-parallel, batch {batch}, "
                                   "context 8192, greedy decode"),
    # prefill (time to first token); its own line, not the decode metric
    "llama3-8b-q8_0-prefill": dict(shape="LLAMA3_8B", context=2048, batch=4,
                                   name="Llama-3-8B-shape decoder, Q8_0 linears, f16 KV, prefill of 4 x 2048-token "
                                        "prompts (time to first token)"),
}
METRIC = "decode tok/s"
# What the timed decode computes in (fast numerics).
FAST_DTYPE = ("q4_k weights; activations quantised to int16 per 32-element block (fast numerics), integer dot "
              "products; attention scores and P.V on f16 MMAs (query split into f16 high/low parts, P rounded to "
              "f16); f32 accumulation and softmax")
# The op-level dequant-GEMV sweep (weight shapes out x in, formats, batches).
SWEEP_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
SWEEP_BATCHES = (1, 4, 16)


def workload_name(wl, batch, layers=0):
    return WORKLOADS[wl]["name"].format(batch=batch) + (f" (REDUCED to {layers} layers)" if layers else "")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=256)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["auto"] + list(WORKLOADS), default="auto")
    p.add_argument("--batch", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-sweep", action="store_true", help="skip the op-level dequant-GEMV sweep")
    p.add_argument("--no-exact", action="store_true", help="skip the exact-numerics decode figure")
    p.add_argument("--layers", type=int, default=0,
                   help="profiling only: build the workload with this many layers (the line says so)")
    p.add_argument("--profile-run", action="store_true",
                   help="profiling only: run warm-up and timed steps, skip the e2e, roofline and CPU legs")
    p.add_argument("--prefill", action="store_true",
                   help="measure prefill instead: 4 x 2048-token prompts through the tensor-core GEMM (one JSON line)")
    a = p.parse_args()
    if a.warmup < 3:
        a.warmup = 3
    if a.workload == "auto":
        a.workload = "llama3-8b-q4k" if a.gpus == 1 else "llama3-70b-q4k-tp"
    return a


def shape_of(wl):
    from beacon_cuda import synthetic
    return dict(getattr(synthetic, WORKLOADS[wl]["shape"]))


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_for(kernel_key):
    """dram bytes per launch from the committed ncu summary, if captured."""
    path = os.path.join(REPO, "profiles", "traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == kernel_key:
                return int(float(parts[1]))
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi samples every 200 ms while the timed region runs."""

    def __init__(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        lr = int(os.environ.get("LOCAL_RANK", "0"))
        idx = vis.split(",")[lr] if vis else str(lr)
        self.tmp = tempfile.NamedTemporaryFile(prefix="clocks", suffix=".csv", delete=False)
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap,utilization.gpu")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", idx, f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.tmp.close()
        rows = []
        for line in open(self.tmp.name):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                rows.append((float(f[0]), float(f[1]), f[3:7], float(f[7])))
            except ValueError:
                continue
        os.unlink(self.tmp.name)
        if not rows:
            return None
        busy = [r for r in rows if r[3] > 0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in busy for i, v in enumerate(r[2]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in busy), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# --- CPU restatement (oracle) on a depth-truncated sample -------------------------

class CpuDecodeSample:
    """The oracle engine on 1- and 2-layer copies of the workload's model
    (full vocabulary, same context); one step times one decode token per
    sequence on both and extrapolates to full depth."""

    def __init__(self, wl, batch, ref_faithful=False):
        import numpy as np

        import oracle as orc
        self.orc = orc
        shp = shape_of(wl)
        self.ctx = WORKLOADS[wl]["context"]
        self.batch = batch
        self.layers = shp["num_layers"]
        H, F, V = shp["hidden_size"], shp["intermediate_size"], shp["vocab_size"]
        QD, KD = shp["num_heads"] * shp["head_dim"], shp["num_kv_heads"] * shp["head_dim"]
        rng = np.random.default_rng(0)

        def rows(n, k):  # one quantized N(0, 0.02) row, tiled: the CPU cost does not depend on values
            row = orc.quantize((rng.standard_normal(k) * 0.02).astype(np.float32), orc.Q4_K)
            return np.tile(row, n)

        emb_row = rng.standard_normal(H).astype(np.float16)
        self.models = {}
        for nl in (1, 2):
            cfg = orc.OracleModelConfig(V, H, nl, shp["num_heads"], shp["num_kv_heads"], shp["head_dim"], F,
                                        self.ctx + 2, shp["rope_theta"], shp["rms_norm_eps"], kv_persist=True,
                                        causal_prefill=True, weights_rtz=True, threads=1 if ref_faithful else 0,
                                        ref_faithful=ref_faithful)
            m = orc.OracleModel(cfg)
            m.set_weight(0, orc.W_EMBED, np.tile(emb_row, V), orc.F16)
            m.set_weight(0, orc.W_FINAL_NORM, np.ones(H, np.float16), orc.F16)
            m.set_weight(0, orc.W_LM_HEAD, rows(V, H), orc.Q4_K)
            for li in range(nl):
                m.set_weight(li, orc.W_ATTN_NORM, np.ones(H, np.float16), orc.F16)
                m.set_weight(li, orc.W_FFN_NORM, np.ones(H, np.float16), orc.F16)
                for w, (n, k) in ((orc.W_Q, (QD, H)), (orc.W_K, (KD, H)), (orc.W_V, (KD, H)), (orc.W_O, (H, QD)),
                                  (orc.W_GATE, (F, H)), (orc.W_UP, (F, H)), (orc.W_DOWN, (H, F))):
                    m.set_weight(li, w, rows(n, k), orc.Q4_K)
            if not ref_faithful:
                m.forward([1], self.ctx)  # warm the caches
            self.models[nl] = m

    def step(self):
        """(extrapolated tok/s, {layers: seconds}, seconds this sample took)."""
        t = {}
        w0 = time.perf_counter()
        for nl, m in self.models.items():
            t0 = time.perf_counter()
            for b in range(self.batch):
                m.forward([1 + b], self.ctx)  # one token per sequence at position `ctx`
            t[nl] = time.perf_counter() - t0
        t_tok = t[1] + (self.layers - 1) * max(t[2] - t[1], 0.0)
        return self.batch / t_tok, t, time.perf_counter() - w0


def cpu_decode_sample(wl, batch, reps=3, ref_faithful=False):
    s = CpuDecodeSample(wl, batch, ref_faithful)
    best = None
    for _ in range(reps):
        v, t, _ = s.step()
        if best is None or v > best[0]:
            best = (v, t)
    return best


def host_threads():
    try:
        import oracle as orc  # noqa: F401
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# --- our arm ---------------------------------------------------------------------------

def run_ours(a):
    import numpy as np
    import torch
    import torch.distributed as dist

    from beacon_cuda import CudaBackend, CudaModel, DecoderConfig
    from beacon_cuda import _lib as L
    from beacon_cuda.synthetic import load_synthetic

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    wl = a.workload
    shp = shape_of(wl)
    if a.layers:
        shp["num_layers"] = a.layers
    ctx_len = WORKLOADS[wl]["context"]
    batch = a.batch or WORKLOADS[wl]["batch"]
    max_ctx = ctx_len + 2 * (a.warmup + a.steps) + 16

    be = CudaBackend(local, L.NUMERICS_FAST)
    if world > 1:
        import ctypes
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            buf = (ctypes.c_uint8 * 128)()
            L.check(L.lib().beacon_cuda_comm_unique_id(buf))
            uid.copy_(torch.tensor(list(buf), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        idb = (ctypes.c_uint8 * 128)(*uid.cpu().tolist())
        L.check(L.lib().beacon_cuda_comm_init(be.ctx, world, rank, idb, 120000))
    cfg = DecoderConfig(**shp, max_context=max_ctx, max_batch=batch, numerics=L.NUMERICS_FAST,
                        kv_dtype=L.DTYPE_F16, tp_size=world, tp_rank=rank)
    model = CudaModel(be, cfg)
    load_synthetic(model, L.DTYPE_Q4_K, seed=0)
    model.fill_kv_random(ctx_len, seed=1)
    ts = torch.cuda.ExternalStream(model.stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    tok0 = torch.tensor([17 + b for b in range(batch)], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    # warm-up: captures both graphs (host-fed and device-continuing)
    model.decode_step_device(tok0.data_ptr(), batch, ctx_len)
    for _ in range(a.warmup - 1):
        model.decode_step_device(None, batch, -1)
    model.stream.synchronize()
    launches = model.launches_per_step(batch, True)

    # --- value: device-resident greedy decode ---
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ts)
    for _ in range(a.steps):
        model.decode_step_device(None, batch, -1)
    e1.record(ts)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1))
    value = a.steps * batch / (ms / 1e3)
    if a.profile_run:
        model.close()
        be.close()
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"profile_run": True, "workload": wl, "layers": shp["num_layers"],
                              "ms_per_step": ms / a.steps, "launches_per_step": launches}), flush=True)
        return

    # --- e2e: public C-ABI call with host buffers, logits to the host each step ---
    pos = ctx_len + a.warmup + a.steps
    toks = np.arange(batch, dtype=np.uint32) + 5
    for _ in range(2):
        toks, _lg = model.decode_step(toks, pos, want_logits=True)
        pos += 1
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    f0.record(ts)
    for _ in range(a.steps):
        toks, _lg = model.decode_step(toks, pos, want_logits=True)
        pos += 1
    f1.record(ts)
    f1.synchronize()
    wall = time.perf_counter() - wall0
    barrier()
    e2e_ms = max_over_ranks(max(f0.elapsed_time(f1), wall * 1e3))
    e2e_value = a.steps * batch / (e2e_ms / 1e3)

    # --- roofline of the dominant kernel: fused gate/up projection over all layers ---
    us, nbytes = model.profile_linear(L.W_GATE, batch, 3)
    achieved = nbytes / (us * 1e-6) / 1e9
    peak, peak_kind = peaks()
    traffic = traffic_for(f"gate_up_{wl}_b{batch}")
    kernel = ("qgemv3_kernel<Q4_K, FAST, B=%d> (persistent dequant-GEMV, fused gate/up + SwiGLU)" % batch
              if batch <= 16 else
              "qgemm_tc_kernel<Q4_K> (tcgen05 dequant-GEMM, fused gate/up + SwiGLU, M=%d)" % batch)
    mem_gb = model.memory_bytes() / 1e9
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": FAST_DTYPE,
        "data": "synthetic (seeded random weights; KV context filled with seeded random rows)",
        "config": {"workload": workload_name(wl, batch, a.layers),
                   "model_shape": wl, "batch": batch, "context": ctx_len,
                   "parallelism": f"tp{world}", "l2": f"inputs larger than L2: {mem_gb:.1f} GB "
                                                     "of weights and cache are read every step"},
        "e2e": {"value": round(e2e_value, 2), "unit": "tok/s",
                "h2d_bytes_per_step": 4 + 4 * batch,
                "d2h_bytes_per_step": 4 * batch + 4 * batch * shp["vocab_size"]},
        "gpu_launches": launches * a.steps,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the same kernel and "
                                       "shape (profiles/traffic.txt); null when not captured",
                     "kernel": "%s, %.2f us/launch (CUDA events, back-to-back over every layer's weights), "
                               "%d algorithmic bytes/launch, peak %s" % (kernel, us, nbytes, peak_kind)},
    }
    if clk:
        out["clocks"] = clk
    model.close()
    del model
    # the same decode in the exact numerics (f32 activations, f32 attention)
    if world == 1 and not a.no_exact:
        out["exact_numerics"] = exact_decode(a, shp, ctx_len, batch, max_ctx)
    if world == 1 and not a.no_sweep:
        out["gemv_sweep"] = gemv_sweep(be, peak)
        out["gemv_sweep_note"] = ("quantized_matmul's decode path through beacon_cuda_profile_quantized_matmul, fp16 "
                                  "activations, fast numerics, weights cycled over copies totalling >= 4x L2 (every "
                                  "launch reads its weights from HBM); bytes = N*K*bpe + B*K*2 + B*N*4; frac of the "
                                  "%s HBM peak" % peak_kind)
    be.close()
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        tps, parts = cpu_decode_sample(wl, batch)
        out["cpu_baseline"] = {"value": round(tps, 4), "unit": "tok/s", "cores": host_threads(), "kind": "port",
                               "sample": "oracle engine (row-parallel on all host cores, same sums as the reference), "
                                         "1- and 2-layer copies of the model (full vocab) decoding one token at "
                                         "position %d; t1=%.3fs t2=%.3fs, extrapolated to %d layers"
                                         % (ctx_len, parts[1], parts[2], shp["num_layers"])}
        tps1, parts1 = cpu_decode_sample(wl, batch, reps=1, ref_faithful=True)
        out["cpu_baseline_ref_faithful"] = {
            "value": round(tps1, 5), "unit": "tok/s", "cores": 1, "kind": "port",
            "sample": "the reference's own loop order, one thread: per-call transposed copy of each weight "
                      "(cpu_backend.rs:330-366) and the column-strided matmul_f32 (ops.rs:16-30); 1- and 2-layer "
                      "copies of the model decoding one token at position %d; t1=%.2fs t2=%.2fs, extrapolated to "
                      "%d layers" % (ctx_len, parts1[1], parts1[2], shp["num_layers"])}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def exact_decode(a, shp, ctx_len, batch, max_ctx):
    """Device-resident greedy decode of the same workload in the exact numerics."""
    import torch

    from beacon_cuda import CudaBackend, CudaModel, DecoderConfig
    from beacon_cuda import _lib as L
    from beacon_cuda.synthetic import load_synthetic
    be = CudaBackend(0, L.NUMERICS_EXACT)
    model = CudaModel(be, DecoderConfig(**shp, max_context=max_ctx, max_batch=batch, numerics=L.NUMERICS_EXACT,
                                        kv_dtype=L.DTYPE_F16))
    load_synthetic(model, L.DTYPE_Q4_K, seed=0)
    model.fill_kv_random(ctx_len, seed=1)
    ts = torch.cuda.ExternalStream(model.stream.cuda_stream)
    tok0 = torch.tensor([17 + b for b in range(batch)], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    model.decode_step_device(tok0.data_ptr(), batch, ctx_len)
    for _ in range(a.warmup - 1):
        model.decode_step_device(None, batch, -1)
    model.synchronize()
    steps = min(a.steps, 64)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ts)
    for _ in range(steps):
        model.decode_step_device(None, batch, -1)
    e1.record(ts)
    e1.synchronize()
    model.synchronize()
    ms = e0.elapsed_time(e1)
    model.close()
    be.close()
    return {"value": round(steps * batch / (ms / 1e3), 2), "unit": "tok/s", "steps": steps,
            "ms_per_step": round(ms / steps, 4),
            "dtype": "q4_k weights dequantised to their f32 values (q*d), f32 activations, f32 attention on the "
                     "CUDA cores, f32 accumulation; f16 KV cache"}


def gemv_sweep(be, peak):
    """Op-level dequant-GEMV sweep: every shape x format x batch of the
    configuration, through the op's decode path, L2-cold."""
    import numpy as np
    import torch

    from beacon_cuda import _lib as L
    from beacon_cuda.synthetic import quantize_on_device
    s = be.new_stream()
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    rng = np.random.default_rng(0)
    rows = []
    for dt, name in ((L.DTYPE_Q4_0, "q4_0"), (L.DTYPE_Q8_0, "q8_0"), (L.DTYPE_Q4_K, "q4_k")):
        for n, k in SWEEP_SHAPES:
            raw = quantize_on_device(be, s, n, k, dt, seed=3, layer=n // 1024, slot=k // 1024)
            copies = max(2, -(-4 * l2 // raw.numel()))
            ws = [be.from_device_blocks(raw.data_ptr(), (n, k), dt) for _ in range(copies)]
            del raw
            x = rng.standard_normal((16, k)).astype(np.float16)
            for b in SWEEP_BATCHES:
                us, nb = be.profile_quantized_matmul(s, ws, be.upload(x[:b]), iters=max(3, 240 // copies))
                gbs = nb / (us * 1e-6) / 1e9
                rows.append({"format": name, "n": n, "k": k, "batch": b, "us": round(us, 3), "gb_s": round(gbs, 1),
                             "frac": round(gbs / peak, 4)})
            del ws
            torch.cuda.empty_cache()
    return rows


def run_prefill(a):
    """Prefill of config 4: 4 prompts x 2048 tokens, Q8_0 8B shape, one GPU.
    value = prompt tokens/s over the batch; ttft_ms = time to prefill all four.
    roofline: the fused gate/up dequant-GEMM at M = 2048 through the C-ABI op,
    FLOPs 2*M*N*K over CUDA-event time, against the measured bf16 peak."""
    import numpy as np
    import torch

    from beacon_cuda import CudaBackend, CudaModel, DecoderConfig
    from beacon_cuda import _lib as L
    from beacon_cuda.synthetic import load_synthetic

    wl = "llama3-8b-q8_0-prefill"
    shp = shape_of(wl)
    if a.layers:
        shp["num_layers"] = a.layers
    P, NB = WORKLOADS[wl]["context"], WORKLOADS[wl]["batch"]
    be = CudaBackend(0, L.NUMERICS_FAST)
    model = CudaModel(be, DecoderConfig(**shp, max_context=P + 16, max_batch=1, numerics=L.NUMERICS_FAST,
                                        kv_dtype=L.DTYPE_F16))
    load_synthetic(model, L.DTYPE_Q8_0, seed=0)
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, shp["vocab_size"], size=(NB, P)).tolist()
    ts = torch.cuda.ExternalStream(model.stream.cuda_stream)
    for i in range(min(a.warmup, 3)):
        model.forward(prompts[i % NB], 0, want_logits=False)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(1, min(a.steps, 4))
    e0.record(ts)
    for _ in range(steps):
        for b in range(NB):
            model.forward(prompts[b], 0, want_logits=False)
    e1.record(ts)
    e1.synchronize()
    ttft_ms = e0.elapsed_time(e1) / steps
    value = NB * P / (ttft_ms / 1e3)

    # GEMM roofline: the model's fused gate/up (2F x H) at M = P rows, every
    # layer's weights in turn (L2-cold), through the model's own linear path
    H, F = shp["hidden_size"], shp["intermediate_size"]
    gemm_us, _nb = model.profile_linear(L.W_GATE, P, 2)
    tflops = 2.0 * P * (2 * F) * H / (gemm_us * 1e-6) / 1e12
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            peak, peak_kind = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        peak, peak_kind = 1590.0, "fallback"
    out = {"metric": "prefill tok/s", "value": round(value, 1), "unit": "tok/s", "n_gpus": 1, "steps": steps,
           "warmup": min(a.warmup, 3), "ms_per_step": round(ttft_ms, 3), "ttft_ms": round(ttft_ms, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights, f16 MMA, f32 accumulate",
           "data": "synthetic (seeded random weights and prompt tokens)",
           "config": {"workload": workload_name(wl, NB, a.layers),
                      "model_shape": wl, "batch": NB, "prompt": P, "parallelism": "tp1"},
           "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tflops / peak, 4), "traffic": None,
                        "kernel": "qgemm_tc_kernel<Q8_0> (fused gate/up, M=%d N=%d K=%d; weights from the model's f16 "
                                  "copies, dequantised by its first prefill and kept), %.1f us/launch incl. the "
                                  "f16 activation copy, peak %s (dense bf16)" % (P, 2 * F, H, gemm_us, peak_kind)}}
    model.close()
    del model
    be.close()
    print(json.dumps(out), flush=True)


def run_reference(a):
    """The reference's CPU path (the oracle port: the reference is Rust and no
    Rust toolchain exists here) on the host cores, on rank 0 only. Each step is
    one bounded sample: one decode token through 1- and 2-layer copies of the
    model, extrapolated to full depth. ms_per_step is the wall time a sample
    actually took; value is the extrapolated full-depth rate."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = a.workload
    batch = a.batch or WORKLOADS[wl]["batch"]
    sample = CpuDecodeSample(wl, batch)
    vals, walls = [], []
    steps = min(a.steps, 32)  # each step is a bounded CPU sample; keep the run to a few minutes
    for i in range(a.warmup + steps):
        tps, _, wall = sample.step()
        if i >= a.warmup:
            vals.append(tps)
            walls.append(wall)
    v = statistics.mean(vals)
    shp = shape_of(wl)
    out = {"metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": a.gpus, "steps": len(vals),
           "warmup": a.warmup, "ms_per_step": round(1e3 * statistics.mean(walls), 2), "higher_is_better": True,
           "extrapolated_ms_per_token": round(1e3 * batch / v, 2),
           "scaling": "strong" if a.gpus > 1 else "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "impl": "reference",
           "config": {"workload": workload_name(wl, batch), "model_shape": wl, "batch": batch,
                      "context": WORKLOADS[wl]["context"], "parallelism": "host cores"},
           "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": host_threads(), "kind": "port",
                            "sample": "CPU restatement of the reference engine (oracle/, row-parallel on all host "
                                      "cores, the reference's sums and their order), one decode token through 1- and "
                                      "2-layer copies of the model at the full context, extrapolated to %d layers"
                                      % shp["num_layers"]},
           "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.prefill:
        run_prefill(args)
    else:
        run_ours(args)

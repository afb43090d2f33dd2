"""Benchmark: full TESMLMHeadModel INT2 prefill on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

A step is one prefill of batch 32 x 4096 tokens per GPU through the public API
(``TESMLMHeadModel.forward(ids, logits_to_keep=1)``): 32 layers, d_model 4096,
d_state 256, window 16, vocab 32000, d_intermediate 11008, ent_rank 64, random
weights (seed 0) and uniform token ids.  Multi-GPU runs are data-parallel replicas
(weak scaling: every rank prefills its own 32 sequences; no collective on the data
path).  Rank 0 prints one JSON line.

``--impl reference`` times the reference's own torch path (the package installed
under ``baseline/_ref``, ``kernel_backend="torch"``) on the host cores: a full
32-layer config-5-width prefill of 1 x 64 tokens per step (see ``ReferenceCPU``).
Without that install it falls back to the numpy restatement and says so.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(n_layer=32, d_model=4096, d_state=256, entanglement_window=16, vocab_size=32000, d_intermediate=11008,
           max_seq_len=4608, ent_rank=64)
BATCH, SEQ = 32, 4096
METRIC = "prefill tokens/s"
UNIT = "tokens/s"


def workload(n):
    return {"workload": "config5: TESMLMHeadModel INT2 prefill, batch 32 x 4096 per GPU", "model": "TESM 32L d4096",
            "global_batch": BATCH * n, "seq_len": SEQ, "parallelism": f"dp{n}", "logits_to_keep": 1,
            "layers": CFG["n_layer"], "d_model": CFG["d_model"], "d_state": CFG["d_state"],
            "d_intermediate": CFG["d_intermediate"], "vocab": CFG["vocab_size"], "window": 16,
            "l2": "inputs larger than L2: per-step activations are GBs (no flush needed)"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ CPU legs (oracle port)
def cpu_sample(layers=2, tokens=128):
    """Time the CPU restatement of the reference prefill on `layers` full-width layers and
    `tokens` tokens (last-token logits).  Returns (tokens/s for the 32-layer model, seconds):
    the layer time is scaled by 32/layers, embedding and head are counted once."""
    import numpy as np
    import oracle as O
    rng = np.random.default_rng(0)
    D, Dm, R, Fd, V = CFG["d_state"], CFG["d_model"], CFG["ent_rank"], CFG["d_intermediate"], CFG["vocab_size"]

    def w(n, k):
        return (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))

    P = {"backbone.embedding.weight": w(V, Dm), "backbone.position_embedding.weight": w(CFG["max_seq_len"], Dm),
         "backbone.norm_f.weight": np.ones(Dm, np.float32)}
    P["lm_head.weight"] = P["backbone.embedding.weight"]
    for i in range(layers):
        pre = f"backbone.layers.{i}."
        P.update({pre + "norm.weight": np.ones(Dm, np.float32), pre + "norm2.weight": np.ones(Dm, np.float32),
                  pre + "mixer.in_proj.weight": w(2 * Dm + 3 * D + 2 * R, Dm),
                  pre + "mixer.state_proj.weight": w(Dm, D), pre + "mixer.ent_proj.weight": w(Dm, D),
                  pre + "mixer.out_proj.weight": w(Dm, Dm), pre + "mixer.cross_layer_q_proj.weight": w(R, D),
                  pre + "mixer.decay_bias": np.full(D, 3.0, np.float32),
                  pre + "mixer.local_entanglement_bias": (rng.standard_normal(16) * 0.3).astype(np.float32),
                  pre + "mlp.gate_proj.weight": w(Fd, Dm), pre + "mlp.up_proj.weight": w(Fd, Dm),
                  pre + "mlp.down_proj.weight": w(Dm, Fd)})
    cfg = dict(CFG, n_layer=layers, entanglement_threshold=0.1, entanglement_scale=0.2, bit_eps=1e-5, rope_base=1e4,
               state_scan_chunk_size=16, use_mimo=False, n_heads=4, mimo_rank=4, norm_epsilon=1e-5)
    ids = rng.integers(0, V, size=(1, tokens))
    O.memo_weights(True)
    O.model_forward(P, cfg, ids[:, :16], logits_to_keep=1)  # ternarise once, as the reference caches in eval
    tm = {}
    t0 = time.perf_counter()
    O.model_forward(P, cfg, ids, logits_to_keep=1, timings=tm)
    t1 = time.perf_counter()
    O.memo_weights(False)
    t_layers, t_head = tm["layers_done"] - t0, t1 - tm["layers_done"]
    t_model = t_layers * CFG["n_layer"] / layers + t_head
    return tokens / t_model, t1 - t0


REF_LAYERS_DISTINCT = 2   # distinct full-width layers built by the reference's own constructor
REF_TOKENS = 64           # prefill tokens per reference step (1 sequence)
REF_DEC_BATCH, REF_DEC_STEPS = 8, 4


def _reference_package():
    """The installed reference (``pip install --target baseline/_ref``), or None."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "tesm_ssm")):
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        from tesm_ssm.models.config_tesm import TESMConfig as RefConfig
        from tesm_ssm.models.mixer_seq_simple import TESMLMHeadModel as RefModel
    except Exception:
        return None
    return RefConfig, RefModel


class ReferenceCPU:
    """The reference's own torch path (``kernel_backend="torch"``, eval, no_grad) on the host
    cores, at config 5's full width and full depth.

    Host memory and build time are bounded by constructing ``REF_LAYERS_DISTINCT`` layers with
    the reference's constructor (seed 0) and running them 16 times over in the reference's own
    ``MixerModel.forward`` (the 32 entries of ``backbone.layers`` alternate between the two
    module objects; every layer keeps its own decode cache).  All 32 layers execute, so a step
    is a real, measured 32-layer forward; sharing weight objects does not change the work
    (fp32 weights of 0.76 GB per layer stream from DRAM either way)."""

    def __init__(self):
        import torch
        import torch.nn as nn
        pkg = _reference_package()
        if pkg is None:
            raise RuntimeError("reference package not installed under baseline/_ref")
        RefConfig, RefModel = pkg
        torch.set_num_threads(cpu_threads())
        t0 = time.perf_counter()
        torch.manual_seed(0)
        cfg = RefConfig(**dict(CFG, n_layer=REF_LAYERS_DISTINCT), kernel_backend="torch")
        self.model = RefModel(cfg).eval()
        layers = list(self.model.backbone.layers)
        self.model.backbone.layers = nn.ModuleList([layers[i % len(layers)] for i in range(CFG["n_layer"])])
        self.model.backbone.config.n_layer = CFG["n_layer"]
        self.build_s = time.perf_counter() - t0
        g = torch.Generator().manual_seed(7)
        self.ids = torch.randint(0, CFG["vocab_size"], (1, REF_TOKENS), generator=g)
        self.dec_prompt = torch.randint(0, CFG["vocab_size"], (REF_DEC_BATCH, 16), generator=g)

    def prefill_step(self):
        """One timed 32-layer prefill of 1 x REF_TOKENS tokens; returns seconds."""
        import torch
        with torch.no_grad():
            t0 = time.perf_counter()
            self.model(self.ids, logits_to_keep=1)
            return time.perf_counter() - t0

    def decode(self, steps):
        """Batch REF_DEC_BATCH: 16-token prompt, then `steps` timed one-token steps; tokens/s."""
        import torch
        with torch.no_grad():
            ip = {"state_cache": self.model.backbone.allocate_inference_cache(REF_DEC_BATCH, CFG["max_seq_len"])}
            o, _ = self.model(self.dec_prompt, inference_params=ip, logits_to_keep=1)
            tok = o.logits[:, -1:].argmax(-1)
            t0 = time.perf_counter()
            for _ in range(steps):
                o, _ = self.model(tok, inference_params=ip)
                tok = o.logits[:, -1:].argmax(-1)
            return REF_DEC_BATCH * steps / (time.perf_counter() - t0)

    def describe(self):
        return (f"reference torch TESMLMHeadModel (kernel_backend='torch', eval, no_grad, fp32), config-5 width, "
                f"32 layers run ({REF_LAYERS_DISTINCT} distinct layer objects alternating), 1 x {REF_TOKENS} "
                f"tokens prefill per step, logits_to_keep=1; build {self.build_s:.0f} s")


def cpu_port_sample(layers=2, tokens=128):
    """Fallback when the reference package is absent: the numpy restatement (oracle port) on
    `layers` full-width layers; returns (tokens/s scaled to 32 layers, seconds measured)."""
    return cpu_sample(layers, tokens)


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    n = cpu_threads()
    try:
        ref = ReferenceCPU()
    except Exception as e:  # reference not installed: labelled oracle-port fallback
        print(f"reference package unavailable ({e}); timing the oracle port", file=sys.stderr)
        ref = None
    if ref is None:
        for _ in range(args.warmup):
            cpu_sample(layers=1, tokens=32)
        meas = [cpu_sample(layers=2, tokens=128) for _ in range(args.steps)]
        v = statistics.median(m[0] for m in meas)
        ms = statistics.median(m[1] for m in meas) * 1e3
        kind, sample = "port", ("oracle port (reference package absent), 2 of 32 full-width layers, 1 x 128 tokens "
                                "per step; reported value scales the layer time x16 (extrapolated)")
        dec = None
    else:
        for _ in range(args.warmup):
            ref.prefill_step()
        ts = [ref.prefill_step() for _ in range(args.steps)]
        t = statistics.median(ts)
        v, ms = REF_TOKENS / t, t * 1e3
        kind, sample = "reference", ref.describe()
        dec = {"metric": "decode tokens/s", "value": ref.decode(REF_DEC_STEPS), "unit": UNIT,
               "batch": REF_DEC_BATCH, "prompt": 16, "steps": REF_DEC_STEPS}
    import torch
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 (reference torch path on CPU)" if kind == "reference" else "f32 (numpy restatement)",
            "data": "synthetic (uniform token ids, random-init weights seed 0)", "impl": "reference",
            "config": workload(world),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": n, "torch_threads": torch.get_num_threads(),
                             "kind": kind, "sample": sample, "cpu": cpu_model()},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if dec:
        line["decode"] = dec
    print(json.dumps(line), flush=True)
    return 0


def cpu_model():
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


# ------------------------------------------------------------------ GPU leg
class Clocks:
    """nvidia-smi sampling during the timed region."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu):
        self.path = tempfile.mktemp(suffix=".csv")
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        for ln in open(self.path):
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(self.NAMES, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def run_gpu(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from tesm_b200 import _lib, ops
    from tesm_b200.models import TESMConfig, TESMLMHeadModel

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    torch.manual_seed(0)
    cfg = TESMConfig(kernel_backend="b200", **CFG)
    with torch.device(dev):
        model = TESMLMHeadModel(cfg, dtype=torch.bfloat16).eval()
    g = torch.Generator().manual_seed(1000 + rank)
    ids_host = torch.randint(0, CFG["vocab_size"], (BATCH, SEQ), generator=g).pin_memory()
    ids = ids_host.to(dev)
    logits_host = torch.empty(BATCH, 1, CFG["vocab_size"], dtype=torch.bfloat16).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def ev():
        return torch.cuda.Event(enable_timing=True)

    with torch.no_grad():
        for _ in range(args.warmup):
            model(ids, logits_to_keep=1)
        barrier()
        clocks = Clocks(local_rank) if rank == 0 else None
        n0 = _lib.launch_count
        e0, e1 = ev(), ev()
        e0.record()
        for _ in range(args.steps):
            model(ids, logits_to_keep=1)
        e1.record()
        barrier()
        launches = (_lib.launch_count - n0) // args.steps
        clk = clocks.stop() if clocks else None
        t_dev = max_over_ranks(e0.elapsed_time(e1) / 1e3)

        # end to end: pinned host ids -> device, forward, next-token logits -> pinned host
        barrier()
        f0, f1 = ev(), ev()
        f0.record()
        for _ in range(args.steps):
            ids.copy_(ids_host, non_blocking=True)
            out, _ = model(ids, logits_to_keep=1)
            logits_host.copy_(out.logits, non_blocking=True)
        f1.record()
        barrier()
        t_e2e = max_over_ranks(f0.elapsed_time(f1) / 1e3)

        # roofline of the dominant kernel (the tcgen05 int8 GEMM: in_proj, out_proj, the SwiGLU
        # gate/up GEMM and down_proj): events around each of its launches in one extra
        # instrumented step, on the launching (current) stream
        rec = []
        orig = ops.gemm

        def timed_gemm(codes, inv, pw, M, out_dtype, out=None, acc=False):
            a, b = ev(), ev()
            a.record()
            r = orig(codes, inv, pw, M, out_dtype, out, acc)
            b.record()
            rec.append((a, b, 2.0 * M * pw.N * pw.K, M * pw.K + pw.N * pw.K + M * pw.N * 2, pw.N, pw.K))
            return r

        orig_sw = ops.gemm_swiglu

        def timed_swiglu(q, pw, out_dtype, out=None):
            if q.M <= 256:  # decode-size batches route through ops.gemm (timed there)
                return orig_sw(q, pw, out_dtype, out)
            a, b = ev(), ev()
            a.record()
            r = orig_sw(q, pw, out_dtype, out)
            b.record()
            rec.append((a, b, 2.0 * q.M * pw.N * pw.K, q.M * pw.K + pw.N * pw.K + q.M * (pw.N // 2) * 2, pw.N, pw.K))
            return r

        ops.gemm, ops.gemm_swiglu = timed_gemm, timed_swiglu
        s0, s1 = ev(), ev()
        s0.record()
        model(ids, logits_to_keep=1)
        s1.record()
        torch.cuda.synchronize()
        ops.gemm, ops.gemm_swiglu = orig, orig_sw
        g_ms = sum(a.elapsed_time(b) for a, b, *_ in rec)
        g_ops = sum(r[2] for r in rec)
        g_bytes = sum(r[3] for r in rec)
        step_ms = s0.elapsed_time(s1)

        # decode (config 5): batch 256, 16-token prompt, greedy steps replayed from a CUDA graph
        from tesm_b200.layers import DecodeGraph
        del out
        torch.cuda.empty_cache()
        dec = {}
        if args.decode_steps > 0:
            Bd = 256
            ip = {"state_cache": model.backbone.allocate_inference_cache(Bd, CFG["max_seq_len"])}
            prompt = torch.randint(0, CFG["vocab_size"], (Bd, 16), generator=g).to(dev)
            o, _ = model(prompt, inference_params=ip, logits_to_keep=1)
            dg = DecodeGraph(model, ip, o.logits[:, -1, :].argmax(-1, keepdim=True))
            for _ in range(3):
                dg.step()
            barrier()
            d0, d1 = ev(), ev()
            d0.record()
            for _ in range(args.decode_steps):
                dg.step()
            d1.record()
            barrier()
            t_dec = max_over_ranks(d0.elapsed_time(d1) / 1e3)
            dec = {"metric": "decode tokens/s", "value": Bd * args.decode_steps * world / t_dec, "unit": UNIT,
                   "batch_per_gpu": Bd, "prompt": 16, "steps": args.decode_steps,
                   "ms_per_step": t_dec / args.decode_steps * 1e3, "cuda_graph": True, "sampling": "greedy argmax"}
            del dg, ip
            if world > 1:
                # tensor-parallel decode over all ranks (FFN column/row split, SISO mixer channel-
                # parallel with all-gathers, NCCL collectives inside the captured graph): one batch
                # of 256 shared by the ranks
                from tesm_b200 import parallel
                parallel.enable_mixer_parallel(model)
                torch.cuda.empty_cache()
                ip = {"state_cache": model.backbone.allocate_inference_cache(Bd, CFG["max_seq_len"])}
                o, _ = model(prompt, inference_params=ip, logits_to_keep=1)
                dg = DecodeGraph(model, ip, o.logits[:, -1, :].argmax(-1, keepdim=True))
                for _ in range(3):
                    dg.step()
                n_tp = min(args.decode_steps, 128)
                barrier()
                d0, d1 = ev(), ev()
                d0.record()
                for _ in range(n_tp):
                    dg.step()
                d1.record()
                barrier()
                t_tp = max_over_ranks(d0.elapsed_time(d1) / 1e3)
                dec["tensor_parallel"] = {"tp": world, "batch": Bd, "steps": n_tp, "value": Bd * n_tp / t_tp,
                                          "unit": UNIT, "ms_per_step": t_tp / n_tp * 1e3,
                                          "note": "whole job: one batch shared by all ranks; data-parallel "
                                                  "replicas (the value above) are faster at this batch"}
                del dg, ip
        status = ops.device_status()

    if rank != 0:
        return 0
    peaks, src = load_peaks()
    # MEASURED_PEAKS.json carries bf16 only; the int8 denominator is measured here with the
    # vendor library (torch._int_mm -> cuBLASLt int8, 8192^3, best of 5).
    a8 = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    b8 = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a8, b8.t())
    best = 1e9
    for _ in range(5):
        x0, x1 = ev(), ev()
        x0.record()
        torch._int_mm(a8, b8.t())
        x1.record()
        torch.cuda.synchronize()
        best = min(best, x0.elapsed_time(x1) / 1e3)
    peak_int8 = 2.0 * 8192 ** 3 / best / 1e12
    del a8, b8
    achieved = g_ops / (g_ms / 1e3) / 1e12
    traffic = None
    tp = os.path.join(ROOT, "profiles", "gemm_i8_traffic.json")
    if os.path.exists(tp):
        # ncu DRAM bytes measured per GEMM shape at this M (bench.py --kernel prefill_gemms),
        # averaged over the step's launches of those shapes (the small cross_layer_q_proj
        # launches, not captured, count as their algorithmic bytes)
        with open(tp) as f:
            tj = json.load(f)
        meas = {(sh["N"], sh["K"]): sh["dram_read"] + sh["dram_write"] for sh in tj["shapes"] if tj["M"] == BATCH * SEQ}
        tot = 0.0
        for (_, _, _, bb, n, k) in rec:
            tot += meas.get((n, k), bb)
        traffic = tot / len(rec)
    tokens = BATCH * SEQ * world
    try:  # the reference's own torch path on the host cores, 3 timed 32-layer steps
        ref = ReferenceCPU()
        ref.prefill_step()
        ts = [ref.prefill_step() for _ in range(3)]
        cpu_b = {"value": REF_TOKENS / statistics.median(ts), "unit": UNIT, "cores": cpu_threads(),
                 "kind": "reference", "sample": ref.describe() + f"; median of 3 steps ({sum(ts):.1f} s)",
                 "cpu": cpu_model()}
        del ref
    except Exception as e:
        cpu_v, cpu_dt = cpu_sample(layers=2, tokens=96)
        cpu_b = {"value": cpu_v, "unit": UNIT, "cores": cpu_threads(), "kind": "port",
                 "sample": f"reference package unavailable ({e}); oracle port, 2 of 32 full-width layers, 1 x 96 "
                           f"tokens ({cpu_dt:.1f} s), layer time x16 + head (extrapolated)"}
    line = {
        "metric": METRIC, "value": tokens / (t_dev / args.steps), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_dev / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 x int2 -> int32 GEMMs; fp32 scan/entanglement; bf16 activations",
        "data": "synthetic (uniform token ids, random-init weights seed 0)", "config": workload(world),
        "e2e": {"value": tokens / (t_e2e / args.steps), "unit": UNIT, "h2d_bytes_per_step": BATCH * SEQ * 8,
                "d2h_bytes_per_step": BATCH * CFG["vocab_size"] * 2},
        "roofline": {"bound": "tensor", "kernel": "tesm::tc::k_gemm_i8 (tcgen05.mma kind::i8)",
                     "achieved": achieved, "peak": peak_int8, "unit": "TOPS", "frac": achieved / peak_int8,
                     "traffic": traffic, "launches_per_step": len(rec), "avg_launch_ms": g_ms / len(rec),
                     "algorithmic_bytes_per_launch": g_bytes / len(rec), "share_of_step": g_ms / step_ms,
                     "peak_source": "cuBLASLt int8 GEMM 8192^3 measured in this run (torch._int_mm, burst)",
                     "frac_of_2x_bf16_sustained": achieved / (2.0 * peaks["bf16_tflops_sustained"]),
                     "peaks_file": src},
        "cpu_baseline": cpu_b,
        "decode": dec, "clocks": clk, "gpu_launches": launches, "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_combine_case(args):
    """Config-5 shaped dual-accumulator combine GEMM (state_proj + ent_proj + output combine) on
    M = 32768 tokens, d_state 256, d_model 4096, bf16 proj / output (for ncu captures)."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    M, D, Dm = 32768, 256, 4096
    Np = 2 * Dm + 3 * D + 128
    proj = torch.randn(M, Np, device="cuda").to(torch.bfloat16)
    codes = torch.randint(-127, 127, (M, 2 * D), device="cuda", dtype=torch.int8)
    inv1 = torch.rand(M, device="cuda") * 0.01
    inv2 = torch.rand(M, device="cuda") * 0.01
    tern = torch.randint(-1, 2, (Dm, 2 * D), device="cuda", dtype=torch.int8)
    deq = torch.full((1,), 0.02, device="cuda")
    y = torch.empty(M, Dm, device="cuda", dtype=torch.bfloat16)
    for _ in range(args.warmup + args.steps):
        ops.gemm_combine(codes, D, inv1, inv2, tern, deq, deq, proj, 0, Dm + 3 * D, M, Dm, y)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    ops.gemm_combine(codes, D, inv1, inv2, tern, deq, deq, proj, 0, Dm + 3 * D, M, Dm, y)
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / 1e3
    byts = M * Dm * 2 * 3 + M * 2 * D
    print(json.dumps({"kernel": "gemm_i8_combine", "M": M, "ms": t * 1e3, "GB_s": byts / t / 1e9}), flush=True)
    return 0


def run_quant_case(args):
    """The activation quantisers at prefill and decode shapes of config 5, graph-timed, for
    ncu captures and their HBM fractions: k_quant_act on the SwiGLU output h (M x 11008 bf16 in,
    int8 codes out) and k_add_rmsnorm_quant on a block boundary (M x 4096 bf16 hidden + fp32
    residual in, fp32 residual + int8 codes out).  Prefill M = 16384 (inputs > L2); decode M = 256."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    peaks, _ = load_peaks()
    F, Dm = CFG["d_intermediate"], CFG["d_model"]
    for M in (16384, 256):
        h = torch.randn(M, F, device="cuda").to(torch.bfloat16)
        t = _graph_time(lambda i: ops.quant_act(h, 1e-5, ops.LAYOUT_ROWMAJOR), inner=4)
        byts = M * F * 3
        print(json.dumps({"kernel": "k_quant_act", "M": M, "K": F, "us": t * 1e6, "GB_s": byts / t / 1e9,
                          "hbm_frac": byts / t / 1e9 / peaks["hbm_gbs"]}), flush=True)
        del h
        x = torch.randn(M, Dm, device="cuda").to(torch.bfloat16)
        res = torch.randn(M, Dm, device="cuda")
        res_out = torch.empty_like(res)
        w = torch.rand(Dm, device="cuda") + 0.5
        q = ops.alloc_quant(M, Dm, x.device, ops.LAYOUT_ROWMAJOR)
        t = _graph_time(lambda i: ops.add_rmsnorm_quant(x, res, res_out, w, 1e-5, 1e-5, q), inner=4)
        byts = M * Dm * (2 + 4 + 4 + 1)
        print(json.dumps({"kernel": "k_add_rmsnorm_quant", "M": M, "K": Dm, "us": t * 1e6, "GB_s": byts / t / 1e9,
                          "hbm_frac": byts / t / 1e9 / peaks["hbm_gbs"]}), flush=True)
        del x, res, res_out
    return 0


def run_kernel_case(args):
    """Small standalone case of the dominant kernel for ncu captures: one int8 tcgen05 GEMM
    of in_proj-like shape M=16384, N=11008, K=4096 (operands 109 MB + 360 MB output > L2)."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    M, N, K = 16384, 11008, 4096
    w = torch.randn(N, K, device="cuda") * 0.02
    pw = ops.pack_weight(w, 1e-5, with_tern=True)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    codes, inv, _ = ops.quant_act(x, 1e-5, ops.LAYOUT_ROWMAJOR)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    for _ in range(args.warmup):
        ops.gemm(codes, inv, pw, M, torch.bfloat16, out)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        ops.gemm(codes, inv, pw, M, torch.bfloat16, out)
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / args.steps / 1e3
    print(json.dumps({"kernel": "gemm_i8", "M": M, "N": N, "K": K, "ms": t * 1e3, "TOPS": 2.0 * M * N * K / t / 1e12,
                      "algorithmic_bytes": M * K + N * K + M * N * 2, "ops": 2.0 * M * N * K}), flush=True)
    return 0


PREFILL_GEMMS = [("in_proj", 9088, 4096), ("out_proj", 4096, 4096), ("gate_up", 22016, 4096), ("down_proj", 4096, 11008)]


def run_prefill_gemms_case(args):
    """The four BitLinear GEMMs of one config-5 prefill layer at the benchmark's M = 32 x 4096 rows,
    one launch each (in_proj, out_proj, the SwiGLU gate/up GEMM, down_proj), for the ncu traffic
    capture that bench.py's roofline object reads (profiles/gemm_i8_traffic.json)."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    M = BATCH * SEQ
    for name, N, K in PREFILL_GEMMS:
        w = torch.randn(N, K, device="cuda") * 0.02
        pw = ops.pack_weight(w, 1e-5, per_row=name == "gate_up", with_tern=True)
        del w
        codes = torch.randint(-127, 128, (M, K), device="cuda", dtype=torch.int8)
        inv = torch.rand(M, device="cuda") * 0.01
        q = ops.QuantAct(codes, inv, None, ops.LAYOUT_ROWMAJOR, M)
        if name == "gate_up":
            out = ops.gemm_swiglu(q, pw, torch.bfloat16)
        else:
            out = ops.gemm(codes, inv, pw, M, torch.bfloat16)
        torch.cuda.synchronize()
        print(json.dumps({"gemm": name, "M": M, "N": N, "K": K}), flush=True)
        del pw, codes, inv, q, out
        torch.cuda.empty_cache()
    return 0


def run_skinny_case(args):
    """Decode-batch BitLinear GEMMs of config 5 (M = 256 rows, int8 codes x ternary weights on
    tcgen05): in_proj, out_proj and down_proj shapes, graph-timed with rotating weight copies
    (> L2) so every call streams its weights from HBM.  One JSON line per shape."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    peaks, _ = load_peaks()
    M = 256
    for name, N, K in [("in_proj", 9088, 4096), ("out_proj", 4096, 4096), ("down_proj", 4096, 11008)]:
        ncopy = max(2, int(3 * 126e6 // (N * K)) + 1)
        w = torch.randn(N, K, device="cuda") * 0.02
        pws = [ops.pack_weight(w.roll(i, 0), 1e-5, with_tern=True) for i in range(ncopy)]
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        codes, inv, _ = ops.quant_act(x, 1e-5, ops.LAYOUT_ROWMAJOR)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t = _graph_time(lambda i: ops.gemm(codes, inv, pws[i % ncopy], M, torch.bfloat16, out), inner=ncopy)
        wbytes = N * ((K + 255) // 256 * 256)  # int8 ternary operand the tensor cores read
        print(json.dumps({"kernel": "skinny gemm_i8", "shape": name, "M": M, "N": N, "K": K, "us": t * 1e6,
                          "TOPS": 2.0 * M * N * K / t / 1e12, "weight_GB_s": wbytes / t / 1e9,
                          "hbm_frac": wbytes / t / 1e9 / peaks["hbm_gbs"]}), flush=True)
        del pws
    # the SwiGLU gate/up GEMM (2 x 11008 interleaved rows, per-row dequantisation)
    N, K = 2 * CFG["d_intermediate"], CFG["d_model"]
    ncopy = max(2, int(3 * 126e6 // (N * K)) + 1)
    w = torch.randn(N, K, device="cuda") * 0.02
    pws = [ops.pack_weight(w.roll(i, 0), 1e-5, per_row=True, with_tern=True) for i in range(ncopy)]
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    q = ops.quantize(x, 1e-5)
    h = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
    t = _graph_time(lambda i: ops.gemm_swiglu(q, pws[i % ncopy], torch.bfloat16, h), inner=ncopy)
    wbytes = N * K
    print(json.dumps({"kernel": "skinny gemm_i8 swiglu", "shape": "gate_up", "M": M, "N": N, "K": K, "us": t * 1e6,
                      "TOPS": 2.0 * M * N * K / t / 1e12, "weight_GB_s": wbytes / t / 1e9,
                      "hbm_frac": wbytes / t / 1e9 / peaks["hbm_gbs"]}), flush=True)
    return 0


def run_decode_case(args):
    """Config-5 model, batch 256: 16-token prefill then `steps` eager one-token decode steps
    (the kernels a decode graph replays), for launch-list captures."""
    import torch
    from tesm_b200.models import TESMConfig, TESMLMHeadModel
    torch.manual_seed(0)
    cfg = TESMConfig(kernel_backend="b200", **CFG)
    with torch.device("cuda"):
        model = TESMLMHeadModel(cfg, dtype=torch.bfloat16).eval()
    with torch.no_grad():
        ip = {"state_cache": model.backbone.allocate_inference_cache(256, CFG["max_seq_len"])}
        prompt = torch.randint(0, CFG["vocab_size"], (256, 16), device="cuda")
        o, _ = model(prompt, inference_params=ip, logits_to_keep=1)
        tok = o.logits[:, -1, :].argmax(-1, keepdim=True)
        for _ in range(args.warmup + args.steps):
            o, _ = model(tok, inference_params=ip)
            tok = o.logits[:, -1, :].argmax(-1, keepdim=True)
        torch.cuda.synchronize()
    print(json.dumps({"kernel": "decode", "batch": 256, "steps": args.warmup + args.steps}), flush=True)
    return 0


def _graph_time(fn, reps=10, inner=8):
    """Median per-call device time of `fn` replayed from a CUDA graph of `inner` calls."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(inner):
            fn(i)
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) / inner / 1e3)
    return statistics.median(ts)


def run_cfg2(args, peaks, rank=0, world=1):
    """BitLinear INT2 microbench, per-tensor and per-row scales.  One call =
    activation quantisation + GEMV (M <= 64) or tensor-core GEMM; weights rotate over enough
    copies to exceed L2 so every call reads them from HBM."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    out = []
    for (N, K) in [(11008, 4096), (4096, 11008)]:
        for per_row in (False, True):
            w = torch.randn(N, K, device="cuda") * 0.02
            ncopy = 14
            pws = [ops.pack_weight(w.roll(i, 0), 1e-5, per_row=per_row, with_tern=True) for i in range(ncopy)]
            for M in (1, 16, 128, 4096):
                x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
                y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
                t = _graph_time(lambda i: ops.bitlinear_2d(x, pws[i % ncopy], 1e-5, torch.bfloat16, y),
                                inner=ncopy if M <= 128 else 4)
                byts = N * K / 4 + M * K * 2 + M * N * 2 + 4 * N + 4 * M
                ops_ = 2.0 * M * N * K
                gbs, tops = byts / t / 1e9, ops_ / t / 1e12
                bound = "hbm" if M <= 16 else ("mixed" if M <= 128 else "tensor")
                out.append({"workload": "cfg2 BitLinear", "N": N, "K": K, "M": M, "scale": "row" if per_row else "tensor",
                            "path": "quant + row-block gemv (mma.sync, packed int2)" if M <= 64 else "tcgen05 int8",
                            "us": t * 1e6, "tokens_per_s": M / t, "GB_s": gbs, "TOPS": tops, "bound": bound,
                            "hbm_frac": gbs / peaks["hbm_gbs"]})
            del pws
    return out


def run_cfg3(args, peaks, rank=0, world=1):
    """standalone SISO scan + local entanglement (+ codes) + global entanglement
    + fused output GEMM at batch 8 x 8192, d_state 256, d_model 2048, window 16, ent_rank 64.
    Synthetic in_proj output: decay pre-activation ~ N(0,1) with decay_bias 0 (a = sigmoid(N(0,1))),
    write / value / q / k / local / gate ~ N(0,1), bf16."""
    import torch
    from tesm_b200 import ops
    torch.manual_seed(0)
    B, L, D, Dm, R, W = 8, 8192, 256, 2048, 64, 16
    if B % world:
        raise SystemExit(f"config 3 splits its batch of {B} over the ranks; {world} does not divide it")
    B //= world  # this rank's sequences; byte / flop counts below are per rank, scaled by world
    M = B * L
    Np = 2 * Dm + 3 * D + 2 * R
    proj = torch.randn(M, Np, device="cuda").to(torch.bfloat16)
    db = torch.zeros(D, device="cuda")
    bias = torch.randn(W, device="cuda") * 0.3
    states = torch.empty(M, D, device="cuda")
    f32 = torch.empty(B, D, device="cuda")
    f64 = torch.empty(B, D, device="cuda", dtype=torch.float64)
    th = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    ch = torch.empty_like(th)
    res = []

    def rec(name, t, byts=None, flops=None, **extra):
        t = _max_over_ranks(t, world)  # whole job: every rank's share, slowest rank's time
        r = {"kernel": name, "ms": t * 1e3, "n_gpus": world}
        if byts is not None:
            r.update(GB_s=byts * world / t / 1e9, hbm_frac=byts / t / 1e9 / peaks["hbm_gbs"],
                     algorithmic_bytes=byts * world)
        if flops is not None:
            r.update(TFLOPS=flops * world / t / 1e12, tensor_frac=flops / t / 1e12 / peaks["bf16_tflops"])
        r.update(extra)
        res.append(r)

    t = _graph_time(lambda i: ops.siso_scan(proj, B, L, Dm, D, R, db, None, states, f32, f64), inner=4)
    rec("k_scan (SISO)", t, M * D * (3 * 2 + 4))  # decay, write, value bf16 in; fp32 states out
    t = _graph_time(lambda i: ops.siso_local_ent(proj, B, L, Dm, D, R, W, None, bias, states, 0.1, 0.2, 1e4, th, ch),
                    inner=4)
    rec("k_win_ent<16> SISO local entanglement (bf16 out)", t, M * (2 * R * 2 + D * 4 + 2 * D * 2))
    t = _graph_time(lambda i: ops.siso_local_ent_codes(proj, B, L, Dm, D, R, W, None, bias, states, 0.1, 0.2, 1e4,
                                                       torch.bfloat16, 1e-5, 1e-5), inner=4)
    rec("k_win_ent<16> SISO local entanglement (int8 codes out)", t, M * (2 * R * 2 + D * 4 + 2 * D + 8))
    emb = torch.randn(64, device="cuda") * 0.02
    relb = ops.global_relbias(emb, 1.0, 0.0, L)
    fl = B * (L * L / 2) * (2 * R + 2 * D)  # algorithmic: causal half, q.k and t.v once each
    t = _graph_time(lambda i: ops.siso_global_ent(proj, B, L, Dm, D, R, None, relb, states, 0.1, 0.2, 1e4, th, ch,
                                                  force="tc"), reps=5, inner=2)
    rec("k_global_ent_tc (tcgen05 kind::f16, incl. prep kernels)", t, flops=fl,
        note="causal half counted once; the kernel issues 3 q.k (hi/lo) and 2 t.v (hi/lo) MMAs, "
             "2.2x the algorithmic flops at R=64, D=256")
    if world == 1:
        t = _graph_time(lambda i: ops.siso_global_ent(proj, B, L, Dm, D, R, None, relb, states, 0.1, 0.2, 1e4, th,
                                                      ch, force="simt"), reps=3, inner=1)
        rec("k_siso_global_ent (SIMT fp32, fallback for ent_rank > 64 / d_state > 256)", t, flops=fl)
    return res


def run_cfg4(args, peaks, rank=0, world=1):
    """TESMMIMO_Optimized layer forward, batch 4 x 16384, d_model 2048, 16 heads,
    d_state 64, ent_rank 48, mimo_rank 4, window 16, bf16 activations, random init seed 0."""
    import torch
    from tesm_b200 import ops
    from tesm_b200.modules import TESMMIMO_Optimized
    import math
    torch.manual_seed(0)
    B, L = 4, 16384
    # (b, h) units: the batch over gcd(4, world) rank groups, the 16 heads over the ranks of a
    # group (8 GPUs: 4 sequences x 2 head halves), head-parallel through NCCL within a group
    bsplit = math.gcd(B, world)
    hsplit = world // bsplit
    if 16 % hsplit:
        raise SystemExit(f"config 4 at {world} GPUs: 16 heads do not split over {hsplit} ranks")
    B //= bsplit
    with torch.device("cuda"):
        m = TESMMIMO_Optimized(d_model=2048, n_heads=16, d_state=64, entanglement_window=16, max_seq_len=L,
                               kernel_backend="b200").eval()
    if hsplit > 1:
        import torch.distributed as dist
        from tesm_b200 import parallel
        groups = [dist.new_group(list(range(g * hsplit, (g + 1) * hsplit))) for g in range(bsplit)]
        parallel.enable_mimo_head_parallel(m, parallel.TPGroup(rank % hsplit, hsplit, groups[rank // hsplit]))
    g = torch.Generator(device="cuda").manual_seed(100 + rank // hsplit)
    x = torch.randn(B, L, 2048, device="cuda", generator=g).to(torch.bfloat16)
    with torch.no_grad():
        t = _max_over_ranks(_graph_time(lambda i: m(x), reps=5, inner=2), world)
        if hsplit > 1:  # the kernel-level lines below are single-GPU measurements
            return [{"workload": "cfg4 MIMO layer", "n_gpus": world, "split": f"batch {bsplit} x heads {hsplit}",
                     "tokens_per_s": B * bsplit * L / t, "ms": t * 1e3}]
        H, D, R, RM, Dm = 16, 64, 48, 4, 2048
        proj = torch.randn(B * L, 2 * Dm + 3 * H * D + 2 * H * R, device="cuda").to(torch.bfloat16)
        states = torch.empty(B * L, RM, H * D, device="cuda")
        f32 = torch.empty(B, H * D, device="cuda")
        f64 = torch.empty(B, H * D, device="cuda", dtype=torch.float64)
        ts = _max_over_ranks(_graph_time(lambda i: ops.mimo_scan(proj, B, L, Dm, H, D, R, RM,
                                                                 m.decay_bias.float().contiguous(),
                                                                 m.mimo_x.float().contiguous(), states, f32, f64),
                                         inner=2), world)
        th = torch.empty(B * L, H * D, device="cuda", dtype=torch.bfloat16)
        ch = torch.empty_like(th)
        bias = m.local_entanglement_bias.float().contiguous()
        mo = m.mimo_o.float().contiguous()
        te = _max_over_ranks(_graph_time(lambda i: ops.mimo_local_ent(proj, B, L, Dm, H, D, R, RM, 16, bias, mo,
                                                                      states, 0.5, 0.2, 1e4, True, th, ch),
                                         inner=2), world)
    E = B * L * H * D * world  # whole job
    ent_bytes = E * (16 + 4) + B * world * L * H * R * 4
    return [{"workload": "cfg4 MIMO layer", "n_gpus": world, "split": f"batch {bsplit}",
             "tokens_per_s": B * world * L / t, "ms": t * 1e3},
            {"kernel": "k_scan (MIMO, 4 ranks)", "n_gpus": world, "ms": ts * 1e3, "GB_s": E * (6 + 16) / ts / 1e9,
             "hbm_frac": E * (6 + 16) / ts / 1e9 / world / peaks["hbm_gbs"], "algorithmic_bytes": E * 22},
            {"kernel": "k_win_ent<16,4> MIMO local entanglement", "n_gpus": world, "ms": te * 1e3, "GB_s": ent_bytes / te / 1e9,
             "hbm_frac": ent_bytes / te / 1e9 / world / peaks["hbm_gbs"], "algorithmic_bytes": ent_bytes}]


def run_workload(args):
    """Supplementary configs.  Under torchrun (WORLD_SIZE > 1) configs 3 and 4 shard their batch
    over the ranks (the split BASELINE names for them; no collective on the data path): every
    rank runs batch / world sequences, each time is the max over ranks, and throughputs are for
    the whole job (strong scaling: the total batch is fixed)."""
    import torch
    peaks, _ = load_peaks()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        fn = {"cfg2": run_cfg2, "cfg3": run_cfg3, "cfg4": run_cfg4}[args.workload]
        if world > 1 and args.workload == "cfg2":
            raise SystemExit("config 2 is a single-GPU microbenchmark (replicas only)")
        recs = fn(args, peaks, rank, world)
        if rank == 0:
            for rec in recs:
                print(json.dumps(rec), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


def _max_over_ranks(t, world):
    if world == 1:
        return t
    import torch
    import torch.distributed as dist
    x = torch.tensor([t], device="cuda", dtype=torch.float64)
    dist.all_reduce(x, op=dist.ReduceOp.MAX)
    return x.item()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default=None, choices=["cfg2", "cfg3", "cfg4"],
                    help="supplementary measurements of BASELINE configs 2-4 (one JSON line per measurement)")
    ap.add_argument("--decode-steps", type=int, default=512, help="config-5 decode steps at batch 256 (0: skip)")
    ap.add_argument("--kernel", default=None, choices=["gemm", "decode", "combine", "skinny", "prefill_gemms", "quant"],
                    help="run a small ncu case")
    args = ap.parse_args()
    if args.workload:
        return run_workload(args)
    if args.kernel == "decode":
        return run_decode_case(args)
    if args.kernel == "combine":
        return run_combine_case(args)
    if args.kernel == "quant":
        return run_quant_case(args)
    if args.kernel == "skinny":
        return run_skinny_case(args)
    if args.kernel == "prefill_gemms":
        return run_prefill_gemms_case(args)
    if args.kernel:
        return run_kernel_case(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        return run_gpu(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())

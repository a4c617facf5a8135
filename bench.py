#!/usr/bin/env python
"""bench.py — the north-star workload: one SDXL UNet step at 1024x1024 (128x128 latent) with
the CFG pair stacked as batch 2, random-init weights of the SDXL architecture, synthetic seeded
inputs.  One process per GPU; every GPU runs its own replica on its own CFG pair (replica data
parallelism, no collective on the path), so `value` (UNet steps/s) is the whole-job aggregate.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line on rank 0.  Legs of our arm:
  value        K steps replayed from the CUDA graph with inputs resident in HBM, CUDA events on
               the launching stream, barrier + synchronize on both sides, max over ranks;
  e2e          the same steps through dlm_unet_forward_host with pinned HOST buffers: every step
               copies latent / text conditioning in and the noise prediction out;
  roofline     the dominant kernel class (tcgen05 GEMM / implicit-GEMM conv): its launches of
               one step replayed alone as one CUDA graph right after the timed region (CUDA
               events), so the per-class times add up to about the step's;
  cpu_baseline the CPU fp32 oracle of the same step (oracle/sdxl_unet.py) on this host's cores
               (rank 0, N = 1 only).
`--impl reference` times the reference's CPU path for this workload: the reference has no CPU
UNet (its UNet is CUDA-only and its golden path needs diffusers + pretrained weights), so the
arm is the fp32 restatement (`kind: port`) on all host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "UNet steps/s per GPU at 1024² CFG-b2; images/s at 1/2/4/8 B200; % fp16 TC peak"
UNIT = "steps/s"
LATENT = 128
BATCH = 2
STEPS_PER_IMAGE = 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--legs", choices=["all", "device"], default="all",
                    help="'device' stops after the device-resident timed leg (for ncu launch lists)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), \
            d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def config(n):
    return {
        "workload": "SDXL UNet2DConditionModel step, 1024x1024 image (latent 128x128), CFG pair as batch 2",
        "model": "sdxl-unet (2.57 G params, random-init)",
        "global_batch": BATCH * n,
        "latent": [LATENT, LATENT],
        "parallelism": f"replica-dp{n}",
        "steps_per_image": STEPS_PER_IMAGE,
        "l2": "inputs larger than L2: every step streams 5.1 GB of weights and a 0.58 GB "
              "activation arena through the 126 MB L2",
    }


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.idx = set(gpu_indices)
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                if int(parts[0]) not in self.idx:
                    continue
                rows.append(parts)
            except ValueError:
                continue
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if "Active" in r[5 + k]
                          and "Not" not in r[5 + k]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def max_over_ranks(ms_local: float, ws: int, device=None) -> float:
    """The timed duration of the whole job: the maximum of every rank's device-timed duration
    (one all-reduce MAX; a plain value when there is one rank)."""
    if ws <= 1:
        return float(ms_local)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(ms_local)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(ws: int, steps: int, ms_total: float) -> float:
    """Whole-job steps/s: every rank runs `steps` steps of its own replica (weak scaling)."""
    return ws * steps / (ms_total / 1000.0)


def make_inputs(device, seed=6, pin=True):
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    lat = torch.randn(1, 4, LATENT, LATENT, generator=g).expand(BATCH, -1, -1, -1).contiguous()
    ehs = torch.randn(BATCH, 77, 2048, generator=g)
    te = torch.randn(BATCH, 1280, generator=g)
    tid = torch.tensor([1024.0, 1024.0, 0.0, 0.0, 1024.0, 1024.0])
    host = [t.half().contiguous() for t in (lat, ehs, te, tid)]
    if pin and torch.cuda.is_available():
        host = [t.pin_memory() for t in host]
    dev = [t.to(device) for t in host]
    return host, dev


def cpu_oracle_step(sd_gpu, host_inputs, timestep=999.0):
    """One UNet step of the CPU fp32 oracle on the same weights / inputs; returns (seconds, threads)."""
    import torch
    from oracle.sdxl_unet import UNetConfig, unet_forward
    torch.set_num_threads(os.cpu_count() or 1)
    sdf = {k: v.float().cpu() for k, v in sd_gpu.items()}
    lat, ehs, te, tid = host_inputs
    with torch.no_grad():
        t0 = time.perf_counter()
        unet_forward(sdf, lat.float(), timestep, ehs.float(), te.float(), tid.float(), UNetConfig())
        dt = time.perf_counter() - t0
    return dt, torch.get_num_threads()


def reference_gpu_leg(sd_gpu, dev_inputs, out, our_value, e0, e1, stream, steps=5, warmup=2):
    """Steps/s of the reference's own CUDA UNet (launch_unet_batched, B=2, default and FAST
    modes) recompiled for sm_100a, on the same weights and device-resident inputs, timed with
    CUDA events over back-to-back steps on the default stream it launches on."""
    import torch
    try:
        from baseline import ref_gpu
        if not ref_gpu.available():
            return {"unavailable": "baseline/_ref_gpu/libref_sdxl_gpu.so not built (no reference tree)"}
        ref = ref_gpu.RefUNet({k: v.cpu() for k, v in sd_gpu.items()})
    except Exception as exc:  # pragma: no cover - reported, not fatal
        return {"unavailable": f"{type(exc).__name__}: {exc}"}
    lat, ehs, te, tid = dev_inputs
    res = {}
    try:
        for mode, fast in (("default", False), ("fast", True)):
            for i in range(warmup):
                ref.forward(lat, 999.0 - 50.0 * i, ehs, te, tid, out, attn_fast=fast, epilogue=fast)
            torch.cuda.synchronize()
            e0.record(stream)
            for i in range(steps):
                ref.forward(lat, 999.0 - 50.0 * i, ehs, te, tid, out, attn_fast=fast,
                            epilogue=fast, sync=False)
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
            res[mode] = {"ms_per_step": ms, "steps_per_s": 1000.0 / ms}
    except Exception as exc:  # pragma: no cover
        res["error"] = f"{type(exc).__name__}: {exc}"
    finally:
        ref.close()
    best = max((v["steps_per_s"] for k, v in res.items() if isinstance(v, dict)), default=None)
    return {"what": "the reference's own CUDA UNet (src/infer/unet.cu launch_unet_batched with its "
                    "kernels and cuBLAS), unchanged, recompiled for sm_100a; same weights and inputs",
            "steps": steps, "warmup": warmup, **res,
            "ours_over_reference_fast": (our_value / res["fast"]["steps_per_s"]) if "fast" in res else None,
            "ours_over_reference_best": (our_value / best) if best else None}


LM_SEQS, LM_PROMPT, LM_NEW = 256, 64, 64   # the LM benchmark: 256 sequences, 64 + 64 tokens


def lm_leg(dev, ws, rank, e0, e1, stream, hbm_peak, peak_src, barrier, cpu=True):
    """The LM benchmark, the ternary BitNet tag LM: greedy decode of LM_SEQS sequences split over
    the ranks by sequence (each rank decodes its share; no exchange).  Whole-job generated tokens/s
    with prompts resident on the device (CUDA events, max over ranks), the same through the host
    API (prompts in, generated ids out), the decode step against HBM (its packed ternary weights
    and activations per step), and — rank 0, N = 1 — the reference's own BitNet::forward
    (src/models/bitnet.hpp:376-440, compiled from its header) timed on a slice on one host core."""
    import numpy as np
    import torch
    from dollama_b200.bitnet_lm import BitNetConfig, BitNetLM, random_weights
    cfg = BitNetConfig(max_seq=LM_PROMPT + LM_NEW)
    lm = BitNetLM(cfg, random_weights(cfg, seed=10, device=dev))
    B = LM_SEQS // ws + (1 if rank < LM_SEQS % ws else 0)
    g = torch.Generator().manual_seed(11 + rank)
    prompts_h = torch.randint(4, cfg.vocab, (B, LM_PROMPT), generator=g, dtype=torch.int32)
    prompts = prompts_h.to(dev)
    out = torch.zeros(B, LM_NEW, dtype=torch.int32, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    L_full = LM_PROMPT + LM_NEW

    def timed(max_len, reps):
        for _ in range(2):
            lm.generate_device(prompts, max_len, out, lens)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            lm.generate_device(prompts, max_len, out, lens)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / reps, ws, dev)

    ms_gen = timed(L_full, 5)
    ms_prefill = timed(LM_PROMPT + 1, 5)          # prefill + the first greedy token
    step_ms = (ms_gen - ms_prefill) / (LM_NEW - 1)
    tokens = LM_SEQS * LM_NEW
    # through the host API: numpy prompts in, generated ids back on the host, per call
    ph = prompts_h.numpy()
    lm.generate(ph, L_full)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(3):
        lm.generate(ph, L_full)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms_host = max_over_ranks(e0.elapsed_time(e1) / 3, ws, dev)
    # algorithmic HBM bytes of one decode step (B tokens, one per sequence), averaged over the
    # decode: the 2-bit ternary weights and their row scales; the BitLinears' int8 inputs and fp32
    # outputs (the residual updates read and written); the tied embedding at its fp32 size (the
    # lm_head reads a transposed double copy of it, twice these bytes; the fp32 size is the
    # algorithmic minimum); the fp32 K / V cache each sequence attends over (P + G / 2 positions on
    # average)
    D, F, NL, V = cfg.d_model, cfg.ffn_dim, cfg.n_layers, cfg.vocab
    tern = NL * (4 * D * D + 3 * D * F)
    w_bytes = tern / 4 + NL * 4 * (5 * D + 2 * F)
    act_bytes = B * NL * ((3 * D + F) + 4 * (7 * D + 2 * F))
    head_bytes = V * D * 4 + B * D * 4
    kv_bytes = B * NL * 2 * D * 4 * (LM_PROMPT + LM_NEW / 2)
    step_bytes = w_bytes + act_bytes + head_bytes + kv_bytes
    res = {
        "workload": f"BitNet tag LM (vocab {cfg.vocab}, d {D}, {NL} layers, {cfg.n_heads} heads, "
                    f"FFN {F} SwiGLU, ternary weights): greedy decode of {LM_SEQS} sequences x "
                    f"{LM_PROMPT} prompt + {LM_NEW} generated tokens, sequences split over {ws} rank(s)",
        "metric": "generated tokens/s", "value": tokens / (ms_gen / 1000.0), "unit": "tokens/s",
        "scaling": "strong", "ms_per_generate": ms_gen, "ms_prefill": ms_prefill,
        "ms_per_decode_step": step_ms,
        "e2e": {"value": tokens / (ms_host / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": int(ph.nbytes), "d2h_bytes_per_step": int(B * (LM_NEW + 1) * 4)},
        "roofline": {"kernel": "one decode step (the 32 ternary BitLinear GEMMs and the context "
                               "kernels around them, 77 launches, one CUDA graph)",
                     "bound": "hbm", "achieved": step_bytes / (step_ms / 1000.0) / 1e9,
                     "peak": hbm_peak, "unit": "GB/s",
                     "frac": step_bytes / (step_ms / 1000.0) / 1e9 / hbm_peak,
                     "traffic": None, "peak_source": f"{peak_src} hbm_gbs",
                     "algorithmic_bytes_per_step": step_bytes,
                     "bytes_split": {"ternary_weights": w_bytes, "activations": act_bytes,
                                     "lm_head_embedding": head_bytes, "kv_cache": kv_bytes}},
    }
    lm.close()
    if cpu and rank == 0 and ws == 1:
        res["cpu_baseline"] = lm_reference_cpu()
    return res


def lm_reference_cpu(n_tokens=8):
    """The reference's own BitNet::forward (oracle/_ref/libref_bitnet.so, compiled from
    src/models/bitnet.hpp at the reference's own dimensions) on one host core: one forward over
    n_tokens positions of one sequence, random ternary weights."""
    import numpy as np
    try:
        from oracle import bitnet as ob
        dims = ob.ref_dims()
        if dims is None:
            return {"value": None, "unit": "tokens/s", "cores": 1, "kind": "reference",
                    "sample": "unavailable: oracle/_ref/libref_bitnet.so not built"}
        V, D, NL, H, F, _ = dims
        rng = np.random.default_rng(10)
        w = {"embed": (0.02 * rng.standard_normal((V, D))).astype(np.float32),
             "final_norm": np.ones(D, np.float32)}
        for l in range(NL):
            for k, shp in (("attn_norm", (D,)), ("wq", (D, D)), ("wk", (D, D)), ("wv", (D, D)),
                           ("wo", (D, D)), ("ffn_norm", (D,)), ("w_gate", (F, D)), ("w_up", (F, D)),
                           ("w_down", (D, F))):
                w[f"layers.{l}.{k}"] = (np.ones(shp, np.float32) if "norm" in k
                                        else rng.integers(-1, 2, shp).astype(np.float32))
        toks = rng.integers(4, V, n_tokens).astype(np.int32)
        t0 = time.perf_counter()
        ob.ref_forward(w, toks)
        dt = time.perf_counter() - t0
        return {"value": n_tokens / dt, "unit": "tokens/s", "cores": 1, "kind": "reference",
                "sample": f"the reference's BitNet::forward (compiled from src/models/bitnet.hpp, "
                          f"its own dims vocab {V} / FFN {F}) over {n_tokens} positions of one "
                          f"sequence, one call, one host thread: {dt:.2f} s"}
    except Exception as exc:  # pragma: no cover - reported, not fatal
        return {"value": None, "unit": "tokens/s", "cores": 1, "kind": "reference",
                "sample": f"failed: {exc}"}


def run_reference(args, ws, rank):
    """The reference arm: the CPU fp32 restatement of the step on all host cores, with its
    weights drawn on the CPU by the oracle's own initialiser.  Nothing of this library (no
    dollama_b200 import, no CUDA) is on this path; it runs exactly --warmup untimed and --steps
    timed steps, on rank 0 only."""
    if rank != 0:
        return 0
    import torch
    from oracle.sdxl_unet import UNetConfig, init_weights, unet_forward
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sdf = {k: v.float() for k, v in init_weights(UNetConfig(), seed=7).items()}
    host, _ = make_inputs("cpu", pin=False)
    lat, ehs, te, tid = (t.float() for t in host)
    steps, warm = max(1, args.steps), max(0, args.warmup)
    ts = [999.0 - 50.0 * i for i in range(STEPS_PER_IMAGE)]
    with torch.no_grad():
        for i in range(warm):
            unet_forward(sdf, lat, ts[i % len(ts)], ehs, te, tid, UNetConfig())
        t0 = time.perf_counter()
        for i in range(steps):
            unet_forward(sdf, lat, ts[i % len(ts)], ehs, te, tid, UNetConfig())
        dt = time.perf_counter() - t0
    v = steps / dt
    sample = (f"{steps} full UNet steps (B=2, 128x128 latent, all 70 transformer blocks) after "
              f"{warm} warm-up, fp32 torch on {threads} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws,
        "steps": steps, "warmup": warm, "ms_per_step": 1000.0 / v, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config(1),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's UNet exists only as CUDA + cuBLAS (src/infer/unet.cu); its CPU "
                "golden path needs diffusers and pretrained weights, absent here; this arm is the "
                "CPU fp32 restatement of the same step, weights drawn on the CPU",
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, ws, rank)
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from dollama_b200.unet import SDXLUNet, random_weights
    from dollama_b200 import _lib as L

    dev = torch.device("cuda", local)
    sd = random_weights(seed=7, device=dev)
    net = SDXLUNet(sd)
    keep_sd = (rank == 0 and ws == 1 and not args.no_cpu_baseline)
    if not keep_sd:
        del sd
        sd = None
    host, (lat, ehs, te, tid) = make_inputs(dev)
    out = torch.empty_like(lat)
    stream = torch.cuda.current_stream(dev)
    ts = [999.0 - 50.0 * i for i in range(STEPS_PER_IMAGE)]

    def barrier():
        if ws > 1:
            dist.barrier()

    # ---------------------------------------------------------------- device-resident leg
    for i in range(max(3, args.warmup)):
        net(lat, ts[i % len(ts)], ehs, te, tid, out)
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_ids = [int(x) for x in vis.split(",")] if vis else list(range(max(ws, 1)))
    sampler = ClockSampler(gpu_ids if rank == 0 else []) if rank == 0 else None
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("dlm_timed")
    e0.record(stream)
    for i in range(args.steps):
        net(lat, ts[i % len(ts)], ehs, te, tid, out)
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms_total = max_over_ranks(e0.elapsed_time(e1), ws, dev)
    ms_step = ms_total / args.steps
    value = job_throughput(ws, args.steps, ms_total)
    finite = bool(torch.isfinite(out).all().item())

    if args.legs == "device":
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws,
                              "steps": args.steps, "ms_per_step": ms_step, "legs": "device"}))
        if ws > 1:
            dist.destroy_process_group()
        net.close()
        return 0

    # ---------------------------------------------------------------- end-to-end leg (host buffers)
    hl, he, ht, hi = host
    hout = torch.empty(tuple(lat.shape), dtype=torch.float16).pin_memory()
    for i in range(max(3, args.warmup)):
        net.forward_host(hl, ts[i % len(ts)], he, ht, hi, hout)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(args.steps):
        net.forward_host(hl, ts[i % len(ts)], he, ht, hi, hout)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_value = job_throughput(ws, args.steps, max_over_ranks(e0.elapsed_time(e1), ws, dev))
    h2d = sum(x.numel() * x.element_size() for x in host)
    d2h = hout.numel() * hout.element_size()

    # ---------------------------------------------------------------- dominant-kernel roofline
    ops = net.time_ops()
    info = net.info()
    burst, sustained, hbm, peak_src = peaks()
    g = ops["gemm"]
    gemm_tf = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] > 0 else 0.0
    step_flops = sum(v["flops"] for v in ops.values())
    roofline = {
        "kernel": "gemm_tc_kernel (tcgen05 GEMM + implicit-GEMM conv), all launches of one step",
        "bound": "tensor", "achieved": gemm_tf, "peak": sustained, "unit": "TFLOP/s",
        "frac": gemm_tf / sustained, "traffic": None,
        "traffic_note": "DRAM bytes are not measurable inside a timed run; single-launch ncu "
                        "captures of the step's GEMM shapes are summarised under profiles/",
        "peak_source": f"{peak_src} bf16_tflops_sustained (kernel timed inside a long step)",
        "frac_of_burst_peak": gemm_tf / burst,
        "launches": g["launches"], "avg_launch_us": 1000.0 * g["ms"] / max(1, g["launches"]),
        "algorithmic_flops_per_launch": g["flops"] / max(1, g["launches"]),
        "step": {"flops": step_flops, "achieved_tflops": step_flops / (ms_step / 1000.0) / 1e12,
                 "frac_of_sustained": step_flops / (ms_step / 1000.0) / 1e12 / sustained},
        "by_class_ms": {k: round(v["ms"], 4) for k, v in ops.items()},
        "by_class_note": "each class's launches replayed alone as one CUDA graph (step order, "
                         "5 replays, CUDA events); the classes' sum against ms_per_step is "
                         "class_sum_over_step",
        "class_sum_over_step": sum(v["ms"] for v in ops.values()) / ms_step,
    }

    # ---------------------------------------------------------------- whole image (txt2img)
    # 20 Euler steps with CFG on the device + the VAE decode (dlm_sdxl_generate): one image per
    # replica, no host round trip between steps
    from dollama_b200.pipeline import euler_schedule, generate
    from dollama_b200.vae import SDXLVAEDecoder, random_weights as vae_weights
    vae = SDXLVAEDecoder(vae_weights(seed=9, device=dev))
    sig, _ = euler_schedule(STEPS_PER_IMAGE)
    g = torch.Generator(device="cpu").manual_seed(8)
    init = (torch.randn(1, 4, LATENT, LATENT, generator=g) * sig[0]).to(dev)
    generate(net, vae, init, ehs, te, tid, steps=STEPS_PER_IMAGE, guidance=7.5)  # warm-up
    runs = []
    for _ in range(3):  # median of three images
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        img = generate(net, vae, init, ehs, te, tid, steps=STEPS_PER_IMAGE, guidance=7.5)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        runs.append(max_over_ranks(e0.elapsed_time(e1), ws, dev))
    img_ms = sorted(runs)[1]
    txt2img = {"ms_per_image": img_ms, "images_per_s": ws * 1000.0 / img_ms,
               "steps": STEPS_PER_IMAGE, "guidance": 7.5,
               "note": "dlm_sdxl_generate: 20 UNet steps (CFG batch 2) + Euler on the device + "
                       "VAE decode to [1, 3, 1024, 1024]; text encoders not included",
               "image_finite": bool(torch.isfinite(img).all().item())}
    vae.close()

    # ---------------------------------------------------------------- BitNet tag LM
    lm = lm_leg(dev, ws, rank, e0, e1, stream, hbm, peak_src, barrier, cpu=keep_sd)

    # ---------------------------------------------------------------- reference GPU comparator
    # the reference's own CUDA UNet (src/infer/unet.cu + its kernels and cuBLAS), unchanged and
    # recompiled for sm_100a, on the same weights and inputs (rank 0, N = 1 only)
    ref_gpu_line = None
    if keep_sd:
        ref_gpu_line = reference_gpu_leg(sd, (lat, ehs, te, tid), out, value, e0, e1, stream)

    # ---------------------------------------------------------------- CPU baseline (rank 0, N=1)
    cpu = None
    if keep_sd:
        try:
            dt, thr = cpu_oracle_step(sd, host)
            cpu = {"value": 1.0 / dt, "unit": UNIT, "cores": thr, "kind": "port",
                   "sample": "1 full UNet step (B=2, 128x128 latent, 70 transformer blocks), "
                             "CPU fp32 torch oracle, same weights and inputs"}
        except Exception as exc:  # pragma: no cover - reported, not fatal
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": config(ws),
            "images_per_s": value / STEPS_PER_IMAGE,
            "txt2img": txt2img,
            "pct_fp16_tc_peak": 100.0 * roofline["step"]["achieved_tflops"] / sustained,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "reference_gpu": ref_gpu_line,
            "lm": lm,
            "clocks": clocks,
            "gpu_launches": args.steps * (info["launches_per_step"] + 1),
            "output_finite": finite,
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    net.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())

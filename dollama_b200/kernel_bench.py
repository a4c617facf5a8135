"""Single-op timing tool for the B200 kernels (CUDA events, warm-up, L2-sized inputs).

    python -m dollama_b200.kernel_bench gemm --m 8192 --n 640 --k 640
    python -m dollama_b200.kernel_bench conv --n 8 --cin 320 --h 128 --w 128 --cout 320
    python -m dollama_b200.kernel_bench attn --b 2 --heads 10 --sq 4096 --sk 4096
    python -m dollama_b200.kernel_bench gn --n 1 --h 512 --w 512 --cin 512
    python -m dollama_b200.kernel_bench vae --h 128 --w 128            # whole decode (graph)
    python -m dollama_b200.kernel_bench lm --b 256 --sq 64 --sk 128    # prefill 64 + greedy to 128

Prints one JSON line: shape, microseconds per launch, achieved TFLOP/s and the fraction of the
measured bf16 peak (MEASURED_PEAKS.json next to the repository, when present).  Used for the
per-kernel ncu captures under profiles/.
"""
from __future__ import annotations

import argparse
import ctypes
import json
from pathlib import Path

import torch

from . import _lib as L


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _time_graph(fn, iters, warm=3):
    """Device time per call with the calls captured in one CUDA graph, so that host-side planning
    and the ctypes call (a few microseconds each) do not gate launches of short kernels."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _time(fn, iters, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemm", "conv", "attn", "ternary", "gn", "vae", "lm"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=640)
    ap.add_argument("--k", type=int, default=640)
    ap.add_argument("--cin", type=int, default=320)
    ap.add_argument("--h", type=int, default=128)
    ap.add_argument("--w", type=int, default=128)
    ap.add_argument("--cout", type=int, default=320)
    ap.add_argument("--b", type=int, default=2)
    ap.add_argument("--heads", type=int, default=10)
    ap.add_argument("--sq", type=int, default=4096)
    ap.add_argument("--sk", type=int, default=4096)
    ap.add_argument("--dh", type=int, default=64, help="attention head dim (64, or 128..512)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--eager", action="store_true",
                    help="time back-to-back ABI calls instead of a captured graph of them")
    ap.add_argument("--tile-mode", type=int, default=0,
                    help="GEMM tile choice: 0 auto, 1 single CTA, 2 CTA pair, 3 stream-K "
                         "(+16 * forced N tile)")
    a = ap.parse_args(argv)
    if a.tile_mode and a.op in ("gemm", "conv"):
        L.call("dlm_gemm_set_tile_mode", a.tile_mode)
    torch.manual_seed(0)
    dev = "cuda"
    if a.op == "gemm":
        A = torch.randn(a.m, a.k, device=dev).half()
        W = (torch.randn(a.n, a.k, device=dev) * a.k ** -0.5).half()
        C = torch.empty(a.m, a.n, device=dev, dtype=torch.half)
        nws = L.lib().dlm_gemm_workspace_bytes()
        ws = torch.zeros(nws, dtype=torch.uint8, device=dev)  # stream-K workspace
        fn = lambda: L.call("dlm_gemm_fp16_ws", _p(A), a.k, _p(W), _p(C), a.n, a.m, a.n, a.k, 0,
                            None, None, 0, _p(ws), nws, _s())
        flops = 2.0 * a.m * a.n * a.k
        shape = {"m": a.m, "n": a.n, "k": a.k}
    elif a.op == "conv":
        x = torch.randn(a.n, a.h, a.w, a.cin, device=dev).half()
        w = (torch.randn(a.cout, 3, 3, a.cin, device=dev) * (9 * a.cin) ** -0.5).half()
        b = torch.zeros(a.cout, device=dev).half()
        o = torch.empty(a.n, a.h, a.w, a.cout, device=dev, dtype=torch.half)
        fn = lambda: L.call("dlm_conv2d_nhwc", _p(x), a.n, a.h, a.w, a.cin, _p(w), _p(b), _p(o), a.cout,
                            3, 1, None, 0, _s())
        flops = 2.0 * a.n * a.h * a.w * a.cout * 9 * a.cin
        shape = {"n": a.n, "cin": a.cin, "h": a.h, "w": a.w, "cout": a.cout, "k": 3}
    elif a.op == "ternary":
        w = (torch.randn(a.n, a.k, device=dev) * 0.05).float()
        packed = torch.zeros(a.n * a.k // 16, dtype=torch.int32, device=dev)
        alpha = torch.zeros(a.n, dtype=torch.float32, device=dev)
        L.call("dlm_ternary_pack", _p(w), a.n, a.k, _p(packed), _p(alpha), _s())
        xq = torch.randint(-127, 128, (a.m, a.k), dtype=torch.int8, device=dev)
        xs = torch.rand(a.m, device=dev)
        y = torch.empty(a.m, a.n, dtype=torch.float32, device=dev)
        fn = lambda: L.call("dlm_ternary_gemm_i8", _p(packed), _p(alpha), _p(xq), _p(xs), _p(y), a.m, a.n,
                            a.k, _s())
        flops = 2.0 * a.m * a.n * a.k  # int8 ops
        shape = {"m": a.m, "n": a.n, "k": a.k,
                 "bytes": a.n * a.k / 4 + a.m * a.k + 4 * a.m * a.n + 4 * (a.m + a.n)}
    elif a.op == "vae":
        from .vae import SDXLVAEDecoder, random_weights
        dec = SDXLVAEDecoder(random_weights(seed=9))
        lat = torch.randn(1, 4, a.h, a.w, device=dev).half()
        img = dec(lat)
        fn = lambda: dec(lat, out=img)
        flops = 10.47e12 * (a.h * a.w) / (128 * 128)
        shape = {"latent": [1, 4, a.h, a.w], "launches": dec.info()["launches_per_decode"]}
    elif a.op == "lm":
        from .bitnet_lm import BitNetConfig, BitNetLM, random_weights
        cfg = BitNetConfig(max_seq=max(a.sk, 1))
        lm = BitNetLM(cfg, random_weights(cfg, seed=10))
        prompts = torch.randint(0, cfg.vocab, (a.b, a.sq), dtype=torch.int32, device=dev)
        out = torch.zeros(a.b, max(a.sk - a.sq, 1), dtype=torch.int32, device=dev)
        lens = torch.zeros(a.b, dtype=torch.int32, device=dev)
        fn = lambda: lm.generate_device(prompts, a.sk, out, lens)
        flops = 0.0
        shape = {"sequences": a.b, "prompt": a.sq, "max_len": a.sk,
                 "generated_tokens": a.b * (a.sk - a.sq)}
    elif a.op == "gn":
        # GroupNorm(32) + SiLU over NHWC fp16 [n, h*w, cin]: two launches (statistics, apply)
        x = torch.randn(a.n, a.h * a.w, a.cin, device=dev).half()
        g = torch.ones(a.cin, device=dev).half()
        bt = torch.zeros(a.cin, device=dev).half()
        o = torch.empty_like(x)
        sb = L.lib().dlm_group_norm_nhwc_scratch_bytes(a.n, a.h * a.w)
        scr = torch.empty(sb, dtype=torch.uint8, device=dev)
        fn = lambda: L.call("dlm_group_norm_nhwc", _p(x), a.cin, None, 0, a.n, a.h * a.w, _p(g), _p(bt),
                            1e-6, 32, 1, _p(o), _p(scr), sb, _s())
        flops = 0.0
        shape = {"n": a.n, "hw": a.h * a.w, "c": a.cin, "bytes": 3.0 * x.numel() * 2}
    else:
        q = torch.randn(a.b, a.heads, a.sq, a.dh, device=dev).half()
        k = torch.randn(a.b, a.heads, a.sk, a.dh, device=dev).half()
        v = torch.randn_like(k)
        o = torch.empty_like(q)
        if a.dh != 64:         # wide heads (the VAE's Dh = 512)
            sc = a.dh ** -0.5
            fn = lambda: L.call("dlm_launch_attention", _p(q), _p(k), _p(v), _p(o), a.b, a.heads,
                                a.sq, a.sk, a.dh, sc, _s())
        elif a.tile_mode == 1:   # one CTA per 256-query block (no load balancing)
            fn = lambda: L.call("dlm_launch_attention", _p(q), _p(k), _p(v), _p(o), a.b, a.heads,
                                a.sq, a.sk, 64, 0.125, _s())
        else:
            nws = L.lib().dlm_attention_workspace_bytes(a.b, a.heads, a.sq)
            ws = torch.zeros(nws, dtype=torch.uint8, device=dev)
            fn = lambda: L.call("dlm_launch_attention_ws", _p(q), _p(k), _p(v), _p(o), a.b, a.heads,
                                a.sq, a.sk, 64, 0.125, _p(ws), nws, _s())
        flops = 4.0 * a.b * a.heads * a.sq * a.sk * a.dh
        shape = {"b": a.b, "heads": a.heads, "sq": a.sq, "sk": a.sk, "dh": a.dh}
    ms = _time_graph(fn, a.iters) if a.op in ("gemm", "attn", "gn") and not a.eager else _time(fn, a.iters)
    peak = None
    pk = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    if pk.exists():
        peak = json.loads(pk.read_text()).get("bf16_tflops")
    tf = flops / (ms / 1e3) / 1e12 if flops else None
    if "bytes" in shape:
        shape["gbs"] = shape["bytes"] / (ms / 1e3) / 1e9
    if "generated_tokens" in shape:
        shape["tokens_per_s"] = shape["generated_tokens"] / (ms / 1e3)
    print(json.dumps({"op": a.op, **shape, "us": ms * 1e3, "tflops": tf,
                      "frac_of_measured_bf16_burst": (tf / peak) if (peak and tf) else None}))


if __name__ == "__main__":
    main()

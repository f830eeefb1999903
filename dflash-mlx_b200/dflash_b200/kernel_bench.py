"""Per-kernel roofline measurements of the hot-path kernels at the benchmark configurations' shapes.

    python -m dflash_b200.kernel_bench [--only gdr,attn,gemm] [--iters N]

Prints one JSON line per case: the kernel, the workload, the algorithmic bytes
(or FLOPs) one launch must move, the CUDA-event time per launch (mean over
``iters`` launches after warm-up, L2 flushed between launches by reading a
256 MB buffer, which leaves the cache full of clean lines) and the fraction of the measured peak (MEASURED_PEAKS.json at the
repository root; the profiling fallback 6650 GB/s / 1590 TFLOP/s when absent).

Cases (synthetic inputs, shapes and distributions of the benchmark configurations):
  gdr_t16     gated-delta recurrence, B=1, T=16, 16 QK / 32 V heads of 128, with
              per-token snapshots (config 2): bytes = state in + q,k,v,g,beta + o +
              T snapshots (the last one is the final state)
  gdr_t64     (only when named) T=64 with snapshots: 134 MB of snapshots, more than the
              126 MB L2, so a profile attributes the snapshot writes to DRAM (at T=16 they
              stay in L2 until after the kernel)
  gdr_t4096   the same over T=4096 without snapshots (final state only); a
              sequential recurrence, reported against both roofs
  attn_c3     verify attention, 1 sequence x 16 rows, Qwen3-4B heads, context 1536
  attn_c4     batched verify attention, 64 sequences x 16 rows, contexts U[512, 4096]
  gemm_c4     verify GEMMs at 1024 rows (64 sequences x 16): QKV, O, gate/up, down, lm_head
              (wide form; "gemm_streaming" runs the M <= 16 form on the same shapes)
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from . import ops

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks() -> tuple[float, float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Timer:
    """CUDA-event time of ``fn`` per launch with an L2 flush before each launch. ``fn``
    is captured once as a CUDA graph so that the timed region holds the kernels only,
    not the host-side argument checks of the Python wrappers."""

    def __init__(self, iters: int, warmup: int = 3):
        self.iters, self.warmup = iters, warmup
        self.flush = torch.ones(128 << 20, dtype=torch.float16, device="cuda")

    def __call__(self, fn) -> float:
        for _ in range(self.warmup):
            fn()
        torch.cuda.synchronize()
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(st):
            with torch.cuda.graph(graph, stream=st):
                fn()
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(self.iters):
            self.flush.sum()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            graph.replay()
            e.record()
            torch.cuda.synchronize()
            total += s.elapsed_time(e)
        return total / self.iters * 1e-3  # seconds per launch


def _line(case, what, seconds, bytes_=None, flops=None, extra=None):
    hbm, tf, kind = peaks()
    out = {"case": case, "kernel": what, "us": round(seconds * 1e6, 2)}
    if bytes_ is not None:
        gbs = bytes_ / seconds / 1e9
        out.update({"alg_bytes": int(bytes_), "achieved_gbs": round(gbs, 1), "hbm_peak_gbs": hbm,
                    "hbm_frac": round(gbs / hbm, 3)})
    if flops is not None:
        t = flops / seconds / 1e12
        out.update({"alg_flops": int(flops), "achieved_tflops": round(t, 1), "tensor_peak_tflops": tf,
                    "tensor_frac": round(t / tf, 3)})
    out["peak_kind"] = kind
    if extra:
        out.update(extra)
    print(json.dumps(out), flush=True)
    return out


def bench_gdr(timer: Timer, T: int, snapshots: bool):
    """Config 2 (seed 1): q,k ~ N(0,1) then L2-normalised, v ~ N(0,1), g = exp(-softplus(N)),
    beta = sigmoid(N), S0 ~ N(0, 0.01)."""
    B, Hk, Hv, D = 1, 16, 32, 128
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, device="cuda", generator=g), dim=-1).bfloat16()
    k = torch.nn.functional.normalize(torch.randn(B, T, Hk, D, device="cuda", generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, Hv, D, device="cuda", generator=g).bfloat16()
    alpha = torch.exp(-torch.nn.functional.softplus(torch.randn(B, T, Hv, device="cuda", generator=g)))
    beta = torch.sigmoid(torch.randn(B, T, Hv, device="cuda", generator=g))
    S0 = torch.randn(B, Hv, D, D, device="cuda", generator=g) * 0.01
    out = torch.empty_like(S0)
    snaps = torch.empty((B, T, Hv, D, D), device="cuda") if snapshots else None
    o = torch.empty((B, T, Hv, D), dtype=torch.bfloat16, device="cuda")

    def run():
        ops.gdr_recurrence(q, k, v, alpha, beta, S0, state_out=None if snapshots else out, snapshots=snaps, o=o)

    sec = timer(run)
    S = B * Hv * D * D * 4
    io = (q.numel() + k.numel() + v.numel() + o.numel()) * 2 + (alpha.numel() + beta.numel()) * 4
    by = S + io + (B * T * Hv * D * D * 4 if snapshots else S)
    flops = 7.0 * D * D * Hv * T * B
    return _line(f"gdr_t{T}", "gdr_kernel", sec, bytes_=by,
                 extra={"fp32_flops": int(flops), "snapshots": snapshots,
                        "workload": f"B=1 T={T} Hk=16 Hv=32 D=128"})


def bench_attention(timer: Timer, B: int, rows: int, ctxs: list[int], case: str, key_chunk: int = 0):
    Hq, Hkv, hd = 32, 8, 128
    cap = max(ctxs) + rows
    gen = torch.Generator(device="cuda").manual_seed(3)
    kc = torch.randn((B, Hkv, cap, hd), device="cuda", generator=gen).bfloat16()
    vc = torch.randn((B, Hkv, cap, hd), device="cuda", generator=gen).bfloat16()
    M = B * rows
    q = torch.randn((M, Hq, hd), device="cuda", generator=gen).bfloat16()
    pos = torch.tensor([c + i for c in ctxs for i in range(rows)], dtype=torch.int32, device="cuda")
    row_seq = (torch.arange(M, dtype=torch.int32, device="cuda") // rows) if B > 1 else None
    out = torch.empty((M, Hq * hd), dtype=torch.bfloat16, device="cuda")
    ws = ops.Workspace(torch.device("cuda"))

    def run():
        ops.attention(q, kc, vc, pos, True, max_kv=cap, row_seq=row_seq, out=out, ws=ws, seq_rows=rows,
                      key_chunk=key_chunk)

    sec = timer(run)
    kv = sum(c + rows for c in ctxs) * Hkv * hd * 2 * 2
    by = kv + q.numel() * 2 + out.numel() * 2
    return _line(case, "attn_chunk_kernel+attn_combine_kernel", sec, bytes_=by,
                 extra={"workload": f"B={B} rows={rows} Hq={Hq} Hkv={Hkv} hd={hd} ctx mean "
                                    f"{sum(ctxs) / len(ctxs):.0f}", "kv_bytes": int(kv),
                        "key_chunk": key_chunk or 128})


def bench_gemm_c4(timer: Timer, M: int = 1024, wide: bool = True, wide_split: int = 1):
    """The verify GEMMs at C4's 1024 rows; wide=True is the whole-K tile form batched
    sessions use, wide=False the M <= 16 weight-streaming form for comparison."""
    H, I, Hq, Hkv, hd = 2560, 9728, 32, 8, 128
    gen = torch.Generator(device="cuda").manual_seed(3)
    res = []
    kern = "gemm_wide_kernel" if wide else "gemm_tc_kernel"
    for name, N, K in (("qkv", (Hq + 2 * Hkv) * hd, H), ("o", H, Hq * hd), ("gate_up", 2 * I, H), ("down", H, I),
                       ("lm_head", 151936, H)):
        w = ops.pack_weight((torch.randn((N, K), device="cuda", generator=gen) * 0.02).bfloat16())
        x = torch.randn((M, K), device="cuda", generator=gen).bfloat16()
        y = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        ws = ops.Workspace(torch.device("cuda"), wide=wide, wide_split=wide_split)
        sec = timer(lambda: ops.gemm(x, w, out=y, ws=ws))
        res.append(_line(f"gemm_c4_{name}" + ("" if wide else "_streaming"), kern, sec,
                         bytes_=N * K * 2 + M * K * 2 + M * N * 2, flops=2.0 * M * N * K,
                         extra={"workload": f"M={M} N={N} K={K}",
                                "k_split": ops.wide_split(N, K, ws) if wide else None}))
        del w, x, y
    return res


def bench_verify_gemms(timer: Timer, M: int = 1024, wide: bool = True):
    """The verify forward's own GEMM launches (fused RMSNorm prologues, residual / tap /
    SiLU·up / argmax epilogues) for one Qwen3-4B layer plus the lm_head, at M rows."""
    from .config import TargetConfig
    from .model import TargetModel
    from .weights import random_target_weights
    cfg = TargetConfig(num_hidden_layers=1)
    target = TargetModel(cfg, random_target_weights(cfg, 3, device="cuda"), "cuda")
    ws = ops.Workspace(torch.device("cuda"), wide=wide)
    b = target.buffers(M)
    b["h"].normal_()
    b["attn"].normal_()
    b["act"].normal_()
    b["ss"].fill_(float(cfg.hidden_size))
    names = ["qkv+norm", "o+residual", "gate_up+norm+silu", "down+residual", "lm_head+norm+argmax"]
    out = []
    for (fn, by, fl), name in zip(target.verify_gemms(M, ws=ws), names):
        sec = timer(fn)
        out.append(_line(f"verify_{name}", "gemm_wide_kernel" if wide else "gemm_tc_kernel", sec, bytes_=by,
                         flops=fl, extra={"workload": f"M={M}"}))
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gdr,attn,gemm")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--key-chunk", type=int, default=0, help="attn_c3 / attn_c4: one key chunk instead of the sweep")
    ap.add_argument("--wide-split", type=int, default=1, help="gemm: most K ranges of a wide GEMM (session limit)")
    args = ap.parse_args(argv)
    sel = set(args.only.split(","))
    timer = Timer(args.iters, args.warmup)
    if sel & {"gdr", "gdr_t16"}:
        bench_gdr(timer, 16, True)
    if "gdr_t64" in sel:  # snapshots (134 MB) larger than L2: the capture attributes their DRAM writes
        bench_gdr(timer, 64, True)
    if sel & {"gdr", "gdr_t4096"}:
        bench_gdr(timer, 4096, False)
    if sel & {"attn", "attn_c3"}:
        for kc in ([args.key_chunk] if args.key_chunk else (128, 256, 512)):
            bench_attention(timer, 1, 16, [1536], "attn_c3", key_chunk=kc)
    if sel & {"attn", "attn_c4"}:
        g = torch.Generator().manual_seed(3)
        ctxs = torch.randint(512, 4097, (64,), generator=g).tolist()
        for kc in ([args.key_chunk] if args.key_chunk else (128, 512, 1024, 4224)):
            bench_attention(timer, 64, 16, ctxs, "attn_c4", key_chunk=kc)
    if "gemm" in sel:
        bench_gemm_c4(timer, wide_split=args.wide_split)
    if "verify" in sel:
        bench_verify_gemms(timer)
    if "gemm_streaming" in sel:
        bench_gemm_c4(timer, wide=False)


if __name__ == "__main__":
    main()

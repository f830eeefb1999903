"""Phase timeline of one weight-streaming GEMM launch (the cluster split-K kernel) at the
Qwen3-4B verify shapes, M = 16 rows.

    python dflash-mlx_b200/dflash_b200/_build.py --trace
    DFLASH_B200_LIB=dflash-mlx_b200/dflash_b200/libdflash_b200_trace.so \\
        python -m dflash_b200.gemm_trace qkv      # or o, gate_up, down

Needs the diagnostic build (-DDFL_TC_TRACE): every CTA records %globaltimer at fixed
points of the kernel. One JSON line per call: the launch time alone and per launch in a
chain of 8 (CUDA events), and per phase [max, median, min] over the CTAs, in us after the
first CTA started:
  p0 start  p1 setup done  p2 producer past the dependency wait  p3 first stage in
  p4 last MMA issued  p5 accumulator ready  p6/p7 before/after the pre-push cluster wait
  p8/p9 before/after the exit cluster wait  p10/p11 owner: pushes received
  p12/p13 owner: rank sum done  p14/p15 owner: epilogue stores issued
One shape per process: the timestamp table is not cleared between launches.
"""
from __future__ import annotations

import ctypes
import json
import sys

import torch

from . import _lib, ops

SHAPES = {"qkv": (6144, 2560, 0), "o": (2560, 4096, 1), "gate_up": (19456, 2560, 2), "down": (2560, 9728, 1)}


def main(argv=None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    name = argv[0] if argv else "o"
    N, K, epi = SHAPES[name]
    lib = _lib.load()
    if not hasattr(lib, "dfl_debug_tc_trace"):
        raise SystemExit("not a trace build: build with `_build.py --trace` and set DFLASH_B200_LIB")
    dev, M = "cuda", 16
    g = torch.Generator(device=dev).manual_seed(0)
    ws = ops.Workspace(torch.device(dev))
    weights = [ops.pack_weight((torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()) for _ in range(8)]
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    y = torch.zeros(M, N // 2 if epi == 2 else N, device=dev, dtype=torch.bfloat16)

    def run(w):
        if epi == 1:
            ops.gemm(x, w, 1, residual=y, out=y, ws=ws)
        else:
            ops.gemm(x, w, epi, out=y, ws=ws)

    for _ in range(3):
        for w in weights:
            run(w)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(200000)
    e0.record()
    for w in weights:
        run(w)
    e1.record()
    torch.cuda.synchronize()
    chain = e0.elapsed_time(e1) * 1000 / len(weights)
    torch.cuda._sleep(200000)
    e0.record()
    run(weights[0])
    e1.record()
    torch.cuda.synchronize()
    alone = e0.elapsed_time(e1) * 1000
    torch.cuda._sleep(1000000)
    run(weights[1])
    torch.cuda.synchronize()
    buf = (ctypes.c_ulonglong * (8192 * 16))()
    lib.dfl_debug_tc_trace(buf, 8192)
    t = torch.tensor(list(buf), dtype=torch.float64).reshape(8192, 16)
    t = t[t[:, 0] > 0]
    t0 = t[:, 0].min()
    t[t == 0] = float("nan")
    rel = (t - t0) / 1000.0

    def q(k):
        col = rel[:, k]
        if torch.isnan(col).all():
            return None
        return [round(float(col.nan_to_num(-1).max()), 2), round(float(col.nanmedian()), 2),
                round(float(col.nan_to_num(1e9).min()), 2)]

    out = {"gemm": name, "N": N, "K": K, "ctas": int(t.shape[0]), "alone_us": round(alone, 2),
           "chain_us": round(chain, 2)}
    out.update({f"p{k}": q(k) for k in range(16) if q(k) is not None})
    print(json.dumps(out))


if __name__ == "__main__":
    main()

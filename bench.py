#!/usr/bin/env python
"""Benchmark: accepted tokens/s of DFlash speculative decoding at the Qwen3-4B shape.

Workload (benchmark config 3): Qwen3-4B-shaped bf16 random-init target (36 layers,
hidden 2560, 32 q / 8 kv heads of 128, FFN 9728, vocab 151936) and a 5-layer DFlash
draft (block 16, 5 taps), one stream per GPU, 512-token random prompt, seed 2.
Drafts are oracle-injected: the block carries the target's own greedy tokens for a
prefix whose acceptance length is Geometric with mean 6.5 capped at 16, then random
tokens. A step = one speculative step (draft forward + 16-token verify + accept).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c3|c4]

N > 1 runs N independent replicas (one process per GPU under torchrun, no
collective on the data path: weak scaling). Rank 0 prints one JSON line.

--workload c4 (benchmark config 4, not the default line): 64 sequences per GPU with
contexts U[512, 4096] (seed 3), block 16, per-sequence oracle-injected acceptance
(tau 6.5) and rollback, decoded together in one batched step per GPU.

--workload c5 (benchmark config 5): Qwen3.5-27B-shaped hybrid target (64 layers) with a
5-layer DFlash draft, tensor-parallel over the N ranks (N = 1, 2, 4 or 8), batch 8,
context --ctx (default 32768), block 16, oracle-injected acceptance tau 4.0 (seed 4).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "dflash-mlx_b200"))

import torch  # noqa: E402

METRIC = "accepted tokens/sec/GPU at Qwen3-4B shape (block 16, tau=6.5); p50 verify-step us"
UNIT = "accepted tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=150)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--tau", type=float, default=6.5)
    ap.add_argument("--seed", type=int, default=2)
    ap.add_argument("--layers", type=int, default=36, help="target depth (36 = the Qwen3-4B shape)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-steps", type=int, default=3, help="speculative steps in the CPU baseline sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--workload", choices=["c3", "c4", "c5"], default="c3")
    ap.add_argument("--mid-context", type=int, default=1024,
                    help="c3: untimed steps first advance the context so that the timed steps centre on this "
                         "context (config 3: prompt 512 + 1024 new tokens, mean context 1024)")
    ap.add_argument("--batch", type=int, default=0, help="c4: sequences per GPU (64); c5: sequences (8)")
    ap.add_argument("--ctx", type=int, default=32768, help="c5: prompt length of every sequence")
    ap.add_argument("--ncu-region", action="store_true",
                    help="bracket the timed steps with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
def draft_taps(layers: int) -> list[int]:
    """The draft's tap layers: five evenly spaced ones at full depth, else the first and the
    last (distinct) for the shallow profiling targets."""
    from dflash_b200.config import evenly_spaced_layers
    return evenly_spaced_layers(layers, 5) if layers >= 8 else sorted({0, layers - 1} if layers < 3 else {1, layers - 1})


def geometric_p(tau: float, cap: int) -> float:
    """p with E[min(G, cap)] = tau for G ~ Geometric(p) on {1, 2, ...}."""
    lo, hi = 1e-6, 1.0
    for _ in range(200):
        p = 0.5 * (lo + hi)
        mean = (1 - (1 - p) ** cap) / p
        if mean > tau:
            lo = p
        else:
            hi = p
    return 0.5 * (lo + hi)


def injection_plan(n_steps: int, bs: int, tau: float, vocab: int, seed: int):
    """Per step: number of leading drafted tokens taken from the greedy trace
    (acceptance length - 1) and the random tokens that fill the rest of the block."""
    g = torch.Generator().manual_seed(seed + 1000)
    p = geometric_p(tau, bs)
    u = torch.rand(n_steps, generator=g, dtype=torch.float64)
    acc = torch.clamp(torch.floor(torch.log1p(-u) / math.log1p(-p)) + 1, max=bs).to(torch.int32)
    noise = torch.randint(0, vocab, (n_steps, bs), generator=g, dtype=torch.int32)
    return acc - 1, noise


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        loaded = [x for x in sm if x > 500] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "samples": len(sm), "reasons": sorted(reasons)}


def measured_peaks() -> tuple[float, float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
def build_models(args, device):
    from dflash_b200.config import DraftConfig, TargetConfig
    from dflash_b200.model import DraftModel, TargetModel
    from dflash_b200.weights import random_draft_weights, random_target_weights
    tcfg = TargetConfig(num_hidden_layers=args.layers)
    dcfg = DraftConfig(target_layer_ids=draft_taps(args.layers))
    tw = random_target_weights(tcfg, args.seed, device=device)
    dw = random_draft_weights(dcfg, args.seed, device=device)
    target = TargetModel(tcfg, tw, device)
    draft = DraftModel(dcfg, dw, target)
    return tcfg, dcfg, tw, dw, target, draft


def greedy_trace(target, prompt, n_new):
    """The target's own greedy continuation (plain decode: block of 1 through the same kernels)."""
    from dflash_b200.runtime import SpecSession
    sess = SpecSession(target, None, 1, len(prompt) + n_new, 1, set(), use_graph=True)
    sess.prefill([prompt], n_new)
    sess.run(n_new + 2)
    return sess.outputs()[0][0]


def gemm_roofline(sess, reps: int = 3) -> dict:
    """Times the verify step's weight-streaming GEMM launches alone (same shapes, weights and
    activation buffers as the step; 8 GB of weights per pass, far above the 126 MB L2)."""
    M = sess.B * sess.bs
    from dflash_b200.model import chain_ok
    use_chain = getattr(sess.target, "use_chain", False) and chain_ok(M, sess.ws)
    launches = (sess.target.verify_chains(M, ws=sess.ws) if use_chain
                else sess.target.verify_gemms(M, ws=sess.ws))
    total_bytes = sum(nb for _, nb, _ in launches)
    total_flops = sum(f for _, _, f in launches)

    def run_all():
        for fn, _, _ in launches:
            fn()

    run_all()  # eager once (tensor maps, function attributes), then replay as a CUDA graph
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            run_all()
    torch.cuda.current_stream().wait_stream(st)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    times = []
    for _ in range(reps):
        torch.cuda.synchronize()
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e-3)
    t_pass = min(times)
    per_launch_s = t_pass / len(launches)
    per_launch_bytes = total_bytes / len(launches)
    return {"launches": len(launches), "chain": use_chain, "bytes_per_pass": total_bytes, "s_per_pass": t_pass,
            "per_launch_s": per_launch_s, "per_launch_bytes": per_launch_bytes,
            "achieved_gbs": per_launch_bytes / per_launch_s / 1e9,
            "per_launch_flops": total_flops / len(launches),
            "achieved_tflops": total_flops / t_pass / 1e12}


def cpu_sample(tcfg, dcfg, tw, dw, sess, trace, lengths, noise, n_steps: int) -> dict:
    """Times the CPU oracle (the restated reference algorithm) on a bounded sample of the same
    workload: ``n_steps`` speculative steps from the GPU run's post-prefill state."""
    from oracle import dflash_oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cpu_w = lambda w: _fp32_weights({k: (v.cpu() if torch.is_tensor(v) else  # noqa: E731
                                         [{kk: vv.cpu() for kk, vv in l.items()} for l in v]) for k, v in w.items()})
    ot = O.OracleTarget(tcfg, cpu_w(tw))
    od = O.OracleDraft(dcfg, cpu_w(dw), ot)
    P = int(sess.state[0, 9].item())
    # oracle caches from the GPU prefill (positions [0, P))
    tcache = ot.make_cache(P + 16 * (n_steps + 2))
    for l, c in enumerate(tcache):
        k, v = sess.tcache.gather(l, 0, P)
        c.k[:, :P], c.v[:, :P] = k.float().cpu(), v.float().cpu()
        c.offset = P
    dcache = od.make_cache(P + 16 * (n_steps + 2))
    for l, c in enumerate(dcache):
        k, v = sess.dcache.gather(l, 0, P)
        c.k[:, :P], c.v[:, :P] = k.float().cpu(), v.float().cpu()
        c.offset = P
    bs = dcfg.block_size
    hidden = torch.zeros((0, len(dcfg.target_layer_ids) * tcfg.hidden_size))
    start = P
    out = list(trace[:P + 1])
    accepted = 0
    t0 = time.perf_counter()
    for s in range(n_steps):
        block = [out[start]] + [dcfg.mask_token_id] * (bs - 1)
        dh = od(ot.embed_tokens(block), hidden, dcache)
        O.argmax_first(ot.lm_head_logits(dh[1:]))
        for c in dcache:
            c.trim(bs)
        L = int(lengths[s])
        for i in range(1, bs):
            block[i] = trace[start + i] if i - 1 < L else int(noise[s, i])
        logits, hid = ot.forward_with_hidden_states(block, tcache, dcfg.target_layer_ids)
        post = O.argmax_first(logits).tolist()
        m = O.longest_prefix_match(block[1:], post[:-1])
        acc = m + 1
        for c in tcache:
            c.trim(bs - acc)
        hidden = hid[:acc]
        out = out[:start] + block[:acc] + [post[m]]
        start += acc
        accepted += acc
    dt = time.perf_counter() - t0
    return {"value": accepted / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n_steps} speculative steps (draft + 16-token verify + accept) of the config-3 workload "
                      f"from context {P}, CPU oracle restatement, {dt:.1f} s"}


def _fp32_weights(w: dict) -> dict:
    """The same (bf16-valued) weights held as fp32: the oracle computes in fp32, so this
    saves a conversion per projection call."""
    f = lambda t: t.float() if torch.is_tensor(t) and t.is_floating_point() else t  # noqa: E731
    out = {k: f(v) for k, v in w.items() if k != "layers"}
    out["layers"] = [{k: f(v) for k, v in lw.items()} for lw in w["layers"]]
    return out


def run_reference(args, world: int, rank: int) -> None:
    """The reference arm: the reference's algorithm for this path (the oracle restatement,
    pinned to the reference's own runtime / draft / adapters by golden fixtures; MLX itself
    does not install here) timed on the host cores. It touches no GPU and loads no library
    of this repository: weights, prefill, the greedy trace behind the injected drafts and
    the timed steps are all computed by the oracle on the CPU. Rank 0 alone runs it."""
    if rank != 0:
        return
    from oracle import dflash_oracle as O
    from dflash_b200.config import DraftConfig, TargetConfig
    from dflash_b200.weights import random_draft_weights, random_target_weights
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    t_setup = time.perf_counter()
    tcfg = TargetConfig(num_hidden_layers=args.layers)
    dcfg = DraftConfig(target_layer_ids=draft_taps(args.layers))
    tw = _fp32_weights(random_target_weights(tcfg, args.seed))
    dw = _fp32_weights(random_draft_weights(dcfg, args.seed))
    ot = O.OracleTarget(tcfg, tw)
    od = O.OracleDraft(dcfg, dw, ot)
    bs = dcfg.block_size
    n_steps = max(1, min(args.steps, args.cpu_steps))
    n_warm = max(0, min(args.warmup, args.cpu_steps))  # untimed steps first, as the GPU arm
    total = n_warm + n_steps
    lengths, noise = injection_plan(total + 4, bs, args.tau, tcfg.vocab_size, args.seed)
    g = torch.Generator().manual_seed(args.seed)
    prompt = torch.randint(0, tcfg.vocab_size, (args.prompt_len,), generator=g).tolist()
    P = len(prompt)
    cap = P + bs * (total + 4)
    tcache, dcache = ot.make_cache(cap), od.make_cache(cap)
    logits, hidden = ot.forward_with_hidden_states(prompt, tcache, dcfg.target_layer_ids)
    out = prompt + [int(O.argmax_first(logits[-1]))]
    # the target's greedy continuation, far enough for every injected prefix (untimed)
    need = P + 1 + sum(int(x) + 1 for x in lengths[:total]) + bs
    gcache = ot.make_cache(need + 1)
    for c, src in zip(gcache, tcache):
        c.k[:, :P] = src.k[:, :P]
        c.v[:, :P] = src.v[:, :P]
        c.offset = P
    trace = list(out)
    while len(trace) < need:
        lg, _ = ot.forward_with_hidden_states([trace[-1]], gcache, [])
        trace.append(int(O.argmax_first(lg[-1])))
    del gcache
    setup_s = time.perf_counter() - t_setup
    start, accepted = P, 0
    t0 = time.perf_counter()
    for s in range(total):
        if s == n_warm:  # the timed steps start here
            t0, accepted = time.perf_counter(), 0
        block = [out[start]] + [dcfg.mask_token_id] * (bs - 1)
        dh = od(ot.embed_tokens(block), hidden, dcache)
        O.argmax_first(ot.lm_head_logits(dh[1:]))
        for c in dcache:
            c.trim(bs)
        L = int(lengths[s])
        for i in range(1, bs):
            block[i] = trace[start + i] if i - 1 < L else int(noise[s, i])
        lg, hid = ot.forward_with_hidden_states(block, tcache, dcfg.target_layer_ids)
        post = O.argmax_first(lg).tolist()
        m = O.longest_prefix_match(block[1:], post[:-1])
        acc = m + 1
        for c in tcache:
            c.trim(bs - acc)
        hidden = hid[:acc]
        out = out[:start] + block[:acc] + [post[m]]
        start += acc
        accepted += acc
    dt = time.perf_counter() - t0
    value = accepted / dt
    sample = (f"{n_steps} speculative steps (draft + 16-token verify + accept) of the config-3 workload after "
              f"{n_warm} untimed ones from context {P}, {dt:.1f} s timed ({setup_s:.0f} s untimed set-up: seeded "
              f"weights, prefill and the greedy trace behind the injected drafts, all on the CPU)")
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": n_steps,
            "warmup": n_warm, "ms_per_step": dt / n_steps * 1e3, "higher_is_better": True, "impl": "reference",
            "scaling": "weak", "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt, oracle-injected drafts)",
            "config": {"workload": f"config3: Qwen3-4B-shaped target ({args.layers} layers) + 5-layer DFlash draft, "
                                   f"block 16, prompt {args.prompt_len}, oracle-injected acceptance tau {args.tau}",
                       "global_batch": 1, "seq_len": args.prompt_len, "parallelism": "cpu (host cores)",
                       "target_layers": args.layers},
            "tau_measured": accepted / n_steps,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "vs_baseline": None, "gpu_launches": 0,
            "note": "MLX (the reference's array library) has no wheel here, so the reference itself cannot run; "
                    "its algorithm is timed as restated in oracle/dflash_oracle.py (bf16 storage, fp32 math), "
                    "which golden fixtures pin to the reference's own runtime.py, draft.py and adapters.py"}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":  # CPU only: no process group, no device, no library of ours
        return run_reference(args, world, rank)
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    device = torch.device("cuda", local if torch.cuda.is_available() else 0)
    torch.cuda.set_device(device)

    from dflash_b200 import _lib
    from dflash_b200.runtime import SpecSession, S_START

    _lib.load()
    if args.workload == "c4":
        return run_c4(args, world, rank, device)
    if args.workload == "c5":
        return run_c5(args, world, rank, device)
    tcfg, dcfg, tw, dw, target, draft = build_models(args, device)
    bs = dcfg.block_size
    g = torch.Generator().manual_seed(args.seed + rank)
    prompt = torch.randint(0, tcfg.vocab_size, (args.prompt_len,), generator=g).tolist()
    # untimed steps before the timed ones: the warm-up, or more, so that the timed steps sit
    # around the configuration's mean context instead of at the prompt's end
    pre = max(args.warmup, int(max(0.0, args.mid_context - args.prompt_len - args.steps * args.tau / 2) / args.tau))
    total_steps = pre + args.steps
    n_new = bs * (total_steps + 2)
    trace = greedy_trace(target, prompt, n_new + 2 * bs)
    trace_t = torch.zeros(len(prompt) + n_new + 4 * bs, dtype=torch.int32)
    trace_t[:len(trace)] = torch.tensor(trace, dtype=torch.int32)
    lengths, noise = injection_plan(total_steps + 4, bs, args.tau, tcfg.vocab_size, args.seed + rank)

    def new_session():
        sess = SpecSession(target, draft, 1, len(prompt) + n_new, bs, set(), use_graph=True,
                           max_steps=total_steps + 8)
        sess.set_injection(trace_t[None], lengths[None], noise.reshape(1, -1))
        sess.prefill([prompt], n_new)
        return sess

    # ---------------- our arm: device-timed value ----------------
    sess = new_session()
    for _ in range(pre):
        sess.step()
    torch.cuda.synchronize()
    ctx_start = int(sess.state[0, S_START].item())
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start_before = int(sess.state[0, S_START].item())
    if args.ncu_region:
        torch.cuda.profiler.start()
    t_start.record()
    for k in range(args.steps):
        sess.step(events=evs[k])
    t_end.record()
    torch.cuda.synchronize()
    if args.ncu_region:
        torch.cuda.profiler.stop()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    elapsed = t_start.elapsed_time(t_end) * 1e-3
    log = sess.accept_log[0].cpu()
    accepted = int(log[pre:pre + args.steps].sum())
    tau_real = accepted / args.steps
    verify_us = sorted(evs[k][1].elapsed_time(evs[k][2]) * 1e3 for k in range(args.steps))
    draft_us = sorted(evs[k][0].elapsed_time(evs[k][1]) * 1e3 for k in range(args.steps))
    ctx_end = int(sess.state[0, S_START].item())
    if world > 1:
        t = torch.tensor([elapsed, float(accepted)], dtype=torch.float64, device=device)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        elapsed_max, total_acc = float(tmax[0]), float(t[1])
    else:
        elapsed_max, total_acc = elapsed, float(accepted)
    value = total_acc / elapsed_max

    # ---------------- e2e: public run loop, host copies every step ----------------
    e2e = None
    if not args.no_e2e:
        sess2 = new_session()
        for _ in range(pre):
            sess2.step()
        torch.cuda.synchronize()
        # per step the host supplies that step's draft record (injected-prefix length and
        # filler tokens) from pinned memory; the device copy the kernels read is overwritten
        inj_host = torch.cat([lengths[:, None], noise], 1).contiguous().pin_memory()
        h2d = inj_host.shape[1] * 4

        def before_step(k):
            row = inj_host[k]
            sess2.inject_len[0, k:k + 1].copy_(row[:1], non_blocking=True)
            sess2.inject_noise[0, k * bs:(k + 1) * bs].copy_(row[1:], non_blocking=True)

        t0 = time.perf_counter()
        for _ in sess2.run_iter(args.steps, copy_tokens=True, before_step=before_step, first_index=pre):
            pass
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        acc2 = int(sess2.accept_log[0, pre:pre + args.steps].sum())
        d2h = sess2.state.numel() * 4 + sess2.out_tokens.numel() * 4
        e2e = {"value": acc2 / dt, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "path": "SpecSession.run_iter (the loop behind dflash_generate_stream): per step a pinned H2D "
                       "copy of the step's draft record and pinned D2H copies of the state and token row"}
        del sess2

    # ---------------- roofline of the dominant kernel ----------------
    hbm_peak, _, peak_kind = measured_peaks()
    roof = None
    if not args.no_roofline:
        r = gemm_roofline(sess)
        # DRAM bytes per launch from one ncu capture of the same kernel (profiles/), scaled to
        # this pass's average launch by the algorithmic bytes
        traffic = None
        tp = os.path.join(ROOT, "profiles", "gemm_chain_traffic.json" if r["chain"] else "gemm_stream_traffic.json")
        if os.path.exists(tp):
            try:
                t = json.load(open(tp))
                if r["chain"]:
                    traffic = int(t["dram_bytes"] / t["alg_bytes"] * r["per_launch_bytes"])
                else:
                    traffic = t.get("dram_bytes_per_launch_full")
            except Exception:
                traffic = None
        kern = ("gemm_chain_kernel (the verify forward's projections as one launch per run between two attention "
                f"calls, M=16; per-launch average over the {r['launches']}-launch verify pass)" if r["chain"] else
                "gemm_csk_kernel + gemm_tc_kernel (verify weight streaming, M=16; per-launch average over the "
                f"{r['launches']}-launch verify pass)")
        roof = {"bound": "hbm", "kernel": kern,
                "achieved": round(r["achieved_gbs"], 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(r["achieved_gbs"] / hbm_peak, 4), "traffic": traffic,
                "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                "algorithmic_bytes_per_launch": int(r["per_launch_bytes"]), "launches_per_pass": r["launches"],
                "us_per_launch": round(r["per_launch_s"] * 1e6, 2),
                "verify_gemm_pass_ms": round(r["s_per_pass"] * 1e3, 3)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            sess3 = new_session()
            torch.cuda.synchronize()
            cpu = cpu_sample(tcfg, dcfg, tw, dw, sess3, trace, lengths, noise, args.cpu_steps)
        except Exception as exc:  # report, do not fail the bench line
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {exc}"}

    # launches of our kernels per timed step (one verify + one draft)
    n_layers_t, n_layers_d = tcfg.num_hidden_layers, dcfg.num_hidden_layers
    q = _lib.query
    att_t = int(q("dfl_attention_launches", tcfg.num_attention_heads, tcfg.num_key_value_heads, tcfg.head_dim,
                  sess.cap, sess.key_chunk))
    att_d = int(q("dfl_attention_launches", dcfg.num_attention_heads, dcfg.num_key_value_heads, dcfg.head_dim,
                  sess.cap, sess.key_chunk))
    # per layer: qkv gemm (+norm) and q/k norm+rope+append (1 launch fused, else 2), attention (1 or 2),
    # o gemm, gu gemm (+norm), down
    from dflash_b200.model import qkv_rope_ok
    rows = sess.B * sess.bs

    def qkv_launches(c):
        if not qkv_rope_ok(sess.ws, c.head_dim, getattr(c, "rope_dim", c.head_dim)):
            return 2
        return int(q("dfl_gemm_qkv_rope_launches", rows, c.hidden_size, c.num_attention_heads,
                     c.num_key_value_heads, c.head_dim))
    qkv_t, qkv_d = qkv_launches(tcfg), qkv_launches(dcfg)
    # draft context rows: fc, then the stacked K/V projection with every layer's append fused
    # (one launch) or followed by one append launch per layer
    ingest_fused = qkv_rope_ok(sess.ws, dcfg.head_dim, dcfg.head_dim) and int(q(
        "dfl_gemm_qkv_rope_launches", rows, dcfg.hidden_size, 0, n_layers_d * dcfg.num_key_value_heads,
        dcfg.head_dim)) == 1
    ingest = 2 + (0 if ingest_fused else n_layers_d)
    draft_launches = 1 + ingest + 1 + (3 + qkv_d + att_d) * n_layers_d + 1 + 1
    verify_launches = 1 + (3 + qkv_t + att_t) * n_layers_t + 1 + 1
    launches_step = draft_launches + verify_launches
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_max / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompt, oracle-injected drafts)",
            "config": {"workload": "config3: Qwen3-4B-shaped target (36 layers) + 5-layer DFlash draft, block 16, "
                                   f"prompt {args.prompt_len}, oracle-injected acceptance tau {args.tau}",
                       "global_batch": world, "seq_len": args.prompt_len, "parallelism": f"replicas x{world}",
                       "l2": "working set per step ~9.9 GB of weights > 126 MB L2 (no flush needed)",
                       "target_layers": n_layers_t},
            "p50_verify_step_us": round(verify_us[len(verify_us) // 2], 1),
            "p50_draft_step_us": round(draft_us[len(draft_us) // 2], 1),
            "tau_measured": round(tau_real, 3), "context_start": ctx_start, "context_end": ctx_end,
            "untimed_steps_before": pre,
            "gpu_launches": launches_step * args.steps,
            "clocks": clk, "e2e": e2e, "roofline": roof, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_c4(args, world, rank, device):
    """Config 4: B sequences per GPU, contexts U[512, 4096], one batched step per GPU."""
    from dflash_b200.runtime import SpecSession
    if world > 1:
        import torch.distributed as dist
    tcfg, dcfg, tw, dw, target, draft = build_models(args, device)
    bs, B = dcfg.block_size, args.batch or 64
    seed = 3
    g = torch.Generator().manual_seed(seed + 7919 * rank)
    lens = torch.randint(512, 4097, (B,), generator=g).tolist()
    prompts = [torch.randint(0, tcfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    total_steps = args.warmup + args.steps
    n_new = bs * (total_steps + 2)
    # each sequence's own greedy continuation: plain decode of the same batch (same kernel forms)
    plain = SpecSession(target, None, B, max(lens) + n_new + 2 * bs, 1, set(), use_graph=True)
    plain.prefill(prompts, n_new + 2 * bs)
    plain.run(n_new + 2 * bs + 2)
    traces = plain.outputs()[0]
    del plain
    L = max(len(t) for t in traces) + 4 * bs
    trace_t = torch.zeros((B, L), dtype=torch.int32)
    for b, t in enumerate(traces):
        trace_t[b, :len(t)] = torch.tensor(t, dtype=torch.int32)
    lengths, noise = [], []
    for b in range(B):
        le, no = injection_plan(total_steps + 4, bs, args.tau, tcfg.vocab_size, seed * 1000 + b + 7919 * rank)
        lengths.append(le)
        noise.append(no.reshape(-1))
    lengths, noise = torch.stack(lengths), torch.stack(noise)
    sess = SpecSession(target, draft, B, max(lens) + n_new, bs, set(), use_graph=True, max_steps=total_steps + 8)
    sess.set_injection(trace_t, lengths, noise)
    sess.prefill(prompts, n_new)
    for _ in range(args.warmup):
        sess.step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for k in range(args.steps):
        sess.step(events=evs[k])
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    elapsed = t0.elapsed_time(t1) * 1e-3
    accepted = int(sess.accept_log[:, args.warmup:args.warmup + args.steps].sum())
    if world > 1:
        t = torch.tensor([elapsed, float(accepted)], dtype=torch.float64, device=device)
        tmax = t.clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        elapsed_max, total_acc = float(tmax[0]), float(t[1])
    else:
        elapsed_max, total_acc = elapsed, float(accepted)
    verify_us = sorted(evs[k][1].elapsed_time(evs[k][2]) * 1e3 for k in range(args.steps))
    draft_us = sorted(evs[k][0].elapsed_time(evs[k][1]) * 1e3 for k in range(args.steps))
    _, tf_peak, peak_kind = measured_peaks()
    r = gemm_roofline(sess)
    roof = {"bound": "tensor", "kernel": "gemm_wide_kernel (verify GEMMs at M = B x 16, average over the pass)",
            "achieved": round(r["achieved_tflops"], 1), "peak": tf_peak, "unit": "TFLOP/s",
            "frac": round(r["achieved_tflops"] / tf_peak, 4), "traffic": None, "peak_kind": peak_kind,
            "algorithmic_flops_per_launch": int(r["per_launch_flops"]), "launches_per_pass": r["launches"],
            "verify_gemm_pass_ms": round(r["s_per_pass"] * 1e3, 3)}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(total_acc / elapsed_max, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed_max / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompts, oracle-injected drafts)",
            "config": {"workload": f"config4: Qwen3-4B shape, {B} sequences per GPU, contexts U[512,4096], block 16, "
                                   f"oracle-injected acceptance tau {args.tau}, per-sequence rollback",
                       "global_batch": B * world, "seq_len": int(sum(lens) / len(lens)),
                       "parallelism": f"data-parallel x{world} (no collective)",
                       "l2": "working set per step ~9.9 GB of weights + ~20 GB KV > 126 MB L2"},
            "p50_verify_step_us": round(verify_us[len(verify_us) // 2], 1),
            "p50_draft_step_us": round(draft_us[len(draft_us) // 2], 1),
            "tau_measured": round(accepted / (args.steps * B), 3),
            "clocks": clk, "roofline": roof, "e2e": None, "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_c5(args, world, rank, device):
    """Config 5: the 27B hybrid, tensor-parallel over the ranks (every rank decodes the
    same batch; each holds 1 / N of every layer)."""
    from dflash_b200.config import qwen35_27b_pair
    from dflash_b200.hybrid import HybridTargetModel
    from dflash_b200.model import DraftModel
    from dflash_b200.runtime import SpecSession
    from dflash_b200.tp import TPComm, shard_config, shard_layer
    from dflash_b200.weights import random_draft_weights, random_target_weights
    if world > 1:
        import torch.distributed as dist
    n_layers = 64 if args.layers == 36 else args.layers
    tcfg, dcfg = qwen35_27b_pair(n_layers)
    bs, B, seed, tau = dcfg.block_size, args.batch or 8, 4, 4.0 if args.tau == 6.5 else args.tau
    comm = TPComm(rank, world, device, max_rows=max(128, B * bs), hidden=tcfg.hidden_size)
    w = random_target_weights(tcfg, seed, device="cuda", layer_hook=lambda i, lw: shard_layer(tcfg, i, lw, rank, world))
    target = HybridTargetModel(shard_config(tcfg, world), w, device, tp=comm)
    del w
    draft = DraftModel(dcfg, random_draft_weights(dcfg, seed, device="cuda"), target, mask_mode="causal")
    torch.cuda.empty_cache()
    g = torch.Generator().manual_seed(seed)  # the same prompts on every rank
    prompts = [torch.randint(0, tcfg.vocab_size, (args.ctx,), generator=g).tolist() for _ in range(B)]
    total_steps = args.warmup + args.steps
    n_new = bs * (total_steps + 2)
    plain = SpecSession(target, None, B, args.ctx + n_new + 2 * bs, 1, set(), use_graph=True)
    plain.prefill(prompts, n_new + 2 * bs)
    plain.run(n_new + 2 * bs + 2)
    traces = plain.outputs()[0]
    del plain
    torch.cuda.empty_cache()
    L = max(len(t) for t in traces) + 4 * bs
    trace_t = torch.zeros((B, L), dtype=torch.int32)
    for b, t in enumerate(traces):
        trace_t[b, :len(t)] = torch.tensor(t, dtype=torch.int32)
    lengths, noise = [], []
    for b in range(B):
        le, no = injection_plan(total_steps + 4, bs, tau, tcfg.vocab_size, seed * 1000 + b)
        lengths.append(le)
        noise.append(no.reshape(-1))
    sess = SpecSession(target, draft, B, args.ctx + n_new, bs, set(), use_graph=True, max_steps=total_steps + 8)
    sess.set_injection(trace_t, torch.stack(lengths), torch.stack(noise))
    sess.prefill(prompts, n_new)
    for _ in range(args.warmup):
        sess.step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(device.index)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.ncu_region:
        torch.cuda.profiler.start()
    t0.record()
    for k in range(args.steps):
        sess.step(events=evs[k])
    t1.record()
    torch.cuda.synchronize()
    if args.ncu_region:
        torch.cuda.profiler.stop()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    elapsed = t0.elapsed_time(t1) * 1e-3
    accepted = int(sess.accept_log[:, args.warmup:args.warmup + args.steps].sum())
    if world > 1:
        t = torch.tensor([elapsed], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t[0])
    from dflash_b200 import ops
    err = ops.device_error()
    verify_us = sorted(evs[k][1].elapsed_time(evs[k][2]) * 1e3 for k in range(args.steps))
    draft_us = sorted(evs[k][0].elapsed_time(evs[k][1]) * 1e3 for k in range(args.steps))
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(accepted / elapsed, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, random prompts, oracle-injected drafts)",
            "config": {"workload": f"config5: Qwen3.5-27B-shaped hybrid ({n_layers} layers) + 5-layer DFlash draft, "
                                   f"batch {B}, context {args.ctx}, block 16, oracle-injected acceptance tau {tau}",
                       "global_batch": B, "seq_len": args.ctx, "parallelism": f"tensor-parallel x{world}",
                       "l2": "weights per rank far above the 126 MB L2"},
            "value_note": "accepted tokens/s of the whole job (one batch decoded by all ranks together)",
            "p50_verify_step_us": round(verify_us[len(verify_us) // 2], 1),
            "p50_draft_step_us": round(draft_us[len(draft_us) // 2], 1),
            "tau_measured": round(accepted / (args.steps * B), 3), "device_error": err,
            "clocks": clk, "roofline": None, "e2e": None, "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark: evk::ai flash-attention forward on B200.

One step = one evk::ai flash-attention forward over one batch of the C2
configuration (B=4, H=16, S=2048, Dh=64, causal, fp16 Q/K/V ~ N(0,1), seeded,
per-head K/V), launched through the C ABI (evkcu_flash_attention).

  value  device throughput, inputs resident in HBM: algorithmic FLOPs
         (4*B*H*S^2*Dh / 2 for causal) / CUDA-event time of K steps.  Steps
         rotate over input sets totalling > 3x the 126 MB L2, so no step
         reads a predecessor's inputs from L2.
  e2e    the same metric through the same C ABI call with HOST buffers:
         per step, pinned-host Q/K/V -> device, the kernel, O -> pinned host,
         all inside the timed region; steps are pipelined over three streams
         (step i+1's upload overlaps step i's kernel and download), as a
         serving loop would run them.
  roofline  tensor-bound; achieved TFLOP/s of the flash kernel (measured with
         CUDA events on its launch stream) over the measured bf16 dense peak.
  cpu_baseline  the CPU oracle (C++ restatement of the reference's shader
         math) on a bounded sample of (batch, head) pairs of the same workload.

With --impl reference the CPU implementation (the reference's Vulkan path
cannot run on a machine without a graphics stack) is timed on the host cores on the same
workload and metric.  Multi-GPU (torchrun): each rank runs its own C2 batch
(weak scaling, no collective); value = total FLOPs / max over ranks.
Extra keys report the GEMM leg (8192^3 bf16 matmul TFLOP/s) for context.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, H, S, DH = 4, 16, 2048, 64
CAUSAL = True
FLOPS = 4.0 * B * H * S * S * DH / (2.0 if CAUSAL else 1.0)
METRIC = "flash-attn fwd TFLOP/s (C2: B4 H16 S2048 Dh64 causal)"
CONFIG = {
    "workload": "evk::ai flash_attention fwd, C2 B=4 H=16 S=2048 Dh=64 causal, per-head K/V",
    "global_batch": B,
    "seq_len": S,
    "heads": H,
    "head_dim": DH,
    "causal": CAUSAL,
    "l2": "inputs rotate over sets totalling > 3x L2",
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = "clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        mx = max((float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples)}


def cpu_baseline(budget_s: float = 10.0, threads: int | None = None):
    """Times the CPU oracle on whole (batch, head) slices of the C2 workload."""
    import numpy as np

    import oracle

    if threads:
        os.environ["EVK_ORACLE_THREADS"] = str(threads)
    n = S * DH
    q, k, v = (oracle.normal(n, s) for s in (11, 12, 13))
    o = np.empty_like(q)
    done, t0 = 0, time.perf_counter()
    while True:
        oracle.flash_attention(q, k, v, o, 1, S, 1, 1, DH, 0.0, 1 if CAUSAL else 0, 0)
        done += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    flops = done * 4.0 * S * S * DH / (2.0 if CAUSAL else 1.0)
    return {
        "value": flops / dt / 1e12,
        "unit": "TFLOP/s",
        "cores": oracle.num_threads(),
        "sample": f"{done} of the {B * H} (batch, head) slices of C2 (S=2048, Dh=64, causal), {dt:.1f} s",
    }


def cpu_extra():
    """The CPU oracle on the other configurations the survey plans a CPU
    baseline for: C1 (matmul 1024^3, fp16) and C3 decode steps (the oracle
    decoder, tests/llm_ref.py: KV-cached, batch 1, after a 128-token prompt).
    A few seconds each, on all host threads."""
    import numpy as np

    import oracle

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from llm_ref import RefModel

    n = 1024
    a, b = oracle.normal(n * n, 1), oracle.normal(n * n, 2)
    c = np.empty(n * n, np.uint16)
    oracle.matmul(a, b, c, 1, n, n, n, 0, 0, 0, 0, 0)
    reps, t0 = 0, time.perf_counter()
    while reps < 2 or time.perf_counter() - t0 < 2.0:
        oracle.matmul(a, b, c, 1, n, n, n, 0, 0, 0, 0, 0)
        reps += 1
    c1 = 2.0 * n ** 3 * reps / (time.perf_counter() - t0) / 1e9
    m = RefModel(6, 512, 8, 2048, 32000, True, dtype=0, seed=42)
    prompt = oracle.uniform_ids(128, 7, 0, 32000, 4).astype(np.int64).reshape(1, 128)
    logits = m.start(prompt, 128 + 257)
    ids = m.greedy(logits)
    steps, t0 = 0, time.perf_counter()
    while steps < 256 and (steps < 3 or time.perf_counter() - t0 < 3.0):
        ids = m.greedy(m.step(ids))
        steps += 1
    c3 = (time.perf_counter() - t0) / steps * 1e3
    return {"c1_matmul_gflops": round(c1, 2), "c3_decode_ms_per_step": round(c3, 2),
            "sample": f"C1: {reps} matmuls; C3: {steps} decode steps after a 128-token prompt"}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    # The reference runs its kernels as Vulkan compute shaders; neither Vulkan
    # nor a software renderer exists on these machines, so the reference arm
    # is the reference's algorithm restated on the CPU (the oracle), timed on
    # all host threads over a bounded sample per step.
    vals = []
    for _ in range(args.warmup):
        cpu_baseline(budget_s=0.5)
    for _ in range(args.steps):
        vals.append(cpu_baseline(budget_s=2.0)["value"])
    cb = cpu_baseline(budget_s=2.0)
    value = sorted(vals)[len(vals) // 2]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": FLOPS / (value * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cb["cores"], "kind": "port",
                         "sample": "per step: " + cb["sample"]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU oracle (restatement of the reference shaders); the reference's Vulkan path is unavailable on this box",
    }
    print(json.dumps(line), flush=True)


def gemm_leg(torch, evk, dtype, n=8192, reps=20):
    a = torch.randn(n, n, device="cuda").to(dtype)
    b = torch.randn(n, n, device="cuda").to(dtype)
    c = torch.empty(n, n, device="cuda", dtype=dtype)
    for _ in range(3):
        evk.matmul(a, b, c)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if n <= 2048:
        # Small products take a few microseconds: replay them from a CUDA
        # graph so host launch overhead is not what is timed.
        st = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for _ in range(reps):
                evk.matmul(a, b, c, stream=st)
        g.replay()
        torch.cuda.synchronize()
        s.record()
        g.replay()
        e.record()
    else:
        s.record()
        for _ in range(reps):
            evk.matmul(a, b, c)
        e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    return 2.0 * n ** 3 / (ms * 1e-3) / 1e12


# LLM configurations of BASELINE.json (random weights, synthetic prompts):
# name -> (layers, d_model, heads, hidden, vocab, batch, prompt, decode steps, dtype, tied)
LLM_CONFIGS = {
    "C3_tiny": (6, 512, 8, 2048, 32000, 1, 128, 256, 0, True),
    "C4_1.3B": (24, 2048, 16, 8192, 32000, 8, 2048, 64, 1, False),
    "C5_8B_shape": (32, 4096, 32, 14336, 128256, 16, 4096, 16, 1, False),
}


def llm_leg(torch, evk, name, comm=None, rank=0, world=1):
    """Prefill TFLOP/s and decode tok/s of one LLM config through the C ABI
    (evkcu_llm_*), tensor-parallel over `world` GPUs.  Device-timed with CUDA
    events; decode steps replay the captured CUDA graph.  FLOPs count the
    projection GEMMs (2 * params * tokens), causal attention and the LM head."""
    L, D, H, F, V, B, S, steps, dt, tied = LLM_CONFIGS[name]
    if world > 1 and (H % world or V % world):
        return None
    m = evk.Llm(L, D, H, F, V, B, S + steps + 8, dtype=dt, tied_embeddings=tied, tp_rank=rank, tp_size=world,
                comm=comm)
    m.init_random(42, 0.02)
    st = torch.cuda.Stream()
    g = torch.Generator(device="cuda").manual_seed(7)
    tok = torch.randint(0, V, (B, S), dtype=torch.int32, device="cuda", generator=g)
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        m.prefill(tok, nxt, stream=st)
        st.synchronize()
        if world > 1:
            torch.distributed.barrier()
        ev0.record(st)
        m.prefill(tok, nxt, stream=st)
        ev1.record(st)
        st.synchronize()
        pf_ms = ev0.elapsed_time(ev1)
        bufs = [torch.zeros(B, dtype=torch.int32, device="cuda") for _ in range(2)]
        cur = nxt.clone()
        warm = 3
        for i in range(warm):
            m.decode(cur, bufs[i % 2], stream=st)
            cur = bufs[i % 2]
        st.synchronize()
        if world > 1:
            torch.distributed.barrier()
        ev0.record(st)
        for i in range(steps - warm):
            m.decode(cur, bufs[i % 2], stream=st)
            cur = bufs[i % 2]
        ev1.record(st)
        st.synchronize()
        dec_ms = ev0.elapsed_time(ev1) / (steps - warm)
    m.close()
    if world > 1:
        t = torch.tensor([pf_ms, dec_ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        pf_ms, dec_ms = t.tolist()
    params = L * (4 * D * D + 2 * D * F) + (0 if tied else D * V)
    flops = 2.0 * params * B * S + L * 4.0 * B * S * S * D / 2 + 2.0 * D * V * B
    return {"prefill_ms": round(pf_ms, 2), "prefill_tflops": round(flops / pf_ms / 1e9, 1),
            "decode_ms_per_step": round(dec_ms, 3), "decode_tok_s": round(B / dec_ms * 1e3, 1),
            "batch": B, "prompt": S, "tp": world}


def profile_leg(leg):
    """A few launches of one leg on resident inputs: the small case ncu captures."""
    import torch

    import evk_b200 as evk

    evk.init(0)
    if leg == "flash":
        q, k, v = (torch.randn(B, S, H * DH, device="cuda").half() for _ in range(3))
        o = torch.empty_like(q)
        for _ in range(5):
            evk.flash_attention(q, k, v, o, heads=H, causal=CAUSAL)
    elif leg == "flash128":
        # C4 prefill attention: B=8, H=16, S=2048, Dh=128, causal, bf16
        q, k, v = (torch.randn(8, 2048, 16 * 128, device="cuda").bfloat16() for _ in range(3))
        o = torch.empty_like(q)
        for _ in range(5):
            evk.flash_attention(q, k, v, o, heads=16, causal=True)
    elif leg == "gemm":
        a, b = (torch.randn(8192, 8192, device="cuda").bfloat16() for _ in range(2))
        c = torch.empty_like(a)
        for _ in range(3):
            evk.matmul(a, b, c)
    elif leg == "gemv":
        # C5 decode W1 shape: 16 rows x [4096, 14336] bf16 weight (117 MB)
        x = torch.randn(16, 4096, device="cuda").bfloat16()
        w = torch.randn(4096, 14336, device="cuda").bfloat16()
        y = torch.empty(16, 14336, device="cuda").bfloat16()
        for _ in range(3):
            evk.matmul(x, w, y)
    elif leg == "llm-decode":
        # C4 (random weights): one prefill, then four eager decode steps (the
        # launch list of one step is the last quarter of the decode launches).
        L, D, Hh, F, V, Bb, Sp, _, dt, tied = LLM_CONFIGS["C4_1.3B"]
        m = evk.Llm(L, D, Hh, F, V, Bb, Sp + 16, dtype=dt, tied_embeddings=tied)
        m.init_random(42, 0.02)
        tok = torch.randint(0, V, (Bb, Sp), dtype=torch.int32, device="cuda")
        nxt = torch.zeros(Bb, dtype=torch.int32, device="cuda")
        m.prefill(tok, nxt)
        cur, out = nxt.clone(), torch.zeros_like(nxt)
        for _ in range(4):
            m.decode(cur, out)
            cur, out = out, cur
        torch.cuda.synchronize()
        m.close()
    elif leg == "decode":
        # C4 decode attention: B=8, H=16, Dh=128 over 2048 cached positions (bf16)
        q = torch.randn(8, 16 * 128, device="cuda").bfloat16()
        kc = torch.randn(8, 2048, 16 * 128, device="cuda").bfloat16()
        vc = torch.randn_like(kc)
        o = torch.empty_like(q)
        for _ in range(3):
            evk.single_query_attention(q, kc, vc, o, 16, 2048)
    torch.cuda.synchronize()
    evk.check_device_error()


# Projection GEMM shapes of the LLM configs' prefill (bf16, M = batch x prompt
# rows), with the residual add (C +=) where the driver fuses it.
GEMM_SHAPES = [("C4 QKV", 16384, 2048, 6144, False), ("C4 Wo", 16384, 2048, 2048, True),
               ("C4 W1", 16384, 2048, 8192, False), ("C4 W2", 16384, 8192, 2048, True),
               ("8192^3", 8192, 8192, 8192, False), ("C5 QKV", 65536, 4096, 12288, False),
               ("C5 Wo", 65536, 4096, 4096, True)]


def gemm_shapes():
    """TFLOP/s of evkcu_matmul on the prefill projection shapes (CUDA events,
    10 launches after 3 warm-up, inputs resident).  EVKCU_GEMM_PLAIN_EPILOGUE=1
    selects the per-row-store epilogue for comparison."""
    import torch

    import evk_b200 as evk

    evk.init(0)
    for name, M, K, N, acc in GEMM_SHAPES:
        a = torch.randn(M, K, device="cuda").bfloat16()
        b = (torch.randn(K, N, device="cuda") * 0.02).bfloat16()
        c = torch.zeros(M, N, device="cuda").bfloat16()
        for _ in range(3):
            evk.matmul(a, b, c, acc_c=acc)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(10):
            evk.matmul(a, b, c, acc_c=acc)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 10
        print(json.dumps({"shape": name, "M": M, "K": K, "N": N, "acc_c": acc, "us": round(ms * 1e3, 1),
                          "tflops": round(2.0 * M * N * K / ms / 1e9, 1)}), flush=True)
        del a, b, c
    evk.check_device_error()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="evk_b200", choices=["evk_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--profile-leg", choices=["flash", "flash128", "gemm", "gemv", "decode", "llm-decode"], default=None,
                    help="run a few launches of one leg and exit (for ncu captures; prints no JSON)")
    ap.add_argument("--gemm-shapes", action="store_true",
                    help="print TFLOP/s of the prefill projection GEMM shapes (one JSON line each) and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.profile_leg:
        return profile_leg(args.profile_leg)
    if args.gemm_shapes:
        return gemm_shapes()

    import torch

    import evk_b200 as evk

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    evk.init(local)
    dtype = torch.float16
    stream = torch.cuda.current_stream()

    # Input sets: enough that the rotation never hits L2 (3x 126 MB).
    set_bytes = 4 * B * S * H * DH * 2
    nsets = max(2, int((3 * 126e6) // set_bytes) + 1)
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    sets = []
    for _ in range(nsets):
        q, k, v = (torch.randn(B, S, H * DH, device="cuda", generator=g).to(dtype) for _ in range(3))
        sets.append((q, k, v, torch.empty_like(q)))

    def step(i):
        q, k, v, o = sets[i % nsets]
        evk.flash_attention(q, k, v, o, heads=H, causal=CAUSAL, stream=stream)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    # ------------------------------------------------ device-timed region --
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        evk.reset_launch_count()
        start.record(stream)
        for i in range(args.steps):
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
        launches = evk.launch_count()
        if ws > 1:
            torch.distributed.barrier()
    ms_total = start.elapsed_time(end)
    if ws > 1:
        t = torch.tensor([ms_total], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_total = t.item()
    ms_step = ms_total / args.steps
    value = FLOPS * ws / (ms_step * 1e-3) / 1e12
    kernel_tflops = FLOPS / (ms_step * 1e-3) / 1e12
    evk.check_device_error()

    # ------------------------------------------------------ end-to-end leg --
    # Each step copies its Q/K/V from pinned host memory, runs the C-ABI call
    # and copies O back to pinned host memory, all inside the timed region.
    # Steps are pipelined like a serving loop: H2D, compute and D2H run on
    # three streams with double-buffered device tensors, so step i + 1's
    # upload overlaps step i's kernel and download.
    # Host inputs rotate over up to four pinned sets (one per device set).
    host_sets = [tuple(t.cpu().pin_memory() for t in st[:3]) for st in sets[:4]]
    hq = host_sets[0][0]
    ho = [torch.empty_like(hq).pin_memory() for _ in range(2)]
    dbuf = [[torch.empty_like(sets[0][0]) for _ in range(4)] for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_run = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    e2e_steps = max(20, min(200, args.steps))
    step_no = [0]

    def e2e_step():
        i = step_no[0]
        step_no[0] += 1
        b = i & 1
        dq, dk, dv, do = dbuf[b]
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(ev_run[b])  # step i-2 no longer reads these inputs
            hq_i, hk_i, hv_i = host_sets[i % len(host_sets)]
            dq.copy_(hq_i, non_blocking=True)
            dk.copy_(hk_i, non_blocking=True)
            dv.copy_(hv_i, non_blocking=True)
            ev_in[b].record(h2d)
        stream.wait_event(ev_in[b])
        if i >= 2:
            stream.wait_event(ev_out[b])  # step i-2's output has been downloaded
        evk.flash_attention(dq, dk, dv, do, heads=H, causal=CAUSAL, stream=stream)
        ev_run[b].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(ev_run[b])
            ho[b].copy_(do, non_blocking=True)
            ev_out[b].record(d2h)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    step_no[0] = 0
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        torch.distributed.barrier()
    es.record(stream)
    h2d.wait_event(es)
    d2h.wait_event(es)
    for _ in range(e2e_steps):
        e2e_step()
    for b in range(2):
        stream.wait_event(ev_out[b])
    ee.record(stream)
    torch.cuda.synchronize()
    e2e_ms = es.elapsed_time(ee) / e2e_steps
    if ws > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = t.item()
    e2e_val = FLOPS * ws / (e2e_ms * 1e-3) / 1e12
    ho = ho[(e2e_steps - 1) & 1]
    # Parity spot-check of the last copied result against the resident run
    # of the same input set.
    last = sets[(e2e_steps - 1) % len(host_sets)]
    evk.flash_attention(*last, heads=H, causal=CAUSAL, stream=stream)
    torch.cuda.synchronize()
    assert torch.equal(ho.cuda(), last[3]), "e2e output differs from the device-resident run"

    extra = {}
    if not args.no_extra:
        extra["gemm_8192_bf16_tflops"] = round(gemm_leg(torch, evk, torch.bfloat16), 1)
        extra["gemm_8192_f16_tflops"] = round(gemm_leg(torch, evk, torch.float16), 1)
        # C1 (1024^3, fp16): 64 output tiles of 128 x 128 for 148 SMs, L2-resident; plumbing and parity size
        extra["c1_matmul_f16_tflops"] = round(gemm_leg(torch, evk, torch.float16, n=1024, reps=200), 1)
        comm = None
        if ws > 1:
            uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
            if rank == 0:
                uid.copy_(torch.frombuffer(bytearray(evk.Comm.unique_id()), dtype=torch.uint8))
            torch.distributed.broadcast(uid, 0)
            comm = evk.Comm(bytes(uid.cpu().numpy()), rank, ws)
        llm = {}
        for name in ("C3_tiny", "C4_1.3B", "C5_8B_shape"):
            llm[name] = llm_leg(torch, evk, name, comm, rank, ws)
        extra["llm"] = llm
        if comm:
            comm.close()

    if ws > 1:
        torch.distributed.barrier()
    if rank != 0:
        torch.distributed.destroy_process_group()
        return

    tf_peak, _, peak_kind = peaks()
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get("flash_tc_kernel_c2_bytes_per_launch")
        except Exception:
            traffic = None
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": ws,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": dict(CONFIG, parallelism=f"replicas x{ws} (independent C2 batches)"),
        "e2e": {"value": round(e2e_val, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": 3 * hq.numel() * 2,
                "d2h_bytes_per_step": ho.numel() * 2},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": round(kernel_tflops, 2), "peak": tf_peak, "unit": "TFLOP/s",
                     "frac": round(kernel_tflops / tf_peak, 4), "peak_kind": f"bf16 dense burst, {peak_kind}",
                     "traffic": traffic},
        "clocks": clocks.summary(),
        "extra": extra,
    }
    if not args.no_cpu_baseline and ws == 1:  # the CPU baseline is timed at N = 1 only
        line["cpu_baseline"] = dict(cpu_baseline(budget_s=10.0), kind="port")
        if not args.no_extra:
            line["cpu_baseline"]["extra"] = cpu_extra()
    print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

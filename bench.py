#!/usr/bin/env python
"""Benchmark of the attention hot path: causal flash-attention forward +
backward through libctfa_b200.so (C ABI, tcgen05 kernels).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config2|config3|config5|...]

One step = forward (o, lse) + backward (dq, dk, dv) of one batch.  Default
workload = BASELINE config 2 (GPT-2-small attention: B=8 per GPU, H=12,
T=1024, D=64, fp32 I/O through tf32 MMAs, causal).  With N GPUs (torchrun,
one rank per GPU) every rank owns its own 8 sequences (batch x head shards,
no collective in the step): weak scaling, value = all ranks' FLOPs / max time.
Config 3 (bf16, B=16, H=16, T=2048, D=128) is strong-scaled: its fixed 256
(batch, head) problems are divided among the ranks (16/N sequences each).

FLOP convention (algorithmic): causal fwd + bwd = 7 * B*H*T^2*D
(2 GEMMs forward + 5 backward, each half-masked); non-causal = 14 * B*H*T^2*D.

Printed JSON line (rank 0): value = device-resident throughput (inputs in HBM
when the timed region starts); e2e = same metric through the C ABI with
pinned host buffers, every step's H2D of q/k/v/dO and D2H of o/dq/dk/dv inside
the timed region (on copy streams that overlap the neighbouring steps'
compute, device buffers double-buffered; at least 100 steps, so that the
pipeline's fill and drain stay below 1 % of it); roofline for the dominant kernel,
timed with CUDA events on its own launch stream, against the tf32 cuBLAS peak
measured in the run and, beside it, half and all of the bf16 burst peak;
per-rank step times and SM clocks; cpu_baseline = the fp32 OpenMP CPU
attention (oracle) on a bounded sample of heads, on this host.  The default
line also carries `config3_bf16`: config 3 timed the same way (its own timed
region, strong-scaled over the N GPUs), with its kernel split and its
fraction of the bf16 dense peak.

--impl reference times the reference's own CUDA FlashAttentionLayer<float>
(computeAttention(saveStates=true) + computeBackward + clearCache, compiled
unmodified from its sources into oracle/_ref/libctref.so) on one GPU, on the
same shape.  The reference has no causal mask, so it computes the full
(non-causal) attention; its FLOPs are counted at 14 * B*H*T^2*D, the work it
does.  Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "causal attention fwd+bwd TFLOP/s and % of B200 tensor peak at 1/2/4/8 GPUs"

WORKLOADS = {
    "config2": dict(desc="BASELINE config 2: GPT-2-small attention shape", B=8, H=12, T=1024, D=64, dtype="f32",
                    causal=True, qkv_scale=0.5, do_scale=1.0, seed=1),
    "config3": dict(desc="BASELINE config 3: bf16 I/O, D=128", B=16, H=16, T=2048, D=128, dtype="bf16",
                    causal=True, qkv_scale=1.0, do_scale=0.1, seed=2, strong=True),
    "config5": dict(desc="BASELINE config 5: long context, bf16, sequence sharded over the GPUs (ring)", B=1, H=32,
                    T=131072, D=128, dtype="bf16", causal=True, qkv_scale=1.0, do_scale=1.0, seed=4),
    "config4": dict(desc="BASELINE config 4: NanoGPT training step (6 layers, d=384, 6 heads x 64, T=256, vocab 65, "
                         "batch 64, fp32, Adam lr 3e-4)", B=64, H=6, T=256, D=64, dtype="f32", causal=False,
                    layers=6, vocab=65, mlp=1536, lr=3e-4, seed=3),
    "proj_config4": dict(desc="QKV + output projection GEMMs of one config-4 block (B=64, T=256, E=384, 6 heads x 64), "
                              "fp32", B=64, T=256, E=384, H=6, D=64, dtype="f32", seed=5),
    "proj_bf16": dict(desc="QKV + output projection GEMMs, bf16, B=8, T=2048, E=2048, 16 heads x 128", B=8, T=2048,
                      E=2048, H=16, D=128, dtype="bf16", seed=6),
    "config4causal": dict(desc="BASELINE config 4 with the causal mask (language-model semantics)", B=64, H=6, T=256,
                          D=64, dtype="f32", causal=True, layers=6, vocab=65, mlp=1536, lr=3e-4, seed=3),
}


def path_flops(B, H, T, D, causal):
    return (7 if causal else 14) * B * H * T * T * D


def gemm_flops(B, H, T, D, causal):
    """One T x T x D GEMM per head, halved under the causal mask."""
    return (1 if causal else 2) * B * H * T * T * D


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


# ---------------------------------------------------------------------------
# clocks sampled with nvidia-smi during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.tmp, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.tmp.flush()
        rows = []
        for line in Path(self.tmp.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]), power=float(parts[3]),
                                 util=float(parts[4]), hw=parts[6], hwt=parts[7], swt=parts[8], pcap=parts[9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r["util"] >= 50] or rows
        reasons = sorted({name for r in loaded for name, key in
                          (("hw_slowdown", "hw"), ("hw_thermal_slowdown", "hwt"), ("sw_thermal_slowdown", "swt"),
                           ("sw_power_cap", "pcap")) if r[key].lower() == "active"})
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": max(r["smax"] for r in rows),
                "power_w_max": max(r["power"] for r in rows), "samples": len(rows),
                "samples_under_load": len(loaded), "reasons": reasons}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_init(n_gpus):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------
def tf32_peak_tflops():
    """cuBLAS tf32 GEMM 8192^3, best of 10 (the denominator for fp32 I/O)."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(3):
        a @ b
    best = 0.0
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        a @ b
        e.record()
        e.synchronize()
        best = max(best, 2 * n ** 3 / (s.elapsed_time(e) * 1e-3) / 1e12)
    torch.backends.cuda.matmul.allow_tf32 = False
    del a, b
    return best


def cpu_baseline(w, min_seconds: float = 10.0):
    """fp32 CPU attention forward + backward on this host, on a bounded sample
    of the workload: (i) the OpenMP online-softmax restatement
    (oracle/liboracle.so, all host threads) over a block of (batch, head)
    problems, repeated until at least `min_seconds` of wall time; (ii) PyTorch
    CPU scaled_dot_product_attention + autograd backward on the same block,
    for about a quarter of that time."""
    import numpy as np

    from oracle import oracle as orc

    cores = os.cpu_count() or 1
    n_heads = min(w["B"] * w["H"], max(8, cores))
    rng = np.random.default_rng(w["seed"])
    shape = (1, n_heads, w["T"], w["D"])
    q, k, v = (rng.standard_normal(shape, dtype=np.float32) * w["qkv_scale"] for _ in range(3))
    do = rng.standard_normal(shape, dtype=np.float32) * w["do_scale"]
    flops = path_flops(1, n_heads, w["T"], w["D"], w["causal"])
    reps, t0 = 0, time.perf_counter()
    while True:
        orc.cpu_attention_fwd_bwd_f32(q, k, v, do, w["causal"], threads=cores)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    out = {"value": flops * reps / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
           "sample": f"{n_heads} of {w['B'] * w['H']} (batch, head) problems of the workload, fp32 fwd+bwd, "
                     f"repeated {reps}x in {dt:.1f} s wall (OpenMP restatement, oracle/liboracle.so)",
           "seconds": round(dt, 2)}
    try:
        import torch

        torch.set_num_threads(cores)
        nt = max(1, n_heads // 4)  # PyTorch's CPU path is much slower: a quarter of the block
        tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x[:, :nt])).requires_grad_() for x in (q, k, v))
        tdo = torch.from_numpy(np.ascontiguousarray(do[:, :nt]))
        tflops = path_flops(1, nt, w["T"], w["D"], w["causal"])
        treps, t0 = 0, time.perf_counter()
        while True:
            o = torch.nn.functional.scaled_dot_product_attention(tq, tk, tv, is_causal=bool(w["causal"]))
            o.backward(tdo)
            treps += 1
            tdt = time.perf_counter() - t0
            if tdt >= min_seconds / 4:
                break
        out["torch_sdpa_cpu"] = {"value": round(tflops * treps / tdt / 1e12, 4), "unit": "TFLOP/s",
                                 "threads": cores,
                                 "sample": f"{nt} (batch, head) problems, repeated {treps}x in {tdt:.1f} s"}
    except Exception as e:  # the OpenMP figure above is the reported baseline
        out["torch_sdpa_cpu"] = {"unavailable": str(e)[:200]}
    return out


def run_ring(args, w, rank, world, local):
    """Config 5 on N >= 2 GPUs: each rank holds 2 of the 2N zig-zag chunks of
    the sequence; forward + backward through RingAttention (NCCL send/recv of
    K/V and dK/dV between neighbours, overlapped with the block kernels)."""
    import torch

    from cudatransformer_b200 import ring_attention as ra

    B, H, T, D = w["B"], w["H"], w["T"], w["D"]
    Tl = T // world
    dev = torch.device("cuda", local)
    gen = torch.Generator().manual_seed(w["seed"] * 1000 + rank)
    shape = (B, H, Tl, D)

    def host(scale):
        return (torch.randn(shape, generator=gen) * scale).to(torch.bfloat16).pin_memory()

    q_h, k_h, v_h, do_h = host(1.0), host(1.0), host(1.0), host(w["do_scale"])
    q, k, v, do = (x.to(dev) for x in (q_h, k_h, v_h, do_h))
    outs_h = [torch.empty(shape, dtype=torch.bfloat16).pin_memory() for _ in range(4)]
    ring = ra.RingAttention()
    stream = torch.cuda.current_stream(dev)
    res = {}

    def step():
        o, lse = ring.forward(q, k, v)
        res["g"] = (o,) + ring.backward(q, k, v, o, lse, do)

    def e2e_step():
        for dst, src in ((q, q_h), (k, k_h), (v, v_h), (do, do_h)):
            dst.copy_(src, non_blocking=True)
        step()
        for dst, src in zip(outs_h, res["g"]):
            dst.copy_(src, non_blocking=True)

    def timed(fn, steps):
        barrier(world)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            fn()
        e.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        return max_over_ranks(s.elapsed_time(e), world)

    for _ in range(args.warmup):
        step()
    with ClockSampler(local) as clocks:
        ms = timed(step, args.steps)
    clk = clocks.summary()
    for _ in range(args.warmup):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps)

    # The same schedule with every exchange replaced by a local device copy of
    # the same buffers (each rank computes the same blocks on its own K/V): the
    # compute time of a step; the ring step minus it is communication left
    # exposed (not hidden under the block kernels).
    class LocalRing(ra.RingAttention):
        def _exchange(self, send, recv):
            recv.copy_(send)
            return []

    local_ring = LocalRing()

    def compute_step():
        o, lse = local_ring.forward(q, k, v)
        local_ring.backward(q, k, v, o, lse, do)

    for _ in range(2):
        compute_step()
    ms_compute = timed(compute_step, args.steps)
    kv_hop_bytes = 2 * B * H * Tl * D * 2       # bf16 K and V of this rank's two chunks
    dkv_hop_bytes = 2 * B * H * Tl * D * 4      # fp32 dK / dV partial sums
    # kernel launches per step: forward = one block kernel per block (the merge is in its epilogue),
    # backward = delta pass + dK/dV + dQ per block; plus per-step zeroing / accumulation and the final
    # conversions
    n_blocks = sum(len(ra.block_plan(world, rank, s)) for s in range(world))
    launches = n_blocks + 3 * n_blocks + 2 * world + 4
    total = path_flops(B, H, T, D, True)
    peaks = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    if rank == 0:
        value = total / (ms / args.steps * 1e-3) / 1e12
        per_rank = value / world
        nbytes = B * H * Tl * D * 2
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16 I/O, bf16 tcgen05 MMA",
            "data": "synthetic: q,k,v,dO ~ N(0,1) bf16, seeded per rank",
            "config": {"workload": w["desc"], "batch": B, "heads": H, "seq_len": T, "head_dim": D, "causal": True,
                       "parallelism": f"zig-zag sequence shards over {world} GPUs, ring K/V + dK/dV exchange "
                                      "with NCCL send/recv overlapped with the block kernels",
                       "local_seq_len": Tl, "l2": "inputs far above 126 MB L2; no flush"},
            "pct_of_tensor_peak": {"of_dtype_peak": round(100 * per_rank / peak, 1), "dtype_peak_tflops": peak,
                                   "dtype_peak_source": "bf16 dense burst, MEASURED_PEAKS.json"},
            "e2e": {"value": round(total / (ms_e2e / args.steps * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "h2d_bytes_per_step": 4 * nbytes, "d2h_bytes_per_step": 4 * nbytes,
                    "ms_per_step": round(ms_e2e / args.steps, 3), "path": "RingAttention (C ABI block calls)"},
            "gpu_launches": launches * args.steps,
            "ring": {"compute_only_ms_per_step": round(ms_compute / args.steps, 3),
                     "exposed_comm_ms_per_step": round((ms - ms_compute) / args.steps, 3),
                     "hops_per_step": {"kv": world - 1, "dkv": world},
                     "kv_bytes_per_hop": kv_hop_bytes, "dkv_bytes_per_hop": dkv_hop_bytes,
                     "note": "compute_only = the same step with each NCCL exchange replaced by a local copy; "
                             "max over ranks"},
            "roofline": {"kernel": "ring step (all block kernels of one rank)", "bound": "tensor",
                         "achieved": round(per_rank, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(per_rank / peak, 3), "traffic": None},
            "cpu_baseline": None,
            "clocks": clk,
        }
        print(json.dumps(out), flush=True)
    barrier(world)


def gather_over_ranks(values, world):
    """All ranks' lists of floats (rank order); the local list when world == 1."""
    if world == 1:
        return [list(values)]
    import torch
    import torch.distributed as dist

    t = torch.tensor(list(values), dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


KERNELS = ("attn_fwd_sm100", "attn_bwd_prep", "attn_bwd_dkdv_sm100", "attn_bwd_dq_sm100")


def measure_attention(args, w, B, rank, world, local, with_e2e):
    """Times one attention shard of B sequences (all of its heads) through the
    C ABI on this rank's GPU: `steps` forward + backward steps after `warmup`
    untimed ones, bracketed by a barrier and synchronize, max over ranks; then
    (with_e2e) the same steps with host buffers; then each kernel alone with
    CUDA events on the launch stream.  Inputs are seeded per rank."""
    import torch

    from cudatransformer_b200 import _lib

    lib = _lib.load()
    H, T, D = w["H"], w["T"], w["D"]
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[w["dtype"]]
    code = {"f32": _lib.CTFA_DTYPE_F32, "bf16": _lib.CTFA_DTYPE_BF16}[w["dtype"]]
    causal = int(w["causal"])
    dev = torch.device("cuda", local)
    gen = torch.Generator().manual_seed(w["seed"] * 1000 + rank)
    shape = (B, H, T, D)

    def host(scale):
        t = (torch.randn(shape, generator=gen) * scale).to(tdt)
        return t.pin_memory() if with_e2e else t

    q_h, k_h, v_h = (host(w["qkv_scale"]) for _ in range(3))
    do_h = host(w["do_scale"])
    q, k, v, do = (x.to(dev) for x in (q_h, k_h, v_h, do_h))
    if not with_e2e:
        del q_h, k_h, v_h, do_h
    o, dq, dk, dv = (torch.empty(shape, dtype=tdt, device=dev) for _ in range(4))
    lse = torch.empty((B, H, T), dtype=torch.float32, device=dev)
    fws_bytes = lib.ctfa_forward_workspace_bytes(B, H, T, D, code)
    fws = torch.empty(max(fws_bytes, 256), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def fwd():
        _lib.check(lib.ctfa_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
                                    B, H, T, D, code, causal, fws.data_ptr(), fws.numel(), sh), "ctfa_forward")

    # fp32: the backward reads the tf32-rounded q, k, v the forward left in its
    # workspace (what FlashAttentionLayer does with saveStates), so it only
    # rounds dO.
    if fws_bytes:
        qb, kb, vb = _lib.rounded_copies(fws, B, H, T, D)
        bcode = _lib.CTFA_DTYPE_TF32
    else:
        qb, kb, vb, bcode = q.data_ptr(), k.data_ptr(), v.data_ptr(), code
    bws = torch.empty(lib.ctfa_backward_workspace_bytes(B, H, T, D, bcode), dtype=torch.uint8, device=dev)

    def bwd(events=None):
        ptrs = (qb, kb, vb, o.data_ptr(), do.data_ptr(), lse.data_ptr(),
                dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), bws.data_ptr(), bws.numel(), B, H, T, D, bcode, causal,
                sh)
        if events is None:
            _lib.check(lib.ctfa_backward(*ptrs), "ctfa_backward")
        else:
            import ctypes

            for ev_ in events:  # torch creates the CUDA event lazily, on first record
                ev_.record(stream)
            arr = (ctypes.c_void_p * 4)(*[ev_.cuda_event for ev_ in events])
            _lib.check(lib.ctfa_backward_with_events(*ptrs, arr), "ctfa_backward_with_events")

    def step():
        fwd()
        bwd()

    def timed(fn, steps):
        barrier(world)
        torch.cuda.synchronize(dev)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(steps):
            fn()
        e.record(stream)
        torch.cuda.synchronize(dev)
        barrier(world)
        return s.elapsed_time(e)

    for _ in range(args.warmup):
        step()
    _lib.check(lib.ctfa_check_device_error(sh), "warm-up (device)")
    with ClockSampler(local) as clocks:
        ms_local = timed(step, args.steps)
    _lib.check(lib.ctfa_check_device_error(sh), "timed steps (device)")
    clk = clocks.summary()
    ms = max_over_ranks(ms_local, world)
    res = {"ms": ms, "ms_local": ms_local, "clocks": clk, "fws_bytes": fws_bytes}

    if with_e2e:
        # e2e: every step copies its q, k, v, dO in from pinned host memory and
        # its o, dq, dk, dv out, through the same C-ABI calls.  The copies run on
        # their own streams and overlap the neighbouring steps' compute (device
        # inputs and outputs double-buffered; PCIe carries both directions at
        # once).
        o_h, dq_h, dk_h, dv_h = (torch.empty(shape, dtype=tdt).pin_memory() for _ in range(4))
        h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        e2e_sets = []
        for _ in range(2):
            ins = [torch.empty(shape, dtype=tdt, device=dev) for _ in range(4)]
            outs = [torch.empty(shape, dtype=tdt, device=dev) for _ in range(4)]
            e2e_sets.append({"in": ins, "out": outs, "ev_in": torch.cuda.Event(), "ev_comp": torch.cuda.Event(),
                             "ev_out": torch.cuda.Event()})

        def e2e_compute(st):
            qi, ki, vi, doi = (t.data_ptr() for t in st["in"])
            oo, dqo, dko, dvo = (t.data_ptr() for t in st["out"])
            _lib.check(lib.ctfa_forward(qi, ki, vi, oo, lse.data_ptr(), B, H, T, D, code, causal, fws.data_ptr(),
                                        fws.numel(), sh), "ctfa_forward")
            bq, bk, bv = (qb, kb, vb) if fws_bytes else (qi, ki, vi)
            _lib.check(lib.ctfa_backward(bq, bk, bv, oo, doi, lse.data_ptr(), dqo, dko, dvo, bws.data_ptr(),
                                         bws.numel(), B, H, T, D, bcode, causal, sh), "ctfa_backward")

        def e2e_run(steps, compute=True):
            """Runs `steps` end-to-end steps; returns the device time from the
            first step's first H2D copy to the last step's last D2H copy.
            compute=False: the same copies with no kernels between them (the
            PCIe floor of the pipeline; reported beside the e2e number)."""
            torch.cuda.synchronize(dev)
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record(h2d_s)
            for i in range(steps):
                st = e2e_sets[i % 2]
                with torch.cuda.stream(h2d_s):
                    if i >= 2:
                        h2d_s.wait_event(st["ev_comp"])  # step i-2's compute has read these inputs
                    for dst, src in zip(st["in"], (q_h, k_h, v_h, do_h)):
                        dst.copy_(src, non_blocking=True)
                    st["ev_in"].record(h2d_s)
                stream.wait_event(st["ev_in"])
                if i >= 2:
                    stream.wait_event(st["ev_out"])  # step i-2's outputs have left the device
                if compute:
                    e2e_compute(st)
                st["ev_comp"].record(stream)
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(st["ev_comp"])
                    for dst, src in zip((o_h, dq_h, dk_h, dv_h), st["out"]):
                        dst.copy_(src, non_blocking=True)
                    st["ev_out"].record(d2h_s)
            e_ev.record(d2h_s)
            torch.cuda.synchronize(dev)
            return s_ev.elapsed_time(e_ev)

        # at least 100 steps: the pipeline's fill (the first step's inputs) and
        # drain (the last step's outputs) are then <= 1 % of the timed region
        e2e_steps = max(args.steps, 100)
        res["e2e_steps"] = e2e_steps
        e2e_run(args.warmup)
        barrier(world)
        res["ms_e2e"] = max_over_ranks(e2e_run(e2e_steps), world)
        barrier(world)
        res["ms_copies"] = max_over_ranks(e2e_run(e2e_steps, compute=False), world)
        barrier(world)
        del e2e_sets

    # per-kernel durations (events recorded on the launch stream around each launch)
    acc = {n: 0.0 for n in KERNELS}
    for _ in range(args.steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        # keep the stream busy while the host prepares the forward's launch
        # (tensor-map encoding), so that ev[0] -> ev[1] spans the kernel only
        if hasattr(torch.cuda, "_sleep"):
            torch.cuda._sleep(200_000)
        ev[0].record(stream)
        fwd()
        ev[1].record(stream)
        bwd(events=ev[2:6])
        torch.cuda.synchronize(dev)
        acc[KERNELS[0]] += ev[0].elapsed_time(ev[1])
        acc[KERNELS[1]] += ev[2].elapsed_time(ev[3])
        acc[KERNELS[2]] += ev[3].elapsed_time(ev[4])
        acc[KERNELS[3]] += ev[4].elapsed_time(ev[5])
    res["per_kernel_ms"] = {n: acc[n] / args.steps for n in KERNELS}
    per_rank = gather_over_ranks([ms_local / args.steps, clk.get("sm_mhz") or 0.0], world)
    res["per_rank"] = [{"rank": r, "ms_per_step": round(x[0], 4), "sm_mhz_median": x[1]}
                       for r, x in enumerate(per_rank)]
    del q, k, v, do, o, dq, dk, dv, fws, bws
    torch.cuda.empty_cache()
    return res


def shard_batch(w, world):
    """Sequences per rank.  Config 3 is strong-scaled: its fixed 16 x 16
    (batch, head) problems are divided among the ranks (each rank owns
    16/world whole sequences, all heads).  Every other workload keeps its
    batch per rank (weak scaling)."""
    if w.get("strong"):
        if w["B"] % world:
            raise SystemExit(f"{w['desc']}: batch {w['B']} does not divide over {world} GPUs")
        return w["B"] // world, "strong"
    return w["B"], "weak"


def attention_kernel_table(w, B, res):
    g = gemm_flops(B, w["H"], w["T"], w["D"], w["causal"])
    kflops = {KERNELS[0]: 2 * g, KERNELS[1]: 0, KERNELS[2]: 4 * g, KERNELS[3]: 3 * g}
    per = res["per_kernel_ms"]
    table = {n: {"ms": round(per[n], 4), "share": round(per[n] / sum(per.values()), 3),
                 "tflops": round(kflops[n] / (per[n] * 1e-3) / 1e12, 1) if kflops[n] else None,
                 "flops_per_launch": kflops[n]}
             for n in KERNELS}
    return kflops, table


def run_ours(args, w):
    rank, world, local = dist_init(args.gpus)
    if w is WORKLOADS["config5"] and world > 1:
        try:
            run_ring(args, w, rank, world, local)
        finally:
            import torch.distributed as dist_

            dist_.destroy_process_group()
        return
    B, scaling = shard_batch(w, world)
    H, T, D = w["H"], w["T"], w["D"]
    res = measure_attention(args, w, B, rank, world, local, with_e2e=True)
    # the bf16 configuration closest to the tensor-peak target, beside the
    # headline fp32 line (strong-scaled: 256 / N heads per GPU)
    sub = None
    if args.workload == "config2":
        w3 = WORKLOADS["config3"]
        B3, scaling3 = shard_batch(w3, world)
        sub = (w3, B3, scaling3, measure_attention(args, w3, B3, rank, world, local, with_e2e=False))

    peaks = measured_peaks()
    bf16_peak = float(peaks.get("bf16_tflops", 1590.0))
    bf16_src = "bf16 dense burst, MEASURED_PEAKS.json" if peaks else "bf16 dense, fallback 1.59 PF (no MEASURED_PEAKS.json)"
    if w["dtype"] == "f32":
        peak = tf32_peak_tflops() if rank == 0 else 0.0
        peak_note = "tf32 dense, cuBLAS 8192^3 measured in this run (best of 10)"
    else:
        peak, peak_note = bf16_peak, bf16_src
    cpu = cpu_baseline(w) if (world == 1 and rank == 0) else None

    if rank != 0:
        barrier(world)
        if world > 1:
            import torch.distributed as dist_

            dist_.destroy_process_group()
        return
    kflops, kernel_table = attention_kernel_table(w, B, res)
    per = res["per_kernel_ms"]
    total = world * path_flops(B, H, T, D, w["causal"])
    ms = res["ms"]
    value = total / (ms / args.steps * 1e-3) / 1e12
    e2e_steps = res["e2e_steps"]
    e2e_value = total / (res["ms_e2e"] / e2e_steps * 1e-3) / 1e12
    dom = max((n for n in KERNELS if kflops[n] > 0), key=lambda n: per[n])
    achieved = kflops[dom] / (per[dom] * 1e-3) / 1e12
    traffic = None
    tpath = ROOT / "profiles" / "roofline_traffic.json"
    if tpath.exists():
        try:
            tj = json.loads(tpath.read_text())
            entry = tj.get(f"{args.workload}/{dom}")
            if entry:
                traffic = entry["dram_bytes_per_launch"]
        except Exception:
            traffic = None
    eb = {"f32": 4, "bf16": 2}[w["dtype"]]
    nbytes = B * H * T * D * eb
    tf32_half = bf16_peak / 2
    roofline = {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(achieved / peak, 3) if peak else None,
                "peak_source": peak_note, "flops_per_launch": kflops[dom], "traffic": traffic,
                "frac_of_bf16_burst": round(achieved / bf16_peak, 3)}
    if w["dtype"] == "f32":
        roofline["frac_of_tf32_half_bf16"] = round(achieved / tf32_half, 3)
        roofline["tf32_half_bf16_tflops"] = round(tf32_half, 1)
    per_gpu = value / world
    pct = {"of_dtype_peak": round(100 * per_gpu / peak, 1) if peak else None, "dtype_peak_tflops": round(peak, 1),
           "dtype_peak_source": peak_note, "of_bf16_dense_peak": round(100 * per_gpu / bf16_peak, 1)}
    if w["dtype"] == "f32":
        pct["of_tf32_half_bf16_peak"] = round(100 * per_gpu / tf32_half, 1)
    par = (f"batch x head shards over {world} GPU(s), no collective in the step: "
           + ("each GPU owns its own sequences (weak scaling)" if scaling == "weak"
              else f"the fixed {w['B']} x {H} (batch, head) problems divided among the GPUs (strong scaling)"))
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": "fp32 I/O, tf32 tcgen05 MMA" if w["dtype"] == "f32" else "bf16 I/O, bf16 tcgen05 MMA",
        "data": f"synthetic: q,k,v ~ {w['qkv_scale']}*N(0,1), dO ~ {w['do_scale']}*N(0,1), seeded per rank",
        "config": {"workload": w["desc"], "batch_per_gpu": B, "global_batch": B * world, "heads": H, "seq_len": T,
                   "head_dim": D, "causal": w["causal"], "parallelism": par,
                   "l2": f"working set {9 * nbytes / 1e6:.0f} MB per GPU > 126 MB L2; no flush"},
        "pct_of_tensor_peak": pct,
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "h2d_bytes_per_step": 4 * nbytes,
                "d2h_bytes_per_step": 4 * nbytes, "ms_per_step": round(res["ms_e2e"] / e2e_steps, 4),
                "steps": e2e_steps,
                "path": "ctfa_forward + ctfa_backward (C ABI) with pinned host buffers; each step's H2D and D2H "
                        "copies run on their own streams, overlapping the neighbouring steps' compute",
                "copies_only_ms_per_step": round(res["ms_copies"] / e2e_steps, 4),
                "of_copy_floor": round(res["ms_copies"] / res["ms_e2e"], 3),
                "copy_floor_gbs_per_direction": round(4 * nbytes / (res["ms_copies"] / e2e_steps * 1e-3) / 1e9, 1)},
        # per step: forward (tf32 rounding inside it), delta pass, dK/dV, dQ
        "gpu_launches": 4 * args.steps,
        "roofline": roofline,
        "kernels": kernel_table,
        "per_rank": res["per_rank"],
        "cpu_baseline": cpu,
        "clocks": res["clocks"],
    }
    if sub is not None:
        w3, B3, scaling3, r3 = sub
        k3, t3 = attention_kernel_table(w3, B3, r3)
        total3 = world * path_flops(B3, w3["H"], w3["T"], w3["D"], True)
        v3 = total3 / (r3["ms"] / args.steps * 1e-3) / 1e12
        dom3 = max((n for n in KERNELS if k3[n] > 0), key=lambda n: r3["per_kernel_ms"][n])
        out["config3_bf16"] = {
            "workload": w3["desc"], "batch": w3["B"], "heads": w3["H"], "seq_len": w3["T"], "head_dim": w3["D"],
            "causal": True, "scaling": scaling3, "batch_per_gpu": B3,
            "value": round(v3, 2), "unit": "TFLOP/s", "ms_per_step": round(r3["ms"] / args.steps, 4),
            "frac_of_bf16_burst_per_gpu": round(v3 / world / bf16_peak, 3), "bf16_peak_tflops": bf16_peak,
            "bf16_peak_source": bf16_src, "kernels": t3,
            "dominant_kernel": {"kernel": dom3, "tflops": t3[dom3]["tflops"],
                                "frac_of_bf16_burst": round(t3[dom3]["tflops"] / bf16_peak, 3)},
            "per_rank": r3["per_rank"], "clocks": r3["clocks"],
            "gpu_launches": 4 * args.steps,
        }
    print(json.dumps(out), flush=True)
    barrier(world)
    if world > 1:
        import torch.distributed as dist_

        dist_.destroy_process_group()


# ---------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------
def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as orc

    lib = orc.load_reference_cuda()
    if lib is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libctref.so was not built "
                          "(needs the reference tree at build time)"}))
        return
    import torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, H, T, D = w["B"], w["H"], w["T"], w["D"]
    if w["dtype"] != "f32":
        print(json.dumps({"impl": "reference", "unavailable": "bench reference arm runs the fp32 workload only"}))
        return
    gen = torch.Generator().manual_seed(w["seed"] * 1000)
    shape = (B, H, T, D)
    q, k, v = ((torch.randn(shape, generator=gen) * w["qkv_scale"]).to(dev) for _ in range(3))
    do = (torch.randn(shape, generator=gen) * w["do_scale"]).to(dev)

    def step():
        rc = lib.ctref_forward_backward(0, q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(), None, None,
                                        None, None, B, H, T, D)
        if rc != 0:
            raise RuntimeError(f"reference FlashAttentionLayer returned CUDA error {rc}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize(dev)
    ms = s.elapsed_time(e)
    flops = path_flops(B, H, T, D, False)  # the reference computes the full (non-causal) attention
    value = flops / (ms / args.steps * 1e-3) / 1e12
    out = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 4),
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32 (SIMT CUDA cores)",
        "data": "synthetic, same distributions as the ours arm",
        "config": {"workload": w["desc"], "batch_per_gpu": B, "global_batch": B, "heads": H, "seq_len": T,
                   "head_dim": D, "causal": False,
                   "note": "the reference kernel has no causal mask; FLOPs counted at 14*B*H*T^2*D, the work it does"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "kind": "reference", "cores": 0,
                         "sample": "full workload; the reference's own implementation of this path is CUDA "
                                   "(FlashAttentionLayer<float> from oracle/_ref), timed on one B200"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "clocks": clocks.summary(),
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# config 4: NanoGPT training step around this repository's attention
# ---------------------------------------------------------------------------
def run_config4(args, w):
    """The reference NanoGPT architecture (token + position embedding, 6 blocks
    of LayerNorm -> attention -> LayerNorm -> ReLU MLP with no residuals,
    unembedding, softmax, cross-entropy on the probabilities, the reference's
    Adam) from cudatransformer_b200.nanogpt: every block's LayerNorms, QKV
    projection, attention, output projection and ReLU MLP run on this
    library's kernels, the embeddings, unembedding, softmax, loss and Adam as
    PyTorch ops (plumbing), fp32.  A step = forward, backward and
    one Adam update on a fresh batch; steps are stateful, so the warm-up steps
    are part of the training run and the loss of every step is kept.

    Reported: step time; the share of it spent in attention and in the two
    projections (the same work timed alone with CUDA events); and the loss of
    each step against an fp64 restatement of the same model and optimizer
    (oracle/nanogpt_oracle.py, the checker) fed the same weights and tokens.
    The reference's own NanoGPT is not run: its position embedding reads and
    writes past its table for batch > 1 and its AttentionLayer backward
    divides by zero (F3)."""
    import numpy as np
    import torch

    from cudatransformer_b200 import FlashAttentionLayer
    from cudatransformer_b200 import nanogpt as model
    from cudatransformer_b200 import projection_layers as pl

    rank, world, local = dist_init(args.gpus)
    if rank != 0:
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, T, D, L, V, E = w["B"], w["H"], w["T"], w["D"], w["layers"], w["vocab"], w["H"] * w["D"]

    init = model.init_parameters(model.parameter_shapes(L, H, D, V, T, w["mlp"]), w["seed"])
    n_steps = args.warmup + args.steps
    brng = np.random.default_rng(w["seed"] + 1000)
    data = []
    for _ in range(n_steps):
        ids = brng.integers(0, V, size=(B, T + 1), dtype=np.int64)
        data.append((ids[:, :-1].copy(), ids[:, 1:].copy()))

    params = {k: torch.tensor(v, device=dev).requires_grad_() for k, v in init.items()}
    opt = model.ReferenceAdam(params, lr=w["lr"])
    losses, times = [], []
    with ClockSampler(local) as clocks:
        for ids_np, tgt_np in data:
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s_ev.record()
            ids = torch.as_tensor(ids_np, device=dev)
            tgt = torch.as_tensor(tgt_np, device=dev)
            loss = model.train_step(params, opt, ids, tgt, L, H, D, w["causal"])
            lval = float(loss)  # device -> host read of the step's loss
            e_ev.record()
            torch.cuda.synchronize()
            times.append(s_ev.elapsed_time(e_ev))
            losses.append(lval)
    timed = times[args.warmup:]
    ms = float(np.median(timed))

    def time_unit(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(reps):
            fn()
        e_ev.record()
        torch.cuda.synchronize()
        return s_ev.elapsed_time(e_ev) / reps

    # attention alone: per layer one forward (saving states) and one backward
    q, k, v, do = (torch.randn(B, H, T, D, device=dev) for _ in range(4))
    att = FlashAttentionLayer(D, H, causal=w["causal"])

    def att_unit():
        for _ in range(L):
            att.computeAttention(q, k, v, saveStates=True)
            att.computeBackward(q, k, v, do)
            att.clearCache()

    att_ms = time_unit(att_unit)

    # the two projections alone: per layer forward, input and parameter gradients
    x, dy = torch.randn(B, T, E, device=dev), torch.randn(B, T, E, device=dev)
    wts = [torch.randn(E, E, device=dev) * 0.02 for _ in range(4)]
    bs = [torch.zeros(E, device=dev) for _ in range(4)]
    gw = [torch.zeros(E, E, device=dev) for _ in range(4)]
    gb = [torch.zeros(E, device=dev) for _ in range(4)]

    def proj_unit():
        for _ in range(L):
            qq, kk, vv = pl.qkv_forward(x, wts[0], bs[0], wts[1], bs[1], wts[2], bs[2], H, D)
            pl.out_proj_forward(qq, wts[3], bs[3])
            pl.out_proj_backward(qq, dy, wts[3], gw[3], gb[3])
            pl.qkv_backward(x, qq, kk, vv, wts[0], wts[1], wts[2], gw[0], gb[0], gw[1], gb[1], gw[2], gb[2])

    proj_ms = time_unit(proj_unit)
    proj_flops = 24.0 * B * T * E * E * L  # QKV fwd 6, out fwd 2, dx 6 + dW 6, da 2 + dWo 2 (x B*T*E*H*D)

    # fp64 restatement of the same training run (loss oracle), on the GPU for
    # the full run; one step of it timed on the host cores as the CPU baseline
    from oracle import nanogpt_oracle as nano

    t0 = time.perf_counter()
    ref_losses = nano.train(init, data, L, H, D, causal=w["causal"], lr=w["lr"], device=str(dev))
    ref_seconds = time.perf_counter() - t0
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    t0 = time.perf_counter()
    nano.train(init, data[:1], L, H, D, causal=w["causal"], lr=w["lr"], device="cpu")
    cpu_step = time.perf_counter() - t0
    diffs = [abs(a - b) for a, b in zip(losses, ref_losses)]
    tokens = B * T
    out = {
        "metric": "NanoGPT training step time and attention share (config 4)",
        "value": round(tokens / (ms * 1e-3), 1),
        "unit": "tokens/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "dtype": "fp32 I/O; LayerNorm, attention, QKV / output projections and the ReLU MLP on this library "
                 "(tf32 tcgen05 GEMMs); embeddings, unembedding, softmax, loss and Adam PyTorch fp32",
        "data": "synthetic: weights N(0,0.02) (LayerNorm scale 1, biases 0), token ids uniform [0,65), seeded",
        "config": {"workload": w["desc"], "batch": B, "seq_len": T, "layers": L, "heads": H, "head_dim": D,
                   "causal": w["causal"],
                   "note": "causal (language-model mask)" if w["causal"] else "non-causal, as the reference's attention"},
        "attention_ms_per_step": round(att_ms, 3),
        "attention_share_of_step": round(att_ms / ms, 4),
        "projection_ms_per_step": round(proj_ms, 3),
        "projection_share_of_step": round(proj_ms / ms, 4),
        "projection_tflops": round(proj_flops / (proj_ms * 1e-3) / 1e12, 1),
        "losses": [round(x, 6) for x in losses],
        "restatement_fp64_losses": [round(x, 6) for x in ref_losses],
        "max_abs_loss_diff_vs_restatement": round(max(diffs), 6),
        "restatement": {"device": str(dev), "seconds": round(ref_seconds, 2),
                        "source": "oracle/nanogpt_oracle.py (fp64, PyTorch)"},
        "cpu_baseline": {"value": round(tokens / cpu_step, 1), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": "one training step of the fp64 restatement on the host cores"},
        "reference": {"unavailable": "the reference NanoGPT's embeddings replace the sequence dimension of a "
                                     "[batch, seq] input with the embedding width (Embedding.cu:43-46, :194-197), so "
                                     "no [batch, seq, vocab] output or loss curve exists (NanoGPT.cu:92-93); two runs "
                                     "of it faulted on a B200; its AttentionLayer backward divides by zero (F3); "
                                     "not run"},
        "clocks": clocks.summary(),
    }
    print(json.dumps(out), flush=True)


def run_projections(args, w):
    """The six projection GEMMs of one attention layer (QKV forward, output
    forward, output backward: dWo + dbo and da, QKV backward: dW + db and dx)
    through the C ABI.  The step and each GEMM alone are captured once into
    CUDA graphs, so the timed replays measure the device (at the config-4
    shapes a GEMM is shorter than the host's cost of preparing its launch);
    CUDA events on the replay stream.  value = the algorithmic FLOPs
    (24 * B*T*E*H*D) per step time."""
    import numpy as np
    import torch

    from cudatransformer_b200 import projection_layers as pl

    rank, world, local = dist_init(args.gpus)
    if rank != 0:
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, T, E, H, D = w["B"], w["T"], w["E"], w["H"], w["D"]
    HD = H * D
    dt = torch.float32 if w["dtype"] == "f32" else torch.bfloat16
    g = torch.Generator(device="cpu").manual_seed(w["seed"])
    mk = lambda *shape, scale=1.0: (torch.randn(*shape, generator=g) * scale).to(dt).to(dev)
    x, dy = mk(B, T, E), mk(B, T, E)
    wq, wk, wv = (mk(HD, E, scale=E ** -0.5) for _ in range(3))
    bq, bk, bv = (mk(HD, scale=0.1) for _ in range(3))
    wo, bo = mk(E, HD, scale=HD ** -0.5), mk(E, scale=0.1)
    gw = [torch.zeros_like(t) for t in (wq, wk, wv, wo)]
    gb = [torch.zeros_like(t) for t in (bq, bk, bv, bo)]
    q, k, v = (torch.empty(B, H, T, D, dtype=dt, device=dev) for _ in range(3))
    lib = pl._lib.load()
    code = pl._code(x)
    P = lambda t: None if t is None else t.data_ptr()
    y, dx, da = torch.empty(B, T, E, dtype=dt, device=dev), torch.empty(B, T, E, dtype=dt, device=dev), \
        torch.empty(B, H, T, D, dtype=dt, device=dev)

    def stream_ptr():
        return torch.cuda.current_stream(dev).cuda_stream

    # the C ABI directly (preallocated outputs), so each captured graph holds
    # exactly one library launch
    gemms = {
        "qkv_fwd": lambda: lib.ctfa_qkv_forward(P(x), P(wq), P(bq), P(wk), P(bk), P(wv), P(bv), P(q), P(k), P(v),
                                                B, T, E, H, D, code, stream_ptr()),
        "out_fwd": lambda: lib.ctfa_out_proj_forward(P(q), P(wo), P(bo), P(y), B, T, E, H, D, code, stream_ptr()),
        "out_dw": lambda: lib.ctfa_out_proj_backward(P(q), P(dy), None, P(gw[3]), P(gb[3]), None, B, T, E, H, D,
                                                     code, stream_ptr()),
        "out_da": lambda: lib.ctfa_out_proj_backward(None, P(dy), P(wo), None, None, P(da), B, T, E, H, D, code,
                                                     stream_ptr()),
        "qkv_dw": lambda: lib.ctfa_qkv_backward(P(x), P(q), P(k), P(v), None, None, None, P(gw[0]), P(gb[0]),
                                                P(gw[1]), P(gb[1]), P(gw[2]), P(gb[2]), None, B, T, E, H, D, code,
                                                stream_ptr()),
        "qkv_dx": lambda: lib.ctfa_qkv_backward(None, P(q), P(k), P(v), P(wq), P(wk), P(wv), None, None, None, None,
                                                None, None, P(dx), B, T, E, H, D, code, stream_ptr()),
    }
    names = list(gemms)
    f1 = 2.0 * B * T * E * HD
    flops = {"qkv_fwd": 3 * f1, "out_fwd": f1, "out_dw": f1, "out_da": f1, "qkv_dw": 3 * f1, "qkv_dx": 3 * f1}

    def run(fn):
        st = fn()
        if st != 0:
            raise RuntimeError(f"projection call failed: {pl._lib.status_name(st)}: {pl._lib.last_error()}")

    def step():
        for n in names:
            run(gemms[n])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    graphs = {}
    with torch.cuda.stream(side):
        for n in names + ["step"]:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=side):
                step() if n == "step" else run(gemms[n])
            graphs[n] = gr
    torch.cuda.synchronize()

    def timed(gr, reps):
        gr.replay()
        torch.cuda.synchronize()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(reps):
            gr.replay()
        e_ev.record()
        torch.cuda.synchronize()
        return s_ev.elapsed_time(e_ev) / reps

    with ClockSampler(local) as clocks:
        ms = timed(graphs["step"], args.steps)
        per = {n: timed(graphs[n], args.steps) for n in names}
    total = sum(flops.values())
    value = total / (ms * 1e-3) / 1e12
    dom = max(per, key=per.get)
    if dt == torch.float32:
        peak, peak_note = tf32_peak_tflops(), "tf32 dense, cuBLAS 8192^3 measured in this run (best of 10)"
    else:
        peak = float(measured_peaks().get("bf16_tflops", 1590.0))
        peak_note = "bf16 dense burst, MEASURED_PEAKS.json"
    achieved = flops[dom] / (per[dom] * 1e-3) / 1e12
    traffic = None
    try:
        entry = json.loads((ROOT / "profiles" / "roofline_traffic.json").read_text()).get(f"{args.workload}/{dom}")
        traffic = entry["dram_bytes_per_launch"] if entry else None
    except (OSError, ValueError, KeyError):
        traffic = None

    # CPU baseline: the same six products with PyTorch fp32 on the host cores,
    # on a sample of the rows (the reference has no CPU implementation)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    Bs = max(1, min(B, 2))
    xr = x[:Bs].float().cpu().reshape(-1, E)
    dyr = dy[:Bs].float().cpu().reshape(-1, E)
    wcat = torch.cat([wq, wk, wv], 0).float().cpu()
    woc = wo.float().cpu()

    def cpu_step():
        qkv = xr @ wcat.T
        a = qkv[:, :HD]
        a @ woc.T
        dyr.T @ a
        dyr @ woc
        qkv.T @ xr
        qkv @ wcat

    cpu_step()
    t0, n_cpu = time.perf_counter(), 0
    while time.perf_counter() - t0 < 3.0:
        cpu_step()
        n_cpu += 1
    cpu_s = (time.perf_counter() - t0) / n_cpu
    cpu_value = total * Bs / B / cpu_s / 1e12
    del graphs
    out = {
        "metric": "projection GEMMs of one attention layer, TFLOP/s",
        "value": round(value, 1),
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32 I/O, tf32 tcgen05 MMA" if dt == torch.float32 else "bf16 I/O, bf16 tcgen05 MMA",
        "data": "synthetic: N(0,1) activations and gradients, weights N(0,1/fan_in), seeded",
        "config": {"workload": w["desc"], "batch": B, "seq_len": T, "E": E, "heads": H, "head_dim": D,
                   "l2": "inputs reused across replays (the L2-resident regime of a training step)",
                   "timing": "CUDA-graph replays (one graph per GEMM, one for the step)"},
        "kernels": {n: {"ms": round(per[n], 4), "tflops": round(flops[n] / (per[n] * 1e-3) / 1e12, 1)}
                    for n in names},
        "roofline": {"kernel": dom, "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 3), "peak_source": peak_note,
                     "traffic": traffic, "flops_per_launch": flops[dom]},
        "cpu_baseline": {"value": round(cpu_value, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"the same six GEMMs on {Bs} of {B} sequences, PyTorch fp32 on the host"},
        "gpu_launches": 6 * args.steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    w = WORKLOADS[args.workload]
    if args.workload in ("config4", "config4causal"):
        run_config4(args, w)
    elif args.workload.startswith("proj_"):
        run_projections(args, w)
    elif args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()

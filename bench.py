#!/usr/bin/env python
"""bench.py -- decode-attention KV GB/s of BASELINE cfg 2 on 1..8 B200s (+ prefill TFLOP/s).

Workload: one batched decode step of a Qwen3-ASR-1.7B-shaped
decoder over 28 layers -- 256 independent sequences, KV lengths drawn uniformly from
[1024, 8192] (seed 0), 16 Q / 8 KV heads, head_dim 128, RoPE theta 1e6, bf16 K / fp16 V
cache ~N(0,1).  With N GPUs the fixed batch of 256 is split by KV bytes (greedy
longest-first, workload.shard_by_bytes): strong scaling, `value` = all 256 sequences'
KV bytes / the slowest rank's step time.  Per layer the step runs the fused QK-RMSNorm + RoPE +
cache-append kernel for the new token of every sequence and the split-KV decode
attention over [0, L+1).  Synthetic data; the cache (~135 GB) is far larger than L2,
so no flush is needed between steps.

Arms
  default            libsmol_b200 on N GPUs (one process per GPU; the 256 sequences are
                     sharded across the ranks, no collective on the data path;
                     --scaling weak gives every rank its own 256 instead)
  --impl reference   the reference's own CPU implementation (oracle/_ref, compiled
                     from the reference sources) on the host cores, rank 0 only

The JSON line carries `value` (device-timed, inputs resident), `e2e` (the same step
through the C ABI with host buffers: H2D of q/k/v and D2H of the output inside the
timed region), `roofline` of the decode kernel pair, `cpu_baseline`, `clocks`, a
`prefill` block with the cfg 5 causal prefill TFLOP/s (one layer, batch 4 x 32768,
KV heads split across the ranks with one all-gather of the outputs), and
`other_configs`: cfg 3 (128 images split by image) and cfg 4 (32 sequences split by
sequence) at every N, and at N = 1 also cfg 1, the device decoder step (Qwen3 and Gemma
settings), the whole SigLIP encoder, the audio encoder's attention windows, the device
prefill and the reference decoder driver against its decoder-level drop-in.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "smol-genius_b200"))

import numpy as np  # noqa: E402

import workload  # noqa: E402

DECODE_TRAFFIC_PER_ALG_BYTE = (304.548352e6 + 4.445440e6) / 304.381952e6
METRIC = "decode attn KV GB/s (% of HBM peak); prefill TFLOP/s; at 1/2/4/8 B200 vs CPU"
UNIT = "GB/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prefill-gather", choices=["kernel", "nccl"], default="kernel",
                    help="N>1: all-gather the prefill outputs inside the kernel (stores to every peer) or with NCCL "
                         "after it (measured: the in-kernel form is faster at 2, 4 and 8 GPUs)")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample budget in seconds (--impl reference: the cap per step)")
    ap.add_argument("--seqs", type=int, default=workload.CFG2["n_seqs"],
                    help="sequences of the cfg 2 batch (split across the GPUs; per GPU with --scaling weak)")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="strong: one fixed batch split across the GPUs (BASELINE cfg 2); weak: every GPU its own")
    ap.add_argument("--layers", type=int, default=workload.CFG2["layers"])
    ap.add_argument("--no-decode", action="store_true", help="prefill measurement only (profiling helper)")
    ap.add_argument("--no-configs", action="store_true", help="skip the cfg 1/3/4 block")
    ap.add_argument("--only-config", choices=["cfg1", "cfg3", "cfg4", "decoder", "audio", "siglip", "so400m",
                                              "gemma", "prefill", "dropin"],
                    default=None,
                    help="run one of the other measurements alone: cfg 1/3/4, the decoder step, the audio-encoder "
                         "windows, the whole SigLIP encoder, the So400m (head dim 72) attention, the Gemma-"
                         "configured decoder step, the device prefill, or the decoder-level drop-in against the "
                         "reference decoder on the host")
    ap.add_argument("--images", type=int, default=None, help="cfg 3 image count override")
    ap.add_argument("--prefill-shape", default=None, help="B,L override of the cfg 5 prefill shape")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return dict(FALLBACK_PEAKS, source="fallback")


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def allreduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def gpu_index(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = [p for p in vis.split(",") if p.strip()]
        if local < len(parts) and parts[local].strip().isdigit():
            return int(parts[local])
    return local


# ---------------------------------------------------------------------------
# CPU baseline: the reference's smol_causal_attention on the host cores
# ---------------------------------------------------------------------------
class CpuReference:
    """The compiled reference (oracle/_ref) on cfg-2 decode, on the host cores.

    Each call is smol_causal_attention(seq_q=1, seq_k=L+1) of one sequence and one layer
    (qkn_decoder.c:658-677) over fp32 K/V.  Six distinct full-length K/V buffers
    (~400 MB, more than a CPU's last-level cache) are generated once and cycled, so the
    timed calls stream their cache from DRAM like the GPU does; GB/s counts
    bf16-equivalent KV bytes so it is the same figure as the GPU's."""

    HQ, HKV, HD = 16, 8, 128

    def __init__(self, lens: np.ndarray, threads: int | None = None):
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import ctypes

        import pyoracle
        self.path = pyoracle.ref_path()
        self.lens = lens
        if self.path is None:
            return
        self.lib = ctypes.CDLL(self.path)
        self.nproc = os.cpu_count() or 1
        self.lib.smol_set_threads(ctypes.c_int(threads or min(self.nproc, 16)))
        self.threads = int(self.lib.smol_get_thread_count())
        f = self.lib.smol_causal_attention
        f.restype = None
        f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int]
        self.f = f
        rng = np.random.default_rng(7)
        maxl = int(lens.max()) + 1
        kv = self.HKV * self.HD
        self.bufs = [(rng.standard_normal((maxl, kv), dtype=np.float32),
                      rng.standard_normal((maxl, kv), dtype=np.float32)) for _ in range(6)]
        self.q = rng.standard_normal((1, self.HQ * self.HD), dtype=np.float32)
        self.out = np.zeros_like(self.q)
        self.i = 0

    @property
    def available(self) -> bool:
        return self.path is not None

    def run(self, seconds: float) -> dict:
        total_bytes, total_t, calls = 0, 0.0, 0
        scale = 1 / np.sqrt(self.HD)
        while total_t < seconds:
            L = int(self.lens[self.i % len(self.lens)]) + 1
            K, V = self.bufs[calls % len(self.bufs)]
            t0 = time.perf_counter()
            self.f(self.out.ctypes.data, self.q.ctypes.data, K.ctypes.data, V.ctypes.data, 1, L, self.HQ, self.HKV,
                   self.HD, scale, L - 1)
            total_t += time.perf_counter() - t0
            total_bytes += L * self.HKV * self.HD * 2 * 2
            calls += 1
            self.i += 1
        return {"value": total_bytes / total_t / 1e9, "unit": UNIT, "cores": self.threads, "nproc": self.nproc,
                "kind": "reference",
                "sample": f"{calls} single-query decode calls of smol_causal_attention from oracle/_ref (cfg-2 "
                          f"lengths+1, 16/8 heads, hd 128, one layer each, fp32 KV cycled over 6 buffers); "
                          f"GB/s counts bf16-equivalent KV bytes",
                "seconds": round(total_t, 3)}


def cpu_reference_decode(lens: np.ndarray, seconds: float) -> dict:
    ref = CpuReference(lens)
    if not ref.available:
        return {"unavailable": "compiled reference (oracle/_ref) not present"}
    return ref.run(seconds)


def cpu_reference_prefill() -> dict:
    """The compiled reference (oracle/_ref) on the host cores for the tensor-bound configs,
    one bounded sample each, reported as GFLOP/s of visible pairs (4 * hd FLOPs per pair
    and head) so it scales to the full workloads:
      cfg 3: smol_bidirectional_attention (single-threaded in the reference) on one image
             and one layer (1024 patches, 12 heads, hd 64, window {0, 1024});
      cfg 5: smol_causal_attention on one sequence of 4096 tokens, 16 / 8 heads, hd 128
             (the full 32768-token layer is 64x the pairs)."""
    import ctypes
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle
    path = pyoracle.ref_path()
    if path is None:
        return {"unavailable": "compiled reference (oracle/_ref) not present"}
    lib = ctypes.CDLL(path)
    lib.smol_set_threads(ctypes.c_int(min(os.cpu_count() or 1, 16)))
    threads = int(lib.smol_get_thread_count())
    rng = np.random.default_rng(11)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)   # noqa: E731
    out = {}
    N, h, hd = 1024, 12, 64
    q, k, v = (rng.standard_normal((N, h * hd), dtype=np.float32) for _ in range(3))
    o = np.zeros_like(q)
    ws = np.array([0, N], np.int32)
    t0 = time.perf_counter()
    lib.smol_bidirectional_attention(p(o), p(q), p(k), p(v), ctypes.c_int(N), ctypes.c_int(h), ctypes.c_int(hd),
                                     ctypes.c_float(0.125), p(ws), ctypes.c_int(1))
    t = time.perf_counter() - t0
    out["cfg3"] = {"gflops": round(workload.full_flops(N, h, hd) / t / 1e9, 2), "cores": 1,
                   "sample": "smol_bidirectional_attention, 1 image x 1 layer (1024 patches, 12 heads, hd 64)"}
    L, hq, hkv, hd = 4096, 16, 8, 128
    q = rng.standard_normal((L, hq * hd), dtype=np.float32)
    k, v = (rng.standard_normal((L, hkv * hd), dtype=np.float32) for _ in range(2))
    o = np.zeros_like(q)
    t0 = time.perf_counter()
    lib.smol_causal_attention(p(o), p(q), p(k), p(v), ctypes.c_int(L), ctypes.c_int(L), ctypes.c_int(hq),
                              ctypes.c_int(hkv), ctypes.c_int(hd), ctypes.c_float(1 / np.sqrt(hd)), ctypes.c_int(0))
    t = time.perf_counter() - t0
    out["cfg5"] = {"gflops": round(workload.causal_flops_square(L, hq, hd) / t / 1e9, 2), "cores": threads,
                   "sample": "smol_causal_attention, 1 sequence of 4096 tokens, 16/8 heads, hd 128 (causal)"}
    return out


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lens = workload.decode_lengths(workload.CFG2["n_seqs"], workload.CFG2["len_lo"], workload.CFG2["len_hi"], 0)
    # each step a bounded sample: the whole run stays near two minutes of CPU time
    per_step = max(0.1, min(args.cpu_seconds, 120.0 / max(1, args.steps + args.warmup)))
    ref = CpuReference(lens)
    if not ref.available:
        print(json.dumps({"impl": "reference", "unavailable": "compiled reference (oracle/_ref) not present"}))
        return
    vals = []
    cb = None
    for s in range(args.warmup + args.steps):
        cb = ref.run(per_step)
        if s >= args.warmup:
            vals.append(cb["value"])
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg2 batched decode attention (reference CPU, sampled sequences)",
                       "lengths": "U[1024,8192] seed 0", "heads": "16/8", "head_dim": 128},
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": cb["cores"], "kind": "reference",
                             "sample": cb["sample"]},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def fill_randn(t, gen, chunk_rows=1 << 20):
    import torch
    for r in range(0, t.shape[0], chunk_rows):
        seg = t[r:r + chunk_rows]
        seg.copy_(torch.randn(seg.shape, device=t.device, generator=gen, dtype=torch.float32))


def run_prefill(args, world, rank, pk):
    """cfg 5 causal prefill, one layer: batch 4 x 32768, 16/8 heads, hd 128.  With N
    GPUs rank r owns KV heads r*8/N.. (and their Q heads) and the per-rank outputs are
    all-gathered once per layer: by the prefill kernel itself, which stores every output
    tile to its slot in each peer's gather buffer (CUDA IPC mappings, NVLink), or by a
    separate NCCL all-gather (--prefill-gather nccl)."""
    import torch

    import smol_b200
    c = workload.CFG5
    B, L, hq, hkv, hd = c["batch"], c["seq"], c["n_heads"], c["n_kv_heads"], c["head_dim"]
    if args.prefill_shape:
        B, L = (int(x) for x in args.prefill_shape.split(","))
    heads = workload.kv_head_groups(hkv, world, rank)
    hkv_r = len(heads)
    hq_r = hq // hkv * hkv_r
    g = torch.Generator(device="cuda").manual_seed(55 + rank)
    q = torch.randn((B, L, hq_r * hd), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((B, L, hkv_r * hd), device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn((B, L, hkv_r * hd), device="cuda", generator=g).to(torch.float16)
    # bf16 output: the consumer (the output projection) takes bf16 operands, and the
    # all-gather moves 2 bytes per element
    out = torch.empty((B, L, hq_r * hd), device="cuda", dtype=torch.bfloat16)
    gathered = torch.empty((world,) + tuple(out.shape), device="cuda", dtype=out.dtype) if world > 1 else None
    stream = torch.cuda.current_stream()
    scale = 1 / np.sqrt(hd)
    # Measured on one box (ms per layer, fused vs NCCL): 4 GPUs 4.37 vs 5.56, 8 GPUs 2.72 vs 3.71.
    fused = world > 1 and args.prefill_gather == "kernel"
    opened, outs, check = [], None, None
    if world > 1:
        import torch.distributed as dist
        sync_t = torch.zeros(1, device="cuda")
    if fused:
        # Every rank maps every peer's gather buffer (CUDA IPC) and its prefill writes each
        # output tile to its own slot in all of them: the all-gather runs inside the kernel.
        handle, off = smol_b200.ipc_handle(gathered)
        meta = torch.tensor(list(handle) + list(off.to_bytes(8, "little")), dtype=torch.uint8, device="cuda")
        allmeta = torch.empty(world * 72, dtype=torch.uint8, device="cuda")
        dist.all_gather_into_tensor(allmeta, meta)
        allmeta = allmeta.cpu().numpy().reshape(world, 72)
        slot = out.numel() * out.element_size()
        bases = []
        for peer in range(world):
            if peer == rank:
                bases.append(gathered.data_ptr())
            else:
                b0 = smol_b200.ipc_open(bytes(allmeta[peer, :64]))
                opened.append(b0)
                bases.append(b0 + int.from_bytes(bytes(allmeta[peer, 64:]), "little"))
        outs = [bases[rank] + rank * slot] + [bases[peer] + rank * slot for peer in range(world) if peer != rank]

    def layer():
        if fused:
            smol_b200.prefill_attention_multi(outs, hq_r * hd, L * hq_r * hd, q, k, v, B, L, L, hq_r, hkv_r, hd, scale,
                                              stream=stream, bf16=True)
            dist.all_reduce(sync_t)   # device-side barrier: every rank's stores have landed
        else:
            smol_b200.prefill_attention(out, q, k, v, B, L, L, hq_r, hkv_r, hd, scale, stream=stream)
            if world > 1:
                dist.all_gather_into_tensor(gathered, out)

    if fused:   # the fused result equals prefill + NCCL all-gather, bit for bit
        layer()
        torch.cuda.synchronize()
        fused_copy = gathered.clone()
        smol_b200.prefill_attention(out, q, k, v, B, L, L, hq_r, hkv_r, hd, scale, stream=stream)
        dist.all_gather_into_tensor(gathered, out)
        torch.cuda.synchronize()
        check = bool(torch.equal(fused_copy, gathered))
        del fused_copy
        if not check:
            raise SystemExit(f"rank {rank}: fused prefill all-gather differs from prefill + NCCL all-gather")
    for _ in range(2):
        layer()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        layer()
    e1.record()
    torch.cuda.synchronize()
    ms = allreduce_max(e0.elapsed_time(e1) / reps, world)
    flops = workload.causal_flops_square(L, hq, hd) * B
    tf = flops / (ms * 1e-3) / 1e12
    smol_b200.check(smol_b200.last_error(), "prefill")
    for b0 in opened:
        smol_b200.ipc_close(b0)
    gather = ("" if world == 1 else
              (f", KV heads split over {world} GPUs; outputs all-gathered inside the prefill kernel (every output "
               "row stored to each peer's buffer over NVLink, CUDA IPC)" if fused
               else f", KV heads split over {world} GPUs + NCCL all-gather"))
    return {"workload": f"cfg5 causal prefill, 1 layer, batch {B} x {L}, GQA 16/8, hd 128, bf16 output" + gather,
            "gather_matches_nccl": check,
            "gather_bytes_per_layer": (world - 1) * world * out.numel() * out.element_size(),
            "gather_bytes_per_gpu_out": (world - 1) * out.numel() * out.element_size(),
            "tflops": round(tf, 1), "ms_per_layer": round(ms, 3), "flops_per_layer": flops,
            "frac_of_bf16_peak": round(tf / world / pk["bf16_tflops"], 4), "per_gpu_tflops": round(tf / world, 1),
            "peak": pk["bf16_tflops"], "peak_source": pk["source"], "kernel": "tcgen05 prefill2_kernel<128>"}


def _ev():
    import torch
    return torch.cuda.Event(enable_timing=True)


def _graph(fn):
    """Capture fn's launches into a CUDA graph (warm-up on the capture stream first, so
    one-time set-up such as kernel attributes happens outside the capture)."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def _time_graph(g, reps: int) -> float:
    """Mean ms per replay of graph g (3 warm-up replays)."""
    import torch
    for _ in range(3):
        g.replay()
    a, b = _ev(), _ev()
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_cfg1() -> dict:
    """cfg 1: one layer, prefill 512 then 128 decode steps (batch 1, 16/8, hd 128)."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(11)
    c = workload.CFG1
    hq, hkv, hd, P, T = c["n_heads"], c["n_kv_heads"], c["head_dim"], c["prefill"], c["decode_steps"]
    cap = P + T + 8
    kv = hkv * hd
    kp = torch.zeros((cap, kv), dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros((cap, kv), dtype=torch.float16, device="cuda")
    cos_h = np.zeros((cap, hd), np.float32)
    sin_h = np.zeros((cap, hd), np.float32)
    smol_b200.compute_rope(cos_h, sin_h, np.arange(cap, dtype=np.int32), cap, hd, c["theta"])
    dc, ds = torch.from_numpy(cos_h).cuda(), torch.from_numpy(sin_h).cuda()
    qn = (1 + 0.02 * torch.randn(hd, device="cuda", generator=g))
    kn = (1 + 0.02 * torch.randn(hd, device="cuda", generator=g))
    q = torch.randn((P, hq * hd), device="cuda", generator=g)
    k = torch.randn((P, kv), device="cuda", generator=g)
    v = torch.randn((P, kv), device="cuda", generator=g)
    qb = torch.empty((P, hq * hd), dtype=torch.bfloat16, device="cuda")
    out = torch.empty((1, P, hq * hd), device="cuda")
    pos = torch.arange(P, dtype=torch.int32, device="cuda")
    slots = pos.to(torch.int64)
    scale = 1 / np.sqrt(hd)

    def prefill():
        smol_b200.qknorm_rope_append(q, k, v, P, hq, hkv, hd, qn, kn, 1e-6, dc, ds, False, pos, slots, None, qb,
                                     kp, vp, cap)
        smol_b200.prefill_attention(out, qb, kp, vp, 1, P, P, hq, hkv, hd, scale,
                                    strides=((hq * hd, 0), (hq * hd, 0), (kv, 0), (kv, 0)))
    pre_ms = _time_graph(_graph(prefill), 20)
    q1 = torch.randn((1, hq * hd), device="cuda", generator=g)
    k1 = torch.randn((1, kv), device="cuda", generator=g)
    v1 = torch.randn((1, kv), device="cuda", generator=g)
    qr = torch.empty_like(q1)
    o1 = torch.empty_like(q1)
    lens = [torch.tensor([P + t], dtype=torch.int32, device="cuda") for t in range(T)]
    lens1 = [torch.tensor([P + t + 1], dtype=torch.int32, device="cuda") for t in range(T)]
    slot = [l.to(torch.int64) for l in lens]
    r0 = torch.zeros(1, dtype=torch.int64, device="cuda")
    ws = torch.empty(smol_b200.decode_workspace_bytes(1, cap, hq, hkv, hd), dtype=torch.uint8, device="cuda")

    def decode_all():
        for t in range(T):
            smol_b200.qknorm_rope_append(q1, k1, v1, 1, hq, hkv, hd, qn, kn, 1e-6, dc, ds, False, lens[t], slot[t],
                                         qr, None, kp, vp, cap)
            smol_b200.decode_attention(o1, qr, kp, vp, cap, r0, lens1[t], 1, cap, hq, hkv, hd, scale, ws)
    dec_ms = _time_graph(_graph(decode_all), 3) / T
    smol_b200.check(smol_b200.last_error(), "cfg1")
    return {"prefill_512_ms": round(pre_ms, 4),
            "prefill_tflops": round(workload.causal_flops_square(P, hq, hd) / (pre_ms * 1e-3) / 1e12, 1),
            "decode_step_us": round(dec_ms * 1e3, 2),
            "note": "one layer, batch 1: latency-bound; prefill (append + attention) and the 128-step decode "
                    "loop (append + split + combine per step) each replayed as one CUDA graph"}


def run_cfg3(pk, images: int | None = None, layers: int | None = None, world: int = 1, rank: int = 0) -> dict:
    """cfg 3: SigLIP attention, 128 images x 12 layers, 1024 patches, 12 heads, hd 64.
    With N GPUs rank r attends images workload.shard_evenly(128, N, r); the time is the
    slowest rank's and the TFLOP/s count all 128 images."""
    import torch

    import smol_b200
    ev = _ev
    g = torch.Generator(device="cuda").manual_seed(13 + rank)
    c = dict(workload.CFG3)
    if images:
        c["images"] = images
    if layers:
        c["layers"] = layers
    total_images = c["images"]
    B = len(workload.shard_evenly(total_images, world, rank))
    N, h3, hd3 = c["patches"], c["n_heads"], c["head_dim"]
    q3 = torch.randn((B, N, h3 * hd3), device="cuda", generator=g).to(torch.bfloat16)
    k3 = torch.randn((B, N, h3 * hd3), device="cuda", generator=g).to(torch.bfloat16)
    v3 = torch.randn((B, N, h3 * hd3), device="cuda", generator=g).to(torch.float16)
    o3 = torch.empty((B, N, h3 * hd3), device="cuda")

    a, b = ev(), ev()

    def siglip():
        for _ in range(c["layers"]):
            smol_b200.prefill_attention(o3, q3, k3, v3, B, N, N, h3, h3, hd3, 1 / 8.0, mask_kind=smol_b200.MASK_FULL)
    siglip()
    torch.cuda.synchronize()
    barrier(world)
    a.record()
    siglip()
    b.record()
    torch.cuda.synchronize()
    ms3 = allreduce_max(a.elapsed_time(b), world)
    fl3 = workload.full_flops(N, h3, hd3) * total_images * c["layers"]
    tf = fl3 / (ms3 * 1e-3) / 1e12
    return {"workload": f"{total_images} images x {c['layers']} layers" +
                        (f", {B} images per GPU on {world} GPUs (split by image, no collective)" if world > 1 else ""),
            "ms": round(ms3, 3), "tflops": round(tf, 1),
            "frac_of_bf16_peak": round(tf / world / pk["bf16_tflops"], 4),
            "flops": fl3, "kernel": "prefill2_kernel<64> (full mask)"}


def run_audio_windows(pk, segments: int = 64) -> dict:
    """Windowed bidirectional attention of the Qwen3-ASR audio encoder (encoder.c:426-465):
    ten 104-token windows per segment, 16 heads, hd 64, one layer; FLOPs count only the
    pairs inside a window (4 * hd per pair and head)."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(19)
    win, n_win, h, hd = 104, 10, 16, 64
    N = win * n_win
    q = torch.randn((segments, N, h * hd), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((segments, N, h * hd), device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn((segments, N, h * hd), device="cuda", generator=g).to(torch.float16)
    o = torch.empty((segments, N, h * hd), device="cuda")
    ws = torch.arange(0, N + 1, win, dtype=torch.int32, device="cuda")

    def layer():
        smol_b200.prefill_attention(o, q, k, v, segments, N, N, h, h, hd, 1 / 8.0, mask_kind=smol_b200.MASK_WINDOWS,
                                    window_starts=ws)
    layer()
    a, b = _ev(), _ev()
    a.record()
    for _ in range(5):
        layer()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / 5
    fl = 4 * hd * h * n_win * win * win * segments
    return {"workload": f"{segments} segments x {n_win} windows of {win} tokens, 16 heads, hd 64, one layer",
            "ms": round(ms, 4), "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
            "frac_of_bf16_peak": round(fl / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4), "flops": fl,
            "kernel": "prefill2_kernel<64> (window mask)"}


def run_so400m_attention(pk, images: int = 128, layers: int = 27) -> dict:
    """SmolVLM's vision tower attention (SigLIP-So400m: 729 patches of a 378-pixel tile,
    16 heads of 72, 27 layers): bidirectional, one call per layer over 128 tiles.  The
    72-column heads run the 128-wide kernel (columns past 72 read as zero), and FLOPs
    count the real head dim, so that padding shows in the fraction."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(29)
    N, h, hd = 729, 16, 72
    q = torch.randn((images, N, h * hd), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((images, N, h * hd), device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn((images, N, h * hd), device="cuda", generator=g).to(torch.float16)
    o = torch.empty((images, N, h * hd), device="cuda", dtype=torch.bfloat16)

    def tower():
        for _ in range(layers):
            smol_b200.prefill_attention(o, q, k, v, images, N, N, h, h, hd, 1 / hd ** 0.5,
                                        mask_kind=smol_b200.MASK_FULL)
    tower()
    a, b = _ev(), _ev()
    torch.cuda.synchronize()
    a.record()
    tower()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    fl = workload.full_flops(N, h, hd) * images * layers
    tf = fl / (ms * 1e-3) / 1e12
    return {"workload": f"SigLIP-So400m attention, {images} tiles x {layers} layers, 729 patches, 16 heads of 72, "
                        "bf16 output (q/k/v 215 MB each, more than L2)",
            "ms": round(ms, 3), "tflops": round(tf, 1), "frac_of_bf16_peak": round(tf / pk["bf16_tflops"], 4),
            "flops": fl, "kernel": "prefill2_kernel<128> on 72-column heads (full mask)"}


def run_siglip_encoder(pk, images: int | None = None) -> dict:
    """The whole SigLIP-base encoder on the device (siglip_forward, Part 5): cfg 3's 128
    images of 512 x 512 (1024 patches of 16 x 16), 12 layers, hidden 768, 12 heads, ffn
    3072; random weights.  FLOPs: the GEMMs (patch embedding and per layer Q, K, V, O,
    fc1, fc2) plus the attention's 4 * hd per pair and head."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(23)
    n_img = images or workload.CFG3["images"]
    H, NH, F, L, P, S = 768, 12, 3072, workload.CFG3["layers"], 16, 512
    NP = (S // P) ** 2
    kin = 3 * P * P

    def mat(r, c):
        return (torch.randn((r, c), device="cuda", generator=g) / c ** 0.5).to(torch.bfloat16)

    def vec(n, mean=0.0):
        return mean + 0.02 * torch.randn(n, device="cuda", generator=g)

    layers = [{"ln1_w": vec(H, 1.0), "ln1_b": vec(H), "wq": mat(H, H), "wk": mat(H, H), "wv": mat(H, H),
               "wo": mat(H, H), "bq": vec(H), "bk": vec(H), "bv": vec(H), "bo": vec(H), "ln2_w": vec(H, 1.0),
               "ln2_b": vec(H), "fc1": mat(F, H), "b1": vec(F), "fc2": mat(H, F), "b2": vec(H)} for _ in range(L)]
    keep = dict(patch_w=mat(H, kin), patch_b=vec(H), pos=vec(NP * H), post_w=vec(H, 1.0), post_b=vec(H))
    model = smol_b200.siglip_model(H, NH, F, P, S, NP, 1e-6, keep["patch_w"], kin, keep["patch_b"], keep["pos"],
                                   keep["post_w"], keep["post_b"], layers)
    imgs = torch.rand((n_img, 3, S, S), device="cuda", generator=g) * 2 - 1
    out = torch.empty((n_img, NP, H), device="cuda")
    ws = torch.empty(smol_b200.siglip_workspace_bytes(model, n_img), dtype=torch.uint8, device="cuda")
    smol_b200.siglip_forward(out, imgs, n_img, model, ws)
    a, b = _ev(), _ev()
    a.record()
    smol_b200.siglip_forward(out, imgs, n_img, model, ws)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    T = n_img * NP
    gemm = 2 * T * H * kin + L * 2 * T * H * (4 * H + 2 * F)
    attn = L * workload.full_flops(NP, NH, H // NH) * n_img
    fl = gemm + attn
    return {"workload": f"SigLIP-base encoder, {n_img} images x {L} layers, 1024 patches, hidden 768, ffn 3072",
            "ms": round(ms, 3), "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
            "frac_of_bf16_peak": round(fl / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4), "flops": fl,
            "gemm_flops": gemm, "attention_flops": attn,
            "kernels": "gemm_bf16_kernel (tcgen05), prefill2_kernel<64>, layer_norm_kernel, unfold / convert"}


def run_cfg4(pk=None, world: int = 1, rank: int = 0) -> dict:
    """cfg 4: PaliGemma prefix-LM, batch 32, 18 layers, MQA 8/1, hd 256; 128-step suffix.
    With N GPUs rank r owns sequences workload.shard_evenly(32, N, r); times are the
    slowest rank's, FLOPs and bytes count all 32 sequences."""
    import torch

    import smol_b200
    ev = _ev
    g = torch.Generator(device="cuda").manual_seed(17 + rank)
    c = workload.CFG4
    P4, S4, h4, hkv4, hd4, L4 = c["prefix"], c["suffix"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["layers"]
    B_all = c["batch"]
    B4 = len(workload.shard_evenly(B_all, world, rank))
    tot = P4 + S4
    kv4 = hkv4 * hd4
    q4 = torch.randn((B4, P4, h4 * hd4), device="cuda", generator=g).to(torch.bfloat16)
    # every layer has its own cache slab (18 x 32 x 448 rows = 264 MB for K+V, more than L2)
    kp4 = torch.randn((L4 * B4 * tot, kv4), device="cuda", generator=g).to(torch.bfloat16)
    vp4 = torch.randn((L4 * B4 * tot, kv4), device="cuda", generator=g).to(torch.float16)
    o4 = torch.empty((B4, P4, h4 * hd4), device="cuda")
    # the same prefix with a bf16 output (the o-projection's operand type): half the
    # output bytes, which a layer writes in one burst at the end of every work item
    o4h = torch.empty((B4, P4, h4 * hd4), device="cuda", dtype=torch.bfloat16)

    a, b = ev(), ev()

    def prefix(out=o4):
        for layer in range(L4):
            base = layer * B4 * tot
            smol_b200.prefill_attention(out, q4, kp4[base:], vp4[base:], B4, P4, P4, h4, hkv4, hd4, 1 / 16.0,
                                        mask_kind=smol_b200.MASK_PREFIX_LM, prefix_len=P4,
                                        strides=((h4 * hd4, P4 * h4 * hd4), (h4 * hd4, P4 * h4 * hd4),
                                                 (kv4, tot * kv4), (kv4, tot * kv4)))
    prefix()
    torch.cuda.synchronize()
    barrier(world)
    a.record()
    prefix()
    b.record()
    torch.cuda.synchronize()
    ms4 = allreduce_max(a.elapsed_time(b), world)
    prefix(o4h)
    torch.cuda.synchronize()
    barrier(world)
    a.record()
    prefix(o4h)
    b.record()
    torch.cuda.synchronize()
    ms4h = allreduce_max(a.elapsed_time(b), world)
    fl4 = workload.prefix_lm_flops(P4, P4, h4, hd4) * B_all * L4
    qd = torch.randn((B4, h4 * hd4), device="cuda", generator=g)
    od = torch.empty_like(qd)
    r04 = [torch.arange(B4, dtype=torch.int64, device="cuda") * tot + layer * B4 * tot for layer in range(L4)]
    ws4 = torch.empty(smol_b200.decode_workspace_bytes(B4, tot, h4, hkv4, hd4), dtype=torch.uint8, device="cuda")
    lens4 = [torch.full((B4,), P4 + t + 1, dtype=torch.int32, device="cuda") for t in range(S4)]

    def suffix():
        for t in range(S4):
            for layer in range(L4):
                smol_b200.decode_attention(od, qd, kp4, vp4, L4 * B4 * tot, r04[layer], lens4[t], B4, tot, h4, hkv4,
                                           hd4, 1 / 16.0, ws4)
    graph = _graph(suffix)
    torch.cuda.synchronize()
    barrier(world)
    ms_s = allreduce_max(_time_graph(graph, 3), world)
    del graph
    suf_bytes = sum(B_all * (P4 + t + 1) * kv4 * 2 * 2 for t in range(S4)) * L4
    smol_b200.check(smol_b200.last_error(), "cfg4")
    tf = fl4 / (ms4 * 1e-3) / 1e12
    gbs = suf_bytes / (ms_s * 1e-3) / 1e9
    res = {"prefix_ms_18_layers": round(ms4, 3), "prefix_tflops": round(tf, 1),
           "prefix_bf16_out_ms": round(ms4h, 3), "prefix_bf16_out_tflops": round(fl4 / (ms4h * 1e-3) / 1e12, 1),
           "suffix_128_steps_ms": round(ms_s, 2), "suffix_step_us": round(ms_s * 1e3 / S4, 1),
           "suffix_kv_gbs": round(gbs, 1),
           "kernels": "prefill_kernel<256> (prefix-LM mask) + decode_split_kernel<256> (MQA group 8); "
                      "the 128-step x 18-layer suffix replayed as one CUDA graph"}
    if pk is not None:
        res["prefix_frac_of_bf16_peak"] = round(tf / world / pk["bf16_tflops"], 4)
        res["prefix_bf16_out_frac_of_bf16_peak"] = round(fl4 / (ms4h * 1e-3) / 1e12 / world / pk["bf16_tflops"], 4)
        res["suffix_hbm_frac"] = round(gbs / world / pk["hbm_gbs"], 4)
    if world > 1:
        res["workload"] = f"{B_all} sequences, {B4} per GPU on {world} GPUs (split by sequence, no collective)"
    return res


def run_decoder(pk, batch: int = 1, steps: int = 50) -> dict:
    """The device-resident decoder step (smol_b200_qkn_decode_step) at Qwen3-0.6B size:
    28 layers, hidden 1024, 16/8 heads, head_dim 128, SwiGLU 3072, vocab 151936 (tied
    lm_head), random bf16 weights, `batch` sequences with 512 cached tokens each.  One
    step = one greedy token per sequence, replayed from a CUDA graph.  Bytes per step =
    every weight once (the products stream them) + the attended K/V."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(21)
    H, Lr, HQ, HKV, HD, I, V = 1024, 28, 16, 8, 128, 3072, 151936
    qd, kvd, P, cap = HQ * HD, HKV * HD, 512, 1024

    def bf(rows, cols):
        return (torch.randn((rows, cols), device="cuda", generator=g) / np.sqrt(cols)).to(torch.bfloat16)

    def near(n, mean):
        return (mean + 0.02 * torch.randn(n, device="cuda", generator=g)).contiguous()

    emb = torch.randn((V, H), device="cuda", generator=g).to(torch.bfloat16)
    layers = [{"wq": bf(qd, H), "wk": bf(kvd, H), "wv": bf(kvd, H), "wo": bf(H, qd), "gate_up": bf(2 * I, H),
               "down": bf(H, I), "input_norm": near(H, 1.0), "post_attn_norm": near(H, 1.0),
               "q_norm": near(HD, 1.0), "k_norm": near(HD, 1.0)} for _ in range(Lr)]
    model = smol_b200.qkn_model(H, HQ, HKV, HD, I, V, 1e-6, emb, near(H, 1.0), layers)
    rows = Lr * batch * cap
    k_pool = torch.randn((rows, kvd), device="cuda", generator=g).to(torch.bfloat16)
    v_pool = torch.randn((rows, kvd), device="cuda", generator=g).to(torch.float16)
    row0 = (torch.arange(Lr * batch, device="cuda", dtype=torch.int64) * cap).contiguous()   # [layer][seq]
    kv_len = torch.full((batch,), P, dtype=torch.int32, device="cuda")
    cos_h = np.zeros((cap, HD), np.float32)
    sin_h = np.zeros((cap, HD), np.float32)
    smol_b200.compute_rope(cos_h, sin_h, np.arange(cap, dtype=np.int32), cap, HD, 1e6)
    cos_d, sin_d = torch.from_numpy(cos_h).cuda(), torch.from_numpy(sin_h).cuda()
    ws = torch.empty(smol_b200.qkn_step_workspace_bytes(model, batch, cap - 1), dtype=torch.uint8, device="cuda")
    tokens = torch.randint(0, V, (batch,), dtype=torch.int32, device="cuda", generator=g)

    def step():
        smol_b200.qkn_decode_step(model, batch, tokens, tokens, k_pool, v_pool, rows, row0, kv_len, cap - 1, cos_d,
                                  sin_d, ws, advance=True)
    ms = _time_graph(_graph(step), steps)
    smol_b200.check(smol_b200.last_error(), "decoder step")
    weight_bytes = (Lr * (qd * H + 2 * kvd * H + H * qd + 2 * I * H + H * I) + V * H) * 2
    mean_len = P + 4 + steps / 2 + 1          # cached tokens attended on average over the timed replays
    kv_bytes = int(Lr * batch * mean_len * kvd * 2 * 2)
    gbs = (weight_bytes + kv_bytes) / (ms * 1e-3) / 1e9
    return {"workload": f"Qwen3-0.6B-size decode step (28 layers, vocab 151936), batch {batch}, ~{P} cached tokens",
            "us_per_step": round(ms * 1e3, 1), "tokens_per_s": round(batch / (ms * 1e-3), 1),
            "bytes_per_step": weight_bytes + kv_bytes, "gbs": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm_gbs"], 4),
            "kernels": "gemv_bf16_kernel, qknorm_rope_append, decode_split_kernel (cluster), "
                       "argmax_part/final_kernel; one CUDA graph per step"}


def run_gemma_decoder(pk, batch: int = 1, steps: int = 30) -> dict:
    """The device decoder step in the Gemma configuration at PaliGemma's Gemma-2B size
    (paligemma.c:206-222 settings): 18 layers, hidden 2048, 8 heads / 1 KV head, head_dim
    256, GeGLU 16384, vocab 257216, embedding scale sqrt(2048), interleaved RoPE,
    attention softcap 50, every other layer sliding (window 4096, local theta 1e4),
    pre/post-FFN norms, no QK-norm; random bf16 weights, 512 cached tokens per sequence,
    replayed from a CUDA graph.  Bytes per step = every weight once + the attended K/V."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(29)
    H, Lr, HQ, HKV, HD, I, V = 2048, 18, 8, 1, 256, 16384, 257216
    qd, kvd, P, cap = HQ * HD, HKV * HD, 512, 1024

    def bf(rows, cols):
        return (torch.randn((rows, cols), device="cuda", generator=g) / np.sqrt(cols)).to(torch.bfloat16)

    def near(n, mean):
        return (mean + 0.02 * torch.randn(n, device="cuda", generator=g)).contiguous()

    emb = (torch.randn((V, H), device="cuda", generator=g) / np.sqrt(H)).to(torch.bfloat16)
    layers = [{"wq": bf(qd, H), "wk": bf(kvd, H), "wv": bf(kvd, H), "wo": bf(H, qd), "gate_up": bf(2 * I, H),
               "down": bf(H, I), "input_norm": near(H, 1.0), "post_attn_norm": near(H, 1.0),
               "pre_ffn_norm": near(H, 1.0), "post_ffn_norm": near(H, 1.0)} for _ in range(Lr)]
    tabs = {}
    for theta in (1e6, 1e4):
        c = np.zeros((cap, HD), np.float32)
        s_ = np.zeros((cap, HD), np.float32)
        smol_b200.compute_rope(c, s_, np.arange(cap, dtype=np.int32), cap, HD, theta, interleaved=True)
        tabs[theta] = (torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda())
    model = smol_b200.qkn_model(H, HQ, HKV, HD, I, V, 1e-6, emb, near(H, 1.0), layers, rope_interleaved=True,
                                activation=smol_b200.ACT_GEGLU, embed_normalizer=float(np.sqrt(H)),
                                attn_softcap=50.0, sliding_window=4096, rope_cos_local=tabs[1e4][0],
                                rope_sin_local=tabs[1e4][1], sliding=[l % 2 == 0 for l in range(Lr)])
    rows = Lr * batch * cap
    k_pool = torch.randn((rows, kvd), device="cuda", generator=g).to(torch.bfloat16)
    v_pool = torch.randn((rows, kvd), device="cuda", generator=g).to(torch.float16)
    row0 = (torch.arange(Lr * batch, device="cuda", dtype=torch.int64) * cap).contiguous()   # [layer][seq]
    kv_len = torch.full((batch,), P, dtype=torch.int32, device="cuda")
    ws = torch.empty(smol_b200.qkn_step_workspace_bytes(model, batch, cap - 1), dtype=torch.uint8, device="cuda")
    tokens = torch.randint(0, V, (batch,), dtype=torch.int32, device="cuda", generator=g)

    def step():
        smol_b200.qkn_decode_step(model, batch, tokens, tokens, k_pool, v_pool, rows, row0, kv_len, cap - 1,
                                  tabs[1e6][0], tabs[1e6][1], ws, advance=True)
    ms = _time_graph(_graph(step), steps)
    smol_b200.check(smol_b200.last_error(), "gemma decoder step")
    weight_bytes = (Lr * (qd * H + 2 * kvd * H + H * qd + 2 * I * H + H * I) + V * H) * 2
    mean_len = P + 4 + steps / 2 + 1
    kv_bytes = int(Lr * batch * mean_len * kvd * 2 * 2)
    gbs = (weight_bytes + kv_bytes) / (ms * 1e-3) / 1e9
    return {"workload": f"Gemma-2B-size decode step (PaliGemma settings, 18 layers, vocab 257216), batch {batch}",
            "us_per_step": round(ms * 1e3, 1), "tokens_per_s": round(batch / (ms * 1e-3), 1),
            "bytes_per_step": weight_bytes + kv_bytes, "gbs": round(gbs, 1), "hbm_frac": round(gbs / pk["hbm_gbs"], 4)}


def run_decoder_prefill(pk, n_tokens: int = 2048) -> dict:
    """The device prefill (smol_b200_qkn_prefill) at Qwen3-0.6B size: one sequence of
    n_tokens, 28 layers, hidden 1024, 16/8 heads, head_dim 128, SwiGLU 3072; random bf16
    weights.  FLOPs: the projections (2 * weights per token) plus the causal attention
    (4 * hd per visible pair and head)."""
    import torch

    import smol_b200
    g = torch.Generator(device="cuda").manual_seed(37)
    H, Lr, HQ, HKV, HD, I, V = 1024, 28, 16, 8, 128, 3072, 151936
    qd, kvd = HQ * HD, HKV * HD

    def bf(rows, cols):
        return (torch.randn((rows, cols), device="cuda", generator=g) / np.sqrt(cols)).to(torch.bfloat16)

    def near(n, mean):
        return (mean + 0.02 * torch.randn(n, device="cuda", generator=g)).contiguous()

    emb = torch.randn((V, H), device="cuda", generator=g).to(torch.bfloat16)
    layers = [{"wq": bf(qd, H), "wk": bf(kvd, H), "wv": bf(kvd, H), "wo": bf(H, qd), "gate_up": bf(2 * I, H),
               "down": bf(H, I), "input_norm": near(H, 1.0), "post_attn_norm": near(H, 1.0),
               "q_norm": near(HD, 1.0), "k_norm": near(HD, 1.0)} for _ in range(Lr)]
    model = smol_b200.qkn_model(H, HQ, HKV, HD, I, V, 1e-6, emb, near(H, 1.0), layers)
    cap = n_tokens
    rows = Lr * cap
    k_pool = torch.zeros((rows, kvd), dtype=torch.bfloat16, device="cuda")
    v_pool = torch.zeros((rows, kvd), dtype=torch.float16, device="cuda")
    row0 = np.arange(Lr, dtype=np.int64) * cap
    c = np.zeros((cap, HD), np.float32)
    s_ = np.zeros((cap, HD), np.float32)
    smol_b200.compute_rope(c, s_, np.arange(cap, dtype=np.int32), cap, HD, 1e6)
    cos_d, sin_d = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
    tokens = torch.randint(0, V, (n_tokens,), dtype=torch.int32, device="cuda", generator=g)
    ws = torch.empty(smol_b200.qkn_prefill_workspace_bytes(model, n_tokens), dtype=torch.uint8, device="cuda")

    def run():
        smol_b200.qkn_prefill(model, tokens, n_tokens, 0, k_pool, v_pool, rows, row0, cos_d, sin_d, ws)
    run()
    a, b = _ev(), _ev()
    a.record()
    run()
    b.record()
    torch.cuda.synchronize()
    smol_b200.check(smol_b200.last_error(), "decoder prefill")
    ms = a.elapsed_time(b)
    gemm = 2 * n_tokens * Lr * (qd * H + 2 * kvd * H + H * qd + 2 * I * H + H * I)
    attn = Lr * workload.causal_flops_square(n_tokens, HQ, HD)
    fl = gemm + attn
    return {"workload": f"Qwen3-0.6B-size prefill of {n_tokens} tokens (28 layers)", "ms": round(ms, 3),
            "tokens_per_s": round(n_tokens / (ms * 1e-3), 1), "tflops": round(fl / (ms * 1e-3) / 1e12, 1),
            "frac_of_bf16_peak": round(fl / (ms * 1e-3) / 1e12 / pk["bf16_tflops"], 4)}


def run_decoder_dropin(layers: int = 1) -> dict:
    """The reference's decoder driver (tests/dropin/qkn_dropin_main.c: Qwen3-shaped,
    hidden 1024, 16/8 heads, `layers` layers) through the reference's own
    qkn_decoder_prefill / _forward on the host cores (oracle/_ref/qkn_dropin_ref) and
    through the decoder-level drop-in on the device (oracle/_ref/qkn_dropin_device):
    wall-clock time of the calls with host buffers in and out, and token identity.
    Each program runs twice: as a process's first generation (`first_run`: the device
    context, module loading and the weight upload fall inside the first calls) and with
    SMOL_DROPIN_WARM=1 (the same generation after one unreported run and a cache reset:
    the steady state a serving process sees); the speed-ups compare the warm runs."""
    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    # the decisive copy model of tests/test_dropin_device_gpu.py (smallest top-2 logit margin
    # ~9): with more layers the reference itself changes tokens once its cache is rounded
    # to the device formats, so identity would not be a property of the drop-in
    args = ["512", "128", "2", "4", "2", str(layers), "1"]
    res = {}
    for kind in ("ref", "device"):
        exe = os.path.join(ref_dir, f"qkn_dropin_{kind}")
        if not os.path.exists(exe):
            return {"unavailable": f"{exe} not built"}
        for warm in (0, 1):
            p = subprocess.run([exe, *args], capture_output=True, text=True, timeout=900,
                               env={**os.environ, "SMOL_DROPIN_WARM": str(warm)})
            if p.returncode != 0:
                return {"error": f"{kind} (warm={warm}): exit {p.returncode}: {p.stderr[-300:]}"}
            t = p.stderr.split("prefill_ms")[1].split()
            res[(kind, warm)] = {"prefill_ms": float(t[0]), "forward_ms_per_step": float(t[2]),
                                 "tokens": p.stdout.split()}

    def times(kind):
        warm, first = res[(kind, 1)], res[(kind, 0)]
        return {"prefill_ms": warm["prefill_ms"], "forward_ms_per_step": warm["forward_ms_per_step"],
                "first_run": {"prefill_ms": first["prefill_ms"], "forward_ms_per_step": first["forward_ms_per_step"]}}

    ref, dev = res[("ref", 1)], res[("device", 1)]
    streams = [res[(k, w)]["tokens"] for k in ("ref", "device") for w in (0, 1)]
    return {"workload": f"reference decoder driver, hidden 1024, {layers} layer(s), vocab 4096, "
                        "prefill 511 + 128 steps",
            "reference_cpu": times("ref"),
            "device_dropin": times("device"),
            "forward_speedup": round(ref["forward_ms_per_step"] / dev["forward_ms_per_step"], 2),
            "prefill_speedup": round(ref["prefill_ms"] / dev["prefill_ms"], 2),
            "tokens_equal": all(x == streams[0] for x in streams),
            "first_differing_step": next((i for i, (x, y) in enumerate(zip(ref["tokens"], dev["tokens"]))
                                          if x != y), None),
            "note": "warm runs (one unreported generation first); first_run = a process's first generation, "
                    "whose first device call includes context creation and the weight upload; the device "
                    "prefill call returns once its work is queued (about 0.15 ms of GPU time at this size), "
                    "which the first forward call's copy then waits for"}


def run_other_configs(pk, world: int = 1, rank: int = 0) -> dict:
    """The remaining BASELINE configs (latency- or tensor-bound; not the headline).

    cfg 3 and cfg 4 shard across the ranks (by image, by sequence) and report the
    slowest rank's time; cfg 1 (batch 1, replicas only) and the decoder step run at
    N = 1 only.  Each runs on its own: a library error in one is reported in its entry
    ("error") and does not stop the others or the headline measurement.  Every rank
    runs the same list, so the collectives inside line up."""
    import smol_b200
    runs = {"cfg3": lambda: run_cfg3(pk, world=world, rank=rank),
            "cfg4": lambda: run_cfg4(pk, world=world, rank=rank)}
    if world == 1:
        runs = {"cfg1": run_cfg1, **runs,
                "decoder_step_b1": lambda: run_decoder(pk, 1), "decoder_step_b8": lambda: run_decoder(pk, 8),
                # the rows beside the attention path: whole SigLIP encoder, the audio encoder's
                # window shape, the device prefill, the Gemma-configured step, and the
                # reference decoder driver against its decoder-level drop-in
                "siglip_encoder": lambda: run_siglip_encoder(pk), "so400m_attention": lambda: run_so400m_attention(pk),
                "audio_windows": lambda: run_audio_windows(pk),
                "device_prefill": lambda: run_decoder_prefill(pk),
                "gemma_step_b1": lambda: run_gemma_decoder(pk, 1), "gemma_step_b8": lambda: run_gemma_decoder(pk, 8),
                "decoder_dropin": run_decoder_dropin}
    import torch
    res = {}
    for name, fn in runs.items():
        smol_b200.clear_error()
        try:
            res[name] = fn()
            smol_b200.check(smol_b200.last_error(), name)
        except smol_b200.SmolB200Error as e:
            res[name] = {"error": str(e)}
            smol_b200.clear_error()
        except (RuntimeError, OSError, subprocess.SubprocessError, ValueError) as e:   # e.g. a missing binary
            if world > 1:
                raise   # the ranks must keep taking the same collective steps
            res[name] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        torch.cuda.empty_cache()
    return res


def run_ours(args):
    import torch

    import smol_b200
    world, rank, local = dist_setup(args)
    pk = peaks()
    cfg = workload.CFG2
    hq, hkv, hd, layers = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], args.layers
    kv_dim = hkv * hd
    lens_all = workload.decode_lengths(args.seqs, cfg["len_lo"], cfg["len_hi"], seed=0)
    if args.scaling == "strong":
        # BASELINE cfg 2: one batch of 256 split by KV bytes; no data crosses ranks
        mine = workload.shard_by_bytes(lens_all, world)[rank]
        job_lens = lens_all
    else:
        mine = np.arange(args.seqs)
        job_lens = np.tile(lens_all, world)
    lens = lens_all[mine]
    n = len(lens)
    lay = workload.pool_layout(lens, layers, reserve=1)
    max_len = int(lens.max())
    kv_bytes_job = workload.pool_layout(job_lens, layers, reserve=1).kv_bytes(kv_dim, extra_tokens=1)

    prefill = None
    if not args.no_prefill:
        prefill = run_prefill(args, world, rank, pk)
        torch.cuda.empty_cache()
    others = None
    if not args.no_configs and not args.no_decode:
        others = run_other_configs(pk, world, rank)
        torch.cuda.empty_cache()
    if args.no_decode:
        if rank == 0:
            print(json.dumps({"prefill": prefill}))
        return

    # ---- device state: the pooled cache, weights, tables, per-layer indices ----
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    k_pool = torch.empty((lay.rows, kv_dim), dtype=torch.bfloat16, device="cuda")
    v_pool = torch.empty((lay.rows, kv_dim), dtype=torch.float16, device="cuda")
    fill_randn(k_pool, gen)
    fill_randn(v_pool, gen)
    q_in = torch.randn((n, hq * hd), device="cuda", generator=gen)
    k_in = torch.randn((n, kv_dim), device="cuda", generator=gen)
    v_in = torch.randn((n, kv_dim), device="cuda", generator=gen)
    qn_w = (1 + 0.02 * torch.randn(hd, device="cuda", generator=gen)).contiguous()
    kn_w = (1 + 0.02 * torch.randn(hd, device="cuda", generator=gen)).contiguous()
    n_pos = max_len + 2
    cos_h = np.zeros((n_pos, hd), np.float32)
    sin_h = np.zeros((n_pos, hd), np.float32)
    smol_b200.compute_rope(cos_h, sin_h, np.arange(n_pos, dtype=np.int32), n_pos, hd, cfg["theta"])
    rope_cos = torch.from_numpy(cos_h).cuda()
    rope_sin = torch.from_numpy(sin_h).cuda()
    q_rot = torch.empty_like(q_in)
    out = torch.empty_like(q_in)
    positions = torch.from_numpy(lens.astype(np.int32)).cuda()
    kv_next = torch.from_numpy((lens + 1).astype(np.int32)).cuda()
    row0 = [torch.from_numpy(lay.row0(l)).cuda() for l in range(layers)]
    slots = [torch.from_numpy(lay.row0(l) + lens).cuda() for l in range(layers)]
    ws = torch.empty(smol_b200.decode_workspace_bytes(n, max_len + 1, hq, hkv, hd), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    scale = 1.0 / np.sqrt(hd)

    kv_events = []

    def step(record=False):
        for l in range(layers):
            smol_b200.qknorm_rope_append(q_in, k_in, v_in, n, hq, hkv, hd, qn_w, kn_w, 1e-6, rope_cos, rope_sin,
                                         False, positions, slots[l], q_rot, None, k_pool, v_pool, lay.rows,
                                         stream=stream)
            if record:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
            smol_b200.decode_attention(out, q_rot, k_pool, v_pool, lay.rows, row0[l], kv_next, n, max_len + 1, hq,
                                       hkv, hd, scale, ws, stream=stream)
            if record:
                b.record(stream)
                kv_events.append((a, b))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    smol_b200.check(smol_b200.last_error(), "warm-up")
    barrier(world)
    clocks = Clocks(gpu_index(local)) if rank == 0 else None
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier(world)
    t_start.record(stream)
    for _ in range(args.steps):
        step(record=True)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop() if clocks else None
    ms_total = t_start.elapsed_time(t_end)
    ms_step = allreduce_max(ms_total / args.steps, world)
    dev_err = smol_b200.device_error()
    if dev_err or smol_b200.last_error():
        raise SystemExit(f"kernel error: device word {dev_err}, last error {smol_b200.last_error()}")

    kv_bytes_rank = lay.kv_bytes(kv_dim, extra_tokens=1)          # attends L+1 per layer
    value = kv_bytes_job / (ms_step * 1e-3) / 1e9                  # whole job / slowest rank
    ms_rank = ms_total / args.steps                                 # this rank's own step time
    rank_ms = [0.0] * world
    if world > 1:
        import torch.distributed as dist
        t = torch.zeros(world, dtype=torch.float64, device="cuda")
        t[rank] = ms_rank
        dist.all_reduce(t)
        rank_ms = [float(x) for x in t.cpu()]
        rank_bytes = torch.zeros(world, dtype=torch.float64, device="cuda")
        rank_bytes[rank] = float(kv_bytes_rank)
        dist.all_reduce(rank_bytes)
        rank_bytes = [float(x) for x in rank_bytes.cpu()]
    else:
        rank_ms = [ms_rank]
        rank_bytes = [float(kv_bytes_rank)]
    # roofline of the decode kernel pair (split-KV + combine), live CUDA events
    dec_ms = statistics.mean(a.elapsed_time(b) for a, b in kv_events)
    qo_bytes = n * hq * hd * 4 * 2                                 # fp32 q read + fp32 out write
    alg_bytes_launch = kv_bytes_rank / layers + qo_bytes
    achieved = alg_bytes_launch / (dec_ms * 1e-3) / 1e9
    # DRAM traffic per launch: ncu (dram__bytes_read.sum + dram__bytes_write.sum) on the
    # 16-sequence, 1-layer case of this workload read 304.55 MB and wrote 4.45 MB
    # (partials + output) for 304.38 MB of algorithmic bytes; both grow with the KV
    # bytes (reads) and the number of 2048-key chunks (partials), so the full launch is
    # scaled by its algorithmic bytes.
    traffic_launch = alg_bytes_launch * DECODE_TRAFFIC_PER_ALG_BYTE

    # ---- e2e through the C ABI with host buffers ----
    e2e = None
    if not args.no_e2e:
        qh = torch.randn((n, hq * hd), generator=torch.Generator().manual_seed(3)).pin_memory()
        kh = torch.randn((n, kv_dim), generator=torch.Generator().manual_seed(4)).pin_memory()
        vh = torch.randn((n, kv_dim), generator=torch.Generator().manual_seed(5)).pin_memory()
        oh = torch.empty((n, hq * hd)).pin_memory()
        lens_d = torch.from_numpy(lens.astype(np.int32)).cuda()
        scratch = torch.empty(smol_b200.decode_step_scratch_bytes(n, max_len, hq, hkv, hd), dtype=torch.uint8,
                              device="cuda")

        def e2e_step():
            for l in range(layers):
                smol_b200.decode_step_host(oh.numpy(), qh.numpy(), kh.numpy(), vh.numpy(), n, hq, hkv, hd, qn_w, kn_w,
                                           1e-6, rope_cos, rope_sin, False, k_pool, v_pool, lay.rows, row0[l], lens_d,
                                           max_len, scale, scratch, stream=stream)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = allreduce_max(e0.elapsed_time(e1) / args.steps, world)
        e2e = {"value": round(kv_bytes_job / (e2e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
               "ms_per_step": round(e2e_ms, 3),
               "h2d_bytes_per_step": world * layers * (qh.numel() + kh.numel() + vh.numel()) * 4 if
               args.scaling == "weak" else len(lens_all) * layers * (hq * hd + 2 * kv_dim) * 4,
               "d2h_bytes_per_step": (world * n if args.scaling == "weak" else len(lens_all)) * layers * hq * hd * 4,
               "api": "smol_b200_decode_step_host (pinned host q/k/v in, host out; 28 calls per step)"}
        smol_b200.check(smol_b200.last_error(), "e2e")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference_decode(lens, args.cpu_seconds)
        if prefill is not None or others is not None:   # the tensor-bound configs' CPU reference too
            try:
                cpu["other_configs"] = cpu_reference_prefill()
            except Exception as e:   # a missing or failing reference must not cost the headline
                cpu["other_configs"] = {"error": str(e)[:200]}

    if rank != 0:
        return
    strong = args.scaling == "strong"
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": ("cfg2: batched decode attention step, 28 layers x 256 sequences "
                                + ("split across the GPUs by KV bytes" if strong else "per GPU")
                                + ", KV len ~U[1024,8192] seed 0, GQA 16/8, hd 128, theta 1e6, "
                                  "QK-norm+RoPE+append fused"),
                   "global_batch": len(job_lens), "layers": layers, "kv_cache": "K bf16 / V fp16, pooled in HBM",
                   "parallelism": f"dp{world} (sequences sharded, no collective)",
                   "l2": "cache of %.1f GB per GPU >> 126 MB L2: no flush needed" % (2 * lay.rows * kv_dim * 2 / 1e9)},
        "kv_bytes_per_step": kv_bytes_job,
        "hbm_frac": round(value / world / pk["hbm_gbs"], 4),
        "shards": {"sequences_per_rank": ([len(x) for x in workload.shard_by_bytes(lens_all, world)] if strong
                                          else [len(lens_all)] * world), "rank_ms_per_step": [round(x, 4) for x in rank_ms],
                   "rank_kv_bytes": [int(x) for x in rank_bytes],
                   "balance": round(min(rank_bytes) / max(rank_bytes), 4),
                   "limit": ("slowest rank: the byte split leaves at most one sequence's bytes of imbalance, and "
                             "each rank keeps the per-layer fixed cost of its launches")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": int(traffic_launch),
                     "traffic_source": "ncu dram bytes of the 16-seq 1-layer case x (full / small algorithmic bytes)",
                     "kernel": "decode_split_kernel<128> + decode_combine_kernel<128> (per layer)",
                     "alg_bytes_per_launch": int(alg_bytes_launch), "ms_per_launch": round(dec_ms, 4),
                     "peak_source": pk["source"]},
        "gpu_launches": args.steps * layers * 3,   # append + split + combine per layer (n >= 32 never clusters)
        "e2e": e2e,
        "cpu_baseline": None if cpu is None else {k: (round(v, 3) if isinstance(v, float) else v)
                                                  for k, v in cpu.items()},
        "clocks": clk,
        "prefill": prefill,
        "other_configs": others,
    }
    print(json.dumps(line))


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.only_config:
        import torch
        torch.cuda.set_device(0)
        pk = peaks()
        fn = {"cfg1": run_cfg1, "cfg3": lambda: run_cfg3(pk, args.images, 1 if args.images else None),
              "cfg4": lambda: run_cfg4(pk), "decoder": lambda: [run_decoder(pk, 1), run_decoder(pk, 8)],
              "audio": lambda: run_audio_windows(pk),
              "siglip": lambda: run_siglip_encoder(pk, args.images),
              "so400m": lambda: run_so400m_attention(pk, args.images or 128, 1 if args.images else 27),
              "gemma": lambda: [run_gemma_decoder(pk, 1), run_gemma_decoder(pk, 8)],
              "prefill": lambda: run_decoder_prefill(pk),
              "dropin": run_decoder_dropin}[args.only_config]
        print(json.dumps({args.only_config: fn()}))
        return
    run_ours(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

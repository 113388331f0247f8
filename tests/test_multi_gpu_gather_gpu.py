"""Prefill with the all-gather inside the kernel, on two GPUs (skipped with fewer).

cfg 5's layout at small size: the KV heads are split over the ranks, each rank runs
the causal prefill for its Q heads and the per-rank outputs are all-gathered.  With
smol_b200_prefill_attention_multi every output tile is stored to this rank's slot in
each rank's gather buffer (a CUDA IPC mapping for the peer) by the prefill kernel
itself.  The gathered tensor must equal prefill + NCCL all-gather bit for bit on every
rank, with fp32 and with bf16 outputs.  Ranks are child processes with NCCL over 127.0.0.1 and a short process-group
timeout; NVLS is off so no multicast object is involved.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, B, L, bf16, q_err):
    import datetime

    import torch.distributed as dist

    import smol_b200
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        hq, hkv, hd = 16, 8, 128
        hq_r, hkv_r = hq // world, hkv // world
        g = torch.Generator(device="cuda").manual_seed(7 + rank)
        q = torch.randn((B, L, hq_r * hd), device="cuda", generator=g).to(torch.bfloat16)
        k = torch.randn((B, L, hkv_r * hd), device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn((B, L, hkv_r * hd), device="cuda", generator=g).to(torch.float16)
        dt = torch.bfloat16 if bf16 else torch.float32
        out = torch.empty((B, L, hq_r * hd), device="cuda", dtype=dt)
        gathered = torch.full((world, B, L, hq_r * hd), float("nan"), device="cuda", dtype=dt)
        handle, off = smol_b200.ipc_handle(gathered)
        meta = torch.tensor(list(handle) + list(off.to_bytes(8, "little")), dtype=torch.uint8, device="cuda")
        allmeta = torch.empty(world * 72, dtype=torch.uint8, device="cuda")
        dist.all_gather_into_tensor(allmeta, meta)
        allmeta = allmeta.cpu().numpy().reshape(world, 72)
        slot = out.numel() * out.element_size()
        bases, opened = [], []
        for peer in range(world):
            if peer == rank:
                bases.append(gathered.data_ptr())
            else:
                b0 = smol_b200.ipc_open(bytes(allmeta[peer, :64]))
                opened.append(b0)
                bases.append(b0 + int.from_bytes(bytes(allmeta[peer, 64:]), "little"))
        outs = [bases[rank] + rank * slot] + [bases[p] + rank * slot for p in range(world) if p != rank]
        dist.barrier()
        scale = 1 / np.sqrt(hd)
        smol_b200.prefill_attention_multi(outs, hq_r * hd, L * hq_r * hd, q, k, v, B, L, L, hq_r, hkv_r, hd, scale,
                                          bf16=bf16)
        torch.cuda.synchronize()
        dist.barrier()                 # every rank's kernel (and its stores) has finished
        fused = gathered.clone()
        smol_b200.prefill_attention(out, q, k, v, B, L, L, hq_r, hkv_r, hd, scale)
        ref = torch.empty_like(gathered)
        dist.all_gather_into_tensor(ref, out)
        torch.cuda.synchronize()
        assert smol_b200.last_error() == 0 and smol_b200.device_error() == 0
        assert not torch.isnan(fused).any(), "a slot of the gather buffer was not written"
        assert torch.equal(fused, ref), float((fused - ref).abs().max())
        dist.barrier()
        for b0 in opened:
            smol_b200.ipc_close(b0)
        dist.destroy_process_group()
    except BaseException as e:   # report to the parent, exit non-zero
        q_err.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("B,L,bf16", [(2, 1024, False), (1, 1000, False), (2, 1024, True), (1, 1000, True)])
def test_fused_allgather_matches_nccl(B, L, bf16):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_err = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, B, L, bf16, q_err)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not q_err.empty():
        errs.append(q_err.get())
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), errs or [p.exitcode for p in procs]

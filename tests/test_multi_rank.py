"""Host-side multi-GPU logic, run as gloo ranks on the CPU (world size 2).

bench.py splits work across the GPUs of one box without a collective on the data
path (cfg 2 sequences, cfg 3 images, cfg 4 sequences) or with one all-gather per
layer (cfg 5 KV-head groups), and reports the max over ranks of the device time.
These tests check the partitions and that flow on gloo, and that a rank which dies
between steps makes the survivor's next collective fail within the process-group
timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import workload


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_by_bytes_covers_every_sequence_once():
    lens = workload.decode_lengths(256, 1024, 8192, seed=0)
    for world in (1, 2, 4, 8):
        shards = workload.shard_by_bytes(lens, world)
        allidx = np.sort(np.concatenate(shards))
        assert np.array_equal(allidx, np.arange(256))
        loads = [int(lens[s].sum()) for s in shards]
        assert max(loads) - min(loads) <= int(lens.max())   # greedy LPT bound


def test_partitions():
    assert [list(workload.kv_head_groups(8, 8, r)) for r in range(8)] == [[r] for r in range(8)]
    assert list(workload.kv_head_groups(8, 2, 1)) == [4, 5, 6, 7]
    with pytest.raises(ValueError):
        workload.kv_head_groups(8, 3, 0)
    got = sorted(i for r in range(4) for i in workload.shard_evenly(128, 4, r))
    assert got == list(range(128))
    assert workload.causal_flops_square(512, 16, 128) == 4 * 128 * 16 * (512 * 513 // 2)
    assert workload.causal_flops(3, 3, 1, 1) == 4 * (1 + 2 + 3)
    assert workload.prefix_lm_flops(4, 2, 1, 1) == 4 * (4 + 3 + 4)


def test_pool_layout_addressing():
    lay = workload.pool_layout(np.array([3, 5], np.int32), layers=2, reserve=1)
    # sequence 0: rows [0, 8) (2 layers x cap 4); sequence 1: rows [8, 20)
    assert list(lay.row0(0)) == [0, 8] and list(lay.row0(1)) == [4, 14] and lay.rows == 20
    assert lay.kv_bytes(kv_dim=4, extra_tokens=1) == (4 + 6) * 2 * 4 * 2 * 2


def _rank_main(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "flow":
            lens = workload.decode_lengths(256, 1024, 8192, seed=0)
            mine = workload.shard_by_bytes(lens, world)[rank]
            t = torch.tensor([float(lens[mine].sum())], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)                     # max over ranks
            heads = list(workload.kv_head_groups(8, world, rank))
            out = torch.tensor(heads, dtype=torch.float32)
            gathered = torch.empty(world * len(heads), dtype=torch.float32)
            dist.all_gather_into_tensor(gathered, out)                   # cfg 5 output exchange
            q.put((rank, float(t.item()), gathered.tolist(), [int(i) for i in mine[:3]]))
        else:   # "rank_dies": rank 1 leaves between steps, rank 0's next collective must fail
            t = torch.ones(1)
            dist.all_reduce(t)                                            # step 1, both ranks
            if rank == 1:
                q.put((1, "left"))
                q.close()
                q.join_thread()          # make sure the message left before the process does
                os._exit(0)
            try:
                dist.all_reduce(t)                                        # step 2: peer is gone
                q.put((0, "completed"))
            except Exception as e:                                        # noqa: BLE001
                q.put((0, "error:" + type(e).__name__))
    finally:
        if mode == "flow":
            dist.destroy_process_group()


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(res, key=lambda r: r[0])


def test_two_gloo_ranks_shard_reduce_and_gather():
    res = _run("flow")
    lens = workload.decode_lengths(256, 1024, 8192, seed=0)
    shards = workload.shard_by_bytes(lens, 2)
    expect_max = max(float(lens[s].sum()) for s in shards)
    for rank, tmax, gathered, first in res:
        assert tmax == expect_max
        assert gathered == [0.0, 1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0]
        assert first == [int(i) for i in shards[rank][:3]]


def test_rank_that_leaves_makes_peer_collective_fail():
    res = _run("rank_dies")
    assert res[1] == (1, "left")
    assert res[0][0] == 0 and res[0][1].startswith("error:"), res[0]

"""Host side of the sharded engine (no GPU): the row/expert ranges each rank holds, and the NCCL
id exchange over a world-size-2 gloo process group."""
import ctypes
import os

import pytest

from sardyne_b200 import capi


def shard_range(n, world, rank, align):
    b, e = ctypes.c_int64(), ctypes.c_int64()
    capi.lib().sdy_shard_range(n, world, rank, align, ctypes.byref(b), ctypes.byref(e))
    return b.value, e.value


@pytest.mark.parametrize("n,align", [(11008, 8), (2048, 8), (151936, 8), (49152, 8), (1536, 8), (128, 1), (576, 8),
                                     (13, 8), (7, 1)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_ranges_partition(n, align, world):
    """Consecutive ranks hold consecutive, aligned, non-overlapping ranges covering [0, n)."""
    end = 0
    for r in range(world):
        b, e = shard_range(n, world, r, align)
        assert b == end and b <= e <= n
        assert b % align == 0
        end = e
    assert end == n


def test_expert_split_qwen3():
    assert [shard_range(128, 8, r, 1) for r in range(8)] == [(16 * r, 16 * r + 16) for r in range(8)]


def test_set_shard_validation():
    lib = capi.lib()
    lib.sdy_clear_error()
    assert lib.sdy_engine_set_shard(2, 2, None) == -1 and "invalid" in capi.last_error()
    assert lib.sdy_engine_set_shard(0, 2, None) == -1  # a sharded world needs the NCCL id
    assert lib.sdy_engine_set_shard(0, 1, None) == 0
    r, w = ctypes.c_int32(), ctypes.c_int32()
    lib.sdy_engine_get_shard(ctypes.byref(r), ctypes.byref(w))
    assert (r.value, w.value) == (0, 1)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from sardyne_b200 import runtime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        obj = [runtime.new_nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        runtime.set_shard(rank, world, obj[0])
        r, w = ctypes.c_int32(), ctypes.c_int32()
        capi.lib().sdy_engine_get_shard(ctypes.byref(r), ctypes.byref(w))
        q.put((rank, r.value, w.value, obj[0]))
    finally:
        dist.destroy_process_group()


def test_nccl_id_exchange_gloo():
    """Two ranks agree on one 128-byte id and record their own rank (gloo, CPU only)."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert [g[:3] for g in got] == [(0, 0, 2), (1, 1, 2)]
    assert got[0][3] == got[1][3] and len(got[0][3]) == 128


@pytest.mark.parametrize("n_head,n_kv,hd", [(16, 2, 128), (32, 4, 128), (9, 3, 64), (4, 2, 64), (8, 8, 64)])
@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_attention_split_covers_every_head_once(n_head, n_kv, hd, world):
    """Query heads split over the ranks exactly once, each rank holding the KV heads its query heads
    read (GQA: head h reads KV head h / (n_head / n_kv)), and the local grouping consistent."""
    lib = capi.lib()
    n_rep = n_head // n_kv
    owners = [0] * n_head
    modes = set()
    for r in range(world):
        rng = (ctypes.c_int32 * 4)()
        mode = lib.sdy_attention_split(n_head, n_kv, hd, world, r, rng)
        assert mode in (0, 1)
        modes.add(mode)
        h0, h1, k0, k1 = list(rng)
        if mode == 0:
            assert (h0, h1, k0, k1) == (0, n_head, 0, n_kv)
            continue
        assert 0 <= h0 < h1 <= n_head and 0 <= k0 < k1 <= n_kv
        assert (h1 - h0) % (k1 - k0) == 0
        rep_local = (h1 - h0) // (k1 - k0)
        for h in range(h0, h1):
            owners[h] += 1
            assert h // n_rep == k0 + (h - h0) // rep_local  # the local KV head is the global one
        assert ((h1 - h0) * hd) % 8 == 0 and ((k1 - k0) * hd) % 8 == 0
    assert len(modes) == 1  # every rank agrees on split or replicated
    if modes == {1}:
        assert owners == [1] * n_head


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sweep_slices_fit_the_fused_gather(world):
    """bench.py's multi-GPU sweep: every rank's row slice of every matrix (whole 8-row groups)
    fits its place in the per-rank gather slice (out_off[i] + rows <= count, the check
    sdy_qmatvec_batch_f32_gather_dev makes), and the slices of all ranks cover every row once."""
    import bench
    share, offs = 0, []
    for _, n_out, _ in [(f, o, i) for f in bench.FORMATS for o, i in bench.SHAPES]:
        per = [bench.shard_rows(n_out, r, world) for r in range(world)]
        assert per[0][0] == 0 and per[-1][1] == n_out
        assert all(per[r][1] == per[r + 1][0] for r in range(world - 1))
        assert all(b % 8 == 0 for b, _ in per)
        offs.append((share, max(e - b for b, e in per), per))
        share += max(e - b for b, e in per)
    for off, width, per in offs:
        for b, e in per:
            assert off + (e - b) <= share and e - b <= width


def _failing_worker(rank, world, port, mode, q):
    import datetime
    import time

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:  # the failing rank: leaves at once, or stays but never takes part
        if mode == "silent":
            time.sleep(8)
        os._exit(0)
    from sardyne_b200 import runtime
    t0 = time.time()
    try:
        runtime.shard_from_torch()
        outcome = "returned"
    except RuntimeError:
        outcome = "raised"
    r, w = ctypes.c_int32(), ctypes.c_int32()
    capi.lib().sdy_engine_get_shard(ctypes.byref(r), ctypes.byref(w))
    q.put((outcome, time.time() - t0, r.value, w.value))
    q.close()
    q.join_thread()  # the queue's feeder thread sends the result before the process ends
    os._exit(0)


@pytest.mark.parametrize("mode", ["exits", "silent"])
def test_shard_setup_fails_when_a_rank_is_gone(mode):
    """Failure detection on the host (gloo, CPU only): when another rank has exited, or stays alive
    without taking part, shard_from_torch raises within the process group's timeout (3 s here)
    instead of waiting, and this process's shard stays unset (world 1), so no sharded load
    starts."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    outcome, seconds, rank, world = q.get(timeout=120)
    for p in procs:
        p.join(60)
    assert outcome == "raised" and seconds < 30, (outcome, seconds)
    assert (rank, world) == (0, 1)

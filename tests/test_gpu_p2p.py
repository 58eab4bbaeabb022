"""sdy_allgather_p2p: the all-gather over NVLink peer memory between two processes (one GPU each).

Each rank shares its buffer through a CUDA IPC handle (exchanged over a gloo group), then the ranks
run rounds of the gather with new data each round: eagerly, then replayed from a CUDA graph (the
round counter lives on the device). After every round each rank's buffer must hold every rank's
slice. Counts that are and are not multiples of 4 take the vector and the scalar copy. Needs two
GPUs; skipped otherwise.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pattern(rank, rnd, count):
    return (rank * 1000.0 + rnd * 10.0 + np.arange(count, dtype=np.float32) * 1e-3).astype(np.float32)


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        from sardyne_b200 import capi
        lib = capi.lib()
        results = []
        for count in (1000, 4096):
            nbytes = lib.sdy_allgather_p2p_bytes(count, world)
            buf = lib.sdy_p2p_alloc(nbytes)
            assert buf, capi.last_error()
            handle = (ctypes.c_char * 64)()
            assert lib.sdy_p2p_handle(buf, handle) == 0, capi.last_error()
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle))
            bases = []
            for r in range(world):
                if r == rank:
                    bases.append(buf)
                else:
                    h = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                    p = lib.sdy_p2p_open(h)
                    assert p, capi.last_error()
                    bases.append(p)
            arr = (ctypes.c_void_p * world)(*bases)
            send = torch.empty(count, dtype=torch.float32, device="cuda")
            stream = torch.cuda.Stream()
            got = np.empty(world * count, np.float32)

            def gather():
                assert lib.sdy_allgather_p2p(ctypes.c_void_p(send.data_ptr()), count, arr, rank, world,
                                             ctypes.c_void_p(stream.cuda_stream)) == 0, capi.last_error()

            for rnd in range(3):  # eager rounds
                send.copy_(torch.from_numpy(_pattern(rank, rnd, count)))
                torch.cuda.synchronize()
                with torch.cuda.stream(stream):
                    gather()
                stream.synchronize()
                lib.sdy_p2p_read(got.ctypes.data, buf, got.nbytes)
                results.append((count, rnd, got.copy()))
                dist.barrier()  # nobody writes the next round before everyone has read this one
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                gather()
            for rnd in range(3, 5):  # graph replays
                send.copy_(torch.from_numpy(_pattern(rank, rnd, count)))
                torch.cuda.synchronize()
                with torch.cuda.stream(stream):
                    g.replay()
                stream.synchronize()
                lib.sdy_p2p_read(got.ctypes.data, buf, got.nbytes)
                results.append((count, rnd, got.copy()))
                dist.barrier()
            del g
            status = lib.sdy_p2p_status()
            for r, p in enumerate(bases):
                if r != rank:
                    lib.sdy_p2p_close(p)
            dist.barrier()
            lib.sdy_p2p_free(buf)
            results.append((count, "status", status))
        q.put((rank, results))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_allgather_over_peer_memory():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(60)
    for rank in range(world):
        assert not isinstance(got[rank], str), got[rank]
        for count, rnd, value in got[rank]:
            if rnd == "status":
                assert value == 0
                continue
            want = np.concatenate([_pattern(r, rnd, count) for r in range(world)])
            assert np.array_equal(value, want), (rank, count, rnd)

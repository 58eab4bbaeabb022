"""sdy_allgather_p2p: the all-gather over NVLink peer memory between two processes (one GPU each);
and sdy_qmatvec_batch_f32_gather_dev, the grouped products with that all-gather fused into their
launch (each rank's row slices of every matrix, gathered, equal the one-GPU products bit for bit).

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


def _fused_rank(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        import oracle
        from sardyne_b200 import capi
        lib = capi.lib()
        shapes = [("Q4_K", 1000, 2048), ("Q6_K", 304, 1024), ("Q4_K", 77, 256)]
        # this rank's rows of each matrix (whole 8-row groups) and their place in the slice
        ranges, offs, share = [], [], 0
        for _, n_out, _ in shapes:
            b, e = ctypes.c_int64(), ctypes.c_int64()
            per = []
            for r in range(world):
                lib.sdy_shard_range(n_out, world, r, 8, ctypes.byref(b), ctypes.byref(e))
                per.append((b.value, e.value))
            ranges.append(per)
            offs.append(share)
            share += max(e - b for b, e in per)
        nbytes = lib.sdy_allgather_p2p_bytes(share, world)
        buf = lib.sdy_p2p_alloc(nbytes)
        handle = (ctypes.c_char * 64)()
        assert buf and lib.sdy_p2p_handle(buf, handle) == 0, capi.last_error()
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle))
        bases = [buf if r == rank else lib.sdy_p2p_open((ctypes.c_char * 64).from_buffer_copy(handles[r]))
                 for r in range(world)]
        assert all(bases), capi.last_error()
        hs, xs, full = [], [], []
        for i, (kind, n_out, n_in) in enumerate(shapes):
            w = oracle.random_blocks(kind, n_out * n_in // 256, seed=70 + i).reshape(n_out, -1)
            full.append(w)
            r0, r1 = ranges[i][rank]
            part = np.ascontiguousarray(w[r0:r1])
            h = lib.sdy_qmat_upload(part.ctypes.data, oracle.TYPE_ID[kind], r1 - r0, n_in)
            assert h, capi.last_error()
            hs.append(h)
            xs.append(torch.from_numpy(np.random.default_rng(i).standard_normal(n_in).astype(np.float32)).cuda())
        arr = lambda vals: (ctypes.c_void_p * len(vals))(*vals)  # noqa: E731
        offa = (ctypes.c_int64 * len(shapes))(*offs)
        stream = torch.cuda.Stream()
        got = np.empty(world * share, np.float32)
        for _ in range(3):  # rounds: every one must leave the whole gathered y
            with torch.cuda.stream(stream):
                assert lib.sdy_qmatvec_batch_f32_gather_dev(len(shapes), arr(hs), arr([x.data_ptr() for x in xs]),
                                                            offa, share, arr(bases), rank, world,
                                                            ctypes.c_void_p(stream.cuda_stream)) == 0, \
                    capi.last_error()
            stream.synchronize()
            lib.sdy_p2p_read(got.ctypes.data, buf, got.nbytes)
            dist.barrier()
        status = lib.sdy_kernel_status()
        # the one-GPU products of the full matrices, through the oracle
        ok = True
        for i, (kind, n_out, n_in) in enumerate(shapes):
            xq = oracle.quantize(xs[i].cpu().numpy()[None], "Q8_K")
            want = oracle.matmul_q(full[i], kind, xq, 1, n_in, n_out)[0]
            for r in range(world):
                b, e = ranges[i][r]
                seg = got[r * share + offs[i]: r * share + offs[i] + (e - b)]
                ok = ok and np.array_equal(seg, want[b:e])
        for r, p in enumerate(bases):
            if r != rank:
                lib.sdy_p2p_close(p)
        dist.barrier()
        lib.sdy_p2p_free(buf)
        for h in hs:
            lib.sdy_qmat_free(h)
        q.put((rank, (ok, status)))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_products_with_fused_allgather():
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
    procs = [ctx.Process(target=_fused_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(60)
    for rank in range(world):
        assert not isinstance(got[rank], str), got[rank]
        assert got[rank] == (True, 0), got[rank]

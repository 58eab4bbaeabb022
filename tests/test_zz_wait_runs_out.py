"""Failure detection of the NVLink peer-memory gathers, on one GPU: when another rank never arrives,
the wait of the last CTA gives up after its one-second limit. It sets the status word that the host
reads, and the context stays usable.

Rank 1 of a two-rank gather is a second buffer on the same GPU that no kernel ever signals. Only one
kernel is launched, and no second rank runs, so no kernel waits on another; the wait runs out on a
flag that nothing sets. Both gathers are covered: the standalone all-gather (sdy_allgather_p2p,
sdy_p2p_status) and the all-gather fused into the grouped products
(sdy_qmatvec_batch_f32_gather_dev, sdy_kernel_status). The stores of the rank that did arrive must
still be complete in both buffers. After the status is cleared, a one-rank gather and the same
product must run with status 0 and give the same values.

The checks run in a child process, because a status word stays set until it is cleared and must
not reach the other tests. The file name sorts last, so that a run stopping at the first failure
has run everything else.
"""
import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WAIT_S = 1.0  # the kernels' wait limit


def _read(lib, ptr, n, dtype, offset=0):
    out = np.empty(n, dtype)
    assert lib.sdy_p2p_read(out.ctypes.data, ctypes.c_void_p(ptr + offset), out.nbytes) == 0
    return out


def _child(q):
    try:
        import torch

        import oracle
        from sardyne_b200 import capi
        lib = capi.lib()
        arr = lambda vals: (ctypes.c_void_p * len(vals))(*vals)  # noqa: E731
        res = {}

        # the standalone all-gather: rank 0 of two, rank 1 never runs
        count, world = 1000, 2
        flags_at = -(-world * count * 4 // 256) * 256  # the flag words follow the world * count floats
        bufs = [lib.sdy_p2p_alloc(lib.sdy_allgather_p2p_bytes(count, world)) for _ in range(world)]
        assert all(bufs), capi.last_error()
        send = torch.arange(count, dtype=torch.float32, device="cuda") * 0.5 + 1.0
        lib.sdy_p2p_clear_status()
        torch.cuda.synchronize()
        t = time.perf_counter()
        assert lib.sdy_allgather_p2p(ctypes.c_void_p(send.data_ptr()), count, arr(bufs), 0, world, None) == 0, \
            capi.last_error()
        torch.cuda.synchronize()
        res["p2p_s"] = time.perf_counter() - t
        res["p2p_status"] = lib.sdy_p2p_status()
        want = send.cpu().numpy()
        res["p2p_delivered"] = all(np.array_equal(_read(lib, b, count, np.float32), want) for b in bufs)
        res["p2p_flags"] = [_read(lib, b, world, np.uint32, flags_at).tolist() for b in bufs]
        lib.sdy_p2p_clear_status()
        one = lib.sdy_p2p_alloc(lib.sdy_allgather_p2p_bytes(count, 1))
        assert one, capi.last_error()
        assert lib.sdy_allgather_p2p(ctypes.c_void_p(send.data_ptr()), count, arr([one]), 0, 1, None) == 0
        torch.cuda.synchronize()
        res["p2p_after"] = (lib.sdy_p2p_status(), np.array_equal(_read(lib, one, count, np.float32), want))
        for b in bufs + [one]:
            lib.sdy_p2p_free(b)

        # the all-gather fused into the grouped products: rank 0 holds every row of the matrix
        kind, n_out, n_in = "Q4_K", 1000, 2048
        w = oracle.random_blocks(kind, n_out * n_in // 256, seed=5).reshape(n_out, -1)
        h = lib.sdy_qmat_upload(w.ctypes.data, oracle.TYPE_ID[kind], n_out, n_in)
        assert h, capi.last_error()
        x = torch.from_numpy(np.random.default_rng(5).standard_normal(n_in).astype(np.float32)).cuda()
        want = oracle.matmul_q(w, kind, oracle.quantize(x.cpu().numpy()[None], "Q8_K"), 1, n_in, n_out)[0]
        off = (ctypes.c_int64 * 1)(0)
        bufs = [lib.sdy_p2p_alloc(lib.sdy_allgather_p2p_bytes(n_out, world)) for _ in range(world)]
        assert all(bufs), capi.last_error()
        lib.sdy_kernel_clear_status()
        res["fused_status_before"] = lib.sdy_kernel_status()
        t = time.perf_counter()
        assert lib.sdy_qmatvec_batch_f32_gather_dev(1, arr([h]), arr([x.data_ptr()]), off, n_out, arr(bufs), 0,
                                                    world, None) == 0, capi.last_error()
        torch.cuda.synchronize()
        res["fused_s"] = time.perf_counter() - t
        res["fused_status"] = lib.sdy_kernel_status()
        res["fused_delivered"] = all(np.array_equal(_read(lib, b, n_out, np.float32), want) for b in bufs)
        lib.sdy_kernel_clear_status()
        one = lib.sdy_p2p_alloc(lib.sdy_allgather_p2p_bytes(n_out, 1))
        assert one, capi.last_error()
        assert lib.sdy_qmatvec_batch_f32_gather_dev(1, arr([h]), arr([x.data_ptr()]), off, n_out, arr([one]), 0, 1,
                                                    None) == 0, capi.last_error()
        torch.cuda.synchronize()
        res["fused_after"] = (lib.sdy_kernel_status(), np.array_equal(_read(lib, one, n_out, np.float32), want))
        for b in bufs + [one]:
            lib.sdy_p2p_free(b)
        lib.sdy_qmat_free(h)
        q.put(res)
    except Exception as e:  # reported to the parent, which fails the test with it
        q.put(repr(e))


def test_gather_waits_run_out_and_leave_the_context_usable():
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_child, args=(q,))
    p.start()
    res = q.get(timeout=600)
    p.join(60)
    assert not isinstance(res, str), res
    # the standalone gather: gave up after its limit, this rank's slice stored in both buffers,
    # this rank's flag raised in both, the absent rank's flag never
    assert res["p2p_status"] == 1 and WAIT_S * 0.5 < res["p2p_s"] < 60, res
    assert res["p2p_delivered"], res
    assert res["p2p_flags"] == [[1, 0], [1, 0]], res
    assert res["p2p_after"] == (0, True), res
    # the fused gather: the same, through the library's kernel status
    assert res["fused_status_before"] == 0, res
    assert res["fused_status"] == 1 and WAIT_S * 0.5 < res["fused_s"] < 60, res
    assert res["fused_delivered"], res
    assert res["fused_after"] == (0, True), res

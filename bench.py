#!/usr/bin/env python
"""Headline benchmark: quantized decode matvec (batch 1) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One step = one pass of the hot path over the config-2 sweep at batch 1: Q4_K and Q6_K weights of
2048x11008, 11008x2048 and 151936x2048 ([n_out][n_in], N(0, 0.02) quantized by the package's
quantizer; the 151936-row LM heads are filled from a pool of quantized Gaussian blocks), and an
f32 N(0, 1) activation vector per input width quantized on the device to Q8_K once per step (the
reference quantizes each distinct input once and reuses it). The metric
is weight+activation bytes streamed per second (GB/s).

  value  device-resident inputs (weights in the slab layout, activations in HBM), device time
         with CUDA events on the launching stream; the step (the two activation quantizations and
         the six products as one grouped launch, sdy_qmatvec_batch_dev) replays as a CUDA graph;
         its working set (492 MB) exceeds the 126 MB L2, so every matrix is re-read from HBM.
  e2e    the same products through the reference-facing C-ABI (op_matmul: host f32 activations
         in pinned memory, host outputs), weights resident after sdy_weights_register (the
         counterpart of the reference's mmap); includes the H2D copy of x and the D2H of y.
  decode the second half of the metric, in the same line: BASELINE config 5 (Qwen3-30B-A3B
         shape, random-init Q4_K_M mix) through engine_eval, host token ids in and host logits
         out: a 256-token prompt, then 256 greedy decode steps; tok/s, prefill tok/s, the
         whole-step HBM roofline, and the reference engine's own CPU decode on a bounded sample.
  --impl reference  the reference's own CPU kernels (oracle/_ref/libsardyne_ref.so, built from
         its sources) on all host threads, row ranges split as its thread pool does, and its
         engine's CPU decode of the same model.

Multi-GPU (torchrun, one rank per GPU): every matrix of the sweep is split by rows over the
ranks and each step ends with one NCCL all-gather of the y slices (strong scaling: value = the
full matrices' bytes / the slowest rank's time); decode runs the sharded engine (experts split
across the ranks, NCCL inside the engine), one token stream, times as the max over ranks.
"""
import argparse
import concurrent.futures as cf
import ctypes
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "Q4_K/Q6_K matvec HBM GB/s (% of 8 TB/s); decode tok/s Qwen3-30B-A3B-shape"
SHAPES = [(2048, 11008), (11008, 2048), (151936, 2048)]  # [n_out][n_in]
FORMATS = ["Q4_K", "Q6_K"]
FORMATS32 = ["Q8_0", "Q4_0", "Q5_0"]  # the rest of config 2's formats (not in the headline value)
TYPE_ID = {"Q4_0": 2, "Q5_0": 6, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14, "Q8_K": 15}
BLOCK = {"Q4_K": (256, 144), "Q6_K": (256, 210), "Q8_0": (32, 34), "Q4_0": (32, 18), "Q5_0": (32, 22)}


def act_type(fmt):
    """The activation layout a weight format multiplies with (quant.c: vec_dot_type)."""
    return "Q8_0" if fmt in FORMATS32 else "Q8_K"
WORKLOAD = ("BASELINE config 2 at batch 1: Q4_K and Q6_K matvec over 2048x11008, 11008x2048 and "
            "151936x2048 ([n_out][n_in]), f32 inputs quantized to Q8_K (quant_q8_K) for the products")


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def weight_bytes(fmt, n_out, n_in):
    qk, bb = BLOCK[fmt]
    return n_out * (n_in // qk) * bb


def alg_bytes(fmt, n_out, n_in):
    """Algorithmic bytes of one matvec: weights + f32 x + f32 y."""
    return weight_bytes(fmt, n_out, n_in) + 4 * n_in + 4 * n_out


INPUTS_VERSION = 1  # bump when the generated matrices change


def _generate_inputs(seed, only, formats):
    from sardyne_b200 import kquant
    rng = np.random.default_rng(seed)
    mats = []
    for fmt in formats:
        for n_out, n_in in SHAPES:
            if only and only != f"{fmt}:{n_out}":
                continue
            if n_out * n_in <= 32 * 1024 * 1024:
                w = (rng.standard_normal((n_out, n_in)) * 0.02).astype(np.float32)
                raw = kquant.quantize(w, fmt)
            else:
                raw = kquant.synth_tensor(fmt, n_out, n_in, rng)
            mats.append((fmt, n_out, n_in, np.frombuffer(raw, np.uint8).reshape(n_out, -1).copy()))
    return mats


def inputs_cache_path(seed=0, only=None, formats=FORMATS) -> pathlib.Path:
    from sardyne_b200 import synth
    tag = "-".join(formats) + (f"-{only.replace(':', '_')}" if only else "")
    return pathlib.Path(synth.model_cache_dir()) / f"sardyne-sweep-v{INPUTS_VERSION}-s{seed}-{tag}.npz"


def make_inputs(seed=0, only=None, formats=FORMATS):
    """The sweep's matrices; `only` ("Q6_K:151936") keeps one format/row count (profiling runs).
    Quantizing ~0.5 GB takes minutes on the host, so the bytes are kept in the synthetic-model
    cache directory (written atomically; a cache whose arrays do not have the expected sizes is
    rebuilt)."""
    from sardyne_b200 import kquant
    xs = {n_in: np.random.default_rng(1).standard_normal(n_in).astype(np.float32) for _, n_in in SHAPES}
    wanted = [(fmt, n_out, n_in) for fmt in formats for n_out, n_in in SHAPES if not only or only == f"{fmt}:{n_out}"]
    path = inputs_cache_path(seed, only, formats)
    try:
        with np.load(path) as z:
            mats = [(fmt, n_out, n_in, z[f"{fmt}_{n_out}_{n_in}"]) for fmt, n_out, n_in in wanted]
        if all(w.shape == (n_out, n_in // kquant.QK[fmt] * kquant.BLOCK_BYTES[fmt]) for fmt, n_out, n_in, w in mats):
            return mats, xs
    except Exception:  # noqa: BLE001 -- absent, truncated or foreign: generated again below
        pass
    mats = _generate_inputs(seed, only, formats)
    tmp = path.with_name(f"{path.name}.{os.getpid()}.tmp")
    try:
        with open(tmp, "wb") as f:
            np.savez(f, **{f"{fmt}_{n_out}_{n_in}": w for fmt, n_out, n_in, w in mats})
        os.replace(tmp, path)
    except OSError:  # no room or no permission: run without the cache
        tmp.unlink(missing_ok=True)
    return mats, xs


# ------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples of this GPU's clocks and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if not self.proc:
            return
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        rows = []
        for line in getattr(self, "lines", []):
            p = [v.strip() for v in line.split(",")]
            if len(p) < 8:
                continue
            try:
                rows.append((float(p[0]), float(p[1]), p[4:8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------ reference CPU arm

def cpu_sample(mats, lm_head_rows=18992):
    """Bounded sample of the same workload for the CPU: every matrix, LM heads cut to their first
    lm_head_rows rows (1/8)."""
    return [(fmt, min(n_out, lm_head_rows) if n_out > 100000 else n_out, n_in, w) for fmt, n_out, n_in, w in mats]


def reference_pass(ref, sample, xs, threads, pool):
    """One pass of the reference's CPU path: op_quantize_rows once per input, then
    op_matmul_q_rows over `threads` contiguous row ranges (csrc/model_llama.c:569-611)."""
    xq = {}
    for n_in, x in xs.items():
        buf = np.zeros(n_in // 256 * 292, np.uint8)
        ref.op_quantize_rows(TYPE_ID["Q8_K"], x.ctypes.data, buf.ctypes.data, n_in, 0, 1)
        xq[n_in] = buf
    for fmt, n_out, n_in, w in sample:
        out = np.empty(n_out, np.float32)
        cuts = [n_out * i // threads for i in range(threads + 1)]
        futs = [pool.submit(ref.op_matmul_q_rows, out.ctypes.data, xq[n_in].ctypes.data, w.ctypes.data,
                            TYPE_ID[fmt], 1, n_in, n_out, cuts[i], cuts[i + 1]) for i in range(threads)]
        for f in futs:
            f.result()


def sample_bytes(sample):
    return sum(alg_bytes(fmt, n_out, n_in) for fmt, n_out, n_in, _ in sample)


def host_cores():
    """Threads for the CPU baselines: the CPUs this process may run on (its affinity mask), capped
    by a cgroup v2 CPU quota when one is set (a container's share of a larger host)."""
    try:
        n = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        n = os.cpu_count() or 1
    try:
        quota, period = pathlib.Path("/sys/fs/cgroup/cpu.max").read_text().split()[:2]
        if quota != "max":
            n = min(n, -(-int(quota) // int(period)))
    except (OSError, ValueError):
        pass
    return max(1, n)


def time_reference(mats, xs, min_seconds=3.0, threads=None):
    import oracle
    ref = oracle.ref()
    ref.op_set_simd(1)
    threads = threads or host_cores()
    sample = cpu_sample(mats)
    nbytes = sample_bytes(sample)
    best, spent, n = float("inf"), 0.0, 0
    with cf.ThreadPoolExecutor(threads) as pool:
        reference_pass(ref, sample, xs, threads, pool)  # warm-up
        while spent < min_seconds or n < 3:
            t0 = time.perf_counter()
            reference_pass(ref, sample, xs, threads, pool)
            dt = time.perf_counter() - t0
            best, spent, n = min(best, dt), spent + dt, n + 1
    return {"value": round(nbytes / best / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"reference AVX2 op_quantize_rows + op_matmul_q_rows on {threads} host threads, all six "
                      f"matrices with the LM heads cut to their first 18992 rows ({nbytes / 1e6:.0f} MB per pass), "
                      f"best of {n} passes ({spent:.1f} s)"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libsardyne_ref.so was not built"}))
        return 0
    mats, xs = make_inputs()
    ref = oracle.ref()
    ref.op_set_simd(1)
    threads = host_cores()
    sample = cpu_sample(mats)
    nbytes = sample_bytes(sample)
    with cf.ThreadPoolExecutor(threads) as pool:
        for _ in range(args.warmup):
            reference_pass(ref, sample, xs, threads, pool)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            reference_pass(ref, sample, xs, threads, pool)
        dt = time.perf_counter() - t0
    value = nbytes * args.steps / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config(),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": f"each step: the six matrices with LM heads cut to 18992 rows "
                                       f"({nbytes / 1e6:.0f} MB), reference AVX2 kernels on {threads} threads"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if not args.no_decode:
        from sardyne_b200 import synth
        path = synth.baseline_model("qwen3moe", args.model_dir)
        n_prompt = DECODE_MODELS["qwen3moe"][0]
        info_vocab = synth.QWEN3_30B_A3B["vocab"]
        prompt = np.random.default_rng(0).integers(0, info_vocab, n_prompt).tolist()
        d = decode_reference("qwen3moe", path, prompt)
        line["decode"] = {"metric": "decode tok/s qwen3moe shape (greedy, e2e through engine_eval)",
                          "value": d["value"], "unit": "tok/s", "prefill_tok_s": d["prefill_tok_s"],
                          "cpu_baseline": d}
    print(json.dumps(line))
    return 0


def config(world=1, gather="p2p"):
    c = {"workload": WORKLOAD, "formats": FORMATS, "shapes_out_in": SHAPES, "batch": 1,
         "l2": "inputs larger than L2: 492 MB of weights per step against a 126 MB L2",
         "weights": "N(0,0.02), package quantizer; LM heads from a pool of quantized Gaussian blocks"}
    c["parallelism"] = (f"rows of every matrix split over {world} GPUs, y all-gathered "
                        f"({'over NVLink peer memory, fused into the product launch' if gather == 'p2p' else 'NCCL'})"
                        if world > 1 else "1 GPU")
    return c


# ------------------------------------------------------------------------------ B200 arm

def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def load_traffic():
    """DRAM bytes per launch of the grouped sweep kernel and of the single Q6_K LM-head kernel, from
    the committed ncu summaries where present."""
    out = []
    for name in ("qmvb_config2_sweep_traffic.json", "qmv_q6k_lmhead_traffic.json"):
        p = REPO / "profiles" / name
        try:
            out.append(json.loads(p.read_text()).get("dram_bytes_per_launch") if p.exists() else None)
        except (ValueError, KeyError):
            out.append(None)
    return tuple(out)


def shard_rows(n_out, rank, world):
    """Rows [r0, r1) of an n_out-row matrix for `rank` of `world`: whole 8-row groups, as the
    engine shards its matrices (sdy_shard_range)."""
    from sardyne_b200 import capi
    b, e = ctypes.c_int64(), ctypes.c_int64()
    capi.lib().sdy_shard_range(n_out, world, rank, 8, ctypes.byref(b), ctypes.byref(e))
    return b.value, e.value


def measure_formats32(lib, dev, reps=20):
    """Config 2's 32-element formats (Q8_0, Q4_0, Q5_0) at batch 1, one matvec per matrix with Q8_0
    activations: per-matrix device time by the same sweep-with/without-it difference as the headline
    breakdown (each matrix cold in L2 when it runs). Informational; not part of `value`."""
    import torch
    from sardyne_b200 import capi
    mats, xs = make_inputs(seed=2, formats=FORMATS32)
    stream = torch.cuda.Stream(device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    handles, outs, d_xq = [], [], {}
    for fmt, n_out, n_in, w in mats:
        h = lib.sdy_qmat_upload(w.ctypes.data, TYPE_ID[fmt], n_out, n_in)
        if not h:
            raise RuntimeError(capi.last_error())
        handles.append(h)
        outs.append(torch.empty(n_out, dtype=torch.float32, device=dev))
    for n_in, x in xs.items():
        d_x = torch.from_numpy(x).to(dev)
        d_xq[n_in] = torch.empty(lib.sdy_xq_bytes(TYPE_ID["Q8_0"], n_in, 1), dtype=torch.uint8, device=dev)
        lib.sdy_quantize_rows_dev(TYPE_ID["Q8_0"], ctypes.c_void_p(d_x.data_ptr()), 1, n_in,
                                  ctypes.c_void_p(d_xq[n_in].data_ptr()), sp)

    def sweep(skip=-1):
        for i, (fmt, n_out, n_in, _) in enumerate(mats):
            if i != skip:
                lib.sdy_qmatvec_dev(handles[i], ctypes.c_void_p(d_xq[n_in].data_ptr()), 1,
                                    ctypes.c_void_p(outs[i].data_ptr()), n_out, 0, n_out, sp)

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            fn()
        return g

    with torch.cuda.stream(stream):
        for _ in range(3):
            sweep()
    torch.cuda.synchronize()
    capi.check()
    g_all = capture(lambda: [sweep() for _ in range(reps)])
    rows = []
    for i, (fmt, n_out, n_in, _) in enumerate(mats):
        g_wo = capture(lambda i=i: [sweep(skip=i) for _ in range(reps)])
        ts = []
        for g in (g_wo, g_all, g_wo, g_all):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = (min(ts[1], ts[3]) - min(ts[0], ts[2])) / reps
        rows.append({"format": fmt, "n_out": n_out, "n_in": n_in, "us": round(ms * 1e3, 2),
                     "GB/s": round(alg_bytes(fmt, n_out, n_in) / (ms * 1e-3) / 1e9, 1)})
        del g_wo
    del g_all
    capi.check()
    for h in handles:
        lib.sdy_qmat_free(h)
    return {"note": "batch 1, Q8_0 activations, per-matrix device time (sweep with / without it)",
            "per_matrix": rows}


def run_b200(args, rank, world, local_rank):
    """The config-2 sweep at batch 1. With N ranks every matrix is split by rows (whole 8-row
    groups): each GPU streams its slice and the step ends with one all-gather of every matrix's
    y slices (NCCL), so value = all bytes of the full matrices / the slowest rank's time."""
    import torch
    import torch.distributed as dist
    from sardyne_b200 import capi

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    lib = capi.lib()
    full, xs = make_inputs(only=args.only)
    if not full:
        raise SystemExit(f"--only {args.only}: no such matrix in the sweep")
    stream = torch.cuda.Stream(device=dev)
    sp = ctypes.c_void_p(stream.cuda_stream)

    # this rank's row slices; each matrix's y slice goes to a fixed place of the gather buffer
    mats, ranges, share_off, share = [], [], [], 0
    for fmt, n_out, n_in, w in full:
        r0, r1 = shard_rows(n_out, rank, world)
        mats.append((fmt, r1 - r0, n_in, np.ascontiguousarray(w[r0:r1])))
        ranges.append((r0, r1))
        share_off.append(share)
        share += max(e - b for b, e in (shard_rows(n_out, q, world) for q in range(world)))
    handles, d_out, d_x, d_xq = [], [], {}, {}
    send = torch.zeros(share, dtype=torch.float32, device=dev)
    recv = torch.zeros(world * share, dtype=torch.float32, device=dev) if world > 1 else None
    # N > 1: the y slices are gathered over NVLink peer memory (sdy_allgather_p2p: each rank's GPU
    # stores its slice into every rank's buffer), or with NCCL's all-gather (--gather nccl)
    p2p = world > 1 and args.gather == "p2p"
    p2p_buf, p2p_bases = None, None
    if p2p:
        p2p_buf = lib.sdy_p2p_alloc(lib.sdy_allgather_p2p_bytes(share, world))
        if not p2p_buf:
            raise RuntimeError(capi.last_error())
        hbuf = (ctypes.c_char * 64)()
        if lib.sdy_p2p_handle(p2p_buf, hbuf) != 0:
            raise RuntimeError(capi.last_error())
        peer_handles = [None] * world
        dist.all_gather_object(peer_handles, bytes(hbuf))
        bases = []
        for q in range(world):
            p = p2p_buf if q == rank else lib.sdy_p2p_open((ctypes.c_char * 64).from_buffer_copy(peer_handles[q]))
            if not p:
                raise RuntimeError(capi.last_error())
            bases.append(p)
        p2p_bases = (ctypes.c_void_p * world)(*bases)

    def gather(stream_handle):
        if p2p:
            if lib.sdy_allgather_p2p(ctypes.c_void_p(send.data_ptr()), share, p2p_bases, rank, world,
                                     stream_handle) != 0:
                raise RuntimeError(capi.last_error())
        else:
            dist.all_gather_into_tensor(recv, send)

    def gathered_all():
        """Every rank's y slices as this rank holds them after the last gather (host copy)."""
        if p2p:
            out = torch.empty(world * share, dtype=torch.float32)
            torch.cuda.synchronize()
            lib.sdy_p2p_read(ctypes.c_void_p(out.data_ptr()), p2p_buf, out.numel() * 4)
            return out
        return recv.cpu()
    for i, (fmt, n_out, n_in, w) in enumerate(mats):
        h = lib.sdy_qmat_upload(w.ctypes.data, TYPE_ID[fmt], n_out, n_in)
        if not h:
            raise RuntimeError(capi.last_error())
        handles.append(h)
        d_out.append(send[share_off[i]:share_off[i] + n_out])
    for n_in, x in xs.items():
        d_x[n_in] = torch.from_numpy(x).to(dev)
        d_xq[n_in] = torch.empty(lib.sdy_xq_bytes(TYPE_ID["Q8_K"], n_in, 1), dtype=torch.uint8, device=dev)
    dominant = max(range(len(mats)), key=lambda i: alg_bytes(*mats[i][:3]))
    step_bytes = sum(alg_bytes(fmt, n_out, n_in) for fmt, n_out, n_in, _ in mats)

    def quantize_inputs():
        # once per distinct input, as the reference reuses its quantized activations across the
        # products that share them (csrc/model_llama.c:590-611)
        for n_in in xs:
            lib.sdy_quantize_rows_dev(TYPE_ID["Q8_K"], ctypes.c_void_p(d_x[n_in].data_ptr()), 1, n_in,
                                      ctypes.c_void_p(d_xq[n_in].data_ptr()), sp)

    def matvecs(skip=-1):
        """The sweep as single-product launches (the per-matrix breakdown), without product `skip`."""
        quantize_inputs()
        for i, (fmt, n_out, n_in, _) in enumerate(mats):
            if i != skip:
                lib.sdy_qmatvec_dev(handles[i], ctypes.c_void_p(d_xq[n_in].data_ptr()), 1,
                                    ctypes.c_void_p(d_out[i].data_ptr()), n_out, 0, n_out, sp)

    hs_arr = (ctypes.c_void_p * len(mats))(*handles)
    xq_arr = (ctypes.c_void_p * len(mats))(*[d_xq[n_in].data_ptr() for _, _, n_in, _ in mats])
    out_arr = (ctypes.c_void_p * len(mats))(*[o.data_ptr() for o in d_out])

    x_arr = (ctypes.c_void_p * len(mats))(*[d_x[n_in].data_ptr() for _, _, n_in, _ in mats])

    def grouped():
        """This rank's products of the sweep in one launch, each CTA quantizing its product's f32
        input row to Q8_K itself (sdy_qmatvec_batch_f32_dev): no quantization launch."""
        if lib.sdy_qmatvec_batch_f32_dev(len(mats), hs_arr, x_arr, out_arr, sp) != 0:
            raise RuntimeError(capi.last_error())

    off_arr = (ctypes.c_int64 * len(mats))(*share_off)

    def fused():
        """The products with the all-gather fused into the same launch: every output value is also
        stored into the peers' gather buffers, and the launch's last CTA exchanges round flags
        (sdy_qmatvec_batch_f32_gather_dev)."""
        if lib.sdy_qmatvec_batch_f32_gather_dev(len(mats), hs_arr, x_arr, off_arr, share, p2p_bases, rank, world,
                                                sp) != 0:
            raise RuntimeError(capi.last_error())

    def step():
        if p2p:  # every rank ends the step with every matrix's full y, in one launch
            fused()
            return
        grouped()
        if world > 1:
            gather(sp)

    def gathered_y(i, allv=None):
        if world == 1:
            return d_out[i].cpu()
        parts = []
        for q in range(world):
            b, e = shard_rows(full[i][1], q, world)
            parts.append(allv[q * share + share_off[i]: q * share + share_off[i] + (e - b)])
        return torch.cat(parts)

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
    torch.cuda.synchronize()
    capi.check()

    def capture(fn):
        """fn's launches (on `stream`) as a CUDA graph, replayed without host launch overhead."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
            fn()
        return g

    # per-matrix device time of this rank's slices (informational, outside the timed region):
    # 20 sweeps with and without the matrix, each as one graph (interleaved, so every matrix is
    # cold in L2 when it runs)
    reps = 20
    sweep_all = capture(lambda: [matvecs() for _ in range(reps)])
    per = []
    for i, (fmt, n_out, n_in, _) in enumerate(mats):
        sweep_wo = capture(lambda i=i: [matvecs(skip=i) for _ in range(reps)])
        ts = []
        for g in (sweep_wo, sweep_all, sweep_wo, sweep_all):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):  # a graph replays on the current stream
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        ms = (min(ts[1], ts[3]) - min(ts[0], ts[2])) / reps
        per.append({"format": fmt, "n_out": n_out, "n_in": n_in, "us": round(ms * 1e3, 2),
                    "GB/s": round(alg_bytes(fmt, n_out, n_in) / (ms * 1e-3) / 1e9, 1)})
        del sweep_wo
    del sweep_all

    # the timed step as one CUDA graph: the grouped launch of the 6 products with their input
    # quantization (N > 1: and the all-gather of y, fused into the same launch; --gather nccl: an
    # NCCL all-gather after it)
    step_graph = capture(step)
    with torch.cuda.stream(stream):
        step_graph.replay()
    torch.cuda.synchronize()

    # timed region
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = lib.sdy_kernel_launches()
    with ClockSampler(torch.cuda.current_device()) as clk:
        barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            start.record(stream)
            for k in range(args.steps):
                step_graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
        barrier()
    # launches recorded in the graph once, replayed every step
    launches_per_step = 1
    # The step's dominant kernel, the grouped launch, timed per launch: eager launches each bracketed
    # by events on its stream, queued behind a ~10 ms spin kernel so that the host is ahead of the
    # GPU and no host launch gap falls inside a bracket. The single largest product (the Q6_K LM
    # head) is timed the same way for comparison.
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    evs1 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    fmt_d, o_d, i_d, _ = mats[dominant]
    with torch.cuda.stream(stream):
        torch.cuda._sleep(20_000_000)
        for k in range(args.steps):
            evs[k][0].record(stream)
            grouped()
            evs[k][1].record(stream)
        torch.cuda._sleep(20_000_000)
        for k in range(args.steps):
            evs1[k][0].record(stream)
            lib.sdy_qmatvec_dev(handles[dominant], ctypes.c_void_p(d_xq[i_d].data_ptr()), 1,
                                ctypes.c_void_p(d_out[dominant].data_ptr()), o_d, 0, o_d, sp)
            evs1[k][1].record(stream)
            grouped()  # the rest of the sweep between launches (the next LM head launch is cold in L2)
    torch.cuda.synchronize()
    launches = launches_per_step * args.steps
    capi.check()
    ms_total = start.elapsed_time(end)
    tm = torch.tensor([ms_total], dtype=torch.float64, device=dev)
    tb = torch.tensor([step_bytes], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
    ms_max, all_bytes = float(tm.item()), float(tb.item())
    value = all_bytes * args.steps / (ms_max * 1e-3) / 1e9
    grp_ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    dom_ms = statistics.mean(a.elapsed_time(b) for a, b in evs1)
    fmt, n_out, n_in, _ = mats[dominant]
    peak, peak_kind = load_peaks()
    achieved = step_bytes / (grp_ms * 1e-3) / 1e9
    achieved1 = alg_bytes(fmt, n_out, n_in) / (dom_ms * 1e-3) / 1e9
    traffic, traffic1 = load_traffic() if world == 1 and not args.only else (None, None)
    allv = gathered_all() if world > 1 else None
    y_dev = [gathered_y(i, allv) for i in range(len(mats))]

    # e2e through the reference-facing C-ABI with host buffers: op_matmul of this rank's slices
    # (pinned f32 x in, host y out), then (N > 1) the host slices gathered over NCCL
    x_pin = {n_in: torch.from_numpy(x).pin_memory() for n_in, x in xs.items()}
    y_pin = [torch.empty(n_out, dtype=torch.float32).pin_memory() for _, n_out, _, _ in mats]
    h_send = torch.empty(share, dtype=torch.float32).pin_memory()
    h_recv = torch.empty(world * share, dtype=torch.float32).pin_memory()
    for fmt, n_out, n_in, w in mats:
        if lib.sdy_weights_register(w.ctypes.data, TYPE_ID[fmt], n_out, n_in) != 0:
            raise RuntimeError(capi.last_error())

    def e2e_step():
        for i, (fmt, n_out, n_in, w) in enumerate(mats):
            lib.op_matmul(ctypes.c_void_p(y_pin[i].data_ptr()), ctypes.c_void_p(x_pin[n_in].data_ptr()),
                          w.ctypes.data, TYPE_ID[fmt], 1, n_in, n_out)
        if world > 1:
            for i, y in enumerate(y_pin):
                h_send[share_off[i]:share_off[i] + y.numel()].copy_(y)
            send.copy_(h_send)
            if p2p:
                gather(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
                torch.cuda.current_stream().synchronize()
                lib.sdy_p2p_read(ctypes.c_void_p(h_recv.data_ptr()), p2p_buf, h_recv.numel() * 4)
            else:
                dist.all_gather_into_tensor(recv, send)
                h_recv.copy_(recv)

    for _ in range(max(args.warmup, 3)):
        e2e_step()
    e2e_steps = max(10, args.steps // 4)
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    capi.check()
    # the product through the C-ABI equals the device-resident one, and (N > 1) the gathered y
    # equals every rank's slices in row order
    for i in range(len(mats)):
        assert torch.equal(y_pin[i], d_out[i].cpu()), "e2e/device mismatch"
    if world > 1:
        for i in range(len(mats)):
            r0, r1 = ranges[i]
            assert torch.equal(y_dev[i][r0:r1], y_pin[i]), "gathered y differs from this rank's slice"
    e2e_value = all_bytes * e2e_steps / float(te.item()) / 1e9
    for _, _, _, w in mats:
        lib.sdy_weights_unregister(w.ctypes.data)
    for h in handles:
        lib.sdy_qmat_free(h)
    if p2p:
        if lib.sdy_p2p_status() != 0:
            raise RuntimeError("a peer-memory gather wait gave up")
        del step_graph  # holds launches that name the peers' buffers
        barrier()
        for q in range(world):
            if q != rank:
                lib.sdy_p2p_close(p2p_bases[q])
        barrier()
        lib.sdy_p2p_free(p2p_buf)

    formats32 = measure_formats32(lib, dev) if world == 1 and not args.only else None
    decode = None
    if not args.no_decode:
        decode = measure_decode("qwen3moe", args, rank, world, cpu_baseline=not args.no_cpu_baseline)
    if rank != 0:
        return 0
    line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config(world, args.gather),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": f"grouped qmv: this rank's {len(mats)} products and their input "
                                   f"quantization in one launch",
                         "peak_source": peak_kind, "algorithmic_bytes": step_bytes,
                         "launch_us": round(grp_ms * 1e3, 2)},
            "roofline_single": {"bound": "hbm", "achieved": round(achieved1, 1), "peak": peak, "unit": "GB/s",
                                "frac": round(achieved1 / peak, 4), "traffic": traffic1,
                                "kernel": f"qmv {fmt} {n_out}x{n_in} batch 1", "peak_source": peak_kind,
                                "algorithmic_bytes": alg_bytes(fmt, n_out, n_in), "launch_us": round(dom_ms * 1e3, 2)},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": sum(4 * n_in for _, _, n_in, _ in mats),
                    "d2h_bytes_per_step": sum(4 * n_out for _, n_out, _, _ in mats),
                    "steps": e2e_steps, "api": "op_matmul (C-ABI), weights resident via sdy_weights_register"
                                               + (f", y slices all-gathered ({args.gather})" if world > 1 else "")},
            "gpu_launches": int(launches), "clocks": clk.summary(),
            "frac_of_8tbs": round(value / world / 8000.0, 4), "per_matrix": per}
    if world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = time_reference(full, xs)
        except OSError as e:
            line["cpu_baseline"] = {"value": None, "unavailable": str(e)}
    if formats32 is not None:
        line["formats_32"] = formats32
    if decode is not None:
        line["decode"] = decode
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------------------ GEMM workload

def run_gemm(args):
    """BASELINE config 2 at batches 128 and 512: the sweep's matrices of every format times many
    tokens, through the tensor-core GEMM (int8 tcgen05 MMAs, exact per-superblock / per-block
    combine). Reports useful multiply-add throughput (2 * n_out * n_in * tokens per product) per
    matrix and batch; `value` is the best Q4_K/Q6_K product."""
    import torch
    from sardyne_b200 import capi
    torch.cuda.set_device(0)
    lib = capi.lib()
    mats, _ = make_inputs(only=args.only, formats=FORMATS + FORMATS32)
    stream = torch.cuda.Stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    rows = []
    peak_tf = None
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        peak_tf = json.loads(p.read_text()).get("bf16_tflops")
    launches0 = lib.sdy_kernel_launches()
    for fmt, n_out, n_in, w in mats:
        h = lib.sdy_qmat_upload(w.ctypes.data, TYPE_ID[fmt], n_out, n_in)
        if not h:
            raise RuntimeError(capi.last_error())
        vt = TYPE_ID[act_type(fmt)]
        for batch in (128, 512):
            x = torch.randn(batch, n_in, device="cuda")
            xq = torch.empty(lib.sdy_xq_bytes(vt, n_in, batch), dtype=torch.uint8, device="cuda")
            y = torch.empty(batch, n_out, device="cuda")
            with torch.cuda.stream(stream):
                lib.sdy_quantize_rows_dev(vt, ctypes.c_void_p(x.data_ptr()), batch, n_in,
                                          ctypes.c_void_p(xq.data_ptr()), sp)

                def prod():
                    lib.sdy_qmatvec_dev(h, ctypes.c_void_p(xq.data_ptr()), batch, ctypes.c_void_p(y.data_ptr()),
                                        n_out, 0, n_out, sp)
                for _ in range(max(args.warmup, 3)):
                    prod()
                reps = max(3, min(args.steps, 50))
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    prod()
                e1.record(stream)
            torch.cuda.synchronize()
            capi.check()
            if lib.sdy_kernel_status() != 0:
                raise RuntimeError("GEMM completion wait timed out")
            us = e0.elapsed_time(e1) / reps * 1e3
            tops = 2.0 * n_out * n_in * batch / (us * 1e-6) / 1e12
            rows.append({"format": fmt, "n_out": n_out, "n_in": n_in, "batch": batch, "us": round(us, 1),
                         "TOPS": round(tops, 1), "tok_s": round(batch / (us * 1e-6), 1)})
        lib.sdy_qmat_free(h)
    best = max((r for r in rows if r["format"] in FORMATS), key=lambda r: r["TOPS"])
    line = {"metric": "Q4_K/Q6_K prefill GEMM useful int8 TOPS (exact per-superblock combine)",
            "value": best["TOPS"], "unit": "TOPS", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "BASELINE config 2 at batches 128 and 512 (Q8_K activations resident)"},
            "roofline": {"bound": "tensor", "achieved": best["TOPS"], "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": round(best["TOPS"] / peak_tf, 4) if peak_tf else None,
                         "peak_source": "measured bf16 cuBLAS (int8 dense nominal is 2x bf16)",
                         "kernel": f"qgemm {best['format']} {best['n_out']}x{best['n_in']} batch {best['batch']}"},
            "gpu_launches": int(lib.sdy_kernel_launches() - launches0), "per_matrix": rows}
    print(json.dumps(line))
    return 0


# ------------------------------------------------------------------------------ decode workload

DECODE_MODELS = {  # prompt length, decode steps, max context
    "smollm2": (128, 256, 2048),
    "qwen25_3b": (512, 512, 4096),
    "qwen3moe": (256, 256, 4096),
}
REF_DECODE_SAMPLE = (32, 16)  # reference CPU sample: prompt tokens, decode steps


def engine_open(lib, path, max_seq, n_batch, n_threads=0):
    """(model, context, info) handles of the engine_* C-ABI of `lib` (this build or the reference)."""
    from sardyne_b200 import capi
    err = ctypes.create_string_buffer(512)
    model = lib.engine_model_load(str(path).encode(), err, len(err))
    if not model:
        raise RuntimeError(err.value.decode(errors="replace"))
    info = capi.EngineModelInfo()
    lib.engine_model_get_info(model, ctypes.byref(info))
    ctx = lib.engine_ctx_new(model, max_seq, n_batch, 0, n_threads, err, len(err))
    if not ctx:
        lib.engine_model_free(model)
        raise RuntimeError(err.value.decode(errors="replace"))
    return model, ctx, info


def engine_next(lib, ctx, tokens, n_vocab):
    """engine_eval of `tokens`, then the greedy choice from the host logits it returns."""
    arr = (ctypes.c_int32 * len(tokens))(*tokens)
    if lib.engine_eval(ctx, arr, len(tokens)) != 0:
        raise RuntimeError(lib.engine_last_error(ctx).decode(errors="replace"))
    logits = np.ctypeslib.as_array(lib.engine_logits(ctx), shape=(n_vocab,))
    return int(np.argmax(logits))


def weight_bytes_per_token(path, info):
    """Weight bytes one decode token reads: every matrix; of the experts only k of n; of an
    untied embedding table only the looked-up row."""
    from sardyne_b200 import capi
    lib = capi.lib()
    err = ctypes.create_string_buffer(256)
    h = lib.gguf_open(str(path).encode(), err, len(err))
    total = 0
    for i in range(lib.gguf_n_tensors(h)):
        t = lib.gguf_get_tensor(h, i).contents
        name, nb = t.name.decode(), t.nbytes
        if "_exps" in name:
            nb = nb * info.n_expert_used // info.n_expert
        if name == "token_embd.weight" and not info.tied_embeddings:
            nb = nb // info.n_vocab
        total += nb
    lib.gguf_close(h)
    return total


def decode_reference(name, path, prompt):
    """The reference engine (oracle/_ref, AVX2 kernels, one thread per host core) on a bounded
    sample of the same workload: the first 32 prompt tokens, then 16 greedy decode steps."""
    import oracle
    n_prompt, n_decode = REF_DECODE_SAMPLE
    ref = oracle.ref()
    ref.op_set_simd(1)
    cores = min(host_cores(), 256)  # the reference's thread pool takes 1..256 (csrc/model_llama.c:475-487)
    model, ctx, info = engine_open(ref, path, n_prompt + n_decode + 1, n_prompt, n_threads=cores)
    try:
        t0 = time.perf_counter()
        nxt = engine_next(ref, ctx, prompt[:n_prompt], info.n_vocab)
        t1 = time.perf_counter()
        for _ in range(n_decode):
            nxt = engine_next(ref, ctx, [nxt], info.n_vocab)
        t2 = time.perf_counter()
    finally:
        ref.engine_ctx_free(ctx)
        ref.engine_model_free(model)
    return {"value": round(n_decode / (t2 - t1), 3), "unit": "tok/s", "cores": cores, "kind": "reference",
            "prefill_tok_s": round(n_prompt / (t1 - t0), 2),
            "sample": f"reference engine_eval (oracle/_ref, AVX2, {cores} threads) on the same model: "
                      f"{n_prompt}-token prompt, then {n_decode} greedy decode steps"}


def measure_decode(name, args, rank, world, cpu_baseline=True):
    """Decode of a BASELINE config 3-5 model through engine_eval (host token ids in, host logits
    out): the prompt's prefill, then greedy single-token steps. Under torchrun every rank runs the
    same token stream with its shard of the model (attention heads where they divide, FFN rows,
    experts, vocabulary) and the engine's exchanges: strong scaling of one stream; times are the max
    over ranks. Returns the decode object (rank 0) or None."""
    import torch
    import torch.distributed as dist
    from sardyne_b200 import capi, runtime, synth
    n_prompt, n_decode, ctx_len = DECODE_MODELS[name]
    n_decode = args.decode_steps or n_decode
    layers = getattr(args, "layers", 0) or 0
    if world > 1:
        if rank == 0:
            synth.baseline_model(name, args.model_dir, layers)  # written once, before the other ranks open it
        dist.barrier()
        runtime.shard_from_torch()
    path = synth.baseline_model(name, args.model_dir, layers)
    lib = capi.lib()
    t0 = time.perf_counter()
    model, ctx, info = engine_open(lib, path, ctx_len, n_prompt)
    load_s = time.perf_counter() - t0
    prompt = np.random.default_rng(0).integers(0, info.n_vocab, n_prompt).tolist()
    try:
        nxt = engine_next(lib, ctx, prompt, info.n_vocab)  # warm-up: prefill, then decode steps
        for _ in range(max(args.warmup, 3)):               # (the second one captures the graphs)
            nxt = engine_next(lib, ctx, [nxt], info.n_vocab)
        lib.engine_reset(ctx)
        launches0 = lib.sdy_kernel_launches()
        with ClockSampler(torch.cuda.current_device()) as clk:
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            nxt = engine_next(lib, ctx, prompt, info.n_vocab)
            t1 = time.perf_counter()
            tokens = []
            for _ in range(n_decode):
                tokens.append(nxt)
                nxt = engine_next(lib, ctx, [nxt], info.n_vocab)
            t2 = time.perf_counter()
        launches = int(lib.sdy_kernel_launches() - launches0)
        capi.check()
        # the same stream with the greedy choice made on the device (sdy_engine_eval_greedy): no
        # logits copied back; every rank must choose the same ids as through the host logits
        lib.engine_reset(ctx)
        nxt_dev = ctypes.c_int32()
        arr = (ctypes.c_int32 * n_prompt)(*prompt)
        if world > 1:
            dist.barrier()
        t3 = time.perf_counter()
        if lib.sdy_engine_eval_greedy(ctx, arr, n_prompt, ctypes.byref(nxt_dev)) != 0:
            raise RuntimeError(lib.engine_last_error(ctx).decode(errors="replace"))
        t4 = time.perf_counter()
        dev_tokens = []
        for _ in range(n_decode):
            dev_tokens.append(nxt_dev.value)
            one = (ctypes.c_int32 * 1)(nxt_dev.value)
            if lib.sdy_engine_eval_greedy(ctx, one, 1, ctypes.byref(nxt_dev)) != 0:
                raise RuntimeError(lib.engine_last_error(ctx).decode(errors="replace"))
        t5 = time.perf_counter()
        if dev_tokens != tokens:
            raise RuntimeError("device greedy choice differs from numpy.argmax of the logits")
        # two more prefills of the same prompt: prefill_tok_s is the median of four
        prefills = [t1 - t0, t4 - t3]
        for _ in range(2):
            lib.engine_reset(ctx)
            if world > 1:
                dist.barrier()
            ta = time.perf_counter()
            engine_next(lib, ctx, prompt, info.n_vocab)
            prefills.append(time.perf_counter() - ta)
    finally:
        lib.engine_ctx_free(ctx)  # graphs and NCCL communicator released before the process group
        lib.engine_model_free(model)
        if world > 1:
            runtime.set_shard(0, 1)
    if world > 1:  # the slowest rank's times; every rank must agree on the tokens
        dev = torch.device("cuda", torch.cuda.current_device())
        tt = torch.tensor([t1 - t0, t2 - t1, t5 - t4] + prefills, dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t0, t1, t2 = 0.0, float(tt[0]), float(tt[0] + tt[1])
        t4, t5 = 0.0, float(tt[2])
        prefills = [float(v) for v in tt[3:]]
        toks = [None] * world
        dist.all_gather_object(toks, tokens)
        if any(tk != tokens for tk in toks):
            raise RuntimeError("ranks disagree on the greedy tokens")
    if rank != 0:
        return None
    wbytes = weight_bytes_per_token(path, info)
    peak, peak_kind = load_peaks()
    tps = n_decode / (t2 - t1)
    out = {"metric": f"decode tok/s {name} shape (greedy, e2e through engine_eval)", "value": round(tps, 2),
           "unit": "tok/s", "n_gpus": world, "steps": n_decode, "ms_per_step": round((t2 - t1) / n_decode * 1e3, 4),
           "prefill_tok_s": round(n_prompt / statistics.median(prefills), 1),
           "prefill_ms_samples": [round(v * 1e3, 2) for v in prefills],
           "scaling": "strong" if world > 1 else "weak",
           "workload": f"BASELINE {name} shape{f' cut to {layers} layers' if layers else ''}: {n_prompt}-token "
                       f"prompt (uniform ids, seed 0), {n_decode} greedy decode steps, context {ctx_len}; "
                       f"random-init Q4_K_M mix",
           "model_gb": round(path.stat().st_size / 1e9, 2), "weight_bytes_per_token": wbytes,
           "parallelism": (f"x{world}: " + ("attention replicated" if os.environ.get("SARDYNE_ATTN_TP") == "off"
                                            else "attention heads split where they divide")
                           + ", ffn rows / experts / vocabulary split; single-token exchanges over NVLink peer "
                             "memory" + (" (NCCL)" if os.environ.get("SARDYNE_EXCHANGE") == "nccl" else ""))
           if world > 1 else "1 GPU",
           "roofline": {"bound": "hbm", "achieved": round(wbytes * tps / 1e9, 1), "peak": round(peak * world, 1),
                        "unit": "GB/s", "frac": round(wbytes * tps / 1e9 / (peak * world), 4), "traffic": None,
                        "kernel": "whole decode step (weight bytes per token x tok/s, against N x peak)",
                        "peak_source": peak_kind},
           "e2e": {"value": round(tps, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                   "d2h_bytes_per_step": 4 * info.n_vocab},
           "greedy_on_device_tok_s": round(n_decode / (t5 - t4), 2),
           "gpu_launches": launches, "clocks": clk.summary(), "load_s": round(load_s, 2),
           "first_tokens": tokens[:8]}
    if cpu_baseline and world == 1:
        try:
            out["cpu_baseline"] = decode_reference(name, path, prompt)
        except (OSError, RuntimeError) as e:
            out["cpu_baseline"] = {"value": None, "unavailable": str(e)}
    return out


def run_decode(args, rank, world):
    """--workload decode: the decode measurement alone, as the line's value."""
    d = measure_decode(args.model, args, rank, world, cpu_baseline=not args.no_cpu_baseline)
    if d is None:
        return 0
    line = {k: d[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "ms_per_step", "scaling")}
    line.update({"warmup": args.warmup, "higher_is_better": True, "vs_baseline": None, "dtype": "int8",
                 "data": "synthetic", "config": {"workload": d["workload"], "parallelism": d["parallelism"]}})
    line.update({k: v for k, v in d.items() if k not in line and k not in ("workload", "parallelism")})
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["matvec", "decode", "gemm"], default="matvec")
    ap.add_argument("--model", choices=sorted(DECODE_MODELS), default="qwen3moe")
    ap.add_argument("--model-dir", default=None, help="where the synthetic GGUFs are cached (default: "
                                                         "SARDYNE_MODEL_DIR, /dev/shm or the temp dir)")
    ap.add_argument("--no-decode", action="store_true", help="matvec: leave out the decode object")
    ap.add_argument("--gather", choices=["p2p", "nccl"], default="p2p",
                    help="matvec, N > 1: all-gather of y over peer memory (own kernel) or with NCCL")
    ap.add_argument("--decode-steps", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0,
                    help="decode: the model's shape with only this many layers (small cases for ncu captures)")
    ap.add_argument("--profile-step", action="store_true",
                    help="decode: run one extra step between cudaProfilerStart/Stop (ncu --profile-from-start off)")
    ap.add_argument("--only", default=None, help="matvec: keep one matrix, e.g. Q6_K:151936 (for ncu captures)")
    args = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.workload == "gemm":
        return run_gemm(args)
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "decode":
            return run_decode(args, rank, world)
        return run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())

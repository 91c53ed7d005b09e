#!/usr/bin/env python3
"""bench.py -- throughput of the B200 resident-weight matmul engine on BASELINE configs[1].

Workload (one "step"): the w8a8 per-channel GEMM sweep of configs[1] -- (K,N) in {(2048,2048),
(2048,6144),(6144,2048)} x M in {1,8,128,512}, twelve ork_i8_mm_run calls -- with B ~ N(0,0.02) given as
f32 [N][K] to ork_i8_mm_pack_f32 and A int8 ~ U[-127,127]. Metric: algorithmic HBM GB/s,
bytes = K*N (weight) + M*K (A) + 4*M*N (int32 C) per call, summed over the step and divided by the step
time; every config is HBM-bound by that formula on B200 (int32 C is heavy), so GB/s is the common unit.

- value: device-resident inputs, the twelve calls queued back to back on the library's stream
  (ork_b200_i8_mm_run_async, with programmatic dependent launch) and replayed as one CUDA graph per step,
  timed with CUDA events on that stream, max over ranks.
- e2e: the same sweep through the synchronous public call ork_i8_mm_run with pinned host buffers: each
  call copies A in, runs, copies C out and synchronises.
- L2: inputs larger than L2 -- 9 distinct packed copies of every weight (265 MB) plus per-copy A/C
  buffers, cycled so no call finds its weight in the 126 MB L2.
- roofline: the dominant kernel (largest share of the step) timed alone with CUDA events.
- cpu_baseline / --impl reference: the reference's own CPU int8 GEMM (orki_cpu_gemm_i32 via
  ork_i8_mm_run_cpu in oracle/_ref, OpenMP over M on all host cores) on the same sweep.

Multi-GPU (torchrun, --gpus N): configs[1] does not shard, so every rank runs an independent replica of
the sweep; value = total bytes of all ranks / max rank time (weak scaling).
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ork-driver_b200"))

SHAPES = [(2048, 2048), (2048, 6144), (6144, 2048)]
MS = [1, 8, 128, 512]
CONFIGS = [(K, N, M) for (K, N) in SHAPES for M in MS]
NCOPIES = 9
WORKLOAD = ("w8a8 per-channel GEMM (BASELINE configs[1]): (K,N) in {(2048,2048),(2048,6144),(6144,2048)} x "
            "M in {1,8,128,512}; B~N(0,0.02) f32 -> ork_i8_mm_pack_f32, A int8~U[-127,127], C int32")
METRIC = "w8a8 GEMM algorithmic HBM GB/s (configs[1] sweep)"


def alg_bytes(K, N, M):
    return K * N + M * K + 4 * M * N


STEP_BYTES = sum(alg_bytes(K, N, M) for K, N, M in CONFIGS)
STEP_OPS = sum(2 * M * K * N for K, N, M in CONFIGS)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock and throttle reasons sampled every ~2 ms (NVML) while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, dev):
        self.dev, self.samples, self.stop, self.t = dev, [], threading.Event(), None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self.max = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def loop():
                while not self.stop.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, rs))
                    except Exception:
                        pass
                    time.sleep(0.002)

            self.t = threading.Thread(target=loop, daemon=True)
            self.t.start()
        except Exception:
            self.max = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.t:
            self.t.join(timeout=2)

    def summary(self):
        sm = [s for s, _ in self.samples]
        reasons = sorted({n for _, rs in self.samples for n, bit in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max, "reasons": reasons,
                "samples": len(sm), "source": "nvml"}


def cpu_model():
    """The host CPU's model name (the CPU baseline runs on it)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def host_cores():
    """Host CPU threads this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_reference_sweep(min_seconds, max_reps=3):
    """The reference's CPU int8 GEMM over the sweep: oracle/_ref (its own code) if built, else the
    restatement, with an OpenMP team of every host core (set explicitly: torchrun exports
    OMP_NUM_THREADS=1). Returns (GB/s, cores, kind, sample description, seconds per sweep)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_ffi as of

    of.restated().orc_set_threads(host_cores())

    ref = of.reference()
    kind = "reference" if ref is not None else "port"
    rng = np.random.default_rng(0)
    data = []
    for K, N in SHAPES:
        f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        codes, _ = of.i8_quant_f32(f32)
        B = np.ascontiguousarray(codes.T)
        for M in MS:
            A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
            data.append((K, N, M, A, B, np.zeros((M, N), np.int32)))
    fn = ref.ork_i8_mm_run_cpu if ref is not None else of.restated().orc_gemm_i32
    reps, t_total = 0, 0.0
    while reps < max_reps and (reps == 0 or t_total < min_seconds):
        t0 = time.perf_counter()
        for K, N, M, A, B, Cm in data:
            fn(M, K, N, of._p(A), of._p(B), of._p(Cm))
        t_total += time.perf_counter() - t0
        reps += 1
    cores = of.restated().orc_threads()
    gbs = STEP_BYTES * reps / t_total / 1e9
    sample = f"{reps} full sweep(s) of the 12 configs[1] calls ({t_total:.2f} s)"
    return gbs, cores, kind, sample, t_total / reps


def run_reference(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    per_step = []
    cores = kind = sample = None
    for _ in range(args.warmup):
        cpu_reference_sweep(0.0, 1)
    for _ in range(args.steps):
        gbs, cores, kind, sample, t = cpu_reference_sweep(0.0, 1)
        per_step.append(t)
    t = statistics.mean(per_step)
    value = STEP_BYTES / t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": "host CPU, OpenMP over M"},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": kind, "cpu": cpu_model(),
                             "sample": f"each step = one full sweep of the 12 calls on the host ({sample})"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def other_configs(ctx, L, stream, ncopies=10, reps=10):
    """The remaining BASELINE configs, timed like the breakdown (each config alone, CUDA graph of
    `ncopies` calls over distinct weight copies): configs[0] fp16, configs[2] w4a8 (uniform and NF4, with
    an imatrix) and W4A4. Algorithmic bytes per call: fp16 2KN+2MK+4MN, int4 KN/2+MK+4MN."""
    import torch

    import ork_b200

    rng = np.random.default_rng(99)
    out = {}

    def check(kind, fmt, w, A, Cm, K, N):
        """C of one call against an exact int32 GEMM of the weight's codes (integer formats), or an fp32
        matmul of the same fp16 values within 1e-3 * sqrt(K) * max|A| * max|B| (fp16)."""
        if kind == "f16":
            raw = np.zeros(K * N * 2, np.uint8)
            assert L.ork_b200_weight_read(w.h, raw.ctypes.data, raw.nbytes) == raw.nbytes
            Wt = torch.from_numpy(raw.view(np.float16).reshape(N, K)).cuda().float()
            ref = A.float() @ Wt.t()
            tol = 1e-3 * np.sqrt(K) * float(A.float().abs().max()) * float(Wt.abs().max())
            return float((Cm - ref).abs().max()) <= tol
        return bool(torch.equal(Cm, exact_i32(A, resident_codes(ctx, w, fmt))))

    def timed(kind, w_list, K, N, M, fmt):
        dtype_in = torch.float16 if kind == "f16" else torch.int8
        dtype_out = torch.float32 if kind == "f16" else torch.int32
        if kind == "f16":
            A = [(torch.rand((M, K), device="cuda") * 2 - 1).to(torch.float16) for _ in range(ncopies)]
        else:
            lo, hi = (-7, 8) if kind == "i4" else (-127, 128)
            A = [torch.randint(lo, hi, (M, K), dtype=dtype_in, device="cuda") for _ in range(ncopies)]
        C = [torch.empty((M, N), dtype=dtype_out, device="cuda") for _ in range(ncopies)]
        fn = {"f16": L.ork_b200_f16_mm_run_async, "i8": L.ork_b200_i8_mm_run_async, "i4": L.ork_b200_i4_mm_run_async}[kind]
        for i in range(ncopies):
            assert fn(ctx.ctx, w_list[i].h, M, A[i].data_ptr(), C[i].data_ptr()) == 0
        torch.cuda.synchronize()
        assert L.ork_b200_sync(ctx.ctx) == 0
        if not check(kind, fmt, w_list[0], A[0], C[0], K, N):
            print(json.dumps({"error": f"{fmt} {K}x{N} M{M}: C differs from the checker"}), flush=True)
            raise SystemExit(3)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(ncopies):
                fn(ctx.ctx, w_list[i].h, M, A[i].data_ptr(), C[i].data_ptr())
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (reps * ncopies), L.ork_b200_route(w_list[0].h, M)

    def record(name, kind, ws, K, N, Ms, wbytes, fmt):
        for M in Ms:
            ms, route = timed(kind, ws, K, N, M, fmt)
            abytes = M * K * (2 if kind == "f16" else 1)
            by = wbytes + abytes + 4 * M * N
            out[f"{name} {K}x{N} M{M}"] = {"us": ms * 1e3, "GB/s": by / (ms / 1e3) / 1e9,
                                           "TOPS": 2 * M * K * N / (ms / 1e3) / 1e12, "route": route,
                                           "parity": "within tolerance" if kind == "f16" else "exact"}

    # fp16 K=2048 N=6144, M in {1, 64}; B ~ N(0, 0.02)
    K, N = 2048, 6144
    B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    ws = [ctx.f16_pack(B) for _ in range(ncopies)]
    record("fp16", "f16", ws, K, N, (1, 64), 2 * K * N, "f16")
    for w in ws:
        w.free()
    # w4a8 uniform / NF4 with imatrix ~ U(0.5, 2), and W4A4 with A ~ U[-7, 7]
    for K, N in ((6144, 2048), (2048, 12288)):
        f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        im = (rng.random(K, dtype=np.float32) * np.float32(1.5) + np.float32(0.5)).astype(np.float32)
        for nf4 in (False, True):
            blob = ork_b200.cpu_blob(f32, im, nf4=nf4)
            ws = [ctx.i4a8_load(blob, K, N) for _ in range(ncopies)]
            record("w4a8-" + ("nf4" if nf4 else "uniform"), "i8", ws, K, N, (1, 32, 256), K * N // 2,
                   "nf4" if nf4 else "u4")
            for w in ws:
                w.free()
        B4 = rng.integers(-7, 8, size=(K, N), dtype=np.int8)
        ws = [ctx.i4_pack(B4) for _ in range(ncopies)]
        record("w4a4", "i4", ws, K, N, (1, 32, 256), K * N // 2, "u4")
        for w in ws:
            w.free()
    return out


# Llama-70B-shaped linear stack of BASELINE configs[4]: hidden 8192, FFN 28672, 80 layers, vocab 128256;
# GQA 64 query / 8 key-value heads of 128 (QKV N = 8192 + 2*1024), gate and up fused into one N = 57344
# weight. (K, N) per linear; the LM head runs once per pass.
L70 = {"layers": 80, "linears": [("qkv", 8192, 10240), ("o", 8192, 8192), ("gate_up", 8192, 57344),
                                 ("down", 28672, 8192)], "lm_head": (8192, 128256)}
# NF4 codebook as int8 codes, lut[i] = rint(level[i] * 127) (ork-driver src/npu/i4/pack.c:128-131 over the
# levels of src/npu.c:888-892): the format's decoding table, used to rebuild a weight's int8 codes from
# its resident nibbles for the benchmark's own result checks
NF4_LUT = [-127, -88, -67, -50, -36, -23, -12, 0, 10, 20, 31, 43, 56, 71, 92, 127]


def resident_codes(ctx, w, fmt):
    """The int8 codes [N][K] of a packed weight as a device tensor, rebuilt from its resident bytes (int8
    as stored; uniform int4 nibbles sign-extended; NF4 nibbles through the codebook), low nibble = even k."""
    import torch

    raw = np.zeros(ctx.L.ork_b200_weight_read(w.h, None, 0), np.uint8)
    assert ctx.L.ork_b200_weight_read(w.h, raw.ctypes.data, raw.nbytes) == raw.nbytes
    t = torch.from_numpy(raw).cuda()
    if fmt == "i8":
        return t.view(torch.int8).view(w.N, w.K)
    lo, hi = (t & 15).to(torch.int16), (t >> 4).to(torch.int16)
    if fmt == "nf4":
        lut = torch.tensor(NF4_LUT, dtype=torch.int16, device="cuda")
        lo, hi = lut[lo.long()], lut[hi.long()]
    else:
        lo, hi = (lo ^ 8) - 8, (hi ^ 8) - 8
    return torch.stack((lo, hi), dim=-1).view(w.N, w.K).to(torch.int8)


def exact_i32(A, codes_nk):
    """C = A . codes^T in exact int32 on the device through torch._int_mm (cuBLASLt): an independent exact
    GEMM that checks the benchmark's own calls outside the timed regions (integer sums have one right
    answer, so any exact int32 GEMM is a valid checker). A [M][K] int8, codes [N][K] int8."""
    import torch

    M, K = A.shape
    Mp = max(32, (M + 7) // 8 * 8)
    Ap = torch.zeros((Mp, K), dtype=torch.int8, device=A.device)
    Ap[:M] = A
    return torch._int_mm(Ap, codes_nk.t().contiguous())[:M]


def sharded_70b(args, Ms, dist=None):
    """every weight NF4 (w4a8, B ~ N(0, 0.02)), column-sharded over the ranks of the job; each
    matmul runs on the local shard and its int32 C reaches every rank -- over NVLink peer memory (the
    library's fused gather: the shard's columns stored into every rank's C, a bounded signal wait) or,
    with --gather nccl, by an NCCL all-gather. One step = one pass of M tokens through the 80 layers' four
    linears and the LM head, captured as one CUDA graph. Each rank quantizes its own channel slice once on
    the host and loads enough distinct copies of a layer that its per-pass working set exceeds L2. Before
    timing, every linear's C is checked: this rank's columns against an exact int32 GEMM of its own
    resident codes, and the whole gathered C by a checksum that must agree on every rank.
    Returns ({"M<m>": result}, description)."""
    import torch

    import ork_b200
    import shard

    world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
    rank = dist.get_rank() if world > 1 else 0
    local = int(os.environ.get("LOCAL_RANK", "0"))
    L = ork_b200.lib()
    ctx = ork_b200.Context()
    stream = torch.cuda.Stream()
    L.ork_b200_set_stream(ctx.ctx, stream.cuda_stream)
    layer_bytes = sum(K * N // 2 for _, K, N in L70["linears"]) // world
    ncopies = max(2, -(-400 * 2 ** 20 // layer_bytes))
    gen = torch.Generator(device="cuda").manual_seed(4242 + rank)

    def packed(K, N, copies):
        n0, n1 = shard.shard_range(N, rank, world)
        # N(0, 0.02) weights drawn on the device (fast), quantized to NF4 on the host by the library's packer
        f32 = (torch.randn((n1 - n0, K), device="cuda", generator=gen) * 0.02).cpu().numpy()
        blob = ork_b200.cpu_blob(f32, None, nf4=True)
        del f32
        return [ctx.i4a8_load(blob, K, n1 - n0) for _ in range(copies)]

    lin = {name: (K, N, packed(K, N, ncopies)) for name, K, N in L70["linears"]}
    Kh, Nv = L70["lm_head"]
    # quantized in 3 channel blocks to bound host memory (same bytes and work); 128256 = 256 * 501, so 3
    # blocks keep every rank's slice a multiple of 32 channels for 1, 2, 4 and 8 ranks
    head_chunks = 3
    head = [(Kh, Nv // head_chunks, packed(Kh, Nv // head_chunks, 1)[0]) for _ in range(head_chunks)]
    # (the LM head's C holds its last chunk's result after a pass)
    shapes = [(name, K, N, ws[0]) for name, (K, N, ws) in lin.items()] + [("lm_head", Kh, Nv // head_chunks, head[-1][2])]
    p2p = world > 1 and args.gather == "p2p"
    peers = shard.PeerGroup(ctx, dist) if p2p else None
    results = {}
    for M in Ms:
        A = {8192: torch.randint(-127, 128, (M, 8192), dtype=torch.int8, device="cuda", generator=gen),
             28672: torch.randint(-127, 128, (M, 28672), dtype=torch.int8, device="cuda", generator=gen)}
        Cfull = {}
        if p2p:
            tab = {}
            for name, K, N, _ in shapes:  # with landing buffers: the tagged-word gather
                tab[name], Cfull[name] = peers.table(M, N, N // world, land=True)
        else:
            Cl = {name: torch.empty((M, N // world), dtype=torch.int32, device="cuda") for name, K, N, _ in shapes}
            Cf = {name: torch.empty((M, N), dtype=torch.int32, device="cuda") for name, K, N, _ in shapes}
            Cfull = {name: (Cf[name] if world > 1 else Cl[name]).data_ptr() for name, K, N, _ in shapes}

        def run(name, w, a):
            if p2p:  # matmul + push of the shard to every rank + bounded wait for every rank's shard
                assert L.ork_b200_i8_mm_run_gather_async(ctx.ctx, w.h, M, a.data_ptr(), tab[name]) == 0
            else:
                assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, a.data_ptr(), Cl[name].data_ptr()) == 0
                if world > 1:
                    shard.gather_columns(Cl[name], dist, out=Cf[name])

        def one_pass():
            for layer in range(L70["layers"]):
                for name, K, N in L70["linears"]:
                    run(name, lin[name][2][layer % ncopies], A[K])
            for K, N, w in head:
                run("lm_head", w, A[K])

        with torch.cuda.stream(stream):
            one_pass()  # eager warm-up: kernel attributes, tensor maps, NCCL communicator
            torch.cuda.synchronize()
            assert L.ork_b200_sync(ctx.ctx) == 0
        # every linear's C after the pass (all copies of a weight are identical): own columns exact,
        # the gathered whole identical on every rank
        sums = []
        for name, K, N, w in shapes:
            full = np.zeros((M, N), np.int32)
            assert L.ork_b200_copy(ctx.ctx, full.ctypes.data, Cfull[name], full.nbytes) == 0
            n0, n1 = shard.shard_range(N, rank, world)
            want = exact_i32(A[K], resident_codes(ctx, w, "nf4")).cpu().numpy()
            if not np.array_equal(full[:, n0:n1], want):
                raise SystemExit(f"70B {name} M={M}: C differs from the exact int32 GEMM of the shard")
            sums.append(int(full.astype(np.int64).sum()) ^ int((full.astype(np.int64) * np.arange(N)).sum()))
        if world > 1:
            every = [None] * world
            dist.all_gather_object(every, sums)
            if any(e != sums for e in every):
                raise SystemExit(f"70B M={M}: gathered C differs between ranks")
        with torch.cuda.stream(stream):
            g = torch.cuda.CUDAGraph()
            l0 = ctx.launches()
            with torch.cuda.graph(g, stream=stream):
                one_pass()
            launches_per_pass = ctx.launches() - l0
            for _ in range(args.warmup):
                g.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with Clocks(local) as clk:
                e0.record(stream)
                for _ in range(args.steps):
                    g.replay()
                e1.record(stream)
                torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        del g
        per_pass = ms / args.steps
        rank_bytes = L70["layers"] * layer_bytes + Kh * Nv // 2 // world
        results[f"M{M}"] = {"tok_s": M / (per_pass / 1e3), "ms_per_pass": per_pass,
                            "per_gpu_weight_GBs": rank_bytes / (per_pass / 1e3) / 1e9,
                            "weight_bytes_per_rank_per_pass": rank_bytes,
                            "gpu_launches": int(launches_per_pass * args.steps), "steps": args.steps,
                            "parity": "exact", "clocks": clk.summary()}
    desc = {"workload": "Llama-70B-shaped linears, NF4 weights ~N(0,0.02), 80 layers x (QKV 8192x10240, "
                        "O 8192x8192, gate+up 8192x57344, down 28672x8192) + LM head 8192x128256, "
                        f"column-sharded over {world} GPU(s), "
                        + ("gather fused into each matmul over NVLink peer memory (each value stored as a "
                           "tagged 8-byte word into every peer's landing buffer, bounded poll and unpack; "
                           "no signal)" if p2p else "NCCL all-gather of each int32 C" if world > 1
                           else "one GPU, no gather"),
            "parallelism": f"column shard x{world}",
            "l2": f"inputs larger than L2: {ncopies} distinct copies of the per-rank layer weights "
                  f"({ncopies * layer_bytes / 2**20:.0f} MiB) cycled over the 80 layers",
            "parity": "before timing, every linear's C: this rank's columns equal an exact int32 GEMM "
                      "(torch._int_mm) of its resident codes; the gathered C's checksum equal on every rank"}
    for _, _, ws in lin.values():
        for w in ws:
            w.free()
    for _, _, w in head:
        w.free()
    if peers is not None:
        peers.close()
    ctx.close()
    return results, desc


def run_70b(args):
    """--workload 70b: configs[4] at M = --tokens alone, as its own JSON line (see sharded_70b)."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    res, desc = sharded_70b(args, [args.tokens], dist if world > 1 else None)
    r = res[f"M{args.tokens}"]
    line = {"metric": "70B-shape NF4 linear stack tok/s (configs[4])", "value": r["tok_s"], "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_pass"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": {**desc, "M": args.tokens},
            **{k: v for k, v in r.items() if k not in ("tok_s", "ms_per_pass")}}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# Qwen3-1.7B shape of BASELINE configs[3]: 28 layers, hidden 2048, 16 query / 8 key-value heads of 128,
# SwiGLU FFN 6144, vocab 151936, RMSNorm (eps 1e-6) incl. per-head q/k norms, RoPE theta 1e6.
Q3 = {"H": 2048, "NH": 16, "NKV": 8, "D": 128, "FF": 6144, "layers": 28, "V": 151936, "theta": 1e6, "eps": 1e-6}


def run_qwen3(args):
    """--workload qwen3: the Qwen3 decode / prefill measurement of qwen3() as its own JSON line."""
    line = qwen3(args)
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)


def qwen3(args):
    """random-init (~N(0,0.02)) Qwen3-1.7B-shaped w8a8 stack; every projection's weight is
    packed per output channel by ork_i8_mm_pack_f32. Decode (the headline): the 28 layers are one
    ork_b200_i8_mm_layers_async call (one persistent launch) -- the library's decode layer: RMSNorm + int8 quantization, q/k/v in one
    batched launch, q/k RMSNorm + RoPE + attention over the fp32 KV cache (the token's k/v appended at the
    device-side position), o, residual + RMSNorm + quantization, gate/up in one launch, SwiGLU +
    quantization, down, residual -- then the final norm + quantization (ork_b200_rmsnorm_q8_async), the LM
    head (ork_b200_i8_mm_run_async) and the greedy pick (ork_b200_argmax_scaled_async); a whole token is one
    CUDA graph. Prefill of the 128-token prompt runs the same layer arithmetic over the rows (the
    library's row glue around ork_b200_i8_mm_run_async; PyTorch's attention), captured as one CUDA graph.
    Four distinct layer weight sets (200 MB, > L2) cycle over the 28 layers. value = decode tokens/s;
    prefill tokens/s beside it."""
    import ctypes as C

    import torch
    import torch.nn.functional as F

    import ork_b200
    from ork_b200 import LayerDims, LayerKV, LayerW

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    L = ork_b200.lib()
    ctx = ork_b200.Context()
    stream = torch.cuda.Stream()
    L.ork_b200_set_stream(ctx.ctx, stream.cuda_stream)
    H, NH, NKV, D, FF, NLY, V = (Q3[k] for k in ("H", "NH", "NKV", "D", "FF", "layers", "V"))
    PRE, DEC = 128, 256
    MAXT = PRE + DEC
    NDIST = 4
    rng = np.random.default_rng(1234 + rank)
    dev = "cuda"

    wgen = torch.Generator(device=dev).manual_seed(1234 + rank)

    def pack(N, K):  # N(0, 0.02) drawn on the device (fast), quantized per channel by ork_i8_mm_pack_f32
        f32 = (torch.randn((N, K), device=dev, generator=wgen) * 0.02).cpu().numpy()
        w, bs = ctx.i8_pack_f32(f32)
        assert w
        return w, torch.from_numpy(bs).to(dev)

    names = ("q", "k", "v", "o", "g", "u", "d")
    wsets = [dict(zip(names, (pack(NH * D, H), pack(NKV * D, H), pack(NKV * D, H), pack(H, NH * D),
                              pack(FF, H), pack(FF, H), pack(H, FF)))) for _ in range(NDIST)]
    lm = pack(V, H)
    g = torch.Generator(device=dev).manual_seed(5)
    emb = (torch.randn((V, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    ones_h = torch.ones(H, device=dev)
    ones_d = torch.ones(D, device=dev)
    kc = [torch.zeros((NKV, MAXT, D), device=dev, dtype=torch.float32) for _ in range(NLY)]
    vc = [torch.zeros((NKV, MAXT, D), device=dev, dtype=torch.float32) for _ in range(NLY)]
    tok = torch.zeros(1, dtype=torch.long, device=dev)
    q8h = torch.empty(H, dtype=torch.int8, device=dev)
    c_lm = torch.empty(V, dtype=torch.int32, device=dev)

    def head(x_row):  # final norm + quantization, the LM head and the greedy pick into tok
        assert L.ork_b200_rmsnorm_q8_async(ctx.ctx, x_row.data_ptr(), ones_h.data_ptr(), H, q8h.data_ptr(), None) == 0
        assert L.ork_b200_i8_mm_run_async(ctx.ctx, lm[0].h, 1, q8h.data_ptr(), c_lm.data_ptr()) == 0
        assert L.ork_b200_argmax_scaled_async(ctx.ctx, c_lm.data_ptr(), lm[1].data_ptr(), V, tok.data_ptr()) == 0

    # prefill buffers: the rows' codes and scales, the matmul results, the dequantized projections
    pq8 = torch.empty((PRE, max(H, NH * D, FF)), dtype=torch.int8, device=dev)
    psc = torch.empty(PRE, dtype=torch.float32, device=dev)
    pC = {n: torch.empty((PRE, N), dtype=torch.int32, device=dev)
          for n, N in (("q", NH * D), ("k", NKV * D), ("v", NKV * D), ("o", H), ("g", FF), ("u", FF), ("d", H))}
    pf = {n: torch.empty((PRE, N), dtype=torch.float32, device=dev) for n, N in (("q", NH * D), ("k", NKV * D),
                                                                                   ("v", NKV * D))}
    px = [torch.empty((PRE, H), dtype=torch.float32, device=dev) for _ in range(2)]
    pqh = torch.empty((NH, PRE, D), dtype=torch.float32, device=dev)

    def mm(w, T, a, c):
        assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, T, a.data_ptr(), c.data_ptr()) == 0

    def prefill_layer(x, li, T):  # x [T, H] fp32, positions 0..T-1; fills the fp32 caches
        # the decode layer's arithmetic over T rows (weights are int8 codes, activations per-row int8):
        # the library's row glue around the library matmuls, PyTorch's attention over the caches
        ws = wsets[li % NDIST]
        x1, xo = px[0][:T], px[1][:T]
        a = pq8[:T]
        assert L.ork_b200_rows_q8_async(ctx.ctx, x.data_ptr(), ones_h.data_ptr(), T, H, 1, a.data_ptr(),
                                        psc.data_ptr()) == 0
        for n in ("q", "k", "v"):
            mm(ws[n][0], T, a, pC[n])
            assert L.ork_b200_rows_dequant_async(ctx.ctx, pC[n].data_ptr(), T, pC[n].shape[1], psc.data_ptr(), None,
                                                 None, pf[n].data_ptr()) == 0
        # q / k norms + RoPE, k and v into the caches at rows 0..T-1, q head-major: one library launch
        assert L.ork_b200_rows_qk_rope_async(ctx.ctx, pf["q"].data_ptr(), pf["k"].data_ptr(), pf["v"].data_ptr(), T,
                                             NH, NKV, D, ones_d.data_ptr(), ones_d.data_ptr(), 0, Q3["theta"],
                                             pqh.data_ptr(), kc[li].data_ptr(), vc[li].data_ptr(), MAXT) == 0
        q = pqh.view(-1)[:NH * T * D].view(NH, T, D)
        o = F.scaled_dot_product_attention(q, kc[li][:, :T], vc[li][:, :T], is_causal=True, enable_gqa=True)
        o = o.transpose(0, 1).reshape(T, NH * D)
        assert L.ork_b200_rows_q8_async(ctx.ctx, o.data_ptr(), None, T, NH * D, 0, a.data_ptr(), psc.data_ptr()) == 0
        mm(ws["o"][0], T, a, pC["o"])
        assert L.ork_b200_rows_dequant_async(ctx.ctx, pC["o"].data_ptr(), T, H, psc.data_ptr(), None, x.data_ptr(),
                                             x1.data_ptr()) == 0  # x1 = x + Co / s
        assert L.ork_b200_rows_q8_async(ctx.ctx, x1.data_ptr(), ones_h.data_ptr(), T, H, 1, a.data_ptr(),
                                        psc.data_ptr()) == 0
        mm(ws["g"][0], T, a, pC["g"])
        mm(ws["u"][0], T, a, pC["u"])
        assert L.ork_b200_rows_swiglu_q8_async(ctx.ctx, pC["g"].data_ptr(), pC["u"].data_ptr(), T, FF,
                                               psc.data_ptr(), a.data_ptr(), psc.data_ptr()) == 0
        mm(ws["d"][0], T, a, pC["d"])
        assert L.ork_b200_rows_dequant_async(ctx.ctx, pC["d"].data_ptr(), T, H, psc.data_ptr(), None, x1.data_ptr(),
                                             xo.data_ptr()) == 0  # x_out = x1 + Cd / s
        return xo

    def prefill(tokens):  # the prompt's rows through the layers, then the first generated token into tok
        x = emb.index_select(0, tokens).float()
        for li in range(NLY):
            x = prefill_layer(x, li, x.shape[0])  # layer outputs alternate between two buffers
        head(x[-1])

    prompt = torch.randint(0, V, (PRE,), device=dev, generator=g)
    pos = torch.zeros(1, dtype=torch.int32, device=dev)
    xa = torch.zeros(H, dtype=torch.float32, device=dev)
    xb = torch.zeros(H, dtype=torch.float32, device=dev)
    dims = LayerDims(H, NH, NKV, D, D, FF, PRE, PRE, 1.0 / float(np.sqrt(D)), Q3["theta"])
    kv = LayerKV(ones_d.data_ptr(), 1, MAXT, pos.data_ptr())

    # the 28 layers as one ork_b200_i8_mm_layers_async call (one persistent launch per token)
    stack = (LayerW * NLY)(*[LayerW(*[wsets[li % NDIST][n][0].h for n in names], ones_h.data_ptr(), ones_d.data_ptr(),
                                    ones_h.data_ptr(), ones_d.data_ptr(), kc[li].data_ptr(), vc[li].data_ptr())
                             for li in range(NLY)])

    def decode_step():
        xa.copy_(emb.index_select(0, tok).float().view(-1))
        assert L.ork_b200_i8_mm_layers_async(ctx.ctx, C.byref(dims), NLY, stack, xa.data_ptr(), xb.data_ptr(),
                                        C.byref(kv)) == 0
        head(xb)  # the final norm + quantization, the LM head and the greedy pick: three library launches
        pos.add_(1)

    with torch.cuda.stream(stream):
        for _ in range(2):  # warm-up prefill (kernel attributes, tensor maps, SDPA selection)
            prefill(prompt)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        prefill(prompt)  # eager: PyTorch's host-side launch rate bounds this one
        e1.record(stream)
        torch.cuda.synchronize()
        prefill_eager_ms = e0.elapsed_time(e1)
        # the prompt as one CUDA graph (glue + library matmuls), replayed: the device time of prefill
        pgraph = torch.cuda.CUDAGraph()
        l0 = ctx.launches()
        with torch.cuda.graph(pgraph, stream=stream):
            prefill(prompt)
        prefill_launches = ctx.launches() - l0
        pgraph.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        pgraph.replay()  # leaves the first generated token in tok
        e1.record(stream)
        torch.cuda.synchronize()
        prefill_ms = e0.elapsed_time(e1)
        del pgraph
        pos.fill_(PRE)
        decode_step()  # eager warm-up of the decode shapes (sizes the layer workspace before capture)
        pos.fill_(PRE)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        l0 = ctx.launches()
        with torch.cuda.graph(graph, stream=stream):
            decode_step()
        launches_per_token = ctx.launches() - l0
        pos.fill_(PRE)
        torch.cuda.synchronize()
        with Clocks(local) as clk:
            e0.record(stream)
            for _ in range(DEC):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
        decode_ms = e0.elapsed_time(e1)
        assert int(pos.item()) == PRE + DEC
    del graph
    weight_bytes = NLY * ((NH + 2 * NKV) * D * H + H * NH * D + 2 * FF * H + H * FF) + V * H
    tps = DEC / (decode_ms / 1e3)
    hbm, _, src = peaks()
    roof_tps = hbm * 1e9 / weight_bytes
    line = {"metric": "Qwen3-1.7B-shape w8a8 decode tok/s (configs[3])", "value": tps * world, "unit": "tok/s",
            "n_gpus": world, "steps": DEC, "warmup": 1, "ms_per_step": decode_ms / DEC, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "Qwen3-1.7B-shaped w8a8 stack, random weights ~N(0,0.02): 28 layers, hidden 2048, "
                                   "16/8 heads x 128, SwiGLU 6144, vocab 151936, q/k norms, RoPE 1e6; prefill 128 "
                                   "then 256 greedy decode steps, batch 1",
                       "linears": "decode: the 28 layers as one ork_b200_i8_mm_layers_async call (the library's decode "
                                  "layer, one persistent launch), final norm + quantization, LM head "
                                  "(ork_b200_i8_mm_run_async) and greedy pick as three library launches; "
                                  "prefill: the same layer arithmetic over 128 rows -- the library's row glue "
                                  "(norm + quantization, dequantization + residual, q/k norms + RoPE + cache "
                                  "writes, SwiGLU + quantization) around ork_b200_i8_mm_run_async, PyTorch's "
                                  "scaled_dot_product_attention -- captured as one CUDA graph (prefill_eager_ms: "
                                  "the same prompt launched eagerly)",
                       "l2": f"{NDIST} distinct layer weight sets cycled (~{NDIST * 50} MB) + 311 MB LM head",
                       "parallelism": "replicas" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": tps * weight_bytes / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": tps / roof_tps, "traffic": None, "kernel": "decode token (weights once)",
                         "peak_source": src},
            "prefill_tok_s": PRE / (prefill_ms / 1e3) * world, "prefill_ms": prefill_ms,
            "prefill_eager_ms": prefill_eager_ms,
            "decode_ms_per_token": decode_ms / DEC, "int8_weight_bytes_per_token": weight_bytes,
            "linear_weight_GBs_decode": weight_bytes / (decode_ms / DEC / 1e3) / 1e9,
            "gpu_launches": int(launches_per_token * DEC), "library_launches_per_token": launches_per_token,
            "library_launches_prefill": prefill_launches, "clocks": clk.summary()}
    for ws in wsets:
        for w, _ in ws.values():
            w.free()
    lm[0].free()
    ctx.close()
    return line


# grouped scales (per-K-group aScale/bScale, fp32 C): the reference's own grouped W4A8 test shapes
# (examples/test_grouped_i8.c:84-87, G = 512 / 1024) plus a G = 128 decode shape, at M = 1 and 8
GROUPED_SHAPES = [(2048, 4096, 512), (2048, 16384, 512), (4096, 20480, 1024), (3072, 12288, 1024), (4096, 4096, 128)]
GROUPED_MS = [1, 8]


def grouped_bytes(K, N, G, M):
    """Algorithmic bytes of one grouped run: int4 weight + bScale + A + aScale + fp32 C."""
    return K * N // 2 + (K // G) * N * 4 + M * K + M * (K // G) * 4 + 4 * M * N


def run_grouped(args):
    """Grouped-scale W4A8 decode: int4 weights written by ork_i4_w_dump_cpu, loaded with
    ork_i4a8_mm_load_tiled(G), run by ork_i8_mm_run_grouped(_async) with int8 activations, fp32 C. One step
    = every (shape, M) once; 3 distinct weight copies (>= 240 MB) cycle so no call finds its weight in L2.
    value = algorithmic GB/s of the step (device-resident inputs, one CUDA graph, events); e2e = the
    synchronous host-buffer call; cpu_baseline = the reference's orki_cpu_gemm_grouped (oracle/_ref) on a
    bounded sample of the same calls."""
    import torch

    import ork_b200

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_ffi as of

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    ctx = ork_b200.Context()
    L = ctx.L
    stream = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))
    NC = 3
    rng = np.random.default_rng(77 + rank)
    calls, host, weights = [], [], []
    for K, N, G in GROUPED_SHAPES:
        B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
        blob = ctx.dump_cpu(B, "i4")
        ws = [ctx.i4a8_load_tiled(blob, K, N, G) for _ in range(NC)]
        assert all(ws)
        weights += ws
        for M in GROUPED_MS:
            A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
            aS = rng.uniform(1e-3, 3e-2, size=(M, K // G)).astype(np.float32)
            bS = rng.uniform(1e-3, 3e-2, size=(K // G, N)).astype(np.float32)
            host.append((K, N, G, M, A, B, aS, bS))
            for ci in range(NC):
                dev = [torch.from_numpy(x).cuda() for x in (A, aS, bS)]
                dC = torch.empty((M, N), dtype=torch.float32, device="cuda")
                calls.append((ci, (K, N, G, M), ws[ci], dev, dC))
    step_bytes = sum(grouped_bytes(K, N, G, M) for K, N, G, M, *_ in host)

    def enqueue(sel):
        for _, _, w, (dA, daS, dbS), dC in sel:
            assert L.ork_b200_i8_mm_run_grouped_async(ctx.ctx, w.h, dA.shape[0], dA.data_ptr(), daS.data_ptr(),
                                                 dbS.data_ptr(), dC.data_ptr()) == 0

    def graph_of(sel):
        enqueue(sel)
        assert L.ork_b200_sync(ctx.ctx) == 0
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            enqueue(sel)
        return g

    def timed(g, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3

    # correctness of the timed calls (first copy) against the restated oracle, before timing
    for ci, key, w, (dA, daS, dbS), dC in calls:
        if ci == 0:
            K, N, G, M = key
            hA, haS, hbS = dA.cpu().numpy(), daS.cpu().numpy(), dbS.cpu().numpy()
            B = next(h[5] for h in host if h[:4] == key)
            enqueue([(ci, key, w, (dA, daS, dbS), dC)])
            assert L.ork_b200_sync(ctx.ctx) == 0
            assert np.array_equal(dC.cpu().numpy().view(np.uint32),
                                  of.gemm_grouped(hA, B, G, haS, hbS).view(np.uint32)), key
    g_all = graph_of(calls)
    for _ in range(max(args.warmup, 3)):
        g_all.replay()
    torch.cuda.synchronize()
    reps = max(1, args.steps // NC)
    with Clocks(local) as clk:
        t = timed(g_all, reps)
    ms_per_step = t / (reps * NC) * 1e3
    value = step_bytes / (ms_per_step / 1e3) / 1e9
    breakdown, dom = {}, None
    for K, N, G, M, *_ in host:
        sel = [c for c in calls if c[1] == (K, N, G, M)]
        g = graph_of(sel)
        for _ in range(3):
            g.replay()
        tt = timed(g, 20) / (20 * NC)
        gbs = grouped_bytes(K, N, G, M) / tt / 1e9
        name = f"{K}x{N}_G{G}_M{M}"
        breakdown[name] = {"us": tt * 1e6, "GB/s": gbs}
        if dom is None or tt > breakdown[dom]["us"] / 1e6:
            dom = name
        del g
    # e2e: the synchronous public call over host buffers, one pass of the step per iteration
    pinned = [(torch.from_numpy(A).pin_memory().numpy(), torch.from_numpy(aS).pin_memory().numpy(),
               torch.from_numpy(bS).pin_memory().numpy(), np.zeros((M, N), np.float32), K, N, G, M)
              for K, N, G, M, A, B, aS, bS in host]
    hw = {key: [c[2] for c in calls if c[1] == key and c[0] == 0][0] for key in {c[1] for c in calls}}
    t0 = time.perf_counter()
    e2e_reps = 5
    for _ in range(e2e_reps):
        for A, aS, bS, Cm, K, N, G, M in pinned:
            assert L.ork_i8_mm_run_grouped(ctx.ctx, hw[(K, N, G, M)].h, M, of._p(A), of._p(aS), of._p(bS),
                                           of._p(Cm)) == 0
    e2e_t = (time.perf_counter() - t0) / e2e_reps
    h2d = sum(A.nbytes + aS.nbytes + bS.nbytes for A, aS, bS, *_ in pinned)
    d2h = sum(Cm.nbytes for _, _, _, Cm, *_ in pinned)
    hbm, _, src = peaks()
    line = {"metric": "grouped-scale W4A8 decode algorithmic HBM GB/s", "value": value * world, "unit": "GB/s",
            "n_gpus": world, "steps": reps * NC, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "grouped W4A8: ork_i4_w_dump_cpu -> ork_i4a8_mm_load_tiled(G) -> "
                                   "ork_i8_mm_run_grouped, fp32 C; (K,N,G) in "
                                   + ", ".join(f"({K},{N},{G})" for K, N, G in GROUPED_SHAPES)
                                   + " (examples/test_grouped_i8.c shapes + G=128), M in {1,8}",
                       "l2": f"{NC} distinct weight copies cycled", "step_bytes": step_bytes,
                       "parallelism": "replicas" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": breakdown[dom]["GB/s"], "peak": hbm, "unit": "GB/s",
                         "frac": breakdown[dom]["GB/s"] / hbm, "traffic": None, "kernel": dom,
                         "peak_source": src},
            "e2e": {"value": step_bytes / e2e_t / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": e2e_t * 1e3},
            "clocks": clk.summary(), "gpu_launches": int(len(calls) * reps),
            "breakdown": breakdown}
    if rank == 0 and not args.no_cpu:
        of.restated().orc_set_threads(host_cores())
        ref = of.reference()
        fn = ref.orki_cpu_gemm_grouped if ref is not None else of.restated().orc_gemm_grouped
        sample = [h for h in host if h[3] == 1]
        t0, n = time.perf_counter(), 0
        while n == 0 or (time.perf_counter() - t0 < 10 and n < 3):
            for K, N, G, M, A, B, aS, bS in sample:
                Cm = np.zeros((M, N), np.float32)
                assert fn(M, K, N, G, of._p(A), of._p(B), of._p(aS), of._p(bS), of._p(Cm)) == 0
            n += 1
        tc = (time.perf_counter() - t0) / n
        line["cpu_baseline"] = {"value": sum(grouped_bytes(K, N, G, M) for K, N, G, M, *_ in sample) / tc / 1e9,
                                "unit": "GB/s", "cores": of.restated().orc_threads(),
                                "kind": "reference" if ref is not None else "port",
                                "sample": f"{n} pass(es) of the M=1 calls of the step ({tc * n:.2f} s)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del g_all
    for w in weights:
        w.free()
    ctx.close()


def run_moe(args):
    """Batches of independent matmuls (ork_b200_i8_mm_run_chain_async): an MoE decode layer of 64 experts, each a
    2048 x 1408 w4a8 NF4 weight (ork_i4a8_mm_pack with ORK_NF4) seeing 1-4 tokens, as one batch; 4 distinct
    expert sets (>= 180 MB of nibbles) cycle so no batch finds its weights in L2. value = algorithmic GB/s of
    the batch (device-resident inputs, one CUDA graph per step, events); breakdown: the same 64 matmuls
    issued as 64 separate ork_b200_i8_mm_run_async launches; e2e: the synchronous ork_i8_mm_run_chain over host
    buffers; cpu_baseline: the reference's own chain semantics (orki_cpu_gemm_i32 per task, oracle/_ref)."""
    import torch

    import ork_b200
    from ork_b200 import TaskI8

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_ffi as of

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    ctx = ork_b200.Context()
    L = ctx.L
    stream = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))
    E, K, N, NSET = 64, 2048, 1408, 4
    rng = np.random.default_rng(99 + rank)
    os.environ["ORK_NF4"] = "1"
    sets, host = [], []
    for si in range(NSET):
        ws, tasks, keep = [], [], []
        for e in range(E):
            f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            w, _ = ctx.i4a8_pack(f32)
            M = 1 + (e * 7 + si) % 4
            A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
            Cd = torch.empty((M, N), dtype=torch.int32, device="cuda")
            ws.append(w)
            keep += [A, Cd]
            tasks.append(TaskI8(w.h, M, A.data_ptr(), Cd.data_ptr(), 0))
            if si == 0:
                codes, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
                host.append((w, M, A.cpu().numpy(), codes, Cd))
        sets.append((ws, (TaskI8 * E)(*tasks), keep))
    os.environ.pop("ORK_NF4", None)
    step_bytes = sum(K * N // 2 + t.M * K + 4 * t.M * N for t in sets[0][1])

    # correctness of the batched launch against the oracle, before timing
    assert L.ork_b200_i8_mm_run_chain_async(ctx.ctx, E, sets[0][1]) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    for w, M, A, codes, Cd in host:
        assert np.array_equal(Cd.cpu().numpy(), of.gemm_i32(A, codes))

    def graph(fn):
        fn()
        assert L.ork_b200_sync(ctx.ctx) == 0
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        return g

    def batched():
        for ws, arr, _ in sets:
            assert L.ork_b200_i8_mm_run_chain_async(ctx.ctx, E, arr) == 0

    def separate():
        for ws, arr, _ in sets:
            for t in arr:
                assert L.ork_b200_i8_mm_run_async(ctx.ctx, t.w, t.M, t.A, t.C) == 0

    def timed(g, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / (reps * NSET)

    gb, gs = graph(batched), graph(separate)
    reps = max(1, args.steps // NSET)
    with Clocks(local) as clk:
        t_b = timed(gb, reps)
    t_s = timed(gs, reps)
    # e2e: the synchronous public call with host buffers (staged A in, C out, one launch for the batch)
    hA = [np.ascontiguousarray(A) for _, _, A, _, _ in host]
    hC = [np.zeros((M, N), np.int32) for _, M, _, _, _ in host]
    harr = (TaskI8 * E)(*[TaskI8(w.h, M, a.ctypes.data, c.ctypes.data, 0)
                          for (w, M, _, _, _), a, c in zip(host, hA, hC)])
    t0 = time.perf_counter()
    for _ in range(10):
        assert L.ork_i8_mm_run_chain(ctx.ctx, E, harr) == 0
    t_e2e = (time.perf_counter() - t0) / 10
    hbm, _, src = peaks()
    line = {"metric": "MoE batch (64 experts, w4a8 NF4 decode) algorithmic HBM GB/s", "value": step_bytes / t_b / 1e9 * world,
            "unit": "GB/s", "n_gpus": world, "steps": reps * NSET, "warmup": 3, "ms_per_step": t_b * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"ork_i8_mm_run_chain(_async): {E} experts of K={K}, N={N} NF4 (ork_i4a8_mm_pack), "
                                   "1-4 tokens each", "l2": f"{NSET} distinct expert sets cycled",
                       "step_bytes": step_bytes, "parallelism": "replicas" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": step_bytes / t_b / 1e9, "peak": hbm, "unit": "GB/s",
                         "frac": step_bytes / t_b / 1e9 / hbm, "traffic": None, "kernel": "gemv_batched_kernel",
                         "peak_source": src},
            "e2e": {"value": step_bytes / t_e2e / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": int(sum(a.nbytes for a in hA)),
                    "d2h_bytes_per_step": int(sum(c.nbytes for c in hC)), "ms_per_step": t_e2e * 1e3},
            "breakdown": {"batched_one_launch_us": t_b * 1e6, "separate_64_launches_us": t_s * 1e6,
                          "separate_GBs": step_bytes / t_s / 1e9},
            "clocks": clk.summary(), "gpu_launches": int(reps * NSET)}
    if rank == 0 and not args.no_cpu:
        of.restated().orc_set_threads(host_cores())
        ref = of.reference()
        fn = ref.ork_i8_mm_run_cpu if ref is not None else of.restated().orc_gemm_i32
        Cm = [np.zeros((M, N), np.int32) for _, M, _, _, _ in host]
        t0 = time.perf_counter()
        for (w, M, A, codes, _), c in zip(host, Cm):
            fn(M, K, N, of._p(A), of._p(np.ascontiguousarray(codes)), of._p(c))
        tc = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": step_bytes / tc / 1e9, "unit": "GB/s", "cores": of.restated().orc_threads(),
                                "kind": "reference" if ref is not None else "port",
                                "sample": f"one batch of {E} expert matmuls on inflated int8 codes ({tc:.2f} s)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    del gb, gs
    for ws, _, _ in sets:
        for w in ws:
            w.free()
    ctx.close()


def run_profile(spec):
    """`K,N,M[,route]`: one config, packed once, run 5 times with a synchronisation after each -- a small,
    self-contained workload for `ncu -k <kernel> -s <skip> -c <count>` captures -- then 50 back-to-back
    calls timed with events (a tuning aid). `all`: the 12 configs[1] calls once each, in sweep order,
    synchronised (one launch per config, for per-config ncu metrics such as DRAM traffic)."""
    import torch

    import ork_b200

    L = ork_b200.lib()
    ctx = ork_b200.Context()
    rng = np.random.default_rng(0)
    if spec == "all":
        for K, N in SHAPES:
            f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
            w, _ = ctx.i8_pack_f32(f32)
            for M in MS:
                a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
                c = torch.empty((M, N), dtype=torch.int32, device="cuda")
                torch.cuda.synchronize()
                assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, a.data_ptr(), c.data_ptr()) == 0
                assert L.ork_b200_sync(ctx.ctx) == 0
            w.free()
        print(json.dumps({"profile": "all", "configs": [f"{K}x{N}xM{M}" for K, N, M in CONFIGS]}))
        ctx.close()
        return
    fields = spec.split(",")
    fmt = fields[4] if len(fields) > 4 else "i8"  # i8 | u4 | nf4 (int4 stores of ork_i4a8_mm_pack)
    parts = [int(x) for x in fields[:4]]
    K, N, M = parts[:3]
    route = parts[3] if len(parts) > 3 else -1
    L.ork_b200_force_route(ctx.ctx, route)
    f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if fmt == "i8":
        w, _ = ctx.i8_pack_f32(f32)
    else:
        if fmt == "nf4":
            os.environ["ORK_NF4"] = "1"
        w, _ = ctx.i4a8_pack(f32)
        os.environ.pop("ORK_NF4", None)
    a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
    c = torch.empty((M, N), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    for _ in range(5):
        assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, a.data_ptr(), c.data_ptr()) == 0
        assert L.ork_b200_sync(ctx.ctx) == 0
    # back-to-back timing of the same call (weight L2-warm after the first): a tuning aid only
    stream = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(50):
        assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, a.data_ptr(), c.data_ptr()) == 0
    e1.record(stream)
    assert L.ork_b200_sync(ctx.ctx) == 0
    us = e0.elapsed_time(e1) * 1e3 / 50
    print(json.dumps({"profile": spec, "route": L.ork_b200_route(w.h, M), "launches": ctx.launches(),
                      "us_per_call_warm": us, "env": {k: v for k, v in os.environ.items() if k.startswith("ORKB_")}}))
    w.free()
    ctx.close()


def run_tc_peak(args):
    """The tensor pipe's ceiling: the library's tcgen05 GEMM (ork_b200_i8_mm_run_async, ork_b200_f16_mm_run_async) at
    M = K = N = 8192, where the work is compute-bound (1.1 T ops against ~0.4 GB), timed beside the GPU's
    measured dense peak on the same shapes (torch._int_mm and torch.mm, i.e. cuBLASLt). Not a BASELINE
    config: it measures the denominator the prefill fractions need and how close the kernel comes to it.
    The int8 result is checked equal to torch._int_mm's (exact int32)."""
    import torch

    import ork_b200

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    L = ork_b200.lib()
    ctx = ork_b200.Context()
    stream = torch.cuda.Stream()
    L.ork_b200_set_stream(ctx.ctx, stream.cuda_stream)
    S = 8192
    ops = 2.0 * S * S * S
    g = torch.Generator(device="cuda").manual_seed(7)

    def timed(fn, reps=10):
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    out = {}
    with Clocks(local) as clk:
        A8 = torch.randint(-127, 128, (S, S), dtype=torch.int8, device="cuda", generator=g)
        B8 = torch.randint(-127, 128, (S, S), dtype=torch.int8, device="cuda", generator=g)
        w8 = ctx.i8_pack(B8.cpu().numpy())
        C32 = torch.empty((S, S), dtype=torch.int32, device="cuda")
        ms = timed(lambda: L.ork_b200_i8_mm_run_async(ctx.ctx, w8.h, S, A8.data_ptr(), C32.data_ptr()))
        out["int8_ours_tops"] = ops / (ms * 1e-3) / 1e12
        try:
            ms_lib = timed(lambda: torch._int_mm(A8, B8))
            out["int8_torch_int_mm_tops"] = ops / (ms_lib * 1e-3) / 1e12
            with torch.cuda.stream(stream):
                same = bool(torch.equal(C32, torch._int_mm(A8, B8)))
            torch.cuda.synchronize()
            out["int8_equal_to_torch"] = same
        except RuntimeError as e:
            out["int8_torch_int_mm"] = f"unavailable: {str(e).splitlines()[0][:120]}"
        w8.free()
        del A8, B8, C32
        A16 = (torch.randn((S, S), device="cuda", generator=g) * 0.5).to(torch.float16)
        B16 = (torch.randn((S, S), device="cuda", generator=g) * 0.02).to(torch.float16)
        w16 = ctx.f16_pack(B16.cpu().numpy())
        C = torch.empty((S, S), dtype=torch.float32, device="cuda")
        ms = timed(lambda: L.ork_b200_f16_mm_run_async(ctx.ctx, w16.h, S, A16.data_ptr(), C.data_ptr()))
        out["f16_ours_tflops"] = ops / (ms * 1e-3) / 1e12
        ms_lib = timed(lambda: torch.mm(A16, B16))
        out["f16_torch_mm_tflops"] = ops / (ms_lib * 1e-3) / 1e12
        w16.free()
    line = {"metric": "tcgen05 GEMM throughput at 8192^3 (ours vs the cuBLASLt peak on this GPU)",
            "value": out["int8_ours_tops"], "unit": "TOPS", "n_gpus": 1, "steps": 10, "warmup": 3,
            "higher_is_better": True, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "M = K = N = 8192, int8 (A, B ~ U[-127, 127]) and fp16; C int32 / fp32"},
            **{k: (round(v, 1) if isinstance(v, float) else v) for k, v in out.items()},
            "clocks": clk.summary()}
    if "int8_torch_int_mm_tops" in out:
        line["int8_frac_of_measured_peak"] = out["int8_ours_tops"] / out["int8_torch_int_mm_tops"]
    line["f16_frac_of_measured_peak"] = out["f16_ours_tflops"] / out["f16_torch_mm_tflops"]
    print(json.dumps(line), flush=True)
    ctx.close()


def run_pack(args):
    """Pack-time quantization, timed on the host beside the reference's own CPU code (the measurement
    plan times the pack-time quantizers apart from the runs). BASELINE configs[2] inputs: B f32[N][K] ~
    N(0, 0.02), imatrix ~ U(0.5, 2), (K, N) in {(6144, 2048), (2048, 12288)}; uniform and NF4, with and
    without an imatrix. Ours: ork_i4a8_pack_cpu_blob, the library's host-only O4N1 writer -- the same
    quantizer ork_i4a8_mm_pack(_im) runs before its upload. Reference: ork-driver's
    ork_i4a8_pack_cpu_blob_qerr (src/npu/i4/pack.c:787-795, byte-identical to its pack_im + w_dump)
    from oracle/_ref, compiled from its sources. Every blob is compared byte for byte. No GPU needed."""
    import ork_b200

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_ffi as of

    L = ork_b200.lib()
    R = of.reference()
    reps = max(1, min(args.steps, 3))
    rng = np.random.default_rng(2)
    table, t_ours, t_ref, weights, identical = {}, 0.0, 0.0, 0, True

    def best(fn):
        fn()  # warm-up (page faults of the output buffer)
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return min(ts)

    for K, N in ((6144, 2048), (2048, 12288)):
        f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        im = (rng.random(K, dtype=np.float32) * np.float32(1.5) + np.float32(0.5)).astype(np.float32)
        for nf4 in (False, True):
            for imx in (None, im):
                imp = None if imx is None else imx.ctypes.data
                need = L.ork_i4a8_pack_cpu_blob(None, K, N, f32.ctypes.data, imp, int(nf4), None, 0)
                ours = np.zeros(need, np.uint8)
                to = best(lambda: L.ork_i4a8_pack_cpu_blob(None, K, N, f32.ctypes.data, imp, int(nf4),
                                                           ours.ctypes.data, need))
                row = {"ours_ms": to * 1e3}
                if R is not None:
                    ref = np.zeros(need, np.uint8)
                    tr = best(lambda: R.ork_i4a8_pack_cpu_blob_qerr(None, K, N, f32.ctypes.data, imp, int(nf4),
                                                                    ref.ctypes.data, need, None))
                    same = bool(np.array_equal(ours, ref))
                    identical &= same
                    row.update({"reference_ms": tr * 1e3, "speedup": tr / to, "identical": same})
                    t_ref += tr
                name = f"{'nf4' if nf4 else 'uniform'}{'+imatrix' if imx is not None else ''} {K}x{N}"
                table[name] = row
                t_ours += to
                weights += K * N
    out = {"metric": "w4a8 pack-time quantization (ork_i4a8_mm_pack(_im) host quantizer), configs[2] inputs",
           "value": weights / t_ours / 1e6, "unit": "Mweights/s", "n_gpus": 0, "steps": reps, "warmup": 1,
           "ms_per_step": t_ours * 1e3, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "pack: 2 shapes x {uniform, NF4} x {no imatrix, imatrix}; best of steps",
                      "threads": os.cpu_count()},
           "table": table}
    if R is not None:
        out["cpu_baseline"] = {"value": weights / t_ref / 1e6, "unit": "Mweights/s", "cores": os.cpu_count(),
                               "kind": "reference", "cpu": cpu_model(),
                               "sample": "the same 8 packs, best of steps, by ork-driver's own pack code"}
        out["bytes_identical"] = identical
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-others", action="store_true", help="skip the other BASELINE configs' table")
    ap.add_argument("--ncu-step", action="store_true",
                    help="after warm-up, replay one cycle of step graphs between cudaProfilerStart/Stop and exit "
                         "(for `ncu --profile-from-start off` launch lists of exactly the timed work)")
    ap.add_argument("--workload", default="w8a8", choices=["w8a8", "70b", "qwen3", "grouped", "moe", "tc_peak", "pack"],
                    help="w8a8: BASELINE configs[1] sweep (default); 70b: configs[4] column-sharded NF4 stack; "
                         "qwen3: configs[3] Qwen3-1.7B-shape w8a8 stack; grouped: grouped-scale W4A8 decode; "
                         "moe: a batch of 64 NF4 expert matmuls through ork_i8_mm_run_chain; tc_peak: the GEMM "
                         "at 8192^3 beside torch._int_mm / torch.mm; pack: the pack-time quantizers on the host beside "
                         "the reference's (no GPU)")
    ap.add_argument("--tokens", type=int, default=1, help="70b workload: tokens per pass M (1, 8 or 256)")
    ap.add_argument("--gather", default="p2p", choices=["p2p", "nccl"],
                    help="70b workload at N > 1: the C gather fused into the matmul over peer memory, or NCCL")
    ap.add_argument("--profile", default=None,
                    help="K,N,M[,route[,fmt]]: run one config a few times eagerly (for ncu captures); fmt i8|u4|nf4")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args.profile)
    if args.workload == "70b":
        return run_70b(args)
    if args.workload == "qwen3":
        return run_qwen3(args)
    if args.workload == "grouped":
        return run_grouped(args)
    if args.workload == "moe":
        return run_moe(args)
    if args.workload == "tc_peak":
        return run_tc_peak(args)
    if args.workload == "pack":
        return run_pack(args)

    import torch

    import ork_b200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    L = ork_b200.lib()
    ctx = ork_b200.Context()
    stream = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))

    # ---- weights: NCOPIES distinct packs of each shape (inputs larger than L2) ----------------
    rng = np.random.default_rng(1234 + rank)
    weights = {}
    for K, N in SHAPES:
        f32 = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        weights[(K, N)] = []
        for _ in range(NCOPIES):
            w, _ = ctx.i8_pack_f32(f32)
            assert w, "pack failed"
            weights[(K, N)].append(w)
    g = torch.Generator(device="cuda").manual_seed(7 + rank)
    bufs = {}
    for K, N, M in CONFIGS:
        bufs[(K, N, M)] = [(torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda", generator=g),
                            torch.empty((M, N), dtype=torch.int32, device="cuda")) for _ in range(NCOPIES)]
    torch.cuda.synchronize()

    def call(K, N, M, i):
        w = weights[(K, N)][i % NCOPIES]
        a, c = bufs[(K, N, M)][i % NCOPIES]
        rc = L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, a.data_ptr(), c.data_ptr())
        assert rc == 0

    # Step s issues the 12 calls; call i of a shape (i = 0..3 over the M values) uses packed copy
    # (4*s + i) % NCOPIES of that shape, so a copy is reused only after NCOPIES calls of its shape
    # (~270 MB of other weights in between). The copy pattern repeats every NCOPIES steps, so one CUDA
    # graph per residue class replays a step without per-call host overhead.
    def step_calls(s):
        for K, N in SHAPES:
            for i, M in enumerate(MS):
                call(K, N, M, 4 * s + i)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for s in range(NCOPIES):  # eager warm-up of every call (kernel attributes, tensor maps)
        step_calls(s)
    torch.cuda.synchronize()
    codes = {(K, N): resident_codes(ctx, weights[(K, N)][0], "i8") for K, N in SHAPES}

    def check_sweep(when):
        """Every config's C (all NCOPIES buffers, each last written by a call with identical weights)
        equal to an exact int32 GEMM of its A and the packed codes; a mismatch ends the run."""
        assert L.ork_b200_sync(ctx.ctx) == 0
        out = {}
        for K, N, M in CONFIGS:
            ok = all(torch.equal(c, exact_i32(a, codes[(K, N)])) for a, c in bufs[(K, N, M)])
            out[f"{K}x{N}xM{M}"] = "exact" if ok else "MISMATCH"
            if not ok:
                print(json.dumps({"error": f"{K}x{N}xM{M}: C differs from the exact int32 GEMM {when}"}),
                      flush=True)
                raise SystemExit(3)
        return out

    parity = check_sweep("before timing")
    graphs = []
    launches_per_step = []
    for s in range(NCOPIES):
        g = torch.cuda.CUDAGraph()
        l0 = ctx.launches()
        with torch.cuda.graph(g, stream=stream):
            step_calls(s)
        launches_per_step.append(ctx.launches() - l0)
        graphs.append(g)
    torch.cuda.synchronize()

    for s in range(args.warmup):
        graphs[s % NCOPIES].replay()
    barrier()
    if args.ncu_step:
        torch.cuda.cudart().cudaProfilerStart()
        for s in range(NCOPIES):
            graphs[s].replay()
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps({"ncu_step": NCOPIES, "launches_per_step": launches_per_step}), flush=True)
        return
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for s in range(args.steps):
                graphs[(args.warmup + s) % NCOPIES].replay()
            ev1.record(stream)
        barrier()
    launches = sum(launches_per_step[(args.warmup + s) % NCOPIES] for s in range(args.steps))
    ms = ev0.elapsed_time(ev1)
    check_sweep("after the timed graph replays")
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * STEP_BYTES * args.steps / (ms / 1e3) / 1e9

    # ---- per-config breakdown and the dominant kernel: each config alone, NCOPIES calls per graph ----
    breakdown = {}
    reps = 20
    def time_config(K, N, M):
        g = torch.cuda.CUDAGraph()
        l0 = ctx.launches()
        with torch.cuda.graph(g, stream=stream):
            for i in range(NCOPIES):
                call(K, N, M, i)
        nl = (ctx.launches() - l0) / NCOPIES
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        del g
        return e0.elapsed_time(e1) / (reps * NCOPIES), nl

    for K, N, M in CONFIGS:
        per, nl = time_config(K, N, M)
        entry = {"ms": per, "GB/s": alg_bytes(K, N, M) / (per / 1e3) / 1e9,
                 "TOPS": 2 * M * K * N / (per / 1e3) / 1e12, "launches": nl,
                 "route": L.ork_b200_route(weights[(K, N)][0].h, M)}
        for route, name in ((0, "ms_gemv"), (1, "ms_tc")):  # both kernel paths, for the router threshold
            L.ork_b200_force_route(ctx.ctx, route)
            entry[name] = time_config(K, N, M)[0]
        L.ork_b200_force_route(ctx.ctx, -1)
        breakdown[f"{K}x{N}xM{M}"] = entry
    tot = sum(b["ms"] for b in breakdown.values())
    dom = max(breakdown, key=lambda k: breakdown[k]["ms"])
    K, N, M = (int(x) for x in dom.replace("M", "").split("x"))
    hbm, bf16, src = peaks()
    int8_peak = 2.0 * bf16  # dense int8 = 2x the measured dense bf16 burst (no int8 figure measured here)
    db = breakdown[dom]
    nl = max(db["launches"], 1)
    per_launch_s = db["ms"] / nl / 1e3
    bytes_l, ops_l = alg_bytes(K, N, M) / nl, 2.0 * M * K * N / nl
    t_hbm, t_tc = bytes_l / (hbm * 1e9), ops_l / (int8_peak * 1e12)
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            traffic = json.load(f).get(dom)
    except Exception:
        pass
    roofs = {"hbm": {"achieved": bytes_l / per_launch_s / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": t_hbm / per_launch_s, "peak_source": f"{src} (copy)"},
             "tensor": {"achieved": ops_l / per_launch_s / 1e12, "peak": int8_peak, "unit": "TOPS",
                        "frac": t_tc / per_launch_s,
                        "peak_source": f"2 x {src} dense bf16 burst ({bf16:.0f} TFLOP/s): int8 dense"}}
    bound = "tensor" if t_tc > t_hbm else "hbm"
    roofline = {"bound": bound, **{k: roofs[bound][k] for k in ("achieved", "peak", "unit", "frac")},
                "traffic": traffic, "kernel": dom, "share": db["ms"] / tot, "peak_source": roofs[bound]["peak_source"],
                "algorithmic_bytes_per_launch": bytes_l, "algorithmic_ops_per_launch": ops_l,
                "us_per_launch": per_launch_s * 1e6, "roofs": roofs,
                "bound_rule": "the larger of algorithmic bytes / HBM peak and ops / int8 tensor peak"}
    del graphs

    # ---- e2e through the synchronous public call with pinned host buffers ---------------------
    host = {}
    for K, N, M in CONFIGS:
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8).pin_memory()
        c = torch.empty((M, N), dtype=torch.int32).pin_memory()
        host[(K, N, M)] = (a, c)
    h2d = sum(M * K for K, N, M in CONFIGS)
    d2h = sum(4 * M * N for K, N, M in CONFIGS)

    def e2e_step(s):
        for r, (K, N, M) in enumerate(CONFIGS):
            a, c = host[(K, N, M)]
            w = weights[(K, N)][(s * len(CONFIGS) + r) % NCOPIES]
            assert L.ork_i8_mm_run(ctx.ctx, w.h, M, a.data_ptr(), c.data_ptr()) == 0

    for s in range(args.warmup):
        e2e_step(s)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        e2e_step(s)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if dist is not None:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": world * STEP_BYTES * args.steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms / args.steps}
    for K, N, M in CONFIGS:  # the last e2e step's host results
        a, c = host[(K, N, M)]
        if not torch.equal(c.cuda(), exact_i32(a.cuda(), codes[(K, N)])):
            print(json.dumps({"error": f"{K}x{N}xM{M}: e2e C differs from the exact int32 GEMM"}), flush=True)
            raise SystemExit(3)
    for ws in weights.values():
        for w in ws:
            w.free()
    del bufs, codes

    # configs[4] column-sharded over the job's ranks, at every N (one GPU included): decode-sized passes
    s70, d70 = sharded_70b(args, [1, 8], dist)
    sharded = {"workload": d70["workload"], "parallelism": d70["parallelism"], "l2": d70["l2"],
               "parity": d70["parity"], "scaling": "strong (the same 70B-shape stack at every N)",
               **{m: {k: v for k, v in r.items() if k != "steps"} for m, r in s70.items()}}

    others = other_configs(ctx, L, stream) if (rank == 0 and not args.no_others) else None

    q3 = None
    if rank == 0 and world == 1 and not args.no_others:
        q = qwen3(args)
        q3 = {"decode_tok_s": q["value"], "prefill_tok_s": q["prefill_tok_s"], "decode_ms_per_token": q["ms_per_step"],
              "prefill_ms": q["prefill_ms"], "roofline": q["roofline"], "config": q["config"]["workload"],
              "gpu_launches_per_token": q["library_launches_per_token"], "clocks": q["clocks"]}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, cores, kind, sample, _ = cpu_reference_sweep(10.0)
        cpu = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": kind, "cpu": cpu_model(), "sample": sample}

    dec = [k for k in breakdown if k.endswith("M1") or k.endswith("M8")]
    pre = [k for k in breakdown if k not in dec]
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": WORKLOAD,
                       "l2": f"inputs larger than L2: {NCOPIES} distinct packed copies per weight "
                             f"({NCOPIES * sum(K * N for K, N in SHAPES) / 1e6:.0f} MB) plus per-copy A/C, cycled",
                       "parallelism": "replicas" if world > 1 else "single GPU",
                       "step_bytes": STEP_BYTES, "step_ops": STEP_OPS},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk.summary(),
            "gpu_launches": int(launches),
            "parity": parity,
            "parity_check": "every config's C, before and after the timed replays and after the e2e steps, equal "
                            "to an exact int32 GEMM (torch._int_mm) of the same A and the packed codes",
            "decode_gbs": sum(alg_bytes(*map(int, k.replace("M", "").split("x"))) for k in dec)
            / (sum(breakdown[k]["ms"] for k in dec) / 1e3) / 1e9,
            "prefill_tops": sum(2 * np.prod([int(x) for x in k.replace("M", "").split("x")]) for k in pre)
            / (sum(breakdown[k]["ms"] for k in pre) / 1e3) / 1e12,
            "sharded_70b": sharded, "qwen3": q3,
            "qwen3_decode_tok_s": q3["decode_tok_s"] if q3 else None,
            "qwen3_prefill_tok_s": q3["prefill_tok_s"] if q3 else None,
            "breakdown": breakdown, "other_configs": others}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

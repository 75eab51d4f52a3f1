"""Benchmark of the B200 contraction hot path (one JSON line on rank 0).

Headline workload: dense permutedims of a rank-6 16^6 tensor (16,777,216
elements) in f64 with perm (5,3,1,0,4,2), entries N(0,1) from a seed.  A
step permutes one batch of `--batch` such tensors (distinct buffers, so every
input comes from HBM: each tensor is 134 MB and the batch is ~4.3 GB, far
larger than the 126 MB L2).  Metric unit: GB/s of algorithmic traffic,
2 * 16^6 * 8 bytes per tensor.  With --gpus N the permute runs as N
independent replicas (one process per GPU, no collective on the data path);
`value` is the sum over ranks.

Also reported on the same line (`contraction`), each with its roofline: the
batched and complex128 permutes of the same 16^6 shape, the dense f64 MPS
two-site merge A[256,4,256] x B[256,4,256] -> C[256,4,4,256], a 4096^3 GEMM,
the DMRG environment chain at bond 1024 (per step), and the block-sparse
U(1) rank-4 (half scale) and c128 two-site MPS contractions (sharded across
ranks with --gpus N > 1, plus the gathered output on every rank).  At one GPU each contraction
also carries a CPU baseline: the reference's TTGT / per-pair algorithm with
MKL (through torch) standing in for faer's GEMM, at one thread and at all
host threads.

--impl reference times the reference's CPU algorithm for the same workload
on the host cores (the C restatement of GenericBackend::permute_into,
backend/generic.rs:15-39, spread over all host threads).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "ndtensors-rs_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "f64 contraction TFLOP/s and permutedims GB/s at 1/2/4/8 B200 vs host CPU"
SHAPE = (16,) * 6
PERM = (5, 3, 1, 0, 4, 2)
NELEM = 16**6
BYTES_F64 = 2 * NELEM * 8  # algorithmic bytes per tensor (read + write)
_FP64_PEAK = {}


def fp64_peak(stream=None):
    """FP64 tensor-core peak (TFLOP/s) measured live on this GPU by a
    register-only mma.sync f64 microbenchmark (csrc/fp64_peak.cu)."""
    if "v" not in _FP64_PEAK:
        lib = ctypes.CDLL(str(ROOT / "ndtensors-rs_b200" / "lib" / "libndt_fp64_peak.so"))
        lib.ndt_fp64_tensor_peak_tflops.restype = ctypes.c_double
        lib.ndt_fp64_tensor_peak_tflops.argtypes = [ctypes.c_void_p]
        v = lib.ndt_fp64_tensor_peak_tflops(ctypes.c_void_p(stream.cuda_stream if stream is not None else 0))
        if v <= 0:
            raise RuntimeError("FP64 peak microbenchmark failed")
        _FP64_PEAK["v"] = v
    return _FP64_PEAK["v"]


def fp64_roofline(tflops_per_gpu, complex_3m=False):
    """FP64 tensor-core roofline of a contraction rate counted as 2mnk (f64)
    or 8mnk (complex).  Complex GEMM tiles run the 3M form (three real
    products per complex multiply-add), so they execute 6mnk real flop: the
    executed rate is 3/4 of the counted one and is reported beside it."""
    p = fp64_peak()
    r = {"bound": "fp64_tensor", "achieved": tflops_per_gpu, "peak": p, "unit": "TFLOP/s per GPU",
         "frac": tflops_per_gpu / p,
         "peak_source": "live mma.sync f64 register-only microbenchmark (csrc/fp64_peak.cu), measured"}
    if complex_3m:
        r["executed_achieved"] = 0.75 * tflops_per_gpu
        r["executed_frac"] = 0.75 * tflops_per_gpu / p
        r["executed_note"] = "3M complex: 6mnk real flop executed per 8mnk counted"
    return r


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ helpers
def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def ncu_traffic(key):
    """Per-launch DRAM bytes (read + write) recorded from an ncu capture."""
    p = ROOT / "profiles" / "ncu_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == key:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML during the timed
    region (the same data nvidia-smi's clocks query reports)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report nothing rather than guess
            log("clock sampling unavailable:", e)
        self._stop = threading.Event()

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def result(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------ CPU baseline
def cpu_permute_time(threads, sample_tensors=1, seed=2002):
    """Times the oracle's restatement of GenericBackend::permute_into over
    the full 16^6 f64 tensor, `threads` host threads splitting the source
    index range (ctypes releases the GIL)."""
    import numpy as np

    from oracle import oracle as o

    L = o.lib()
    rng = np.random.default_rng(seed)
    a = np.ascontiguousarray(rng.standard_normal(NELEM))
    dst = np.zeros(NELEM)
    shape = o._sz(SHAPE)
    perm = o._sz(PERM)
    chunks = [(NELEM * i // threads, NELEM * (i + 1) // threads) for i in range(threads)]

    def work(lo, hi):
        L.ndo_permutedims_range(0, a.ctypes.data_as(ctypes.c_void_p), shape, ctypes.c_size_t(6), perm,
                                dst.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(lo), ctypes.c_size_t(hi))

    t0 = time.perf_counter()
    for _ in range(sample_tensors):
        ts = [threading.Thread(target=work, args=c) for c in chunks]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    dt = time.perf_counter() - t0
    return dt / sample_tensors


def _blocks_as_mats(sizes, coords, data, split):
    """Each stored block of a packed column-major block-sparse tensor as a
    matrix (first `split` axes = rows), keyed by block coordinates."""
    import numpy as np

    out, off = {}, 0
    for c in coords:
        shp = [sizes[ax][b] for ax, b in enumerate(c)]
        n = int(np.prod(shp))
        r = int(np.prod(shp[:split]))
        out[tuple(c)] = data[off:off + n].reshape((r, n // r), order="F")
        off += n
    return out


def cpu_contraction_baselines():
    """CPU times of the contraction workloads the way the reference computes
    them: TTGT with faer's GEMM at Par::Seq (contract/gemm.rs:158, :215) and
    the per-pair loop of contract_blocksparse (contract/blocksparse.rs:144-180).
    faer is not available; MKL through torch stands in for its GEMM, at one
    thread (the reference's setting) and at all host threads.  Each sample is
    bounded to a few seconds of CPU work.  Returns {workload key: baseline}."""
    import numpy as np
    import torch

    sys.path.insert(0, str(ROOT / "tests"))
    import workloads as W

    ncores = os.cpu_count() or 1
    out = {}

    def rate(fn, flop, reps):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return flop / statistics.median(ts) / 1e12

    def both(key, fn, flop, reps, sample):
        res = {}
        for th in (1, ncores):
            torch.set_num_threads(th)
            res[th] = rate(fn, flop, reps)
        torch.set_num_threads(ncores)
        out[key] = {"value": res[1], "unit": "TFLOP/s", "cores": 1, "kind": "port", "sample": sample,
                    "all_threads": {"value": res[ncores], "cores": ncores}}

    g = torch.Generator().manual_seed(7)
    # MPS merge: one GEMM m = n = 1024, k = 256
    a = torch.randn(1024, 256, dtype=torch.float64, generator=g)
    b = torch.randn(256, 1024, dtype=torch.float64, generator=g)
    both("mps_merge", lambda: torch.matmul(a, b), 2.0 * 1024 * 1024 * 256, 5,
         "full workload: A[256,4,256] x B[256,4,256] as one MKL dgemm (faer stand-in)")
    # the reference's C-ABI contract is the naive loop (naive.rs:45-187), far
    # too slow at this size: timed through the oracle's restatement of it on
    # the same pattern scaled down (A[48,4,48] x B[48,4,48]), one thread
    from oracle import oracle as orc

    rng = np.random.default_rng(5)
    na, nb = rng.standard_normal((48, 4, 48)), rng.standard_normal((48, 4, 48))
    orc.contract_naive(na, [1, 2, -1], nb, [-1, 3, 4])
    t0 = time.perf_counter()
    orc.contract_naive(na, [1, 2, -1], nb, [-1, 3, 4])
    naive_s = time.perf_counter() - t0
    out["mps_merge"]["abi_naive_contract"] = {
        "value": 2.0 * 192 * 192 * 48 / naive_s / 1e12, "unit": "TFLOP/s", "cores": 1, "kind": "port",
        "sample": "A[48,4,48] x B[48,4,48] through the oracle's restatement of naive.rs (the C ABI's contract)"}
    # square GEMM: a 2048^3 sample of the 4096^3 workload
    a = torch.randn(2048, 2048, dtype=torch.float64, generator=g)
    b = torch.randn(2048, 2048, dtype=torch.float64, generator=g)
    both("gemm4096", lambda: torch.matmul(a, b), 2.0 * 2048 ** 3, 2, "2048^3 sample, MKL dgemm (faer stand-in)")
    # DMRG chain at bond 1024, every step as einsum (TTGT on MKL)
    L, psi, W1, W2, R = [torch.from_numpy(np.ascontiguousarray(x)) for x in W.cfg3_tensors(1024)]
    eqs = ["awx,xpqb->awpqb", "awpqb,wvpr->aqbvr", "aqbvr,vuqt->abrut", "abrut,zub->artz"]

    def chain():
        cur = L
        for eq, rhs in zip(eqs, [psi, W1, W2, R]):
            cur = torch.einsum(eq, cur, rhs)
        return cur

    both("dmrg_chain", chain, sum(W.cfg3_flops(1024)), 1,
         "full chain at bond 1024, torch.einsum per step (permute + MKL dgemm)")
    # c128 two-site MPS chain (A.S).B over its 128 block pairs
    (sa, ca, ad), (ss, cs_, sd), (sb, cb, bd) = W.cfg5_tensors()
    Am = _blocks_as_mats(sa, ca, ad, 2)
    Bm = _blocks_as_mats(sb, cb, bd, 1)
    offs = np.concatenate([[0], np.cumsum(sa[2])])
    Am = {c: torch.from_numpy(m * sd[offs[c[2]]:offs[c[2]] + m.shape[1]][None, :]) for c, m in Am.items()}
    Bm = {c: torch.from_numpy(m) for c, m in Bm.items()}
    pairs = [(ca_, cb_) for ca_ in ca for cb_ in cb if ca_[2] == cb_[0]]
    flop5 = W.flops_blocksparse((sa, ca, None), [1, 2, -1], (sb, cb, None), [-1, 3, 4], True)
    diag_t = torch.from_numpy(sd)

    def bs5():
        outb = {}
        for c in ca:  # diagonal scale of A's last axis
            m = Am[c]
            _ = m * diag_t[offs[c[2]]:offs[c[2]] + m.shape[1]][None, :]
        for x, y in pairs:
            key = (x[0], x[1], y[1], y[2])
            r = torch.matmul(Am[x], Bm[y])
            if key in outb:
                outb[key] += r
            else:
                outb[key] = r
        return outb

    both("bs_c128_mps", bs5, flop5, 1,
         "full chain: diagonal scale + 128 block-pair zgemm (MKL, faer stand-in) with per-block accumulation")
    # U(1) rank-4 half scale: a strided sample of the block pairs (~2e10 flop)
    dims = W.cfg4_dims(2)
    sizes, coords = W.cfg4_structure(dims)
    cset = set(coords)
    allp = []
    for x in coords:
        for y in coords:
            if x[2] == y[0] and x[3] == y[1]:
                allp.append((x, y, 2.0 * dims[x[0]] * dims[x[1]] * dims[x[2]] * dims[x[3]] * dims[y[2]] * dims[y[3]]))
    total = sum(f for _, _, f in allp)
    stride = max(1, int(total / 2e10))
    sample = allp[::stride]
    flop4 = sum(f for _, _, f in sample)
    mats = {}
    for x, y, _ in sample:
        for c, split, tag in ((x, 2, "a"), (y, 2, "b")):
            if (tag, c) not in mats:
                r = dims[c[0]] * dims[c[1]]
                k2 = dims[c[2]] * dims[c[3]]
                mats[(tag, c)] = torch.randn(r, k2, dtype=torch.float64, generator=g)
    assert all(c in cset for c in [p[0] for p in sample])

    def bs4():
        outb = {}
        for x, y, _ in sample:
            key = (x[0], x[1], y[2], y[3])
            r = torch.matmul(mats[("a", x)], mats[("b", y)])
            if key in outb:
                outb[key] += r
            else:
                outb[key] = r
        return outb

    both("bs_u1_rank4", bs4, flop4, 1,
         f"{len(sample)} of {len(allp)} block pairs ({flop4:.3g} of {total:.3g} flop, every {stride}th pair), "
         "dgemm per pair (MKL, faer stand-in) with per-block accumulation")
    torch.set_num_threads(ncores)
    return out


def host_info():
    """CPU model, logical cores and RAM of the host the CPU legs ran on."""
    cpu, ram = None, None
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    cpu = ln.split(":", 1)[1].strip()
                    break
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemTotal"):
                    ram = round(int(ln.split()[1]) / 1024 ** 2, 1)
                    break
    except OSError:
        pass
    return {"cpu": cpu, "logical_cores": os.cpu_count(), "ram_gib": ram}


def run_reference(args, world, rank):
    if rank != 0:
        return  # rank 0 alone runs the host-CPU reference
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_permute_time(threads)
    times = [cpu_permute_time(threads) for _ in range(args.steps)]
    t = sum(times)
    value = BYTES_F64 * args.steps / t / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "permutedims 16^6 f64 perm (5,3,1,0,4,2)", "batch": 1,
                   "l2": "input 134 MB > 126 MB L2"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"full 16^6 f64 tensor per step, {threads} host threads over the source index range"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host": host_info(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours
def _r3(x):
    return None if x is None else float(f"{x:.3g}")


def summary_rows(line_head, extras):
    """One short row per configuration, printed as the line's last key so that
    a reader of the line's tail sees every configuration's number:
    [cfg, value, unit, roofline fraction (executed for 3M complex), ms, n_gpus,
    parity (max relative error checked in this run, or null)]."""
    rows = [["c2 permute f64 (headline)", _r3(line_head["value"]), "GB/s", _r3(line_head["achieved"] /
             line_head["peak"]), _r3(line_head["ms"]), line_head["world"], 0.0]]
    if line_head.get("e2e"):
        rows.append(["c2 permute f64 e2e (C ABI, host buffers)", _r3(line_head["e2e"]["value"]), "GB/s", None,
                     None, line_head["world"], None])
    for e in extras:
        if "cfg" not in e:
            continue
        rf = e.get("roofline") or {}
        frac = rf.get("executed_frac", rf.get("frac"))
        par = e.get("parity")
        perr = None
        if isinstance(par, dict):
            perr = _r3(par.get("max_block_rel_err", par.get("rel_err")))
            if not par.get("ok", False):
                perr = "FAIL"
        unit = {"TFLOP/s": "TF/s", "GB/s": "GB/s"}.get(e.get("unit"), e.get("unit"))
        rows.append([e["cfg"], _r3(e.get("value")), unit, _r3(frac), _r3(e.get("ms")), e.get("n_gpus", 1), perr])
        if e.get("e2e"):
            rows.append([e["cfg"] + " e2e", _r3(e["e2e"]["value"]), unit, None, _r3(e["e2e"].get("ms")),
                         e.get("n_gpus", 1), None])
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--no-extras", action="store_true", help="skip the contraction sub-results")
    args = ap.parse_args()
    world, rank, local = dist_setup(args)

    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import numpy as np
    import torch

    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        pg = dist

    import ndtensors_b200 as ndt

    lib = ndt.get_lib()
    # one dedicated stream: the library's kernels and the timing events share it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ndt.set_stream(stream.cuda_stream)

    # ---- inputs resident in HBM: `batch` distinct tensors (seeded)
    g = torch.Generator(device="cuda")
    g.manual_seed(1002 + rank)
    B = args.batch
    src = torch.randn(B, NELEM, dtype=torch.float64, device="cuda", generator=g)
    dst = torch.empty_like(src)
    shape_c = (ctypes.c_size_t * 6)(*SHAPE)
    perm_c = (ctypes.c_size_t * 6)(*PERM)
    sptr = ctypes.c_void_p(stream.cuda_stream)

    def step():
        for i in range(B):
            st = lib.ndt_b200_permutedims_dev(0, ctypes.c_void_p(src[i].data_ptr()), ctypes.c_void_p(dst[i].data_ptr()),
                                              shape_c, 6, perm_c, 6, sptr)
            if st != 0:
                raise RuntimeError(f"permutedims failed: {st} {ndt.last_error()}")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # parity spot check of the timed kernel on a slice (bit-exact vs torch permute)
    ref0 = src[0].view(*reversed(SHAPE)).permute(*[5 - p for p in reversed(PERM)]).contiguous()
    assert torch.equal(ref0.flatten(), dst[0]), "permute mismatch"
    # The B launches of a step are replayed from a CUDA graph (launch gaps
    # between the per-tensor kernels are the only host cost left).
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    dst.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(ref0.flatten(), dst[0]), "permute mismatch (graph replay)"

    def step():  # noqa: F811  (the timed step: one graph replay of B kernels)
        graph.replay()

    for _ in range(2):
        step()

    # per-launch durations of the dominant kernel inside the timed region
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    launches0 = ndt.launch_count()
    sampler = ClockSampler(torch.cuda.current_device())
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with sampler:
        t0.record()
        for k in range(args.steps):
            ev[k][0].record()
            step()
            ev[k][1].record()
        t1.record()
        torch.cuda.synchronize()
    if pg:
        pg.barrier()
    # kernels in the timed region: the graph holds the B launches captured above
    launches = B * args.steps
    assert ndt.launch_count() == launches0, "graph replays only"
    ms = t0.elapsed_time(t1)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    ms_t = torch.tensor([ms], device="cuda")
    if pg:
        pg.all_reduce(ms_t, op=pg.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    total_bytes = BYTES_F64 * B * args.steps * world
    value = total_bytes / (ms_max * 1e-3) / 1e9
    launch_ms = statistics.mean(step_ms) / B
    achieved = BYTES_F64 / (launch_ms * 1e-3) / 1e9
    peaks, peak_src = measured_peaks()

    # The same batch as ONE launch: a rank-7 permute whose last axis (the
    # batch, unmoved) becomes an outer tile dimension -- no launch gaps, one
    # tail for the whole batch.
    shape7 = (ctypes.c_size_t * 7)(*(SHAPE + (B,)))
    perm7 = (ctypes.c_size_t * 7)(*(PERM + (6,)))

    def batched():
        st = lib.ndt_b200_permutedims_dev(0, ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
                                          shape7, 7, perm7, 7, sptr)
        assert st == 0, ndt.last_error()

    for _ in range(3):
        batched()
    torch.cuda.synchronize()
    assert torch.equal(ref0.flatten(), dst[0]), "permute mismatch (batched launch)"
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record()
    for _ in range(args.steps):
        batched()
    b1.record()
    torch.cuda.synchronize()
    batched_gbs = BYTES_F64 * B * args.steps / (b0.elapsed_time(b1) * 1e-3) / 1e9
    batched_line = {"cfg": "c2 permute f64 x32 1 launch", "workload": f"permutedims 16^6 f64 perm (5,3,1,0,4,2), batch of {B} as one rank-7 launch",
                    "value": batched_gbs, "unit": "GB/s",
                    "roofline": {"bound": "hbm", "achieved": batched_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                 "frac": batched_gbs / peaks["hbm_gbs"]}}

    # ---- end to end through the C ABI with host buffers (pinned)
    e2e = None
    host_in = torch.empty(NELEM, dtype=torch.float64, pin_memory=True)
    host_in.copy_(src[0].cpu())
    hp = ctypes.cast(host_in.data_ptr(), ctypes.POINTER(ctypes.c_double))
    st = ctypes.c_int(-999)

    dev_index = torch.cuda.current_device()

    def e2e_steps_on_thread(count, errs):
        # one host thread's share of the steps; ctypes releases the GIL inside each C call
        torch.cuda.set_device(dev_index)
        stl = ctypes.c_int(-999)
        for _ in range(count):
            t = lib.ndt_tensor_f64_from_data(hp, NELEM, shape_c, 6, ctypes.byref(stl))
            p = lib.ndt_tensor_f64_permutedims(t, perm_c, 6, ctypes.byref(stl))
            d = lib.ndt_tensor_f64_data(p)  # device -> host read of the result
            if not d or stl.value != 0:
                errs.append(stl.value)
            lib.ndt_tensor_f64_release(p)
            lib.ndt_tensor_f64_release(t)

    def e2e_run(nsteps, nthreads):
        """Wall time of nsteps H2D -> permutedims -> D2H steps through the C ABI,
        split over nthreads host threads (the library uploads on one stream,
        computes on another and reads back on a third, so one thread's read
        overlaps another's upload on the two PCIe directions)."""
        errs = []
        share = [nsteps // nthreads + (1 if i < nsteps % nthreads else 0) for i in range(nthreads)]
        ths = [threading.Thread(target=e2e_steps_on_thread, args=(c, errs)) for c in share]
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        torch.cuda.synchronize()
        dt = time.perf_counter() - w0
        assert not errs, f"C ABI step failed: {errs[:3]}"
        w = torch.tensor([dt], device="cuda")
        if pg:
            pg.all_reduce(w, op=pg.ReduceOp.MAX)
        return float(w.item())

    # the C ABI's host result equals the device reference, bit for bit
    import numpy as np
    t = lib.ndt_tensor_f64_from_data(hp, NELEM, shape_c, 6, ctypes.byref(st))
    p = lib.ndt_tensor_f64_permutedims(t, perm_c, 6, ctypes.byref(st))
    d = lib.ndt_tensor_f64_data(p)
    assert d and st.value == 0 and np.array_equal(np.ctypeslib.as_array(d, shape=(NELEM,)),
                                                  ref0.flatten().cpu().numpy()), "C ABI permute mismatch"
    lib.ndt_tensor_f64_release(p)
    lib.ndt_tensor_f64_release(t)
    E2E_THREADS = 2
    # warm-up: hold 2 x E2E_THREADS steps' tensors at once, so the library's pinned host
    # mirrors and device pool already hold what the threads can have in flight, then run
    # the threaded loop itself
    held = []
    for _ in range(2 * E2E_THREADS):
        t = lib.ndt_tensor_f64_from_data(hp, NELEM, shape_c, 6, ctypes.byref(st))
        p = lib.ndt_tensor_f64_permutedims(t, perm_c, 6, ctypes.byref(st))
        assert lib.ndt_tensor_f64_data(p) and st.value == 0
        held += [t, p]
    for h in held:
        lib.ndt_tensor_f64_release(h)
    e2e_run(4 * E2E_THREADS, E2E_THREADS)
    e2e_steps = max(6, min(args.steps, 40))
    t_multi = e2e_run(e2e_steps, E2E_THREADS)
    t_single = e2e_run(e2e_steps, 1)
    e2e = {"value": BYTES_F64 * e2e_steps * world / t_multi / 1e9, "unit": "GB/s",
           "h2d_bytes_per_step": NELEM * 8, "d2h_bytes_per_step": NELEM * 8,
           "host_threads": E2E_THREADS,
           "single_thread_value": BYTES_F64 * e2e_steps * world / t_single / 1e9,
           "path": "ndt_tensor_f64_from_data (pinned host) -> ndt_tensor_f64_permutedims -> ndt_tensor_f64_data, "
                   f"steps split over {E2E_THREADS} host threads"}

    # ---- extras: complex permute and the dense f64 MPS merge (DMMA GEMM)
    extras = [batched_line]
    del src, dst
    torch.cuda.empty_cache()
    if not args.no_extras:
        fp64_peak(stream)
        if world == 1:
            extras += run_extras(args, torch, lib, ndt, stream, peaks)
        extras += run_dmrg(args, torch, ndt, peaks, world, rank, pg)
        extras += run_blocksparse(args, torch, ndt, world, rank, pg)

    if world == 1 and not args.no_extras:
        e2e_c = contraction_e2e(torch, ndt, lib)
        for e in extras:
            if e.get("cfg") in e2e_c and e.get("n_gpus", 1) == 1:
                e["e2e"] = e2e_c[e["cfg"]]

    # ---- parity of every checked configuration, max over ranks (each rank
    # checked its own output blocks / slab against the CPU reference)
    parity_ok = True
    for e in extras:
        par = e.get("parity")
        if not isinstance(par, dict):
            continue
        key = "max_block_rel_err" if "max_block_rel_err" in par else "rel_err"
        t = torch.tensor([float(par.get(key, 0.0)), 0.0 if par.get("ok", False) else 1.0], device="cuda")
        if pg:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        par[key] = float(t[0].item())
        par["ok"] = bool(t[1].item() == 0.0)
        par["over_ranks"] = world
        parity_ok = parity_ok and par["ok"]

    # ---- CPU baseline (rank 0, N=1 only): the oracle port on one host thread
    if rank == 0 and world == 1 and not args.no_extras:
        cb = cpu_contraction_baselines()
        keymap = [("contract A[256,4,256]", "mps_merge"), ("f64 GEMM 4096^3", "gemm4096"), ("DMRG", "dmrg_chain"),
                  ("block-sparse c128 two-site MPS (A.S).B", "bs_c128_mps"), ("block-sparse U(1)", "bs_u1_rank4")]
        for e in extras:
            for prefix, key in keymap:
                if e["workload"].startswith(prefix) and key in cb:
                    e["cpu_baseline"] = cb[key]

    cpu = None
    if rank == 0 and world == 1:
        t_cpu = cpu_permute_time(1)
        cpu = {"value": BYTES_F64 / t_cpu / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": "one full 16^6 f64 tensor, GenericBackend::permute_into restated in C (oracle), 1 thread"}

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f64",
            "data": "synthetic (seeded N(0,1), torch generator on device)",
            "config": {"workload": "permutedims 16^6 f64 perm (5,3,1,0,4,2)", "batch": B,
                       "parallelism": f"replicas x{world}",
                       "l2": f"inputs larger than L2: {B} distinct 134 MB tensors per step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"], "traffic": ncu_traffic("permute_16p6_f64"),
                         "traffic_read": ncu_traffic("permute_16p6_f64_read"),
                         "traffic_note": "ncu dram bytes inside the launch; part of the 134.2 MB of writes drains "
                                         "from L2 after the kernel ends and is not counted, so compare traffic_read "
                                         "with the 134.2 MB of algorithmic reads",
                         "kernel": "permute_tiled_kernel<8>", "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_src})",
                         "algorithmic_bytes_per_launch": BYTES_F64},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": sampler.result(),
            "host": host_info(),
            "contraction": extras,
            "summary": summary_rows(line_head={"value": value, "achieved": achieved, "peak": peaks["hbm_gbs"],
                                               "ms": ms_max / args.steps, "world": world, "e2e": e2e},
                                    extras=extras),
        }
        print(json.dumps(line), flush=True)
    if pg:
        ndt.blocksparse.Comm._by_group.clear()  # the library's communicators, before the group goes
        pg.barrier()
        pg.destroy_process_group()
    if not parity_ok:
        # a rate whose result differs from the reference is not a result
        raise SystemExit("parity check failed: see the 'parity' keys of the line")


def _host_threads(torch, world):
    """Share the host cores between the ranks of this node for CPU checks."""
    torch.set_num_threads(max(1, (os.cpu_count() or 8) // max(1, world)))


def _device_blocks(torch, bs, t, coords):
    """{coords: numpy block} of a library block-sparse tensor, copying only
    the listed blocks from the device."""
    _, allc, offs = t._structure()
    allc = [tuple(int(x) for x in c) for c in allc]
    ends = list(offs[1:]) + [t.nnz]
    where = {c: (int(o), int(e)) for c, o, e in zip(allc, offs, ends)}
    cplx = isinstance(t, bs.BlockSparseC64)
    span = torch.as_tensor(bs._DeviceSpan(t.device_ptr(), t.nnz * (2 if cplx else 1)), device="cuda")
    out = {}
    for c in coords:
        o, e = where[tuple(c)]
        v = span[(2 if cplx else 1) * o:(2 if cplx else 1) * e].cpu().numpy()
        out[tuple(c)] = v.view(np.complex128) if cplx else v
    return out


def block_parity(torch, bs, result, A, B, nfree_a, nc, world, kscale=None, cplx=False, every=10,
                 flop_budget=None, expect_coords=None):
    """Check a seeded sample of `result`'s output blocks (every `every`-th in
    sorted order, plus the one with the most flops, within `flop_budget`)
    against the CPU block reference (tests/blockref.py: per output block, the
    sum of its pair GEMMs in float64 / complex128, as
    contract/blocksparse.rs:144-180 computes it).  With `expect_coords`, the
    result's block list must equal it exactly.  Returns the parity record."""
    import blockref

    coords = [tuple(int(x) for x in c) for c in result.coords]
    rec = {"tol": 1e-12, "blocks": len(coords)}
    if expect_coords is not None:
        rec["structure_ok"] = coords == [tuple(c) for c in expect_coords]
    fl = blockref.pair_flops(A, B, nfree_a, nc, coords, cplx)
    pick = list(coords[::every])
    if coords:
        big = max(coords, key=lambda c: fl[c])
        if big not in pick:
            pick.append(big)
    if flop_budget is not None:
        pick.sort(key=lambda c: fl[c])
        chosen, used = [], 0.0
        for c in pick:
            if used + fl[c] <= flop_budget:
                chosen.append(c)
                used += fl[c]
        pick = chosen
    _host_threads(torch, world)
    ref = blockref.reference_blocks(A, B, nfree_a, nc, pick, kscale=kscale)
    got = _device_blocks(torch, bs, result, pick)
    errs = [blockref.rel_fro(got[c], ref[c]) for c in pick]
    num = sum(float(np.linalg.norm(got[c] - ref[c]) ** 2) for c in pick)
    den = sum(float(np.linalg.norm(ref[c]) ** 2) for c in pick)
    rec.update({"checked": len(pick), "checked_flop_frac": (sum(fl[c] for c in pick) / max(sum(fl.values()), 1.0)),
                "max_block_rel_err": max(errs) if errs else 0.0,
                "rel_err": (num / den) ** 0.5 if den > 0 else 0.0})
    rec["ok"] = bool(rec["max_block_rel_err"] <= 1e-12 and rec.get("structure_ok", True) and
                     (len(pick) > 0 or not coords))
    return rec


def run_blocksparse(args, torch, ndt, world, rank, pg):
    """Block-sparse contractions (U(1) rank-4 at half scale, c128 two-site MPS) on
    FP64 tensor cores; with N ranks each computes its FLOP-balanced share of
    the output blocks (strong scaling: the total work is fixed)."""
    sys.path.insert(0, str(ROOT / "tests"))
    import workloads as W

    bs = ndt.blocksparse
    out = []

    def timed(fn, reps, warm=3, groups=3):
        """Median over `groups` runs of `reps` back-to-back calls (ms per call)."""
        for _ in range(warm):
            r = fn()
        r = None  # the timed calls reuse the warm-up's memory instead of growing the pool
        per = []
        for _ in range(groups):
            if pg:
                pg.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                r = fn()
            e1.record()
            torch.cuda.synchronize()
            per.append(e0.elapsed_time(e1) / reps)
        t = torch.tensor([statistics.median(per)], device="cuda")
        if pg:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item()), r

    # ---- U(1) rank-4 x rank-4, 9 sectors, dims halved
    dims = W.cfg4_dims(2)
    sizes, coords = W.cfg4_structure(dims)
    total = sum(W.block_elems(sizes, coords))
    g = torch.Generator(device="cuda")
    g.manual_seed(1004)
    dA = torch.randn(total, dtype=torch.float64, device="cuda", generator=g)
    dB = torch.randn(total, dtype=torch.float64, device="cuda", generator=g)
    A = bs.BlockSparseF64.from_torch(sizes, coords, dA)
    B = bs.BlockSparseF64.from_torch(sizes, coords, dB)
    la, lb = [1, 2, -1, -2], [-1, -2, 3, 4]
    flops = W.flops_blocksparse((sizes, coords, None), la, (sizes, coords, None), lb, False)
    if world == 1:
        ms, r = timed(lambda: bs.contract(A, la, B, lb), 3, warm=2, groups=1)
    else:
        ms, r = timed(lambda: bs.contract_shard(A, la, B, lb, rank, world), 3, warm=2, groups=1)
    # the timed result checked against the CPU block reference (the operands
    # stay on the device; only the blocks a sampled pair uses are copied)
    par = block_parity(torch, bs, r, (sizes, coords, dA), (sizes, coords, dB), 2, 2, world)
    tf = flops / (ms * 1e-3) / 1e12
    out.append({"cfg": "c4 U1 half", "value": tf, "unit": "TFLOP/s", "ms": ms, "flop": flops, "n_gpus": world,
                "scaling": "strong" if world > 1 else None, "parity": par,
                "roofline": fp64_roofline(tf / world),
                "workload": "block-sparse U(1) rank-4 x rank-4 f64, sector dims halved [4,12,28,48,72,48,28,12,4] "
                            "(489 blocks, 4.25 GB per operand)"})
    del A, B, r, dA, dB
    torch.cuda.empty_cache()

    # ---- c128 two-site MPS (A . S) . B, bond 8192, 33 sectors
    Ah, Sh, Bh = W.cfg5_tensors()
    (sa, ca, a), (ss, cs_, sd), (sb, cb, b) = Ah, Sh, Bh
    A = bs.BlockSparseC64.from_blocks(sa, ca, a)
    S = bs.DiagBlockSparseC64.from_blocks(ss, cs_, sd)
    B = bs.BlockSparseC64.from_blocks(sb, cb, b)
    flops5 = W.flops_blocksparse((sa, ca, None), [1, 2, -1], (sb, cb, None), [-1, 3, 4], True)

    def chain():
        # one grouped launch per rank: S's diagonal scales A's loads (no A.S pass)
        return bs.contract_through_diag(A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4], rank, world)

    ms5, r5 = timed(chain, 10)
    import blockref

    all5 = blockref.output_coords(Ah, Bh, 2, 1)
    par5 = block_parity(torch, bs, r5, Ah, Bh, 2, 1, world, kscale=np.asarray(sd), cplx=True, every=1,
                        expect_coords=all5 if world == 1 else None)
    tf5 = flops5 / (ms5 * 1e-3) / 1e12
    entry = {"cfg": "c5 c128 MPS", "value": tf5, "unit": "TFLOP/s", "ms": ms5, "flop": flops5, "n_gpus": world,
             "scaling": "strong" if world > 1 else None, "gather": "none (compute only)", "parity": par5,
             "roofline": fp64_roofline(tf5 / world, complex_3m=True),
             "workload": "block-sparse c128 two-site MPS (A.S).B, bond 8192 in 33 sectors, DiagBlockSparse S"}
    out.append(entry)
    del r5
    if world > 1:
        comm = bs.Comm.from_group()
        msg, rg = timed(lambda: bs.contract_through_diag_gathered(A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4], comm),
                        5)
        # the gathered tensor: the unsharded block list, every block checked
        parg = block_parity(torch, bs, rg, Ah, Bh, 2, 1, world, kscale=np.asarray(sd), cplx=True, every=1,
                            expect_coords=all5)
        out.append({"cfg": "c5 c128 MPS+gather", "value": flops5 / (msg * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms": msg, "n_gpus": world, "scaling": "strong", "parity": parg,
                    "gather": "gathered in the library (ndt_blocksparse_c64_contract_through_diag_gathered): "
                              "the grouped kernel's epilogue stores each tile into every rank's IPC-mapped buffer "
                              "over NVLink, one NCCL barrier, one copy into the result (NCCL all-gather per chunk "
                              "when the buffers cannot be mapped)",
                    "workload": "block-sparse c128 two-site MPS, sharded + gathered on every rank"})
        del rg
    if world >= 4:
        del A, S, B
        torch.cuda.empty_cache()
        out.append(literal_u1_rank4(torch, ndt, W, world, rank, timed))
    return out


def literal_u1_rank4(torch, ndt, W, world, rank, timed):
    """U(1) rank-4 x rank-4 at its literal size: 489 blocks per operand, 68 GB per
    operand, 6.39e14 flop.  A+B+C do not fit one GPU; each rank keeps only the
    A and B blocks its output blocks reference and computes its output blocks
    with contract_select.  Output blocks go to ranks by longest processing
    time (balanced FLOPs; 105 GB per rank at 8 ranks) when every rank's
    referenced blocks fit in 65% of the device memory, else as the
    contiguous FLOP-balanced ranges of contract_shard (104 GB per rank at 4).
    Block data: N(0,1) from a generator seeded by (operand, block index), so
    a block shared by several ranks holds the same values on all of them."""
    from math import prod

    bs = ndt.blocksparse
    dims = W.cfg4_dims(1)
    sizes, coords = W.cfg4_structure(dims)
    la, lb = [1, 2, -1, -2], [-1, -2, 3, 4]
    elems = {c: prod(dims[x] for x in c) for c in coords}
    pairs = {}
    for x in coords:
        for y in coords:
            if x[2:] == y[:2]:
                pairs.setdefault((x[0], x[1], y[2], y[3]), []).append(
                    (x, y, 2.0 * elems[x] * dims[y[2]] * dims[y[3]]))
    outs = sorted(pairs)
    work = {o: sum(f for _, _, f in pairs[o]) for o in outs}
    total = sum(work.values())

    def footprint(lst):  # bytes of referenced A, B blocks and output blocks
        a = {x for o in lst for x, _, _ in pairs[o]}
        b = {y for o in lst for _, y, _ in pairs[o]}
        return 8 * (sum(elems[c] for c in a) + sum(elems[c] for c in b) + sum(elems[o] for o in lst))

    # contiguous FLOP-balanced ranges of the sorted output blocks (the
    # library's contract_shard rule): small footprints, coarse balance
    contiguous, acc, r = [[] for _ in range(world)], 0.0, 0
    for o in outs:
        while r < world - 1 and acc >= total * (r + 1) / world:
            r += 1
        contiguous[r].append(o)
        acc += work[o]
    # longest-processing-time assignment: balanced FLOPs, larger footprints;
    # used when every rank's blocks fit in 65% of the device memory
    lpt = [[] for _ in range(world)]
    load = [0.0] * world
    for o in sorted(outs, key=lambda o: -work[o]):
        q = min(range(world), key=lambda i: load[i])
        lpt[q].append(o)
        load[q] += work[o]
    budget = 0.65 * torch.cuda.mem_get_info()[1]
    use_lpt = max(footprint(lst) for lst in lpt) <= budget
    plan = lpt if use_lpt else contiguous
    mine = sorted(plan[rank])
    used_a = {x for o in mine for x, _, _ in pairs[o]}
    used_b = {y for o in mine for _, y, _ in pairs[o]}

    def make(keep, seed):
        kept = [(i, c) for i, c in enumerate(coords) if c in keep]
        t = bs.BlockSparseF64.zeros(sizes, [c for _, c in kept])
        if t.nnz:
            view = torch.as_tensor(bs._DeviceSpan(t.device_ptr_mut(), t.nnz), device="cuda")
            off = 0
            for i, c in kept:
                g = torch.Generator(device="cuda").manual_seed(seed * 1000 + i)
                view[off:off + elems[c]].normal_(generator=g)
                off += elems[c]
        return t, [c for _, c in kept]

    A, ka = make(used_a, 1)
    B, kb = make(used_b, 2)
    torch.cuda.synchronize()
    ms, r = timed(lambda: bs.contract_select(A, la, B, lb, mine), 1, warm=1, groups=1)
    tf = total / (ms * 1e-3) / 1e12
    # a sample of this rank's output blocks against the CPU block reference,
    # within 3e11 flop of host work per rank (the largest blocks are 1e13)
    span = lambda t: torch.as_tensor(bs._DeviceSpan(t.device_ptr(), t.nnz), device="cuda")  # noqa: E731
    par = block_parity(torch, bs, r, (sizes, ka, span(A)), (sizes, kb, span(B)), 2, 2, world, flop_budget=3e11,
                       expect_coords=mine)
    return {"cfg": "c4 U1 literal", "parity": par,
            "workload": "block-sparse U(1) rank-4 x rank-4 f64 at the literal size [8,24,56,96,144,96,56,24,8] "
                        "(489 blocks, 68 GB per operand, 6.39e14 flop), each rank holding only the blocks its "
                        "output blocks reference",
            "value": tf, "unit": "TFLOP/s", "ms": ms, "flop": total, "n_gpus": world, "scaling": "strong",
            "roofline": fp64_roofline(tf / world),
            "assignment": "longest-processing-time" if use_lpt else "contiguous FLOP-balanced ranges",
            "max_rank_flop_share": max(sum(work[o] for o in lst) for lst in plan) / total,
            "max_rank_gb": max(footprint(lst) for lst in plan) / 1e9}


def contraction_e2e(torch, ndt, lib):
    """End-to-end times of contraction configurations through the C ABI with
    host buffers (pinned), one host thread, wall clock: every step uploads
    the inputs (from_data), contracts, and reads the result back (data()).
    Returns {cfg: {"value": TFLOP/s, "ms", "h2d_bytes_per_step",
    "d2h_bytes_per_step", "path"}}."""
    sys.path.insert(0, str(ROOT / "tests"))
    import workloads as W

    def pinned(x):
        t = torch.empty(x.size, dtype=torch.float64 if x.dtype == np.float64 else torch.complex128, pin_memory=True)
        t.numpy()[:] = np.asarray(x).ravel(order="F")
        return t

    def wall(fn, reps, warm=2):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - w0) / reps * 1e3

    res = {}
    st = ctypes.c_int(-999)
    dp = ctypes.POINTER(ctypes.c_double)
    # ---- c1: MPS merge A[256,4,256] x B[256,4,256] through ndt_tensor_f64_contract
    rng = np.random.default_rng(1001)
    a, b = rng.standard_normal((256, 4, 256)), rng.standard_normal((256, 4, 256))
    pa, pb = pinned(a), pinned(b)
    shp = (ctypes.c_size_t * 3)(256, 4, 256)
    la, lb = (ctypes.c_long * 3)(1, 2, -1), (ctypes.c_long * 3)(-1, 3, 4)

    def c1():
        ta = lib.ndt_tensor_f64_from_data(ctypes.cast(pa.data_ptr(), dp), pa.numel(), shp, 3, ctypes.byref(st))
        tb = lib.ndt_tensor_f64_from_data(ctypes.cast(pb.data_ptr(), dp), pb.numel(), shp, 3, ctypes.byref(st))
        tc = lib.ndt_tensor_f64_contract(ta, la, 3, tb, lb, 3, ctypes.byref(st))
        assert st.value == 0 and lib.ndt_tensor_f64_data(tc)
        for t in (ta, tb, tc):
            lib.ndt_tensor_f64_release(t)

    ms = wall(c1, 20)
    res["c1 MPS merge"] = {"value": 2.0 * 1024 * 1024 * 256 / (ms * 1e-3) / 1e12, "ms": ms,
                           "h2d_bytes_per_step": 2 * a.nbytes, "d2h_bytes_per_step": 1024 * 1024 * 8,
                           "path": "from_data x2 -> ndt_tensor_f64_contract -> data"}
    # ---- c3: DMRG chain, bond 1024, through contract_gemm
    host = [pinned(x).numpy().reshape(x.shape, order="F") for x in W.cfg3_tensors(1024)]
    flops3 = sum(W.cfg3_flops(1024))

    def c3():
        ts = [ndt.TensorF64.from_numpy(x) for x in host]
        cur = ts[0]
        for (la3, lb3), t in zip(W.CFG3_STEPS, ts[1:]):
            cur = ndt.contract_gemm(cur, la3, t, lb3)
        assert lib.ndt_tensor_f64_data(cur._ptr)

    ms = wall(c3, 5)
    res["c3 DMRG chain"] = {"value": flops3 / (ms * 1e-3) / 1e12, "ms": ms,
                            "h2d_bytes_per_step": sum(x.nbytes for x in host),
                            "d2h_bytes_per_step": 1024 * 2 * 2 * 1024 * 8,
                            "path": "from_data x5 -> contract_gemm x4 -> data"}
    # ---- c5: c128 two-site MPS (A.S).B, bond 8192
    (sa, ca, a5), (ss, cs5, sd), (sb, cb, b5) = W.cfg5_tensors()
    pa5, pb5 = pinned(a5).numpy(), pinned(b5).numpy()
    flops5 = W.flops_blocksparse((sa, ca, None), [1, 2, -1], (sb, cb, None), [-1, 3, 4], True)
    bs = ndt.blocksparse
    out_bytes = []

    def c5():
        A = bs.BlockSparseC64.from_blocks(sa, ca, pa5)
        S = bs.DiagBlockSparseC64.from_blocks(ss, cs5, sd)
        B = bs.BlockSparseC64.from_blocks(sb, cb, pb5)
        C = bs.contract_through_diag(A, [1, 2, -1], S, [-1, -2], B, [-2, 3, 4])
        assert lib.ndt_blocksparse_c64_data(C._ptr)
        out_bytes.append(C.nnz * 16)

    ms = wall(c5, 5)
    res["c5 c128 MPS"] = {"value": flops5 / (ms * 1e-3) / 1e12, "ms": ms,
                          "h2d_bytes_per_step": pa5.nbytes + pb5.nbytes + sd.nbytes,
                          "d2h_bytes_per_step": out_bytes[-1],
                          "path": "from_data (A, S, B) -> contract_through_diag -> data"}
    return res


def run_extras(args, torch, lib, ndt, stream, peaks):
    out = []
    sptr = ctypes.c_void_p(stream.cuda_stream)
    # complex128 permute of the same shape, timed like the f64 line: 32
    # distinct tensors per step (8.6 GB in, 8.6 GB out)
    src = torch.randn(32, NELEM, dtype=torch.complex128, device="cuda")
    dst = torch.empty_like(src)
    shape_c = (ctypes.c_size_t * 6)(*SHAPE)
    perm_c = (ctypes.c_size_t * 6)(*PERM)

    def cstep():
        for i in range(src.shape[0]):
            st = lib.ndt_b200_permutedims_dev(1, ctypes.c_void_p(src[i].data_ptr()),
                                              ctypes.c_void_p(dst[i].data_ptr()), shape_c, 6, perm_c, 6, sptr)
            assert st == 0, ndt.last_error()

    for _ in range(3):
        cstep()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record()
    for _ in range(reps):
        cstep()
    e1.record()
    torch.cuda.synchronize()
    per = e0.elapsed_time(e1) / (reps * src.shape[0])
    gbs = 2 * NELEM * 16 / (per * 1e-3) / 1e9
    out.append({"cfg": "c2 permute c128", "workload": "permutedims 16^6 c128 perm (5,3,1,0,4,2), 32 tensors per step",
                "value": gbs, "unit": "GB/s",
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": gbs / peaks["hbm_gbs"], "traffic": ncu_traffic("permute_16p6_c128")}})
    del src, dst
    # dense f64 MPS merge: A[256,4,256] x B[256,4,256] (labels (1,2,-1),(-1,3,4)) as one DMMA GEMM.
    # Timed as a stream of NM independent merges on distinct operands (12 MB each, NM x 12 MB > L2),
    # launched back to back between one event pair: a single launch between two events carries a
    # fixed event / launch cost of several microseconds on this part, a fifth of this 20 us kernel.
    m, n, k = 1024, 1024, 256
    NM = 16
    As = torch.randn(NM, m * k, dtype=torch.float64, device="cuda")
    Bs = torch.randn(NM, k * n, dtype=torch.float64, device="cuda")
    Cs = torch.empty(NM, m * n, dtype=torch.float64, device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 8, dtype=torch.float64, device="cuda")

    def g(i):
        st = lib.ndt_b200_gemm_dev(0, m, n, k, ctypes.c_void_p(As[i].data_ptr()), m, 0,
                                   ctypes.c_void_p(Bs[i].data_ptr()), k, 1, ctypes.c_void_p(Cs[i].data_ptr()), m, 0,
                                   sptr)
        assert st == 0

    for i in range(NM):
        g(i)
    reps = 10
    per = []
    for _ in range(reps):
        flush.zero_()  # L2 flush before each stream (outside the events)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(NM):
            g(i)
        b.record()
        torch.cuda.synchronize()
        per.append(a.elapsed_time(b) / NM)
    t = statistics.mean(per)
    single = []
    for _ in range(20):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g(0)
        b.record()
        torch.cuda.synchronize()
        single.append(a.elapsed_time(b))
    # cuBLAS DGEMM (torch.matmul) on the same operands and layout, timed the same way
    Am = [As[i].view(k, m).t() for i in range(NM)]
    Bm = [Bs[i].view(n, k).t() for i in range(NM)]
    for i in range(NM):
        torch.matmul(Am[i], Bm[i])
    lib_per = []
    for _ in range(reps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(NM):
            torch.matmul(Am[i], Bm[i])
        b.record()
        torch.cuda.synchronize()
        lib_per.append(a.elapsed_time(b) / NM)
    tf = 2.0 * m * n * k / (t * 1e-3) / 1e12
    # 64x64 tiles of four 32x32 warp tiles; FP64 MMA throughput is per SM sub-partition (4 per SM)
    tiles, parts = (m // 64) * (n // 64), torch.cuda.get_device_properties(0).multi_processor_count * 4
    out.append({"cfg": "c1 MPS merge", "workload": "contract A[256,4,256] x B[256,4,256] -> C[256,4,4,256] f64 (MPS merge)",
                "value": tf, "unit": "TFLOP/s", "ms": t,
                "timing": f"{NM} independent merges back to back per event pair, L2 flushed before each stream",
                "single_launch_ms": statistics.mean(single),
                "cublas_dgemm_ms": statistics.mean(lib_per),
                "balance_ceiling": tiles * 4 / (math.ceil(tiles * 4 / parts) * parts),
                "roofline": fp64_roofline(tf)})
    del As, Bs, Cs, Am, Bm
    # a large square f64 GEMM for the kernel's steady-state rate
    def g():
        st = lib.ndt_b200_gemm_dev(0, m, n, k, ctypes.c_void_p(A.data_ptr()), m, 0, ctypes.c_void_p(Bt.data_ptr()),
                                   k, 1, ctypes.c_void_p(Ct.data_ptr()), m, 0, sptr)
        assert st == 0

    m = n = k = 4096
    A = torch.randn(m * k, dtype=torch.float64, device="cuda")
    Bt = torch.randn(k * n, dtype=torch.float64, device="cuda")
    Ct = torch.empty(m * n, dtype=torch.float64, device="cuda")
    for _ in range(2):
        g()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(5):
        g()
    b.record()
    torch.cuda.synchronize()
    t = a.elapsed_time(b) / 5
    tf = 2.0 * m * n * k / (t * 1e-3) / 1e12
    out.append({"cfg": "gemm 4096^3", "workload": "f64 GEMM 4096^3 (DMMA kernel steady state)", "value": tf, "unit": "TFLOP/s",
                "roofline": fp64_roofline(tf)})
    return out


def run_dmrg(args, torch, ndt, peaks, world=1, rank=0, pg=None):
    """DMRG environment-update chain, bond 1024: T1 = L.psi, T2 = T1.W1,
    T3 = T2.W2, E = T3.R through contract_gemm (8.67e10 flop).  Steps 1 and 4
    are DMMA GEMMs (step 4 packs its permuted operand); steps 2 and 3 run on
    the skinny kernel (k = n = 10 against 2^21 rows, HBM bound, permutation
    folded into the loads).  Inputs resident on the device; each step's
    output is the next step's input (168 MB intermediates, larger than L2).
    With N ranks the chain is split along the free index a (axis 0 of L and
    of every intermediate): rank r runs all four steps on L[a0:a1], no
    collective (strong scaling, times are the max over ranks)."""
    sys.path.insert(0, str(ROOT / "tests"))
    import numpy as np
    import workloads as W

    D = 1024
    T = ndt.TensorF64
    host = list(W.cfg3_tensors(D))
    ts = [T.from_numpy(x) for x in host]
    for t in ts:
        t.device_ptr()
    if world > 1:  # this rank's slab of L, for the host check below
        a0, a1 = rank * D // world, (rank + 1) * D // world
        host[0] = np.asfortranarray(host[0][a0:a1])
    L, psi, W1, W2, R = ts
    rhs = [psi, W1, W2, R]
    flops = W.cfg3_flops(D)

    def chain(ev=None):
        cur = L
        for i, ((la, lb), b) in enumerate(zip(W.CFG3_STEPS, rhs)):
            if ev:
                ev[i][0].record()
            if i == 0 and world > 1:
                # the library's dense split: this rank's range of the free index a
                cur = ndt.contract_gemm_shard(cur, la, b, lb, 1, rank, world)
            else:
                cur = ndt.contract_gemm(cur, la, b, lb)
            if ev:
                ev[i][1].record()
        return cur

    for _ in range(3):
        chain()
    torch.cuda.synchronize()
    reps = 10
    step_ms = [[] for _ in range(4)]
    tot = []
    for _ in range(reps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(4)]
        if pg:
            pg.barrier()
        torch.cuda.synchronize()
        chain(ev)
        torch.cuda.synchronize()
        for i in range(4):
            step_ms[i].append(ev[i][0].elapsed_time(ev[i][1]))
        tot.append(ev[0][0].elapsed_time(ev[3][1]))
    ms = [statistics.median(x) for x in step_ms]
    chain_ms = statistics.median(tot)
    # this rank's result against the same chain on the host (torch CPU
    # einsum in float64 over the rank's slab of L)
    _host_threads(torch, world)
    got = chain().to_numpy()
    tL, tpsi, tW1, tW2, tR = (torch.from_numpy(x) for x in host)
    t1 = torch.einsum("abx,xcde->abcde", tL, tpsi)
    t2 = torch.einsum("axyde,xfyg->adefg", t1, tW1)
    t3 = torch.einsum("aycxe,xfyg->acefg", t2, tW2)
    want = torch.einsum("axbyc,dyx->abcd", t3, tR).numpy()
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    par = {"tol": 1e-12, "rel_err": err, "ok": bool(err <= 1e-12),
           "reference": "torch CPU float64 einsum of the four steps on this rank's slab"}
    if pg:  # max over ranks
        t = torch.tensor(ms + [chain_ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        vals = t.tolist()
        ms, chain_ms = vals[:4], vals[4]
    skinny_bytes = 2 * (2 * D * D) * 10 * 8 + 100 * 8  # read 2D^2 x 10, write 2D^2 x 10, W
    out = {"cfg": "c3 DMRG chain", "parity": par,
           "workload": "DMRG environment chain L[1024,5,1024].psi[1024,2,2,1024].W1.W2.R[1024,5,1024] f64, "
                       "contract_gemm x4" + (f", split along a over {world} ranks" if world > 1 else ""),
           "value": sum(flops) / (chain_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": chain_ms, "flop": sum(flops),
           "n_gpus": world, "scaling": "strong" if world > 1 else None, "steps": []}
    for i in range(4):
        tf = flops[i] / (ms[i] * 1e-3) / 1e12
        st = {"step": i + 1, "ms": ms[i], "flop": flops[i], "tflops": tf}
        if i in (1, 2):
            gbs = skinny_bytes / (ms[i] * 1e-3) / 1e9 / world
            st["kernel"] = "skinny_kernel (k=n=10, strided loads)"
            st["roofline"] = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s per GPU",
                              "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes": skinny_bytes / world}
        else:
            st["kernel"] = "dmma_gemm_kernel" + (" (+ run-copy pack of the permuted A)" if i == 3 else "")
            st["roofline"] = fp64_roofline(tf / world)
        out["steps"].append(st)
    res = [out]
    if world == 1:
        # the same update as one network: greedy order contracts W1.W2 first
        # (400 entries) and applies it to T1 in one skinny pass (k = n = 20)
        labels = [[1, -1, -2], [-2, -3, -4, -5], [-1, -6, -3, 2], [-6, -7, -4, 3], [4, -7, -5]]
        net = lambda: ndt.contract_network([L, psi, W1, W2, R], labels)  # noqa: E731
        for _ in range(3):
            net()
        torch.cuda.synchronize()
        tn = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            net()
            e1.record()
            torch.cuda.synchronize()
            tn.append(e0.elapsed_time(e1))
        net_ms = statistics.median(tn)
        tf = sum(flops) / (net_ms * 1e-3) / 1e12
        res.append({"cfg": "c3 DMRG network", "workload": "DMRG environment update as one network (contract_network: W1.W2 fused into one "
                                "skinny pass), bond 1024", "value": tf, "unit": "TFLOP/s", "ms": net_ms,
                    "flop": sum(flops), "roofline": fp64_roofline(tf)})
    return res


if __name__ == "__main__":
    main()

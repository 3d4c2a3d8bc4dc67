"""Benchmark of the Arctic-embed-xs forward on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config c2|c1|c4] [--mode w8a8|w8a32|f32]
    python bench.py --model lenet [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Default workload: Arctic-embed-xs with int8 weights from the reference's
quantiser, batch 256 per GPU, seq 128, valid lengths U{16..128}, leading CLS 101, body ids
U{1000..30521}; the W8A8 tensor-core path.  Weak scaling: every rank runs its own 256 sequences
(the 256*N-sequence global batch is sharded by work) and the embeddings are gathered to rank 0.

`value`   : sequences/s over all ranks, inputs resident in HBM, device time (CUDA events around
            each step's forward + gather, L2 flushed before every step), max over ranks.
`e2e`     : the same metric through the public host API (tz_arctic_forward: host ids in, host
            embeddings out; H2D + D2H inside the timed call), wall time of the synchronous call.
`roofline`: the dominant kernel class, its algorithmic FLOPs and bytes per launch over its
            average launch duration, measured with CUDA events recorded between launches on the
            launching stream during the timed steps; `bound` is the binding limit (the larger of
            FLOPs / tensor peak and bytes / HBM peak), `limits` carries both fractions.
`--impl reference`: the reference's CPU algorithm (C restatement; the Zig reference cannot be
            built here) on the host cores, rank 0 only.
`--model lenet`: BASELINE configs[4], LeNet-5 (padded variant, softmax) over 65536 seeded U[0,1]
            images with Kaiming-uniform weights; the batch is split across the N ranks (strong
            scaling) and the [65536, 10] probabilities are gathered to rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "c1": dict(batch=8, seq=128, lmin=16, lmax=128, desc="configs[0] B=8 S=128"),
    "c2": dict(batch=256, seq=128, lmin=16, lmax=128, desc="configs[1] B=256 S=128"),
    "c4": dict(batch=8192, seq=512, lmin=32, lmax=512, desc="configs[3] B=8192 S=512"),
}
LIN_FLOP_PER_TOKEN = 2 * (4 * 384 * 384 + 2 * 384 * 1536)  # per layer
NCCL_SMS = 4  # N > 1: SMs left to the NCCL gather that overlaps the next forward
CLASS_NAMES = ["embed_ln", "qkv_gemm", "attention", "oproj_gemm_ln", "layernorm", "ffn1_gemm",
               "ffn_fused", "ffn2_gemm_ln", "pool_l2"]


def arctic_metric(config, mode):
    """The metric name both arms print for a config and mode: BASELINE's seq/s at the config's
    sequence length, for the f32 or the int8-weight model.  The arithmetic each arm runs (W8A8 on the
    GPU, the reference's W8A32 on the CPU) is in `dtype`, not in the name."""
    return f"Arctic-embed-xs seq/s @seq{CONFIGS[config]['seq']} ({'f32' if mode == 'f32' else 'int8'})"


def flop_useful(lens):
    L = np.asarray(lens, np.float64)
    return float(6 * (3538944 * L.sum() + 1536 * (L * L).sum()))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), d.get("bf16_tflops_sustained", 1400.0), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def class_bytes(cls, T, B, int8):
    """Algorithmic HBM bytes of one launch of a forward kernel class: the operands it must read and
    the results it must write, each once (weights once per launch), for T packed tokens.  Per token:
    the GEMM operand XA is int8 + an f32 scale (W8A8) or f16; QKV, the attention output OA and the
    FFN hidden H are f16 (W8A8 adds a u32 row |max| to OA and H); the residual stream X is f32, read
    and rewritten by each GEMM+LayerNorm kernel, which also writes the next XA.  The fused W8A8 FFN
    block (6) reads XA and X and writes X and the next XA; its hidden H stays on chip."""
    a_in = 384 + 4 if int8 else 768
    amax = 4 if int8 else 0
    wb = 1 if int8 else 2
    return {0: T * 384 * (4 + 1 + 4) + T * 384 * 2,
            1: T * (a_in + 1152 * 2) + 1152 * 384 * wb,
            2: T * (1152 * 2 + 384 * 2),
            3: T * (384 * 2 + amax + 384 * 4 * 2 + a_in) + 384 * 384 * wb,
            4: T * 384 * (4 + 4 + 1) + T * 4,
            5: T * (a_in + 1536 * 2 + amax) + 1536 * 384 * wb,
            6: T * (a_in + 384 * 4 * 2 + a_in) + 2 * 1536 * 384 * wb,
            7: T * (1536 * 2 + amax + 384 * 4 * 2 + a_in) + 384 * 1536 * wb,
            8: B * 384 * 8}[cls]


def measured_int8_peak():
    """Dense int8 tensor throughput measured on this GPU with cuBLAS (torch._int_mm, 8192^3, best of 5):
    the int8 roofline denominator (MEASURED_PEAKS.json carries only bf16)."""
    import torch
    a = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (8192, 8192), dtype=torch.int8, device="cuda").t()
    best = float("inf")
    for i in range(7):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        torch.cuda.synchronize()
        if i >= 2:
            best = min(best, s.elapsed_time(e))
    del a, b
    return 2.0 * 8192 ** 3 / (best / 1e3) / 1e12


def traffic_table():
    """Per-launch DRAM bytes from the committed ncu summary (profiles/ncu_traffic.txt), if any."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    out = {}
    if os.path.exists(p):
        for line in open(p):
            line = line.strip()
            if line and not line.startswith("#") and "=" in line:
                k, v = line.split("=", 1)
                try:
                    out[k.strip()] = float(v.split()[0])
                except ValueError:
                    pass
    return out


class Clocks:
    """SM clock, power and clock-event reasons sampled DURING the timed region.

    NVML (the library nvidia-smi reads) is polled every ~2 ms from a thread, so even a timed region of
    a few tens of milliseconds gets samples; `mark()` is called from the timing loop right after the
    steps are enqueued (the GPU is busy then) and only samples taken between `begin()` and `end()`
    count.  Falls back to `nvidia-smi -lms 200` when NVML is unavailable.  With `poll` false there is
    no thread, only the `mark()` sample: under torchrun only rank 0 (whose clocks the JSON line
    reports) polls, so that eight processes do not each make ~2000 NVML driver calls per second
    during the timed steps."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu: int, poll: bool = True):
        self.gpu = gpu
        self.poll = poll
        self.rows = []  # (t, sm_mhz, max_mhz, power_w, [reason names])
        self.window = []
        self.proc = None
        self.nv = None
        self.t = None
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml as N
        N.nvmlInit()
        try:
            import torch
            p = torch.cuda.get_device_properties(self.gpu)
            return N, N.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")
        except Exception:
            return N, N.nvmlDeviceGetHandleByIndex(self.gpu)

    def _sample_nvml(self):
        N, h = self.nv
        r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
        bits = [N.nvmlClocksEventReasonHwSlowdown, N.nvmlClocksEventReasonHwThermalSlowdown,
                N.nvmlClocksEventReasonSwThermalSlowdown, N.nvmlClocksEventReasonSwPowerCap]
        self.rows.append((time.perf_counter(), float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)),
                          float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)),
                          N.nvmlDeviceGetPowerUsage(h) / 1000.0, [n for n, b in zip(self.NAMES, bits) if r & b]))

    def _poll(self):
        while not self.stop.is_set():
            try:
                self._sample_nvml()
            except Exception:
                return
            time.sleep(0.002)

    def __enter__(self):
        try:
            self.nv = self._nvml_handle()
            self._sample_nvml()
            if self.poll:
                self.t = threading.Thread(target=self._poll, daemon=True)
                self.t.start()
            return self
        except Exception:
            self.nv = None
        if not self.poll:
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read_smi(self):
        for line in self.proc.stdout:
            r = [x.strip() for x in line.split(",")]
            if len(r) > 8 and r[1].replace(".", "").isdigit():
                self.rows.append((time.perf_counter(), float(r[1]), float(r[2]) if r[2].replace(".", "").isdigit() else None,
                                  None, [self.NAMES[i] for i in range(4) if r[5 + i] == "Active"]))

    def begin(self):
        self.window.append([time.perf_counter(), None])

    def mark(self):
        """Called while the GPU is busy with the timed steps: one sample inside the window."""
        if self.nv:
            try:
                self._sample_nvml()
            except Exception:
                pass

    def end(self):
        self.window[-1][1] = time.perf_counter()

    def __exit__(self, *a):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        elif self.t is not None:
            self.t.join(timeout=1)

    def summary(self):
        rows = [r for r in self.rows if any(a <= r[0] <= (b or a) for a, b in self.window)] if self.window else []
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock sample inside the timed region"],
                    "samples": 0}
        sm = [r[1] for r in rows]
        mx = [r[2] for r in rows if r[2]]
        pw = [r[3] for r in rows if r[3] is not None]
        reasons = sorted({n for r in rows for n in r[4]})
        out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
               "samples": len(rows), "source": "nvml" if self.nv else "nvidia-smi"}
        if pw:
            out["power_w_median"] = statistics.median(pw)
        return out


def cpu_forward_timing(w_ckpt, ids, lens, mode_name, budget_s=12.0, max_seqs=None):
    """Times the C restatement of the reference CPU forward (forwardBatchParallel semantics: one
    sequence per task on all host threads) on a bounded sample.  Returns (seq/s, sample, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not os.environ.get("TENZOR_BLAS_LIB"):
        found = find_cblas()
        if found:
            os.environ["TENZOR_BLAS_LIB"] = found
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    om = O.OracleModel(w_ckpt)
    mode = {"f32": O.MODE_F32, "w8a32": O.MODE_W8A32, "w8a8": O.MODE_W8A8}[mode_name]
    threads = os.cpu_count() or 1
    # probe: a small batch, then size the sample to ~budget_s
    n0 = min(len(lens), max(threads, 8))
    p, cu = _pack(ids[:n0], lens[:n0])
    t0 = time.perf_counter()
    om.forward(p, cu, mode, nthreads=threads)
    dt = time.perf_counter() - t0
    n = int(max(n0, min(len(lens), n0 * budget_s / max(dt, 1e-3))))
    if max_seqs:
        n = min(n, max_seqs)
    p, cu = _pack(ids[:n], lens[:n])
    t0 = time.perf_counter()
    om.forward(p, cu, mode, nthreads=threads)
    dt = time.perf_counter() - t0
    sample = f"first {n} sequences of the batch ({int(cu[-1])} tokens), {O.blas_status()}"
    return n / dt, sample, threads


def find_cblas():
    """A CBLAS for the CPU baseline when TENZOR_BLAS_LIB is unset: the reference's candidate
    library names (blas.zig:206-220) on the loader's search path first (the oracle tries those
    itself), else an OpenBLAS bundled with an installed Python package (``<pkg>.libs/libopenblas*``,
    which exports the standard cblas_* names).  None when neither exists."""
    import ctypes.util
    import glob
    import site
    for name in ("openblas", "openblas64_", "openblas64", "openblasp", "cblas", "blas", "mkl_rt"):
        if ctypes.util.find_library(name):
            return None  # the oracle's own search finds it
    roots = list(site.getsitepackages()) + [site.getusersitepackages()]
    for root in roots:
        for path in sorted(glob.glob(os.path.join(root, "*.libs", "libopenblas*.so*"))):
            return path
    return None


def _pack(ids, lens):
    from tenzor_b200 import synthetic as S
    return S.pack(ids, lens)


def make_inputs(cfg, world, batch_override=None):
    """(ids [B, S], lengths [B], the global row ids of each rank).  configs[0] / configs[1] scale
    weakly: rank r runs its own block of `batch` sequences whose lengths are those of the one-GPU
    batch (seed 7) and whose tokens are drawn from seed 7 + r, so every rank does the one-GPU work.
    configs[3] scales strongly: its fixed 8192-sequence batch is dealt by work (shard_by_tokens)."""
    from tenzor_b200 import synthetic as S
    from tenzor_b200.shard import shard_by_tokens
    c = CONFIGS[cfg]
    batch = batch_override or c["batch"]
    ids0, lens0 = S.token_batch(batch, c["seq"], c["lmin"], c["lmax"], seed=7)
    if cfg == "c4":
        return ids0, lens0, shard_by_tokens(lens0, world) if world > 1 else [np.arange(len(lens0))]
    ids = np.concatenate([ids0] + [S.token_batch_with_lengths(lens0, c["seq"], seed=7 + r) for r in range(1, world)])
    lens = np.concatenate([lens0] * world)
    return ids, lens, [np.arange(r * batch, (r + 1) * batch) for r in range(world)]


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    from tenzor_b200 import synthetic as S
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    w = S.arctic_weights(1234)
    ck = O.quantize_checkpoint(w) if a.mode != "f32" else w
    ids, lens, _ = make_inputs(a.config, world, a.batch)
    ref_mode = "w8a32" if a.mode != "f32" else "f32"  # the reference's own int8 path is W8A32
    vals = []
    sample = ""
    threads = os.cpu_count() or 1
    per_step_budget = max(2.0, 150.0 / max(1, a.steps + a.warmup))
    for i in range(a.warmup + a.steps):
        v, sample, threads = cpu_forward_timing(ck, ids, lens, ref_mode, budget_s=per_step_budget)
        if i >= a.warmup:
            vals.append(v)
    value = float(np.median(vals))
    line = {
        "impl": "reference", "metric": arctic_metric(a.config, a.mode),
        "value": value, "unit": "seq/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if ref_mode == "f32" else "int8-weight/f32 (W8A32)", "data": "synthetic",
        "config": {"workload": CONFIGS[a.config]["desc"], "mode": ref_mode, "global_batch": int(len(lens)),
                   "seq_len": CONFIGS[a.config]["seq"], "parallelism": "host threads (one sequence per task)"},
        "cpu_baseline": {"value": value, "unit": "seq/s", "cores": threads, "kind": "port",
                         "sample": sample + "; C restatement of arctic.zig forwardBatchParallel (Zig reference unbuildable here)"},
        "e2e": {"value": value, "unit": "seq/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(a):
    import torch
    import torch.distributed as dist
    from tenzor_b200 import synthetic as S
    from tenzor_b200 import _lib as L
    from tenzor_b200.arctic import ArcticModel
    from tenzor_b200.quantize import quantize_checkpoint
    from tenzor_b200.runtime import Context
    from tenzor_b200 import ops
    from tenzor_b200.shard import RankGather, shard_by_tokens
    import ctypes as C

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        # The gather of step i overlaps step i + 1's forward: NCCL gets at most NCCL_SMS CTAs and the
        # forward's persistent GEMM grids leave that many SMs free, so neither waits for the other's SMs.
        os.environ.setdefault("NCCL_MAX_CTAS", str(NCCL_SMS))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = Context(local)
    if world > 1:
        ctx.set_sm_reserve(NCCL_SMS)
    w = S.arctic_weights(1234)
    ck = quantize_checkpoint(ctx, w) if a.mode != "f32" else w
    model = ArcticModel.from_checkpoint(ctx, ck, a.mode, prec=a.prec)
    model.set_ffn_fusion(a.ffn == "fused")

    ids, lens, shards = make_inputs(a.config, world, a.batch)
    mine = shards[rank]
    l_ids, l_lens = ids[mine], lens[mine]
    packed, cu = S.pack(l_ids, l_lens)
    B, T, maxL = len(l_lens), int(cu[-1]), int(l_lens.max())
    model.reserve(B, T)
    d_ids = torch.from_numpy(packed.view(np.int32)).cuda()
    d_cu = torch.from_numpy(cu).cuda()
    gather = None
    if world > 1:
        gather = RankGather(mine, len(lens), 384, torch.device("cuda", local),
                            lambda table, ids, out: ops.gather_rows(ctx, table, ids, out=out))
    # two output buffers: step i's gather reads one while step i + 1's forward writes the other
    d_outs = [torch.zeros((gather.cap if gather else B, 384), device="cuda", dtype=torch.float32) for _ in range(2)]
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)  # > 126 MB L2
    # A dedicated stream: the forward, the L2 flush and the timing events all on it; with N > 1 the
    # gather of step i runs on a second stream, overlapping step i + 1's forward.
    stream = torch.cuda.Stream()
    gstream = torch.cuda.Stream() if gather else None
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0
    fdone = [torch.cuda.Event(), torch.cuda.Event()]  # forward of the buffer's step finished
    gdone = [torch.cuda.Event(), torch.cuda.Event()]  # gather of the buffer's step finished

    overlap = gather is not None and a.gather == "overlap"

    def step(i):
        buf = i % 2
        if overlap:
            stream.wait_event(gdone[buf])  # step i - 2's gather has read this buffer
        model.forward_device(d_ids.data_ptr(), d_cu.data_ptr(), B, T, maxL, d_outs[buf].data_ptr(), stream.cuda_stream)
        if overlap:
            fdone[buf].record(stream)
            with torch.cuda.stream(gstream):
                gstream.wait_event(fdone[buf])
                gather.step(d_outs[buf])
                gdone[buf].record(gstream)
        elif gather is not None:  # serial: the gather follows the forward on the same stream
            gather.step(d_outs[buf])

    def join(i):
        """Makes the main stream wait for step i's gather (every gather ends inside a timed step)."""
        if overlap and i >= 0:
            stream.wait_event(gdone[i % 2])

    # warm-up (also captures nothing: the device path launches directly)
    for i in range(max(a.warmup, 3)):
        step(i)
        join(i)
    torch.cuda.synchronize()

    def timed_loop(clk=None):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if clk:
            clk.begin()
        for i in range(a.steps):
            flush.zero_()
            evs[i][0].record(stream)
            step(i)
            join(i - 1)  # the previous step's gather ran under this forward; it closes in this window
            if i == a.steps - 1:
                join(i)
            evs[i][1].record(stream)
        if clk:
            clk.mark()
        torch.cuda.synchronize()
        if clk:
            clk.end()
        if world > 1:
            dist.barrier()
        per = [s_.elapsed_time(e_) for s_, e_ in evs]
        t = sum(per)
        if world > 1 and a.verbose_steps:
            print(f"rank {rank} step ms: " + " ".join(f"{x:.3f}" for x in per), file=sys.stderr, flush=True)
        t_t = torch.tensor([t], device="cuda")
        if world > 1:
            dist.all_reduce(t_t, op=dist.ReduceOp.MAX)
        return float(t_t.item())

    # 1) the headline: K steps, nothing but the forward (+ gather) on the stream
    with Clocks(local, poll=rank == 0 and a.clock_poll) as clk:
        ms = timed_loop(clk)
    # 2) the same K steps with CUDA events recorded between the forward's launches on the launching
    #    stream: per-kernel-class durations for the roofline
    L.check(L.lib().tz_arctic_profile(model.handle, a.steps))
    ms_prof = timed_loop()
    cls_ms = (C.c_float * 9)()
    cls_n = (C.c_int * 9)()
    L.check(L.lib().tz_arctic_profile_read(model.handle, cls_ms, cls_n))
    L.check(L.lib().tz_arctic_profile(model.handle, 0))
    nfwd = max(1, int(cls_n[0]))  # forwards recorded (one embedding launch each; 1 when replayed from a graph)
    launches_per_fwd = int(sum(cls_n)) // nfwd

    # end to end through the public host API (graph replay inside; H2D of ids + cu from pinned host
    # memory, as a serving pipeline stages them, and D2H of the embeddings into pinned host memory).
    # One GPU: tz_arctic_forward.  N GPUs: ShardedForward, whose call also gathers every rank's rows
    # to rank 0 and copies the whole batch back there; wall time per call, max over ranks.
    def pinned(arr):  # a page-locked copy (the torch tensor owns it) and its numpy view of arr's dtype
        t = torch.empty(arr.shape, dtype=torch.int32, pin_memory=True)
        v = t.numpy().view(arr.dtype)
        v[...] = arr
        return t, v
    keep_ids, h_ids = pinned(np.ascontiguousarray(packed, dtype=np.uint32))
    keep_cu, h_cu = pinned(np.ascontiguousarray(cu, dtype=np.int32))
    h_out_t = torch.empty((B, 384), dtype=torch.float32, pin_memory=True)
    host_out = h_out_t.numpy()
    if world > 1:
        from tenzor_b200.shard import ShardedForward
        sharded = ShardedForward(ctx, model, mine, len(lens), T, stream=stream)
        call = lambda: sharded.forward(h_ids, h_cu, maxL)
    else:
        call = lambda: model.forward_packed(h_ids, h_cu, out=host_out)
    for _ in range(3):
        call()
    e2e_t = 0.0
    for i in range(a.steps):
        flush.zero_()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        call()
        e2e_t += time.perf_counter() - t0
    e2e_t_t = torch.tensor([e2e_t], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t_t, op=dist.ReduceOp.MAX)
    e2e_t = float(e2e_t_t.item())

    total_seqs = len(lens) * a.steps if world > 1 else B * a.steps
    value = total_seqs / (ms / 1e3)
    e2e_value = total_seqs / e2e_t

    line = None
    if rank == 0:
        hbm, bf16, bf16_sus, src = peaks()
        # The roofline kernel: the FFN GEMM class that takes longer (FFN2 + residual + LayerNorm in
        # practice), tensor-bound by the path's own roofline (int8 dense peak for W8A8, f16 for the
        # f16-operand modes); its HBM side is reported beside it.  The class that takes the most time
        # overall is named too.
        per = [(cls_ms[c], c) for c in range(9) if cls_n[c] > 0]
        top_ms, top = max(per)
        dom_ms, dom = max((cls_ms[c], c) for c in (5, 6, 7) if cls_n[c] > 0)
        avg_ms = dom_ms / cls_n[dom]
        Tl = T
        int8 = a.mode == "w8a8"
        # (6: the fused FFN block's algorithmic FLOPs, FFN1 + FFN2; its second FFN1 pass is not counted)
        flops = {1: 2 * Tl * 384 * 1152, 3: 2 * Tl * 384 * 384, 5: 2 * Tl * 384 * 1536, 7: 2 * Tl * 1536 * 384,
                 6: 4 * Tl * 384 * 1536,
                 2: 4 * 384 * float((l_lens.astype(np.float64) ** 2).sum())}
        byts = class_bytes(dom, Tl, B, int8)
        t_hbm = byts / (hbm * 1e9)
        hbm_side = {"achieved": byts / (avg_ms / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                    "peak_source": f"{src} HBM copy", "bytes_per_launch": byts}
        hbm_side["frac"] = hbm_side["achieved"] / hbm
        sides = {"hbm": hbm_side}
        if dom in flops:
            if dom == 2:
                tpeak, tnote = bf16_sus, f"dense f16 = {src} bf16 sustained"
            elif int8:
                tpeak, tnote = measured_int8_peak(), "int8 dense, cuBLAS torch._int_mm 8192^3 measured in this run"
            else:
                tpeak, tnote = bf16_sus, f"f16 = {src} bf16 sustained"
            ach = flops[dom] / (avg_ms / 1e3) / 1e12
            sides["tensor"] = {"achieved": ach, "peak": tpeak, "unit": "TFLOP/s", "peak_source": tnote,
                               "flops_per_launch": flops[dom], "frac": ach / tpeak}
        bound = "tensor"
        sides["hbm"]["binding_at_measured_peaks"] = bool(t_hbm > flops[dom] / (sides["tensor"]["peak"] * 1e12))
        b_side = sides[bound]
        achieved, peak, unit, peak_note = b_side["achieved"], b_side["peak"], b_side["unit"], b_side["peak_source"]
        tr = traffic_table().get(f"{CLASS_NAMES[dom]}_{a.mode}_{a.config}")
        if tr:  # DRAM bytes ncu counted for one launch (cold cache), over the live launch time
            sides["hbm"]["ncu_dram_bytes_per_launch"] = tr
            sides["hbm"]["ncu_dram_frac"] = tr / (avg_ms / 1e3) / 1e9 / hbm
        dom_flops_or_bytes = flops.get(dom)
        cfg = CONFIGS[a.config]
        line = {
            "metric": arctic_metric(a.config, a.mode),
            "value": value, "unit": "seq/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms / a.steps, "higher_is_better": True,
            "scaling": "strong" if a.config == "c4" else "weak", "vs_baseline": None,
            "dtype": "int8 (W8A8, int32 acc)" if int8 else (f"{a.prec} operands / f32 acc" if a.mode == "f32"
                                                             else f"int8 weights as {a.prec} / f32 acc"),
            "data": "synthetic (seeded N(0,0.02) weights, U ids / lengths)",
            "config": {"workload": cfg["desc"] + (" per GPU" if world > 1 else "") +
                       (f" (batch overridden to {a.batch}: a profiling case, not the config)" if a.batch else ""),
                       "model": "Arctic-embed-xs",
                       "mode": a.mode, "ffn_block": (a.ffn if int8 else None), "global_batch": int(len(lens)), "per_gpu_batch": B, "tokens_per_gpu": T,
                       "seq_len": cfg["seq"], "parallelism": f"sequence-sharded x{world}, gather to rank 0",
                       "l2": "flushed (256 MB write) before every timed step",
                       "gather": ("N > 1: step i's NCCL gather to rank 0 runs on a second stream under step i + 1's "
                                  "forward and completes inside step i + 1's timed window (the last one inside the last)")
                                 if a.gather == "overlap" else
                                 "N > 1: each step's NCCL gather to rank 0 follows its forward on the same stream, inside its timed window",
                       "useful_gflop_per_step": flop_useful(lens) / 1e9},
            "roofline": {"kernel": CLASS_NAMES[dom], "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                         "frac": achieved / peak, "peak_source": peak_note, "traffic": tr,
                         "per_launch_work": dom_flops_or_bytes, "avg_launch_ms": avg_ms,
                         "limits": sides, "largest_class": CLASS_NAMES[top],
                         "class_ms_per_forward": {CLASS_NAMES[c]: round(cls_ms[c] / nfwd, 4) for c in range(9) if cls_n[c]},
                         "profiled_ms_per_step": ms_prof / a.steps},
            "e2e": {"value": e2e_value, "unit": "seq/s", "h2d_bytes_per_step": int(T * 4 + (B + 1) * 4),
                    "d2h_bytes_per_step": int(len(lens) * 384 * 4),
                    "api": "tz_arctic_forward" if world == 1 else "tenzor_b200.shard.ShardedForward (forward + NCCL gather to rank 0 + D2H of the whole batch on rank 0)"},
            "gpu_launches": launches_per_fwd * a.steps,
            "clocks": clk.summary(),
        }
        if world == 1 and not a.no_cpu:
            v, sample, thr = cpu_forward_timing(ck, ids, lens, "w8a32" if a.mode != "f32" else "f32", budget_s=12.0)
            line["cpu_baseline"] = {"value": v, "unit": "seq/s", "cores": thr, "kind": "port",
                                    "sample": sample + "; reference CPU algorithm (W8A32 int8 path) restated in C"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    model.close()
    ctx.close()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def run_micro(a):
    """the fused-op microbenchmarks, one JSON line each (not the headline metric).
    Inputs are seeded U[-1, 1]; each timed region is K launches with the L2 flushed before each."""
    import torch
    from tenzor_b200 import expr as E
    from tenzor_b200 import ops
    from tenzor_b200 import synthetic as S
    from tenzor_b200.runtime import Context
    ctx = Context(0)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    hbm, bf16, bf16_sus, src = peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)

    def timed(fn, flush_l2=True):
        # The K iterations (flush, start event, op, end event) are captured into one CUDA graph and
        # replayed, so the device runs them back to back and the host's per-call overhead (Python,
        # ctypes, tensor-map encoding) never lands between an op's two events.  flush_l2=False for
        # ops whose inputs rotate over more than L2 holds (126 MB): no flush write-backs then
        # compete with the op's own traffic.
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        # external=True: captured as event-record nodes, which keep their timestamps
        evs = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
               for _ in range(a.steps)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            if flush_l2:  # events around each launch, a flush before each
                for s_, e_ in evs:
                    flush.zero_()
                    s_.record()
                    fn()
                    e_.record()
            else:  # the K launches back to back between one pair of events
                evs[0][0].record()
                for _ in evs:
                    fn()
                evs[0][1].record()
        g.replay()
        torch.cuda.synchronize()
        if flush_l2:
            t = sum(s_.elapsed_time(e_) for s_, e_ in evs) / a.steps
        else:
            t = evs[0][0].elapsed_time(evs[0][1]) / a.steps
        del g
        return t

    def u(seed, shape):
        return torch.from_numpy(S.uniform(seed, shape, -1.0, 1.0)).cuda()

    lines = []
    # (a) [8192,384] x [384,1536] + bias + GELU (B not transposed), tf32 tensor cores
    A, B, bias = u(1, (8192, 384)), u(2, (384, 1536)), u(3, (1536,))
    e = E.matmul(A, B).add(bias).gelu()
    ms = timed(lambda: e.eval(ctx))
    fl = 2.0 * 8192 * 384 * 1536
    lines.append({"metric": "fused matmul+bias+GELU [8192,384]x[384,1536] TFLOP/s (f32 in, tf32 tensor cores)",
                  "value": fl / ms / 1e9, "unit": "TFLOP/s", "ms": ms, "plan": E.analyze(e),
                  "roofline": {"bound": "tensor", "peak": bf16_sus / 2, "frac": fl / ms / 1e9 / (bf16_sus / 2),
                               "peak_source": f"tf32 = half of {src} bf16 sustained (nominal ratio)"}})
    # (b) exp((a + b) * c), a, c [16384, 4096], b [4096]
    a_, b_, c_ = u(4, (16384, 4096)), u(5, (4096,)), u(6, (16384, 4096))
    e = E.tensor(a_).add(b_).mul(c_).exp()
    out = torch.empty_like(a_)
    ms = timed(lambda: ops.ew_add_mul_exp(ctx, a_, b_, c_, out=out), flush_l2=False)  # 768 MB touched per launch
    byts = 3 * 64 * 2 ** 20 * 4 + 4096 * 4
    lines.append({"metric": "elementwise chain a.add(b).mul(c).exp() 64M elems GB/s", "value": byts / ms / 1e6,
                  "unit": "GB/s", "ms": ms, "plan": E.analyze(e),
                  "roofline": {"bound": "hbm", "peak": hbm, "frac": byts / ms / 1e6 / hbm, "peak_source": f"{src} HBM copy"}})
    del a_, c_, out
    # (c) LayerNorm [32768, 384]; three input/output sets round-robin (300 MB > L2)
    g, bb = torch.ones(384, device="cuda"), torch.zeros(384, device="cuda")
    lx = [u(7 + i, (32768, 384)) for i in range(3)]
    ly = [torch.empty_like(t) for t in lx]
    lit = [0]

    def ln():
        i = lit[0] % 3
        lit[0] += 1
        ops.layer_norm_last_dim(ctx, lx[i], g, bb, 1e-5, out=ly[i])
    ms = timed(ln, flush_l2=False)
    byts = 2 * 32768 * 384 * 4 + 2 * 384 * 4
    lines.append({"metric": "LayerNorm [32768,384] GB/s", "value": byts / ms / 1e6, "unit": "GB/s", "ms": ms,
                  "roofline": {"bound": "hbm", "peak": hbm, "frac": byts / ms / 1e6 / hbm,
                               "peak_source": f"{src} HBM copy; 3 distinct 100 MB buffer sets round-robin"}})
    del lx, ly
    # (c) masked softmax [96, 128, 128], key lengths U{16..128}; 32 distinct buffers round-robin (> L2)
    nb = 32
    xs = [u(100 + i, (96, 128, 128)) for i in range(nb)]
    ys = [torch.empty_like(t) for t in xs]
    kl = torch.from_numpy(S.randint(9, 96, 16, 128).astype(np.int32)).cuda()
    it = [0]

    def sm():
        i = it[0] % nb
        it[0] += 1
        ops.softmax_keylen(ctx, xs[i], kl, out=ys[i])
    ms = timed(sm, flush_l2=False)
    byts = 2 * 96 * 128 * 128 * 4
    lines.append({"metric": "masked softmax [96,128,128] GB/s", "value": byts / ms / 1e6, "unit": "GB/s", "ms": ms,
                  "roofline": {"bound": "hbm", "peak": hbm, "frac": byts / ms / 1e6 / hbm,
                               "peak_source": f"{src} HBM copy; 32 distinct 6.3 MB buffers round-robin"}})
    for ln in lines:
        ln.update({"steps": a.steps, "warmup": a.warmup, "data": "synthetic U[-1,1]",
                   "config": {"workload": "configs[2]",
                              "l2": "flushed (256 MB write) before each launch" if "matmul" in ln["metric"]
                              else "inputs rotate over more than L2 (no flush)",
                              "timing": "K launches captured in one CUDA graph; CUDA events around each launch"
                              if "matmul" in ln["metric"] else
                              "K launches back to back in one CUDA graph between two CUDA events, divided by K"}})
        print(json.dumps(ln), flush=True)
    ctx.close()
    return 0


LENET_BATCH = 65536


def lenet_flop_per_image():
    return 2 * (6 * 28 * 28 * 25 + 16 * 10 * 10 * 150 + 400 * 120 + 120 * 84 + 84 * 10)


def lenet_cpu_timing(w, images, budget_s=12.0):
    """The C restatement of lenet.zig's forward on all host threads (images independent), on a
    bounded sample sized to ~budget_s.  Returns (img/s, sample, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = os.cpu_count() or 1
    probe = images[:2048]
    t0 = time.perf_counter()
    O.lenet_forward(w, O.LENET_PAD2, probe)
    dt = max(time.perf_counter() - t0, 1e-6)
    n = int(min(len(images), max(2048, 2048 * budget_s / dt)))
    t0 = time.perf_counter()
    O.lenet_forward(w, O.LENET_PAD2, images[:n])
    dt = time.perf_counter() - t0
    return n / dt, f"first {n} images of the 65536-image batch; C restatement of lenet.zig forward, OpenMP over images", threads


def run_lenet_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from tenzor_b200 import synthetic as S
    w = S.lenet_weights(4321, S.LENET_PAD2)
    x = S.lenet_images(LENET_BATCH, seed=11)
    vals = []
    budget = max(2.0, 150.0 / max(1, a.steps + a.warmup))
    for i in range(a.warmup + a.steps):
        v, sample, threads = lenet_cpu_timing(w, x, budget_s=budget)
        if i >= a.warmup:
            vals.append(v)
    v = float(np.median(vals))
    line = {"impl": "reference", "metric": "LeNet-5 img/s (f32, batch 65536)", "value": v, "unit": "img/s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": a.steps, "warmup": a.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (Kaiming-uniform weights, U[0,1] images)",
            "config": {"workload": "configs[4] LeNet-5 batch 65536 (pad-2 variant, softmax)", "global_batch": LENET_BATCH,
                       "parallelism": "host threads (one image per task)"},
            "cpu_baseline": {"value": v, "unit": "img/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": "img/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def run_lenet(a):
    import torch
    import torch.distributed as dist
    from tenzor_b200 import synthetic as S
    from tenzor_b200.lenet import LeNet
    from tenzor_b200.runtime import Context

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = Context(local)
    w = S.lenet_weights(4321, S.LENET_PAD2)
    x_all = S.lenet_images(LENET_BATCH, seed=11)
    per = LENET_BATCH // world
    x = x_all[rank * per:(rank + 1) * per]
    model = LeNet(ctx, w, S.LENET_PAD2)
    model.reserve(per)
    d_x = torch.from_numpy(x).cuda()
    d_o = torch.empty((per, 10), device="cuda")
    gathered = [torch.empty_like(d_o) for _ in range(world)] if (world > 1 and rank == 0) else None
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)

    def step():
        model.forward_device(d_x.data_ptr(), per, d_o.data_ptr(), stream.cuda_stream)
        if world > 1:
            dist.gather(d_o, gathered, dst=0)

    for _ in range(max(a.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    with Clocks(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clk.begin()
        for i in range(a.steps):
            flush.zero_()
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        clk.mark()
        torch.cuda.synchronize()
        clk.end()
    if world > 1:
        dist.barrier()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in evs)
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # e2e: host images (pinned, as a serving pipeline stages them) in, host probabilities out,
    # through the synchronous host API
    pinned = torch.empty((per, 28, 28, 1), dtype=torch.float32, pin_memory=True)
    pinned.numpy()[:] = x
    host = pinned.numpy()
    model.forward(host)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        model.forward(host)
    e2e_t = (time.perf_counter() - t0) / a.steps
    e2e = torch.tensor([e2e_t], device="cuda")
    if world > 1:
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
    e2e_t = float(e2e.item())
    if rank == 0:
        value = LENET_BATCH * a.steps / (ms / 1e3)
        clk_s = clk.summary()
        sm_mhz = clk_s.get("sm_mhz") or 1965.0
        fma_peak = ctx.sm_count * 128 * 2 * sm_mhz * 1e6 / 1e12  # f32 FMA lanes x 2 flop x clock
        achieved = lenet_flop_per_image() * per * a.steps / (ms / 1e3) / 1e12
        line = {"metric": "LeNet-5 img/s (f32, batch 65536)", "value": value, "unit": "img/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (Kaiming-uniform weights, U[0,1] images)",
                "config": {"workload": "configs[4] LeNet-5 batch 65536 (pad-2 variant, softmax)", "global_batch": LENET_BATCH,
                           "per_gpu_batch": per, "parallelism": f"image-sharded x{world}, gather to rank 0",
                           "l2": "flushed (256 MB write) before every timed step; inputs 205 MB > L2"},
                "roofline": {"kernel": "whole forward: lenet_conv (f32 FMA) + FC1 split-tf32 GEMM + lenet_fc_tail",
                             "bound": "fma", "achieved": achieved,
                             "peak": fma_peak, "unit": "TFLOP/s", "frac": achieved / fma_peak,
                             "peak_source": "f32 CUDA-core FMA: SMs x 128 lanes x 2 flop x median SM clock under load",
                             "traffic": None},
                "e2e": {"value": LENET_BATCH / e2e_t, "unit": "img/s", "h2d_bytes_per_step": int(per * 784 * 4),
                        "d2h_bytes_per_step": int(per * 10 * 4)},
                "gpu_launches": 3 * a.steps, "clocks": clk_s}
        if world == 1 and not a.no_cpu:
            v, sample, threads = lenet_cpu_timing(w, x_all)
            line["cpu_baseline"] = {"value": v, "unit": "img/s", "cores": threads, "kind": "port", "sample": sample}
        print(json.dumps(line))
    model.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="c2", choices=list(CONFIGS))
    ap.add_argument("--mode", default="w8a8", choices=["w8a8", "w8a32", "f32"])
    ap.add_argument("--prec", default="f16", choices=["f16", "bf16"],
                    help="16-bit GEMM operand type of the f32 / w8a32 modes")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--gather", default="overlap", choices=["overlap", "serial"],
                    help="N > 1: step i's gather runs under step i + 1's forward (overlap) or after step i's forward")
    ap.add_argument("--verbose-steps", action="store_true", help="N > 1: print each rank's per-step times to stderr")
    ap.add_argument("--no-clock-poll", dest="clock_poll", action="store_false",
                    help="no NVML polling thread (one clock sample inside the timed region only)")
    ap.add_argument("--ffn", default="split", choices=["fused", "split"],
                    help="W8A8 feed-forward block: the FFN1 + FFN2 kernel pair (default) or one kernel")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences per GPU instead of the config's (small cases for profiling; not a bench line)")
    ap.add_argument("--micro", action="store_true", help="configs[2] fused-op microbenchmarks (one line each)")
    ap.add_argument("--model", default="arctic", choices=["arctic", "lenet"])
    a = ap.parse_args()
    if a.warmup < 3:
        a.warmup = 3
    if a.model == "lenet":
        return run_lenet_reference(a) if a.impl == "reference" else run_lenet(a)
    if a.impl == "reference":
        return run_reference(a)
    if a.micro:
        return run_micro(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())

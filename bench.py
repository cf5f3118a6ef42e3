#!/usr/bin/env python
"""Decode-attention benchmark: prints ONE JSON line (rank 0).

Headline workload: KIVI-style 2-bit KV-cache decode at the metric's 32K context with the
config-1 head shapes: batch 8 per GPU, 28 query / 4 KV heads, head_dim 128, context 32768
of which the last 128 tokens are a bf16 residual window; keys quantised per channel over
groups of 32 tokens, values per token over groups of 32 channels (f16 scale / minimum).
Synthetic seeded inputs (N(0,1) bf16 with 4 of 128 key channels x8), packed once by the
engine's own packer before timing.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (batch-sharded, weak scaling)

value      device time per decode step (us, max over ranks): a CUDA graph of exactly K
           steps of the public API call, replayed once after a graph of exactly W warm-up
           steps (both graphs uploaded to the device before either runs); the steps rotate
           over 4 input sets (416 MB > 3x L2) so no step reads its inputs from L2.
e2e        the same K steps through the public Python API with host buffers: every step
           copies its queries host->device from pinned memory and reads the output back,
           the copies on their own streams so they overlap neighbouring steps' kernels
           (events order each step's upload -> decode -> read-back).
roofline   the packed-cache kernel alone (no residual window), algorithmic bytes per launch
           / its CUDA-event time, against MEASURED_PEAKS.json's copy bandwidth.
cpu_baseline / --impl reference: the reference's own CPU-runnable KIVI path
           (benchmarks/kivi_latency.py dequant_k + dequant_v + kivi_decode_attn_ref, from
           the installed reference in baseline/_ref), else the fp32 torch restatement of it
           in oracle/, on the host cores.
split_kv   (every N) one 1M-token bf16 sequence split across the N ranks: per-rank split-KV
           partial, the exchange of the (max, sum, numerator) partials and the log-sum-exp
           combine inside the timed step; at N > 1 the exchange is NVLink peer stores fused
           with the combine (one kernel), with the NCCL all-gather step timed beside it. The
           result is checked against single-GPU decode of the whole sequence before timing
           (parity_ok).
"""
import argparse
import hashlib
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "decode-attn µs/step & HBM GB/s (% of 8 TB/s) at 32K ctx; top-k select µs"
HEAD = dict(B=8, Hq=28, Hk=4, D=128, S=32768, R=128, bits=2, group=32)  # config-1 heads at 32K
CFG1 = dict(HEAD, S=16384)  # config 1 as stated (16K context)
NBUF = 4
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
TRAFFIC_FILE = os.path.join(ROOT, "profiles", "kivi_decode_kernel_32k.traffic.json")
KIVI_SOURCES = ("bytes_b200/csrc/kivi.cu", "bytes_b200/csrc/common.cuh")


def _workload(c):
    return (f"KIVI-{c['bits']} decode B={c['B']} Hq={c['Hq']} Hk={c['Hk']} D={c['D']} S={c['S']} R={c['R']} "
            f"group={c['group']}")


def _metric():
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            return json.load(f).get("metric", METRIC)
    except Exception:
        return METRIC


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _host_cores():
    """Cores this process may run on (its CPU affinity), for the host-side baselines."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _sources_sha():
    h = hashlib.sha256()
    for rel in KIVI_SOURCES:
        with open(os.path.join(ROOT, rel), "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _measured_traffic(workload):
    """DRAM bytes per launch of the packed-cache kernel from an ncu capture recorded for
    the current kernel sources and this workload; None when no such record exists (a
    record made for other sources is stale and not used)."""
    try:
        with open(TRAFFIC_FILE) as f:
            rec = json.load(f)
        if rec.get("source_sha256") == _sources_sha() and rec.get("workload") == workload:
            return int(rec["dram_bytes_per_launch"])
    except Exception:
        pass
    return None


# ----------------------------------------------------------------------------- inputs
def kivi_inputs(dev, seed, c=HEAD):
    from bytes_b200 import kivi as kv
    g = torch.Generator(device=dev).manual_seed(seed)
    B, Hq, Hk, D, S, R = c["B"], c["Hq"], c["Hk"], c["D"], c["S"], c["R"]
    Sq = S - R
    k = torch.randn(B, Hk, S, D, device=dev, generator=g)
    ch = torch.randperm(D, device=dev, generator=g)[:4]
    k[..., ch] *= 8
    k = k.bfloat16()
    v = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    q = torch.randn(B, Hq, 1, D, device=dev, generator=g).bfloat16()
    Kq, Ks, Km = kv.triton_quantize_and_pack_along_last_dim(k[:, :, :Sq].transpose(2, 3).contiguous().half(),
                                                            c["group"], c["bits"])
    Vq, Vs, Vm = kv.triton_quantize_and_pack_along_last_dim(v[:, :, :Sq].contiguous().half(), c["group"], c["bits"])
    Kr, Vr = k[:, :, Sq:].contiguous(), v[:, :, Sq:].contiguous()
    return q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr


def nbytes(*ts):
    return sum(t.numel() * t.element_size() for t in ts)


# ----------------------------------------------------------------------------- timing
def graph_of(calls):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for c in calls:
            c()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for c in calls:
            c()
    torch.cuda.synchronize()
    return g


def upload_graph(g):
    """Upload an instantiated graph to the device ahead of its first replay (otherwise the
    first replay pays the upload: measured +5 us per step on a 20-step KIVI graph). Setup,
    like instantiation: no step of the graph runs. A no-op when the runtime bindings or
    the graph's exec handle are unavailable."""
    try:
        try:
            from cuda.bindings import runtime as cr
        except ImportError:
            from cuda import cudart as cr
        cr.cudaGraphUpload(g.raw_cuda_graph_exec(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
    except Exception:
        pass


def time_graph(g, reps):
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e3  # µs


class ClockSampler:
    """Polls SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(index)
            self.max = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max = None
        self._stop = threading.Event()

    def _sample(self):
        nv = self.nv
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.005)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()
            if not self.samples:
                self._sample()  # a timed region shorter than one polling interval

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU side
def _reference_kivi():
    """The reference's own KIVI helpers (benchmarks/kivi_latency.py) from the installed
    reference, or None. Its module insists on a KIVI checkout at import; the engine's
    ``quant`` shim satisfies that (only the pure-torch helpers are called here)."""
    if not os.path.isdir(os.path.join(REF_DIR, "benchmarks")):
        return None
    os.environ.setdefault("KIVI_REPO", os.path.join(ROOT, "bytes_b200", "kivi_shim"))
    if REF_DIR not in sys.path:
        sys.path.append(REF_DIR)
    try:
        import importlib
        return importlib.import_module("benchmarks.kivi_latency")
    except Exception:
        return None


def cpu_step_fn(c):
    """(step(inputs, b, tok_frac), kind, what) for one sequence of the KIVI step on the host."""
    kl = _reference_kivi()
    fpi = 32 // c["bits"]

    def cut(inp, b, tok_frac):
        q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr = (t[b:b + 1] for t in inp)
        if tok_frac < 1.0:
            ng = max(1, int(Ks.shape[-1] * tok_frac))
            Kq, Ks, Km = Kq[..., :ng * 32 // fpi], Ks[..., :ng], Km[..., :ng]
            Vq, Vs, Vm = Vq[:, :, :ng * 32], Vs[:, :, :ng * 32], Vm[:, :, :ng * 32]
        return q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr

    if kl is not None:
        G = c["Hq"] // c["Hk"]

        def step(inp, b, tok_frac=1.0):
            q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr = cut(inp, b, tok_frac)
            Kd = kl.dequant_k(Kq, Ks, Km, c["group"], c["bits"]).to(torch.bfloat16)
            Vd = kl.dequant_v(Vq, Vs, Vm, c["group"], c["bits"]).to(torch.bfloat16)
            return kl.kivi_decode_attn_ref(q, Kd, Kr, Vd, Vr, G)
        return step, "reference", "benchmarks/kivi_latency.py dequant_k + dequant_v + kivi_decode_attn_ref"

    import oracle

    def step(inp, b, tok_frac=1.0):
        return oracle.kivi_decode_attn(*cut(inp, b, tok_frac), c["bits"], c["group"])
    return step, "port", "oracle.kivi_decode_attn (fp32 torch restatement)"


def cpu_inputs(c):
    """Inputs of the workload built on the host (same generator recipe as the GPU inputs)."""
    import oracle
    g = torch.Generator().manual_seed(1000)
    B, Hq, Hk, D, S, R = c["B"], c["Hq"], c["Hk"], c["D"], c["S"], c["R"]
    Sq = S - R
    k = torch.randn(B, Hk, S, D, generator=g)
    ch = torch.randperm(D, generator=g)[:4]
    k[..., ch] *= 8
    k = k.bfloat16()
    v = torch.randn(B, Hk, S, D, generator=g).bfloat16()
    q = torch.randn(B, Hq, 1, D, generator=g).bfloat16()
    Kq, Ks, Km = oracle.kivi_pack_last_dim(k[:, :, :Sq].transpose(2, 3).contiguous().half(), 32, c["bits"])
    Vq, Vs, Vm = oracle.kivi_pack_last_dim(v[:, :, :Sq].contiguous().half(), 32, c["bits"])
    return q, Kq, Ks, Km, k[:, :, Sq:].contiguous(), Vq, Vs, Vm, v[:, :, Sq:].contiguous()


def cpu_baseline(c, budget_s=10.0):
    """Time the host-side step on a bounded sample: single sequences, scaled to the full batch."""
    cores = _host_cores()
    torch.set_num_threads(cores)
    step, kind, what = cpu_step_fn(c)
    inp = cpu_inputs(c)
    t0 = time.perf_counter()
    step(inp, 0)
    one = time.perf_counter() - t0
    frac = min(1.0, budget_s / 2 / max(one, 1e-9))
    t0 = time.perf_counter()
    n = 0
    while n < 2 or (time.perf_counter() - t0 < budget_s / 2 and n < 20):
        step(inp, n % c["B"], frac)
        n += 1
    us = (time.perf_counter() - t0) / n * 1e6 * c["B"] / frac
    sample = f"{n} single-sequence steps of {what}" + (f" over the first {frac:.3f} of the packed tokens"
                                                       if frac < 1 else "") + f", scaled to the {c['B']}-sequence step"
    return {"value": round(us, 1), "unit": "us/step", "cores": cores, "kind": kind, "sample": sample}


def run_reference(args, rank):
    """--impl reference: the reference's CPU path for the workload, timed on host cores."""
    if rank != 0:
        return None
    c = HEAD
    cores = _host_cores()
    torch.set_num_threads(cores)
    step, kind, what = cpu_step_fn(c)
    inp = cpu_inputs(c)
    t0 = time.perf_counter()
    step(inp, 0)
    one_seq = time.perf_counter() - t0
    # size the per-step sample so the whole run stays within ~2 minutes
    frac = min(1.0, 110.0 / max(one_seq * (args.steps + args.warmup), 1e-9))
    for i in range(args.warmup):
        step(inp, i % c["B"], frac)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(inp, i % c["B"], frac)
    dt = (time.perf_counter() - t0) / args.steps
    us = dt * 1e6 * c["B"] / frac  # one sequence (and a token fraction) per step, scaled to the full step
    sample = (f"{what}: one of {c['B']} sequences per step"
              + (f", first {frac:.3f} of the packed tokens" if frac < 1 else "") + ", time scaled to the full step")
    return {
        "impl": "reference", "metric": _metric(), "value": round(us, 1), "unit": "us/step", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if kind == "port" else "bf16", "data": "synthetic",
        "config": {"workload": _workload(c), "global_batch": c["B"], "seq_len": c["S"], "parallelism": "host cores"},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ----------------------------------------------------------------------------- extras
def _rot(make, n):
    return [make() for _ in range(n)]


def _line(us, b, peak):
    return {"us": round(us, 2), "GBps": round(b / us / 1e3, 1), "frac": round(b / us / 1e3 / peak, 3)}


def path_c1(dev, peak, g):
    """Config 1 as stated: KIVI-2 decode at 16K context (B=8, 28/4), whole step and the
    packed-cache kernel alone."""
    from bytes_b200 import kivi as kv, _ops
    c = CFG1
    sets = [kivi_inputs(dev, 2000 + i, c) for i in range(8)]
    gr = graph_of([lambda s=s: kv.kivi_decode_attn(*s, c["bits"], c["group"]) for s in sets])
    time_graph(gr, 2)
    us = time_graph(gr, 20) / (20 * len(sets))
    scal = 1.0 / math.sqrt(c["D"])
    outs = [torch.empty(c["B"], c["Hq"], c["D"], dtype=torch.bfloat16, device=dev) for _ in sets]
    gk = graph_of([lambda s=s, o=o: _ops.kivi_decode(s[0][:, :, 0, :], *s[1:], c["bits"], c["group"], scal, o,
                                                     stages=1) for s, o in zip(sets, outs)])
    time_graph(gk, 2)
    us_k = time_graph(gk, 20) / (20 * len(sets))
    kb = nbytes(*(sets[0][i] for i in (1, 2, 3, 5, 6, 7)))
    out = {"c1_kivi2_16k_B8": dict(_line(us, nbytes(*sets[0][1:]), peak), kernel=_line(us_k, kb, peak))}
    return out


def path_c0(dev, peak, g):
    """c0: bf16 dense decode, B=1, 28/4 heads, S=8192, q pre-scaled by 1/sqrt(D)."""
    from bytes_b200 import attention_kernels as ak
    D = 128
    sets = _rot(lambda: ((torch.randn(1, 28, 1, D, device=dev, generator=g) / math.sqrt(D)).bfloat16(),
                         torch.randn(1, 4, 8192, D, device=dev, generator=g).bfloat16(),
                         torch.randn(1, 4, 8192, D, device=dev, generator=g).bfloat16()), 16)
    gr = graph_of([lambda s=s: ak.decode_attn_bf16(*s) for s in sets])
    us = time_graph(gr, 20) / (20 * len(sets))
    return {"c0_bf16_decode": _line(us, nbytes(*sets[0][1:]), peak)}


def path_bf16_32k(dev, peak, g):
    """bf16 and fp8 dense decode at 32K context with the c1 head shapes (B=8, 28/4)."""
    from bytes_b200 import attention_kernels as ak
    D = 128
    sets = _rot(lambda: (torch.randn(8, 28, 1, D, device=dev, generator=g).bfloat16(),
                         torch.randn(8, 4, 32768, D, device=dev, generator=g).bfloat16(),
                         torch.randn(8, 4, 32768, D, device=dev, generator=g).bfloat16()), 2)
    gr = graph_of([lambda s=s: ak.decode_attn_bf16(*s) for s in sets])
    us = time_graph(gr, 10) / (10 * len(sets))
    out = {"bf16_decode_32k_B8": _line(us, nbytes(*sets[0][1:]), peak)}
    sets8 = [(q, k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)) for q, k, v in sets]
    del sets
    gr = graph_of([lambda s=s: ak.decode_attn_fp8(*s) for s in sets8])
    us = time_graph(gr, 10) / (10 * len(sets8))
    out["fp8_decode_32k_B8"] = _line(us, nbytes(*sets8[0][1:]), peak)
    return out


def path_c2(dev, peak, g):
    """c2: PQ-LUT keys (16 x 8-dim subspaces, 256 centroids) + int8 V with f16 per-token scale."""
    from bytes_b200 import attention_kernels as ak
    B, Hq, Hk, S, M, K, D = 4, 32, 8, 32768, 16, 256, 128

    def mk2():
        lut = torch.randn(B, Hq, M, K, device=dev, generator=g) * 0.3
        codes = torch.randint(0, 256, (B, Hk, S, M), device=dev, generator=g, dtype=torch.int32).to(torch.uint8)
        v8 = torch.randint(-127, 128, (B, Hk, S, D), device=dev, generator=g, dtype=torch.int32).to(torch.int8)
        vs = (torch.rand(B, Hk, S, device=dev, generator=g) * 0.02).half()
        return lut, codes, v8, vs
    sets = _rot(mk2, 3)
    gr = graph_of([lambda s=s: ak.decode_attn_pq_lut_int8v(*s) for s in sets])
    us = time_graph(gr, 10) / (10 * len(sets))
    b = nbytes(*sets[0]) + M * K * 8 * 2 * Hk  # + per-head fp16 codebooks of the configuration
    return {"c2_pq_lut_int8v": _line(us, b, peak)}


def path_c3(dev, peak, g):
    """c3: Quest top-64 pages + gather, exact token top-k k=1024 (B=16, 32/8, S=32768), top-k alone."""
    from bytes_b200 import attention_kernels as ak, sparse_attention as sa, _ops
    out = {}
    B, Hq, Hk, S, kb, page, D = 16, 32, 8, 32768, 1024, 16, 128
    q = torch.randn(B, Hq, 1, D, device=dev, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    kmin, kmax = sa.quest_page_metadata(k, page)
    sc = 1 / math.sqrt(D)

    def quest_step():
        idx = sa.quest_select_decode(q, kmin, kmax, S, kb, page, sc)
        return ak.sparse_gather_attn(q, k, v, idx, sc)

    gr = graph_of([quest_step])
    us = time_graph(gr, 20) / 20
    meta = nbytes(kmin, kmax)
    gathered = B * Hq * kb * D * 2 * 2
    out["c3_quest_select_gather"] = {"us": round(us, 2), "metadata_MB": round(meta / 1e6, 1),
                                     "gathered_MB": round(gathered / 1e6, 1),
                                     "GBps": round((meta + gathered) / us / 1e3, 1),
                                     "frac": round((meta + gathered) / us / 1e3 / peak, 3)}

    def exact_step():
        s_ = ak.sparse_score_scalar(q, k, sc, score_bits=16)
        _, idx = _ops.topk(s_, kb, sorted=False, want_values=False, idx_dtype=torch.int32)
        return ak.sparse_gather_attn(q, k, v, idx, sc)

    gr = graph_of([exact_step])
    us = time_graph(gr, 10) / 10
    kscan = nbytes(k)
    nscore = B * Hq * S
    out["c3_exact_topk_decode"] = {"us": round(us, 2), "bytes_MB": round((kscan + 2 * nscore * 4 + gathered) / 1e6, 1),
                                   "frac": round((kscan + 2 * nscore * 4 + gathered) / us / 1e3 / peak, 3)}
    s_ = ak.sparse_score_scalar(q, k, sc, score_bits=16)
    gr = graph_of([lambda: _ops.topk(s_, kb, sorted=False, want_values=False, idx_dtype=torch.int32)])
    us_tk = time_graph(gr, 20) / 20
    gr2 = graph_of([lambda: s_.topk(kb, dim=-1)])
    us_torch = time_graph(gr2, 20) / 20
    out["topk_select"] = {"rows": B * Hq, "n": S, "k": kb, "us": round(us_tk, 2), "torch_topk_us": round(us_torch, 2)}
    return out


def path_sparse_published(dev, peak, g):
    """The reference's published sparse configurations on config 3's tensors (B=16, 32/8,
    S=32768): two-pass sparse decode at k = 5 % with fp8, int4 and int2 score keys
    (tables/profiling_latency.tex of the reference), each with its score / top-k / gather
    split and the score pass's roofline fraction."""
    from bytes_b200 import attention_kernels as ak, _ops
    B, Hq, Hk, S, D = 16, 32, 8, 32768, 128
    sc = 1 / math.sqrt(D)
    q = torch.randn(B, Hq, 1, D, device=dev, generator=g).bfloat16()
    k = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    v = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    kb = max(1, int(round(0.05 * S)))
    out = {}
    for bits in (8, 4, 2):
        if bits == 8:
            ks, s_, z_ = k.to(torch.float8_e4m3fn), None, None
            score = lambda: ak.sparse_score_scalar(q, ks, sc, score_bits=8)
            sbytes = nbytes(ks)
        else:
            ks, s_, z_ = ak.quantize_and_pack_score_keys(k, bits, 32)
            score = lambda: ak.sparse_score_packed(q, ks, s_, z_, sc, score_bits=bits, group_size=32)
            sbytes = nbytes(ks, s_, z_)
        full = lambda: ak.sparse_decode_scalar(q, ks, s_, z_, k, v, 0.05, sc, score_bits=bits, group_size=32)
        gr = graph_of([full])
        us_full = time_graph(gr, 10) / 10
        gr = graph_of([score])
        us_s = time_graph(gr, 10) / 10
        scores = score()
        gr = graph_of([lambda: _ops.topk(scores, kb, sorted=False, want_values=False, idx_dtype=torch.int32)])
        us_t = time_graph(gr, 10) / 10
        _, idx = _ops.topk(scores, kb, sorted=False, want_values=False, idx_dtype=torch.int32)
        gr = graph_of([lambda: ak.sparse_gather_attn(q, k, v, idx, sc)])
        us_g = time_graph(gr, 10) / 10
        name = {8: "fp8", 4: "int4", 2: "int2"}[bits]
        out[f"sparse_{name}_score_k5pct"] = {
            "us": round(us_full, 2), "kb": kb, "score_us": round(us_s, 2), "topk_us": round(us_t, 2),
            "gather_us": round(us_g, 2), "score_bytes_MB": round((sbytes + B * Hq * S * 4) / 1e6, 1),
            "score_frac": round((sbytes + B * Hq * S * 4) / us_s / 1e3 / peak, 3)}
        del gr, scores, idx
    return out


def path_topk(dev, peak, g):
    """Top-k select alone: 512 rows x 32768 fp32 scores (c3's B*Hq rows), k = 1024, vs torch.topk."""
    from bytes_b200 import _ops
    rows, n, kb = 16 * 32, 32768, 1024
    s_ = torch.randn(rows, n, device=dev, generator=g)
    gr = graph_of([lambda: _ops.topk(s_, kb, sorted=False, want_values=False, idx_dtype=torch.int32)])
    us_tk = time_graph(gr, 20) / 20
    gr2 = graph_of([lambda: s_.topk(kb, dim=-1)])
    us_torch = time_graph(gr2, 20) / 20
    return {"topk_alone": {"rows": rows, "n": n, "k": kb, "us": round(us_tk, 2), "torch_topk_us": round(us_torch, 2),
                           "GBps": round(rows * n * 4 / us_tk / 1e3, 1)}}


def c4_batch_shard(dev, peak, g):
    """c4, one GPU's batch shard: 8 sequences x 131072 tokens with the c1 head shapes
    (28/4, D=128) as bf16 and as KIVI-2."""
    from bytes_b200 import attention_kernels as ak, kivi as kv
    out = {}
    D, S = 128, 131072
    q = torch.randn(8, 28, 1, D, device=dev, generator=g).bfloat16()
    k = torch.randn(8, 4, S, D, device=dev, generator=g).bfloat16()
    v = torch.randn(8, 4, S, D, device=dev, generator=g).bfloat16()
    gr = graph_of([lambda: ak.decode_attn_bf16(q, k, v)])
    time_graph(gr, 2)
    us = time_graph(gr, 10) / 10
    out["c4_bf16_131k_B8"] = _line(us, nbytes(k, v), peak)
    del k, v, gr
    torch.cuda.empty_cache()
    c = dict(HEAD, S=S)
    s = kivi_inputs(dev, 4242, c)
    gr = graph_of([lambda: kv.kivi_decode_attn(*s, c["bits"], c["group"])])
    time_graph(gr, 2)
    us = time_graph(gr, 10) / 10
    out["c4_kivi2_131k_B8"] = dict(_line(us, nbytes(*s[1:]), peak), MB=round(nbytes(*s[1:]) / 1e6, 1))
    return out


def path_c4(dev, peak, g):
    return c4_batch_shard(dev, peak, g)


def path_ref_gpu(dev, peak, g):
    """The reference's own Triton kernels (the installed reference in baseline/_ref,
    unmodified) on this GPU beside this engine's kernels, on the same inputs: dense bf16 /
    fp8 decode at 32K (B=8, 28/4) and c0, the fp8 / int4 / int2 score passes and the gather
    at config 3's shape (B=16, 32/8, S=32768, k = 5 %), PQ-LUT decode with bf16 values at
    config 2's shape, and the two-pass sparse decode (fp8 / int2 scores, k = 5 %) as whole
    chains. Each op is CUDA-graph replayed after a warm-up call (the reference's own harness
    times ops the same way); `max_abs_diff` compares the two outputs."""
    if not os.path.isdir(os.path.join(REF_DIR, "src")):
        return {"ref_gpu": {"unavailable": "the reference is not installed in baseline/_ref"}}
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import src.attention_kernels as ref
    from bytes_b200 import attention_kernels as ak

    def timed(fn, reps=10):
        fn()
        torch.cuda.synchronize()
        gr = graph_of([fn])
        time_graph(gr, 2)
        return round(time_graph(gr, reps) / reps, 2)

    def both(name, f_ref, f_ours):
        a, b = f_ref(), f_ours()
        torch.cuda.synchronize()
        d = (a.float() - b.float()).abs().max().item()
        out[name] = {"ref_us": timed(f_ref), "ours_us": timed(f_ours), "max_abs_diff": d}
        out[name]["speedup"] = round(out[name]["ref_us"] / out[name]["ours_us"], 2)

    out = {}
    D = 128
    q = torch.randn(8, 28, 1, D, device=dev, generator=g).bfloat16()
    k = torch.randn(8, 4, 32768, D, device=dev, generator=g).bfloat16()
    v = torch.randn(8, 4, 32768, D, device=dev, generator=g).bfloat16()
    qs = (q.float() / math.sqrt(D)).bfloat16()
    both("bf16_decode_32k_B8", lambda: ref.decode_attn_bf16(qs, k, v), lambda: ak.decode_attn_bf16(qs, k, v))
    k8, v8 = k.to(torch.float8_e4m3fn), v.to(torch.float8_e4m3fn)
    both("fp8_decode_32k_B8", lambda: ref.decode_attn_fp8(qs, k8, v8), lambda: ak.decode_attn_fp8(qs, k8, v8))
    del k, v, k8, v8
    q0 = (torch.randn(1, 28, 1, D, device=dev, generator=g) / math.sqrt(D)).bfloat16()
    k0 = torch.randn(1, 4, 8192, D, device=dev, generator=g).bfloat16()
    v0 = torch.randn(1, 4, 8192, D, device=dev, generator=g).bfloat16()
    both("c0_bf16_decode", lambda: ref.decode_attn_bf16(q0, k0, v0), lambda: ak.decode_attn_bf16(q0, k0, v0))
    torch.cuda.empty_cache()
    B, Hq, Hk, S = 16, 32, 8, 32768
    sc = 1 / math.sqrt(D)
    q3 = torch.randn(B, Hq, 1, D, device=dev, generator=g).bfloat16()
    k3 = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    v3 = torch.randn(B, Hk, S, D, device=dev, generator=g).bfloat16()
    k38 = k3.to(torch.float8_e4m3fn)
    both("c3_score_fp8", lambda: ref.sparse_score_scalar(q3, k38, sc, score_bits=8),
         lambda: ak.sparse_score_scalar(q3, k38, sc, score_bits=8))
    del k38
    for bits in (4, 2):
        kp, s_, z_ = ak.quantize_and_pack_score_keys(k3, bits, 32)
        both(f"c3_score_int{bits}", lambda: ref.sparse_score_packed(q3, kp, s_, z_, sc, score_bits=bits, group_size=32),
             lambda: ak.sparse_score_packed(q3, kp, s_, z_, sc, score_bits=bits, group_size=32))
        del kp, s_, z_
    # the two-pass sparse decode at k = 5 % (scores -> top-k -> gather), whole chain
    k38 = k3.to(torch.float8_e4m3fn)
    both("c3_sparse_decode_fp8_k5pct",
         lambda: ref.sparse_decode_scalar(q3, k38, None, None, k3, v3, 0.05, sc, score_bits=8),
         lambda: ak.sparse_decode_scalar(q3, k38, None, None, k3, v3, 0.05, sc, score_bits=8))
    del k38
    kp, s_, z_ = ak.quantize_and_pack_score_keys(k3, 2, 32)
    both("c3_sparse_decode_int2_k5pct",
         lambda: ref.sparse_decode_scalar(q3, kp, s_, z_, k3, v3, 0.05, sc, score_bits=2, group_size=32),
         lambda: ak.sparse_decode_scalar(q3, kp, s_, z_, k3, v3, 0.05, sc, score_bits=2, group_size=32))
    del kp, s_, z_
    kb = max(1, int(round(0.05 * S)))
    scores = ak.sparse_score_scalar(q3, k3, sc, score_bits=16)
    _, idx = ak.topk(scores, kb, sorted=False)
    del scores
    both("c3_gather_k5pct", lambda: ref.sparse_gather_attn(q3, k3, v3, idx, sc),
         lambda: ak.sparse_gather_attn(q3, k3, v3, idx, sc))
    del q3, k3, v3, idx
    torch.cuda.empty_cache()
    lut = torch.randn(4, 32, 16, 256, device=dev, generator=g) * 0.3
    codes = torch.randint(0, 256, (4, 8, 32768, 16), device=dev, generator=g, dtype=torch.int32).to(torch.uint8)
    vp = torch.randn(4, 8, 32768, D, device=dev, generator=g).bfloat16()
    both("c2_pq_lut_bf16v", lambda: ref.decode_attn_pq_lut(lut, codes, vp), lambda: ak.decode_attn_pq_lut(lut, codes, vp))
    return {"ref_gpu": out}


PATHS = {"c0": path_c0, "c1": path_c1, "bf16_32k": path_bf16_32k, "c2": path_c2, "c3": path_c3,
         "sparse_published": path_sparse_published, "topk": path_topk, "c4": path_c4, "ref_gpu": path_ref_gpu}
OPT_IN = {"ref_gpu"}  # run only when asked for by --path (it JIT-compiles the reference's Triton kernels)


def extras(dev, peak, only=None):
    """Other decode paths at their configuration shapes (rank 0, single GPU)."""
    import gc
    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    for name, fn in PATHS.items():
        if (only is not None and name != only) or (only is None and name in OPT_IN):
            continue
        out.update(fn(dev, peak, g))
        gc.collect()
        torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------- split-KV
SPLIT_TOKENS = 1 << 20  # config 4's long sequence


def _split_shard(dev, i, n, Hk, D):
    """Tokens [i*S/n, (i+1)*S/n) of the long sequence (a seed per shard: any rank can rebuild any shard)."""
    g = torch.Generator(device=dev).manual_seed(90000 + 131 * n + i)
    L = SPLIT_TOKENS // n
    return (torch.randn(1, Hk, L, D, device=dev, generator=g).bfloat16(),
            torch.randn(1, Hk, L, D, device=dev, generator=g).bfloat16())


def split_kv_bench(dev, rank, world, dist, steps, warmup, peak):
    """One 1M-token bf16 sequence (28/4 heads, D=128) split along its tokens across the ranks.

    Step = this rank's split-KV partial over its shard, then the exchange of the (max, sum,
    numerator) partials and their log-sum-exp combine. Two exchanges are timed: the split
    pass followed by one kernel that merges the splits, stores the merged partials into every
    rank's buffer over NVLink and combines (bytes_b200.distributed.PeerExchange.decode; one
    CUDA graph per step), and NCCL's all-gather between the partial and combine graphs.
    Before timing, every rank checks each combined output against single-GPU decode of the
    whole sequence; the ranks agree on the verdict through an all-reduce."""
    from bytes_b200 import _ops, attention_kernels as ak
    Hq, Hk, D = 28, 4, 128
    scal = 1.0 / math.sqrt(D)
    g = torch.Generator(device=dev).manual_seed(424242)
    q3 = torch.randn(1, Hq, D, device=dev, generator=g).bfloat16()
    k_sh, v_sh = _split_shard(dev, rank, world, Hk, D)
    n_ml = Hq
    width = 2 * n_ml + Hq * D
    send = torch.empty(width, dtype=torch.float32, device=dev)
    recv = torch.empty(world, width, dtype=torch.float32, device=dev)
    out = torch.empty(1, Hq, D, dtype=torch.bfloat16, device=dev)

    def partial():
        m, l, o = _ops.decode_attn_partial(q3, k_sh, v_sh, scal)
        send[:n_ml].copy_(m.view(-1))
        send[n_ml:2 * n_ml].copy_(l.view(-1))
        send[2 * n_ml:].copy_(o.view(-1))

    def exchange():
        if dist is not None:
            dist.all_gather_into_tensor(recv, send)
        else:
            recv[0].copy_(send)

    def combine():
        out.copy_(_ops.lse_combine(recv[:, :n_ml].reshape(world, 1, Hq), recv[:, n_ml:2 * n_ml].reshape(world, 1, Hq),
                                   recv[:, 2 * n_ml:].reshape(world, 1, Hq, D), torch.bfloat16))

    g_part, g_comb = graph_of([partial]), graph_of([combine])

    def step():
        g_part.replay()
        exchange()
        g_comb.replay()

    # the peer exchange (N > 1 with symmetric memory): partial + exchange + combine, one graph
    peer, peer_note = None, None
    if dist is not None:
        ok = 1.0
        try:
            from bytes_b200.distributed import PeerExchange
            peer = PeerExchange(1, Hq, D, dev)
        except Exception as e:  # symmetric memory unavailable: NCCL only
            peer_note = f"{type(e).__name__}: {e}"[:160]
            ok = 0.0
        t = torch.tensor([ok], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        if t.item() < 1.0:
            peer = None
    out_peer = torch.empty(1, Hq, D, dtype=torch.bfloat16, device=dev)

    def peer_step():
        out_peer.copy_(peer.decode(q3, k_sh, v_sh, scal, torch.bfloat16))

    g_peer = graph_of([peer_step]) if peer is not None else None
    if peer is not None:  # the exchange kernel alone, on fixed partials
        part_fixed = _ops.decode_attn_partial(q3, k_sh, v_sh, scal)
        g_ex = graph_of([lambda: peer(*part_fixed, torch.bfloat16)])

    # parity: the split result against single-GPU decode of the whole sequence
    step()
    if g_peer is not None:
        g_peer.replay()
    torch.cuda.synchronize()
    parts = [_split_shard(dev, i, world, Hk, D) for i in range(world)]
    k_full = torch.cat([p[0] for p in parts], 2)
    v_full = torch.cat([p[1] for p in parts], 2)
    del parts
    ref = ak.decode_attn_bf16((q3.float() * scal).bfloat16().unsqueeze(2), k_full, v_full)[:, :, 0]
    # the reference call takes a pre-scaled bf16 query; compare both against fp32 math too
    ref32 = torch.softmax((k_full[0].float() @ (q3[0].float().view(Hk, Hq // Hk, D).transpose(1, 2)) * scal)
                          .transpose(1, 2), -1) @ v_full[0].float()
    del k_full, v_full
    def agrees(x):
        d = (x[0].float() - ref32.reshape(Hq, D)).abs()
        d2 = (x.float() - ref.float()).abs()
        return bool(torch.isfinite(x.float()).all().item() and d.max().item() <= 2e-2 and d.mean().item() <= 1e-3
                    and d2.max().item() <= 2e-2)

    ok = agrees(out) and (g_peer is None or agrees(out_peer))
    flag = torch.tensor([1.0 if ok else 0.0], device=dev)
    if dist is not None:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    parity_ok = bool(flag.item() == 1.0)
    torch.cuda.empty_cache()

    for _ in range(max(warmup, 3)):
        step()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(steps):
        step()
    e1.record(st)
    e1.synchronize()
    us_step = e0.elapsed_time(e1) * 1e3 / steps
    # the all-gather alone, same loop length
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(steps):
        exchange()
    e1.record(st)
    e1.synchronize()
    us_ag = e0.elapsed_time(e1) * 1e3 / steps
    # the peer-exchange step, and the partial alone (to attribute the exchange's share)
    us_peer = us_part = us_ex = 0.0
    if g_peer is not None:
        for gr in (g_peer, g_ex):
            for _ in range(max(warmup, 3)):
                gr.replay()
            dist.barrier()
            torch.cuda.synchronize()
            e0.record(st)
            for _ in range(steps):
                gr.replay()
            e1.record(st)
            e1.synchronize()
            if gr is g_peer:
                us_peer = e0.elapsed_time(e1) * 1e3 / steps
            else:
                us_ex = e0.elapsed_time(e1) * 1e3 / steps
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(steps):
        g_part.replay()
    e1.record(st)
    e1.synchronize()
    us_part = e0.elapsed_time(e1) * 1e3 / steps
    t = torch.tensor([us_step, us_ag, us_peer, us_part, us_ex], device=dev)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us_nccl, us_ag, us_peer, us_part, us_ex = (float(x) for x in t.tolist())
    us_best = us_peer if g_peer is not None else us_nccl
    shard_bytes = nbytes(k_sh, v_sh)
    used_peer = g_peer is not None
    del g_part, g_comb, g_peer
    if used_peer:
        del g_ex
    line = {"tokens": SPLIT_TOKENS, "ranks": world, "shard_tokens": SPLIT_TOKENS // world, "us": round(us_best, 2),
            "exchange": "split merge + nvlink peer stores + combine, one kernel behind the split pass"
                        if used_peer else ("nccl all-gather" if dist is not None else "none (one rank)"),
            "partial_us": round(us_part, 2), "exchange_share": round(max(0.0, us_best - us_part) / us_best, 3),
            "peer_exchange_alone_us": round(us_ex, 2) if used_peer else None,
            "nccl_step_us": round(us_nccl, 2), "nccl_allgather_us": round(us_ag, 2),
            "exchange_bytes_per_rank": width * 4 * max(1, world - 1), "tokens_per_s": round(1e6 / us_best, 1),
            "shard_GBps": round(shard_bytes / us_best / 1e3, 1),
            "shard_frac": round(shard_bytes / us_best / 1e3 / peak, 3), "parity_ok": parity_ok,
            "steps": steps, "timing": "CUDA graphs (the NCCL all-gather eager between two), CUDA events, "
                                      "max over ranks"}
    if peer_note:
        line["peer_exchange_unavailable"] = peer_note
    if peer is not None:
        peer.buf = None
    return line


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--path", choices=sorted(PATHS), help="time only this secondary path and print its numbers")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.steps < 1:
        raise SystemExit("--steps must be at least 1")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # host-core work on rank 0 only; the other ranks exit at once (no process group, so
        # nothing spins on a core the CPU sample needs)
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    from bytes_b200 import kivi as kv
    from bytes_b200 import _ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak, peak_kind = _peaks()
    if args.path:
        print(json.dumps(extras(dev, peak, only=args.path)), flush=True)
        return
    c = HEAD
    sets = [kivi_inputs(dev, 1000 + rank * NBUF + i) for i in range(NBUF)]
    step_bytes = nbytes(*sets[0][1:])
    kern_bytes = nbytes(*(sets[0][i] for i in (1, 2, 3, 5, 6, 7)))
    scal = 1.0 / math.sqrt(c["D"])

    # device-time value: a graph of exactly `steps` decode steps (after one of `warmup`),
    # rotating over the NBUF input sets
    def step_call(i):
        s = sets[i % NBUF]
        return lambda: kv.kivi_decode_attn(*s, c["bits"], c["group"])

    g_warm = graph_of([step_call(i) for i in range(args.warmup)])
    g_step = graph_of([step_call(i) for i in range(args.steps)])
    upload_graph(g_warm)
    upload_graph(g_step)
    g_warm.replay()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        us_total = time_graph(g_step, 1)
    torch.cuda.synchronize()
    us_step = us_total / args.steps
    if dist is not None:
        t = torch.tensor([us_step], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us_step = float(t.item())
    del g_warm, g_step

    # roofline: the packed-cache kernel alone
    outs = [torch.empty(c["B"], c["Hq"], c["D"], dtype=torch.bfloat16, device=dev) for _ in sets]
    kcalls = [lambda s=s, o=o: _ops.kivi_decode(s[0][:, :, 0, :], *s[1:], c["bits"], c["group"], scal, o, stages=1)
              for s, o in zip(sets, outs)]
    g_k = graph_of(kcalls)
    time_graph(g_k, 3)
    reps_k = max(5, min(200, args.steps // NBUF))
    us_kern = time_graph(g_k, reps_k) / (reps_k * NBUF)
    achieved = kern_bytes / us_kern / 1e3  # GB/s
    del g_k

    # e2e through the public API with host buffers, exactly `steps` steps after `warmup`
    q_host = [s[0].cpu().pin_memory() for s in sets]
    out_host = [torch.empty(c["B"], c["Hq"], 1, c["D"], dtype=torch.bfloat16).pin_memory() for _ in sets]
    q_dev = [torch.empty_like(s[0]) for s in sets]
    st = torch.cuda.current_stream()
    # a serving loop's overlap: the copies run on their own streams, so step i's query upload
    # and step i-1's output read-back proceed while decode kernels run; per input slot j,
    # events order upload -> decode -> read-back and keep a slot's buffers from being reused
    # before its read-back is done
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_up = [torch.cuda.Event() for _ in sets]
    ev_dec = [torch.cuda.Event() for _ in sets]
    ev_down = [torch.cuda.Event() for _ in sets]
    for e in ev_down:
        e.record(st)

    def e2e_step(i):
        j = i % NBUF
        with torch.cuda.stream(up):
            up.wait_event(ev_down[j])
            q_dev[j].copy_(q_host[j], non_blocking=True)
            ev_up[j].record(up)
        st.wait_event(ev_up[j])
        o = kv.kivi_decode_attn(q_dev[j], *sets[j][1:], c["bits"], c["group"])
        o.record_stream(down)  # the allocator keeps it until its read-back is done
        ev_dec[j].record(st)
        with torch.cuda.stream(down):
            down.wait_event(ev_dec[j])
            out_host[j].copy_(o, non_blocking=True)
            ev_down[j].record(down)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    up.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    for j in range(NBUF):  # every read-back of the timed steps is inside the timed region
        st.wait_event(ev_down[j])
    e1.record(st)
    e1.synchronize()
    us_e2e = e0.elapsed_time(e1) * 1e3 / args.steps
    if dist is not None:
        t = torch.tensor([us_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us_e2e = float(t.item())
    del sets, q_host, out_host, q_dev, outs
    torch.cuda.empty_cache()

    # the long sequence split across the ranks (NCCL all-gather inside the step)
    split = split_kv_bench(dev, rank, world, dist, max(10, min(args.steps, 200)), args.warmup, peak)
    torch.cuda.empty_cache()

    extra = None
    cpu_base = None
    c4 = None
    if world > 1:
        # every rank times its own c4 batch shard; max over ranks
        c4 = c4_batch_shard(dev, peak, torch.Generator(device=dev).manual_seed(11 + rank))
        t = torch.tensor([c4["c4_bf16_131k_B8"]["us"], c4["c4_kivi2_131k_B8"]["us"]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        c4 = {"bf16_us": round(float(t[0].item()), 2), "kivi2_us": round(float(t[1].item()), 2),
              "sequences": 8 * world, "tokens_per_sequence": 131072}
        torch.cuda.empty_cache()
    if rank == 0 and world == 1:
        if not args.no_extras:
            extra = extras(dev, peak)
        cpu_base = cpu_baseline(c)

    if rank == 0:
        wl = _workload(c)
        line = {
            "metric": _metric(), "value": round(us_step, 2), "unit": "us/step", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us_step / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": wl, "global_batch": c["B"] * world, "seq_len": c["S"],
                       "parallelism": f"batch-shard x{world}",
                       "l2": f"{NBUF} rotating input sets ({NBUF * step_bytes / 1e6:.0f} MB > 3x L2)",
                       "timing": "one CUDA graph of exactly `steps` steps, CUDA events, max over ranks"},
            "tokens_per_s": round(c["B"] * world / (us_step * 1e-6), 1),
            "hbm_GBps_step": round(step_bytes * world / us_step / 1e3, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": _measured_traffic(wl),
                         "kernel": "kivi_decode_kernel (packed-cache pass)", "algorithmic_bytes_per_launch": kern_bytes,
                         "kernel_us": round(us_kern, 2)},
            "cpu_baseline": cpu_base,
            "e2e": {"value": round(us_e2e, 2), "unit": "us/step", "h2d_bytes_per_step": nbytes(q_dev_shape(c)),
                    "d2h_bytes_per_step": nbytes(q_dev_shape(c))},
            # per step: the packed-cache pass and the residual-window pass, which also
            # merges the split partials (R = 128 takes one window CTA per group)
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
            "split_kv": split,
        }
        if c4 is not None:
            line["c4_batch_shard"] = c4
        if extra is not None:
            line["paths"] = extra
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def q_dev_shape(c):
    """A meta tensor of one step's query (and output) shape, for byte counts."""
    return torch.empty(c["B"], c["Hq"], 1, c["D"], dtype=torch.bfloat16, device="meta")


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Decode-attention benchmark: prints ONE JSON line (rank 0).

Headline workload (config 1 of the reference study's B200 plan): KIVI-style 2-bit KV
cache decode, batch 8 per GPU, 28 query / 4 KV heads, head_dim 128, context 16384 of which
the last 128 tokens are a bf16 residual window; keys quantised per channel over groups of
32 tokens, values per token over groups of 32 channels (f16 scale / minimum). Synthetic
seeded inputs (N(0,1) bf16 with 4 of 128 key channels x8), packed once by the engine's own
packer before timing.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N ...   (batch-sharded, weak scaling)

value      device time per decode step (µs, max over ranks), CUDA-graph replay of the
           public API call with the packed cache resident in HBM; 8 rotating input sets
           (416 MB > 3x L2) so no step reads its inputs from L2.
e2e        the same step through the public Python API with host buffers: every step copies
           its queries host->device from pinned memory and reads the output back.
roofline   the packed-cache kernel alone (no residual window / combine), algorithmic bytes
           per launch / its CUDA-event time, against MEASURED_PEAKS.json's copy bandwidth.
cpu_baseline / --impl reference: the CPU oracle (a fp32 torch restatement of the
           reference's kivi_decode_attn) on the host cores.
"""
import argparse
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
CFG1 = dict(B=8, Hq=28, Hk=4, D=128, S=16384, R=128, bits=2, group=32)
NBUF = 8


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


def _profile_traffic(name):
    """bytes per launch from a committed ncu summary line 'traffic_bytes_per_launch: N'."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except Exception:
        pass
    return None


# ----------------------------------------------------------------------------- inputs
def kivi_inputs(dev, seed, c=CFG1):
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

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
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

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ----------------------------------------------------------------------------- CPU side
def cpu_kivi_step(inputs_cpu, b=None, tok_frac=1.0):
    """The oracle's KIVI step on host cores; optional sample of one sequence / a token slice."""
    import oracle
    q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr = inputs_cpu
    if b is not None:
        sl = slice(b, b + 1)
        q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr = (t[sl] for t in (q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr))
    if tok_frac < 1.0:
        fpi = 32 // CFG1["bits"]
        ng = max(1, int(Ks.shape[-1] * tok_frac))
        Kq, Ks, Km = Kq[..., :ng * 32 // fpi], Ks[..., :ng], Km[..., :ng]
        Vq, Vs, Vm = Vq[:, :, :ng * 32], Vs[:, :, :ng * 32], Vm[:, :, :ng * 32]
    return oracle.kivi_decode_attn(q, Kq, Ks, Km, Kr, Vq, Vs, Vm, Vr, CFG1["bits"], CFG1["group"])


def cpu_inputs():
    """Config-1 inputs built on the host (same generator recipe as the GPU inputs)."""
    import oracle
    g = torch.Generator().manual_seed(1000)
    c = CFG1
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


def run_reference(args, rank):
    """--impl reference: the CPU restatement of the reference path, timed on host cores."""
    if rank != 0:
        return None
    cores = _host_cores()
    torch.set_num_threads(cores)
    inp = cpu_inputs()
    # size the per-step sample so the whole run stays within ~2 minutes
    t0 = time.perf_counter()
    cpu_kivi_step(inp, b=0)
    one_seq = time.perf_counter() - t0
    total_steps = args.steps + args.warmup
    frac = min(1.0, 110.0 / max(one_seq * total_steps, 1e-9))
    for i in range(args.warmup):
        cpu_kivi_step(inp, b=i % CFG1["B"], tok_frac=frac)
    t0 = time.perf_counter()
    for i in range(args.steps):
        cpu_kivi_step(inp, b=i % CFG1["B"], tok_frac=frac)
    dt = (time.perf_counter() - t0) / args.steps
    us = dt * 1e6 * CFG1["B"] / frac  # one sequence (and a token fraction) per step, scaled to the full step
    sample = f"one of {CFG1['B']} sequences per step" + (f", first {frac:.3f} of the packed tokens" if frac < 1 else "")
    line = {
        "impl": "reference", "metric": _metric(), "value": round(us, 1), "unit": "us/step", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "c1 KIVI-2 decode B=8 Hq=28 Hk=4 D=128 S=16384 R=128 group=32",
                   "global_batch": CFG1["B"], "seq_len": CFG1["S"], "parallelism": "host cores"},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": cores, "kind": "port",
                         "sample": sample + ", time scaled to the full step"},
        "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# ----------------------------------------------------------------------------- extras
def _rot(make, n):
    return [make() for _ in range(n)]


def path_c0(dev, peak, g):
    """c0: bf16 dense decode, B=1, 28/4 heads, S=8192, q pre-scaled by 1/sqrt(D)."""
    from bytes_b200 import attention_kernels as ak
    D = 128
    sets = _rot(lambda: ((torch.randn(1, 28, 1, D, device=dev, generator=g) / math.sqrt(D)).bfloat16(),
                         torch.randn(1, 4, 8192, D, device=dev, generator=g).bfloat16(),
                         torch.randn(1, 4, 8192, D, device=dev, generator=g).bfloat16()), 16)
    gr = graph_of([lambda s=s: ak.decode_attn_bf16(*s) for s in sets])
    us = time_graph(gr, 20) / (20 * len(sets))
    b = nbytes(*sets[0][1:])
    return {"c0_bf16_decode": {"us": round(us, 2), "GBps": round(b / us / 1e3, 1),
                               "frac": round(b / us / 1e3 / peak, 3)}}


def path_bf16_32k(dev, peak, g):
    """bf16 dense decode at 32K context with the c1 head shapes (B=8, 28/4)."""
    from bytes_b200 import attention_kernels as ak
    D = 128
    sets = _rot(lambda: (torch.randn(8, 28, 1, D, device=dev, generator=g).bfloat16(),
                         torch.randn(8, 4, 32768, D, device=dev, generator=g).bfloat16(),
                         torch.randn(8, 4, 32768, D, device=dev, generator=g).bfloat16()), 2)
    gr = graph_of([lambda s=s: ak.decode_attn_bf16(*s) for s in sets])
    us = time_graph(gr, 10) / (10 * len(sets))
    b = nbytes(*sets[0][1:])
    return {"bf16_decode_32k_B8": {"us": round(us, 2), "GBps": round(b / us / 1e3, 1),
                                   "frac": round(b / us / 1e3 / peak, 3)}}


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
    return {"c2_pq_lut_int8v": {"us": round(us, 2), "GBps": round(b / us / 1e3, 1),
                                "frac": round(b / us / 1e3 / peak, 3)}}


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


def path_c4(dev, peak, g):
    """c4 (8-GPU box), one GPU's share: 8 sequences x 131072 tokens with the c1 head shapes
    (28/4, D=128) as bf16 and as KIVI-2; and one rank's shard of a 1M-token sequence split
    8 ways (B=1, 131072 tokens): its split-KV partial, then the combine of 8 shard partials
    (the partials of this shard stand in for the all-gather's result on one GPU)."""
    from bytes_b200 import attention_kernels as ak, kivi as kv, _ops
    out = {}
    D, S = 128, 131072
    q = torch.randn(8, 28, 1, D, device=dev, generator=g).bfloat16()
    k = torch.randn(8, 4, S, D, device=dev, generator=g).bfloat16()
    v = torch.randn(8, 4, S, D, device=dev, generator=g).bfloat16()
    gr = graph_of([lambda: ak.decode_attn_bf16(q, k, v)])
    time_graph(gr, 2)
    us = time_graph(gr, 10) / 10
    b = nbytes(k, v)
    out["c4_bf16_131k_B8"] = {"us": round(us, 2), "GBps": round(b / us / 1e3, 1), "frac": round(b / us / 1e3 / peak, 3)}
    del k, v, gr
    torch.cuda.empty_cache()
    c = dict(CFG1, S=S)
    s = kivi_inputs(dev, 4242, c)
    gr = graph_of([lambda: kv.kivi_decode_attn(*s, c["bits"], c["group"])])
    time_graph(gr, 2)
    us = time_graph(gr, 10) / 10
    b = nbytes(*s[1:])
    out["c4_kivi2_131k_B8"] = {"us": round(us, 2), "MB": round(b / 1e6, 1), "GBps": round(b / us / 1e3, 1),
                               "frac": round(b / us / 1e3 / peak, 3)}
    del s, gr
    torch.cuda.empty_cache()
    q1 = torch.randn(1, 28, D, device=dev, generator=g).bfloat16()
    k1 = torch.randn(1, 4, S, D, device=dev, generator=g).bfloat16()
    v1 = torch.randn(1, 4, S, D, device=dev, generator=g).bfloat16()
    scal = 1.0 / math.sqrt(D)
    gr = graph_of([lambda: _ops.decode_attn_partial(q1, k1, v1, scal)])
    time_graph(gr, 2)
    us_p = time_graph(gr, 10) / 10
    m, l, o = _ops.decode_attn_partial(q1, k1, v1, scal)
    m8, l8, o8 = (t.unsqueeze(0).repeat(8, *([1] * t.dim())).contiguous() for t in (m, l, o))
    gr2 = graph_of([lambda: _ops.lse_combine(m8, l8, o8, torch.bfloat16)])
    time_graph(gr2, 2)
    us_c = time_graph(gr2, 20) / 20
    b = nbytes(k1, v1)
    out["c4_1M_shard_of_8"] = {"partial_us": round(us_p, 2), "combine8_us": round(us_c, 2),
                               "GBps": round(b / us_p / 1e3, 1), "frac": round(b / us_p / 1e3 / peak, 3),
                               "exchange_bytes_per_rank": int(m.numel() * 8 + o.numel() * 4)}
    return out


PATHS = {"c0": path_c0, "bf16_32k": path_bf16_32k, "c2": path_c2, "c3": path_c3, "topk": path_topk, "c4": path_c4}


def extras(dev, peak, only=None):
    """Other decode paths at their configuration shapes (rank 0, single GPU)."""
    import gc
    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    for name, fn in PATHS.items():
        if only is not None and name != only:
            continue
        out.update(fn(dev, peak, g))
        gc.collect()
        torch.cuda.empty_cache()
    return out


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
    args.warmup = max(args.warmup, 3)

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
    c = CFG1
    sets = [kivi_inputs(dev, 1000 + rank * NBUF + i) for i in range(NBUF)]
    step_bytes = nbytes(*sets[0][1:])
    kern_bytes = nbytes(*(sets[0][i] for i in (1, 2, 3, 5, 6, 7)))
    scal = 1.0 / math.sqrt(c["D"])

    # device-time value: graph replay of the public call, NBUF rotating input sets per replay
    calls = [lambda s=s: kv.kivi_decode_attn(*s, c["bits"], c["group"]) for s in sets]
    g_step = graph_of(calls)
    reps_w = max(1, math.ceil(args.warmup / NBUF))
    reps = max(1, math.ceil(args.steps / NBUF))
    steps_timed = reps * NBUF
    time_graph(g_step, reps_w)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        us_total = time_graph(g_step, reps)
    torch.cuda.synchronize()
    us_step = us_total / steps_timed
    if dist is not None:
        t = torch.tensor([us_step], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us_step = float(t.item())

    # roofline: the packed-cache kernel alone
    outs = [torch.empty(c["B"], c["Hq"], c["D"], dtype=torch.bfloat16, device=dev) for _ in sets]
    kcalls = [lambda s=s, o=o: _ops.kivi_decode(s[0][:, :, 0, :], *s[1:], c["bits"], c["group"], scal, o, stages=1)
              for s, o in zip(sets, outs)]
    g_k = graph_of(kcalls)
    time_graph(g_k, 2)
    us_kern = time_graph(g_k, max(2, reps // 2)) / (max(2, reps // 2) * NBUF)
    achieved = kern_bytes / us_kern / 1e3  # GB/s

    # e2e through the public API with host buffers
    q_host = [s[0].cpu().pin_memory() for s in sets]
    out_host = [torch.empty(c["B"], c["Hq"], 1, c["D"], dtype=torch.bfloat16).pin_memory() for _ in sets]
    q_dev = [torch.empty_like(s[0]) for s in sets]
    n_e2e = max(NBUF, min(args.steps, 400))
    st = torch.cuda.current_stream()

    def e2e_step(i):
        j = i % NBUF
        q_dev[j].copy_(q_host[j], non_blocking=True)
        o = kv.kivi_decode_attn(q_dev[j], *sets[j][1:], c["bits"], c["group"])
        out_host[j].copy_(o, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(n_e2e):
        e2e_step(i)
    e1.record(st)
    e1.synchronize()
    us_e2e = e0.elapsed_time(e1) * 1e3 / n_e2e
    if dist is not None:
        t = torch.tensor([us_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us_e2e = float(t.item())

    extra = None
    cpu_base = None
    if rank == 0 and world == 1:
        if not args.no_extras:
            extra = extras(dev, peak)
        cores = _host_cores()
        torch.set_num_threads(cores)
        inp = cpu_inputs()
        t0 = time.perf_counter()
        n_cpu = 0
        while n_cpu < 2 or (time.perf_counter() - t0 < 10.0 and n_cpu < 20):
            cpu_kivi_step(inp, b=n_cpu % c["B"])
            n_cpu += 1
        us_cpu = (time.perf_counter() - t0) / n_cpu * 1e6 * c["B"]
        cpu_base = {"value": round(us_cpu, 1), "unit": "us/step", "cores": cores, "kind": "port",
                    "sample": f"{n_cpu} single-sequence steps of the config-1 cache (fp32 torch oracle), x{c['B']}"}

    if rank == 0:
        line = {
            "metric": _metric(), "value": round(us_step, 2), "unit": "us/step", "n_gpus": world,
            "steps": steps_timed, "warmup": reps_w * NBUF, "ms_per_step": round(us_step / 1e3, 5),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic",
            "config": {"workload": "c1 KIVI-2 decode B=8 Hq=28 Hk=4 D=128 S=16384 R=128 group=32",
                       "global_batch": c["B"] * world, "seq_len": c["S"], "parallelism": f"batch-shard x{world}",
                       "l2": f"{NBUF} rotating input sets ({NBUF * step_bytes / 1e6:.0f} MB > 3x L2)",
                       "timing": "CUDA-graph replay, CUDA events, max over ranks"},
            "tokens_per_s": round(c["B"] * world / (us_step * 1e-6), 1),
            "hbm_GBps_step": round(step_bytes * world / us_step / 1e3, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": _profile_traffic("kivi_decode_kernel_c1.md"),
                         "kernel": "kivi_decode_kernel<2,1,3>", "algorithmic_bytes_per_launch": kern_bytes,
                         "kernel_us": round(us_kern, 2)},
            "cpu_baseline": cpu_base,
            "e2e": {"value": round(us_e2e, 2), "unit": "us/step", "h2d_bytes_per_step": nbytes(sets[0][0]),
                    "d2h_bytes_per_step": nbytes(outs[0])},
            # per step: the packed-cache pass and the residual-window pass, which also
            # merges the split partials (R = 128 takes one window CTA per group)
            "gpu_launches": 2 * steps_timed,
            "clocks": clk.summary(),
        }
        if extra is not None:
            line["paths"] = extra
        print(json.dumps(line), flush=True)
    del g_step, g_k
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

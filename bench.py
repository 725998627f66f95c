"""Benchmark of the HALO chunked-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload all|cfg5|cfg2|cfg3|cfg4] [--no-cpu-baseline]

Headline workload (all N): 1M-token sequence-sharded decode of one
Llama-3-70B-shaped attention layer (B1, 64 q-heads / 8 KV heads, head_dim
128, bf16, 256 chunks of 4096 rows).  Rank r of N owns a contiguous 1/N of
the chunks; a step is one decode query: split-KV kernel over the local
chunks, then one fused kernel that merges the local splits, pushes the fp32
(o, lse) row to every rank over NVLink peer stores and merges the N parts
(halo_sharded_merge).  Total context is fixed as N grows (strong scaling).
K/V are seeded N(0,1) synthetic data resident in HBM; the working set per
GPU (4.3 GB / N) is far larger than L2, so no flush is needed between steps.
After timing, one KV-head group of the last output is checked against a
float64 attention (``parity`` in the line).

With N = 1 the default run (``--workload all``) also measures the other
three workloads and reports them under ``workloads`` in the same line:

* ``cfg2`` -- tiered decode: 32 layers of B8 / 32 q-heads / 8 KV heads /
  32K context in chunks of 1024; hot chunks (first + 7 most recent) in HBM,
  24 cold chunks per layer in pinned host DRAM; per layer and step the chunk
  scorer picks the top-8 cold chunks for a fresh query, the ones not already
  in the layer's GPU slot cache are refetched on a copy stream while the hot
  chunks are attended, then the selected chunks are folded in
  (``halo_b200.tiered.TieredLayer``);
* ``cfg3`` -- chunked prefill of a 131072-token prompt in 32 slices of 4096
  queries against the accumulated KV, causal, 32 q-heads / 8 KV heads,
  head_dim 128, on the tcgen05 prefill kernel; a step is the whole prompt of
  one layer;
* ``cfg4`` -- KIVI 2-bit decode of B4 / 32 q-heads / 8 KV heads / head_dim
  128 over a 65536-token context -- 65408 quantised rows (packed 2-bit
  codes, fp16 scale and zero per group of 32 along head_dim) plus the 128
  most recent rows in fp16 -- through ``KIVICache.compute_attention``.

and, under ``reference_gpu``, the reference's own Triton decode kernel
(``halo/triton_chunked.py`` from the reference installed in
``baseline/_ref``) timed on the same GPU and inputs.  ``--workload cfgX``
runs one workload alone and prints its own line.

``--seq-len T`` shrinks the cfg5 context (a multiple of 4096 x N) or the cfg3
prompt (a multiple of 4096), and ``--layers L`` the cfg2 layer count, for
small profiling captures; the line then names the reduced workload.

Rank 0 prints one JSON line.  ``--impl reference`` times the reference's CPU
implementation of the path (its torch ops restated in ``oracle/``) on this
host's cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# 1M-token sequence-sharded decode of one Llama-3-70B-shaped layer
CFG5 = dict(B=1, H=64, H_kv=8, D=128, T=1 << 20, chunk=4096)
METRIC = "decode-attn tokens/s & achieved HBM GB/s at 32K-1M ctx, 1/2/4/8 B200"

# DRAM traffic per algorithmic byte, from one ncu capture of each kernel
# (dram__bytes_read.sum + dram__bytes_write.sum of the launch over the bytes
# it must read); the captures and their commands are summarised under
# profiles/.  kd_dyn_kernel: cfg5 reduced to 262144 tokens, scaled to a full
# launch by the K/V bytes it processes.  kk_kernel: the cfg4 launch itself
# (transposed tile math, K into MMA registers).  kd_kernel at cfg2: the hot
# and selected launches of one layer.
NCU_TRAFFIC_RATIO = 1.0040      # kd_dyn_kernel, ncu at 262144 tokens: (1073.795 + 4.311) MB read+write / 1073.742 MB algorithmic
NCU_TRAFFIC_RATIO_KK = 1.0200      # kk_kernel, ncu of the cfg4 launch: (201.00 + 3.95) MB / 200.93 MB
NCU_TRAFFIC_RATIO_KD_CFG2 = 1.0139  # kd_kernel, ncu of one layer's hot + selected launches (cfg2)


def _tensor_peak():
    """Sustained dense bf16 TFLOP/s (a kernel timed inside a long step)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.idx, self.period = device_index, period_s
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        self._thr = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return self
        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append(self._nv.nvmlDeviceGetClockInfo(self._h, self._nv.NVML_CLOCK_SM))
                    self.reasons |= int(self._nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
                except Exception:
                    pass
                time.sleep(self.period)
        self._thr = threading.Thread(target=loop, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr is not None:
            self._thr.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def _dist_setup(n_gpus: int):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _cfg5_shard(world: int, rank: int, dev):
    """This rank's K/V shard of the 1M-token context and the replicated query."""
    import torch
    from halo_b200.sharded import shard_range
    c = CFG5
    n_chunks = c["T"] // c["chunk"]
    lo, hi = shard_range(n_chunks, world, rank)
    rows = (hi - lo) * c["chunk"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    k = torch.randn(c["B"], c["H_kv"], rows, c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    v = torch.randn(c["B"], c["H_kv"], rows, c["D"], device=dev, dtype=torch.bfloat16, generator=g)
    gq = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(c["B"], c["H"], c["D"], device=dev, dtype=torch.bfloat16, generator=gq)
    return q, k, v, lo * c["chunk"]


def _cpu_cfg5_sample(n_chunks_sample: int, seed: int = 1000):
    """CPU copies of the first chunks of rank 0's shard (bf16) and the query."""
    import torch
    c = CFG5
    g = torch.Generator().manual_seed(seed)
    rows = n_chunks_sample * c["chunk"]
    k = torch.randn(c["B"], c["H_kv"], rows, c["D"], generator=g).bfloat16()
    v = torch.randn(c["B"], c["H_kv"], rows, c["D"], generator=g).bfloat16()
    q = torch.randn(c["B"], c["H"], 1, c["D"], generator=g).bfloat16()
    chunks = [(k[..., a:a + c["chunk"], :], v[..., a:a + c["chunk"], :], a, False)
              for a in range(0, rows, c["chunk"])]
    return q, chunks


def _time_cpu_oracle(n_chunks_sample: int, repeats: int):
    """Seconds per sample of the CPU oracle port (reference torch ops)."""
    import torch
    from oracle import attention as OA
    torch.set_num_threads(os.cpu_count() or 1)
    q, chunks = _cpu_cfg5_sample(n_chunks_sample)
    OA.chunked_attention(q, chunks[:1])  # warm the thread pool
    ts = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        OA.chunked_attention(q, chunks)
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), torch.get_num_threads()


def cpu_baseline_cfg5(budget_s: float = 15.0):
    """Bounded CPU sample of cfg5 through the oracle port, scaled to a step."""
    n_total = CFG5["T"] // CFG5["chunk"]
    t1, _ = _time_cpu_oracle(1, 1)
    n = int(max(1, min(n_total, budget_s / 3 / max(t1, 1e-3))))
    t, cores = _time_cpu_oracle(n, 3)
    step_s = t * n_total / n
    return {"value": CFG5["B"] / step_s, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n} of {n_total} chunks (x{CFG5['chunk']} rows) of rank-0 data, "
                      f"median of 3, scaled x{n_total / n:.1f} to the full 1M-token step",
            "s_per_step": step_s}


def run_reference(args):
    """The reference arm: the reference's CPU torch path (restated in the
    oracle) on this host's cores, each step a bounded sample of cfg5."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    n_total = CFG5["T"] // CFG5["chunk"]
    t1, cores = _time_cpu_oracle(1, 1)
    budget = 150.0 / max(1, args.steps + args.warmup)
    n = int(max(1, min(n_total, budget / max(t1, 1e-3))))
    import torch
    from oracle import attention as OA
    q, chunks = _cpu_cfg5_sample(n)
    for _ in range(args.warmup):
        OA.chunked_attention(q, chunks)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        OA.chunked_attention(q, chunks)
    el = time.perf_counter() - t0
    step_s = el / args.steps * n_total / n
    value = CFG5["B"] / step_s
    sample = (f"each step: {n} of {n_total} chunks of the 1M-token context through the "
              f"reference torch ops on CPU, time scaled x{n_total / n:.1f}")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": _cfg5_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _cfg5_config(n: int):
    c = CFG5
    n_chunks = c["T"] // c["chunk"]
    name = ("cfg5: 1M-token sequence-sharded decode" if c["T"] == 1 << 20 else
            f"cfg5 reduced to {c['T']} tokens (profiling case)")
    return {"workload": f"{name}, one Llama-3-70B-shaped attention layer (64 q-heads / "
                        f"8 KV heads, head_dim 128), {n_chunks} chunks x {c['chunk']}",
            "global_batch": c["B"], "seq_len": c["T"], "chunk": c["chunk"],
            "parallelism": f"sequence-sharded x{n} (fused LSE merge with NVLink peer-store "
                           f"exchange of (o, lse))"
                           if n > 1 else "single GPU",
            "l2": "inputs larger than L2 (K+V %.2f GB per GPU); no flush" %
                  (2 * c["B"] * c["H_kv"] * c["T"] * c["D"] * 2 / n / 1e9)}


def run_ours_cfg5(args):
    import torch
    import torch.distributed as dist
    world, rank, local = _dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    from halo_b200 import _lib as L
    from halo_b200.sharded import ShardedDecoder
    q, k, v, start = _cfg5_shard(world, rank, dev)
    dec = ShardedDecoder(k, v, start=start, chunk_size=CFG5["chunk"],
                         group=dist.group.WORLD if world > 1 else None)
    B, H, D = q.shape
    out = torch.empty(B, H, D, device=dev, dtype=q.dtype)
    lse = torch.empty(B, H, device=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        dec(q, out=out, lse=lse)
    torch.cuda.synchronize()
    # a decode step as a serving loop runs it: one CUDA graph replay per step
    # (split-KV kernel + merge, or + the NVLink exchange merge when sharded);
    # --eager times plain calls instead
    graph = None if args.eager else dec.capture(q, out=out, lse=lse)
    step = graph.replay if graph is not None else (lambda: dec(q, out=out, lse=lse))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device throughput: K steps, events only around the whole loop (an
    # event between the split-KV kernel and its dependent merge would cancel
    # the merge's early launch)
    K = args.steps
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    n0 = L.launch_count()
    with ClockSampler(local) as clocks:
        t0.record()
        for i in range(K):
            step()
        t1.record()
        torch.cuda.synchronize()
    # graph replays launch the captured kernels without passing the host
    # counter: count them from the kernels one step holds
    launches = (K * dec.launches_per_call if graph is not None else L.launch_count() - n0)
    barrier()
    ms = t0.elapsed_time(t1)
    # ---- roofline pass: the same K steps with the split-KV kernel bracketed
    # by events on its stream
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    for e in ev_b + ev_e:          # materialise the raw events
        e.record()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks_kd:
        for i in range(K):
            dec(q, out=out, lse=lse, events=(ev_b[i].cuda_event, ev_e[i].cuda_event))
        torch.cuda.synchronize()
    barrier()
    kd_ms = sum(ev_b[i].elapsed_time(ev_e[i]) for i in range(K)) / K
    ms_t = torch.tensor([ms, kd_ms], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, kd_ms_max = ms_t.tolist()
    ms_step = ms / K

    # ---- end to end through the public API with host buffers: the query
    # comes from pinned host memory into the step's input buffer, the output
    # goes back, every step synchronised
    q_host = q.cpu().pin_memory()
    out_host = torch.empty_like(out, device="cpu").pin_memory()
    for _ in range(3):
        q.copy_(q_host, non_blocking=True)
        step()
        out_host.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        q.copy_(q_host, non_blocking=True)
        step()
        out_host.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / K], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    barrier()

    # parity of the last output (outside timing): one KV-head group against
    # float64 attention, each rank over its own shard, merged across ranks
    parity = _cfg5_parity(q, k, v, out, lse, world, group_kv=0)
    local_bytes = 2 * k.numel() * k.element_size()
    peak, peak_kind = _peaks()
    achieved = local_bytes / (kd_ms_max / 1e3) / 1e9
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        ref_gpu = reference_gpu_cfg5(q, k, v, out)
    line = None
    if rank == 0:
        cpu = cpu_baseline_cfg5() if world == 1 and not args.no_cpu_baseline else None
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_kind": f"of {peak_kind}",
                "kernel": "kd_dyn_kernel (split-KV decode, dynamic schedule)",
                "timing": "second pass of K steps with events around the split-KV kernel",
                "clocks_kd_pass": clocks_kd.summary(),
                "bytes_per_launch": local_bytes,
                "traffic": (local_bytes * NCU_TRAFFIC_RATIO) if NCU_TRAFFIC_RATIO else None,
                "step_gbs": 2 * CFG5["B"] * CFG5["H_kv"] * CFG5["T"] * CFG5["D"] * 2
                            / (ms_step / 1e3) / 1e9}
        line = {"metric": METRIC, "value": CFG5["B"] / (ms_step / 1e3), "unit": "tokens/s",
                "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic", "config": _cfg5_config(world),
                "roofline": roof,
                "cpu_baseline": cpu and {kk: cpu[kk] for kk in ("value", "unit", "cores",
                                                               "kind", "sample")},
                "e2e": {"value": CFG5["B"] / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": q.numel() * q.element_size(),
                        "d2h_bytes_per_step": out.numel() * out.element_size()},
                "clocks": clocks.summary(),
                "gpu_launches": launches,
                "parity": parity}
        if ref_gpu is not None:
            line["reference_gpu"] = ref_gpu
        line["config"]["step"] = ("one CUDA graph replay per step" if graph is not None
                                  else "eager calls")
    del graph, step
    torch.cuda.synchronize()
    dec.close()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return line


def _cfg5_parity(q, k, v, out, lse, world: int, group_kv: int = 0):
    """Max |error| of the decode output and LSE of one KV-head group against
    float64 attention computed with torch on this GPU.  Each rank attends
    its own shard; the ranks' (out, lse) rows are all-gathered (a few KB)
    and merged with log-sum-exp, so every rank takes the same collective
    step.  ``out`` is the bf16 output the timed loop kept, so its error
    includes one bf16 rounding."""
    import torch
    import torch.distributed as dist
    B, H, D = q.shape
    H_kv = k.shape[1]
    G = H // H_kv
    hs = slice(group_kv * G, (group_kv + 1) * G)
    scale = 1.0 / (D ** 0.5)
    qg = q[:, hs].double()                                   # (B, G, D)
    o_loc = torch.empty(B, G, D, dtype=torch.float64, device=q.device)
    l_loc = torch.empty(B, G, dtype=torch.float64, device=q.device)
    for b in range(B):
        s = torch.matmul(qg[b], k[b, group_kv].double().T) * scale      # (G, T_local)
        l = torch.logsumexp(s, dim=-1)
        o_loc[b] = torch.matmul(torch.exp(s - l[:, None]), v[b, group_kv].double())
        l_loc[b] = l
        del s
    row = torch.cat([o_loc.reshape(-1), l_loc.reshape(-1)])
    if world > 1:
        rows = torch.empty(world * row.numel(), dtype=row.dtype, device=row.device)
        dist.all_gather_into_tensor(rows, row)
        rows = rows.view(world, -1)
    else:
        rows = row.view(1, -1)
    o_parts = rows[:, :B * G * D].view(-1, B, G, D)
    l_parts = rows[:, B * G * D:].view(-1, B, G)
    l_all = torch.logsumexp(l_parts, dim=0)
    o_all = (torch.exp(l_parts - l_all)[..., None] * o_parts).sum(dim=0)
    err_o = (out[:, hs].double() - o_all).abs().max().item()
    err_l = (lse[:, hs].double() - l_all).abs().max().item()
    return {"kv_head_group": group_kv, "max_abs_out": err_o, "max_abs_lse": err_l,
            "checker": "float64 torch attention on the GPU (per-rank shard, LSE-merged)",
            "tolerance": {"out": 2e-3 + 2 ** -8 * o_all.abs().max().item(), "lse": 1e-4},
            "ok": bool(err_o <= 2e-3 + 2 ** -8 * o_all.abs().max().item() and err_l <= 1e-4)}


def _reference_triton():
    """The reference's Triton module from its unmodified install under
    ``baseline/_ref`` (``pip install --target baseline/_ref``), or a reason
    why it cannot run here."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "halo")):
        return None, "reference not installed under baseline/_ref"
    if ref_root not in sys.path:
        sys.path.append(ref_root)
    try:
        from halo import triton_chunked as RT
    except Exception as e:          # noqa: BLE001 - reported in the line
        return None, f"import halo.triton_chunked failed: {type(e).__name__}: {e}"
    if not getattr(RT, "HAS_TRITON", False):
        return None, "triton is not importable on this box"
    return RT, None


def _time_events(fn, steps: int, warmup: int):
    """Mean ms per call of ``fn`` on the current stream (CUDA events)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        res = fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, res


def reference_gpu_cfg5(q, k, v, ours_out, steps: int = 5, warmup: int = 3):
    """The reference's own GPU decode path (its Triton kernel,
    ``halo/triton_chunked.py:47-138``) on this GPU and on the same resident
    inputs as the timed decode: (a) ``update_chunk`` once over the whole
    context (the kernel alone, grid B x H) + ``finalize``; (b) its
    single-launch driver ``triton_chunked_attention_single_launch`` with the
    context passed as its GPU part (it stages the rows into one buffer with a
    device-to-device copy, then launches the kernel once).  Not causal (the
    query sits after every key).  Also reports the largest difference
    between the reference kernel's output and this build's."""
    import torch
    RT, why = _reference_triton()
    if RT is None:
        return {"unavailable": why}
    B, H, D = q.shape
    T = k.shape[-2]
    scale = 1.0 / (D ** 0.5)
    q_pos = torch.full((B,), T - 1, dtype=torch.int64, device=q.device)
    nbytes = 2 * k.numel() * k.element_size()

    def kernel_only():
        m, l, o = RT.init_acc(B=B, H=H, D_v=v.shape[-1], device=q.device)
        RT.update_chunk(q=q, k=k, v=v, m=m, l=l, o=o, scale=scale, chunk_start=0, q_pos=q_pos,
                        apply_causal=False)
        return RT.finalize(m=m, l=l, o=o, out_dtype=torch.float32)

    def single_launch():
        return RT.triton_chunked_attention_single_launch(q.unsqueeze(2), None, None, k, v,
                                                         scale=scale, q_pos=q_pos,
                                                         apply_causal=False)

    try:
        ms_k, o_ref = _time_events(kernel_only, steps, warmup)
        ms_s, _ = _time_events(single_launch, steps, warmup)
    except Exception as e:          # noqa: BLE001 - reported in the line
        return {"unavailable": f"reference Triton kernel failed: {type(e).__name__}: {e}"}
    diff = (o_ref - ours_out.float()).abs().max().item()
    return {"impl": "reference halo/triton_chunked.py (unmodified, baseline/_ref), Triton on "
                    "this B200",
            "workload": "the timed 1M-token decode: same q, K, V in HBM",
            "kernel_only": {"ms_per_step": ms_k, "tokens_per_s": B / (ms_k / 1e3),
                            "algorithmic_gbs": nbytes / (ms_k / 1e3) / 1e9,
                            "call": "init_acc + update_chunk over all rows + finalize"},
            "single_launch": {"ms_per_step": ms_s, "tokens_per_s": B / (ms_s / 1e3),
                              "algorithmic_gbs": nbytes / (ms_s / 1e3) / 1e9,
                              "call": "triton_chunked_attention_single_launch (includes its "
                                      "device-to-device staging copy)"},
            "max_abs_vs_ours": diff, "steps": steps, "warmup": warmup}


# ---------------------------------------------------------------- cfg2 (tiered decode)
CFG2 = dict(L=32, B=8, H=32, H_kv=8, D=128, T=32768, chunk=1024, k_sel=8)
METRIC2 = ("tiered decode tokens/s & achieved HBM GB/s, Llama-3-8B shapes, 32K ctx, "
           "hot 25% + top-8 cold chunks refetched, 1 B200")


def _cfg2_hot(P: int):
    """hot_ratio 0.25: the first chunk plus the most recent ones."""
    n_hot = max(1, P // 4)
    return [0] + list(range(P - (n_hot - 1), P))


def _cfg2_config():
    c = CFG2
    P = c["T"] // c["chunk"]
    name = "cfg2: tiered decode" if c["L"] == 32 else "cfg2 reduced (profiling case): tiered decode"
    return {"workload": f"{name}, {c['L']} layers, B{c['B']}, 32 q-heads / 8 KV "
                        f"heads, head_dim 128, {c['T']} ctx in {P} chunks of {c['chunk']}; hot = "
                        f"chunk 0 + {len(_cfg2_hot(P)) - 1} most recent (HBM), {P - len(_cfg2_hot(P))} "
                        f"cold chunks in pinned host DRAM; per layer and step the chunk scorer picks "
                        f"the top-{c['k_sel']} cold chunks for a fresh N(0,1) query and the ones not "
                        f"already in the GPU slot cache are refetched; keys with 4 outlier channels",
            "global_batch": c["B"], "seq_len": c["T"], "chunk": c["chunk"],
            "parallelism": "single GPU",
            "l2": "attended K/V 0.54 GB per layer > L2 (126 MB); no flush"}


def cpu_baseline_cfg2(budget_s: float = 15.0):
    """The reference's CPU decode attention over the same 16 chunks of one
    layer (torch ops restated in the oracle), scaled by the layer count."""
    import torch
    from oracle import attention as OA
    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG2
    g = torch.Generator().manual_seed(2)
    n_chunks = len(_cfg2_hot(c["T"] // c["chunk"])) + c["k_sel"]
    q = torch.randn(c["B"], c["H"], 1, c["D"], generator=g).bfloat16()

    def run(n):
        chunks = []
        for i in range(n):
            k = torch.randn(c["B"], c["H_kv"], c["chunk"], c["D"], generator=g).bfloat16()
            v = torch.randn(c["B"], c["H_kv"], c["chunk"], c["D"], generator=g).bfloat16()
            chunks.append((k, v, i * c["chunk"], False))
        t0 = time.perf_counter()
        OA.chunked_attention(q, chunks)
        return time.perf_counter() - t0

    t1 = run(1)
    n = int(max(1, min(n_chunks, budget_s / 2 / max(t1, 1e-3))))
    t = run(n)
    step_s = t * (n_chunks / n) * c["L"]
    return {"value": c["B"] / step_s, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"{n} of the {n_chunks} attended chunks of one of {c['L']} layers "
                      f"(fp32 torch ops), scaled x{n_chunks / n * c['L']:.0f}",
            "s_per_step": step_s}


def run_ours_cfg2(args):
    import torch
    from halo_b200 import _lib as L
    from halo_b200.tiered import TieredLayer
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("cfg2 runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = CFG2
    P = c["T"] // c["chunk"]
    hot = _cfg2_hot(P)
    copy_stream = torch.cuda.Stream(dev)
    layers = []
    g = torch.Generator(device=dev).manual_seed(2)
    for li in range(c["L"]):
        k = torch.randn(c["B"], c["H_kv"], c["T"], c["D"], device=dev, generator=g)
        k = _outlier_keys(k, 200 + li).bfloat16()
        v = torch.randn(c["B"], c["H_kv"], c["T"], c["D"], device=dev, generator=g,
                        dtype=torch.bfloat16)
        layers.append(TieredLayer(k, v, chunk_size=c["chunk"], hot_chunks=hot,
                                  n_slots=c["k_sel"], copy_stream=copy_stream))
        del k, v
    n_q = args.warmup + args.steps + 4
    qs = torch.randn(n_q, c["L"], c["B"], c["H"], c["D"], device=dev, generator=g,
                     dtype=torch.bfloat16)
    out = torch.empty(c["B"], c["H"], c["D"], device=dev, dtype=torch.bfloat16)
    lse = torch.empty(c["B"], c["H"], device=dev)

    def step(i, evs=None, cevs=None):
        for li, lay in enumerate(layers):
            lay.step(qs[i, li], k_sel=c["k_sel"], out=out, lse=lse,
                     events=evs[li] if evs else None,
                     copy_events=cevs[li] if cevs else None)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    for lay in layers:
        for kk in lay.stats:
            lay.stats[kk] = 0
    K = args.steps
    mk = lambda: torch.cuda.Event(enable_timing=True)
    evs = [[[(mk(), mk()), (mk(), mk())] for _ in range(c["L"])] for _ in range(K)]
    for e in (x for s_ in evs for l_ in s_ for pr in l_ for x in pr):
        e.record()
    torch.cuda.synchronize()
    raw = [[((a.cuda_event, b.cuda_event), (c2.cuda_event, d.cuda_event))
            for (a, b), (c2, d) in s_] for s_ in evs]
    cevs = [[(mk(), mk()) for _ in range(c["L"])] for _ in range(K)]
    for e in (x for s_ in cevs for pr in s_ for x in pr):
        e.record()
    torch.cuda.synchronize()
    t0, t1 = mk(), mk()
    n0 = L.launch_count()
    with ClockSampler(0) as clocks:
        t0.record()
        for i in range(K):
            step(args.warmup + i, raw[i], cevs[i])
        t1.record()
        torch.cuda.synchronize()
    launches = L.launch_count() - n0
    ms_step = t0.elapsed_time(t1) / K
    kd_ms = sum(a.elapsed_time(b) + c2.elapsed_time(d)
                for s_ in evs for (a, b), (c2, d) in s_) / K
    hot_ms = sum(a.elapsed_time(b) for s_ in evs for (a, b), _ in s_) / K
    copy_ms = sum(a.elapsed_time(b) for s_ in cevs for (a, b) in s_) / K
    # compute-stream idle time between the hot attention and the fold of
    # the selected chunks: waiting for the indices on the host and for the
    # refetch copies (the part of the refetch not hidden behind attention)
    exposed_ms = sum(max(0.0, hb.elapsed_time(sb)) for s_ in evs
                     for (_ha, hb), (sb, _se) in s_) / K
    refetched = sum(l_.stats["refetched_chunks"] for l_ in layers) / K
    refetch_bytes = sum(l_.stats["refetch_bytes"] for l_ in layers) / K
    att_bytes = (len(hot) + c["k_sel"]) * layers[0].chunk_bytes * c["L"]

    # e2e: the query comes from pinned host memory, the output goes back
    q_host = qs[:, :, :, :, :].cpu().pin_memory()
    out_host = torch.empty(c["B"], c["H"], c["D"], dtype=torch.bfloat16).pin_memory()
    q_dev = torch.empty_like(qs[0])

    def e2e_step(i):
        q_dev.copy_(q_host[i], non_blocking=True)
        for li, lay in enumerate(layers):
            lay.step(q_dev[li], k_sel=c["k_sel"], out=out, lse=lse)
        out_host.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step(0)
    e0, e1 = mk(), mk()
    n_e2e = max(1, min(K, 5))
    e0.record()
    for i in range(n_e2e):
        e2e_step(1 + i)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / n_e2e

    peak, peak_kind = _peaks()
    achieved = att_bytes / (kd_ms / 1e3) / 1e9
    cpu = None if args.no_cpu_baseline else cpu_baseline_cfg2()
    line = {"metric": METRIC2, "value": c["B"] / (ms_step / 1e3), "unit": "tokens/s",
            "n_gpus": 1, "steps": K, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": _cfg2_config(),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": f"of {peak_kind}",
                         "kernel": "kd_kernel (split-KV decode), hot + selected launches",
                         "bytes_per_step": att_bytes, "kernel_ms_per_step": kd_ms,
                         "traffic": (att_bytes * NCU_TRAFFIC_RATIO_KD_CFG2
                                     if NCU_TRAFFIC_RATIO_KD_CFG2 else None)},
            "refetch": {"chunks_per_step": refetched, "bytes_per_step": refetch_bytes,
                        "chunks_selected_per_step": c["k_sel"] * c["L"],
                        "copy_stream_ms_per_step": copy_ms,
                        "copy_gbs": refetch_bytes / max(copy_ms, 1e-9) / 1e6,
                        "hot_attention_ms_per_step": hot_ms,
                        "attention_ms_per_step": kd_ms,
                        "exposed_ms_per_step": exposed_ms,
                        "hidden": exposed_ms <= 0.05 * ms_step,
                        "exposed_note": "compute-stream gap between the hot-chunk attention "
                                        "and the fold of the selected chunks, summed over "
                                        "layers (host wait for the indices + copies)"},
            "cpu_baseline": cpu and {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind",
                                                           "sample")},
            "e2e": {"value": c["B"] / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": qs[0].numel() * 2,
                    "d2h_bytes_per_step": out.numel() * 2},
            "clocks": clocks.summary(), "gpu_launches": launches}
    if not args.no_reference_gpu:
        line["reference_gpu"] = reference_gpu_cfg2(layers[0], qs[0, 0])
    del layers
    return line


def reference_gpu_cfg2(lay, q, steps: int = 10, warmup: int = 3):
    """One layer's attention of the tiered decode on the reference's Triton
    kernel (``halo/triton_chunked.py:47-138``): the 16 chunks a step attends
    (8 hot + the 8 in the refetch slots, 16384 rows) staged in one buffer,
    one ``update_chunk`` over it, against this build's split-KV decode over
    the same chunks in place."""
    import torch
    from halo_b200 import ops
    RT, why = _reference_triton()
    if RT is None:
        return {"unavailable": why}
    C = lay.C
    ks = [lay.k_hot] + [lay.k_slots[i] for i in range(lay.n_slots)]
    vs = [lay.v_hot] + [lay.v_slots[i] for i in range(lay.n_slots)]
    k = torch.cat(ks, dim=2)
    v = torch.cat(vs, dim=2)
    B, H, D = q.shape
    T = k.shape[2]
    scale = 1.0 / (D ** 0.5)
    q_pos = torch.full((B,), T - 1, dtype=torch.int64, device=q.device)
    nbytes = 2 * k.numel() * k.element_size()
    chunks = [(k[:, :, a:a + C], v[:, :, a:a + C], a, False) for a in range(0, T, C)]
    table = ops.ChunkTable(chunks)
    out = torch.empty(B, H, D, device=q.device)
    lse = torch.empty(B, H, device=q.device)

    def ref():
        m, l, o = RT.init_acc(B=B, H=H, D_v=D, device=q.device)
        RT.update_chunk(q=q, k=k, v=v, m=m, l=l, o=o, scale=scale, chunk_start=0, q_pos=q_pos,
                        apply_causal=False)
        return RT.finalize(m=m, l=l, o=o, out_dtype=torch.float32)

    def ours():
        ops.chunked_decode(q, table, scale=scale, out=out, lse=lse)
        return out

    try:
        ms_r, o_r = _time_events(ref, steps, warmup)
    except Exception as e:          # noqa: BLE001 - reported in the line
        return {"unavailable": f"reference Triton kernel failed: {type(e).__name__}: {e}"}
    ms_o, o_o = _time_events(ours, steps, warmup)
    return {"impl": "reference halo/triton_chunked.py (unmodified, baseline/_ref), Triton on "
                    "this B200",
            "workload": f"one layer's attended chunks: B{B}, {H}/{k.shape[1]} heads, {T} rows",
            "reference_ms_per_layer": ms_r, "reference_gbs": nbytes / (ms_r / 1e3) / 1e9,
            "ours_ms_per_layer": ms_o, "ours_gbs": nbytes / (ms_o / 1e3) / 1e9,
            "max_abs_vs_ours": (o_r - o_o).abs().max().item(), "steps": steps,
            "call": "init_acc + update_chunk over the staged rows + finalize"}


def run_reference_cfg2(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cpu = cpu_baseline_cfg2(budget_s=max(10.0, 150.0 / max(1, args.steps + args.warmup)))
    v = cpu["value"]
    line = {"impl": "reference", "metric": METRIC2, "value": v, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cpu["s_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": _cfg2_config(),
            "cpu_baseline": {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- cfg4 (KIVI)
CFG4 = dict(B=4, H=32, H_kv=8, D=128, T=65536, bits=2, group=32, recent=128)
METRIC4 = "KIVI 2-bit decode tokens/s & achieved HBM GB/s (packed bytes), B4 x 64K ctx, 1 B200"


def _outlier_keys(k, seed: int):
    """Scale 4 seeded channels of every KV head by 10 (outlier key channels)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    for h in range(k.shape[1]):
        idx = torch.randperm(k.shape[-1], generator=g)[:4].to(k.device)
        k[:, h, :, idx] *= 10
    return k


def _cfg4_inputs(dev, rows=None, batch=None):
    import torch
    c = CFG4
    B = c["B"] if batch is None else batch
    T = c["T"] if rows is None else rows
    g = torch.Generator(device=dev).manual_seed(4)
    k = torch.randn(B, c["H_kv"], T, c["D"], device=dev, generator=g)
    v = torch.randn(B, c["H_kv"], T, c["D"], device=dev, generator=g)
    q = torch.randn(B, c["H"], 1, c["D"], device=dev, generator=g)
    k = _outlier_keys(k, 44)
    return q.half(), k.half(), v.half()


def _cfg4_bytes():
    """Packed bytes the fused kernel must read per step: 2-bit codes plus an
    fp16 scale and zero per group of 32, for K and V, over the quantised
    prefix."""
    c = CFG4
    rows = c["T"] - c["recent"]
    per_row = c["D"] * c["bits"] // 8 + (c["D"] // c["group"]) * 2 * 2
    return 2 * c["B"] * c["H_kv"] * rows * per_row


def _cfg4_config():
    c = CFG4
    return {"workload": "cfg4: KIVI 2-bit decode, B4, 32 q-heads / 8 KV heads, head_dim 128, "
                        "65536 ctx (65408 quantised + 128 fp16 recent), group 32, fp16 "
                        "scale/zero, keys with 4 outlier channels x10 per head",
            "global_batch": c["B"], "seq_len": c["T"], "parallelism": "single GPU",
            "l2": "packed prefix %.0f MB > L2 (126 MB); no flush" % (_cfg4_bytes() / 1e6)}


def cpu_baseline_cfg4(budget_s: float = 15.0):
    """The reference's CPU decode step for cfg4 -- dequantise the whole
    prefix (its update() does so on every call) and attend in fp32 -- through
    the oracle port, on a sample of rows of one batch element, scaled."""
    import torch
    from oracle import attention as OA
    from oracle import kivi as OK
    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG4

    def prepare(rows):
        q, k, v = _cfg4_inputs(torch.device("cpu"), rows=rows, batch=1)
        return (q.float(),
                OK.quantize_per_group(k.float().numpy(), bits=2, group_size=32, dtype="f16"),
                OK.quantize_per_group(v.float().numpy(), bits=2, group_size=32, dtype="f16"))

    def run(prep):
        q, (ck, sk, zk), (cv, sv, zv) = prep
        t0 = time.perf_counter()
        kd = torch.from_numpy(OK.dequantize_per_group(ck, sk, zk, dtype="f16"))
        vd = torch.from_numpy(OK.dequantize_per_group(cv, sv, zv, dtype="f16"))
        OA.chunk_attention(q, kd, vd)
        return time.perf_counter() - t0

    t1 = run(prepare(1024))
    rows = int(max(1024, min(c["T"], budget_s / 3 / max(t1, 1e-4) * 1024)))
    rows = rows // 1024 * 1024
    prep = prepare(rows)
    t = statistics.median(run(prep) for _ in range(3))
    step_s = t * (c["T"] / rows) * c["B"]
    return {"value": c["B"] / step_s, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"1 of {c['B']} batch rows x {rows} of {c['T']} tokens (dequantise K and "
                      f"V + fp32 attention), median of 3, scaled x{c['B'] * c['T'] / rows:.0f}",
            "s_per_step": step_s}


def run_ours_cfg4(args):
    import torch
    from halo_b200 import _lib as L
    from halo_b200.baselines.kivi_cache import KIVICache
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("cfg4 runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = CFG4
    q, k, v = _cfg4_inputs(dev)
    cache = KIVICache(bits=c["bits"], group_size=c["group"], residual_length=c["recent"],
                      fused_attention=True)
    cache.update(k, v, layer_idx=0)
    del k, v
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        cache.compute_attention(q, layer_idx=0)
    K = args.steps
    # device throughput: events only around the loop (the merge kernel is a
    # dependent launch; an event in between would cancel its early launch)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    n0 = L.launch_count()
    with ClockSampler(0) as clocks:
        t0.record()
        for i in range(K):
            cache.compute_attention(q, layer_idx=0)
        t1.record()
        torch.cuda.synchronize()
    launches = L.launch_count() - n0
    ms_step = t0.elapsed_time(t1) / K
    # roofline pass: the same K steps with events around the fused kernel
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    for e in ev_b + ev_e:
        e.record()
    torch.cuda.synchronize()
    for i in range(K):
        cache.compute_attention(q, layer_idx=0, events=(ev_b[i].cuda_event, ev_e[i].cuda_event))
    torch.cuda.synchronize()
    kk_ms = sum(ev_b[i].elapsed_time(ev_e[i]) for i in range(K)) / K

    q_host = q.cpu().pin_memory()
    out_host = torch.empty(c["B"], c["H"], 1, c["D"], dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        o = cache.compute_attention(q_dev, layer_idx=0)
        out_host.copy_(o, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(3):
        e2e_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / K

    nbytes = _cfg4_bytes()
    peak, peak_kind = _peaks()
    achieved = nbytes / (kk_ms / 1e3) / 1e9
    cpu = None if args.no_cpu_baseline else cpu_baseline_cfg4()
    line = {"metric": METRIC4, "value": c["B"] / (ms_step / 1e3), "unit": "tokens/s",
            "n_gpus": 1, "steps": K, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic", "config": _cfg4_config(),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": f"of {peak_kind}",
                         "kernel": "kk_kernel (fused 2-bit dequant-and-attend)",
                         "bytes_per_launch": nbytes, "traffic": nbytes * NCU_TRAFFIC_RATIO_KK},
            "cpu_baseline": cpu and {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind",
                                                           "sample")},
            "e2e": {"value": c["B"] / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": q.numel() * q.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "clocks": clocks.summary(), "gpu_launches": launches}
    del cache
    return line


def run_reference_cfg4(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cpu = cpu_baseline_cfg4(budget_s=max(10.0, 150.0 / max(1, args.steps + args.warmup)))
    v = cpu["value"]
    line = {"impl": "reference", "metric": METRIC4, "value": v, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cpu["s_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic", "config": _cfg4_config(),
            "cpu_baseline": {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- cfg3 (chunked prefill)
CFG3 = dict(B=1, H=32, H_kv=8, D=128, T=131072, slice=4096)
METRIC3 = "chunked-prefill attention: prompt tokens/s & TFLOP/s (causal), 131072 tokens, 1 B200"


def _cfg3_flops(T=None):
    """Algorithmic causal FLOPs of one layer's prefill: 4 H D per visible
    (query, key) pair, T (T + 1) / 2 pairs."""
    c = CFG3
    T = c["T"] if T is None else T
    return 4 * c["H"] * c["D"] * T * (T + 1) // 2


def _cfg3_config():
    c = CFG3
    name = ("cfg3: chunked prefill of a 131072-token prompt" if c["T"] == 131072 else
            f"cfg3 reduced to a {c['T']}-token prompt (profiling case)")
    return {"workload": f"{name} in {c['T'] // c['slice']} slices of {c['slice']} against the "
                        "accumulated KV (causal), 32 q-heads / 8 KV heads, head_dim 128, B1, "
                        "keys with 4 outlier channels x10 per head",
            "global_batch": c["B"], "seq_len": c["T"], "slice": c["slice"],
            "parallelism": "single GPU",
            "l2": "Q/K/V/out %.2f GB per step > L2 (126 MB); no flush" %
                  ((2 * c["H"] + 2 * c["H_kv"]) * c["T"] * c["D"] * 2 / 1e9)}


def _cfg3_inputs(dev, T=None, H=None, H_kv=None):
    import torch
    c = CFG3
    T = c["T"] if T is None else T
    H = c["H"] if H is None else H
    H_kv = c["H_kv"] if H_kv is None else H_kv
    g = torch.Generator(device=dev).manual_seed(3)
    q = torch.randn(c["B"], H, T, c["D"], device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(c["B"], H_kv, T, c["D"], device=dev, generator=g)
    v = torch.randn(c["B"], H_kv, T, c["D"], device=dev, generator=g, dtype=torch.bfloat16)
    k = _outlier_keys(k, 33).bfloat16()
    return q, k, v


def cpu_baseline_cfg3(budget_s: float = 15.0):
    """The reference's CPU path for one slice (fp32 attention of the slice's
    queries over the accumulated keys, causal), through the oracle port, on a
    sample: one KV head group and the last rows of the last slice, scaled by
    the causal pair count of the whole prompt."""
    import torch
    from oracle import attention as OA
    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG3
    G = c["H"] // c["H_kv"]
    T = c["T"]

    def run(n_q):
        q, k, v = _cfg3_inputs(torch.device("cpu"), T=T, H=G, H_kv=1)
        qs = q[..., T - n_q:, :]
        t0 = time.perf_counter()
        OA.chunked_attention(qs, [(k, v, 0, True)], q_pos=T - n_q)
        return time.perf_counter() - t0, n_q * T - n_q * (n_q - 1) // 2

    t1, p1 = run(16)
    n_q = int(max(256, min(c["slice"], 16 * budget_s / 3 / max(t1, 1e-3))))
    t, pairs = run(n_q)
    s_per_pair_group = t / pairs
    step_s = s_per_pair_group * (T * (T + 1) // 2) * c["H_kv"]
    return {"value": T / step_s, "unit": "prompt tokens/s", "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"last {n_q} queries of the prompt x 1 of {c['H_kv']} KV head groups "
                      f"against all {T} keys (causal, fp32), time scaled by causal pair count "
                      f"x{(T * (T + 1) // 2) * c['H_kv'] / pairs:.0f}",
            "s_per_step": step_s}


def run_ours_cfg3(args):
    import torch
    from halo_b200 import _lib as L
    from halo_b200 import ops
    if args.gpus != 1 or int(os.environ.get("WORLD_SIZE", "1")) != 1:
        raise SystemExit("cfg3 runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    c = CFG3
    T, S = c["T"], c["slice"]
    q, k, v = _cfg3_inputs(dev)
    out = torch.empty_like(q)
    lse = torch.empty(c["B"], c["H"], T, device=dev)

    def step(qq, kk, vv, oo):
        for s0 in range(0, T, S):
            ops.prefill_attention(qq[:, :, s0:s0 + S], [(kk[..., :s0 + S, :], vv[..., :s0 + S, :],
                                                         0, True)],
                                  query_pos_offset=s0, out=oo[:, :, s0:s0 + S],
                                  lse=lse[:, :, s0:s0 + S])

    for _ in range(args.warmup):
        step(q, k, v, out)
    torch.cuda.synchronize()
    K = args.steps
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = L.launch_count()
    with ClockSampler(0) as clocks:
        t0.record()
        for _ in range(K):
            step(q, k, v, out)
        t1.record()
        torch.cuda.synchronize()
    launches = L.launch_count() - n0
    ms_step = t0.elapsed_time(t1) / K

    # e2e: the step's Q/K/V come from pinned host memory, the output goes back
    qh, kh, vh = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def e2e_step():
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        step(qd, kd, vd, out)
        oh.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n_e2e = max(1, min(K, 5))
    e0.record()
    for _ in range(n_e2e):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / n_e2e

    flops = _cfg3_flops()
    tflops = flops / (ms_step / 1e3) / 1e12
    peak, peak_kind = _tensor_peak()
    cpu = None if args.no_cpu_baseline else cpu_baseline_cfg3()
    line = {"metric": METRIC3, "value": T / (ms_step / 1e3), "unit": "prompt tokens/s",
            "n_gpus": 1, "steps": K, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": _cfg3_config(),
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": tflops / peak, "peak_kind": f"of {peak_kind}",
                         "kernel": "kp3_kernel (tcgen05 chunked-prefill attention) + v16_kernel "
                                   "(fp16 copy of V) per slice",
                         "flops_per_step": flops, "traffic": None,
                         "note": "algorithmic causal FLOPs; the kernel also runs the masked "
                                 "halves of diagonal tiles"},
            "cpu_baseline": cpu and {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind",
                                                           "sample")},
            "e2e": {"value": T / (e2e_ms / 1e3), "unit": "prompt tokens/s",
                    "h2d_bytes_per_step": (q.numel() + k.numel() + v.numel()) * 2,
                    "d2h_bytes_per_step": out.numel() * 2},
            "clocks": clocks.summary(), "gpu_launches": launches}
    return line


def run_reference_cfg3(args):
    if int(os.environ.get("RANK", "0")) != 0:
        return
    cpu = cpu_baseline_cfg3(budget_s=max(10.0, 150.0 / max(1, args.steps + args.warmup)))
    v = cpu["value"]
    line = {"impl": "reference", "metric": METRIC3, "value": v, "unit": "prompt tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cpu["s_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": _cfg3_config(),
            "cpu_baseline": {kk: cpu[kk] for kk in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": v, "unit": "prompt tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours_all(args):
    """The headline decode line; with one GPU, the other three workloads
    measured after it (each with its own roofline, CPU baseline, e2e and
    clock record) under ``workloads``."""
    import torch
    line = run_ours_cfg5(args)
    if int(os.environ.get("WORLD_SIZE", "1")) != 1 or args.gpus != 1 or args.no_workloads:
        return line
    sub = argparse.Namespace(**vars(args))
    sub.steps = min(args.steps, 20)
    sub.warmup = max(3, min(args.warmup, 5))
    workloads = {}
    for name, fn in (("cfg4", run_ours_cfg4), ("cfg3", run_ours_cfg3), ("cfg2", run_ours_cfg2)):
        torch.cuda.empty_cache()
        try:
            workloads[name] = fn(sub if name != "cfg4" else args)
        except Exception as e:      # noqa: BLE001 - one workload failing is reported, not fatal
            workloads[name] = {"error": f"{type(e).__name__}: {e}"}
    line["workloads"] = workloads
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all", "cfg5", "cfg4", "cfg3", "cfg2"], default="all")
    ap.add_argument("--seq-len", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-workloads", action="store_true",
                    help="headline decode only (skip cfg2/3/4 in the default run)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's Triton kernel")
    ap.add_argument("--eager", action="store_true",
                    help="time the decode step as eager calls instead of CUDA graph replays")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.seq_len and args.workload in ("cfg5", "all"):
        n = args.gpus * CFG5["chunk"]
        if args.seq_len % n:
            raise SystemExit(f"--seq-len must be a multiple of {n}")
        CFG5["T"] = args.seq_len
    if args.seq_len and args.workload == "cfg3":
        if args.seq_len % CFG3["slice"]:
            raise SystemExit(f"--seq-len must be a multiple of {CFG3['slice']}")
        CFG3["T"] = args.seq_len
    if args.layers:
        CFG2["L"] = args.layers
    if args.impl == "reference":
        if args.workload == "cfg4":
            return run_reference_cfg4(args)
        if args.workload == "cfg2":
            return run_reference_cfg2(args)
        if args.workload == "cfg3":
            return run_reference_cfg3(args)
        return run_reference(args)
    runner = {"cfg4": run_ours_cfg4, "cfg2": run_ours_cfg2, "cfg3": run_ours_cfg3,
              "cfg5": run_ours_cfg5, "all": run_ours_all}[args.workload]
    line = runner(args)
    if line is not None:
        print(json.dumps(line), flush=True)
    return line


if __name__ == "__main__":
    main()

"""Benchmark: fused causal top-K retrieval + sparse attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wayfinder|reference] [--config cfg2]

One rank per GPU (torchrun for N > 1).  Each rank runs its own batch element of
the workload (batch sharding, no collective on the data path: weak scaling).
Prints ONE JSON line on rank 0.

Timing: W untimed warm-up steps, then exactly K steps between a barrier +
cuda.synchronize() on both sides.  Before every timed step a 256 MiB memset
(2x the 126 MB L2) flushes the cache; each step is bracketed by CUDA events on
the launching stream, so the flush is outside the timed region.  The per-rank
time is the sum of step times; the job time is the max over ranks.

``value`` is queries/s (token positions B*T per step, all ranks) with inputs
resident in HBM; ``e2e`` is the same metric through the public API with the
inputs copied from pinned host memory and the outputs read back every step.
``--impl reference`` times the CPU oracle port of the reference path on the
host cores instead (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from wayfinder_attention_b200.workloads import CONFIGS, Workload, make_inputs, scaled, to_device  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
E2E_CHUNKS = 4  # query-row chunks of the host pipeline
L2_FLUSH_BYTES = 256 << 20
METRIC = "fused top-K+sparse-attn fwd queries/s @T=16K,K=128"
# dram__bytes_read.sum + dram__bytes_write.sum of one sparse-attention launch: constants
# from the named ncu captures (not measured in this run).
ATTN_DRAM_BYTES = {"cfg2": 62.0e6, "cfg4": 7.89e9 + 0.54e9, "cfg5": 3.48e9 + 1.06e9}
ATTN_DRAM_SOURCE = {"cfg2": "profiles/sparse_attention_cfg2.md", "cfg4": "profiles/sparse_attention_cfg4_cfg5.md",
                    "cfg5": "profiles/sparse_attention_cfg4_cfg5.md"}


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


_JSON_OUT = None


def emit(line: dict) -> None:
    """Write the one JSON result line to the process's real stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def claim_stdout() -> None:
    """Route fd 1 to stderr so library banners (NCCL prints its version on stdout)
    cannot interleave with the JSON line, which goes to a private copy of stdout."""
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class ClockSampler:
    """Samples SM clock and clock-event reasons during the timed region.

    Reads NVML (read-only queries) every ~2 ms from a background thread, so even a
    timed region of a few tens of milliseconds gets samples; without NVML the
    summary reports no samples.
    """

    REASONS = {
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = False
        self._thread = None

    def _run(self):
        import pynvml

        h = None
        try:  # map the CUDA device to NVML through its PCI address (CUDA_VISIBLE_DEVICES may renumber)
            pr = torch.cuda.get_device_properties(self.gpu_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu_index)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        while not self._stop:
            self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
            r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            for name, bit in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
            time.sleep(0.002)

    def __enter__(self):
        try:
            import pynvml
            import threading

            pynvml.nvmlInit()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
            t0 = time.time()  # the first sample lands before the timed region starts
            while not self.samples and self._thread.is_alive() and time.time() - t0 < 2.0:
                time.sleep(0.001)
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=2)
        return False

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sample_rows(T: int, n: int) -> np.ndarray:
    """Evenly spread query rows: their mean causal length is T/2, like the full job."""
    return np.unique(np.linspace(0, T - 1, n).astype(np.int64))


def time_cpu_reference(w: Workload, inputs: dict, n_rows: int, chunk: int | None = None) -> tuple[float, int]:
    """Seconds for the reference's CPU execution restated in torch (``oracle/reference_torch``:
    row-blocked fp32 bmm + topk, (B,H,n,K,D) gather, softmax, weighted sum) on ``n_rows``
    sampled rows of batch element 0, all in one call like the reference's (or ``chunk``
    rows at a time), all host threads."""
    chunk = chunk or n_rows
    from oracle import reference_torch  # CPU baseline leg only

    x = {k: v[:1].float().contiguous() for k, v in inputs.items()}
    rows = torch.from_numpy(cpu_sample_rows(w.T, n_rows))
    t0 = time.perf_counter()
    for a in range(0, rows.numel(), chunk):
        reference_torch.fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], w.K,
                                               w.D ** -0.5, rows[a:a + chunk])
    return time.perf_counter() - t0, rows.numel()


def run_reference_arm(args, w: Workload) -> None:
    rank, _, world = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    inputs = make_inputs(w, B=1)
    n_rows = args.cpu_rows
    for _ in range(max(args.warmup, 0)):
        time_cpu_reference(w, inputs, min(n_rows, 64))
    secs = []
    for _ in range(args.steps):
        s, n = time_cpu_reference(w, inputs, n_rows)
        secs.append(s)
    total = sum(secs)
    value = n * args.steps / total
    line = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seed 45)",
        "config": {"workload": w.name, "B": 1, "H": w.H, "T": w.T, "D": w.D, "d_A": w.R, "K": w.K,
                   "sample_rows_per_step": n},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": threads, "kind": "port",
                         "cpu": cpu_model(),
                         "sample": f"{n} evenly spaced query rows of one T={w.T} sequence per step "
                                   f"(retrieval over their causal prefixes + attention over {w.H} heads), "
                                   "the reference's torch CPU operations restated (oracle/reference_torch.py)"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="wayfinder", choices=["wayfinder", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--cpu-rows", type=int, default=1024, help="rows per reference-arm step")
    ap.add_argument("--cpu-baseline-rows", type=int, default=4096, help="rows of the one-off cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dense", action="store_true")
    ap.add_argument("--no-decoder", action="store_true", help="skip the whole-decoder prefill measurements")
    ap.add_argument("--profile-op", choices=["topk", "attention", "both", "fused", "backward", "projection"],
                    help="profiling mode: run only this op --iters times on --config (L2 flushed before each) "
                         "and print 'ok'; for ncu captures")
    ap.add_argument("--iters", type=int, default=3, help="calls in --profile-op mode")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="skip the cfg4 / cfg5 measurements (and the sequence-sharded cfg4 run at N > 1)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    claim_stdout()

    w = CONFIGS[args.config]
    if args.profile_op:
        profile_op(args.profile_op, w, args.iters)
        return
    if args.impl == "reference":
        run_reference_arm(args, w)
        return

    import torch.distributed as dist

    from wayfinder_attention_b200 import _lib
    from wayfinder_attention_b200.causal_topk import _launch_topk
    from wayfinder_attention_b200.fused_sparse import _launch_attention, fused_sparse_attention

    rank, local_rank, world = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    if args.config == "cfg4" and world > 1:
        run_sequence_sharded(args, w, rank, world, dev)
        dist.barrier()
        dist.destroy_process_group()
        return

    # batch sharding: each rank owns batch element(s) `rank` of a global batch of world * B
    w_local = scaled(w, B=w.B)
    host = make_inputs(w_local, batch_offset=rank)
    x = to_device(host, dev)
    K = w.K
    scale = w.D ** -0.5
    idx = torch.empty(w.B, w.T, min(K, w.T), dtype=torch.int32, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], K, scale)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()

    # timed region: the product call (wf_fused_sparse_attention through the Python API)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    torch.cuda.reset_peak_memory_stats(dev)
    mem0 = torch.cuda.memory_allocated(dev)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        barrier()
    peak_mb = (torch.cuda.max_memory_allocated(dev) - mem0) / 2**20
    total_ms = sum(a.elapsed_time(b) for a, b in ev)

    # per-kernel durations for the roofline: the same kernels launched one after the other
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    for i in range(args.steps):
        flush.zero_()
        kev[i][0].record(stream)
        _launch_topk(x["q_addr"], x["k_addr"], K, "reference", out=idx)
        kev[i][1].record(stream)
        _launch_attention(x["q"], x["k"], x["v"], idx, scale, mask_negative=False, out_dtype=None)
        kev[i][2].record(stream)
    torch.cuda.synchronize()
    topk_tot = sum(e[0].elapsed_time(e[1]) for e in kev)
    attn_tot = sum(e[1].elapsed_time(e[2]) for e in kev)
    ceiling_gbs = gather_ceiling(x, idx, args.steps, flush, stream)
    bulk = bulk_gather_rates(x, idx, args.steps, flush, stream)
    t = torch.tensor([total_ms, topk_tot, attn_tot], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, topk_tot, attn_tot = t.tolist()
    ms_per_step = total_ms / args.steps
    queries = w.B * w.T * world
    value = queries / (ms_per_step / 1e3)

    # end-to-end through the public API with pinned host tensors in and out.
    # Headline: HostFusedSparseAttention (upload, retrieval/attention and download
    # overlapped on three streams).  Also reported: the serial form (upload all,
    # fused_sparse_attention, download all).
    from wayfinder_attention_b200.host_pipeline import HostFusedSparseAttention

    pin = {k: (v.transpose(1, 2).contiguous() if v.dim() == 4 else v.contiguous()).pin_memory()
           for k, v in host.items()}
    dbuf = {k: torch.empty_like(v, device=dev) for k, v in pin.items()}
    out_h = torch.empty(w.B, w.T, w.H, w.D, dtype=w.dtype).pin_memory().transpose(1, 2)
    idx_h = torch.empty(w.B, w.T, min(K, w.T), dtype=torch.int32).pin_memory()
    out_hs = torch.empty(w.B, w.H, w.T, w.D, dtype=w.dtype).pin_memory()  # serial form: the op's own layout
    h2d = sum(v.numel() * v.element_size() for v in pin.values())
    d2h = out_h.numel() * out_h.element_size() + idx_h.numel() * idx_h.element_size()
    host_op = HostFusedSparseAttention(K, scale, chunks=E2E_CHUNKS, device=dev)
    host_op_out = HostFusedSparseAttention(K, scale, chunks=E2E_CHUNKS, device=dev, download_indices=False)

    def e2e_serial():
        for k_ in pin:
            dbuf[k_].copy_(pin[k_], non_blocking=True)
        q, k, v = (dbuf[n].transpose(1, 2) for n in ("q", "k", "v"))
        out, ii = fused_sparse_attention(dbuf["q_addr"], dbuf["k_addr"], q, k, v, K, scale)
        out_hs.copy_(out, non_blocking=True)
        idx_h.copy_(ii, non_blocking=True)

    def e2e_pipelined():
        host_op(pin["q_addr"], pin["k_addr"], *(pin[n].transpose(1, 2) for n in ("q", "k", "v")),
                out=out_h, idx_out=idx_h)

    def e2e_pipelined_out_only():
        host_op_out(pin["q_addr"], pin["k_addr"], *(pin[n].transpose(1, 2) for n in ("q", "k", "v")), out=out_h)

    def time_e2e(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            e_ev[i][0].record(stream)
            fn()
            e_ev[i][1].record(stream)
        torch.cuda.synchronize()
        barrier()
        t_ = torch.tensor([sum(a.elapsed_time(b) for a, b in e_ev)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        return t_.item() / args.steps

    # The copies alone, as the pipelined call issues them (uploads on one stream,
    # downloads on another, both directions at once), on every rank at the same time:
    # the host-link ceiling of the e2e number.
    s_up, s_dn = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    dn_src = torch.empty(d2h, dtype=torch.uint8, device=dev)
    dn_dst = torch.empty(d2h, dtype=torch.uint8).pin_memory()

    def copies_only():
        s_up.wait_stream(stream)
        s_dn.wait_stream(stream)
        with torch.cuda.stream(s_up):
            for k_ in pin:
                dbuf[k_].copy_(pin[k_], non_blocking=True)
        with torch.cuda.stream(s_dn):
            dn_dst.copy_(dn_src, non_blocking=True)
        stream.wait_stream(s_up)
        stream.wait_stream(s_dn)

    e2e_serial_ms = time_e2e(e2e_serial)
    e2e_ms_step = time_e2e(e2e_pipelined)
    e2e_out_only_ms = time_e2e(e2e_pipelined_out_only)
    copy_ms = time_e2e(copies_only)
    e2e_value = queries / (e2e_ms_step / 1e3)

    # the one data path with a collective: cfg4's long sequence over all ranks, and the
    # same call on one GPU (rank 0, the others wait) for the strong-scaling efficiency
    seq = None
    batch_sharded = {}
    if world > 1 and not args.no_extra_configs:
        seq = sequence_sharded_measure(CONFIGS["cfg4"], rank, world, dev, max(3, args.steps // 4), 3)
        if rank == 0:
            one = config_measurement("cfg4", dev, flush, max(3, args.steps // 4))
            seq["single_gpu_ms"] = one["ms"]
            seq["strong_scaling_efficiency"] = one["ms"] / (world * seq["ms"])
        dist.barrier()
        # batch-sharded configs: cfg5 (B=64, K=128) and the cfg3 decoder (B=8), each rank
        # its share of the batch, no collective; the job time is the slowest rank's
        w5 = CONFIGS["cfg5"]
        if w5.B % world == 0:
            m5 = config_measurement("cfg5", dev, flush, 3, B=w5.B // world, seed=45 + rank)
            t5 = torch.tensor([m5["ms"]], dtype=torch.float64, device=dev)
            dist.all_reduce(t5, op=dist.ReduceOp.MAX)
            batch_sharded["cfg5_k128"] = {"ms": t5.item(), "B_per_rank": w5.B // world,
                                          "queries_per_s": w5.B * w5.T / (t5.item() / 1e3)}
        if 8 % world == 0 and not args.no_decoder:
            d3 = decoder_forward(8 // world, 4096, flush, 5, dev)
            t3 = torch.tensor([d3["ms"]], dtype=torch.float64, device=dev)
            dist.all_reduce(t3, op=dist.ReduceOp.MAX)
            batch_sharded["cfg3_decoder"] = {"ms": t3.item(), "B_per_rank": 8 // world,
                                             "tokens_per_s": 8 * 4096 / (t3.item() / 1e3)}
        dist.barrier()

    result = None
    if rank == 0:
        peaks, peak_kind = load_peaks()
        attn_ms_launch = attn_tot / args.steps
        topk_ms_launch = topk_tot / args.steps
        gathered = w.gathered_bytes()
        achieved_gbs = gathered / (attn_ms_launch / 1e3) / 1e9
        hbm = float(peaks["hbm_gbs"])
        tens = float(peaks["bf16_tflops"]) * 1e12
        roof_s = max(w.score_flops() / tens, gathered / (hbm * 1e9))
        roof_l2_s = max(w.score_flops() / tens, gathered / (ceiling_gbs * 1e9))
        dram = ATTN_DRAM_BYTES.get(w.name)
        result = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else str(w.dtype).split(".")[-1],
            "data": "synthetic (seeded N(0,1) q/k/v, N(0,1/32) addresses)",
            "config": {"workload": w.name, "B": w.B, "H": w.H, "T": w.T, "D": w.D, "d_A": w.R, "K": K,
                       "global_batch": w.B * world, "seq_len": w.T,
                       "parallelism": f"batch-sharded x{world} (no collective)",
                       "l2": "flushed before every timed step (256 MiB memset, outside the events)"},
            "latency_ms": ms_per_step,
            "query_heads_per_s": value * w.H,
            "kernels_ms": {"causal_topk": topk_ms_launch, "sparse_attention": attn_ms_launch,
                           "note": "each kernel timed alone, same launches as the step"},
            # cfg2's K/V (33.5 MB) stay in the 126 MB L2, so the gathers are served from L2:
            # the binding resource is the L2 -> SM load stream, whose ceiling for this
            # access pattern is measured in this run by wf_gather_rows_bench (same loads,
            # same indices, no math).  The HBM view uses the DRAM bytes of a named capture.
            "roofline": {"kernel": "sparse_attention", "bound": "l2", "achieved": achieved_gbs,
                         "peak": ceiling_gbs, "unit": "GB/s", "frac": achieved_gbs / ceiling_gbs,
                         "peak_kind": "measured in this run (wf_gather_rows_bench: the kernel's K/V row loads "
                                      "over the same indices, nothing computed)",
                         "traffic": dram,
                         "traffic_source": (ATTN_DRAM_SOURCE.get(w.name, "") +
                                            " (constant from that ncu capture, not measured in this run)"),
                         "hbm": {"achieved": (dram / (attn_ms_launch / 1e3) / 1e9) if dram else None, "peak": hbm,
                                 "frac": (dram / (attn_ms_launch / 1e3) / 1e9 / hbm) if dram else None,
                                 "peak_kind": peak_kind},
                         "alternative_bulk_copy": bulk,
                         "note": "achieved = gathered K/V bytes (2*B*H*T*K*D*2) / kernel time; "
                                 "alternative_bulk_copy: the same rows through cp.async.bulk into shared memory"},
            "path_roofline": {"roofline_ms": roof_l2_s * 1e3, "frac": roof_l2_s * 1e3 / ms_per_step,
                              "score_tflops_achieved": w.score_flops() / (topk_ms_launch / 1e3) / 1e12,
                              "definition": "max(score FLOPs / bf16 peak, gathered bytes / measured gather "
                                            "ceiling) / latency",
                              "north_star_form": {"roofline_ms": roof_s * 1e3, "frac": roof_s * 1e3 / ms_per_step,
                                                  "definition": "max(score FLOPs / bf16 peak, gathered bytes / "
                                                                "HBM peak); above 1 because the gathers hit L2"}},
            "peak_mb": peak_mb,
            "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms_step, "api": "HostFusedSparseAttention (copies overlapped, "
                    f"{E2E_CHUNKS} row chunks)", "serial_ms_per_step": e2e_serial_ms,
                    "copies_only_ms_per_step": copy_ms,
                    "out_only_ms_per_step": e2e_out_only_ms,
                    "out_only_d2h_bytes_per_step": out_h.numel() * out_h.element_size(),
                    "host_link_gbs_per_rank": (h2d + d2h) / (copy_ms / 1e3) / 1e9,
                    "frac_of_copy_ceiling": copy_ms / e2e_ms_step,
                    "note": "copies_only: the same uploads and downloads on every rank at once, no kernels"},
            "gpu_launches": 4 * args.steps,  # per step: scoring, rescoring, finalisation, attention
            "clocks": clk.summary(),
        }
        if not args.no_dense:
            result["dense_sdpa"] = dense_baseline(w, x, flush, args.steps)
        if not args.no_decoder and args.config == "cfg2":
            # the reference publishes this model's forward latency (B=1, T=16384: 38.35 ms on an RTX 5090,
            # fp32 + TF32; dense flash 84.33 ms), and cfg3 is the same family at B=8, T=4096
            result["decoder_prefill"] = {
                "systems_T16384": decoder_forward(1, 16384, flush, 5, dev),
                "systems_T16384_dense": decoder_forward(1, 16384, flush, 5, dev, attention_type="dense_flash"),
                "cfg3_B8_T4096": decoder_forward(8, 4096, flush, 5, dev),
                "published_rtx5090_ms": {"wayfinder_T16384": 38.35, "dense_flash_T16384": 84.33},
            }
        if seq is not None:
            result["cfg4_sequence_sharded"] = seq
        if batch_sharded:
            result["batch_sharded"] = batch_sharded
        if world == 1 and not args.no_extra_configs:
            result["overlap_probe"] = overlap_probe(w, dev, flush, args.steps)
        if world == 1 and not args.no_extra_configs:
            # configurations whose K/V outgrow the 126 MB L2 (cfg4: 1.07 GB; cfg5: 2.1 GB per call)
            result["cfg4_single_gpu"] = config_measurement("cfg4", dev, flush, max(3, args.steps // 4))
            for name in ("cfg5_k64", "cfg5", "cfg5_k256"):
                result[name.replace("cfg5", "cfg5_k128") if name == "cfg5" else name] = config_measurement(
                    name, dev, flush, 3)
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(os.cpu_count() or 1)
            secs, n = time_cpu_reference(w, host, args.cpu_baseline_rows)
            result["cpu_baseline"] = {
                "value": n / secs, "unit": "queries/s", "cores": os.cpu_count() or 1, "kind": "port",
                "cpu": cpu_model(),
                "sample": f"{n} evenly spaced query rows of the T={w.T} sequence "
                          f"(retrieval + {w.H}-head attention) in one call, the reference's torch CPU operations "
                          "restated (oracle/reference_torch.py)",
            }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        emit(result)


def sequence_sharded_measure(w: Workload, rank: int, world: int, dev, steps: int, warmup: int,
                             transports=("peer", "nccl")) -> dict:
    """cfg4 on ``world`` ranks: query-row blocks cyclic over ranks, k_addr and K/V exchanged.

    For each K/V transport (copy-engine pulls from the peers' buffers, or NCCL
    all-gathers) returns the per-step time (max over ranks, CUDA events, L2 flushed
    before each step) and, for the limiter, the parts timed alone: the K/V
    exchange, the rank's retrieval (with its address all-gather) and its attention
    over landed K/V.  The first transport is the headline.
    """
    import torch.distributed as dist

    from wayfinder_attention_b200.sharding import (SequenceShardedAttention, _all_gather_rows, _chunked_attention,
                                                   gather_sequence, local_rows, sharded_causal_topk)

    tile = 256
    if w.T % (world * tile):
        raise SystemExit(f"T={w.T} is not a multiple of world*tile={world * tile}")
    full = device_inputs(w, dev)  # identical on every rank (same seed)
    rows = torch.from_numpy(local_rows(w.T, world, rank, tile)).to(dev)
    qa_l, ka_l = full["q_addr"][:, rows].contiguous(), full["k_addr"][:, rows].contiguous()
    q_l, k_l, v_l = (full[n].transpose(1, 2)[:, rows].contiguous().transpose(1, 2) for n in ("q", "k", "v"))
    del full
    torch.cuda.empty_cache()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for _ in range(2):  # warm-up (first collectives of a kind set up their channels)
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        for a, b in ev:
            flush.zero_()
            dist.barrier()  # all ranks enter the step together, outside the timed events
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        tot = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
        return tot.item() / steps

    kt, vt = k_l.transpose(1, 2), v_l.transpose(1, 2)
    k_addr = gather_sequence(ka_l, tile)
    idx = sharded_causal_topk(qa_l, k_addr, w.K, world, rank, tile)
    retrieval_ms = timed(lambda: sharded_causal_topk(qa_l, gather_sequence(ka_l, tile), w.K, world, rank, tile))
    kv_recv = 2.0 * (world - 1) / world * w.B * w.T * w.H * w.D * q_l.element_size()
    res = {"n_gpus": world, "kv_bytes_received_per_rank": kv_recv}
    for i, transport in enumerate(transports):
        op = SequenceShardedAttention(w.K, w.D ** -0.5, tile=tile, transport=transport)
        for _ in range(warmup):
            flush.zero_()
            op(qa_l, ka_l, q_l, k_l, v_l)
        torch.cuda.synchronize()
        with ClockSampler(int(os.environ.get("LOCAL_RANK", 0))) as clk:
            ms = timed(lambda: op(qa_l, ka_l, q_l, k_l, v_l))
        # the parts alone, same buffers and chunking as the op
        C = op._n_chunks(q_l.shape[2], world)
        Tc = q_l.shape[2] // C
        shape = (C, world, w.B, Tc, w.H, w.D)
        if transport == "peer":
            peer = op._peer
            side = torch.cuda.Stream(device=dev)

            def exchange():
                side.wait_stream(stream)
                peer.exchange(kt, vt, side)
                for e in peer.events:
                    stream.wait_event(e)

            kb, vb = peer.k_base, peer.v_base
        else:
            k_g, v_g = op._kg, op._vg

            def exchange():
                for c in range(C):
                    _all_gather_rows(kt[:, c * Tc:(c + 1) * Tc], world, None, k_g[c])
                    _all_gather_rows(vt[:, c * Tc:(c + 1) * Tc], world, None, v_g[c])

            kb, vb = k_g.data_ptr(), v_g.data_ptr()
        exchange_ms = timed(exchange)
        attention_ms = timed(lambda: _chunked_attention(q_l, idx, kb, vb, shape, w.D ** -0.5, tile, "reference",
                                                        None, None))
        op.close()
        r = {"ms": ms, "chunks": C, "clocks": clk.summary(),
             "parts_ms": {"kv_exchange": exchange_ms, "retrieval_with_addr_gather": retrieval_ms,
                          "attention": attention_ms},
             "kv_exchange_gbs_per_rank": kv_recv / (exchange_ms / 1e3) / 1e9}
        if i == 0:
            res.update(r)
            res["transport"] = transport
        else:
            res[transport] = r
    return res


def run_sequence_sharded(args, w: Workload, rank: int, world: int, dev) -> None:
    """cfg4 as the workload: one T=65536 sequence over the ranks (strong scaling)."""
    m = sequence_sharded_measure(w, rank, world, dev, args.steps, args.warmup)
    ms = m["ms"]
    if rank == 0:
        peaks, peak_kind = load_peaks()
        roof_ms = 1e3 * max(w.score_flops() / (float(peaks["bf16_tflops"]) * 1e12),
                            w.gathered_bytes() / (float(peaks["hbm_gbs"]) * 1e9)) / world
        emit({
            "metric": METRIC, "value": w.B * w.T / (ms / 1e3), "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, generated on device)",
            "config": {"workload": w.name, "B": w.B, "H": w.H, "T": w.T, "D": w.D, "d_A": w.R, "K": w.K,
                       "parallelism": f"query-row blocks of 256 cyclic over {world} ranks; "
                                      "k_addr and K/V all-gathered with NCCL",
                       "l2": "flushed before every timed step"},
            "path_roofline": {"roofline_ms_per_gpu": roof_ms, "frac": roof_ms / ms, "peak_kind": peak_kind},
            "parts_ms": m["parts_ms"], "transport": m["transport"], "nccl_transport": m.get("nccl"),
            "gpu_launches": (3 + m["chunks"]) * args.steps,  # per step: scoring, rescoring, finalisation, attention chunks
            "clocks": m["clocks"],
        })


def profile_op(op: str, w: Workload, iters: int) -> None:
    """One hot-path op ``iters`` times on seeded device inputs of ``w``, L2 flushed before each call.

    ``projection`` runs the fused address projection at the decoder's shape (32768 x 256
    bf16 hidden states, d_A = 32, both addresses).  Prints only a final ``ok``.
    """
    from wayfinder_attention_b200.causal_topk import causal_topk
    from wayfinder_attention_b200.fused_sparse import (_launch_attention_backward, fused_sparse_attention,
                                                       sparse_meat_attention)

    dev = torch.device("cuda:0")
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    if op == "projection":
        from wayfinder_attention_b200.address_projection import address_projection

        g = torch.Generator(device=dev).manual_seed(45)
        hid = torch.randn(32768, 256, generator=g, device=dev).to(torch.bfloat16)
        wgt = (torch.randn(64, 256, generator=g, device=dev) / 16).to(torch.bfloat16)
        bias = torch.zeros(64, dtype=torch.bfloat16, device=dev)
        for _ in range(iters):
            flush.zero_()
            address_projection(hid, wgt, bias, 32)
    else:
        x = device_inputs(w, dev)
        scale = w.D ** -0.5
        idx = causal_topk(x["q_addr"], x["k_addr"], w.K)
        for _ in range(iters):
            flush.zero_()
            if op in ("topk", "both"):
                idx = causal_topk(x["q_addr"], x["k_addr"], w.K)
            if op in ("attention", "both"):
                sparse_meat_attention(x["q"], x["k"], x["v"], idx, scale)
            if op == "fused":
                fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], w.K, scale)
            if op == "backward":
                _launch_attention_backward(x["q"], x["k"], x["v"], idx, x["q"], scale, False)
    torch.cuda.synchronize()
    print("ok")


def overlap_probe(w: Workload, dev, flush: torch.Tensor, steps: int) -> dict:
    """Retrieval and attention of two independent cfg2 problems, serial and on two streams at once.

    If the two kernels left each other's resources idle, the concurrent form would
    approach max(topk, attention); it stays near their sum, which is why this build
    does not fuse retrieval with attention per query tile.
    """
    from wayfinder_attention_b200.causal_topk import _launch_topk
    from wayfinder_attention_b200.fused_sparse import _launch_attention

    x1, x2 = device_inputs(w, dev, 1), device_inputs(w, dev, 2)
    i1 = torch.empty(w.B, w.T, w.K, dtype=torch.int32, device=dev)
    i2 = torch.empty_like(i1)
    _launch_topk(x2["q_addr"], x2["k_addr"], w.K, "reference", out=i2)
    main = torch.cuda.current_stream(dev)
    s1, s2 = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    topk = lambda: _launch_topk(x1["q_addr"], x1["k_addr"], w.K, "reference", out=i1)  # noqa: E731
    attn = lambda: _launch_attention(x2["q"], x2["k"], x2["v"], i2, w.D ** -0.5, mask_negative=False,  # noqa: E731
                                     out_dtype=None)

    def both_serial():
        topk()
        attn()

    def both_concurrent():
        s1.wait_stream(main)
        s2.wait_stream(main)
        with torch.cuda.stream(s1):
            topk()
        with torch.cuda.stream(s2):
            attn()
        main.wait_stream(s1)
        main.wait_stream(s2)

    res = {}
    for name, fn in (("topk_ms", topk), ("attention_ms", attn), ("serial_ms", both_serial),
                     ("concurrent_ms", both_concurrent)):
        for _ in range(3):
            fn()
        res[name] = time_events(fn, steps, flush, main)
    return res


def device_inputs(w: Workload, dev, seed: int = 45) -> dict:
    """Seeded inputs of workload ``w`` drawn on the device (large configs: no host round trip)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    if w.clustered:
        centres = torch.randn(64, w.R, generator=g, device=dev) / 32 ** 0.5
        pick = lambda: centres[torch.randint(0, 64, (w.B, w.T), generator=g, device=dev)]  # noqa: E731
        qa = pick() + 0.05 * torch.randn(w.B, w.T, w.R, generator=g, device=dev)
        ka = pick() + 0.05 * torch.randn(w.B, w.T, w.R, generator=g, device=dev)
    else:
        qa = torch.randn(w.B, w.T, w.R, generator=g, device=dev) / 32 ** 0.5
        ka = torch.randn(w.B, w.T, w.R, generator=g, device=dev) / 32 ** 0.5
    out = {"q_addr": qa.to(w.dtype), "k_addr": ka.to(w.dtype)}
    for n in ("q", "k", "v"):
        out[n] = torch.randn(w.B, w.T, w.H, w.D, generator=g, device=dev).to(w.dtype).transpose(1, 2)
    return out


def time_events(fn, steps: int, flush: torch.Tensor, stream) -> float:
    """Mean ms of ``fn`` over ``steps`` launches, L2 flushed before each, CUDA events on ``stream``."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        flush.zero_()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / steps


def gather_ceiling(x: dict, idx: torch.Tensor, steps: int, flush: torch.Tensor, stream) -> float:
    """GB/s of wf_gather_rows_bench: the attention kernel's K/V row loads over the same indices, no math."""
    from wayfinder_attention_b200 import _lib

    lib = _lib.load_library()
    k, v = x["k"], x["v"]  # (B, H, T, D) views of (B, T, H, D) memory: one token's heads are contiguous
    B, H, T, D = k.shape
    esz = k.element_size()
    sink = torch.empty(B * T, dtype=torch.int32, device=k.device)
    K = idx.shape[-1]

    def run():
        for b in range(B):
            rc = lib.wf_gather_rows_bench(k[b].data_ptr(), v[b].data_ptr(), H * D * esz, k.stride(2) * esz,
                                          idx[b].data_ptr(), T, K, T, sink[b * T:].data_ptr(),
                                          stream.cuda_stream)
            _lib.check(rc)

    for _ in range(3):
        run()
    ms = time_events(run, steps, flush, stream)
    return 2.0 * B * T * K * H * D * esz / (ms / 1e3) / 1e9


def bulk_gather_rates(x: dict, idx: torch.Tensor, steps: int, flush: torch.Tensor, stream) -> dict:
    """GB/s of the same gather through cp.async.bulk into shared memory, without and with read-back."""
    from wayfinder_attention_b200 import _lib

    lib = _lib.load_library()
    k, v = x["k"], x["v"]
    B, H, T, D = k.shape
    esz = k.element_size()
    if H * D * esz != 1024:
        return {}
    sink = torch.empty(B * T, dtype=torch.int32, device=k.device)
    K = idx.shape[-1]
    res = {}
    for name, rb in (("bulk_copy_only_gbs", 0), ("bulk_copy_and_read_gbs", 1)):
        def run():
            for b in range(B):
                _lib.check(lib.wf_gather_rows_bulk_bench(k[b].data_ptr(), v[b].data_ptr(), k.stride(2) * esz,
                                                         idx[b].data_ptr(), T, K, T, rb, sink[b * T:].data_ptr(),
                                                         stream.cuda_stream))

        for _ in range(3):
            run()
        ms = time_events(run, steps, flush, stream)
        res[name] = 2.0 * B * T * K * H * D * esz / (ms / 1e3) / 1e9
    return res


def config_measurement(name: str, dev, flush: torch.Tensor, steps: int, B: int | None = None,
                       seed: int = 45) -> dict:
    """One more configuration on this GPU (fused step and its two kernels), for configs beyond cfg2.

    ``B`` overrides the batch (a rank's share of a batch-sharded config)."""
    from wayfinder_attention_b200.causal_topk import _launch_topk
    from wayfinder_attention_b200.fused_sparse import _launch_attention, fused_sparse_attention

    w = CONFIGS[name] if B is None else scaled(CONFIGS[name], B=B)
    x = device_inputs(w, dev, seed)
    stream = torch.cuda.current_stream(dev)
    scale = w.D ** -0.5
    idx = torch.empty(w.B, w.T, min(w.K, w.T), dtype=torch.int32, device=dev)
    step = lambda: fused_sparse_attention(x["q_addr"], x["k_addr"], x["q"], x["k"], x["v"], w.K, scale)  # noqa: E731
    for _ in range(3):
        step()
    ms = time_events(step, steps, flush, stream)
    topk_ms = time_events(lambda: _launch_topk(x["q_addr"], x["k_addr"], w.K, "reference", out=idx), steps, flush,
                          stream)
    attn_ms = time_events(lambda: _launch_attention(x["q"], x["k"], x["v"], idx, scale, mask_negative=False,
                                                    out_dtype=None), steps, flush, stream)
    peaks, kind = load_peaks()
    kv_bytes = 2.0 * w.B * w.T * w.H * w.D * x["k"].element_size()
    res = {"ms": ms, "queries_per_s": w.queries / (ms / 1e3), "B": w.B, "H": w.H, "T": w.T, "D": w.D, "K": w.K,
           "kernels_ms": {"causal_topk": topk_ms, "sparse_attention": attn_ms},
           "gathered_bytes": w.gathered_bytes(), "kv_bytes": kv_bytes,
           "gathered_gbs": w.gathered_bytes() / (attn_ms / 1e3) / 1e9}
    dram = ATTN_DRAM_BYTES.get(name)
    if dram is not None:
        gbs = dram / (attn_ms / 1e3) / 1e9
        res["hbm"] = {"dram_bytes": dram, "source": ATTN_DRAM_SOURCE[name], "achieved_gbs": gbs,
                      "peak_gbs": float(peaks["hbm_gbs"]), "frac": gbs / float(peaks["hbm_gbs"]),
                      "peak_kind": kind}
    del x
    torch.cuda.empty_cache()
    return res


def decoder_forward(B: int, T: int, flush: torch.Tensor, steps: int, dev, attention_type: str = "learned_address",
                    graph: bool = True) -> dict:
    """Whole-model prefill forward of the reference's systems-benchmark model family
    (4 layers, d_model 256, 4 heads, FFN 1024, vocab 128, K 128; transformer.py:76-312)
    with this build's attention, bf16 weights, random init, uniform token ids."""
    from wayfinder_attention_b200 import TransformerLM

    torch.manual_seed(45)
    m = TransformerLM(128, d_model=256, n_layers=4, n_heads=4, d_ff=1024, max_seq_len=T, dropout=0.0,
                      attention_type=attention_type, routing_top_k=128,
                      retrieval_config={"use_fused_sparse": True, "method": "fused_causal"})
    m = m.to(dev, torch.bfloat16).eval()
    ids = torch.randint(0, 128, (B, T), device=dev, generator=torch.Generator(device=dev).manual_seed(45))
    with torch.no_grad():
        for _ in range(3):
            m(ids)
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(steps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            m(ids)
            b.record()
            torch.cuda.synchronize()
            tot += a.elapsed_time(b)
    ms = tot / steps
    res = {"ms": ms, "tokens_per_s": B * T / (ms / 1e3), "B": B, "T": T, "attention": attention_type,
           "model": "4 layers, d_model 256, H 4, FFN 1024, vocab 128, K 128, bf16"}
    if graph:
        # the same forward replayed from a CUDA graph (wayfinder_attention_b200.CapturedForward)
        from wayfinder_attention_b200 import CapturedForward

        cap = CapturedForward(lambda x: m(x)["logits"], ids)
        stream = torch.cuda.current_stream(dev)
        for _ in range(3):
            cap(ids)
        res["graph_ms"] = time_events(lambda: cap(ids), steps, flush, stream)
    return res


def dense_baseline(w: Workload, x: dict, flush: torch.Tensor, steps: int) -> dict:
    """Dense causal SDPA at the same shape (the reference's DenseSDPAAttention call), for comparison."""
    import torch.nn.functional as F

    dev = x["q"].device
    q, k, v = x["q"], x["k"], x["v"]
    for _ in range(3):
        F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=w.D ** -0.5)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats(dev)
    m0 = torch.cuda.memory_allocated(dev)
    tot = 0.0
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=w.D ** -0.5)
        b.record()
        torch.cuda.synchronize()
        tot += a.elapsed_time(b)
    return {"ms": tot / steps, "peak_mb": (torch.cuda.max_memory_allocated(dev) - m0) / 2**20,
            "queries_per_s": w.B * w.T / (tot / steps / 1e3)}


if __name__ == "__main__":
    main()

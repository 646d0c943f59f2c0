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
import subprocess
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
# dram__bytes_read.sum + dram__bytes_write.sum of one sparse-attention launch, from the
# ncu capture summarised in profiles/sparse_attention_cfg2.md (58.0 MB + 4.4 MB).
ATTN_DRAM_BYTES = {"cfg2": 62.3e6}


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
    timed region of a few tens of milliseconds gets samples; falls back to an
    `nvidia-smi` poll if NVML is unavailable.
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
            time.sleep(0.005)  # first sample before the timed region starts
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


def time_cpu_oracle(w: Workload, inputs: dict, n_rows: int) -> tuple[float, int]:
    """Seconds for the oracle port on ``n_rows`` sampled rows of batch element 0 (all host threads)."""
    from oracle import wayfinder_oracle as oracle  # CPU baseline leg only

    xn = {k: v[:1].float().contiguous().numpy() for k, v in inputs.items()}
    rows = cpu_sample_rows(w.T, n_rows)
    t0 = time.perf_counter()
    oracle.fused_sparse_attention(xn["q_addr"], xn["k_addr"], xn["q"], xn["k"], xn["v"], w.K, w.D ** -0.5,
                                  rows=rows)
    return time.perf_counter() - t0, rows.size


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
        time_cpu_oracle(w, inputs, min(n_rows, 64))
    secs = []
    for _ in range(args.steps):
        s, n = time_cpu_oracle(w, inputs, n_rows)
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
                                   f"(retrieval over their causal prefixes + attention over {w.H} heads)"},
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
    ap.add_argument("--cpu-baseline-rows", type=int, default=16384, help="rows of the one-off cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-dense", action="store_true")
    ap.add_argument("--no-decoder", action="store_true", help="skip the whole-decoder prefill measurements")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    claim_stdout()

    w = CONFIGS[args.config]
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

    e2e_serial_ms = time_e2e(e2e_serial)
    e2e_ms_step = time_e2e(e2e_pipelined)
    e2e_value = queries / (e2e_ms_step / 1e3)

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
            "roofline": {"kernel": "sparse_attention", "bound": "hbm", "achieved": achieved_gbs, "peak": hbm,
                         "unit": "GB/s", "frac": achieved_gbs / hbm,
                         "traffic": ATTN_DRAM_BYTES.get(w.name),
                         "peak_kind": peak_kind,
                         "note": "achieved = gathered K/V bytes (2*B*H*T*K*D*2) / kernel time; K/V fit in L2"},
            "path_roofline": {"roofline_ms": roof_s * 1e3, "frac": roof_s * 1e3 / ms_per_step,
                              "score_tflops_achieved": w.score_flops() / (topk_ms_launch / 1e3) / 1e12,
                              "definition": "max(score FLOPs / bf16 peak, gathered bytes / HBM peak) / latency"},
            "peak_mb": peak_mb,
            "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms_step, "api": "HostFusedSparseAttention (copies overlapped, "
                    f"{E2E_CHUNKS} row chunks)", "serial_ms_per_step": e2e_serial_ms},
            "gpu_launches": 3 * args.steps,  # per step: retrieval, finalisation, attention
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
        if world == 1 and not args.no_cpu_baseline:
            secs, n = time_cpu_oracle(w, host, args.cpu_baseline_rows)
            result["cpu_baseline"] = {
                "value": n / secs, "unit": "queries/s", "cores": os.cpu_count() or 1, "kind": "port",
                "cpu": cpu_model(),
                "sample": f"{n} evenly spaced query rows of the T={w.T} sequence "
                          f"(retrieval + {w.H}-head attention), numpy fp32 oracle",
            }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        emit(result)


def run_sequence_sharded(args, w: Workload, rank: int, world: int, dev) -> None:
    """cfg4: one T=65536 sequence, query-row blocks over ranks, address and K/V all-gathers (strong scaling)."""
    import torch.distributed as dist

    from wayfinder_attention_b200.sharding import SequenceShardedAttention, local_rows

    tile = 256
    if w.T % (world * tile):
        raise SystemExit(f"T={w.T} is not a multiple of world*tile={world * tile}")
    g = torch.Generator(device=dev).manual_seed(45)  # identical full inputs on every rank
    qa = (torch.randn(w.B, w.T, w.R, generator=g, device=dev) / 32 ** 0.5).to(w.dtype)
    ka = (torch.randn(w.B, w.T, w.R, generator=g, device=dev) / 32 ** 0.5).to(w.dtype)
    qkv = [torch.randn(w.B, w.T, w.H, w.D, generator=g, device=dev).to(w.dtype) for _ in range(3)]
    rows = torch.from_numpy(local_rows(w.T, world, rank, tile)).to(dev)
    qa_l, ka_l = qa[:, rows].contiguous(), ka[:, rows].contiguous()
    q_l, k_l, v_l = (t[:, rows].contiguous().transpose(1, 2) for t in qkv)
    del qa, ka, qkv
    op = SequenceShardedAttention(w.K, w.D ** -0.5, tile=tile)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        flush.zero_()
        op(qa_l, ka_l, q_l, k_l, v_l)
    torch.cuda.synchronize()
    dist.barrier()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    torch.cuda.synchronize()
    dist.barrier()
    with ClockSampler(int(os.environ.get("LOCAL_RANK", 0))) as clk:
        for i in range(args.steps):
            flush.zero_()
            dist.barrier()  # all ranks enter the step together, outside the timed events
            ev[i][0].record(stream)
            op(qa_l, ka_l, q_l, k_l, v_l)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    dist.barrier()
    tot = torch.tensor([sum(a.elapsed_time(b) for a, b in ev)], dtype=torch.float64, device=dev)
    dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    ms = tot.item() / args.steps
    if rank == 0:
        peaks, peak_kind = load_peaks()
        roof_ms = 1e3 * max(w.score_flops() / (float(peaks["bf16_tflops"]) * 1e12),
                            w.gathered_bytes() / (float(peaks["hbm_gbs"]) * 1e9)) / world
        emit({
            "metric": METRIC, "value": w.B * w.T / (ms / 1e3), "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, generated on device)",
            "config": {"workload": w.name, "B": w.B, "H": w.H, "T": w.T, "D": w.D, "d_A": w.R, "K": w.K,
                       "parallelism": f"query-row blocks of {tile} cyclic over {world} ranks; "
                                      "k_addr and K/V all-gathered with NCCL",
                       "l2": "flushed before every timed step"},
            "path_roofline": {"roofline_ms_per_gpu": roof_ms, "frac": roof_ms / ms, "peak_kind": peak_kind},
            "gpu_launches": 3 * args.steps,  # per step: retrieval, finalisation, attention
            "clocks": clk.summary(),
        })


def decoder_forward(B: int, T: int, flush: torch.Tensor, steps: int, dev, attention_type: str = "learned_address") -> dict:
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
    return {"ms": ms, "tokens_per_s": B * T / (ms / 1e3), "B": B, "T": T, "attention": attention_type,
            "model": "4 layers, d_model 256, H 4, FFN 1024, vocab 128, K 128, bf16"}


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

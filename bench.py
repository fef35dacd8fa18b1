"""Benchmark of the B200 scale-sweep MSE NVFP4 quantizer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: row-sharded quantization of a bf16 [524288, 8192] activation
(seeded N(0,1), 0.5% of columns x20; global scale amax/(6*448)), split by rows
over N GPUs (strong scaling).  One step = per-GPU |x| max -> NCCL MAX
all-reduce (N > 1) -> device-side multiplier 2688/amax -> scale-sweep MSE
quantization (11 candidates, swizzled scales).  The metric is algorithmic
GB/s = M*K*2.5625 B (bf16 in, E2M1 codes + E4M3 scales out) per step time.

At N=1 the line also carries the shape sweep of the standalone quantizer
(M in {1..16384} x K in {4096, 8192, 14336}, scale-sweep vs plain RTN) and the
CPU baseline (the oracle on a bounded sample on this host's cores).

``--impl reference`` times the reference algorithm's CPU implementation (the
plain-C restatement under oracle/, all host threads) on a bounded sample of
the same workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_TOTAL = 524288
K_DIM = 8192
FP8_MAX = 448.0
BYTES_PER_ELEM = 2.5625
METRIC = "scalesweep-MSE NVFP4 quant GB/s (algorithmic M*K*2.5625 B)"
UNIT = "GB/s"
WORKLOAD = "row-sharded scale-sweep MSE NVFP4 quantization of bf16 [524288, 8192]"
# config-2 rows, plus 128 and 8192, the other rows the reference publishes latencies for
SWEEP_M = (1, 16, 64, 128, 256, 1024, 4096, 8192, 16384)
# Llama-3.1-8B linear layers (K -> N): qkv, o, gate_up, down
GEMM_SHAPES = ((4096, 6144), (4096, 4096), (4096, 28672), (14336, 4096))
GEMM_M = (16, 128, 1024, 8192)
FP4_DENSE_NOMINAL_TFLOPS = 9000.0
SWEEP_K = (4096, 8192, 14336)
ALU_OPS_PER_ELEM = 35  # sweep's FP32 op count per element (roofline definition)
SM_COUNT = 148
FP32_LANES_PER_SM = 128
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
# vLLM end-to-end arms: the backend passed to vllm_e2e.run, and whether the
# activation quantizer is the reference's own Triton kernel
VLLM_ARMS = {
    "cutlass": "vLLM's own RTN activation quantizer (CUTLASS path)",
    "reference_triton": "the reference's Triton scalesweep_mse kernel "
                        "(bench_kernel/scalesweep_mse_nvfp4_utils.py:498-519), registered as "
                        "torch.ops.vllm.scalesweep_mse_nvfp4_quant with its own fake "
                        "implementation (:546-560), SCALESWEEP_TUNE=0 as in run_bench_tune.sh",
    "scalesweep_mse": "this package's scalesweep_mse quantizer",
    "scalesweep_mse_fused_norm_act": "this package's quantizer with RMSNorm and SiLU-and-mul fused "
                                     "into it (Llama module hooks); the fused RMSNorm is vLLM's "
                                     "vllm_c kernel bit for bit, so under Inductor its last bits "
                                     "can differ from the unfused compiled run",
    "scalesweep_mse_fusion_pass": "the same fusions reached through a vLLM compile pass "
                                  "(vllm_fusion.py) instead of module hooks",
    "scalesweep_mse_dispatch": "this package's quantizer; each linear layer's GEMM from this "
                               "package (quantizer + GEMM in one call) at token counts where it "
                               "is faster, vLLM's CUTLASS GEMM elsewhere",
    "scalesweep_mse_fused_norm_act_dispatch": "the fused RMSNorm/SiLU-and-mul hooks with the "
                                              "same per-call GEMM choice",
    "scalesweep_mse_fusion_pass_dispatch": "the compile-pass fusions (any model) with the GEMM "
                                           "alone dispatched per call",
}
# (input tokens, output tokens, batch sizes): config 4, and the reference's
# own 256-request run (benchmark_nvfp4_tokens.py defaults, run_bench_tune.sh)
VLLM_WORKLOADS = {"decode": (1024, 256, (1, 16, 64, 256)), "reference": (2048, 256, (256,))}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=M_TOTAL, help="total rows (default 524288)")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-gemm", action="store_true")
    ap.add_argument("--no-ref-triton", action="store_true",
                    help="skip the same-GPU timing of the reference's Triton kernels")
    ap.add_argument("--write-config5-digests", default=None, metavar="FILE",
                    help="one GPU: write the per-chunk SHA-256 digests of the whole tensor's "
                         "codes and scales (the record N-GPU runs are checked against)")
    ap.add_argument("--profile-case", default=None, metavar="MxK",
                    help="only run the scale-sweep quantizer 4 times on one [M, K] input "
                         "(the command used for ncu captures) and exit")
    ap.add_argument("--profile-backend", default="scalesweep_mse",
                    choices=["scalesweep_mse", "scalesweep_mse_reference", "rtn", "scalesweep"])
    ap.add_argument("--profile-gemm", default=None, metavar="MxNxK",
                    help="only run the NVFP4 GEMM 4 times on one shape and exit (for ncu)")
    ap.add_argument("--profile-amax", default=None, metavar="MxK",
                    help="only run the fused amax + global-scale kernel 4 times and exit")
    ap.add_argument("--profile-amax-noalloc", default=None, metavar="MxK",
                    help="only run the allocation-free global-scale entry point 4 times and "
                         "exit (for ncu)")
    ap.add_argument("--profile-act", default=None, metavar="MxN",
                    help="only run silu_and_mul and the fused SiLU-and-mul quantizer on a "
                         "[M, 2N] input 4 times each and exit (for ncu)")
    ap.add_argument("--profile-norm", default=None, metavar="MxN",
                    help="only run the RMSNorm-fused quantizer (plain, then with a residual) "
                         "on an [M, N] input 4 times each and exit (for ncu)")
    ap.add_argument("--vllm-e2e", action="store_true",
                    help="Llama-3.1-8B W4A4 in vLLM on one GPU: output tok/s of each arm "
                         "(--vllm-arms), one engine process per run, arms interleaved over "
                         "--vllm-repeats rounds; prints one JSON line and exits")
    ap.add_argument("--vllm-arms", nargs="+", default=list(VLLM_ARMS), choices=list(VLLM_ARMS))
    ap.add_argument("--vllm-repeats", type=int, default=3)
    ap.add_argument("--vllm-workload", choices=sorted(VLLM_WORKLOADS), default="decode")
    ap.add_argument("--gemm-crossover", action="store_true",
                    help="time the whole linear layer from this package against the quantizer "
                         "+ vLLM's GEMM over token counts; prints one JSON line and exits")
    ap.add_argument("--vllm-arm", default=None, choices=list(VLLM_ARMS),
                    help=argparse.SUPPRESS)  # one engine run (a child of --vllm-e2e)
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("sm_max_mhz", 1965.0)), "measured"
    except Exception:
        return 6650.0, 1965.0, "fallback"


def load_traffic_profile():
    """DRAM bytes per 16-element block of the quantizer, from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "quant_kernel_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_block:"):
                    return (float(line.split(":", 1)[1].split()[0]),
                            os.path.relpath(path, ROOT))
    except OSError:
        pass
    return None, None


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 200 ms for one GPU."""

    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, bus_id: str | None):
        self.index = None
        self.proc = None
        try:
            out = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id",
                                  "--format=csv,noheader"], capture_output=True, text=True,
                                 timeout=30).stdout
            for line in out.splitlines():
                idx, bus = [f.strip() for f in line.split(",")]
                if bus_id and bus.lower() == bus_id.lower():
                    self.index = idx
        except Exception:
            pass

    def start(self):
        if self.index is None:
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.index, f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            reasons.update(n for n, v in zip(self.REASONS, f[3:7]) if v == "Active")
        if not sm:
            return None
        loaded = sorted(sm)[len(sm) // 2:]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm), "gpu_index": self.index}


# ------------------------------------------------------------- workload ----
def make_shard(rows: int, k: int, seed: int, device):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.empty(rows, k, dtype=torch.bfloat16, device=device)
    chunk = 16384
    for r in range(0, rows, chunk):
        n = min(chunk, rows - r)
        x[r:r + n] = torch.randn(n, k, generator=g, device=device, dtype=torch.float32)
    gc = torch.Generator().manual_seed(seed ^ 0x5EED)
    cols = torch.randperm(k, generator=gc)[: -(-5 * k // 1000)].to(device)
    x[:, cols] *= 20
    return x


CHUNK_ROWS = 16384  # config-5 rows are generated (and digested) in chunks of this many
CONFIG5_SEED = 5000
DIGEST_PATH = os.path.join(ROOT, "tests", "golden", "config5_digests.json")


def config5_outlier_cols(k: int):
    """The one set of ceil(0.5% * K) outlier columns of the whole config-5 tensor."""
    import torch
    gc = torch.Generator().manual_seed(CONFIG5_SEED ^ 0x5EED)
    return torch.randperm(k, generator=gc)[: -(-5 * k // 1000)]


def make_global_rows(start: int, rows: int, k: int, device):
    """Rows [start, start + rows) of the config-5 tensor, the same bits at
    every GPU count: chunk c (rows c*16384 ...) is N(0,1) from a generator
    seeded with CONFIG5_SEED + c on the device, then the tensor-wide outlier
    columns are multiplied by 20.  ``start`` and ``rows`` are whole chunks."""
    import torch
    if start % CHUNK_ROWS or rows % CHUNK_ROWS:
        raise ValueError("config-5 shards are whole 16384-row chunks")
    x = torch.empty(rows, k, dtype=torch.bfloat16, device=device)
    for r in range(0, rows, CHUNK_ROWS):
        g = torch.Generator(device=device).manual_seed(CONFIG5_SEED + (start + r) // CHUNK_ROWS)
        x[r:r + CHUNK_ROWS] = torch.randn(CHUNK_ROWS, k, generator=g, device=device,
                                          dtype=torch.float32)
    x[:, config5_outlier_cols(k).to(device)] *= 20
    return x


def chunk_digests(codes, scales, start: int):
    """SHA-256 of each 16384-row chunk's codes plus its rows of the swizzled
    scale buffer (a contiguous slab of 128 row tiles), keyed by global chunk."""
    import hashlib
    out = {}
    c_host = codes.cpu()
    s_host = scales.view(-1, scales.shape[-1]).cpu()
    for r in range(0, codes.shape[0], CHUNK_ROWS):
        h = hashlib.sha256(c_host[r:r + CHUNK_ROWS].numpy().tobytes())
        h.update(s_host[r:r + CHUNK_ROWS].numpy().tobytes())
        out[str((start + r) // CHUNK_ROWS)] = h.hexdigest()
    return out


def time_events(fn, iters: int, stream):
    import torch
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / iters


def kernel_avg_ms(fn, iters: int, stream, flush=None):
    """Average duration of one launch, each bracketed by its own events."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(iters)]
    for a, b in evs:
        if flush is not None:
            flush()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in evs) / iters


def graph_avg_ms(fn, reps: int, device) -> float:
    """Per-launch device time of ``fn`` replayed ``reps`` times from one CUDA graph
    (no L2 flush between launches: the reference's do_bench_cudagraph method)."""
    import torch
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b) / reps
    del g
    return ms


def dequant_mse(x, codes, scales, gsi) -> float:
    """Mean squared error of the dequantized NVFP4 result against the input,
    the quality figure the reference reports per backend.  Plain torch on the
    GPU: E2M1 lookup, E4M3 scales read through the 128x4 swizzle."""
    import torch
    m, n = x.shape
    dev = x.device
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], device=dev)
    c = codes.view(torch.uint8).to(torch.int64)
    vals = torch.stack([lut[c & 0xF], lut[c >> 4]], dim=-1).reshape(m, n)
    kb = n // 16
    kpad = (kb + 3) // 4 * 4
    r = torch.arange(m, device=dev)[:, None]
    col = torch.arange(kb, device=dev)[None, :]
    off = (r >> 7) * (kpad * 128) + (col >> 2) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (col & 3)
    sb = scales.view(torch.uint8).reshape(-1)[off]
    s = sb.view(torch.float8_e4m3fn).to(torch.float32)
    deq = vals.reshape(m, kb, 16) * (s / gsi.reshape(1)).unsqueeze(-1)
    return float((deq.reshape(m, n) - x.float()).square().mean().item())


def run_quality(device):
    """Dequantized MSE on N(0,1) bf16 [M, 4096], the reference's quality
    benchmark: fp8_max 256 for the scale-sweep backends, 448 for RTN."""
    import torch
    from test_speed_scalesweep_b200 import custom
    out = {"input": "torch.randn bf16 [M, 4096], seeded; gsi = fp8_max*6/amax"}
    g = torch.Generator(device=device).manual_seed(1234)
    backends = (("scalesweep_mse", 256.0), ("scalesweep_mse_reference", 256.0), ("rtn", 448.0),
                ("cutlass", 448.0))
    for m in (1024, 8192):
        x = torch.randn(m, 4096, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
        row = {}
        for backend, fp8_max in backends:
            gsi = ((fp8_max * 6.0) / x.abs().max().to(torch.float32)).reshape(1)
            try:
                codes, scales = custom.nvfp4_quant(x, gsi, True, backend)
            except Exception as exc:  # vLLM's comparator may be missing
                row[backend] = f"unavailable: {type(exc).__name__}"
                continue
            row[backend] = round(dequant_mse(x, codes, scales, gsi), 8)
        out[f"M{m}_K4096"] = row
    return out


def run_sweep(device, reps: int = 20):
    """Standalone quantizer at the shape-sweep configs, scale-sweep vs RTN."""
    import torch
    from test_speed_scalesweep_b200 import custom, global_scale
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    out = {}
    for k in SWEEP_K:
        for m in SWEEP_M:
            x = make_shard(m, k, 7 + m + k, device)
            gsi = global_scale.global_scale_inv_from_max(x, FP8_MAX)
            codes, scales = custom.create_fp4_output_tensors(m, k, device, True)
            res = {}
            for name, fn in (("scalesweep_mse", mse.scalesweep_mse_nvfp4_quant_out),
                             ("rtn", mse.rtn_nvfp4_quant_out)):
                call = lambda fn=fn: fn(x, gsi, True, output=codes, output_scale=scales)  # noqa
                ms = graph_avg_ms(call, reps, device)
                res[name] = {"us": round(ms * 1e3, 3),
                             "GB/s": round(m * k * BYTES_PER_ELEM / (ms * 1e-3) / 1e9, 1)}
            out[f"{m}x{k}"] = res
            del x
    out["method"] = ("per-launch time from one CUDA graph of 20 launches, no L2 flush "
                     "(inputs of M>=16384 exceed L2)")
    return out




def load_reference_dispatcher():
    """The reference's own ``bench_kernel/custom.py:nvfp4_quant`` from the
    unmodified install under baseline/_ref (baseline/install_ref.py), with the
    scale-sweep kernels autotuned as in its published latency runs
    (SCALESWEEP_TUNE=1, read when the module is imported).  None if absent."""
    if not os.path.isdir(os.path.join(REF_DIR, "bench_kernel")):
        return None
    os.environ.setdefault("SCALESWEEP_TUNE", "1")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from bench_kernel import custom as ref_custom
    return ref_custom.nvfp4_quant


def run_reference_triton_sweep(device, rep: int = 20):
    """Config 2 on this GPU: the reference's Triton kernels (K1 scalesweep_mse,
    K2 scalesweep_mse_reference) against this package's kernels, both through
    their ``nvfp4_quant(x, gsi, True, backend)`` dispatcher and both timed with
    the reference's method (``triton.testing.do_bench_cudagraph``, mean,
    bench_kernel/test_kernel_latency.py:144-158).  Each shape also compares the
    two outputs byte for byte (codes and the written scale bytes)."""
    import torch
    from triton.testing import do_bench_cudagraph
    from test_speed_scalesweep_b200 import custom
    ref_quant = load_reference_dispatcher()
    if ref_quant is None:
        return {"unavailable": "reference not installed under baseline/_ref"}
    out = {"method": "triton.testing.do_bench_cudagraph(rep=20, return_mode='mean') on both "
                     "arms' nvfp4_quant dispatchers; reference kernels autotuned "
                     "(SCALESWEEP_TUNE=1); gsi = 256*6/amax (the reference's convention for "
                     "scale-sweep backends)"}
    ratios = {"scalesweep_mse": [], "scalesweep_mse_reference": []}
    for k in SWEEP_K:
        for m in SWEEP_M:
            x = make_shard(m, k, 7 + m + k, device)
            gsi = ((256.0 * 6.0) / x.abs().max().to(torch.float32)).reshape(1)
            row = {}
            for backend in ("scalesweep_mse", "scalesweep_mse_reference"):
                rc, rs = ref_quant(x, gsi, True, backend)
                oc, os_ = custom.nvfp4_quant(x, gsi, True, backend)
                # the swizzled slab's padding rows/columns are never written by either
                kb = k // 16
                r_idx = torch.arange(m, device=device)[:, None]
                c_idx = torch.arange(kb, device=device)[None, :]
                kpad = (kb + 3) // 4 * 4
                off = ((r_idx >> 7) * (kpad * 128) + (c_idx >> 2) * 512 + (r_idx & 31) * 16 +
                       ((r_idx & 127) >> 5) * 4 + (c_idx & 3)).reshape(-1)
                same = bool(torch.equal(rc, oc)) and bool(torch.equal(
                    rs.view(torch.uint8).reshape(-1)[off], os_.view(torch.uint8).reshape(-1)[off]))
                ref_ms = do_bench_cudagraph(lambda: ref_quant(x, gsi, True, backend), rep=rep)
                our_ms = do_bench_cudagraph(lambda: custom.nvfp4_quant(x, gsi, True, backend),
                                            rep=rep)
                row[backend] = {"reference_triton_us": round(ref_ms * 1e3, 3),
                                "ours_us": round(our_ms * 1e3, 3),
                                "ours_over_reference_time": round(our_ms / ref_ms, 4),
                                "bytes_equal": same}
                ratios[backend].append(our_ms / ref_ms)
            out[f"{m}x{k}"] = row
            del x
    for backend, r in ratios.items():
        big = [v for (mk, v) in zip([f"{m}x{k}" for k in SWEEP_K for m in SWEEP_M], r)
               if int(mk.split("x")[0]) >= 1024]
        out[f"{backend}_geomean_time_ratio"] = round(statistics.geometric_mean(r), 4)
        out[f"{backend}_worst_time_ratio_m_ge_1024"] = round(max(big), 4) if big else None
    out["all_bytes_equal"] = all(v[b]["bytes_equal"] for kk, v in out.items()
                                 if isinstance(v, dict) and "scalesweep_mse" in v
                                 for b in ("scalesweep_mse", "scalesweep_mse_reference"))
    return out


ACT_FUSION_M = (16, 128, 1024, 8192)
ACT_FUSION_N = 14336  # Llama-3.1-8B intermediate width: the down projection's input


def run_act_fusion_sweep(device, reps: int = 20):
    """SiLU-and-mul + scalesweep_mse, unfused (two launches, bf16 intermediate
    in HBM) against the fused kernel, on [M, 2 x 14336] gate_up outputs."""
    import torch
    from test_speed_scalesweep_b200 import act_quant
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    n = ACT_FUSION_N
    out = {"n": n, "method": "per-launch time from one CUDA graph of 20 launches"}
    gsi = torch.tensor([FP8_MAX * 6.0 / 40.0], dtype=torch.float32, device=device)
    for m in ACT_FUSION_M:
        x = make_shard(m, 2 * n, 17 + m, device)
        h = torch.empty(m, n, dtype=x.dtype, device=device)
        codes, scales = act_quant.alloc_outputs(x, True)

        def unfused():
            act_quant.silu_and_mul(x, h)
            mse.scalesweep_mse_nvfp4_quant_out(h, gsi, True, output=codes, output_scale=scales)

        def fused():
            act_quant.silu_and_mul_scalesweep_mse_nvfp4_quant_out(x, gsi, True, output=codes,
                                                                  output_scale=scales)

        u_ms = graph_avg_ms(unfused, reps, device)
        f_ms = graph_avg_ms(fused, reps, device)
        s_ms = graph_avg_ms(lambda: act_quant.silu_and_mul(x, h), reps, device)
        out[f"M{m}"] = {"unfused_us": round(u_ms * 1e3, 2), "silu_and_mul_us": round(s_ms * 1e3, 2),
                        "fused_us": round(f_ms * 1e3, 2), "speedup": round(u_ms / f_ms, 3)}
        del x, h
    return out


NORM_FUSION_M = (16, 128, 1024, 8192)
NORM_FUSION_N = 4096  # Llama-3.1-8B hidden size: the qkv and gate_up projections' input


def run_norm_fusion_sweep(device, reps: int = 20):
    """RMSNorm + scalesweep_mse on [M, 4096] decoder-layer inputs: vLLM's
    rms_norm / fused_add_rms_norm, then the quantizer on the bf16 result (the
    reference's pipeline, fuse_norm_quant off), against the fused op (row
    statistics, then the quantizer normalising while it loads).  Needs vLLM's
    compiled ops for the unfused leg; the fused times are reported either way."""
    import torch
    from test_speed_scalesweep_b200 import norm_quant
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    try:
        import vllm._custom_ops  # noqa: F401
        have_vllm = hasattr(torch.ops._C, "rms_norm")
    except Exception:
        have_vllm = False
    n, eps = NORM_FUSION_N, 1e-5
    out = {"n": n, "method": "per-launch time from one CUDA graph of 20 launches"}
    gsi = torch.tensor([FP8_MAX * 6.0 / 40.0], dtype=torch.float32, device=device)
    g = torch.Generator(device=device).manual_seed(n)
    w = (1.0 + 0.3 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)
    for m in NORM_FUSION_M:
        x = make_shard(m, n, 29 + m, device)
        res = make_shard(m, n, 31 + m, device)
        h = torch.empty_like(x)
        rstd = torch.empty(m, dtype=torch.float32, device=device)
        codes, scales = norm_quant.alloc_outputs(x, True)
        r = {}

        def fused():
            norm_quant.rms_norm_scalesweep_mse_nvfp4_quant_out(
                x, w, eps, gsi, True, output=codes, output_scale=scales, rstd=rstd)

        def fused_add():
            norm_quant.rms_norm_scalesweep_mse_nvfp4_quant_out(
                x, w, eps, gsi, True, output=codes, output_scale=scales, residual=res, rstd=rstd)

        r["fused_us"] = round(graph_avg_ms(fused, reps, device) * 1e3, 2)
        r["fused_add_us"] = round(graph_avg_ms(fused_add, reps, device) * 1e3, 2)
        if have_vllm:
            def unfused():
                torch.ops._C.rms_norm(h, x, w, eps)
                mse.scalesweep_mse_nvfp4_quant_out(h, gsi, True, output=codes,
                                                   output_scale=scales)

            def unfused_add():
                torch.ops._C.fused_add_rms_norm(h, res, w, eps)
                mse.scalesweep_mse_nvfp4_quant_out(h, gsi, True, output=codes,
                                                   output_scale=scales)

            h.copy_(x)
            r["vllm_rms_norm_us"] = round(
                graph_avg_ms(lambda: torch.ops._C.rms_norm(h, x, w, eps), reps, device) * 1e3, 2)
            r["unfused_us"] = round(graph_avg_ms(unfused, reps, device) * 1e3, 2)
            r["unfused_add_us"] = round(graph_avg_ms(unfused_add, reps, device) * 1e3, 2)
            r["speedup"] = round(r["unfused_us"] / r["fused_us"], 3)
            r["speedup_add"] = round(r["unfused_add_us"] / r["fused_add_us"], 3)
        out[f"M{m}"] = r
        del x, res, h
    return out


def measure_fp4_peak(device, iters: int = 4096):
    """Dense FP4 tensor-core rate of this B200, measured: one CTA per SM
    issues back-to-back kind::mxf4nvf4 MMAs (ssw_nvfp4_mma_rate_probe, the
    GEMM's own instruction and layouts, no loads).  Returns TFLOP/s over the
    whole GPU from CUDA events (best of 3 launches) and FLOPs per SM cycle."""
    import ctypes
    import torch
    from test_speed_scalesweep_b200 import _lib
    lib = _lib.lib()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    cycles = torch.zeros(sms, dtype=torch.int64, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    best = {}
    for bn in (128, 256):
        flops = 2.0 * 128 * bn * 64 * 4 * iters * sms
        times = []
        for _ in range(4):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            st = lib.ssw_nvfp4_mma_rate_probe(bn, iters, ctypes.c_void_p(cycles.data_ptr()),
                                              ctypes.c_void_p(status.data_ptr()),
                                              ctypes.c_void_p(stream.cuda_stream))
            b.record(stream)
            _lib.check(st)
            b.synchronize()
            times.append(a.elapsed_time(b))
        if status.item() != 0 or int(cycles.min().item()) <= 0:
            raise RuntimeError("tensor-core rate probe: a bounded wait gave up")
        per_cycle = 2.0 * 128 * bn * 64 * 4 * iters / float(cycles.median().item())
        best[bn] = {"tflops": round(flops / (min(times[1:]) * 1e-3) / 1e12, 1),
                    "flops_per_sm_cycle": round(per_cycle, 1)}
    top = max(best.values(), key=lambda v: v["tflops"])
    return {"peak_tflops": top["tflops"], "by_tile_n": best,
            "method": f"ssw_nvfp4_mma_rate_probe: {sms} CTAs, 4 x {iters} back-to-back "
                      "kind::mxf4nvf4 MMAs (128 x N x 64) each, CUDA events, best of 3"}


def run_gemm_sweep(device, reps: int = 20):
    """Config 3: quantize + tcgen05 NVFP4 GEMM on the Llama-3.1-8B linear shapes.

    Times (one CUDA graph of ``reps`` launches each): our GEMM, vLLM's CUTLASS
    NVFP4 GEMM on the same operands when vLLM's compiled ops are importable, and
    scale-sweep quantization of the activations followed by our GEMM."""
    import torch
    from test_speed_scalesweep_b200 import custom, global_scale
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm, scalesweep_nvfp4_linear
    try:
        import vllm._custom_ops as vops
        vllm_mm = vops.cutlass_scaled_fp4_mm if hasattr(torch.ops._C, "cutlass_scaled_fp4_mm") \
            else None
    except Exception:
        vllm_mm = None
    try:
        peak = measure_fp4_peak(device)
        peak_tflops = peak["peak_tflops"]
        peak_source = {"measured": peak, "nominal_tflops": FP4_DENSE_NOMINAL_TFLOPS}
    except Exception as e:  # the probe needs the whole GPU
        peak_tflops = FP4_DENSE_NOMINAL_TFLOPS
        peak_source = f"nominal dense FP4 (tensor-core rate probe failed: {e})"
    out = {"peak_tflops": peak_tflops, "peak_source": peak_source,
           "method": "per-launch time from one CUDA graph of 20 launches"}
    for k, n in GEMM_SHAPES:
        g = torch.Generator(device=device).manual_seed(k + n)
        w = (torch.randn(n, k, generator=g, device=device) * 0.02).to(torch.bfloat16)
        w_gsi = global_scale.global_scale_inv_from_max(w, FP8_MAX)
        qb, sb = mse.rtn_nvfp4_quant_impl(w, w_gsi, True)
        del w
        for m in GEMM_M:
            x = make_shard(m, k, 3 + m + k, device)
            a_gsi = global_scale.global_scale_inv_from_max(x, FP8_MAX)
            qa, sa = mse.scalesweep_mse_nvfp4_quant_impl(x, a_gsi, True)
            alpha = (1.0 / (a_gsi * w_gsi)).reshape(1).float()
            flops = 2.0 * m * n * k
            res = {}
            ms = graph_avg_ms(lambda: cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha), reps, device)
            res["gemm_us"] = round(ms * 1e3, 2)
            res["gemm_tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
            res["gemm_frac"] = round(res["gemm_tflops"] / peak_tflops, 4)
            if vllm_mm is not None:
                vms = graph_avg_ms(lambda: vllm_mm(qa, qb, sa, sb, alpha, torch.bfloat16), reps,
                                   device)
                res["vllm_cutlass_gemm_us"] = round(vms * 1e3, 2)
                res["vllm_cutlass_gemm_tflops"] = round(flops / (vms * 1e-3) / 1e12, 1)

            def two_calls():
                ca, csa = mse.scalesweep_mse_nvfp4_quant_impl(x, a_gsi, True)
                return cutlass_scaled_fp4_mm(ca, qb, csa, sb, alpha)
            qms = graph_avg_ms(two_calls, reps, device)
            res["quant_plus_gemm_us"] = round(qms * 1e3, 2)
            # one call: the GEMM as a programmatic dependent launch of the quantizer
            lms = graph_avg_ms(lambda: scalesweep_nvfp4_linear(x, a_gsi, qb, sb, alpha), reps,
                               device)
            res["quant_gemm_linear_us"] = round(lms * 1e3, 2)
            out[f"M{m}_K{k}_N{n}"] = res
            del x, qa, sa
        del qb, sb
    return out


CROSSOVER_M = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512, 1024, 2048, 8192)


def run_gemm_crossover(args):
    """Where the whole linear layer from this package (scale-sweep quantizer,
    then this GEMM as its programmatic dependent) beats scale-sweep
    quantization followed by vLLM's CUTLASS NVFP4 GEMM, per Llama-3.1-8B
    shape and token count M.  Prints one JSON line."""
    import torch
    import vllm._custom_ops as vops
    from test_speed_scalesweep_b200 import global_scale
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    from test_speed_scalesweep_b200.gemm import scalesweep_nvfp4_linear
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    out = {"gemm_crossover": "per-launch us, one CUDA graph of 20 launches; 'ours' = "
                             "scalesweep_nvfp4_linear (quantizer + this GEMM, one call), "
                             "'vllm' = scale-sweep quantizer + vLLM cutlass_scaled_fp4_mm",
           "shapes": {}}
    for k, n in GEMM_SHAPES:
        g = torch.Generator(device=device).manual_seed(k + n)
        w = (torch.randn(n, k, generator=g, device=device) * 0.02).to(torch.bfloat16)
        w_gsi = global_scale.global_scale_inv_from_max(w, FP8_MAX)
        qb, sb = mse.rtn_nvfp4_quant_impl(w, w_gsi, True)
        del w
        rows = {}
        for m in CROSSOVER_M:
            x = make_shard(m, k, 3 + m + k, device)
            a_gsi = global_scale.global_scale_inv_from_max(x, FP8_MAX)
            alpha = (1.0 / (a_gsi * w_gsi)).reshape(1).float()

            def vllm_path():
                ca, csa = mse.scalesweep_mse_nvfp4_quant_impl(x, a_gsi, True)
                return vops.cutlass_scaled_fp4_mm(ca, qb, csa, sb, alpha, torch.bfloat16)
            ours = graph_avg_ms(lambda: scalesweep_nvfp4_linear(x, a_gsi, qb, sb, alpha), 20,
                                device)
            theirs = graph_avg_ms(vllm_path, 20, device)
            rows[str(m)] = {"ours_us": round(ours * 1e3, 2), "vllm_us": round(theirs * 1e3, 2),
                            "vllm_over_ours": round(theirs / ours, 3)}
            del x
        out["shapes"][f"K{k}_N{n}"] = rows
        del qb, sb
    print(json.dumps(out), flush=True)


def cpu_sample_rate(rows_hint: int, budget_s: float = 12.0):
    """Oracle (all host threads) on a bounded sample of the workload."""
    import numpy as np
    import oracle
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import golden_inputs as gi
    threads = os.cpu_count() or 1
    probe_rows = 64
    x = gi.outlier_activations(probe_rows, K_DIM, seed=4242)
    gsi = gi.torch_style_gsi(x, FP8_MAX)
    t = time.perf_counter()
    oracle.quantize(x, gsi, nthreads=threads)
    dt = max(time.perf_counter() - t, 1e-4)
    rows = int(min(rows_hint, max(probe_rows, probe_rows * budget_s / dt)))
    rows = max(probe_rows, rows // 64 * 64)
    # at most 16384 freshly drawn rows, quantized as often as the budget asks
    chunk = min(rows, 16384)
    reps = max(1, rows // chunk)
    rows = reps * chunk
    x = gi.outlier_activations(chunk, K_DIM, seed=4243)
    gsi = gi.torch_style_gsi(x, FP8_MAX)
    t = time.perf_counter()
    for _ in range(reps):
        oracle.quantize(x, gsi, nthreads=threads)
    dt = time.perf_counter() - t
    # config 1 (128 x 4096) and the config-2 shapes with M <= 1024 at K = 4096:
    # median of 5 runs after one warm-up, ms per call
    shapes = {}
    for m, k in ((128, 4096), (1, 4096), (16, 4096), (64, 4096), (256, 4096), (1024, 4096)):
        xs = gi.outlier_activations(m, k, seed=4300 + m)
        g = gi.torch_style_gsi(xs, FP8_MAX)
        oracle.quantize(xs, g, nthreads=threads)
        times = []
        for _ in range(5):
            t = time.perf_counter()
            oracle.quantize(xs, g, nthreads=threads)
            times.append(time.perf_counter() - t)
        ms = sorted(times)[2] * 1e3
        shapes[f"{m}x{k}"] = {"ms": round(ms, 4),
                              "GB/s": round(m * k * BYTES_PER_ELEM / (ms * 1e-3) / 1e9, 4)}
    return {"value": round(rows * K_DIM * BYTES_PER_ELEM / dt / 1e9, 4), "unit": UNIT,
            "cores": threads, "kind": "port",
            "sample": f"{rows} x {K_DIM} rows of the workload ({rows * K_DIM // 16} blocks; "
                      f"{reps} x a {chunk}-row draw), {dt:.2f} s, oracle/scalesweep_oracle.c "
                      f"with {threads} OpenMP threads",
            "shapes": shapes}


def run_reference(args):
    """Reference arm: the reference algorithm on the host cores, bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np  # noqa: F401
    import oracle
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import golden_inputs as gi
    oracle.lib()
    threads = os.cpu_count() or 1
    rows = 256
    x = gi.outlier_activations(rows, K_DIM, seed=4244)
    gsi = gi.torch_style_gsi(x, FP8_MAX)
    # size the per-step sample so W+K steps take about two minutes in total
    t = time.perf_counter()
    oracle.quantize(x, gsi, nthreads=threads)
    dt = max(time.perf_counter() - t, 1e-4)
    per_step_budget = 120.0 / max(1, args.steps + args.warmup)
    rows = max(64, int(rows * per_step_budget / dt) // 64 * 64)
    rows = min(rows, args.rows)
    # at most 16384 freshly drawn rows (drawing and rounding them in numpy
    # costs more than quantizing them), quantized as often as the step budget
    # asks: the per-row work of the oracle does not depend on the values
    chunk = min(rows, 16384)
    reps = max(1, rows // chunk)
    rows = reps * chunk
    x = gi.outlier_activations(chunk, K_DIM, seed=4245)
    gsi = gi.torch_style_gsi(x, FP8_MAX)

    def one_step():
        for _ in range(reps):
            oracle.quantize(x, gsi, nthreads=threads)
    for _ in range(args.warmup):
        one_step()
    t = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    dt = (time.perf_counter() - t) / args.steps
    value = rows * K_DIM * BYTES_PER_ELEM / dt / 1e9
    sample = (f"{rows} x {K_DIM} rows of the workload per step ({reps} x a {chunk}-row draw), "
              f"oracle/scalesweep_oracle.c (plain-C restatement of the reference kernel), "
              f"{threads} OpenMP threads")
    line = {"metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "rows": args.rows, "k": K_DIM,
                       "sample_rows": rows, "backend": "scalesweep_mse"},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist
    from test_speed_scalesweep_b200 import _lib, custom, global_scale, sharded
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    _lib.lib()  # fail loudly if the CUDA library is missing
    if world > 1:
        from datetime import timedelta
        # NCCL's init lines (rank count, NVLink/NVLS transport) go to stderr
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    if args.rows % (CHUNK_ROWS * world):
        raise SystemExit(f"rows must be a multiple of {CHUNK_ROWS} * world_size")
    rows = args.rows // world
    k = K_DIM
    row0 = rank * rows
    x = make_global_rows(row0, rows, k, device)
    codes, scales = custom.create_fp4_output_tensors(rows, k, device, True)
    amax = torch.empty(1, dtype=torch.float32, device=device)
    gsi = torch.empty(1, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    def step(inp=x):
        if world == 1:
            global_scale.global_scale_inv_from_max(inp, FP8_MAX, out=gsi)
        else:
            global_scale.absmax(inp, out=amax)
            sharded.all_reduce_amax(amax)
            global_scale.global_scale_from_amax(amax, FP8_MAX, out=gsi)
        mse.scalesweep_mse_nvfp4_quant_out(inp, gsi, True, output=codes, output_scale=scales)

    launches_per_step = 2 if world == 1 else 3

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    bus = None
    try:
        p = torch.cuda.get_device_properties(device)
        bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        pass
    sampler = ClockSampler(bus)
    sampler.start()
    time.sleep(0.3)
    # Ranks leave the sampler start-up at different times; line them up right
    # before the first timed step, or an early rank's window would include
    # waiting for the others in its first all-reduce.
    barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms_total = start.elapsed_time(end)
    clocks = sampler.stop()
    t = torch.tensor([ms_total], dtype=torch.float64, device=device)
    rank_ms = [round(ms_total / args.steps, 4)]
    if world > 1:
        every = torch.zeros(world, dtype=torch.float64, device=device)
        every[rank] = ms_total / args.steps
        dist.all_reduce(every, op=dist.ReduceOp.SUM)
        rank_ms = [round(v, 4) for v in every.tolist()]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = t.item() / args.steps
    total_bytes = args.rows * k * BYTES_PER_ELEM
    value = total_bytes / (ms_step * 1e-3) / 1e9

    # dominant kernel alone: the quantizer, each launch bracketed by events
    quant = lambda: mse.scalesweep_mse_nvfp4_quant_out(x, gsi, True, output=codes,  # noqa: E731
                                                       output_scale=scales)
    q_ms = kernel_avg_ms(quant, max(3, args.steps), stream)
    amax_ms = kernel_avg_ms(lambda: global_scale.global_scale_inv_from_max(x, FP8_MAX, out=gsi),
                            max(3, args.steps), stream)
    hbm_peak, sm_max, peak_src = load_peaks()
    shard_bytes = rows * k * BYTES_PER_ELEM
    achieved = shard_bytes / (q_ms * 1e-3) / 1e9
    per_block, traffic_src = load_traffic_profile()
    traffic = round(per_block * rows * k / 16) if per_block else None
    clk = (clocks or {}).get("sm_mhz") or sm_max
    alu_peak_gbs = (SM_COUNT * FP32_LANES_PER_SM * clk * 1e6 / ALU_OPS_PER_ELEM) * \
        BYTES_PER_ELEM / 1e9
    # The binding roofline is the slower of HBM and the sweep's FP32-ALU bound
    # (35 FP32 operations per element at 148 SMs x 128 lanes x the SM clock
    # sampled during the timed region), both in algorithmic GB/s.
    bound = "alu" if alu_peak_gbs < hbm_peak else "hbm"
    peak = min(alu_peak_gbs, hbm_peak)
    roofline = {"bound": bound, "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                "peak_source": (f"FP32-ALU bound: {SM_COUNT} SMs x {FP32_LANES_PER_SM} lanes x "
                                f"{clk:.0f} MHz / {ALU_OPS_PER_ELEM} ops per element x "
                                f"{BYTES_PER_ELEM} B per element (HBM bound: MEASURED_PEAKS.json "
                                f"hbm_gbs {hbm_peak:.0f}, {peak_src})"),
                "kernel": "quant_kernel (scale-sweep MSE, 11 candidates)",
                "kernel_ms": round(q_ms, 4),
                "algorithmic_bytes_per_launch": shard_bytes,
                "traffic_source": traffic_src,
                "alu": {"ops_per_elem": ALU_OPS_PER_ELEM, "sm_mhz": clk,
                        "peak_equiv_gbs": round(alu_peak_gbs, 1),
                        "frac": round(achieved / alu_peak_gbs, 4)},
                "hbm": {"peak_gbs": hbm_peak, "frac": round(achieved / hbm_peak, 4),
                        "source": f"MEASURED_PEAKS.json hbm_gbs ({peak_src})"},
                "amax_kernel_ms": round(amax_ms, 4),
                "amax_achieved_gbs": round(rows * k * 2 / (amax_ms * 1e-3) / 1e9, 1)}

    # end to end: pinned host input -> device -> quantize -> codes+scales back to pinned host
    e2e = None
    if not args.no_e2e:
        h_in = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        h_in.copy_(x)
        h_codes = torch.empty(codes.shape, dtype=codes.dtype, pin_memory=True)
        h_scales = torch.empty(scales.shape, dtype=scales.dtype, pin_memory=True)
        x_dev = torch.empty_like(x)

        def e2e_step():
            x_dev.copy_(h_in, non_blocking=True)
            step(x_dev)
            h_codes.copy_(codes, non_blocking=True)
            h_scales.copy_(scales, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e_steps = max(3, min(args.steps, 5))
        e_ms = time_events(e2e_step, e_steps, stream)
        et = torch.tensor([e_ms], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e_ms = et.item()
        e2e = {"value": round(total_bytes / (e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": int(x.numel() * 2 * world),
               "d2h_bytes_per_step": int((codes.numel() + scales.numel() * 4) * world),
               "ms_per_step": round(e_ms, 3), "steps": e_steps,
               "path": "pinned host -> cudaMemcpyAsync -> global_scale + nvfp4 quant (public API) "
                       "-> codes and scales to pinned host"}
        del h_in, h_codes, h_scales, x_dev

    # whole-tensor bit-exactness against one GPU: every rank hashes its
    # 16384-row chunks (codes + scale slab) and compares them with the
    # committed digests of a one-GPU run of the same tensor
    step()
    torch.cuda.synchronize()
    mine = chunk_digests(codes, scales, row0)
    gsi_bits = int(gsi.view(torch.int32).item())
    record = None
    if os.path.exists(DIGEST_PATH):
        with open(DIGEST_PATH) as f:
            record = json.load(f)
    comparable = (record is not None and record.get("rows") == args.rows and
                  record.get("k") == k and record.get("chunk_rows") == CHUNK_ROWS)
    ok = comparable and all(record["digests"].get(c) == d for c, d in mine.items()) and \
        record.get("gsi_bits") == gsi_bits
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    if world > 1:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    bitexact = {"bitexact_vs_1gpu": bool(flag.item()) if comparable else None,
                "chunks_checked": len(mine) * world, "chunk_rows": CHUNK_ROWS,
                "record": os.path.relpath(DIGEST_PATH, ROOT) if comparable else
                "no one-GPU record for this tensor size",
                "gsi_bits": f"0x{gsi_bits & 0xFFFFFFFF:08X}"}
    if args.write_config5_digests:
        if world != 1:
            raise SystemExit("--write-config5-digests is a one-GPU run")
        with open(args.write_config5_digests, "w") as f:
            json.dump({"rows": args.rows, "k": k, "chunk_rows": CHUNK_ROWS,
                       "gsi_bits": gsi_bits, "digests": mine,
                       "made_by": "python bench.py --no-sweep --no-gemm --no-cpu --no-e2e "
                                  "--write-config5-digests <file> on one B200",
                       "hash": "sha256 of each chunk's codes bytes then its scale slab bytes"},
                      f, indent=1)

    sweep = None
    ref_triton = None
    cpu = None
    gemm_res = None
    quality = None
    act_fusion = None
    norm_fusion = None
    if rank == 0 and world == 1:
        del x
        torch.cuda.empty_cache()
        if not args.no_sweep:
            sweep = run_sweep(device)
        if not args.no_ref_triton:
            ref_triton = run_reference_triton_sweep(device)
        if not args.no_gemm:
            gemm_res = run_gemm_sweep(device)
        if not args.no_sweep:
            quality = run_quality(device)
            act_fusion = run_act_fusion_sweep(device)
            norm_fusion = run_norm_fusion_sweep(device)
        if not args.no_cpu:
            cpu = cpu_sample_rate(args.rows)

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "rows": args.rows, "k": k,
                           "rows_per_gpu": rows, "backend": "scalesweep_mse",
                           "candidates": 11, "swizzled_scales": True, "fp8_max": FP8_MAX,
                           "l2": "inputs larger than L2 (no flush needed)",
                           "step": "amax -> (NCCL MAX all-reduce if N>1) -> scale -> quantize"},
                "gpu_launches": launches_per_step * args.steps,
                "rank_ms_per_step": rank_ms,
                "roofline": roofline, "clocks": clocks, "e2e": e2e, **bitexact}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if sweep is not None:
            line["sweep"] = sweep
        if ref_triton is not None:
            line["sweep_vs_reference_triton"] = ref_triton
        if quality is not None:
            line["quality_mse"] = quality
        if gemm_res is not None:
            line["gemm"] = gemm_res
        if act_fusion is not None:
            line["act_fusion"] = act_fusion
        if norm_fusion is not None:
            line["norm_fusion"] = norm_fusion
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_profile_case(args):
    import torch
    from test_speed_scalesweep_b200 import custom, global_scale
    m, k = (int(v) for v in args.profile_case.lower().split("x"))
    device = torch.device("cuda", 0)
    x = make_shard(m, k, 99, device)
    gsi = global_scale.global_scale_inv_from_max(x, FP8_MAX)
    for _ in range(4):
        custom.nvfp4_quant(x, gsi, True, args.profile_backend)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": [m, k], "backend": args.profile_backend}))


def run_profile_gemm(args):
    import torch
    from test_speed_scalesweep_b200 import global_scale
    from test_speed_scalesweep_b200 import scalesweep_mse_nvfp4_utils as mse
    from test_speed_scalesweep_b200.gemm import cutlass_scaled_fp4_mm
    m, n, k = (int(v) for v in args.profile_gemm.lower().split("x"))
    device = torch.device("cuda", 0)
    x = make_shard(m, k, 5, device)
    w = make_shard(n, k, 6, device)
    gx = global_scale.global_scale_inv_from_max(x, FP8_MAX)
    gw = global_scale.global_scale_inv_from_max(w, FP8_MAX)
    qa, sa = mse.scalesweep_mse_nvfp4_quant_impl(x, gx, True)
    qb, sb = mse.rtn_nvfp4_quant_impl(w, gw, True)
    alpha = (1.0 / (gx * gw)).reshape(1).float()
    for _ in range(4):
        cutlass_scaled_fp4_mm(qa, qb, sa, sb, alpha)
    torch.cuda.synchronize()
    print(json.dumps({"profile_gemm": [m, n, k]}))


def run_profile_amax(args):
    import torch
    from test_speed_scalesweep_b200 import global_scale
    m, k = (int(v) for v in args.profile_amax.lower().split("x"))
    x = make_shard(m, k, 7, torch.device("cuda", 0))
    for _ in range(4):
        global_scale.global_scale_inv_from_max(x, FP8_MAX)
    torch.cuda.synchronize()
    print(json.dumps({"profile_amax": [m, k]}))


def run_profile_amax_noalloc(args):
    """The allocation-free global-scale entry point (fixed device scratch) 4
    times on one [M, K] bf16 input, through the C ABI; for ncu."""
    import ctypes
    import torch
    from test_speed_scalesweep_b200 import _lib
    lib = _lib.lib()
    m, k = (int(v) for v in args.profile_amax_noalloc.lower().split("x"))
    if m * k > lib.ssw_global_scale_inv_noalloc_max_numel():
        raise SystemExit("above the allocation-free entry point's maximum size")
    x = make_shard(m, k, 7, torch.device("cuda", 0))
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(4):
        st = lib.ssw_global_scale_inv_noalloc(ctypes.c_void_p(x.data_ptr()), 0, x.numel(),
                                              FP8_MAX, ctypes.c_void_p(out.data_ptr()), None,
                                              ctypes.c_void_p(stream))
        if st != 0:
            raise SystemExit(f"ssw_global_scale_inv_noalloc returned {st}")
    torch.cuda.synchronize()
    print(json.dumps({"profile_amax_noalloc": [m, k]}))


def run_profile_act(args):
    import torch
    from test_speed_scalesweep_b200 import act_quant
    m, n = (int(v) for v in args.profile_act.lower().split("x"))
    device = torch.device("cuda", 0)
    x = make_shard(m, 2 * n, 17, device)
    gsi = torch.tensor([FP8_MAX * 6.0 / 40.0], dtype=torch.float32, device=device)
    h = torch.empty(m, n, dtype=x.dtype, device=device)
    codes, scales = act_quant.alloc_outputs(x, True)
    for _ in range(4):
        act_quant.silu_and_mul(x, h)
    for _ in range(4):
        act_quant.silu_and_mul_scalesweep_mse_nvfp4_quant_out(x, gsi, True, output=codes,
                                                              output_scale=scales)
    torch.cuda.synchronize()
    print(json.dumps({"profile_act": [m, n]}))


def run_profile_norm(args):
    import torch
    from test_speed_scalesweep_b200 import norm_quant
    m, n = (int(v) for v in args.profile_norm.lower().split("x"))
    device = torch.device("cuda", 0)
    x = make_shard(m, n, 29, device)
    res = make_shard(m, n, 31, device)
    w = torch.ones(n, dtype=torch.bfloat16, device=device)
    gsi = torch.tensor([FP8_MAX * 6.0 / 40.0], dtype=torch.float32, device=device)
    codes, scales = norm_quant.alloc_outputs(x, True)
    for resid in (None, res):
        for _ in range(4):
            norm_quant.rms_norm_scalesweep_mse_nvfp4_quant_out(
                x, w, 1e-5, gsi, True, output=codes, output_scale=scales, residual=resid)
    torch.cuda.synchronize()
    print(json.dumps({"profile_norm": [m, n]}))


def register_reference_quant_op():
    """The reference's Triton ``scalesweep_mse_nvfp4_quant_impl`` as a torch op,
    registered the way the reference's vLLM fork registers it (the names in
    test_kernel_latency.py:41-47; its fake implementation
    bench_kernel/scalesweep_mse_nvfp4_utils.py:546-560), from the unmodified
    install under baseline/_ref.  SCALESWEEP_TUNE=0: one kernel configuration,
    as run_bench_tune.sh exports for its end-to-end runs."""
    import torch
    os.environ["SCALESWEEP_TUNE"] = "0"
    if not os.path.isdir(os.path.join(REF_DIR, "bench_kernel")):
        raise SystemExit("reference not installed under baseline/_ref "
                         "(python baseline/install_ref.py)")
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    from bench_kernel import scalesweep_mse_nvfp4_utils as k1
    from vllm.utils.torch_utils import direct_register_custom_op
    direct_register_custom_op("scalesweep_mse_nvfp4_quant", k1.scalesweep_mse_nvfp4_quant_impl,
                              mutates_args=[], fake_impl=k1._scalesweep_mse_nvfp4_quant_fake)
    return torch.ops.vllm.scalesweep_mse_nvfp4_quant


def run_vllm_arm(args):
    """One vLLM engine with one arm; prints its result as one JSON line."""
    from test_speed_scalesweep_b200 import vllm_e2e
    input_len, output_len, batches = VLLM_WORKLOADS[args.vllm_workload]
    arm = args.vllm_arm
    if arm == "reference_triton":
        res = vllm_e2e.run("cutlass", batches, input_len, output_len,
                           quant_op=register_reference_quant_op())
    else:
        res = vllm_e2e.run(arm, batches, input_len, output_len)
    res["arm"] = arm
    print("VLLM_ARM_RESULT " + json.dumps(res), flush=True)


def run_vllm_e2e(args):
    """Arms interleaved over repeats (arm order rotated each round), one engine
    process per run; per batch size the mean, min and max output tok/s of
    each arm, and each arm's mean over the reference Triton arm's mean."""
    input_len, output_len, batches = VLLM_WORKLOADS[args.vllm_workload]
    arms = list(args.vllm_arms)
    runs = {a: [] for a in arms}
    meta = {}
    failures = []
    for r in range(args.vllm_repeats):
        order = arms[r % len(arms):] + arms[:r % len(arms)]
        for arm in order:
            cmd = [sys.executable, os.path.abspath(__file__), "--vllm-arm", arm,
                   "--vllm-workload", args.vllm_workload]
            env = dict(os.environ, VLLM_ENABLE_V1_MULTIPROCESSING="0")
            t0 = time.time()
            proc = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=1800)
            line = [ln for ln in proc.stdout.splitlines() if ln.startswith("VLLM_ARM_RESULT ")]
            if proc.returncode != 0 or not line:
                failures.append({"arm": arm, "repeat": r, "rc": proc.returncode,
                                 "tail": (proc.stdout + proc.stderr)[-800:]})
                continue
            res = json.loads(line[-1][len("VLLM_ARM_RESULT "):])
            res["process_seconds"] = round(time.time() - t0, 1)
            runs[arm].append(res)
            meta.setdefault(arm, []).append(
                {k: v for k, v in res.items()
                 if "_calls" in k or k.endswith(("_matches", "_names", "_seconds", "_layers"))})
    out = {"vllm_e2e": f"Llama-3.1-8B architecture W4A4 in vLLM, one B200, {input_len} in / "
                       f"{output_len} out, CUDA graphs, fusion passes off",
           "workload": args.vllm_workload, "repeats": args.vllm_repeats,
           "order": "arms interleaved, order rotated each repeat; one engine process per run",
           "arms": {a: VLLM_ARMS[a] for a in arms}, "batch": {}, "failures": failures,
           "per_run": meta}
    for bs in batches:
        row = {}
        for arm in arms:
            vals = [r["batch"][str(bs)]["output_tok_s"] for r in runs[arm]]
            if vals:
                row[arm] = {"mean": round(statistics.mean(vals), 2), "min": min(vals),
                            "max": max(vals), "runs": vals}
        ref = row.get("reference_triton", {}).get("mean")
        if ref:
            for arm in arms:
                if arm in row:
                    row[arm]["over_reference_triton"] = round(row[arm]["mean"] / ref, 4)
        out["batch"][str(bs)] = row
    print(json.dumps(out), flush=True)


def main():
    args = parse_args()
    if args.vllm_arm:
        run_vllm_arm(args)
        return
    if args.vllm_e2e:
        run_vllm_e2e(args)
        return
    if args.gemm_crossover:
        run_gemm_crossover(args)
        return
    if args.profile_case:
        run_profile_case(args)
        return
    if args.profile_gemm:
        run_profile_gemm(args)
        return
    if args.profile_amax:
        run_profile_amax(args)
        return
    if args.profile_amax_noalloc:
        run_profile_amax_noalloc(args)
        return
    if args.profile_act:
        run_profile_act(args)
        return
    if args.profile_norm:
        run_profile_norm(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()

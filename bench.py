"""Benchmark of the B200 Conformer conv-module kernels.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--scaling strong|weak]
                    [--workload stack|module|module_i8|module_w8a8|dw|dw_cf|dw_cf_glu|ff|attn|block|encoder|ctc]

Default workload ("stack"): 16 conv-module layers (independent seeds) over 512 synthetic utterances with lognormal
lengths (median 600 frames, sigma 0.5, clipped to [64, 1536]), sorted by length, logical batches of 128 cut into
execution chunks of <= 48 padded to the 128-frame grid.  One step = every chunk through all 16 layers.  On N GPUs
(one process per GPU under torchrun) the one set of 512 utterances is split over the ranks (strong scaling, the
default: length-sorted utterances dealt round robin, each rank chunking its share), or with --scaling weak every rank
owns its own 512.  No collective runs in the loop; value = valid frames x 16 layers of all ranks / the slowest
rank's time.  Inputs are resident in HBM and larger than L2 (~0.7 GB per step on one GPU).

Other workloads (single-GPU measurements): "module" = one conv module on one B=48 chunk (lognormal lengths, T on
the 128 grid), "module_i8" = the same with int8 weights, "module_w8a8" = int8 weights and activations, "dw" = the
depthwise kernel alone on [48, 1024, 2048] channels-last, "dw_cf" / "dw_cf_glu" = the depthwise op at the
reference's call site, (48, 2048, 1024) channels-first (and its GLU form on the (48, 4096, 1024) up_conv output),
"ff" = one feed-forward half on the B=48 chunk, "attn" = one attention step (block-local, Shaw relative positions),
"block" = one whole Conformer block (FF/2, attention, conv, FF/2, post norm), "encoder" = the whole CTC encoder
over the stack's 512 utterances: 160-dim input features projected to 1024, 16 Conformer blocks, the
self-conditioning CTC head after block 8 and the BPE CTC head (100352-word vocabulary, argmax fused into the GEMM,
CTC collapse) at the end, "ctc" = those heads alone on the B=48 chunk.

The CPU baseline (``cpu_baseline`` and ``--impl reference``, rank 0 only) times, for the conv-module and depthwise
workloads, the torch restatement of the reference's eager op calls (oracle/torch_eager.py) on every host core in
float32 and bfloat16 and keeps the faster; for the other workloads the numpy oracle.  It runs on a bounded sample
(up to 8 utterances of every chunk at the chunk's padded T) and ``--impl reference`` prints the same JSON line with
"impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "granite-speech-4.1-2b-nar-turbo_b200"))

if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    # NCCL's own log on stderr (version, and with this NCCL the communicator lines where it prints them); NCCL reads
    # these when the library loads, i.e. before torch is imported below.  The bench also prints the process group
    # (backend, world size, each rank's GPU) from the ranks themselves
    os.environ.setdefault("NCCL_DEBUG", "INFO")

from granite_conv_b200 import dispatch, synth  # noqa: E402

N_LAYERS = 16
N_UTTS = 512
D, I = synth.D_MODEL, synth.D_INNER
GEMM1_FLOP_PER_FRAME = 2 * D * 2 * I          # 8.389 MFLOP
GEMM2_FLOP_PER_FRAME = 2 * I * D              # 4.194 MFLOP
FF_FLOP_PER_FRAME = 2 * D * 4 * D             # 8.389 MFLOP per feed-forward GEMM
HEADS, DIM_HEAD, CONTEXT = synth.NUM_HEADS, synth.DIM_HEAD, synth.CONTEXT
QKV_FLOP_PER_FRAME = 2 * D * 3 * HEADS * DIM_HEAD       # 6.291 MFLOP
OUT_FLOP_PER_FRAME = 2 * HEADS * DIM_HEAD * D           # 2.097 MFLOP
# attention: per valid query frame, head and valid key of its block: q.k, q.rel[i - j] and p.v (2 x 128 each)
ATTN_FLOP_PER_QUERY_KEY = 3 * 2 * DIM_HEAD * HEADS      # 6144
# DRAM bytes (read + write) of the fused up_conv + GLU + depthwise kernel (LayerNorm folded) per row of the 128-row
# tiles it computes, from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of the module workload's
# B=48, T=1536 chunk: 72.66 + 84.82 MB over 31,104 rows.  The traffic of a launch scales with the rows it computes.
# A constant: it is re-captured whenever the kernel changes (the command is in the kernel's ncu summary).
GEMM1DW_DRAM_BYTES_PER_ROW = 5063
DW_BYTES_PER_FRAME = 2 * I * 2                # read + write bf16: 8192 B
DW_GLU_BYTES_PER_FRAME = 3 * I * 2            # GLU form: read value + gate, write: 12288 B
DW_WORKLOADS = ("dw", "dw_cf", "dw_cf_glu")
METRIC = "conv-module frames/s at 1/2/4/8 B200; % of HBM / tensor-pipe roofline"


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _int8_peak_tops(dev, sustained_s: float = 3.0):
    """Dense int8 tensor-core throughput of this GPU, measured here: torch._int_mm (cuBLASLt, s32 accumulate) on
    8192^3 int8, 2 * 8192^3 ops per call, timed by CUDA events -- best of 10 single calls (burst) and back to back
    for `sustained_s` seconds (sustained, under the power cap).  The denominator of the W8A8 kernels' fractions."""
    import torch
    n = 8192
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev, generator=g).t()   # column-major operand
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize(dev)
    ops = 2.0 * n ** 3
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    calls = max(1, int(sustained_s * 1e3 / best))
    e0.record()
    for _ in range(calls):
        torch._int_mm(a, b)
    e1.record()
    e1.synchronize()
    sus = e0.elapsed_time(e1) / calls
    return {"int8_tops": ops / (best / 1e3) / 1e12, "int8_tops_sustained": ops / (sus / 1e3) / 1e12,
            "how": f"torch._int_mm int8 8192^3, best of 10 (burst) and {calls} calls back to back (sustained)"}


# ----------------------------------------------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML every 200 ms while running."""

    REASONS = {
        0x0000000000000004: "sw_power_cap", 0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown", 0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown", 0x0000000000000002: "applications_clocks_setting",
    }

    def __init__(self, torch_device_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        self._handle = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(torch_device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
            self._nvml = pynvml
        except Exception as e:  # noqa: BLE001
            self.error = f"nvml unavailable: {e}"

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        if self._handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "note": getattr(self, "error", "no samples")}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------------------------------
def _dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _workload_plan(rank: int, workload: str, world: int = 1, scaling: str = "strong", shard: str = "utterances"):
    """Chunks of this rank (list of dispatch.Chunk) for the workload.  stack / encoder: strong scaling splits one set
    of 512 utterances over the ranks (dealt as utterances, each rank chunking its share, or as whole chunks of the
    one plan); weak scaling gives every rank its own 512."""
    if workload in ("stack", "encoder"):
        plan = lambda ls: dispatch.plan_chunks(ls, exec_batch=dispatch.EXEC_BATCH,  # noqa: E731
                                               logical_batch=dispatch.LOGICAL_BATCH, frame_grid=dispatch.FRAME_GRID)
        if scaling == "weak":
            return plan(synth.sample_lengths(1005 + 7919 * rank, N_UTTS))
        lens = synth.sample_lengths(1005, N_UTTS)
        if shard == "chunks":
            return dispatch.shard_chunks(plan(lens), world)[rank].chunks
        mine = dispatch.shard_utterances(lens, world)[rank]
        return plan(lens[mine])
    if workload in ("module", "module_i8", "module_w8a8", "ff", "attn", "block", "ctc"):
        lens = synth.sample_lengths(1003 + 7919 * rank, 48)
        T = synth.round_up(int(lens.max()), synth.FRAME_GRID)
        return [dispatch.Chunk(index=np.arange(48), lengths=lens, T=T)]
    if workload in DW_WORKLOADS:
        return [dispatch.Chunk(index=np.arange(48), lengths=np.full(48, 1024, np.int32), T=1024)]
    raise ValueError(workload)


def _layers_for(workload: str) -> int:
    return N_LAYERS if workload in ("stack", "encoder") else 1


# ----------------------------------------------------------------------------------------------------------------
def cpu_oracle_rate(workload: str, budget_s: float, rank: int = 0):
    """frames/s (valid frames x layers per second) of the numpy oracle (float32, all host threads through BLAS) on a
    bounded sample of the workload: the shortest chunks of the plan, one layer each, until budget_s is spent."""
    from oracle import conv_module as O
    from oracle import attention as ATO
    from oracle import feed_forward as FFO
    chunks = _workload_plan(rank, workload)
    if workload in DW_WORKLOADS:
        w, b = synth.make_dw_weights(1002)
        wb, bb = O.bf16_round(w), O.bf16_round(b)
    elif workload == "ff":
        ffprep = FFO.prepare_ff_fp32(synth.make_ff_params(1006))
    elif workload == "attn":
        atprep = ATO.prepare_attn_fp32(synth.make_attn_params(1007))
    elif workload in ("block", "encoder"):
        from oracle import block as BKO
        bkprep = BKO.prepare_block(synth.make_block_params(1008), mode="fp32")
    elif workload == "ctc":
        from oracle import ctc_head as CHO
        chprep = CHO.prepare_ctc_fp32(synth.make_ctc_params(1009))
    else:
        params = synth.make_params(1005)
        prep = O.prepare_fp32(params)
    frames = 0
    t0 = time.perf_counter()
    done = 0
    sample_desc = []
    i = 0
    while True:
        c = chunks[i % len(chunks)]
        B = min(c.B, 4)
        T = int(c.lengths[:B].max())
        x = synth.make_activations(77 + i, (B, T, (2 * I if workload == "dw_cf_glu" else I)
                                               if workload in DW_WORKLOADS else D))
        lens = c.lengths[:B]
        if workload == "dw_cf_glu":
            O.dwconv_silu_glu(x, wb, bb, lengths=lens)
        elif workload in DW_WORKLOADS:
            O.dwconv_silu(x, wb, bb, lengths=lens, round_out=False)
        elif workload == "ff":
            FFO.feed_forward_half(x, ffprep, lengths=lens, mode="fp32", dtype=np.float32)
        elif workload == "attn":
            ATO.attention_block(x, atprep, lengths=lens, mode="fp32", dtype=np.float32)
        elif workload in ("block", "encoder"):
            BKO.conformer_block(x, bkprep, lengths=lens, mode="fp32", dtype=np.float32)
        elif workload == "ctc":
            hh, bl = CHO.selfcond(x, chprep, lengths=lens, mode="fp32", dtype=np.float32)
            CHO.decode(hh, bl, chprep, lengths=lens, mode="fp32")
        else:
            O.conv_module(x, prep, lengths=lens, mode="fp32", dtype=np.float32)
        frames += int(lens.sum())
        done += 1
        sample_desc.append((B, T))
        i += 1
        if time.perf_counter() - t0 >= budget_s:
            break
    dt = time.perf_counter() - t0
    cores = len(os.sched_getaffinity(0))
    desc = (f"{done} chunk slices (first 4 utterances of each chunk, 1 layer each, float32 numpy oracle), "
            f"{frames} valid frames in {dt:.1f} s")
    return frames / dt, cores, desc


EAGER_WORKLOADS = ("stack", "module", "module_i8", "module_w8a8", "dw", "dw_cf", "dw_cf_glu")


def _eager_sample(workload: str, rank: int = 0):
    """The bounded CPU sample: from every chunk of the workload's plan, 8 utterances evenly spaced in the chunk (all
    of them if fewer), at the chunk's padded T -- the reference's eager path processes a chunk as its padded tensor.
    Returns [(B, T, valid frames)]."""
    out = []
    for c in _workload_plan(rank, workload):
        idx = np.unique(np.linspace(0, c.B - 1, min(8, c.B)).round().astype(int))
        out.append((len(idx), c.T, int(c.lengths[idx].sum())))
    return out


class EagerBaseline:
    """CPU baseline of the conv-module and depthwise workloads: the torch restatement of the reference's eager op
    calls (oracle/torch_eager.py, bit-identical to the reference on its goldens) on every host core, in float32 and
    bfloat16 (the reference module's dtype; oneDNN uses the host's bf16 units where it has them).  A pass runs one
    layer over the sample; the faster dtype is the baseline."""

    def __init__(self, workload: str):
        import torch

        from oracle import torch_eager as TE
        self.torch, self.TE, self.workload = torch, TE, workload
        self.cores = TE.host_threads()
        torch.set_num_threads(self.cores)
        self.sample = _eager_sample(workload)
        self.mods = {}
        w, b = synth.make_dw_weights(1002)
        for dt in (torch.float32, torch.bfloat16):
            if workload in DW_WORKLOADS:
                self.mods[dt] = (torch.from_numpy(w).to(dt), torch.from_numpy(b).to(dt))
            else:
                self.mods[dt] = TE.EagerConvModule(synth.make_params(1005), dt)
        g = torch.Generator().manual_seed(77)
        cin = {"dw_cf_glu": 2 * I}.get(workload, I if workload in DW_WORKLOADS else D)
        self.inputs = {dt: [torch.randn((B, cin, T) if workload in DW_WORKLOADS else (B, T, cin), generator=g).to(dt)
                            for B, T, _ in self.sample] for dt in self.mods}

    def _one(self, dt, x):
        if self.workload in DW_WORKLOADS:
            w, b = self.mods[dt]
            return (self.TE.dwconv_silu_glu if self.workload == "dw_cf_glu" else self.TE.dwconv_silu)(x, w, b)
        return self.mods[dt](x)

    def pass_rate(self, dt) -> float:
        """valid frames per second of one pass over the sample"""
        t0 = time.perf_counter()
        for x in self.inputs[dt]:
            self._one(dt, x)
        return sum(v for _, _, v in self.sample) / (time.perf_counter() - t0)

    def describe(self, dt, rates) -> str:
        frames = sum(v for _, _, v in self.sample)
        padded = sum(B * T for B, T, _ in self.sample)
        what = ("depthwise conv + SiLU" + (" after GLU" if self.workload == "dw_cf_glu" else "")
                if self.workload in DW_WORKLOADS else "conv module + residual, 1 layer")
        per_dtype = ", ".join(f"{_dtype_name(k)} {v / 1e3:.1f} k" for k, v in rates.items())
        return (f"torch eager restatement of the reference's op calls ({what}) on {self.cores} host threads; a pass = "
                f"{len(self.sample)} chunks x up to 8 utterances at the chunk's padded T ({frames} valid / {padded} "
                f"padded frames); {_dtype_name(dt)} was the faster dtype ({per_dtype} frames/s)")


def _dtype_name(dt) -> str:
    return {"torch.float32": "f32", "torch.bfloat16": "bf16"}.get(str(dt), str(dt))


def cpu_baseline_rate(workload: str, budget_s: float):
    """(frames/s, cores, kind, description) of the CPU baseline on a bounded sample of the workload."""
    if workload not in EAGER_WORKLOADS:
        r, cores, desc = cpu_oracle_rate(workload, budget_s)
        return r, cores, desc
    eb = EagerBaseline(workload)
    rates = {}
    for dt in eb.mods:
        eb.pass_rate(dt)                          # warm: oneDNN primitives for every shape of the sample
        rates[dt] = eb.pass_rate(dt)
    best = max(rates, key=rates.get)
    return rates[best], eb.cores, eb.describe(best, rates)


def run_reference(args):
    world, rank, _ = _dist_env()
    if rank != 0:
        return 0
    if args.workload in EAGER_WORKLOADS:
        eb = EagerBaseline(args.workload)
        probe = {}
        for dt in eb.mods:                        # a warm pass, then a timed one, of each dtype picks the faster
            eb.pass_rate(dt)
            probe[dt] = eb.pass_rate(dt)
        best = max(probe, key=probe.get)
        for _ in range(max(0, args.warmup - 1)):
            eb.pass_rate(best)
        rates = [eb.pass_rate(best) for _ in range(args.steps)]
        v = float(statistics.median(rates))
        cores, desc = eb.cores, eb.describe(best, probe) + f"; value = median of {args.steps} passes"
        dtype = _dtype_name(best)
    else:
        budget = max(0.5, min(20.0, 60.0 / max(1, args.steps + args.warmup)))
        for _ in range(args.warmup):
            cpu_oracle_rate(args.workload, min(budget, 1.0))
        rates = []
        for _ in range(args.steps):
            r, cores, desc = cpu_oracle_rate(args.workload, budget)
            rates.append(r)
        v = float(statistics.median(rates))
        dtype = "f32"
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "frames/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": _scaling(args),
        "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": _config(args, world),
        "cpu_baseline": {"value": v, "unit": "frames/s", "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _scaling(args) -> str:
    return args.scaling if args.workload in ("stack", "encoder") else "weak"


def _config(args, world):
    w = args.workload
    cfg = {"workload": {
        "stack": "16-layer Conformer conv-module stack (LN, 1024->4096 GEMM+GLU, dw k15+SiLU, 2048->1024 GEMM+"
                 "residual), 512 utterances/rank, lognormal lengths, chunks<=48 on the 128-frame grid",
        "module": "one conv module, B=48 chunk, lognormal lengths, T on the 128-frame grid, length mask",
        "module_i8": "one conv module with int8 per-channel weights, B=48 chunk, lognormal lengths, length mask",
        "module_w8a8": "one conv module with int8 per-channel weights and per-row int8 activations (kind::i8 MMAs, "
                       "s32 accumulate), B=48 chunk, lognormal lengths, length mask",
        "dw": "depthwise k15 + bias + SiLU alone, bf16 [48, 1024, 2048] channels-last, all frames valid",
        "dw_cf": "depthwise k15 + bias + SiLU alone at the reference op's call site: bf16 (48, 2048, 1024) "
                 "channels-first (T innermost, contiguous), all frames valid",
        "dw_cf_glu": "GLU + depthwise k15 + bias + SiLU alone (granite::dwconv_silu_glu at the reference's call site): "
                     "bf16 (48, 4096, 1024) channels-first up_conv output -> (48, 2048, 1024), all frames valid",
        "ff": "one feed-forward half of the Conformer block (LN, 1024->4096 GEMM+SiLU, 4096->1024 GEMM + 0.5x "
              "residual), B=48 chunk, lognormal lengths, T on the 128-frame grid, length mask",
        "attn": "one attention step of the Conformer block (LN, 1024->3072 q|k|v GEMM, block-local attention over "
                "200-frame blocks with Shaw relative positions, 8 heads x 128, 1024->1024 GEMM + residual), B=48 "
                "chunk, lognormal lengths, T on the 128-frame grid, length mask",
        "block": "one Conformer block (FF/2, block-local Shaw attention, conv module, FF/2, post LayerNorm; 14 "
                 "launches), B=48 chunk, lognormal lengths, T on the 128-frame grid, length mask",
        "encoder": "the whole CTC encoder: 160-dim features -> 1024 projection, 16 Conformer blocks (FF/2, attention, "
                   "conv, FF/2, post norm) with the self-conditioning CTC head after block 8 and the BPE CTC head "
                   "(V=100352, fused argmax, collapse) at the end; 512 utterances/rank, lognormal lengths, chunks<=48 "
                   "on the 128-frame grid",
        "ctc": "the encoder's CTC heads alone: self-conditioning (1024->348 GEMM, softmax, 348->1024 GEMM + residual), "
               "posterior-weighted pooling by 4, BPE head 1024->100352 GEMM with the argmax in its epilogue, CTC "
               "collapse; B=48 chunk, lognormal lengths, T on the 128-frame grid"}[w],
        "d_model": D, "d_inner": I, "kernel": 15, "layers": _layers_for(w),
        "exec_batch": dispatch.EXEC_BATCH,
        "frame_grid": dispatch.FRAME_GRID, "parallelism": f"dp{world} (independent shards, no collective)",
        "l2": "inputs larger than L2 (no flush)",
        "frames": "valid encoder frames x layers (padding excluded)"}
    if w in ("stack", "encoder"):
        if args.scaling == "strong":
            cfg["utterances"] = N_UTTS
            cfg["split"] = (f"one set of {N_UTTS} utterances over {world} rank(s): " +
                            ("length-sorted utterances dealt round robin, each rank chunking its share"
                             if args.shard == "utterances" else "whole chunks of one plan, greedy by padded frames"))
        else:
            cfg["utterances_per_rank"] = N_UTTS
    else:
        cfg["utterances_per_rank"] = 48
    return cfg


# ----------------------------------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    from granite_conv_b200 import _lib, ops
    from granite_conv_b200.weights import prepare_from_params

    world, rank, local = _dist_env()
    pg_info = None
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        # which GPU every rank drives, from the ranks themselves (one all_gather before any timing)
        props = torch.cuda.get_device_properties(local)
        mine = {"rank": rank, "local_rank": local, "device": f"cuda:{local}",
                "pci_bus_id": f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}"}
        ranks = [None] * world
        dist.all_gather_object(ranks, mine)
        pg_info = {"backend": dist.get_backend(), "world_size": dist.get_world_size(), "ranks": ranks}
        if rank == 0:
            print(f"process group: {json.dumps(pg_info)}", file=sys.stderr, flush=True)
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    workload = args.workload
    int8 = workload == "module_i8"
    w8a8 = workload == "module_w8a8"
    n_layers = _layers_for(workload)

    chunks = _workload_plan(rank, workload, world, args.scaling, args.shard)
    if not chunks:
        raise RuntimeError(f"rank {rank} of {world} received no chunks; use fewer GPUs or weak scaling")
    valid_frames = sum(c.valid_frames for c in chunks) * n_layers
    padded_frames = sum(c.padded_frames for c in chunks) * n_layers

    # ---- resident inputs and weights
    gen = torch.Generator(device=dev).manual_seed(1005 + rank)
    if workload in DW_WORKLOADS:
        w, b = synth.make_dw_weights(1002)
        dw_w = torch.from_numpy(w).to(torch.bfloat16).to(dev)
        dw_b = torch.from_numpy(b).to(torch.bfloat16).to(dev)
        if workload == "dw":          # [B, T, C] rows
            xs = [torch.randn((c.B, c.T, I), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
            ys = [torch.empty_like(x) for x in xs]
        else:                         # (B, C_in, T) contiguous, T innermost
            cin = 2 * I if workload == "dw_cf_glu" else I
            xs = [torch.randn((c.B, cin, c.T), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
            ys = [torch.empty((c.B, I, c.T), dtype=torch.bfloat16, device=dev) for c in chunks]
        layers = []
    elif workload == "ff":
        from granite_conv_b200.weights import prepare_ff_from_params
        layers = [prepare_ff_from_params(synth.make_ff_params(1006), device=dev)]
        xs = [torch.randn((c.B, c.T, D), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
    elif workload == "attn":
        from granite_conv_b200.weights import prepare_attn_from_params
        layers = [prepare_attn_from_params(synth.make_attn_params(1007), device=dev)]
        xs = [torch.randn((c.B, c.T, D), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
    elif workload in ("block", "encoder"):
        from granite_conv_b200 import prepare_block_from_params
        layers = [prepare_block_from_params(synth.make_block_params(1008 + l), device=dev) for l in range(n_layers)]
        xs = [torch.randn((c.B, c.T, D), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
        if workload == "encoder":       # the input features and the projection 160 -> 1024
            feats = [torch.randn((c.B, c.T, synth.INPUT_DIM), generator=gen, device=dev).to(torch.bfloat16)
                     for c in chunks]
            wi, bi = synth.make_input_params(1010)
            w_in = torch.from_numpy(wi).to(torch.bfloat16).to(dev)
            b_in = torch.from_numpy(bi).to(torch.bfloat16).float().to(dev)
    elif workload == "ctc":
        layers = []
        xs = [torch.randn((c.B, c.T, D), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
    else:
        # bf16: the LayerNorm folded into the up_conv GEMM (the module op's path for T on the 128 grid)
        layers = [prepare_from_params(synth.make_params(1005 + l), device=dev, int8=int8 or w8a8,
                                      ln_fold=not (int8 or w8a8))
                  for l in range(n_layers)]
        xs = [torch.randn((c.B, c.T, D), generator=gen, device=dev).to(torch.bfloat16) for c in chunks]
    heads = None
    if workload in ("encoder", "ctc"):
        from granite_conv_b200.weights import prepare_bpe_head_from_tensors, prepare_selfcond_from_tensors
        cp = synth.make_ctc_params(1009)
        bfh = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
        heads = (prepare_selfcond_from_tensors(bfh(cp.out_weight), bfh(cp.out_bias), bfh(cp.mid_weight),
                                               bfh(cp.mid_bias), device=dev),
                 prepare_bpe_head_from_tensors(bfh(cp.bpe_weight), bfh(cp.bpe_bias), cp.blank_id, cp.window,
                                               device=dev))
    lens_dev = [torch.from_numpy(c.lengths).to(dev) for c in chunks]
    max_m = max(c.padded_frames for c in chunks)
    ws_bytes = int(L.gsn_conv_module_workspace_bytes(1, max_m, D, I))
    if w8a8:
        ws_bytes = max(ws_bytes, int(L.gsn_conv_module_w8a8_workspace_bytes(1, max_m, D, I)))
    if workload == "ff":
        ws_bytes = max(ws_bytes, int(L.gsn_ff_half_workspace_bytes(1, max_m, D, 4 * D)))
    if workload in ("ff", "block", "encoder"):
        ws_bytes = max(ws_bytes, int(L.gsn_ff_half_workspace_bytes(1, max_m, D, 4 * D)))
    if workload in ("attn", "block", "encoder"):
        ws_bytes = max(ws_bytes, int(L.gsn_attention_block_workspace_bytes(1, max_m, D, HEADS, DIM_HEAD)))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    h_buf = ws                                                         # [M, I] GLU output
    t_off = ((max_m * I * 2 + 255) // 256) * 256
    if heads is not None:
        from granite_conv_b200.ops import pooled_frames
        hsc, hbpe = heads
        sc_ws = torch.empty(int(L.gsn_ctc_selfcond_workspace_bytes(1, max_m, hsc.n_cls)), dtype=torch.uint8, device=dev)
        blank_buf = torch.empty(max_m, dtype=torch.float32, device=dev)
        max_pp = max(c.B * pooled_frames(c.T) for c in chunks)
        pooled_buf = torch.empty((max_pp, D), dtype=torch.bfloat16, device=dev)
        plen_buf = torch.empty(max(c.B for c in chunks), dtype=torch.int32, device=dev)
        ids_buf = torch.empty(max_pp, dtype=torch.int32, device=dev)
        tok_buf = torch.empty(max_pp, dtype=torch.int32, device=dev)
        cnt_buf = torch.empty(max(c.B for c in chunks), dtype=torch.int32, device=dev)
        key_ws = torch.empty(int(L.gsn_bpe_head_workspace_bytes(1, max_pp)), dtype=torch.uint8, device=dev)
    act = [torch.empty((c.B, c.T, D), dtype=torch.bfloat16, device=dev) for c in chunks]   # ping-pong buffers
    stats_buf = torch.empty((max_m, D // 256, 2), dtype=torch.float32, device=dev)   # chained layers' row statistics
    act2 = [torch.empty((c.B, c.T, D), dtype=torch.bfloat16, device=dev) for c in chunks]

    layer_events = []      # per recorded layer: (events[4], chunk) around layernorm, gemm1 + dwconv, gemm2
    widen_events = []      # int8: per recorded layer, the events around the weight widening
    w8_events = []         # W8A8: per recorded module call, (start, end, chunk)

    def layer_kernels(x, out, c, p, lens, record, li=0, n_li=1):
        """The kernels of one conv module (the same launches the module op makes for T on the 128 grid): bf16
        weights, layer li of n_li chained as ConvModuleStack runs them (gsn_conv_module_lnfold_chain_bf16): LayerNorm
        statistics (first layer only; later layers read the row statistics the previous down_conv wrote), up_conv +
        GLU + depthwise + SiLU on the raw frames with the LayerNorm folded in, down_conv + residual (writing the row
        statistics of its output unless it is the last layer); int8 weights (widened to bf16 once, when the layer was
        prepared): LayerNorm, the fused up_conv kernel on the LayerNorm output with the column scales, down_conv +
        residual (gsn_conv_module_i8w_widened).  CUDA events between them when `record`."""
        M = c.padded_frames
        if w8a8:
            # the four launches of gsn_conv_module_w8a8 for T on the 128 grid (LayerNorm + quantise, kind::i8 up_conv
            # + GLU + depthwise + SiLU, quantise, kind::i8 down_conv + residual), timed as one call
            e = [torch.cuda.Event(enable_timing=True) for _ in range(2)] if record else None
            if record:
                e[0].record(stream)
            _lib.check(L.gsn_conv_module_w8a8(x.data_ptr(), p.ln_w.data_ptr(), p.ln_b.data_ptr(), p.w1q_glu.data_ptr(),
                                              p.s1_glu.data_ptr(), p.b1_glu.data_ptr(), p.dw_w.data_ptr(),
                                              p.dw_b.data_ptr(), p.w2q.data_ptr(), p.s2.data_ptr(), p.b2.data_ptr(),
                                              lens.data_ptr(), 1, out.data_ptr(), c.B, c.T, D, I, p.ln_eps,
                                              ws.data_ptr(), ws.numel(), sp), "w8a8 module")
            if record:
                e[1].record(stream)
                w8_events.append((e[0], e[1], c))
            return
        dp = h_buf.data_ptr()                   # depthwise output [M, I]
        tp = h_buf.data_ptr() + t_off           # LayerNorm output [M, D]
        lp, T = lens.data_ptr(), c.T
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            ev[0].record(stream)
        has_ln = int8 or li == 0
        if int8:
            _lib.check(L.gsn_layernorm_bf16(x.data_ptr(), D, p.ln_w.data_ptr(), p.ln_b.data_ptr(), tp, D, M, D,
                                            p.ln_eps, lp, T, sp), "layernorm")
        elif has_ln:
            _lib.check(L.gsn_layernorm_stats_bf16(x.data_ptr(), D, tp, M, D, p.ln_eps, lp, T, sp), "ln_stats")
        if record:
            ev[1].record(stream)
        if int8:
            _lib.check(L.gsn_gemm1_glu_dwconv_bf16(tp, p.w1w_glu.data_ptr(), p.s1_glu.data_ptr(), p.b1_glu.data_ptr(),
                                                   p.dw_w.data_ptr(), p.dw_b.data_ptr(), dp, c.B, T, D, 2 * I, lp,
                                                   sp), "gemm1_dw")
        elif has_ln:
            _lib.check(L.gsn_gemm1_lnfold_glu_dwconv_bf16(x.data_ptr(), p.w1g_glu.data_ptr(), p.b1g_glu.data_ptr(),
                                                          p.c1_glu.data_ptr(), tp, p.dw_w.data_ptr(),
                                                          p.dw_b.data_ptr(), dp, c.B, T, D, 2 * I, lp, sp),
                       "gemm1_dw")
        else:
            _lib.check(L.gsn_gemm1_lnfold_partials_glu_dwconv_bf16(
                x.data_ptr(), p.w1g_glu.data_ptr(), p.b1g_glu.data_ptr(), p.c1_glu.data_ptr(), stats_buf.data_ptr(),
                p.ln_eps, p.dw_w.data_ptr(), p.dw_b.data_ptr(), dp, c.B, T, D, 2 * I, lp, sp), "gemm1_dw")
        if record:
            ev[2].record(stream)
        if int8:
            _lib.check(L.gsn_gemm2_residual_bf16s(dp, p.w2w.data_ptr(), p.s2.data_ptr(), p.b2.data_ptr(),
                                                  x.data_ptr(), D, out.data_ptr(), D, M, I, D, lp, T, sp), "gemm2")
        elif li + 1 < n_li:
            _lib.check(L.gsn_gemm2_residual_stats_bf16(dp, p.w2.data_ptr(), p.b2.data_ptr(), x.data_ptr(), D,
                                                       out.data_ptr(), D, M, I, D, lp, T, stats_buf.data_ptr(), sp),
                       "gemm2")
        else:
            _lib.check(L.gsn_gemm2_residual_bf16(dp, p.w2.data_ptr(), p.b2.data_ptr(), x.data_ptr(), D,
                                                 out.data_ptr(), D, M, I, D, lp, T, sp), "gemm2")
        if record:
            ev[3].record(stream)
            layer_events.append((ev, c, has_ln))

    def ff_kernels(x, out, c, p, lens, record):
        """The three launches of gsn_ff_half_bf16: LayerNorm, up_proj + SiLU, down_proj + half-step residual."""
        M, T, F = c.padded_frames, c.T, p.d_ff
        tp = ws.data_ptr()                                   # LayerNorm output [M, D]
        hp = ws.data_ptr() + ((M * D * 2 + 255) // 256) * 256   # SiLU output [M, F]
        lp = lens.data_ptr()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if record else None
        if record:
            ev[0].record(stream)
        _lib.check(L.gsn_layernorm_bf16(x.data_ptr(), D, p.ln_w.data_ptr(), p.ln_b.data_ptr(), tp, D, M, D,
                                        p.ln_eps, lp, T, sp), "layernorm")
        if record:
            ev[1].record(stream)
        _lib.check(L.gsn_gemm_silu_bf16(tp, p.w_up.data_ptr(), p.b_up.data_ptr(), hp, M, D, F, lp, T, sp), "ff up")
        if record:
            ev[2].record(stream)
        _lib.check(L.gsn_gemm_residual_scaled_bf16(hp, p.w_down.data_ptr(), p.b_down.data_ptr(), x.data_ptr(), D,
                                                   out.data_ptr(), D, M, F, D, 0.5, lp, T, sp), "ff down")
        if record:
            ev[3].record(stream)
            layer_events.append((ev, c))

    def attn_kernels(x, out, c, p, lens, record):
        """The four launches of gsn_attention_block_bf16: LayerNorm (valid frames), the q|k|v GEMM (tiles holding
        valid frames), the attention, to_out + residual."""
        M, T = c.padded_frames, c.T
        inner = HEADS * DIM_HEAD
        tp = ws.data_ptr()                                          # LayerNorm output [M, D]
        qp = tp + ((M * D * 2 + 255) // 256) * 256                  # q | k | v [M, 3 inner]
        cp = qp + ((M * 3 * inner * 2 + 255) // 256) * 256          # context [M, inner]
        lp = lens.data_ptr()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if record else None
        if record:
            ev[0].record(stream)
        _lib.check(L.gsn_layernorm_bf16(x.data_ptr(), D, p.ln_w.data_ptr(), p.ln_b.data_ptr(), tp, D, M, D,
                                        p.ln_eps, lp, T, sp), "layernorm")
        if record:
            ev[1].record(stream)
        _lib.check(L.gsn_gemm_linear_bf16(tp, p.w_qkv.data_ptr(), p.b_qkv.data_ptr(), qp, 3 * inner, M, D, 3 * inner,
                                          lp, T, sp), "qkv")
        if record:
            ev[2].record(stream)
        _lib.check(L.gsn_attention_core_bf16(qp, 3 * inner, p.rel.data_ptr(), p.rel.shape[0], cp, inner, lp, c.B, T,
                                             HEADS, DIM_HEAD, CONTEXT, p.max_pos, DIM_HEAD ** -0.5, sp), "attention")
        if record:
            ev[3].record(stream)
        _lib.check(L.gsn_gemm2_residual_bf16(cp, p.w_out.data_ptr(), p.b_out.data_ptr(), x.data_ptr(), D,
                                             out.data_ptr(), D, M, inner, D, lp, T, sp), "to_out")
        if record:
            ev[4].record(stream)
            layer_events.append((ev, c))

    kev = []       # block / encoder: (kernel name, start event, end event, chunk) of every recorded launch

    def timed(name, c, record, fn):
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            kev.append((name, e0, e1, c))
        else:
            fn()

    def block_kernels(x, out, tmp, c, p, lens, record):
        """One Conformer block, the launches run_conformer_block makes: FF/2 (3), attention (4), conv module with
        the LayerNorm folded (3), FF/2 (3), post LayerNorm over every frame (1).  x -> tmp -> out -> tmp -> out."""
        M, T = c.padded_frames, c.T
        lp = lens.data_ptr()
        inner = HEADS * DIM_HEAD

        def ff(tag, src, dst, q):
            tp = ws.data_ptr()
            hp = ws.data_ptr() + ((M * D * 2 + 255) // 256) * 256
            timed(tag + ".layernorm", c, record, lambda: _lib.check(L.gsn_layernorm_bf16(
                src.data_ptr(), D, q.ln_w.data_ptr(), q.ln_b.data_ptr(), tp, D, M, D, q.ln_eps, lp, T, sp), "ln"))
            timed(tag + ".up_silu", c, record, lambda: _lib.check(L.gsn_gemm_silu_bf16(
                tp, q.w_up.data_ptr(), q.b_up.data_ptr(), hp, M, D, q.d_ff, lp, T, sp), "ff up"))
            timed(tag + ".down_residual", c, record, lambda: _lib.check(L.gsn_gemm_residual_scaled_bf16(
                hp, q.w_down.data_ptr(), q.b_down.data_ptr(), src.data_ptr(), D, dst.data_ptr(), D, M, q.d_ff, D, 0.5,
                lp, T, sp), "ff down"))

        ff("ff1", x, tmp, p.ff1)
        a = p.attn
        tp = ws.data_ptr()
        qp = tp + ((M * D * 2 + 255) // 256) * 256
        cp = qp + ((M * 3 * inner * 2 + 255) // 256) * 256
        timed("attn.layernorm", c, record, lambda: _lib.check(L.gsn_layernorm_bf16(
            tmp.data_ptr(), D, a.ln_w.data_ptr(), a.ln_b.data_ptr(), tp, D, M, D, a.ln_eps, lp, T, sp), "ln"))
        timed("attn.qkv", c, record, lambda: _lib.check(L.gsn_gemm_linear_bf16(
            tp, a.w_qkv.data_ptr(), a.b_qkv.data_ptr(), qp, 3 * inner, M, D, 3 * inner, lp, T, sp), "qkv"))
        timed("attn.attention", c, record, lambda: _lib.check(L.gsn_attention_core_bf16(
            qp, 3 * inner, a.rel.data_ptr(), a.rel.shape[0], cp, inner, lp, c.B, T, HEADS, DIM_HEAD, CONTEXT,
            a.max_pos, DIM_HEAD ** -0.5, sp), "attention"))
        timed("attn.out_proj", c, record, lambda: _lib.check(L.gsn_gemm2_residual_bf16(
            cp, a.w_out.data_ptr(), a.b_out.data_ptr(), tmp.data_ptr(), D, out.data_ptr(), D, M, inner, D, lp, T,
            sp), "to_out"))
        v = p.conv
        dp = ws.data_ptr()
        sp_ = ws.data_ptr() + t_off
        timed("conv.ln_stats", c, record, lambda: _lib.check(L.gsn_layernorm_stats_bf16(
            out.data_ptr(), D, sp_, M, D, v.ln_eps, lp, T, sp), "ln_stats"))
        timed("conv.gemm1_glu_dw", c, record, lambda: _lib.check(L.gsn_gemm1_lnfold_glu_dwconv_bf16(
            out.data_ptr(), v.w1g_glu.data_ptr(), v.b1g_glu.data_ptr(), v.c1_glu.data_ptr(), sp_, v.dw_w.data_ptr(),
            v.dw_b.data_ptr(), dp, c.B, T, D, 2 * I, lp, sp), "gemm1_dw"))
        timed("conv.gemm2_residual", c, record, lambda: _lib.check(L.gsn_gemm2_residual_bf16(
            dp, v.w2.data_ptr(), v.b2.data_ptr(), out.data_ptr(), D, tmp.data_ptr(), D, M, I, D, lp, T, sp),
            "gemm2"))
        ff("ff2", tmp, out, p.ff2)
        timed("post_ln", c, record, lambda: _lib.check(L.gsn_layernorm_bf16(
            out.data_ptr(), D, p.post_ln_w.data_ptr(), p.post_ln_b.data_ptr(), out.data_ptr(), D, M, D, p.post_ln_eps,
            None, T, sp), "post ln"))

    def selfcond_kernels(x, out, c, lens, record):
        """gsn_ctc_selfcond_bf16 (three launches: the 1024->348 (padded 512) linear GEMM, the softmax, the 348
        (padded 384) -> 1024 GEMM + residual), timed as one."""
        nb = int(L.gsn_ctc_selfcond_workspace_bytes(c.B, c.T, hsc.n_cls))
        timed("ctc.selfcond", c, record, lambda: _lib.check(L.gsn_ctc_selfcond_bf16(
            x.data_ptr(), hsc.w_out.data_ptr(), hsc.b_out.data_ptr(), hsc.n_cls, hsc.w_mid.data_ptr(),
            hsc.b_mid.data_ptr(), lens.data_ptr(), out.data_ptr(), blank_buf.data_ptr(), c.B, c.T, D,
            sc_ws.data_ptr(), nb, sp), "selfcond"))

    def decode_kernels(h, c, lens, record):
        """gsn_bpe_pool_bf16 and gsn_bpe_head_ctc_bf16: pooling, the argmax GEMM (keys zeroed first), collapse."""
        from granite_conv_b200.ops import pooled_frames
        T = c.T
        Pp = pooled_frames(T)
        nb = int(L.gsn_bpe_head_workspace_bytes(c.B, Pp))
        timed("ctc.pool", c, record, lambda: _lib.check(L.gsn_bpe_pool_bf16(
            h.data_ptr(), blank_buf.data_ptr(), lens.data_ptr(), pooled_buf.data_ptr(), plen_buf.data_ptr(), c.B, T,
            D, Pp, 4, sp), "pool"))
        timed("ctc.head_argmax_collapse", c, record, lambda: _lib.check(L.gsn_bpe_head_ctc_bf16(
            pooled_buf.data_ptr(), plen_buf.data_ptr(), hbpe.w.data_ptr(), hbpe.b.data_ptr(), hbpe.w.shape[0],
            hbpe.blank_id, ids_buf.data_ptr(), tok_buf.data_ptr(), cnt_buf.data_ptr(), c.B, Pp, D, key_ws.data_ptr(),
            nb, sp), "head"))

    dw_events = []

    def step(record=False):
        n = 0
        for ci, c in enumerate(chunks):
            if workload in DW_WORKLOADS:
                x, y = xs[ci], ys[ci]
                if record:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e1 = torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                if workload == "dw":
                    _lib.check(L.gsn_dwconv_silu_bf16(x.data_ptr(), dw_w.data_ptr(), dw_b.data_ptr(), y.data_ptr(),
                                                      c.B, I, c.T, 15, c.T * I, 1, I, c.T * I, 1, I, 0, sp), "dwconv")
                else:
                    entry = L.gsn_dwconv_silu_glu_bf16 if workload == "dw_cf_glu" else L.gsn_dwconv_silu_bf16
                    _lib.check(entry(x.data_ptr(), dw_w.data_ptr(), dw_b.data_ptr(), y.data_ptr(), c.B, I, c.T, 15,
                                     *x.stride(), *y.stride(), 0, sp), "dwconv")
                if record:
                    e1.record(stream)
                    dw_events.append((e0, e1, c.padded_frames))
                n += 1
                continue
            src = xs[ci]
            if workload == "encoder":
                x0 = xs[ci]
                timed("input_linear", c, record, lambda: _lib.check(L.gsn_gemm_linear_bf16(
                    feats[ci].data_ptr(), w_in.data_ptr(), b_in.data_ptr(), x0.data_ptr(), D, c.padded_frames,
                    synth.INPUT_DIM, D, None, 0, sp), "input_linear"))
                n += 1
            for li, p in enumerate(layers):
                dst = act[ci] if li % 2 == 0 else act2[ci]
                if workload == "ff":
                    ff_kernels(src, dst, c, p, lens_dev[ci], record)
                    n += 3
                elif workload == "attn":
                    attn_kernels(src, dst, c, p, lens_dev[ci], record)
                    n += 4
                elif workload in ("block", "encoder"):
                    dst = act[ci]
                    block_kernels(src, dst, act2[ci], c, p, lens_dev[ci], record)
                    n += 14
                    if heads is not None and li + 1 == len(layers) // 2:
                        selfcond_kernels(dst, act2[ci], c, lens_dev[ci], record)
                        dst = act2[ci]
                        n += 3
                else:
                    layer_kernels(src, dst, c, p, lens_dev[ci], record, li, len(layers))
                    n += 4 if w8a8 else 3
                src = dst
            if workload == "ctc":
                selfcond_kernels(xs[ci], act[ci], c, lens_dev[ci], record)
                src = act[ci]
                n += 3
            if heads is not None:
                decode_kernels(src, c, lens_dev[ci], record)
                n += 3          # pool, argmax GEMM, collapse (+ the keys' memset, a driver kernel, not counted)
        return n

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step()
    barrier()
    status = _lib.device_status(sp)
    if status:
        raise RuntimeError(f"kernel status word {status:#x} after warm-up")

    launches = 0
    with ClockSampler(dev.index) as clocks:
        barrier()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for _ in range(args.steps):
            launches += step(record=True)
        t_end.record(stream)
        barrier()
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        tot = torch.tensor([valid_frames, padded_frames], device=dev, dtype=torch.float64)
        dist.all_reduce(tot)
        valid_all, padded_all = float(tot[0].item()), float(tot[1].item())
    else:
        valid_all, padded_all = float(valid_frames), float(padded_frames)
    ms_per_step = ms / args.steps
    value = valid_all * args.steps / (ms / 1e3)

    peaks = _peaks()
    if workload in DW_WORKLOADS:
        dur = sum(a.elapsed_time(b) for a, b, _ in dw_events) / len(dw_events)
        frames = sum(m for _, _, m in dw_events) / len(dw_events)
        bpf = DW_GLU_BYTES_PER_FRAME if workload == "dw_cf_glu" else DW_BYTES_PER_FRAME
        achieved = frames * bpf / (dur / 1e3) / 1e9
        roof = {"kernel": "dwconv_cl_kernel" if workload == "dw" else
                          "dwconv_cf_mma_kernel<GLU>" if workload == "dw_cf_glu" else "dwconv_cf_mma_kernel",
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                "per_launch_ms": dur, "algorithmic_bytes_per_frame": bpf,
                "peak_source": f"hbm_gbs of {peaks['source']}"}
        if workload in ("dw_cf", "dw_cf_glu"):
            try:                              # a comparison, never a reason to lose the bench line
                roof["gpu_comparator"] = _dw_torch_eager(xs[0], ys[0], dw_w, dw_b, workload == "dw_cf_glu", stream,
                                                         dur, frames * bpf)
            except Exception as exc:  # noqa: BLE001
                roof["gpu_comparator"] = {"error": repr(exc)[:300]}
    elif w8a8:
        dur = sum(a.elapsed_time(b) for a, b, _ in w8_events) / len(w8_events)
        rows = sum(sum(-(-int(L_) // 128) * 128 for L_ in c.lengths) for _, _, c in w8_events) / len(w8_events)
        i8 = _int8_peak_tops(dev)
        peak = i8["int8_tops_sustained"]
        achieved = rows * (GEMM1_FLOP_PER_FRAME + GEMM2_FLOP_PER_FRAME) / (dur / 1e3) / 1e12
        roof = {"kernel": "whole W8A8 module call (LayerNorm + row quantisation, kind::i8 up_conv + GLU + depthwise + "
                          "SiLU, row quantisation, kind::i8 down_conv + residual), timed as one unit: a lower bound "
                          "for the GEMMs",
                "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s", "frac": achieved / peak,
                "traffic": None, "per_launch_ms": dur,
                "algorithmic_ops_per_frame": GEMM1_FLOP_PER_FRAME + GEMM2_FLOP_PER_FRAME,
                "frames_counted": "rows of the 128-row tiles holding valid frames",
                "peak_source": "int8 dense, sustained, measured in this run: " + i8["how"],
                "int8_peak": i8, "frac_of_burst": achieved / i8["int8_tops"]}
    elif workload == "ff":
        kernels = _ff_breakdown(layer_events, peaks)
        g1 = kernels["ff_up_silu"]
        roof = {"kernel": "gemm_kernel<SILU> (up_proj 1024->4096 + SiLU)", "bound": "tensor",
                "achieved": g1["achieved"], "peak": g1["peak"], "unit": "TFLOP/s", "frac": g1["frac"],
                "traffic": None, "per_launch_ms": g1["ms_per_launch"], "algorithmic_flop_per_frame": FF_FLOP_PER_FRAME,
                "frames_counted": "rows of the 128-row tiles holding valid frames",
                "peak_source": f"bf16_tflops_sustained of {peaks['source']}", "kernels": kernels}
    elif workload in ("block", "encoder", "ctc"):
        kernels = _named_breakdown(kev, peaks)
        top = max(kernels, key=lambda n: kernels[n]["share"])
        k = kernels[top]
        roof = {"kernel": top, "bound": "hbm" if k["unit"] == "GB/s" else "tensor", "achieved": k["achieved"],
                "peak": k["peak"], "unit": k["unit"], "frac": k["frac"], "traffic": None,
                "per_launch_ms": k["ms_per_launch"],
                "peak_source": f"bf16_tflops_sustained / hbm_gbs of {peaks['source']}", "kernels": kernels}
    elif workload == "attn":
        kernels = _attn_breakdown(layer_events, peaks)
        top = max(kernels, key=lambda n: kernels[n]["share"])
        k = kernels[top]
        roof = {"kernel": top, "bound": "hbm" if k["unit"] == "GB/s" else "tensor", "achieved": k["achieved"],
                "peak": k["peak"], "unit": k["unit"], "frac": k["frac"], "traffic": None,
                "per_launch_ms": k["ms_per_launch"],
                "work": "q|k|v and to_out GEMMs: 6.291 / 2.097 MFLOP per row of the 128-row tiles holding valid "
                        "frames; attention: 6144 FLOP per (valid query, valid key of its 200-frame block) "
                        "(q.k, q.rel[i-j], p.v over 8 heads x 128); LayerNorm: 4 KB per valid frame",
                "peak_source": f"bf16_tflops_sustained / hbm_gbs of {peaks['source']}", "kernels": kernels}
    else:
        kernels = _kernel_breakdown(layer_events, peaks, widen_events, ln_name="layernorm" if int8 else "ln_stats")
        g1 = kernels["gemm1_glu_dw"]
        traffic = None if GEMM1DW_DRAM_BYTES_PER_ROW is None else g1["rows_per_launch"] * GEMM1DW_DRAM_BYTES_PER_ROW
        roof = {"kernel": "gemm_glu_dw_kernel (up_conv 1024->4096 + GLU + depthwise k15 + SiLU)", "bound": "tensor",
                "achieved": g1["achieved"], "peak": g1["peak"], "unit": "TFLOP/s", "frac": g1["frac"],
                "traffic": traffic,
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per computed row from one capture "
                                  "of the module workload's B=48, T=1536 chunk (a constant of this build, not "
                                  "measured in this run), scaled to the average launch",
                "algorithmic_bytes": g1["rows_per_launch"] * (2 * D + 2 * I), "per_launch_ms": g1["ms_per_launch"],
                "algorithmic_flop_per_frame": GEMM1_FLOP_PER_FRAME,
                "frames_counted": "rows of the 128-row tiles holding valid frames (tiles of pure padding are "
                                  "skipped by the kernel)",
                "peak_source": f"bf16_tflops_sustained of {peaks['source']}", "kernels": kernels}
        if workload == "module":
            try:                              # a comparison, never a reason to lose the bench line
                roof["gpu_comparator"] = _module_torch_eager(xs[0], act[0], chunks[0], stream, ms_per_step)
            except Exception as exc:  # noqa: BLE001
                roof["gpu_comparator"] = {"error": repr(exc)[:300]}

    # ---- end to end through the public op with pinned host buffers
    e2e = None
    if workload in ("dw_cf", "dw_cf_glu") and not args.no_e2e:
        e2e = _e2e_dw(args, chunks, xs[0].shape, workload == "dw_cf_glu", dw_w, dw_b, dev, stream, world)
    elif workload not in ("dw", "module_w8a8") and not args.no_e2e:
        e2e = _e2e(args, chunks, layers, int8, dev, stream, world, barrier, ff=workload == "ff",
                   attn=workload == "attn", block=workload in ("block", "encoder"), heads=heads)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r, cores, desc = cpu_baseline_rate(workload, args.cpu_seconds)
        cpu = {"value": r, "unit": "frames/s", "cores": cores, "kind": "port", "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "frames/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": _scaling(args),
            "vs_baseline": None, "dtype": "int8 x int8 (s32 accumulate), bf16 in/out" if w8a8 else ("bf16" if not int8 else "bf16 x int8-weight"), "data": "synthetic",
            "config": dict(_config(args, world), padded_frames_per_s=padded_all * args.steps / (ms / 1e3)),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(),
            **({"process_group": pg_info} if pg_info else {}),
            "gpu_launches": launches,
        }
    if world > 1:
        dist.destroy_process_group()
    return line if rank == 0 else None


# The other configurations of the conv-module path, measured after the headline on one GPU so that every bench run
# carries them: the depthwise kernel alone (channels-last rows as the standalone op's layout, and the reference
# call site's channels-first layout, plain and GLU), one bf16 module, the int8-weight module and the W8A8 module.
SECONDARY_WORKLOADS = ("dw", "dw_cf", "dw_cf_glu", "module", "module_i8", "module_w8a8")


def secondary_configs(args) -> dict:
    out = {}
    for w in SECONDARY_WORKLOADS:
        a = argparse.Namespace(**vars(args))
        a.workload, a.steps, a.warmup, a.no_cpu, a.no_e2e = w, 20, 5, True, True
        ln = run_ours(a)
        r = ln["roofline"]
        out[w] = {"config": ln["config"]["workload"], "value": ln["value"], "unit": ln["unit"], "dtype": ln["dtype"],
                  "kernel": r["kernel"], "achieved": r["achieved"], "peak": r["peak"], "roofline_unit": r["unit"],
                  "frac": r["frac"], "bound": r["bound"], "per_launch_us": r["per_launch_ms"] * 1e3,
                  "peak_source": r.get("peak_source"), "clocks": ln["clocks"], "steps": 20, "warmup": 5,
                  "gpu_launches": ln["gpu_launches"]}
    return out


def _dw_torch_eager(x, y_ours, dw_w, dw_b, glu, stream, our_ms, algo_bytes):
    """The comparison the reference's own depthwise microbenchmark makes (script/cuda_kernels/conv1d.py:118-145),
    on this GPU: torch's eager ops for the same call -- [F.glu(x, dim=1)], F.conv1d(groups=C, padding=7) (cuDNN) and
    F.silu, bf16 -- timed with CUDA events over 20 launches after 5 warm-up calls, and their largest difference from
    this package's output."""
    import torch
    import torch.nn.functional as F
    C = dw_w.shape[0]
    w3 = dw_w.view(C, 1, -1)

    def eager():
        h = F.glu(x, dim=1) if glu else x
        return F.silu(F.conv1d(h, w3, dw_b, padding=w3.shape[-1] // 2, groups=C))

    for _ in range(5):
        ref = eager()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(20):
        ref = eager()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    d = (ref.float() - y_ours.float()).abs()
    return {"what": "torch eager on this GPU: " + ("F.glu, " if glu else "") +
                    "depthwise F.conv1d (cuDNN) and F.silu in bf16, the reference microbenchmark's comparison",
            "per_launch_us": ms * 1e3, "achieved_gbs": algo_bytes / (ms / 1e3) / 1e9,
            "this_kernel_speedup": ms / our_ms,
            "max_abs_diff": float(d.max()), "max_rel_to_gate": float((d / (2e-2 * ref.float().abs().clamp(min=1.0))).max())}


def _module_torch_eager(x, y_ours, c, stream, our_ms):
    """The reference module's own eager path on this GPU (ConformerConvModule.forward, conformer.py:175-189, after
    the BatchNorm fold, plus the residual add of :207), bf16, on the same chunk and weights: F.layer_norm, the 1x1
    up_conv as F.conv1d, F.glu, the depthwise F.conv1d (cuDNN), F.silu, the 1x1 down_conv, the residual.  Timed
    with CUDA events over 20 calls after 3 warm-up calls.  The reference module has no length mask, so the last 7
    valid frames of each utterance see the padding frames through the depthwise window there; the largest
    difference from this package's output is taken over the frames whose window lies inside the utterance."""
    import torch
    import torch.nn.functional as F
    q = synth.make_params(1005)
    dev = x.device
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
    ln_w, ln_b = bf(q.norm_weight), bf(q.norm_bias)
    w1, b1 = bf(q.up_weight)[:, :, None], bf(q.up_bias)
    w2, b2 = bf(q.down_weight)[:, :, None], bf(q.down_bias)
    scale = bf(q.bn_weight).float() * torch.rsqrt(bf(q.bn_var).float() + float(q.bn_eps))
    dw_w = (bf(q.dw_weight).float() * scale[:, None]).to(torch.bfloat16)[:, None, :]
    dw_b = (bf(q.bn_bias).float() - bf(q.bn_mean).float() * scale).to(torch.bfloat16)
    inner = dw_w.shape[0]

    def eager():
        h = F.layer_norm(x, (x.shape[-1],), ln_w, ln_b, float(q.ln_eps)).transpose(1, 2)
        h = F.glu(F.conv1d(h, w1, b1), dim=1)
        h = F.silu(F.conv1d(h, dw_w, dw_b, padding=dw_w.shape[-1] // 2, groups=inner))
        return F.conv1d(h, w2, b2).transpose(1, 2) + x

    for _ in range(3):
        ref = eager()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(20):
        ref = eager()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 20
    worst = 0.0
    for b, L in enumerate(c.lengths):
        n = max(int(L) - 7, 0)
        if n == 0:
            continue
        d = (ref[b, :n].float() - y_ours[b, :n].float()).abs()
        worst = max(worst, float((d / (2e-2 * ref[b, :n].float().abs().clamp(min=1.0))).max()))
    return {"what": "the reference module's eager path on this GPU (F.layer_norm, 1x1 F.conv1d, F.glu, depthwise "
                    "F.conv1d, F.silu, 1x1 F.conv1d, residual) in bf16 on the same chunk and weights",
            "per_call_us": ms * 1e3, "valid_frames_per_s": c.valid_frames / (ms / 1e3),
            "this_module_speedup": ms / our_ms, "max_rel_to_gate_inner_frames": worst}


def _tile_rows(c, tile=128):
    """Rows of the 128-row tiles that hold at least one valid frame (T is on the 128 grid)."""
    return int(sum(((int(L) + tile - 1) // tile) * tile for L in c.lengths))


def _ff_breakdown(layer_events, peaks):
    """Per-kernel launch time and rate of the feed-forward half: LayerNorm (2 x 2 KB per valid frame), the two
    GEMMs (8.389 MFLOP per computed row each)."""
    names = ("layernorm", "ff_up_silu", "ff_down_residual")
    tot = {n: 0.0 for n in names}
    work = {n: 0.0 for n in names}
    for ev, c in layer_events:
        for k, n in enumerate(names):
            tot[n] += ev[k].elapsed_time(ev[k + 1])
        rows = _tile_rows(c)
        work["layernorm"] += c.valid_frames * 2 * D * 2
        work["ff_up_silu"] += rows * FF_FLOP_PER_FRAME
        work["ff_down_residual"] += rows * FF_FLOP_PER_FRAME
    all_ms = sum(tot.values())
    out = {}
    for n in names:
        tensor = n.startswith("ff_")
        ach = work[n] / (tot[n] / 1e3) / (1e12 if tensor else 1e9)
        pk = peaks["bf16_tflops_sustained"] if tensor else peaks["hbm_gbs"]
        out[n] = {"ms_per_launch": tot[n] / len(layer_events), "share": tot[n] / all_ms, "achieved": ach,
                  "unit": "TFLOP/s" if tensor else "GB/s", "peak": pk, "frac": ach / pk}
    return out


def _attn_query_keys(c):
    """Sum over valid query frames of the valid keys in their 200-frame block."""
    n = 0
    for L in c.lengths:
        L = int(L)
        for m0 in range(0, L, CONTEXT):
            k = min(CONTEXT, L - m0)
            n += k * k
    return n


# work of each named launch of the block / encoder workloads: (kind, per-chunk work function)
def _named_work(name, c):
    rows = _tile_rows(c)
    kind = name.split(".")[-1]
    if kind == "layernorm":
        return "hbm", c.valid_frames * 2 * D * 2
    if name == "post_ln":
        return "hbm", c.padded_frames * 2 * D * 2
    if kind == "ln_stats":
        return "hbm", c.valid_frames * (D * 2 + 8)
    if kind in ("up_silu", "down_residual", "gemm1_glu_dw"):
        return "tensor", rows * FF_FLOP_PER_FRAME
    if kind == "gemm2_residual":
        return "tensor", rows * GEMM2_FLOP_PER_FRAME
    if kind == "qkv":
        return "tensor", rows * QKV_FLOP_PER_FRAME
    if kind == "out_proj":
        return "tensor", rows * OUT_FLOP_PER_FRAME
    if kind == "attention":
        return "tensor", _attn_query_keys(c) * ATTN_FLOP_PER_QUERY_KEY
    if name == "input_linear":
        return "tensor", c.padded_frames * 2 * synth.INPUT_DIM * D
    if kind == "selfcond":
        return "tensor", rows * (2 * D * 512 + 2 * 384 * D)
    if kind == "pool":
        return "hbm", c.valid_frames * (D * 2 + 4) + sum(-(-int(L) // 4) for L in c.lengths) * D * 2
    if kind == "head_argmax_collapse":
        prow = sum(-(-(-(-int(L) // 4)) // 128) * 128 for L in c.lengths)
        return "tensor", prow * 2 * D * synth.BPE_VOCAB
    raise KeyError(name)


def _named_breakdown(kev, peaks):
    """Per named launch: average duration, share of the recorded time, achieved rate against the measured peak."""
    tot, work, cnt, kinds = {}, {}, {}, {}
    for name, e0, e1, c in kev:
        kind, w = _named_work(name, c)
        tot[name] = tot.get(name, 0.0) + e0.elapsed_time(e1)
        work[name] = work.get(name, 0.0) + w
        cnt[name] = cnt.get(name, 0) + 1
        kinds[name] = kind
    all_ms = sum(tot.values())
    out = {}
    for n in tot:
        tensor = kinds[n] == "tensor"
        ach = work[n] / (tot[n] / 1e3) / (1e12 if tensor else 1e9)
        pk = peaks["bf16_tflops_sustained"] if tensor else peaks["hbm_gbs"]
        out[n] = {"ms_per_launch": tot[n] / cnt[n], "share": tot[n] / all_ms, "achieved": ach,
                  "unit": "TFLOP/s" if tensor else "GB/s", "peak": pk, "frac": ach / pk}
    return out


def _attn_breakdown(layer_events, peaks):
    """Per-kernel launch time and rate of the attention step: LayerNorm over the valid frames (2 x 2 KB), the q|k|v and
    to_out GEMMs (rows of the 128-row tiles holding valid frames), the attention (ATTN_FLOP_PER_QUERY_KEY per valid
    query-key pair of a block)."""
    names = ("layernorm", "qkv_proj", "attention", "out_proj")
    tot = {n: 0.0 for n in names}
    work = {n: 0.0 for n in names}
    for ev, c in layer_events:
        for k, n in enumerate(names):
            tot[n] += ev[k].elapsed_time(ev[k + 1])
        rows = _tile_rows(c)
        work["layernorm"] += c.valid_frames * 2 * D * 2
        work["qkv_proj"] += rows * QKV_FLOP_PER_FRAME
        work["attention"] += _attn_query_keys(c) * ATTN_FLOP_PER_QUERY_KEY
        work["out_proj"] += rows * OUT_FLOP_PER_FRAME
    all_ms = sum(tot.values())
    out = {}
    for n in names:
        tensor = n != "layernorm"
        ach = work[n] / (tot[n] / 1e3) / (1e12 if tensor else 1e9)
        pk = peaks["bf16_tflops_sustained"] if tensor else peaks["hbm_gbs"]
        out[n] = {"ms_per_launch": tot[n] / len(layer_events), "share": tot[n] / all_ms, "achieved": ach,
                  "unit": "TFLOP/s" if tensor else "GB/s", "peak": pk, "frac": ach / pk}
    return out


def _kernel_breakdown(layer_events, peaks, widen_events=(), ln_name="layernorm"):
    """Average launch time, share of the recorded kernel time and achieved rate of each kernel.
    Work per launch: LayerNorm reads and writes the valid frames (2 x 2 KB); the GEMMs compute the rows of the
    128-row tiles that hold valid frames (the up_conv kernel also runs GLU and the depthwise conv on them, counted
    as its GEMM FLOPs only); the LayerNorm statistics read 2 KB and write 8 B per valid frame; the int8 weight
    widening reads 1 byte and writes 2 per weight."""
    names = (ln_name, "gemm1_glu_dw", "gemm2_residual")
    tot = {n: 0.0 for n in names}
    work = {n: 0.0 for n in names}
    if widen_events:
        names = ("widen_i8",) + names
        tot["widen_i8"] = sum(a.elapsed_time(b) for a, b in widen_events) * len(layer_events) / len(widen_events)
        work["widen_i8"] = 3.0 * (2 * I * D + D * I) * len(layer_events)
    ln_launches = 0
    for ev, c, has_ln in layer_events:
        for k, n in enumerate(names[-3:]):
            if k > 0 or has_ln:
                tot[n] += ev[k].elapsed_time(ev[k + 1])
        valid = c.valid_frames
        rows = _tile_rows(c)
        if has_ln:
            ln_launches += 1
            work[ln_name] += valid * (2 * D * 2 if ln_name == "layernorm" else D * 2 + 8)
        work["gemm1_glu_dw"] += rows * GEMM1_FLOP_PER_FRAME
        work["gemm2_residual"] += rows * GEMM2_FLOP_PER_FRAME
    all_ms = sum(tot.values())
    out = {}
    for n in names:
        tensor = n.startswith("gemm")
        ach = work[n] / (tot[n] / 1e3) / (1e12 if tensor else 1e9)
        pk = peaks["bf16_tflops_sustained"] if tensor else peaks["hbm_gbs"]
        launches = ln_launches if n == ln_name else len(layer_events)
        out[n] = {"ms_per_launch": tot[n] / max(1, launches), "launches": launches, "share": tot[n] / all_ms,
                  "achieved": ach, "unit": "TFLOP/s" if tensor else "GB/s", "peak": pk, "frac": ach / pk}
    out["gemm1_glu_dw"]["rows_per_launch"] = work["gemm1_glu_dw"] / GEMM1_FLOP_PER_FRAME / len(layer_events)
    return out


def _e2e(args, chunks, layers, int8, dev, stream, world, barrier, ff=False, attn=False, block=False, heads=None):
    """Same work through the public API (ConvModuleStack, the feed-forward / attention / block ops, the encoder)
    with each chunk's input copied from pinned host memory and its output copied back inside the timed region.
    Consecutive steps are pipelined as a streaming server runs them: a chunk's next upload waits only for the
    compute that read its device buffer, so the next step's first uploads overlap this step's last chunks; every
    step still moves all of its inputs and outputs across the host link inside the timed region, which ends when
    the last step's last download has landed."""
    import torch

    from granite_conv_b200 import ConvModuleStack, ops
    if ff:
        def stack(x, lengths):
            return ops.run_feed_forward_half(x, layers[0], lengths)
    elif attn:
        def stack(x, lengths):
            return ops.run_attention_block(x, layers[0], lengths)
    elif block and heads is not None:
        from granite_conv_b200 import GraniteCTCEncoder
        wi, bi = synth.make_input_params(1010)
        genc = GraniteCTCEncoder(torch.from_numpy(wi).to(torch.bfloat16).to(dev),
                                 torch.from_numpy(bi).to(torch.bfloat16).float().to(dev), layers, heads[0], heads[1],
                                 selfcond_layer=len(layers) // 2)

        def stack(x, lengths):            # features in, the transcript (collapsed token ids, int32 [B, Pp]) back
            return genc(x, lengths)["tokens"]
    elif block:
        from granite_conv_b200 import ConformerEncoderStack
        stack = ConformerEncoderStack(layers)
    elif heads is not None:
        def stack(x, lengths):
            h, blank = ops.run_ctc_selfcond(x, heads[0], lengths)
            return ops.run_bpe_ctc_decode(h, blank, heads[1], lengths)[1]
    else:
        stack = ConvModuleStack(layers, int8=int8)
    g = torch.Generator().manual_seed(4242)
    din = synth.INPUT_DIM if (block and heads is not None) else D       # the encoder takes the 160-dim features
    hx = [torch.randn((c.B, c.T, din), generator=g).to(torch.bfloat16).pin_memory() for c in chunks]
    hl = [torch.from_numpy(c.lengths).pin_memory() for c in chunks]
    # the output of one call: bf16 [B, T, D] frames, or with the heads int32 [B, Pp] tokens
    out_dtype = torch.bfloat16 if heads is None else torch.int32
    ho = [torch.empty((c.B, c.T, D) if heads is None else (c.B, ops.pooled_frames(c.T)), dtype=out_dtype).pin_memory()
          for c in chunks]
    h2d = sum(x.numel() * 2 + l.numel() * 4 for x, l in zip(hx, hl))
    d2h = sum(o.numel() * o.element_size() for o in ho)

    # copies run on their own streams so chunk i+1's upload and chunk i-1's download overlap chunk i's layers;
    # a chunk's device input is overwritten only after the previous step's compute of that chunk has finished.
    # Chunks alternate between two compute streams (ConvModuleStack.run_chunks' schedule), so each persistent
    # kernel's tail is filled by the other chunk's next kernel.
    copy_in = torch.cuda.Stream(dev)
    copy_out = torch.cuda.Stream(dev)
    comp = [stream, torch.cuda.Stream(dev)]
    xd = [torch.empty((c.B, c.T, din), dtype=torch.bfloat16, device=dev) for c in chunks]
    ld = [torch.empty((c.B,), dtype=torch.int32, device=dev) for c in chunks]
    done = [None] * len(chunks)

    def start():
        begin = torch.cuda.Event()          # the copies start after everything queued before them (e.g. the start
        begin.record(stream)                #   event of the timed region)
        copy_in.wait_event(begin)
        comp[1].wait_event(begin)

    def finish():
        fin = torch.cuda.Event()            # the current stream waits for the last download and the side stream
        fin.record(copy_out)
        stream.wait_event(fin)
        side = torch.cuda.Event()
        side.record(comp[1])
        stream.wait_event(side)

    def step():
        for ci in range(len(chunks)):
            cs = comp[ci % 2]
            with torch.cuda.stream(copy_in):
                if done[ci] is not None:
                    copy_in.wait_event(done[ci])
                xd[ci].copy_(hx[ci], non_blocking=True)
                ld[ci].copy_(hl[ci], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(copy_in)
            cs.wait_event(ready)
            with torch.cuda.stream(cs):
                y = stack(xd[ci], ld[ci])
                done[ci] = torch.cuda.Event()
                done[ci].record(cs)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done[ci])
                ho[ci].copy_(y, non_blocking=True)
                y.record_stream(copy_out)

    start()
    for _ in range(max(1, args.warmup)):
        step()
    finish()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    start()
    for _ in range(args.steps):
        step()
    finish()
    e1.record(stream)
    barrier()
    ms = e0.elapsed_time(e1)
    valid = sum(c.valid_frames for c in chunks) * len(layers)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        v = torch.tensor([float(valid)], device=dev, dtype=torch.float64)
        dist.all_reduce(v)
        valid = float(v.item())
    return {"value": valid * args.steps / (ms / 1e3), "unit": "frames/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms / args.steps,
            "path": ("GraniteCTCEncoder (features in, granite:: ops per step, CTC heads; tokens come back)"
                     if block and heads is not None else
                     "granite::ctc_selfcond + granite::bpe_ctc_decode (tokens come back)" if heads is not None else
                     "ConformerEncoderStack (granite:: ops per step of each block)" if block else
                     "torch.ops.granite." + ("feed_forward_half" if ff else "attention_block" if attn else
                                             "conv_module per layer")) + ", pinned host in/out on two copy streams"}


def _e2e_dw(args, chunks, shape, glu, dw_w, dw_b, dev, stream, world):
    """The depthwise op at the reference's call site end to end: torch.ops.granite.dwconv_silu[_glu] on a (B, C, T)
    tensor copied from pinned host memory, its output copied back, every step inside the timed region."""
    import torch

    from granite_conv_b200 import ops  # noqa: F401  (registers the ops)
    op = torch.ops.granite.dwconv_silu_glu if glu else torch.ops.granite.dwconv_silu
    g = torch.Generator().manual_seed(4243)
    hx = torch.randn(shape, generator=g).to(torch.bfloat16).pin_memory()
    ho = torch.empty((shape[0], I, shape[2]), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    w3 = dw_w[:, None, :]

    def step():
        xd.copy_(hx, non_blocking=True)
        y = op(xd, w3, dw_b)
        ho.copy_(y, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    frames = sum(c.valid_frames for c in chunks)
    return {"value": frames * args.steps / (ms / 1e3), "unit": "frames/s", "h2d_bytes_per_step": hx.numel() * 2,
            "d2h_bytes_per_step": ho.numel() * 2, "ms_per_step": ms / args.steps,
            "path": "torch.ops.granite." + ("dwconv_silu_glu" if glu else "dwconv_silu") +
                    " on (B, C, T) contiguous, pinned host in/out"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["stack", "module", "module_i8", "module_w8a8", "dw", "dw_cf", "dw_cf_glu", "ff",
                                           "attn", "block", "encoder", "ctc"], default="stack")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="stack / encoder over N GPUs: one set of 512 utterances split over the ranks (strong) or "
                         "512 per rank (weak)")
    ap.add_argument("--shard", choices=["utterances", "chunks"], default="utterances",
                    help="strong scaling: deal sorted utterances to ranks, each chunking its share, or deal the "
                         "chunks of one plan")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="stack on one GPU: skip the other configurations measured after the headline")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("note: --warmup raised to 3", file=sys.stderr)
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    line = run_ours(args)
    if line is None:
        return 0
    if args.workload == "stack" and line["n_gpus"] == 1 and not args.no_configs:
        line["other_configs"] = secondary_configs(args)
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

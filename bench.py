"""Benchmark of the MoE expert-FFN path (one JSON line on rank 0).

Workload: a Qwen-Next-style decode MoE layer,
H=2048, 512 routed experts of I=512 + 1 shared expert, MXFP4 blobs, top-10
softmax routing, 64 tokens per step and per GPU, seeded synthetic inputs.
A step is one layer forward through the public API (router -> sort -> expert
GEMVs -> shared expert -> combine).  Each step uses the next of 8 token
batches, so routes change; L2 is flushed (a 256 MB write) before every timed
step.  `value` is whole-job tokens/s from device events (inputs resident);
`e2e` is the same through the public call for a repeated decode shape
(Engine.replay: pinned host input and output, the copies inside the timed
region, the layer replayed from a graph captured on the first call).
With --gpus N > 1 the layer runs expert-parallel (whallm_b200.ep): every rank owns E/N experts and its own
64-token batch, and pairs travel to their experts' ranks and back through
NVLink peer memory (--exchange nccl: NCCL all-to-all), fixed-capacity
exchanges, one CUDA graph per step (weak scaling).  At N = 1 the line also
carries a `prefill` section: the config-2
layer (16,384 tokens, Zipf(1.1) routing) through the grouped-GEMM path.
At N = 1 it also carries `decode_batches` (the same layer at batch 1 and 8)
and `long_calls`: one config-3 layer (DeepSeek-style
FP8, 8192 tokens) and one layer of config 4 (256 decode + 4096 prefill
tokens, 384 MXFP4 experts of H = 7168, I = 2048), both on the grouped GEMM.
`--impl reference` times the CPU oracle (the restatement of the reference's
arithmetic) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s (prefill, decode) at 1/2/4/8 B200; % of HBM / FP4-TC roofline"
H, I, E, K = 2048, 512, 512, 10
BLOB = 1_671_168  # bytes of one expert blob (gate_up + scales + down + scales)
GATE_UP_BYTES = 2 * I * H // 2 + 2 * I * H // 32
# dram bytes (read + write) of one gate/up decode launch at this workload, from an ncu capture
# (profiles/decode_bs_config1_b64.txt: block-scaled kernel; profiles/decode_mma_config1_b64.txt: --decode mma)
NCU_GATE_UP_TRAFFIC = {"bs": 436.316416e6 + 6.585344e6, "mma": 412.166656e6 + 3.397376e6, "fused": None}
DECODE_KERNEL = {"bs": "bs_decode_kernel<0> (gate/up + SwiGLU; block-scaled tcgen05, kind::mxf8f6f4)",
                 "mma": "decode_mma_kernel<0> (gate/up + SwiGLU; register-direct mma.sync)",
                 "fused": "bs_decode_fused_kernel (gate/up + SwiGLU and down in one launch; block-scaled tcgen05)"}
DECODE_PROFILE = {"bs": "profiles/decode_bs_config1_b64.txt", "mma": "profiles/decode_mma_config1_b64.txt",
                  "fused": None}
DECODE_FLAGS = {"bs": 0, "mma": "FLAG_MMA_DECODE", "fused": "FLAG_FUSED_DECODE"}
DOWN_BYTES = H * I // 2 + H * I // 32


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Clocks:
    """SM clocks and clock-event reasons sampled during the timed region: NVML
    polled every millisecond from a side thread, with one sample as the region
    starts and one as it ends (so even a few-millisecond region has samples);
    nvidia-smi at 200 ms when NVML is not there.  Samples go to a CSV too."""

    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index: int, log_dir: str | None = None):
        self.index = index
        self.proc = None
        self.nvml = None
        self.rows: list[tuple[float, float, int]] = []
        self.path = Path(log_dir or tempfile.gettempdir()) / f"clocks_rank{index}.csv"

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.index).uuid)
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)

    def _sample(self):
        nv, h = self.nvml
        sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        self.rows.append((sm, mx, int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))

    def __enter__(self):
        import threading
        try:
            self.nvml = self._nvml_handle()
            self._sample()
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self.stop = threading.Event()

            def poll():
                while not self.stop.wait(0.001):
                    try:
                        self._sample()
                    except Exception:
                        return
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return self
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.nvml is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self._sample()
            except Exception:
                pass
            try:
                self.path.parent.mkdir(parents=True, exist_ok=True)
                self.path.write_text("".join(f"{a},{b},{c:#x}\n" for a, b, c in self.rows))
            except OSError:
                pass
        elif self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait(timeout=5)
            self.f.close()

    def summary(self) -> dict:
        if self.nvml is not None:
            sm = [r[0] for r in self.rows]
            reasons = sorted({name for name, bit in self.REASONS for r in self.rows if r[2] & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.rows[-1][1] if sm else None,
                    "reasons": reasons, "samples": len(sm), "source": "nvml, 1 ms"}
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], None, set()
        names = [name for name, _ in self.REASONS]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def cpu_sample(layer_np, xb, idx, w, min_seconds: float, tokens: int):
    """Oracle forward on `tokens` tokens, repeated for at least min_seconds; tokens/s."""
    import numpy as np
    sub = np.arange(tokens, dtype=np.int32)
    n, t0 = 0, time.perf_counter()
    while True:
        layer_np.forward(xb, idx, w, tokens=sub)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            return tokens * n / dt


def run_reference(args) -> None:
    """The reference arm: the CPU oracle on the box's host cores."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    import torch
    import oracle
    from oracle import adapter
    from whallm_b200 import synth

    cores = len(os.sched_getaffinity(0))
    oracle.set_threads(cores)  # torchrun sets OMP_NUM_THREADS=1 for every rank
    threads = oracle.max_threads()
    wl = synth.config(1, device="cpu", batch=64)
    layer_np = adapter.from_layer(wl.layer)
    xb = adapter.bits(wl.x)
    logits = oracle.router_logits(xb, adapter.bits(wl.layer.router.weight))
    idx, w = oracle.route(oracle.ROUTER_SOFTMAX, logits, K)
    sample = 8
    sub = np.arange(sample, dtype=np.int32)
    for _ in range(args.warmup):
        layer_np.forward(xb, idx, w, tokens=sub)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        layer_np.forward(xb, idx, w, tokens=sub)
    dt = time.perf_counter() - t0
    tps = sample * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, BASELINE configs[1] shapes)",
        "config": {"workload": "config1 decode layer, 64-token batch (8-token sample per step)", "H": H, "I": I,
                   "E": E, "K": K, "shared_expert": True},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} tokens of a 64-token config-1 batch per step, OpenMP threads {threads} "
                                   f"on {cores} cores"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Long-call sections at N = 1: (config, label, mma kind note).
LONG_CONFIGS = {
    2: "config2 prefill layer, 16384 tokens, Zipf(1.1) expert popularity",
    3: "config3 DeepSeek-style FP8 layer, 8192 tokens, 256 experts (I=2048) + shared, sigmoid group-limited top-8",
    4: "config4 single layer (of the 8-layer stack): 256 decode + 4096 prefill tokens, 384 MXFP4 experts (I=2048)"
       " + shared, top-8",
}


def prefill_section(args, dev, pk, n: int = 2) -> dict:
    """A long call of config n through the public call (grouped-GEMM path)."""
    import torch
    from whallm_b200 import synth
    from whallm_b200.moe import Engine

    wl = synth.config(n, device=dev)
    T, Hn = wl.x.shape
    lay = wl.layer
    En, In, Kn = lay.E, lay.I, wl.K
    eng = Engine(dev.index, max_tokens=T, hidden=Hn, inter=In, experts=En, topk=Kn)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(3):
        flush.zero_()
        eng.forward(lay, wl.x, Kn)
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 10))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        evs[i][0].record()
        eng.forward(lay, wl.x, Kn)
        evs[i][1].record()
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    eng.ctx.profile(True)
    eng.ctx.profile_reset()
    _, (w, idx) = eng.forward(lay, wl.x, Kn, return_routes=True)
    torch.cuda.synchronize()
    prof = eng.ctx.profile_read()
    eng.ctx.profile(False)
    counts = torch.bincount(idx.reshape(-1).long(), minlength=En).cpu()
    rows = T * Kn + T  # routed pairs + shared-expert rows
    gu_flops, dn_flops = 2.0 * rows * Hn * 2 * In, 2.0 * rows * In * Hn
    gu_n, gu_ms = prof.get("gemm_gate_up", (1, float("nan")))
    dn_n, dn_ms = prof.get("gemm_down", (1, float("nan")))
    tf_gu = gu_flops / (gu_ms / gu_n / 1e3) / 1e12
    tf_dn = dn_flops / (dn_ms / dn_n / 1e3) / 1e12
    layer_tf = (gu_flops + dn_flops) / (ms / 1e3) / 1e12
    fp8 = lay.layout == lib_layout_fp8()
    nominal = 4500.0 if fp8 else 9000.0
    bs = eng.ctx.counters().bs_gemm_calls > 0
    # rows the 128-row tiles cover (each expert's group padded to 128; the MMA runs on them all)
    tile_rows = int(((counts + 127) // 128).sum()) * 128 + (T + 127) // 128 * 128
    mma = ("kind::mxf8f6f4.block_scale (E2M1 weights with E8M0 scale factors; activation rows as hi + lo "
           "E4M3 parts, two MMAs per K step)" if bs else "kind::f16 (bf16 operands, exact dequantised weights)")
    out = {
        "workload": LONG_CONFIGS[n], "tokens_per_s": T / (ms / 1e3),
        "ms_per_layer": ms, "layer_tflops": layer_tf,
        "roofline": {"bound": "tensor", "kernel": "gemm_gate_up", "achieved": tf_gu, "unit": "TFLOP/s",
                     "peak_bf16": pk["bf16_tflops"], "frac_bf16": tf_gu / pk["bf16_tflops"],
                     ("peak_fp8_nominal" if fp8 else "peak_fp4_nominal"): nominal,
                     ("frac_fp8_nominal" if fp8 else "frac_fp4_nominal"): tf_gu / nominal,
                     "mma_kind": mma, "peak_source": pk["source"],
                     "down_tflops": tf_dn, "algorithmic_flops_per_launch": gu_flops,
                     "tile_row_utilisation": rows / tile_rows,
                     **({"tensor_pipe_tflops": 2.0 * tf_gu * tile_rows / rows, "peak_mxf8f6f4_nominal": 4500.0,
                         "frac_tensor_pipe_nominal": 2.0 * tf_gu * tile_rows / rows / 4500.0} if bs else {})},
        "kernels": {nm: {"launches": c, "avg_us": 1e3 * t / c} for nm, (c, t) in prof.items()},
        "expert_rows": {"max": int(counts.max()), "median": float(counts.float().median()), "min": int(counts.min())},
        "l2": "flushed before every timed step",
    }
    eng.ctx.close()
    del wl, lay, eng
    torch.cuda.empty_cache()
    return out


def lib_layout_fp8() -> int:
    from whallm_b200 import lib
    return lib.LAYOUT_W13_FP8_B128


# Expert-parallel long-call sections (strong scaling: the tokens and the
# routed experts split evenly over the ranks; router and shared expert on
# every rank).  config 3: one DeepSeek-style FP8 layer, 8192 tokens.  config 4:
# the 8-layer MXFP4 stack, 256 decode + 4096 prefill tokens per step, bf16
# residual adds between layers.
EP_SECTIONS = {
    3: ("ep_config3", "config3 FP8 layer (H=7168, 256 experts of I=2048 + shared, sigmoid group-limited top-8), "
                      "8192 tokens per step split over the GPUs"),
    4: ("config4_stack", "config4 8-layer MXFP4 stack (H=7168, 384 experts of I=2048 + shared, top-8), "
                         "256 decode + 4096 prefill tokens per step split over the GPUs, bf16 residual adds"),
}


def long_ep_section(args, n: int, world: int, rank: int, local: int, pk: dict) -> dict:
    """Config n (3 or 4) over `world` GPUs, expert-parallel over NVLink peer
    memory when world > 1.  Every rank holds the whole model (so it can check
    its expert-parallel result against the one-GPU result bit for bit, and
    rank 0 can time the whole batch on one GPU in the same run); the
    expert-parallel step reads only the rank's shard of the routed experts."""
    import torch
    import torch.distributed as dist

    from whallm_b200 import synth
    from whallm_b200.ep import ExpertParallelMoE
    from whallm_b200.moe import Engine

    dev = torch.device("cuda", local)
    if n == 3:
        layers, T_total = [synth.deepseek_fp8_layer(device=dev, seed=0)], 8192
    else:
        # pre-norm residual blocks, h <- h + MoE(RMSNorm(h)): without the norm
        # random layers grow the residual stream past fp32 range within a few layers
        from whallm_b200.moe import PreNorm
        layers, T_total = [synth.deepseek_mxfp4_layer(device=dev, seed=l) for l in range(8)], 256 + 4096
        for l, lay in enumerate(layers):
            g = torch.Generator(device=dev).manual_seed(700 + l)
            lay.norm = PreNorm((1.0 + 0.1 * torch.randn((lay.H,), generator=g, device=dev)).to(torch.bfloat16), 1e-6)
    lay0 = layers[0]
    Hn, In, En, Kn = lay0.H, lay0.I, lay0.E, 8
    if T_total % world or En % world:
        return {"workload": EP_SECTIONS[n][1], "skipped": f"{T_total} tokens / {En} experts do not split over {world}"}
    T_loc = T_total // world
    x_all = synth.activations(T_total, Hn, torch.Generator(device=dev).manual_seed(1), dev)
    x = x_all[rank * T_loc:(rank + 1) * T_loc].contiguous()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    steps = max(3, min(args.steps, 10))

    def stack(fwd, h):
        for i, lay in enumerate(layers):
            y = fwd(i, lay, h)
            h = y if len(layers) == 1 else h + y  # bf16 residual add between layers
        return h

    step_ms = []

    def timed(fwd, h0, nsteps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nsteps)]
        for i in range(nsteps):
            flush.zero_()
            evs[i][0].record()
            stack(fwd, h0)
            evs[i][1].record()
        torch.cuda.synchronize()
        step_ms[:] = [a.elapsed_time(b) for a, b in evs]
        return sum(step_ms) / nsteps

    # one GPU, the whole batch (rank 0; the grouped GEMM throughout)
    single = None
    if rank == 0:
        eng1 = Engine(local, max_tokens=T_total, hidden=Hn, inter=In, experts=En, topk=Kn, gemv_max_tokens=-1)
        fwd1 = lambda i, lay, h: eng1.forward(lay, h, Kn)  # noqa: E731
        for _ in range(2):
            flush.zero_()
            stack(fwd1, x_all)
        torch.cuda.synchronize()
        single = T_total / (timed(fwd1, x_all, steps) / 1e3)
        single_finite = bool(torch.isfinite(stack(fwd1, x_all).float()).all())
        eng1.ctx.close()
        del eng1
    out = {"workload": EP_SECTIONS[n][1], "tokens_per_step": T_total, "tokens_per_gpu": T_loc, "layers": len(layers),
           "l2": "flushed (256 MB write) before every timed step",
           "pre_moe_norm": n == 4}
    if world == 1:
        out.update({"tokens_per_s": single, "ms_per_step": T_total / single * 1e3, "single_gpu_tokens_per_s": single,
                    "efficiency": 1.0, "parallelism": "single GPU", "output_finite": single_finite})
        torch.cuda.empty_cache()
        return out

    # expert parallel: routing / combine handle, owner handle (single routes
    # from every peer), shared-expert handle; one exchange buffer for all layers
    C = T_loc * Kn
    eng = Engine(local, max_tokens=T_loc, hidden=Hn, inter=In, experts=En, topk=Kn, gemv_max_tokens=-1)
    owner = Engine(local, max_tokens=world * C, hidden=Hn, inter=In, experts=En // world, topk=1,
                   gemv_max_tokens=-1)
    shared = Engine(local, max_tokens=T_loc, hidden=Hn, inter=In, experts=1, topk=1, gemv_max_tokens=-1)
    eps = []
    for lay in layers:
        eps.append(ExpertParallelMoE(eng, lay, Kn, shared_engine=shared, fixed_capacity=T_loc, peer_memory=True,
                                     owner_engine=owner, peer_buffer=eps[0].ep_buf if eps else None))
    fwd = lambda i, lay, h: eps[i](h)  # noqa: E731
    for _ in range(2):
        flush.zero_()
        stack(fwd, x)
    torch.cuda.synchronize()
    dist.barrier()
    ms = timed(fwd, x, steps)
    # per-rank step statistics (mean, min, median, max): a slow rank or a slow step shows here
    mine = torch.tensor([ms, min(step_ms), statistics.median(step_ms), max(step_ms)], device=dev)
    every = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    per_rank = [[round(float(v), 3) for v in r.tolist()] for r in every]
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    # per-kernel split of one step on this rank (library events, eager)
    for e_ in (eng, owner, shared):
        e_.ctx.profile(True)
        e_.ctx.profile_reset()
    stack(fwd, x)
    torch.cuda.synchronize()
    kernels = {}
    for tag, e_ in (("", eng), ("owner_", owner), ("shared_", shared)):
        for name, (c, tt) in e_.ctx.profile_read().items():
            kernels[tag + name] = {"launches": c, "avg_us": 1e3 * tt / c, "total_us": 1e3 * tt}
        e_.ctx.profile(False)
    # parity: the expert-parallel stack against the one-GPU stack on this rank's tokens
    got = stack(fwd, x)
    ref_eng = Engine(local, max_tokens=T_loc, hidden=Hn, inter=In, experts=En, topk=Kn, gemv_max_tokens=-1)
    want = stack(lambda i, lay, h: ref_eng.forward(lay, h, Kn), x)
    torch.cuda.synchronize()
    exact = torch.tensor([1.0 if torch.equal(got.view(torch.int16), want.view(torch.int16)) else 0.0], device=dev)
    finite = torch.isfinite(got.float()).all().float().reshape(1)
    max_abs = (got.float() - want.float()).abs().max().reshape(1)
    dist.all_reduce(exact, op=dist.ReduceOp.MIN)
    dist.all_reduce(finite, op=dist.ReduceOp.MIN)
    dist.all_reduce(max_abs, op=dist.ReduceOp.MAX)
    eps[0].close()  # the shared exchange buffer (collective)
    for e_ in (eng, owner, shared, ref_eng):
        e_.ctx.close()
    tps = T_total / (ms / 1e3)
    top = max(kernels.items(), key=lambda kv: kv[1]["total_us"])[0] if kernels else None
    out.update({"tokens_per_s": tps, "ms_per_step": ms, "parallelism": f"expert-parallel x{world} "
                f"({En // world} experts per GPU per layer), NVLink peer-memory exchanges",
                "single_gpu_tokens_per_s": single,
                "efficiency": (tps / (world * single)) if single else None,
                "step_ms_per_rank": per_rank, "step_ms_fields": "mean, min, median, max over the timed steps",
                "efficiency_note": "tokens/s over N GPUs / (N x one GPU's tokens/s on the whole batch, rank 0, same run)",
                "parity": {"bit_exact": bool(exact.item() == 1.0), "finite": bool(finite.item() == 1.0),
                           "max_abs": float(max_abs.item()),
                           "against": "the one-GPU stack on each rank's tokens (grouped GEMM on both)"},
                "kernels_rank0_per_step": kernels if rank == 0 else None, "limiting_kernel": top})
    del eps, layers
    torch.cuda.empty_cache()
    return out


def run_ep(args, world: int, rank: int, local: int) -> None:
    """--gpus N > 1: the config-1 layer expert-parallel over N ranks."""
    import torch
    import torch.distributed as dist

    from whallm_b200 import lib, synth
    from whallm_b200.ep import ExpertParallelMoE
    from whallm_b200.moe import Engine

    dev = torch.device("cuda", local)
    B = args.batch
    wl = synth.config(1, device=dev, batch=B, seed=0)  # same seed: every rank holds the same layer
    layer = wl.layer
    nb = 8
    xs = [synth.activations(B, H, torch.Generator(device=dev).manual_seed(1000 * rank + i), dev) for i in range(nb)]
    # rows a rank receives are at most all ranks' pairs; decode kernels throughout
    cap = world * B * K
    eng = Engine(local, max_tokens=cap, hidden=H, inter=I, experts=E, topk=K, gemv_max_tokens=cap,
                 flags=lib.FLAG_SKIP_NEGATIVE_ROUTES)
    shared_eng = Engine(local, max_tokens=B, hidden=H, inter=I, experts=1, topk=1, gemv_max_tokens=B)
    # fixed-capacity exchanges (B * K slots per peer): no host round trip, so a
    # whole step is one CUDA graph (router, plan, the exchanges, experts,
    # shared expert on a side stream, combine); over NVLink peer memory by
    # default, NCCL all-to-all with --exchange nccl or when peer mapping fails
    exchange = args.exchange
    try:
        ep = ExpertParallelMoE(eng, layer, K, shared_engine=shared_eng, fixed_capacity=B,
                               peer_memory=exchange == "peer")
    except RuntimeError:  # every rank sees the same failure: all fall back together
        exchange = "nccl"
        ep = ExpertParallelMoE(eng, layer, K, shared_engine=shared_eng, fixed_capacity=B)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    x_static = xs[0].clone()

    def fwd(x):
        return ep(x)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            fwd(xs[i % nb])
    torch.cuda.synchronize()
    if exchange == "peer":
        # a bounded wait that ran out shows in the device status: if it did on
        # any rank, every rank measures the NCCL exchange instead
        healthy = torch.ones(1, device=dev)
        try:
            eng.sync()
        except lib.WMError:
            healthy.zero_()
        dist.all_reduce(healthy, op=dist.ReduceOp.MIN)
        if healthy.item() == 0:
            ep.close()
            exchange = "nccl"
            ep = ExpertParallelMoE(eng, layer, K, shared_engine=shared_eng, fixed_capacity=B)
            with torch.cuda.stream(stream):
                for i in range(args.warmup):
                    fwd(xs[i % nb])
            torch.cuda.synchronize()
    c0 = eng.ctx.counters().launches + shared_eng.ctx.counters().launches
    with torch.cuda.stream(stream):
        fwd(xs[0])
    torch.cuda.synchronize()
    launches_per_step = eng.ctx.counters().launches + shared_eng.ctx.counters().launches - c0
    graph, graph_error = None, None
    try:
        with torch.cuda.stream(stream):
            fwd(x_static)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out_static = fwd(x_static)
        torch.cuda.synchronize()
    except Exception as exc:  # eager steps then
        graph, graph_error = None, f"{type(exc).__name__}: {exc}"[:200]
        torch.cuda.synchronize()
    dist.barrier()

    def step(i, ev=None):
        if graph is not None:
            x_static.copy_(xs[i % nb])
        flush.zero_()
        if ev is not None:
            ev[0].record(stream)
        if graph is not None:
            graph.replay()
        else:
            fwd(xs[i % nb])
        if ev is not None:
            ev[1].record(stream)

    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with Clocks(local, args.clocks_dir) as clocks:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(args.warmup):
                step(i)
            for i in range(args.steps):
                step(i, evs[i])
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs)
    t = torch.tensor([ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = world * B * args.steps / (ms / 1e3)

    # per-kernel durations on this rank (library CUDA events), eager
    eng.ctx.profile(True)
    eng.ctx.profile_reset()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush.zero_()
            fwd(xs[i % nb])
    torch.cuda.synchronize()
    prof = eng.ctx.profile_read()
    eng.ctx.profile(False)
    kernels = {name: {"launches": n, "avg_us": 1e3 * tt / n} for name, (n, tt) in prof.items()}
    # the same steps' host-side time split (rank 0): where an eager step goes
    t_host = []
    with torch.cuda.stream(stream):
        for i in range(min(args.steps, 10)):
            torch.cuda.synchronize()
            h0 = time.perf_counter()
            fwd(xs[i % nb])
            torch.cuda.synchronize()
            t_host.append(1e3 * (time.perf_counter() - h0))

    # end to end with pinned host buffers
    xh = [x.cpu().pin_memory() for x in xs]
    oh = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()
    e_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            flush.zero_()
            e_evs[i][0].record(stream)
            if graph is not None:
                x_static.copy_(xh[i % nb], non_blocking=True)
                graph.replay()
                oh.copy_(out_static, non_blocking=True)
            else:
                oh.copy_(fwd(xh[i % nb].to(dev, non_blocking=True)), non_blocking=True)
            e_evs[i][1].record(stream)
    torch.cuda.synchronize()
    e_ms = sum(a.elapsed_time(b) for a, b in e_evs)
    t = torch.tensor([e_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e_ms = float(t.item())
    e2e = world * B * args.steps / (e_ms / 1e3)
    del graph  # holds NCCL work: release before the process group goes

    # parity: each rank's expert-parallel layer against the one-GPU layer on the same tokens (decode kernels on both)
    exact, max_abs = torch.ones(1, device=dev), torch.zeros(1, device=dev)
    with torch.cuda.stream(stream):
        for i in range(nb):
            got = fwd(xs[i]).clone()
            want = eng.forward(layer, xs[i], K)
            if not torch.equal(got.view(torch.int16), want.view(torch.int16)):
                exact.zero_()
            max_abs = torch.maximum(max_abs, (got.float() - want.float()).abs().max().reshape(1))
    torch.cuda.synchronize()
    dist.all_reduce(exact, op=dist.ReduceOp.MIN)
    dist.all_reduce(max_abs, op=dist.ReduceOp.MAX)
    parity = {"bit_exact": bool(exact.item() == 1.0), "max_abs": float(max_abs.item()),
              "against": f"the one-GPU layer on every rank's {nb} batches"}
    ep.close()
    eng.ctx.close()
    shared_eng.ctx.close()
    del ep, eng, shared_eng
    torch.cuda.empty_cache()
    long_sections = {}
    if not args.no_long:
        pk = peaks()
        for n in (3, 4):
            long_sections[EP_SECTIONS[n][0]] = long_ep_section(args, n, world, rank, local, pk)
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32-accumulate MXFP4 x bf16",
        "data": "synthetic (seeded; BASELINE configs[1] value distributions)",
        "config": {"workload": f"config1 decode layer, {B} tokens per step per GPU", "H": H, "I": I, "E": E,
                   "K": K, "shared_expert": True, "router": "softmax top-10",
                   "l2": "flushed (256 MB write) before every timed step",
                   "timing": ("CUDA graph replay per step" if graph_error is None else "eager steps")
                   + ", device events, max over ranks",
                   "graph_error": graph_error,
                   "parallelism": f"expert-parallel x{world} ({E // world} experts per GPU)",
                   "exchange": (f"NVLink peer-memory stores of the real pairs ({B * K} slots per peer), "
                                "device flags" if exchange == "peer"
                                else f"NCCL all-to-all, fixed {B * K} slots per peer each way"),
                   "wall_ms_per_step_rank0": statistics.median(t_host)},
        "roofline": None,
        "kernels": kernels,
        "cpu_baseline": None,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": world * B * H * 2,
                "d2h_bytes_per_step": world * B * H * 2},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "parity": parity,
        **long_sections,
    }
    print(json.dumps(line), flush=True)


def decode_batch_line(eng, layer, dev, B: int, steps: int, flush) -> dict:
    """Config-1 decode at batch B (graph replay per step, L2 flushed, device
    events): latency, tokens/s and the layer's bytes per second."""
    import torch
    from whallm_b200 import synth

    xs = [synth.activations(B, H, torch.Generator(device=dev).manual_seed(500 + i), dev) for i in range(8)]
    x_static = xs[0].clone()
    out = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(2):
            eng.forward(layer, x_static, K, out=out)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            eng.forward(layer, x_static, K, out=out)
    torch.cuda.synchronize()
    uniq = []
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    with torch.cuda.stream(stream):
        for i in range(3 + steps):
            x_static.copy_(xs[i % 8])
            flush.zero_()
            if i >= 3:
                evs[i - 3][0].record(stream)
            graph.replay()
            if i >= 3:
                evs[i - 3][1].record(stream)
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    for i in range(8):
        _, (_, ri) = eng.forward(layer, xs[i], K, return_routes=True)
        uniq.append(int(torch.unique(ri).numel()))
    torch.cuda.synchronize()
    # where the time goes: per-kernel CUDA-event durations of eager calls (each
    # includes its launch; the graph-replayed step above has no host gaps)
    eng.ctx.profile(True)
    eng.ctx.profile_reset()
    for i in range(steps):
        x_static.copy_(xs[i % 8])
        flush.zero_()
        eng.forward(layer, x_static, K, out=out)
    torch.cuda.synchronize()
    kernels = {n: round(1e3 * t / c, 2) for n, (c, t) in eng.ctx.profile_read().items()}
    eng.ctx.profile(False)
    del graph
    U = sum(uniq) / len(uniq)
    layer_bytes = (U + 1) * BLOB + E * H * 2 + H * 2 + 4 * B * H  # experts + router + shared gate + x/out
    return {"batch": B, "ms_per_step": ms, "tokens_per_s": B / (ms / 1e3), "unique_experts": U,
            "layer_bytes": layer_bytes, "achieved_gbs": layer_bytes / (ms / 1e3) / 1e9,
            "kernels_avg_us_eager": kernels}


def cpu_baselines(dev, cores: int, threads: int) -> dict:
    """The CPU oracle (OpenMP over the host cores) on bounded samples of
    configs 0, 2 and 3 (config 1 is the headline cpu_baseline): routes come
    from the GPU layer, only the experts the sampled tokens reach are copied
    to the host, each sample repeats for at least 4 s."""
    import numpy as np
    import torch
    from oracle import adapter
    from whallm_b200 import synth
    from whallm_b200.moe import Engine

    out = {}
    wl = synth.config(0, device=dev)
    layer_np = adapter.from_layer(wl.layer)
    T0 = wl.x.shape[0]
    idx0, w0 = np.zeros((T0, 1), np.int32), np.ones((T0, 1), np.float32)
    out["config0"] = {"value": cpu_sample(layer_np, adapter.bits(wl.x), idx0, w0, 4.0, T0), "unit": "tokens/s",
                      "sample": f"the whole config-0 call ({T0} tokens, one expert)"}
    for n, sample in ((2, 8), (3, 2)):
        wl = synth.config(n, device=dev)
        T, Hn = wl.x.shape
        eng = Engine(dev.index, max_tokens=T, hidden=Hn, inter=wl.layer.I, experts=wl.layer.E, topk=wl.K)
        _, (w, idx) = eng.forward(wl.layer, wl.x, wl.K, return_routes=True)
        torch.cuda.synchronize()
        tokens = np.random.default_rng(n).choice(T, sample, replace=False)
        ii, ww = idx.cpu().numpy()[tokens], w.cpu().numpy()[tokens]
        experts = sorted(set(ii.reshape(-1).tolist()))
        remap = {e: i for i, e in enumerate(experts)}
        sub_np = adapter.from_layer(wl.layer, experts=experts)
        tps = cpu_sample(sub_np, adapter.bits(wl.x[torch.as_tensor(tokens, device=dev)]),
                         np.vectorize(remap.get)(ii).astype(np.int32), ww, 4.0, sample)
        out[f"config{n}"] = {"value": tps, "unit": "tokens/s",
                             "sample": f"{sample} tokens of the {T}-token config-{n} call (their {len(experts)} experts)"}
        eng.ctx.close()
        del wl, eng, sub_np
        torch.cuda.empty_cache()
    for v in out.values():
        v.update({"cores": threads, "kind": "port", "threads_note": f"OpenMP threads {threads} on {cores} cores"})
    return out


def run(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from whallm_b200 import lib, synth
    from whallm_b200.moe import Engine

    world, rank, local = dist_init()
    if world > 1:
        run_ep(args, world, rank, local)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B = args.batch
    wl = synth.config(1, device=dev, batch=B, seed=0)
    layer = wl.layer
    nb = 8
    xs = [synth.activations(B, H, torch.Generator(device=dev).manual_seed(1000 * rank + i), dev) for i in range(nb)]
    flag = DECODE_FLAGS[args.decode]
    eng = Engine(local, max_tokens=max(B, 64), hidden=H, inter=I, experts=E, topk=K,
                 flags=getattr(lib, flag) if flag else 0)
    x_static = xs[0].clone()
    out_static = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)

    # launches of our kernels in one step (counted on an eager call)
    c0 = eng.ctx.counters().launches
    eng.forward(layer, x_static, K, out=out_static)
    eng.sync()
    launches_per_step = eng.ctx.counters().launches - c0

    # capture one step as a CUDA graph (router -> plan -> GEMVs -> combine)
    with torch.cuda.stream(stream):
        for _ in range(2):
            eng.forward(layer, x_static, K, out=out_static)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            eng.forward(layer, x_static, K, out=out_static)
    torch.cuda.synchronize()

    def step(i, timed_events=None):
        x_static.copy_(xs[i % nb])
        flush.zero_()
        if timed_events is not None:
            timed_events[0].record(stream)
        graph.replay()
        if timed_events is not None:
            timed_events[1].record(stream)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with Clocks(local, args.clocks_dir) as clocks:
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                step(i, evs[i])
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in evs)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    value = world * B * args.steps / (ms / 1e3)

    # per-kernel durations (library CUDA events) over the same steps, eager
    eng.ctx.profile(True)
    eng.ctx.profile_reset()
    uniq = []
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            x_static.copy_(xs[i % nb])
            flush.zero_()
            _, (rw, ri) = eng.forward(layer, x_static, K, out=out_static, return_routes=True)
            uniq.append(int(torch.unique(ri).numel()))
    torch.cuda.synchronize()
    prof = eng.ctx.profile_read()
    eng.ctx.profile(False)
    U = statistics.mean(uniq)
    gu_n, gu_ms = prof.get("decode_gate_up", (1, float("nan")))
    dn_n, dn_ms = prof.get("decode_down", (1, float("nan")))
    gu_bytes = (U + 1) * GATE_UP_BYTES + B * H * 2 + B * 2 * I * 2  # weights + x + act written
    dn_bytes = (U + 1) * DOWN_BYTES + (B * K + B) * (I * 2 + H * 2)
    pk = peaks()
    if args.decode == "fused":  # one launch streams both projections: its bytes over its time
        fu_n, fu_ms = prof.get("decode_fused", (1, float("nan")))
        gu_bytes, gu_avg = gu_bytes + dn_bytes, fu_ms / fu_n
        dn_n, dn_ms = fu_n, fu_ms
    else:
        gu_avg = gu_ms / gu_n
    achieved = gu_bytes / (gu_avg / 1e3) / 1e9
    kernels = {name: {"launches": n, "avg_us": 1e3 * t / n} for name, (n, t) in prof.items()}

    # end to end through the public call with pinned host buffers
    xh = [x.cpu().pin_memory() for x in xs]
    oh = torch.empty((B, H), dtype=torch.bfloat16).pin_memory()
    e_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            eng.replay(layer, xh[i % nb], K, out=oh)
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            e_evs[i][0].record(stream)
            eng.replay(layer, xh[i % nb], K, out=oh)
            e_evs[i][1].record(stream)
    torch.cuda.synchronize()
    e_ms = sum(a.elapsed_time(b) for a, b in e_evs)
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e = world * B * args.steps / (e_ms / 1e3)

    del graph
    # the small batches before the CPU baseline: its OpenMP threads keep
    # spinning for a while after it returns, and a short step's time depends
    # on the host enqueueing its launches promptly
    decode_batches = [decode_batch_line(eng, layer, dev, b, max(10, min(args.steps, 30)), flush) for b in (1, 8)]
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        from oracle import adapter
        layer_np = adapter.from_layer(layer)
        xb = adapter.bits(xs[0])
        _, (rw, ri) = eng.forward(layer, xs[0], K, return_routes=True)
        cores = len(os.sched_getaffinity(0))
        oracle.set_threads(cores)
        threads = oracle.max_threads()
        tps = cpu_sample(layer_np, xb, ri.cpu().numpy(), rw.cpu().numpy(), min_seconds=10.0, tokens=16)
        cpu = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"16 tokens of a config-1 batch, repeated for >= 10 s, OpenMP threads {threads} on {cores} cores"}
        if not args.no_prefill:
            cpu["other_configs"] = cpu_baselines(dev, cores, threads)

    prefill = None if args.no_prefill else prefill_section(args, dev, pk, 2)
    long_calls = None
    long_sections = {}
    if not args.no_prefill and not args.no_long:
        long_calls = {"config3": prefill_section(args, dev, pk, 3), "config4_layer": prefill_section(args, dev, pk, 4)}
        for n in (3, 4):
            long_sections[EP_SECTIONS[n][0]] = long_ep_section(args, n, 1, 0, local, pk)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32-accumulate MXFP4 x bf16",
        "data": "synthetic (seeded; BASELINE configs[1] value distributions)",
        "config": {"workload": f"config1 decode layer, {B} tokens per step per GPU", "H": H, "I": I, "E": E,
                   "K": K, "shared_expert": True, "router": "softmax top-10",
                   "l2": "flushed (256 MB write) before every timed step",
                   "timing": "CUDA graph replay per step, device events, max over ranks",
                   "parallelism": "single GPU",
                   "unique_experts_per_step": U},
        "roofline": {"bound": "hbm", "kernel": DECODE_KERNEL[args.decode], "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_source": pk["source"], "traffic": NCU_GATE_UP_TRAFFIC[args.decode],
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch, "
                                        + DECODE_PROFILE[args.decode]) if DECODE_PROFILE[args.decode]
                                       else "no ncu capture of this kernel yet",
                     "algorithmic_bytes_per_launch": gu_bytes,
                     "down_achieved_gbs": (None if args.decode == "fused"
                                           else dn_bytes / (dn_ms / dn_n / 1e3) / 1e9)},
        "kernels": kernels,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "decode_batches": decode_batches,
        "prefill": prefill,
        "long_calls": long_calls,
        **long_sections,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-long", action="store_true", help="skip the config-3 and config-4 long-call sections")
    ap.add_argument("--clocks-dir", default=None,
                    help="folder for the raw nvidia-smi clock samples (default: the system temp folder)")
    ap.add_argument("--decode", default="bs", choices=["bs", "mma", "fused"],
                    help="decode expert kernels: block-scaled tcgen05 (bs, the default), register-direct warp MMAs, "
                         "or the block-scaled gate/up and down in one launch (fused)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1: expert-parallel exchanges over peer memory (default) or NCCL all-to-all")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    # Python's cyclic collector stays off while the bench runs (reference
    # counting still frees almost everything): a collection pause on one rank
    # in a timed region stalls every rank's bounded peer waits with it
    gc.collect()
    gc.disable()
    if args.impl == "reference":
        run_reference(args)
    else:
        run(args)


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark: MoE-layer decode tokens/s of the B200 routed-expert hot path.

Workload: a stack of 48 FP8 MoE layers (hidden 2048, 128
experts, top-8, intermediate 768, E4M3 with fp32 128x128 block scales, RMSNorm
with gamma 1+N(0,0.01)), decode batch 1, 512 consecutive decode steps captured
in one CUDA graph, all experts resident in HBM (29 GB). One bench step = one
replay of that graph (512 tokens). Inputs are seeded synthetic bf16 N(0,1)
rows; every token reads ~1.84 GB of expert weights, far more than L2.

Arms:
  python bench.py [--gpus N --steps K --warmup W]        this repository
  python bench.py --impl reference [...]                  the reference's own
        CPU expert core (native/src/*.cpp built under oracle/_ref) timed on
        the host cores on a bounded sample of the same workload.
Under torchrun each rank runs an independent replica (the decode path has no
exchange step at batch 1); timing is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "drama3-studio_b200"))
sys.path.insert(0, str(REPO))

METRIC = "MoE-layer decode tokens/s and expert-weight HBM GB/s vs ~8 TB/s at 1/2/4/8 B200"
HIDDEN, EXPERTS, TOP_K, INTER = 2048, 128, 8, 768


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--decode-steps", type=int, default=512, help="decode tokens per CUDA graph")
    p.add_argument("--workload", choices=("decode", "prefill", "ep", "offload", "int4", "w8a8", "shared"),
                   default="decode",
                   help="decode: config 1 (the headline); prefill: config 3 (4096 tokens, one layer, Zipf); "
                        "ep: config 4 expert-parallel decode of 256 tokens over the torchrun ranks; "
                        "offload: config 4's 1-GPU offload variant (32 of 128 experts resident per layer); "
                        "int4: config 2 (one W4A16 asymmetric layer, decode batches 1/4/16, uniform routes); "
                        "w8a8: config 2's measurement on a W8A8 bank of --mode 1, 2 or 3; "
                        "shared: the shared expert + gate fused with the routed sum and residual, 48 layers")
    p.add_argument("--shared-inter", type=int, default=768,
                   help="shared: shared_expert_intermediate_size (the checkpoint's value is not available here)")
    p.add_argument("--mode", type=int, choices=(1, 2, 3), default=1,
                   help="w8a8: 1 INT8-ConvRot, 2 W6A8, 3 W4A8 codebook")
    p.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p",
                   help="ep: NVLink peer-memory exchange (default) or NCCL all-to-alls")
    p.add_argument("--host-layers", type=int, default=48,
                   help="offload: distinct pinned host stores (layers beyond reuse them in turn)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--router", choices=("fused", "torch"), default="fused",
                   help="decode: router in the fused layer kernel, or torch's RMSNorm/linear in front (bit-exact ids)")
    p.add_argument("--contract", choices=("w8a8", "w16a16"), default="w8a8",
                   help="prefill: the production W8A8 contract on tcgen05 (default) or the W16A16 dequant contract")
    p.add_argument("--no-ep", action="store_true",
                   help="decode: skip the config-4 expert-parallel sub-record (\"ep\") of the headline line")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    return p.parse_args()


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and throttle reasons sampled while the timed region runs.

    NVML is polled every 2 ms from a thread, so a timed region of a few tens
    of milliseconds still gets samples; ``nvidia-smi -lms 200`` is the
    fallback when NVML cannot be loaded. ``__enter__`` returns after the first
    sample (or 2 s), so the sampler is running when the region starts.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                   ("sw_power_cap", 0x4))

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.samples: list[tuple[float, float, int]] = []   # (sm MHz, max MHz, reason mask)
        self.lines: list[str] = []
        self.proc = None
        self.thread = None
        self.stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            if self.gpu_id.startswith("GPU-"):
                handle = pynvml.nvmlDeviceGetHandleByUUID(self.gpu_id)
            else:
                handle = pynvml.nvmlDeviceGetHandleByIndex(int(self.gpu_id))
            max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))

            def poll():
                while not self.stop.is_set():
                    try:
                        mhz = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                        mask = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
                        self.samples.append((mhz, max_mhz, mask))
                    except pynvml.NVMLError:
                        pass
                    self.stop.wait(0.002)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
        except Exception:  # NVML missing or the device not found: nvidia-smi instead
            self.thread = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                     "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.thread = threading.Thread(target=self._read, daemon=True)
                self.thread.start()
            except (OSError, ValueError):
                self.proc = None
        deadline = time.monotonic() + 2.0
        while self.thread is not None and not (self.samples or self.lines) and time.monotonic() < deadline:
            time.sleep(0.002)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self) -> dict:
        mhz, max_mhz, reasons = [], None, set()
        for sm, mx, mask in self.samples:
            mhz.append(sm)
            max_mhz = mx
            reasons.update(name for name, bit in self.REASON_BITS if mask & bit)
        names = [name for name, _ in self.REASON_BITS]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for name, value in zip(names, parts[5:9]):
                if value.lower() == "active":
                    reasons.add(name)
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz),
                "source": "nvml 2 ms" if self.samples else "nvidia-smi 200 ms"}


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def committed_traffic(name: str = "moe_layer_traffic.json") -> float | None:
    """DRAM bytes per launch of a bench's dominant kernel from a committed ncu
    summary under profiles/ (read + write, one capture)."""
    path = REPO / "profiles" / name
    if path.is_file():
        return json.loads(path.read_text()).get("dram_bytes_per_layer")
    return None


# ---------------------------------------------------------------------------
# CPU baseline: the reference's native expert core (W8A8 contract) plus the
# oracle's RMSNorm/router restatement, timed on the host cores.
# ---------------------------------------------------------------------------
class CpuReference:
    """One config-1 layer on the host: bank, router, and the native executor."""

    def __init__(self, bank=None):
        import torch

        from drama_b200 import synthetic
        from oracle.ref_native import ReferenceNative

        self.threads = os.cpu_count() or 1
        self.lib = ReferenceNative()
        if bank is None:
            bank = synthetic.fp8_bank(EXPERTS, HIDDEN, INTER, 0, chunk=EXPERTS)
        bank = {k: v.detach().cpu() for k, v in bank.items()}
        self.bank = {k: (v.view(torch.uint8).numpy() if v.dtype == torch.float8_e4m3fn else v.numpy())
                     for k, v in bank.items()}
        self.gate = synthetic.gate_weight(EXPERTS, HIDDEN, 500).float().numpy()
        self.gamma = synthetic.norm_gamma(HIDDEN, 700).numpy()
        self.x = synthetic.hidden_states(1, HIDDEN, 11).float().numpy()
        self.executor = self.lib.executor(HIDDEN, INTER, capacity=TOP_K, threads=self.threads)

    def layer(self) -> None:
        from oracle import restate as R

        normed = R.rms_norm(self.x, self.gamma)
        logits = R.gate_logits(normed, self.gate)
        ids, w, _ = R.route_topk(logits, TOP_K, True, "bfloat16")
        partials = self.executor.forward(self.bank, R.bf16_bits(normed[0]), ids[0], w[0])
        self.x = R.round_bf16(self.x + R.round_bf16(partials.sum(0))[None, :])

    def sample(self, seconds: float, layers: int) -> dict:
        done, start = 0, time.perf_counter()
        while True:
            self.layer()
            done += 1
            elapsed = time.perf_counter() - start
            if elapsed >= seconds:
                break
        per_layer = elapsed / done
        return {
            "value": 1.0 / (per_layer * layers), "unit": "tokens/s", "cores": self.threads, "kind": "reference",
            "sample": (f"{done} token-layers in {elapsed:.1f}s: the reference's native expert core "
                       f"(native/src/*.cpp, W8A8 contract, {self.threads} threads) for the 8 routed experts "
                       f"plus the oracle's RMSNorm/router; one config-1 layer bank stands in for every "
                       f"layer position; value = 1 / ({layers} x mean token-layer time)"),
        }


class TorchDequantReference:
    """The reference's PyTorch dequant path on the host: TorchExpertBackend.forward.

    ``src/drama_low_vram/offload.py:199-244`` run unmodified from the copy that
    build() places under oracle/_ref, on CPU tensors, one config-0 token-layer
    per call (the 8 routed experts dequantised to bf16, F.linear, weighted slot
    sum), with the oracle's RMSNorm and router in front as in CpuReference.
    """

    def __init__(self, bank):
        import torch

        sys.path.insert(0, str(REPO / "oracle" / "_ref"))
        from drama_low_vram.offload import StagedExperts, TorchExpertBackend

        from drama_b200 import synthetic

        self.torch = torch
        self.threads = torch.get_num_threads()
        self.staged = StagedExperts(**{k: v.detach().cpu().contiguous() for k, v in bank.items()})
        self.backend = TorchExpertBackend()
        self.gate = synthetic.gate_weight(EXPERTS, HIDDEN, 500).float().numpy()
        self.gamma = synthetic.norm_gamma(HIDDEN, 700).numpy()
        self.x = synthetic.hidden_states(1, HIDDEN, 11).float().numpy()

    def layer(self) -> None:
        from oracle import restate as R

        torch = self.torch
        normed = R.rms_norm(self.x, self.gamma)
        logits = R.gate_logits(normed, self.gate)
        ids, w, _ = R.route_topk(logits, TOP_K, True, "bfloat16")
        x = torch.from_numpy(normed).to(torch.bfloat16)
        moe = self.backend.forward(x, torch.from_numpy(ids), torch.from_numpy(w).to(torch.bfloat16), self.staged)
        self.x = R.round_bf16(self.x + moe.float().numpy())

    def sample(self, seconds: float, layers: int) -> dict:
        done, start = 0, time.perf_counter()
        while True:
            self.layer()
            done += 1
            elapsed = time.perf_counter() - start
            if elapsed >= seconds:
                break
        per_layer = elapsed / done
        return {
            "value": 1.0 / (per_layer * layers), "unit": "tokens/s", "cores": self.threads, "kind": "reference",
            "sample": (f"{done} token-layers in {elapsed:.1f}s: the reference's TorchExpertBackend.forward "
                       f"(offload.py:199-244, W16A16 dequant path, torch on {self.threads} threads) for the 8 "
                       f"routed experts plus the oracle's RMSNorm/router; value = 1 / ({layers} x mean "
                       f"token-layer time)"),
        }


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    ref = CpuReference()
    for _ in range(max(1, args.warmup)):
        ref.layer()
    # One bench step = one decode token through every layer position.
    start = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(args.layers):
            ref.layer()
    total = time.perf_counter() - start
    value = args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8-e4m3 weights and activations (W8A8), fp32 accumulate", "data": "synthetic",
        "config": config_dict(args, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ref.threads, "kind": "reference",
                         "sample": (f"{args.steps} decode tokens x {args.layers} layer positions through the "
                                    f"reference's native expert core (native/src/*.cpp, {ref.threads} "
                                    f"threads) with the oracle's RMSNorm/router; one layer bank reused")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def config_dict(args, world: int) -> dict:
    return {
        "workload": (f"config1: {args.layers} FP8 MoE layers (hidden {HIDDEN}, {EXPERTS} experts, top-{TOP_K}, "
                     f"intermediate {INTER}, E4M3 128x128 block scales), decode batch 1, "
                     f"{args.decode_steps} steps per CUDA graph, all experts resident"),
        "layers": args.layers, "hidden": HIDDEN, "experts": EXPERTS, "top_k": TOP_K, "intermediate": INTER,
        "batch": 1, "decode_steps_per_graph": args.decode_steps, "router": getattr(args, "router", "fused"),
        "parallelism": f"replicas{world}" if world > 1 else "single",
        "l2": "inputs larger than L2: 29 GB of resident banks, ~1.84 GB of routed weights per token",
    }


# ---------------------------------------------------------------------------
# this repository's arm
# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))

    from drama_b200 import stack, synthetic

    t0 = time.perf_counter()
    layers = stack.synthetic_stack(args.layers, experts=EXPERTS, hidden=HIDDEN, intermediate=INTER,
                                   seed=rank, device=device)
    st = stack.DecodeStack(layers, tokens=1, top_k=TOP_K, router=args.router)
    steps_per_graph = args.decode_steps
    inputs = torch.stack([synthetic.hidden_states(1, HIDDEN, 10_000 + s, device=device)
                          for s in range(steps_per_graph)])
    outputs = torch.empty_like(inputs)
    build_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    graph = st.capture(inputs, outputs, timed_steps=1)
    capture_s = time.perf_counter() - t0

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier()
    props = torch.cuda.get_device_properties(device)
    gpu_id = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    layer_ms = st.layer_time_ms()
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # e2e: public API with host buffers (inputs H2D from pinned memory, outputs D2H).
    host_in = inputs.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        inputs.copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(outputs, non_blocking=True)
    f1.record()
    f1.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    tokens = args.steps * steps_per_graph * world
    value = tokens / (ms / 1000.0)
    expert_bytes = synthetic.expert_nbytes_fp8(HIDDEN, INTER) * TOP_K
    # per layer: the routed experts, the router weight, gamma, the hidden row in and out
    layer_bytes = expert_bytes + EXPERTS * HIDDEN * 2 + HIDDEN * 4 + HIDDEN * 2 * 2
    peaks = measured_peaks()
    # average duration of one layer launch over the timed region (the graph
    # holds only the layer launches; consecutive layers overlap by programmatic
    # dependent launch, so this is their spacing), and the same layer bracketed
    # by events on its own in the graph's first step
    launches = args.steps * steps_per_graph * args.layers * st.launches_per_layer()
    launch_ms = ms / (args.steps * steps_per_graph * args.layers)
    achieved = layer_bytes / (launch_ms / 1000.0) / 1e9
    traffic = committed_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp8-e4m3 weights, bf16/f16 activations, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and hidden rows)", "config": config_dict(args, world),
        "hbm_gbs_per_gpu": layer_bytes * args.layers * value / world / 1e9,
        "roofline": {
            "kernel": ("one MoE layer: decode_layer_kernel (RMSNorm, router, gate/up, down and slot combine in "
                       "one launch)" if st.launches_per_layer() == 1 else
                       "one MoE layer: routed_up_kernel (router + gate/up) + routed_down_kernel (down + combine)"),
            "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)",
            "traffic": traffic, "algorithmic_bytes_per_launch": layer_bytes, "launch_ms": launch_ms,
            "isolated_launch_ms": layer_ms,
        },
        "e2e": {"value": tokens / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": inputs.numel() * 2, "d2h_bytes_per_step": outputs.numel() * 2},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "setup_s": {"build": round(build_s, 1), "capture": round(capture_s, 1)},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = CpuReference({"w13_weight": layers[0].w13_weight, "w13_scale_inv": layers[0].w13_scale_inv,
                            "w2_weight": layers[0].w2_weight, "w2_scale_inv": layers[0].w2_scale_inv})
        ref.layer()
        line["cpu_baseline"] = ref.sample(args.cpu_seconds, args.layers)
        if (REPO / "oracle" / "_ref" / "drama_low_vram").is_dir():
            bank = {"w13_weight": layers[0].w13_weight, "w13_scale_inv": layers[0].w13_scale_inv,
                    "w2_weight": layers[0].w2_weight, "w2_scale_inv": layers[0].w2_scale_inv}
            torch_ref = TorchDequantReference(bank)
            torch_ref.layer()
            line["cpu_baseline"]["torch_dequant"] = torch_ref.sample(args.cpu_seconds / 2, args.layers)
    del graph
    if not args.no_ep:
        # config 4 at the same N: the driver's 1 -> 8 runs then also time expert parallelism
        del st, layers, inputs, outputs
        torch.cuda.empty_cache()
        ep_line, model, ep_graph = measure_ep(args, world, rank, device, gpu_id)
        line["ep"] = {k: ep_line[k] for k in ("metric", "value", "unit", "n_gpus", "ms_per_step", "scaling",
                                                 "roofline", "e2e", "gpu_launches", "checksum", "clocks")}
        line["ep"]["workload"] = ep_line["config"]["workload"]
        line["ep"]["exchange"] = ep_line["config"]["exchange"]
        line["ep"]["peer_wait_timed_out"] = ep_line["peer_wait_timed_out"]
        del ep_graph
        model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def fp8_gemm_peak(device) -> dict:
    """Dense E4M3 tensor throughput measured here: cuBLASLt through
    torch._scaled_mm, 8192^3, best of 10 (a burst, like MEASURED_PEAKS.json's
    bf16 figure). Falls back to twice the measured bf16 burst (the B200's
    FP8 : BF16 dense ratio) when the FP8 GEMM is unavailable."""
    import torch

    n = 8192
    try:
        a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
        b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()
        one = torch.ones((), device=device)
        for _ in range(3):
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return {"tflops": 2.0 * n ** 3 / (best / 1000.0) / 1e12,
                "source": "measured in this run: torch._scaled_mm E4M3 x E4M3 -> bf16, 8192^3, best of 10"}
    except (RuntimeError, TypeError) as exc:
        path = REPO / "MEASURED_PEAKS.json"
        bf16 = json.loads(path.read_text())["bf16_tflops"] if path.is_file() else 1590.0
        return {"tflops": 2.0 * bf16, "source": f"2 x MEASURED_PEAKS.json bf16_tflops ({exc.__class__.__name__})"}


def run_prefill(args) -> None:
    """Config 3: one FP8 MoE layer over 4096 prefill tokens, Zipf(1.1) routes.

    ``--contract w8a8`` (default): one step = ``drama_b200_fp8_w8a8_prefill``
    (permute, sorted-row quantisation, gate/up and down grouped GEMMs on the
    tcgen05 tensor cores, combine), the arithmetic of the reference's
    production GPU backend; the roofline is the E4M3 tensor pipe.
    ``--contract w16a16``: ``fp8_prefill`` (TorchExpertBackend's dequant
    arithmetic on bf16 mma.sync tensor cores) against the bf16 peak.
    FLOPs = 2 * pairs * (2I * H + H * I) per step.
    """
    import ctypes

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))
    from drama_b200 import _lib, synthetic
    from drama_b200.backend import _fp8_bank, fp8_prefill

    tokens = 4096
    bank = synthetic.fp8_bank(EXPERTS, HIDDEN, INTER, rank, device=device, chunk=EXPERTS)

    class Staged:
        w13_weight = bank["w13_weight"]
        w13_scale_inv = bank["w13_scale_inv"]
        w2_weight = bank["w2_weight"]
        w2_scale_inv = bank["w2_scale_inv"]

    ids, w = synthetic.zipf_routes(tokens, TOP_K, EXPERTS, 100 + rank, device=device)
    ids = ids.to(torch.int64).contiguous()
    w = w.to(torch.bfloat16).contiguous()
    x = synthetic.hidden_states(tokens, HIDDEN, 200 + rank, device=device)
    out = torch.empty_like(x)
    if args.contract == "w8a8":
        lib = _lib.library()
        desc, keep = _fp8_bank(Staged, HIDDEN)
        nbytes = lib.dll.drama_b200_fp8_w8a8_prefill_workspace_bytes(tokens, TOP_K, HIDDEN, INTER, EXPERTS)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
        stream = _lib.stream_handle(device)

        def step():
            lib.check(lib.dll.drama_b200_fp8_w8a8_prefill(
                ctypes.byref(desc), x.data_ptr(), tokens, TOP_K, ids.data_ptr(), _lib.I64, w.data_ptr(), _lib.BF16,
                out.data_ptr(), None, ws.data_ptr(), ws.numel(), stream))
            return out

        launches, kernel = 5, ("prefill step: permute + sorted-row quantisation + gate/up and down grouped GEMMs "
                               "(tcgen05, TMEM accumulators) + combine")
        dtype = "fp8-e4m3 weights and activations (1x128 / 128x128 block scales), fp32 accumulate"
    else:
        def step():
            return fp8_prefill(x, ids, w, Staged, validate_ids=False)

        launches, kernel = 4, "prefill step: permute + gate/up GEMM + down GEMM + combine (bf16 mma.sync)"
        dtype = "fp8-e4m3 weights dequantised to bf16, bf16 activations, fp32 accumulate"
    for _ in range(max(3, args.warmup)):
        step()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    barrier()
    props = torch.cuda.get_device_properties(device)
    gpu_id = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    host_x = x.cpu().pin_memory()
    host_out = torch.empty_like(host_x).pin_memory()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        x.copy_(host_x, non_blocking=True)
        result = step()
        host_out.copy_(result, non_blocking=True)
    f1.record()
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    pairs = tokens * TOP_K
    flops = 2.0 * pairs * (2 * INTER * HIDDEN + HIDDEN * INTER)
    if args.contract == "w8a8":
        fp8 = fp8_gemm_peak(device)
        peak, peak_source = fp8["tflops"], fp8["source"]
    else:
        peak_path = REPO / "MEASURED_PEAKS.json"
        peak = json.loads(peak_path.read_text())["bf16_tflops"] if peak_path.is_file() else 1590.0
        peak_source = "measured (MEASURED_PEAKS.json bf16_tflops, cuBLAS bf16 burst)"
    achieved = flops / (ms / 1000.0) / 1e12
    line = {
        "metric": "FP8 MoE-layer prefill tokens/s (config 3)", "value": tokens * world / (ms / 1000.0),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": dtype, "data": "synthetic (seeded random-init weights, hidden rows, Zipf(1.1) routes)",
        "config": {"workload": (f"config3: prefill {tokens} tokens through one FP8 MoE layer (hidden {HIDDEN}, "
                                f"{EXPERTS} experts, top-{TOP_K}, intermediate {INTER}), Zipf(1.1) routing"),
                   "contract": args.contract, "tokens": tokens, "hidden": HIDDEN, "experts": EXPERTS,
                   "top_k": TOP_K, "intermediate": INTER,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2: 604 MB bank, 268 MB of fp32 per-pair down rows"},
        "roofline": {"kernel": kernel, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_source, "traffic": None,
                     "algorithmic_flops_per_launch": flops},
        "e2e": {"value": tokens * world / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2},
        "gpu_launches": args.steps * launches,
        "clocks": clocks.summary(),
    }
    if world > 1:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


# ---------------------------------------------------------------------------
# config 4: expert-parallel decode of 256 tokens, and the offload variant
# ---------------------------------------------------------------------------
EP_TOKENS = 256
EP_CHUNK = 16          # experts generated per seed, so every G sees the same banks


def _dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=device, timeout=timedelta(seconds=300))
    props = torch.cuda.get_device_properties(device)
    gpu_id = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(local)
    return world, rank, device, gpu_id


def _max_over_ranks(values, world, device):
    import torch
    import torch.distributed as dist

    if world == 1:
        return values
    t = torch.tensor(values, device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _ep_bank(layer: int, experts: range, device):
    """This rank's experts of one layer; expert e's bytes do not depend on the shard."""
    import torch

    from drama_b200 import synthetic

    parts = [synthetic.fp8_bank(EP_CHUNK, HIDDEN, INTER, 90_000 + layer * 100 + c // EP_CHUNK, device=device,
                                chunk=EP_CHUNK)
             for c in range(experts.start, experts.stop, EP_CHUNK)]
    return {n: torch.cat([p[n] for p in parts]) for n in parts[0]}


def _ep_bank_of(layer: int, experts: list[int], device):
    """The listed experts of one layer, in that order (same bytes as ``_ep_bank`` gives them)."""
    import torch

    chunks = sorted({e // EP_CHUNK for e in experts})
    full = {c: _ep_bank(layer, range(c * EP_CHUNK, (c + 1) * EP_CHUNK), device) for c in chunks}
    return {n: torch.stack([full[e // EP_CHUNK][n][e % EP_CHUNK] for e in experts]) for n in full[chunks[0]]}


def _ep_routes(layers: int, device):
    import torch

    from drama_b200 import synthetic

    out = []
    for l in range(layers):
        ids, w = synthetic.zipf_routes(EP_TOKENS, TOP_K, EXPERTS, 95_000 + l, device=device)
        out.append((ids.to(torch.int32).contiguous(), w.to(torch.bfloat16).contiguous()))
    return out


def run_ep(args) -> None:
    """Config 4: 256 decode tokens through 48 FP8 MoE layers, experts sharded over the ranks.

    Strong scaling: the 256 tokens and 128 experts per layer are split over
    the G ranks (tokens T/G per rank, experts E/G per rank); one step is one
    replay of a CUDA graph holding all 48 layers (dispatch, NCCL all-to-alls,
    grouped GEMMs, combine). ``value`` = 256 tokens / max-over-ranks step time.
    """
    import torch.distributed as dist

    world, rank, device, gpu_id = _dist_setup()
    line, model, graph = measure_ep(args, world, rank, device, gpu_id)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = CpuReference(_ep_bank(0, range(0, EXPERTS), device))
        ref.layer()
        cpu = ref.sample(args.cpu_seconds, args.layers)
        cpu["sample"] += "; one token per step (the workload's 256 tokens would take 256x as long)"
        line["cpu_baseline"] = cpu
    del graph
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def measure_ep(args, world: int, rank: int, device, gpu_id: str):
    """Build, capture and time the config-4 EP step on this rank; returns (line, model, graph)."""
    import torch
    import torch.distributed as dist

    from drama_b200 import synthetic
    from drama_b200.expert_parallel import (ExpertParallelMoE, balanced_placement, experts_of_rank, nccl_all_to_all,
                                            shard_tokens)

    t0 = time.perf_counter()
    rows = shard_tokens(EP_TOKENS, world, rank)

    class Bank:
        def __init__(self, d):
            self.__dict__.update(d)

    routes = _ep_routes(args.layers, device)
    # experts placed on ranks by their observed route counts (balanced rows per rank)
    placements, banks = [], []
    for l in range(args.layers):
        counts = torch.bincount(routes[l][0].reshape(-1).long(), minlength=EXPERTS).tolist()
        placement = balanced_placement(counts, world) if world > 1 else list(range(EXPERTS))
        placements.append(torch.tensor(placement, dtype=torch.int32, device=device) if world > 1 else None)
        banks.append(Bank(_ep_bank_of(l, experts_of_rank(placement, world, rank), device)))
    local_routes = [(i[rows].contiguous(), w[rows].contiguous()) for i, w in routes]
    h0 = synthetic.hidden_states(EP_TOKENS, HIDDEN, 97_000, device=device)[rows].contiguous()
    model = ExpertParallelMoE(banks, experts=EXPERTS, top_k=TOP_K, tokens=EP_TOKENS // world, ranks=world,
                              rank=rank, all_to_all=nccl_all_to_all() if world > 1 else None, placements=placements,
                              exchange=args.exchange if world > 1 else "nccl")   # one GPU: no exchange at all
    x = h0.clone()
    model.step(x, local_routes)                       # eager pass: checks, lazy init
    torch.cuda.synchronize(device)
    dropped = model.dropped()
    timed_out = model.timed_out() if model.exchange == "p2p" else False
    x.copy_(h0)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        model.step(x, local_routes)
    x.copy_(h0)
    graph.replay()                                    # one step from h0: the checksum below
    torch.cuda.synchronize(device)
    checksum = float(x.double().sum())
    checksum = _sum_over_ranks(checksum, world, device)
    build_s = time.perf_counter() - t0

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    host_in = h0.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        x.copy_(host_in, non_blocking=True)
        graph.replay()
        host_out.copy_(x, non_blocking=True)
    f1.record()
    f1.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    ms, e2e_ms = _max_over_ranks([ms, e2e_ms], world, device)

    # Algorithmic weight bytes: every expert touched on this rank, every layer.
    nbytes = synthetic.expert_nbytes_fp8(HIDDEN, INTER)
    touched = 0
    for l, (ids, _) in enumerate(routes):
        held = set(experts_of_rank(placements[l].tolist(), world, rank)) if world > 1 else set(range(EXPERTS))
        touched += len(set(torch.unique(ids.long()).tolist()) & held)
    step_bytes = touched * nbytes + 2 * (EP_TOKENS // world) * HIDDEN * 2 * args.layers
    peaks = measured_peaks()
    achieved = step_bytes / (ms / 1000.0) / 1e9
    if world == 1:
        link_bytes = 0
    elif args.exchange == "nccl":
        link_bytes = 2 * world * model.capacity * HIDDEN * 2 * args.layers
    else:   # the real rows only, each way
        link_bytes = 2 * (EP_TOKENS // world) * TOP_K * HIDDEN * 2 * args.layers
    line = {
        "metric": METRIC, "value": EP_TOKENS / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8-e4m3 weights dequantised to bf16, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and hidden rows, Zipf(1.1) routes per layer)",
        "config": {"workload": (f"config4: expert-parallel decode of {EP_TOKENS} tokens through {args.layers} FP8 "
                                f"MoE layers (hidden {HIDDEN}, {EXPERTS} experts, top-{TOP_K}, intermediate {INTER}),"
                                f" Zipf(1.1) routing, {EXPERTS // world} experts and {EP_TOKENS // world} tokens "
                                f"per GPU, " + ("no exchange" if world == 1 else "NVLink peer-memory dispatch/combine"
                                                if args.exchange == "p2p" else "NCCL all-to-all dispatch/combine")
                                + ", one CUDA graph per step"),
                   "tokens": EP_TOKENS, "layers": args.layers, "experts_per_gpu": EXPERTS // world,
                   "parallelism": f"ep{world}", "capacity_rows_per_peer": model.capacity,
                   "exchange": model.exchange if world > 1 else "none",
                   "placement": "by observed route counts (balanced rows per rank)" if world > 1 else "all local",
                   "l2": "inputs larger than L2: every step reads the touched experts of 48 layers"},
        "roofline": {"kernel": "one EP decode step on one rank (dispatch, all-to-alls, grouped GEMMs, combine)",
                     "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"],
                     "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)", "traffic": None,
                     "algorithmic_bytes_per_launch": step_bytes},
        "nvlink_bytes_per_step_per_gpu": link_bytes,
        "e2e": {"value": EP_TOKENS / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": h0.numel() * 2 * world, "d2h_bytes_per_step": h0.numel() * 2 * world},
        "gpu_launches": args.steps * args.layers * model.launches_per_layer(),
        "clocks": clocks.summary(),
        "checksum": checksum, "dropped_pairs": list(dropped), "peer_wait_timed_out": timed_out,
        "setup_s": round(build_s, 1),
    }
    return line, model, graph


def _sum_over_ranks(value: float, world: int, device) -> float:
    import torch
    import torch.distributed as dist

    if world == 1:
        return value
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return float(t.item())


def _pinned_h2d_gbs(device) -> float:
    """Pinned host -> HBM copy bandwidth of this box (1 GiB, best of 3, CUDA events)."""
    import torch

    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    best = 0.0
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        best = max(best, (1 << 30) / (a.elapsed_time(b) / 1000.0) / 1e9)
    del src, dst
    return best


def run_offload(args) -> None:
    """Config 4, offload variant: 1 GPU, 32 of 128 experts resident per layer.

    The resident 32 are each layer's most-routed experts (the ranking the
    reference's host-budget/hot-cache logic makes from observed routes); the
    other 96 live in page-locked host memory and the touched ones are staged
    through ``StagingArena`` on a copy stream every layer, one layer ahead of
    the compute. One step = 256 decode tokens through every layer.
    """
    import torch

    from drama_b200 import synthetic
    from drama_b200.backend import fp8_prefill
    from drama_b200.staging import PackedExperts, StagingArena

    world, rank, device, gpu_id = _dist_setup()
    t0 = time.perf_counter()
    resident_n = EXPERTS // 4
    # Layer l is a copy of layer l % host_layers (weights, routes, residency);
    # at least 3 distinct layers, so no slot set ever holds the ids its next
    # stage asks for and every layer's cold experts really cross PCIe.
    host_layers = max(3, min(args.host_layers, args.layers))
    routes = _ep_routes(host_layers, device)
    residents, stores, plans = [], [], []
    for l in range(host_layers):
        ids = routes[l][0].long()
        counts = torch.bincount(ids.reshape(-1), minlength=EXPERTS).cpu()
        order = sorted(range(EXPERTS), key=lambda e: (-int(counts[e]), e))
        hot = sorted(order[:resident_n])
        cold = sorted(order[resident_n:])
        bank = _ep_bank(l, range(0, EXPERTS), device)
        stores.append(PackedExperts.from_bank({n: t[cold].cpu() for n, t in bank.items()}, pin_memory=True))
        residents.append(PackedExperts.from_bank({n: t[hot] for n, t in bank.items()}, device=device))
        del bank
        touched = sorted(set(torch.unique(ids).tolist()) - set(hot))
        cold_pos = {e: i for i, e in enumerate(cold)}
        stage_ids = torch.tensor([cold_pos[e] for e in touched], dtype=torch.int64)
        local = {e: i for i, e in enumerate(touched)}
        local.update({e: len(touched) + i for i, e in enumerate(hot)})
        lut = torch.tensor([local.get(e, -1) for e in range(EXPERTS)], dtype=torch.int32, device=device)
        plans.append((l, stage_ids, lut[ids].contiguous(), routes[l][1], len(touched)))
    plans = [plans[l % host_layers] for l in range(args.layers)]
    arena = StagingArena(EXPERTS, buffers=2)
    h0 = synthetic.hidden_states(EP_TOKENS, HIDDEN, 97_000, device=device)
    x = h0.clone()
    build_s = time.perf_counter() - t0
    hot_slots = list(range(resident_n))

    def step(x):
        for src_layer, stage_ids, local_ids, w, n_cold in plans:
            store = stores[src_layer]
            with arena.session(store, device):
                if n_cold:
                    arena.stage(store, stage_ids)
                    bank = arena.combine_resident(n_cold, residents[src_layer], hot_slots)
                else:
                    bank = residents[src_layer].staged()
                moe = fp8_prefill(x, local_ids, w, bank, validate_ids=False)
                torch.add(x, moe, out=x)
        return x

    for _ in range(max(3, args.warmup)):
        x.copy_(h0)
        step(x)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        e0.record()
        for _ in range(args.steps):
            step(x)
        e1.record()
        e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    host_in = h0.cpu().pin_memory()
    host_out = torch.empty_like(host_in).pin_memory()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        x.copy_(host_in, non_blocking=True)
        step(x)
        host_out.copy_(x, non_blocking=True)
    f1.record()
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    ms, e2e_ms = _max_over_ranks([ms, e2e_ms], world, device)
    nbytes = synthetic.expert_nbytes_fp8(HIDDEN, INTER)
    staged_bytes = sum(p[4] for p in plans) * nbytes
    pcie = _pinned_h2d_gbs(device)
    achieved = staged_bytes / (ms / 1000.0) / 1e9
    line = {
        "metric": METRIC, "value": EP_TOKENS * world / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8-e4m3 weights dequantised to bf16, bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and hidden rows, Zipf(1.1) routes per layer)",
        "config": {"workload": (f"config4 offload: {EP_TOKENS} decode tokens through {args.layers} FP8 MoE layers "
                                f"on one GPU, {resident_n} of {EXPERTS} experts resident per layer (the most "
                                f"routed), the touched others staged from page-locked host memory each layer"),
                   "tokens": EP_TOKENS, "layers": args.layers, "resident_per_layer": resident_n,
                   "host_stores": host_layers, "parallelism": f"replicas{world}" if world > 1 else "single",
                   "staged_experts_per_step": sum(p[4] for p in plans),
                   "l2": "inputs larger than L2: ~20 GB staged per step"},
        "roofline": {"kernel": "one offload step (host->HBM staging on a copy stream + grouped GEMMs)",
                     "bound": "pcie", "achieved": achieved, "peak": pcie, "unit": "GB/s", "frac": achieved / pcie,
                     "peak_source": "measured in this run: 1 GiB pinned host -> HBM cudaMemcpyAsync, best of 3",
                     "traffic": None, "algorithmic_bytes_per_launch": staged_bytes},
        "e2e": {"value": EP_TOKENS * world / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": h0.numel() * 2, "d2h_bytes_per_step": h0.numel() * 2},
        "gpu_launches": args.steps * args.layers * 4,
        "clocks": clocks.summary(),
        "staging": {"h2d_bytes": arena.stats.h2d_bytes, "stage_calls": arena.stats.h2d_copy_calls,
                    "reuse_hits": arena.stats.expert_cache_hits},
        "setup_s": round(build_s, 1),
    }
    arena.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


# ---------------------------------------------------------------------------
# config 2: one INT4 W4A16 layer, decode batches of 1, 4 and 16 tokens
# ---------------------------------------------------------------------------
INT4_CALLS = 64      # calls per CUDA graph, each with its own uniform routes


W8A8_NAMES = {1: "INT8-ConvRot", 2: "W6A8", 3: "W4A8 codebook"}


def w8a8_expert_nbytes(mode: int, hidden: int, inter: int) -> int:
    """Bytes of one W8A8 expert: weights plus scale rows (quantized_model.py:45-68)."""
    total = 0
    for n, k in ((2 * inter, hidden), (hidden, inter)):
        cols = k if mode == 1 else k * 3 // 4 if mode == 2 else k // 2
        scale = 4 if mode == 1 else k // 16 + (8 if mode == 3 else 4)
        total += n * (cols + scale)
    return total


def _w8a8_device_bank(mode: int, device, seed: int):
    """The 128-expert W8A8 bank on the device, generated 16 experts at a time."""
    import torch

    from drama_b200 import synthetic

    parts = [synthetic.w8a8_bank(mode, 16, HIDDEN, INTER, seed + c) for c in range(0, EXPERTS, 16)]
    return {k: torch.cat([p[k] for p in parts]).to(device) for k in parts[0]}


def run_int4(args, mode: int = 0) -> None:
    """Config 2: QuantizedB200Backend(mode) on a quantized bank, batches 1/4/16.

    mode 0 is config 2 itself (asymmetric W4A16); modes 1-3 run the same
    measurement on a W8A8 bank (INT8-ConvRot, W6A8, W4A8 codebook). One step =
    one replay of a CUDA graph holding 64 expert calls, each with its own
    seeded uniform routes (so consecutive calls read different experts of a
    bank larger than L2). ``value`` is the batch-1 tokens/s; every batch is
    reported under ``by_batch`` with its algorithmic bytes (the distinct
    experts of each call) and GB/s.
    """
    import torch

    from drama_b200 import QuantizedB200Backend, QuantizedBank, synthetic

    world, rank, device, gpu_id = _dist_setup()
    if mode == 0:
        bank = synthetic.int4_bank(EXPERTS, HIDDEN, INTER, 2024 + rank, device=device, asymmetric=True)
        qb = QuantizedBank(**bank)
        nbytes = synthetic.expert_nbytes_int4(HIDDEN, INTER)
    else:
        from types import SimpleNamespace

        qb = SimpleNamespace(**_w8a8_device_bank(mode, device, 3000 + 1000 * mode + rank))
        nbytes = w8a8_expert_nbytes(mode, HIDDEN, INTER)
    backend = QuantizedB200Backend(mode, validate_ids=False)
    peaks = measured_peaks()
    results = {}
    clocks_summary = None
    for batch in (1, 4, 16):
        routes = [synthetic.uniform_routes(batch, TOP_K, EXPERTS, 300 + 100 * batch + c, device=device)
                  for c in range(INT4_CALLS)]
        routes = [(i.to(torch.int32).contiguous(), w.to(torch.bfloat16).contiguous()) for i, w in routes]
        xs = [synthetic.hidden_states(batch, HIDDEN, 900 + c, device=device) for c in range(INT4_CALLS)]
        outs = [None] * INT4_CALLS
        cap_stream = torch.cuda.Stream(device)          # the backend's workspace is per (device, stream)
        cap_stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(cap_stream):
            for c in range(INT4_CALLS):                 # eager: workspace, checks
                outs[c] = backend.forward(xs[c], routes[c][0], routes[c][1], qb)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap_stream):
            for c in range(INT4_CALLS):
                outs[c] = backend.forward(xs[c], routes[c][0], routes[c][1], qb)
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(gpu_id) as clocks:
            e0.record()
            for _ in range(args.steps):
                graph.replay()
            e1.record()
            e1.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        ms = _max_over_ranks([ms], world, device)[0]
        unique = sum(int(torch.unique(i).numel()) for i, _ in routes)
        call_bytes = unique * nbytes / INT4_CALLS + 2 * batch * HIDDEN * 2
        call_ms = ms / INT4_CALLS
        results[batch] = {"tokens_per_s": batch * INT4_CALLS * world / (ms / 1000.0), "call_us": call_ms * 1000.0,
                          "unique_experts_per_call": unique / INT4_CALLS,
                          "algorithmic_bytes_per_call": call_bytes,
                          "achieved_gbs": call_bytes / (call_ms / 1000.0) / 1e9}
        if batch == 1:
            clocks_summary = clocks.summary()
            host_x = [x.cpu().pin_memory() for x in xs]
            host_o = torch.empty(INT4_CALLS, batch, HIDDEN, dtype=torch.bfloat16).pin_memory()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record()
            for _ in range(args.steps):
                for c in range(INT4_CALLS):
                    xs[c].copy_(host_x[c], non_blocking=True)
                graph.replay()
                for c in range(INT4_CALLS):
                    host_o[c].copy_(outs[c], non_blocking=True)
            f1.record()
            f1.synchronize()
            e2e_ms = _max_over_ranks([f0.elapsed_time(f1) / args.steps], world, device)[0]
        del graph
    b1 = results[1]
    if mode == 0:
        dtype = ("int4 weights (asymmetric, group 128, bf16 scales, uint4 zero-points), exact levels on bf16 MMA, "
                 "fp32 block scales and accumulate")
        layer = "W4A16"
        # batch 1 at this shape is the one-launch layer (int4_layer.cu)
        kernel = ("one W4A16 MoE layer for one decode row in one launch (4-CTA clusters: gate/up GEMV, SwiGLU, "
                  "down GEMV, ordered combine), batch 1")
        launches = 1
    else:
        dtype = (f"{W8A8_NAMES[mode]} weights, ConvRot-rotated int8 activations, s8 MMA, int32 accumulate, "
                 "bf16 projections")
        layer = f"W8A8 mode {mode} ({W8A8_NAMES[mode]})"
        kernel = (f"one {W8A8_NAMES[mode]} expert call (grouping + token rotation, up GEMV, SwiGLU rotation, "
                  "down GEMV with the fused combine), batch 1")
        launches = 4
    line = {
        "metric": METRIC, "value": b1["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": INT4_CALLS * b1["call_us"] / 1000.0, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": dtype,
        "data": "synthetic (seeded random-init weights and hidden rows, uniform routes)",
        "config": {"workload": ((f"config2: one {layer} MoE layer" if mode == 0 else f"one {layer} MoE layer")
                                + f" (hidden {HIDDEN}, {EXPERTS} experts, top-{TOP_K}, "
                                f"intermediate {INTER}), decode batches 1/4/16 (value: batch 1), "
                                f"{INT4_CALLS} calls per CUDA graph with distinct uniform routes"),
                   "batches": [1, 4, 16], "calls_per_graph": INT4_CALLS,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": f"bank of {EXPERTS * nbytes / 1e6:.0f} MB (> L2), routes differ call to call"},
        "roofline": {"kernel": kernel, "bound": "hbm",
                     "achieved": b1["achieved_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": b1["achieved_gbs"] / peaks["hbm_gbs"],
                     "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": committed_traffic("int4_layer_traffic.json") if mode == 0 else None,
                     "algorithmic_bytes_per_launch": b1["algorithmic_bytes_per_call"]},
        "by_batch": results,
        "e2e": {"value": INT4_CALLS * world / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": INT4_CALLS * HIDDEN * 2, "d2h_bytes_per_step": INT4_CALLS * HIDDEN * 2},
        "gpu_launches": args.steps * INT4_CALLS * launches,
        "clocks": clocks_summary,
    }
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def run_shared(args) -> None:
    """Shared expert + sigmoid gate fused with the routed sum and the residual
    (``_shared_impl`` + ``_post_impl``, backbone_graph.py:327-337), batches 1/4/16.

    One step = one replay of a CUDA graph holding one call per layer of a
    48-layer stack of distinct bf16 shared experts (48 x 3 x H x I x 2 bytes,
    larger than L2). ``value`` is the batch-1 tokens/s of the 48-layer pass.
    """
    import torch

    from drama_b200 import synthetic
    from drama_b200.shared import SharedExpertB200

    world, rank, device, gpu_id = _dist_setup()
    inter, layers = args.shared_inter, args.layers
    gen = torch.Generator(device=device)
    gen.manual_seed(4000 + rank)

    def w(*shape):
        return (torch.randn(*shape, generator=gen, device=device) * 0.03).to(torch.bfloat16)

    mods = [SharedExpertB200(w(inter, HIDDEN), w(inter, HIDDEN), w(HIDDEN, inter), w(1, HIDDEN))
            for _ in range(layers)]
    layer_bytes = 3 * HIDDEN * inter * 2 + HIDDEN * 2
    one_launch = HIDDEN == 2048 and inter == 768  # batch 1 at this shape is one launch (shared_layer.cu)
    peaks = measured_peaks()
    results = {}
    clocks_summary = e2e_ms = None
    for batch in (1, 4, 16):
        x = synthetic.hidden_states(batch, HIDDEN, 50 + batch, device=device)
        routed = synthetic.hidden_states(batch, HIDDEN, 60 + batch, device=device) * 0.1
        hid = [synthetic.hidden_states(batch, HIDDEN, 70 + batch, device=device)]
        cap = torch.cuda.Stream(device)
        cap.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(cap):
            h = hid[0]
            for m in mods:
                h = m.post(h, routed, x)
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            h = hid[0]
            for m in mods:
                h = m.post(h, routed, x)
            final = h
        for _ in range(max(3, args.warmup)):
            graph.replay()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(gpu_id) as clocks:
            e0.record()
            for _ in range(args.steps):
                graph.replay()
            e1.record()
            e1.synchronize()
        ms = _max_over_ranks([e0.elapsed_time(e1) / args.steps], world, device)[0]
        call_us = ms * 1000.0 / layers
        step_bytes = layers * (layer_bytes + 4 * batch * HIDDEN * 2)
        results[batch] = {"tokens_per_s": batch * world / (ms / 1000.0), "layer_us": call_us,
                          "algorithmic_bytes_per_layer": layer_bytes + 4 * batch * HIDDEN * 2,
                          "achieved_gbs": step_bytes / (ms / 1000.0) / 1e9}
        if batch == 1:
            clocks_summary = clocks.summary()
            host_in = hid[0].cpu().pin_memory()
            host_out = torch.empty_like(host_in).pin_memory()
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            f0.record()
            for _ in range(args.steps):
                hid[0].copy_(host_in, non_blocking=True)
                graph.replay()
                host_out.copy_(final, non_blocking=True)
            f1.record()
            f1.synchronize()
            e2e_ms = _max_over_ranks([f0.elapsed_time(f1) / args.steps], world, device)[0]
        del graph
    b1 = results[1]
    line = {
        "metric": METRIC, "value": b1["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": layers * b1["layer_us"] / 1000.0, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 weights and activations, bf16 MMA, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and hidden rows)",
        "config": {"workload": (f"shared expert + gate fused with the routed sum and residual, {layers} layers "
                                f"(hidden {HIDDEN}, shared intermediate {inter} assumed), batches 1/4/16 "
                                "(value: batch 1), one CUDA graph per batch"),
                   "batches": [1, 4, 16], "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": f"{layers} distinct experts, {layers * layer_bytes / 1e6:.0f} MB (> L2)"},
        "roofline": {"kernel": ("one layer's shared expert in one launch (4-CTA clusters: gate/up rows, SwiGLU, "
                                "down rows, ordered sum with the gate, routed sum and residual), batch 1"
                                if one_launch else
                                "one layer's shared expert (gate/up GEMV, SwiGLU, down GEMV + fused sum), batch 1"),
                     "bound": "hbm", "achieved": b1["achieved_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": b1["achieved_gbs"] / peaks["hbm_gbs"],
                     "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": committed_traffic("shared_layer_traffic.json") if one_launch else None,
                     "algorithmic_bytes_per_launch": b1["algorithmic_bytes_per_layer"]},
        "by_batch": results,
        "e2e": {"value": world / (e2e_ms / 1000.0), "unit": "tokens/s",
                "h2d_bytes_per_step": HIDDEN * 2, "d2h_bytes_per_step": HIDDEN * 2},
        "gpu_launches": args.steps * layers * (1 if one_launch else 2),
        "clocks": clocks_summary,
    }
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line))


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "ep":
        run_ep(args)
    elif args.workload == "offload":
        run_offload(args)
    elif args.workload == "int4":
        run_int4(args)
    elif args.workload == "w8a8":
        run_int4(args, mode=args.mode)
    elif args.workload == "shared":
        run_shared(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

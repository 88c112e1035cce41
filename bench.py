"""Benchmark: batch-1 SmolLM2-135M FP32 decode at context 8192 on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flux_b200|reference]

Workload (the benchmark's configs[1]): SmolLM2-135M geometry with seeded
N(0, 0.02) weights, a seeded uniform-random 8192-token prompt prefilled into
the compact cache by the native prefill, then W warm-up and K timed greedy
decode steps replayed from the CUDA graph (context 8192+W -> 8192+W+K).  One
step = one token.  ``value`` is ms/token (lower is better), timed with CUDA
events on the launching stream between barriers, max over ranks.  Every step
streams ~0.92 GB (> the 126 MB L2), so no L2 flush is needed.

Under torchrun with N > 1 every rank runs an independent replica (the batch-1
path does not shard; no collective is on the data path): the job decodes N
tokens per step, so ``value`` is the max-over-ranks step time divided by N
(ms per token of the whole job; ``config.per_replica_ms_per_token`` keeps the
per-GPU figure).

The line also carries ``sweep`` (configs[2]: the batch-1 step after a
native prefill at each context 128 ... 8192, N = 1), ``batched`` (configs[3]: 64 ragged sequences per GPU,
greedy steps through the batched runtime, sequences sharded by rank with no
collective; aggregate tokens/s over all ranks, max-over-ranks time) and, at
N = 1, ``attention`` (configs[4]: the isolated decode attention GB/s over
B in {1, 16, 64, 256} x L in {128, 1024, 8192}, L2 flushed per launch).

``--impl reference`` times the reference's own FP32 CPU path (transformers
``LlamaForCausalLM`` eager, as ``benchmarks/benchmark_flux.py:533-564`` drives
it) on the host cores for the same config, rank 0 only.
"""

from __future__ import annotations

import argparse
import copy
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

WEIGHT_BYTES = 538_062_336      # FP32 weights streamed per step (incl. the 113 MB tied LM head)
KV_BYTES_PER_ROW = 46_080       # 30 layers x (K + V) x 3 heads x 64 x 4 B
METRIC = "bs1 decode ms/token @ctx8192"
FALLBACK_HBM_GBS = 6650.0


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=("flux_b200", "reference"), default="flux_b200")
    p.add_argument("--context", type=int, default=8192)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--batched-steps", type=int, default=256, help="greedy steps of the batched configuration")
    p.add_argument("--batch", type=int, default=64, help="sequences per GPU of the batched configuration")
    p.add_argument("--no-batched", action="store_true", help="skip the batched configuration")
    p.add_argument("--no-attention", action="store_true", help="skip the isolated-attention sweep")
    p.add_argument("--no-sweep", action="store_true", help="skip the context sweep of the batch-1 decode")
    p.add_argument("--no-generation", action="store_true",
                   help="skip configs[0] (128-token prompt, 128 greedy tokens end to end)")
    return p.parse_args(argv)


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except ValueError:
            pass
    return {}


def measured_traffic(bytes_per_step: float) -> dict | None:
    """DRAM bytes per step-kernel launch from the committed ncu capture of
    this workload (profiles/decode_step_traffic.json), scaled from the
    captured step's algorithmic bytes to the timed steps' (traffic grows with
    the K/V rows read)."""
    path = ROOT / "profiles" / "decode_step_traffic.json"
    try:
        rec = json.loads(path.read_text())
    except (OSError, ValueError):
        return None
    captured = rec["dram_read_bytes"] + rec["dram_write_bytes"]
    scaled = captured * bytes_per_step / rec["algorithmic_bytes"]
    return {"bytes_per_launch": int(scaled), "ratio_to_algorithmic": round(captured / rec["algorithmic_bytes"], 4),
            "captured_context_rows": rec["context_rows"], "source": rec["source"]}


# ----------------------------------------------------------- clock sampling


_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
            0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """Reads (never sets) the SM clock and clock-event reasons through NVML
    every ``interval`` seconds while the timed region runs."""

    def __init__(self, device_index: int, interval: float = 0.001):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._interval = interval
        self._handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            try:
                self._handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self._handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML missing: report no clocks rather than fail the bench
            self._handle = None

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((mhz, reasons))
            except Exception:
                return
            time.sleep(self._interval)

    def __enter__(self):
        if self._handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._handle is not None:
            self._stop.set()
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mask = 0
        for _, r in self.samples:
            mask |= r
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": [name for bit, name in _REASONS.items() if mask & bit and bit != 0x1],
                "samples": len(self.samples)}


# ----------------------------------------------------------------- workload


def build_models(context: int, steps_total: int, seed: int):
    from tests.golden.inputs import build_model, smollm2_config
    config = smollm2_config(vocab_size=49152, max_positions=max(8320, context + steps_total + 1))
    return config, build_model(config, seed)


def run_native(args) -> dict | None:
    import torch.distributed as dist

    from tests.host import limit_threads, usable_cpus
    world, rank, local = dist_info()
    limit_threads(max(1, usable_cpus() // world))  # one process per GPU share the host cores

    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    from flux_b200.runtime import NativeSmolLM2Prefill
    from tests.golden.inputs import uniform_prompt

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    K, W, ctx = args.steps, args.warmup, args.context
    e2e_steps = K
    decode_steps = W + K + 2 * (W + e2e_steps)  # device-timed, then the two end-to-end legs
    config, cpu_model = build_models(ctx, decode_steps, args.seed)
    model = enable_flux_ops(copy.deepcopy(cpu_model).to(device), operators=FINAL_FLUX_OPERATOR_CATEGORIES)
    prompt = uniform_prompt(ctx, seed=args.seed + rank).to(device)
    with torch.inference_mode():
        runtime = NativeSmolLM2Prefill.capture(model, prompt, max_decode_steps=decode_steps)
        torch.cuda.synchronize()
        # prefill time of the same prompt (the native prefill re-run; not part of ms/token)
        p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p_start.record()
        runtime.prefill(prompt)
        p_end.record()
        torch.cuda.synchronize()
        prefill_ms = p_start.elapsed_time(p_end)
        native = runtime.native_object()
        stream = torch.cuda.current_stream(device)

        # ---- device-timed region: K graph replays, device-resident greedy loop
        for _ in range(W):
            runtime.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            start.record(stream)
            for _ in range(K):
                runtime.replay()
            end.record(stream)
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        elapsed_ms = start.elapsed_time(end)

        # ---- end-to-end, host buffers: the token goes in from host memory and the
        # sampled token comes back to host memory every step.  (1) the C-ABI
        # host-buffer step (fx_decode_replay_host through replay_host); (2) the
        # tensor API: pinned host tensor -> device tensor -> replay(token) ->
        # pinned host tensor.
        def timed_loop(step) -> float:
            for _ in range(W):
                step()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e_start.record(stream)
            for _ in range(e2e_steps):
                step()
            e_end.record(stream)
            torch.cuda.synchronize()
            return e_start.elapsed_time(e_end)

        host_token = [int(runtime.current_token.item())]

        def host_step():
            host_token[0] = runtime.replay_host(host_token[0])

        e2e_ms = timed_loop(host_step)

        host_in = torch.empty((1, 1), dtype=torch.int64, pin_memory=True)
        host_out = torch.empty((1, 1), dtype=torch.int64, pin_memory=True)
        dev_in = torch.empty((1, 1), dtype=torch.int64, device=device)
        host_in.copy_(runtime.current_token.cpu())
        ready = torch.cuda.Event()

        def tensor_step():
            dev_in.copy_(host_in, non_blocking=True)
            runtime.replay(dev_in)
            host_out.copy_(runtime.current_token, non_blocking=True)
            ready.record(stream)
            ready.synchronize()
            host_in.copy_(host_out)

        e2e_tensor_ms = timed_loop(tensor_step)
        kernels_per_step = native._decode.kernels_per_step()

    times = torch.tensor([elapsed_ms, e2e_ms, e2e_tensor_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms, e2e_tensor_ms = times.tolist()
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or FALLBACK_HBM_GBS
    del runtime, native
    torch.cuda.empty_cache()
    batched = None
    if not args.no_batched:
        with torch.inference_mode():
            batched = run_batched(args, model, device, world, rank, peak, peak_src)
        torch.cuda.empty_cache()
    if rank != 0:
        return None

    ms_per_step = elapsed_ms / K
    # Algorithmic bytes: weights + K/V rows read (position + 1 each step) + the row written.
    first_len = ctx + W + 1
    mean_len = first_len + (K - 1) / 2.0
    bytes_per_step = WEIGHT_BYTES + KV_BYTES_PER_ROW * mean_len + KV_BYTES_PER_ROW
    achieved = bytes_per_step / (ms_per_step * 1e-3) / 1e9
    # Whole-job aggregate: with N replicas (one sequence per GPU, no collective)
    # the job decodes N tokens per step time, so ms per token of the job is the
    # max-over-ranks step time over N (at N = 1, the step time itself).
    aggregate_ms = ms_per_step / world
    line = {
        "metric": METRIC,
        "value": round(aggregate_ms, 5),
        "unit": "ms/token",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights, seeded uniform prompt)",
        "config": {
            "workload": "configs[1]: bs1 greedy decode after an 8192-token native prefill",
            "model": "SmolLM2-135M architecture (30x576, 9/3 heads, vocab 49152, tied)",
            "context_start": ctx + W, "context_end": ctx + W + K,
            "tokens_per_s_per_gpu": round(1e3 / ms_per_step, 1),
            "tokens_per_s_aggregate": round(world * 1e3 / ms_per_step, 1),
            "per_replica_ms_per_token": round(ms_per_step, 5),
            "prefill_ms": round(prefill_ms, 2),
            "parallelism": "replicas" if world > 1 else "single",
            "l2": "inputs larger than L2 (~0.92 GB streamed per step)",
        },
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "traffic": (measured_traffic(bytes_per_step) or {}).get("bytes_per_launch"),
            "traffic_source": measured_traffic(bytes_per_step),
            "kernel": "decode step (one CUDA graph replay)",
            "algorithmic_bytes_per_launch": int(bytes_per_step), "peak_source": peak_src,
        },
        "e2e": {"value": round(e2e_ms / e2e_steps / world, 5), "unit": "ms/token", "h2d_bytes_per_step": 8 * world,
                "d2h_bytes_per_step": 8 * world, "per_replica_ms_per_token": round(e2e_ms / e2e_steps, 5),
                "api": "NativeSmolLM2Prefill.replay_host(token) -> next token (C-ABI fx_decode_replay_host: host "
                       "token in, one replay, sampled token back in host memory, every step)",
                "tensor_api_value": round(e2e_tensor_ms / e2e_steps, 5),
                "tensor_api": "NativeSmolLM2Prefill.replay(token) with a pinned host token copied in and the next "
                              "token read back through torch copies"},
        "gpu_launches": int(kernels_per_step * K),
        "clocks": clocks.summary(),
    }
    if batched is not None:
        line["batched"] = batched
    if world == 1 and not args.no_attention:
        line["attention"] = run_attention_sweep(device, peak)
    if world == 1 and not args.no_sweep:
        line["sweep"] = run_context_sweep(model, device, args.seed, peak)
    if world == 1 and not args.no_generation:
        line["generation"] = run_generation(model, device, args.seed)
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cpu_model, config, ctx, sweep=not args.no_sweep,
                                            generation=line.get("generation"), seed=args.seed)
    return line


BATCH_CONTEXT = (512, 4096)     # ragged contexts drawn uniformly (seeded)


def run_batched(args, model, device, world: int, rank: int, peak: float, peak_src: str) -> dict | None:
    """64 independent sequences per GPU, ragged contexts ~U[512, 4096]
    (seeded per rank), greedy steps through ``NativeSmolLM2BatchedDecode``;
    sequences are sharded by rank with no collective on the data path.  Caches
    are seeded N(0, 0.5) rows (no prefill; the step does not depend on how the
    rows were produced)."""
    import torch.distributed as dist
    from flux_b200 import sharding
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    steps, warm = args.batched_steps, max(3, args.warmup)
    batch = args.batch
    shard = sharding.sequence_shard(world * batch, world, rank)
    lengths, tokens = sharding.shard_contexts(args.seed, shard, *BATCH_CONTEXT)
    capacity = BATCH_CONTEXT[1] + warm + steps + 1
    runtime = NativeSmolLM2BatchedDecode(model, batch, capacity)
    dgen = torch.Generator(device=device)
    for i, n in enumerate(lengths):
        dgen.manual_seed(args.seed * 1_000_003 + 29 + shard[i])  # cache rows depend on the global sequence only
        keys = torch.randn(30, 3, n, 64, device=device, generator=dgen) * 0.5
        values = torch.randn(30, 3, n, 64, device=device, generator=dgen) * 0.5
        runtime.load(i, tokens[i], list(keys), list(values), n)
        runtime.check()
        del keys, values
    stream = torch.cuda.current_stream(device)
    runtime.step(warm)
    runtime.check()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    runtime.step(steps)
    end.record(stream)
    torch.cuda.synchronize()
    runtime.check()
    if world > 1:
        dist.barrier()
    ms = sharding.max_over_ranks([start.elapsed_time(end)], device)[0]
    if rank != 0:
        return None
    ms_per_step = ms / steps
    mean_rows = sum(lengths) / batch + warm + (steps - 1) / 2.0 + 1
    bytes_per_step = WEIGHT_BYTES + KV_BYTES_PER_ROW * batch * mean_rows
    achieved = bytes_per_step / (ms_per_step * 1e-3) / 1e9
    return {
        "metric": f"batched decode tokens/s ({batch} sequences per GPU)",
        "value": round(sharding.aggregate_tokens_per_s(batch * steps, world, ms), 1),
        "unit": "tokens/s", "higher_is_better": True, "n_gpus": world, "scaling": "weak", "steps": steps,
        "warmup": warm, "ms_per_step": round(ms_per_step, 4),
        "tokens_per_s_per_gpu": round(batch * steps / (ms * 1e-3), 1),
        "config": {"workload": f"configs[3]: {batch} independent sequences per GPU, ragged contexts ~U[512,4096] "
                               "(seeded per global sequence), greedy steps, contiguous sequence blocks per rank, "
                               "no collective",
                   "contexts_rank0": {"min": min(lengths), "max": max(lengths), "mean": round(sum(lengths) / batch, 1)},
                   "data": "seeded N(0,0.5) cache rows, seeded uniform tokens"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "algorithmic_bytes_per_step": int(bytes_per_step),
                     "peak_source": peak_src},
        "gpu_launches": int(runtime.kernels_per_step * steps),
    }


SWEEP_CONTEXTS = (128, 512, 1024, 2048, 4096, 8192)


def run_context_sweep(model, device, seed: int, peak: float, steps: int = 32, warm: int = 4) -> dict:
    """the batch-1 decode step after a native prefill of a seeded
    prompt of each context length; ms/token over ``steps`` graph replays and
    the fraction of the HBM roofline of those steps' algorithmic bytes."""
    from flux_b200.runtime import NativeSmolLM2Prefill
    from tests.golden.inputs import uniform_prompt
    rows = []
    for ctx in SWEEP_CONTEXTS:
        prompt = uniform_prompt(ctx, seed=seed + ctx).to(device)
        with torch.inference_mode():
            runtime = NativeSmolLM2Prefill.capture(model, prompt, max_decode_steps=warm + steps + 1)
            for _ in range(warm):
                runtime.replay()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(steps):
                runtime.replay()
            e.record()
            torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
        mean_len = ctx + warm + 1 + (steps - 1) / 2.0
        nbytes = WEIGHT_BYTES + KV_BYTES_PER_ROW * (mean_len + 1)
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"context": ctx, "ms_per_token": round(ms, 4), "GBps": round(gbs, 1), "frac": round(gbs / peak, 4)})
        del runtime
        torch.cuda.empty_cache()
    return {"metric": "bs1 decode ms/token by context (configs[2])", "unit": "ms/token", "steps": steps,
            "warmup": warm, "rows": rows}


def run_attention_sweep(device, peak: float) -> dict:
    """the compact decode attention alone through the C ABI,
    Q/K/V ~ N(0, 1) seeded, B x L grid, L2 flushed before every launch (a
    256 MB write in the same graph); 20 graph replays per timing, minus the
    same replays of the flush alone, so host submission is not timed and the
    event clock's ~2 us tick does not quantise small launches."""
    from flux_b200 import _native
    lib = _native.load()
    flush = torch.empty(64 * 1024 * 1024, device=device)  # 256 MB > L2
    stream = torch.cuda.Stream(device)
    rows = []
    for batch in (1, 16, 64, 256):
        for length in (128, 1024, 8192):
            g = torch.Generator(device=device).manual_seed(batch * 7 + length)
            q = torch.randn(batch, 9, 1, 64, device=device, generator=g)
            k = torch.randn(batch, 3, length, 64, device=device, generator=g)
            v = torch.randn(batch, 3, length, 64, device=device, generator=g)
            ln = torch.tensor(length, device=device)
            out = torch.empty(batch, 9, 1, 64, device=device)
            # partials + zeroed merge counters: the merge runs in the chunk kernel (one launch)
            floats = lib.fx_gqa_decode_attention_workspace_floats(batch, 9, length, 64) + batch * 3
            ws = torch.zeros(floats, device=device)
            args = (q.data_ptr(), _native.int64_array(q.stride()), k.data_ptr(), _native.int64_array(k.stride()),
                    v.data_ptr(), _native.int64_array(v.stride()), None, None, None, ln.data_ptr(), out.data_ptr(),
                    ws.data_ptr(), floats, 0.125, batch, 9, 3, length, 64)
            with torch.cuda.stream(stream):
                _native.check(lib.fx_gqa_decode_attention_f32(*args, stream.cuda_stream))  # loads the kernels
                stream.synchronize()
                # graph A: L2 flush + attention; graph B: the flush alone.  Each is
                # replayed `reps` times between two events (the event clock ticks
                # ~2 us on this GPU); attention time = (A - B) / reps.
                with_attention, flush_only = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                with torch.cuda.graph(with_attention, stream=stream):
                    flush.fill_(1.0)
                    _native.check(lib.fx_gqa_decode_attention_f32(*args, stream.cuda_stream))
                with torch.cuda.graph(flush_only, stream=stream):
                    flush.fill_(2.0)
                reps = 20

                def timed(graph):
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record(stream)
                    for _ in range(reps):
                        graph.replay()
                    e.record(stream)
                    stream.synchronize()
                    return s.elapsed_time(e) / reps

                times = []
                for it in range(5):
                    ta, tb = timed(with_attention), timed(flush_only)
                    if it >= 1:
                        times.append(ta - tb)
            t = statistics.median(times) * 1e-3
            nbytes = batch * (1536 * length + 4608)
            rows.append({"B": batch, "L": length, "us": round(t * 1e6, 2), "GBps": round(nbytes / t / 1e9, 1),
                         "frac": round(nbytes / t / 1e9 / peak, 3)})
            del with_attention, flush_only, q, k, v, out, ws
    return {"metric": "isolated decode attention GB/s (configs[4])", "unit": "GB/s", "peak": peak,
            "algorithmic_bytes": "B*(1536*L + 4608)", "l2": "flushed (256 MB write) before every launch",
            "timing": "20 graph replays of (flush + attention) minus 20 of the flush alone, median of 4",
            "rows": rows}


GENERATION_PROMPT, GENERATION_TOKENS = 128, 128   # configs[0]


def run_generation(model, device, seed: int, rounds: int = 5) -> dict:
    """a seeded 128-token prompt, then 128 greedy tokens, on the
    GPU.  Two timings, median of ``rounds``: the reference's generation number
    (native prefill + ``generate_greedy``, runtime set-up excluded,
    ``benchmarks/benchmark_flux.py:685-702``), and the whole public call
    ``native_smollm2_greedy_generate`` with the prompt copied from pinned host
    memory and the tokens read back (set-up included)."""
    from flux_b200.runtime import NativeSmolLM2Prefill, native_smollm2_greedy_generate
    from tests.golden.inputs import uniform_prompt
    prompt_host = uniform_prompt(GENERATION_PROMPT, seed=seed + 1).pin_memory()
    prompt = prompt_host.to(device)
    reference_ms, prefill_ms, e2e_ms = [], [], []
    with torch.inference_mode():
        for _ in range(rounds):
            runtime = NativeSmolLM2Prefill.capture(model, prompt, max_decode_steps=GENERATION_TOKENS - 1)
            torch.cuda.synchronize()
            s, m, e = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            s.record()
            runtime.prefill(prompt)
            m.record()
            tokens = runtime.generate_greedy(GENERATION_TOKENS)
            e.record()
            e.synchronize()
            prefill_ms.append(s.elapsed_time(m))
            reference_ms.append(s.elapsed_time(e))
            del runtime
            t0 = time.perf_counter()
            out = native_smollm2_greedy_generate(model, prompt_host.to(device, non_blocking=True),
                                                 max_new_tokens=GENERATION_TOKENS).cpu()
            e2e_ms.append((time.perf_counter() - t0) * 1e3)
    return {"metric": "configs[0] greedy generation ms (128-token prompt, 128 new tokens, incl. native prefill)",
            "unit": "ms", "value": round(statistics.median(reference_ms), 3),
            "prefill_ms": round(statistics.median(prefill_ms), 3),
            "ms_per_token": round(statistics.median(reference_ms) / GENERATION_TOKENS, 4),
            "e2e_ms": round(statistics.median(e2e_ms), 3),
            "e2e": "native_smollm2_greedy_generate(prompt from pinned host memory) -> tokens on the host, "
                   "runtime set-up (weights, graph capture) included",
            "rounds": rounds, "tokens": [int(t) for t in tokens.reshape(-1).tolist()[:8]],
            "h2d_bytes": GENERATION_PROMPT * 8, "d2h_bytes": (GENERATION_PROMPT + GENERATION_TOKENS) * 8}


CPU_SWEEP_STEPS = 16


def cpu_baseline(cpu_model, config, ctx: int, budget_s: float = 15.0, sweep: bool = True,
                 generation: dict | None = None, seed: int = 0) -> dict:
    """The reference's FP32 path (transformers eager) on the host cores: decode
    at the benchmark context (the headline sample), at every sweep context
    (median of up to 16 steps each) and, with the GPU's configs[0] result
    beside it, the 128 + 128 greedy generation."""
    from oracle import hf_reference as hf
    from oracle.host import cpu_model_name, usable_cpus
    from tests.golden.inputs import uniform_prompt
    threads = usable_cpus()
    result = hf.time_cpu_decode(cpu_model, config, ctx, steps=64, threads=threads, budget_s=budget_s)
    line = {"value": round(result["ms_per_token"], 3), "unit": "ms/token", "cores": threads, "kind": "reference",
            "cpu": cpu_model_name(),
            "sample": (f"transformers LlamaForCausalLM eager FP32 decode (the reference's CPU path), "
                       f"{result['steps']} greedy steps over a {ctx}-row seeded synthetic cache, median")}
    if sweep:
        rows = []
        for context in SWEEP_CONTEXTS:
            r = hf.time_cpu_decode(cpu_model, config, context, steps=CPU_SWEEP_STEPS, threads=threads, budget_s=4.0)
            rows.append({"context": context, "ms_per_token": round(r["ms_per_token"], 3), "steps": r["steps"]})
        line["sweep"] = rows
    if generation is not None:
        g = hf.time_cpu_generation(cpu_model, uniform_prompt(GENERATION_PROMPT, seed=seed + 1), GENERATION_TOKENS,
                                   threads=threads)
        line["generation"] = {"total_ms": round(g["total_ms"], 1), "prefill_ms": round(g["prefill_ms"], 1),
                              "decode_ms": round(g["decode_ms"], 1),
                              "sample": "configs[0]: transformers eager prefill of the same 128-token prompt, "
                                        "then 127 greedy steps (128 tokens), wall clock",
                              "tokens_match_gpu": g["tokens"][:8] == generation.get("tokens")}
    return line


def run_reference(args) -> dict | None:
    """The reference's FP32 CPU path, timed on the host cores (rank 0 only)."""
    world, rank, _ = dist_info()
    if rank != 0:
        return None
    from oracle import hf_reference as hf
    from oracle.host import limit_threads
    threads = limit_threads()
    K, W, ctx = args.steps, args.warmup, args.context
    config, cpu_model = build_models(ctx, W + K, args.seed)
    keys, values = hf.synthetic_cache(config, ctx, seed=args.seed)
    cache = hf.dynamic_cache(config, keys, values)
    token = 17
    for _ in range(W):
        token = int(torch.argmax(hf.decode_step(cpu_model, token, cache)))
    start = time.perf_counter()
    for _ in range(K):
        token = int(torch.argmax(hf.decode_step(cpu_model, token, cache)))
    ms = (time.perf_counter() - start) * 1e3 / K
    return {
        "impl": "reference", "metric": METRIC, "value": round(ms, 4), "unit": "ms/token", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(ms, 4), "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,0.02) weights, seeded synthetic cache)",
        "config": {"workload": "configs[1]: bs1 greedy decode at context 8192 (synthetic cache rows)",
                   "model": "SmolLM2-135M architecture (30x576, 9/3 heads, vocab 49152, tied)",
                   "context_start": ctx + W, "context_end": ctx + W + K},
        "cpu_baseline": {"value": round(ms, 4), "unit": "ms/token", "cores": threads, "kind": "reference",
                         "sample": f"transformers eager FP32 decode, {K} timed steps after {W} warm-up"},
        "e2e": {"value": round(ms, 4), "unit": "ms/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv=None) -> int:
    args = parse_args(argv)
    world, rank, local = dist_info()
    if args.impl == "reference":
        line = run_reference(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    try:
        line = run_native(args)
    finally:
        if world > 1:
            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

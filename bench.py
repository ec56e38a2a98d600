"""Headline benchmark: output tok/s at concurrency 64 (with p50 TTFT and ITL) for the GPT-OSS-120B shape,
TP=EP=N on N GPUs of one node, random-init MXFP4 experts, FP8 KV cache, bf16 elsewhere.

    python bench.py --gpus 1 --steps 200 --warmup 5
    torchrun --nproc-per-node 8 bench.py --gpus 8 ...

Workload: requests of 1024 input / 1024 output tokens (token ids uniform from a seed),
64 in flight. The engine is brought to the steady state of that closed loop before timing: the 64 initial
requests carry staggered progress (request i holds 1024 + 16*i context tokens and 1024 - 16*i outputs
remain), and whenever one finishes a fresh 1024/1024 request takes its place, so the timed steps mix
decode rows with the prefill chunks of arriving requests at the rate the trace implies.

A "step" is one scheduler iteration (one forward over the running batch). K steps are timed with CUDA
events on the compute stream between two synchronizes (max over ranks); the inputs of every step (token
ids, positions, slots, block-table updates, sampling params) are copied host->device from pinned memory and
every step's sampled tokens are read back device->host, inside the timed region.
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

METRIC = "output tok/s at concurrency 64; p50 TTFT & ITL (GPT-OSS-120B-shape TP8 EP8)"
BASELINE_VALUE = None  # no published reference number exists for this metric
OUT_DIR = os.environ.get("SNB_BENCH_OUT", os.path.join(ROOT, "bench_out"))  # clock samples, profiler tables


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--baseline", default="", choices=["", "nccl"],
                   help="nccl: this engine with cuBLAS dense GEMMs and NCCL collectives (no fused kernels), the "
                        "comparison build the repository's baseline tables quote")
    p.add_argument("--model", default="gpt-oss-120b")
    p.add_argument("--concurrency", type=int, default=64)
    p.add_argument("--input-len", type=int, default=1024)
    p.add_argument("--output-len", type=int, default=1024)
    p.add_argument("--stagger", type=int, default=0, help="context stagger between slots (0: output_len / concurrency, at most 16)")
    p.add_argument("--kv", default="", help="KV cache dtype (default: fp8_e4m3 for GPT-OSS, the model's default otherwise)")
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--chunked-prefill", type=int, default=4096)
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    return p.parse_args()


def reference_arm(a):
    """The reference (sgl-project/sglang-neuron) is a Trainium plugin: it needs torch_neuronx, neuronx-cc,
    NKI and libnrt, and SGLang itself; none exist for B200, so its serving path cannot run here."""
    reason = None
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    try:
        import sglang_neuron  # noqa: F401
        if sglang_neuron.activate() is None:
            reason = ("reference installed (baseline/_ref) but its platform entry point returns None: it requires "
                      "torch_neuronx/neuronx-cc/libnrt (AWS Trainium) and SGLang, which have no B200 build")
    except Exception as e:  # not installed
        reason = f"reference not importable ({type(e).__name__}); it targets AWS Trainium (torch_neuronx) only"
    if reason is None:
        reason = "reference has no CUDA serving path"
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


class ClockSampler:
    def __init__(self, index: int):
        self.proc = None
        self.path = os.path.join(OUT_DIR, f"clocks_rank{index}.csv")
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def _profile_steps(eng, sched, refill, rank, n, dev, mode_filter=None):
    """Profile steps under torch.profiler (CUPTI kernel activity, graph-replayed kernels included): n
    consecutive steps, or with mode_filter ("mixed" or "decode") the next single step of that kind. Writes
    the per-kernel device-time table of this rank to <SNB_BENCH_OUT>/torchprof_rank<r>[_<mode>].txt.
    Eagerly launched kernels run without programmatic dependent launch here: with it, a kernel is timed from
    the moment it becomes resident while its predecessor still runs, so durations would overlap."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from sglang_neuron_b200._ext import kernels
    kernels().set_pdl(False)

    from sglang_neuron_b200.model_executor.forward_batch import ForwardMode
    torch.cuda.synchronize(dev)
    p = profile(activities=[ProfilerActivity.CUDA])
    taken, started = 0, False
    for _ in range(max(n, 1) * 64):
        if taken >= (1 if mode_filter else n):
            break
        refill()
        sched._sync_arrivals()
        step = sched.schedule()
        if step is None:
            continue
        kind = "decode" if step.mode == ForwardMode.DECODE else "mixed"
        hit = mode_filter is None or kind == mode_filter
        if hit and not started:
            sched.drain()
            torch.cuda.synchronize(dev)
            p.start()
            started = True
        ids_host, ev = eng.runner.run_step(step)
        sched.inflight.append((step, ids_host, ev))
        taken += int(hit)
        while len(sched.inflight) > 1:
            sched._process(*sched.inflight.popleft())
    sched.drain()
    torch.cuda.synchronize(dev)
    if not started:
        return
    p.stop()
    os.makedirs(OUT_DIR, exist_ok=True)
    suffix = f"_{mode_filter}" if mode_filter else ""
    with open(os.path.join(OUT_DIR, f"torchprof_rank{rank}{suffix}.txt"), "w") as f:
        f.write(f"{taken} profiled step(s)\n")
        f.write(p.key_averages().table(sort_by="cuda_time_total", row_limit=40, max_name_column_width=90))


def main():
    a = parse()
    if a.impl == "reference":
        reference_arm(a)
        return
    if a.baseline:
        os.environ["SGLANG_B200_BASELINE"] = a.baseline
    import numpy as np
    import torch
    import torch.distributed as dist

    from sglang_neuron_b200.engine import Engine
    from sglang_neuron_b200.managers.schedule_batch import SamplingParams
    from sglang_neuron_b200.model_executor.forward_batch import ForwardMode
    from sglang_neuron_b200.parallel.state import get_state
    from sglang_neuron_b200.server_args import ServerArgs
    from sglang_neuron_b200 import _ext

    world = int(os.environ.get("WORLD_SIZE", "1"))
    assert world == a.gpus, f"--gpus {a.gpus} but WORLD_SIZE={world}"
    C, IL, OL = a.concurrency, a.input_len, a.output_len
    S = a.stagger or max(1, min(16, OL // max(1, C)))
    headline = a.model == "gpt-oss-120b"
    kv = a.kv or ("fp8_e4m3" if headline else "auto")
    ctx = IL + OL + 64
    bs_list = sorted({b for b in (1, 2, 4, 8, 16, 32, 48, 56, 60, 62, 63, 64, 96, 112, 120, 124, 126, 127, C) if b <= C})
    args = ServerArgs(model=a.model, load_format="random", device="cuda", tp_size=a.gpus, page_size=a.page_size,
                      context_length=ctx, max_running_requests=C + 8, chunked_prefill_size=a.chunked_prefill,
                      max_prefill_tokens=a.chunked_prefill, cuda_graph_bs=bs_list, disable_cuda_graph=a.no_graph,
                      disable_radix_cache=True, kv_cache_dtype=kv, seed=a.seed, mem_fraction_static=0.9)
    t_init = time.perf_counter()
    eng = Engine(args)
    st = get_state()
    rank = st.rank
    dev = eng.runner.device
    init_s = time.perf_counter() - t_init
    rng = np.random.default_rng(a.seed)
    V = eng.cfg.vocab_size
    sched = eng.scheduler
    counter = [0]

    # Every rank runs this same code (SPMD): rank 0 owns intake and broadcasts arrivals inside
    # scheduler steps; requests are tracked by rid so followers see the same state once they arrive.
    def new_req(ctx_len, out_len):
        counter[0] += 1
        rid = f"b{counter[0]}"
        ids = rng.integers(0, V, size=ctx_len).tolist()
        eng.submit(ids, SamplingParams(max_new_tokens=out_len, temperature=0.0, ignore_eos=True), rid=rid)
        return rid

    def req(rid):
        return sched.reqs_by_rid.get(rid)

    def done(rid):
        r = req(rid)
        return r is not None and r.finished

    # steady-state construction (untimed): staggered progress across the 64 slots
    live = [new_req(IL + S * i, max(1, OL - S * i)) for i in range(C)]
    while any(req(rid) is None or req(rid).first_token_time is None for rid in live):
        sched.step()
    sched.drain()

    def refill():
        live[:] = [rid for rid in live if not done(rid)]
        for _ in range(C - len(live)):
            live.append(new_req(IL, OL))

    # warm-up: at least W steps, and until a mixed (prefill + decode) step of the steady state has run once,
    # so one-time costs of that shape (library heuristics, allocator growth) stay out of the timed steps
    warm, seen_mixed = 0, False
    while warm < a.warmup or (not seen_mixed and warm < a.warmup + 4 * S + 40):
        refill()
        n0 = sched.stats.get("extend_steps", 0)
        sched.step()
        seen_mixed = seen_mixed or sched.stats.get("extend_steps", 0) > n0
        warm += 1
    sched.drain()
    refill()

    # ---------------- timed region ----------------
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(torch.cuda.current_device() if world == 1 else int(os.environ.get("LOCAL_RANK", "0")))
    io = eng.runner.io
    h2d0, d2h0 = io.h2d_bytes, io.d2h_bytes
    launches0 = _ext.launch_count()
    steps_before = len(sched.step_times)
    start_ev = torch.cuda.Event(enable_timing=True)
    end_ev = torch.cuda.Event(enable_timing=True)
    produced = 0
    delivered0 = sched.stats["output_tokens"]
    wall0 = time.perf_counter()
    prof = os.environ.get("SNB_PROFILE_WINDOW") == "1"
    if prof:  # ncu --profile-from-start off captures only the timed steps
        torch.cuda.cudart().cudaProfilerStart()
    start_ev.record()
    timed_steps = []
    step_evs = []  # one event at each step's launch point: consecutive pairs time each step on the device
    for _ in range(a.steps):
        refill()
        sched._sync_arrivals()
        step = sched.schedule()
        if step is None:
            continue
        sev = torch.cuda.Event(enable_timing=True)
        sev.record()
        step_evs.append(sev)
        ids_host, ev = eng.runner.run_step(step)
        sched.inflight.append((step, ids_host, ev))
        sched.stats["steps"] += 1
        produced += sum(1 for s in step.sampled if s)
        timed_steps.append(step)
        while len(sched.inflight) > 1:
            sched._process(*sched.inflight.popleft())
    end_ev.record()
    if prof:
        torch.cuda.cudart().cudaProfilerStop()
    sched.drain()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    dev_ms = start_ev.elapsed_time(end_ev)
    step_ms = [e0.elapsed_time(e1) for e0, e1 in zip(step_evs, step_evs[1:] + [end_ev])]
    delivered = sched.stats["output_tokens"] - delivered0
    launches = _ext.launch_count() - launches0
    n_steps = len(timed_steps)
    h2d = (io.h2d_bytes - h2d0) / max(1, n_steps)
    d2h = (io.d2h_bytes - d2h0) / max(1, n_steps)
    if world > 1:
        t = torch.tensor([dev_ms, wall] + step_ms, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_ms, wall = float(t[0]), float(t[1])
        step_ms = t[2:].tolist()
    # latency stats from the requests that received tokens in the window
    ttfts, itls = [], []
    for r in sched.finished_reqs + [req(rid) for rid in live if req(rid) is not None]:
        if r.first_token_time is not None and r.first_token_time >= wall0 and r.arrival >= wall0:
            ttfts.append((r.first_token_time - r.arrival) * 1e3)
        tt = [t for t in r.token_times if t >= wall0]
        itls += [(b - a_) * 1e3 for a_, b in zip(tt, tt[1:])]
    value = produced / (dev_ms / 1e3)
    e2e = delivered / wall
    mixed = sum(1 for s in timed_steps if s.mode != ForwardMode.DECODE)
    dec_ms = [t for s, t in zip(timed_steps, step_ms) if s.mode == ForwardMode.DECODE]
    mix_ms = [t for s, t in zip(timed_steps, step_ms) if s.mode != ForwardMode.DECODE]
    step_stats = {"decode_p50_ms": round(statistics.median(dec_ms), 3) if dec_ms else None,
                  "decode_mean_ms": round(statistics.fmean(dec_ms), 3) if dec_ms else None,
                  "mixed_ms": [round(t, 3) for t in mix_ms],
                  "mixed_tokens": [int(s.num_tokens) for s in timed_steps if s.mode != ForwardMode.DECODE],
                  "how": "CUDA events at each step's launch point, max over ranks"}
    if rank == 0:
        metric = METRIC if headline and C == 64 else (
            f"output tok/s at concurrency {C}; p50 TTFT & ITL ({a.model}-shape, TP{a.gpus})")
        model_desc = ("GPT-OSS-120B-shape (36 layers, hidden 2880, 64q/8kv heads x 64, 128 experts top-4, "
                      "MXFP4 experts, FP8 KV, alternating SWA-128/full, sinks, YaRN)" if headline
                      else f"{a.model}-shape (architecture of the named checkpoint, random init), KV {kv}")
        line = {
            "metric": metric, "value": round(value, 1), "unit": "tok/s", "n_gpus": a.gpus, "steps": n_steps,
            "warmup": a.warmup, "warmup_steps_run": warm, "ms_per_step": round(dev_ms / max(1, n_steps), 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "impl": "baseline-nccl-cublas" if a.baseline else "ours",
            "data": "synthetic token ids (uniform, seeded); random-init weights of the named architecture",
            "config": {"model": model_desc,
                       "global_batch": C, "seq_len": IL + OL, "input_len": IL, "output_len": OL,
                       "parallelism": f"tp{a.gpus}ep{a.gpus}", "concurrency": C,
                       "l2": ("inputs larger than L2 (60+ GB of expert weights streamed per step)" if headline else
                              "inputs larger than L2 (the model's weights, > 126 MB, streamed every step)"),
                       "steps_mixed_prefill": mixed, "cuda_graph": not a.no_graph},
            "p50_ttft_ms": round(statistics.median(ttfts), 2) if ttfts else None,
            "ttft_samples": len(ttfts),
            "p50_itl_ms": round(statistics.median(itls), 3) if itls else None,
            "step_device_ms": step_stats,
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h),
                    "how": "host wall clock around the same steps via Engine scheduler/runner (pinned H2D inputs, "
                           "D2H sampled ids, tokens delivered to requests)"},
            "gpu_launches": int(launches),
            "clocks": clk,
            "init_s": round(init_s, 1),
        }
        print(json.dumps(line), flush=True)
    if os.environ.get("SNB_TORCH_PROFILE"):
        # attribution only (after the timed region): per-kernel device time of a few more steps, every rank
        _profile_steps(eng, sched, refill, rank, int(os.environ.get("SNB_TORCH_PROFILE")), dev,
                       os.environ.get("SNB_TORCH_PROFILE_MODE") or None)
    eng.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

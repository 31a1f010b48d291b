"""bench.py -- prefill tokens/s of the full RidgeFill step at 32K on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]

A step is one approximate pass of the RidgeFill step over a 32,768-row prefill chunk of the 48-layer stack:
the 24 late layers, 18 Gated DeltaNet and 6 attention layers, through this library's sm_100a
device rows (late_pass.LatePass): the class mask (30 % of rows exact) and the layer-S stream's codes once, then per
layer the int8 projector d 2,048 (per-column scales, fused bias, written straight into the block input's
approximated rows: the select fused into its epilogue) and the block input's codes; per DeltaNet
layer the int8 mixed q|k|v projection, the bf16 a|b projection and conv_prep (16 q/k, 32 v heads x 128); per
attention layer the int8 k|v projection and the K/V cache write (2 kv heads x 256, imrope); then one fill launch over
all 18 DeltaNet layers' 576 heads between a state undo and apply over the same heads, rho per layer, the hazard record.
Synthetic inputs with the published benchmark's shapes and distributions, seeded; the pass reads > 10 GB, far past the 126 MB L2, so
no flush is needed between steps.

value   device time of K passes with inputs resident in HBM (CUDA events, max over ranks)
e2e     the same passes through the same C-ABI rows with each step's inputs (h_S, token ids, positions) copied
        host->device from pinned memory and its results (every DeltaNet state, every attention cache, the mask,
        the decay sums, the hazard record) copied back, inside the timed region; two buffer sets let one step's copies
        overlap the neighbouring steps' passes
N > 1   one process per GPU (torchrun), tensor parallel over ONE prompt: each rank the DeltaNet value heads of its
        span (with their k heads) and its attention kv heads, the projector's output columns split across ranks and
        all-gathered over NVLink by the library's peer kernels ("scaling": "strong"; value = the prompt's tokens / the
        slowest rank's time)
extra   the mixed ragged batch (one 32K prompt after six of U[256, 2,048] rows) and the one-layer pass, device time
--impl reference   the CPU arm: the same pass on the host -- the reference's own host rows compiled from its sources
        (oracle/_ref) for mask, select, correction, rho, hazard, and the CPU restatement for the GEMMs, quantiser,
        conv_prep, K/V write and fill the reference does not contain -- on a bounded sample (2,048 rows, the first 4
        late layers), scaled to the pass; every host core; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "radiance-ridgefill_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

METRIC = "prefill tokens/s at 32K (RidgeFill step)"
T_FULL = 32768
WORKLOAD = ("the full RidgeFill step over the 24 late layers of a 48-layer stack (18 Gated "
            "DeltaNet + 6 attention), hidden 2,048, int8 per-column projectors, 32,768-row prompt, 30 % of rows exact")
CPU_ROWS, CPU_LAYERS = 2048, 4


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled while the timed region runs: through NVML every
    millisecond (a region of a few tens of milliseconds still gets samples), else nvidia-smi every 200 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h): sw power cap 0x4, hw slowdown 0x8, sw thermal 0x20, hw thermal 0x40
    NVML_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                 ("sw_power_cap", 0x4))

    def __init__(self, gpu_index: int):
        self.idx, self.rows, self.proc, self.nvml, self.samples = gpu_index, [], None, None, []
        self.stop_flag = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.idx)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.idx)

    def start(self):
        try:
            self.nvml = self._nvml_handle()
            self.max_mhz = self.nvml[0].nvmlDeviceGetMaxClockInfo(self.nvml[1], self.nvml[0].NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _poll(self):
        nv, h = self.nvml
        while not self.stop_flag.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                try:
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                except AttributeError:
                    bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append((mhz, bits))
            except Exception:
                return
            time.sleep(0.001)

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.nvml:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            sm = [float(m) for m, _ in self.samples]
            reasons = sorted({name for _, b in self.samples for name, bit in self.NVML_BITS if b & bit})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(self.max_mhz),
                    "reasons": reasons, "samples": len(sm), "source": "nvml, 1 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm), "source": "nvidia-smi, 200 ms"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------------------------------ the CPU arm

def cpu_arm(passes: int, warmup: int) -> dict:
    """The pass on the host over a bounded sample: CPU_ROWS rows of the prompt through the first CPU_LAYERS late
    layers (one period of the 3:1 DeltaNet / attention interleave); the whole pass's time is taken as the sample's
    time x 24 / CPU_LAYERS, and the rows per second of the sample stand for the chunk's (the CPU rows are linear in
    the rows, except the mask's O(w^2) rank count, which is a small part at this size)."""
    import cpu_path
    import late_pass as LP
    shape = LP.full_step(CPU_ROWS)
    inputs = cpu_path.to_host(LP.late_inputs(shape, "cpu", 7))
    c = cpu_path.CpuLatePass(shape, inputs, layers=CPU_LAYERS)
    sec = c.time_passes(passes, warmup)
    scale = len(shape.layers) / CPU_LAYERS
    per_pass = sec * scale
    return {"value": CPU_ROWS / per_pass, "unit": "tokens/s", "cores": c.threads, "kind": c.kind,
            "sample": f"{CPU_ROWS} rows of the prompt through the first {CPU_LAYERS} of the 24 late layers "
                      f"(G G G A), {passes} timed passes of {sec:.2f} s; the full pass taken as x{scale:g} (24 layers); "
                      f"mask, select, correction, rho, hazard: the reference's host rows ({c.kind}); GEMMs, quantiser, "
                      f"conv_prep, K/V write, fill: the CPU restatement, OpenMP on {c.threads} threads",
            "sec_per_pass": per_pass}


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    base = cpu_arm(args.steps, args.warmup)
    line = {"metric": METRIC, "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": base["sec_per_pass"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "i8/bf16/f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "rows": T_FULL, "d": 2048, "late_layers": 24,
                       "parallelism": "host cores of rank 0 (each step a bounded sample: cpu_baseline.sample)"},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------ the device arm

def per_op_times(p, stream, reps: int = 2) -> dict:
    """Device milliseconds per pass of each row (every launch of it), from an ordered pass with events."""
    import torch
    counts = p.op_counts()
    total = {op: 0.0 for op in counts}
    for _ in range(reps):
        ev = {op: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
              for op, n in counts.items()}
        with torch.cuda.stream(stream):
            p.run(stream.cuda_stream, events=ev)
        stream.synchronize()
        for op, pairs in ev.items():
            total[op] += sum(a.elapsed_time(b) for a, b in pairs) / reps
    return total


def roofline(op: str, ms: float, alg: dict, pk: dict) -> dict:
    """The roofline of one row's launches in a pass (all of its launches: `ms` their summed device time)."""
    if op == "ridgefill_gemm_nt_q_bias":
        peak = 2.0 * pk["bf16_tflops"]
        r = {"bound": "tensor", "achieved": alg["int8_ops"] / (ms * 1e-3) / 1e12, "peak": peak, "unit": "TOP/s",
             "traffic": None, "note": f"int8 dense peak = 2 x the {pk['source']} bf16 figure ({pk['bf16_tflops']} TF/s); "
                                      "the pass's ridgefill_gemm_nt_q_bias launches together (projectors, q tails, attention k|v)"}
    elif op == "ridgefill_gdn_in_proj":
        peak = 2.0 * pk["bf16_tflops"]
        r = {"bound": "tensor", "achieved": alg["int8_ops_in_proj"] / (ms * 1e-3) / 1e12, "peak": peak, "unit": "TOP/s",
             "traffic": None, "note": f"int8 dense peak = 2 x the {pk['source']} bf16 figure ({pk['bf16_tflops']} TF/s); "
                                      "the DeltaNet k|v projections with the convolution, SiLU and k norm in their "
                                      "epilogue (the 3-row tile overlap's extra 2.4 % of MMAs not counted)"}
    elif op == "ridgefill_gdn_fill":
        # DRAM bytes over algorithmic bytes of the per-head fill, from one ncu capture of it (8,192 rows, 128 heads:
        # 424.2 MB read + written against 427.4 MB, profiles/gdn_fill_heads_T8192.md); the traffic grows with the
        # heads and rows it processes, so the pass's launch is taken as that ratio times its algorithmic bytes
        traffic_ratio = (419.5 + 4.7) / 427.4
        r = {"bound": "hbm", "achieved": alg["fill_bytes"] / (ms * 1e-3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
             "traffic": alg["fill_bytes"] * traffic_ratio / 1e9, "traffic_unit": "GB per launch",
             "note": f"the batched fill (state-only bytes: k, v, g, beta read, state read and written), one launch a "
                     f"pass; traffic scaled from an ncu capture of 8,192 rows x 128 heads; peak {pk['source']}"}
        r["tensor"] = {"achieved": alg["fill_chunk_flops"] / (ms * 1e-3) / 1e12, "peak": pk["bf16_tflops"],
                       "unit": "TFLOP/s"}
        r["tensor"]["frac"] = r["tensor"]["achieved"] / r["tensor"]["peak"]
    else:
        return {"kernel": op, "kernel_ms": ms}
    r["frac"] = r["achieved"] / r["peak"]
    r["kernel"] = op
    r["kernel_ms"] = ms
    return r


def run_mine(args):
    import torch
    import torch.distributed as dist
    import late_pass as LP

    world, rank, local = dist_setup()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    shape = LP.full_step(T_FULL)
    team = LP.Team.create(world, rank, dist) if world > 1 else None
    p = LP.LatePass(shape, str(dev), seed=1234, team=team)
    stream = torch.cuda.Stream(device=dev)
    alg = p.algorithmic()
    kernels = p.kernels

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            p.run(stream.cuda_stream)
    stream.synchronize()
    per_op = per_op_times(p, stream)
    dominant = max(per_op, key=per_op.get)

    # ---------------------------------------------------------- device-resident timing
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            p.run(stream.cuda_stream)
        stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        clocks.start()
        start.record(stream)
        for _ in range(args.steps):
            p.run(stream.cuda_stream)
        end.record(stream)
        stream.synchronize()
    clock_info = clocks.stop()
    torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps

    # ---------------------------------------------------------- end to end, host buffers in and out
    # Two buffer sets (two passes' buffers) and three streams: step i+1's upload and step i-1's readback run on the
    # copy engines while step i computes; a set is reused only after its previous pass and readback. The results
    # final before the fill (the attention caches, the conv states, the mask) are read back while the fill runs,
    # the rest once the pass is done.
    sets = [p, LP.LatePass(shape, str(dev), seed=4321, team=team)]
    ins = [s_.inputs_per_step() for s_ in sets]
    outs = [s_.results_split() for s_ in sets]
    host_in = [t.cpu().pin_memory() for t in ins[0]]
    host_out = [tuple([torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in part] for part in o) for o in outs]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for part in host_out[0] for t in part)
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def e2e_steps(n, start_event=None, end_event=None):
        done_comp, done_out = [None, None], [None, None]
        if start_event is not None:
            start_event.record(s_in)
        for i in range(n):
            b_ = i % 2
            with torch.cuda.stream(s_in):
                if done_comp[b_] is not None:
                    s_in.wait_event(done_comp[b_])
                for d_, h in zip(ins[b_], host_in):
                    d_.copy_(h, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            stream.wait_event(ev_in)
            if done_out[b_] is not None:
                stream.wait_event(done_out[b_])
            blocks_done = torch.cuda.Event()
            with torch.cuda.stream(stream):
                sets[b_].run(stream.cuda_stream, before_tail=lambda: blocks_done.record(stream))
            done_comp[b_] = torch.cuda.Event()
            done_comp[b_].record(stream)
            with torch.cuda.stream(s_out):
                for ev_, h_part, d_part in ((blocks_done, host_out[b_][0], outs[b_][0]),
                                            (done_comp[b_], host_out[b_][1], outs[b_][1])):
                    s_out.wait_event(ev_)
                    for h, d_ in zip(h_part, d_part):
                        h.copy_(d_, non_blocking=True)
                done_out[b_] = torch.cuda.Event()
                done_out[b_].record(s_out)
        if end_event is not None:
            for e in done_out:
                if e is not None:
                    s_out.wait_event(e)
            end_event.record(s_out)

    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps(3)
    torch.cuda.synchronize()
    barrier()
    e2e_steps(args.steps, e_start, e_end)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e_start.elapsed_time(e_end) / args.steps
    del sets[1]

    # ---------------------------------------------------------- extras (one GPU): the ragged batch and the one-layer pass
    extra = {}
    if world == 1 and not args.no_extra:
        del p
        torch.cuda.empty_cache()
        extra["ragged_batch"] = time_extra(LP.LatePass(LP.ragged_batch(), str(dev), seed=99), stream, args.steps)
        torch.cuda.empty_cache()
        extra["one_layer_pass"] = time_one_layer(stream, args.steps)

    import shard
    dom_ms = per_op[dominant]
    ms, e2e_ms, dom_ms = shard.max_over_ranks([ms, e2e_ms, dom_ms], dist if world > 1 else None)

    if rank == 0:
        pk = peaks()
        roof = roofline(dominant, dom_ms, alg, pk)
        second = max((op for op in per_op if op != dominant), key=per_op.get)
        fill_key = "ridgefill_gdn_fill"
        line = {"metric": METRIC, "value": T_FULL / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "i8/bf16/f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "rows": T_FULL, "d": 2048, "late_layers": "GGGA x 6",
                           "l2": "inputs larger than L2 (no flush)",
                           "parallelism": (f"tp{world}: value heads and attention kv heads by rank span, projector "
                                           f"columns split and all-gathered by peer kernels" if world > 1 else "tp1")},
                "gpu_launches": kernels * args.steps,
                "per_op_ms": {k: round(v, 4) for k, v in sorted(per_op.items(), key=lambda kv: -kv[1])},
                "roofline": roof,
                "roofline_next": roofline(second, per_op[second], alg, pk) if second in (fill_key, "ridgefill_gemm_nt_q_bias", "ridgefill_gdn_in_proj") else None,
                "clocks": clock_info,
                "e2e": {"value": T_FULL / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h}}
        if extra:
            line["extra"] = extra
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = {k: v for k, v in cpu_arm(2, 1).items() if k != "sec_per_pass"}
        print(json.dumps(line), flush=True)
    if team is not None:
        team.close()
    if world > 1:
        dist.destroy_process_group()


def time_extra(p, stream, steps: int) -> dict:
    import torch
    with torch.cuda.stream(stream):
        for _ in range(3):
            p.run(stream.cuda_stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        a.record(stream)
        for _ in range(steps):
            p.run(stream.cuda_stream)
        b.record(stream)
        stream.synchronize()
    ms = a.elapsed_time(b) / steps
    s = p.s
    return {"workload": f"mixed ragged batch: prompts of {list(s.lengths)} rows, the last approximated, the 24 late "
                        f"layers; the fill over every sequence (varlen)", "rows": s.T, "ms_per_step": ms,
            "tokens_per_s": s.T / (ms * 1e-3)}


def time_one_layer(stream, steps: int) -> dict:
    import torch
    import ridgefill_step as RS
    step = RS.Step(RS.StepShape(T=T_FULL), device="cuda", seed=1234)
    with torch.cuda.stream(stream):
        for _ in range(3):
            step.run(stream.cuda_stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        a.record(stream)
        for _ in range(steps):
            step.run(stream.cuda_stream)
        b.record(stream)
        stream.synchronize()
    ms = a.elapsed_time(b) / steps
    return {"workload": "one late layer: projector d 2,048 + DeltaNet fill (16 q/k and 32 v heads of 128, inputs given) + mask, "
                        "select, correction, rho, hazard", "rows": T_FULL, "ms_per_step": ms,
            "tokens_per_s": T_FULL / (ms * 1e-3)}


def run_only(args):
    """Launch only one row's launches of the pass (every launch of it, in the pass's order), after --warmup whole
    passes that fill their inputs, at --rows rows and --layers late layers: a small, self-contained command for an
    ncu capture of that row's kernels."""
    import torch
    import late_pass as LP
    shape = LP.LateShape(T=args.rows, layers=args.layers)
    p = LP.LatePass(shape, "cuda", seed=1234)
    calls = [c for c in p.calls if c[0] == args.only]
    if not calls:
        raise SystemExit(f"--only {args.only}: not a row of the pass")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            p.run(stream.cuda_stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        a.record(stream)
        for _ in range(args.steps):
            for op, r, tens, params, _tag in calls:
                p._launch(op, r, tens, params, stream.cuda_stream)
        b.record(stream)
        stream.synchronize()
    print(json.dumps({"op": args.only, "rows": args.rows, "layers": args.layers, "launches": args.steps * len(calls),
                      "ms_per_launch": a.elapsed_time(b) / (args.steps * len(calls))}), flush=True)


def run_profile_pass(args):
    """Issue --warmup whole passes of the full step, then one more between cudaProfilerStart and
    cudaProfilerStop, and nothing else (no timing, no extras): the command an ncu launch list of one pass runs
    (`ncu --profile-from-start off` sees that pass's launches only, not the input set-up's nor the warm-up's)."""
    import torch
    import late_pass as LP
    p = LP.LatePass(LP.LateShape(T=args.rows, layers=args.layers), "cuda", seed=1234)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            p.run(stream.cuda_stream)
    stream.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    with torch.cuda.stream(stream):
        p.run(stream.cuda_stream)
    stream.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"profile_pass": True, "rows": args.rows, "layers": args.layers, "kernels_per_pass": p.kernels}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the ragged-batch and one-layer extras")
    ap.add_argument("--only", default=None, help="profile mode: launch only this row's launches of the pass")
    ap.add_argument("--rows", type=int, default=T_FULL, help="rows of the chunk in --only mode")
    ap.add_argument("--layers", default="GGGA" * 6, help="late layers in --only / --profile-pass mode (G DeltaNet, A attention)")
    ap.add_argument("--profile-pass", action="store_true", help="profile mode: --warmup passes, then one pass, untimed")
    args = ap.parse_args()
    if args.profile_pass:
        run_profile_pass(args)
    elif args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_mine(args)


if __name__ == "__main__":
    main()

"""bench.py -- prefill tokens/s of one RidgeFill approximate pass at 32K on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]

A step is one pass of the RidgeFill hot path over a 32,768-row prefill chunk (ridgefill_step.Step):
mask -> activation codes -> int8 projector (d 2,048, per-column scales, fused bias) -> select ->
state undo -> Gated DeltaNet chunk fill (16 q/k heads, 32 v heads, 128 dims, state [32,128,128] f32)
-> rho -> state apply -> hazard, every op a launch of the library's sm_100a device rows through the C
ABI. Synthetic inputs with BASELINE's shapes and distributions, seeded; inputs (> 700 MB) exceed the
126 MB L2, so no flush is needed between steps. The timed passes are issued pipelined (Step.run_pipelined):
the projector path (codes, projector) from the top of the pass and select after the mask on a normal-priority
stream, the rest (mask, undo, fill, rho, apply, hazard) on a high-priority stream, as a pass over the late layers
runs the next layer's projection of the shared h_S beside this layer's fill; every op of every pass still runs,
and a pass ends when both streams have finished it.

value   device time of K passes with inputs resident in HBM (CUDA events, max over ranks)
e2e     the same passes with each step's inputs copied host->device from pinned memory and the results
        (projected block input x, DeltaNet state, mask) copied back, inside the timed region; two buffer sets
        let one step's copies overlap the neighbouring steps' passes (copy engines and SMs run together)
N > 1   one process per GPU (torchrun), each rank an independent 32K prompt: prompts are independent
        units, no data-path collective ("scaling": "weak"); value = all ranks' tokens / max rank time.
--impl reference   the CPU arm: the reference's own host rows (compiled from kernels/host_ref.cpp into
        oracle/_ref) plus the CPU restatement of the projector and the fill it lacks, on a 2,048-row
        sample of the workload, all host threads; rank 0 only.
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
WORKLOAD = ("RidgeFill approximate pass over a 32,768-row prefill chunk: projector d 2,048 (int8, per-column scales), "
            "Gated DeltaNet fill 16 qk / 32 v heads x 128, class mask share 0.30")
T_FULL = 32768
CPU_SAMPLE_ROWS = 2048


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


def cpu_arm(steps: int, warmup: int) -> dict:
    import cpu_path
    s = cpu_path.CpuStep(CPU_SAMPLE_ROWS)
    sec = s.time_steps(steps, warmup)
    return {"value": CPU_SAMPLE_ROWS / sec, "unit": "tokens/s", "cores": s.threads, "kind": s.kind,
            "sample": f"the same pass on a {CPU_SAMPLE_ROWS}-row chunk (T={CPU_SAMPLE_ROWS} of {T_FULL}; "
                      f"the mask's rank count is O(w^2), so the full chunk is slower per row on the CPU), "
                      f"{steps} timed passes", "sec_per_pass": sec}


def run_reference(args):
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    base = cpu_arm(args.steps, args.warmup)
    line = {"metric": METRIC, "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": base["sec_per_pass"] * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "i8/bf16/f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "rows": T_FULL, "d": 2048,
                       "parallelism": "host cores of rank 0 (each step a bounded sample: cpu_baseline.sample)"},
            "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_mine(args):
    import torch
    import torch.distributed as dist
    import ridgefill_step as RS

    world, rank, local = dist_setup()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    step = RS.Step(RS.StepShape(T=T_FULL), device=str(dev), seed=1234 + rank)
    # the pass's main stream at high priority; the projector path and select beside it at normal priority (run_pipelined)
    stream = torch.cuda.Stream(device=dev, priority=-1)
    side = torch.cuda.Stream(device=dev, priority=0)
    alg = step.algorithmic()

    def barrier():
        if world > 1:
            dist.barrier()

    # per-op device times (untimed pass), to name the dominant kernel
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step.run(stream.cuda_stream)
        ops = {name: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for name in {c[0] for c in step.calls}}
        per_op = {n: 0.0 for n in ops}
        for _ in range(3):
            step.run(stream.cuda_stream, events=ops)
            stream.synchronize()
            for n, (a, b) in ops.items():
                per_op[n] += a.elapsed_time(b) / 3
    dominant = max(per_op, key=per_op.get)

    # ---------------------------------------------------------- device-resident timing
    dom_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    pipelined = dominant not in RS.Step.SIDE_OPS
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step.run_pipelined(stream, side)
        stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        clocks.start()
        start.record()
        for i in range(args.steps):
            if pipelined:
                step.run_pipelined(stream, side, events={dominant: dom_ev[i]})
            else:
                step.run(stream.cuda_stream, events={dominant: dom_ev[i]})
        end.record()
        stream.synchronize()
    clock_info = clocks.stop()
    torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    dom_ms = statistics.mean(a.elapsed_time(b) for a, b in dom_ev)

    # ---------------------------------------------------------- end to end through the C ABI, host buffers
    # Each step uploads its inputs from pinned host memory, runs the pass and reads its results back. Two
    # buffer sets (two Step objects) and three streams let step i+1's upload and step i-1's readback run on
    # the copy engines while step i computes; a set is reused only after its previous pass and readback.
    steps2 = [step, RS.Step(RS.StepShape(T=T_FULL), device=str(dev), seed=4321 + rank)]
    ins = [[s_.h_s, s_.k, s_.v, s_.g, s_.beta, s_.ab, s_.token_ids, s_.positions] for s_ in steps2]
    outs = [[s_.x, s_.state, s_.mask] for s_ in steps2]
    host_in = [t.cpu().pin_memory() for t in ins[0]]
    host_out = [[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in o] for o in outs]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out[0])
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
            steps2[b_].run_pipelined(stream, side)
            done_comp[b_] = torch.cuda.Event()
            done_comp[b_].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done_comp[b_])
                for h, d_ in zip(host_out[b_], outs[b_]):
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

    # the job's time is its slowest rank's
    import shard
    ms, e2e_ms, dom_ms = shard.max_over_ranks([ms, e2e_ms, dom_ms], dist if world > 1 else None)

    if rank == 0:
        pk = peaks()
        if dominant == "ridgefill_gemm_nt_q_bias":
            int8_peak = 2.0 * pk["bf16_tflops"]
            roof = {"bound": "tensor", "achieved": alg["gemm_ops"] / (dom_ms * 1e-3) / 1e12, "peak": int8_peak,
                    "unit": "TOP/s", "traffic": None,
                    "note": f"int8 dense peak = 2 x the {pk['source']} bf16 figure ({pk['bf16_tflops']} TF/s)"}
        else:
            by = {"ridgefill_gdn_fill": alg["gdn_bytes"], "ridgefill_quant_act_i8g": alg["quant_bytes"],
                  "ridgefill_select": alg["select_bytes"]}.get(dominant, 0)
            roof = {"bound": "hbm", "achieved": by / (dom_ms * 1e-3) / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                    "traffic": None, "note": f"peak {pk['source']}"}
            if dominant == "ridgefill_gdn_fill":
                # DRAM bytes of one fill from an ncu capture at 16,384 rows (plan + fill kernels: 0.009 + 564.9
                # MB: 208.1 read, 356.9 written), scaled by rows: every term (k, v, g, beta reads, the chunk
                # slots written and read back) grows in proportion to the rows.
                roof["traffic"] = 564.9e6 * T_FULL / 16384
                roof["traffic_note"] = "ncu dram__bytes_read+write at 16,384 rows, scaled by rows"
                roof["tensor"] = {"achieved": alg["gdn_chunk_flops"] / (dom_ms * 1e-3) / 1e12, "peak": pk["bf16_tflops"],
                                  "unit": "TFLOP/s"}
                roof["tensor"]["frac"] = roof["tensor"]["achieved"] / roof["tensor"]["peak"]
        roof["frac"] = roof["achieved"] / roof["peak"]
        roof["kernel"] = dominant
        roof["kernel_ms"] = dom_ms
        line = {"metric": METRIC, "value": world * T_FULL / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "i8/bf16/f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "rows": T_FULL, "d": 2048, "l2": "inputs larger than L2 (no flush)",
                           "parallelism": f"independent prompts x{world}",
                           "streams": "projector path beside the fill (two streams, pipelined pass)"},
                "gpu_launches": Step_launches(step) * args.steps,
                "per_op_ms": {k: round(v, 4) for k, v in sorted(per_op.items(), key=lambda kv: -kv[1])},
                "roofline": roof, "clocks": clock_info,
                "e2e": {"value": world * T_FULL / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h}}
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = {k: v for k, v in cpu_arm(2, 1).items() if k != "sec_per_pass"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def side_op_call(op: str, rows: int):
    """Operands of a row the pass does not issue, at the served layer's shapes and `rows` rows (synthetic, seeded):
    ridgefill_gdn_conv_prep (16 q/k and 32 v heads of 128, one sequence with a conv history) and
    ridgefill_attn_kv_fill (2 kv heads of 256, rope 64 of imrope sections 11/11/10, every row stored). Returns
    (row, tensors, params, keep) -- `keep` holds the torch buffers for as long as the launches run."""
    import torch
    import ridgefill_abi as abi
    lib = abi.product()
    g = torch.Generator(device="cuda").manual_seed(1234)
    t = lambda x, code=None: abi.tensor(code or {torch.float32: abi.F32, torch.bfloat16: abi.BF16,   # noqa: E731
                                                  torch.int32: abi.I32}[x.dtype], list(x.shape), x.data_ptr(), list(x.stride()))
    T = rows
    if op == "ridgefill_gdn_conv_prep":
        hk, hv = 16, 32
        C = 2 * hk * 128 + hv * 128
        keep = dict(x=torch.randn(T, C, device="cuda", generator=g).bfloat16(),
                    w=(0.5 * torch.randn(C, 4, device="cuda", generator=g)).bfloat16(),
                    al=torch.randn(hv, device="cuda", generator=g), dt=torch.randn(hv, device="cuda", generator=g),
                    st=torch.zeros(2, 3, C, device="cuda").bfloat16(), cu=torch.tensor([0, T], dtype=torch.int32, device="cuda"),
                    ab=torch.randn(T, 2 * hv, device="cuda", generator=g).bfloat16(),
                    idx=torch.tensor([1], dtype=torch.int32, device="cuda"), ctx=torch.tensor([5], dtype=torch.int32, device="cuda"),
                    q=torch.empty(T, hk, 128, device="cuda").bfloat16(), k=torch.empty(T, hk, 128, device="cuda").bfloat16(),
                    v=torch.empty(T, hv, 128, device="cuda").bfloat16(), g=torch.empty(T, hv, device="cuda"),
                    be=torch.empty(T, hv, device="cuda"))
        k = keep
        tens = [t(k["x"]), t(k["w"]), abi.absent(), t(k["al"]), t(k["dt"]), t(k["st"]), t(k["cu"]),
                abi.tensor(abi.BF16, [T, hv], k["ab"].data_ptr(), [2 * hv, 1]),
                abi.tensor(abi.BF16, [T, hv], k["ab"].data_ptr() + 2 * hv, [2 * hv, 1]),
                t(k["idx"]), t(k["ctx"]), t(k["q"]), t(k["k"]), t(k["v"]), t(k["g"]), t(k["be"])]
        params = [abi.pint("M", T), abi.pint("n_head_k", hk), abi.pint("n_head_v", hv), abi.pint("head_k", 128),
                  abi.pint("head_v", 128), abi.pint("conv", 4)]
    elif op == "ridgefill_attn_kv_fill":
        hkv = 2
        keep = dict(k=torch.randn(T, hkv, 256, device="cuda", generator=g).bfloat16(),
                    v=torch.randn(T, hkv, 256, device="cuda", generator=g).bfloat16(),
                    w=torch.ones(256, device="cuda").bfloat16(),
                    pos=(torch.arange(3 * T, dtype=torch.int32, device="cuda") % 30000).view(3, T),
                    slots=torch.randperm(T + 1000, device="cuda", generator=g)[:T].int(),
                    cache=torch.zeros(2, T + 1000, hkv, 256, device="cuda").bfloat16())
        k = keep
        tens = [t(k["k"]), t(k["v"]), t(k["w"]), t(k["pos"]), t(k["slots"]), t(k["cache"]), abi.absent()]
        params = [abi.pint("M", T), abi.pint("n_head_kv", hkv), abi.pint("head_dim", 256), abi.pint("rope_dim", 64),
                  abi.pf64("rope_theta", 1e7), abi.pstr("rope_mode", "imrope"), abi.pstr("rope_sections", "11,11,10")]
    else:
        return None
    return lib.find_row(op, abi.DOMAIN_DEVICE), tens, params, keep


def run_only(args):
    """Launch one op of the pass repeatedly at --rows rows (after --warmup full passes that fill its
    inputs), or one of the rows beside the pass (ridgefill_gdn_conv_prep, ridgefill_attn_kv_fill) on synthetic
    operands: a small, self-contained command for an ncu capture of that op's kernels."""
    import torch
    import ridgefill_step as RS
    side = side_op_call(args.only, args.rows)
    if side is not None:
        row, tens, params, keep = side
        import ridgefill_abi as abi
        lib = abi.product()
        stream = torch.cuda.Stream()
        for _ in range(args.warmup):
            if lib.launch(row, tens, params, stream=stream.cuda_stream) != 0:
                raise SystemExit(f"{args.only}: refused")
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        a.record(stream)
        for _ in range(args.steps):
            if lib.launch(row, tens, params, stream=stream.cuda_stream) != 0:
                raise SystemExit(f"{args.only}: refused")
        b.record(stream)
        stream.synchronize()
        print(json.dumps({"op": args.only, "rows": args.rows, "launches": args.steps,
                          "ms_per_launch": a.elapsed_time(b) / args.steps}), flush=True)
        del keep
        return
    step = RS.Step(RS.StepShape(T=args.rows), device="cuda", seed=1234)
    stream = torch.cuda.Stream()
    calls = [c for c in step._args if c[0] == args.only]
    if not calls:
        raise SystemExit(f"--only {args.only}: not an op of the pass")
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step.run(stream.cuda_stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.synchronize()
        a.record()
        for _ in range(args.steps):
            for name, r, tens, params in calls:
                sb = step.gdn_scratch if name == "ridgefill_gdn_fill" else 0
                rc = step.lib.launch(r, tens, params, stream=stream.cuda_stream,
                                     scratch=step.scratch.data_ptr() if sb else None, scratch_bytes=sb)
                if rc != 0:
                    raise SystemExit(f"{name}: rc {rc}")
        b.record()
        stream.synchronize()
    print(json.dumps({"op": args.only, "rows": args.rows, "launches": args.steps * len(calls),
                      "ms_per_launch": a.elapsed_time(b) / (args.steps * len(calls))}), flush=True)


def Step_launches(step) -> int:
    return step.LAUNCHES_PER_PASS


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--only", default=None, help="profile mode: launch only this op of the pass, or ridgefill_gdn_conv_prep / ridgefill_attn_kv_fill on synthetic operands")
    ap.add_argument("--rows", type=int, default=T_FULL, help="rows of the chunk in --only mode")
    args = ap.parse_args()
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_mine(args)


if __name__ == "__main__":
    main()

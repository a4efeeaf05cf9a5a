#!/usr/bin/env python
"""BaseLM per-token decode benchmark (one JSON line on rank 0).

Workloads (seeded synthetic models):
  cfg2 (default)  28 layers, H=2048, 16x128 heads, 2 KV heads, F=6144, Q8_0; one stream per GPU,
                  KV prefilled to 1023 positions, decoding towards a 4096 context
  cfg3            cfg2 with F16 projections
  cfg1            24 layers at H=1024 (config[0]'s layer), F16 token table, 128-token prefill
  cfg0            config[0]: one layer at H=1024, 512 prior positions
  residual        ResidualLM + FSQ + fusion at VoxCPM2's shape (8 layers, H=2048, F16), positions/s
  cfg4            16 streams per GPU at cfg2's shape with ragged KV lengths ~U[64, 4096]; a step
                  advances every stream by one token (vg_decode_batch)

A step is one decode token of one stream. `value` is the whole-job aggregate tok/s over all
GPUs (independent replicas, weights replicated, no collectives on the data path), device-timed
with CUDA events on the engine's stream, max over ranks. `e2e` is the same metric through the
C ABI with host buffers: every step copies its token from pinned host memory and reads the
output hidden state back to the host.

`--impl reference` times the reference's CPU path on all host cores, on the same workload: the
reference's own BaseLM shaders compiled as C++ (oracle/_ref) where that library was built, else
the C restatement of the shaders (oracle/). The reference's Rust host and its Vulkan path cannot
be built or run here.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # span: the decode positions the config covers; the timed steps are spread over it
    "cfg2": dict(preset="cfg2", prefill=1023, ctx=4096, span=(1024, 4095),
                 desc="BaseLM 28L H2048 16x128 GQA 2 KV F6144 Q8_0"),
    "cfg3": dict(preset="cfg3", prefill=1023, ctx=4096, span=(1024, 4095),
                 desc="BaseLM 28L H2048 16x128 GQA 2 KV F6144 F16"),
    "cfg1": dict(preset="cfg1", prefill=128, ctx=512, span=(128, 383),
                 desc="BaseLM 24L H1024 16x64 GQA 2 KV F4096 Q8_0"),
    "cfg0": dict(preset="cfg0", prefill=512, ctx=1024, span=(512, 1023),
                 desc="one BaseLM layer H1024 16x64 GQA 2 KV F4096 Q8_0"),
    # ResidualLM + FSQ + fusion after BaseLM (src/acoustic.rs:851-1035), VoxCPM2's shape
    "residual": dict(acoustic="res_cfg2", prefill=0, ctx=4096,
                     desc="ResidualLM 8L H2048 16x128 GQA 2 KV F6144 F16 + FSQ 512 + fusion"),
    # batched prefill (vg_prefill_tokens): config[1]'s 128-token prompt, and a longer prompt at
    # config[2]'s shape; one step is one whole prompt from position 0
    "prefill": dict(preset="cfg1", prompt=128, desc="prefill of a 128-token prompt, BaseLM 24L H1024 Q8_0"),
    "prefill_cfg2": dict(preset="cfg2", prompt=512, desc="prefill of a 512-token prompt, BaseLM 28L H2048 Q8_0"),
    # BASELINE cfg4: many streams per GPU, each with its own KV cache (runtime.rs's engines)
    "cfg4": dict(preset="cfg2", streams=16, ctx=4096, slack=256, prefill=2080,
                 desc="16 streams per GPU, BaseLM 28L H2048 Q8_0, ragged KV ~U[64,4096]"),
}


# The JSON line goes to the process's original stdout; everything else that
# writes to file descriptor 1 (NCCL prints its version line there at
# communicator set-up) is sent to stderr, so stdout holds the one line.
_JSON_OUT = None


def quiet_stdout():
    global _JSON_OUT
    if _JSON_OUT is None:
        sys.stdout.flush()
        _JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(line):
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=sorted(WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-profile", action="store_true")
    return ap.parse_args()


def dist_env():
    from voxgen_b200 import replicas
    return replicas.env()


def model_cache() -> Path:
    return Path(os.environ.get("VOXGEN_MODEL_CACHE", "/tmp/voxgen_b200_models"))


def ensure_model(spec, rank, world, pg_barrier):
    from voxgen_b200 import synth
    if rank == 0:
        p = synth.model_path(spec, model_cache())
    pg_barrier()
    if rank != 0:
        p = synth.model_path(spec, model_cache())
    return p


def launch_traffic(workload, kernel="decode_step_kernel"):
    """DRAM bytes of one launch of `kernel` on this workload from an ncu capture
    (profiles/traffic.json), or None."""
    tr = ROOT / "profiles" / "traffic.json"
    if not tr.exists():
        return None
    return json.loads(tr.read_text()).get(workload, {}).get(kernel)


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# NVML clock-event reason bits (nvmlClocksEventReason*): reported by name when active.
_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
            0x80: "hw_power_brake_slowdown"}


class ClockSampler:
    """SM clock and clock-event reasons sampled during the timed region: NVML in a thread every
    10 ms (plus one sample at start and one at stop, so a region of a few milliseconds still has
    samples), else nvidia-smi. Reads only; nothing is set."""

    def __init__(self, device_index: int):
        import threading
        self.rows = []
        self.proc = None
        self.nv = None
        self.stop_ev = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                self.h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._sample()
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
        except Exception:
            self.nv = None
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={device_index}", "--query-gpu=clocks.sm,clocks.max.sm,"
                     "clocks_event_reasons.active", "--format=csv,noheader,nounits", "-lms", "20"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except (FileNotFoundError, OSError):
                self.proc = None

    def _sample(self):
        nv = self.nv
        sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
        try:
            bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except AttributeError:
            bits = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        self.rows.append((float(sm), float(self.max_mhz), int(bits)))

    def _loop(self):
        while not self.stop_ev.wait(0.01):
            try:
                self._sample()
            except Exception:
                return

    def stop(self):
        if self.nv is not None:
            self.stop_ev.set()
            self.thread.join(timeout=1)
            try:
                self._sample()
            except Exception:
                pass
            rows = self.rows
        elif self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            rows = []
            for r in out.strip().splitlines():
                f = [x.strip() for x in r.split(",")]
                try:
                    rows.append((float(f[0]), float(f[1]), int(f[2], 16)))
                except (ValueError, IndexError):
                    pass
        else:
            return None
        if not rows:
            return None
        reasons = sorted({n for _, _, b in rows for bit, n in _REASONS.items() if b & bit})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "source": "nvml" if self.nv else "nvidia-smi"}


def spread_blocks(k, lo, hi, max_blocks=16):
    """k decode steps as blocks (start position, steps) whose starts are spread evenly over the
    positions [lo, hi], every block inside the range: at most max_blocks blocks, more only when
    one block would not fit in the range."""
    span = hi - lo + 1
    nb = max(1, min(max_blocks, k), -(-k // span))
    sizes = [k // nb + (1 if b < k % nb else 0) for b in range(nb)]
    out = []
    for b, n in enumerate(sizes):
        last = hi - n + 1                          # latest start that keeps the block in range
        out.append((lo + (round(b * (last - lo) / (nb - 1)) if nb > 1 else 0), n))
    return [(p, n) for p, n in out if n > 0]


def algorithmic_bytes(info, positions):
    """Weights + norm weights + KV rows read + KV row written, per token (embedding row added
    separately). positions: decode positions of the steps."""
    kv = info["block_count"] * info["kv_dim"] * 2 * 2  # K+V fp16 per position per token
    base = info["layer_weight_bytes"] + info["norm_weight_bytes"]
    return [base + kv * (p + 1) + kv for p in positions]


def run_reference(args, rank, world):
    """The reference's own CPU path on this host's cores, rank 0 only: its BaseLM shaders compiled
    as C++ (oracle/_ref, run under a workgroup emulator, the stand-in for the lavapipe run the
    reference would use) when that library was built, else the oracle port."""
    if rank != 0:
        return
    from oracle import oracle as O
    from oracle import ref as R
    from voxgen_b200 import synth
    wl = WORKLOADS[args.workload]
    spec = synth.preset(wl["preset"])
    path = synth.model_path(spec, model_cache())
    shaders = R.LIB.exists()
    if shaders:
        eng = R.RefEngine(path, wl["ctx"])
        kind, what = "reference", "the reference's BaseLM GLSL shaders compiled as C++, workgroups emulated"
        budget, min_steps = float(os.environ.get("VOXGEN_REF_SECONDS", "45")), 2
    else:
        m = O.OracleModel(path)
        eng = O.OracleState(m, wl["ctx"])
        kind, what = "port", "C restatement of the reference shaders"
        budget, min_steps = float(os.environ.get("VOXGEN_REF_SECONDS", "120")), 3
    k, v = synth.kv_prefill(spec, wl["prefill"])
    toks = synth.token_ids(spec, args.warmup + args.steps)
    cores = O.threads()
    # each bench step is one decode token; the run is bounded so that it ends in minutes
    warm = 1 if shaders else min(args.warmup, 3)
    eng.write_kv(k, v)
    for t in toks[:warm]:
        eng.decode_token(int(t))
    eng.write_kv(k, v)
    t0 = time.perf_counter()
    n = 0
    for t in toks[: args.steps]:
        eng.decode_token(int(t))
        n += 1
        if n >= min_steps and time.perf_counter() - t0 > budget:
            break
    el = time.perf_counter() - t0
    val = n / el
    line = {
        "metric": "decode tok/s", "value": val, "unit": "tok/s", "n_gpus": world, "steps": n,
        "warmup": warm, "ms_per_step": 1000 * el / n, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{args.workload}: {wl['desc']}", "positions": [wl["prefill"], wl["prefill"] + n - 1],
                   "streams_per_gpu": 1, "parallelism": "cpu"},
        "cpu_baseline": {"value": val, "unit": "tok/s", "cores": cores, "kind": kind,
                         "sample": f"{n} decode steps from position {wl['prefill']} ({what}, {cores} threads)"},
        "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def cpu_baseline_sample(args, spec, path, wl):
    """The oracle on the host cores, bounded to about args.cpu_seconds of work."""
    from oracle import oracle as O
    from voxgen_b200 import synth
    m = O.OracleModel(path)
    st = O.OracleState(m, wl["ctx"])
    k, v = synth.kv_prefill(spec, wl["prefill"])
    st.write_kv(k, v)
    toks = synth.token_ids(spec, 64)
    st.decode_token(int(toks[0]))  # warm caches
    t0 = time.perf_counter()
    n = 0
    while n < 63 and (n < 2 or time.perf_counter() - t0 < args.cpu_seconds):
        st.decode_token(int(toks[n + 1]))
        n += 1
    el = time.perf_counter() - t0
    return {"value": n / el, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": f"{n} decode steps from position {wl['prefill'] + 1} of {args.workload} "
                      f"({el:.1f} s, C restatement of the reference shaders, OpenMP)"}


def run_residual(args, rank, world, local):
    """ResidualLM positions per second: one step is FSQ(BaseLM hidden) + fusion + the ResidualLM
    layers (an audio position), device-timed over K steps with device-resident inputs; e2e
    copies the step's BaseLM hidden and acoustic embedding from host memory and reads the output
    back. The CPU baseline is the oracle restatement (oracle/residual.py)."""
    import torch

    from voxgen_b200 import api, replicas, synth
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = replicas.init("nccl", world, timeout_s=600, device=dev)
    wl = WORKLOADS[args.workload]
    aspec = synth.acoustic_preset(wl["acoustic"])
    if rank == 0:
        synth.model_path(aspec.base, model_cache())
        synth.acoustic_model_path(aspec, model_cache())
    replicas.barrier(pg)
    bpath = synth.model_path(aspec.base, model_cache())
    apath = synth.acoustic_model_path(aspec, model_cache())
    K, W = args.steps, args.warmup
    ctx = api.Context(local)
    base = api.Model(ctx, bpath)
    res = api.ResidualModel(ctx, apath, base)
    info = res.info
    H = info["embedding_length"]
    eng = api.ResidualEngine(res, max(wl["ctx"], W + K + 8))
    hs = torch.from_numpy(synth.hidden_inputs(aspec.base, 8, seed_index=2000 + rank)).to(dev)
    em = torch.from_numpy(synth.hidden_inputs(aspec.base, 8, seed_index=2100 + rank) * 0.5).to(dev)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(eng.cuda_stream, device=dev)
    for i in range(W):
        eng.step(hs[i % 8].data_ptr(), em[i % 8].data_ptr(), fsq_applied=True)
    eng.sync()
    p0 = eng.position
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replicas.barrier(pg)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    start.record(stream)
    for i in range(K):
        eng.step(hs[i % 8].data_ptr(), em[i % 8].data_ptr(), fsq_applied=True)
    end.record(stream)
    eng.sync(timeout_s=600)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms_max = replicas.max_over_ranks(start.elapsed_time(end), pg, dev)
    # e2e: host inputs in, the output hidden state out, every step
    KE = args.e2e_steps or min(K, 300)
    eng.reset()
    hh = synth.hidden_inputs(aspec.base, 8, seed_index=2000 + rank)
    he = synth.hidden_inputs(aspec.base, 8, seed_index=2100 + rank) * 0.5
    out = np.empty(H, np.float32)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(KE):
        eng.step(hh[i % 8], he[i % 8], fsq_applied=True)
        out[:] = eng.output()
    e_end.record(stream)
    torch.cuda.synchronize()
    e_ms_max = replicas.max_over_ranks(e_start.elapsed_time(e_end), pg, dev)
    # algorithmic bytes of a step: every matrix once (F16), norms, biases, KV rows read and written
    L, F, KV, LAT = info["block_count"], info["feed_forward_length"], info["kv_dim"], aspec.latent
    layer_w = L * 2 * (H * (H + 2 * KV) + H * H + 3 * H * F)
    other_w = 2 * (2 * LAT * H + 2 * H * H) + 4 * (LAT + 2 * H) + 4 * (2 * L + 1) * H
    kv_row = L * KV * 2 * 2
    positions = range(p0, p0 + K)
    avg_bytes = layer_w + other_w + sum(kv_row * (p + 2) for p in positions) / K
    step_ms = ms_max / K
    peak, peak_kind = measured_peaks()
    ach = avg_bytes / (step_ms * 1e-3) / 1e9
    line = {
        "metric": "ResidualLM positions/s", "value": round(world * K / (ms_max / 1e3), 2), "unit": "positions/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(step_ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {wl['desc']}", "weights": "F16",
                   "positions": [p0, p0 + K - 1], "streams_per_gpu": 1,
                   "parallelism": f"replicas x{world} (weights replicated, no collectives)",
                   "l2": f"inputs larger than L2: {layer_w / 1e9:.2f} GB of layer weights per step",
                   "input": "seeded BaseLM hidden states and acoustic embeddings, FSQ on"},
        "roofline": {"kernel": "decode_step_kernel with the FSQ and fusion phases (one launch per position)"
                               if eng.kernel_mode == 1 else
                               "FSQ + fusion matvecs and the ResidualLM layers (whole position)",
                     "bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(ach / peak, 4),
                     "traffic": launch_traffic(args.workload) if eng.kernel_mode == 1 else None,
                     "bytes_per_launch": int(avg_bytes), "peak_source": f"{peak_kind} hbm_gbs"},
        "e2e": {"value": round(world * KE / (e_ms_max / 1e3), 2), "unit": "positions/s", "steps": KE,
                "h2d_bytes_per_step": 2 * H * 4, "d2h_bytes_per_step": H * 4},
        "gpu_launches": K * (1 if eng.kernel_mode == 1 else 4 + 5 * L + 1),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        from oracle.residual import ResidualOracle
        o = ResidualOracle(apath, bpath, KE + 8)
        o.step(hh[0], he[0], True)
        n, c0 = 0, time.perf_counter()
        while n < 2 or (time.perf_counter() - c0 < args.cpu_seconds and n < KE):
            o.step(hh[n % 8], he[n % 8], True)
            n += 1
        el = time.perf_counter() - c0
        line["cpu_baseline"] = {"value": n / el, "unit": "positions/s", "cores": O.threads(), "kind": "port",
                                "sample": f"{n} ResidualLM positions ({el:.1f} s, oracle restatement, OpenMP)"}
    eng.close()
    res.close()
    base.close()
    ctx.close()
    if rank == 0:
        emit(line)
    replicas.barrier(pg)
    replicas.shutdown(pg)


def run_batch(args, rank, world, local):
    """cfg4: S streams per GPU over one model, each with its own KV cache prefilled to a seeded
    ragged length ~U[64, 4096]. A step advances every stream by one token through
    vg_decode_batch: one launch of the batched step kernel reads the weights once for all the
    streams (or, for a model that kernel does not take, one step-kernel launch per stream).
    value = tokens of all streams on all ranks / device time (events on every engine stream, max
    over streams and ranks). e2e copies the S token ids from host memory and reads the S output
    hidden states back every step, with one wait for all of them (vg_copy_outputs)."""
    import torch

    from voxgen_b200 import api, replicas, synth
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = replicas.init("nccl", world, timeout_s=600, device=dev)

    def barrier():
        replicas.barrier(pg)

    wl = WORKLOADS[args.workload]
    spec = synth.preset(wl["preset"])
    path = ensure_model(spec, rank, world, barrier)
    K, W, S = args.steps, args.warmup, wl["streams"]
    KE = args.e2e_steps or min(K, 20)
    lens = np.random.default_rng([4, rank]).integers(64, wl["ctx"] + 1, size=S)
    max_ctx = int(max(wl["ctx"] + wl["slack"], lens.max() + W + K + KE + 1))
    ctx = api.Context(local)
    model = api.Model(ctx, path)
    info = model.info
    batched = model.batch_columns >= S
    engs = [api.BaseLmEngine(model, max_ctx) for _ in range(S)]
    kpre, vpre = synth.kv_prefill(spec, int(lens.max()))

    def prefill():
        for e, n in zip(engs, lens):
            e.write_kv(kpre[:, :n], vpre[:, :n])

    toks = synth.token_ids(spec, (W + K + KE) * S, seed_index=4000 + rank).reshape(W + K + KE, S)
    streams = [torch.cuda.ExternalStream(e.cuda_stream, device=dev) for e in engs]

    def timed(rows, read_back):
        start = torch.cuda.Event(enable_timing=True)
        ends = [torch.cuda.Event(enable_timing=True) for _ in engs]
        barrier()
        torch.cuda.synchronize()
        start.record(torch.cuda.current_stream())
        for st in streams:
            st.wait_event(start)
        for row in rows:
            api.decode_batch(engs, [int(t) for t in row])   # S token ids from host memory
            if read_back:
                api.outputs(engs)                             # D2H of every stream's hidden state, one wait
        for st, ev in zip(streams, ends):
            ev.record(st)
        for e in engs:
            e.sync(timeout_s=600)
        torch.cuda.synchronize()
        barrier()
        return max(start.elapsed_time(ev) for ev in ends)

    prefill()
    for row in toks[:W]:
        api.decode_batch(engs, [int(t) for t in row])
    for e in engs:
        e.sync()
    p0 = [e.position for e in engs]
    clocks = ClockSampler(local)
    ms = timed(toks[W:W + K], False)
    clk = clocks.stop()
    ms_max = replicas.max_over_ranks(ms, pg, dev)
    prefill()
    e_ms_max = replicas.max_over_ranks(timed(toks[W + K:W + K + KE], True), pg, dev)

    peak, peak_kind = measured_peaks()
    kv = info["block_count"] * info["kv_dim"] * 2 * 2
    wbytes = info["layer_weight_bytes"] + info["norm_weight_bytes"]
    emb = S * info["embedding_length"] * 2                                   # the S token-table rows
    kv_step = sum(kv * (p + j + 1) + kv for p in p0 for j in range(K)) / K   # all streams, per step
    step_ms = ms_max / K
    # per batched step, counting the weights once (the roofline of a shared weight pass)
    batch_bytes = wbytes + kv_step + emb
    batch_ach = batch_bytes / (step_ms * 1e-3) / 1e9
    if batched:
        # one launch per step reads the weights once and every stream's KV
        launch_bytes, launch_ach, launches = batch_bytes, batch_ach, K
        kname = (f"decode_batch_kernel (one launch per step for all {S} streams, every weight byte read once; "
                 f"split-K over CTAs, fp16 hi+lo operand, f16 mma.sync)")
    else:
        # per launch of the step kernel (one stream's token): its weights and that stream's KV
        launch_bytes = wbytes + kv_step / S
        launch_ach = launch_bytes * S / (step_ms * 1e-3) / 1e9
        launches = K * S
        kname = "decode_step_kernel (one launch per stream token; the weight pass is not shared between streams)"
    line = {
        "metric": "decode tok/s", "value": round(replicas.aggregate_rate(K * S, world, ms_max), 2),
        "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(step_ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"{args.workload}: {wl['desc']}", "weights": "Q8_0", "streams_per_gpu": S,
            "kv_lengths": [int(x) for x in lens], "step": f"one token for each of the {S} streams",
            "parallelism": f"replicas x{world} (weights replicated, streams partitioned, no collectives)",
            "l2": (f"inputs larger than L2: {info['layer_weight_bytes'] / 1e9:.2f} GB of weights per batched step"
                   if batched else
                   f"inputs larger than L2: {info['layer_weight_bytes'] / 1e9:.2f} GB of weights per stream token"),
            "input": "seeded token ids",
        },
        "roofline": {"kernel": kname, "bound": "hbm", "achieved": round(launch_ach, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(launch_ach / peak, 4),
                     "traffic": launch_traffic(args.workload, "decode_batch_kernel" if batched else "decode_step_kernel"),
                     "bytes_per_launch": int(launch_bytes),
                     "avg_launch_ms": round(step_ms * K / launches, 5), "peak_source": f"{peak_kind} hbm_gbs"},
        "batch_roofline": {"bytes_per_step": int(batch_bytes), "achieved": round(batch_ach, 1), "peak": peak,
                           "unit": "GB/s", "frac": round(batch_ach / peak, 4),
                           "note": "weights counted once per batched step"},
        "e2e": {"value": round(replicas.aggregate_rate(KE * S, world, e_ms_max), 2), "unit": "tok/s",
                "steps": KE, "h2d_bytes_per_step": 4 * S,
                "d2h_bytes_per_step": S * info["embedding_length"] * 4},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        mean_len = int(np.mean(lens))
        line["cpu_baseline"] = cpu_baseline_sample(args, spec, path, {"ctx": mean_len + 80, "prefill": mean_len})
        line["cpu_baseline"]["sample"] += f"; the {S} streams would run one after another"
    for e in engs:
        e.close()
    model.close()
    ctx.close()
    if rank == 0:
        emit(line)
    replicas.barrier(pg)
    replicas.shutdown(pg)


def run_prefill(args, rank, world, local):
    """Prompt tokens per second through vg_prefill_tokens: one step is a whole prompt from
    position 0, runs of up to 16 positions per launch of the batched kernel (one weight pass
    each). Device-timed with events on the engine's stream; e2e passes the prompt from host
    memory through the public call and reads the final hidden state back. The same prompt decoded
    one token per step (the batched kernel switched off for a second copy of the model) is timed
    beside it."""
    import ctypes

    import torch

    from voxgen_b200 import api, replicas, synth
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = replicas.init("nccl", world, timeout_s=600, device=dev)

    def barrier():
        replicas.barrier(pg)

    wl = WORKLOADS[args.workload]
    spec = synth.preset(wl["preset"])
    path = ensure_model(spec, rank, world, barrier)
    n, K, W = wl["prompt"], args.steps, args.warmup
    toks = np.ascontiguousarray(synth.token_ids(spec, n, seed_index=3500 + rank), np.uint32)
    tp = toks.ctypes.data_as(ctypes.c_void_p)
    ctx = api.Context(local)
    L = api.lib()

    def timed(model, reps, e2e):
        eng = api.BaseLmEngine(model, n + 8)
        stream = torch.cuda.ExternalStream(eng.cuda_stream, device=dev)
        out = np.empty(model.info["embedding_length"], np.float32)
        for _ in range(W):
            eng.reset()
            ctx.check(L.vg_prefill_tokens(eng.h, tp, n, 0))
        eng.sync()
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            eng.reset()
            ctx.check(L.vg_prefill_tokens(eng.h, tp, n, 0))
            if e2e:
                out[:] = eng.output()
        b.record(stream)
        eng.sync(timeout_s=600)
        torch.cuda.synchronize()
        barrier()
        ms = replicas.max_over_ranks(a.elapsed_time(b), pg, dev)
        eng.close()
        return ms

    model = api.Model(ctx, path)
    info = model.info
    cols = model.batch_columns
    clocks = ClockSampler(local)
    ms = timed(model, K, False)
    clk = clocks.stop()
    e_ms = timed(model, max(1, min(K, 20)), True)
    model.close()
    os.environ["VOXGEN_BATCH_KERNEL"] = "0"     # the same prompt, one decode step per token
    seq_model = api.Model(ctx, path)
    seq_reps = max(1, min(K, 5))
    seq_ms = timed(seq_model, seq_reps, False)
    seq_model.close()
    del os.environ["VOXGEN_BATCH_KERNEL"]
    passes = -(-n // cols) if cols else n
    kv = info["block_count"] * info["kv_dim"] * 2 * 2
    wbytes = info["layer_weight_bytes"] + info["norm_weight_bytes"]
    byt = passes * wbytes + sum(kv * (p + 1) + kv for p in range(n)) + n * info["embedding_length"] * 2
    step_ms = ms / K
    peak, peak_kind = measured_peaks()
    ach = byt / (step_ms * 1e-3) / 1e9
    line = {
        "metric": "prefill tok/s", "value": round(world * n * K / (ms / 1e3), 2), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.workload}: {wl['desc']}", "prompt_tokens": n, "positions_per_pass": cols,
                   "weight_passes_per_prompt": passes, "streams_per_gpu": 1,
                   "parallelism": f"replicas x{world} (weights replicated, no collectives)",
                   "l2": f"inputs larger than L2: {wbytes / 1e9:.2f} GB of weights per pass",
                   "input": "seeded token ids"},
        "roofline": {"kernel": "decode_batch_kernel (up to 16 positions per launch)", "bound": "hbm",
                     "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                     "traffic": None, "bytes_per_launch": int(byt / passes),
                     "avg_launch_ms": round(step_ms / passes, 5), "peak_source": f"{peak_kind} hbm_gbs"},
        "one_token_per_step": {"value": round(world * n * seq_reps / (seq_ms / 1e3), 2),
                               "unit": "tok/s", "note": "the same prompt through one decode step per token"},
        "e2e": {"value": round(world * n * max(1, min(K, 20)) / (e_ms / 1e3), 2), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * n + 960 * passes, "d2h_bytes_per_step": info["embedding_length"] * 4},
        "gpu_launches": K * passes,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(args, spec, path, {"ctx": n + 80, "prefill": 0})
        line["cpu_baseline"]["sample"] += "; a prompt is prefilled one decode step per token"
    ctx.close()
    if rank == 0:
        emit(line)
    replicas.barrier(pg)
    replicas.shutdown(pg)


def main():
    args = parse()
    quiet_stdout()
    rank, world, local = dist_env()
    if args.workload == "cfg4" and args.impl == "ours":
        run_batch(args, rank, world, local)
        return
    if args.workload.startswith("prefill"):
        if args.impl == "reference":
            if rank == 0:
                emit({"impl": "reference", "unavailable":
                      "the prefill workloads have no reference CPU arm (the reference arm covers BaseLM decode)"})
            return
        run_prefill(args, rank, world, local)
        return
    if args.workload == "residual":
        if args.impl == "reference":
            if rank == 0:
                emit({"impl": "reference", "unavailable":
                      "the ResidualLM workload has no reference CPU arm (the reference arm covers BaseLM)"})
            return
        run_residual(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch

    from voxgen_b200 import api, replicas, synth

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = replicas.init("nccl", world, timeout_s=600, device=dev)

    def barrier():
        replicas.barrier(pg)

    wl = WORKLOADS[args.workload]
    spec = synth.preset(wl["preset"])
    path = ensure_model(spec, rank, world, barrier)
    K, W = args.steps, args.warmup
    lo, hi = wl["span"]
    max_ctx = max(wl["ctx"], hi + 1)

    ctx = api.Context(local)
    model = api.Model(ctx, path)
    info = model.info
    eng = api.BaseLmEngine(model, max_ctx)
    kpre, vpre = synth.kv_prefill(spec, hi)
    toks = synth.token_ids(spec, W + max(K, args.e2e_steps or 0), seed_index=3000 + rank)
    stream = torch.cuda.ExternalStream(eng.cuda_stream, device=torch.device("cuda", local))

    # ---- device-timed decode: W warm-up steps, then K timed steps spread over the span ----
    # The cache holds seeded rows up to the end of the span, and the K steps run in blocks
    # that start at evenly spaced positions (vg_stream_seek between blocks, inside the timed
    # region), so the rate represents the whole context range the config decodes over.
    eng.write_kv(kpre, vpre)
    eng.seek(lo)
    for t in toks[:W]:
        eng.decode_token_gpu_only(int(t))
    eng.sync()
    blocks = spread_blocks(K, lo, hi)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    start.record(stream)
    i = W
    for b0, n in blocks:
        eng.seek(b0)
        for t in toks[i:i + n]:
            eng.decode_token_gpu_only(int(t))
        i += n
    end.record(stream)
    eng.sync(timeout_s=600)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = start.elapsed_time(end)
    ms_max = replicas.max_over_ranks(ms, pg, dev)
    positions = [b0 + j for b0, n in blocks for j in range(n)]

    # ---- e2e through the C ABI with host buffers, over the same spread of positions ----
    KE = args.e2e_steps or min(K, 500)
    e_blocks = spread_blocks(KE, lo, hi)
    host_out = np.empty(info["embedding_length"], np.float32)
    eng.seek(lo)
    for t in toks[:min(W, 5)]:
        eng.decode_token_gpu_only(int(t))
        eng.output()
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    i = W
    for b0, n in e_blocks:
        eng.seek(b0)
        for t in toks[i:i + n]:
            eng.decode_token_gpu_only(int(t))          # token id copied from pinned host memory
            host_out[:] = eng.output()                  # D2H of the final hidden state + sync
        i += n
    e_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    e_ms = e_start.elapsed_time(e_end)
    e_ms_max = replicas.max_over_ranks(e_ms, pg, dev)

    # ---- roofline of the dominant kernel ----
    # Persistent mode (kernel_mode 1): the step is one kernel launch, so the dominant kernel is
    # the step kernel itself: algorithmic bytes of a step / its device time (the events above
    # bracket exactly the K launches). Per-kernel mode: gate_up from one instrumented step.
    roof = None
    peak, peak_kind = measured_peaks()
    peak_src = f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback 6650 GB/s"
    mode = eng.kernel_mode
    prof = None
    traffic = {}
    tr = ROOT / "profiles" / "traffic.json"
    if tr.exists():
        traffic = json.loads(tr.read_text()).get(args.workload, {})
    if mode == 1:
        byt = int(sum(algorithmic_bytes(info, positions)) / K)
        avg_ms = ms_max / K
        ach = byt / (avg_ms * 1e-3) / 1e9
        roof = {"kernel": "decode_step_kernel (persistent, the whole decode step)", "bound": "hbm",
                "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "traffic": traffic.get("decode_step_kernel"), "bytes_per_launch": byt,
                "avg_launch_ms": round(avg_ms, 5), "peak_source": peak_src}
    elif not args.no_profile:
        eng.seek(lo)
        for t in toks[:3]:
            eng.profile_step(int(t))       # warm
        eng.seek(lo)
        prof = [eng.profile_step(int(t)) for t in toks[3:8]]
        rows = [r for step in prof for r in step if r["name"] == "gate_up"]
        avg_ms = sum(r["ms"] for r in rows) / len(rows)
        byt = rows[0]["bytes"]
        ach = byt / (avg_ms * 1e-3) / 1e9
        roof = {"kernel": "gate_up (fused gate/up matvec + SwiGLU)", "bound": "hbm", "achieved": round(ach, 1),
                "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4), "traffic": traffic.get("gate_up"),
                "bytes_per_launch": byt, "avg_launch_ms": round(avg_ms, 5), "peak_source": peak_src}

    # ---- whole-step numbers ----
    bytes_tok = algorithmic_bytes(info, positions)
    emb_row = info["embedding_length"] * 2
    avg_bytes = (sum(bytes_tok) / K) + emb_row
    step_ms = ms_max / K
    value = replicas.aggregate_rate(K, world, ms_max)
    e2e_val = replicas.aggregate_rate(KE, world, e_ms_max)
    line = {
        "metric": "decode tok/s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(step_ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {
            "workload": f"{args.workload}: {wl['desc']}",
            "weights": "Q8_0" if info["format"] == 8 else "F16",
            "compute": ("Q8_0: activation as three int8 digits with one shared power of two per vector, "
                        "exact s8 MMA (mma.sync), fp32 rescale by the fp16 block scales"
                        if info["format"] == 8 else
                        "F16: activation as fp16 hi + lo with one shared power of two per vector, "
                        "f16 MMA (mma.sync) with fp32 accumulation"),
            "streams_per_gpu": 1, "positions": [[b0, b0 + n - 1] for b0, n in blocks],
            "position_sampling": (f"{K} timed steps in {len(blocks)} blocks whose starts are spread evenly over "
                                  f"positions {lo}-{hi} (vg_stream_seek between blocks, inside the timed region; "
                                  f"the cache holds seeded rows below every position)"),
            "parallelism": f"replicas x{world} (weights replicated, no collectives)",
            "l2": f"inputs larger than L2: {info['layer_weight_bytes'] / 1e9:.2f} GB of weights per step",
            "input": "seeded token ids",
        },
        "per_stream_tok_s": round(K / (ms_max / 1e3), 2),
        "step_roofline": {"bound": "hbm", "bytes_per_token": int(avg_bytes),
                          "achieved": round(avg_bytes / (step_ms * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                          "frac": round(avg_bytes / (step_ms * 1e-3) / 1e9 / peak, 4)},
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 2), "unit": "tok/s", "steps": KE, "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": info["embedding_length"] * 4 + 64},
        "gpu_launches": K * (1 if mode == 1 else 5 * info["block_count"] + 2),
        "kernel_mode": "persistent step kernel" if mode == 1 else "one kernel per projection / attention / norm",
        "clocks": clk,
    }
    if prof:
        agg = {}
        for step in prof:
            for r in step:
                a = agg.setdefault(r["name"], [0.0, 0, 0])
                a[0] += r["ms"]
                a[1] += 1
                a[2] = r["bytes"]
        line["kernels"] = {n: {"avg_ms": round(a[0] / a[1], 5), "launches_per_step": a[1] // len(prof),
                               "gbs": round(a[2] / (a[0] / a[1] * 1e-3) / 1e9, 1)} for n, a in agg.items()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(args, spec, path, wl)
    eng.close()
    model.close()
    ctx.close()
    if rank == 0:
        emit(line)
    replicas.barrier(pg)
    replicas.shutdown(pg)


if __name__ == "__main__":
    main()

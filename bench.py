#!/usr/bin/env python3
"""Headline benchmark: batched Llama-3.1-8B decode on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (config 4): B=16 streams, S=512 cache, per-stream past length
U[64, 384] (seed 3) so that 128 more steps fit, seeded bf16 KV ~N(0,1), token
ids U[0, 128256) (seed 2), random-init bf16 weights ~N(0, 0.02) (seed 0).
A step is one batched decode step (32 layers + lm_head + greedy argmax) for
the 16 streams.  Weights (15.0 GB/step) are far larger than L2, so no flush is
needed between steps.

  value    16 * K / device time of K steps with inputs resident in HBM
           (CUDA-graph replays that feed each argmax back as the next token)
  e2e      the same through the public API BatchDecodeEngine.step(): host
           token/position lists in (pinned H2D), next tokens out (D2H), per step
  N > 1    one independent replica per GPU (decode does not shard),
           value = all ranks' tokens / max-over-ranks device time

--impl reference times the CPU fp32 path (the test oracle's C restatement of
the reference's cpu_layer, on all host cores) on the same workload; rank 0
only under torchrun.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "rngd-pd_b200"))
sys.path.insert(0, REPO)

METRIC = "decode tok/s/GPU (Llama-3.1-8B, B=16, S=512); KV handoff GB/s over NVLink"
B, S = 16, 512
WEIGHT_BYTES = 15_009_316_864
KV_BYTES_PER_POS = 131_072          # K+V, 32 layers x 8 heads x 128 x 2 B x 2
WORKLOAD = "config4: batched decode B=16 S=512, past lengths U[64,384] (seed 3)"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def lengths_and_tokens():
    # the same integer recipe as rngd_pd.synth (numpy copy so the reference arm needs no GPU)
    from oracle import synth_np as sy
    lens = [64 + int(v) for v in sy.uniform_ints(3, sy.T_CTXLEN, B, 384 - 64 + 1)]
    toks = [int(v) for v in sy.uniform_ints(2, sy.T_TOKENS, B, 128256)]
    return lens, toks


class Clocks:
    """nvidia-smi sampling during the timed region (the recipe's clocks line)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        self.p.wait()
        rows = [r.split(",") for r in open(self.f.name).read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_steps(n_steps, warmup):
    """The CPU fp32 path (C restatement of the reference's cpu_layer) on all host cores."""
    from oracle import corc
    from oracle.ref_np import LLAMA8B
    lens, toks = lengths_and_tokens()
    corc.set_threads(len(os.sched_getaffinity(0)))
    m = corc.CModel(LLAMA8B, seed=0)
    Kc, Vc = m.new_cache(B, S)
    for b in range(B):
        m.fill_lane(Kc, Vc, b, 100 + b, lens[b])
    pos = list(lens)
    times = []
    for i in range(warmup + n_steps):
        t0 = time.perf_counter()
        nxt, _, _ = m.decode_step(toks, pos, Kc, Vc, want_logits=False)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
        toks, pos = [int(t) for t in nxt], [p + 1 for p in pos]
    m.close()
    return times, corc.threads()


def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    times, cores = cpu_reference_steps(args.steps, args.warmup)
    step_s = sum(times) / len(times)
    v = B / step_s
    sample = f"{len(times)} full decode steps (32 layers + lm_head, B=16, S=512) after {args.warmup} warm-up"
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": B, "seq_len": S, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def gemv_roofline(eng, reps=20):
    """Dominant kernel (the decode GEMV) timed alone with CUDA events on its stream."""
    import torch
    from rngd_pd import _lib
    w = eng.w
    c = eng.cfg
    H, M = c.hidden, c.inter
    shapes = {"gate_up": (w.wgu[0], 2 * M, H), "qkv": (w.wqkv[0], w.NQKV, H), "o": (w.wo[0], H, H),
              "down": (w.wd[0], H, M)}
    X = torch.randn(B, max(H, M), device=eng.dev)
    Y = torch.empty(B, 2 * M, device=eng.dev)
    s = torch.cuda.current_stream(eng.dev)
    h = _lib.stream_handle(s)
    out = {}
    for name, (Wt, N, K) in shapes.items():
        Wl = [eng.w.wgu[l] if name == "gate_up" else (eng.w.wqkv[l] if name == "qkv" else
              (eng.w.wo[l] if name == "o" else eng.w.wd[l])) for l in range(c.n_layers)]
        for i in range(3):
            _lib.call("rngd_gemv_bf16", _lib.ptr(Wl[i]), N, K, _lib.ptr(X), max(H, M), B, _lib.ptr(Y), N, 0, h)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(reps):   # rotate layers: each launch reads cold weights
            _lib.call("rngd_gemv_bf16", _lib.ptr(Wl[i % c.n_layers]), N, K, _lib.ptr(X), max(H, M), B,
                      _lib.ptr(Y), N, 0, h)
        e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / reps
        nbytes = N * K * 2 + B * K * 4 + B * N * 4
        out[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6}
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist
    from rngd_pd import synth
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = ModelConfig.llama31_8b()
    eng = BatchDecodeEngine(cfg, synth.SyntheticState(cfg, seed=0), B=B, S=S, group=8, chip=local)
    lens, toks0 = lengths_and_tokens()
    Ks, Vs = zip(*[synth.request_kv(cfg, S, 100 + b, lens[b], device=dev) for b in range(B)])
    Kd, Vd = eng.adopt_kv_device(list(Ks), list(Vs))
    del Ks, Vs
    max_steps = S - max(lens) - 1            # positions must stay inside the cache

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---------------------------------------------------- value: device loop
    eng.step(toks0, lens, Kd, Vd)            # builds + captures the step graph
    W, K = args.warmup, args.steps
    if W + K > max_steps:
        raise SystemExit(f"--warmup + --steps must be <= {max_steps} (cache positions)")
    eng.set_inputs(toks0, lens)
    eng.step_device(Kd, Vd, W)
    barrier()
    clocks = Clocks() if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(eng.stream)
    eng.step_device(Kd, Vd, K)
    e1.record(eng.stream)
    barrier()
    clk = clocks.stop() if clocks else None
    ms_total = e0.elapsed_time(e1)
    t = torch.tensor([ms_total], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / K
    value = world * B * K / (ms_total / 1e3)
    mid_pos = [l + W + K // 2 for l in lens]
    kv_bytes = sum(p + 1 for p in mid_pos) * KV_BYTES_PER_POS + B * KV_BYTES_PER_POS
    step_bytes = WEIGHT_BYTES + kv_bytes

    # ------------------------------------------------- e2e: public step() API
    toks, pos = list(toks0), list(lens)
    for _ in range(3):
        toks, Kd, Vd = eng.step(toks, pos, Kd, Vd)
        pos = [p + 1 for p in pos]
    toks, pos = list(toks0), list(lens)
    barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        toks, Kd, Vd = eng.step(toks, pos, Kd, Vd)
        pos = [p + 1 for p in pos]
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())

    roof = gemv_roofline(eng) if rank == 0 else None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    import json as _j
    peaks = {}
    try:
        peaks = _j.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    peak_kind = "measured" if "hbm_gbs" in peaks else "fallback"
    dom = roof["gate_up"]
    traffic = None
    try:
        traffic = _j.load(open(os.path.join(REPO, "profiles", "traffic.json"))).get("gemv_gate_up")
    except (OSError, ValueError):
        pass
    cpu = None
    if not args.no_cpu_baseline:
        times, cores = cpu_reference_steps(1, 0)
        cpu = {"value": B / times[0], "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": "1 full decode step (32 layers + lm_head, B=16, S=512) of the C restatement"}
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": B * world, "seq_len": S,
                   "parallelism": f"replicas x{world}", "per_gpu_tok_s": value / world,
                   "l2": "no flush: 15.0 GB of weights per step >> 126 MB L2"},
        "step_roofline": {"bound": "hbm", "bytes_per_step": step_bytes,
                          "achieved": step_bytes / (ms_step / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                          "frac": step_bytes / (ms_step / 1e3) / 1e9 / hbm, "peak_kind": peak_kind},
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel (gate/up 28672x4096, B=16)",
                     "achieved": dom["gbs"], "peak": hbm, "unit": "GB/s", "frac": dom["gbs"] / hbm,
                     "traffic": traffic, "peak_kind": peak_kind,
                     "per_shape": {k: round(v["gbs"], 1) for k, v in roof.items()}},
        "cpu_baseline": cpu,
        "clocks": clk,
        "e2e": {"value": world * B * K / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 2 * B * 4,
                "d2h_bytes_per_step": B * 4},
        "gpu_launches": eng.launches_per_step * K,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

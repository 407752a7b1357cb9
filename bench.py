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
  N > 1    one independent replica per GPU (decode does not shard: every GPU holds
           the whole model and its own streams), value = all ranks' tokens /
           max-over-ranks device time

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


def lengths_and_tokens(cpu=False):
    """Config 4's past lengths U[64, 384] (seed 3) and first tokens (seed 2).  The GPU arm draws
    them with the package's device generator; the CPU reference arm (no GPU) with the test
    oracle's numpy copy of the same integer recipe."""
    if cpu:
        from oracle import synth_np as sy
        lens = [64 + int(v) for v in sy.uniform_ints(3, sy.T_CTXLEN, B, 384 - 64 + 1)]
        toks = [int(v) for v in sy.uniform_ints(2, sy.T_TOKENS, B, 128256)]
        return lens, toks
    from rngd_pd import synth
    return synth.context_lengths(B, 3, 64, 384), synth.tokens(B, 2, 128256)


class Clocks:
    """nvidia-smi sampling during the timed region (the recipe's clocks line)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
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
    lens, toks = lengths_and_tokens(cpu=True)
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
        "handoff": {"cpu_baseline": handoff_cpu_baseline()},
    }), flush=True)


class TcGemm:
    """One decode GEMM shape through rngd_tc_gemv: weights [L][N][K], the hi/lo operand prepared once."""

    def __init__(self, weights, N, K, dev):
        import ctypes
        import torch
        from rngd_pd import _lib
        self.W, self.N, self.K = weights, N, K
        pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.call("rngd_tc_gemv_workspace", N, K, ctypes.byref(pf), ctypes.byref(ct))
        self.X = torch.randn(B, K, device=dev)
        self.Y = torch.zeros(B, N, device=dev)
        self.act = torch.zeros(32, K, dtype=torch.bfloat16, device=dev)
        self.part = torch.zeros(max(pf.value, 1), device=dev)
        self.cnt = torch.zeros(max(ct.value, 1), dtype=torch.int32, device=dev)
        self.run(0, prep=1)
        self.nbytes = N * K * 2 + 32 * K * 2 + B * N * 4 * 2   # weights + operand + y read/write

    def run(self, layer, prep=0, stream=None):
        from rngd_pd import _lib
        _lib.call("rngd_tc_gemv", _lib.ptr(self.W[layer]), self.N, self.K, _lib.ptr(self.X), self.K, B,
                  _lib.ptr(self.Y), self.N, _lib.ptr(self.act), _lib.ptr(self.part), _lib.ptr(self.cnt), prep,
                  _lib.stream_handle(stream))

    def time(self, reps, stream, trace=None):
        """Mean launch duration (ms) over `reps` back-to-back launches (captured in a CUDA graph so host
        launch cost does not gate short kernels), rotating through the layers so weights are cold.
        trace: optional int64 device buffer [reps][1024][16] for per-launch CTA timelines."""
        import torch
        from rngd_pd import _lib
        L = len(self.W)
        if trace is not None:        # raises before any capture when the library has no tracing
            _lib.call("rngd_tc_gemv_trace", _lib.ptr(trace[0]))
            _lib.call("rngd_tc_gemv_trace", None)
        side = torch.cuda.Stream(device=self.X.device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for i in range(3):
                self.run(i % L, stream=side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                for i in range(reps):
                    if trace is not None:
                        _lib.call("rngd_tc_gemv_trace", _lib.ptr(trace[i]))
                    self.run(i % L, stream=side)
            if trace is not None:
                _lib.call("rngd_tc_gemv_trace", None)
            g.replay()                                   # warm
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(side)
            g.replay()
            e1.record(side)
        e1.synchronize()
        stream.wait_stream(side)
        return e0.elapsed_time(e1) / reps


def gemm_roofline(eng, reps=32):
    """The dominant kernel (the tcgen05 decode GEMM, skgemm_kernel) per weight shape, CUDA events on its stream."""
    import torch
    w, c = eng.w, eng.cfg
    H, M = c.hidden, c.inter
    s = torch.cuda.current_stream(eng.dev)
    out = {}
    for name, W, N, K in (("gate_up", w.wgu, 2 * M, H), ("qkv", w.wqkv, w.NQKV, H), ("o", w.wo, H, H),
                          ("down", w.wd, H, M)):
        g = TcGemm(W, N, K, eng.dev)
        ms = g.time(reps, s)
        out[name] = {"ms": ms, "bytes": g.nbytes, "gbs": g.nbytes / ms / 1e6}
        del g
    return out


def run_micro_attn(args):
    """The decode attention (split-S partials + combine) for one layer at config 4's lengths."""
    import torch
    from rngd_pd import _lib
    dev = torch.device("cuda", 0)
    NH, NKV, HD = 32, 8, 128
    lens, _ = lengths_and_tokens()
    pos = torch.tensor([l + 64 for l in lens], dtype=torch.int32, device=dev)
    layers = 8                                       # rotate layers: 8 x 33.5 MB of cache > L2
    K = torch.randn(layers, B, NKV, S, HD, device=dev).to(torch.bfloat16)
    V = torch.randn(layers, B, NKV, S, HD, device=dev).to(torch.bfloat16)
    q = torch.randn(B, NH * HD, device=dev)
    part = torch.empty(B, NH, S // 128, HD + 2, device=dev)
    ao = torch.empty(B, NH * HD, device=dev)
    side = torch.cuda.Stream(device=dev)
    def run(l, st):
        _lib.call("rngd_attn_decode", _lib.ptr(q), _lib.ptr(K[l]), _lib.ptr(V[l]), _lib.ptr(pos), B, B, NH, NKV, HD,
                  S, _lib.ptr(part), _lib.ptr(ao), _lib.stream_handle(st))
    with torch.cuda.stream(side):
        for l in range(3):
            run(l, side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(args.steps):
                run(i % layers, side)
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(side)
        g.replay()
        e1.record(side)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    nbytes = sum(int(p) + 1 for p in pos.tolist()) * NKV * HD * 2 * 2
    print(json.dumps({"micro": "attn", "B": B, "S": S, "ms": ms, "kv_bytes": nbytes, "gbs": nbytes / ms / 1e6}),
          flush=True)


def run_micro_prefill(args):
    """One prefill GEMM shape (C=256 tokens) through rngd_tc_gemm_tokens (pfgemm_kernel)."""
    import ctypes
    import torch
    from rngd_pd import _lib, synth
    shapes = {"pf_gate_up": (28672, 4096), "pf_qkv": (6144, 4096), "pf_o": (4096, 4096), "pf_down": (4096, 14336)}
    N, K = shapes[args.micro]
    C = 256
    dev = torch.device("cuda", 0)
    W = torch.empty((2, N, K), dtype=torch.bfloat16, device=dev)
    synth.fill_gauss(W, 0, 4, 0.02)
    X = torch.randn(C, K, device=dev)
    Y = torch.zeros(C, N, device=dev)
    act = torch.zeros(2 * C, K, dtype=torch.bfloat16, device=dev)
    pf, ct = ctypes.c_size_t(0), ctypes.c_size_t(0)
    _lib.call("rngd_tc_gemm_tokens_workspace", N, K, C, ctypes.byref(pf), ctypes.byref(ct))
    part = torch.zeros(max(pf.value, 1), device=dev)
    cnt = torch.zeros(max(ct.value, 1), dtype=torch.int32, device=dev)
    def run(l, prep, st):
        _lib.call("rngd_tc_gemm_tokens", _lib.ptr(W[l]), N, K, _lib.ptr(X), C, _lib.ptr(Y), _lib.ptr(act),
                  _lib.ptr(part), _lib.ptr(cnt), prep, _lib.stream_handle(st))
    side = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(side):
        run(0, 1, side)
        for i in range(3):
            run(i % 2, 0, side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(args.steps):
                run(i % 2, 0, side)
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(side)
        g.replay()
        e1.record(side)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    flops = 2 * 2 * C * N * K                      # hi and lo operand rows
    print(json.dumps({"micro": args.micro, "N": N, "K": K, "C": C, "ms": ms, "tflops_mma": flops / ms / 1e9,
                      "weight_gbs": N * K * 2 / ms / 1e6, "status": _lib.device_status()}), flush=True)


HANDOFF_BATCHES = (1, 4, 16)
NVLINK_NOMINAL_GBS = 900.0     # NVLink 5, per direction per GPU (nominal; the measured copy is taken in the run)


def handoff_bytes(cfg):
    """Config 3's unit: one 512-token request, K and V of every layer and head, bf16."""
    return cfg.n_layers * 2 * cfg.n_kv * S * cfg.head_dim * 2


def handoff_cpu_baseline():
    """The reference's host-staged handoff of one 512-token request on the host (the connector's
    bf16 wire: ser -> /dev/shm file -> deser, per layer k and v), restated in
    rngd_pd.connector.transport; GB/s of payload."""
    import numpy as np
    from rngd_pd.connector import transport as tr
    from rngd_pd.engines.model import ModelConfig
    cfg = ModelConfig.llama31_8b()
    rng = np.random.default_rng(5)
    shape = (cfg.n_kv, S, cfg.head_dim)
    k = (rng.standard_normal(shape, dtype=np.float32).view(np.uint32) >> 16 << 16).view(np.float32)
    root = tempfile.mkdtemp(dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else None)
    t = tr.ShmTransport(root)
    t0 = time.perf_counter()
    for l in range(cfg.n_layers):
        for kv in ("k", "v"):
            key = f"req/layer.{l}/{kv}"
            t.push(key, tr.ser(k, wire="bf16"))
            out = tr.deser(t.pull(key, timeout=5))
            os.unlink(t._path(key))
    dt = time.perf_counter() - t0
    os.rmdir(root)
    assert out.shape == shape
    return {"value": handoff_bytes(cfg) / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": "1 request of 512 tokens (64 layer tensors): ser bf16 -> /dev/shm -> deser"}


def run_micro_handoff(args):
    import torch
    dsts = [0] + ([1] if torch.cuda.device_count() > 1 else [])
    out = handoff_one_process(dsts, args.steps, args.warmup)
    print(json.dumps({"micro": "handoff", "unit": "GB/s", "results": out}), flush=True)


SLEEP_CYCLES = 400_000     # ~0.2 ms of torch.cuda._sleep ahead of a timed launch hides host enqueue time


def _time_pushes(tx, items, s):
    """One batched push (a single launch for <= 16 requests) timed with CUDA events on its stream;
    a short clock sleep queued first keeps the stream busy while the host enqueues the launch, so
    the events bracket the kernel and not the Python call."""
    import torch
    with torch.cuda.stream(s):
        torch.cuda._sleep(SLEEP_CYCLES)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    tx.push_many(items, stream=s)
    e1.record(s)
    return e0, e1


def handoff_one_process(dsts, reps, warmup):
    """Config 3 in one process: 1/4/16 requests of 512 tokens pushed by the fused handoff kernel
    (one launch per batch) from GPU 0 into decode lanes on each GPU of `dsts` (GPU 0: HBM -> HBM;
    another GPU: over NVLink with peer access); byte-exact check of every lane.  Per batch size:
    the kernel's device time, and the API time (push_many + the receiver's wait() seeing every
    flag through wait_all, host wall clock); for a peer, a copy-engine peer copy of the same bytes.""" 
    import ctypes
    import torch
    from rngd_pd import _lib, synth
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.nvlink import NvlinkTransport
    cfg = ModelConfig.llama31_8b()
    L, NKV, HD = cfg.n_layers, cfg.n_kv, cfg.head_dim
    per_req = handoff_bytes(cfg)
    src = torch.device("cuda", 0)
    torch.cuda.set_device(src)
    kvs = [synth.handoff_kv(cfg, S, 1000 + i, device=src) for i in range(B)]
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = []
    for dst in dsts:
        ddev = torch.device("cuda", dst)
        rx = NvlinkTransport(dst)
        K = torch.zeros((L, B, NKV, S, HD), dtype=torch.bfloat16, device=ddev)
        V = torch.zeros_like(K)
        rx.bind_cache(K, V)
        tx = rx if dst == 0 else NvlinkTransport(0)
        key = tx.set_remote_handshake(rx.handshake_metadata()) if tx is not rx else None
        s = torch.cuda.Stream(device=src)
        for n in HANDOFF_BATCHES:
            dev_ms, api_ms, used = [], [], []
            for rep in range(2 * (warmup + reps)):
                timed_dev = rep % 2 == 0                         # alternate device-timed / API-timed
                ids = [f"r{n}.{rep}.{b}" for b in range(n)]
                used = [(rep * n + b) % B for b in range(n)]      # rotate sources: > L2 across reps
                for b, r in enumerate(ids):
                    tk = rx.reserve(r, b, sender_device=0)
                    if key is not None:
                        tx.add_lease(key, tk)
                items = [(r, kvs[used[b]], None) for b, r in enumerate(ids)]
                if timed_dev:
                    e0, e1 = _time_pushes(tx, items, s)
                    for r in ids:
                        rx.wait(r, timeout=10)
                    e1.synchronize()
                    if rep // 2 >= warmup:
                        dev_ms.append(e0.elapsed_time(e1))
                else:
                    t0 = time.perf_counter()
                    tx.push_many(items, stream=s)
                    rx.wait_all(ids, timeout=10)
                    if rep // 2 >= warmup:
                        api_ms.append((time.perf_counter() - t0) * 1e3)
                for r in ids:
                    rx.release(r)
            exact = all(torch.equal(K[:, b].view(torch.int16), kvs[used[b]][:, 0].to(ddev).view(torch.int16)) and
                        torch.equal(V[:, b].view(torch.int16), kvs[used[b]][:, 1].to(ddev).view(torch.int16))
                        for b in range(n))
            ms, ams = statistics.median(dev_ms), statistics.median(api_ms)
            gbs = n * per_req / ms / 1e6
            row = {"dst": f"cuda:{dst}", "requests": n, "launches": 1, "ms": ms, "payload_bytes": n * per_req,
                   "gbs": gbs, "api_ms": ams, "api_gbs": n * per_req / ams / 1e6, "byte_exact": exact}
            if dst == 0:
                row.update(bound="hbm", frac=2 * gbs / hbm, peak=hbm, note="frac counts read + write")
            else:
                flat = torch.empty(n * per_req // 2, dtype=torch.bfloat16, device=ddev)
                ce = []
                for rep in range(3 + reps):
                    with torch.cuda.stream(s):
                        torch.cuda._sleep(SLEEP_CYCLES)
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record(s)
                        for b in range(n):
                            _lib.call("rngd_peer_copy", ctypes.c_void_p(flat.data_ptr() + b * per_req), dst,
                                      _lib.ptr(kvs[(rep * n + b) % B]), 0, per_req, _lib.stream_handle(s))
                        e1.record(s)
                    e1.synchronize()
                    if rep >= 3:
                        ce.append(e0.elapsed_time(e1))
                del flat
                copy_gbs = n * per_req / statistics.median(ce) / 1e6
                row.update(bound="nvlink", peak=copy_gbs, peak_kind="peer copy of the same bytes, measured here",
                           frac=gbs / copy_gbs, copy_engine_gbs=copy_gbs, frac_of_nominal=gbs / NVLINK_NOMINAL_GBS,
                           nominal_gbs=NVLINK_NOMINAL_GBS)
            out.append(row)
        if tx is not rx:
            tx.close()
        rx.close()
        del K, V
    return out


def config1_measure(eng, steps=20, warmup=3):
    """BASELINE config 1's decode rate: B=4 streams with 256 past tokens each (KV seeds 100..103,
    tokens seed 2), a B=4 engine on the weights of `eng`, device time of self-feeding graph
    replays.  Its roofline bytes: the weights plus the KV read and written per step."""
    import torch
    from rngd_pd import synth
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    b4, past = 4, 256
    e4 = BatchDecodeEngine(eng.cfg, eng.w, B=b4, S=S, group=8)
    Ks, Vs = zip(*[synth.request_kv(eng.cfg, S, 100 + b, past, device=eng.dev) for b in range(b4)])
    Kd, Vd = e4.adopt_kv_device(list(Ks), list(Vs))
    del Ks, Vs
    toks = synth.tokens(b4, seed=2)
    e4.step(toks, [past] * b4, Kd, Vd)
    e4.set_inputs(toks, [past] * b4)
    e4.step_device(Kd, Vd, warmup)
    torch.cuda.synchronize(eng.dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(e4.stream)
    e4.step_device(Kd, Vd, steps)
    e1.record(e4.stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    mid = past + warmup + steps // 2
    nbytes = WEIGHT_BYTES + b4 * (mid + 1) * KV_BYTES_PER_POS + b4 * KV_BYTES_PER_POS
    del Kd, Vd, e4
    return {"workload": "config1: batched decode B=4, S=512, 256 past tokens per stream", "ms_per_step": ms,
            "tok_s": b4 / ms * 1e3, "bytes_per_step": nbytes, "achieved_gbs": nbytes / ms / 1e6}


def prefill_flops(cfg, C):
    """Useful FLOPs of one prefill_full pass over C tokens (config 2): the layer GEMMs, causal
    attention (QK^T and PV over the lower triangle) and the last position's lm_head."""
    layer_params = (cfg.hidden * (cfg.n_heads + 2 * cfg.n_kv) * cfg.head_dim + cfg.n_heads * cfg.head_dim * cfg.hidden
                    + 3 * cfg.hidden * cfg.inter)
    gemm = 2 * C * layer_params * cfg.n_layers
    attn = cfg.n_layers * 4 * cfg.n_heads * cfg.head_dim * (C // 2) * C
    return gemm + attn + 2 * cfg.hidden * cfg.vocab


def prefill_measure(eng, reps=5, warmup=2):
    """Config 2 on the decode engine's card and weights: one 256-token prompt (ids U[0, V),
    seed 4) through FullPrefillEngine.prefill_kv_device, CUDA events on the prefill stream."""
    import torch
    from rngd_pd import synth
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    C = 256
    pf = FullPrefillEngine(eng.cfg, eng.w, C=C, group=2, S=S)
    toks = synth.tokens(C, seed=4)
    for _ in range(warmup):
        pf.prefill_kv_device(toks)
    ms = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(pf.stream)
        kv, nxt = pf.prefill_kv_device(toks)
        e1.record(pf.stream)
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
    t = statistics.median(ms)
    flops = prefill_flops(eng.cfg, C)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    peak = peaks.get("bf16_tflops", 1590.0)
    tf = flops / (t / 1e3) / 1e12
    del pf
    return {"workload": "config2: prefill_full, one prompt of C=256 tokens, Llama-3.1-8B shape", "ms": t,
            "tflops_useful": tf, "peak_tflops": peak, "frac": tf / peak,
            "flops_per_pass": flops, "note": "GEMMs issue hi and lo activation halves: tensor work is ~2x the useful"}


def prefill_timeline(eng, layers=2):
    """Per-CTA timelines of the first `layers` layers' prefill GEMM launches of one config-2 pass
    (needs a library built with `make TRACE=1`; None for a product build).  Per launch, in us
    from its earliest CTA start, [min, median, max] over CTAs of: start, TMA past the dependency
    wait, first full stage, last MMA commit, last unit's accumulator ready / pieces acquired /
    epilogue done; plus the median MMA span, the tail from the last commit to the last epilogue,
    and the median epilogue time of the CTAs that finish their last unit themselves."""
    import torch
    from rngd_pd import _lib, synth
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    n = 4 * layers
    tr = torch.zeros((n, 1024, 16), dtype=torch.int64, device=eng.dev)
    try:
        _lib.call("rngd_trace_decode_gemms", _lib.ptr(tr), 0)     # records nothing: a support check
    except _lib.RngdError:           # a product build: the stamps are compiled out
        return None
    pf = FullPrefillEngine(eng.cfg, eng.w, C=256, group=2, S=S)
    toks = synth.tokens(256, seed=4)
    pf.prefill_kv_device(toks)
    _lib.call("rngd_trace_decode_gemms", _lib.ptr(tr), n)
    try:
        pf.prefill_kv_device(toks)
        torch.cuda.synchronize(eng.dev)
    finally:
        _lib.call("rngd_trace_decode_gemms", None, 0)
    out = []
    prev_end = None
    for i in range(n):
        t = tr[i].cpu().double()
        t = t[t[:, 0] > 0]
        rel = (t - t[:, 0].min()) / 1e3
        q = lambda c: [round(float(v), 1) for v in (rel[:, c].min(), rel[:, c].median(), rel[:, c].max())]
        own = t[:, 9] == 0
        row = {"gemm": ("qkv", "o", "gate_up", "down")[i % 4], "layer": i // 4}
        row.update({k: q(c) for k, c in (("start", 0), ("tma_dep", 1), ("first_full", 2), ("last_commit", 3),
                                         ("last_acc", 4), ("pieces", 5), ("epi_done", 6))})
        row["mma_span_med"] = round(float(((t[:, 3] - t[:, 2]) / 1e3).median()), 1)
        row["tail"] = round(float((t[:, 6].max() - t[:, 3].max()) / 1e3), 1)
        row["last_unit_epi_med"] = round(float(((t[own, 6] - t[own, 5]) / 1e3).median()), 1) if own.any() else None
        row["last_unit_epi_by_owners"] = {int(k): round(float(((t[own & (t[:, 8] == k), 6] - t[own & (t[:, 8] == k), 5])
                                                                / 1e3).median()), 1)
                                          for k in sorted(set(t[own, 8].long().tolist()))}
        # from the previous traced GEMM's last epilogue to this launch's dependency release: the
        # kernels in between (for O, the attention) and the boundary
        row["dep_after_prev_end"] = (round(float((t[:, 1].median() - prev_end) / 1e3), 1)
                                     if prev_end is not None else None)
        prev_end = float(t[:, 6].max())
        out.append(row)
    del pf
    return out


def prefill_chunk_measure(eng, reps=3, warmup=1):
    """Chunked prefill (ChunkPrefillEngine, engines/prefill_chunk.py): one 256-token prompt
    (seed 4) in chunks of 16 positions against a one-lane cache, on the decode engine's card and
    weights.  Every chunk is one decode step of 16 streams sharing the lane, so it streams the
    whole 15 GB of weights: HBM-bound, reported as weight GB/s of the median pass."""
    import torch
    from rngd_pd import synth
    from rngd_pd.engines.prefill_chunk import ChunkPrefillEngine
    C, P = 16, 256
    ck = ChunkPrefillEngine(eng.cfg, None, S=S, C=C, group=eng.NG, share=eng)
    toks = synth.tokens(P, seed=4)
    for _ in range(warmup):
        ck.prefill_device(toks)
    ms = []
    for _ in range(reps):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ck._e.stream)
        ck.prefill_device(toks)
        e1.record(ck._e.stream)
        e1.synchronize()
        ms.append(e0.elapsed_time(e1))
    t = statistics.median(ms)
    chunks = P // C
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    gbs = WEIGHT_BYTES * chunks / (t / 1e3) / 1e9
    del ck
    return {"workload": "chunked prefill: one prompt of 256 tokens in chunks of 16 (one decode step of 16 "
                        "streams sharing a cache lane per chunk), Llama-3.1-8B shape",
            "ms": t, "chunks": chunks, "ms_per_chunk": t / chunks, "weight_gbs": gbs, "peak_gbs": hbm,
            "frac": gbs / hbm, "note": "includes the host->device upload of each chunk's 16 tokens"}


def handoff_pairs(rank, world, dev, reps, warmup):
    """Config 3 across processes: GPU 2i prefills (seeded caches) and pushes into GPU 2i+1's
    decode cache, mapped through CUDA IPC; 1/4/16 requests per batch.  Returns, on every rank,
    {requests: max-over-senders ms} of the handoff kernel, of a copy-engine peer copy and of NCCL
    send/recv moving the same requests (the two comparators), and whether every receiver's lanes
    were byte-exact."""
    import ctypes
    import torch
    import torch.distributed as dist
    from rngd_pd import _lib, synth
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.nvlink import NvlinkTransport, ipc_empty
    cfg = ModelConfig.llama31_8b()
    L, NKV, HD = cfg.n_layers, cfg.n_kv, cfg.head_dim
    sender = rank % 2 == 0
    partner = rank + 1 if sender else rank - 1
    t = NvlinkTransport(dev.index)
    kvs = K = V = None
    if sender:
        kvs = [synth.handoff_kv(cfg, S, 1000 + i, device=dev) for i in range(B)]
    else:
        K = ipc_empty((L, B, NKV, S, HD), torch.bfloat16, dev)
        V = ipc_empty((L, B, NKV, S, HD), torch.bfloat16, dev)
        t.bind_cache(K, V)
    metas = [None] * world
    dist.all_gather_object(metas, None if sender else t.handshake_metadata())
    key = t.set_remote_handshake(metas[partner]) if sender else None
    s = torch.cuda.Stream(device=dev)
    out, copies, nccl, exact = {}, {}, {}, True
    pdev = torch.device("cuda", partner)
    for n in HANDOFF_BATCHES:
        times = []
        for rep in range(warmup + reps):
            used = [(rep * n + b) % B for b in range(n)]
            tickets = None
            if not sender:
                tickets = [t.reserve(f"r{n}.{rep}.{b}", b, sender_device=partner) for b in range(n)]
            allt = [None] * world
            dist.all_gather_object(allt, tickets)
            if sender:
                for tk in allt[partner]:
                    t.add_lease(key, tk)
            dist.barrier()
            if sender:
                e0, e1 = _time_pushes(t, [(tk["req"], kvs[used[b]], None) for b, tk in enumerate(allt[partner])], s)
                e1.synchronize()
                if rep >= warmup:
                    times.append(e0.elapsed_time(e1))
            else:
                for tk in tickets:
                    t.wait(tk["req"], timeout=20)
            dist.barrier()
            if not sender:
                if rep == warmup + reps - 1:
                    for b in range(n):
                        ref = synth.handoff_kv(cfg, S, 1000 + used[b], device=dev)
                        exact &= bool(torch.equal(K[:, b].view(torch.int16), ref[:, 0].view(torch.int16)) and
                                      torch.equal(V[:, b].view(torch.int16), ref[:, 1].view(torch.int16)))
                        del ref
                for tk in tickets:
                    t.release(tk["req"])
        ms = torch.tensor([statistics.median(times) if times else 0.0], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        out[n] = float(ms.item())
        # the copy engine moving the same bytes GPU 2i -> GPU 2i+1 (a peer copy from the sender's
        # process), the measured peak the handoff is compared with
        cms = []
        if sender:
            _lib.call("rngd_peer_enable", dev.index, partner)          # a direct copy over NVLink
            flat = torch.empty(n * kvs[0].numel(), dtype=torch.bfloat16, device=pdev)
            nbytes = kvs[0].numel() * 2
            for rep in range(warmup + reps):
                with torch.cuda.stream(s):
                    torch.cuda._sleep(SLEEP_CYCLES)
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(s)
                    for b in range(n):
                        _lib.call("rngd_peer_copy", ctypes.c_void_p(flat.data_ptr() + b * nbytes), partner,
                                  _lib.ptr(kvs[(rep * n + b) % B]), dev.index, nbytes, _lib.stream_handle(s))
                    e1.record(s)
                e1.synchronize()
                if rep >= warmup:
                    cms.append(e0.elapsed_time(e1))
            del flat
        cm = torch.tensor([statistics.median(cms) if cms else 0.0], device=dev)
        dist.all_reduce(cm, op=dist.ReduceOp.MAX)
        copies[n] = float(cm.item())
        # NCCL point-to-point moving the same requests (send on GPU 2i, recv on GPU 2i+1): the
        # library comparator.  Every rank posts its side of the batch; device time of the batch on
        # each rank, max over ranks
        rbuf = None if sender else torch.empty((n, L, 2, NKV, S, HD), dtype=torch.bfloat16, device=dev)
        nms = []
        for rep in range(warmup + reps):
            if sender:
                ops = [dist.P2POp(dist.isend, kvs[(rep * n + b) % B].contiguous(), partner) for b in range(n)]
            else:
                ops = [dist.P2POp(dist.irecv, rbuf[b], partner) for b in range(n)]
            dist.barrier()
            cur = torch.cuda.current_stream(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(cur)
            for w in dist.batch_isend_irecv(ops):
                w.wait()
            e1.record(cur)
            e1.synchronize()
            if rep >= warmup:
                nms.append(e0.elapsed_time(e1))
        del rbuf
        nm = torch.tensor([statistics.median(nms)], device=dev)
        dist.all_reduce(nm, op=dist.ReduceOp.MAX)
        nccl[n] = float(nm.item())
    ok = torch.tensor([1 if exact else 0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    t.close()                      # senders unmap before receivers free
    dist.barrier()
    del K, V, kvs
    return out, copies, nccl, bool(ok.item())


def run_micro_step_small(args):
    """Config 4's decode step (B=16, S=512, same lengths and per-layer shapes) on a 2-layer model
    of the Llama-3.1-8B shape: ~3 GB on the device, for ncu captures of any decode-step kernel
    (the fused attention, the GEMM epilogues) on a small case.  Eager launches, one per kernel."""
    import torch
    from rngd_pd import synth
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    os.environ["RNGD_CUDA_GRAPH"] = "0"
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = ModelConfig.from_dims(L=2)
    eng = BatchDecodeEngine(cfg, synth.SyntheticState(cfg, seed=0), B=B, S=S, group=2)
    lens, toks = lengths_and_tokens()
    Ks, Vs = zip(*[synth.request_kv(cfg, S, 100 + b, lens[b], device=dev) for b in range(B)])
    Kd, Vd = eng.adopt_kv_device(list(Ks), list(Vs))
    del Ks, Vs
    pos = list(lens)
    for _ in range(args.warmup):
        toks, Kd, Vd = eng.step(toks, pos, Kd, Vd)
        pos = [p + 1 for p in pos]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(eng.stream)
    for _ in range(args.steps):
        toks, Kd, Vd = eng.step(toks, pos, Kd, Vd)
        pos = [p + 1 for p in pos]
    e1.record(eng.stream)
    torch.cuda.synchronize()
    from rngd_pd import _lib
    print(json.dumps({"micro": "step_small", "layers": 2, "B": B, "S": S, "ms_per_step": e0.elapsed_time(e1) / args.steps,
                      "status": _lib.device_status()}), flush=True)


def run_micro_serve_box(args):
    """The end-to-end PD box in one process over every visible GPU (serving/pd.py build_pd):
    P prefill GPUs push each prompt's cache over NVLink into the lanes of D decode GPUs, each a
    continuous-batching scheduler (B=16, S=512) behind one gateway.  SERVE_SPLIT picks the split
    ("2P:6D"; default half and half, i.e. 1P:1D pairs), SERVE_N the requests (default 512),
    SERVE_RATE the Poisson arrival rate of the box (default 40 req/s per decode GPU) or
    SERVE_RATES a sweep of per-decode-GPU rates ("24,40"), all on the same box and prompts.
    Prompts U[128, 448] tokens, 64 output tokens, seeded.  Box tok/s = output tokens / (last
    completion - first arrival); TTFT = arrival -> first token; TPOT = a request's median decode
    step.  Afterwards every request is served again solo on one GPU (SERVE_SOLO=0 skips it) and
    its greedy tokens compared with each run's."""
    import threading
    import numpy as np
    import torch
    from rngd_pd import _lib, synth
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.serving.pd import build_pd, parse_split
    n = torch.cuda.device_count()
    split = parse_split(os.environ["SERVE_SPLIT"]) if os.environ.get("SERVE_SPLIT") else (n // 2, n - n // 2)
    if n < 2 or split[0] + split[1] > n:
        print(json.dumps({"micro": "serve_box", "unavailable": f"split {split} needs more than the {n} GPUs visible"}),
              flush=True)
        return
    cfg = ModelConfig.llama31_8b()
    box = build_pd(cfg, synth.SyntheticState(cfg, seed=0), split=split, B=B, S=S)
    out_tok = 64
    n_req = int(os.environ.get("SERVE_N", "512"))
    if os.environ.get("SERVE_RATES"):        # per decode GPU, a sweep
        rates = [float(r) * split[1] for r in os.environ["SERVE_RATES"].split(",")]
    else:
        rates = [float(os.environ.get("SERVE_RATE", str(40.0 * split[1])))]
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab, int(rng.integers(128, 449))).tolist() for _ in range(n_req)]
    for P in (200, 400):                    # warm-up outside the trace: both buckets on every pairing
        for _ in range(max(split)):
            box.gateway.complete({"tokens": [1] * P, "max_tokens": 4})
    pct = lambda v, q: float(np.percentile([x for x in v if x is not None], q)) if any(
        x is not None for x in v) else None
    runs = []
    for k, rate in enumerate(rates):
        box.gateway.window.recs.clear()
        arrivals = np.cumsum(np.random.default_rng(6 + k).exponential(1.0 / rate, n_req))
        ttft, tpot, done_at, errors = [None] * n_req, [None] * n_req, [None] * n_req, []
        outs = [None] * n_req
        lane0 = [(sc.steps, sc.lane_steps) for sc in box.schedulers]
        t_start = time.perf_counter() + 0.2

        def client(i):
            t_arr = t_start + arrivals[i]
            time.sleep(max(0.0, t_arr - time.perf_counter()))
            first = []
            try:
                resp = box.gateway.complete({"tokens": prompts[i], "max_tokens": out_tok},
                                            on_token=lambda t: first.append(time.perf_counter()) if not first else None)
                ttft[i] = (first[0] - t_arr) * 1e3
                tpot[i] = resp["pd"]["tpot_ms"]
                outs[i] = list(resp["choices"][0]["tokens"])
                done_at[i] = time.perf_counter()
            except Exception as e:   # noqa: BLE001 - reported
                errors.append(repr(e))
        threads = [threading.Thread(target=client, args=(i,)) for i in range(n_req)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        ok = [i for i in range(n_req) if done_at[i] is not None]
        span = max(done_at[i] for i in ok) - (t_start + arrivals[0]) if ok else float("nan")
        occ = [(sc.lane_steps - l0) / max((sc.steps - s0) * sc.B, 1) for sc, (s0, l0) in zip(box.schedulers, lane0)]
        runs.append({"rate_req_s": rate, "rate_per_decode_gpu": rate / split[1], "requests": n_req,
                     "completed": len(ok), "errors": errors[:3],
                     "box_tok_s": len(ok) * out_tok / span if ok else 0.0, "span_s": span,
                     "ttft_ms_p50": pct(ttft, 50), "ttft_ms_p90": pct(ttft, 90),
                     "tpot_ms_p50": pct(tpot, 50), "tpot_ms_p90": pct(tpot, 90),
                     "decode_occupancy": occ, "airm": box.gateway.window.summary(), "_outs": outs, "_ok": ok})
        print(json.dumps({"micro": "serve_box", "split": f"{split[0]}P:{split[1]}D", "gpus": n,
                          **{k2: v for k2, v in runs[-1].items() if not k2.startswith("_")}}), flush=True)
    box.close()
    solo = None
    if os.environ.get("SERVE_SOLO", "1") != "0":
        every = sorted(set(i for r in runs for i in r["_ok"]))
        # the gateway keeps a prompt's first S - max_tokens - 1 tokens (as the reference's gateway
        # does, serving/cluster.py:1516); the solo run is given the same prompt
        served = [p[:S - out_tok - 1] for p in prompts]
        got = _solo_tokens(cfg, box.decode_engines, served, every, out_tok)
        solo = [dict(_solo_report(r["_outs"], got, r["_ok"]), rate_req_s=r["rate_req_s"]) for r in runs]
    best = max(runs, key=lambda r: r["box_tok_s"])
    print(json.dumps({"micro": "serve_box", "split": f"{split[0]}P:{split[1]}D", "gpus": n,
                      "workload": "PD box in one process: prefill GPUs -> NVLink -> decode lanes, continuous "
                                  "batching B=16, S=512, seeded Poisson trace, prompts U[128,448], 64 output "
                                  "tokens, Llama-3.1-8B shape",
                      "runs": [{k2: v for k2, v in r.items() if not k2.startswith("_")} for r in runs],
                      "box_tok_s": best["box_tok_s"], "ttft_ms_p50": best["ttft_ms_p50"],
                      "tpot_ms_p50": best["tpot_ms_p50"], "solo": solo,
                      "status": _lib.device_status()}), flush=True)


def _solo_tokens(cfg, engines, prompts, which, out_tok):
    """Every request of `which` served again as a solo single-GPU run: each decode GPU takes a
    share and runs prefill and decode on itself (a FullPrefillEngine on the decode engine's
    weights under a one-card continuous-batching scheduler).  Returns {request: tokens}."""
    import threading
    import torch
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd.serving.scheduler import ContinuousScheduler, OneCardProducer
    got, errs = {}, []

    def card(eng, share):
        with torch.cuda.device(eng.dev):
            pre = FullPrefillEngine(cfg, eng.w, C=256, group=2, S=eng.S)
            pre.add_bucket(512)
            prod = OneCardProducer(pre)
            sched = ContinuousScheduler(eng.B, eng, prod.produce, produce_owner=prod, stage_admission=False)

            def one(i):
                try:
                    got[i] = list(sched.submit({"tokens": prompts[i], "max_new": out_tok})["tokens"])
                except Exception as e:   # noqa: BLE001 - reported
                    errs.append(repr(e))
            ts = [threading.Thread(target=one, args=(i,)) for i in share]
            for t in ts:
                t.start()
            for t in ts:
                t.join()
            sched.close()
    cards = [threading.Thread(target=card, args=(e, which[k::len(engines)])) for k, e in enumerate(engines)]
    for t in cards:
        t.start()
    for t in cards:
        t.join()
    if errs:
        got["_errors"] = errs[:3]
    return got


def _solo_report(outs, solo, which):
    same = [i for i in which if solo.get(i) is not None and solo[i] == outs[i]]
    differ = [i for i in which if i not in same]
    first = None
    if differ:
        i = differ[0]
        a, b = outs[i] or [], solo.get(i) or []
        at = next((k for k in range(min(len(a), len(b))) if a[k] != b[k]), min(len(a), len(b)))
        first = {"request": i, "position": at, "box": a[at:at + 4], "solo": b[at:at + 4]}
    return {"checked": len(which), "identical": len(same), "first_difference": first,
            "errors": solo.get("_errors", []),
            "how": "each decode GPU re-serves its share of the trace alone: prefill and decode on that one GPU "
                   "(one-card scheduler), greedy tokens compared request by request"}


def run_micro_serve(args, pd=False):
    """Continuous batching (serving/scheduler.py over BatchDecodeEngine B=16): a seeded Poisson
    trace in the shape of the end-to-end PD configuration (prompts U[128, 448] tokens, 64 output
    tokens each) sent through the in-process Gateway by one client thread per request at its
    arrival time; the line carries the gateway Window's airm summary too.  One card (pd=False): a
    FullPrefillEngine on the decode engine's weights, prompts admitted between steps.  PD on two
    GPUs of one process (pd=True): prefill on GPU 0 pushes each prompt's cache over NVLink into
    the decode lane leased on GPU 1 while GPU 1 keeps stepping.  Box tok/s = output tokens /
    (last completion - first arrival); TTFT = arrival -> first token; TPOT = a request's median
    decode step."""
    import threading
    import numpy as np
    import torch
    from rngd_pd import synth
    from rngd_pd.engines.decode_batch import BatchDecodeEngine
    from rngd_pd.engines.model import ModelConfig
    from rngd_pd.engines.prefill_full import FullPrefillEngine
    from rngd_pd import _lib
    from rngd_pd.serving.gateway import Gateway
    from rngd_pd.serving.scheduler import ContinuousScheduler, NvlinkProducer, OneCardProducer
    cfg = ModelConfig.llama31_8b()
    if pd:
        if torch.cuda.device_count() < 2:
            print(json.dumps({"micro": "serve_pd", "unavailable": "needs two GPUs"}), flush=True)
            return
        eng = BatchDecodeEngine(cfg, synth.SyntheticState(cfg, seed=0), B=B, S=S, group=8, chip=1)
        pre = FullPrefillEngine(cfg, synth.SyntheticState(cfg, seed=0), C=256, group=2, S=S, chip=0)
    else:
        torch.cuda.set_device(0)
        eng = BatchDecodeEngine(cfg, synth.SyntheticState(cfg, seed=0), B=B, S=S, group=8)
        pre = FullPrefillEngine(cfg, eng.w, C=256, group=2, S=S)
    pre.add_bucket(512)
    rate, n_req, out_tok = float(os.environ.get("SERVE_RATE", "40")), int(os.environ.get("SERVE_N", "96")), 64
    rng = np.random.default_rng(5)
    arrivals = np.cumsum(rng.exponential(1.0 / rate, n_req))
    prompts = [rng.integers(0, cfg.vocab, int(rng.integers(128, 449))).tolist() for _ in range(n_req)]
    if pd:
        kv = eng.blank_kv()
        prod = NvlinkProducer(pre, eng, kv)
        sched = ContinuousScheduler(B, eng, None, produce_owner=prod, idle_pos=S - 1, kv=kv)
        stage = False
    else:
        prod = OneCardProducer(pre)
    # admission: waiting prompts prefilled back to back between decode steps (RNGD_ADMIT=block;
    # measured here against staging 4 or 16 layer groups per iteration, the reference's default
    # for a card whose prefill group costs as much as a decode step: a B200 prefill costs a few
    # decode steps, and blocking gave the best TTFT and box throughput); SERVE_ADMIT=stage for the other
    if not pd:
        stage = os.environ.get("SERVE_ADMIT", "block") == "stage"
        sched = ContinuousScheduler(B, eng, prod.produce, produce_owner=prod, stage_admission=stage)
    # warm-up outside the trace: every prefill bucket and the captured step
    for P in (200, 400):
        sched.submit({"tokens": [1] * P, "max_new": 4})
    gw = Gateway({"llama-3.1-8b": sched}, S=S)      # requests enter as the reference's gateway takes them
    ttft, tpot, done_at, errors = [None] * n_req, [None] * n_req, [None] * n_req, []
    t_start = time.perf_counter() + 0.2

    def client(i):
        t_arr = t_start + arrivals[i]
        time.sleep(max(0.0, t_arr - time.perf_counter()))
        first = []
        body = {"model": "llama-3.1-8b", "tokens": prompts[i], "max_tokens": out_tok}
        try:
            resp = gw.complete(body, on_token=lambda t: first.append(time.perf_counter()) if not first else None)
            ttft[i] = (first[0] - t_arr) * 1e3
            tpot[i] = resp["pd"]["tpot_ms"]
            done_at[i] = time.perf_counter()
        except Exception as e:   # noqa: BLE001 - reported
            errors.append(repr(e))
    threads = [threading.Thread(target=client, args=(i,)) for i in range(n_req)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    sched.close()
    if pd:
        prod.close()
    ok = [i for i in range(n_req) if done_at[i] is not None]
    span = max(done_at[i] for i in ok) - (t_start + arrivals[0])
    pct = lambda v, q: float(np.percentile([x for x in v if x is not None], q))
    print(json.dumps({"micro": "serve_pd" if pd else "serve",
                      "workload": ("PD on two GPUs (prefill GPU 0 -> NVLink -> decode lanes on GPU 1)" if pd else
                                   "one card") + ": continuous batching B=16, S=512, seeded Poisson trace, prompts "
                                   "U[128,448], 64 output tokens, Llama-3.1-8B shape",
                      "admission": "nvlink lane fill" if pd else ("stage" if stage else "block"),
                      "rate_req_s": rate, "requests": n_req, "completed": len(ok), "errors": errors[:3],
                      "box_tok_s": len(ok) * out_tok / span, "span_s": span,
                      "ttft_ms_p50": pct(ttft, 50), "ttft_ms_p90": pct(ttft, 90),
                      "tpot_ms_p50": pct(tpot, 50), "tpot_ms_p90": pct(tpot, 90),
                      "occupancy": sched.occupancy(), "steps": sched.steps, "admissions": sched.admits,
                      "staged_steps": sched.stage_steps, "airm": gw.window.summary(),
                      "status": _lib.device_status()}), flush=True)


def run_micro(args):
    """One decode GEMM shape alone (small device footprint; for ncu captures of skgemm_kernel)."""
    import torch
    from rngd_pd import _lib, synth
    if args.micro == "attn":
        return run_micro_attn(args)
    if args.micro == "step_small":
        return run_micro_step_small(args)
    if args.micro in ("serve", "serve_pd"):
        return run_micro_serve(args, pd=args.micro == "serve_pd")
    if args.micro == "serve_box":
        return run_micro_serve_box(args)
    if args.micro == "handoff":
        return run_micro_handoff(args)
    if args.micro in ("prefill", "prefill_small"):
        # prefill_small: the same pass on a 2-layer model of the same shape (~3 GB, for captures)
        from rngd_pd.engines.decode_batch import BatchDecodeEngine
        from rngd_pd.engines.model import ModelConfig
        torch.cuda.set_device(0)
        cfg = ModelConfig.llama31_8b() if args.micro == "prefill" else ModelConfig.from_dims(L=2)
        eng = BatchDecodeEngine(cfg, synth.SyntheticState(cfg, seed=0), B=B, S=S,
                                group=8 if args.micro == "prefill" else 2)
        res = prefill_measure(eng, reps=args.steps, warmup=args.warmup)
        tl = prefill_timeline(eng)
        if tl is not None:
            res["timeline_us"] = tl
        print(json.dumps({"micro": args.micro, **res}), flush=True)
        return
    if args.micro.startswith("pf_"):
        return run_micro_prefill(args)
    shapes = {"gate_up": (28672, 4096), "qkv": (6144, 4096), "o": (4096, 4096), "down": (4096, 14336),
              "lm": (128256, 4096)}
    N, K = shapes[args.micro]
    dev = torch.device("cuda", 0)
    W = torch.empty((2, N, K), dtype=torch.bfloat16, device=dev)   # two layers' worth: > L2, alternated
    synth.fill_gauss(W, 0, 4, 0.02)
    g = TcGemm(W, N, K, dev)
    ms = g.time(args.steps, torch.cuda.current_stream(dev))
    # traced graph of 4 launches: per launch, CTA stamps relative to launch 0's earliest start (us)
    tr = torch.zeros((4, 1024, 16), dtype=torch.int64, device=dev)
    timeline = []
    try:
        g.time(4, torch.cuda.current_stream(dev), trace=tr)
    except _lib.RngdError:           # a product build (no TRACE=1): the stamps are compiled out
        tr = None
    t = tr.cpu().double() if tr is not None else None
    t0 = t[0, :, 0][t[0, :, 0] > 0].min() if t is not None else None
    for i in range(4 if t is not None else 0):
        ti = t[i][t[i, :, 0] > 0]
        rel = (ti - t0) / 1e3
        q = lambda col: [round(float(v), 2) for v in (rel[:, col].min(), rel[:, col].median(), rel[:, col].max())]
        timeline.append({k: q(c) for c, k in enumerate(("start", "operand", "last_tma", "last_arrival", "last_mma",
                                                         "last_acc", "epi_done", "end"))})
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json")))
    except OSError:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    print(json.dumps({"micro": args.micro, "N": N, "K": K, "B": B, "ms": ms, "bytes": g.nbytes,
                      "gbs": g.nbytes / ms / 1e6, "frac_hbm": g.nbytes / ms / 1e6 / hbm,
                      "pdl": os.environ.get("RNGD_PDL", "1"), "timeline_us_min_med_max": timeline}), flush=True)


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
    # the clock sampler starts before ~0.4 s of untimed steps (the same steps at the same
    # positions), so its samples cover the load the timed region runs under, and it is
    # stopped right after the timed region
    clocks = Clocks() if rank == 0 else None
    t_pre = time.perf_counter() + 0.4
    while time.perf_counter() < t_pre:
        eng.set_inputs(toks0, lens)
        eng.step_device(Kd, Vd, W)
        torch.cuda.synchronize(dev)
    eng.set_inputs(toks0, lens)
    eng.step_device(Kd, Vd, W)
    barrier()
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
    # a bounded device wait that ran out leaves a wrong result and a step cut short by it
    from rngd_pd import _lib
    t = torch.tensor([_lib.device_status()], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    status = int(t.item())
    if status != 0:
        raise RuntimeError(f"device status {status} after the timed steps: a bounded wait ran out, "
                           "so these timings are not valid")

    roof = gemm_roofline(eng) if rank == 0 else None
    config1 = config1_measure(eng) if rank == 0 else None
    prefill = prefill_measure(eng) if rank == 0 else None
    prefill_chunk = prefill_chunk_measure(eng) if rank == 0 else None

    # ------------------------------------------------- KV handoff (config 3)
    from rngd_pd.engines.model import ModelConfig as _MC
    per_req = handoff_bytes(_MC.llama31_8b())
    hreps = 10
    if world >= 2 and world % 2 == 0:
        hms, hcopy, hnccl, hexact = handoff_pairs(rank, world, dev, hreps, 3)
        pairs = world // 2
        handoff = {"unit": "GB/s", "pairs": pairs, "per_request_bytes": per_req, "byte_exact": hexact,
                   "path": "GPU 2i -> GPU 2i+1, separate processes, CUDA IPC + NVLink P2P stores",
                   "results": [{"requests": n, "ms": ms, "gbs": pairs * n * per_req / ms / 1e6,
                                "gbs_per_pair": n * per_req / ms / 1e6,
                                "peak": n * per_req / hcopy[n] / 1e6, "peak_kind": "peer copy of the same bytes, "
                                "measured here (max over pairs)",
                                "frac": hcopy[n] / ms, "frac_of_nominal": n * per_req / ms / 1e6 / NVLINK_NOMINAL_GBS,
                                "nominal_gbs": NVLINK_NOMINAL_GBS, "bound": "nvlink",
                                "nccl_ms": hnccl[n], "nccl_gbs_per_pair": n * per_req / hnccl[n] / 1e6}
                               for n, ms in hms.items()]}
    elif rank == 0:
        rows = handoff_one_process([local], hreps, 3)
        handoff = {"unit": "GB/s", "pairs": 0, "per_request_bytes": per_req,
                   "byte_exact": all(r["byte_exact"] for r in rows),
                   "path": "one GPU: prefill-layout cache -> decode lanes on the same GPU (HBM read + write)",
                   "results": rows}
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
        traffic = _j.load(open(os.path.join(REPO, "profiles", "traffic.json"))).get("skgemm_gate_up")
    except (OSError, ValueError):
        pass
    cpu = None
    if not args.no_cpu_baseline:
        handoff["cpu_baseline"] = handoff_cpu_baseline()
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
        "roofline": {"bound": "hbm", "kernel": "skgemm_kernel (tcgen05 stream-K, gate/up 28672x4096, B=16)",
                     "achieved": dom["gbs"], "peak": hbm, "unit": "GB/s", "frac": dom["gbs"] / hbm,
                     "traffic": traffic, "peak_kind": peak_kind,
                     "per_shape": {k: round(v["gbs"], 1) for k, v in roof.items()}},
        "cpu_baseline": cpu,
        "clocks": clk,
        "e2e": {"value": world * B * K / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 2 * B * 4,
                "d2h_bytes_per_step": B * 4},
        "gpu_launches": eng.launches_per_step * K,
        "handoff": handoff,
        "prefill": prefill,
        "prefill_chunk": prefill_chunk,
        "config1": None if config1 is None else dict(config1, frac=config1["achieved_gbs"] / hbm, peak=hbm,
                                                     unit="GB/s", peak_kind=peak_kind),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--micro", choices=["gate_up", "qkv", "o", "down", "lm", "attn", "pf_gate_up", "pf_qkv", "pf_o",
                                        "pf_down", "handoff", "prefill", "prefill_small", "step_small", "serve",
                                        "serve_pd", "serve_box"],
                    help="time one decode GEMM shape alone (small footprint, for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.micro:
        run_micro(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

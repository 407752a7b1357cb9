"""Iteration-level (continuous) batching over the B200 decode engines
(the reference's _ContinuousScheduler, src/rngd_pd/serving/cluster.py:832-1134, and its
one-card producer, serving/cluster.py:646-818).

Before every decode step the loop admits whatever is waiting into the free lanes and
retires whatever finished, so a batch can mix a stream on its third token with one on its
hundredth.  A stream's cache comes from `produce(item) -> (K, V, first, pos, aux_ms)`, the
only thing that differs between a one-card server (prefill on the same card) and a
disaggregated one; admission writes it into one lane of the resident cache
(BatchDecodeEngine.write_slot_kv) and leaves the other lanes alone.  With a TieredDecode
engine the loop reports the live lanes before each step (set_live), so the step runs at the
narrowest width that covers them.

While streams are running, a new prompt's prefill can be staged: `produce_owner.begin_produce`
hands back a stage whose `advance(n)` runs n layer groups, and the loop runs a few groups
per iteration between decode steps, so an arriving prompt does not stall every stream in
flight for a whole prefill.  With nothing running, waiting prompts are admitted at once.

A producer that writes the lane itself (`produce_owner.start_lane(item, lane) -> Future`, e.g.
a prefill on another GPU pushing into the reserved lane over NVLink) gets a free lane when a
request is taken; the lane stays out of the batch while it fills, the other lanes keep
stepping, and the stream is seated when the future completes.  Lanes without a stream step at
position `idle_pos`: pass S - 1 when lanes fill asynchronously, so the appends of idle lanes
stay clear of the rows a push is writing (a prompt never reaches the last row).  Given such a
fixed cache (`kv=`), the constructor runs one all-idle step on it, so the step's CUDA graph is
captured before any producer thread starts.

Items are dicts: "tokens" (the prompt) and "max_new" (tokens to return, the prefill's next
token included), optionally "on_token" (called with each token as it is produced; it must
not block).  submit(item) blocks and returns the item's result dict, or raises the error
that ended it; an error in a step ends the streams of that step only and the loop goes on.
"""
import collections
import os
import threading
import time
from concurrent.futures import ThreadPoolExecutor


def _emit(item, token):
    cb = item.get("on_token")
    if cb is not None:
        cb(token)


class ContinuousScheduler:
    def __init__(self, B, engine, produce, admit_min=1, produce_owner=None, produce_on_device=True,
                 stage_groups=None, stage_admission=None, idle_pos=0, kv=None):
        self.B, self.eng, self.produce = B, engine, produce
        self._kv0 = kv                   # a resident cache to use (e.g. one a transport writes into)
        self.idle_pos = int(idle_pos)
        self._start_lane = getattr(produce_owner, "start_lane", None)
        self.filling = {}                # lane -> (item, future) while its cache is produced elsewhere
        self.admit_min = max(1, int(admit_min))
        self.produce_owner = produce_owner
        # a producer that reads host memory only (a disaggregated load) runs in the background
        # from arrival on; the loop admits streams whose cache is ready.  One that uses the
        # card runs inside the loop, in order with the decode steps.
        self._loader = None if produce_on_device else ThreadPoolExecutor(
            max_workers=int(os.environ.get("PD_KV_LOADERS", "2")))
        self.stage_groups = int(stage_groups if stage_groups is not None
                                else os.environ.get("PD_STAGE_GROUPS", "4"))
        self.stage_admission = (stage_admission if stage_admission is not None
                                else os.environ.get("RNGD_ADMIT", "stage") != "block")
        self.slots = [None] * B
        self.pending = collections.deque()
        self.cv = threading.Condition()
        self._staging = None             # (lane, item, stage) of a prefill in progress
        self._closed = False
        # counters: steps, lane-steps that carried a stream, and the empty lane-steps split into
        # starved (nothing was waiting) and held (something waited, admit_min kept it out)
        self.steps = self.lane_steps = 0
        self.starved_lane_steps = self.held_lane_steps = 0
        self.admits, self.admit_ms, self.admit_stall_ms = 0, 0.0, 0.0
        self.stage_steps = 0
        if kv is not None:
            # a fixed cache: run (and so capture) its first decode step now, before any producer
            # thread exists, with every lane idle at idle_pos (rows no stream reads)
            engine.step([0] * B, [self.idle_pos] * B, *kv)
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()

    # ---------------------------------------------------------------- callers
    def submit(self, item):
        """Queue one request and wait for it; returns its result dict."""
        item["ev"] = threading.Event()
        item["out"] = item["err"] = None
        if self._loader is not None:
            item["_fut"] = self._loader.submit(self.produce, item)
            item["_fut"].add_done_callback(lambda _f: self._wake())
        with self.cv:
            if self._closed:
                raise RuntimeError("scheduler is closed")
            self.pending.append(item)
            self.cv.notify()
        item["ev"].wait()
        if item["err"] is not None:
            raise item["err"]
        return item["out"]

    def close(self):
        """Stop the loop after the current iteration; queued requests fail."""
        with self.cv:
            self._closed = True
            self.cv.notify()
        self._thread.join(timeout=60)
        err = RuntimeError("scheduler closed")
        for item in list(self.pending):
            if not item["ev"].is_set():
                item["err"] = err
                item["ev"].set()
        self.pending.clear()
        if self._loader is not None:
            self._loader.shutdown(wait=False)

    def occupancy(self):
        return self.lane_steps / max(self.steps * self.B, 1)

    # ---------------------------------------------------------------- loop
    def _wake(self):
        with self.cv:
            self.cv.notify()

    def _live(self):
        return [i for i, s in enumerate(self.slots) if s is not None]

    def _free(self):
        return [i for i, s in enumerate(self.slots) if s is None and i not in self.filling]

    def _collect_filled(self):
        """Seat the streams whose lanes finished filling; a failed fill fails its request only."""
        for lane in [ln for ln, (_it, fut) in self.filling.items() if fut.done()]:
            item, fut = self.filling.pop(lane)
            if fut.exception() is not None:
                item["err"] = fut.exception()
                item["ev"].set()
            else:
                self._seat(lane, item, fut.result())

    def _ready(self):
        """Pending items the loop may take now (called with cv held); a background load that
        failed fails its own request only."""
        if self._loader is None:
            return len(self.pending)
        ready, waiting = [], []
        for item in self.pending:
            fut = item["_fut"]
            if not fut.done():
                waiting.append(item)
            elif fut.exception() is not None:
                item["err"] = fut.exception()
                item["ev"].set()
            else:
                item["_produced"] = fut.result()
                ready.append(item)
        self.pending = collections.deque(ready + waiting)
        return len(ready)

    def _seat(self, lane, item, produced):
        K, V, first, pos, aux_ms = produced
        self.slots[lane] = {"item": item, "cur": int(first), "pos": int(pos), "pos0": int(pos),
                            "outs": [int(first)], "aux_ms": aux_ms, "step_ms": [],
                            "t0": time.perf_counter(), "s0": self.steps, "l0": self.lane_steps,
                            "v0": self.starved_lane_steps, "h0": self.held_lane_steps}
        _emit(item, int(first))

    def _admit(self, taking, Kd, Vd):
        """Produce, write and seat one stream at a time (its first token goes out while the
        rest of the admission is still running)."""
        ms = 0.0
        for lane, item in taking:
            produced = item.pop("_produced", None) or self.produce(item)
            t0 = time.perf_counter()
            Kd, Vd = self.eng.write_slot_kv(Kd, Vd, lane, produced[0], produced[1])
            ms += (time.perf_counter() - t0) * 1e3
            self._seat(lane, item, produced)
        self.admits += 1
        self.admit_ms += ms
        self.admit_stall_ms += ms
        return Kd, Vd

    def _finish(self, lane):
        s, self.slots[lane] = self.slots[lane], None
        st = sorted(s["step_ms"])
        n = max(self.steps - s["s0"], 1)
        s["item"]["out"] = {
            "tokens": s["outs"], "pos": s["pos0"], "prefill_ms": round(s["aux_ms"], 1),
            "tpot_ms": round(st[len(st) // 2], 3) if st else 0.0,
            "decode_ms": round((time.perf_counter() - s["t0"]) * 1e3, 1),
            "batch": len(self._live()) + 1, "batch_width": self.B, "sched": "continuous",
            "admit_ms": round(self.admit_ms / max(self.admits, 1), 2),
            "occupancy": round((self.lane_steps - s["l0"]) / n, 2),
            "starved_lanes": round((self.starved_lane_steps - s["v0"]) / n, 2),
            "held_lanes": round((self.held_lane_steps - s["h0"]) / n, 2),
            "occupancy_all": round(self.lane_steps / max(self.steps, 1), 2),
            "admit_stall_ms": round(self.admit_stall_ms, 1)}
        s["item"]["ev"].set()

    def _fail_all(self, e, taking):
        # lanes still filling keep filling: their requests are seated (or failed) later
        for lane in self._live():
            s, self.slots[lane] = self.slots[lane], None
            s["item"]["err"] = e
            s["item"]["ev"].set()
        for _lane, item in taking:
            if not item["ev"].is_set():
                item["err"] = item.get("err") or e
                item["ev"].set()
        if self._staging is not None:
            item = self._staging[1]
            self._staging = None
            if not item["ev"].is_set():
                item["err"] = e
                item["ev"].set()

    def _loop(self):
        Kd, Vd = self._kv0 if self._kv0 is not None else (None, None)
        while True:
            with self.cv:
                while True:
                    if self._closed:
                        return
                    ready = self._ready()
                    if self.filling and (ready or any(f.done() for _i, f in self.filling.values())):
                        break
                    if (ready and self._free()) or self._live() or self._staging is not None:
                        break
                    self.cv.wait(timeout=0.05 if (self.pending or self.filling) else None)
                free = self._free()
                n = 0 if self._staging is not None else min(len(free), ready)
                if self._live() and n < min(self.admit_min, len(free)):
                    n = 0                        # not worth an admission yet
                taking = [(free[k], self.pending.popleft()) for k in range(n)]
                waiting = len(self.pending)
                empty = len(free) - n
                self.starved_lane_steps += max(0, empty - waiting)
                self.held_lane_steps += min(empty, waiting)
            try:
                if Kd is None:
                    Kd, Vd = self.eng.blank_kv()
                tell = getattr(self.eng, "set_live", None)    # TieredDecode
                if self._start_lane is not None:
                    # lanes filled elsewhere: start each taken request's fill, seat finished ones
                    for lane, item in taking:
                        fut = self._start_lane(item, lane)
                        fut.add_done_callback(lambda _f: self._wake())
                        self.filling[lane] = (item, fut)
                    taking = []
                    self._collect_filled()
                if tell is not None:
                    tell(self._live())
                if self._staging is not None:
                    lane, item, stage = self._staging
                    self.stage_steps += 1
                    if stage.advance(self.stage_groups):
                        produced = stage.result()
                        self._staging = None
                        t0 = time.perf_counter()
                        Kd, Vd = self.eng.write_slot_kv(Kd, Vd, lane, produced[0], produced[1])
                        self.admit_stall_ms += (time.perf_counter() - t0) * 1e3
                        self._seat(lane, item, produced)
                elif (taking and self._live() and self.stage_admission
                      and hasattr(self.produce_owner, "begin_produce") and "_produced" not in taking[0][1]):
                    # protect the running streams: one prompt a few layer groups per iteration
                    lane, item = taking[0]
                    self._staging = (lane, item, self.produce_owner.begin_produce(item))
                    with self.cv:
                        for _lane, rest in reversed(taking[1:]):
                            self.pending.appendleft(rest)
                    taking = []
                elif taking:
                    Kd, Vd = self._admit(taking, Kd, Vd)
                live = self._live()
                if not live:
                    continue
                if tell is not None:
                    tell(live)
                cur = [self.slots[i]["cur"] if self.slots[i] else 0 for i in range(self.B)]
                pos = [self.slots[i]["pos"] if self.slots[i] else self.idle_pos for i in range(self.B)]
                t1 = time.perf_counter()
                nxt, Kd, Vd = self.eng.step(cur, pos, Kd, Vd)
                dt = (time.perf_counter() - t1) * 1e3
                done = []
                for i in live:
                    s = self.slots[i]
                    if len(s["outs"]) >= s["item"]["max_new"]:   # max_new = 1: the prefill's token
                        done.append(i)
                        continue
                    s["step_ms"].append(dt)
                    s["outs"].append(int(nxt[i]))
                    _emit(s["item"], int(nxt[i]))
                    s["cur"] = int(nxt[i])
                    s["pos"] += 1
                    if len(s["outs"]) >= s["item"]["max_new"]:
                        done.append(i)
                self.lane_steps += len(live)
                self.steps += 1
                for i in done:
                    self._finish(i)
            except Exception as e:   # a bad step fails its own streams; the loop goes on
                self._fail_all(e, taking)
                Kd, Vd = self._kv0 if self._kv0 is not None else (None, None)


class OneCardProducer:
    """Prefill on the decode card and hand the scheduler the device cache directly (the
    reference's SoloWorker producers, serving/cluster.py:747-776).  The cache stays in the
    prefill layout (a PrefillKV): the decode engine's write_slot_kv moves the prompt's positions
    into the lane with the handoff kernel."""

    def __init__(self, prefill_engine):
        self.pre = prefill_engine

    def produce(self, item):
        from rngd_pd.engines.decode_batch import PrefillKV
        t0 = time.perf_counter()
        P = len(item["tokens"])
        kv, nxt = self.pre.prefill_kv_device(item["tokens"])
        return PrefillKV(kv, P), None, nxt, P, (time.perf_counter() - t0) * 1e3

    def begin_produce(self, item):
        stage = self.pre.begin_device_prefill(item["tokens"])
        t0 = time.perf_counter()
        P = len(item["tokens"])

        class _Stage:
            def advance(self, n=1):
                return stage.advance(n)

            def result(self):
                from rngd_pd.engines.decode_batch import PrefillKV
                kv, nxt = stage.result_kv()
                return PrefillKV(kv, P), None, nxt, P, (time.perf_counter() - t0) * 1e3

        return _Stage()


class PrefillPool:
    """Prefill engines (one per GPU) shared by several producers, e.g. 2 prefill GPUs feeding 6
    decode GPUs (the reference's gateway round-robins prefill pods: serving/cluster.py:1490-1501).
    A prompt takes the engine with the fewest prompts holding or waiting for it (ties go
    round-robin) and holds it from its prefill to the launch of its push, so an engine's
    output is never overwritten before the push that reads it is queued behind it."""

    def __init__(self, engines):
        import itertools
        self.engines = list(engines)
        if not self.engines:
            raise ValueError("prefill pool needs at least one engine")
        self._busy = [0] * len(self.engines)
        self._locks = [threading.Lock() for _ in self.engines]
        self._mu = threading.Lock()
        self._rr = itertools.count()

    def take(self):
        """Context manager: the chosen engine, held exclusively inside the block."""
        import contextlib
        n = len(self.engines)
        with self._mu:
            first = next(self._rr) % n
            i = min(range(n), key=lambda j: (self._busy[j], (j - first) % n))
            self._busy[i] += 1

        @contextlib.contextmanager
        def held():
            try:
                with self._locks[i]:
                    yield self.engines[i]
            finally:
                with self._mu:
                    self._busy[i] -= 1
        return held()


class NvlinkProducer:
    """Disaggregated producer inside one process: the prompt is prefilled on one GPU and its
    cache pushed over NVLink straight into the decode lane the scheduler leased (the reference
    moves it host-staged through /dev/shm: serving/cluster.py:1329-1334).  Prefills run on
    worker threads (one per prefill engine), so they overlap the decode steps on the other GPU;
    the fill ends when the host sees every layer's flag of the lane.  `prefill_engine` is one
    engine or a PrefillPool shared with other producers.  Use with the scheduler's
    `kv=(Kd, Vd)` (the cache bound here) and `idle_pos=S-1`.  `transport` builds the
    transports (NvlinkTransport; a test passes a fake)."""

    def __init__(self, prefill_engine, decode_engine, kv, timeout=10.0, transport=None):
        import itertools
        if transport is None:
            from rngd_pd.nvlink import NvlinkTransport as transport
        self.pool = prefill_engine if isinstance(prefill_engine, PrefillPool) else PrefillPool([prefill_engine])
        self.pre, self.timeout = self.pool.engines[0], timeout
        self.rx = transport(decode_engine.dev)
        self.rx.bind_cache(*decode_engine.full_kv(*kv))
        self._tx = {}                    # prefill GPU -> (its sending transport, the receiver's key)
        for e in self.pool.engines:
            d = e.dev.index
            if d not in self._tx:
                tx = transport(e.dev)
                self._tx[d] = (tx, tx.set_remote_handshake(self.rx.handshake_metadata()))
        self._ids = itertools.count()
        self._pool = ThreadPoolExecutor(max_workers=len(self.pool.engines))

    def start_lane(self, item, lane):
        req = f"pd-{next(self._ids)}"
        tokens = item["tokens"]

        def fill():
            t0 = time.perf_counter()
            leased = False
            try:
                with self.pool.take() as pre:
                    tq = time.perf_counter()
                    d = pre.dev.index
                    tx, peer = self._tx[d]
                    tx.add_lease(peer, self.rx.reserve(req, lane, sender_device=d))
                    leased = True
                    kv, nxt = pre.prefill_kv_device(tokens)
                    t1 = time.perf_counter()
                    moved = tx.push_device(req, kv, stream=pre.stream, tokens=len(tokens))
                    t2 = time.perf_counter()
                self.rx.wait(req, timeout=self.timeout)
                t3 = time.perf_counter()
            finally:
                if leased:
                    self.rx.release(req)
            # the request's transfer record (the reference's pd fields): prefill, the push's
            # launch, and the wait until every layer flag of the lane was seen; queue_ms is the
            # wait for a prefill engine
            item["_xfer"] = {"prefill_ms": round((t1 - tq) * 1e3, 2), "kv_save_ms": round((t2 - t1) * 1e3, 3),
                             "kv_load_ms": round((t3 - t2) * 1e3, 3), "kv_mb": round(moved / 1e6, 2),
                             "queue_ms": round((tq - t0) * 1e3, 2)}
            return None, None, nxt, len(tokens), (t3 - t0) * 1e3
        return self._pool.submit(fill)

    def close(self):
        self._pool.shutdown(wait=True)
        for tx, _peer in self._tx.values():
            tx.close()
        self.rx.close()


_ContinuousScheduler = ContinuousScheduler   # the reference's private name

__all__ = ["ContinuousScheduler", "OneCardProducer", "NvlinkProducer", "PrefillPool"]

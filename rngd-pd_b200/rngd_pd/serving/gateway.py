"""One front for several prefill/decode pairings inside a process (the reference's Gateway,
src/rngd_pd/serving/cluster.py:1457-1598, without its HTTP hop).

The reference runs every prefill and decode card as its own HTTP worker and the gateway
calls them in turn (prefill, then decode with the KV moved through shm).  On B200 a pairing
is a ContinuousScheduler in this process: its producer either prefills on the decode card
(OneCardProducer: "single-card") or on another GPU and pushes the cache over NVLink into the
leased lane (NvlinkProducer: "disaggregated-kv-transfer").  The gateway picks the pairing by
the request's model name, round-robin when a name has several (the reference's round-robin
over prefill pods), submits the request, and answers with the reference's completion record:
choices, usage and the `pd` timing fields, with TTFT measured to the first token the
scheduler emits.  Every answer goes into an airm Window (p90 TTFT/TPOT, tok/s, KV transfer
time as airm_* gauges).

Prompts are token ids: "tokens", or "prompt" as a list of ids; a text prompt needs a
`tokenizer` (encode / decode), which this image does not ship.
"""
import itertools
import threading
import time

from rngd_pd.airm import Window

MODEL = "meta-llama/Llama-3.1-8B"


class Gateway:
    def __init__(self, targets, S, tokenizer=None, window=None, model=MODEL):
        """targets: {model name: scheduler or [schedulers]}; S: the decode cache length."""
        if not targets:
            raise ValueError("gateway needs at least one pairing")
        self.targets = {k: (list(v) if isinstance(v, (list, tuple)) else [v]) for k, v in targets.items()}
        self.S, self.tk, self.model = int(S), tokenizer, model
        self.window = window if window is not None else Window()
        self._rr = {k: itertools.count() for k in self.targets}
        self._ids = itertools.count(1)
        self._lock = threading.Lock()

    def _route(self, body):
        """(scheduler, config name) for this request: ValueError for an unknown model name."""
        name = body.get("model", "")
        if name not in self.targets:
            if name or len(self.targets) != 1:
                raise ValueError(f"unknown model {name!r}; have {sorted(self.targets)}")
            name = next(iter(self.targets))
        pool = self.targets[name]
        with self._lock:
            k = next(self._rr[name])
        return pool[k % len(pool)], name

    def _tokens(self, body, max_new):
        toks = body.get("tokens")
        if toks is None:
            prompt = body.get("prompt")
            if not prompt and body.get("messages"):
                prompt = "\n".join(m.get("content", "") for m in body["messages"])
            if isinstance(prompt, str):
                if self.tk is None:
                    raise ValueError("a text prompt needs a tokenizer; send token ids in 'tokens'")
                toks = self.tk.encode(prompt, add_special_tokens=False)
            else:
                toks = prompt
        toks = [int(t) for t in (toks or [])][:self.S - max_new - 1]
        if not toks:
            raise ValueError(f"empty prompt (body keys: {sorted(body)})")
        return toks

    def complete(self, body, on_token=None):
        """One request, answered when its last token is out.  on_token(token) streams tokens."""
        max_new = int(body.get("max_tokens", 8))
        if max_new < 1:
            raise ValueError("max_tokens must be at least 1")
        toks = self._tokens(body, max_new)
        sched, name = self._route(body)
        req_id = f"pd-{int(time.time() * 1000)}-{next(self._ids)}"
        first = []

        def tap(tok):
            if not first:
                first.append(time.perf_counter())
            if on_token is not None:
                on_token(tok)
        item = {"tokens": toks, "max_new": max_new, "on_token": tap}
        t0 = time.perf_counter()
        out = sched.submit(item)
        t1 = time.perf_counter()
        xfer = item.get("_xfer")
        gen = out["tokens"]
        pd = {"mode": "disaggregated-kv-transfer" if xfer else "single-card", "config": name,
              "prefill_ms": (xfer or {}).get("prefill_ms", out.get("prefill_ms")),
              "ttft_ms": round(((first[0] if first else t1) - t0) * 1e3, 1),
              "kv_mb": (xfer or {}).get("kv_mb", 0.0),
              "kv_save_ms": (xfer or {}).get("kv_save_ms", 0.0),
              "kv_load_ms": (xfer or {}).get("kv_load_ms", 0.0),
              "tpot_ms": out.get("tpot_ms"), "decode_ms": out.get("decode_ms"),
              "wall_ms": round((t1 - t0) * 1e3, 1)}
        for k in ("batch", "batch_width", "sched", "admit_ms", "occupancy", "starved_lanes", "held_lanes"):
            pd[k] = out.get(k)
        resp = {"id": req_id, "object": "text_completion", "model": self.model,
                "choices": [{"index": 0, "text": self.tk.decode(gen) if self.tk is not None else None,
                             "tokens": gen, "finish_reason": "length"}],
                "usage": {"prompt_tokens": len(toks), "completion_tokens": len(gen),
                          "total_tokens": len(toks) + len(gen)},
                "pd": pd}
        self.window.record(t0, t1, resp)
        return resp


__all__ = ["Gateway"]

"""A prefill/decode box in one process: P prefill GPUs and D decode GPUs behind one gateway
(the end-to-end PD configurations of the reference's deployment: 1P:1D pairs, and 2P:6D with
the gateway round-robining prefill pods, serving/cluster.py:1457-1598).

Every decode GPU runs a BatchDecodeEngine under a ContinuousScheduler whose producer is an
NvlinkProducer: a prompt is prefilled on a prefill GPU and its cache pushed over NVLink into
the decode lane the scheduler leased.  With as many prefill GPUs as decode GPUs each decode
GPU has its own prefill GPU (pairs); otherwise all decode GPUs share a PrefillPool of the
prefill GPUs.  The gateway spreads requests round-robin over the decode GPUs.

    box = build_pd(cfg, state, split=(2, 6))          # GPUs 0-1 prefill, 2-7 decode
    resp = box.gateway.complete({"tokens": prompt, "max_tokens": 64})
    box.close()

`make_prefill(gpu)` / `make_decode(gpu)` build the engines (defaults: FullPrefillEngine with
buckets 256 and 512, BatchDecodeEngine B=16), each GPU with its own copy of the weights.
"""
from rngd_pd.serving.gateway import Gateway
from rngd_pd.serving.scheduler import ContinuousScheduler, NvlinkProducer, PrefillPool

MODEL_NAME = "llama-3.1-8b"


def parse_split(text):
    """'2P:6D' -> (2, 6)."""
    p, _, d = text.upper().partition(":")
    if not (p.endswith("P") and d.endswith("D")):
        raise ValueError(f"split {text!r}: expected the form '2P:6D'")
    return int(p[:-1]), int(d[:-1])


class PDBox:
    def __init__(self, gateway, schedulers, producers, prefill, decode):
        self.gateway, self.schedulers, self.producers = gateway, schedulers, producers
        self.prefill_engines, self.decode_engines = prefill, decode

    def occupancy(self):
        return [s.occupancy() for s in self.schedulers]

    def close(self):
        for s in self.schedulers:
            s.close()
        for p in self.producers:
            p.close()


def build_pd(cfg, state=None, split=(1, 1), B=16, S=512, gpus=None, make_prefill=None, make_decode=None,
             transport=None, model=MODEL_NAME, timeout=10.0):
    """Engines, producers, schedulers and the gateway of one box.  split = (P, D) prefill and
    decode GPUs; gpus = the device indices to use (default 0 .. P+D-1: prefill GPUs first)."""
    n_pre, n_dec = split
    if n_pre < 1 or n_dec < 1:
        raise ValueError(f"split {split}: needs at least one prefill and one decode GPU")
    gpus = list(range(n_pre + n_dec)) if gpus is None else list(gpus)
    if len(gpus) < n_pre + n_dec:
        raise ValueError(f"split {n_pre}P:{n_dec}D needs {n_pre + n_dec} GPUs, have {len(gpus)}")
    if make_prefill is None or make_decode is None:
        from rngd_pd.engines.decode_batch import BatchDecodeEngine
        from rngd_pd.engines.prefill_full import FullPrefillEngine

        def default_prefill(g):
            e = FullPrefillEngine(cfg, state, C=256, group=2, S=S, chip=g)
            e.add_bucket(512)
            return e
        make_prefill = make_prefill or default_prefill
        make_decode = make_decode or (lambda g: BatchDecodeEngine(cfg, state, B=B, S=S, group=8, chip=g))
    pre = [make_prefill(g) for g in gpus[:n_pre]]
    dec = [make_decode(g) for g in gpus[n_pre:n_pre + n_dec]]
    shared = None if n_pre == n_dec else PrefillPool(pre)
    scheds, prods = [], []
    try:
        for i, d in enumerate(dec):
            kv = d.blank_kv()
            prod = NvlinkProducer(pre[i] if shared is None else shared, d, kv, timeout=timeout, transport=transport)
            prods.append(prod)
            scheds.append(ContinuousScheduler(B, d, None, produce_owner=prod, idle_pos=S - 1, kv=kv))
    except BaseException:
        for s in scheds:
            s.close()
        for p in prods:
            p.close()
        raise
    return PDBox(Gateway({model: scheds}, S=S), scheds, prods, pre, dec)


__all__ = ["build_pd", "parse_split", "PDBox"]

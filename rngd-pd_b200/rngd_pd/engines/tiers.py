"""Several decode widths on one card, each step run at the narrowest width that covers every
live lane (API of src/rngd_pd/engines/tiers.py:4-79).

A B=16 step reads the same 15 GB of weights as a B=4 step, but its attention and epilogues
still grow with B, so a lone request should not pay for 16 lanes.  One BatchDecodeEngine per
width shares the weights (BatchDecodeEngine(share=...)); each width keeps its own resident
cache, allocated on first use.  Lane i is lane i at every width, so switching widths copies
only the live lanes' K/V, device to device, on the switching engine's stream.

The caller sees one engine of the widest width: it calls set_live() with the live lanes
before a step, and the (Kd, Vd) it holds are opaque handles (the caches live here).
"""
import torch


class TieredDecode:
    def __init__(self, engines):
        if not engines:
            raise ValueError("TieredDecode needs at least one engine")
        self.tiers = sorted(engines, key=lambda e: e.B)
        widths = [e.B for e in self.tiers]
        if len(set(widths)) != len(widths):
            raise ValueError(f"duplicate widths {widths}")
        self.B = self.tiers[-1].B
        self.by_B = {e.B: e for e in self.tiers}
        self.kv = {}          # width -> (Kd, Vd)
        self.cur = None       # current width
        self.live = []        # sorted live lanes
        self.switches = 0
        self.steps_at = {b: 0 for b in widths}

    # ------------------------------------------------------------ widths
    def _cache(self, width):
        if width not in self.kv:
            self.kv[width] = self.by_B[width].blank_kv()
        return self.kv[width]

    def _width_for(self, top_lane):
        """Narrowest width whose lanes include lane `top_lane`."""
        for e in self.tiers:
            if e.B > top_lane:
                return e.B
        raise ValueError(f"lane {top_lane} outside the widest engine (B={self.B})")

    def _switch(self, width):
        """Make `width` current, carrying the live lanes' caches over (one gather-copy per
        cache group, on the new width's stream, ordered after the old width's stream)."""
        if self.cur == width:
            return
        Kn, Vn = self._cache(width)
        if self.cur is not None and self.live:
            Ko, Vo = self.kv[self.cur]
            new, old = self.by_B[width], self.by_B[self.cur]
            idx = torch.tensor(self.live, dtype=torch.long, device=Kn[0].device)

            def copy():
                for g in range(len(Kn)):
                    Kn[g].index_copy_(1, idx, Ko[g].index_select(1, idx))
                    Vn[g].index_copy_(1, idx, Vo[g].index_select(1, idx))

            if Kn[0].is_cuda:
                with torch.cuda.device(Kn[0].device):
                    new.stream.wait_stream(old.stream)
                    with torch.cuda.stream(new.stream):
                        copy()
                    old.stream.wait_stream(new.stream)
            else:
                copy()
            self.switches += 1
        self.cur = width

    # -------------------------------------------------- engine interface
    def blank_kv(self):
        self._switch(self.tiers[0].B)
        return self, self

    def set_live(self, live):
        self.live = sorted(int(i) for i in live)
        if self.live and self.live[-1] >= self.B:
            raise ValueError(f"lane {self.live[-1]} outside the widest engine (B={self.B})")

    def write_slot_kv(self, Kd, Vd, idx, K, V):
        """Admit a request's K/V into lane idx (widening first if the lane needs it)."""
        need = self._width_for(max(self.live + [idx]))
        if self.cur is None or need > self.cur:
            self._switch(need)
        Kc, Vc = self.kv[self.cur]
        self.kv[self.cur] = self.by_B[self.cur].write_slot_kv(Kc, Vc, idx, K, V)
        if idx not in self.live:
            self.live = sorted(self.live + [idx])
        return Kd, Vd

    def adopt_kv_device(self, Ks, Vs):
        """Per-request device caches into lanes 0..n-1 (the widest engine's API)."""
        for i, (K, V) in enumerate(zip(Ks, Vs)):
            self.write_slot_kv(self, self, i, K, V)
        return self, self

    def _lanes(self, width, toks, positions):
        toks, positions = list(toks), list(positions)
        return toks[:width], positions[:width]

    def step(self, toks, positions, Kd, Vd):
        """One greedy step at the narrowest width covering the live lanes; returns B tokens
        (zeros past the width), like the widest engine's step()."""
        if not self.live:
            return [0] * self.B, Kd, Vd
        self._switch(self._width_for(self.live[-1]))
        width = self.cur
        e = self.by_B[width]
        t, p = self._lanes(width, toks, positions)
        Kc, Vc = self.kv[width]
        nxt, Kc, Vc = e.step(t, p, Kc, Vc)
        self.kv[width] = (Kc, Vc)
        self.steps_at[width] += 1
        return list(nxt) + [0] * (self.B - width), Kd, Vd

    def step_logits(self, toks, positions, Kd, Vd):
        """step() returning the current width's logits ([32, Vp/32, width] bf16 layout of the
        reference) instead of tokens."""
        if not self.live:
            raise ValueError("step_logits with no live lane")
        self._switch(self._width_for(self.live[-1]))
        width = self.cur
        e = self.by_B[width]
        t, p = self._lanes(width, toks, positions)
        Kc, Vc = self.kv[width]
        lg, Kc, Vc = e.step_logits(t, p, Kc, Vc)
        self.kv[width] = (Kc, Vc)
        self.steps_at[width] += 1
        return lg, Kd, Vd

    def download_kv(self, Kd=None, Vd=None):
        """The current width's cache on the host (reference layout)."""
        Kc, Vc = self.kv[self.cur]
        return self.by_B[self.cur].download_kv(Kc, Vc)


__all__ = ["TieredDecode"]

"""Cross-node KV through NIXL's UCX backend (the `nixl-ucx` path of the reference's
src/rngd_pd/connector/ucxkv.py, same public names and descriptor bytes).

A pushing process copies a blob into a NIXL-registered host pool and publishes a small
descriptor (where the bytes are, how many, their CRC-32, and the agent to read them from)
under the blob's key in a TcpKVServer; the pulling process takes the descriptor and READs the
bytes one-sidedly over UCX into its own registered pool.  The READ carries a notification
that lets the pusher reuse the space.  Only descriptors cross the relay.  UCX_TLS chooses the
wire (tcp, or verbs when an RDMA NIC is present) without a code change.  Nothing falls back:
no NIXL, a failed READ or a CRC mismatch raises.

How this module is built:

  HostPool   an anonymous mmap (page-aligned by construction, as registration wants) cut into
             4 KiB pages.  A byte map marks used pages, and a cursor makes allocation go round
             the pool in ring order: KV blobs are mostly read in the order they were pushed, so
             the space freed first is the space reached next and the pool does not fragment at
             its start.  A request that finds no room waits on a condition, bounded.
  _Outbox    the pushing side.  It holds the send pool and a ledger of the slots still
             published.  Reclaiming is lazy: every push, every pending() and every wait for room
             drains the agent's notifications and expires slots older than the TTL.  There is no
             reaper thread, so a store that is only pushed to costs no CPU between pushes.
  _Inbox     the pulling side: the receive pool, the agents already loaded, and the READ
             itself, polled with a backoff from 20 us to 1 ms.
  UcxKVStore push / pull / pending / describe / close, and stats.

The descriptor is a wire format shared with the reference's pods: magic b"AKU1", then
little-endian address:u64, n:u64, crc:u32, name length:i32, metadata length:i32, the agent
name and the agent metadata.

Environment: AIRM_KV_UCX_POOL_MB (pool per side, 1024), AIRM_KV_UCX_XFER_TIMEOUT_S (60),
AIRM_KV_TCP_TTL_S (900), AIRM_KV_TCP_CRC (1), and UCX's own UCX_* variables.
"""
import ctypes
import json
import mmap
import os
import socket
import struct
import threading
import time
import uuid
import zlib

import numpy as np

BACKEND = "UCX"
MAGIC = b"AKU1"
DESC = struct.Struct("<4sQQIii")
FREE_TAG = b"airm-free:"
# UCX's tcp transport moves 8 KiB segments unless told otherwise; 64 KiB segments carry a
# 1 MiB READ markedly faster.  Verbs transports ignore both; values already set win.
UCX_DEFAULTS = {"UCX_TCP_TX_SEG_SIZE": "65536", "UCX_TCP_RX_SEG_SIZE": "65536"}
PAGE = 4096


def crc_enabled():
    return os.environ.get("AIRM_KV_TCP_CRC", "1").strip().lower() not in ("0", "false", "no")


def make_agent(name):
    """A NIXL agent named `name` with the UCX backend created (UCX reads UCX_* here)."""
    for var, value in UCX_DEFAULTS.items():
        os.environ.setdefault(var, value)
    from nixl._api import nixl_agent, nixl_agent_config
    agent = nixl_agent(name, nixl_agent_config(backends=[]))
    agent.create_backend(BACKEND, {})
    return agent


def pack_desc(name, metadata, address, n, crc):
    """Descriptor bytes for `n` bytes at `address` in agent `name`'s registered memory."""
    name_b, md = name.encode(), bytes(metadata)
    head = DESC.pack(MAGIC, int(address), int(n), int(crc), len(name_b), len(md))
    return b"".join((head, name_b, md))


def unpack_desc(blob):
    """Descriptor bytes -> (agent name, agent metadata, address, n, crc); IOError if the bytes
    are not one well-formed descriptor."""
    raw = bytes(blob)
    if len(raw) >= DESC.size:
        magic, address, n, crc, name_len, md_len = DESC.unpack_from(raw)
        body = raw[DESC.size:]
        if magic == MAGIC and name_len >= 0 and md_len >= 0 and len(body) == name_len + md_len:
            return body[:name_len].decode(), body[name_len:], address, n, crc
    raise IOError("ucxkv: malformed descriptor")


class HostPool:
    """Page-granular host memory for registered transfers (see the module docstring).

    take(n, timeout) -> (offset, pages) reserves ceil(n / page) contiguous pages; give(offset,
    pages) returns them.  view(offset, n) is a numpy uint8 view.  Thread-safe."""

    def __init__(self, nbytes, page=PAGE):
        self.page = int(page)
        self.pages = max(1, -(-int(nbytes) // self.page))
        self.size = self.pages * self.page
        self._map = mmap.mmap(-1, self.size, flags=mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS)
        self.buf = np.frombuffer(self._map, dtype=np.uint8)
        self.address = ctypes.addressof(ctypes.c_char.from_buffer(self._map))
        self._used = np.zeros(self.pages, np.uint8)
        self._cursor = 0
        self._in_use = 0
        self._cv = threading.Condition()

    def _find(self, k):
        """Start page of a free run of k pages, from the cursor onwards, else from page 0."""
        c = self._cursor
        if c + k <= self.pages and not self._used[c:c + k].any():
            return c
        free = np.concatenate(([0], np.cumsum(self._used == 0, dtype=np.int64)))
        fits = np.flatnonzero(free[k:] - free[:-k] == k)
        if fits.size == 0:
            return None
        later = fits[fits >= c]
        return int(later[0] if later.size else fits[0])

    def take(self, n, timeout=0.0, while_waiting=None):
        """Reserve room for n bytes, waiting up to `timeout` s.  while_waiting() is called
        (outside the pool's lock) before each wait, so an owner can reclaim space meanwhile."""
        k = max(1, -(-int(n) // self.page))
        if k > self.pages:
            raise ValueError(f"ucxkv: {n} bytes do not fit a pool of {self.size} (AIRM_KV_UCX_POOL_MB)")
        deadline = time.monotonic() + max(0.0, float(timeout))
        while True:
            with self._cv:
                start = self._find(k)
                if start is not None:
                    self._used[start:start + k] = 1
                    self._cursor = (start + k) % self.pages
                    self._in_use += k
                    return start * self.page, k
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"ucxkv: no room for {n} bytes in the pool within {timeout:.1f} s")
                if while_waiting is None:
                    self._cv.wait(left)
                    continue
            while_waiting()
            with self._cv:
                if self._find(k) is None:
                    self._cv.wait(min(0.002, max(0.0, deadline - time.monotonic())))

    def give(self, offset, pages):
        first = offset // self.page
        with self._cv:
            self._used[first:first + pages] = 0
            self._in_use -= pages
            self._cv.notify_all()

    def view(self, offset, n):
        return self.buf[offset:offset + n]

    def free_bytes(self):
        with self._cv:
            return (self.pages - self._in_use) * self.page

    def close(self):
        self.buf = None
        try:
            self._map.close()
        except BufferError:          # a caller still holds a view; the mapping goes with it
            pass


class _Outbox:
    """Pushing side: the registered send pool and the ledger of published slots."""

    def __init__(self, store):
        self.store = store
        self.pool = None
        self.metadata = None
        self.ledger = {}                  # key -> (offset, pages, published at)
        self.lock = threading.Lock()

    def ready(self):
        if self.pool is None:
            s = self.store
            with s.nixl_lock:
                if self.pool is None:
                    pool = HostPool(s.pool_bytes)
                    s.registrations.append(s.agent().register_memory([(pool.address, pool.size, 0, "")], "DRAM",
                                                                     [BACKEND]))
                    self.metadata = s.agent().get_agent_metadata()   # describes the send pool
                    self.pool = pool
        return self.pool

    def _drop(self, key, counter):
        with self.lock:
            slot = self.ledger.pop(key, None)
        if slot is not None:
            self.pool.give(slot[0], slot[1])
            self.store.stats[counter] += 1

    def reclaim(self):
        """Free the slots whose READ notification came in, and those past the TTL."""
        if self.pool is None:
            return
        s = self.store
        try:
            with s.nixl_lock:
                notes = s.agent().get_new_notifs()
        except Exception:                 # a broken agent frees nothing; TTL still applies
            notes = {}
        for messages in notes.values():
            for m in messages:
                m = bytes(m)
                if m.startswith(FREE_TAG):
                    self._drop(m[len(FREE_TAG):].decode(), "freed")
        cutoff = time.monotonic() - s.ttl_s
        with self.lock:
            old = [k for k, (_o, _p, t) in self.ledger.items() if t < cutoff]
        for key in old:
            self._drop(key, "expired")

    def publish(self, key, data):
        pool = self.ready()
        self.reclaim()
        n = data.nbytes
        offset, pages = pool.take(n, timeout=self.store.xfer_timeout_s, while_waiting=self.reclaim)
        try:
            pool.view(offset, n)[:] = np.frombuffer(data, np.uint8)
            crc = zlib.crc32(data) if crc_enabled() else 0
            with self.lock:
                self.ledger[key] = (offset, pages, time.monotonic())
            desc = pack_desc(self.store.name, self.metadata, pool.address + offset, n, crc)
            self.store.control.push(key, desc)
        except BaseException:
            with self.lock:
                self.ledger.pop(key, None)
            pool.give(offset, pages)
            raise


def _backoff():
    delay = 20e-6
    while True:
        yield delay
        delay = min(1e-3, delay * 2)


class _Inbox:
    """Pulling side: the registered receive pool, the loaded agents and the READ."""

    def __init__(self, store):
        self.store = store
        self.pool = None
        self.peers = set()

    def ready(self):
        if self.pool is None:
            s = self.store
            with s.nixl_lock:
                if self.pool is None:
                    pool = HostPool(s.pool_bytes)
                    s.registrations.append(s.agent().register_memory([(pool.address, pool.size, 0, "")], "DRAM",
                                                                     [BACKEND]))
                    self.pool = pool
        return self.pool

    def read(self, key, name, metadata, address, n):
        """READ n bytes at `address` of agent `name` and return a copy of them."""
        s = self.store
        pool = self.ready()
        offset, pages = pool.take(n, timeout=s.xfer_timeout_s)
        try:
            with s.nixl_lock:
                agent = s.agent()
                if name != s.name and name not in self.peers:        # own agent: UCX loopback
                    agent.add_remote_agent(metadata)
                    self.peers.add(name)
                here = agent.get_xfer_descs([(pool.address + offset, n, 0)], "DRAM")
                there = agent.get_xfer_descs([(address, n, 0)], "DRAM")
                xfer = agent.initialize_xfer("READ", here, there, name, FREE_TAG + key.encode(), [BACKEND])
                state = agent.transfer(xfer)
            give_up = time.monotonic() + s.xfer_timeout_s
            pause = _backoff()
            while state == "PROC" and time.monotonic() < give_up:
                time.sleep(next(pause))
                with s.nixl_lock:
                    state = agent.check_xfer_state(xfer)
            with s.nixl_lock:
                xfer.release()
            if state != "DONE":
                outcome = "did not finish in time" if state == "PROC" else f"ended as {state}"
                raise IOError(f"ucxkv pull {key}: the NIXL READ from {name} {outcome}")
            return bytearray(pool.view(offset, n))
        finally:
            pool.give(offset, pages)


class UcxKVStore:
    """push / pull of blobs between processes on any hosts, the bytes over NIXL UCX.

    control: anything with push(key, bytes) and take(key, timeout), normally a TcpKVClient, for
    the descriptors.  agent: a NIXL agent with the UCX backend (tests pass a fake), else one is
    made on first use.  One store can push and pull; each role registers its own pool once."""

    def __init__(self, control, agent=None, pool_bytes=None, name=None, xfer_timeout_s=None, ttl_s=None):
        self.control = control
        self._agent = agent
        self.name = name or getattr(agent, "name", None) or \
            "rngd-ucx-%s-%d-%s" % (socket.gethostname(), os.getpid(), uuid.uuid4().hex[:8])
        self.pool_bytes = int(pool_bytes) if pool_bytes else int(os.environ.get("AIRM_KV_UCX_POOL_MB", "1024")) << 20
        self.xfer_timeout_s = float(xfer_timeout_s if xfer_timeout_s is not None
                                    else os.environ.get("AIRM_KV_UCX_XFER_TIMEOUT_S", "60"))
        self.ttl_s = float(ttl_s if ttl_s is not None else os.environ.get("AIRM_KV_TCP_TTL_S", "900"))
        self.nixl_lock = threading.RLock()       # NIXL agents are driven by one thread at a time
        self.registrations = []
        self.stats = dict.fromkeys(("pushed", "pulled", "freed", "expired", "bytes_out", "bytes_in"), 0)
        self.outbox = _Outbox(self)
        self.inbox = _Inbox(self)

    def agent(self):
        if self._agent is None:
            try:
                self._agent = make_agent(self.name)
            except Exception as e:
                raise RuntimeError(f"ucxkv: no NIXL agent with the {BACKEND} backend "
                                   f"({type(e).__name__}: {e}); the nixl wheel ships the UCX plugin") from e
        return self._agent

    def push(self, key, buf):
        """Stage `buf` (any contiguous buffer) and publish its descriptor under `key`."""
        data = memoryview(buf).cast("B")
        self.outbox.publish(key, data)
        self.stats["pushed"] += 1
        self.stats["bytes_out"] += data.nbytes

    def pull(self, key, timeout=5.0):
        """The bytes pushed under `key` (a bytearray).  TimeoutError if no descriptor came within
        `timeout` s; IOError if the READ failed or the bytes fail their CRC."""
        name, metadata, address, n, crc = unpack_desc(self.control.take(key, timeout=timeout))
        data = self.inbox.read(key, name, metadata, address, n)
        if crc and crc_enabled() and zlib.crc32(data) != crc:
            raise IOError(f"ucxkv pull {key}: CRC mismatch (the sender's slot was reused or expired)")
        self.stats["pulled"] += 1
        self.stats["bytes_in"] += n
        return data

    def pending(self):
        """Keys pushed here whose slots are still held (not read, not expired)."""
        self.outbox.reclaim()
        with self.outbox.lock:
            return sorted(self.outbox.ledger)

    def describe(self):
        return {"agent": self.name, "backend": BACKEND,
                "ucx_tls": os.environ.get("UCX_TLS", "(UCX default)"),
                "ucx_net_devices": os.environ.get("UCX_NET_DEVICES", "(UCX default)")}

    def close(self):
        agent = self._agent
        if agent is not None:
            with self.nixl_lock:
                for name in sorted(self.inbox.peers):
                    try:
                        agent.remove_remote_agent(name)
                    except Exception:
                        pass
                for reg in self.registrations:
                    try:
                        agent.deregister_memory(reg, [BACKEND])
                    except Exception:
                        pass
        self.inbox.peers.clear()
        self.registrations = []
        with self.outbox.lock:
            self.outbox.ledger.clear()


def probe():
    """What this host's NIXL / UCX set-up would use, and whether an agent can be made."""
    store = UcxKVStore(control=None, pool_bytes=PAGE)
    report = dict(store.describe())
    try:
        store.agent()
        report["ok"] = True
    except RuntimeError as e:
        report.update(ok=False, error=str(e))
    finally:
        store.close()
    return report


if __name__ == "__main__":
    print(json.dumps(probe()))

"""Cross-node KV through NIXL's UCX backend (API and descriptor format of
src/rngd_pd/connector/ucxkv.py): host-staged blobs, one-sided READ, descriptors through the
TCP relay.

Each process owns host arenas registered with NIXL once.  The pushing side copies a blob
into a slot of its send arena and publishes a descriptor under the blob's key in a
TcpKVServer (the `tcp` transport's relay, or one beside decode); the pulling side takes the
descriptor, loads the sender's agent metadata once, READs the bytes into its receive arena
over UCX (RDMA READ on verbs, TCP otherwise: UCX_TLS decides, the code does not change),
checks the CRC-32, and the READ's notification tells the sender to free the slot.  Only
descriptors (a few KB) cross the relay.  A slot nobody reads within the TTL
($AIRM_KV_TCP_TTL_S, 900 s) is freed, and a READ after that fails its CRC instead of returning
stale bytes.  Nothing falls back: no NIXL, no UCX or a failed READ raises.

The descriptor is the reference's byte for byte, so pods of either build read each other's
blobs: magic b"AKU1", then little-endian address:u64, n:u64, crc:u32, name length:i32,
metadata length:i32, the agent name and the agent metadata.

Environment: AIRM_KV_UCX_POOL_MB (arena per side, 1024), AIRM_KV_UCX_XFER_TIMEOUT_S (60),
AIRM_KV_TCP_CRC (1), UCX_* (UCX's own; UCX_TCP_TX/RX_SEG_SIZE default to 64 KiB here).
"""
import json
import os
import socket
import struct
import threading
import time
import uuid
import zlib

BACKEND = "UCX"
MAGIC = b"AKU1"
DESC = struct.Struct("<4sQQIii")           # magic, address, n, crc, name length, metadata length
FREE_TAG = b"airm-free:"
# larger UCX tcp segments than UCX's 8 KiB default (the reference measured 0.26 -> 0.44 GB/s
# for a 1 MiB READ); verbs transports ignore them, and the environment wins
UCX_DEFAULTS = {"UCX_TCP_TX_SEG_SIZE": "65536", "UCX_TCP_RX_SEG_SIZE": "65536"}


def crc_enabled():
    return os.environ.get("AIRM_KV_TCP_CRC", "1") not in ("0", "false", "no")


def make_agent(name):
    """A NIXL agent with the UCX backend (UCX reads its UCX_* environment here)."""
    for k, v in UCX_DEFAULTS.items():
        os.environ.setdefault(k, v)
    from nixl._api import nixl_agent, nixl_agent_config
    agent = nixl_agent(name, nixl_agent_config(backends=[]))
    agent.create_backend(BACKEND, {})
    return agent


def pack_desc(name, metadata, address, n, crc):
    nb = name.encode()
    return DESC.pack(MAGIC, address, n, crc, len(nb), len(metadata)) + nb + bytes(metadata)


def unpack_desc(blob):
    """descriptor bytes -> (agent name, agent metadata, address, n, crc); IOError if malformed."""
    blob = bytes(blob)
    if len(blob) < DESC.size:
        raise IOError("ucxkv: malformed descriptor")
    magic, address, n, crc, nl, ml = DESC.unpack_from(blob)
    if magic != MAGIC or nl < 0 or ml < 0 or len(blob) != DESC.size + nl + ml:
        raise IOError("ucxkv: malformed descriptor")
    return blob[DESC.size:DESC.size + nl].decode(), blob[DESC.size + nl:], address, n, crc


class Arena:
    """A page-aligned host buffer with a first-fit allocator of 64-byte-aligned slots.
    alloc(n, timeout) waits up to `timeout` s for room; free() merges neighbours.  Thread-safe."""

    ALIGN = 64

    def __init__(self, nbytes):
        import numpy as np
        self.size = int(nbytes)
        self._mem = np.empty(self.size + 4096, np.uint8)
        skip = (-self._mem.ctypes.data) % 4096
        self.buf = self._mem[skip:skip + self.size]
        self.address = self._mem.ctypes.data + skip
        self._holes = [(0, self.size)]                 # (offset, length), sorted, disjoint
        self._cv = threading.Condition()

    def alloc(self, n, timeout=0.0):
        span = max(self.ALIGN, -(-int(n) // self.ALIGN) * self.ALIGN)
        if span > self.size:
            raise ValueError(f"ucxkv: {n} bytes do not fit an arena of {self.size} (AIRM_KV_UCX_POOL_MB)")
        deadline = time.monotonic() + max(0.0, timeout)
        with self._cv:
            while True:
                for i, (off, length) in enumerate(self._holes):
                    if length >= span:
                        if length == span:
                            del self._holes[i]
                        else:
                            self._holes[i] = (off + span, length - span)
                        return off, span
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"ucxkv: no {n} free bytes in the arena within {timeout:.1f} s")
                self._cv.wait(left)

    def free(self, off, span):
        with self._cv:
            holes = sorted(self._holes + [(off, span)])
            merged = [holes[0]]
            for o, l in holes[1:]:
                po, pl = merged[-1]
                if po + pl == o:
                    merged[-1] = (po, pl + l)
                else:
                    merged.append((o, l))
            self._holes = merged
            self._cv.notify_all()

    def free_bytes(self):
        with self._cv:
            return sum(l for _o, l in self._holes)


class UcxKVStore:
    """push / pull of blobs between processes on any hosts, the bytes over NIXL UCX.

    control: anything with push(key, bytes) / take(key, timeout) (a TcpKVClient) for the
    descriptors.  agent: a NIXL agent with the UCX backend (tests pass a fake); made on first
    use otherwise.  One store serves both roles, with one registered arena per role."""

    def __init__(self, control, agent=None, pool_bytes=None, name=None, xfer_timeout_s=None, ttl_s=None,
                 poll_s=0.0005):
        self.control = control
        self.name = name or getattr(agent, "name", None) or \
            f"airm-kv-{socket.gethostname()}-{os.getpid()}-{uuid.uuid4().hex[:6]}"
        self.pool_bytes = int(pool_bytes or int(os.environ.get("AIRM_KV_UCX_POOL_MB", "1024")) << 20)
        self.xfer_timeout_s = float(xfer_timeout_s or os.environ.get("AIRM_KV_UCX_XFER_TIMEOUT_S", "60"))
        self.ttl_s = float(ttl_s if ttl_s is not None else os.environ.get("AIRM_KV_TCP_TTL_S", "900"))
        self.poll_s = poll_s
        self._agent = agent
        self._lock = threading.RLock()          # every NIXL call and the tables below
        self._send = self._recv = None          # registered arenas
        self._regs, self._metadata, self._remotes = [], None, {}
        self._slots = {}                        # key -> (offset, span, published at)
        self._stop = threading.Event()
        self._reaper = None
        self.stats = {"pushed": 0, "pulled": 0, "freed": 0, "expired": 0, "bytes_out": 0, "bytes_in": 0}

    # -- set-up -------------------------------------------------------------------------
    def _nixl(self):
        if self._agent is None:
            try:
                self._agent = make_agent(self.name)
            except Exception as e:
                raise RuntimeError(f"ucxkv: no NIXL agent with the {BACKEND} backend ({type(e).__name__}: {e}); "
                                   "install nixl (its wheel ships the UCX plugin)") from e
        return self._agent

    def _registered(self, role):
        """The send or receive arena, allocated and registered with NIXL on first use."""
        with self._lock:
            have = self._send if role == "send" else self._recv
            if have is not None:
                return have
            agent = self._nixl()
            arena = Arena(self.pool_bytes)
            self._regs.append(agent.register_memory([(arena.address, arena.size, 0, "")], "DRAM", [BACKEND]))
            if role == "send":
                self._send = arena
                self._metadata = agent.get_agent_metadata()          # now carries the send arena
                self._reaper = threading.Thread(target=self._reap, daemon=True, name="ucxkv-reaper")
                self._reaper.start()
            else:
                self._recv = arena
            return arena

    # -- sending side -------------------------------------------------------------------
    def push(self, key, buf):
        """Stage `buf` in the send arena and publish its descriptor under `key`."""
        mv = memoryview(buf).cast("B")
        n = mv.nbytes
        arena = self._registered("send")
        off, span = arena.alloc(n, timeout=self.xfer_timeout_s)
        try:
            arena.buf[off:off + n] = mv
            crc = zlib.crc32(mv) if crc_enabled() else 0
            with self._lock:
                self._slots[key] = (off, span, time.monotonic())
            self.control.push(key, pack_desc(self.name, self._metadata, arena.address + off, n, crc))
        except BaseException:
            with self._lock:
                self._slots.pop(key, None)
            arena.free(off, span)
            raise
        self.stats["pushed"] += 1
        self.stats["bytes_out"] += n

    def _drop(self, key, expired=False):
        with self._lock:
            slot = self._slots.pop(key, None)
        if slot is not None:
            self._send.free(slot[0], slot[1])
            self.stats["expired" if expired else "freed"] += 1

    def _reap(self):
        """Free a slot when its reader's READ notification arrives, or once its TTL has passed."""
        agent = self._nixl()
        while not self._stop.is_set():
            try:
                with self._lock:
                    notes = agent.get_new_notifs()
            except Exception:
                notes = {}
            freed = False
            for msgs in notes.values():
                for m in msgs:
                    m = bytes(m)
                    if m.startswith(FREE_TAG):
                        self._drop(m[len(FREE_TAG):].decode())
                        freed = True
            now = time.monotonic()
            with self._lock:
                stale = [k for k, (_o, _s, t) in self._slots.items() if now - t > self.ttl_s]
            for k in stale:
                self._drop(k, expired=True)
            if not freed:
                self._stop.wait(0.002)

    def pending(self):
        """Keys pushed here whose slots are still held (not read yet)."""
        with self._lock:
            return sorted(self._slots)

    # -- receiving side -------------------------------------------------------------------
    def pull(self, key, timeout=5.0):
        """The bytes pushed under `key` (a bytearray), READ over UCX; TimeoutError if the
        descriptor never came, IOError if the READ failed or the CRC does not match."""
        name, md, address, n, crc = unpack_desc(self.control.take(key, timeout=timeout))
        arena = self._registered("recv")
        agent = self._nixl()
        off, span = arena.alloc(n, timeout=self.xfer_timeout_s)
        try:
            with self._lock:
                if name != self.name and name not in self._remotes:     # own agent: UCX loopback
                    self._remotes[name] = agent.add_remote_agent(md)
                mine = agent.get_xfer_descs([(arena.address + off, n, 0)], "DRAM")
                theirs = agent.get_xfer_descs([(address, n, 0)], "DRAM")
                h = agent.initialize_xfer("READ", mine, theirs, name, FREE_TAG + key.encode(), [BACKEND])
                state = agent.transfer(h)
            deadline = time.monotonic() + self.xfer_timeout_s
            while state == "PROC" and time.monotonic() < deadline:
                if self.poll_s:
                    time.sleep(self.poll_s)
                with self._lock:
                    state = agent.check_xfer_state(h)
            with self._lock:
                h.release()
            if state != "DONE":
                why = "timed out" if state == "PROC" else f"ended in state {state}"
                raise IOError(f"ucxkv pull {key}: NIXL READ from {name} {why}")
            data = bytearray(arena.buf[off:off + n])
        finally:
            arena.free(off, span)
        if crc and crc_enabled() and zlib.crc32(data) != crc:
            raise IOError(f"ucxkv pull {key}: crc mismatch (the source slot was freed or overwritten)")
        self.stats["pulled"] += 1
        self.stats["bytes_in"] += n
        return data

    # -- lifecycle --------------------------------------------------------------------------
    def describe(self):
        return {"agent": self.name, "backend": BACKEND, "ucx_tls": os.environ.get("UCX_TLS", "(UCX default)"),
                "ucx_net_devices": os.environ.get("UCX_NET_DEVICES", "(UCX default)")}

    def close(self):
        self._stop.set()
        if self._reaper is not None:
            self._reaper.join(1.0)
        agent = self._agent
        if agent is None:
            return
        with self._lock:
            for name in list(self._remotes):
                try:
                    agent.remove_remote_agent(name)
                except Exception:
                    pass
            self._remotes.clear()
            for reg in self._regs:
                try:
                    agent.deregister_memory(reg, [BACKEND])
                except Exception:
                    pass
            self._regs.clear()
            self._slots.clear()


def main(argv=None):
    """Print what this host's NIXL/UCX would use: python -m rngd_pd.connector.ucxkv"""
    s = UcxKVStore(control=None, pool_bytes=1 << 20)
    try:
        s._nixl()
        print(json.dumps(dict(s.describe(), ok=True)))
    except RuntimeError as e:
        print(json.dumps(dict(s.describe(), ok=False, error=str(e))))
    finally:
        s.close()


if __name__ == "__main__":
    main()

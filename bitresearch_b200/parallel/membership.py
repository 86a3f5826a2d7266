"""Rendezvous, ring formation, heartbeats and dynamic timeouts over a ``torch.distributed`` store.

This replaces the reference's WebSocket signalling server and WebRTC keep-alive:

* peers register in a room; the ring is the alive compute peers sorted by id, each with a left and
  a right neighbour, and a version counter bumped on every re-formation (server/signaling.ts:75-119);
* each peer refreshes a heartbeat key every ``heartbeat_s`` seconds (the reference pings every 2 s,
  webrtc-mesh.ts:173-196) and keeps an EMA (beta 0.9) of its store round-trip time
  (webrtc-mesh.ts:514-528);
* ``dynamic_timeout_s = max(10, 3 * max_rtt + 5)`` seconds (webrtc-mesh.ts:99-109);
* a peer whose heartbeat is older than ``dead_after_s`` is dropped at the next ``form_ring``, the
  equivalent of the server's ``peer-left`` + re-formation (server/signaling.ts:264-295);
* a re-formation that must include newcomers (the server re-forms on join too, :210-213) is decided by
  one member, which publishes the new peer list under a sequence number (``publish_ring``); every
  member and every joining peer forms its ring from that list (``wait_published``), so all of them
  build the same group even when they read the heartbeats at different times.

``ElasticGroup`` is a gloo process group over the members of one ring version, built from the job's
store under a per-version prefix. Forming it needs no collective over the old group, so the survivors
of a lost rank can build it on their own; the trainer's ``elastic`` ring path re-forms this way
(``Trainer._reform``). The in-kernel NVLink path and NCCL keep a fixed group: a lost rank there ends the
job with an error at the next collective's timeout.
"""
from __future__ import annotations

import datetime
import threading
import time
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class RingTopology:
    position: int
    total: int
    left: str
    right: str
    version: int
    peers: list[str]


class Membership:
    def __init__(self, store, peer_id: str, room: str = "default", heartbeat_s: float = 2.0,
                 dead_after_s: float = 10.0, peer_type: str = "compute", heartbeat_store=None):
        self.store = store
        # the heartbeat thread writes through its own store client when given one, so a long blocking
        # store call of the main thread never delays a beat
        self.hb_store = heartbeat_store if heartbeat_store is not None else store
        self.beat_errors = 0
        self.peer_id = peer_id
        self.room = room
        self.heartbeat_s = heartbeat_s
        self.dead_after_s = dead_after_s
        self.peer_type = peer_type
        self.smoothed_rtt_s = 0.0
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def _k(self, *parts: str) -> str:
        return "/".join((self.room, *parts))

    def register(self) -> int:
        idx = self.store.add(self._k("count"), 1) - 1
        self.store.set(self._k("peer", str(idx)), f"{self.peer_id}|{self.peer_type}")
        self.beat()
        return idx

    def beat(self, store=None) -> None:
        store = self.store if store is None else store
        t0 = time.time()
        store.set(self._k("hb", self.peer_id), repr(t0))
        store.get(self._k("hb", self.peer_id))
        rtt = time.time() - t0
        self.smoothed_rtt_s = rtt if self.smoothed_rtt_s == 0 else 0.9 * self.smoothed_rtt_s + 0.1 * rtt

    def leave(self) -> None:
        self.stop()
        self.store.set(self._k("hb", self.peer_id), repr(0.0))

    def start(self) -> None:
        def run():
            while not self._stop.wait(self.heartbeat_s):
                try:
                    self.beat(self.hb_store)
                except Exception:  # a transient store error skips one beat; peers tolerate dead_after_s
                    self.beat_errors += 1
        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()

    def registered_peers(self) -> list[tuple[str, str]]:
        n = int(self.store.add(self._k("count"), 0))
        out = []
        for i in range(n):
            pid, _, ptype = self.store.get(self._k("peer", str(i))).decode().partition("|")
            out.append((pid, ptype))
        return out

    def last_seen(self, pid: str) -> float:
        try:
            return float(self.store.get(self._k("hb", pid)).decode())
        except Exception:
            return 0.0

    def alive_peers(self, now: float | None = None) -> list[str]:
        now = time.time() if now is None else now
        # a peer id registered twice (a process that re-registered) counts once
        return sorted({pid for pid, ptype in self.registered_peers()
                       if ptype == "compute" and now - self.last_seen(pid) <= self.dead_after_s})

    def form_ring(self) -> RingTopology | None:
        return self.ring_from(self.alive_peers())

    def ring_from(self, peers: list[str]) -> RingTopology | None:
        """This peer's place in the ring over ``peers`` (None if it is not one of them)."""
        peers = sorted(set(peers))
        if self.peer_id not in peers:
            return None
        N = len(peers)
        i = peers.index(self.peer_id)
        key = self._k("ring", ",".join(peers))
        # every member of the same peer set agrees on one version number
        if self.store.add(key + "/claim", 1) == 1:
            self.store.set(key, str(self.store.add(self._k("ring_version"), 1)))
        version = int(self.store.get(key).decode())
        return RingTopology(i, N, peers[(i - 1) % N], peers[(i + 1) % N], version, peers)

    @property
    def dynamic_timeout_s(self) -> float:
        if self.smoothed_rtt_s <= 0:
            return 10.0
        return max(10.0, 3 * self.smoothed_rtt_s + 5.0)

    def wait_for(self, n: int, timeout_s: float = 60.0) -> RingTopology:
        """Waits until ``n`` compute peers are registered and alive, then forms the ring."""
        deadline = time.time() + timeout_s
        while True:
            if len(self.alive_peers()) >= n:
                ring = self.form_ring()
                if ring is not None and ring.total >= n:
                    return ring
            if time.time() > deadline:
                raise TimeoutError(f"only {len(self.alive_peers())} of {n} peers joined room {self.room!r}")
            time.sleep(min(0.05, self.heartbeat_s))

    def latest_published(self) -> int:
        return int(self.store.add(self._k("ring_seq"), 0))

    def publish_ring(self, peers: list[str]) -> int:
        """Makes ``peers`` the next ring (called by one member); returns its sequence number."""
        seq = int(self.store.add(self._k("ring_seq"), 1))
        self.store.set(self._k("ring_list", str(seq)), ",".join(sorted(set(peers))))
        return seq

    def wait_published(self, after: int, timeout_s: float = 60.0) -> tuple[int, RingTopology]:
        """Waits for a ring list published after sequence number ``after`` that includes this peer;
        returns (its sequence number, this peer's place in it)."""
        deadline = time.time() + timeout_s
        seen = after
        while True:
            latest = self.latest_published()
            for seq in range(seen + 1, latest + 1):
                peers = self.store.get(self._k("ring_list", str(seq))).decode().split(",")
                ring = self.ring_from(peers)
                if ring is not None:
                    return seq, ring
            seen = max(seen, latest)
            if time.time() > deadline:
                raise TimeoutError(f"no ring including {self.peer_id} was published in room {self.room!r} "
                                   f"within {timeout_s:.0f} s")
            time.sleep(min(0.05, self.heartbeat_s))

    def wait_for_change(self, peers: list[str], timeout_s: float = 60.0) -> RingTopology:
        """After a failed step: waits until the alive set differs from ``peers`` (the lost peer's heartbeat
        has aged past ``dead_after_s``), then forms the new ring."""
        deadline = time.time() + timeout_s
        while True:
            alive = self.alive_peers()
            if alive != sorted(peers) and self.peer_id in alive:
                ring = self.form_ring()
                if ring is not None:
                    return ring
            if time.time() > deadline:
                raise TimeoutError(f"ring did not re-form within {timeout_s:.0f} s (alive: {alive})")
            time.sleep(min(0.1, self.heartbeat_s))


def store_client(prefix: str = "bitresearch/elastic", timeout_s: float = 60.0):
    """A fresh client connection to the job's TCPStore (``MASTER_ADDR:MASTER_PORT``) under ``prefix``."""
    import os
    host = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ["MASTER_PORT"])
    raw = dist.TCPStore(host, port, is_master=False, timeout=datetime.timedelta(seconds=timeout_s))
    return dist.PrefixStore(prefix, raw)


class ElasticGroup:
    """A gloo group over one ring version's members (rank = ring position)."""

    def __init__(self, store, ring: RingTopology, room: str = "default", timeout_s: float = 30.0,
                 host: str = "127.0.0.1"):
        import os
        opts = dist.ProcessGroupGloo._Options()
        opts._timeout = datetime.timedelta(seconds=timeout_s)
        iface = os.environ.get("GLOO_SOCKET_IFNAME", "").split(",")[0]
        # loopback by default (one node); GLOO_SOCKET_IFNAME, gloo's own switch, names the interface otherwise
        opts._devices = [dist.ProcessGroupGloo.create_device(interface=iface) if iface
                         else dist.ProcessGroupGloo.create_device(hostname=host)]
        self.pg = dist.ProcessGroupGloo(dist.PrefixStore(f"{room}/pg/v{ring.version}", store), ring.position,
                                        ring.total, opts)
        self.ring = ring
        self.rank, self.size, self.version = ring.position, ring.total, ring.version
        self.timeout_s = timeout_s

    def isend(self, t: torch.Tensor, dst: int):
        return self.pg.send([t], dst, 0)

    def irecv(self, t: torch.Tensor, src: int):
        return self.pg.recv([t], src, 0)

    def all_reduce(self, t: torch.Tensor, op=dist.ReduceOp.SUM) -> bool:
        """In place on a CPU tensor; False if a member is gone (error or timeout)."""
        o = dist.AllreduceOptions()
        o.reduceOp = op
        return self._wait(self.pg.allreduce([t], o))

    def broadcast(self, t: torch.Tensor, root: int = 0) -> bool:
        o = dist.BroadcastOptions()
        o.rootRank = root
        o.rootTensor = 0
        return self._wait(self.pg.broadcast([t], o))

    def _wait(self, work) -> bool:
        try:
            return bool(work.wait(timeout=datetime.timedelta(seconds=self.timeout_s)))
        except Exception:
            return False

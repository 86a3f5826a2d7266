"""Rendezvous, ring formation, heartbeats and dynamic timeouts over a ``torch.distributed`` store.

This replaces the reference's WebSocket signalling server and WebRTC keep-alive:

* peers register in a room; the ring is the alive compute peers sorted by id, each with a left and
  a right neighbour, and a version counter bumped on every re-formation (server/signaling.ts:75-119);
* each peer refreshes a heartbeat key every ``heartbeat_s`` seconds (the reference pings every 2 s,
  webrtc-mesh.ts:173-196) and keeps an EMA (beta 0.9) of its store round-trip time
  (webrtc-mesh.ts:514-528);
* ``dynamic_timeout_s = max(10, 3 * max_rtt + 5)`` seconds (webrtc-mesh.ts:99-109);
* a peer whose heartbeat is older than ``dead_after_s`` is dropped at the next ``form_ring``, the
  equivalent of the server's ``peer-left`` + re-formation (server/signaling.ts:264-295).

Within one NVSwitch node the data path does not depend on the ring (the in-kernel collectives are
direct), but the trainer uses membership to detect a lost rank between steps and to skip or stop,
since a NCCL/P2P collective cannot continue with a missing rank.
"""
from __future__ import annotations

import threading
import time
from dataclasses import dataclass


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
                 dead_after_s: float = 10.0, peer_type: str = "compute"):
        self.store = store
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

    def beat(self) -> None:
        t0 = time.time()
        self.store.set(self._k("hb", self.peer_id), repr(t0))
        self.store.get(self._k("hb", self.peer_id))
        rtt = time.time() - t0
        self.smoothed_rtt_s = rtt if self.smoothed_rtt_s == 0 else 0.9 * self.smoothed_rtt_s + 0.1 * rtt

    def leave(self) -> None:
        self.stop()
        self.store.set(self._k("hb", self.peer_id), repr(0.0))

    def start(self) -> None:
        def run():
            while not self._stop.wait(self.heartbeat_s):
                try:
                    self.beat()
                except Exception:
                    return
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
        return sorted(pid for pid, ptype in self.registered_peers()
                      if ptype == "compute" and now - self.last_seen(pid) <= self.dead_after_s)

    def form_ring(self) -> RingTopology | None:
        peers = self.alive_peers()
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

import datetime
import time

from torch.distributed import TCPStore

from dist_utils import free_port
from bitresearch_b200.parallel.membership import Membership


def test_ring_formation_and_dead_peer_dropped():
    port = free_port()
    master = TCPStore("127.0.0.1", port, 3, True, timeout=datetime.timedelta(seconds=10), wait_for_workers=False)
    peers = [Membership(master if i == 0 else TCPStore("127.0.0.1", port, 3, False,
                                                        timeout=datetime.timedelta(seconds=10)),
                        f"peer-{c}", dead_after_s=1.0) for i, c in enumerate("bca")]
    for p in peers:
        p.register()
    rings = {p.peer_id: p.form_ring() for p in peers}
    assert rings["peer-a"].position == 0 and rings["peer-a"].right == "peer-b" and rings["peer-a"].left == "peer-c"
    assert len({r.version for r in rings.values()}) == 1
    v0 = rings["peer-a"].version
    time.sleep(1.3)
    peers[0].beat()  # peer-b alive
    peers[2].beat()  # peer-a alive, peer-c silent
    r = peers[2].form_ring()
    assert r.peers == ["peer-a", "peer-b"] and r.version > v0
    assert peers[1].form_ring() is None  # the silent peer is no longer a member
    assert 10.0 <= peers[0].dynamic_timeout_s < 11.0


def test_ring_timeout_follows_config_or_membership_rtt():
    from types import SimpleNamespace

    from bitresearch_b200.train import Trainer
    tr = Trainer.__new__(Trainer)
    tr.cfg = SimpleNamespace(comm_timeout_s=4.0)
    tr.membership = SimpleNamespace(dynamic_timeout_s=17.0)
    assert tr._ring_timeout() == 4.0
    tr.cfg.comm_timeout_s = 0
    assert tr._ring_timeout() == 17.0
    tr.membership = None
    assert tr._ring_timeout() == 10.0

"""The extension proxy: launch counting per entry point (kernels per call) and argument forwarding."""
from bitresearch_b200.ops import _ext


def test_counting_proxy_counts_launches_and_forwards_keywords():
    class Mod:
        @staticmethod
        def attn_bwd_tc(a, b=2):
            return a + b

        @staticmethod
        def rms_fwd(x):
            return -x

    _ext.reset_launch_counts()
    p = _ext._Counting(Mod())
    assert p.attn_bwd_tc(1) == 3 and p.attn_bwd_tc(1, b=5) == 6 and p.rms_fwd(4) == -4
    assert _ext.launch_counts() == {"attn_bwd_tc": 4, "rms_fwd": 1}  # the tcgen05 backward is two kernels
    _ext.reset_launch_counts()
    assert _ext.launch_counts() == {}

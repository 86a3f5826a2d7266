"""Loads the compiled sm_100a extension (``bitresearch_b200._C``).

On a machine with a CUDA device the extension is required: importing a kernel wrapper without it
raises, so a GPU run can never fall back silently to a PyTorch path. Build it in-tree with
``python setup.py build_ext --inplace`` (``__graft_entry__.build()`` does this).

``ext()`` returns a thin proxy that counts kernel launches per entry point (``launch_counts``), which
the benchmark reports as the number of this library's kernels launched in a timed region.
"""
from __future__ import annotations

import torch

_EXT = None
_ERR: Exception | None = None
# kernels launched by one call of a multi-kernel entry point
_KERNELS_PER_CALL = {"attn_bwd": 3, "attn_bwd_tc": 2, "muon_prepare": 2, "muon_finish": 2, "read_status": 0,
                     "reset_status": 0, "muon_prepare_scratch": 0, "muon_finish_scratch": 0, "gemm_set_pair": 0,
                     "gemm_pair": 0, "status_snapshot": 0}
_COUNTS: dict[str, int] = {}


def _load():
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            from .. import _C  # type: ignore
            _EXT = _C
        except Exception as e:  # pragma: no cover - depends on the build
            _ERR = e
    return _EXT


def available() -> bool:
    return _load() is not None


class _Counting:
    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            raw = getattr(self._mod, name)
            k = _KERNELS_PER_CALL.get(name, 1)

            def fn(*a, _raw=raw, _k=k, _n=name, **kw):
                _COUNTS[_n] = _COUNTS.get(_n, 0) + _k
                return _raw(*a, **kw)
            self._cache[name] = fn
        return fn


_PROXY = None


def ext():
    global _PROXY
    m = _load()
    if m is None:
        raise RuntimeError(f"bitresearch_b200._C is not built or failed to load ({_ERR!r}); "
                           "run `python setup.py build_ext --inplace`")
    if _PROXY is None:
        _PROXY = _Counting(m)
    return _PROXY


def reset_launch_counts() -> None:
    _COUNTS.clear()


def launch_counts() -> dict[str, int]:
    return dict(_COUNTS)


def check_status(device: int | None = None) -> int:
    """Reads (and clears) the device status word that kernels set when a bounded wait gave up."""
    m = ext()
    d = torch.cuda.current_device() if device is None else device
    s = int(m.read_status(d))
    if s:
        m.reset_status(d)
    return s

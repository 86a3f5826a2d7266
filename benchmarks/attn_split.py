"""Where the tcgen05 attention kernels spend their time: MMA/TMA pipeline versus softmax warps.

  python benchmarks/attn_split.py --build        # CPU is enough: compiles the three variants for sm_100a
  python benchmarks/attn_split.py [--tokens 131072] [--windows 1024,2048]   # times the built variants

Builds ``csrc/kernels/attention_tc.cu`` three times with ``ATTN_SPLIT_MODE``:

* 0: the kernels as shipped;
* 1: softmax arithmetic removed (the softmax warps keep their TMEM loads and barrier protocol, so
  this is the MMA/TMA pipeline plus synchronisation);
* 2: MMA and softmax decoupled (the MMA lane does not wait for P, the softmax warps do not wait for
  S), so the kernel takes as long as the slower of the two sides run on their own.

Modes 1 and 2 compute wrong values on purpose and exist only for this timing. Times are CUDA-event
medians on the launching stream after warm-up. The variants are built in-tree under
``benchmarks/_attn_split/`` so they travel with the repository snapshot.
"""
from __future__ import annotations

import argparse
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KDIR = os.path.join(ROOT, "csrc", "kernels")
OUT = os.path.join(ROOT, "benchmarks", "_attn_split")
MODES = {0: "as shipped", 1: "softmax arithmetic removed", 2: "MMA and softmax decoupled"}

WRAP = """
#include <torch/extension.h>
namespace br {
void attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t T, int64_t H,
                 int64_t KV, int64_t hd, int64_t window);
void attn_bwd_tc(const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout, const torch::Tensor& lse,
                 torch::Tensor& dqkv, torch::Tensor& delta, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t hd,
                 int64_t window, int64_t which);
}
PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fwd", [](const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t T, int64_t H,
                  int64_t KV, int64_t window) { br::attn_fwd_tc(qkv, o, lse, B, T, H, KV, 128, window); });
  m.def("bwd", [](const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout, const torch::Tensor& lse,
                  torch::Tensor& dqkv, torch::Tensor& delta, int64_t B, int64_t T, int64_t H, int64_t KV, int64_t window,
                  int64_t which) { br::attn_bwd_tc(qkv, o, dout, lse, dqkv, delta, B, T, H, KV, 128, window, which); });
}
"""


def load(mode: int):
    from torch.utils.cpp_extension import load as load_ext
    d = os.path.join(OUT, f"mode{mode}")
    os.makedirs(d, exist_ok=True)
    wrap = os.path.join(d, "bind.cpp")
    if not os.path.exists(wrap) or open(wrap).read() != WRAP:
        with open(wrap, "w") as fh:
            fh.write(WRAP)
    srcs = [os.path.join(KDIR, f) for f in ("attention_tc.cu", "attention.cu", "status.cu")] + [wrap]
    return load_ext(name=f"attn_split{mode}", sources=srcs,
                    extra_cuda_cflags=["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math",
                                       "-std=c++17", "-lineinfo", f"-DATTN_SPLIT_MODE={mode}"],
                    extra_cflags=["-O3"], extra_ldflags=["-lcuda"], build_directory=d, verbose=False)


def load_built(mode: int):
    """Imports a variant built by ``--build`` (no compiler run: the build tree may come from another machine)."""
    import glob
    import importlib.util
    hits = glob.glob(os.path.join(OUT, f"mode{mode}", f"attn_split{mode}*.so"))
    if not hits:
        raise SystemExit(f"variant {mode} is not built: run `python benchmarks/attn_split.py --build` first")
    spec = importlib.util.spec_from_file_location(f"attn_split{mode}", hits[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def timeit(fn, reps=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--build", action="store_true", help="only compile the variants")
    ap.add_argument("--tokens", type=int, default=131072)
    ap.add_argument("--windows", default="1024,2048")
    args = ap.parse_args()
    if args.build:
        for m in MODES:
            load(m)
        print("built", sorted(MODES))
        return
    mods = {m: load_built(m) for m in MODES}
    T, H, KV, hd = 2048, 4, 4, 128
    B = args.tokens // T
    torch.manual_seed(0)
    qkv = (torch.randn(B * T, (H + 2 * KV) * hd, device="cuda") * 0.5).bfloat16()
    o = torch.empty(B * T, H * hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, H, T, device="cuda")
    dout = torch.randn(B * T, H * hd, device="cuda").bfloat16()
    dqkv = torch.empty_like(qkv)
    delta = torch.zeros(B, H, T, device="cuda")
    for w in (int(x) for x in args.windows.split(",")):
        for m, x in mods.items():
            x.fwd(qkv, o, lse, B, T, H, KV, w)  # lse for the backward
            tf = timeit(lambda: x.fwd(qkv, o, lse, B, T, H, KV, w))
            tq = timeit(lambda: x.bwd(qkv, o, dout, lse, dqkv, delta, B, T, H, KV, w, 1))
            tk = timeit(lambda: x.bwd(qkv, o, dout, lse, dqkv, delta, B, T, H, KV, w, 2))
            print(f"window={w:5d} mode={m} ({MODES[m]:28s}) fwd={tf:.3f} ms  dq={tq:.3f} ms  dkdv={tk:.3f} ms",
                  flush=True)


if __name__ == "__main__":
    sys.exit(main())

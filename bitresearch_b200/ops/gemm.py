"""tcgen05 GEMM wrapper: ``C = epilogue(A @ B)`` for strided bf16 views.

Operand majors are read from the strides, so transposed views need no copies:
``a`` is logical [M, K] (row-major -> K-major, ``a.T`` of a contiguous tensor -> MN-major) and ``b`` is
logical [K, N] (row-major -> MN-major B, ``w.T`` of a contiguous [N, K] weight -> K-major B).
Batched operands are 3-D with a leading batch dimension.

Epilogues (fused into the TMEM read-out):
  BF16       C = alpha*AB + beta*aux           (bf16 out)
  F32        C = alpha*AB + beta*aux           (fp32 out; aux may be C itself: residual add)
  RELU2      C = relu(alpha*AB)^2              (bf16)
  RELU2_BWD  C = alpha*AB * 2*sqrt(aux)        (bf16; aux = relu(u)^2 saved by the forward)
  ATOMIC     C += alpha*AB                     (fp32, split-K over the reduction dimension)
  SOFTCAP    C = beta*tanh(alpha*AB)           (bf16; alpha = 1/cap, beta = cap)
"""
from __future__ import annotations

import torch

from ._ext import ext

BF16, F32, RELU2, RELU2_BWD, ATOMIC, SOFTCAP = range(6)
_F32_OUT = (F32, ATOMIC)


def _layout_a(a: torch.Tensor):
    """(mn_major, ld, batch_stride) of a logical [.., M, K] operand."""
    if a.stride(-1) == 1:
        return False, a.stride(-2)
    if a.stride(-2) == 1:
        return True, a.stride(-1)
    raise ValueError("gemm: A needs a unit stride in one of its last two dims")


def _layout_b(b: torch.Tensor):
    """(mn_major, ld) of a logical [.., K, N] operand (B of the kernel is its transpose)."""
    if b.stride(-1) == 1:
        return True, b.stride(-2)
    if b.stride(-2) == 1:
        return False, b.stride(-1)
    raise ValueError("gemm: B needs a unit stride in one of its last two dims")


def matmul(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, epi: int = BF16,
           aux: torch.Tensor | None = None, alpha: float = 1.0, beta: float = 0.0, k_splits: int = 1,
           block_n: int = 0) -> torch.Tensor:
    batched = a.dim() == 3
    M, K = a.shape[-2:]
    K2, N = b.shape[-2:]
    assert K == K2, f"gemm: inner dims differ {a.shape} x {b.shape}"
    batch = a.shape[0] if batched else 1
    if out is None:
        dt = torch.float32 if epi in _F32_OUT else torch.bfloat16
        shape = (batch, M, N) if batched else (M, N)
        out = (torch.zeros if epi == ATOMIC else torch.empty)(shape, dtype=dt, device=a.device)
    a_mn, lda = _layout_a(a)
    b_mn, ldb = _layout_b(b)
    assert out.stride(-1) == 1, "gemm: output rows must be contiguous"
    bsa = a.stride(0) if batched else 0
    bsb = b.stride(0) if batched else 0
    bsc = out.stride(0) if batched else 0
    ld_aux = bs_aux = 0
    if aux is not None:
        assert aux.stride(-1) == 1
        ld_aux = aux.stride(-2)
        bs_aux = aux.stride(0) if aux.dim() == 3 else 0
    ext().gemm(a, a_mn, lda, bsa, b, b_mn, ldb, bsb, out, out.stride(-2), bsc, M, N, K, batch, epi, aux, ld_aux,
               bs_aux, alpha, beta, k_splits, block_n)
    return out


def qkv_rope(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
             rq: torch.Tensor, rk: torch.Tensor, T: int, H: int, KV: int, idx: torch.Tensor | None = None,
             ve: torch.Tensor | None = None, cur: torch.Tensor | None = None, wg: torch.Tensor | None = None,
             gate: torch.Tensor | None = None) -> torch.Tensor:
    """``out = x @ w`` for the fused QKV projection with RoPE + QK-norm on the q/k heads (rstd into
    ``rq``/``rk``) and, when ``ve`` is given, the value-embedding add on the v heads (gate into
    ``gate``), all in the GEMM epilogue. Needs head_dim 128 and even H and KV."""
    ext().gemm_qkv_rope(x, w, out, cos, sin, rq, rk, T, H, KV, idx, ve, cur, wg, gate)
    return out

"""Hand-scheduled forward/backward of the GPT on sm_100a kernels.

The engine owns all activation buffers (allocated once for a fixed micro-batch), runs the forward
with the fused kernels, and runs the backward explicitly (no autograd graph): every weight
gradient is accumulated by a split-K tcgen05 GEMM or a scatter kernel directly into the trainer's
flat fp32 gradient buffer (reference order), so data-parallel communication can start on a finished
bucket without any copy.

Per layer (forward):
  ladder_rms_fwd      cur = lr*x + l0*x0, xn = bf16(rms(cur))
  GEMM                qkv = xn @ [Wq|Wk|Wv]                        (bf16)
  rope_fwd            q,k <- rms(rope(.)), v += ve[idx]*2sigmoid(cur[:, :32] @ Wg)
  attn_fwd            o = softmax(q k^T / sqrt(hd) + causal/window mask) v, lse
  GEMM (F32 epi)      mid = cur + o @ Wproj                         (fp32 residual add in the epilogue)
  rms_fwd             xn2 = bf16(rms(mid))
  GEMM (RELU2 epi)    h = relu(xn2 @ Wfc)^2
  GEMM (F32 epi)      x_next = mid + h @ Wmlp_proj
Head: rms_fwd -> lm_head GEMM whose epilogue computes the softcapped cross-entropy statistics and writes
G = exp(z - cap) (1 - (z/cap)^2) instead of the logits -> ce_finalize (loss, per-token nats, per-row scale,
the target column's gradient written into G, the scaled activations for dW).
Backward mirrors it: dW via ``X^T @ dY`` split-K GEMMs (fp32 vector reductions), dX via ``dY @ W^T``
GEMMs (the ReLU^2 derivative fused into the mlp_proj dX epilogue), rms/ladder backward kernels,
attention backward, RoPE/QK-norm/VE backward and the embedding scatter.

GEMM B-operands are bf16 shadows of the fp32 master weights; the optimizer kernels rewrite them after
each update. q/k/v shadows are column slices of one [D, Dq + 2 Dkv] matrix so the QKV projection is a
single GEMM.
"""
from __future__ import annotations

import torch

from ..config import effective_window, has_value_embedding
from ..ops import gemm
from ..ops._ext import check_status, ext
from ..utils.timing import traced


class FusedGPTEngine:
    @staticmethod
    def unsupported(cfg) -> str | None:
        """Why the sm_100a engine cannot run this model config, or None. Heads are 128 wide (the tcgen05
        attention and the QKV epilogue with RoPE + QK-norm fused) or 64 wide (the reference's default
        model: register-tiled attention and the separate RoPE/QK-norm/VE kernels); other widths train
        through the eager path (``impl=torch``) on the same GPU."""
        if cfg.head_dim not in (64, 128):
            return f"head_dim {cfg.head_dim} (n_embd {cfg.n_embd} / n_head {cfg.n_head}); the kernels need 64 or 128"
        return None

    def __init__(self, model, grad_views: dict, batch: int, seq: int, flat_grad: torch.Tensor | None = None):
        self.model = model
        self.cfg = cfg = model.cfg
        why = self.unsupported(cfg)
        if why is not None:
            raise ValueError(f"impl=cuda cannot run this model: {why}; use impl=torch")
        self.timer = None  # a PhaseTimer: forward / backward as CUDA-event phases with NVTX ranges
        self.grads = grad_views
        self.flat_grad = flat_grad
        self.dev = next(model.parameters()).device
        self.B, self.T = batch, seq
        self.L, self.D, self.H, self.KV, self.hd = cfg.n_layer, cfg.n_embd, cfg.n_head, cfg.n_kv_head, cfg.head_dim
        self.Dq, self.Dkv, self.F, self.V = cfg.n_head * cfg.head_dim, cfg.kv_dim, 4 * cfg.n_embd, cfg.vocab_size
        self.P = model.named()
        self.E = ext()
        self.windows = [effective_window(w, seq) for w, _ in model.window_sizes]
        self.ve_layers = [i for i in range(self.L) if has_value_embedding(i, self.L)]
        self.cos = model.rope_cos[:seq].contiguous()
        self.sin = model.rope_sin[:seq].contiguous()
        self._alloc_shadows()
        self.refresh_shadows()
        self.bufs: dict[int, dict] = {}
        self.optimizer = None
        # bucket_hook(b, grad_scale) is called on the compute stream when bucket b's gradients are
        # final (b = 0: lm_head, 1..L: layers L-1..0, L+1: embeddings and scalars)
        self.bucket_hook = None
        # tcgen05 attention needs 128-wide heads and whole 128-row tiles; otherwise the register-tiled kernels
        self.tc_attention = seq % 128 == 0 and self.hd == 128
        # the QKV GEMM applies RoPE/QK-norm/VE in its epilogue when each 256-column tile holds two heads
        self.fused_rope = self.hd == 128 and self.H % 2 == 0 and self.KV % 2 == 0
        self._hook_on = False
        self._grad_scale = 1.0
        # param_ready(g) is called on the compute stream before the first kernel that reads parameter
        # group g (0: embeddings and scalars, 1..L: layer g-1 with its value embedding, L+1: lm_head), so
        # a data-parallel parameter exchange still in flight can overlap the forward
        self.param_ready = None

    # ------------------------------------------------------------------ weights
    def _alloc_shadows(self):
        bf = dict(dtype=torch.bfloat16, device=self.dev)
        D, Dq, Dkv = self.D, self.Dq, self.Dkv
        self.wqkv, self.shadows = [], {}
        for i in range(self.L):
            w = torch.empty(D, Dq + 2 * Dkv, **bf)
            self.wqkv.append(w)
            self.shadows[f"layer{i}_q"] = w[:, :Dq]
            self.shadows[f"layer{i}_k"] = w[:, Dq:Dq + Dkv]
            self.shadows[f"layer{i}_v"] = w[:, Dq + Dkv:]
            for n in ("proj", "fc", "mlp_proj"):
                self.shadows[f"layer{i}_{n}"] = torch.empty_like(self.P[f"layer{i}_{n}"], **bf)
        self.shadows["lmHead"] = torch.empty_like(self.P["lmHead"], **bf)

    @torch.no_grad()
    def refresh_shadows(self):
        for n, s in self.shadows.items():
            s.copy_(self.P[n])

    def sync_params_to_model(self):
        """Parameters are the model's own tensors; nothing to copy."""

    def attach_optimizer(self, opt):
        self.optimizer = opt

    # ------------------------------------------------------------------ buffers
    def _buffers(self, B: int):
        if B in self.bufs:
            return self.bufs[B]
        T, D, L, H, KV = self.T, self.D, self.L, self.H, self.KV
        M = B * T
        W = self.Dq + 2 * self.Dkv
        f32 = dict(dtype=torch.float32, device=self.dev)
        bf = dict(dtype=torch.bfloat16, device=self.dev)
        b = {
            "x0": torch.empty(M, D, **f32), "rstd0": torch.empty(M, **f32),
            "xs": [torch.empty(M, D, **f32) for _ in range(L)],  # xs[i] = output of layer i
            "cur": [torch.empty(M, D, **f32) for _ in range(L)],
            "mid": [torch.empty(M, D, **f32) for _ in range(L)],
            "rstd1": [torch.empty(M, **f32) for _ in range(L)],
            "rstd2": [torch.empty(M, **f32) for _ in range(L)],
            "xn": [torch.empty(M, D, **bf) for _ in range(L)],
            "xn2": [torch.empty(M, D, **bf) for _ in range(L)],
            "qkv": [torch.empty(M, W, **bf) for _ in range(L)],
            "rq": [torch.empty(M, H, **f32) for _ in range(L)],
            "rk": [torch.empty(M, KV, **f32) for _ in range(L)],
            "gate": {i: torch.empty(M, KV, **f32) for i in self.ve_layers},
            "o": [torch.empty(M, D, **bf) for _ in range(L)],
            "lse": [torch.empty(B, H, T, **f32) for _ in range(L)],
            "h": [torch.empty(M, self.F, **bf) for _ in range(L)],
            "rstdf": torch.empty(M, **f32), "xf": torch.empty(M, D, **bf),
            # fused head: G (dlogits up to a per-row scale and the target column), CE statistics
            "G": torch.empty(M, self.V, **bf), "ce_part": torch.empty(2 * ((self.V + 255) // 256), M, **f32),
            "zt": torch.empty(M, **f32), "rowscale": torch.empty(M, **f32),
            "xs_head": torch.empty(M, D, **bf), "nats": torch.empty(M, **f32),
            "loss": torch.zeros(1, **f32),
            # backward scratch
            "dx": torch.empty(M, D, **f32), "dx_b": torch.empty(M, D, **bf),
            "dmid": torch.empty(M, D, **f32), "dmid_b": torch.empty(M, D, **bf),
            "dh": torch.empty(M, self.F, **bf), "dxn2": torch.empty(M, D, **bf),
            "do": torch.empty(M, D, **bf), "dqkv": torch.empty(M, W, **bf), "dxn": torch.empty(M, D, **bf),
            "delta": torch.empty(B, H, T, **f32), "dz": torch.empty(M, KV, **f32),
            "dgate_in": torch.empty(M, 32, **f32), "dx0": torch.empty(M, D, **f32),
        }
        self.bufs[B] = b
        return b

    # ------------------------------------------------------------------ forward
    def _forward(self, idx: torch.Tensor, b: dict, B: int):
        E, P = self.E, self.P
        T, D, H, KV, hd = self.T, self.D, self.H, self.KV, self.hd
        Dq, Dkv = self.Dq, self.Dkv
        idx = idx.reshape(-1)
        ready = self.param_ready or (lambda g: None)
        ready(0)
        E.embed_rms_fwd(idx, P["wte"], b["x0"], b["rstd0"])
        x = b["x0"]
        for i in range(self.L):
            ready(i + 1)
            cur, xn = b["cur"][i], b["xn"][i]
            E.ladder_rms_fwd(x, b["x0"], P["residLambdas"], P["x0Lambdas"], i, cur, xn, b["rstd1"][i])
            qkv = b["qkv"][i]
            ve_args = ((idx, P[f"ve_{i}"], cur, P[f"layer{i}_ve_gate"], b["gate"][i]) if i in b["gate"]
                       else (idx, None, None, None, None))
            if self.fused_rope:  # RoPE + QK-norm (+ VE) in the QKV GEMM's epilogue
                gemm.qkv_rope(xn, self.wqkv[i], qkv, self.cos, self.sin, b["rq"][i], b["rk"][i], T, H, KV, *ve_args)
            else:
                gemm.matmul(xn, self.wqkv[i], out=qkv)
                E.rope_fwd(qkv, T, H, KV, hd, self.cos, self.sin, b["rq"][i], b["rk"][i], *ve_args)
            o = b["o"][i]
            if self.tc_attention:
                E.attn_fwd_tc(qkv, o, b["lse"][i], B, T, H, KV, hd, self.windows[i])
            else:
                E.attn_fwd(qkv[:, :Dq], qkv[:, Dq:Dq + Dkv], qkv[:, Dq + Dkv:], o, b["lse"][i], B, T, H, KV, hd,
                           self.windows[i])
            mid = b["mid"][i]
            gemm.matmul(o, self.shadows[f"layer{i}_proj"], out=mid, epi=gemm.F32, aux=cur, beta=1.0)
            E.rms_fwd(mid, b["xn2"][i], b["rstd2"][i])
            gemm.matmul(b["xn2"][i], self.shadows[f"layer{i}_fc"], out=b["h"][i], epi=gemm.RELU2)
            gemm.matmul(b["h"][i], self.shadows[f"layer{i}_mlp_proj"], out=b["xs"][i], epi=gemm.F32, aux=mid,
                        beta=1.0)
            x = b["xs"][i]
        E.rms_fwd(x, b["xf"], b["rstdf"])
        ready(self.L + 1)

    def _head(self, tg: torch.Tensor, b: dict, scale: float, grad: bool):
        """lm_head + softcap 15 + cross-entropy (gpt.ts:296-313) without writing the logits: the GEMM epilogue
        keeps per-row exp-sums and the target logit, ``ce_finalize`` adds ``scale * sum(nats)`` into the loss.
        With ``grad`` it also prepares the backward: G (with the target column's gradient patched in), the
        per-row scale and the scaled activations for the weight-gradient GEMM."""
        E = self.E
        E.gemm_softcap_ce(b["xf"], self.shadows["lmHead"], b["G"], tg, b["ce_part"], b["zt"], 15.0, grad)
        if grad:
            E.ce_finalize(b["ce_part"], b["zt"], tg, self.V, 15.0, scale, nats=b["nats"], loss_sum=b["loss"],
                          rowscale=b["rowscale"], x=b["xf"], xs=b["xs_head"], g=b["G"])
        else:
            E.ce_finalize(b["ce_part"], b["zt"], tg, self.V, 15.0, scale, nats=b["nats"])

    # ------------------------------------------------------------------ backward
    def _backward(self, idx: torch.Tensor, tg: torch.Tensor, b: dict, B: int):
        E, P, G = self.E, self.P, self.grads
        T, D, H, KV, hd = self.T, self.D, self.H, self.KV, self.hd
        Dq, Dkv = self.Dq, self.Dkv
        idx = idx.reshape(-1)
        A = gemm.ATOMIC
        # head: dlogits = rowscale * G (ce_finalize wrote the target column into G), so
        # dlmHead += G^T (rowscale xf) and dxf = rowscale (G lmHead), the scale folded into rms_bwd
        gemm.matmul(b["G"].t(), b["xs_head"], out=G["lmHead"], epi=A, k_splits=0)
        gemm.matmul(b["G"], self.shadows["lmHead"], out=b["dmid"], epi=gemm.F32)
        self._ready(0)
        E.rms_bwd(b["xs"][-1], b["rstdf"], b["dmid"], None, b["dx"], b["dx_b"], b["rowscale"])
        b["dx0"].zero_()
        for i in reversed(range(self.L)):
            # MLP
            gemm.matmul(b["h"][i].t(), b["dx_b"], out=G[f"layer{i}_mlp_proj"], epi=A, k_splits=0)
            gemm.matmul(b["dx_b"], self.shadows[f"layer{i}_mlp_proj"].t(), out=b["dh"], epi=gemm.RELU2_BWD,
                        aux=b["h"][i])
            gemm.matmul(b["xn2"][i].t(), b["dh"], out=G[f"layer{i}_fc"], epi=A, k_splits=0)
            gemm.matmul(b["dh"], self.shadows[f"layer{i}_fc"].t(), out=b["dxn2"])
            E.rms_bwd(b["mid"][i], b["rstd2"][i], b["dxn2"], b["dx"], b["dmid"], b["dmid_b"])
            # attention
            gemm.matmul(b["o"][i].t(), b["dmid_b"], out=G[f"layer{i}_proj"], epi=A, k_splits=0)
            gemm.matmul(b["dmid_b"], self.shadows[f"layer{i}_proj"].t(), out=b["do"])
            qkv, dqkv = b["qkv"][i], b["dqkv"]
            ve = i in b["gate"]
            if self.tc_attention:
                E.attn_bwd_tc(qkv, b["o"][i], b["do"], b["lse"][i], dqkv, b["delta"], B, T, H, KV, hd, self.windows[i])
            else:
                E.attn_bwd(qkv[:, :Dq], qkv[:, Dq:Dq + Dkv], qkv[:, Dq + Dkv:], b["o"][i], b["do"], b["lse"][i],
                           dqkv[:, :Dq], dqkv[:, Dq:Dq + Dkv], dqkv[:, Dq + Dkv:], b["delta"], b["delta"], B, T, H, KV,
                           hd, self.windows[i])
            # RoPE + QK-norm (+ VE) backward as its own pass: folding it into the attention epilogues put
            # its global loads on every CTA's tail and measured slower
            ve_b = (P[f"ve_{i}"], b["gate"][i], G[f"ve_{i}"], b["dz"]) if ve else (None, None, None, None)
            E.rope_bwd(dqkv, qkv, T, H, KV, hd, self.cos, self.sin, b["rq"][i], b["rk"][i], idx, *ve_b)
            if ve:
                E.ve_gate_bwd(b["cur"][i], b["dz"], P[f"layer{i}_ve_gate"], G[f"layer{i}_ve_gate"], b["dgate_in"])
            xn = b["xn"][i]
            gemm.matmul(xn.t(), dqkv[:, :Dq], out=G[f"layer{i}_q"], epi=A, k_splits=0)
            gemm.matmul(xn.t(), dqkv[:, Dq:Dq + Dkv], out=G[f"layer{i}_k"], epi=A, k_splits=0)
            gemm.matmul(xn.t(), dqkv[:, Dq + Dkv:], out=G[f"layer{i}_v"], epi=A, k_splits=0)
            gemm.matmul(dqkv, self.wqkv[i].t(), out=b["dxn"])
            x_in = b["xs"][i - 1] if i > 0 else b["x0"]
            # also writes the bf16 copy of dx that layer i-1's backward GEMMs read
            E.ladder_bwd(x_in, b["x0"], P["residLambdas"], P["x0Lambdas"], i, b["rstd1"][i], b["dxn"], b["dmid"],
                         b["dgate_in"] if ve else None, b["dx"], b["dx0"], G["residLambdas"], G["x0Lambdas"], i == 0,
                         b["dx_b"] if i > 0 else None)
            self._ready(self.L - i)
        E.embed_bwd(idx, P["wte"], b["rstd0"], b["dx0"], G["wte"])
        self._ready(self.L + 1)

    def _ready(self, bucket: int):
        if self._hook_on:
            self.bucket_hook(bucket, self._grad_scale)

    # ------------------------------------------------------------------ API
    def forward_backward(self, idx: torch.Tensor, targets: torch.Tensor, loss_scale: float = 1.0,
                         accumulate: bool = False, last_micro: bool = True, grad_scale: float = 1.0) -> torch.Tensor:
        """Accumulates gradients of ``loss_scale * mean CE`` into the flat buffer; returns the mean CE.

        On the last micro-batch of a step the bucket hook fires as each bucket's gradients become
        final (``grad_scale`` is the loss scale to divide out when packing them)."""
        B = idx.shape[0]
        self._hook_on = last_micro and self.bucket_hook is not None
        self._grad_scale = grad_scale
        assert idx.shape[1] == self.T
        b = self._buffers(B)
        tg = targets.reshape(-1).to(torch.int32).contiguous()
        with traced(self.timer, "forward"):
            self._forward(idx, b, B)
            # zeroed after the forward: it waited for every parameter group of the last exchange, and with
            # it for the last reduce-scatter kernels that read the previous step's gradients
            if not accumulate:
                if self.flat_grad is not None:
                    self.flat_grad.zero_()
                else:
                    for g in self.grads.values():
                        g.zero_()
            b["loss"].zero_()
            self._head(tg, b, loss_scale / (B * self.T), grad=True)
        with traced(self.timer, "backward"):  # includes the bucket hooks that launch the gradient reduce
            self._backward(idx, tg, b, B)
        return b["loss"][0] / loss_scale

    @torch.no_grad()
    def per_token_nats(self, idx: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        B = idx.shape[0]
        b = self._buffers(B)
        self._forward(idx, b, B)
        self._head(targets.reshape(-1).to(torch.int32).contiguous(), b, 1.0, grad=False)
        return b["nats"].view(B, self.T).clone()

    def status(self) -> int:
        return check_status()

"""Configuration: model hyper-parameters, optimiser/schedule/data/comm settings and presets.

Model semantics follow the reference trainer's model config (src/model/config.ts:3-86):

* ``window_pattern`` maps each layer to a window: ``L`` = ``sequence_len``, ``S`` =
  ``sequence_len // 2``; the last layer is always ``L`` (config.ts:29-51).
* value embeddings live on layers with ``i % 2 == (n_layer - 1) % 2`` (config.ts:24-26).
* ``estimate_params`` matches config.ts:54-86; ``estimate_flops_per_token`` matches the
  reference's MFU numerator (src/model/gpt.ts:404-428).

Trainer defaults follow src/distributed/trainer.ts:69-99 and src/train/muon.ts:435-443.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Any

VE_GATE_CHANNELS = 32


@dataclass
class GPTConfig:
    sequence_len: int = 2048
    vocab_size: int = 8192
    n_layer: int = 8
    n_head: int = 4
    n_kv_head: int = 4
    n_embd: int = 512
    window_pattern: str = "SSSL"

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def kv_dim(self) -> int:
        return self.n_kv_head * self.head_dim

    def validate(self) -> None:
        # same checks as src/model/gpt.ts:61-73
        if self.n_embd % self.n_head:
            raise ValueError(f"n_embd ({self.n_embd}) must be divisible by n_head ({self.n_head})")
        if self.n_kv_head <= 0 or self.n_head % self.n_kv_head:
            raise ValueError(f"n_kv_head ({self.n_kv_head}) must be a positive divisor of n_head ({self.n_head})")
        if self.head_dim % 2:
            raise ValueError(f"head dimension ({self.head_dim}) must be even for RoPE")
        if self.n_embd < VE_GATE_CHANNELS:
            raise ValueError(f"n_embd ({self.n_embd}) must be at least {VE_GATE_CHANNELS} for ve_gate")
        if not self.window_pattern:
            raise ValueError("window_pattern must not be empty")
        for ch in self.window_pattern.upper():
            if ch not in "LS":
                raise ValueError(f"unsupported window pattern character: {ch}")

    # camelCase form used by the reference checkpoints' ``config`` metadata (trainer.ts:1136)
    def to_reference_dict(self) -> dict[str, Any]:
        return {
            "sequenceLen": self.sequence_len,
            "vocabSize": self.vocab_size,
            "nLayer": self.n_layer,
            "nHead": self.n_head,
            "nKvHead": self.n_kv_head,
            "nEmbd": self.n_embd,
            "windowPattern": self.window_pattern,
        }

    @classmethod
    def from_reference_dict(cls, d: dict[str, Any]) -> "GPTConfig":
        if "sequenceLen" in d:
            return cls(
                sequence_len=int(d["sequenceLen"]),
                vocab_size=int(d["vocabSize"]),
                n_layer=int(d["nLayer"]),
                n_head=int(d["nHead"]),
                n_kv_head=int(d["nKvHead"]),
                n_embd=int(d["nEmbd"]),
                window_pattern=str(d["windowPattern"]),
            )
        return cls(**{k: v for k, v in d.items() if k in {f.name for f in dataclasses.fields(cls)}})


def has_value_embedding(layer_idx: int, n_layer: int) -> bool:
    """Value-embedding layers (config.ts:24-26)."""
    return layer_idx % 2 == (n_layer - 1) % 2


def compute_window_sizes(cfg: GPTConfig) -> list[tuple[int, int]]:
    """Per-layer ``(window, 0)`` pairs (config.ts:29-51)."""
    pattern = cfg.window_pattern.upper()
    if not pattern:
        raise ValueError("windowPattern must not be empty")
    long_w = cfg.sequence_len
    short_w = long_w // 2
    table = {"L": (long_w, 0), "S": (short_w, 0)}
    out = []
    for i in range(cfg.n_layer):
        ch = pattern[i % len(pattern)]
        if ch not in table:
            raise ValueError(f"unsupported window pattern character: {ch}")
        out.append(table[ch])
    if out:
        out[-1] = (long_w, 0)
    return out


def effective_window(window: int, seq_len: int) -> int:
    """Number of keys (self included) a query sees; ``seq_len`` means plain causal.

    The reference applies the band mask only when ``0 < window < T`` (gpt.ts:262).
    """
    if window <= 0 or window >= seq_len:
        return seq_len
    return window


def estimate_params(cfg: GPTConfig) -> int:
    """Parameter count (config.ts:54-86)."""
    d, v, kv = cfg.n_embd, cfg.vocab_size, cfg.kv_dim
    p = v * d * 2
    for i in range(cfg.n_layer):
        p += d * (cfg.n_head * cfg.head_dim) + 2 * d * kv + d * d + 8 * d * d
        if has_value_embedding(i, cfg.n_layer):
            p += v * kv + VE_GATE_CHANNELS * cfg.n_kv_head
    p += cfg.n_layer * 2
    return p


def estimate_flops_per_token(cfg: GPTConfig) -> int:
    """FLOPs/token used for MFU (gpt.ts:404-428): 6*matrix params + 12*H*hd*window per layer."""
    d, kv = cfg.n_embd, cfg.kv_dim
    matrix = cfg.n_layer * (d * cfg.n_head * cfg.head_dim + 2 * d * kv + d * d + 8 * d * d)
    attn = 0
    for w, _ in compute_window_sizes(cfg):
        eff = min(w, cfg.sequence_len) if w > 0 else cfg.sequence_len
        attn += 12 * cfg.n_head * cfg.head_dim * eff
    return 6 * matrix + attn


def estimate_flops_per_token_with_head(cfg: GPTConfig) -> int:
    """Reference FLOPs/token plus the lm_head's 6*V*D (the reference omits it)."""
    return estimate_flops_per_token(cfg) + 6 * cfg.vocab_size * cfg.n_embd


@dataclass
class SparsifyConfig:
    """Top-k + error feedback settings (src/distributed/gradient-sparsifier.ts:20-36)."""

    enabled: bool = False
    top_k_ratio: float = 0.10
    warmup_steps: int = 100
    sample_size: int = 10000
    momentum_factor: float = 0.9
    value_dtype: str = "fp16"  # wire dtype of the kept values
    # False: the reference's update (residual = the whole velocity, velocity never cleared), whose
    # unsent residuals grow by (1 + momentum) per step; True: Deep Gradient Compression's momentum
    # correction with factor masking (u = m u + g, v += u, send top-k of v, clear v and u where sent)
    momentum_masking: bool = False


@dataclass
class TrainConfig:
    model: GPTConfig = field(default_factory=GPTConfig)
    # batch: ``device_batch`` sequences per rank per micro-step; ``total_batch_tokens`` global per step
    device_batch: int = 128
    total_batch_tokens: int = 2 ** 19
    # MuonAdamW (muon.ts:435-443, trainer.ts:69-99)
    unembedding_lr: float = 0.004
    embedding_lr: float = 0.6
    matrix_lr: float = 0.04
    scalar_lr: float = 0.5
    weight_decay: float = 0.2
    adam_betas: tuple[float, float] = (0.8, 0.95)
    ns_steps: int = 5
    muon_beta2: float = 0.95
    ns_dtype: str = "bf16"  # "fp32" reproduces the reference's fp32 polar express exactly
    # schedules (trainer.ts:577-602)
    warmup_ratio: float = 0.0
    warmdown_ratio: float = 0.5
    final_lr_frac: float = 0.0
    # loop
    max_steps: int = 1 << 62
    time_budget: float = 300.0
    warmup_steps_excluded: int = 10  # trainer.ts:986,1005: first steps not counted in the budget
    seed: int = 0
    # eval
    eval_tokens: int = 40 * 524288
    val_fraction: float = 0.1
    # data: "zipf" (BOS-packed Zipf docs), "markov" (Zipf docs whose tokens follow hashed order-1 /
    # order-2 successor tables), "uniform" (uniform + BOS every 64), "tokens" (.bin shards, a manifest,
    # or a .json token list), "documents" (a .json list of token arrays, best-fit BOS packed)
    data: str = "zipf"
    data_path: str = ""
    token_bytes_path: str = ""
    zipf_s: float = 1.1
    doc_mean_len: int = 512
    markov_p1: float = 0.4  # P(next token is a successor of the previous token)
    markov_p2: float = 0.4  # P(next token is a successor of the previous two tokens)
    markov_branch: int = 4  # successors per context, picked with weights 2^-k
    token_bytes_max: int = 16
    bos_every: int = 64
    document_buffer_size: int = 1000
    documents_bos_prefixed: bool = False  # data=documents: the documents already start with BOS
    bos_token_id: int = -1  # data=documents: -1 = vocab_size - 1
    # compute
    impl: str = "cuda"  # "cuda" (sm_100a kernels) or "torch" (eager oracle path)
    # impl=torch on a GPU: run the eager model under torch.compile with flex attention (a fused
    # sliding-window kernel), the strongest stock-PyTorch form of the model, for baseline runs
    torch_compile: bool = False
    dtype: str = "bf16"
    # distributed communication
    comm: str = "p2p"  # "p2p" (in-kernel NVLink), "nccl", "ring" (reference ring algorithm over the PG)
    wire_dtype: str = "bf16"  # bf16 | fp16 | fp32
    bucket_mb: float = 32.0
    overlap: bool = True
    # p2p path with the fused engine: true runs the sharded optimizer per forward group on the comm
    # stream, interleaved with the parameter exchange; the default (false) runs one optimizer call on the
    # compute stream after the backward, then the exchange on the comm stream. Measured at 8 GPUs: 27.3
    # ms per step with the overlap against 26.1 without, since the optimizer's small GEMM launches only
    # get SMs between the forward's persistent kernels and stretched to 5.5 ms
    overlap_optimizer: bool = False
    sparsify: SparsifyConfig = field(default_factory=SparsifyConfig)
    comm_timeout_s: float = 10.0  # elastic ring: 0 = the membership's dynamic timeout max(10, 3 rtt + 5) s
    # ring path only: re-form the ring without a lost rank (store heartbeats + a new gloo group)
    elastic: bool = False
    heartbeat_s: float = 2.0  # the reference pings every 2 s (webrtc-mesh.ts:173-196)
    dead_after_s: float = 10.0  # a peer silent this long is dropped at the next re-formation
    reform_timeout_s: float = 60.0
    # elastic ring: pause while fewer peers are alive (trainer.ts minRingSize), stop after reform_timeout_s
    min_ring_size: int = 1
    # elastic ring: this process joins a running job's ring instead of forming the first one (it takes
    # part in the next re-formation and receives the state from a member)
    elastic_join: bool = False
    # elastic ring: every this many steps the members take in peers that joined the room (0 = never;
    # a ring paused below min_ring_size always takes them in)
    join_check_steps: int = 10
    # checkpoints / logging
    checkpoint_interval: int = 0
    checkpoint_dir: str = "checkpoints"
    results_tsv: str = "results.tsv"
    metrics_jsonl: str = ""
    status_port: int = -1  # >= 0: rank 0 serves GET /status and GET /metrics on this port (0 picks one)
    trace_phases: bool = False  # CUDA-event + NVTX phases (data, forward, backward, sync, optimizer) per step
    profile_steps: str = ""  # "a:b": torch.profiler over steps [a, b), Chrome trace into profile_dir
    profile_dir: str = "traces"
    log_every: int = 5

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), sort_keys=True)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "TrainConfig":
        d = dict(d)
        model = GPTConfig(**d.pop("model", {}))
        sp = SparsifyConfig(**d.pop("sparsify", {}))
        if "adam_betas" in d:
            d["adam_betas"] = tuple(d["adam_betas"])
        return cls(model=model, sparsify=sp, **d)


def _tiny_cpu() -> TrainConfig:
    # Tiny GPT on CPU, gloo world_size=2: depth 2, d128, 2x64 heads, vocab 512, seq 128, batch 4/rank, fp32
    return TrainConfig(
        model=GPTConfig(sequence_len=128, vocab_size=512, n_layer=2, n_head=2, n_kv_head=2, n_embd=128,
                        window_pattern="L"),
        device_batch=4, total_batch_tokens=4 * 128 * 2, data="uniform", bos_every=64, token_bytes_max=4,
        impl="torch", dtype="fp32", comm="ring", wire_dtype="fp32", ns_dtype="fp32", eval_tokens=4 * 128 * 4,
    )


def _d512() -> TrainConfig:
    # autoresearch default: depth 8, d512, 4x128 heads, vocab 8192, seq 2048, SSSL, 2^19 tokens/step
    return TrainConfig(model=GPTConfig(), device_batch=128, total_batch_tokens=2 ** 19)


def _d1280() -> TrainConfig:
    return TrainConfig(
        model=GPTConfig(sequence_len=2048, vocab_size=65536, n_layer=20, n_head=10, n_kv_head=10, n_embd=1280,
                        window_pattern="SSSL"),
        device_batch=32, total_batch_tokens=2 ** 19,
    )


def _d512_topk() -> TrainConfig:
    # error feedback without sender-side momentum: Muon and AdamW apply momentum to what arrives
    c = _d512()
    c.sparsify = SparsifyConfig(enabled=True, top_k_ratio=0.01, warmup_steps=0, value_dtype="fp16",
                                momentum_factor=0.0)
    return c


def _ref_default() -> TrainConfig:
    # the reference trainer's own DEFAULT_CONFIG (config.ts:14-22), batch 4 (trainer.ts:71). Its heads are
    # 64 wide and the sm_100a engine is built for 128-wide heads, so it trains on the eager path (bf16 on
    # the GPU); multi-GPU runs then all-reduce with NCCL.
    return TrainConfig(
        model=GPTConfig(sequence_len=512, vocab_size=8192, n_layer=4, n_head=4, n_kv_head=4, n_embd=256,
                        window_pattern="L"),
        device_batch=4, total_batch_tokens=4 * 512, impl="cuda",
    )


PRESETS = {
    "tiny-cpu": _tiny_cpu,
    "d512": _d512,
    "d1280": _d1280,
    "d512-topk": _d512_topk,
    "ref-default": _ref_default,
}


def preset(name: str) -> TrainConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    return PRESETS[name]()


def _coerce(old: Any, value: str) -> Any:
    if isinstance(old, bool):
        return value.lower() in ("1", "true", "yes", "on")
    if isinstance(old, int):
        return int(float(value))
    if isinstance(old, float):
        return float(value)
    if isinstance(old, tuple):
        return tuple(float(x) for x in value.split(","))
    return value


def apply_overrides(cfg: TrainConfig, overrides: list[str]) -> TrainConfig:
    """Apply ``key=value`` overrides; nested keys use dots (``model.n_layer=4``)."""
    for item in overrides:
        key, _, value = item.lstrip("-").partition("=")
        key = key.replace("-", "_")
        target: Any = cfg
        parts = key.split(".")
        for p in parts[:-1]:
            target = getattr(target, p)
        if not hasattr(target, parts[-1]):
            raise KeyError(f"unknown config key {key!r}")
        setattr(target, parts[-1], _coerce(getattr(target, parts[-1]), value))
    return cfg

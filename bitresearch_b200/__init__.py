"""bitresearch-b200: a data-parallel GPT pretraining framework for NVIDIA B200 (sm_100a).

Capabilities follow gauravsaini/bitresearch (autoresearch GPT, MuonAdamW, ring all-reduce with f16
wire and top-k + error feedback, fixed-time-budget training scored by val_bpb, safetensors
checkpoints with the reference's names); the compute path is PyTorch plus hand-written sm_100a
CUDA kernels and in-kernel NVLink collectives.
"""
from .config import GPTConfig, TrainConfig, preset  # noqa: F401

__version__ = "0.1.0"

"""The sm_100a engine's loss and every gradient vs the eager fp32 model on the same weights/batch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(cuda, n_kv=2, T=256, pattern="SL"):
    from bitresearch_b200.config import GPTConfig
    from bitresearch_b200.models.gpt import GPT
    cfg = GPTConfig(sequence_len=T, vocab_size=512, n_layer=2, n_head=2, n_kv_head=n_kv, n_embd=256,
                    window_pattern=pattern)
    torch.manual_seed(0)
    m = GPT(cfg, init="normal", seed=0, device=cuda)
    g = torch.Generator(device="cpu").manual_seed(1)
    with torch.no_grad():
        for n, p in m.named().items():
            if n.endswith("_proj") or n.endswith("_ve_gate"):
                p.copy_((torch.randn(p.shape, generator=g) * 0.05).to(cuda))
    return cfg, m


@pytest.mark.parametrize("n_kv", [2, 1])
def test_engine_matches_eager(cuda, n_kv):
    from collections import OrderedDict

    from bitresearch_b200.models.engine import FusedGPTEngine
    cfg, m = _setup(cuda, n_kv)
    B, T = 2, cfg.sequence_len
    idx = torch.randint(0, cfg.vocab_size, (B, T), device=cuda, dtype=torch.int32)
    tgt = torch.randint(0, cfg.vocab_size, (B, T), device=cuda, dtype=torch.int32)
    tgt[0, :5] = -1
    flat = torch.zeros(m.num_params(), device=cuda)
    views, o = OrderedDict(), 0
    for n, p in m.named().items():
        views[n] = flat[o:o + p.numel()].view_as(p)
        o += p.numel()
    eng = FusedGPTEngine(m, views, B, T, flat_grad=flat)
    loss = eng.forward_backward(idx, tgt)
    torch.cuda.synchronize()
    assert eng.status() == 0
    ref_loss = m.forward_torch(idx.long(), tgt.long())
    ref_loss.backward()
    assert abs(loss.item() - ref_loss.item()) < 2e-2 * abs(ref_loss.item())
    for n, p in m.named().items():
        ref = p.grad
        err = (views[n] - ref).abs().max().item()
        scale = ref.abs().max().item() + 1e-8
        assert err <= 0.08 * scale, (n, err, scale)
    nats = eng.per_token_nats(idx, tgt)
    ref_nats = m.forward_torch(idx.long(), tgt.long(), reduction="none")
    assert (nats - ref_nats).abs().max().item() < 0.05

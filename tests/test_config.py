from bitresearch_b200.config import (GPTConfig, apply_overrides, compute_window_sizes, effective_window,
                                     estimate_flops_per_token, estimate_params, has_value_embedding, preset)
from bitresearch_b200.models.gpt import GPT, param_specs


def test_default_d512_param_count_and_flops():
    cfg = GPTConfig()
    assert estimate_params(cfg) == 50_332_176  # 50.33M (program.md:134 "50.3")
    assert round(estimate_flops_per_token(cfg) / 1e6, 1) == 213.9
    specs = param_specs(cfg)
    assert sum(int(__import__("numpy").prod(s)) for _, s, _ in specs) == estimate_params(cfg)


def test_windows_sssl_last_layer_long():
    cfg = GPTConfig(sequence_len=2048, n_layer=8, window_pattern="SSSL")
    w = [a for a, _ in compute_window_sizes(cfg)]
    assert w == [1024, 1024, 1024, 2048, 1024, 1024, 1024, 2048]
    cfg = GPTConfig(sequence_len=512, n_layer=3, window_pattern="S")
    assert [a for a, _ in compute_window_sizes(cfg)] == [256, 256, 512]
    assert effective_window(1024, 2048) == 1024
    assert effective_window(2048, 2048) == 2048
    assert effective_window(1024, 512) == 512


def test_value_embedding_layers():
    assert [i for i in range(8) if has_value_embedding(i, 8)] == [1, 3, 5, 7]
    assert [i for i in range(3) if has_value_embedding(i, 3)] == [0, 2]


def test_param_order_matches_reference():
    cfg = GPTConfig(n_layer=2)
    names = [n for n, _, _ in param_specs(cfg)]
    assert names[:4] == ["wte", "lmHead", "residLambdas", "x0Lambdas"]
    assert names[4:10] == ["layer0_q", "layer0_k", "layer0_v", "layer0_proj", "layer0_fc", "layer0_mlp_proj"]
    assert names[10:17] == ["layer1_q", "layer1_k", "layer1_v", "layer1_proj", "layer1_fc", "layer1_mlp_proj",
                            "layer1_ve_gate"]
    assert names[17:] == ["ve_1"]


def test_presets_and_overrides():
    c = preset("tiny-cpu")
    assert c.model.n_layer == 2 and c.model.n_embd == 128 and c.model.vocab_size == 512
    c = apply_overrides(preset("d512"), ["model.n_layer=4", "matrix_lr=0.02", "overlap=false"])
    assert c.model.n_layer == 4 and c.matrix_lr == 0.02 and c.overlap is False
    m = GPT(GPTConfig(n_layer=2, n_embd=64, n_head=2, n_kv_head=2, vocab_size=64, sequence_len=16))
    assert m.num_params() == estimate_params(m.cfg)


def test_every_preset_runs_on_a_path_that_supports_its_model():
    from bitresearch_b200.config import PRESETS
    from bitresearch_b200.models.engine import FusedGPTEngine
    for name in PRESETS:
        cfg = preset(name)
        if cfg.impl == "cuda":
            assert FusedGPTEngine.unsupported(cfg.model) is None, name

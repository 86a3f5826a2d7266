import json
import os
import struct

import torch

from bitresearch_b200 import checkpoint as ckpt
from bitresearch_b200.config import GPTConfig
from bitresearch_b200.models.gpt import GPT
from bitresearch_b200.optim.muon_adamw import MuonAdamW


def _cfg():
    return GPTConfig(sequence_len=16, vocab_size=64, n_layer=2, n_head=2, n_kv_head=2, n_embd=32, window_pattern="L")


def test_roundtrip_weights_optimizer_metadata(tmp_path):
    m = GPT(_cfg(), seed=1)
    opt = MuonAdamW(m.named(), m.param_groups(), model_dim=32)
    opt.step({n: torch.randn_like(p) for n, p in m.named().items()})
    t, meta = ckpt.build_state(m, opt, step=7, loss_scale=512.0, total_tokens=1234,
                               extra_meta={"smoothLoss": 3.5})
    path = ckpt.save(str(tmp_path / ckpt.checkpoint_filename(7)), t, meta)
    assert "checkpoint_step000007_" in path
    m2 = GPT(_cfg(), seed=2)
    opt2 = MuonAdamW(m2.named(), m2.param_groups(), model_dim=32)
    t2, meta2 = ckpt.load(path)
    assert all(isinstance(v, str) for v in meta2.values())  # safetensors spec: string metadata
    info = ckpt.restore(m2, t2, meta2, opt2)
    assert info["step"] == 7 and info["lossScale"] == 512.0 and info["totalTokens"] == 1234
    assert info["smoothLoss"] == 3.5 and json.loads(meta2["config"])["nEmbd"] == 32
    for n, p in m.named().items():
        assert torch.equal(p, m2.named()[n]), n
    for k, v in opt.state_tensors().items():
        assert torch.equal(v, opt2.state_tensors()[k])
    assert opt2.state_steps() == opt.state_steps()


def test_reads_reference_written_file_with_numeric_metadata_and_exporter_alias(tmp_path):
    # header layout of trainer.ts:1139-1153: numbers in __metadata__ and F32 tensors in order
    cfg = _cfg()
    m = GPT(cfg, seed=3)
    tensors = {n: p.detach().numpy() for n, p in m.named().items()}
    tensors["layer1_value_embed"] = tensors.pop("ve_1")  # exporter alias
    header, off, blobs = {}, 0, []
    for n, a in tensors.items():
        b = a.astype("<f4").tobytes()
        header[n] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"step": 42, "lossScale": 1024, "totalTokens": 99, "config": json.dumps(cfg.to_reference_dict())}
    hb = json.dumps(header).encode()
    (tmp_path / "ref.safetensors").write_bytes(struct.pack("<Q", len(hb)) + hb + b"".join(blobs))
    m2 = GPT(cfg, seed=9)
    t, meta = ckpt.load(str(tmp_path / "ref.safetensors"))
    info = ckpt.restore(m2, t, meta)
    assert info["step"] == 42 and info["restored"] == len(m.named())
    assert torch.equal(m2.named()["ve_1"], m.named()["ve_1"])


def test_safetensors_library_reads_our_files(tmp_path):
    st = __import__("pytest").importorskip("safetensors.torch")
    m = GPT(_cfg())
    t, meta = ckpt.build_state(m, None, step=1)
    ckpt.save(str(tmp_path / "a.safetensors"), t, meta)
    loaded = st.load_file(str(tmp_path / "a.safetensors"))
    assert torch.equal(loaded["wte"], m.named()["wte"])


def test_eval_cli_scores_a_saved_checkpoint(tmp_path, capsys):
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.eval import main
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("tiny-cpu"), ["model.n_layer=1", "model.n_embd=64", "model.n_head=1",
                                               "model.n_kv_head=1", "model.sequence_len=32", "model.vocab_size=128",
                                               "device_batch=2", "total_batch_tokens=64", "eval_tokens=256",
                                               "log_every=0", "results_tsv=", "data=markov", "doc_mean_len=16"])
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    for _ in range(3):
        tr.train_step()
    want = tr.evaluate_bpb()
    path = tr.save_checkpoint(str(tmp_path / "c.safetensors"))
    tr.destroy()
    capsys.readouterr()
    assert main(["--checkpoint", path]) == 0  # the config comes from the checkpoint's metadata
    out = capsys.readouterr().out
    got = float(out.split("val_bpb:")[1].split()[0])
    assert abs(got - want) < 1e-6 and "step:             3" in out and "val_bpb_floor:" in out


def test_eval_cli_takes_the_model_from_a_reference_style_checkpoint(tmp_path, capsys):
    """A checkpoint with only the reference's metadata (step, lossScale, totalTokens, model config)."""
    from bitresearch_b200.eval import main
    cfg = _cfg()
    m = GPT(cfg, seed=4)
    t, meta = ckpt.build_state(m, None, step=11)
    assert "trainConfig" not in meta
    path = ckpt.save(str(tmp_path / "ref.safetensors"), t, meta)
    assert main(["--checkpoint", path, "--preset", "tiny-cpu", "eval_tokens=64", "data=uniform", "bos_every=8",
                 "device_batch=2"]) == 0
    out = capsys.readouterr().out
    assert float(out.split("val_bpb:")[1].split()[0]) > 0 and "step:             11" in out


def _sharded_save(rank, world, out_dir):
    import numpy as np
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    cfg = apply_overrides(preset("tiny-cpu"), ["model.n_layer=1", "model.n_embd=64", "model.n_head=1",
                                               "model.n_kv_head=1", "model.sequence_len=32", "model.vocab_size=128",
                                               "device_batch=2", f"total_batch_tokens={64 * world}",
                                               "eval_tokens=128", "log_every=0", "results_tsv=", "comm=ring"])
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    for _ in range(2):
        tr.train_step()
    path = tr.save_checkpoint(os.path.join(out_dir, "ck"))
    return path, {n: p.detach().numpy().copy() for n, p in tr.model.named().items()}


def test_multi_rank_checkpoint_merges_and_reloads(tmp_path):
    import numpy as np
    from dist_utils import run_world
    from bitresearch_b200.config import apply_overrides, preset
    from bitresearch_b200.train import Trainer
    (p0, w0), (p1, _) = run_world(_sharded_save, 2, str(tmp_path))
    assert p0.endswith(".safetensors") and os.path.isfile(p0)
    t, meta = ckpt.load(p0)
    assert "shard" not in meta and any(k.startswith("adam_") for k in t) and any(k.startswith("muon_") for k in t)
    cfg = apply_overrides(preset("tiny-cpu"), ["model.n_layer=1", "model.n_embd=64", "model.n_head=1",
                                               "model.n_kv_head=1", "model.sequence_len=32", "model.vocab_size=128",
                                               "device_batch=2", "total_batch_tokens=64", "eval_tokens=128",
                                               "log_every=0", "results_tsv="])
    tr = Trainer(cfg, device="cpu", log=lambda m: None)
    tr.initialize()
    info = tr.load_checkpoint(p0)
    assert info["step"] == 2 and info["optimizer_loaded"]
    for n, p in tr.model.named().items():
        assert np.array_equal(p.detach().numpy(), w0[n]), n


def test_resume_takes_the_checkpoint_config(tmp_path, capsys):
    from bitresearch_b200.train import main
    common = ["results_tsv=", "log_every=0", "eval_tokens=256", "model.n_layer=1", "model.n_embd=64",
              "model.n_head=1", "model.n_kv_head=1", "model.sequence_len=32", "model.vocab_size=128",
              "device_batch=2", "total_batch_tokens=64", f"checkpoint_dir={tmp_path}", "checkpoint_interval=3"]
    main(["--preset", "tiny-cpu", "--max-steps", "3"] + common)
    saved = sorted(p for p in os.listdir(tmp_path) if p.endswith(".safetensors"))
    assert len(saved) == 1
    capsys.readouterr()
    main(["--resume", str(tmp_path / saved[0]), "--max-steps", "5", "checkpoint_interval=0"])
    out = capsys.readouterr().out
    assert "num_steps:        5" in out and "depth:            1" in out  # the tiny model, not the d512 default

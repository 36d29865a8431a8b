"""Example trainers and the streamed checkpoint loader, on CPU."""

import json
import os
import subprocess
import sys

import pytest
import torch

import zeroq_b200 as zq
from zeroq_b200.models import DecoderLM, get_config
from zeroq_b200.utils.loading import hf_to_decoder_name, save_hf_checkpoint

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_hf_name_mapping():
    assert hf_to_decoder_name("model.layers.3.self_attn.q_proj.weight") == "layers.3.q_proj.weight"
    assert hf_to_decoder_name("model.layers.0.mlp.down_proj.weight") == "layers.0.down_proj.weight"
    assert hf_to_decoder_name("model.layers.1.post_attention_layernorm.weight") == \
        "layers.1.mlp_norm.weight"
    assert hf_to_decoder_name("model.embed_tokens.weight") == "embed_tokens.weight"
    assert hf_to_decoder_name("model.rotary_emb.inv_freq") is None


@pytest.mark.parametrize("qkv_bias", [False, True])
def test_streamed_load_equals_direct_partition(tmp_path, qkv_bias):
    """Meta skeleton + tensor-by-tensor sharding from an HF-named safetensors file
    gives the same model as partitioning the dense model directly."""
    cfg = get_config("tiny", n_layers=2, vocab_size=1000, qkv_bias=qkv_bias, lora_r=4)
    dense = DecoderLM(cfg).init_dense_(seed=3)
    if qkv_bias:
        with torch.no_grad():
            for layer in dense.layers:
                for m in (layer.q_proj, layer.k_proj, layer.v_proj):
                    m.bias.normal_(0, 0.02)
    ck = tmp_path / "model.safetensors"
    save_hf_checkpoint(dense, str(ck), vocab_size=cfg.vocab_size)

    zcfg = zq.ZeroQConfig(exclude_modules=["lm_head", "embed_tokens"])
    direct = DecoderLM(cfg).init_dense_(seed=3)
    if qkv_bias:
        with torch.no_grad():
            for a, b in zip(direct.layers, dense.layers):
                for n in ("q_proj", "k_proj", "v_proj"):
                    getattr(a, n).bias.copy_(getattr(b, n).bias)
    zq.prepare_model_for_zeroq(direct, zcfg)

    streamed = DecoderLM(cfg).init_meta_()
    zq.prepare_model_for_zeroq(streamed, zcfg, checkpoint=str(ck))
    counts = streamed._zeroq_load_counts
    # 2 layers x (7 projections + 2 norms) + final norm, all frozen and sharded
    assert counts["sharded"] == 2 * 9 + 1 + (6 if qkv_bias else 0) and counts["skipped"] == 0

    # same LoRA weights in both, then identical forward/backward
    with torch.no_grad():
        for (na, pa), (nb, pb) in zip(direct.named_parameters(), streamed.named_parameters()):
            if "lora_" in na:
                pb.copy_(pa)
    x = torch.randint(0, cfg.vocab_size, (2, 32))
    la = direct(x, x)
    lb = streamed(x, x)
    assert torch.equal(la, lb)


@pytest.mark.slow
def test_train_qlora_example_cpu_save_resume(tmp_path):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT)
    ex = os.path.join(ROOT, "examples", "train_qlora.py")
    base = [sys.executable, ex, "--model", "tiny", "--layers", "2", "--seq", "64", "--batch", "2",
            "--lr", "1e-3", "--lora-r", "4", "--save", str(tmp_path / "run")]
    r = subprocess.run(base + ["--steps", "3"], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    logs = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert [l["step"] for l in logs if "step" in l and "loss" in l] == [1, 2, 3]
    assert os.path.exists(tmp_path / "run" / "adapter_model.safetensors")
    r2 = subprocess.run(base + ["--steps", "5", "--resume", str(tmp_path / "run")], env=env,
                        capture_output=True, text=True, timeout=600)
    assert r2.returncode == 0, r2.stdout + r2.stderr
    logs2 = [json.loads(l) for l in r2.stdout.splitlines() if l.startswith("{")]
    assert logs2[0]["resume_step"] == 3
    assert [l["step"] for l in logs2 if "loss" in l] == [4, 5]

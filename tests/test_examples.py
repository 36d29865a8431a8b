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
            "--lr", "1e-3", "--lora-r", "4", "--max-grad-norm", "1.0", "--save", str(tmp_path / "run")]
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


def _run(args, timeout=600, extra_env=None):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT)
    env.update(extra_env or {})
    return subprocess.run(args, env=env, capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("optimizer", ["adamw", "lion-fused", "adamw-offload"])
def test_train_from_scratch_example_learns(optimizer):
    """fp32 master shards (ZeroQTrainConfig): memorising one batch lowers the loss
    with AdamW, the fused Lion step and the CPU-offload path."""
    r = _run([sys.executable, os.path.join(ROOT, "examples", "train_from_scratch.py"), "--layers",
              "2", "--steps", "6", "--seq", "64", "--batch", "2", "--optimizer", optimizer,
              "--fixed-batch"])
    assert r.returncode == 0, r.stdout + r.stderr
    done = [json.loads(l) for l in r.stdout.splitlines() if l.startswith('{"event": "done"')][0]
    assert done["last_loss"] < done["first_loss"] - 0.5


def test_network_test_local_round_trips():
    r = _run([sys.executable, os.path.join(ROOT, "examples", "network_test.py"), "--role", "local",
              "--port", "5597", "--reps", "1"], timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]
    assert [row["elements"] for row in rows] == [1 << 10, 1 << 16, 1 << 20, 1 << 24]


@pytest.mark.distributed
def test_smoke_lora_multinode_two_ranks_agree():
    r = _run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
              "--master-addr", "127.0.0.1", "--master-port", "29563",
              os.path.join(ROOT, "examples", "smoke_lora_multinode.py")], timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    done = [json.loads(l) for l in r.stdout.splitlines() if l.startswith('{"event": "done"')][0]
    assert done["ok"] and done["world"] == 2


def test_prefetch_tool_help():
    r = _run([sys.executable, os.path.join(ROOT, "examples", "prefetch_hf_model.py"), "--help"],
             timeout=120)
    assert r.returncode == 0 and "--local-dir" in r.stdout


def test_launch_script_dry_run_builds_one_torchrun_per_node():
    env = dict(os.environ, HOSTS="node0 node1 node2", NPROC="8", MASTER_ADDR="10.0.0.1",
               DRY_RUN="1")
    r = subprocess.run(["bash", os.path.join(ROOT, "examples", "launch_multinode.sh"), "start",
                        "examples/train_qlora.py", "--model", "qwen2.5-32b"], env=env,
                       capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    cmds = [l for l in r.stdout.splitlines() if l.startswith("[node")]
    assert len(cmds) == 3
    for i, c in enumerate(cmds):
        assert f"--node-rank {i}" in c and "--nnodes 3" in c and "--master-addr 10.0.0.1" in c
        assert "setsid" in c and "qwen2.5-32b" in c


def test_memory_scaling_benchmark_shards_shrink_with_world():
    r = _run([sys.executable, os.path.join(ROOT, "benchmarks", "memory_scaling.py"), "--hidden",
              "256", "--layers", "2", "--world", "1", "2"], timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    rows = {d["world"]: d for d in (json.loads(l) for l in r.stdout.splitlines() if l.startswith("{"))}
    assert rows[1]["ratio_vs_fp16"] > 3.4   # NF4 + fp32 absmax per 64 vs fp16
    assert rows[2]["nf4_shard_bytes_per_rank"] <= rows[1]["nf4_shard_bytes_per_rank"] / 2 + 64

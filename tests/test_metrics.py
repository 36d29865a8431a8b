"""Step metrics: counters and NVTX ranges (CPU), the per-step JSONL logger of
``Trainer`` (GPU: CUDA-event step times)."""

import json

import pytest
import torch

from zeroq_b200.utils import metrics


def test_counters_and_nvtx_noop():
    metrics.reset_counters()
    metrics.count("gather_bytes", 10)
    metrics.count("gather_bytes", 5)
    assert metrics.snapshot() == {"gather_bytes": 15}
    with metrics.nvtx_range("x"):   # tracing off: a no-op
        pass
    metrics.reset_counters()
    assert metrics.snapshot() == {}


@pytest.mark.gpu
def test_trainer_step_logger_writes_jsonl(cuda, tmp_path):
    import zeroq_b200 as zq
    from zeroq_b200.models import DecoderLM, get_config
    from zeroq_b200.train import Trainer, synthetic_batch

    cfg = get_config("4.7b", d_model=256, n_layers=2, n_heads=2, n_kv_heads=2, ffn_dim=1024,
                     vocab_size=1000, lora_r=16, lora_alpha=32.0)
    model = DecoderLM(cfg, device=cuda).init_dense_(seed=0)
    zq.initialize(model, zq.ZeroQConfig(compute_dtype=torch.bfloat16, compute_in_4bit=True,
                                        gather_once=True,
                                        exclude_modules=["lm_head", "embed_tokens"]),
                  trainable_patterns=("lora_", "norm"))
    opt = zq.ShardedAdamW(model.trainable_parameters(), lr=1e-3, max_grad_norm=1.0)
    path = tmp_path / "m.jsonl"
    log = metrics.StepLogger(str(path), flush_every=2, flops_per_token=model.flops_per_token(128),
                             peak_tflops=1000.0)
    tr = Trainer(model, opt, cuda, logger=log)
    x, y = synthetic_batch(2, 128, cfg.vocab_size, seed=0)
    losses = [tr.step(x, y) for _ in range(3)]
    log.flush()
    recs = [json.loads(l) for l in path.read_text().splitlines()]
    assert [r["step"] for r in recs] == [0, 1, 2]
    for r, l in zip(recs, losses):
        assert abs(r["loss"] - l) < 1e-4 and r["ms"] > 0 and r["tokens_per_s"] > 0
        assert 0 < r["frac_of_peak"] < 1
    assert opt.grad_norm() is not None and opt.grad_norm() > 0

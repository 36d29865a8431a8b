#!/usr/bin/env python
"""Hugging Face ``Trainer`` path: LoRA + ZeRO-Q on a Hugging Face causal LM.

Counterpart of the reference's ``examples/train_7b_zeroq.py``: the model's
``nn.Linear`` projections become NF4-sharded ``Linear4bit`` modules with LoRA
adapters (``apply_lora_with_zeroq``; PEFT is used when installed), and
``ZeroQTrainer`` trains them with the stock HF training loop.

    python examples/train_hf_trainer.py --model-path /path/to/local/hf/model --steps 100
    python examples/train_hf_trainer.py --arch llama --hidden 256 --layers 2 --steps 3   # random init

Without ``--model-path`` a small Llama/Qwen2 model is built from a config with
random weights (no download).  Data: ``--data FILE`` (bytes as tokens) or
random token ids.  HF's ``Trainer`` needs ``accelerate``; where it is missing
the same prepared model is trained by a plain loop instead (``--plain-loop``
forces that).
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import zeroq_b200 as zq  # noqa: E402


def build_model(args):
    import transformers

    if args.model_path:
        return transformers.AutoModelForCausalLM.from_pretrained(args.model_path,
                                                                 torch_dtype=torch.bfloat16)
    kw = dict(vocab_size=args.vocab, hidden_size=args.hidden, intermediate_size=args.hidden * 2,
              num_hidden_layers=args.layers, num_attention_heads=max(1, args.hidden // 64),
              num_key_value_heads=max(1, args.hidden // 128))
    if args.arch == "qwen2":
        cfg = transformers.Qwen2Config(**kw)
        return transformers.Qwen2ForCausalLM(cfg)
    cfg = transformers.LlamaConfig(**kw)
    return transformers.LlamaForCausalLM(cfg)


class TokenDataset(torch.utils.data.Dataset):
    def __init__(self, tokens: torch.Tensor, seq: int):
        self.t, self.seq = tokens, seq
        self.n = (tokens.numel() - 1) // seq

    def __len__(self):
        return self.n

    def __getitem__(self, i):
        w = self.t[i * self.seq:(i + 1) * self.seq]
        return {"input_ids": w.clone(), "labels": w.clone()}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--model-path", default=None)
    p.add_argument("--arch", choices=["llama", "qwen2"], default="llama")
    p.add_argument("--hidden", type=int, default=256)
    p.add_argument("--layers", type=int, default=2)
    p.add_argument("--vocab", type=int, default=1024)
    p.add_argument("--data", default=None)
    p.add_argument("--seq", type=int, default=128)
    p.add_argument("--batch", type=int, default=2)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--lr", type=float, default=2e-4)
    p.add_argument("--lora-r", type=int, default=8)
    p.add_argument("--output", default="zeroq_hf_out")
    p.add_argument("--plain-loop", action="store_true")
    args = p.parse_args(argv)

    model = build_model(args)
    vocab = model.config.vocab_size
    if args.data:
        with open(args.data, "rb") as f:
            tokens = torch.frombuffer(bytearray(f.read()), dtype=torch.uint8).long() % vocab
    else:
        tokens = torch.randint(0, vocab, ((args.steps * args.batch + 4) * args.seq + 1,),
                               generator=torch.Generator().manual_seed(0))
    zcfg = zq.ZeroQConfig(compute_dtype=torch.bfloat16 if torch.cuda.is_available() else torch.float32,
                          exclude_modules=["lm_head", "embed_tokens"])
    lora = {"r": args.lora_r, "lora_alpha": 2 * args.lora_r,
            "target_modules": ["q_proj", "k_proj", "v_proj", "o_proj"]}
    model = zq.apply_lora_with_zeroq(model, lora, zcfg)
    if torch.cuda.is_available():
        model = model.cuda()
    ds = TokenDataset(tokens, args.seq)
    try:
        if args.plain_loop:
            raise ImportError("plain loop requested")
        import accelerate  # noqa: F401  (HF Trainer needs it)
        from transformers import TrainingArguments
    except ImportError as e:
        print(f"HF Trainer unavailable ({e}); training with a plain loop", flush=True)
        return plain_loop(model, ds, args)
    targs = TrainingArguments(output_dir=args.output, per_device_train_batch_size=args.batch,
                              max_steps=args.steps, learning_rate=args.lr, logging_steps=1,
                              report_to="none", save_strategy="no", dataloader_num_workers=0,
                              use_cpu=not torch.cuda.is_available())
    trainer = zq.ZeroQTrainer(model=model, args=targs, zeroq_config=zcfg, train_dataset=ds)
    out = trainer.train()
    trainer.log_zeroq_stats()
    print(f"final train loss {out.training_loss:.4f}; zeroq stats {zq.get_zeroq_memory_stats(model)}")
    return 0


def plain_loop(model, ds, args) -> int:
    dev = next(p.device for p in model.parameters() if p.requires_grad)
    opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=args.lr)
    loader = torch.utils.data.DataLoader(ds, batch_size=args.batch, shuffle=True)
    it = iter(loader)
    for step in range(args.steps):
        try:
            batch = next(it)
        except StopIteration:
            it = iter(loader)
            batch = next(it)
        out = model(input_ids=batch["input_ids"].to(dev), labels=batch["labels"].to(dev))
        out.loss.backward()
        opt.step()
        opt.zero_grad()
        print(f"step {step + 1} loss {out.loss.item():.4f}", flush=True)
    print(f"zeroq stats {zq.get_zeroq_memory_stats(model)}", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())

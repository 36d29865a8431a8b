"""Coordinator lifecycle, training modes, model, checkpoints - single process on CPU
(reference tests/test_train_from_scratch.py:138-276, tests/test_coordinator.py)."""

import os

import pytest
import torch
import torch.nn as nn

import zeroq_b200 as zq
from zeroq_b200.models import DecoderLM, get_config
from zeroq_b200.ops.qlinear import Linear4bit


class TinyMLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(64, 128)
        self.fc2 = nn.Linear(128, 64)
        self.lm_head = nn.Linear(64, 10)

    def forward(self, x):
        return self.lm_head(torch.relu(self.fc2(torch.relu(self.fc1(x)))))


def _frozen_mlp(seed=0):
    torch.manual_seed(seed)
    m = TinyMLP()
    for p in m.parameters():
        p.requires_grad_(False)
    return m


class TestGatherRelease:
    def test_partition_gather_release(self):
        m = _frozen_mlp()
        w_ref = m.fc1.weight.detach().clone()
        coord = zq.ZeroQCoordinator(zq.ZeroQConfig())
        wrap = zq.ZeroQModuleWrapper(m, coord)
        assert len(coord) == 4  # fc1/fc2 weight+bias; lm_head excluded
        wrap.partition()
        assert m.fc1.weight.numel() == 0
        zp = coord.get_param_for_tensor  # registry still keyed by the original tensors
        assert zp is not None
        p0 = coord._params[0]
        p0.start_gather(async_op=False)
        assert p0.status == zq.ZeroQParamStatus.AVAILABLE
        assert m.fc1.weight.shape == w_ref.shape
        assert ((m.fc1.weight - w_ref).abs().mean() / w_ref.abs().mean()) < 0.12
        p0.release()
        assert m.fc1.weight.numel() == 0 and p0.status == zq.ZeroQParamStatus.NOT_AVAILABLE

    def test_hooks_forward_backward(self):
        m = _frozen_mlp()
        x = torch.randn(8, 64)
        ref = m(x)
        coord = zq.ZeroQCoordinator(zq.ZeroQConfig())
        zq.ZeroQModuleWrapper(m, coord).partition()
        out = m(x)
        assert out.shape == ref.shape
        assert torch.corrcoef(torch.stack([out.flatten(), ref.flatten()]))[0, 1] > 0.99
        assert m.fc1.weight.numel() == 0  # released after forward
        stats = coord.get_memory_stats()
        assert stats["compression_ratio"] > 1.0 and stats["num_params"] == 4

    def test_exclude_and_frozen_rules(self):
        m = _frozen_mlp()
        m.fc2.weight.requires_grad_(True)
        coord = zq.ZeroQCoordinator(zq.ZeroQConfig())
        zq.ZeroQModuleWrapper(m, coord)
        names = {(p.module_path, p.param_name) for p in coord._params.values()}
        assert ("fc2", "weight") not in names and not any(n[0] == "lm_head" for n in names)


class TestTrainingMode:
    def test_master_shards_and_grads(self):
        torch.manual_seed(0)
        m = TinyMLP()
        ref = [p.detach().clone() for p in m.parameters()]
        cfg = zq.ZeroQTrainConfig(exclude_modules=[])
        coord = zq.ZeroQCoordinator(cfg)
        zq.ZeroQModuleWrapper(m, coord).partition()
        masters = coord.trainable_master_params()
        assert len(masters) == 6 and all(p.dtype == torch.float32 for p in masters)
        opt = torch.optim.AdamW(masters, lr=1e-2)
        x = torch.randn(16, 64)
        losses = []
        for _ in range(8):
            loss = m(x).pow(2).mean()
            loss.backward()
            assert all(p.grad is not None for p in masters)
            opt.step()
            opt.zero_grad()
            losses.append(loss.item())
        assert losses[-1] < losses[0]
        st = coord.gather_full_state_dict()
        assert "fc1.weight" in st and st["fc1.weight"].shape == ref[0].shape

    def test_cpu_offload_manual_grad_and_requantise(self):
        torch.manual_seed(0)
        m = TinyMLP()
        cfg = zq.ZeroQTrainConfig(cpu_offload=True, exclude_modules=["lm_head"])
        coord = zq.ZeroQCoordinator(cfg)
        zq.ZeroQModuleWrapper(m, coord).partition()
        zparam = coord._params[0]
        assert zparam.local_packed is not None and zparam.master_shard.device.type == "cpu"
        masters = coord.trainable_master_params()
        opt = torch.optim.SGD(masters, lr=0.1)
        # the manual weight gradient runs in the module's backward hook, which
        # needs a gradient to flow through the module (here: into x)
        x = torch.randn(4, 64, requires_grad=True)
        m(x).sum().backward()
        assert zparam.master_shard.grad is not None
        before = zparam.local_packed.clone()
        opt.step()
        coord.update_4bit_from_masters()
        assert not torch.equal(before, zparam.local_packed)

    def test_fused_lion_step(self):
        torch.manual_seed(0)
        m = TinyMLP()
        cfg = zq.ZeroQTrainConfig(fused_shard_step=True, master_dtype=torch.float16,
                                  exclude_modules=["lm_head"], lion_lr=1e-2)
        coord = zq.ZeroQCoordinator(cfg)
        zq.ZeroQModuleWrapper(m, coord).partition()
        zparam = coord._params[0]
        before = zparam.master_shard.detach().clone()
        m(torch.randn(4, 64, requires_grad=True)).sum().backward()
        after = zparam.master_shard.detach()
        assert after.dtype == torch.float16 and not torch.equal(before, after)
        assert hasattr(zparam, "_lion_m")


class TestModel:
    @pytest.fixture
    def cfg(self):
        return get_config("tiny", lora_r=8, n_layers=2)

    def test_4bit_compute_matches_dequantised_dense(self, cfg):
        torch.manual_seed(0)
        m = DecoderLM(cfg).init_dense_(seed=3)
        x = torch.randint(0, cfg.vocab_size, (2, 32))
        zq.initialize(m, zq.ZeroQConfig(compute_in_4bit=True, gather_once=True,
                                        exclude_modules=["lm_head", "embed_tokens"]))
        assert all(mod.has_nf4 for mod in m.modules() if isinstance(mod, Linear4bit))
        logits = m(x)
        # dense model with the dequantised weights gives the same logits
        d = DecoderLM(cfg)
        d.load_state_dict({k: v for k, v in m.state_dict().items()
                           if not k.endswith(("weight_packed", "weight_absmax"))}, strict=False)
        for (n1, a), (n2, b) in zip(m.named_modules(), d.named_modules()):
            if isinstance(a, Linear4bit):
                b.weight = nn.Parameter(a.dequantized_weight(torch.bfloat16), requires_grad=False)
        ref = d(x)
        assert torch.allclose(logits.float(), ref.float(), atol=5e-2, rtol=5e-2)

    def test_activation_checkpointing_same_grads(self, cfg):
        torch.manual_seed(0)
        x = torch.randint(0, cfg.vocab_size, (2, 32))
        y = torch.randint(0, cfg.vocab_size, (2, 32))
        grads = []
        for ck in (False, True):
            c = get_config("tiny", lora_r=8, n_layers=2, activation_checkpointing=ck)
            torch.manual_seed(1)
            m = DecoderLM(c).init_nf4_(seed=5)
            for mod in m.modules():
                if isinstance(mod, Linear4bit) and mod.lora_r:
                    nn.init.normal_(mod.lora_B, std=0.02)
            m.train()
            m(x, y).backward()
            grads.append(m.layers[0].q_proj.lora_A.grad.clone())
        assert torch.allclose(grads[0], grads[1], atol=1e-5)

    def test_enable_gradient_checkpointing_api(self, cfg):
        m = DecoderLM(cfg).init_nf4_(seed=0)
        zq.enable_gradient_checkpointing(m)
        assert all(getattr(layer, "_zq_ckpt_wrapped", False) for layer in m.layers)
        est = zq.estimate_checkpoint_memory(4096, 32, 2, 512)
        assert est["savings"] > 1

    def test_sharded_checkpoint_roundtrip(self, cfg, tmp_path):
        m = DecoderLM(cfg).init_dense_(seed=1)
        zq.initialize(m, zq.ZeroQConfig(compute_in_4bit=True, gather_once=True,
                                        exclude_modules=["lm_head", "embed_tokens"]),
                      trainable_patterns=("lora_", "norm"))
        opt = zq.ShardedAdamW(m.trainable_parameters(), lr=1e-3)
        x = torch.randint(0, cfg.vocab_size, (2, 16))
        m(x, x).backward()
        opt.step()
        zq.save_sharded_checkpoint(str(tmp_path / "ck"), m, opt, step=7)
        out_ref = m(x).detach()
        m2 = DecoderLM(cfg).init_dense_(seed=99)
        zq.initialize(m2, zq.ZeroQConfig(compute_in_4bit=True, gather_once=True,
                                         exclude_modules=["lm_head", "embed_tokens"]),
                      trainable_patterns=("lora_", "norm"))
        m2.embed_tokens.weight.data.copy_(m.embed_tokens.weight.data)
        opt2 = zq.ShardedAdamW(m2.trainable_parameters(), lr=1e-3)
        step = zq.load_sharded_checkpoint(str(tmp_path / "ck"), m2, opt2)
        assert step == 7 and opt2.step_count == 1
        assert torch.equal(m2(x).detach(), out_ref)

    def test_adapter_save_load(self, cfg, tmp_path):
        m = DecoderLM(cfg).init_nf4_(seed=0)
        for mod in m.modules():
            if isinstance(mod, Linear4bit) and mod.lora_r:
                nn.init.normal_(mod.lora_B)
        zq.save_adapters(m, str(tmp_path / "ad"))
        m2 = DecoderLM(cfg).init_nf4_(seed=0)
        n = zq.load_adapters(m2, str(tmp_path / "ad"))
        assert n == 2 * 2 * 4
        assert torch.equal(m2.layers[1].v_proj.lora_B, m.layers[1].v_proj.lora_B)
        assert os.path.exists(tmp_path / "ad" / "adapter_config.json")


def test_inject_lora_into_plain_model():
    m = _frozen_mlp()
    zq.inject_lora(m, r=4, lora_alpha=8, target_modules=["fc1", "fc2"])
    assert isinstance(m.fc1, Linear4bit) and m.fc1.lora_r == 4
    m = zq.apply_lora_with_zeroq(m, {"r": 4, "lora_alpha": 8, "target_modules": ["fc1"]},
                                 zq.ZeroQConfig())
    trainable = [n for n, p in m.named_parameters() if p.requires_grad]
    assert trainable and all("lora_" in n for n in trainable)
    out = m(torch.randn(3, 64))
    out.sum().backward()
    assert m.fc1.lora_A.grad is not None


def test_gather_release_with_frozen_sharded_norms():
    """Frozen norm weights are sharded too; the decoder must reach them through the
    norm modules so the gather hooks run (a bare ``.weight`` would be empty)."""
    cfg = get_config("tiny", lora_r=4, n_layers=2)
    m = DecoderLM(cfg).init_dense_(seed=0)
    zq.initialize(m, zq.ZeroQConfig(compute_in_4bit=True, gather_once=False,
                                    exclude_modules=["lm_head", "embed_tokens"]),
                  trainable_patterns=("lora_",))
    coord = m._zeroq_coordinator
    norm_params = [p for p in coord._params.values() if "norm" in (p.module_path or "")]
    assert norm_params, "norm weights should be registered and sharded"
    assert m.layers[0].attn_norm.weight.numel() == 0  # released between uses
    x = torch.randint(0, cfg.vocab_size, (2, 32))
    loss = m(x, x)
    loss.backward()
    assert torch.isfinite(loss)
    assert m.layers[0].q_proj.lora_B.grad is not None


def test_linear4bit_peer_source_gathers_when_the_fused_kernel_does_not_apply():
    """A Linear4bit whose weight stays in its owners' shards (set_peer_source): off
    the fused path (CPU, torch backend) forward and backward assemble the NF4 data
    through the pool and match the resident-NF4 module exactly."""
    from zeroq_b200.ops.qlinear import Linear4bit

    torch.manual_seed(0)
    lin = Linear4bit(128, 64, lora_r=4, backend="torch", device="cpu")
    lin.quantize_from(torch.randn(64, 128) * 0.02)
    with torch.no_grad():
        lin.lora_B.normal_(0, 0.05)
    pk, am = lin.weight_packed.clone(), lin.weight_absmax.clone()
    x = torch.randn(3, 5, 128, requires_grad=True)
    ref = lin(x)
    ref.square().sum().backward()
    gx_ref, gA_ref = x.grad.clone(), lin.lora_A.grad.clone()

    class Pool:
        calls = 0

        def gather(self, zq):
            Pool.calls += 1

            class H:
                def wait(self):
                    return pk, am
            return H()

    lin.set_peer_source(Pool(), None)
    assert lin.has_nf4 and lin.weight_packed is None
    x.grad = None
    lin.lora_A.grad = None
    y = lin(x)
    y.square().sum().backward()
    assert torch.equal(y, ref) and torch.equal(x.grad, gx_ref)
    assert torch.equal(lin.lora_A.grad, gA_ref)
    assert Pool.calls == 2  # forward and backward each assemble once
    lin.clear_nf4()
    assert not lin.has_nf4


def test_gelu_mlp_split_form_matches_plain_form_on_cpu():
    """The split GELU MLP (up returns h and a non-differentiable gelu(h), down takes
    the gradient through h) gives the plain form's values and gradients off the
    fused path, including when one layer holds a full-precision weight."""
    from zeroq_b200.ops.activations import gelu
    from zeroq_b200.ops.qlinear import Linear4bit

    torch.manual_seed(1)
    up = Linear4bit(64, 128, lora_r=4, backend="torch", device="cpu")
    down = Linear4bit(128, 64, lora_r=4, backend="torch", device="cpu")
    up.quantize_from(torch.randn(128, 64) * 0.05)
    down.quantize_from(torch.randn(64, 128) * 0.05)
    with torch.no_grad():
        up.lora_B.normal_(0, 0.05)
        down.lora_B.normal_(0, 0.05)
    x = torch.randn(3, 7, 64, requires_grad=True)
    for full_precision_down in (False, True):
        if full_precision_down:
            w = down.dequantized_weight()
            down.clear_nf4()
            down.weight = torch.nn.Parameter(w, requires_grad=False)
        x.grad = None
        h, a = up(x, act_out="gelu")
        assert not a.requires_grad
        y = down(a, pre=h)
        y.square().sum().backward()
        g1, gA1 = x.grad.clone(), up.lora_A.grad.clone()
        x.grad = None
        up.lora_A.grad = None
        y2 = down(gelu(up(x)))
        y2.square().sum().backward()
        torch.testing.assert_close(y, y2, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(g1, x.grad, rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(gA1, up.lora_A.grad, rtol=1e-4, atol=1e-6)
        up.lora_A.grad = None


def test_flat_params_groups_layout_padding_and_binding():
    """FlatParams with groups: each group contiguous and padded to pad_to, every
    parameter (and its .grad) a view at its offset, values preserved."""
    from zeroq_b200.parallel.optimizer import FlatParams

    torch.manual_seed(3)
    ps = [torch.nn.Parameter(torch.randn(n)) for n in (5, 7, 3, 9)]
    vals = [p.detach().clone() for p in ps]
    groups = [[ps[2], ps[0]], [ps[3]], [ps[1]]]
    flat = FlatParams(ps, pad_to=8, groups=groups)
    assert flat.group_ranges == [(0, 8), (8, 24), (24, 32)] and flat.padded == 32
    assert [p is q for p, q in zip(flat.params, [ps[2], ps[0], ps[3], ps[1]])] == [True] * 4
    assert flat.offsets == [0, 3, 8, 24]
    for p, v, off in zip(flat.params, [vals[2], vals[0], vals[3], vals[1]], flat.offsets):
        assert torch.equal(p.detach(), v)
        assert p.data.data_ptr() == flat.data[off:].data_ptr()
        assert p.grad.data_ptr() == flat.grad[off:].data_ptr()
    assert float(flat.data[17:24].abs().sum()) == 0.0   # padding
    with pytest.raises(ValueError):
        FlatParams(ps, groups=[[ps[0]], [ps[0], ps[1], ps[2], ps[3]]])


def test_sharded_adamw_overlap_buckets_fall_back_off_the_fused_backend():
    """overlap_buckets without the fused multi-rank backend (here: one CPU
    process) keeps the single-shard layout; arm_overlap / bucket_ready are
    no-ops and the step equals torch's AdamW."""
    from zeroq_b200.parallel.optimizer import ShardedAdamW
    from zeroq_b200.parallel.gradient_sync import reduce_scatter_grads_async

    torch.manual_seed(4)
    ps = [torch.nn.Parameter(torch.randn(n)) for n in (6, 10)]
    ref = [torch.nn.Parameter(p.detach().clone()) for p in ps]
    opt = ShardedAdamW(ps, lr=1e-2, overlap_buckets=[[ps[1]], [ps[0]]])
    assert not opt.overlap and len(opt._parts) == 1
    opt.arm_overlap()
    opt.bucket_ready(0)   # no-op
    for p, r in zip(ps, ref):
        p.grad.copy_(torch.randn(p.shape))
        r.grad = p.grad.detach().clone()
    opt.step()
    torch.optim.AdamW(ref, lr=1e-2, weight_decay=0.0).step()
    for p, r in zip(ps, ref):
        torch.testing.assert_close(p.detach(), r.detach(), rtol=1e-5, atol=1e-6)
    g = torch.randn(7)
    torch.testing.assert_close(reduce_scatter_grads_async(g, 1, 0)(), g)


def test_exp2_polynomial_range_reduction_error_bound():
    """The attention forward's polynomial 2^x (csrc/attention_sm100.cu
    exp2_poly3_x2), emulated step by step in float32: round-to-nearest by the
    1.5 * 2^23 addition, degree-3 Horner on [-1/2, 1/2], 2^j added to the
    exponent bits.  Relative error <= 8e-5 over the kernel's input range
    (-120, 8], far below the bf16 rounding of P."""
    import numpy as np

    c3, c2, c1, c0 = (np.float32(0.05508868396282196), np.float32(0.24260404706001282),
                      np.float32(0.6932762265205383), np.float32(0.9999289512634277))
    magic = np.float32(12582912.0)
    x = np.concatenate([np.linspace(-120.0, 8.0, 400001), np.arange(-120, 9)]).astype(np.float32)
    t = (x + magic).astype(np.float32)
    j = (t - magic).astype(np.float32)
    f = (x - j).astype(np.float32)
    assert np.abs(f).max() <= 0.5
    p = c3
    for c in (c2, c1, c0):
        p = (p * f + c).astype(np.float32)   # (the kernel's fma rounds once; this rounds twice)
    bits = p.view(np.int32) + (t.view(np.int32) << 23)
    y = bits.view(np.float32).astype(np.float64)
    rel = np.abs(y / np.exp2(x.astype(np.float64)) - 1.0)
    assert rel.max() < 8e-5, rel.max()


def test_swiglu_mlp_split_form_matches_plain_form_on_cpu():
    """The split SwiGLU MLP (up returns u and a non-differentiable silu(g)·u, down
    takes the gradients through g and u) gives the plain form's values and
    gradients off the fused path, including with a full-precision down weight."""
    from zeroq_b200.ops.activations import swiglu
    from zeroq_b200.ops.qlinear import Linear4bit

    torch.manual_seed(2)
    gate = Linear4bit(64, 96, lora_r=4, backend="torch", device="cpu")
    up = Linear4bit(64, 96, lora_r=4, backend="torch", device="cpu")
    down = Linear4bit(96, 64, lora_r=4, backend="torch", device="cpu")
    for m, shape in ((gate, (96, 64)), (up, (96, 64)), (down, (64, 96))):
        m.quantize_from(torch.randn(*shape) * 0.05)
        with torch.no_grad():
            m.lora_B.normal_(0, 0.05)
    x = torch.randn(3, 7, 64, requires_grad=True)
    for full_precision_down in (False, True):
        if full_precision_down:
            w = down.dequantized_weight()
            down.clear_nf4()
            down.weight = torch.nn.Parameter(w, requires_grad=False)
        x.grad = None
        g = gate(x)
        u, a = up(x, act_out="swiglu", gate=g)
        assert not a.requires_grad
        y = down(a, pre=(g, u))
        y.square().sum().backward()
        g1, gA1, uA1 = x.grad.clone(), gate.lora_A.grad.clone(), up.lora_A.grad.clone()
        x.grad = None
        gate.lora_A.grad = up.lora_A.grad = None
        y2 = down(swiglu(gate(x), up(x)))
        y2.square().sum().backward()
        torch.testing.assert_close(y, y2, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(g1, x.grad, rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(gA1, gate.lora_A.grad, rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(uA1, up.lora_A.grad, rtol=1e-4, atol=1e-6)
        gate.lora_A.grad = up.lora_A.grad = None


def test_linear4bit_rope_argument_matches_apply_rope_on_cpu():
    """Off the fused path (CPU) the rope= argument rotates the projection's output
    like apply_rope, values and input gradients."""
    from zeroq_b200.ops.qlinear import Linear4bit
    from zeroq_b200.ops.rope import apply_rope, rope_table

    torch.manual_seed(2)
    B, S, d, H = 2, 6, 64, 2
    lin = Linear4bit(d, H * 128, lora_r=4, backend="torch", device="cpu")
    lin.quantize_from(torch.randn(H * 128, d) * 0.05)
    x = torch.randn(B, S, d, requires_grad=True)
    cs = rope_table(S, 128, 10000.0, "cpu")
    y = lin(x, rope=cs)
    y.square().sum().backward()
    g1 = x.grad.clone()
    x.grad = None
    y0 = lin(x).view(B, S, H, 128)
    y2, _ = apply_rope(y0, y0, 10000.0)
    y2.square().sum().backward()
    torch.testing.assert_close(y.view(B, S, H, 128), y2, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(g1, x.grad, rtol=1e-4, atol=1e-6)


def test_chunked_cross_entropy_falls_back_on_cpu():
    from zeroq_b200.ops.cross_entropy import lm_head_cross_entropy

    torch.manual_seed(0)
    h = torch.randn(16, 64)
    W = torch.randn(256, 64) * 0.1
    t = torch.randint(0, 250, (16,))
    loss = lm_head_cross_entropy(h, W, t, 250, chunk=128)
    ref = torch.nn.functional.cross_entropy(h @ W[:250].t(), t)
    assert abs(loss.item() - ref.item()) < 1e-4

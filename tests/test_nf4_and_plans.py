"""NF4/FP4 codec oracle, double quantisation, shard plans, configs."""

import pytest
import torch

from zeroq_b200 import (MAXWELL_CONFIG, PHOENIX_CLUSTER_CONFIG, TRAIN_FROM_SCRATCH_CONFIG,
                        MultiNodeConfig, ZeroQConfig, ZeroQTrainConfig, make_plan)
from zeroq_b200.ops.nf4 import (FP4_CODE, NF4_CODE, dequantize_4bit, double_quantize_absmax,
                                nf4_code_from_normal_quantiles, quantize_4bit,
                                quantize_4bit_reference)
from zeroq_b200.parallel.shard_plan import ceil_plan, compute_weighted_shard_lengths, uniform_remainder_plan


def test_nf4_code_is_the_normal_quantile_construction():
    pytest.importorskip("scipy")
    rebuilt = nf4_code_from_normal_quantiles()
    assert len(rebuilt) == 16
    for a, b in zip(rebuilt, NF4_CODE):
        assert abs(a - b) < 1e-6


def test_codes_roundtrip_exactly():
    for qt, code in (("nf4", NF4_CODE), ("fp4", FP4_CODE)):
        vals = torch.tensor(code, dtype=torch.float32).repeat(4)  # 64 values, absmax 1
        p, st = quantize_4bit(vals, 64, qt)
        back = dequantize_4bit(p, st)
        assert torch.equal(back.abs(), vals.abs())


def test_packing_high_nibble_first():
    x = torch.zeros(64)
    x[0] = 1.0   # code 15 (NF4 +1.0)
    x[1] = -1.0  # code 0
    p, st = quantize_4bit(x, 64, "nf4")
    assert p[0].item() == 0xF0
    assert p[1].item() == 0x77  # zeros map to code 7


def test_ties_round_to_lower_code():
    mids = [(NF4_CODE[i] + NF4_CODE[i + 1]) / 2 for i in range(15)]
    x = torch.zeros(64)
    x[0] = 1.0
    x[2] = torch.tensor(mids[10], dtype=torch.float32)
    p, _ = quantize_4bit_reference(x, 64, "nf4")
    assert (p[1].item() >> 4) == 10


def test_odd_length_and_zero_block():
    x = torch.randn(129)
    x[:64] = 0
    p, st = quantize_4bit(x, 64, "nf4")
    assert p.numel() == 65 and st.absmax.numel() == 3 and st.absmax[0] == 0
    back = dequantize_4bit(p, st)
    assert torch.all(back[:64] == 0) and back.shape == x.shape


def test_double_quant_roundtrip():
    torch.manual_seed(0)
    x = torch.randn(64 * 1000) * 0.02
    p, st = quantize_4bit(x, 64, "nf4")
    dq = double_quantize_absmax(st)
    assert dq.absmax.dtype == torch.uint8
    a = dequantize_4bit(p, dq)
    b = dequantize_4bit(p, st)
    assert ((a - b).abs().max() / b.abs().max()) < 0.02


class TestShardPlan:
    def test_weighted(self):
        assert compute_weighted_shard_lengths(1000, [24.0, 12.0, 24.0]) == [400, 200, 400]

    def test_sum_and_offsets(self):
        pl = make_plan(1003, [2, 2, 1, 1, 1, 1, 1, 1])
        assert sum(pl.lengths) == 1003
        assert pl.offsets[0] == 0 and all(pl.offsets[i + 1] == pl.offsets[i] + pl.lengths[i]
                                          for i in range(7))
        assert pl.lengths[0] >= pl.lengths[2]

    def test_remainder_to_largest_fraction_then_lower_rank(self):
        assert compute_weighted_shard_lengths(10, [1, 1, 1]) == [4, 3, 3]
        assert compute_weighted_shard_lengths(5, [1, 2]) == [2, 3]

    def test_uniform_fallback_and_errors(self):
        assert compute_weighted_shard_lengths(9, [0, 0, 0]) == [3, 3, 3]
        with pytest.raises(ValueError):
            compute_weighted_shard_lengths(9, [])
        with pytest.raises(ValueError):
            compute_weighted_shard_lengths(9, [-1, 2])

    def test_owner_of_and_table(self):
        pl = make_plan(100, [3, 1])
        assert pl.owner_of(0) == (0, 0) and pl.owner_of(99) == (1, 99 - pl.offsets[1])
        assert pl.table().tolist() == [0, pl.offsets[1], 100]

    def test_uniform_and_ceil(self):
        u = uniform_remainder_plan(10, 3)
        assert u.lengths == [3, 3, 4]
        c = ceil_plan(10, 3)
        assert c.lengths == [4, 4, 2]


class TestConfig:
    def test_defaults(self):
        c = ZeroQConfig()
        assert c.quant_type == "nf4" and c.blocksize == 64 and c.exclude_modules == ["lm_head"]
        assert c.compute_dtype == torch.float32 and c.frozen_only and not c.partition_trainable

    def test_validation(self):
        with pytest.raises(ValueError):
            ZeroQConfig(quant_type="int4")
        with pytest.raises(ValueError):
            ZeroQConfig(blocksize=48)
        with pytest.raises(ValueError):
            ZeroQConfig(compute_dtype=torch.int8)

    def test_roundtrip(self):
        c = ZeroQConfig(compute_dtype=torch.bfloat16, prefetch_count=3)
        d = c.to_dict()
        assert d["compute_dtype"] == "torch.bfloat16"
        assert ZeroQConfig.from_dict(d) == c

    def test_from_reference_dict(self):
        ref = {"enabled": True, "quant_type": "nf4", "blocksize": 64, "double_quant": True,
               "compute_dtype": "torch.float32", "partition_trainable": False,
               "frozen_only": True, "async_gather": True, "prefetch_count": 1,
               "overlap_comm": True, "pin_memory": True, "contiguous_buffers": True,
               "target_modules": None, "exclude_modules": ["lm_head"]}
        assert ZeroQConfig.from_dict(ref).compute_dtype == torch.float32

    def test_presets(self):
        assert MAXWELL_CONFIG.compute_dtype == torch.float32
        assert TRAIN_FROM_SCRATCH_CONFIG.training_mode and TRAIN_FROM_SCRATCH_CONFIG.partition_trainable

    def test_train_config_defaults(self):
        c = ZeroQTrainConfig()
        assert c.training_mode and not c.frozen_only and c.optimizer_cls == "AdamW"
        assert c.lion_beta2 == 0.99 and not c.cpu_offload
        ZeroQTrainConfig(blocksize=48)  # validated only when compress_between_steps
        with pytest.raises(ValueError):
            ZeroQTrainConfig(blocksize=48, compress_between_steps=True)

    def test_multinode(self):
        m = MultiNodeConfig()
        assert m.node_id and m.coordinator_port == 5555
        assert MultiNodeConfig.from_dict(m.to_dict()) == m
        assert PHOENIX_CLUSTER_CONFIG.gradient_compression


@pytest.mark.parametrize("shape,world,weights", [((37, 129), 3, None), ((64, 64), 2, None),
                                                 ((50, 77), 4, [2.0, 2.0, 1.0, 1.0]),
                                                 ((8, 1000), 8, [2, 2, 1, 1, 1, 1, 1, 1])])
def test_local_range_quantisation_equals_full_then_slice(shape, world, weights):
    """Each rank quantises only the blocks covering its bytes; the shards are the
    slices of one full quantisation (uniform and weighted plans, ragged sizes)."""
    import zeroq_b200 as zq
    from zeroq_b200.ops.nf4 import quantize_4bit
    from zeroq_b200.parallel.coordinator import ZeroQParameter
    from zeroq_b200.parallel.hetero import HeteroZeroQParameter

    torch.manual_seed(0)
    w = torch.randn(*shape) * 0.02
    full_p, st = quantize_4bit(w.to(torch.float16), 64, "nf4")
    full_a = st.absmax.reshape(-1)
    cfg = zq.ZeroQConfig(exclude_modules=[])
    for rank in range(world):
        param = torch.nn.Parameter(w.clone(), requires_grad=False)
        if weights is None:
            p = ZeroQParameter(param=param, rank=rank, world_size=world, config=cfg, param_id=0)
        else:
            p = HeteroZeroQParameter(param=param, rank=rank, world_size=world, config=cfg,
                                     param_id=0, rank_weights=weights)
        p.partition_from_full_precision(w)
        p0, p1 = p.packed_plan.range_of(rank)
        a0, a1 = p.absmax_plan.range_of(rank)
        assert torch.equal(p.local_packed, full_p[p0:p1])
        assert torch.equal(p.local_absmax, full_a[a0:a1])
        assert p._quant_meta["shape"] == tuple(shape)

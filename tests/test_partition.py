"""Partition math, quantised partitioning and fp32 sharding (reference tests/test_partition.py,
tests/test_train_from_scratch.py:35-111)."""

import pytest
import torch

from zeroq_b200 import (PartitionInfo, compute_aligned_partition_sizes, estimate_memory_savings,
                        gather_and_dequantize, gather_fp32, partition_fp32,
                        partition_quantized_tensor, reduce_scatter_grads, repartition_tensor)
from zeroq_b200.ops.nf4 import dequantize_4bit_reference, quantize_4bit_reference


class TestAlignedSizes:
    def test_exact_division(self):
        assert compute_aligned_partition_sizes(4096, 4, 64) == (1024, 512, 16, 4096)

    def test_padding(self):
        e, p, a, t = compute_aligned_partition_sizes(4000, 4, 64)
        assert e * 4 >= 4000 and e % 64 == 0 and t == e * 4 and t >= 4000

    @pytest.mark.parametrize("bs", [64, 128, 256, 512])
    def test_blocksizes(self, bs):
        e, p, a, t = compute_aligned_partition_sizes(8192, 4, bs)
        assert e % bs == 0 and p == e // 2 and a == e // bs

    def test_single_gpu(self):
        e, _, _, _ = compute_aligned_partition_sizes(1000, 1, 64)
        assert e % 64 == 0 and e >= 1000

    def test_small_tensor(self):
        e, _, _, t = compute_aligned_partition_sizes(100, 4, 64)
        assert e >= 64 and t >= 100


class TestPartitionQuantized:
    @pytest.fixture
    def w(self):
        torch.manual_seed(42)
        return torch.randn(256, 256)

    def test_basic(self, w):
        p, a, st, info = partition_quantized_tensor(w, rank=0, world_size=4, blocksize=64)
        assert isinstance(info, PartitionInfo)
        assert info.original_shape == w.shape and info.world_size == 4
        assert p.numel() == info.packed_partition_size and a.numel() == info.absmax_partition_size

    def test_shards_concatenate_to_full_quantisation(self, w):
        full_p, full_a = quantize_4bit_reference(w, 64, "nf4")
        parts = [partition_quantized_tensor(w, r, 4, 64) for r in range(4)]
        assert torch.equal(torch.cat([x[0] for x in parts]), full_p)
        assert torch.equal(torch.cat([x[1] for x in parts]), full_a)

    def test_ranks_differ(self, w):
        p0 = partition_quantized_tensor(w, 0, 4)[0]
        p1 = partition_quantized_tensor(w, 1, 4)[0]
        assert not torch.equal(p0, p1)

    def test_invalid_rank(self, w):
        with pytest.raises(ValueError):
            partition_quantized_tensor(w, rank=4, world_size=4)

    @pytest.mark.parametrize("qt", ["nf4", "fp4"])
    def test_single_rank_roundtrip(self, qt):
        torch.manual_seed(0)
        w = torch.randn(512, 512) * 0.02
        p, a, st, info = partition_quantized_tensor(w, 0, 1, 64, qt)
        r = gather_and_dequantize(p, a, st, info)
        assert r.shape == w.shape
        rel = ((r - w).abs().mean() / w.abs().mean()).item()
        assert rel < 0.10 if qt == "nf4" else rel < 0.25
        assert (r - w).abs().max().item() < 1.0
        corr = torch.corrcoef(torch.stack([r.flatten(), w.flatten()]))[0, 1]
        assert corr > 0.98 if qt == "nf4" else corr > 0.95

    def test_repartition(self, w):
        p, a, st, info = partition_quantized_tensor(w, 1, 2)
        p2, a2, _ = repartition_tensor(w, info)
        assert torch.equal(p, p2) and torch.equal(a, a2)

    def test_partition_info_padding(self):
        _, _, _, info = partition_quantized_tensor(torch.randn(100), 0, 4)
        assert info.needs_padding and info.padding_elements == info.padded_numel - 100


def test_memory_estimate():
    est = estimate_memory_savings(32_000_000_000, 8)
    assert est["zeroq_per_gpu_bytes"] < est["zero3_per_gpu_bytes"]
    assert est["memory_reduction"] > 3.5


class TestFP32Shards:
    def test_roundtrip_single(self):
        t = torch.randn(37, 11)
        s, shp = partition_fp32(t, 1, 0)
        assert torch.equal(gather_fp32(s, shp, 1), t)

    def test_multi_rank_simulation(self):
        t = torch.randn(1001)
        shards = [partition_fp32(t, 4, r)[0] for r in range(4)]
        assert all(s.numel() == 251 for s in shards)
        assert torch.equal(torch.cat(shards)[:1001], t)
        assert torch.all(shards[-1][-3:] == 0)

    def test_dtype(self):
        s, _ = partition_fp32(torch.randn(10, dtype=torch.float16), 2, 0)
        assert s.dtype == torch.float32

    def test_reduce_scatter_single_rank(self):
        g = torch.randn(5, 7)
        out = reduce_scatter_grads(g, 1, 0)
        assert torch.equal(out, g.view(-1))

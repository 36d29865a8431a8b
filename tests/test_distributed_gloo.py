"""Multi-rank plumbing on CPU with the gloo backend (reference tests/test_coordinator.py,
tests/test_distributed_comm.py, tests/test_e2e_training.py - there NCCL on GPUs)."""

import os
import socket
import tempfile
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.distributed


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fn_name, errfile, env):
    os.environ.update(env)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        globals()[fn_name](rank, world)
        dist.barrier()
    except BaseException:
        with open(f"{errfile}.{rank}", "w") as f:
            f.write(traceback.format_exc())
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run(fn_name, world=2, env=None):
    port = _free_port()
    err = tempfile.mktemp()
    try:
        mp.spawn(_worker, args=(world, port, fn_name, err, env or {}), nprocs=world, join=True)
    except Exception:
        msgs = []
        for r in range(world):
            if os.path.exists(f"{err}.{r}"):
                msgs.append(open(f"{err}.{r}").read())
        raise AssertionError("\n".join(msgs) or "worker failed")


# ---------------------------------------------------------------------------- workers
def w_uniform_gather(rank, world):
    import zeroq_b200 as zq
    from tests.test_engine_cpu import _frozen_mlp

    m = _frozen_mlp(seed=0)
    ref = {n: p.detach().clone() for n, p in m.named_parameters()}
    coord = zq.ZeroQCoordinator(zq.ZeroQConfig(async_gather=False))
    zq.ZeroQModuleWrapper(m, coord).partition()
    for p in coord._params.values():
        assert p.packed_plan.lengths[rank] == p.local_packed.numel()
        p.start_gather(async_op=True)
        p.wait_gather()
        full = getattr(p.module, p.param_name).detach()
        # every rank reconstructs the identical tensor
        g = [torch.empty_like(full) for _ in range(world)]
        dist.all_gather(g, full)
        assert all(torch.equal(g[0], x) for x in g)
        r = ref[f"{p.module_path}.{p.param_name}"]
        assert ((full - r).abs().mean() / r.abs().mean()) < 0.15
        p.release()
    out = m(torch.ones(2, 64))
    g = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(g, out)
    assert torch.equal(g[0], g[1])


def w_hetero(rank, world):
    import zeroq_b200 as zq
    from tests.test_engine_cpu import _frozen_mlp

    m = _frozen_mlp(seed=1)
    x = torch.randn(3, 64, generator=torch.Generator().manual_seed(0))
    coord = zq.HeteroZeroQCoordinator(zq.ZeroQConfig())
    assert coord.rank_weights == [2.0, 1.0, 1.0][:world]
    wrap = zq.HeteroZeroQModuleWrapper(m, coord)
    wrap.partition()
    coord.verify_registration_consistency()
    p = coord._params[0]
    assert p.packed_plan.lengths[0] >= p.packed_plan.lengths[-1]
    out = m(x)
    g = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(g, out)
    assert torch.equal(g[0], g[-1])
    assert "All" in coord.debug_collective_seq()
    st = coord.get_memory_stats()
    assert st["rank_weight"] == coord.rank_weights[rank]


def w_registration_mismatch(rank, world):
    import torch.nn as nn
    import zeroq_b200 as zq

    m = nn.Sequential(nn.Linear(8, 8), nn.Linear(8, 8 if rank == 0 else 16))
    for p in m.parameters():
        p.requires_grad_(False)
    coord = zq.HeteroZeroQCoordinator(zq.ZeroQConfig(exclude_modules=[]), rank_weights=[1.0] * world)
    zq.HeteroZeroQModuleWrapper(m, coord)
    with pytest.raises(RuntimeError, match="Registration order mismatch"):
        coord.verify_registration_consistency()


def w_collective_seq_divergence(rank, world):
    import zeroq_b200 as zq

    coord = zq.HeteroZeroQCoordinator(zq.ZeroQConfig(), rank_weights=[1.0] * world)
    coord._collective_seq = 5 if rank == 0 else 3
    msg = coord.debug_collective_seq()
    assert "MISMATCH" in msg and "BEHIND" in msg


def w_varlen(rank, world):
    import zeroq_b200 as zq
    from zeroq_b200.parallel.varlen import all_gather_by_plan

    local = torch.arange(rank * 10, rank * 10 + rank + 1, dtype=torch.float32)
    lengths, cat = zq.all_gather_varlen_1d(local)
    assert lengths == [r + 1 for r in range(world)]
    assert cat.tolist() == [float(r * 10 + i) for r in range(world) for i in range(r + 1)]
    plan = zq.make_plan(17, [2.0] + [1.0] * (world - 1))
    full = torch.arange(17, dtype=torch.float32)
    o, l = plan.range_of(rank)
    out = all_gather_by_plan(full[o:l].clone(), plan)
    assert torch.equal(out, full)


def w_reduce_scatter(rank, world):
    import zeroq_b200 as zq

    g = torch.arange(10, dtype=torch.float32) * (rank + 1)
    shard = zq.reduce_scatter_grads(g, world, rank)
    chunk = (10 + world - 1) // world
    full = torch.arange(chunk * world, dtype=torch.float32)
    full[10:] = 0
    mean = full * sum(r + 1 for r in range(world)) / world
    assert torch.allclose(shard, mean[rank * chunk:(rank + 1) * chunk])


def w_sharded_adamw(rank, world):
    import zeroq_b200 as zq
    import torch.distributed as dist

    # replicas initialised from different random states start from rank 0's values
    torch.manual_seed(100 + rank)
    own = [torch.nn.Parameter(torch.randn(6, 4)), torch.nn.Parameter(torch.randn(3))]
    zq.ShardedAdamW(own, lr=1e-2)
    for p in own:
        ref = p.detach().clone()
        dist.broadcast(ref, src=0)
        assert torch.equal(p.detach(), ref)

    for clip in (None, 0.5):  # with clipping: the averaged gradient's global norm
        torch.manual_seed(0)
        ps = [torch.nn.Parameter(torch.randn(7, 3)), torch.nn.Parameter(torch.randn(5))]
        ref = [torch.nn.Parameter(p.detach().clone()) for p in ps]
        opt = zq.ShardedAdamW(ps, lr=1e-2, weight_decay=0.1, max_grad_norm=clip)
        ref_opt = torch.optim.AdamW(ref, lr=1e-2, weight_decay=0.1)
        for step in range(3):
            gens = [torch.Generator().manual_seed(100 * step + r) for r in range(world)]
            grads = [[torch.randn(p.shape, generator=gens[r]) for p in ps] for r in range(world)]
            for p, g in zip(ps, grads[rank]):
                p.grad.copy_(g)
            opt.step()
            opt.zero_grad()
            for i, p in enumerate(ref):
                p.grad = sum(grads[r][i] for r in range(world)) / world
            if clip is not None:
                norm = torch.nn.utils.clip_grad_norm_(ref, clip)
                assert abs(opt.grad_norm() - float(norm)) < 1e-4 * float(norm)
            ref_opt.step()
        for p, r in zip(ps, ref):
            assert torch.allclose(p.detach(), r.detach(), atol=1e-5), (clip, p, r)


def w_tiny_decoder_training(rank, world):
    """The tiny-decoder plumbing workload: NF4 shards in gather/release mode, 20 AdamW steps."""
    import zeroq_b200 as zq
    from zeroq_b200.models import DecoderLM, get_config

    cfg = get_config("tiny")  # vocab 1024, d 256, 4 layers, 4 heads of 64, SwiGLU 688
    model = DecoderLM(cfg).init_dense_(std=0.02, seed=0)
    for n, p in model.named_parameters():
        p.requires_grad_("embed" not in n and ("norm" in n))
    coord = zq.ZeroQCoordinator(zq.ZeroQConfig(exclude_modules=["embed_tokens", "lm_head"],
                                               prefetch_count=1))
    wrap = zq.ZeroQModuleWrapper(model, coord)
    wrap.partition()
    # projections are trainable only through LoRA-free norms here; train the norms
    opt = zq.ShardedAdamW([p for p in model.parameters() if p.requires_grad], lr=1e-2)
    g = torch.Generator().manual_seed(rank)
    losses = []
    for step in range(20):
        ids = torch.randint(0, cfg.vocab_size, (4, 129), generator=torch.Generator().manual_seed(step))
        loss = model(ids[:, :-1], ids[:, 1:])
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(loss.item())
    t = torch.tensor(losses)
    all_l = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(all_l, t)
    assert all(torch.allclose(all_l[0], x) for x in all_l)  # ranks agree
    assert losses[-1] < losses[0]
    assert wrap._prefetcher is not None and len(wrap._prefetcher.order) > 0


def w_prefetch_manager(rank, world):
    import zeroq_b200 as zq
    from zeroq_b200.models import DecoderLM, get_config

    model = DecoderLM(get_config("tiny", n_layers=2)).init_dense_(seed=0)
    for p in model.parameters():
        p.requires_grad_(False)
    lw = zq.LayerWiseZeroQ(model, zq.ZeroQConfig(), layer_attr="layers")
    lw.partition()
    lw.prefetch.prefetch_for_layer(0)
    assert lw.prefetch.get_stats()["inflight_layers"] == 1
    lw.prefetch.wait_for_layer(0)
    q = model.layers[0].q_proj.weight
    assert q.numel() == 256 * 256
    lw.prefetch.release_layer(0)
    assert model.layers[0].q_proj.weight.numel() == 0


def w_train_mode_rs(rank, world):
    import zeroq_b200 as zq
    from tests.test_engine_cpu import TinyMLP

    torch.manual_seed(0)
    m = TinyMLP()
    coord = zq.ZeroQCoordinator(zq.ZeroQTrainConfig(exclude_modules=[]))
    zq.ZeroQModuleWrapper(m, coord).partition()
    masters = coord.trainable_master_params()
    opt = torch.optim.SGD(masters, lr=0.1)
    x = torch.randn(4, 64, generator=torch.Generator().manual_seed(rank))
    m(x).pow(2).mean().backward()
    assert all(p.grad is not None for p in masters)
    # the reduce-scatters started in the gradient hooks were finished at the end of
    # the backward: each master shard holds its slice of the rank-averaged gradient
    torch.manual_seed(0)
    ref = TinyMLP()          # the same initial weights, not sharded
    ref(x).pow(2).mean().backward()
    refp = dict(ref.named_parameters())
    checked = 0
    for zq_ in coord._params.values():
        if getattr(zq_, "master_shard", None) is None or zq_.master_shard.grad is None:
            continue
        checked += 1
        full = refp[f"{zq_.module_path}.{zq_.param_name}"].grad.detach().reshape(-1).clone()
        dist.all_reduce(full)
        full /= world
        n = zq_.master_shard.numel()
        want = torch.nn.functional.pad(full, (0, n * world - full.numel()))[rank * n:(rank + 1) * n]
        torch.testing.assert_close(zq_.master_shard.grad, want.to(zq_.master_shard.dtype),
                                   rtol=1e-5, atol=1e-6)
    assert checked > 0
    opt.step()
    st = coord.gather_full_state_dict()
    if rank == 0:
        assert "fc1.weight" in st


# ---------------------------------------------------------------------------- tests
def test_uniform_gather_2ranks():
    run("w_uniform_gather", 2)


def test_hetero_3ranks():
    run("w_hetero", 3, env={"ZEROQ_HETERO_RANK_WEIGHTS": "2,1,1"})


def test_registration_mismatch_raises():
    run("w_registration_mismatch", 2)


def test_collective_seq_divergence_reported():
    run("w_collective_seq_divergence", 2)


def test_varlen_collectives():
    run("w_varlen", 3)


def test_reduce_scatter_grads():
    run("w_reduce_scatter", 3)


def test_sharded_adamw_matches_torch_adamw():
    run("w_sharded_adamw", 2)


def test_tiny_decoder_gather_release_training():
    run("w_tiny_decoder_training", 2)


def test_prefetch_manager():
    run("w_prefetch_manager", 2)


def test_train_mode_reduce_scatter():
    run("w_train_mode_rs", 2)

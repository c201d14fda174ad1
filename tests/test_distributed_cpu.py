"""Multi-process tests on CPU with the gloo backend (world size 2)."""
import os
import socket
import sys
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(fn, world=2, *args):
    port = _port()
    mp.spawn(_entry, args=(world, port, fn, args), nprocs=world, join=True)


def _entry(rank, world, port, fn, args):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


# ---------------------------------------------------------------- FSDP trainer
def _train_llama_fsdp(rank, world, out_dir):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    cfg = ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel_cpu",
                                      "--training.steps", "4", "--checkpoint.enable", "--checkpoint.interval", "2",
                                      "--dump-folder", out_dir, "--checkpoint.keep-latest-k", "5",
                                      "--validator.enable", "--validator.freq", "4", "--validator.steps", "1"])
    t = Trainer(cfg)
    t.train()
    losses = t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]
    assert 5.0 < losses < 9.0
    t.close()
    # resume from the step-4 checkpoint into a fresh trainer
    cfg2 = ConfigManager().parse_args(["--module", "llama3", "--config", "llama3_debugmodel_cpu",
                                       "--training.steps", "5", "--checkpoint.enable", "--checkpoint.interval", "10",
                                       "--dump-folder", out_dir])
    t2 = Trainer(cfg2)
    t2.checkpointer.load()
    assert t2.step == 4 and t2.ntokens_seen == t.ntokens_seen
    assert t2.dataloader.batches_emitted == t.dataloader.batches_emitted
    t2.close()


def test_fsdp_gloo_training_and_resume():
    with tempfile.TemporaryDirectory() as d:
        _run(_train_llama_fsdp, 2, d)
        assert os.path.exists(os.path.join(d, "checkpoint", "step-4", ".metadata"))


# ---------------------------------------------------------------- peer data parallel (host logic)
def _train_peer_vs_fsdp(rank, world, out_dir):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def make(comm, steps, extra=()):
        return Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", str(steps),
            "--metrics.log-freq", "1", "--parallelism.data-parallel-comm", comm, "--dump-folder",
            os.path.join(out_dir, comm), "--training.global-batch-size", "8", *extra]))

    tf = make("fsdp2", 3)
    tp = make("peer", 3, ("--checkpoint.enable", "--checkpoint.interval", "3"))
    rt = tp.model_parts[0]._dp_runtime
    assert rt.comm == "collective"
    # identical starting weights: FSDP2's full state loaded through the checkpoint wrapper
    full = get_model_state_dict(tf.model_parts[0], options=StateDictOptions(full_state_dict=True))
    tp.checkpointer.states["model"].load_state_dict(full)
    for t in (tf, tp):
        t.train()
    mf, mp_ = (t.metrics_processor.last_metrics for t in (tf, tp))
    lf, lp = mf["loss_metrics/global_avg_loss"], mp_["loss_metrics/global_avg_loss"]
    gf, gp = mf["grad_norm"], mp_["grad_norm"]
    assert abs(lf - lp) < 1e-4 * max(1.0, abs(lf)), (lf, lp)
    assert abs(gf - gp) < 1e-3 * max(1.0, abs(gf)), (gf, gp)
    # the updated weights equal FSDP2's, and every rank holds the same copy
    full = get_model_state_dict(tf.model_parts[0], options=StateDictOptions(full_state_dict=True))
    for n, p in tp.model_parts[0].named_parameters():
        n = n.replace("_checkpoint_wrapped_module.", "")
        torch.testing.assert_close(p.detach(), full[n], rtol=1e-4, atol=1e-5)
    w = rt.wbuf.clone()
    ws = [torch.empty_like(w) for _ in range(world)]
    dist.all_gather(ws, w)
    assert torch.equal(ws[0], ws[1])
    tf.close()
    tp.close()
    # resume: masters, moments and step count come back and the weights are rebuilt from them
    t2 = make("peer", 4, ("--checkpoint.enable",))
    rt2 = t2.model_parts[0]._dp_runtime
    master_before = rt2.master.clone()
    t2.checkpointer.load()
    assert t2.step == 3 and t2.optimizers.optimizers[0].step_count == 3
    assert torch.equal(rt2.master, rt.master) and not torch.equal(rt2.master, master_before)
    assert torch.equal(rt2.wbuf, w)
    torch.testing.assert_close(t2.optimizers.optimizers[0].exp_avg, tp.optimizers.optimizers[0].exp_avg)
    t2.close()


def test_peer_data_parallel_matches_fsdp2_and_resumes():
    with tempfile.TemporaryDirectory() as d:
        _run(_train_peer_vs_fsdp, 2, d)


# ---------------------------------------------------------------- Ulysses a2a
def _ulysses(rank, world):
    from torchtitan_b200.ops import reference as R
    from torchtitan_b200.parallel.context_parallel import head_to_seq, seq_to_head, ulysses_hook

    torch.manual_seed(0)
    B, S, H, D = 1, 8, 4, 4
    q, k, v = (torch.randn(B, S, H, D) for _ in range(3))
    full = R.attention(q, k, v, True)
    sl = slice(rank * S // world, (rank + 1) * S // world)
    x = q[:, sl].contiguous()
    assert torch.equal(head_to_seq(seq_to_head(x, dist.group.WORLD), dist.group.WORLD), x)
    hook = ulysses_hook(dist.group.WORLD)
    o = hook(lambda a, b, c, m: R.attention(a, b, c, True), q[:, sl].contiguous(), k[:, sl].contiguous(),
             v[:, sl].contiguous(), None)
    assert torch.allclose(o, full[:, sl], atol=1e-5)


def test_ulysses_all_to_all_matches_full_attention():
    _run(_ulysses, 2)


# ---------------------------------------------------------------- expert parallel
def _ep(rank, world):
    from torchtitan_b200.models.common.moe import MoE
    from torchtitan_b200.parallel.expert_parallel import make_ep_dispatch

    torch.manual_seed(0)
    m = MoE(8, 16, num_experts=4, top_k=2)
    m.init_weights(0.1)
    for p in m.parameters():
        dist.broadcast(p.data, 0)
    x = torch.randn(1, 6, 8) + rank
    ref = m(x)
    # shard experts: this rank keeps experts [2r, 2r+2)
    e = m.experts
    full = [p.data.clone() for p in (e.w1, e.w2, e.w3)]
    for name, f in zip(("w1", "w2", "w3"), full):
        setattr(e, name, torch.nn.Parameter(f[rank * 2:(rank + 1) * 2].clone()))
    m.ep_dispatch = make_ep_dispatch(dist.group.WORLD, 4)
    xr = x.clone().requires_grad_()
    out = m(xr)
    assert torch.allclose(out, ref, atol=1e-5)
    out.sum().backward()
    assert xr.grad is not None and e.w1.grad.shape[0] == 2


def test_expert_parallel_dispatch_matches_local():
    _run(_ep, 2)


# ---------------------------------------------------------------- DistMuon
def _distmuon(rank, world):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    from torchtitan_b200.components.optimizer import Muon

    mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("fsdp",))
    torch.manual_seed(0)
    # several matrices (uneven row splits, equal shapes batched together) and a 3-D expert stack
    shapes = [(8, 6), (7, 12), (8, 6), (5, 3, 4), (16, 16), (3, 10)]
    ws = [torch.randn(s) for s in shapes]
    gs = [torch.randn(s) for s in shapes]
    refs = [torch.nn.Parameter(w.clone()) for w in ws]
    for p, g in zip(refs, gs):
        p.grad = g.clone()
    opt_ref = Muon([{"params": refs, "use_muon": True}], lr=0.02)
    ps = [torch.nn.Parameter(distribute_tensor(w.clone(), mesh, [Shard(0)])) for w in ws]
    opt = Muon([{"params": ps, "use_muon": True}], lr=0.02, distributed=True)
    for _ in range(2):  # two steps: momentum buffers carry over
        for p, g in zip(ps, gs):
            p.grad = distribute_tensor(g.clone(), mesh, [Shard(0)])
        for p, g in zip(refs, gs):
            p.grad = g.clone()
        opt_ref.step()
        opt.step()
    for p, r in zip(ps, refs):
        assert torch.allclose(p.full_tensor(), r.detach(), atol=1e-5), (p.shape,)


@pytest.mark.parametrize("world", [2, 3])
def test_distmuon_matches_muon(world):
    _run(_distmuon, world)


# ---------------------------------------------------------------- failure detection
def _rank_dies(rank, world):
    import datetime

    t = torch.ones(1)
    dist.all_reduce(t)
    if rank == 1:
        os._exit(0)  # leaves between steps, no collective in flight
    pg = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=3))
    with pytest.raises(Exception):
        dist.all_reduce(t, group=pg)


def test_peer_exit_surfaces_as_error_not_hang():
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_entry, args=(r, 2, port, _rank_dies, ())) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    assert all(not p.is_alive() for p in procs)


# ---------------------------------------------------------------- semi-synchronous replicas
def _semi_sync(rank, world, out_dir):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def make(method, extra=()):
        return Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "4",
            "--training.seq-len", "128", "--parallelism.data-parallel-replicate-degree", "2",
            "--parallelism.data-parallel-shard-degree", "1", "--fault-tolerance.enable",
            "--fault-tolerance.semi-sync-method", method, "--fault-tolerance.sync-steps", "2",
            "--dump-folder", os.path.join(out_dir, method), *extra]))

    def gathered(t):
        w = torch.cat([p.detach().to_local().reshape(-1) if hasattr(p, "to_local") else p.detach().reshape(-1)
                       for p in t.model_parts[0].parameters()])
        ws = [torch.empty_like(w) for _ in range(world)]
        dist.all_gather(ws, w)
        return ws

    t = make("local_sgd")
    for step in range(1, 4):
        t.step = step
        t.train_step(t.batch_generator(t.dataloader))
        ws = gathered(t)
        # replicas see different data: they agree only right after a synchronisation (steps 2, 4, ...)
        assert torch.equal(ws[0], ws[1]) == (step % 2 == 0), step
    t.close()
    # DiLoCo with outer lr 1 and no momentum is exactly weight averaging
    t = make("diloco", ("--fault-tolerance.outer-lr", "1.0", "--fault-tolerance.outer-momentum", "0.0"))
    it = t.batch_generator(t.dataloader)
    for step in range(1, 3):
        t.step = step
        t.train_step(it)
    ws = gathered(t)
    torch.testing.assert_close(ws[0], ws[1])
    t.close()


def test_semi_sync_local_sgd_and_diloco():
    with tempfile.TemporaryDirectory() as d:
        _run(_semi_sync, 2, d)


def test_semi_sync_fragment_schedule():
    from torchtitan_b200.parallel.semi_sync import FaultToleranceConfig, SemiSync

    s = SemiSync.__new__(SemiSync)
    s.cfg = FaultToleranceConfig(enable=True, semi_sync_method="diloco", sync_steps=8, num_fragments=4)
    s.offsets = [0, 2, 4, 6]
    assert [s.due(k) for k in range(1, 17)] == [[], [], [], [], [], [], [], [0], [], [1], [], [2], [], [3], [],
                                                 [0]]


# ---------------------------------------------------------------- async TP collective matmuls
def _async_tp(rank, world):
    from torchtitan_b200.parallel import async_tp
    from torchtitan_b200.parallel.tensor_parallel import all_gather_seq, reduce_scatter_seq

    g = dist.group.WORLD
    torch.manual_seed(0)
    B, S, K, N = 2, 8 * world, 16, 12
    x_full = torch.randn(B, S, K, dtype=torch.float64)
    w_col = torch.randn(N, K, dtype=torch.float64)  # this rank's column shard (same on all ranks here)
    s = S // world
    x = x_full[:, rank * s:(rank + 1) * s].clone().requires_grad_()
    w1 = w_col.clone().requires_grad_()
    y = async_tp.ag_matmul(x, w1, g)
    x_ref = x.detach().clone().requires_grad_()
    w_ref = w_col.clone().requires_grad_()
    y_ref = all_gather_seq(x_ref, g) @ w_ref.t()
    torch.testing.assert_close(y, y_ref)
    gy = torch.randn_like(y)
    y.backward(gy)
    y_ref.backward(gy)
    torch.testing.assert_close(x.grad, x_ref.grad)
    torch.testing.assert_close(w1.grad, w_ref.grad)
    # row-parallel: each rank holds a different K shard of the input features
    xr = torch.randn(B, S, K, dtype=torch.float64, generator=torch.Generator().manual_seed(rank + 1))
    wr = torch.randn(N, K, dtype=torch.float64, generator=torch.Generator().manual_seed(rank + 7))
    a, b = xr.clone().requires_grad_(), wr.clone().requires_grad_()
    out = async_tp.matmul_rs(a, b, g)
    a2, b2 = xr.clone().requires_grad_(), wr.clone().requires_grad_()
    ref = reduce_scatter_seq(a2 @ b2.t(), g)
    torch.testing.assert_close(out, ref)
    go = torch.randn_like(out)
    out.backward(go)
    ref.backward(go)
    torch.testing.assert_close(a.grad, a2.grad)
    torch.testing.assert_close(b.grad, b2.grad)


@pytest.mark.parametrize("world", [2, 3])
def test_async_tp_ring_matmuls_match_collectives(world):
    _run(_async_tp, world)


def _tp_async_trainer(rank, world, out_dir):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    res = []
    for extra in ([], ["--parallelism.enable-async-tensor-parallel"]):
        t = Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "2",
            "--training.seq-len", "128", "--parallelism.tensor-parallel-degree", "2",
            "--parallelism.data-parallel-shard-degree", "1", "--metrics.log-freq", "1",
            "--debug.seed", "0", "--dump-folder", os.path.join(out_dir, str(len(extra))), *extra]))
        t.train()
        res.append(t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"])
        t.close()
    from torchtitan_b200.parallel import async_tp

    async_tp.ENABLED = False
    assert abs(res[0] - res[1]) < 1e-5 * abs(res[0]), res


def test_async_tp_trainer_matches_sync_tp():
    with tempfile.TemporaryDirectory() as d:
        _run(_tp_async_trainer, 2, d)


# ---------------------------------------------------------------- pipeline parallel
def _pp(rank, world, out_dir, module, config):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", module, "--config", config, "--training.steps", "2", "--training.seq-len", "64",
        "--parallelism.pipeline-parallel-degree", "2", "--parallelism.data-parallel-shard-degree", "1",
        "--parallelism.pipeline-parallel-microbatch-size", "2", "--training.local-batch-size", "4",
        "--parallelism.pipeline-parallel-schedule", "Interleaved1F1B", "--training.dtype", "float32",
        "--training.mixed-precision-param", "float32", "--dump-folder", out_dir]))
    t.train()
    loss = t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]
    assert t.pp_has_last_stage == (rank == 1)
    if rank == 1:
        assert 6.0 < loss < 9.0
    t.close()


@pytest.mark.parametrize("module,config", [("llama3", "llama3_debugmodel_cpu"),
                                           ("kimi_linear", "kimi_linear_debugmodel_block_attn_res")])
def test_pipeline_parallel_interleaved_1f1b(module, config):
    with tempfile.TemporaryDirectory() as d:
        _run(_pp, 2, d, module, config)


# ---------------------------------------------------------------- fused (peer-memory layout) EP
def _ep_fused(rank, world):
    from torchtitan_b200.models.common.moe import MoE
    from torchtitan_b200.parallel.ep_fused import make_fused_ep_dispatch

    torch.manual_seed(0)
    E = 2 * world
    m = MoE(8, 16, num_experts=E, top_k=2, load_balance_coeff=None)
    m.init_weights(0.1)
    for p in m.parameters():
        dist.broadcast(p.data, 0)
    x = (torch.randn(1, 40 + 7 * rank, 8, generator=torch.Generator().manual_seed(rank)) + rank).requires_grad_()
    ref = m(x)
    ref.square().sum().backward()
    gx_ref = x.grad.clone()
    e = m.experts
    gw_ref = []
    for w in (e.w1, e.w2, e.w3):
        g = w.grad.clone()
        dist.all_reduce(g)  # the local reference saw only this rank's tokens
        gw_ref.append(g[rank * 2:(rank + 1) * 2])
    full = [p.data.clone() for p in (e.w1, e.w2, e.w3)]
    for name, f in zip(("w1", "w2", "w3"), full):
        setattr(e, name, torch.nn.Parameter(f[rank * 2:(rank + 1) * 2].clone()))
    m.zero_grad()
    m.ep_dispatch = make_fused_ep_dispatch(dist.group.WORLD, E)
    assert m.ep_dispatch.comm.comm is None
    xr = x.detach().clone().requires_grad_()
    out = m(xr)
    assert m.ep_dispatch.comm.comm == "collective"
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    out.square().sum().backward()
    torch.testing.assert_close(xr.grad, gx_ref, rtol=1e-5, atol=1e-5)
    # expert weight gradients are summed over every rank's routed rows
    for g, w in zip(gw_ref, (e.w1, e.w2, e.w3)):
        torch.testing.assert_close(w.grad, g, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("world", [2, 3])
def test_fused_expert_parallel_matches_local(world):
    _run(_ep_fused, world)


def test_fused_ep_plan_layout():
    from torchtitan_b200.parallel.ep_fused import Plan

    M = torch.tensor([[3, 0, 5, 1], [2, 130, 0, 4]])  # 2 ranks x 4 experts (2 per rank)
    p0, p1 = Plan(M, 0, torch.device("cpu")).finalize(M), Plan(M, 1, torch.device("cpu")).finalize(M)
    # owner 0: expert 0 gets 3 + 2 rows -> [0, 128); expert 1 gets 130 -> [128, 384)
    assert p0.P == 384 and p1.P == 256 and p0.P_max == 384
    assert p0.local_counts.tolist() == [5, 130]
    # rank 0's rows: expert 0 -> owner 0 rows 0..2; expert 2 -> owner 1 rows 0..4; expert 3 -> owner 1 row 128
    assert p0.dest_rank.tolist() == [0, 0, 0, 1, 1, 1, 1, 1, 1]
    assert p0.dest_row.tolist() == [0, 1, 2, 0, 1, 2, 3, 4, 128]
    # rank 1's rows for expert 0 follow rank 0's; expert 1 starts at 128; expert 3 after rank 0's row
    assert p1.dest_row[:3].tolist() == [3, 4, 128] and p1.dest_row[-4:].tolist() == [129, 130, 131, 132]
    assert p0.pad_rows.numel() == 384 - 135 and p1.real_rows.numel() == 10


def _ep_trainer(rank, world, out_dir):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    res = []
    for backend in ("standard", "fused"):
        t = Trainer(ConfigManager().parse_args([
            "--module", "qwen3", "--config", "qwen3_debugmodel_moe", "--training.steps", "2",
            "--training.seq-len", "64", "--training.local-batch-size", "2", "--training.dtype", "float32",
            "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "none",
            "--parallelism.expert-parallel-degree", "2", "--parallelism.expert-parallel-comm-backend", backend,
            "--debug.seed", "0", "--metrics.log-freq", "1", "--dump-folder", os.path.join(out_dir, backend)]))
        t.train()
        res.append(t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"])
        t.close()
    assert abs(res[0] - res[1]) < 1e-5 * abs(res[0]), res


def test_fused_ep_trainer_matches_standard():
    with tempfile.TemporaryDirectory() as d:
        _run(_ep_trainer, 2, d)


# ---------------------------------------------------------------- Kimi-Linear tensor parallel
def _kimi_tp(rank, world, out_dir):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.models.kimi_linear import model_registry
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "kimi_linear", "--config", "kimi_linear_debugmodel", "--training.steps", "1",
        "--training.seq-len", "64", "--training.local-batch-size", "2", "--training.dtype", "float32",
        "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "none",
        "--parallelism.tensor-parallel-degree", "2", "--parallelism.data-parallel-shard-degree", "1",
        "--debug.seed", "0", "--dump-folder", out_dir]))
    model = t.model_parts[0]
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    ref = model_registry("debugmodel").model.build()
    ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in full.items()}, strict=False)
    tokens = torch.randint(0, 2048, (2, 64), generator=torch.Generator().manual_seed(3))
    labels = tokens.roll(-1, 1)
    loss_ref = cross_entropy_loss(ref(tokens), labels)
    loss_ref.backward()
    loss_tp = t._loss(model(tokens), labels)
    torch.testing.assert_close(loss_tp, loss_ref, rtol=1e-5, atol=1e-4)
    loss_tp.backward()
    named = dict(ref.named_parameters())
    for n, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
        r = named[n.replace("_checkpoint_wrapped_module.", "")].grad
        # fp32 summation-order noise only: relative to the gradient's scale
        assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-7, n
    t.close()


def test_kimi_tensor_parallel_matches_single_device():
    with tempfile.TemporaryDirectory() as d:
        _run(_kimi_tp, 2, d)


def _llama_tp_grads(rank, world, out_dir, sp, module="llama3", config="llama3_debugmodel_cpu", extra=()):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", module, "--config", config, "--training.steps", "1",
        "--training.seq-len", "64", "--parallelism.tensor-parallel-degree", "2",
        "--parallelism.data-parallel-shard-degree", "1", "--debug.seed", "0", "--dump-folder", out_dir,
        "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
        "--activation-checkpoint.mode", "none", *([] if sp else ["--parallelism.no-enable-sequence-parallel"]),
        *extra]))
    model = t.model_parts[0]
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    import importlib

    ref = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(
        t.config.model_spec.flavor).model.build()
    ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in full.items()}, strict=False)
    ref.rope.init_weights()
    tokens = torch.randint(0, 2048, (2, 64), generator=torch.Generator().manual_seed(3))
    labels = tokens.roll(-1, 1)
    cross_entropy_loss(ref(tokens), labels).backward()
    loss_tp = t._loss(model(tokens), labels)
    loss_tp.backward()
    named = dict(ref.named_parameters())
    for n, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
        r = named[n.replace("_checkpoint_wrapped_module.", "")].grad
        assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-7, (n, sp)
    t.close()


@pytest.mark.parametrize("sp", [True, False])
@pytest.mark.parametrize("module,config", [("llama3", "llama3_debugmodel_cpu"), ("qwen3", "qwen3_debugmodel"),
                                           ("qwen3", "qwen3_debugmodel_moe"), ("llama4", "llama4_debugmodel"),
                                           ("deepseek_v3", "deepseek_v3_debugmodel"),
                                           ("deepseek_v3", "deepseek_v3_debugmodel_qlora"),
                                           ("gpt_oss", "gpt_oss_debugmodel")])
def test_tensor_parallel_gradients(sp, module, config):
    with tempfile.TemporaryDirectory() as d:
        _run(_llama_tp_grads, 2, d, sp, module, config)


@pytest.mark.parametrize("sp", [True, False])
@pytest.mark.parametrize("module,config", [("qwen3", "qwen3_debugmodel_moe"), ("deepseek_v3", "deepseek_v3_debugmodel"),
                                           ("gpt_oss", "gpt_oss_debugmodel")])
def test_expert_tensor_parallel_gradients(sp, module, config):
    with tempfile.TemporaryDirectory() as d:
        _run(_llama_tp_grads, 2, d, sp, module, config, ("--parallelism.expert-tensor-parallel-degree", "2"))


# ---------------------------------------------------------------- context parallel, gradient-exact
def _cp_grads(rank, world, out_dir, module, config, method):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer
    import importlib

    t = Trainer(ConfigManager().parse_args([
        "--module", module, "--config", config, "--training.steps", "1", "--training.seq-len", "64",
        "--training.local-batch-size", "2", "--training.dtype", "float32",
        "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "none",
        "--parallelism.context-parallel-degree", "2", "--parallelism.context-parallel-method", method,
        "--parallelism.data-parallel-shard-degree", "1", "--debug.seed", "0", "--dump-folder", out_dir]))
    model = t.model_parts[0]
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry("debugmodel")
    ref = spec.model.build()
    ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in full.items()}, strict=False)
    if hasattr(ref, "rope"):
        ref.rope.init_weights()
    tokens = torch.randint(0, spec.model.vocab_size, (2, 64), generator=torch.Generator().manual_seed(3))
    labels = tokens.roll(-1, 1)
    loss_ref = cross_entropy_loss(ref(tokens), labels)
    loss_ref.backward()
    inp, lab, _, kw = t.post_dataloading_process({"input": tokens}, labels)
    loss_local = t._loss(model(inp, **kw), lab)
    total = loss_local.detach().clone()
    dist.all_reduce(total)
    torch.testing.assert_close(total, loss_ref, rtol=1e-5, atol=1e-4)
    loss_local.backward()
    named = dict(ref.named_parameters())
    for n, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad.clone()
        # FSDP on gloo averaged the shards' gradients over the cp ranks (the trainer scales the
        # loss by that degree to compensate); summing the average over ranks gives the full gradient
        dist.all_reduce(g)
        r = named[n.replace("_checkpoint_wrapped_module.", "")].grad
        assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-7, (n, method)
    t.close()


@pytest.mark.parametrize("module,config,method", [("llama3", "llama3_debugmodel_cpu", "ring"),
                                                  ("llama3", "llama3_debugmodel_cpu", "ulysses"),
                                                  ("kimi_linear", "kimi_linear_debugmodel", "ulysses")])
def test_context_parallel_gradients_match_single_device(module, config, method):
    with tempfile.TemporaryDirectory() as d:
        _run(_cp_grads, 2, d, module, config, method)


def _pp_grads(rank, world, out_dir, schedule, module="llama3", config="llama3_debugmodel_cpu"):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer
    import importlib

    model_registry = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry
    t = Trainer(ConfigManager().parse_args([
        "--module", module, "--config", config, "--training.steps", "1",
        "--training.seq-len", "64", "--parallelism.pipeline-parallel-degree", "2",
        "--parallelism.data-parallel-shard-degree", "1", "--parallelism.pipeline-parallel-microbatch-size", "1",
        "--training.local-batch-size", "4", "--parallelism.pipeline-parallel-schedule", schedule,
        "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
        "--debug.seed", "0", "--dump-folder", out_dir]))
    full = {}
    for part in t.model_parts:
        full.update(get_model_state_dict(part, options=StateDictOptions(full_state_dict=True)))
    gathered = [None] * world
    dist.all_gather_object(gathered, {k: v for k, v in full.items()})
    merged = {}
    for d in gathered:
        merged.update(d)
    ref = model_registry(t.config.model_spec.flavor).model.build()
    res = ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in merged.items()},
                              strict=False)
    assert not res.unexpected_keys and all("tokens_per_expert" in k for k in res.missing_keys), res
    if hasattr(ref, "rope"):
        ref.rope.init_weights()
    tokens = torch.randint(0, ref.model_args.vocab_size if hasattr(ref.model_args, "vocab_size") else 2048,
                           (4, 64), generator=torch.Generator().manual_seed(3))
    labels = tokens.roll(-1, 1)
    loss_ref = cross_entropy_loss(ref(tokens), labels) / labels.numel()
    loss_ref.backward()
    loss = t.forward_backward_step(input_dict={"input": tokens}, labels=labels,
                                   global_valid_tokens=torch.tensor(float(labels.numel())))
    if t.pp_has_last_stage:
        torch.testing.assert_close(loss.reshape(()), loss_ref, rtol=1e-5, atol=1e-5)
    named = dict(ref.named_parameters())
    for part in t.model_parts:
        for n, p in part.named_parameters():
            g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
            r = named[n.replace("_checkpoint_wrapped_module.", "")].grad
            assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-8, (n, schedule)
    t.close()


@pytest.mark.parametrize("schedule", ["1F1B", "Interleaved1F1B", "GPipe"])
def test_pipeline_parallel_gradients_match_single_device(schedule):
    with tempfile.TemporaryDirectory() as d:
        _run(_pp_grads, 2, d, schedule)


@pytest.mark.parametrize("module,config", [("kimi_linear", "kimi_linear_debugmodel_block_attn_res"),
                                           ("attention_residual", "attention_residual_debugmodel")])
def test_pipeline_parallel_attn_res_gradients_match_single_device(module, config):
    """Attention-Residual models hand their whole residual state (completed blocks + the
    partial block) from stage to stage, so the pipelined model is the unpipelined one."""
    with tempfile.TemporaryDirectory() as d:
        _run(_pp_grads, 2, d, "Interleaved1F1B", module, config)


# ---------------------------------------------------------------- data parallel, gradient-exact
def _dp_grads(rank, world, out_dir, module, config, extra):
    import importlib

    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", module, "--config", config, "--training.steps", "1", "--training.seq-len", "64",
        "--training.local-batch-size", "2", "--training.dtype", "float32",
        "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "none",
        "--debug.seed", "0", "--dump-folder", out_dir, *extra]))
    model = t.model_parts[0]
    rt = getattr(model, "_dp_runtime", None)
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    spec = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry(t.config.model_spec.flavor)
    ref = spec.model.build()
    res = ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in full.items()}, strict=False)
    assert not res.unexpected_keys and all("tokens_per_expert" in k for k in res.missing_keys), res
    if hasattr(ref, "rope"):
        ref.rope.init_weights()
    tokens = torch.randint(0, spec.model.vocab_size, (2 * world, 64), generator=torch.Generator().manual_seed(3))
    labels = tokens.roll(-1, 1)
    (cross_entropy_loss(ref(tokens), labels) / labels.numel()).backward()
    mine = slice(2 * rank, 2 * rank + 2)
    if rt is not None:
        rt.begin_microbatch(0, 1)
    t.forward_backward_step(input_dict={"input": tokens[mine]}, labels=labels[mine],
                            global_valid_tokens=torch.tensor(float(labels.numel())))
    named = dict(ref.named_parameters())
    if rt is not None:  # peer runtime: compare this rank's fp32 gradient shard
        rt.finish_backward()
        flat = torch.zeros(rt.total)
        for i, p in enumerate(rt.params):
            n = [k for k, q in model.named_parameters() if q is p][0]
            flat[rt.offsets[i]:rt.offsets[i] + p.numel()] = named[n.replace("_checkpoint_wrapped_module.", "")].grad.flatten()
        for b, sh in zip(rt.buckets, rt.shard_views(rt.grad_shard)):
            sl = b.shard_len(world)
            r = flat[b.offset + rank * sl:b.offset + (rank + 1) * sl]
            assert float((sh - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-8
    else:
        for n, p in model.named_parameters():
            g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
            r = named[n.replace("_checkpoint_wrapped_module.", "")].grad
            assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-8, n
    t.close()


@pytest.mark.parametrize("module,config,extra", [
    ("llama3", "llama3_debugmodel_cpu", ()),
    ("llama3", "llama3_debugmodel_cpu", ("--parallelism.data-parallel-comm", "peer")),
    ("qwen3", "qwen3_debugmodel_moe", ()),
    ("qwen3", "qwen3_debugmodel_moe", ("--parallelism.expert-parallel-degree", "2")),
])
def test_data_parallel_gradients_match_single_device(module, config, extra):
    with tempfile.TemporaryDirectory() as d:
        _run(_dp_grads, 2, d, module, config, extra)


# ---------------------------------------------------------------- exact resume
def _resume_exact(rank, world, out_dir, extra):
    import json

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def make(steps, folder, ckpt):
        return Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", str(steps),
            "--training.seq-len", "64", "--metrics.log-freq", "1", "--metrics.enable-jsonl", "--debug.seed", "0",
            "--dump-folder", os.path.join(out_dir, folder), *(["--checkpoint.enable", "--checkpoint.interval", "2"]
                                                              if ckpt else []), *extra]))

    def losses(folder):
        with open(os.path.join(out_dir, folder, "tb", "rank_0", "metrics.jsonl")) as f:
            return {r["step"]: r["loss_metrics/global_avg_loss"] for r in map(json.loads, f)}

    t = make(4, "straight", False)
    t.train()
    t.close()
    t = make(2, "resumed", True)
    t.train()
    t.close()
    t = make(4, "resumed", True)
    t.checkpointer.load()
    assert t.step == 2
    t.train()
    t.close()
    if rank == 0:
        a, b = losses("straight"), losses("resumed")
        for s in (3, 4):
            assert a[s] == b[s], (s, a[s], b[s], extra)


@pytest.mark.parametrize("extra", [
    (), ("--parallelism.data-parallel-comm", "peer"),
    ("--parallelism.tensor-parallel-degree", "2", "--parallelism.data-parallel-shard-degree", "1"),
    ("--parallelism.pipeline-parallel-degree", "2", "--parallelism.data-parallel-shard-degree", "1",
     "--parallelism.pipeline-parallel-microbatch-size", "2"),
])
def test_resume_reproduces_uninterrupted_losses(extra):
    with tempfile.TemporaryDirectory() as d:
        _run(_resume_exact, 2, d, extra)


# ---------------------------------------------------------------- async checkpoint
def _resume_async(rank, world, out_dir, mode):
    import json

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def make(steps, folder, extra=()):
        return Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", str(steps),
            "--training.seq-len", "64", "--metrics.log-freq", "1", "--metrics.enable-jsonl", "--debug.seed", "0",
            "--dump-folder", os.path.join(out_dir, folder), *extra]))

    def losses(folder):
        with open(os.path.join(out_dir, folder, "tb", "rank_0", "metrics.jsonl")) as f:
            return {r["step"]: r["loss_metrics/global_avg_loss"] for r in map(json.loads, f)}

    ck = ("--checkpoint.enable", "--checkpoint.interval", "2", "--checkpoint.async-mode", mode,
          "--checkpoint.no-last-save-model-only")
    t = make(5, "straight", ck)  # step 2 is written in the background while steps 3-5 train
    assert t.checkpointer._async_pg is not None
    t.train()
    t.close()
    t = make(5, "straight", ck + ("--checkpoint.load-step", "2"))
    t.checkpointer.load(step=2)
    assert t.step == 2
    t.train()
    t.close()
    if rank == 0:
        a = losses("straight")
        with open(os.path.join(out_dir, "straight", "tb", "rank_0", "metrics.jsonl")) as f:
            rows = [json.loads(r) for r in f]
        resumed = {r["step"]: r["loss_metrics/global_avg_loss"] for r in rows[5:]}
        first = {r["step"]: r["loss_metrics/global_avg_loss"] for r in rows[:5]}
        for s in (3, 4, 5):
            assert first[s] == resumed[s], (s, first[s], resumed[s], mode, a)


@pytest.mark.parametrize("mode", ["async", "async_with_pinned_mem"])
def test_async_checkpoint_saved_while_training_resumes_exactly(mode):
    with tempfile.TemporaryDirectory() as d:
        _run(_resume_async, 2, d, mode)


def _uneven_stage(rank, world):
    from torch.distributed.device_mesh import init_device_mesh
    from torch.distributed.tensor import Shard, distribute_tensor

    from torchtitan_b200.components.checkpoint import _to_pinned_host

    mesh = init_device_mesh("cpu", (world,))
    full = torch.arange(5 * 3, dtype=torch.float32).reshape(5, 3)  # 5 rows over 2 ranks: 3 + 2
    dt = distribute_tensor(full, mesh, [Shard(0)])
    staged = _to_pinned_host({"w": dt}, pin=False, copy_cpu=True)["w"]
    assert staged.shape == full.shape and staged.stride() == dt.stride()
    assert staged.to_local().data_ptr() != dt.to_local().data_ptr()
    assert torch.equal(staged.full_tensor(), full)


def test_pinned_staging_keeps_uneven_shard_shape():
    _run(_uneven_stage, 2)


# ---------------------------------------------------------------- gradient accumulation
def _grad_accum(rank, world, out_dir, extra):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    res = []
    for lbs in ("4", "2"):  # one microbatch of 4 vs two of 2 per rank, same global batch
        t = Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "3",
            "--training.seq-len", "64", "--training.local-batch-size", lbs, "--training.global-batch-size",
            str(4 * world), "--metrics.log-freq", "1", "--debug.seed", "0",
            "--dump-folder", os.path.join(out_dir, lbs), *extra]))
        assert t.gradient_accumulation_steps == (1 if lbs == "4" else 2)
        t.train()
        res.append(t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"])
        t.close()
    assert abs(res[0] - res[1]) <= 2e-5 * abs(res[0]), (res, extra)


@pytest.mark.parametrize("extra", [(), ("--parallelism.data-parallel-comm", "peer")])
def test_gradient_accumulation_matches_large_batch(extra):
    with tempfile.TemporaryDirectory() as d:
        _run(_grad_accum, 2, d, extra)


# ---------------------------------------------------------------- failure handling
def _slow_rank(rank, world):
    import datetime
    import time

    pg = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=2))
    t = torch.ones(1)
    dist.all_reduce(t, group=pg)
    if rank == 1:
        time.sleep(6)  # misses the next collective's deadline; nothing of it is in flight yet
    else:
        with pytest.raises(Exception):
            dist.all_reduce(t, group=pg)


def test_rank_delayed_past_timeout_surfaces_as_error():
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_entry, args=(r, 2, port, _slow_rank, ())) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(not p.is_alive() for p in procs)
    assert procs[0].exitcode == 0


def _dropped_message(rank, world):
    import datetime

    pg = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=2))
    t = torch.zeros(4)
    if rank == 0:  # waits for a pipeline activation that rank 1 never sends
        req = dist.irecv(t, src=1, group=pg)
        with pytest.raises(Exception):
            req.wait(timeout=datetime.timedelta(seconds=2))
    dist.barrier()  # both ranks still answer afterwards


def test_dropped_message_surfaces_as_error():
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_entry, args=(r, 2, port, _dropped_message, ())) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert all(not p.is_alive() for p in procs)
    assert all(p.exitcode == 0 for p in procs)


def _corrupt_resume(rank, world, out_dir):
    import glob

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def make(steps):
        return Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", str(steps),
            "--training.seq-len", "64", "--checkpoint.enable", "--checkpoint.interval", "2", "--debug.seed", "0",
            "--dump-folder", out_dir]))

    t = make(4)
    t.train()
    t.close()
    dist.barrier()
    if rank == 0:  # truncate one shard of the newest checkpoint
        shard = sorted(glob.glob(os.path.join(out_dir, "checkpoint", "step-4", "*.distcp")))[0]
        with open(shard, "r+b") as f:
            f.truncate(64)
    dist.barrier()
    t = make(6)
    assert t.checkpointer.load()
    assert t.step == 2  # fell back to the last good checkpoint
    t.checkpointer.config.fallback_on_load_error = False
    with pytest.raises(RuntimeError, match="no loadable checkpoint"):
        t.checkpointer.load()
    t.close()


def test_corrupt_checkpoint_falls_back_to_previous_step():
    with tempfile.TemporaryDirectory() as d:
        _run(_corrupt_resume, 2, d)


def _hf_backend(rank, world, out_dir):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "hf_transformers", "--config", "hf_transformers_qwen3_debugmodel", "--training.steps", "3",
        "--training.seq-len", "64", "--training.local-batch-size", "2", "--training.dtype", "float32",
        "--training.mixed-precision-param", "float32", "--activation-checkpoint.mode", "full",
        "--metrics.log-freq", "1", "--dump-folder", out_dir]))
    t.train()
    loss = t.metrics_processor.last_metrics["loss_metrics/global_avg_loss"]
    assert 6.0 < loss < 9.0
    t.close()


def test_hf_transformers_backend_trains_with_fsdp():
    with tempfile.TemporaryDirectory() as d:
        _run(_hf_backend, 2, d)


# ---------------------------------------------------------------- Qwen3-VL, gradient-exact
def _qwen3_vl_grads(rank, world, out_dir, mode, module="qwen3_vl"):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    import importlib

    from torchtitan_b200.trainer import Trainer

    model_registry = importlib.import_module(f"torchtitan_b200.models.{module}").model_registry
    par = (["--parallelism.tensor-parallel-degree", "2", "--parallelism.data-parallel-shard-degree", "1"]
           if mode == "tp" else ["--parallelism.data-parallel-shard-degree", "2"])
    t = Trainer(ConfigManager().parse_args([
        "--module", module, "--config", f"{module}_debugmodel", "--training.steps", "1",
        "--training.seq-len", "128", "--training.local-batch-size", "2", "--debug.seed", "0",
        "--dump-folder", out_dir, "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
        "--activation-checkpoint.mode", "none", "--dataloader.image-size", "64", *par]))
    model = t.model_parts[0]
    if mode == "fsdp":  # every vision block is its own FSDP unit
        enc = model.vision_encoder.blocks if module == "qwen3_vl" else model.encoder.layers
        assert type(enc[0]).__name__.startswith("FSDP")
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    ref = model_registry("debugmodel").model.build()
    ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in full.items()}, strict=False)
    ref.rope.init_weights()
    if module == "qwen3_vl":
        ref.vision_encoder.init_buffers()
    inp, labels = next(iter(t.dataloader))  # same batch on both ranks (seeded by dp rank 0 for tp)
    if mode == "fsdp":
        obj = [(inp, labels)]
        dist.broadcast_object_list(obj, src=0)
        inp, labels = obj[0]
    kw = {k: v for k, v in inp.items() if k != "input"}
    cross_entropy_loss(ref(inp["input"], **kw), labels).backward()
    comp = getattr(model, "_fsdp_grad_compensation", 1)
    (t._loss(model(inp["input"], **kw), labels) * comp).backward()
    named = dict(ref.named_parameters())
    scale = world if mode == "fsdp" else 1  # FSDP sums the (identical) per-rank gradients
    for n, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
        r = named[n.replace("_checkpoint_wrapped_module.", "")].grad * scale
        assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-7, (n, mode)
    t.close()


@pytest.mark.parametrize("module", ["qwen3_vl", "vlm"])
@pytest.mark.parametrize("mode", ["tp", "fsdp"])
def test_vision_language_parallel_gradients(mode, module):
    with tempfile.TemporaryDirectory() as d:
        _run(_qwen3_vl_grads, 2, d, mode, module)


# ---------------------------------------------------------------- FLUX under FSDP2
def _flux_fsdp(rank, world, out_dir):
    import pathlib

    sys.path.insert(0, str(pathlib.Path(__file__).parent))
    from test_flux_cpu import _small_cfg

    from torchtitan_b200.models.flux.trainer import FluxTrainer

    cfg = _small_cfg(pathlib.Path(out_dir), steps=2)
    cfg.parallelism.data_parallel_shard_degree = 2
    t = FluxTrainer(cfg)
    assert type(t.model_parts[0].double_blocks[0]).__name__.startswith("FSDP")
    t.train()
    losses = [torch.zeros(1) for _ in range(world)]
    dist.all_gather(losses, t.last_loss.detach().reshape(1).float())
    assert all(torch.isfinite(x).all() for x in losses)
    # replicas stay identical: gathered full parameters match across ranks
    w = t.model_parts[0].final_layer.linear.weight.full_tensor()
    ws = [torch.zeros_like(w) for _ in range(world)]
    dist.all_gather(ws, w)
    assert torch.equal(ws[0], ws[1])
    t.close()


def test_flux_fsdp_training():
    with tempfile.TemporaryDirectory() as d:
        _run(_flux_fsdp, 2, d)


# ---------------------------------------------------------------- ETP combined with EP
def _etp_ep_grads(rank, world, out_dir, sp):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.models.qwen3 import model_registry
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "qwen3", "--config", "qwen3_debugmodel_moe", "--training.steps", "1",
        "--training.seq-len", "64", "--training.local-batch-size", "2", "--parallelism.tensor-parallel-degree", "2",
        "--parallelism.data-parallel-shard-degree", "2", "--parallelism.expert-parallel-degree", "2",
        "--parallelism.expert-tensor-parallel-degree", "2", "--debug.seed", "0", "--dump-folder", out_dir,
        "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
        "--activation-checkpoint.mode", "none", *([] if sp else ["--parallelism.no-enable-sequence-parallel"])]))
    model = t.model_parts[0]
    w1 = next(iter(model.layers.values())).moe.experts.w1
    assert tuple(w1.to_local().shape[:2]) == (w1.shape[0] // 2, w1.shape[1] // 2)  # [ep, etp] shards
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    ref = model_registry("debugmodel_moe").model.build()
    ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in full.items()}, strict=False)
    ref.rope.init_weights()
    for n, b in model.named_buffers():
        if n.endswith("expert_bias"):
            dict(ref.named_buffers())[n].copy_(b)
    tokens = torch.randint(0, 2048, (2, 64), generator=torch.Generator().manual_seed(3))
    labels = tokens.roll(-1, 1)
    cross_entropy_loss(ref(tokens), labels).backward()
    comp = getattr(model, "_fsdp_grad_compensation", 1)
    (t._loss(model(tokens), labels) * comp).backward()
    named = dict(ref.named_parameters())
    for n, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
        r = named[n.replace("_checkpoint_wrapped_module.", "")].grad * 2  # both data-parallel ranks see the batch
        assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-7, (n, sp)
    t.close()


@pytest.mark.parametrize("sp", [True, False])
def test_expert_tensor_parallel_with_expert_parallel(sp):
    with tempfile.TemporaryDirectory() as d:
        _run(_etp_ep_grads, 4, d, sp)


def _flux_cp(rank, world, out_dir):
    """Ulysses context parallelism for FLUX: the sharded loss and gradients equal the
    full-sequence ones of the same weights and batch."""
    import pathlib

    sys.path.insert(0, str(pathlib.Path(__file__).parent))
    from test_flux_cpu import _small_cfg
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.models.flux.trainer import FluxTrainer

    cfg = _small_cfg(pathlib.Path(out_dir), steps=1)
    cfg.parallelism.context_parallel_degree = 2
    cfg.parallelism.data_parallel_shard_degree = 1
    cfg.training.max_norm = 0.0
    t = FluxTrainer(cfg)
    model = t.model_parts[0]
    full = get_model_state_dict(model, options=StateDictOptions(full_state_dict=True))
    ref = t.model_args.build()
    ref.load_state_dict(full)
    inp, labels = next(iter(t.dataloader))
    t._microbatch = 0
    f = t.flow_inputs(inp, labels)
    target = f.pop("target")
    loss_ref = t.loss_fn(ref(**f), target) / target.numel()
    loss_ref.backward()
    t._microbatch = 0
    loss = t.forward_backward_step(input_dict=inp, labels=labels,
                                   global_valid_tokens=torch.tensor(float(labels.numel())))
    total = loss.detach().clone()
    dist.all_reduce(total)
    assert abs(float(total) - float(loss_ref)) < 1e-4 * abs(float(loss_ref)), (float(total), float(loss_ref))
    named = dict(ref.named_parameters())
    for n, p in model.named_parameters():
        g = p.grad.full_tensor() if hasattr(p.grad, "full_tensor") else p.grad
        r = named[n.replace("_checkpoint_wrapped_module.", "")].grad
        assert float((g - r).abs().max()) <= 2e-4 * float(r.abs().max()) + 1e-7, n
    t.close()


def test_flux_context_parallel_matches_full_sequence():
    with tempfile.TemporaryDirectory() as d:
        _run(_flux_cp, 2, d)


# ---------------------------------------------------------------- tensor-parallel generation
def _tp_generate(rank, world):
    from torchtitan_b200.generate import generate, make_tensor_parallel
    from torchtitan_b200.models.llama3 import model_registry

    torch.manual_seed(0)
    m = model_registry("debugmodel").model.build()
    m.init_weights()
    m.eval()
    p = torch.randint(0, 2048, (2, 9), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        ref = generate(m, p, 6, 1.0, 8, torch.Generator().manual_seed(2))
        assert make_tensor_parallel(m) is not None
        out = generate(m, p, 6, 1.0, 8, torch.Generator().manual_seed(2))
    assert torch.equal(out, ref), (out, ref)


def test_tensor_parallel_generation_matches_single_device():
    _run(_tp_generate, 2)


# ---------------------------------------------------------------- validation through the training layout
def _validate_layout(rank, world, out_dir, extra):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.components.validate import Validator
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.models.llama3 import model_registry
    from torchtitan_b200.trainer import Trainer

    t = Trainer(ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "1",
        "--training.seq-len", "64", "--training.local-batch-size", "2", "--training.dtype", "float32",
        "--training.mixed-precision-param", "float32", "--parallelism.data-parallel-shard-degree", "1",
        "--validator.enable", "--validator.steps", "2", "--debug.seed", "0", "--dump-folder", out_dir, *extra]))
    loss = t.validator.validate(t.model_parts, 0)
    full = {}
    for part in t.model_parts:
        full.update(get_model_state_dict(part, options=StateDictOptions(full_state_dict=True)))
    gathered = [None] * world
    dist.all_gather_object(gathered, full)
    merged = {}
    for d in gathered:
        merged.update(d)
    ref = model_registry("debugmodel").model.build()
    ref.load_state_dict({k.replace("_checkpoint_wrapped_module.", ""): v for k, v in merged.items()}, strict=False)
    ref.rope.init_weights()
    v = Validator(t.config.validator, seq_len=64, local_batch_size=2, loss_fn=cross_entropy_loss)
    want = v.validate([ref], 0)
    assert abs(loss - want) < 1e-5 * abs(want), (loss, want, extra)
    t.close()


@pytest.mark.parametrize("extra", [
    ("--parallelism.tensor-parallel-degree", "2"),
    ("--parallelism.pipeline-parallel-degree", "2", "--parallelism.pipeline-parallel-microbatch-size", "1"),
    ("--parallelism.context-parallel-degree", "2"),
])
def test_validation_through_parallel_layouts(extra):
    with tempfile.TemporaryDirectory() as d:
        _run(_validate_layout, 2, d, extra)


# ---------------------------------------------------------------- forge engine under pipeline parallelism
def _forge_pp(rank, world, out_dir, schedule):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.forge import ForgeEngine
    from torchtitan_b200.models.llama3 import model_registry

    eng = ForgeEngine(ConfigManager().parse_args([
        "--module", "llama3", "--config", "llama3_debugmodel_cpu", "--training.steps", "4",
        "--training.seq-len", "32", "--parallelism.pipeline-parallel-degree", "2",
        "--parallelism.data-parallel-shard-degree", "1", "--parallelism.pipeline-parallel-microbatch-size", "1",
        "--training.local-batch-size", "2", "--parallelism.pipeline-parallel-schedule", schedule,
        "--training.dtype", "float32", "--training.mixed-precision-param", "float32",
        "--activation-checkpoint.mode", "none", "--debug.seed", "0", "--dump-folder", out_dir]))
    full = {}
    for part in eng.model_parts:
        full.update(get_model_state_dict(part, options=StateDictOptions(full_state_dict=True)))
    gathered = [None] * world
    dist.all_gather_object(gathered, full)
    merged = {k: v for d in gathered for k, v in d.items()}
    ref = model_registry(eng.config.model_spec.flavor).model.build()
    ref.load_state_dict(merged, strict=False)
    ref.rope.init_weights()
    tokens = torch.randint(0, 2048, (2, 33), generator=torch.Generator().manual_seed(5))
    inp, labels = tokens[:, :-1], tokens[:, 1:]
    # forward only: every pipeline rank gets the last stage's logits, equal to the whole model's
    logits = eng.forward({"input": inp})
    with torch.no_grad():
        want = ref(inp)
    torch.testing.assert_close(logits, want, rtol=1e-5, atol=1e-5)
    # a custom objective (half the cross entropy, normalised by twice the token count) trains
    # through the schedule's last stage
    loss = eng.train_on_batches([({"input": inp}, labels)],
                                loss_fn=lambda pred, lab: 0.5 * cross_entropy_loss(pred, lab),
                                count_valid=lambda lab: 2 * lab.numel())
    if eng.pp_has_last_stage:
        exp = 0.25 * cross_entropy_loss(want, labels) / labels.numel()
        torch.testing.assert_close(loss.reshape(()), exp, rtol=1e-5, atol=1e-6)
    assert eng.step == 1 and eng.trainer.loss_fn is not None and "count_valid" not in eng.trainer.__dict__
    after = eng.forward({"input": inp})
    assert not torch.allclose(after, logits)  # the step changed the weights
    # the default objective is back: the next step's loss is the plain mean cross entropy
    loss2 = eng.train_on_batches([({"input": inp}, labels)])
    if eng.pp_has_last_stage:
        torch.testing.assert_close(loss2.reshape(()), cross_entropy_loss(after, labels) / labels.numel(),
                                   rtol=1e-5, atol=1e-6)
    eng.close()


@pytest.mark.parametrize("schedule", ["1F1B", "Interleaved1F1B"])
def test_forge_engine_pipeline_forward_and_custom_objective(schedule):
    with tempfile.TemporaryDirectory() as d:
        _run(_forge_pp, 2, d, schedule)

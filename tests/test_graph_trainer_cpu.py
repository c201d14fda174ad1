"""Graph trainer on CPU/gloo: SimpleFSDP gradients against an unsharded model, every graph
pass exact against the eager step, and the GraphTrainer loop against its eager mode."""
import copy
import os
import socket

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


def _run(fn, world, *args):
    mp.spawn(_entry, args=(world, _port(), fn, args), nprocs=world, join=True)


def _entry(rank, world, port, fn, args):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def _model(vocab=131):
    from torchtitan_b200.models.llama3 import Llama3ModelArgs

    torch.manual_seed(0)
    m = Llama3ModelArgs(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=vocab, max_seq_len=64).build()
    m.init_weights()
    return m


def _loss_fn(pred, labels):
    from torchtitan_b200 import ops

    return ops.cross_entropy_sum(pred.flatten(0, 1).float(), labels.flatten())


def _shard(t, rank, world):
    per = -(-t.shape[0] // world)
    return t[rank * per:(rank + 1) * per]


def _batch(world):
    g = torch.Generator().manual_seed(1)
    tok = torch.randint(0, 131, (2 * world, 32), generator=g)
    lab = torch.randint(0, 131, (2 * world, 32), generator=g)
    return tok, lab


def _sfsdp_vs_unsharded(rank, world, mode):
    from torch.distributed.device_mesh import init_device_mesh

    from torchtitan_b200.graph.simple_fsdp import data_parallel, disable_active_parametrization

    ref = _model()
    m = copy.deepcopy(ref)
    if mode == "hybrid_shard":
        mesh = init_device_mesh("cpu", (2, world // 2), mesh_dim_names=("dp_replicate", "fsdp"))
        shard_rank, shard_world = mesh.get_local_rank(1), world // 2
    else:
        mesh = init_device_mesh("cpu", (world,))
        shard_rank, shard_world = (rank, world) if mode == "fully_shard" else (0, 1)
    data_parallel(m, mesh, mode)
    with disable_active_parametrization():
        assert type(m.tok_embeddings.weight).__name__ == "DTensor"
    tok, lab = _batch(world)
    norm = float(lab.numel())
    loss = _loss_fn(m(tok[2 * rank:2 * rank + 2]), lab[2 * rank:2 * rank + 2]) / norm
    loss.backward()
    (_loss_fn(ref(tok), lab) / norm).backward()
    for (n, p), q in zip(m.named_parameters(), ref.parameters()):
        want = _shard(q.grad, shard_rank, shard_world)
        torch.testing.assert_close(p.grad.to_local(), want, rtol=1e-5, atol=1e-6, msg=n)


@pytest.mark.parametrize("mode,world", [("fully_shard", 2), ("fully_shard", 3), ("replicate", 2),
                                        ("hybrid_shard", 4)])
def test_simple_fsdp_matches_unsharded(mode, world):
    _run(_sfsdp_vs_unsharded, world, mode)


def _passes_exact(rank, world, pass_sets):
    from torch.distributed.device_mesh import init_device_mesh

    from torchtitan_b200.graph import passes as P
    from torchtitan_b200.graph.simple_fsdp import data_parallel
    from torchtitan_b200.graph.tracer import GraphStepRunner, trace_train_step

    m = _model()
    data_parallel(m, init_device_mesh("cpu", (world,)), "fully_shard")
    tok, lab = _batch(world)
    tok, lab = tok[2 * rank:2 * rank + 2], lab[2 * rank:2 * rank + 2]
    norm = torch.tensor(float(lab.numel() * world))
    eager_loss = _loss_fn(m(tok), lab) / norm
    eager_loss.backward()
    want = [p.grad.to_local().clone() for p in m.parameters()]
    n_params = len(want)
    for names in pass_sets:
        m.zero_grad()
        tr = trace_train_step(m, _loss_fn, tok, lab, norm)
        ag0 = sum(1 for n in tr.gm.graph.nodes if n.target == P.AG)
        assert ag0 == n_params  # one gather per parameter as traced
        P.apply_passes(tr, P.DEFAULT_PASSES + names)
        nodes = list(tr.gm.graph.nodes)
        ags = [n for n in nodes if n.target == P.AG]
        rss = [n for n in nodes if n.target == P.RS]
        if "transformer_block_bucketing" in names:
            # one bucket per block and per top-level module (x2 when backward re-gathers)
            n_buckets = 2 + 2 + 1  # tok_embeddings, layers.0, layers.1, norm, output
            assert len(rss) == n_buckets
            # backward re-gathers every bucket but the embedding (its backward needs no weight)
            assert len(ags) == (n_buckets + 4 if "reshard_after_forward" in names else n_buckets)
            # reductions are waited on only at the end of the graph
            waits = [i for i, n in enumerate(nodes) if n.target == P.WAIT and n.args[0] in rss]
            assert min(waits) > max(i for i, n in enumerate(nodes) if n.target == P.RS)
        elif "reshard_after_forward" in names:
            assert len(ags) > n_params
        loss = GraphStepRunner(m, tr)(tok, lab, norm)
        torch.testing.assert_close(loss, eager_loss.detach(), rtol=1e-6, atol=1e-6)
        for p, w in zip(m.parameters(), want):
            torch.testing.assert_close(p.grad.to_local(), w, rtol=1e-5, atol=1e-6)


def test_graph_passes_exact():
    _run(_passes_exact, 2, [[], ["reshard_after_forward"], ["transformer_block_bucketing"],
                            ["reshard_after_forward", "transformer_block_bucketing"],
                            ["selective_recompute", "auto_bucketing"]])


def test_selective_recompute_moves_cheap_ops_to_backward():
    """Single process: recompute re-creates elementwise forward ops in the backward and
    the traced step still matches eager autograd."""
    from torchtitan_b200.graph import passes as P
    from torchtitan_b200.graph.tracer import GraphStepRunner, backward_nodes, trace_train_step

    m = _model()
    tok, lab = _batch(1)
    norm = torch.tensor(float(lab.numel()))
    (_loss_fn(m(tok), lab) / norm).backward()
    want = [p.grad.clone() for p in m.parameters()]
    m.zero_grad()
    tr = trace_train_step(m, _loss_fn, tok, lab, norm)
    P.apply_passes(tr, P.DEFAULT_PASSES)
    n_before = len(tr.gm.graph.nodes)
    copied = P.selective_recompute(tr)
    assert copied > 0 and len(tr.gm.graph.nodes) > n_before
    bwd = backward_nodes(tr.gm, tr.loss_node)
    # no GEMM is recomputed: every mm in the backward is a backward GEMM (dgrad / wgrad)
    n_mm_fwd = sum(1 for n in tr.gm.graph.nodes if n.target == torch.ops.aten.mm.default and n not in bwd)
    n_mm_bwd = sum(1 for n in tr.gm.graph.nodes if n.target == torch.ops.aten.mm.default and n in bwd)
    assert n_mm_bwd <= 2 * n_mm_fwd
    GraphStepRunner(m, tr)(tok, lab, norm)
    for p, w in zip(m.parameters(), want):
        torch.testing.assert_close(p.grad, w, rtol=1e-5, atol=1e-6)


def _trainer_modes(rank, world, out, accum=1):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.graph.trainer import GraphTrainer

    losses = {}
    for mode in ("eager", "aot_fx_trace"):
        cfg = ConfigManager().parse_args(["--module", "graph", "--config", "graph_trainer_llama3_debugmodel_cpu",
                                          "--training.steps", "3", "--training.seq_len", "64",
                                          "--training.local_batch_size", "2", "--checkpoint.no-enable",
                                          "--validator.no-enable", "--compile.mode", mode,
                                          "--training.global_batch_size", str(2 * world * accum),
                                          "--debug.seed", "7", "--dump-folder", out])
        assert isinstance(cfg, GraphTrainer.Config)
        t = GraphTrainer(cfg)
        it = t.batch_generator(t.dataloader)
        vals = []
        while t.step < 3:
            t.step += 1
            vals.append(float(t.train_step(it)))
        losses[mode] = vals
        t.close()
    torch.testing.assert_close(torch.tensor(losses["aot_fx_trace"]), torch.tensor(losses["eager"]),
                               rtol=1e-5, atol=1e-6)


def test_graph_trainer_matches_eager_mode(tmp_path):
    _run(_trainer_modes, 2, str(tmp_path))


def test_graph_trainer_gradient_accumulation(tmp_path):
    """Two microbatches per step: the traced step's gradients accumulate like eager ones."""
    _run(_trainer_modes, 2, str(tmp_path), 2)


def _precompile(rank, world, out):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.graph.trainer import GraphTrainer

    runs = []
    for _ in range(2):
        cfg = ConfigManager().parse_args(["--module", "graph", "--config", "graph_trainer_llama3_debugmodel_cpu",
                                          "--training.steps", "2", "--training.seq_len", "64",
                                          "--training.local_batch_size", "2", "--checkpoint.no-enable",
                                          "--validator.no-enable", "--debug.seed", "3", "--dump-folder", out,
                                          "--compile.precompile-artifact-dir", os.path.join(out, "artifacts")])
        t = GraphTrainer(cfg)
        it = t.batch_generator(t.dataloader)
        losses = []
        while t.step < 2:
            t.step += 1
            losses.append(float(t.train_step(it)))
        runs.append((losses, getattr(t, "loaded_artifacts", 0)))
        t.close()
    assert runs[0][1] == 0 and runs[1][1] == 1  # the second run loads the first run's graph
    assert os.path.exists(os.path.join(out, "artifacts")) and \
        sum(f.endswith(f"rank{rank}.pt") for f in os.listdir(os.path.join(out, "artifacts"))) == 1
    assert runs[0][0] == runs[1][0]


def test_graph_trainer_precompiled_artifacts(tmp_path):
    _run(_precompile, 2, str(tmp_path))


def _fp8_gather(rank, world):
    import torch.nn as nn
    from torch.distributed.device_mesh import init_device_mesh

    from torchtitan_b200.graph.simple_fsdp import MixedPrecisionPolicy, _fp8_rows, data_parallel

    class Lin(nn.Linear):
        pass

    torch.manual_seed(0)
    ref = nn.Sequential(Lin(16, 37, bias=True), nn.Tanh(), nn.Linear(37, 5))
    m = copy.deepcopy(ref)
    data_parallel(m, init_device_mesh("cpu", (world,)), "fully_shard",
                  MixedPrecisionPolicy(fp8_all_gather_modules=(Lin,)))
    w = m[0].weight  # gathered through FP8 codes with per-row scales
    codes, inv = _fp8_rows(ref[0].weight.detach())
    want = codes.view(torch.float8_e4m3fn).float() * inv[:, None]
    assert torch.equal(w.detach(), want)
    assert not torch.equal(w.detach(), ref[0].weight.detach())  # it is really quantized
    torch.testing.assert_close(m[2].weight.detach(), ref[2].weight.detach())  # other modules: exact
    torch.testing.assert_close(m[0].bias.detach(), ref[0].bias.detach())     # 1-D: exact
    # gradients pass straight through the quantizer and are reduce-scattered as usual
    x = torch.randn(4, 16, generator=torch.Generator().manual_seed(rank))
    m(x).sum().backward()
    xs = torch.cat([torch.randn(4, 16, generator=torch.Generator().manual_seed(r)) for r in range(world)])
    q = copy.deepcopy(ref)
    with torch.no_grad():
        q[0].weight.copy_(want)
    q(xs).sum().backward()
    torch.testing.assert_close(m[0]._parameters["weight"].grad.to_local(),
                               _shard(q[0].weight.grad, rank, world), rtol=1e-5, atol=1e-6)


def test_simple_fsdp_fp8_all_gather():
    _run(_fp8_gather, 2)


def _resume(rank, world, out):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.graph.trainer import GraphTrainer

    def cfg(steps, folder, ckpt):
        args = ["--module", "graph", "--config", "graph_trainer_llama3_debugmodel_cpu",
                "--training.steps", str(steps), "--training.seq_len", "64", "--training.local_batch_size", "2",
                "--validator.no-enable", "--debug.seed", "5", "--dump-folder", folder]
        args += ["--checkpoint.enable", "--checkpoint.interval", "2"] if ckpt else ["--checkpoint.no-enable"]
        return ConfigManager().parse_args(args)

    def losses(t, upto):
        it = t.batch_generator(t.dataloader)
        out_ = []
        while t.step < upto:
            t.step += 1
            out_.append(float(t.train_step(it)))
            t.checkpointer.save(t.step, last_step=t.step == upto)
        return out_

    straight = GraphTrainer(cfg(3, os.path.join(out, "a"), False))
    ref = losses(straight, 3)
    straight.close()
    first = GraphTrainer(cfg(2, os.path.join(out, "b"), True))
    losses(first, 2)
    first.close()
    second = GraphTrainer(cfg(3, os.path.join(out, "b"), True))
    second.checkpointer.load()
    assert second.step == 2
    resumed = losses(second, 3)
    second.close()
    torch.testing.assert_close(torch.tensor(resumed), torch.tensor(ref[2:]), rtol=1e-5, atol=1e-6)


def test_graph_trainer_checkpoint_resume(tmp_path):
    """SimpleFSDP's DTensor shards go through DCP: a resumed run continues the straight run."""
    _run(_resume, 2, str(tmp_path))


def _bitwise(rank, world, out):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.graph.trainer import GraphTrainer
    from torchtitan_b200.utils.hashing import hash_model

    hashes = []
    for _ in range(2):
        cfg = ConfigManager().parse_args(["--module", "graph", "--config", "graph_trainer_llama3_debugmodel_cpu",
                                          "--training.steps", "3", "--training.seq_len", "64",
                                          "--training.local_batch_size", "2", "--checkpoint.no-enable",
                                          "--validator.no-enable", "--debug.seed", "11", "--debug.deterministic",
                                          "--dump-folder", out, "--compile.passes", "selective_recompute",
                                          "reshard_after_forward", "auto_bucketing"])
        t = GraphTrainer(cfg)
        it = t.batch_generator(t.dataloader)
        while t.step < 3:
            t.step += 1
            t.train_step(it)
        hashes.append(hash_model(t.model_parts[0]))
        t.close()
    assert hashes[0] == hashes[1]


def test_graph_trainer_bitwise_deterministic(tmp_path):
    """Two runs of the traced, bucketed, recomputing step from the same seed end with bitwise
    identical weights (parity: the reference graph trainer's bitwise-determinism test)."""
    _run(_bitwise, 2, str(tmp_path))


def test_traced_step_with_packed_documents():
    """Block-causal (packed-document) attention: per-token positions and document ids enter the
    traced step as extra graph inputs; the traced step matches eager autograd."""
    from torchtitan_b200.graph import passes as P
    from torchtitan_b200.graph.tracer import GraphStepRunner, trace_train_step
    from torchtitan_b200.models.llama3 import Llama3ModelArgs

    torch.manual_seed(0)
    m = Llama3ModelArgs(dim=64, n_layers=2, n_heads=4, n_kv_heads=2, vocab_size=131, max_seq_len=64,
                        mask_type="block_causal").build()
    m.init_weights()
    tok, lab = _batch(1)
    pos = torch.cat([torch.arange(12), torch.arange(20)]).repeat(2, 1)  # two documents per row
    extra = {"positions": pos, "attention_masks": torch.cumsum((pos == 0).int(), dim=1)}
    norm = torch.tensor(float(lab.numel()))
    (_loss_fn(m(tok, **extra), lab) / norm).backward()
    want = [p.grad.clone() for p in m.parameters()]
    # the documents really are separated: the unmasked model gives another loss
    with torch.no_grad():
        assert abs(float(_loss_fn(m(tok), lab)) - float(_loss_fn(m(tok, **extra), lab))) > 1e-4
    m.zero_grad()
    tr = trace_train_step(m, _loss_fn, tok, lab, norm, extra)
    P.apply_passes(tr, P.DEFAULT_PASSES + ["selective_recompute"])
    GraphStepRunner(m, tr)(tok, lab, norm, extra)
    for p, w in zip(m.parameters(), want):
        torch.testing.assert_close(p.grad, w, rtol=1e-5, atol=1e-6)


def test_reshard_policy_maps_to_the_graph_pass(tmp_path, monkeypatch):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.graph.trainer import GraphTrainer

    monkeypatch.setenv("LOCAL_RANK", "0")
    got = {}
    for policy in ("never", "always"):
        cfg = ConfigManager().parse_args(["--module", "graph", "--config", "graph_trainer_llama3_debugmodel_cpu",
                                          "--training.steps", "1", "--checkpoint.no-enable", "--validator.no-enable",
                                          "--parallelism.fsdp-reshard-after-forward", policy,
                                          "--compile.passes", "transformer_block_bucketing",
                                          "--dump-folder", str(tmp_path)])
        t = GraphTrainer(cfg)
        got[policy] = list(t._passes)
        t.close()
    assert "reshard_after_forward" not in got["never"]
    assert got["always"][0] == "reshard_after_forward"


def _hsdp_trainer(rank, world, out):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.graph.trainer import GraphTrainer

    losses = {}
    for mode in ("eager", "aot_fx_trace"):
        cfg = ConfigManager().parse_args(["--module", "graph", "--config", "graph_trainer_llama3_debugmodel_cpu",
                                          "--training.steps", "2", "--training.seq_len", "64",
                                          "--training.local_batch_size", "1", "--checkpoint.no-enable",
                                          "--validator.no-enable", "--compile.mode", mode,
                                          "--parallelism.data-parallel-replicate-degree", "2",
                                          "--parallelism.data-parallel-shard-degree", "2",
                                          "--debug.seed", "9", "--dump-folder", out])
        t = GraphTrainer(cfg)
        w = t.model_parts[0].tok_embeddings._parameters["weight"]
        assert w.device_mesh.ndim == 2  # [dp_replicate, fsdp]
        it = t.batch_generator(t.dataloader)
        vals = []
        while t.step < 2:
            t.step += 1
            vals.append(float(t.train_step(it)))
        losses[mode] = vals
        t.close()
    torch.testing.assert_close(torch.tensor(losses["aot_fx_trace"]), torch.tensor(losses["eager"]),
                               rtol=1e-5, atol=1e-6)


def test_graph_trainer_hsdp(tmp_path):
    """HSDP (2 replicas x 2 shards): the traced step with its reduce-scatter + all-reduce nodes
    matches SimpleFSDP's eager step."""
    _run(_hsdp_trainer, 4, str(tmp_path))


def test_graph_trainer_configs_are_data_parallel():
    """Every registered graph-trainer config builds and asks only for the parallelism the graph
    trainer composes (SimpleFSDP data parallelism)."""
    from torchtitan_b200.graph import config_registry as reg
    from torchtitan_b200.graph.trainer import GraphTrainer

    names = [n for n in dir(reg) if n.startswith("graph_trainer_")]
    assert len(names) >= 12
    for n in names:
        c = getattr(reg, n)()
        assert isinstance(c, GraphTrainer.Config), n
        p = c.parallelism
        assert (p.tensor_parallel_degree, p.context_parallel_degree, p.pipeline_parallel_degree,
                p.expert_parallel_degree) == (1, 1, 1, 1), n
        assert c.activation_checkpoint.mode == "none", n
